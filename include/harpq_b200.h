/*
 * harpq_b200.h — C ABI of the B200-native progressive int2 GEMV library.
 *
 * The path: y = x · Wᵀ (+ bias) where W (rows x cols, "out_features x in_features")
 * is stored as up to four signed-int2 residual stages over 128x128 tiles with one
 * FP16 scale per (row, tile, stage), evaluated at a caller-selected prefix depth or
 * a per-tile depth map, without materialising FP16/FP32 weights.
 *
 * Every entry point takes plain pointers and sizes.  Device pointers are CUDA device
 * addresses; `stream` is a cudaStream_t (NULL = legacy default stream).  Status values
 * are cudaError_t codes: 0 success, 1 (cudaErrorInvalidValue) for any rejected argument
 * (nothing is enqueued), 801 (cudaErrorNotSupported) for a geometry the fast path does
 * not cover, otherwise the CUDA error of the failing call.  A sticky CUDA error that is
 * pending before a launch is returned without launching (reference behaviour,
 * native/src/progressive_gemv.cu:427-433).  The caller owns every buffer, the stream
 * ordering and completion, as in the reference (native/include/harpq/progressive_gemv.hpp:49-57).
 *
 * Reference interfaces each group replaces are cited per declaration.
 */
#ifndef HARPQ_B200_H_
#define HARPQ_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define HQB_API __attribute__((visibility("default")))
#else
#define HQB_API
#endif

#define HQB_OK 0
#define HQB_ERR_INVALID 1
#define HQB_ERR_UNSUPPORTED 801

/* element types of activations, bias and outputs */
#define HQB_F32 0
#define HQB_F16 1

/* hqb_gemv_ex flags */
#define HQB_FLAG_PDL 1u  /* launch with programmatic dependent launch (see hqb_gemv_ex) */
#define HQB_FLAG_SIMT 2u /* CUDA-core decode+FFMA consumer instead of tensor-core mma */
#define HQB_FLAG_RING 4u /* force the bulk-copy ring pipeline (comparison/diagnostics) */
#define HQB_FLAG_TCGEN05 8u /* tcgen05 (UMMA, TMEM accumulators) kernel: FP16 x, batch <= 8,
                                 uniform prefix; a comparison path, slower than the default
                                 mma.sync kernels at these shapes */
/* Uniform prefix at batch <= 8 runs one of two kernels, chosen by size: the row-block
 * kernel (no tile row split between CTAs; lowest fixed cost, for small layers) or the
 * stream-K kernel (tile rows split between CTAs, their sums finished through the
 * workspace; best streaming rate, for large layers).  These flags force one of them
 * (both set: HQB_ERR_INVALID; the row-block flag is ignored where its activation
 * fragments would not fit shared memory). */
#define HQB_FLAG_STREAMK 16u
#define HQB_FLAG_ROWBLOCK 32u
/* The GEMV kernels at batch <= 2 with raw FP16 or FP32 x multiply int8 activation limbs
 * (four signed bytes of a 31-bit fixed-point copy of each 128-column tile of x, scaled
 * to the tile's largest |x|) with integer tensor-core MMAs; this flag keeps it on the
 * FP16-fragment MMAs instead (comparison/diagnostics). */
#define HQB_FLAG_F16MMA 64u
/* Batch <= 2 with raw FP16 or FP32 x, uniform prefix or depth map: the bulk-copy kernel
 * (plane chunks of ~40-52 KB moved into shared memory by 1-D bulk copies issued ahead of
 * the programmatic-dependent-launch wait, int8 activation limbs).  It is the default for
 * uniform layers of >= 128 tile columns and >= 96 MB of selected planes at prefix >= 2;
 * this flag selects it for any layer. */
#define HQB_FLAG_BULK 128u

/* Fast-path tiling: 128x128 tiles, one scale group per tile row (group 128). */
#define HQB_TILE 128
/* One stage of one tile in the plane layout: 8 row-blocks x (512 B codes + 32 B scales). */
#define HQB_TILE_RECORD_BYTES 4352
#define HQB_MAX_STAGES 4
#define HQB_MAX_BATCH 16

/* Device-error bits reported through the int flag words below. */
#define HQB_DEVERR_SCALE 1        /* a non-finite or negative FP16 scale was repacked   */
#define HQB_DEVERR_DEPTH 2        /* a depth-map entry outside [1, stage_count]          */
#define HQB_DEVERR_TIMEOUT 4      /* a pipeline wait exceeded its bound (kernel returned) */
#define HQB_DEVERR_LAUNCH 8       /* shared memory sized below a CTA's work (kernel returned) */

/* Matrix geometry, same fields and order as ProgressiveGemvGeometry
 * (reference native/include/harpq/progressive_gemv.hpp:15-23). */
typedef struct hqb_geometry {
  uint64_t original_rows;
  uint64_t original_columns;
  uint64_t padded_rows;
  uint64_t padded_columns;
  uint64_t tile_rows;
  uint64_t tile_columns;
  uint64_t group_size;
} hqb_geometry;

/* One stage in the reference's device layout: row-major packed codes over the padded
 * matrix (4 codes/byte, LSB first) and raw FP16 scale bits in
 * [tile_row][tile_col][row_in_tile][group] order.  Same fields as
 * ProgressiveGemvStageDeviceView (progressive_gemv.hpp:27-32). */
typedef struct hqb_raw_stage {
  const uint8_t* packed_codes;
  uint64_t packed_code_bytes;
  const uint16_t* scale_fp16_bits;
  uint64_t scale_count;
} hqb_raw_stage;

/* Same stage with host-decoded FP32 scales, as DecodedStage carries them
 * (native/include/harpq/native/stage_codec.hpp:26-31); used by the decode and
 * reference-order entry points that must accept any finite non-negative scale. */
typedef struct hqb_raw_stage_f32 {
  const uint8_t* packed_codes;
  uint64_t packed_code_bytes;
  const float* scales;
  uint64_t scale_count;
} hqb_raw_stage_f32;

/* A device-resident matrix in the plane layout: planes[s] holds stage s as
 * grid_rows*grid_cols tile records (row-major over tiles) of HQB_TILE_RECORD_BYTES.
 * Stages are independent buffers, so a newly resident residual stage is one more
 * plane (hqb_repack_stage) without touching the others. */
typedef struct hqb_plane_matrix {
  uint64_t rows;        /* original rows (output features)  */
  uint64_t cols;        /* original columns (input features) */
  uint32_t grid_rows;   /* ceil(rows / 128) */
  uint32_t grid_cols;   /* ceil(cols / 128) */
  uint32_t stage_count; /* planes[0..stage_count) are valid */
  uint32_t reserved;
  const void* planes[HQB_MAX_STAGES];
} hqb_plane_matrix;

HQB_API int hqb_version(void);
HQB_API const char* hqb_status_string(int status);

/* ---- plane layout ---------------------------------------------------------------- */

/* Bytes of one stage plane for geometry g; 0 when g is not 128x128 tiles with group
 * 128 (such matrices run only through hqb_raw_gemv). */
HQB_API uint64_t hqb_plane_bytes(const hqb_geometry* g);

/* Device repack of one reference-layout stage into one plane (16-byte slots in
 * mma-fragment order, codes of padded columns cleared, FP16 scale pairs per row
 * block).  device_flags (optional, device int) gets HQB_DEVERR_SCALE OR-ed in when a
 * scale is NaN/Inf/negative — the checks of DecodeStagePayload
 * (native/src/stage_codec.cpp:205-213), done on the device.  Replaces the reference's
 * per-call use of the row-major layout (native/src/progressive_gemv.cu:359-392). */
HQB_API int hqb_repack_stage(const hqb_geometry* g, const hqb_raw_stage* stage, void* plane,
                             int* device_flags, void* stream);

/* ---- activations ----------------------------------------------------------------- */

/* Bytes of the prepared-activation buffer for `batch` rows of `cols` inputs. */
HQB_API uint64_t hqb_xfrag_bytes(uint64_t cols, uint32_t batch, int x_dtype);

/* Converts x [batch][cols] (FP16 or FP32, row-major) into per-tile tensor-core
 * B fragments plus per-tile correction sums.  One prepared buffer serves every
 * matrix with the same `cols` (e.g. q/k/v).  No reference counterpart (the reference
 * reads FP32 x directly, progressive_gemv.cu:392). */
HQB_API int hqb_prepare_x(const void* x, int x_dtype, uint64_t cols, uint32_t batch,
                          void* xfrag, void* stream);

/* ---- workspace ------------------------------------------------------------------- */

/* Scratch bytes a GEMV on m with this batch needs on `device`: an error word,
 * split-row partial sums and a prepared-activation area.  Calls that overlap on the
 * GPU must not share a workspace. */
HQB_API uint64_t hqb_workspace_bytes(const hqb_plane_matrix* m, uint32_t batch, int x_dtype,
                                     int device);
/* Clears a workspace: its error word, split-row counters and split-row partial sums
 * must start at zero.  Call once after allocation and after a reported device error;
 * counters and partial sums return to zero at the end of every GEMV. */
HQB_API int hqb_workspace_init(void* workspace, uint64_t bytes, void* stream);
/* Copies the workspace error word (HQB_DEVERR_* bits) to *host_flags, synchronously. */
HQB_API int hqb_workspace_error(const void* workspace, int* host_flags, void* stream);

/* ---- mixed depth ------------------------------------------------------------------ */

/* Bytes of the schedule a depth map needs: (grid_rows + 1) uint32 row-cost prefix sums. */
HQB_API uint64_t hqb_depth_plan_bytes(uint32_t grid_rows);
/* Builds the schedule for a device depth map [grid_rows][grid_cols] (uint8, values in
 * [1, stage_count]); bad entries set HQB_DEVERR_DEPTH in device_flags and are clamped.
 * No reference symbol: the reference selects one prefix per matrix
 * (progressive_gemv.hpp:58-62); its allocator emits per-group prefixes
 * (src/harpq/allocator.py:1-9). */
HQB_API int hqb_depth_plan(const uint8_t* depth, uint32_t grid_rows, uint32_t grid_cols,
                           uint32_t stage_count, uint32_t* plan, int* device_flags,
                           void* stream);

/* ---- GEMV ----------------------------------------------------------------------- */

/* y[b][r] = Σ_c x[b][c]·W_prefix[r][c] (+ bias[r]) for b < batch (1..16), FP32
 * accumulation, y FP16 or FP32 [batch][rows].  Replaces LaunchProgressiveGemv
 * (progressive_gemv.hpp:58-62, progressive_gemv.cu:420-439) for plane matrices and
 * extends it to batch 2-16.  prefix 0 writes bias or exact zeros.  x is raw
 * [batch][cols]; it is prepared into the workspace first. */
HQB_API int hqb_gemv(const hqb_plane_matrix* m, uint32_t prefix, const void* x, int x_dtype,
                     uint32_t batch, const void* bias, int bias_dtype, void* y, int y_dtype,
                     void* workspace, uint64_t workspace_bytes, void* stream);

/* Same with a per-tile depth map and its plan (hqb_depth_plan). */
HQB_API int hqb_gemv_mixed(const hqb_plane_matrix* m, const uint8_t* depth,
                           const uint32_t* depth_plan, const void* x, int x_dtype,
                           uint32_t batch, const void* bias, int bias_dtype, void* y,
                           int y_dtype, void* workspace, uint64_t workspace_bytes,
                           void* stream);

/* General form.  depth/depth_plan NULL selects the uniform prefix.  x_prepared != 0
 * means x is a buffer filled by hqb_prepare_x (x_dtype as given to it).
 * HQB_FLAG_PDL launches the GEMV as a programmatic dependent of the previous kernel
 * in the stream: it prefetches weight planes before waiting for that kernel, so that
 * kernel must not write the planes (a preceding hqb_prepare_x or GEMV is fine).
 * HQB_FLAG_SIMT selects the CUDA-core comparison kernel (batch <= 8, FP16 x). */
HQB_API int hqb_gemv_ex(const hqb_plane_matrix* m, uint32_t prefix, const uint8_t* depth,
                        const uint32_t* depth_plan, const void* x, int x_dtype,
                        uint32_t batch, int x_prepared, const void* bias, int bias_dtype,
                        void* y, int y_dtype, void* workspace, uint64_t workspace_bytes,
                        uint32_t flags, void* stream);

/* What one GEMV call would enqueue on the current device, without enqueueing anything:
 * the library's own kernel choice for (m, prefix or depth map, x dtype, batch, prepared x,
 * flags).  No reference counterpart (the reference has one kernel). */
typedef struct hqb_launch_info {
  uint32_t launches;   /* kernels the call enqueues (activation preparation, GEMV, fix-up) */
  uint32_t int8_limbs; /* 1 when the GEMV multiplies int8 activation limbs */
  uint32_t grid;       /* the GEMV kernel's CTAs */
  uint32_t block;      /* its threads per CTA */
  uint32_t smem_bytes; /* its dynamic shared memory per CTA */
  uint32_t reserved;
  char kernel[40];     /* GEMV kernel family, e.g. "gemv_bulk_kernel" (NUL-terminated) */
} hqb_launch_info;

/* mixed != 0: a per-tile depth map (prefix ignored).  Returns the status hqb_gemv_ex would
 * return for invalid arguments, else 0 with *info filled. */
HQB_API int hqb_gemv_query(const hqb_plane_matrix* m, uint32_t prefix, int mixed, int x_dtype, uint32_t batch,
                           int x_prepared, uint32_t flags, hqb_launch_info* info);

/* One GEMV of a batch of calls: the arguments of hqb_gemv_ex. */
typedef struct hqb_gemv_call {
  const hqb_plane_matrix* m;
  uint32_t prefix;
  int x_dtype;
  const uint8_t* depth;       /* NULL: uniform prefix */
  const uint32_t* depth_plan; /* NULL: uniform prefix */
  const void* x;
  uint32_t batch;
  int x_prepared;
  const void* bias;
  int bias_dtype;
  int y_dtype;
  void* y;
  uint32_t flags;
  uint32_t reserved;
} hqb_gemv_call;

/* The calls in order on one stream with one workspace (large enough for every call), one
 * host call for a whole decode step: stops at the first call that fails and returns its
 * status (the calls before it are enqueued).  No reference counterpart. */
HQB_API int hqb_gemv_batch(const hqb_gemv_call* calls, uint32_t count, void* workspace, uint64_t workspace_bytes,
                           void* stream);

/* Independent GEMVs (no call reads another's output) as ONE kernel launch: the calls'
 * (tile, stage) units are dealt to the CTAs of one grid in proportion to their sizes, each
 * CTA working on one call, so every call streams at once and the launch's fixed costs are
 * paid once.  It applies to up to 8 calls that share a uniform prefix, batch (<= 2) and raw
 * activation dtype; other call lists run one by one as in hqb_gemv_batch.  The workspace
 * must be as large as the largest call's.  No reference counterpart. */
HQB_API int hqb_gemv_grouped(const hqb_gemv_call* calls, uint32_t count, void* workspace, uint64_t workspace_bytes,
                             void* stream);

/* A decode step captured once: the calls of hqb_gemv_batch recorded into a CUDA graph
 * (their programmatic-dependent launches kept as graph edges) and instantiated.  Launching
 * it costs one graph launch on the host, whatever the number of GEMVs.  The buffers the
 * calls name are bound into the graph: refill x and read y in place.  No reference
 * counterpart. */
typedef struct hqb_step hqb_step;
HQB_API int hqb_step_create(const hqb_gemv_call* calls, uint32_t count, void* workspace, uint64_t workspace_bytes,
                            hqb_step** step);
/* The same for independent calls, captured as hqb_gemv_grouped (one kernel for the group). */
HQB_API int hqb_step_create_grouped(const hqb_gemv_call* calls, uint32_t count, void* workspace,
                                    uint64_t workspace_bytes, hqb_step** step);

/* One copy of a captured step: bytes from src to dst (cudaMemcpyDefault: host buffers must
 * be page-locked, e.g. cudaHostAlloc, so that the copy can live in a CUDA graph). */
typedef struct hqb_copy {
  void* dst;
  const void* src;
  uint64_t bytes;
} hqb_copy;

/* A step that also moves its inputs and outputs: the n_h2d copies, then the GEMVs
 * (grouped != 0: one grouped launch as hqb_step_create_grouped, else as hqb_step_create),
 * then the n_d2h copies, all in the step's one CUDA graph.  A decode step that feeds
 * host-resident activations and reads its results back is then one hqb_step_launch. */
HQB_API int hqb_step_create_io(const hqb_gemv_call* calls, uint32_t count, void* workspace,
                               uint64_t workspace_bytes, const hqb_copy* h2d, uint32_t n_h2d,
                               const hqb_copy* d2h, uint32_t n_d2h, int grouped, hqb_step** step);
HQB_API int hqb_step_launch(hqb_step* step, void* stream);
HQB_API int hqb_step_destroy(hqb_step* step);

/* ---- GEMV with a fixed scratch (no reference counterpart) --------------------------- */

/* Size of the per-device scratch array built into the library for hqb_gemv_noalloc:
 * 4 MiB.  On a 148-SM B200 that covers batch 1-4 for layers up to 28672 input columns,
 * FP16 or FP32 activations (hqb_workspace_bytes gives the exact need). */
#define HQB_NOALLOC_SCRATCH_BYTES (4u << 20)
/* hqb_gemv_noalloc status when hqb_workspace_bytes(m, batch, x_dtype, device) exceeds
 * HQB_NOALLOC_SCRATCH_BYTES; nothing is enqueued (use hqb_gemv with a workspace). */
#define HQB_ERR_SCRATCH_LIMIT 20001

/* hqb_gemv on the current device without a caller workspace and without allocating:
 * the scratch is a fixed array in the library's device image, one per device.  For
 * callers that cannot allocate device memory at the call: a host that binds only this
 * library and holds no device allocator, and a decode step that must not allocate
 * because cudaMalloc/cudaFree synchronize the device and fail once weights and caches
 * fill the HBM.  The reference has no counterpart (its LaunchProgressiveGemv needs no
 * scratch, progressive_gemv.cu:420-439; this library's GEMV does).
 * - The first call on a device sets up: it resolves the array's address on that device
 *   (cudaGetSymbolAddress) and enqueues a clear of the whole array on `stream`.  Make
 *   that first call before any stream capture.
 * - What must start at zero: the error word, the split-row counters and partial sums
 *   (they return to zero at the end of every call).  The rest is written before it is
 *   read.
 * - One scratch per device: calls whose GPU work overlaps (other streams, other host
 *   threads) race on it.  Order them on one stream or with events.
 * - Device error bits land in the scratch's error word: read them with
 *   hqb_gemv_noalloc_flags.  After a non-zero word (a bounded wait that ran out, for
 *   instance) the split-row counters and partial sums may not have returned to zero:
 *   call hqb_gemv_noalloc_reset before the next call.
 * - Every call checks the array's address on the current device (cudaGetSymbolAddress,
 *   which allocates nothing); when it differs from the cached one (the module was loaded
 *   again after cudaDeviceReset) the array is cleared again before use. */
HQB_API int hqb_gemv_noalloc(const hqb_plane_matrix* m, uint32_t prefix, const void* x,
                             int x_dtype, uint32_t batch, const void* bias, int bias_dtype,
                             void* y, int y_dtype, void* stream);
/* The scratch's device error word (HQB_DEVERR_* bits) of the current device copied to
 * *host_flags after the work on `stream` (synchronises the stream); clear != 0 also sets
 * the word back to zero.  Allocates nothing. */
HQB_API int hqb_gemv_noalloc_flags(int* host_flags, int clear, void* stream);
/* Enqueues a clear of the whole scratch array of the current device on `stream` (the state
 * of the first call).  Allocates nothing. */
HQB_API int hqb_gemv_noalloc_reset(void* stream);
/* Device address of the current device's scratch array (*ptr), for inspection. */
HQB_API int hqb_gemv_noalloc_scratch(void** ptr);

/* ---- output-row shards across GPUs: fused all-gather over peer memory --------------- */

#define HQB_MAX_PEERS 8
#define HQB_IPC_HANDLE_BYTES 64

/* Device buffer that peers of this node can map (cudaMalloc + IPC handle).  The handle
 * (HQB_IPC_HANDLE_BYTES) goes to the peers by any host channel. */
HQB_API int hqb_peer_alloc(uint64_t bytes, void** ptr, void* ipc_handle);
/* Maps a peer's buffer from its handle (P2P over NVLink) / unmaps it. */
HQB_API int hqb_peer_open(const void* ipc_handle, void** ptr);
HQB_API int hqb_peer_close(void* ptr);
HQB_API int hqb_peer_free(void* ptr);

/* One rank's view of a gathered output.  Every rank owns a row shard of the layer; its
 * GEMV writes its outputs straight into every rank's gathered buffer (its own included)
 * at columns [rank * slot_rows, rank * slot_rows + rows) of each batch row, so the
 * gathered buffer is [batch][world * slot_rows] of y_dtype on every rank.  After the
 * last CTA's stores, the kernel adds 1 to counter `rank` of every rank's flag array
 * (world uint32, zero-initialised, peer-mapped).  peer_y[r] / peer_flags[r] are rank r's
 * buffers as mapped here (r == rank: the local ones).  No reference counterpart: the
 * reference GEMV runs on one device (native/src/progressive_gemv.cu:420-439). */
typedef struct hqb_gather {
  uint32_t world;
  uint32_t rank;
  uint64_t slot_rows;
  void* peer_y[HQB_MAX_PEERS];
  uint32_t* peer_flags[HQB_MAX_PEERS];
} hqb_gather;

/* hqb_gemv whose outputs go to every rank's gathered buffer (uniform prefix; the plane
 * matrix is this rank's row shard, rows <= slot_rows).  HQB_ERR_UNSUPPORTED when the
 * shape or batch needs a kernel without the fused gather (activations wider than the
 * resident limit, HQB_FLAG_SIMT/RING/TCGEN05). */
HQB_API int hqb_gemv_gather(const hqb_plane_matrix* m, uint32_t prefix, const void* x, int x_dtype,
                            uint32_t batch, const void* bias, int bias_dtype, int y_dtype,
                            const hqb_gather* gather, void* workspace, uint64_t workspace_bytes,
                            uint32_t flags, void* stream);

/* Waits on the device until every rank has signalled the gathered buffer whose local flag
 * array is `flags` once more than the previous wait: one thread spins (bounded, 2 s) on
 * flags[0..world) >= *epoch + 1, then stores the new epoch.  A timeout sets
 * HQB_DEVERR_TIMEOUT in *device_flags.  Launch it before anything reads the gathered
 * buffer. */
HQB_API int hqb_gather_wait(const uint32_t* flags, uint32_t world, uint32_t* epoch, int* device_flags,
                            void* stream);
/* The same with a caller-chosen bound in nanoseconds (at most the 2 s of hqb_gather_wait):
 * a rank that has not signalled within it ends the wait with HQB_DEVERR_TIMEOUT set and the
 * epoch advanced, and the stream goes on, so a host-side failure detector can act. */
HQB_API int hqb_gather_wait_ex(const uint32_t* flags, uint32_t world, uint32_t* epoch, int* device_flags,
                               uint64_t limit_ns, void* stream);

/* ---- prefill (batch >> 16) ------------------------------------------------------------ */

/* y[batch][rows] = x[batch][cols] · W_prefix^T (+ bias) for a large batch, the product the
 * reference lists as future work (docs/RESEARCH_PLAN.md:104).  The selected stages are
 * decoded once per call into FP16 weights in the workspace (each element the FP32 stage sum of
 * DequantizePrefix, native/src/stage_codec.cpp:254-272, rounded once to FP16) and multiplied
 * by cuBLAS with FP16 inputs and FP32 accumulation.  x: FP16 only (HQB_ERR_UNSUPPORTED
 * otherwise); y, bias: FP16 or FP32.  Prefix 0 writes bias or zeros.  The workspace holds
 * hqb_prefill_workspace_bytes(m) bytes, 256-byte aligned.  The first call on a host thread and
 * device creates that thread's cuBLAS handle (kept until exit); a cuBLAS failure returns
 * cudaErrorUnknown. */
HQB_API uint64_t hqb_prefill_workspace_bytes(const hqb_plane_matrix* m);
HQB_API int hqb_prefill_gemm(const hqb_plane_matrix* m, uint32_t prefix, const void* x, int x_dtype,
                             uint32_t batch, const void* bias, int bias_dtype, void* y, int y_dtype,
                             void* workspace, uint64_t workspace_bytes, void* stream);

/* Dense FP32 weights [rows][cols] decoded from planes, Σ_{s<d} code·scale summed in
 * stage order from 0.0f — bit-identical to DequantizePrefix
 * (native/src/stage_codec.cpp:254-272).  depth NULL: uniform prefix. */
HQB_API int hqb_decode_planes(const hqb_plane_matrix* m, uint32_t prefix, const uint8_t* depth,
                              float* out, uint64_t out_count, void* stream);

/* ---- reference-layout (drop-in) entry points --------------------------------------- */

/* LaunchProgressiveGemv semantics on the reference's own device layout, any tile
 * geometry, FP32 x/bias/y, batch 1 (native/include/harpq/progressive_gemv.hpp:49-62,
 * native/src/progressive_gemv.cu:266-321 validation, :420-439 launch).  stages[] has
 * stage_count entries; entries < prefix must be valid. */
HQB_API int hqb_raw_gemv(const hqb_geometry* g, const hqb_raw_stage* stages, uint32_t stage_count,
                         uint32_t prefix, const float* x, uint64_t x_count, const float* bias,
                         uint64_t bias_count, float* y, uint64_t y_count, void* stream);

/* hqb_raw_gemv's kernel choice.  By default, 128x128 tiles with group 128 at prefix 1..4
 * (8-byte aligned code arrays, at most 48K padded columns) run the int8-limb tensor-core
 * kernel on the raw layout (raw_i8_kernel: no repack, no workspace, bits fixed by the
 * shape); other geometries run the per-element FMA kernel (raw_gemv_kernel).
 *   HQB_RAW_GENERIC       always the per-element FMA kernel.
 *   HQB_RAW_REQUIRE_FAST  HQB_ERR_UNSUPPORTED (nothing enqueued) unless the int8 kernel
 *                         applies. */
#define HQB_RAW_GENERIC 1u
#define HQB_RAW_REQUIRE_FAST 2u
HQB_API int hqb_raw_gemv_ex(const hqb_geometry* g, const hqb_raw_stage* stages, uint32_t stage_count,
                            uint32_t prefix, const float* x, uint64_t x_count, const float* bias,
                            uint64_t bias_count, float* y, uint64_t y_count, uint32_t flags, void* stream);

/* out[rows][cols] = code·scale of one stage, the exact FP32 product
 * (DequantizeStage, native/src/stage_codec.cpp:218-252).  Scales are FP32. */
HQB_API int hqb_raw_dequantize_stage(const hqb_geometry* g, const hqb_raw_stage_f32* stages,
                                     uint32_t stage_count, uint32_t stage, float* out,
                                     void* stream);

/* out[rows][cols] = Σ_{s<prefix} code·scale added in stage order into 0.0f
 * (DequantizePrefix, native/src/stage_codec.cpp:254-272).  Scales are FP32. */
HQB_API int hqb_raw_dequantize_prefix(const hqb_geometry* g, const hqb_raw_stage_f32* stages,
                                      uint32_t stage_count, uint32_t prefix, float* out,
                                      void* stream);

/* ProgressiveLinearReference's exact scalar order on the device: per stage a fresh
 * FP32 dot per (batch,row) over columns, stage-major, bias last, every multiply and
 * add rounded separately (native/src/stage_codec.cpp:274-326).  Bit-identical to the
 * reference's CPU result. */
HQB_API int hqb_raw_linear_ordered(const hqb_geometry* g, const hqb_raw_stage_f32* stages,
                                   uint32_t stage_count, uint32_t prefix, const float* x,
                                   uint64_t batch, const float* bias, float* y, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HARPQ_B200_H_ */
