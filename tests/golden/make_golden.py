"""Generate the committed golden fixtures from the reference implementation itself.

Run in a container where the reference checkout exists (default path below, or
``--reference``).  It never runs on the GPU box; the tests only read its outputs.

What it writes (all under tests/golden/):

* ``native_golden.npz`` — the values of the reference's checked-in C++ fixture
  ``native/tests/generated/golden_vectors.hpp`` (5x9 matrix, tile 4x8, group 4,
  four stage payloads, CRC32Cs, batch-2 inputs, bias, exact prefix weights for
  prefixes 0..4 and scalar-order outputs).  Before parsing, the script re-renders
  the header with the reference's own generator (scripts/generate_native_golden.py)
  and requires it to be byte-identical to the checked-in file, so the fixture is
  exactly what the reference's code produces.
* ``seeded_<name>.npz`` — seeded 128x128/group-128 matrices quantized by the
  reference's ``quantize_progressive`` and serialized by ``encode_stage_payload``,
  with inputs, bias, per-prefix SHA-256 of the reference's ``dequantize_prefix``
  (FP32 bytes), the reference's ``progressive_matmul`` outputs, and the payload
  CRC32Cs from the reference's ``integrity.crc32c``.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib.util
import os
import re
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# (name, rows, cols, weight std, seed, batch)
SEEDED_CASES = [
    ("tile1", 128, 128, 0.02, 303, 2),
    ("ragged", 137, 259, 0.02, 101, 3),
    ("grid2", 256, 256, 0.05, 202, 4),
]


def _load_reference(ref: Path):
    sys.path.insert(0, str(ref / "src"))
    from harpq import integrity, matrix_codec, quantization  # type: ignore

    spec = importlib.util.spec_from_file_location(
        "ref_generate_native_golden", ref / "scripts" / "generate_native_golden.py")
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)  # type: ignore[union-attr]
    return quantization, matrix_codec, integrity, gen


def _parse_array_block(text: str, name: str) -> list[str]:
    start = text.index(name)
    body_start = text.index("{{", start) + 2
    depth, i = 1, body_start
    while depth:
        if text.startswith("{{", i):
            depth += 1
            i += 2
        elif text.startswith("}}", i):
            depth -= 1
            i += 2
        else:
            i += 1
    return [tok for tok in re.split(r"[\s,{}]+", text[body_start:i - 2]) if tok]


def _float(tok: str) -> float:
    return float.fromhex(tok.rstrip("F"))


def native_fixture(ref: Path, gen) -> dict:
    header_path = ref / "native" / "tests" / "generated" / "golden_vectors.hpp"
    text = header_path.read_text(encoding="utf-8")
    if gen.render_header() != text:
        raise SystemExit("reference golden header does not match its own generator")
    geo = re.search(r"kGeometry\{([^}]*)\}", text).group(1)
    geometry = np.array([int(v) for v in geo.split(",")], np.uint64)
    scale_shape = np.array([int(v) for v in re.search(r"kScaleShape\{([^}]*)\}", text).group(1).split(",")], np.uint64)
    payload_bytes = int(re.search(r"kPayloadBytes = (\d+)", text).group(1))
    payloads = np.array([int(t, 16) for t in _parse_array_block(text, "kStagePayloads")], np.uint8)
    payloads = payloads.reshape(-1, payload_bytes)
    crcs = np.array([int(t.rstrip("U"), 16) for t in _parse_array_block(text, "kStageCrc32c")], np.uint32)
    inputs = np.array([_float(t) for t in _parse_array_block(text, "kInputs")], np.float32)
    bias = np.array([_float(t) for t in _parse_array_block(text, "kBias")], np.float32)
    weights = np.array([_float(t) for t in _parse_array_block(text, "kPrefixWeights")], np.float32)
    outputs = np.array([_float(t) for t in _parse_array_block(text, "kPrefixOutputs")], np.float32)
    rows, cols = int(geometry[0]), int(geometry[1])
    return dict(geometry=geometry, scale_shape=scale_shape, payloads=payloads, crc32c=crcs,
                inputs=inputs.reshape(2, cols), bias=bias,
                prefix_weights=weights.reshape(5, rows, cols),
                prefix_outputs=outputs.reshape(5, 2, rows),
                header_sha256=np.frombuffer(hashlib.sha256(text.encode()).digest(), np.uint8))


def seeded_fixture(quantization, matrix_codec, integrity, name, rows, cols, std, seed, batch) -> dict:
    rng = np.random.default_rng(seed)
    weights = rng.normal(0.0, std, size=(rows, cols)).astype(np.float32)
    x = rng.standard_normal((batch, cols)).astype(np.float16).astype(np.float32)
    bias = rng.normal(0.0, 0.1, size=(rows,)).astype(np.float32)
    q = quantization.quantize_progressive(weights)
    payloads = [matrix_codec.encode_stage_payload(st, i) for i, st in enumerate(q.stages)]
    lengths = np.array([len(p) for p in payloads], np.uint64)
    digests, outputs = [], []
    for prefix in range(q.stage_count + 1):
        w = quantization.dequantize_prefix(q, prefix)
        digests.append(np.frombuffer(hashlib.sha256(np.ascontiguousarray(w, np.float32).tobytes()).digest(), np.uint8))
        outputs.append(quantization.progressive_matmul(x, q, prefix=prefix, bias=bias))
    out = dict(
        geometry=np.array([rows, cols, *q.padded_shape, *q.tile_shape, q.group_size], np.uint64),
        weights=weights, x=x, bias=bias,
        payloads=np.frombuffer(b"".join(payloads), np.uint8), payload_lengths=lengths,
        crc32c=np.array([integrity.crc32c(p) for p in payloads], np.uint32),
        prefix_sha256=np.stack(digests), prefix_outputs=np.stack(outputs).astype(np.float32),
    )
    if rows * cols <= 128 * 128:
        out["prefix4_weights"] = quantization.dequantize_prefix(q, 4).astype(np.float32)
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    default_ref = Path(os.environ.get("HQB_REFERENCE", str(Path(__file__).resolve().parents[3] / "reference")))
    ap.add_argument("--reference", type=Path, default=default_ref,
                    help="reference checkout ($HQB_REFERENCE, else 'reference' beside this repository)")
    ap.add_argument("--check", action="store_true", help="fail if committed fixtures differ")
    args = ap.parse_args(argv)
    quantization, matrix_codec, integrity, gen = _load_reference(args.reference)
    produced = {"native_golden.npz": native_fixture(args.reference, gen)}
    for case in SEEDED_CASES:
        produced[f"seeded_{case[0]}.npz"] = seeded_fixture(quantization, matrix_codec, integrity, *case)
    drift = []
    for fname, arrays in produced.items():
        path = HERE / fname
        if args.check:
            old = np.load(path)
            if set(old.files) != set(arrays) or any(not np.array_equal(old[k], arrays[k]) for k in arrays):
                drift.append(fname)
        else:
            np.savez_compressed(path, **arrays)
    if drift:
        print("golden fixtures drifted:", ", ".join(drift), file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
