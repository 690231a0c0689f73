"""The bench's roofline numerator (algorithmic bytes), on the CPU.

Per stage a layer holds its int2 codes (4 per byte) and one FP16 scale per row and 128-column
group, i.e. 17·N·K/64 bytes for N, K multiples of 128 (the reference's own stage format,
quantization.py pack / scale shape [N/128, K/128, 128, 1]). The numerator adds the FP16 input
and output vectors. These tests pin bench.py's formula to that count and to the per-config
figures it reports.
"""

from __future__ import annotations

import pytest

pytest.importorskip("torch")

import bench  # noqa: E402


def _stage_bytes(rows, cols):
    groups = -(-cols // 128)
    return rows * cols // 4 + rows * groups * 2


@pytest.mark.parametrize("rows,cols,prefix,mb", [
    (4096, 4096, 1, 4.473), (4096, 4096, 2, 8.929), (4096, 4096, 3, 13.386), (4096, 4096, 4, 17.842),
    (11008, 4096, 1, 12.007), (11008, 4096, 2, 23.984), (11008, 4096, 4, 47.937),
    (4096, 11008, 2, 23.984), (28672, 8192, 3, 187.245), (8192, 28672, 3, 187.245)])
def test_layer_bytes(rows, cols, prefix, mb):
    b = bench.algorithmic_bytes(rows, cols, prefix)
    assert b == prefix * _stage_bytes(rows, cols) + 2 * cols + 2 * rows
    assert abs(b / 1e6 - mb) < 5e-4
    assert prefix * _stage_bytes(rows, cols) == prefix * 17 * rows * cols // 64


def test_stacked_launch_bytes_count_the_shared_input_once():
    members = [{"nrows": 4096}, {"nrows": 4096}, {"nrows": 4096}]  # q, k, v
    stacked = bench.group_bytes(members, 4096, 2)
    separate = sum(bench.algorithmic_bytes(4096, 4096, 2) for _ in members)
    assert stacked == separate - 2 * 2 * 4096  # two of the three FP16 input reads are shared


def test_llama7b_block_step_bytes():
    prefix, layers, _ = bench.WORKLOADS["llama7b_block_p2"]
    assert prefix == 2 and len(layers) == 7
    per_layer = sum(bench.algorithmic_bytes(r, c, prefix) for _, r, c, _ in layers)
    assert abs(per_layer / 1e6 - 107.67) < 0.01
