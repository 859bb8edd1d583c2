"""Pins of the oracle's Q8_0 LM-head arithmetic (MulQ80Into / MulQ80Argmax).

The oracle (oracle/spt_oracle.c spo_dot_q80, spo_mul_q80) restates
quantQ80AVX2 / quantQ80PairAVX2 (forward/quant_amd64.go:17-45, 92-110):
32 FMA chains (chain c = element c of every 32-element block, weight =
int8 * float16 scale, exact), the a0+a1+a2+a3 / quantSumAVX2 tree, and the
argmax rule of forward/q80.go:64-104 (largest logit, lowest row on ties,
NaN never chosen, row 0 when nothing beats -Inf).  The fixtures are the
reference tests' own byte formulas:
  TestQ80Dot                      tests/testdata/forward/pipeline_test.go:146-172
  TestQuantRowsPairSpecial        tests/testdata/forward/quant_rows_test.go:135-170
  TestMulQ80Into                  tests/testdata/forward/sampling_test.go:179-209
  TestQuantOptimizationNumerics   tests/testdata/forward/quant_optimization_test.go:127-180
"""
import os
import struct
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from oracle import oracle  # noqa: E402
from tests.refdata import q80_fixture, q80_reference_dot  # noqa: E402


def f16(bits):
    return np.frombuffer(struct.pack("<H", bits), np.float16)[0].astype(np.float32)


def test_q80_dot_known_answer():
    row = np.zeros(34, np.uint8)
    row[:2] = np.frombuffer(struct.pack("<H", 0x3C00), np.uint8)
    row[2:] = (np.arange(32) - 16).astype(np.int8).view(np.uint8)
    assert oracle.dot_q80(row, np.ones(32, np.float32)) == np.float32(-16.0)


def test_q80_every_scale():
    """All 65,536 float16 scales with q = 1 and x = 1: every chain holds the
    scale, the tree sums 32 equal values exactly (zeros sum to +0)."""
    rows = np.ones((65536, 34), np.uint8)
    rows[:, :2] = np.arange(65536, dtype=np.uint16).view(np.uint8).reshape(-1, 2)
    y, _, _ = oracle.mul_q80(rows.reshape(-1), 32, 65536, np.ones(32, np.float32), workers=8)
    scales = np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32)
    want = (scales * np.float32(32)).astype(np.float32)
    want[scales == 0] = np.float32(0.0)  # fma(-0, 1, +0) = +0
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(y), nan)
    assert np.array_equal(y[~nan].view(np.uint32), want[~nan].view(np.uint32))


@pytest.mark.parametrize("input_", [32, 96, 512])
def test_q80_rows_match_reference_sum(input_):
    data, x = q80_fixture(input_, 17, x_kind="opt")
    y, best, logit = oracle.mul_q80(data, input_, 17, x)
    rb = input_ // 32 * 34
    want = np.array([q80_reference_dot(data[r * rb:(r + 1) * rb], x) for r in range(17)], np.float32)
    tol = 1e-4 * (1 + np.abs(want))  # compareVectors (rmsnorm_test.go:209-223)
    assert np.all(np.abs(y - want) <= tol)
    assert best == int(np.argmax(y)) and logit == y[best]


def test_mul_q80_into_fixture():
    data, x = q80_fixture(96, 17, x_kind="into")
    y, _, _ = oracle.mul_q80(data, 96, 17, x)
    want = np.array([q80_reference_dot(data[r * 102:(r + 1) * 102], x) for r in range(17)], np.float32)
    assert np.all(np.abs(y - want) <= 1e-4 * (1 + np.abs(want)))


def test_q80_argmax_rule():
    """Ties go to the lowest row; NaN rows never win; -Inf everywhere -> row 0."""
    blk = np.zeros(34, np.uint8)

    def row(scale_bits, q):
        r = blk.copy()
        r[:2] = np.frombuffer(struct.pack("<H", scale_bits), np.uint8)
        r[2:] = np.full(32, q, np.int8).view(np.uint8)
        return r

    x = np.ones(32, np.float32)
    rows = np.stack([row(0x3C00, 1), row(0x3C00, 3), row(0x7E00, 1), row(0x3C00, 3)])  # 32, 96, NaN, 96
    y, best, logit = oracle.mul_q80(rows.reshape(-1), 32, 4, x)
    assert best == 1 and logit == np.float32(96)
    rows = np.stack([row(0xFC00, 1), row(0xFC00, 1)])  # -Inf, -Inf
    y, best, logit = oracle.mul_q80(rows.reshape(-1), 32, 2, x)
    assert best == 0 and np.isneginf(logit)
