"""Pins of the oracle's Q4_0 arithmetic (MulQ40Into / MulQ40BatchInto).

The oracle (oracle/spt_oracle.c spo_dot_q40, spo_dot_q40_batch,
spo_mul_q40) restates the reference's two AVX2 orders:
  one input  quantQ40AVX2 (forward/quant_amd64.go:75-90): 32 FMA chains,
             chain c = element c of every block, a0+a1+a2+a3, quantSumAVX2;
  a batch    quantDotQ40Batch (forward/quant_amd64.go:118-148): one 8-lane
             accumulator per item, lane l takes elements l, 8+l, 16+l, 24+l
             of each block, then quantSumAVX2;
with weight = (nibble - 8) * float16 scale (exact), element c the low
nibble of byte c (c < 16) or the high nibble of byte c - 16
(quantQ40WeightsAVX2, :65-73).  MulQ40BatchInto takes the first for batch 1
and the second otherwise (forward/q40.go:87-92).  The fixtures are the
reference tests' own:
  TestDotQ40, TestDotQ40TwoBlocks       tests/testdata/forward/q40_test.go:12-50
  TestMulQ40StreamingBatch              tests/testdata/forward/q40_stream_test.go:69-105
  TestQuantOptimizationFloat16Scales    tests/testdata/forward/quant_optimization_test.go:64-113
  TestQuantOptimizationNumerics         tests/testdata/forward/quant_optimization_test.go:127-180
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
from tests.refdata import q40_fixture, q40_reference_dot, q40_stream_x  # noqa: E402


def block(scale_bits, fill=0):
    b = np.full(18, fill, np.uint8)
    b[:2] = np.frombuffer(struct.pack("<H", scale_bits), np.uint8)
    return b


def test_dot_q40_known_answer():
    b = block(0x3C00)
    b[2] = 0x0F  # first weight 7 (nibble 15), seventeenth -8 (nibble 0)
    x = np.zeros(32, np.float32)
    x[0], x[16] = 2, 3
    assert oracle.dot_q40(b, x) == np.float32(7 * 2 - 8 * 3)
    assert oracle.mul_q40(b, 32, 1, x)[0, 0] == np.float32(7 * 2 - 8 * 3)


def test_dot_q40_two_blocks():
    row = np.concatenate([block(0x3C00, 0x88), block(0x3C00, 0x88)])
    row[18 + 2] = 0x89
    x = np.zeros(64, np.float32)
    x[32] = 5
    assert oracle.dot_q40(row, x) == np.float32(5)


def test_q40_every_scale():
    """All 65,536 float16 scales, weight bytes 0x99 (both nibbles +1), x = 1:
    the result is 32 * scale exactly (NaN for NaN scales), in both orders."""
    rows = np.full((65536, 18), 0x99, np.uint8)
    rows[:, :2] = np.arange(65536, dtype=np.uint16).view(np.uint8).reshape(-1, 2)
    scales = np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        want = (scales * np.float32(32)).astype(np.float32)
    want[scales == 0] = np.float32(0.0)
    nan = np.isnan(want)
    for batch in (1, 2):
        y = oracle.mul_q40(rows.reshape(-1), 32, 65536, np.ones(32 * batch, np.float32), batch, workers=8)
        for item in range(batch):
            assert np.array_equal(np.isnan(y[item]), nan)
            assert np.array_equal(y[item][~nan].view(np.uint32), want[~nan].view(np.uint32))


@pytest.mark.parametrize("batch", [1, 3, 9, 19])
def test_q40_streaming_batch_fixture(batch):
    """TestMulQ40StreamingBatch: input 96, output 11, batches 1, 3, lanes+1
    (AVX2: 9) and 19, against referenceQ40Dot within compareVectors'
    tolerance 1e-4 * (1 + |want|)."""
    input_, output = 96, 11
    data = q40_fixture(input_, output, "stream")
    x = q40_stream_x(batch, input_)
    y = oracle.mul_q40(data, input_, output, x, batch, workers=3)
    rb = input_ // 32 * 18
    for item in range(batch):
        want = np.array([q40_reference_dot(data[r * rb:(r + 1) * rb], x[item * input_:(item + 1) * input_])
                         for r in range(output)], np.float32)
        assert np.all(np.abs(y[item] - want) <= 1e-4 * (1 + np.abs(want))), item


@pytest.mark.parametrize("input_", [32, 96, 512])
def test_q40_optimization_numerics(input_):
    data = q40_fixture(input_, 17, "opt")
    i = np.arange(input_)
    x = ((i % 23 - 11) / 32).astype(np.float32)
    y = oracle.mul_q40(data, input_, 17, x)[0]
    rb = input_ // 32 * 18
    want = np.array([q40_reference_dot(data[r * rb:(r + 1) * rb], x) for r in range(17)], np.float32)
    finite = np.isfinite(want)
    assert np.array_equal(np.isfinite(y), finite)
    assert np.all(np.abs(y[finite] - want[finite]) <= 1e-4 * (1 + np.abs(want[finite])))


def _chains_one(row, x):
    """quantQ40AVX2's chains, restated as plain float32 loops."""
    a = np.zeros(32, np.float32)
    for b in range(len(row) // 18):
        s = np.frombuffer(bytes(row[18 * b:18 * b + 2]), np.float16)[0].astype(np.float32)
        for c in range(32):
            n = int(row[18 * b + 2 + (c & 15)] >> (4 * (c >> 4))) & 15
            a[c] = np.float32(np.float64(np.float32(np.float32(n - 8) * s)) * np.float64(x[32 * b + c])
                              + np.float64(a[c]))
    s8 = [np.float32(np.float32(np.float32(a[l] + a[8 + l]) + a[16 + l]) + a[24 + l]) for l in range(8)]
    p = [np.float32(s8[i] + s8[4 + i]) for i in range(4)]
    return np.float32(np.float32(p[0] + p[1]) + np.float32(p[2] + p[3]))


def _chains_batch(row, x):
    """quantDotQ40Batch's 8 lanes for one item, restated as plain loops."""
    a = np.zeros(8, np.float32)
    for b in range(len(row) // 18):
        s = np.frombuffer(bytes(row[18 * b:18 * b + 2]), np.float16)[0].astype(np.float32)
        for j in range(4):
            for l in range(8):
                c = 8 * j + l
                n = int(row[18 * b + 2 + (c & 15)] >> (4 * (c >> 4))) & 15
                a[l] = np.float32(np.float64(np.float32(np.float32(n - 8) * s)) * np.float64(x[32 * b + c])
                                  + np.float64(a[l]))
    p = [np.float32(a[i] + a[4 + i]) for i in range(4)]
    return np.float32(np.float32(p[0] + p[1]) + np.float32(p[2] + p[3]))


def test_q40_orders_restated():
    """The C oracle's two orders equal an independent loop restatement bit
    for bit (fp32 fma emulated through float64, exact for these products:
    the weights have 15 significant bits and x has 5)."""
    input_, output, batch = 96, 5, 3
    data = q40_fixture(input_, output, "stream")
    x = q40_stream_x(batch, input_)
    rb = input_ // 32 * 18
    y1 = oracle.mul_q40(data, input_, output, x[:input_], 1)[0]
    yb = oracle.mul_q40(data, input_, output, x, batch)
    for r in range(output):
        row = data[r * rb:(r + 1) * rb]
        assert y1[r].view(np.uint32) == _chains_one(row, x[:input_]).view(np.uint32)
        for item in range(batch):
            want = _chains_batch(row, x[item * input_:(item + 1) * input_])
            assert yb[item, r].view(np.uint32) == want.view(np.uint32)
