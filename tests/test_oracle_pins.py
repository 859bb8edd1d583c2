"""Pin the CPU oracle to the reference's own known-answer tests.

The reference (Go 1.27 GOEXPERIMENT=simd) cannot run here, so the oracle is
checked against every known answer and independent float64 reference its
test suite holds for the MoE path (paths relative to the Stream-PT root):

  TestMXFP4Dot                          tests/testdata/forward/pipeline_test.go:176-201
  TestMXFP4AllScales                    tests/testdata/forward/mxfp4_optimization_test.go:52-78
  TestMXFP4NibbleReference              tests/testdata/forward/mxfp4_optimization_test.go:12-50
  TestSIMDKernelMXFP4DecodeAllEncodings tests/testdata/forward/simd_kernels_test.go:211-246
  TestSIMDKernelGather                  tests/testdata/forward/simd_kernels_test.go:27-72
  TestSIMDKernelRouter                  tests/testdata/forward/simd_kernels_test.go:99-153
  TestGPTOSSExpertBiasesAndSwiGLU       tests/testdata/forward/inference_regression_test.go:44-103
  TestSparseMoEIndependentReference     tests/testdata/forward/moe_sparse_test.go:78-105
  TestForwardMoEBatchMatchesSequential  tests/testdata/forward/moe_batch_test.go:125-168
"""
import math

import numpy as np
import pytest

import refdata
from oracle import oracle
from refdata import bits_equal

LEVELS = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, 0, -.5, -1, -1.5, -2, -3, -4, -6], np.float64)


def test_mxfp4_dot_known_answer():
    row = np.zeros(17, np.uint8)
    row[0] = 127
    row[1:] = 0x22
    x = np.full(32, 2.0, np.float32)
    y = np.zeros(1, np.float32)
    oracle.mul_moe_batch_expert(row, 32, 1, x, [0], None, y, [0])
    assert abs(float(y[0]) - 64.0) <= 1e-4


def test_mxfp4_all_scales():
    data = np.zeros(257 * 17, np.uint8)
    for s in range(256):
        data[s * 17] = s
        data[s * 17 + 1: s * 17 + 17] = 0x22
    data[256 * 17] = 255  # Inf scale times zero must remain NaN, not become zero.
    x = np.full(32, 1.0 / 32, np.float32)
    out = np.zeros(257, np.float32)
    oracle.mul_moe_batch_expert(data, 32, 257, x, [0], None, out, [0], workers=8)
    for s in range(256):
        want = np.float32(math.ldexp(1.0, s - 127)) if s < 255 else np.float32(np.inf)
        assert out[s] == want, (s, out[s], want)
    assert np.isnan(out[256])


def test_decode_all_encodings():
    scale = np.repeat(np.arange(256, dtype=np.uint8), 256)
    packed = np.tile(np.arange(256, dtype=np.uint8), 256)
    row = np.empty((65536, 17), np.uint8)
    row[:, 0] = scale
    row[:, 1:] = packed[:, None]
    got = oracle.decode_mxfp4(row.reshape(-1)).reshape(65536, 32)
    lv = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, -0.0, -.5, -1, -1.5, -2, -3, -4, -6], np.float32)
    factor = np.array([np.float32(math.ldexp(1.0, s - 127)) if s < 255 else np.float32(np.inf)
                       for s in range(256)], np.float32)
    nib = np.concatenate([np.repeat((packed & 15)[:, None], 16, 1), np.repeat((packed >> 4)[:, None], 16, 1)], 1)
    with np.errstate(invalid="ignore", over="ignore"):
        want = (factor[scale][:, None] * lv[nib]).astype(np.float32)
    assert bits_equal(got, want).all()


@pytest.mark.parametrize("input_", [32, 96, 2880])
def test_mxfp4_nibble_reference(input_):
    rows, blocks = 256, input_ // 32
    x = ((np.arange(input_) % 23 - 11).astype(np.float32) / np.float32(32)).astype(np.float32)
    data = np.zeros((rows, blocks, 17), np.uint8)
    want = np.zeros(rows)
    r = np.arange(rows)[:, None, None]
    b = np.arange(blocks)[None, :, None]
    i = np.arange(16)[None, None, :]
    packed = ((r + b * 7 + i * 11) & 0xFF).astype(np.uint8)
    data[:, :, 0] = (120 + np.arange(blocks) % 12)[None, :]
    data[:, :, 1:] = packed
    scale = np.ldexp(1.0, data[:, :, 0].astype(np.int64) - 127)
    xb = x.reshape(blocks, 32).astype(np.float64)
    want = (scale[:, :, None] * (LEVELS[packed & 15] * xb[None, :, :16] + LEVELS[packed >> 4] * xb[None, :, 16:])).sum((1, 2))
    for workers in (1, 8):
        out = np.zeros(rows, np.float32)
        oracle.mul_moe_batch_expert(data.reshape(-1), input_, rows, x, [0], None, out, [0], workers)
        assert np.all(np.abs(out - want) <= 3e-5 * np.maximum(1, np.abs(want)))


@pytest.mark.parametrize("input_", [32, 96, 2880])
@pytest.mark.parametrize("count", [1, 2, 3, 4, 8, 16])
def test_gather_scatter(input_, count):
    row, vector = refdata.simd_kernel_row(input_)
    output = 3
    data = np.tile(row, output)
    x = np.zeros(count * (input_ + 1), np.float32)
    y = np.zeros(count * (output + 1), np.float32)
    starts = [(count - 1 - t) * (input_ + 1) + 1 for t in range(count)]
    ends = [t * (output + 1) + 1 for t in range(count)]
    bias = np.array([.125, -.25, .5], np.float32)
    for t in range(count):
        x[starts[t]: starts[t] + input_] = vector * np.float32(t + 1)
    oracle.mul_moe_batch_expert(data, input_, output, x, starts, bias, y, ends)
    nb = input_ // 32
    rb = row.reshape(nb, 17)
    scale = np.ldexp(1.0, rb[:, 0].astype(np.int64) - 127)
    for t, s in enumerate(starts):
        xb = x[s: s + input_].astype(np.float64).reshape(nb, 32)
        want = (scale[:, None] * (LEVELS[rb[:, 1:] & 15] * xb[:, :16] + LEVELS[rb[:, 1:] >> 4] * xb[:, 16:])).sum()
        for i, bv in enumerate(bias):
            exp = want + float(bv)
            got = float(y[ends[t] + i])
            assert not math.isnan(got) and abs(got - exp) <= 3e-5 * max(1, abs(exp))
        assert y[t * (output + 1)] == 0  # sentinel untouched


@pytest.mark.parametrize("hidden", [3, 31, 32, 96, 2880])
@pytest.mark.parametrize("batch", [1, 2, 17])
def test_router(hidden, batch):
    experts = 5
    bias = np.array([.125, -.25, .5, -1, 2], np.float32)
    n = experts * hidden
    w = ((np.arange(n) % 23 - 11).astype(np.float32) / np.float32(64)).astype(np.float32)
    storage = np.zeros(n * 4 + 1, np.uint8)
    storage[1:] = np.frombuffer(w.astype("<f4").tobytes(), np.uint8)
    data = storage[1:]  # deliberately unaligned view
    x = ((np.arange(batch * hidden) % 31 - 15).astype(np.float32) / np.float32(32)).astype(np.float32)
    logits = oracle.route(data, x, bias, batch, hidden, experts)
    want = (x.reshape(batch, 1, hidden).astype(np.float64) * w.reshape(1, experts, hidden)).sum(-1) + bias
    assert np.all(np.abs(logits - want) <= 3e-5 * np.maximum(1, np.abs(want)))
    for value in (np.nan, np.inf, -np.inf):
        d2 = data.copy()
        d2[:4] = np.frombuffer(np.float32(value).tobytes(), np.uint8)
        x2 = x.copy()
        x2[0] = 1
        got = oracle.route(d2, x2, bias, batch, hidden, experts)[0, 0]
        if np.isnan(value):
            assert np.isnan(got)
        else:
            assert got == value


def test_router_exact_order_matches_avx2_layout():
    """hidden%32==0 uses the dotF32AVX2 chains; spot-check against a direct
    restatement of its 8x8-lane accumulation in numpy float32."""
    hidden = 2880 + 32  # exercises the 32-element tail loop
    rng = np.random.default_rng(7)
    w = rng.standard_normal(hidden).astype(np.float32)
    x = rng.standard_normal(hidden).astype(np.float32)
    acc = np.zeros((8, 8), np.float32)
    o = 0
    while o + 64 <= hidden:
        for j in range(8):
            acc[j] = _fma32(w[o + 8 * j: o + 8 * j + 8], x[o + 8 * j: o + 8 * j + 8], acc[j])
        o += 64
    while o < hidden:
        for j in range(4):
            acc[j] = _fma32(w[o + 8 * j: o + 8 * j + 8], x[o + 8 * j: o + 8 * j + 8], acc[j])
        o += 32
    s0 = ((acc[0] + acc[1]) + acc[2]) + acc[3]
    s1 = ((acc[4] + acc[5]) + acc[6]) + acc[7]
    s = (s0 + s1).astype(np.float32)
    p = (s[:4] + s[4:]).astype(np.float32)
    want = np.float32((p[0] + p[1]) + (p[2] + p[3]))
    got = oracle.route(np.frombuffer(w.tobytes(), np.uint8), x, None, 1, hidden, 1)[0, 0]
    assert got.view(np.uint32) == want.view(np.uint32)


def _fma32(a, b, c):
    """Single-rounding float32 fma (C fmaf through the oracle library)."""
    return oracle.fmaf(a, b, c)


def test_mxfp4_avx2_equals_scalar_chains():
    rng = np.random.default_rng(3)
    for input_ in (32, 96, 2880):
        row = rng.integers(0, 256, input_ // 32 * 17, dtype=np.uint8)
        row[::17] = rng.integers(100, 140, input_ // 32)
        x = rng.standard_normal(input_).astype(np.float32)
        a = oracle.dot_mxfp4(row, x)
        b = oracle.dot_mxfp4(row, x, scalar=True)
        assert np.float32(a).view(np.uint32) == np.float32(b).view(np.uint32)


def test_f16_decode_all_patterns():
    L = oracle.lib()
    got = np.array([L.spo_f16(b) for b in range(65536)], np.float32)
    want = np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32)
    assert bits_equal(got, want).all()


def test_swiglu_known_answer():
    fx = refdata.swiglu_fixture()
    out = oracle.forward_moe_batch(fx.dense, np.zeros(32, np.float32), 1)
    want = 7 / (1 + math.exp(-1.702 * 7)) * 8 + 5
    assert np.all(np.abs(out - want) <= 1e-5)


@pytest.mark.parametrize("mode", ["ties", "normal", "underflow"])
@pytest.mark.parametrize("k", [1, 2, 8])
def test_sparse_independent_reference(mode, k):
    fx = refdata.moe_batch_fixture(96, 64, 8, k, -1, mode)
    batch = 19
    x = ((np.arange(batch * 96) % 13 + 1).astype(np.float32) / np.float32(16)).astype(np.float32)
    for workers in (1, 4):
        out = oracle.forward_moe_batch(fx.dense, x, batch, workers)
        for t in range(batch):
            want = oracle.scalar_sparse_moe_f64(fx.dense, x[t * 96:(t + 1) * 96])
            assert np.all(np.abs(out[t] - want) <= 3e-5 * np.maximum(1, np.abs(want))), (t,)


@pytest.mark.parametrize("experts", [1, 4, 7])
@pytest.mark.parametrize("bias_type", [-1, 0, 1, 30])
def test_batch_matches_sequential(experts, bias_type):
    for top_k in sorted({1, min(2, experts), experts}):
        for mode in refdata.ROUTER_MODES:
            fx = refdata.moe_batch_fixture(96, 64, experts, top_k, bias_type, mode)
            for batch in (1, 5, 37):
                x = refdata.moe_batch_x(batch, 96, mode)
                orig = x.copy()
                want = np.concatenate([oracle.forward_moe_batch(fx.dense, x[t * 96:(t + 1) * 96], 1)
                                       for t in range(batch)])
                for workers in (1, 3):
                    got = oracle.forward_moe_batch(fx.dense, x, batch, workers)
                    assert bits_equal(got, want).all(), (top_k, mode, batch, workers)
                assert np.array_equal(x.view(np.uint32), orig.view(np.uint32))


def test_select_rules():
    # ties -> lowest index; NaN never chosen; no candidate -> (rank, 0)
    sel = oracle.select(np.array([1, 3, 3, np.nan, 2], np.float32), 3)
    assert [s[0] for s in sel] == [1, 2, 4]
    sel = oracle.select(np.array([np.nan, np.nan, np.nan], np.float32), 2)
    assert [s[0] for s in sel] == [0, 1]
    assert all(s[1] == np.float32(0.5) for s in sel)
    # +Inf everywhere: exp(Inf-Inf) = NaN weights, no normalisation
    sel = oracle.select(np.array([np.inf, np.inf], np.float32), 2)
    assert [s[0] for s in sel] == [0, 1] and all(np.isnan(s[1]) for s in sel)
    # underflow: exp(-1000) == 0
    sel = oracle.select(np.array([0, 1000, 2000], np.float32), 2)
    assert sel[0] == (2, np.float32(1)) and sel[1][1] == 0
