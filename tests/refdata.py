"""The reference tests' deterministic fixtures, restated for the parity suite.

Each builder reproduces the byte formulas of a Stream-PT test helper (paths
relative to the Stream-PT repository root) and returns both the "file" bytes
with tensor descriptors (for the C ABI) and the decoded arrays the CPU oracle
takes:

  moe_batch_fixture   tests/testdata/forward/moe_batch_test.go:20-111
  moe_batch_x         tests/testdata/forward/moe_batch_test.go:133-139
  simd_kernel_row     tests/testdata/forward/simd_kernels_test.go:12-24
  swiglu_fixture      tests/testdata/forward/inference_regression_test.go:44-103
"""
from __future__ import annotations

import importlib
import struct
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
spt = importlib.import_module("stream-pt_b200")
from oracle import oracle  # noqa: E402

ROUTER_MODES = ("normal", "ties", "nonfinite", "mixed-nan", "infinite", "underflow", "clamp")
F16_BITS = (0xB800, 0xB400, 0x0000, 0x3400, 0x3800)  # -0.5 -0.25 0 0.25 0.5


class Fixture:
    """A synthetic weight file plus the decoded inputs of the oracle."""

    def __init__(self, cfg, lw, data: bytearray, dense: oracle.Weights):
        self.cfg = cfg
        self.lw = lw
        self.data = bytes(data)
        self.reader = spt.Reader(self.data)
        self.dense = dense


def _quantized(input_, output, experts, salt) -> np.ndarray:
    nblocks = input_ // 32 * output * experts
    blk = np.arange(nblocks, dtype=np.int64)[:, None]
    i = np.arange(1, 17, dtype=np.int64)[None, :]
    enc = np.empty((nblocks, 17), np.uint8)
    enc[:, 0] = (120 + (blk[:, 0] + salt) % 4).astype(np.uint8)
    enc[:, 1:] = ((blk * 13 + i * 7 + salt) & 0xFF).astype(np.uint8)
    return enc.reshape(-1)


def _bias_bytes(dim, count, bias_type) -> tuple[bytes, np.ndarray]:
    n = dim * count
    i = np.arange(n)
    value = ((i % 5 - 2).astype(np.float32) / np.float32(4)).astype(np.float32)
    if bias_type == 0:
        return value.astype("<f4").tobytes(), value
    if bias_type == 30:
        bits = (value.view(np.uint32) >> 16).astype("<u2")
        return bits.tobytes(), (bits.astype(np.uint32) << 16).view(np.float32)
    bits = np.array([F16_BITS[k % 5] for k in range(n)], dtype="<u2")
    return bits.tobytes(), bits.view(np.float16).astype(np.float32)


def moe_batch_fixture(hidden, expert_dim, experts, top_k, bias_type, router_mode) -> Fixture:
    data = bytearray(37)

    def append(name, typ, shape, encoded: bytes):
        start = len(data)
        data.extend(encoded)
        return spt.Tensor(name, typ, shape, start, len(data))

    e = np.arange(experts)[:, None]
    i = np.arange(hidden)[None, :]
    router = ((e * 7 + i * 3) % 19 - 9).astype(np.float32) / np.float32(32)
    if router_mode == "ties":
        router[:] = 0
    elif router_mode == "nonfinite":
        router[:] = np.nan
    elif router_mode == "mixed-nan":
        router[:] = np.nan
        if experts > 1:
            router[1, :] = 0
    elif router_mode == "infinite":
        router[:] = np.inf
    elif router_mode == "underflow":
        router[:] = (e * 1000).astype(np.float32) * np.ones_like(router)
    router_bytes = router.astype("<f4").tobytes()
    lw = spt.LayerWeights()
    lw.ffn_gate_inp = append("router", 0, [hidden, experts], router_bytes)
    gate = _quantized(hidden, expert_dim, experts, 1)
    up = _quantized(hidden, expert_dim, experts, 7)
    down = _quantized(expert_dim, hidden, experts, 17)
    lw.ffn_gate_exps = append("gate", 39, [hidden, expert_dim, experts], gate.tobytes())
    lw.ffn_up_exps = append("up", 39, [hidden, expert_dim, experts], up.tobytes())
    lw.ffn_down_exps = append("down", 39, [expert_dim, hidden, experts], down.tobytes())
    rb = gb = ub = db = None
    if bias_type >= 0:
        def bias(name, dim, count, vector):
            raw, dec = _bias_bytes(dim, count, bias_type)
            shape = [dim] if vector else [dim, count]
            return append(name, bias_type, shape, raw), dec
        lw.ffn_gate_inp_bias, rb = bias("router.bias", experts, 1, True)
        lw.ffn_gate_exps_bias, gb = bias("gate.bias", expert_dim, experts, False)
        lw.ffn_up_exps_bias, ub = bias("up.bias", expert_dim, experts, False)
        lw.ffn_down_exps_bias, db = bias("down.bias", hidden, experts, False)
    cfg = spt.Config(hidden, expert_dim, experts, top_k)
    dense = oracle.Weights(hidden, expert_dim, experts, top_k, np.frombuffer(router_bytes, np.uint8),
                           rb, gate, up, down, gb, ub, db)
    return Fixture(cfg, lw, data, dense)


def moe_batch_x(batch, hidden, mode="normal") -> np.ndarray:
    i = np.arange(batch * hidden, dtype=np.int64)
    x = (((i * 17 + i // hidden) % 31 - 15).astype(np.float32) / np.float32(16)).astype(np.float32)
    if mode == "clamp":
        x = (x * np.float32(1000)).astype(np.float32)
    return x


def simd_kernel_row(input_) -> tuple[np.ndarray, np.ndarray]:
    nb = input_ // 32
    row = np.zeros(nb * 17, np.uint8)
    for b in range(nb):
        row[b * 17] = (123 + b % 8) & 0xFF
        for i in range(16):
            row[b * 17 + i + 1] = (b * 37 + i * 17) & 0xFF
    i = np.arange(input_)
    x = ((i % 31 - 15).astype(np.float32) / np.float32(32)).astype(np.float32)
    return row, x


def f32_bytes(values) -> bytes:
    return np.asarray(values, dtype="<f4").tobytes()


def swiglu_fixture() -> Fixture:
    """TestGPTOSSExpertBiasesAndSwiGLU: dim 32, 2 experts, top-1; router
    zeros with bias [0,1] so expert 1 wins; gate/up weights zero with biases
    10/12; down's first coefficient 1 with bias 5."""
    dim, experts = 32, 2
    data = bytearray()

    def add(name, typ, shape, values: bytes):
        start = len(data)
        data.extend(values)
        return spt.Tensor(name, typ, shape, start, len(data))

    lw = spt.LayerWeights()
    lw.ffn_gate_inp = add("router", 0, [dim, experts], f32_bytes(np.zeros(dim * experts)))
    lw.ffn_gate_inp_bias = add("router.bias", 0, [experts], f32_bytes([0, 1]))
    zero = np.zeros(experts * dim * 17, np.uint8)
    zero[::17] = 127
    lw.ffn_gate_exps = add("gate", 39, [dim, dim, experts], zero.tobytes())
    lw.ffn_up_exps = add("up", 39, [dim, dim, experts], zero.tobytes())
    down = zero.copy()
    down[1::17] = 2  # first coefficient = 1.0
    lw.ffn_down_exps = add("down", 39, [dim, dim, experts], down.tobytes())

    def bias(name, value):
        v = np.zeros(dim * experts, np.float32)
        v[dim:] = value
        return add(name, 0, [dim, experts], f32_bytes(v)), v

    lw.ffn_gate_exps_bias, gb = bias("gate.bias", 10)
    lw.ffn_up_exps_bias, ub = bias("up.bias", 12)
    lw.ffn_down_exps_bias, db = bias("down.bias", 5)
    cfg = spt.Config(dim, dim, experts, 1)
    router = np.frombuffer(f32_bytes(np.zeros(dim * experts)), np.uint8)
    dense = oracle.Weights(dim, dim, experts, 1, router, np.array([0, 1], np.float32), zero, zero,
                           down, gb, ub, db)
    return Fixture(cfg, lw, data, dense)


def bits_equal(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Elementwise Float32bits equality with NaN == NaN (moe_batch_test.go:152)."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return (a.view(np.uint32) == b.view(np.uint32)) | (np.isnan(a) & np.isnan(b))


# ---- Q8_0 fixtures (tests/testdata/forward/quant_optimization_test.go:25-55,
# 115-125; sampling_test.go:179-185) ----------------------------------------
_Q80_SCALES = (0x3C00, 0xB800, 0x3400, 0x0001, 0x03FF, 0x0400, 0x7BFF, 0x8000)


def q80_fixture(input_, output, x_kind="opt"):
    """quantOptimizationFixture(8, input, output) bytes and the test's x."""
    nb = input_ // 32 * output
    data = np.zeros(nb * 34, np.uint8)
    for block in range(nb):
        b = data[block * 34:(block + 1) * 34]
        b[0:2] = np.frombuffer(struct.pack("<H", _Q80_SCALES[block % len(_Q80_SCALES)]), np.uint8)
        for i in range(2, 34):
            b[i] = (block * 13 + i * 7) & 0xFF
    i = np.arange(input_)
    if x_kind == "opt":
        x = ((i % 23 - 11) / 32).astype(np.float32)
    else:
        x = ((i % 7 - 3) / 8).astype(np.float32)
    return data, x


def q80_reference_dot(row, x):
    """referenceQ80Optimization: sequential float32 sum of scale*q*x."""
    s = np.float32(0)
    for block in range(len(row) // 34):
        b = row[block * 34:(block + 1) * 34]
        scale = np.frombuffer(bytes(b[0:2]), np.float16)[0].astype(np.float32)
        q = b[2:].view(np.int8).astype(np.float32)
        for i in range(32):
            s = np.float32(s + np.float32(np.float32(scale * q[i]) * x[block * 32 + i]))
    return s


_Q40_STREAM_SCALES = (0x3C00, 0xB800, 0x3400, 0x0001)


def q40_fixture(input_, output, kind="stream"):
    """Q4_0 bytes of q40Fixture (tests/testdata/forward/q40_stream_test.go:20-29,
    kind "stream") or quantOptimizationFixture(2, ...) (quant_optimization_test.go:25-38,
    kind "opt"): block b gets the scale table's entry b % len and bytes
    (b*13 + i*7) & 0xFF for i = 2..17."""
    scales = _Q40_STREAM_SCALES if kind == "stream" else _Q80_SCALES
    nb = input_ // 32 * output
    blocks = np.arange(nb, dtype=np.int64)[:, None]
    data = ((blocks * 13 + np.arange(18, dtype=np.int64)[None, :] * 7) & 0xFF).astype(np.uint8)
    sc = np.array([scales[b % len(scales)] for b in range(nb)], np.uint16)
    data[:, 0:2] = sc.view(np.uint8).reshape(nb, 2)
    return data.reshape(-1)


def q40_stream_x(batch, input_):
    """x[i] = (i%23 - 11)/32 over the whole batch (q40_stream_test.go:79-81)."""
    i = np.arange(batch * input_)
    return ((i % 23 - 11) / 32).astype(np.float32)


def q40_reference_dot(row, x):
    """referenceQ40Dot (tests/testdata/forward/q40_model_test.go:112-129):
    sequential float32 sum, low then high nibble of each byte."""
    s = np.float32(0)
    for block in range(len(row) // 18):
        b = row[block * 18:(block + 1) * 18]
        scale = np.frombuffer(bytes(b[0:2]), np.float16)[0].astype(np.float32)
        for i in range(16):
            low, high = np.float32(int(b[2 + i] & 15) - 8), np.float32(int(b[2 + i] >> 4) - 8)
            s = np.float32(s + np.float32(np.float32(scale * low) * x[block * 32 + i]))
            s = np.float32(s + np.float32(np.float32(scale * high) * x[block * 32 + i + 16]))
    return s
