"""Q8_0 LM head on the GPU (spt_mul_q80, spt_q80_matrix_*) against the oracle.

Bit-exact: every logit's Float32bits equal the oracle's restatement of
quantQ80AVX2 (forward/quant_amd64.go:92-110; NaN == NaN), and the argmax row
and logit equal MulQ80Argmax's rule (forward/q80.go:64-104).  Shapes: the
reference tests' fixtures, every float16 scale, and GPT-OSS's output head
(201,088 rows x 2,880).
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
from tests.refdata import q80_fixture  # noqa: E402

pytestmark = pytest.mark.gpu


def same(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    na, nb = np.isnan(a), np.isnan(b)
    return bool(np.array_equal(na, nb) and np.array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32)))


@pytest.mark.parametrize("input_", [32, 96, 512])
def test_q80_fixture_bit_exact(ctx, input_):
    data, x = q80_fixture(input_, 17, x_kind="opt")
    want_y, want_i, want_l = oracle.mul_q80(data, input_, 17, x)
    y, i, l = ctx.mul_q80(data, input_, 17, x)
    assert same(y, want_y)
    assert i == want_i and same(l, want_l)


@pytest.mark.parametrize("input_", [2912, 4096])
def test_q80_long_rows_bit_exact(ctx, input_):
    """Rows too long for 16-row stages run in 8-row stages (odd and even block
    counts); 45 rows end in a partial four-row group."""
    rng = np.random.default_rng(input_)
    nb = input_ // 32
    data = rng.integers(0, 256, size=(45, nb, 34), dtype=np.uint8)
    data[:, :, :2] = (rng.standard_normal((45, nb)) * 0.01).astype(np.float16).view(np.uint8).reshape(45, nb, 2)
    data = data.reshape(-1)
    x = rng.standard_normal(input_).astype(np.float32)
    want_y, want_i, want_l = oracle.mul_q80(data, input_, 45, x)
    y, i, l = ctx.mul_q80(data, input_, 45, x)
    assert same(y, want_y)
    assert i == want_i and same(l, want_l)


def test_q80_every_scale(ctx):
    rows = np.ones((65536, 34), np.uint8)
    rows[:, :2] = np.arange(65536, dtype=np.uint16).view(np.uint8).reshape(-1, 2)
    x = np.ones(32, np.float32)
    want_y, want_i, want_l = oracle.mul_q80(rows.reshape(-1), 32, 65536, x, workers=8)
    y, i, l = ctx.mul_q80(rows.reshape(-1), 32, 65536, x)
    assert same(y, want_y)
    assert i == want_i and same(l, want_l)


def test_q80_argmax_rules(ctx):
    def row(scale_bits, q):
        r = np.zeros(34, np.uint8)
        r[:2] = np.frombuffer(struct.pack("<H", scale_bits), np.uint8)
        r[2:] = np.full(32, q, np.int8).view(np.uint8)
        return r
    x = np.ones(32, np.float32)
    cases = [
        [row(0x3C00, 1), row(0x3C00, 3), row(0x7E00, 1), row(0x3C00, 3)],  # tie -> lowest, NaN skipped
        [row(0xFC00, 1), row(0xFC00, 1)],                                     # all -Inf -> row 0
        [row(0x7E00, 1), row(0x7E00, 1)],                                     # all NaN -> row 0, -Inf
        [row(0x8000, 1), row(0x0000, 1)],                                     # -0 ties +0 -> row 0
    ]
    for rows in cases:
        data = np.stack(rows).reshape(-1)
        want_y, want_i, want_l = oracle.mul_q80(data, 32, len(rows), x)
        y, i, l = ctx.mul_q80(data, 32, len(rows), x)
        assert same(y, want_y)
        assert i == want_i and same(l, want_l), (i, want_i, l, want_l)


def test_q80_gpt_oss_lm_head(ctx, spt):
    rows, inp = 201088, 2880
    rng = np.random.default_rng(80)
    data = rng.integers(0, 256, size=rows * inp // 32 * 34, dtype=np.uint8).reshape(rows, inp // 32, 34)
    scales = (rng.standard_normal((rows, inp // 32)) * 0.01).astype(np.float16)
    data[:, :, :2] = scales.view(np.uint8).reshape(rows, inp // 32, 2)
    data = data.reshape(-1)
    x = spt.synth_normal_host(80, 1, inp)
    want_y, want_i, want_l = oracle.mul_q80(data, inp, rows, x, workers=os.cpu_count() or 8)
    m = ctx.q80_matrix(data, inp, rows)
    try:
        for _ in range(2):  # the resident matrix serves repeated calls
            y, i, l = m.mul(x)
            assert same(y, want_y)
            assert i == want_i and same(l, want_l)
        _, i2, l2 = m.mul(x, want_y=False)
        assert i2 == want_i and same(l2, want_l)
    finally:
        m.close()
