"""Q4_0 products on the GPU (spt_mul_q40, spt_mul_q40_batch, spt_q40_matrix_*)
against the oracle, bit for bit (NaN == NaN).

Batch 1 follows quantQ40AVX2 (forward/quant_amd64.go:75-90), larger batches
quantDotQ40Batch (:118-148), as MulQ40BatchInto picks them
(forward/q40.go:87-92).  Cases: the reference tests' fixtures
(q40_test.go:12-50, q40_stream_test.go:69-105 with its 37-byte tensor
offset, quant_optimization_test.go:64-180), every float16 scale, GPT-OSS's
attention projections (Q/K/V fused 5,120 x 2,880 and O 2,880 x 4,096) at
every tile shape of the batched kernel, ragged row counts and an odd block
count per row.
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
from tests.refdata import q40_fixture, q40_stream_x  # noqa: E402

pytestmark = pytest.mark.gpu
WORKERS = os.cpu_count() or 8


def same(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    na, nb = np.isnan(a), np.isnan(b)
    return bool(np.array_equal(na, nb) and np.array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32)))


def random_q40(rows, input_, seed):
    rng = np.random.default_rng(seed)
    nb = input_ // 32
    data = rng.integers(0, 256, size=(rows, nb, 18), dtype=np.uint8)
    data[:, :, :2] = (rng.standard_normal((rows, nb)) * 0.01).astype(np.float16).view(np.uint8).reshape(rows, nb, 2)
    return data.reshape(-1)


def test_q40_known_answers(ctx, spt):
    b = np.zeros(18, np.uint8)
    b[:2] = np.frombuffer(struct.pack("<H", 0x3C00), np.uint8)
    b[2] = 0x0F
    x = np.zeros(32, np.float32)
    x[0], x[16] = 2, 3
    r, t = spt.q40_tensor(b, 32, 1)
    assert ctx.mul_q40(r, t, x)[0] == np.float32(7 * 2 - 8 * 3)
    row = np.zeros(36, np.uint8)
    for blk in range(2):
        row[18 * blk:18 * blk + 2] = np.frombuffer(struct.pack("<H", 0x3C00), np.uint8)
        row[18 * blk + 2:18 * blk + 18] = 0x88
    row[20] = 0x89
    x = np.zeros(64, np.float32)
    x[32] = 5
    r, t = spt.q40_tensor(row, 64, 1)
    assert ctx.mul_q40(r, t, x)[0] == np.float32(5)


@pytest.mark.parametrize("batch", [1, 2])
def test_q40_every_scale(ctx, spt, batch):
    rows = np.full((65536, 18), 0x99, np.uint8)
    rows[:, :2] = np.arange(65536, dtype=np.uint16).view(np.uint8).reshape(-1, 2)
    x = np.ones(32 * batch, np.float32)
    want = oracle.mul_q40(rows.reshape(-1), 32, 65536, x, batch, workers=WORKERS)
    r, t = spt.q40_tensor(rows, 32, 65536)
    got = ctx.mul_q40_batch(r, t, x, batch)
    assert same(got, want)


@pytest.mark.parametrize("batch", [1, 3, 9, 19])
def test_q40_streaming_batch_fixture(ctx, spt, batch):
    data = q40_fixture(96, 11, "stream")
    x = q40_stream_x(batch, 96)
    want = oracle.mul_q40(data, 96, 11, x, batch)
    r, t = spt.q40_tensor(data, 96, 11, prefix=37)
    got = ctx.mul_q40_batch(r, t, x, batch)
    assert same(got, want)
    assert same(ctx.mul_q40_batch(r, t, x, batch), want)  # repeated call


@pytest.mark.parametrize("input_", [32, 96, 512])
def test_q40_optimization_fixture(ctx, spt, input_):
    data = q40_fixture(input_, 17, "opt")
    i = np.arange(input_)
    x = ((i % 23 - 11) / 32).astype(np.float32)
    r, t = spt.q40_tensor(data, input_, 17)
    assert same(ctx.mul_q40(r, t, x), oracle.mul_q40(data, input_, 17, x)[0])


@pytest.mark.parametrize("rows,input_", [(5120, 2880), (2880, 4096), (4099, 2880), (37, 2912), (16, 64)])
@pytest.mark.parametrize("batch", [1, 2, 5, 16, 33, 130])
def test_q40_gpt_oss_projections(ctx, spt, rows, input_, batch):
    """Every tile shape of the batched kernel (batch <= 4, <= 8, <= 16, more)
    and ragged item tiles; row counts off the 16-row stage and 64-row tile;
    91 blocks per row (odd: 8-row copies)."""
    data = random_q40(rows, input_, rows + input_)
    x = spt.synth_normal_host(40 + batch, 1, batch * input_)
    want = oracle.mul_q40(data, input_, rows, x, batch, workers=WORKERS)
    r, t = spt.q40_tensor(data, input_, rows)
    m = ctx.q40_matrix(r, t)
    try:
        assert same(m.mul(x, batch), want)
    finally:
        m.close()


def test_q40_device_entry_and_overlap(ctx, spt):
    import torch
    rows, input_ = 512, 2880
    data = random_q40(rows, input_, 7)
    r, t = spt.q40_tensor(data, input_, rows)
    m = ctx.q40_matrix(r, t)
    try:
        x = spt.synth_normal_host(7, 1, 3 * input_)
        want1 = oracle.mul_q40(data, input_, rows, x[:input_], 1)
        want3 = oracle.mul_q40(data, input_, rows, x, 3)
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty(3 * rows, dtype=torch.float32, device="cuda")
        for batch, want in ((1, want1), (3, want3)):
            m.mul_device(xd.data_ptr(), yd.data_ptr(), batch)
            ctx.sync()
            assert same(yd[:batch * rows].cpu().numpy().reshape(batch, rows), want)
        with pytest.raises(spt.SptError) as e:
            m.mul_device(xd.data_ptr(), xd.data_ptr() + 64, 1)
        assert e.value.status == spt.ERR_OVERLAP
    finally:
        m.close()
