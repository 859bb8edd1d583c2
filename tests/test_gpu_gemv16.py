"""GPU parity of the decode GEMV (SPT_PATH_GEMV16): the packed MXFP4 planes
dequantised to f16 in registers, the activations as two f16 terms, fp32 sums
on the mma.sync tensor path.

Routing and dispatch come from the same bit-exact kernels as every path and
must match the oracle bit for bit.  Block outputs are checked at the block's
tolerance (max |error| / max |reference| <= 1e-3, cosine >= 0.99999 against
the oracle's fp32 output) and, since every product is exact here, at a much
tighter 2e-5 that the design promises.
"""
import numpy as np
import pytest

import refdata
from oracle import oracle

pytestmark = pytest.mark.gpu
spt = refdata.spt

MAX_REL = 1e-3
MIN_COS = 0.99999
TIGHT = 2e-5


def _err(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    err = np.abs(got - want).max() / max(np.abs(want).max(), 1e-30)
    cos = float(np.dot(got, want) / (np.linalg.norm(got) * np.linalg.norm(want) + 1e-300))
    return err, cos


def _check(got, want, tag, tight=True):
    assert np.isfinite(got).all(), tag
    err, cos = _err(got, want)
    assert err <= MAX_REL and cos >= MIN_COS, (tag, err, cos)
    if tight:
        assert err <= TIGHT, (tag, err)
    return err, cos


@pytest.fixture(scope="module")
def layer(ctx):
    cfg = spt.Config(2880, 2880, 128, 4)
    params = spt.SynthParams(seed=0)
    dense = oracle.synth_weights(2880, 2880, 128, 4, oracle.synth_params(seed=0))
    arena = ctx.synthetic_arena(cfg, params, flags=spt.ARENA_MMA)
    yield cfg, dense, arena
    arena.close()
    ctx.set_path(spt.PATH_AUTO)


@pytest.mark.parametrize("T", [1, 2, 5, 8, 32])
def test_gemv16_block_matches_oracle(ctx, layer, T):
    cfg, dense, arena = layer
    x = spt.synth_normal_host(T + 11, 2000, T * 2880)
    ctx.set_path(spt.PATH_GEMV16)
    try:
        got = ctx.forward_moe_batch(arena, x, T)
        kernels = ctx.kernels_per_forward()
        r = ctx.last_routing(T, 128, 4)
    finally:
        ctx.set_path(spt.PATH_AUTO)
    # router (with the f16 split of x), [select], [dispatch], gate/up, down
    # [+ combine]: the router's last CTA selects and
    # dispatches (up to 8 tokens), up to 64 slots combine inside the down launch
    assert kernels == 6 - 2 * (T <= 8) - (T * 4 <= 64)
    want = oracle.forward_moe_batch(dense, x, T, workers=8, want_internals=True)
    assert np.array_equal(r["sel_idx"], want["sel_idx"])
    assert refdata.bits_equal(r["sel_w"], want["sel_w"]).all()
    assert np.array_equal(r["perm"], want["perm"])
    _check(got, want["out"], T)


def test_gemv16_is_the_auto_decode_path(ctx, layer):
    """SPT_PATH_AUTO runs decode batches on the GEMV (no quantisation
    launches) and prefill batches on the tcgen05 GEMM; both meet the
    tolerance on the same tokens."""
    cfg, dense, arena = layer
    ctx.set_path(spt.PATH_AUTO)
    x = spt.synth_normal_host(3, 2100, 4 * 2880)
    got = ctx.forward_moe_batch(arena, x, 4)
    assert ctx.kernels_per_forward() == 3  # router (+ select, dispatch), gate/up, down (+ combine)
    ctx.set_option(spt.OPT_GEMV16_SLOTS, 0)
    try:
        mma = ctx.forward_moe_batch(arena, x, 4)
        assert ctx.kernels_per_forward() == 6
    finally:
        ctx.set_option(spt.OPT_GEMV16_SLOTS, 16)
    want = oracle.forward_moe_batch(dense, x, 4, workers=8)
    _check(got, want, "auto")
    _check(mma, want, "mma", tight=False)


def test_gemv16_many_tokens_per_expert(ctx, layer):
    """T = 300 on the GEMV: experts hold up to dozens of tokens, so the CTAs
    take them in several passes of four; sampled tokens against the oracle
    and the whole batch against the tcgen05 path."""
    cfg, dense, arena = layer
    T = 300
    x = spt.synth_normal_host(9, 2200, T * 2880)
    ctx.set_path(spt.PATH_GEMV16)
    try:
        got = ctx.forward_moe_batch(arena, x, T).reshape(T, 2880)
        counts = ctx.last_routing(T, 128, 4)["counts"]
        ctx.set_path(spt.PATH_MMA)
        mma = ctx.forward_moe_batch(arena, x, T).reshape(T, 2880)
    finally:
        ctx.set_path(spt.PATH_AUTO)
    assert counts.max() > 8
    sample = [0, 1, 77, 150, 299]
    xs = np.concatenate([x[t * 2880:(t + 1) * 2880] for t in sample])
    want = oracle.forward_moe_batch(dense, xs, len(sample), workers=8)
    _check(got[sample], want, "sample")
    _check(mma, got, "vs tcgen05", tight=False)


@pytest.mark.parametrize("mode", ["normal", "ties", "underflow", "clamp"])
@pytest.mark.parametrize("experts,k", [(4, 2), (7, 7), (8, 1)])
def test_gemv16_reference_fixtures(ctx, mode, experts, k):
    """The reference's fixtures (hidden 96, expert dim 64: one K tile, 37
    tokens so experts take several passes; the clamp mode scales x by 1000,
    which the per-row exponent of the f16 split absorbs)."""
    fx = refdata.moe_batch_fixture(96, 64, experts, k, 0, mode)
    batch = 37
    x = refdata.moe_batch_x(batch, 96, mode)
    arena = ctx.arena([fx.reader], fx.cfg, [fx.lw], flags=spt.ARENA_MMA)
    try:
        ctx.set_path(spt.PATH_GEMV16)
        got = ctx.forward_moe_batch(arena, x, batch)
        r = ctx.last_routing(batch, experts, k)
    finally:
        ctx.set_path(spt.PATH_AUTO)
        arena.close()
    want = oracle.forward_moe_batch(fx.dense, x, batch, want_internals=True)
    assert np.array_equal(r["sel_idx"], want["sel_idx"]), mode
    assert np.array_equal(r["perm"], want["perm"]), mode
    _check(got, want["out"], (mode, experts, k))


def test_gemv16_refuses_scales_outside_f16(ctx):
    """Scale bytes outside [104, 140] would not stay exact in f16: such an
    arena refuses the forced decode GEMV and SPT_PATH_AUTO takes the tcgen05
    GEMM instead."""
    cfg = spt.Config(256, 128, 16, 4)
    params = spt.SynthParams(seed=5, scale_lo=100, scale_hi=123)
    arena = ctx.synthetic_arena(cfg, params, flags=spt.ARENA_MMA)
    try:
        x = spt.synth_normal_host(5, 7, 2 * 256)
        ctx.set_path(spt.PATH_GEMV16)
        with pytest.raises(spt.SptError):
            ctx.forward_moe_batch(arena, x, 2)
        ctx.set_path(spt.PATH_AUTO)
        ctx.forward_moe_batch(arena, x, 2)
        assert ctx.kernels_per_forward() == 6
    finally:
        ctx.set_path(spt.PATH_AUTO)
        arena.close()
