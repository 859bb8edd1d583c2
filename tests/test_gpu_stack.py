"""Layer stack (spt_forward_stack): x += MoE(normBatch(post_attention_norm, x))
per layer (forward/layer_batch.go:102-120), checked against the oracle's
composition of the same three steps (spo_rmsnorm, spo_forward_moe_batch,
float32 add).  Exact path: bit-identical residual stream; tensor-core path:
max|err| / max|ref| <= 1e-3 on the residual stream."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from oracle import oracle  # noqa: E402

pytestmark = pytest.mark.gpu
EPS = 1e-5


def oracle_stack(spt, cfg, params, x, T, layers):
    H, D, E, K = cfg.hidden_dim, cfg.expert_hidden_dim, cfg.num_experts, cfg.num_experts_used
    x = np.array(x, np.float32).reshape(T, H)
    for l in range(layers):
        host = spt.synth_layer_host(cfg, params, l)
        w = oracle.Weights(H, D, E, K, host["router"], host["router_bias"], host["gate"], host["up"],
                           host["down"], host["gate_bias"], host["up_bias"], host["down_bias"])
        norm = spt.synth_norm_host(params, l, H)
        normed = oracle.rmsnorm(x, norm, T, H, EPS)
        ffn = oracle.forward_moe_batch(w, normed, T, workers=os.cpu_count() or 8)
        x = (x + ffn).astype(np.float32)
    return x.reshape(-1)


@pytest.mark.parametrize("T", [1, 5])
def test_stack_small_exact(ctx, spt, T):
    cfg = spt.Config(256, 128, 16, 4)
    params = spt.SynthParams(seed=41)
    arena = ctx.synthetic_arena(cfg, params, n_layers=3, flags=spt.ARENA_GEMV)
    try:
        ctx.set_path(spt.PATH_EXACT)
        x = spt.synth_normal_host(41, T, T * 256)
        got = ctx.forward_stack(arena, x, T, eps=EPS)
        want = oracle_stack(spt, cfg, params, x, T, 3)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        # a sub-range of layers continues from the caller's residual stream
        mid = ctx.forward_stack(arena, x, T, first_layer=0, n_layers=1, eps=EPS)
        rest = ctx.forward_stack(arena, mid, T, first_layer=1, n_layers=2, eps=EPS)
        assert np.array_equal(rest.view(np.uint32), want.view(np.uint32))
    finally:
        arena.close()


def test_stack_gpt_oss_two_layers(ctx, spt):
    cfg = spt.Config(2880, 2880, 128, 4)
    params = spt.SynthParams(seed=4)
    T = 64
    arena = ctx.synthetic_arena(cfg, params, n_layers=2, flags=spt.ARENA_GEMV | spt.ARENA_MMA)
    try:
        x = spt.synth_normal_host(4, 1000, T * 2880)
        want = oracle_stack(spt, cfg, params, x, T, 2)
        ctx.set_path(spt.PATH_EXACT)
        got = ctx.forward_stack(arena, x, T, eps=EPS)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
        ctx.set_path(spt.PATH_MMA)
        got = ctx.forward_stack(arena, x, T, eps=EPS)
        err = float(np.max(np.abs(got - want)) / np.max(np.abs(want)))
        assert np.isfinite(got).all() and err <= 1e-3, err
    finally:
        arena.close()


def test_stack_rejects_bad_arguments(ctx, spt):
    cfg = spt.Config(256, 128, 16, 4)
    arena = ctx.synthetic_arena(cfg, spt.SynthParams(seed=1), n_layers=2, flags=spt.ARENA_GEMV)
    try:
        x = np.zeros(256, np.float32)
        with pytest.raises(spt.SptError):
            ctx.forward_stack(arena, x, 1, first_layer=1, n_layers=2)
        with pytest.raises(spt.SptError):
            ctx.forward_stack(arena, x, 1, eps=float("nan"))
    finally:
        arena.close()
