"""GPU parity: the sm_100a library through its C ABI against the CPU oracle.

The bar is bit-exact (Float32bits equal, NaN == NaN) for every stage and the
whole block: the kernels reproduce the reference's AVX2 arithmetic order.
Where a reference test states a tolerance (3e-5 against its float64
oracle, 1e-5 for the SwiGLU known answer) that tolerance is checked too.
"""
import math

import numpy as np
import pytest

import refdata
from oracle import oracle
from refdata import bits_equal

pytestmark = pytest.mark.gpu
spt = refdata.spt
LEVELS = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, 0, -.5, -1, -1.5, -2, -3, -4, -6], np.float64)


def _run_block(ctx, fx, x, batch):
    arena = ctx.arena([fx.reader], fx.cfg, [fx.lw])
    try:
        out = np.full(batch * fx.cfg.hidden_dim, 999, np.float32)
        ctx.forward_moe_batch(arena, x, batch, out=out)
        routing = ctx.last_routing(batch, fx.cfg.num_experts, fx.cfg.num_experts_used)
        seq = np.concatenate([ctx.forward_moe(arena, x[t * fx.cfg.hidden_dim:(t + 1) * fx.cfg.hidden_dim])
                              for t in range(batch)])
    finally:
        arena.close()
    return out, routing, seq


@pytest.mark.parametrize("experts", [1, 4, 7])
@pytest.mark.parametrize("bias_type", [-1, 0, 1, 30])
def test_block_bit_exact_sweep(ctx, experts, bias_type):
    """TestForwardMoEBatchMatchesSequential's sweep, checked against the oracle
    (outputs, logits, selections, dispatch permutation) and batch==sequential."""
    for top_k in sorted({1, min(2, experts), experts}):
        for mode in refdata.ROUTER_MODES:
            fx = refdata.moe_batch_fixture(96, 64, experts, top_k, bias_type, mode)
            for batch in (1, 5, 37):
                x = refdata.moe_batch_x(batch, 96, mode)
                orig = x.copy()
                want = oracle.forward_moe_batch(fx.dense, x, batch, want_internals=True)
                got, r, seq = _run_block(ctx, fx, x, batch)
                tag = (top_k, mode, batch)
                assert bits_equal(got, want["out"].ravel()).all(), tag
                assert bits_equal(seq, got).all(), tag
                assert bits_equal(r["logits"], want["logits"]).all(), tag
                assert np.array_equal(r["sel_idx"], want["sel_idx"]), tag
                assert bits_equal(r["sel_w"], want["sel_w"]).all(), tag
                assert r["dispatched"] == want["dispatched"], tag
                assert np.array_equal(r["perm"], want["perm"]), tag
                assert np.array_equal(r["counts"], want["counts"]), tag
                assert np.array_equal(x.view(np.uint32), orig.view(np.uint32))


def test_fused_selection_matches_separate(ctx):
    """Up to 8 tokens the top-k selection and the dispatch run in the
    router's last CTA (SPT_OPT_FUSED_SELECT = 1, the default: two launches
    fewer), or the selection inside the dispatch kernel (= 2: one fewer);
    = 0 keeps three launches.  All give the same output bits and routing,
    over every router mode of the sweep (20 tokens: separate launches in
    every mode)."""
    for experts, top_k in ((7, 2), (33, 4), (128, 32)):
        for mode in refdata.ROUTER_MODES:
            fx = refdata.moe_batch_fixture(96, 64, experts, top_k, 1, mode)
            for batch in (1, 5, 8, 20):
                x = refdata.moe_batch_x(batch, 96, mode)
                got = {}
                for fused in (1, 2, 0):
                    ctx.set_option(spt.OPT_FUSED_SELECT, fused)
                    out, r, _ = _run_block(ctx, fx, x, batch)
                    got[fused] = (out, r, ctx.kernels_per_forward())
                ctx.set_option(spt.OPT_FUSED_SELECT, 1)
                tag = (experts, top_k, mode, batch)
                b, rb, kb = got[0]
                for fused in (1, 2):
                    a, ra, ka = got[fused]
                    assert bits_equal(a, b).all(), tag
                    assert np.array_equal(ra["sel_idx"], rb["sel_idx"]), tag
                    assert bits_equal(ra["sel_w"], rb["sel_w"]).all(), tag
                    assert np.array_equal(ra["perm"], rb["perm"]), tag
                    assert np.array_equal(ra["counts"], rb["counts"]), tag
                    # the counts are those of the last call, a one-token forward
                    assert ka == kb - (3 - fused), (tag, fused, ka, kb)


@pytest.mark.parametrize("mode", ["ties", "normal", "underflow"])
@pytest.mark.parametrize("k", [1, 2, 8])
def test_sparse_independent_reference(ctx, mode, k):
    fx = refdata.moe_batch_fixture(96, 64, 8, k, -1, mode)
    batch = 19
    x = ((np.arange(batch * 96) % 13 + 1).astype(np.float32) / np.float32(16)).astype(np.float32)
    got, _, _ = _run_block(ctx, fx, x, batch)
    got = got.reshape(batch, 96)
    for t in range(batch):
        want = oracle.scalar_sparse_moe_f64(fx.dense, x[t * 96:(t + 1) * 96])
        assert np.all(np.abs(got[t] - want) <= 3e-5 * np.maximum(1, np.abs(want)))


def test_swiglu_known_answer(ctx):
    fx = refdata.swiglu_fixture()
    out = np.zeros(32, np.float32)
    ctx.forward_moe_batch_reader(fx.reader, fx.cfg, fx.lw, np.zeros(32, np.float32), out, 1)
    want = 7 / (1 + math.exp(-1.702 * 7)) * 8 + 5
    assert np.all(np.abs(out - want) <= 1e-5)
    assert bits_equal(out, oracle.forward_moe_batch(fx.dense, np.zeros(32, np.float32), 1).ravel()).all()


def test_cancel_flag(ctx):
    fx = refdata.moe_batch_fixture(96, 64, 4, 4, 0, "ties")
    arena = ctx.arena([fx.reader], fx.cfg, [fx.lw])
    x = np.zeros(37 * 96, np.float32)
    with pytest.raises(spt.CanceledError):
        ctx.forward_moe_batch(arena, x, 37, cancel=np.ones(1, np.int32))
    arena.close()


# ---- stages -----------------------------------------------------------------

@pytest.mark.parametrize("hidden", [3, 31, 32, 96, 2880])
@pytest.mark.parametrize("batch", [1, 2, 17, 100])
def test_router_stage(ctx, hidden, batch):
    """Up to 64 rows the router stages whole rows in shared memory
    (k_router_smem), beyond that it runs register-blocked from L2
    (k_router); the 64-chain order is the same."""
    experts = 5
    bias = np.array([.125, -.25, .5, -1, 2], np.float32)
    n = experts * hidden
    w = ((np.arange(n) % 23 - 11).astype(np.float32) / np.float32(64)).astype(np.float32)
    storage = np.zeros(n * 4 + 1, np.uint8)
    storage[1:] = np.frombuffer(w.astype("<f4").tobytes(), np.uint8)
    data = storage[1:]
    x = ((np.arange(batch * hidden) % 31 - 15).astype(np.float32) / np.float32(32)).astype(np.float32)
    got = ctx.route_moe_batch(data, x, bias, batch, hidden, experts)
    assert bits_equal(got, oracle.route(data, x, bias, batch, hidden, experts)).all()
    want = (x.reshape(batch, 1, hidden).astype(np.float64) * w.reshape(1, experts, hidden)).sum(-1) + bias
    assert np.all(np.abs(got - want) <= 3e-5 * np.maximum(1, np.abs(want)))
    for value in (np.nan, np.inf, -np.inf):
        d2 = data.copy()
        d2[:4] = np.frombuffer(np.float32(value).tobytes(), np.uint8)
        x2 = x.copy()
        x2[0] = 1
        g = ctx.route_moe_batch(d2, x2, bias, batch, hidden, experts)[0, 0]
        assert np.isnan(g) if np.isnan(value) else g == value


def test_select_stage(ctx):
    rng = np.random.default_rng(11)
    cases = [rng.standard_normal((64, 128)).astype(np.float32),
             np.round(rng.standard_normal((64, 128)) * 2).astype(np.float32),  # many ties
             np.full((4, 16), np.nan, np.float32),
             np.full((4, 16), np.inf, np.float32),
             (np.arange(16, dtype=np.float32) * 1000)[None, :].repeat(3, 0)]
    mixed = rng.standard_normal((8, 32)).astype(np.float32)
    mixed[:, ::3] = np.nan
    mixed[:, 1::5] = -np.inf
    cases.append(mixed)
    for lg in cases:
        for k in (1, 2, 4, 8):
            idx, w = ctx.select_moe_batch(lg, k)
            for t in range(lg.shape[0]):
                want = oracle.select(lg[t], k)
                assert list(idx[t]) == [s[0] for s in want]
                assert bits_equal(w[t], np.array([s[1] for s in want], np.float32)).all()


def test_dispatch_stage(ctx):
    rng = np.random.default_rng(5)
    for batch, k, experts in ((1, 4, 128), (32, 4, 128), (2048, 4, 128), (8192, 4, 128), (37, 3, 7)):
        idx = rng.integers(0, experts, (batch, k)).astype(np.int32)
        w = rng.random((batch, k)).astype(np.float32)
        w[rng.random((batch, k)) < 0.1] = 0
        w[rng.random((batch, k)) < 0.02] = np.nan
        perm, offs = ctx.dispatch_moe_batch(idx, w, experts)
        flat_i, flat_w = idx.ravel(), w.ravel()
        disp = ~(flat_w <= 0)
        want = []
        for e in range(experts):
            slots = [s for s in range(batch * k) if disp[s] and flat_i[s] == e]
            assert offs[e + 1] - offs[e] == len(slots)
            want.extend(sorted(slots, reverse=True))
        assert np.array_equal(perm, np.array(want, np.int32))


@pytest.mark.parametrize("input_", [32, 96, 2880])
@pytest.mark.parametrize("count", [1, 2, 3, 4, 8, 16])
def test_gather_scatter_stage(ctx, input_, count):
    row, vector = refdata.simd_kernel_row(input_)
    output = 3
    data = np.tile(row, output)
    x = np.zeros(count * (input_ + 1), np.float32)
    starts = [(count - 1 - t) * (input_ + 1) + 1 for t in range(count)]
    ends = [t * (output + 1) + 1 for t in range(count)]
    bias = np.array([.125, -.25, .5], np.float32)
    for t in range(count):
        x[starts[t]: starts[t] + input_] = vector * np.float32(t + 1)
    y = np.zeros(count * (output + 1), np.float32)
    want = np.zeros_like(y)
    ctx.mul_moe_batch_expert(data, input_, output, x, starts, bias, y, ends)
    oracle.mul_moe_batch_expert(data, input_, output, x, starts, bias, want, ends)
    assert bits_equal(y, want).all()
    for t in range(count):
        assert y[t * (output + 1)] == 0


def test_all_scales_and_dot_known_answer(ctx):
    data = np.zeros(257 * 17, np.uint8)
    for s in range(256):
        data[s * 17] = s
        data[s * 17 + 1: s * 17 + 17] = 0x22
    data[256 * 17] = 255
    x = np.full(32, 1.0 / 32, np.float32)
    out = np.zeros(257, np.float32)
    ctx.mul_moe_batch_expert(data, 32, 257, x, [0], None, out, [0])
    for s in range(255):
        assert out[s] == np.float32(math.ldexp(1.0, s - 127)), s
    assert np.isinf(out[255]) and np.isnan(out[256])
    row = np.zeros(17, np.uint8)
    row[0] = 127
    row[1:] = 0x22
    y = np.zeros(1, np.float32)
    ctx.mul_moe_batch_expert(row, 32, 1, np.full(32, 2.0, np.float32), [0], None, y, [0])
    assert y[0] == 64.0


def test_decode_all_encodings_one_hot(ctx):
    """Every (scale, byte) block dotted with each one-hot vector: 65536 rows x
    32 tokens, bit-exact against the oracle (NaN == NaN for scale 255)."""
    scale = np.repeat(np.arange(256, dtype=np.uint8), 256)
    packed = np.tile(np.arange(256, dtype=np.uint8), 256)
    row = np.empty((65536, 17), np.uint8)
    row[:, 0] = scale
    row[:, 1:] = packed[:, None]
    data = row.reshape(-1)
    x = np.eye(32, dtype=np.float32).reshape(-1)
    offs = [32 * j for j in range(32)]
    yoffs = [65536 * j for j in range(32)]
    y = np.zeros(32 * 65536, np.float32)
    want = np.zeros_like(y)
    ctx.mul_moe_batch_expert(data, 32, 65536, x, offs, None, y, yoffs)
    oracle.mul_moe_batch_expert(data, 32, 65536, x, offs, None, want, yoffs, workers=8)
    assert bits_equal(y, want).all()
    dec = oracle.decode_mxfp4(data).reshape(65536, 32)
    finite = np.isfinite(dec).all(1)  # an Inf weight times 0 poisons its row's sum
    assert np.array_equal(y.reshape(32, 65536).T[finite], dec[finite])


@pytest.mark.parametrize("input_", [32, 96, 2880])
def test_nibble_reference(ctx, input_):
    rows, blocks = 256, input_ // 32
    x = ((np.arange(input_) % 23 - 11).astype(np.float32) / np.float32(32)).astype(np.float32)
    r = np.arange(rows)[:, None, None]
    b = np.arange(blocks)[None, :, None]
    i = np.arange(16)[None, None, :]
    packed = ((r + b * 7 + i * 11) & 0xFF).astype(np.uint8)
    data = np.zeros((rows, blocks, 17), np.uint8)
    data[:, :, 0] = (120 + np.arange(blocks) % 12)[None, :]
    data[:, :, 1:] = packed
    scale = np.ldexp(1.0, data[:, :, 0].astype(np.int64) - 127)
    xb = x.reshape(blocks, 32).astype(np.float64)
    want = (scale[:, :, None] * (LEVELS[packed & 15] * xb[None, :, :16] + LEVELS[packed >> 4] * xb[None, :, 16:])).sum((1, 2))
    out = np.zeros(rows, np.float32)
    ctx.mul_moe_batch_expert(data.reshape(-1), input_, rows, x, [0], None, out, [0])
    assert np.all(np.abs(out - want) <= 3e-5 * np.maximum(1, np.abs(want)))
    ref = np.zeros(rows, np.float32)
    oracle.mul_moe_batch_expert(data.reshape(-1), input_, rows, x, [0], None, ref, [0])
    assert bits_equal(out, ref).all()


def test_swiglu_stage(ctx):
    rng = np.random.default_rng(2)
    g = np.concatenate([rng.standard_normal(4096) * 4, [np.nan, np.inf, -np.inf, 7, 7.0001, -7, -1e30, 1e30, 0, -0.0]]).astype(np.float32)
    u = np.concatenate([rng.standard_normal(4096) * 4, [1, np.nan, 2, np.inf, -np.inf, 8, -8, 0, -0.0, 3]]).astype(np.float32)
    got = ctx.swiglu(g, u)
    want = np.array([oracle.swiglu(a, b) for a, b in zip(g, u)], np.float32)
    assert bits_equal(got, want).all()


def test_combine_stage(ctx):
    rng = np.random.default_rng(4)
    batch, k, hidden = 9, 4, 2880
    res = rng.standard_normal((batch * k, hidden)).astype(np.float32)
    w = rng.random((batch, k)).astype(np.float32)
    w[0, 1] = 0
    w[1, 2] = np.nan
    w[2, :] = -1
    got = ctx.combine_moe_batch(res, w, batch, k, hidden)
    want = np.zeros((batch, hidden), np.float32)
    for t in range(batch):
        for r in range(k):
            wt = w[t, r]
            if wt <= 0:
                continue
            want[t] = oracle.fmaf(res[t * k + r], wt, want[t])
    assert bits_equal(got, want).all()


def test_rmsnorm_stage(ctx):
    rng = np.random.default_rng(8)
    for dim in (2880, 100, 7):
        x = rng.standard_normal(3 * dim).astype(np.float32)
        w = (1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)
        got = ctx.rmsnorm(x, w, 3, dim, 1e-5)
        want = oracle.rmsnorm(x, w, 3, dim, 1e-5)
        assert bits_equal(got, want).all()


# ---- GPT-OSS-120B shapes with seeded synthetic weights --------------------

GPT_OSS = dict(hidden=2880, expert_dim=2880, experts=128, k=4)


def _gpt_oss_layer(seed=0, **kw):
    cfg = spt.Config(2880, 2880, 128, 4)
    params = spt.SynthParams(seed=seed, **kw)
    host = spt.synth_layer_host(cfg, params)
    dense = oracle.Weights(2880, 2880, 128, 4, host["router"], host["router_bias"], host["gate"],
                           host["up"], host["down"], host["gate_bias"], host["up_bias"], host["down_bias"])
    return cfg, params, dense


@pytest.fixture(scope="module")
def gpt_oss(ctx):
    cfg, params, dense = _gpt_oss_layer(0)
    arena = ctx.synthetic_arena(cfg, params)
    yield cfg, params, dense, arena
    arena.close()


@pytest.mark.parametrize("T", [1, 4, 32])
def test_gpt_oss_block_bit_exact(ctx, gpt_oss, T):
    cfg, params, dense, arena = gpt_oss
    x = spt.synth_normal_host(T, 1000, T * 2880)
    got = ctx.forward_moe_batch(arena, x, T)
    r = ctx.last_routing(T, 128, 4)
    want = oracle.forward_moe_batch(dense, x, T, workers=8, want_internals=True)
    assert np.array_equal(r["sel_idx"], want["sel_idx"])
    assert np.array_equal(r["perm"], want["perm"])
    assert bits_equal(got, want["out"].ravel()).all()
    # north_star tolerances (implied by bit-exactness, asserted explicitly)
    ref = want["out"].ravel().astype(np.float64)
    err = np.abs(got.astype(np.float64) - ref).max() / np.abs(ref).max()
    cos = float(np.dot(got, ref) / (np.linalg.norm(got) * np.linalg.norm(ref)))
    assert err <= 1e-3 and cos >= 0.99999


def test_gpt_oss_large_batch_properties(ctx, gpt_oss):
    """T=2048: sampled tokens against the oracle, plus batch-split and token
    permutation invariance of the whole batch (bit-exact)."""
    cfg, params, dense, arena = gpt_oss
    T = 2048
    x = spt.synth_normal_host(2, 1000, T * 2880)
    got = ctx.forward_moe_batch(arena, x, T).reshape(T, 2880)
    for t in (0, 1, 777, 2047):
        want = oracle.forward_moe_batch(dense, x[t * 2880:(t + 1) * 2880], 1, workers=8)
        assert bits_equal(got[t], want.ravel()).all(), t
    a = ctx.forward_moe_batch(arena, x[: 1000 * 2880], 1000).reshape(1000, 2880)
    assert bits_equal(a, got[:1000]).all()
    perm = np.random.default_rng(0).permutation(T)
    xp = x.reshape(T, 2880)[perm].ravel()
    gp = ctx.forward_moe_batch(arena, xp, T).reshape(T, 2880)
    assert bits_equal(gp, got[perm]).all()


def test_host_call_graph_replay_matches_launches(ctx):
    """spt_forward_moe_batch replays a captured graph of its device work from
    the second call with the same arena, layer and batch on: the outputs of
    replays equal plain launches bit for bit, on every expert path, and a
    new batch size or option captures anew."""
    cfg = spt.Config(512, 256, 16, 4)
    arena = ctx.synthetic_arena(cfg, spt.SynthParams(seed=31), flags=spt.ARENA_GEMV | spt.ARENA_MMA)
    try:
        for path in (spt.PATH_EXACT, spt.PATH_MMA, spt.PATH_GEMV16, spt.PATH_AUTO):
            ctx.set_path(path)
            for T in (1, 3, 40):
                ctx.set_option(spt.OPT_HOST_GRAPHS, 0)
                want = ctx.forward_moe_batch(arena, spt.synth_normal_host(T, 9, T * 512), T)
                ctx.set_option(spt.OPT_HOST_GRAPHS, 1)
                for rep in range(4):  # plain, capture, replay, replay
                    x = spt.synth_normal_host(T + 100 * rep, 9, T * 512)
                    got = ctx.forward_moe_batch(arena, x, T)
                    ctx.set_option(spt.OPT_HOST_GRAPHS, 0)
                    ref = ctx.forward_moe_batch(arena, x, T)
                    ctx.set_option(spt.OPT_HOST_GRAPHS, 1)
                    assert bits_equal(got, ref).all(), (path, T, rep)
                # the first input again, through the replayed graph
                assert bits_equal(ctx.forward_moe_batch(arena, spt.synth_normal_host(T, 9, T * 512), T), want).all()
    finally:
        ctx.set_path(spt.PATH_AUTO)
        arena.close()
