"""The benchmark's own inputs against the oracle
(decode, seed 0), configs[1] (T=32, seed 1, router bias) and configs[2]
(T=2048, seed 2, Zipf(1.1)-skewed router bias), with the same synthetic
weights and activation stream bench.py times.

Routing (logits, selected ids and weights, dispatch permutation) must be
bit-exact for every token on every path; block outputs are checked on all
tokens of the small batches and, for T=2048, on 64 tokens of which 16 are
routed to the most loaded expert: bit-identical on the exact path, else
max|err| / max|ref| <= 1e-3 and cosine >= 0.99999 (the tolerance of the
block; the reference's own check is TestForwardMoEBatchMatchesSequential,
tests/testdata/forward/moe_batch_test.go:125-168).
"""
import os

import numpy as np
import pytest

import refdata
from oracle import oracle

pytestmark = pytest.mark.gpu
spt = refdata.spt

H, D, E, K = 2880, 2880, 128, 4
MAX_REL, MIN_COS = 1e-3, 0.99999
# name: (tokens, seed, zipf_s, zipf_beta, router bias), as bench.CONFIGS
CASES = {"c0": (1, 0, 0.0, 0.0, True), "c1": (32, 1, 0.0, 0.0, True), "c2": (2048, 2, 1.1, 0.9, True)}


@pytest.fixture(scope="module")
def arenas(ctx):
    made = {}
    yield made
    for a in made.values():
        a.close()


def _arena(ctx, arenas, name):
    if name not in arenas:
        for a in arenas.values():
            a.close()
        arenas.clear()
        T, seed, zs, zb, rb = CASES[name]
        params = spt.SynthParams(seed=seed, zipf_s=zs, zipf_beta=zb, router_bias=rb)
        arenas[name] = ctx.synthetic_arena(spt.Config(H, D, E, K), params, flags=spt.ARENA_GEMV | spt.ARENA_MMA)
    return arenas[name]


@pytest.mark.parametrize("name,path", [("c0", "auto"), ("c0", "mma"), ("c0", "exact"),
                                       ("c1", "auto"), ("c1", "exact"),
                                       ("c2", "auto"), ("c2", "fp8")])
def test_bench_inputs_match_oracle(ctx, arenas, name, path):
    T, seed, zs, zb, rb = CASES[name]
    arena = _arena(ctx, arenas, name)
    p = oracle.synth_params(seed=seed, zipf_s=zs, zipf_beta=zb, router_bias=rb)
    x = oracle.synth_normal(seed, 1000, T * H).reshape(T, H)
    ctx.set_path({"auto": spt.PATH_AUTO, "mma": spt.PATH_MMA, "exact": spt.PATH_EXACT, "fp8": spt.PATH_MMA}[path])
    ctx.set_option(spt.OPT_PREFILL_FP8, 1 if path == "fp8" else 0)
    try:
        got = ctx.forward_moe_batch(arena, x.ravel(), T).reshape(T, H)
        r = ctx.last_routing(T, E, K)
    finally:
        ctx.set_path(spt.PATH_AUTO)
        ctx.set_option(spt.OPT_PREFILL_FP8, 0)
    # routing of every token, bit for bit
    head = oracle.synth_layer_experts(H, D, E, p, 0, [])
    lg = oracle.route_threads(head["router"], x, head["router_bias"], T, H, E)
    sel = [oracle.select(lg[t], K) for t in range(T)]
    sel_idx = np.array([[i for i, _ in s] for s in sel], np.int32)
    sel_w = np.array([[v for _, v in s] for s in sel], np.float32)
    perm, counts = oracle.dispatch_perm(sel_idx, sel_w, E)
    assert np.array_equal(lg.view(np.uint32), r["logits"].view(np.uint32))
    assert np.array_equal(sel_idx, r["sel_idx"])
    assert np.array_equal(sel_w.view(np.uint32), r["sel_w"].view(np.uint32))
    assert np.array_equal(perm, r["perm"])
    # block outputs of the sampled tokens
    if T <= 64:
        idx = list(range(T))
    else:
        top = int(np.argmax(counts))
        on_top = [t for t in range(T) if top in sel_idx[t]][:16]
        assert len(on_top) == 16
        idx = sorted(set(on_top + np.linspace(0, T - 1, 48).astype(int).tolist()))
    experts = sorted(set(sel_idx[idx].ravel().tolist()))
    w = oracle.weights_of(oracle.synth_layer_experts(H, D, E, p, 0, experts), H, D, E, K)
    want = oracle.forward_moe_batch(w, x[idx].ravel(), len(idx), workers=os.cpu_count() or 8).reshape(len(idx), H)
    sub = got[idx]
    if path == "exact":
        assert np.array_equal(sub.view(np.uint32), want.view(np.uint32))
    else:
        err = float(np.max(np.abs(sub - want)) / np.max(np.abs(want)))
        g64, w64 = sub.astype(np.float64).ravel(), want.astype(np.float64).ravel()
        cos = float(np.dot(g64, w64) / (np.linalg.norm(g64) * np.linalg.norm(w64)))
        assert err <= MAX_REL and cos >= MIN_COS, (name, path, err, cos)
