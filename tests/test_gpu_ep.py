"""Expert-parallel block on two GPUs through the C ABI.

Each of two processes owns one GPU, half of the 128 experts
(spt_arena_create_synthetic_range over spt_ep_expert_range) and its own
tokens; spt_forward_moe_batch_ep exchanges rows over NCCL.  Every rank's
output must equal the single-GPU block (a full arena on the same GPU) for
its tokens: bit for bit on the exact path, within the tensor-core path's
tolerance (max|err| / max|ref| <= 1e-3) on the MMA path, for the counts-first
exchange and for the fixed-capacity exchange through the NVLink peer windows
and through NCCL.  Skipped on hosts with fewer than two GPUs.
"""
import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

pytestmark = pytest.mark.gpu

WORLD = 2
TOKENS = {0: [32, 1, 300], 1: [17, 4, 64]}  # per call, per rank (ranks differ)


def _log(rank, msg):
    print(f"[ep rank {rank}] {msg}", file=sys.stderr, flush=True)


def _rank_main(rank, world, uid_q, results):
    import faulthandler
    faulthandler.dump_traceback_later(90, repeat=True)  # a stuck rank shows where it waits
    sys.path.insert(0, ROOT)
    spt = importlib.import_module("stream-pt_b200")
    out = {}
    try:
        # the id is made in rank 0's own process, so every rank's NCCL is the
        # same library build
        if rank == 0:
            uid = spt.ep_unique_id()
            for _ in range(world - 1):
                uid_q.put(uid)
        else:
            uid = uid_q.get(timeout=120)
        ctx = spt.Context(rank)
        cfg = spt.Config(2880, 2880, 128, 4)
        params = spt.SynthParams(seed=3)
        flags = spt.ARENA_GEMV | spt.ARENA_MMA
        shard = ctx.synthetic_arena(cfg, params, flags=flags, experts=spt.ep_expert_range(128, world, rank))
        full = ctx.synthetic_arena(cfg, params, flags=flags)
        _log(rank, "arenas ready")
        ep = spt.ExpertParallel(ctx, uid, rank, world)
        _log(rank, "group ready")
        # counts exchanged per call, then the fixed-capacity exchange through
        # the NVLink peer windows and through NCCL
        for mode, capacity in (("counts", 0), ("capacity", 300), ("capacity-nccl", 300)):
          ep.set_capacity(capacity)
          ep.set_exchange(spt.EP_EXCHANGE_NCCL if mode == "capacity-nccl" else spt.EP_EXCHANGE_PEER)
          for call, T in enumerate(TOKENS[rank]):
            x = spt.synth_normal_host(50 + rank, call, T * 2880)
            for path, name in ((spt.PATH_EXACT, "exact"), (spt.PATH_MMA, "mma")):
                ctx.set_path(path)
                got = ctx.forward_moe_batch_ep(ep, shard, x, T)
                want = ctx.forward_moe_batch(full, x, T)
                if name == "exact":
                    ok = bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))
                    err = 0.0 if ok else float(np.max(np.abs(got - want)))
                else:
                    err = float(np.max(np.abs(got - want)) / max(np.max(np.abs(want)), 1e-30))
                    ok = bool(np.isfinite(got).all() and err <= 1e-3)
                out[(mode, call, name)] = (ok, err)
                _log(rank, f"{mode} call {call} T={T} {name}: ok={ok} err={err:.3g}")
        results.put((rank, out, None))
    except Exception as exc:
        _log(rank, f"error: {exc!r}")
        results.put((rank, out, repr(exc)))
    finally:
        for obj in ("ep", "shard", "full", "ctx"):
            if obj in locals():
                locals()[obj].close()


@pytest.mark.timeout(900)
def test_expert_parallel_matches_single_gpu():
    import torch
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import multiprocessing as mp
    mctx = mp.get_context("spawn")
    q, uid_q = mctx.Queue(), mctx.Queue()
    procs = [mctx.Process(target=_rank_main, args=(r, WORLD, uid_q, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(WORLD):
            rank, res, err = q.get(timeout=420)
            got[rank] = (res, err)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.terminate()
    for rank, (res, err) in got.items():
        assert err is None, (rank, err)
        for key, (ok, e) in res.items():
            assert ok, (rank, key, e)
        assert len(res) == 3 * 2 * len(TOKENS[rank])
