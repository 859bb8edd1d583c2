"""Expert-parallel protocol on CPU: two gloo ranks.

The GPU expert-parallel forward (spt_forward_moe_batch_ep) splits the block
into: route and select this rank's tokens; group the dispatched slots by the
rank that owns their expert (spt_ep_expert_range), gather their token rows;
exchange row counts, then rows plus local expert ids; run the expert products
for the received rows; send the result rows back; combine them in rank order
with fma(result, weight, out).  This test runs that exact protocol with the
oracle as the arithmetic and torch.distributed (gloo) as the transport, with
each rank computing only its own experts, and checks that every rank's output
is bit-identical to the single-process oracle block for the same tokens.  It
pins the decomposition (partition, grouping order, exchange layout and
combine order) that the CUDA path implements, on hosts without a GPU.
"""
import importlib
import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

H, D, E, K = 64, 64, 8, 2
TOKENS = {0: 5, 1: 3}  # different batch per rank
WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, results):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    from oracle import oracle
    spt = importlib.import_module("stream-pt_b200")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        cfg = spt.Config(H, D, E, K)
        host = spt.synth_layer_host(cfg, spt.SynthParams(seed=7))
        w = oracle.Weights(H, D, E, K, host["router"], host["router_bias"], host["gate"], host["up"],
                           host["down"], host["gate_bias"], host["up_bias"], host["down_bias"])
        T = TOKENS[rank]
        x = spt.synth_normal_host(100 + rank, 5, T * H).reshape(T, H)
        want = oracle.forward_moe_batch(w, x, T)

        # 1. route + select this rank's tokens (all experts: the router is whole)
        logits = oracle.route(host["router"], x, host["router_bias"], T, H, E)
        sel = [oracle.select(logits[t], K) for t in range(T)]
        # 2. group dispatched slots by owner rank; within a rank, descending slot
        #    (the order of the dispatch kernel's counting sort)
        ranges = [spt.ep_expert_range(E, world, r) for r in range(world)]
        owner = lambda e: next(r for r, (b, en) in enumerate(ranges) if b <= e < en)
        slots = [(t * K + r, e, wt) for t in range(T) for r, (e, wt) in enumerate(sel[t])
                 if not (wt <= 0.0)]
        send_order = sorted(slots, key=lambda s: (owner(s[1]), -s[0]))
        send_counts = [sum(1 for s in send_order if owner(s[1]) == r) for r in range(world)]
        send_pos = {s[0]: p for p, s in enumerate(send_order)}
        xs = np.stack([x[s[0] // K] for s in send_order]) if send_order else np.zeros((0, H), np.float32)
        ms = np.array([s[1] - ranges[owner(s[1])][0] for s in send_order], np.int32)
        # 3. counts, then rows and local expert ids
        sc = torch.tensor(send_counts, dtype=torch.int64)
        rc = torch.empty(world, dtype=torch.int64)
        dist.all_to_all_single(rc, sc)
        recv_counts = rc.tolist()
        R = sum(recv_counts)
        xr = torch.empty(R * H, dtype=torch.float32)
        dist.all_to_all_single(xr, torch.from_numpy(xs.reshape(-1).copy()),
                               [c * H for c in recv_counts], [c * H for c in send_counts])
        mr = torch.empty(R, dtype=torch.int32)
        dist.all_to_all_single(mr, torch.from_numpy(ms.copy()), recv_counts, send_counts)
        xr = xr.numpy().reshape(R, H)
        mr = mr.numpy()
        # 4. expert products for the received rows, this rank's experts only
        b0, b1 = ranges[rank]
        gsz, dsz = D * (H // 32) * 17, H * (D // 32) * 17
        rows_out = np.zeros((R, H), np.float32)
        for j in range(R):
            e = b0 + int(mr[j])
            assert b0 <= e < b1
            g = np.zeros(D, np.float32)
            u = np.zeros(D, np.float32)
            oracle.mul_moe_batch_expert(host["gate"][e * gsz:(e + 1) * gsz], H, D, xr[j], [0],
                                        host["gate_bias"][e * D:(e + 1) * D], g, [0])
            oracle.mul_moe_batch_expert(host["up"][e * gsz:(e + 1) * gsz], H, D, xr[j], [0],
                                        host["up_bias"][e * D:(e + 1) * D], u, [0])
            act = np.array([oracle.swiglu(g[i], u[i]) for i in range(D)], np.float32)
            oracle.mul_moe_batch_expert(host["down"][e * dsz:(e + 1) * dsz], D, H, act, [0],
                                        host["down_bias"][e * H:(e + 1) * H], rows_out[j], [0])
        # 5. results back, rank-ordered combine
        ret = torch.empty(sum(send_counts) * H, dtype=torch.float32)
        dist.all_to_all_single(ret, torch.from_numpy(rows_out.reshape(-1).copy()),
                               [c * H for c in send_counts], [c * H for c in recv_counts])
        ret = ret.numpy().reshape(-1, H)
        out = np.zeros((T, H), np.float32)
        for t in range(T):
            for r in range(K):
                s = t * K + r
                if s in send_pos:
                    out[t] = oracle.fmaf(ret[send_pos[s]], np.full(H, sel[t][r][1], np.float32), out[t])
        same = bool(np.array_equal(out.view(np.uint32), want.view(np.uint32)))
        results.put((rank, same, R, sum(send_counts)))
    except Exception as exc:  # report instead of hanging the peer
        results.put((rank, repr(exc), -1, -1))
        raise
    finally:
        dist.destroy_process_group()


def test_expert_parallel_protocol_matches_single_process():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, WORLD, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(WORLD):
        rank, same, recv, sent = q.get(timeout=240)
        got[rank] = (same, recv, sent)
    for p in procs:
        p.join(timeout=60)
    for rank, (same, recv, sent) in got.items():
        assert same is True, (rank, same)
    # every dispatched slot was received by exactly one rank
    assert sum(v[1] for v in got.values()) == sum(v[2] for v in got.values())


def test_expert_ranges_partition_every_expert():
    spt = importlib.import_module("stream-pt_b200")
    for e, world in [(128, 1), (128, 2), (128, 8), (8, 2), (12, 4)]:
        covered = []
        for r in range(world):
            b, en = spt.ep_expert_range(e, world, r)
            covered.extend(range(b, en))
        assert covered == list(range(e))
    assert spt.ep_expert_range(128, 8, 8) == (0, 0)   # rank out of range
    assert spt.ep_expert_range(128, 0, 0) == (0, 0)
