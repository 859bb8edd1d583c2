"""Failure paths, exercised without a GPU fault.

The reference returns ctx.Err() when its caller cancels
(tests/testdata/forward/moe_batch_test.go:252-261); the B200 block also has
device-side waits (the tcgen05 GEMM's mbarrier ring) and host-side waits on
the expert-parallel exchange, each bounded so that a stalled party turns into
an error status instead of a hang.  These tests make such a wait run out:

* a GEMM whose producer skips one pipeline stage (the test hook
  SPT_OPT_FAULT_STAGE), with a short wait limit: the MMA issuer's wait for
  that stage gives up, the CTA waits for its own copies in flight, frees its
  tensor memory and returns, and the call reports SPT_ERR_TIMEOUT; the next
  normal call on the same context is correct;
* a router CTA that leaves out one row's copy (SPT_OPT_FAULT_STAGE = 1000):
  the router's wait for its rows gives up, the CTA waits for the copies it
  did issue and leaves (still counting itself for the last-CTA selection),
  and the call reports SPT_ERR_TIMEOUT; the next normal call is correct;
* an expert-parallel group whose second rank never joins: the set-up wait
  gives up after SPT_EP_TIMEOUT_MS and the group is aborted (no exchange
  kernel was launched); the context keeps working.
"""
import time

import numpy as np
import pytest

import refdata
from oracle import oracle

pytestmark = pytest.mark.gpu
spt = refdata.spt


HID, DIM = 1024, 256  # gate/up: 8 K tiles, two pipeline stages per row tile


@pytest.fixture()
def small(ctx):
    cfg = spt.Config(HID, DIM, 16, 4)
    params = spt.SynthParams(seed=21)
    arena = ctx.synthetic_arena(cfg, params, flags=spt.ARENA_MMA)
    dense = oracle.synth_weights(HID, DIM, 16, 4, oracle.synth_params(seed=21))
    yield cfg, arena, dense
    arena.close()
    ctx.set_path(spt.PATH_AUTO)
    ctx.set_option(spt.OPT_FAULT_STAGE, -1)
    ctx.set_option(spt.OPT_WAIT_LIMIT, 31)


def _close(got, want):
    got, want = np.ravel(got).astype(np.float64), np.ravel(want).astype(np.float64)
    err = np.abs(got - want).max() / np.abs(want).max()
    return err <= 1e-3


@pytest.mark.parametrize("stage", [0, 1])
def test_gemm_wait_gives_up_and_context_recovers(ctx, small, stage):
    cfg, arena, dense = small
    T = 24
    x = spt.synth_normal_host(21, 5, T * HID)
    want = oracle.forward_moe_batch(dense, x, T)
    ctx.set_path(spt.PATH_MMA)
    ctx.set_option(spt.OPT_WAIT_LIMIT, 20)  # about half a millisecond
    ctx.set_option(spt.OPT_FAULT_STAGE, stage)
    t0 = time.perf_counter()
    with pytest.raises(spt.SptError) as e:
        ctx.forward_moe_batch(arena, x, T)
    assert e.value.status == spt.ERR_TIMEOUT, e.value
    assert time.perf_counter() - t0 < 30
    # the same context, the fault hook off: a normal, correct call
    ctx.set_option(spt.OPT_FAULT_STAGE, -1)
    ctx.set_option(spt.OPT_WAIT_LIMIT, 31)
    got = ctx.forward_moe_batch(arena, x, T)
    assert _close(got, want)


@pytest.mark.parametrize("T", [4, 24])
def test_router_wait_gives_up_and_context_recovers(ctx, small, T):
    """T = 4: the router with the selection and dispatch in its last CTA;
    T = 24: the plain shared-memory router."""
    cfg, arena, dense = small
    x = spt.synth_normal_host(22, 5, T * HID)
    want = oracle.forward_moe_batch(dense, x, T)
    ctx.set_path(spt.PATH_MMA)
    ctx.set_option(spt.OPT_WAIT_LIMIT, 20)
    ctx.set_option(spt.OPT_FAULT_STAGE, 1000)
    t0 = time.perf_counter()
    with pytest.raises(spt.SptError) as e:
        ctx.forward_moe_batch(arena, x, T)
    assert e.value.status == spt.ERR_TIMEOUT, e.value
    assert "router" in str(e.value)
    assert time.perf_counter() - t0 < 30
    ctx.set_option(spt.OPT_FAULT_STAGE, -1)
    ctx.set_option(spt.OPT_WAIT_LIMIT, 31)
    for _ in range(2):  # the counter of the last-CTA selection is back at 0
        got = ctx.forward_moe_batch(arena, x, T)
        assert _close(got, want)


@pytest.mark.timeout(180)
def test_expert_parallel_setup_times_out_without_peer(ctx, small, monkeypatch):
    """Rank 0 of a group of two, whose rank 1 never arrives (the failure is
    made on the host: there is no second process)."""
    cfg, arena, dense = small
    monkeypatch.setenv("SPT_EP_TIMEOUT_MS", "1500")
    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")
    uid = spt.ep_unique_id()
    t0 = time.perf_counter()
    with pytest.raises(spt.SptError) as e:
        spt.ExpertParallel(ctx, uid, 0, 2)
    waited = time.perf_counter() - t0
    assert e.value.status == spt.ERR_NCCL, e.value
    assert 1.0 <= waited < 60, waited
    x = spt.synth_normal_host(22, 5, 3 * HID)
    assert _close(ctx.forward_moe_batch(arena, x, 3), oracle.forward_moe_batch(dense, x, 3))
