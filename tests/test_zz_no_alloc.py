"""The allocation-free entry point (spt_forward_moe_batch_device_static).

It exists for callers that cannot let the library allocate device memory
while they run (an engine that reserved all of HBM at load time, or a decode
loop that must not pay cudaMalloc's device-wide synchronisation), so it keeps
its intermediates in a static device array.  This test calls it through the
C ABI twice in a row, with different batches, and compares each result with
the allocating entry point (spt_forward_moe_batch_device) on the same inputs.
Both run the exact path, so the tolerance is the one the exact-path tests
use: bit-identical outputs.  The file is named to be collected last.
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


def test_static_scratch_matches_allocating_entry_point():
    import torch

    spt = importlib.import_module("stream-pt_b200")
    ctx = spt.Context(0)
    cfg = spt.Config(2880, 2880, 128, 4)
    arena = ctx.synthetic_arena(cfg, spt.SynthParams(seed=11), flags=spt.ARENA_GEMV)
    try:
        for call, (T, seed) in enumerate([(16, 101), (3, 202)]):
            x = torch.from_numpy(spt.synth_normal_host(seed, 3000, T * 2880)).cuda()
            want = torch.full_like(x, float("nan"))
            got = torch.full_like(x, float("nan"))
            torch.cuda.synchronize()
            ctx.forward_moe_batch_device(arena, x.data_ptr(), want.data_ptr(), T)
            ctx.sync()
            ctx.forward_moe_batch_device_static(arena, x.data_ptr(), got.data_ptr(), T)
            ctx.sync()
            g, w = got.cpu().numpy(), want.cpu().numpy()
            assert np.isfinite(w).all(), call
            assert np.array_equal(g.view(np.uint32), w.view(np.uint32)), call
            # the static call's routing stays in the static array: the
            # context's routing record refuses rather than report the
            # previous allocating call
            with pytest.raises(spt.SptError):
                ctx.last_routing(T, 128, 4)
        # sizes beyond the static array are refused before any device work
        x = torch.zeros(17 * 2880, device="cuda")
        with pytest.raises(spt.SptError) as e:
            ctx.forward_moe_batch_device_static(arena, x.data_ptr(), x.data_ptr(), 17)
        assert e.value.status == spt.ERR_UNSUPPORTED
    finally:
        arena.close()
        ctx.close()
