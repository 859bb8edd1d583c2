"""Arenas and the LM head built from GGUF model files (spt_arena_create_gguf,
spt_gguf_tensor) compute exactly what the synthetic arena of the same bytes
computes: the file path repacks the GGUF blocks on the device, the synthetic
path generates the same blocks there."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from oracle import oracle  # noqa: E402
from tests import gguf_writer as gw  # noqa: E402

pytestmark = pytest.mark.gpu


def test_gguf_arena_matches_synthetic(ctx, spt, tmp_path):
    cfg = spt.Config(256, 256, 16, 4)
    params = spt.SynthParams(seed=9)
    a, b = str(tmp_path / "m-00001.gguf"), str(tmp_path / "m-00002.gguf")
    md = gw.moe_metadata(cfg, eps=1e-5)
    gw.write_gguf(a, md + [("split.no", gw.U16, 0), ("split.count", gw.U16, 2)],
                  gw.moe_layer_tensors(spt, cfg, params, 0) + [gw.q80_tensor("output.weight", 1000, 256)])
    gw.write_gguf(b, md + [("split.no", gw.U16, 1), ("split.count", gw.U16, 2)],
                  gw.moe_layer_tensors(spt, cfg, params, 1))
    g = spt.Gguf([b, a])
    flags = spt.ARENA_GEMV | spt.ARENA_MMA
    from_file = ctx.arena_from_gguf(g, flags=flags)
    synth = ctx.synthetic_arena(cfg, params, n_layers=2, flags=flags)
    try:
        for T in (1, 7, 33):
            x = spt.synth_normal_host(9, T, T * 256)
            for path in (spt.PATH_EXACT, spt.PATH_MMA):
                ctx.set_path(path)
                for layer in (0, 1):
                    got = ctx.forward_moe_batch(from_file, x, T, layer=layer)
                    want = ctx.forward_moe_batch(synth, x, T, layer=layer)
                    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (T, path, layer)
                got = ctx.forward_stack(from_file, x, T)
                want = ctx.forward_stack(synth, x, T)
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (T, path, "stack")
        # an expert-parallel shard of the file holds the shard's experts
        shard = ctx.arena_from_gguf(g, flags=spt.ARENA_GEMV, experts=(4, 8))
        shard.close()
        # LM head straight from the file's tensor bytes
        t = g.tensor("output.weight")
        with open(a, "rb") as f:
            f.seek(t.start)
            data = np.frombuffer(f.read(t.end - t.start), np.uint8)
        x = spt.synth_normal_host(9, 77, 256)
        m = ctx.q80_matrix(data, 256, 1000)
        y, i, l = m.mul(x)
        want_y, want_i, want_l = oracle.mul_q80(data, 256, 1000, x)
        assert np.array_equal(y.view(np.uint32), want_y.view(np.uint32)) and i == want_i
        m.close()
    finally:
        from_file.close()
        synth.close()
        g.close()


@pytest.mark.parametrize("flags", ["gemv", "both"])
def test_arena_from_tensor_views_matches_reader_arena(ctx, spt, flags):
    import refdata
    """spt_arena_create_views (each tensor handed over as its own buffer, the
    way the Go shim passes ggufmap.Reader.WithTensor slices) builds the same
    arena as spt_arena_create over the whole file: identical outputs on the
    exact path, and on the tensor-core path when both layouts are built."""
    f = spt.ARENA_GEMV if flags == "gemv" else spt.ARENA_GEMV | spt.ARENA_MMA
    for bias in (-1, 1, 30):
        fx = refdata.moe_batch_fixture(96, 64, 7, 2, bias, "normal")
        x = refdata.moe_batch_x(9, 96, "normal")
        a = ctx.arena([fx.reader], fx.cfg, [fx.lw], flags=f)
        b = ctx.arena_views([fx.reader], fx.cfg, [fx.lw], flags=f)
        try:
            for path in ([spt.PATH_EXACT] if flags == "gemv" else [spt.PATH_EXACT, spt.PATH_MMA, spt.PATH_GEMV16]):
                ctx.set_path(path)
                ya = ctx.forward_moe_batch(a, x, 9)
                yb = ctx.forward_moe_batch(b, x, 9)
                assert refdata.bits_equal(ya, yb).all(), (bias, path)
        finally:
            ctx.set_path(spt.PATH_AUTO)
            a.close()
            b.close()
