"""GGUF model index (spt_gguf_*) on the host: the rules of ggufindex.Open
(ggufindex/index.go:55-575) and the NewLayerWeights suffix lookup
(forward/layer.go:39-86), on model files written by tests/gguf_writer.py."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from tests import gguf_writer as gw  # noqa: E402


@pytest.fixture(scope="module")
def small(spt):
    cfg = spt.Config(64, 64, 8, 2)
    params = spt.SynthParams(seed=5)
    return cfg, params


def file_bytes(path, t):
    with open(path, "rb") as f:
        f.seek(t.start)
        return f.read(t.end - t.start)


def test_single_file_model(spt, small, tmp_path, host_ctx):
    cfg, params = small
    path = str(tmp_path / "m.gguf")
    tensors = gw.moe_layer_tensors(spt, cfg, params, 0) + gw.moe_layer_tensors(spt, cfg, params, 1)
    tensors.append(gw.q80_tensor("output.weight", 40, 64))
    gw.write_gguf(path, gw.moe_metadata(cfg, n_layers=2, eps=2e-5, alignment=64), tensors, alignment=64)
    g = spt.Gguf([path])
    try:
        assert g.layer_count == 2
        c, eps = g.config()
        assert (c.hidden_dim, c.expert_hidden_dim, c.num_experts, c.num_experts_used) == (64, 64, 8, 2)
        assert eps == np.float32(2e-5)
        written = {name: (typ, shape, data) for name, typ, shape, data in tensors}
        for layer in range(2):
            lw = g.layer(layer)
            for field, t in lw.items():
                assert t.name, field
                typ, shape, data = written[t.name]
                assert t.type == typ and tuple(t.shape) == tuple(shape)
                assert file_bytes(path, t) == data
                assert t.start % 64 == 0
            # the layer's facts pass the block's own validation (validateMoEBatch*)
            view = spt.LayerWeights(**{k: v for k, v in lw.items()})
            host_ctx.validate(spt.Reader(np.fromfile(path, np.uint8)), cfg, view)
        out = g.tensor("output.weight")
        assert out.type == 8 and tuple(out.shape) == (64, 40)
        assert file_bytes(path, out) == written["output.weight"][2]
    finally:
        g.close()


def test_split_files_any_order(spt, small, tmp_path):
    cfg, params = small
    a, b = str(tmp_path / "m-00001.gguf"), str(tmp_path / "m-00002.gguf")
    md = gw.moe_metadata(cfg)
    gw.write_gguf(a, md + [("split.no", gw.U16, 0), ("split.count", gw.U16, 2)],
                  gw.moe_layer_tensors(spt, cfg, params, 0) + [gw.q80_tensor("output.weight", 8, 64)])
    gw.write_gguf(b, md + [("split.no", gw.U16, 1), ("split.count", gw.U16, 2)],
                  gw.moe_layer_tensors(spt, cfg, params, 1))
    for order in ([a, b], [b, a]):
        g = spt.Gguf(order)
        assert g.layer_count == 2  # no gpt_oss.block_count: the layers found
        assert g.layer(1)["ffn_down_exps"].name == "blk.1.ffn_down_exps.weight"
        g.close()
    with pytest.raises(spt.SptError, match="incomplete model: 1 of 2 splits provided"):
        spt.Gguf([a])


@pytest.mark.parametrize("case,match", [
    ("magic", "not a GGUF file"),
    ("version", "unsupported GGUF version 4"),
    ("truncated", "unexpected end of file"),
    ("dims", "invalid dimension count"),
    ("type", "unsupported GGML tensor type 99"),
    ("range", "byte range extends beyond the file"),
    ("alignment", "invalid alignment 48"),
    ("dupkey", "duplicate metadata key"),
    ("declared", "expected 3 layers, found 2"),
    ("gap", "layer 1 is missing"),
])
def test_malformed_models(spt, small, tmp_path, case, match):
    cfg, params = small
    path = str(tmp_path / f"{case}.gguf")
    md = gw.moe_metadata(cfg)
    tensors = gw.moe_layer_tensors(spt, cfg, params, 0) + gw.moe_layer_tensors(spt, cfg, params, 1)
    kw = {}
    if case == "magic":
        kw["magic"] = b"GGUG"
    elif case == "version":
        kw["version"] = 4
    elif case == "truncated":
        kw["truncate"] = 40
    elif case == "dims":
        tensors[0] = (tensors[0][0], 0, (), b"")
    elif case == "type":
        tensors[0] = (tensors[0][0], 99, (64,), tensors[0][3])
    elif case == "range":
        kw["truncate"] = 2000
    elif case == "alignment":
        md = md + [("general.alignment", gw.U32, 48)]
    elif case == "dupkey":
        md = md + [md[1]]
    elif case == "declared":
        md = md + [("gpt_oss.block_count", gw.U32, 3)]
    elif case == "gap":
        tensors = gw.moe_layer_tensors(spt, cfg, params, 0) + [
            (n.replace("blk.1.", "blk.2."), t, s, d) for n, t, s, d in gw.moe_layer_tensors(spt, cfg, params, 1)]
        md = md + [("gpt_oss.block_count", gw.U32, 2)]
        md = md[:-1]  # counted from the layers found (0 and 2): two layers, the second missing
    gw.write_gguf(path, md, tensors, **kw)
    with pytest.raises(spt.SptError, match=match) as e:
        spt.Gguf([path])
    assert e.value.status == spt.ERR_FORMAT


def test_model_level_consistency(spt, small, tmp_path):
    cfg, params = small
    a, b = str(tmp_path / "a.gguf"), str(tmp_path / "b.gguf")
    gw.write_gguf(a, gw.moe_metadata(cfg, alignment=64), gw.moe_layer_tensors(spt, cfg, params, 0), alignment=64)
    gw.write_gguf(b, gw.moe_metadata(cfg, alignment=32), gw.moe_layer_tensors(spt, cfg, params, 1), alignment=32)
    with pytest.raises(spt.SptError, match="inconsistent tensor alignment"):
        spt.Gguf([a, b])
    gw.write_gguf(b, gw.moe_metadata(cfg, alignment=64), gw.moe_layer_tensors(spt, cfg, params, 0), alignment=64)
    with pytest.raises(spt.SptError, match="duplicate tensor"):
        spt.Gguf([a, b])
    md = gw.moe_metadata(cfg, alignment=64)
    md[1] = ("gpt-oss.embedding_length", gw.U32, 128)
    gw.write_gguf(b, md, gw.moe_layer_tensors(spt, cfg, params, 1), alignment=64)
    with pytest.raises(spt.SptError, match="inconsistent metadata"):
        spt.Gguf([a, b])
    with pytest.raises(spt.SptError, match="duplicate file"):
        spt.Gguf([a, a])
