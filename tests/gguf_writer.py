"""Minimal GGUF (v2/v3) writer for tests: metadata, tensor directory,
aligned tensor data.  Builds GPT-OSS-style MoE model files from the
library's seeded synthetic layers (the same bytes as a synthetic arena)."""
from __future__ import annotations

import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?",
           U64: "<Q", I64: "<q", F64: "<d"}


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(typ, v) -> bytes:
    if typ == STR:
        return _str(v)
    if typ == ARR:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, x) for x in items)
    return struct.pack(_SCALAR[typ], v)


def write_gguf(path, metadata, tensors, alignment=32, version=3, magic=b"GGUF", truncate=None):
    """metadata: [(key, type, value)], tensors: [(name, ggml_type, shape, bytes)]."""
    head = bytearray(magic + struct.pack("<IQQ", version, len(tensors), len(metadata)))
    for key, typ, val in metadata:
        head += _str(key) + struct.pack("<I", typ) + _value(typ, val)
    offsets, off = [], 0
    for _, _, _, data in tensors:
        off = (off + alignment - 1) // alignment * alignment
        offsets.append(off)
        off += len(data)
    for (name, typ, shape, _), o in zip(tensors, offsets):
        head += _str(name) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in shape)
        head += struct.pack("<IQ", typ, o)
    base = (len(head) + alignment - 1) // alignment * alignment
    out = bytearray(head) + bytes(base - len(head))
    for (_, _, _, data), o in zip(tensors, offsets):
        out += bytes(base + o - len(out)) + bytes(data)
    if truncate is not None:
        out = out[:truncate]
    with open(path, "wb") as f:
        f.write(out)
    return base, offsets


def moe_layer_tensors(spt, cfg, params, layer):
    """GGUF tensors of one synthetic MoE layer (ffn_* and post_attention_norm)."""
    H, D, E = cfg.hidden_dim, cfg.expert_hidden_dim, cfg.num_experts
    h = spt.synth_layer_host(cfg, params, layer)
    norm = spt.synth_norm_host(params, layer, H)
    p = f"blk.{layer}."
    return [
        (p + "post_attention_norm.weight", 0, (H,), norm.tobytes()),
        (p + "ffn_gate_inp.weight", 0, (H, E), h["router"].tobytes()),
        (p + "ffn_gate_inp.bias", 0, (E,), h["router_bias"].tobytes()),
        (p + "ffn_gate_exps.weight", 39, (H, D, E), h["gate"].tobytes()),
        (p + "ffn_gate_exps.bias", 0, (D, E), h["gate_bias"].tobytes()),
        (p + "ffn_up_exps.weight", 39, (H, D, E), h["up"].tobytes()),
        (p + "ffn_up_exps.bias", 0, (D, E), h["up_bias"].tobytes()),
        (p + "ffn_down_exps.weight", 39, (D, H, E), h["down"].tobytes()),
        (p + "ffn_down_exps.bias", 0, (H, E), h["down_bias"].tobytes()),
    ]


def moe_metadata(cfg, n_layers=None, eps=1e-5, alignment=None):
    md = [("general.architecture", STR, "gpt-oss"),
          ("gpt-oss.embedding_length", U32, cfg.hidden_dim),
          ("gpt-oss.expert_count", U32, cfg.num_experts),
          ("gpt-oss.expert_used_count", U32, cfg.num_experts_used),
          ("gpt-oss.expert_feed_forward_length", U32, cfg.expert_hidden_dim),
          ("gpt-oss.attention.layer_norm_rms_epsilon", F32, eps),
          ("tokenizer.ggml.tokens", ARR, (STR, ["<a>", "<b>"]))]
    if n_layers is not None:
        md.append(("gpt_oss.block_count", U32, n_layers))
    if alignment is not None:
        md.append(("general.alignment", U32, alignment))
    return md


def q80_tensor(name, rows, inp, seed=3):
    rng = np.random.default_rng(seed)
    data = rng.integers(0, 256, size=(rows, inp // 32, 34), dtype=np.uint8)
    data[:, :, :2] = (rng.standard_normal((rows, inp // 32)) * 0.05).astype(np.float16).view(np.uint8).reshape(
        rows, inp // 32, 2)
    return (name, 8, (inp, rows), data.tobytes())
