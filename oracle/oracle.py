"""ctypes binding of the CPU oracle (oracle/spt_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()``
as the checker, and by ``bench.py``'s CPU-baseline leg.  The product library
under ``stream-pt_b200/`` never imports this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libspt_oracle.so")


def build() -> str:
    """Compile the oracle with its Makefile (gcc, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class Selection(ctypes.Structure):
    _fields_ = [("index", ctypes.c_int32), ("weight", ctypes.c_float)]


class MoEWeights(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_int64), ("expert_dim", ctypes.c_int64),
        ("experts", ctypes.c_int64), ("top_k", ctypes.c_int64),
        ("router", ctypes.c_void_p), ("router_bias", ctypes.c_void_p),
        ("gate", ctypes.c_void_p), ("up", ctypes.c_void_p), ("down", ctypes.c_void_p),
        ("gate_bias", ctypes.c_void_p), ("up_bias", ctypes.c_void_p),
        ("down_bias", ctypes.c_void_p),
    ]


class SynthParams(ctypes.Structure):
    """The benchmark's synthetic-layer parameters (spo_synth_params)."""
    _fields_ = [("seed", ctypes.c_uint64), ("router_std", ctypes.c_float), ("bias_std", ctypes.c_float),
                ("scale_lo", ctypes.c_uint8), ("scale_hi", ctypes.c_uint8), ("expert_bias", ctypes.c_uint8),
                ("router_bias", ctypes.c_uint8), ("zipf_s", ctypes.c_float), ("zipf_beta", ctypes.c_float)]


def synth_params(seed=0, router_std=0.02, bias_std=0.01, scale_lo=119, scale_hi=123, expert_bias=True,
                 router_bias=True, zipf_s=0.0, zipf_beta=0.0) -> SynthParams:
    return SynthParams(seed, router_std, bias_std, scale_lo, scale_hi, int(expert_bias), int(router_bias),
                       zipf_s, zipf_beta)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        vp, i64, f32, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_float, ctypes.c_int
        L.spo_init.restype = None
        L.spo_e8m0.argtypes = [ctypes.c_uint8]; L.spo_e8m0.restype = f32
        L.spo_scaled_fp4.argtypes = [ctypes.c_uint8, ctypes.c_uint8]; L.spo_scaled_fp4.restype = f32
        L.spo_f16.argtypes = [ctypes.c_uint16]; L.spo_f16.restype = f32
        L.spo_bf16.argtypes = [ctypes.c_uint16]; L.spo_bf16.restype = f32
        L.spo_decode_float_vector.argtypes = [vp, ctypes.c_uint32, i64, vp]
        L.spo_decode_float_vector.restype = i32
        L.spo_decode_mxfp4.argtypes = [vp, i64, vp]; L.spo_decode_mxfp4.restype = None
        L.spo_dot_mxfp4.argtypes = [vp, vp, i64]; L.spo_dot_mxfp4.restype = f32
        L.spo_dot_mxfp4_scalar.argtypes = [vp, vp, i64]; L.spo_dot_mxfp4_scalar.restype = f32
        L.spo_dot_router.argtypes = [vp, vp, i64]; L.spo_dot_router.restype = f32
        L.spo_set_portable_lanes.argtypes = [i32]; L.spo_set_portable_lanes.restype = None
        L.spo_get_portable_lanes.restype = i32
        L.spo_route.argtypes = [vp, vp, vp, i64, i64, i64, vp]; L.spo_route.restype = None
        L.spo_select.argtypes = [vp, i64, i64, vp]; L.spo_select.restype = None
        L.spo_swiglu.argtypes = [f32, f32]; L.spo_swiglu.restype = f32
        L.spo_mul_moe_batch_expert.argtypes = [vp, i64, i64, vp, vp, i64, vp, vp, vp, i32]
        L.spo_mul_moe_batch_expert.restype = None
        L.spo_forward_moe_batch.argtypes = [ctypes.POINTER(MoEWeights), vp, i64, vp, i32,
                                            vp, vp, vp, vp, vp, vp]
        L.spo_forward_moe_batch.restype = i64
        L.spo_scalar_sparse_moe_f64.argtypes = [ctypes.POINTER(MoEWeights), vp, vp]
        L.spo_scalar_sparse_moe_f64.restype = None
        L.spo_rmsnorm.argtypes = [vp, vp, i64, i64, f32, vp]; L.spo_rmsnorm.restype = None
        L.spo_add.argtypes = [vp, vp, i64]; L.spo_add.restype = None
        L.spo_dot_q80.argtypes = [vp, vp, i64]; L.spo_dot_q80.restype = f32
        L.spo_mul_q80.argtypes = [vp, i64, i64, vp, vp, vp, i32]; L.spo_mul_q80.restype = i64
        L.spo_dot_q40.argtypes = [vp, vp, i64]; L.spo_dot_q40.restype = f32
        L.spo_mul_q40.argtypes = [vp, i64, i64, vp, i64, vp, i32]; L.spo_mul_q40.restype = None
        L.spo_has_avx2.restype = i32
        L.spo_synth_layer.argtypes = [ctypes.POINTER(SynthParams), i64, i64, i64, i64, vp, vp, vp, vp, vp, vp,
                                      vp, vp, i32]
        L.spo_synth_layer.restype = i32
        L.spo_synth_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint32, f32, f32, vp, i64]
        L.spo_synth_normal.restype = None
        L.spo_synth_experts.argtypes = [ctypes.POINTER(SynthParams), i64, i64, i64, i64, vp, i64, vp, vp, vp, i32]
        L.spo_synth_experts.restype = i32
        L.spo_synth_norm.argtypes = [ctypes.c_uint64, i64, i64, vp]
        L.spo_synth_norm.restype = None
        L.spo_fmaf_vec.argtypes = [vp, vp, vp, vp, i64]; L.spo_fmaf_vec.restype = None
        L.spo_init()
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def decode_mxfp4(row: np.ndarray) -> np.ndarray:
    row = np.ascontiguousarray(row, dtype=np.uint8)
    nb = row.size // 17
    out = np.empty(nb * 32, np.float32)
    lib().spo_decode_mxfp4(_p(row), nb, _p(out))
    return out


def dot_mxfp4(row, x, scalar=False) -> float:
    row = np.ascontiguousarray(row, dtype=np.uint8)
    x = _f32(x)
    fn = lib().spo_dot_mxfp4_scalar if scalar else lib().spo_dot_mxfp4
    return np.float32(fn(_p(row), _p(x), x.size))


def route(router_bytes, x, bias, batch, hidden, experts) -> np.ndarray:
    rb = np.ascontiguousarray(router_bytes, dtype=np.uint8)
    x = _f32(x)
    bias = _f32(bias)
    logits = np.empty(batch * experts, np.float32)
    lib().spo_route(_p(rb), _p(x), _p(bias), batch, hidden, experts, _p(logits))
    return logits.reshape(batch, experts)


def select(logits_row, k):
    lg = _f32(logits_row)
    sel = (Selection * k)()
    lib().spo_select(_p(lg), lg.size, k, ctypes.byref(sel))
    return [(s.index, np.float32(s.weight)) for s in sel]


def swiglu(g, u) -> np.float32:
    return np.float32(lib().spo_swiglu(float(g), float(u)))


def mul_moe_batch_expert(data, input_, output, x, xoff, bias, y, yoff, workers=1):
    data = np.ascontiguousarray(data, dtype=np.uint8)
    x = _f32(x)
    xo = np.ascontiguousarray(xoff, dtype=np.int64)
    yo = np.ascontiguousarray(yoff, dtype=np.int64)
    bias = _f32(bias)
    assert y.dtype == np.float32 and y.flags.c_contiguous
    lib().spo_mul_moe_batch_expert(_p(data), input_, output, _p(x), _p(xo), xo.size,
                                   _p(bias), _p(y), _p(yo), workers)
    return y


class Weights:
    """Dense decoded inputs for the whole block (keeps the arrays alive)."""

    def __init__(self, hidden, expert_dim, experts, top_k, router, router_bias,
                 gate, up, down, gate_bias=None, up_bias=None, down_bias=None):
        self.arrays = dict(
            router=np.ascontiguousarray(router, dtype=np.uint8),
            router_bias=_f32(router_bias),
            gate=np.ascontiguousarray(gate, dtype=np.uint8),
            up=np.ascontiguousarray(up, dtype=np.uint8),
            down=np.ascontiguousarray(down, dtype=np.uint8),
            gate_bias=_f32(gate_bias), up_bias=_f32(up_bias), down_bias=_f32(down_bias))
        a = self.arrays
        self.hidden, self.expert_dim, self.experts, self.top_k = hidden, expert_dim, experts, top_k
        self.c = MoEWeights(hidden, expert_dim, experts, top_k,
                            _p(a["router"]), _p(a["router_bias"]), _p(a["gate"]),
                            _p(a["up"]), _p(a["down"]), _p(a["gate_bias"]),
                            _p(a["up_bias"]), _p(a["down_bias"]))


def forward_moe_batch(w: Weights, x, batch, workers=1, want_internals=False):
    x = _f32(x)
    H, D, E, K = w.hidden, w.expert_dim, w.experts, w.top_k
    S = batch * K
    out = np.empty(batch * H, np.float32)
    if not want_internals:
        lib().spo_forward_moe_batch(ctypes.byref(w.c), _p(x), batch, _p(out), workers,
                                    None, None, None, None, None, None)
        return out.reshape(batch, H)
    logits = np.empty(batch * E, np.float32)
    sel = (Selection * max(S, 1))()
    perm = np.full(max(S, 1), -1, np.int32)
    counts = np.zeros(E, np.int32)
    act = np.zeros(S * D, np.float32)
    res = np.zeros(S * H, np.float32)
    n = lib().spo_forward_moe_batch(ctypes.byref(w.c), _p(x), batch, _p(out), workers,
                                    _p(logits), ctypes.byref(sel), _p(perm), _p(counts),
                                    _p(act), _p(res))
    sel_idx = np.array([sel[i].index for i in range(S)], np.int32).reshape(batch, K)
    sel_w = np.array([sel[i].weight for i in range(S)], np.float32).reshape(batch, K)
    return dict(out=out.reshape(batch, H), logits=logits.reshape(batch, E), sel_idx=sel_idx,
                sel_w=sel_w, perm=perm[:n], counts=counts, act=act.reshape(S, D),
                results=res.reshape(S, H), dispatched=int(n))


def scalar_sparse_moe_f64(w: Weights, x_row) -> np.ndarray:
    x = _f32(x_row)
    out = np.empty(w.hidden, np.float32)
    lib().spo_scalar_sparse_moe_f64(ctypes.byref(w.c), _p(x), _p(out))
    return out


def rmsnorm(x, weight, batch, dim, eps):
    x = _f32(x); weight = _f32(weight)
    y = np.empty(batch * dim, np.float32)
    lib().spo_rmsnorm(_p(x), _p(weight), batch, dim, float(eps), _p(y))
    return y.reshape(batch, dim)


def dot_q80(row, x) -> np.float32:
    row = np.ascontiguousarray(row, dtype=np.uint8)
    x = _f32(x)
    return np.float32(lib().spo_dot_q80(_p(row), _p(x), x.size))


def mul_q80(data, input_, output, x, workers=1):
    data = np.ascontiguousarray(data, dtype=np.uint8)
    x = _f32(x)
    y = np.empty(output, np.float32)
    best = ctypes.c_float()
    idx = lib().spo_mul_q80(_p(data), input_, output, _p(x), _p(y), ctypes.byref(best), workers)
    return y, int(idx), np.float32(best.value)


def dot_q40(row, x) -> np.float32:
    row = np.ascontiguousarray(row, dtype=np.uint8)
    x = _f32(x)
    return np.float32(lib().spo_dot_q40(_p(row), _p(x), x.size))


def mul_q40(data, input_, output, x, batch=1, workers=1):
    """MulQ40BatchInto: y [batch, output] for x [batch, input]."""
    data = np.ascontiguousarray(data, dtype=np.uint8)
    x = _f32(x)
    assert x.size == batch * input_ and data.size == output * (input_ // 32) * 18
    y = np.empty(batch * output, np.float32)
    lib().spo_mul_q40(_p(data), input_, output, _p(x), batch, _p(y), workers)
    return y.reshape(batch, output)


def fmaf(a, b, c) -> np.ndarray:
    """Elementwise single-rounding float32 fma (C fmaf)."""
    a, b, c = np.broadcast_arrays(_f32(a), _f32(b), _f32(c))
    a, b, c = (np.ascontiguousarray(v, dtype=np.float32) for v in (a, b, c))
    out = np.empty(a.shape, np.float32)
    lib().spo_fmaf_vec(_p(a), _p(b), _p(c), _p(out), out.size)
    return out


def synth_layer(hidden, expert_dim, experts, params: SynthParams, layer=0, threads=None) -> dict:
    """One synthetic layer in GGUF tensor layout, generated by the oracle
    (same bytes as the CUDA library's generator)."""
    H, D, E = hidden, expert_dim, experts
    out = dict(router=np.empty(E * H * 4, np.uint8), router_bias=np.empty(E, np.float32),
               gate=np.empty(E * D * (H // 32) * 17, np.uint8), up=np.empty(E * D * (H // 32) * 17, np.uint8),
               down=np.empty(E * H * (D // 32) * 17, np.uint8), gate_bias=np.empty(E * D, np.float32),
               up_bias=np.empty(E * D, np.float32), down_bias=np.empty(E * H, np.float32))
    o = out
    r = lib().spo_synth_layer(ctypes.byref(params), H, D, E, layer, _p(o["router"]), _p(o["router_bias"]),
                              _p(o["gate"]), _p(o["up"]), _p(o["down"]), _p(o["gate_bias"]), _p(o["up_bias"]),
                              _p(o["down_bias"]), threads or os.cpu_count() or 1)
    if r != 0:
        raise ValueError("invalid synthetic layer dimensions")
    return out


def synth_layer_experts(hidden, expert_dim, experts, params: SynthParams, layer, ids, threads=None) -> dict:
    """A synthetic layer whose expert tensors hold only the experts `ids`
    (the others stay zero; the forward reads only the selected experts):
    for checking a few tokens of a deep stack without generating 1.7 GB per
    layer.  Router and biases are complete."""
    H, D, E = hidden, expert_dim, experts
    out = dict(router=np.empty(E * H * 4, np.uint8), router_bias=np.empty(E, np.float32),
               gate=np.zeros(E * D * (H // 32) * 17, np.uint8), up=np.zeros(E * D * (H // 32) * 17, np.uint8),
               down=np.zeros(E * H * (D // 32) * 17, np.uint8), gate_bias=np.empty(E * D, np.float32),
               up_bias=np.empty(E * D, np.float32), down_bias=np.empty(E * H, np.float32))
    o = out
    r = lib().spo_synth_layer(ctypes.byref(params), H, D, E, layer, _p(o["router"]), _p(o["router_bias"]), None,
                              None, None, _p(o["gate_bias"]), _p(o["up_bias"]), _p(o["down_bias"]), 1)
    ids = np.ascontiguousarray(sorted(set(int(i) for i in ids)), dtype=np.int32)
    if r == 0 and ids.size:
        r = lib().spo_synth_experts(ctypes.byref(params), H, D, E, layer, _p(ids), ids.size, _p(o["gate"]),
                                    _p(o["up"]), _p(o["down"]), threads or os.cpu_count() or 1)
    if r != 0:
        raise ValueError("invalid synthetic layer dimensions")
    return out


def weights_of(layer: dict, hidden, expert_dim, experts, top_k) -> "Weights":
    return Weights(hidden, expert_dim, experts, top_k, layer["router"], layer["router_bias"], layer["gate"],
                   layer["up"], layer["down"], layer["gate_bias"], layer["up_bias"], layer["down_bias"])


def route_threads(router_bytes, x, bias, batch, hidden, experts, threads=None) -> np.ndarray:
    """route() over token chunks on several threads (same values)."""
    from concurrent.futures import ThreadPoolExecutor
    x = _f32(x).reshape(batch, hidden)
    n = max(1, min(threads or os.cpu_count() or 1, batch))
    chunks = [(i * batch // n, (i + 1) * batch // n) for i in range(n)]
    with ThreadPoolExecutor(n) as ex:
        parts = list(ex.map(lambda c: route(router_bytes, x[c[0]:c[1]], bias, c[1] - c[0], hidden, experts), chunks))
    return np.concatenate(parts, axis=0)


def dispatch_perm(sel_idx, sel_w, experts) -> tuple:
    """The reference's dispatch order (moe_batch.go:142-159): slots whose
    weight is > 0 or NaN, grouped by expert ascending, each expert's slots in
    descending slot order.  Returns (perm, per-expert counts)."""
    idx = np.asarray(sel_idx).ravel()
    w = np.asarray(sel_w, np.float32).ravel()
    live = ~(w <= 0)
    slots = np.nonzero(live)[0]
    order = np.lexsort((-slots, idx[slots]))
    return slots[order].astype(np.int32), np.bincount(idx[slots], minlength=experts).astype(np.int32)


def synth_weights(hidden, expert_dim, experts, top_k, params: SynthParams, layer=0, threads=None) -> Weights:
    h = synth_layer(hidden, expert_dim, experts, params, layer, threads)
    return Weights(hidden, expert_dim, experts, top_k, h["router"], h["router_bias"], h["gate"], h["up"],
                   h["down"], h["gate_bias"], h["up_bias"], h["down_bias"])


def synth_normal(seed, stream, n, mean=0.0, std=1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().spo_synth_normal(seed, stream & 0xFFFFFFFF, mean, std, _p(out), n)
    return out


def synth_norm(seed, layer, dim) -> np.ndarray:
    out = np.empty(dim, np.float32)
    lib().spo_synth_norm(seed, layer, dim, _p(out))
    return out
