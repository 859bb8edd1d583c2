"""Stream-PT MoE FFN block on B200: Python host mirror of the C ABI.

The compute path is the sm_100a library ``libspt_moe.so`` built from
``csrc/`` (``include/spt_moe.h`` is its interface).  This module mirrors the
reference's Go interface of package ``forward`` for tests and benchmarks:
``Tensor``/``Reader``/``Config``/``LayerWeights`` stand for ggufindex.Tensor,
ggufmap.Reader, forward.Config and forward.LayerWeights, and each function
raises ``SptError`` where the Go function returns an error.

There is no CPU fallback: if the library is missing or no CUDA device is
present, every compute call raises.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field
from typing import Tuple, Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libspt_moe.so")

# spt_status codes (include/spt_moe.h)
OK, ERR_NULL_ARG, ERR_DIMENSIONS, ERR_OVERLAP, ERR_ROUTER, ERR_EXPERT, ERR_BIAS = range(7)
ERR_FILE_RANGE, ERR_SCRATCH, ERR_CANCELED, ERR_CUDA, ERR_NCCL, ERR_TIMEOUT = range(7, 13)
ERR_UNSUPPORTED, ERR_NO_DEVICE = 13, 14

ARENA_GEMV, ARENA_MMA = 1, 2
ERR_FORMAT = 15
PATH_AUTO, PATH_EXACT, PATH_MMA, PATH_GEMV16 = 0, 1, 2, 3
# spt_context_set_option (include/spt_moe.h)
OPT_TILE_TOKENS, OPT_FUSED_SELECT, OPT_L2_PREFETCH, OPT_GEMV16_SLOTS, OPT_WAIT_LIMIT, OPT_FAULT_STAGE = 1, 2, 3, 4, 5, 6
OPT_HOST_GRAPHS = 7
OPT_PREFILL_FP8 = 8
EP_EXCHANGE_PEER, EP_EXCHANGE_NCCL = 0, 1

GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16, GGML_MXFP4 = 0, 1, 8, 30, 39


class SptError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status
        self.message = message


class CanceledError(SptError):
    """context.Canceled equivalent."""


# ---- C structs ------------------------------------------------------------
class _Tensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("type", ctypes.c_uint32), ("n_dims", ctypes.c_uint32),
                ("shape", ctypes.c_uint64 * 4), ("start", ctypes.c_uint64), ("end", ctypes.c_uint64)]


class _Reader(ctypes.Structure):
    _fields_ = [("base", ctypes.c_void_p), ("size", ctypes.c_uint64)]


class _Config(ctypes.Structure):
    _fields_ = [("hidden_dim", ctypes.c_int64), ("expert_hidden_dim", ctypes.c_int64),
                ("num_experts", ctypes.c_int64), ("num_experts_used", ctypes.c_int64)]


class _LayerWeights(ctypes.Structure):
    _fields_ = [(n, _Tensor) for n in (
        "ffn_gate_inp", "ffn_gate_inp_bias", "ffn_gate_exps", "ffn_gate_exps_bias",
        "ffn_up_exps", "ffn_up_exps_bias", "ffn_down_exps", "ffn_down_exps_bias", "post_attention_norm")]


class _LayerData(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n, _ in _LayerWeights._fields_]


class _SynthParams(ctypes.Structure):
    _fields_ = [("seed", ctypes.c_uint64), ("router_std", ctypes.c_float),
                ("bias_std", ctypes.c_float), ("scale_lo", ctypes.c_uint8),
                ("scale_hi", ctypes.c_uint8), ("expert_bias", ctypes.c_uint8),
                ("router_bias", ctypes.c_uint8), ("zipf_s", ctypes.c_float),
                ("zipf_beta", ctypes.c_float)]


# ---- Go-side value types ---------------------------------------------------
@dataclass
class Tensor:
    """ggufindex.Tensor: name ('' = absent), GGML type, shape (ne0 first), byte range."""
    name: str = ""
    type: int = 0
    shape: Sequence[int] = ()
    start: int = 0
    end: int = 0

    def _c(self) -> _Tensor:
        t = _Tensor()
        t.name = self.name.encode() if self.name else None
        t.type = self.type
        shape = list(self.shape)
        t.n_dims = len(shape)
        for i, v in enumerate(shape[:4]):
            t.shape[i] = int(v) & ((1 << 64) - 1)
        if len(shape) > 4:
            t.n_dims = 5  # never valid for the MoE tensors
        t.start = int(self.start) & ((1 << 64) - 1)
        t.end = int(self.end) & ((1 << 64) - 1)
        return t


@dataclass
class Config:
    """The forward.Config fields the MoE block reads."""
    hidden_dim: int
    expert_hidden_dim: int
    num_experts: int
    num_experts_used: int

    def _c(self) -> _Config:
        m = (1 << 63) - 1
        def clamp(v):
            return max(-(1 << 63), min(m, int(v)))
        return _Config(clamp(self.hidden_dim), clamp(self.expert_hidden_dim),
                       clamp(self.num_experts), clamp(self.num_experts_used))


@dataclass
class LayerWeights:
    ffn_gate_inp: Tensor = field(default_factory=Tensor)
    ffn_gate_inp_bias: Tensor = field(default_factory=Tensor)
    ffn_gate_exps: Tensor = field(default_factory=Tensor)
    ffn_gate_exps_bias: Tensor = field(default_factory=Tensor)
    ffn_up_exps: Tensor = field(default_factory=Tensor)
    ffn_up_exps_bias: Tensor = field(default_factory=Tensor)
    ffn_down_exps: Tensor = field(default_factory=Tensor)
    ffn_down_exps_bias: Tensor = field(default_factory=Tensor)
    post_attention_norm: Tensor = field(default_factory=Tensor)

    def _c(self) -> _LayerWeights:
        lw = _LayerWeights()
        for name, _ in _LayerWeights._fields_:
            setattr(lw, name, getattr(self, name)._c())
        return lw


class Reader:
    """ggufmap.Reader stand-in: a host byte buffer holding the model file."""

    def __init__(self, data: bytes | bytearray | np.ndarray):
        self.buf = np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) \
            else np.ascontiguousarray(data, dtype=np.uint8)

    def _c(self) -> _Reader:
        return _Reader(self.buf.ctypes.data if self.buf.size else None, self.buf.size)


@dataclass
class SynthParams:
    seed: int = 0
    router_std: float = 0.02
    bias_std: float = 0.01
    scale_lo: int = 119
    scale_hi: int = 123
    expert_bias: bool = True
    router_bias: bool = True
    zipf_s: float = 0.0
    zipf_beta: float = 0.0

    def _c(self) -> _SynthParams:
        return _SynthParams(self.seed, self.router_std, self.bias_std, self.scale_lo,
                            self.scale_hi, int(self.expert_bias), int(self.router_bias),
                            self.zipf_s, self.zipf_beta)


# ---- library loading --------------------------------------------------------
_lib = None


def library_path() -> str:
    return LIB_PATH


def lib():
    """Load libspt_moe.so; raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise SptError(ERR_NO_DEVICE, f"{LIB_PATH} not built (run stream-pt_b200/build.py)")
    L = ctypes.CDLL(LIB_PATH)
    vp, i64, i32, f32, st = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float, ctypes.c_int
    P = ctypes.POINTER
    sigs = {
        "spt_context_create": ([ctypes.c_int, P(vp)], st),
        "spt_context_destroy": ([vp], None),
        "spt_last_error": ([vp], ctypes.c_char_p),
        "spt_status_string": ([st], ctypes.c_char_p),
        "spt_context_stream": ([vp], vp),
        "spt_context_set_stream": ([vp, vp], st),
        "spt_context_sync": ([vp], st),
        "spt_validate_moe_layer": ([vp, P(_Reader), P(_Config), P(_LayerWeights)], st),
        "spt_arena_create": ([vp, P(_Reader), P(_Config), P(_LayerWeights), i64, ctypes.c_uint32, P(vp)], st),
        "spt_arena_create_synthetic": ([vp, P(_Config), P(_SynthParams), i64, ctypes.c_uint32, P(vp)], st),
        "spt_arena_destroy": ([vp], None),
        "spt_arena_bytes": ([vp], ctypes.c_uint64),
        "spt_synth_layer_host": ([P(_Config), P(_SynthParams), i64, vp, vp, vp, vp, vp, vp, vp, vp], st),
        "spt_synth_normal_host": ([ctypes.c_uint64, ctypes.c_uint64, f32, f32, vp, i64], st),
        "spt_forward_moe_batch": ([vp, vp, i64, vp, i64, vp, i64, i64, vp], st),
        "spt_forward_moe": ([vp, vp, i64, vp, i64, vp, i64, vp], st),
        "spt_forward_moe_batch_device": ([vp, vp, i64, vp, vp, i64], st),
        "spt_forward_moe_batch_device_static": ([vp, vp, i64, vp, vp, i64], st),
        "spt_forward_moe_batch_reader": ([vp, P(_Reader), P(_Config), P(_LayerWeights), vp, i64, vp, i64, i64, vp], st),
        "spt_last_routing": ([vp, vp, vp, vp, vp, vp, P(i64)], st),
        "spt_route_moe_batch": ([vp, vp, ctypes.c_uint64, vp, i64, vp, i64, i64, i64, vp, vp], st),
        "spt_select_moe_batch": ([vp, vp, i64, i64, i64, vp, vp], st),
        "spt_dispatch_moe_batch": ([vp, vp, vp, i64, i64, i64, vp, vp, P(i64)], st),
        "spt_mul_moe_batch_expert": ([vp, vp, ctypes.c_uint64, i64, i64, vp, i64, vp, i64, vp, vp, i64, vp, vp], st),
        "spt_swiglu": ([vp, vp, vp, vp, i64], st),
        "spt_combine_moe_batch": ([vp, vp, vp, i64, i64, i64, vp], st),
        "spt_rmsnorm": ([vp, vp, vp, i64, i64, f32, vp], st),
        "spt_mul_q80": ([vp, vp, ctypes.c_uint64, i64, i64, vp, vp, P(i64), P(f32)], st),
        "spt_gguf_open": ([P(ctypes.c_char_p), i64, P(vp)], st),
        "spt_gguf_close": ([vp], None),
        "spt_gguf_layer_count": ([vp], i64),
        "spt_gguf_config": ([vp, P(_Config), P(f32)], st),
        "spt_gguf_layer": ([vp, i64, P(_LayerWeights), P(_Reader)], st),
        "spt_gguf_tensor": ([vp, ctypes.c_char_p, P(_Tensor), P(_Reader)], st),
        "spt_arena_create_gguf": ([vp, vp, i64, i64, ctypes.c_uint32, i64, i64, P(vp)], st),
        "spt_forward_stack_device": ([vp, vp, vp, i64, i64, vp, i64, f32], st),
        "spt_forward_stack": ([vp, vp, vp, i64, i64, vp, i64, i64, f32, vp], st),
        "spt_synth_norm_host": ([P(_SynthParams), i64, i64, vp], st),
        "spt_mul_q40": ([vp, vp, vp, vp, i64, vp, i64, vp], st),
        "spt_mul_q40_batch": ([vp, vp, vp, vp, i64, vp, i64, i64, vp], st),
        "spt_q40_matrix_create": ([vp, vp, vp, P(vp)], st),
        "spt_q40_matrix_destroy": ([vp], None),
        "spt_q40_matrix_shape": ([vp, P(i64), P(i64)], st),
        "spt_mul_q40_matrix": ([vp, vp, vp, i64, vp, i64, i64, vp], st),
        "spt_mul_q40_matrix_device": ([vp, vp, vp, vp, i64], st),
        "spt_q80_matrix_create": ([vp, vp, ctypes.c_uint64, i64, i64, P(vp)], st),
        "spt_q80_matrix_destroy": ([vp], None),
        "spt_mul_q80_matrix": ([vp, vp, vp, vp, P(i64), P(f32)], st),
        "spt_mul_q80_matrix_device": ([vp, vp, vp, vp, vp, vp], st),
        "spt_ep_expert_range": ([i64, i32, i32, P(i64), P(i64)], None),
        "spt_last_dispatch": ([vp, P(i64), P(i64)], st),
        "spt_ep_unique_id": ([vp], st),
        "spt_ep_create": ([vp, vp, i32, i32, P(vp)], st),
        "spt_ep_destroy": ([vp], None),
        "spt_ep_set_capacity": ([vp, i64], st),
        "spt_ep_set_exchange": ([vp, i32], st),
        "spt_forward_moe_batch_ep_device": ([vp, vp, vp, i64, vp, vp, i64], st),
        "spt_forward_moe_batch_ep": ([vp, vp, vp, i64, vp, i64, vp, i64, i64, vp], st),
        "spt_arena_create_range": ([vp, vp, P(_Config), vp, i64, ctypes.c_uint32, i64, i64, P(vp)], st),
        "spt_arena_create_synthetic_range": ([vp, P(_Config), P(_SynthParams), i64, ctypes.c_uint32, i64, i64,
                                              P(vp)], st),
        "spt_arena_expert_range": ([vp, P(i64), P(i64)], None),
        "spt_set_stage_timing": ([vp, ctypes.c_int], st),
        "spt_stage_times": ([vp, vp, ctypes.c_int], ctypes.c_int),
        "spt_kernels_per_forward": ([vp], ctypes.c_int),
        "spt_context_set_path": ([vp, ctypes.c_int], st),
        "spt_context_set_option": ([vp, ctypes.c_int, i64], st),
        "spt_last_expert_path": ([vp, P(ctypes.c_int)], ctypes.c_int),
        "spt_arena_create_views": ([vp, P(_Config), vp, vp, i64, ctypes.c_uint32, i64, i64, P(vp)], st),
        "spt_context_get_option": ([vp, ctypes.c_int], i64),
    }
    for name, (args, res) in sigs.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def exported_symbols() -> list[str]:
    """Names this binding expects the library to export (include/spt_moe.h)."""
    lib()
    return sorted(n for n in dir(_lib) if n.startswith("spt_"))


def _p(a: Optional[np.ndarray]):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


class Context:
    """spt_context: one CUDA device + stream (device=-1: host-only validation)."""

    def __init__(self, device: int = 0):
        self._h = ctypes.c_void_p()
        st = lib().spt_context_create(device, ctypes.byref(self._h))
        if st != OK:
            raise SptError(st, lib().spt_last_error(None).decode())
        self.device = device

    @property
    def handle(self):
        return self._h

    def close(self):
        if self._h:
            lib().spt_context_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, st: int):
        if st != OK:
            msg = lib().spt_last_error(self._h).decode()
            if st == ERR_CANCELED:
                raise CanceledError(st, msg)
            raise SptError(st, msg)

    @property
    def stream(self) -> int:
        return lib().spt_context_stream(self._h) or 0

    def set_stream(self, stream_ptr: int):
        self.check(lib().spt_context_set_stream(self._h, ctypes.c_void_p(stream_ptr) if stream_ptr else None))

    def sync(self):
        self.check(lib().spt_context_sync(self._h))

    STAGES = ("router", "select", "dispatch", "quant_x", "gate_up", "quant_act", "down", "combine")

    def set_stage_timing(self, enable: bool = True):
        self.check(lib().spt_set_stage_timing(self._h, int(enable)))

    def stage_times(self) -> dict:
        ms = np.zeros(len(self.STAGES), np.float32)
        n = lib().spt_stage_times(self._h, _p(ms), ms.size)
        return {k: float(v) for k, v in zip(self.STAGES[:n], ms[:n])}

    def kernels_per_forward(self) -> int:
        return int(lib().spt_kernels_per_forward(self._h))

    def set_path(self, path: int):
        """PATH_EXACT (CUDA-core, bit-exact), PATH_MMA (tcgen05), PATH_GEMV16
        (decode GEMV on the packed planes) or PATH_AUTO."""
        self.check(lib().spt_context_set_path(self._h, path))

    def last_expert_path(self) -> Tuple[str, int]:
        """("exact" | "tcgen05" | "gemv16", tcgen05 token-tile width) of the last forward."""
        bn = ctypes.c_int()
        p = int(lib().spt_last_expert_path(self._h, ctypes.byref(bn)))
        return {PATH_EXACT: "exact", PATH_MMA: "tcgen05", PATH_GEMV16: "gemv16"}.get(p, "exact"), bn.value

    def set_option(self, option: int, value: int):
        """spt_context_set_option (OPT_* constants)."""
        self.check(lib().spt_context_set_option(self._h, option, int(value)))

    def get_option(self, option: int) -> int:
        return int(lib().spt_context_get_option(self._h, option))

    # ---- validation -----------------------------------------------------
    def validate(self, reader: Reader, cfg: Config, lw: LayerWeights):
        r, c, w = reader._c(), cfg._c(), lw._c()
        self.check(lib().spt_validate_moe_layer(self._h, ctypes.byref(r), ctypes.byref(c), ctypes.byref(w)))

    # ---- arenas -----------------------------------------------------------
    def arena(self, readers: Sequence[Reader], cfg: Config, layers: Sequence[LayerWeights],
              flags: int = ARENA_GEMV) -> "Arena":
        n = len(layers)
        rs = (_Reader * n)(*[r._c() for r in readers])
        ls = (_LayerWeights * n)(*[l._c() for l in layers])
        c = cfg._c()
        h = ctypes.c_void_p()
        self.check(lib().spt_arena_create(self._h, rs, ctypes.byref(c), ls, n, flags, ctypes.byref(h)))
        return Arena(self, h, cfg, n, keep=(readers,))

    def arena_views(self, readers: Sequence[Reader], cfg: Config, layers: Sequence[LayerWeights],
                    flags: int = ARENA_GEMV) -> "Arena":
        """spt_arena_create_views: every tensor handed over as its own buffer
        (a copy of its [start, end) bytes here), as a reader that maps tensors
        one by one (ggufmap's WithTensor) would."""
        n = len(layers)
        ls = (_LayerWeights * n)(*[l._c() for l in layers])
        ds = (_LayerData * n)()
        keep = []
        for i, (r, lw) in enumerate(zip(readers, layers)):
            raw = r.buf
            for name, _ in _LayerWeights._fields_:
                t = getattr(lw, name)
                if t.name:
                    buf = np.array(raw[t.start:t.end], copy=True)
                    keep.append(buf)
                    setattr(ds[i], name, buf.ctypes.data)
        c = cfg._c()
        h = ctypes.c_void_p()
        self.check(lib().spt_arena_create_views(self._h, ctypes.byref(c), ls, ds, n, flags, 0, 0, ctypes.byref(h)))
        return Arena(self, h, cfg, n)

    def synthetic_arena(self, cfg: Config, params: SynthParams, n_layers: int = 1,
                        flags: int = ARENA_GEMV, experts: Optional[Tuple[int, int]] = None) -> "Arena":
        """Seeded synthetic arena; `experts` = (begin, end) keeps only those
        experts (an expert-parallel shard, same bytes as the full arena's)."""
        c, p = cfg._c(), params._c()
        h = ctypes.c_void_p()
        if experts is None:
            self.check(lib().spt_arena_create_synthetic(self._h, ctypes.byref(c), ctypes.byref(p), n_layers,
                                                        flags, ctypes.byref(h)))
        else:
            self.check(lib().spt_arena_create_synthetic_range(self._h, ctypes.byref(c), ctypes.byref(p), n_layers,
                                                              flags, experts[0], experts[1], ctypes.byref(h)))
        return Arena(self, h, cfg, n_layers)

    def arena_from_gguf(self, g: "Gguf", first_layer: int = 0, n_layers: Optional[int] = None,
                        flags: int = ARENA_GEMV, experts: Optional[Tuple[int, int]] = None) -> "Arena":
        """spt_arena_create_gguf: layers [first, first + n) of a GGUF model."""
        n = g.layer_count - first_layer if n_layers is None else n_layers
        cfg, _ = g.config()
        b, e = experts if experts is not None else (0, 0)
        h = ctypes.c_void_p()
        self.check(lib().spt_arena_create_gguf(self._h, g.handle, first_layer, n, flags, b, e, ctypes.byref(h)))
        return Arena(self, h, cfg, n, keep=(g,))

    def arena_range(self, readers: Sequence[Reader], cfg: Config, layers: Sequence[LayerWeights],
                    experts: Tuple[int, int], flags: int = ARENA_GEMV) -> "Arena":
        """spt_arena_create_range: GGUF arena holding experts [begin, end) only."""
        n = len(layers)
        rs = (_Reader * n)(*[r._c() for r in readers])
        ls = (_LayerWeights * n)(*[l._c() for l in layers])
        c = cfg._c()
        h = ctypes.c_void_p()
        self.check(lib().spt_arena_create_range(self._h, rs, ctypes.byref(c), ls, n, flags, experts[0], experts[1],
                                                ctypes.byref(h)))
        return Arena(self, h, cfg, n, keep=(readers,))

    def last_dispatch(self) -> Tuple[int, int]:
        """(active experts, dispatched rows) of the last dispatch this context ran."""
        a, d = ctypes.c_int64(), ctypes.c_int64()
        self.check(lib().spt_last_dispatch(self._h, ctypes.byref(a), ctypes.byref(d)))
        return a.value, d.value

    # ---- layer stack ---------------------------------------------------------
    def forward_stack(self, arena: "Arena", x: np.ndarray, batch: int, first_layer: int = 0,
                      n_layers: Optional[int] = None, eps: float = 1e-5,
                      ep: Optional["ExpertParallel"] = None, out: Optional[np.ndarray] = None) -> np.ndarray:
        """Residual stream after layers [first, first+n): x += MoE(RMSNorm(x)).
        Returns a new array, or `out` (float32, x's size) filled in place."""
        if out is None:
            x = np.array(_f32(x), copy=True)
        else:
            np.copyto(out.reshape(-1), np.asarray(x, np.float32).reshape(-1))
            x = out
        n = arena.n_layers - first_layer if n_layers is None else n_layers
        self.check(lib().spt_forward_stack(self._h, ep.handle if ep else None, arena.handle, first_layer, n, _p(x),
                                           x.size, batch, eps, None))
        return x

    def forward_stack_device(self, arena: "Arena", x_ptr: int, batch: int, first_layer: int = 0,
                             n_layers: Optional[int] = None, eps: float = 1e-5,
                             ep: Optional["ExpertParallel"] = None):
        n = arena.n_layers - first_layer if n_layers is None else n_layers
        self.check(lib().spt_forward_stack_device(self._h, ep.handle if ep else None, arena.handle, first_layer, n,
                                                  ctypes.c_void_p(x_ptr), batch, eps))

    # ---- expert parallelism ------------------------------------------------
    def forward_moe_batch_ep(self, ep: "ExpertParallel", arena: "Arena", x: np.ndarray, batch: int,
                             layer: int = 0, out: Optional[np.ndarray] = None) -> np.ndarray:
        x = _f32(x)
        if out is None:
            out = np.empty_like(x)
        self.check(lib().spt_forward_moe_batch_ep(self._h, ep.handle, arena.handle, layer, _p(x), x.size, _p(out),
                                                  out.size, batch, None))
        return out

    def forward_moe_batch_ep_device(self, ep: "ExpertParallel", arena: "Arena", x_ptr: int, out_ptr: int,
                                    batch: int, layer: int = 0):
        self.check(lib().spt_forward_moe_batch_ep_device(self._h, ep.handle, arena.handle, layer,
                                                         ctypes.c_void_p(x_ptr), ctypes.c_void_p(out_ptr), batch))

    # ---- the block ----------------------------------------------------------
    def forward_moe_batch(self, arena: "Arena", x: np.ndarray, batch: int, layer: int = 0,
                          out: Optional[np.ndarray] = None, cancel: Optional[np.ndarray] = None,
                          x_len: Optional[int] = None, out_len: Optional[int] = None) -> np.ndarray:
        x = _f32(x)
        if out is None:
            out = np.empty_like(x)
        xl = x.size if x_len is None else x_len
        ol = out.size if out_len is None else out_len
        self.check(lib().spt_forward_moe_batch(self._h, arena.handle, layer, _p(x), xl, _p(out), ol, batch,
                                               _p(cancel)))
        return out

    def forward_moe(self, arena: "Arena", x: np.ndarray, layer: int = 0) -> np.ndarray:
        x = _f32(x)
        out = np.empty_like(x)
        self.check(lib().spt_forward_moe(self._h, arena.handle, layer, _p(x), x.size, _p(out), out.size, None))
        return out

    def forward_moe_batch_device(self, arena: "Arena", x_ptr: int, out_ptr: int, batch: int, layer: int = 0):
        self.check(lib().spt_forward_moe_batch_device(self._h, arena.handle, layer, ctypes.c_void_p(x_ptr),
                                                      ctypes.c_void_p(out_ptr), batch))

    def forward_moe_batch_device_static(self, arena: "Arena", x_ptr: int, out_ptr: int, batch: int,
                                        layer: int = 0):
        """Allocation-free forward on device pointers (static device scratch)."""
        self.check(lib().spt_forward_moe_batch_device_static(self._h, arena.handle, layer, ctypes.c_void_p(x_ptr),
                                                             ctypes.c_void_p(out_ptr), batch))

    def forward_moe_batch_reader(self, reader: Reader, cfg: Config, lw: LayerWeights, x: np.ndarray,
                                 out: np.ndarray, batch: int, cancel: Optional[np.ndarray] = None):
        """Drop-in one-shot forwardMoEBatch (validate + upload + run)."""
        r, c, w = reader._c(), cfg._c(), lw._c()
        self.check(lib().spt_forward_moe_batch_reader(self._h, ctypes.byref(r), ctypes.byref(c), ctypes.byref(w),
                                                      _p(x), x.size, _p(out), out.size, batch, _p(cancel)))
        return out

    def last_routing(self, batch: int, experts: int, k: int) -> dict:
        logits = np.empty(batch * experts, np.float32)
        idx = np.empty(batch * k, np.int32)
        w = np.empty(batch * k, np.float32)
        perm = np.empty(max(batch * k, 1), np.int32)
        counts = np.empty(experts, np.int32)
        n = ctypes.c_int64()
        self.check(lib().spt_last_routing(self._h, _p(logits), _p(idx), _p(w), _p(perm), _p(counts),
                                          ctypes.byref(n)))
        return dict(logits=logits.reshape(batch, experts), sel_idx=idx.reshape(batch, k),
                    sel_w=w.reshape(batch, k), perm=perm[: n.value], counts=counts,
                    dispatched=n.value)

    # ---- stage entry points ------------------------------------------------
    def route_moe_batch(self, data: np.ndarray, x: np.ndarray, router_bias: Optional[np.ndarray],
                        batch: int, hidden: int, experts: int, cancel=None) -> np.ndarray:
        data = np.ascontiguousarray(data, dtype=np.uint8)
        x = _f32(x)
        rb = None if router_bias is None else _f32(router_bias)
        logits = np.empty(batch * experts, np.float32)
        self.check(lib().spt_route_moe_batch(self._h, _p(data), data.size, _p(x), x.size, _p(rb), batch, hidden,
                                             experts, _p(logits), _p(cancel)))
        return logits.reshape(batch, experts)

    def select_moe_batch(self, logits: np.ndarray, k: int):
        logits = _f32(logits)
        batch, experts = logits.shape
        idx = np.empty(batch * k, np.int32)
        w = np.empty(batch * k, np.float32)
        self.check(lib().spt_select_moe_batch(self._h, _p(logits), batch, experts, k, _p(idx), _p(w)))
        return idx.reshape(batch, k), w.reshape(batch, k)

    def dispatch_moe_batch(self, index: np.ndarray, weight: np.ndarray, experts: int):
        index = np.ascontiguousarray(index, dtype=np.int32)
        weight = _f32(weight)
        batch, k = index.shape
        perm = np.empty(batch * k, np.int32)
        offs = np.empty(experts + 1, np.int32)
        n = ctypes.c_int64()
        self.check(lib().spt_dispatch_moe_batch(self._h, _p(index), _p(weight), batch, k, experts, _p(perm),
                                                _p(offs), ctypes.byref(n)))
        return perm[: n.value], offs

    def mul_moe_batch_expert(self, data: np.ndarray, input_: int, output: int, x: np.ndarray,
                             x_offsets: Sequence[int], bias: Optional[np.ndarray], y: np.ndarray,
                             y_offsets: Sequence[int], cancel=None) -> np.ndarray:
        data = np.ascontiguousarray(data, dtype=np.uint8)
        x = _f32(x)
        xo = np.ascontiguousarray(x_offsets, dtype=np.int64)
        yo = np.ascontiguousarray(y_offsets, dtype=np.int64)
        b = None if bias is None else _f32(bias)
        assert y.dtype == np.float32 and y.flags.c_contiguous
        self.check(lib().spt_mul_moe_batch_expert(self._h, _p(data), data.size, input_, output, _p(x), x.size,
                                                  _p(xo), xo.size, _p(b), _p(y), y.size, _p(yo), _p(cancel)))
        return y

    def swiglu(self, gate: np.ndarray, up: np.ndarray) -> np.ndarray:
        g, u = _f32(gate), _f32(up)
        act = np.empty_like(g)
        self.check(lib().spt_swiglu(self._h, _p(g), _p(u), _p(act), g.size))
        return act

    def combine_moe_batch(self, results: np.ndarray, weight: np.ndarray, batch: int, k: int, hidden: int):
        r, w = _f32(results), _f32(weight)
        out = np.empty(batch * hidden, np.float32)
        self.check(lib().spt_combine_moe_batch(self._h, _p(r), _p(w), batch, k, hidden, _p(out)))
        return out.reshape(batch, hidden)

    def rmsnorm(self, x: np.ndarray, weight: np.ndarray, batch: int, dim: int, eps: float):
        x, w = _f32(x), _f32(weight)
        y = np.empty(batch * dim, np.float32)
        self.check(lib().spt_rmsnorm(self._h, _p(x), _p(w), batch, dim, eps, _p(y)))
        return y.reshape(batch, dim)

    def mul_q80(self, data: np.ndarray, input_: int, output: int, x: np.ndarray):
        data = np.ascontiguousarray(data, dtype=np.uint8)
        x = _f32(x)
        y = np.empty(output, np.float32)
        am = ctypes.c_int64()
        best = ctypes.c_float()
        self.check(lib().spt_mul_q80(self._h, _p(data), data.size, input_, output, _p(x), _p(y),
                                     ctypes.byref(am), ctypes.byref(best)))
        return y, am.value, np.float32(best.value)

    def mul_q40_batch(self, reader: "Reader", tensor: "Tensor", x: np.ndarray, batch: int,
                      y: Optional[np.ndarray] = None, cancel: Optional[np.ndarray] = None) -> np.ndarray:
        """MulQ40BatchInto (forward/q40.go:46-101): y [batch, output]."""
        x = _f32(x)
        out = int(tensor.shape[1]) if len(tensor.shape) > 1 else 0
        if y is None:
            y = np.empty(max(batch, 0) * out, np.float32)
        r, t = reader._c(), tensor._c()
        self.check(lib().spt_mul_q40_batch(self._h, ctypes.byref(r), ctypes.byref(t), _p(x), x.size, _p(y), y.size,
                                           batch, _p(cancel)))
        return y.reshape(batch, -1) if batch > 0 else y

    def mul_q40(self, reader: "Reader", tensor: "Tensor", x: np.ndarray, y: Optional[np.ndarray] = None,
                cancel: Optional[np.ndarray] = None) -> np.ndarray:
        """MulQ40Into (forward/q40.go:35-40): y [output]."""
        x = _f32(x)
        if y is None:
            y = np.empty(int(tensor.shape[1]) if len(tensor.shape) > 1 else 0, np.float32)
        r, t = reader._c(), tensor._c()
        self.check(lib().spt_mul_q40(self._h, ctypes.byref(r), ctypes.byref(t), _p(x), x.size, _p(y), y.size,
                                     _p(cancel)))
        return y

    def q40_matrix(self, reader: "Reader", tensor: "Tensor") -> "Q40Matrix":
        """Upload a Q4_0 tensor once (spt_q40_matrix_create)."""
        return Q40Matrix(self, reader, tensor)

    def q80_matrix(self, data: np.ndarray, input_: int, output: int) -> "Q80Matrix":
        """Upload a Q8_0 matrix once (spt_q80_matrix_create)."""
        return Q80Matrix(self, data, input_, output)


def _tensor_view(t: "_Tensor") -> Tensor:
    return Tensor(t.name.decode() if t.name else "", t.type, tuple(t.shape[i] for i in range(min(t.n_dims, 4))),
                  t.start, t.end)


class Gguf:
    """spt_gguf: a GGUF model (split files in any order), mapped read-only."""

    def __init__(self, paths: Sequence[str]):
        arr = (ctypes.c_char_p * len(paths))(*[os.fsencode(p) for p in paths])
        self._h = ctypes.c_void_p()
        st = lib().spt_gguf_open(arr, len(paths), ctypes.byref(self._h))
        if st != OK:
            raise SptError(st, lib().spt_last_error(None).decode())

    @property
    def handle(self):
        return self._h

    @property
    def layer_count(self) -> int:
        return lib().spt_gguf_layer_count(self._h)

    def config(self) -> Tuple[Config, float]:
        c, eps = _Config(), ctypes.c_float()
        self._check(lib().spt_gguf_config(self._h, ctypes.byref(c), ctypes.byref(eps)))
        return Config(c.hidden_dim, c.expert_hidden_dim, c.num_experts, c.num_experts_used), float(eps.value)

    def layer(self, layer: int) -> dict:
        """NewLayerWeights of one layer: field -> Tensor (name '' when absent)."""
        lw, rd = _LayerWeights(), _Reader()
        self._check(lib().spt_gguf_layer(self._h, layer, ctypes.byref(lw), ctypes.byref(rd)))
        return {name: _tensor_view(getattr(lw, name)) for name, _ in _LayerWeights._fields_}

    def tensor(self, name: str) -> Tensor:
        t, rd = _Tensor(), _Reader()
        self._check(lib().spt_gguf_tensor(self._h, name.encode(), ctypes.byref(t), ctypes.byref(rd)))
        return _tensor_view(t)

    def _check(self, st):
        if st != OK:
            raise SptError(st, lib().spt_last_error(None).decode())

    def close(self):
        if self._h:
            lib().spt_gguf_close(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def q40_tensor(data: np.ndarray, input_: int, output: int, name: str = "q40.weight", prefix: int = 0):
    """A Reader holding Q4_0 bytes (after `prefix` bytes) and its Tensor [input, output]."""
    data = np.ascontiguousarray(data, dtype=np.uint8).reshape(-1)
    buf = np.zeros(prefix + data.size, np.uint8)
    buf[prefix:] = data
    return Reader(buf), Tensor(name, 2, (input_, output), prefix, prefix + data.size)


class Q40Matrix:
    """HBM-resident Q4_0 matrix: y = W x for a batch of inputs."""

    def __init__(self, ctx: "Context", reader: "Reader", tensor: "Tensor"):
        self.ctx = ctx
        self._h = ctypes.c_void_p()
        r, t = reader._c(), tensor._c()
        ctx.check(lib().spt_q40_matrix_create(ctx._h, ctypes.byref(r), ctypes.byref(t), ctypes.byref(self._h)))
        i, o = ctypes.c_int64(), ctypes.c_int64()
        lib().spt_q40_matrix_shape(self._h, ctypes.byref(i), ctypes.byref(o))
        self.input, self.output = i.value, o.value

    def mul(self, x: np.ndarray, batch: int = 1, y: Optional[np.ndarray] = None, cancel=None) -> np.ndarray:
        x = _f32(x)
        if y is None:
            y = np.empty(batch * self.output, np.float32)
        self.ctx.check(lib().spt_mul_q40_matrix(self.ctx._h, self._h, _p(x), x.size, _p(y), y.size, batch,
                                                _p(cancel)))
        return y.reshape(batch, self.output)

    def mul_device(self, x_ptr: int, y_ptr: int, batch: int = 1):
        self.ctx.check(lib().spt_mul_q40_matrix_device(self.ctx._h, self._h, ctypes.c_void_p(x_ptr),
                                                       ctypes.c_void_p(y_ptr), batch))

    def close(self):
        if self._h:
            lib().spt_q40_matrix_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Q80Matrix:
    """HBM-resident Q8_0 matrix (LM head): y = W x and its argmax."""

    def __init__(self, ctx: "Context", data: np.ndarray, input_: int, output: int):
        data = np.ascontiguousarray(data, dtype=np.uint8)
        self.ctx, self.input, self.output = ctx, input_, output
        self._h = ctypes.c_void_p()
        ctx.check(lib().spt_q80_matrix_create(ctx._h, _p(data), data.size, input_, output, ctypes.byref(self._h)))

    def mul(self, x: np.ndarray, want_y: bool = True):
        """(y or None, argmax row, best logit) for host x."""
        x = _f32(x)
        y = np.empty(self.output, np.float32) if want_y else None
        am, best = ctypes.c_int64(), ctypes.c_float()
        self.ctx.check(lib().spt_mul_q80_matrix(self.ctx._h, self._h, _p(x), _p(y), ctypes.byref(am),
                                                ctypes.byref(best)))
        return y, am.value, np.float32(best.value)

    def mul_device(self, x_ptr: int, y_ptr: int = 0, argmax_ptr: int = 0, logit_ptr: int = 0):
        self.ctx.check(lib().spt_mul_q80_matrix_device(self.ctx._h, self._h, ctypes.c_void_p(x_ptr),
                                                       ctypes.c_void_p(y_ptr or None),
                                                       ctypes.c_void_p(argmax_ptr or None),
                                                       ctypes.c_void_p(logit_ptr or None)))

    def close(self):
        if self._h:
            lib().spt_q80_matrix_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ep_expert_range(num_experts: int, world: int, rank: int) -> Tuple[int, int]:
    """Experts held by `rank` of `world`: [rank*E/world, (rank+1)*E/world)."""
    b, e = ctypes.c_int64(), ctypes.c_int64()
    lib().spt_ep_expert_range(num_experts, world, rank, ctypes.byref(b), ctypes.byref(e))
    return b.value, e.value


def _nccl_library():
    """Point the library at PyTorch's NCCL (the pip nvidia-nccl package) when
    that is installed and no NCCL is named yet: whichever NCCL the process
    loads first is the one every later user of the soname gets."""
    if os.environ.get("SPT_NCCL_LIBRARY"):
        return
    try:
        import importlib.util
        spec = importlib.util.find_spec("nvidia.nccl")
    except (ImportError, ValueError):
        spec = None
    for base in (spec.submodule_search_locations if spec else []) or []:
        path = os.path.join(base, "lib", "libnccl.so.2")
        if os.path.exists(path):
            os.environ["SPT_NCCL_LIBRARY"] = path
            return


def ep_unique_id() -> bytes:
    """NCCL unique id for spt_ep_create (made on rank 0, shared out of band)."""
    _nccl_library()
    buf = (ctypes.c_uint8 * 128)()
    st = lib().spt_ep_unique_id(buf)
    if st != OK:
        raise SptError(st, lib().spt_last_error(None).decode())
    return bytes(buf)


class ExpertParallel:
    """spt_ep: this rank's member of an expert-parallel group (collective create)."""

    def __init__(self, ctx: "Context", unique_id: bytes, rank: int, world: int):
        if len(unique_id) != 128:
            raise ValueError("unique id must be 128 bytes")
        self.ctx, self.rank, self.world = ctx, rank, world
        _nccl_library()
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(unique_id)
        self._h = ctypes.c_void_p()
        ctx.check(lib().spt_ep_create(ctx._h, buf, rank, world, ctypes.byref(self._h)))

    @property
    def handle(self):
        return self._h

    def set_capacity(self, max_tokens_per_rank: int):
        """Fixed-capacity exchange (no host synchronisation); same value on every rank."""
        self.ctx.check(lib().spt_ep_set_capacity(self._h, max_tokens_per_rank))

    def set_exchange(self, exchange: int):
        """spt_ep_set_exchange: EP_EXCHANGE_PEER (NVLink peer windows) or
        EP_EXCHANGE_NCCL for the fixed-capacity exchange."""
        self.ctx.check(lib().spt_ep_set_exchange(self._h, exchange))

    def close(self):
        if self._h:
            lib().spt_ep_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Arena:
    """HBM-resident expert arena (spt_arena)."""

    def __init__(self, ctx: Context, handle, cfg: Config, n_layers: int, keep=()):
        self.ctx, self._h, self.cfg, self.n_layers = ctx, handle, cfg, n_layers
        self._keep = keep

    @property
    def handle(self):
        return self._h

    @property
    def nbytes(self) -> int:
        return int(lib().spt_arena_bytes(self._h))

    def close(self):
        if self._h:
            lib().spt_arena_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def synth_layer_host(cfg: Config, params: SynthParams, layer: int = 0) -> dict:
    """Host copy of a synthetic layer in GGUF tensor layout (same bytes as the arena)."""
    H, D, E = cfg.hidden_dim, cfg.expert_hidden_dim, cfg.num_experts
    router = np.empty(E * H * 4, np.uint8)
    rb = np.empty(E, np.float32)
    gate = np.empty(E * D * (H // 32) * 17, np.uint8)
    up = np.empty_like(gate)
    down = np.empty(E * H * (D // 32) * 17, np.uint8)
    gb = np.empty(E * D, np.float32)
    ub = np.empty(E * D, np.float32)
    db = np.empty(E * H, np.float32)
    c, p = cfg._c(), params._c()
    st = lib().spt_synth_layer_host(ctypes.byref(c), ctypes.byref(p), layer, _p(router), _p(rb), _p(gate),
                                    _p(up), _p(down), _p(gb), _p(ub), _p(db))
    if st != OK:
        raise SptError(st, lib().spt_last_error(None).decode())
    return dict(router=router, router_bias=rb, gate=gate, up=up, down=down, gate_bias=gb,
                up_bias=ub, down_bias=db)


def synth_norm_host(params: SynthParams, layer: int, dim: int) -> np.ndarray:
    """Norm weights [dim] of a synthetic layer (same values as the arena's)."""
    out = np.empty(dim, np.float32)
    p = params._c()
    st = lib().spt_synth_norm_host(ctypes.byref(p), layer, dim, _p(out))
    if st != OK:
        raise SptError(st, lib().spt_last_error(None).decode())
    return out


def synth_normal_host(seed: int, stream: int, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, np.float32)
    st = lib().spt_synth_normal_host(seed, stream, mean, std, _p(out), n)
    if st != OK:
        raise SptError(st, lib().spt_last_error(None).decode())
    return out


def build(verbose: bool = False, force: bool = False) -> str:
    """Compile csrc/ for sm_100a (see build.py)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("_spt_build", os.path.join(_HERE, "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build(verbose=verbose, force=force)
