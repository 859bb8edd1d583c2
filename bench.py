"""Benchmark of the B200 MoE FFN block (GPT-OSS-120B shapes).

python bench.py [--gpus N] [--steps K] [--warmup W] [--config c1] [--impl ours|reference]
                [--path auto|mma|gemv16|exact] [--no-extras] [--no-cpu-baseline]

Prints ONE JSON line (rank 0).  A step is one forward of the MoE block over
one batch of synthetic tokens: seeded Philox weights with GPT-OSS shapes
generated on the device, N(0, 1) activations (the real checkpoint is not in
the image; no dataset is involved).  `value` times the device path with
inputs resident in HBM (CUDA events on the library's stream); `e2e` times the
C-ABI host call a caller makes (spt_forward_moe_batch: host x -> device ->
block -> host out, returned after completion) on the host clock, after a
synchronised L2 flush, so validation, launch, copies and waiting all count.
The L2 (126 MB) is flushed between timed steps by writing a 256 MB buffer.

The line's workload is --config (default c1).  With one
GPU the line also carries the other configs under "configs" (c0 decode, c2
Zipf prefill, c3 T=8192, c4 36-layer stack), each measured in the same
process with its own parity check.  Under torchrun (N > 1) the block runs
expert-parallel: rank r holds experts [r*128/N, (r+1)*128/N); the line's
workload keeps c1's 32 tokens per rank (weak scaling, fixed-capacity
exchange), and "configs" carries c3 (T = 8192 in total, 8192/N per rank:
strong scaling) and c4 (64 rows in total).

Every line has a "parity" object: tokens of the timed workload recomputed by
the CPU oracle (oracle/, the C restatement of the reference's path) outside
the timed region, with routing (selected ids, dispatch permutation) compared
bit for bit and block outputs by max|err|/max|ref| and cosine.

--impl reference times the oracle on the host cores on the same workload
(rank 0 only): the reference is a Go module that cannot be built here, and
its C restatement is what runs; it never loads the CUDA library.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

H = D = 2880
E, K = 128, 4
MATRIX_BYTES = 2880 * (2880 // 32) * 17          # one MXFP4 expert matrix, GGUF bytes
ROUTER_BYTES = E * H * 4
L2_BYTES = 126 << 20
FLUSH_BYTES = 256 << 20
EPS = 1e-5
MAX_REL, MIN_COS = 1e-3, 0.99999                  # the block's tolerance (north_star)

CONFIGS = {
    "c0": dict(T=1, seed=0, zipf_s=0.0, zipf_beta=0.0, router_bias=True,
               desc="decode, 1 token (BASELINE configs[0])"),
    "c1": dict(T=32, seed=1, zipf_s=0.0, zipf_beta=0.0, router_bias=True,
               desc="prefill batch T=32 (BASELINE configs[1])"),
    "c2": dict(T=2048, seed=2, zipf_s=1.1, zipf_beta=0.9, router_bias=True,
               desc="prefill T=2048, Zipf(1.1)-skewed router bias (BASELINE configs[2])"),
    "c3": dict(T=8192, seed=3, zipf_s=0.0, zipf_beta=0.0, router_bias=False, strong=True,
               desc="T=8192 in total, balanced routing (zero router bias), tokens sharded over ranks "
                    "(BASELINE configs[3])"),
    "c4": dict(T=64, seed=4, zipf_s=0.0, zipf_beta=0.0, router_bias=True, layers=36, strong=True,
               desc="36-layer stack, RMSNorm + MoE + residual per layer, 64 token rows (BASELINE configs[4])"),
}


def dist_info():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def tokens(name, world):
    """(tokens per rank, tokens in total) of config `name` on `world` ranks."""
    c = CONFIGS[name]
    if c.get("strong"):
        return max(1, c["T"] // world), max(1, c["T"] // world) * world
    return c["T"], c["T"] * world


def workload_config(name, world, ep_mode=None):
    """The `config` object of a line: identical in both arms for the same
    workload (it names only the workload, nothing measured)."""
    c = CONFIGS[name]
    t_rank, t_all = tokens(name, world)
    if world == 1:
        par = "single GPU"
    else:
        par = f"ep{world}: {E // world} experts per GPU, {t_rank} tokens per rank, dispatch/combine ({ep_mode})"
    return {"workload": f"{name}: {c['desc']}", "tokens_per_step": t_all, "tokens_per_rank": t_rank,
            "hidden": H, "expert_dim": D, "experts": E, "top_k": K, "layers": c.get("layers", 1),
            "seed": c["seed"], "router_bias": c["router_bias"], "zipf_s": c["zipf_s"], "zipf_beta": c["zipf_beta"],
            "scale_bytes": "uniform 119..123", "parallelism": par,
            "l2": "256 MB buffer written between timed steps"}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", 0.0)), "measured (MEASURED_PEAKS.json)"
    return 6650.0, 1590.0, "fallback (6.65 TB/s, 1.59 PFLOP/s)"


def load_traffic(key):
    """Per-launch DRAM bytes of a kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if not os.path.exists(p):
        return None
    return json.load(open(p)).get(key)


class ClockSampler:
    """SM clock and throttle reasons sampled during the timed region.

    NVML is polled every 2 ms from a thread (the timed regions here last from
    milliseconds to seconds); without pynvml it falls back to nvidia-smi
    every 200 ms.  Reads only: no GPU setting is touched.
    """

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # nvmlClocksEventReason bits: sw_power_cap 0x4, hw_slowdown 0x8,
    # sw_thermal_slowdown 0x20, hw_thermal_slowdown 0x40
    BITS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
            ("sw_power_cap", 0x4))

    def __init__(self, cuda_index):
        self.cuda_index = cuda_index
        self.rows = []       # (sm_mhz, max_mhz, reasons set)
        self.proc = None
        self.stop = threading.Event()
        self.t = None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(self.cuda_index)
        uuid = getattr(props, "uuid", None)
        if uuid is not None:
            try:
                return pynvml.nvmlDeviceGetHandleByUUID("GPU-" + str(uuid))
            except Exception:
                pass
        bus = getattr(props, "pci_bus_id", None)
        if bus is not None:
            try:
                busid = "%08X:%02X:%02X.0" % (getattr(props, "pci_domain_id", 0), bus,
                                               getattr(props, "pci_device_id", 0))
                return pynvml.nvmlDeviceGetHandleByPciBusId(busid)
            except Exception:
                pass
        return pynvml.nvmlDeviceGetHandleByIndex(self.cuda_index)

    def _poll_nvml(self, h):
        import pynvml
        mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        while True:
            try:
                sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.rows.append((float(sm), float(mx), {n for n, b in self.BITS if bits & b}))
            except Exception:
                pass
            if self.stop.wait(0.002):
                break

    def __enter__(self):
        try:
            h = self._nvml_handle()
            self.t = threading.Thread(target=self._poll_nvml, args=(h,), daemon=True)
            self.t.start()
            return self
        except Exception:
            self.t = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.cuda_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read_smi, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read_smi(self):
        names = [n for n, _ in self.BITS]
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                self.rows.append((float(parts[1]), float(parts[2]) if parts[2].replace(".", "").isdigit() else None,
                                  {names[i] for i in range(4) if parts[5 + i].lower() == "active"}))

    def __exit__(self, *exc):
        self.stop.set()
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.t:
            self.t.join(timeout=5)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [r[0] for r in self.rows]
        mx = [r[1] for r in self.rows if r[1]]
        reasons = sorted(set().union(*(r[2] for r in self.rows)))
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ---------------------------------------------------------------------------
# the oracle side (CPU): weights, parity, CPU baseline

def oracle_params(name):
    from oracle import oracle
    c = CONFIGS[name]
    return oracle.synth_params(seed=c["seed"], zipf_s=c["zipf_s"], zipf_beta=c["zipf_beta"],
                               router_bias=c["router_bias"])


_WEIGHTS = {}


def oracle_weights(name, layer=0):
    """The whole synthetic layer, generated by the oracle (cached)."""
    from oracle import oracle
    key = (CONFIGS[name]["seed"], name, layer)
    if key not in _WEIGHTS:
        _WEIGHTS.clear()
        _WEIGHTS[key] = oracle.synth_weights(H, D, E, K, oracle_params(name), layer)
    return _WEIGHTS[key]


def x_rows(name, rank):
    from oracle import oracle
    t_rank, _ = tokens(name, int(os.environ.get("WORLD_SIZE", "1")))
    return oracle.synth_normal(CONFIGS[name]["seed"] + 7919 * rank, 1000, t_rank * H)


def compare(got, want):
    got = np.asarray(got, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    finite = bool(np.isfinite(got).all())
    err = float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30)) if finite else float("inf")
    cos = float(np.dot(got, want) / (np.linalg.norm(got) * np.linalg.norm(want) + 1e-300)) if finite else 0.0
    return err, cos


def parity_block(name, x, T, got, routing=None, sample=64):
    """Sampled tokens of one block against the oracle.  With `routing` (the
    library's logits, selections and dispatch of the same call) the routing
    of every token is compared bit for bit; near-ties (the two logits around
    the k-th choice within 1e-6) are counted."""
    from oracle import oracle
    w = oracle_weights(name)
    x = np.asarray(x, np.float32).reshape(T, H)
    got = np.asarray(got, np.float32).reshape(T, H)
    out = {"tokens": T}
    top = None
    if routing is not None:
        lg = oracle.route_threads(w.arrays["router"], x, w.arrays["router_bias"], T, H, E)
        sel = [oracle.select(lg[t], K) for t in range(T)]
        sel_idx = np.array([[i for i, _ in s] for s in sel], np.int32)
        sel_w = np.array([[v for _, v in s] for s in sel], np.float32)
        perm, counts = oracle.dispatch_perm(sel_idx, sel_w, E)
        out["logits_bit_exact"] = bool(np.array_equal(lg.view(np.uint32), routing["logits"].view(np.uint32)))
        out["ids_equal"] = bool(np.array_equal(sel_idx, routing["sel_idx"]))
        out["weights_bit_exact"] = bool(np.array_equal(sel_w.view(np.uint32), routing["sel_w"].view(np.uint32)))
        out["perm_equal"] = bool(np.array_equal(perm, routing["perm"]))
        srt = np.sort(lg, axis=1)[:, ::-1]
        out["near_ties_1e-6"] = int(np.sum(np.abs(srt[:, K - 1] - srt[:, K]) <= 1e-6))
        top = int(np.argmax(counts))
        out["top_expert_share"] = round(float(counts.max() / max(counts.sum(), 1)), 4)
    # sampled tokens: every 2nd of the first 16 routed to the top expert, the rest spread evenly
    if T <= sample:
        idx = list(range(T))
    else:
        idx = []
        if top is not None:
            idx = [t for t in range(T) if top in routing["sel_idx"][t]][:sample // 4]
        rest = np.linspace(0, T - 1, sample - len(idx)).astype(int).tolist()
        idx = sorted(set(idx + rest))
    want = oracle.forward_moe_batch(w, x[idx].ravel(), len(idx), workers=os.cpu_count() or 8)
    err, cos = compare(got[idx], want)
    out.update({"checked_tokens": len(idx), "max_rel": err, "cos": cos,
                "ok": bool(err <= MAX_REL and cos >= MIN_COS and out.get("ids_equal", True)
                           and out.get("perm_equal", True))})
    return out


def oracle_stack_layer(name, l, xs, rows):
    """One layer of the oracle's stack (RMSNorm -> block -> residual add) on
    `rows` rows; returns (new rows, the rows' selected ids, the gap between
    the k-th and (k+1)-th largest logit of each row).  Only the experts the
    rows select are generated."""
    from oracle import oracle
    c = CONFIGS[name]
    p = oracle_params(name)
    norm = oracle.synth_norm(c["seed"], l, H)
    normed = oracle.rmsnorm(xs, norm, rows, H, EPS)
    head = oracle.synth_layer_experts(H, D, E, p, l, [])
    lg = oracle.route(head["router"], normed, head["router_bias"], rows, H, E)
    ids = np.array([[i for i, _ in oracle.select(lg[t], K)] for t in range(rows)], np.int32)
    srt = np.sort(lg, axis=1)[:, ::-1]
    gap = srt[:, K - 1] - srt[:, K]
    w = oracle.weights_of(oracle.synth_layer_experts(H, D, E, p, l, sorted(set(ids.ravel().tolist()))), H, D, E, K)
    out = (xs + oracle.forward_moe_batch(w, normed, rows, workers=os.cpu_count() or 8)).astype(np.float32)
    return out, ids, gap


def parity_stack(name, runner, got, rows=2):
    """The first `rows` rows of a stack step against the oracle's composition
    RMSNorm -> block -> residual add, two ways:
      teacher-forced: each layer of the library (its timed expert path) on
        the oracle's input to that layer, against the oracle's output; the
        block tolerance applies per layer and the routing must be bit-exact;
      free-running: the timed step's final rows against the oracle's own 36
        layers.  The library's rows are also run layer by layer on their own
        outputs to find where a row's selected experts first differ from the
        oracle's; each such divergence is logged with the oracle's gap
        between the k-th and (k+1)-th logit of that row (a near-tie that the
        path's rounding tipped over)."""
    ctx, spt = runner.ctx, runner.spt
    layers = CONFIGS[name].get("layers", 1)
    x0 = np.array(np.asarray(runner.x_host, np.float32).reshape(runner.T, H)[:rows], copy=True)
    path, _ = ctx.last_expert_path()
    saved = ctx.get_option(spt.OPT_GEMV16_SLOTS)
    if path == "tcgen05":
        ctx.set_option(spt.OPT_GEMV16_SLOTS, 0)  # the rows alone would take the decode GEMV
    worst, worst_cos, ids_ok = 0.0, 1.0, True
    xo, xg = x0, x0.copy()
    divergence = {}
    try:
        for l in range(layers):
            nxt, ids, gap = oracle_stack_layer(name, l, xo, rows)
            tf = ctx.forward_stack(runner.arena, xo, rows, first_layer=l, n_layers=1, eps=EPS).reshape(rows, H)
            r = ctx.last_routing(rows, E, K)
            ids_ok = ids_ok and bool(np.array_equal(r["sel_idx"], ids))
            err, cos = compare(tf, nxt)
            worst, worst_cos = max(worst, err), min(worst_cos, cos)
            xg = ctx.forward_stack(runner.arena, xg, rows, first_layer=l, n_layers=1, eps=EPS).reshape(rows, H)
            gids = ctx.last_routing(rows, E, K)["sel_idx"]
            for t in range(rows):
                if t not in divergence and not np.array_equal(gids[t], ids[t]):
                    divergence[t] = {"layer": l, "oracle_gap": float(gap[t])}
            xo = nxt
    finally:
        ctx.set_option(spt.OPT_GEMV16_SLOTS, saved)
    final = np.asarray(got, np.float32).reshape(runner.T, H)[:rows]
    err, cos = compare(final, xo)
    # rows that kept the oracle's experts in every layer stay close; only a
    # logged divergence may explain a row that does not
    ok_free = all(t in divergence for t in range(rows) if not compare(final[t], xo[t])[0] <= 1e-2)
    return {"tokens": runner.T, "checked_tokens": rows, "layers": layers,
            "teacher_forced": {"max_rel": worst, "min_cos": worst_cos, "ids_equal": ids_ok},
            "free_running": {"max_rel": err, "cos": cos, "diverged_rows": divergence},
            "max_rel": worst, "cos": worst_cos,
            "ok": bool(worst <= MAX_REL and worst_cos >= MIN_COS and ids_ok and ok_free)}


def cpu_baseline(name, seconds=12.0, workers=None):
    """The oracle (C restatement of the reference's AVX2 path, row-partitioned
    threads like mulMoEBatchExpert) on the same workload, all host threads,
    memory-resident weights generated by the oracle itself (the CUDA library
    is never loaded).  Returns (tokens/s, cores, sample text)."""
    from oracle import oracle
    c = CONFIGS[name]
    w = oracle_weights(name)
    layers = c.get("layers", 1)
    workers = workers or os.cpu_count() or 1
    t_rank, _ = tokens(name, 1)
    # bounded sample: at most 64 tokens of the workload per repetition, one
    # layer (a stack's time is the per-layer time times its depth)
    Ts = min(t_rank, 64)
    x = oracle.synth_normal(c["seed"], 1000, Ts * H)
    norm = oracle.synth_norm(c["seed"], 0, H)

    def one():
        xin = oracle.rmsnorm(x, norm, Ts, H, EPS) if layers > 1 else x
        out = oracle.forward_moe_batch(w, xin, Ts, workers)
        if layers > 1:
            out = out + x.reshape(Ts, H)
        return out

    one()  # warm
    reps, t0 = 0, time.perf_counter()
    while True:
        one()
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds or reps >= 1000:
            break
    tps = reps * Ts / el / layers
    what = f"{reps} x {Ts} tokens x 1 of {layers} layers" if layers > 1 else f"{reps} x {Ts} tokens"
    return tps, workers, f"{what} of {name} ({el:.1f} s, memory-resident weights, oracle-generated)"


def native_libraries():
    """Shared objects of this repository mapped into the process."""
    found = set()
    try:
        with open("/proc/self/maps") as f:
            for line in f:
                path = line.split()[-1] if line.strip() else ""
                if path.endswith(".so") and os.path.realpath(path).startswith(os.path.realpath(ROOT) + os.sep):
                    found.add(os.path.relpath(os.path.realpath(path), os.path.realpath(ROOT)))
    except OSError:
        return None
    return sorted(found)


def run_reference(args):
    rank, world, _ = dist_info()
    if rank != 0:
        return
    tps, cores, sample = cpu_baseline(args.config, seconds=max(3.0, 2.0 * args.steps))
    t_rank, t_all = tokens(args.config, world)
    line = {"metric": "moe_block_tokens_per_s", "value": tps, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t_all / tps,
            "higher_is_better": True, "scaling": "strong" if CONFIGS[args.config].get("strong") else "weak",
            "vs_baseline": None, "dtype": "f32 (mxfp4 weights)", "data": "synthetic", "impl": "reference",
            "config": workload_config(args.config, world, ep_mode(args.config)),
            "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "native_so_loaded": native_libraries()}
    print(json.dumps(line), flush=True)


def ep_mode(name):
    """Every config uses the fixed-capacity exchange: through the NVLink peer
    windows only live rows move and no call synchronises with the host."""
    return "fixed capacity, NVLink peer windows, live rows only"


# ---------------------------------------------------------------------------
# the GPU side

class Runner:
    """One workload on this rank: arena, inputs, the step and the host call."""

    def __init__(self, spt, torch, ctx, name, args, rank, world, local):
        self.spt, self.torch, self.ctx, self.name = spt, torch, ctx, name
        self.rank, self.world, self.local = rank, world, local
        c = CONFIGS[name]
        self.layers = c.get("layers", 1)
        self.T, self.T_all = tokens(name, world)
        cfg = spt.Config(H, D, E, K)
        params = spt.SynthParams(seed=c["seed"], zipf_s=c["zipf_s"], zipf_beta=c["zipf_beta"],
                                 router_bias=c["router_bias"])
        flags = spt.ARENA_GEMV if args.path == "exact" else spt.ARENA_MMA
        self.ep = None
        if world > 1:
            # expert parallelism: this rank holds experts [r*E/N, (r+1)*E/N)
            # and the whole router; token rows cross NVLink through the
            # library's NCCL exchange (the id of its communicator comes from
            # rank 0)
            experts = spt.ep_expert_range(E, world, rank)
            self.arena = ctx.synthetic_arena(cfg, params, n_layers=self.layers, flags=flags, experts=experts)
            uid = [spt.ep_unique_id() if rank == 0 else None]
            torch.distributed.broadcast_object_list(uid, src=0)
            self.ep = spt.ExpertParallel(ctx, uid[0], rank, world)
            self.ep.set_capacity(self.T)  # no host synchronisation per step
        else:
            self.arena = ctx.synthetic_arena(cfg, params, n_layers=self.layers, flags=flags)
        self.stream = torch.cuda.ExternalStream(ctx.stream)
        self.x_host = x_rows(name, rank)
        dev = f"cuda:{local}"
        self.x_dev = torch.from_numpy(self.x_host).to(dev)
        self.out_dev = torch.empty_like(self.x_dev)
        self.flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
        self.x_pin = torch.from_numpy(self.x_host).pin_memory()
        self.out_pin = torch.empty_like(self.x_pin).pin_memory()

    def step(self):
        ctx, T = self.ctx, self.T
        if self.layers > 1:
            # the stack updates the residual stream in place: every step
            # starts from the same input rows (a device copy, part of the step)
            with self.torch.cuda.stream(self.stream):
                self.out_dev.copy_(self.x_dev)
            ctx.forward_stack_device(self.arena, self.out_dev.data_ptr(), T, eps=EPS, ep=self.ep)
        elif self.ep is not None:
            ctx.forward_moe_batch_ep_device(self.ep, self.arena, self.x_dev.data_ptr(), self.out_dev.data_ptr(), T)
        else:
            ctx.forward_moe_batch_device(self.arena, self.x_dev.data_ptr(), self.out_dev.data_ptr(), T)

    def host_call(self):
        """The caller-facing C-ABI call: host buffers in, host buffers out."""
        ctx, T = self.ctx, self.T
        xn, on = self.x_pin.numpy(), self.out_pin.numpy()
        if self.layers > 1:
            ctx.forward_stack(self.arena, xn, T, eps=EPS, ep=self.ep, out=on)
        elif self.ep is not None:
            ctx.forward_moe_batch_ep(self.ep, self.arena, xn, T, out=on)
        else:
            ctx.forward_moe_batch(self.arena, xn, T, out=on)

    def do_flush(self, i):
        with self.torch.cuda.stream(self.stream):
            self.flush.fill_(i & 0xFF)

    def barrier(self):
        if self.world > 1:
            self.torch.distributed.barrier()

    def max_over_ranks(self, v):
        if self.world == 1:
            return v
        t = self.torch.tensor([v], device=f"cuda:{self.local}", dtype=self.torch.float64)
        self.torch.distributed.all_reduce(t, op=self.torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        self.torch.cuda.synchronize()
        if self.ep is not None:
            self.ep.close()
        self.arena.close()


def measure(spt, torch, ctx, name, args, rank, world, local, steps, warmup, clocks=None):
    """Device throughput, per-kernel times, host-call e2e and parity of one
    workload.  Returns the fields of its line."""
    r = Runner(spt, torch, ctx, name, args, rank, world, local)
    T, T_all, layers = r.T, r.T_all, r.layers
    torch.cuda.synchronize()
    for _ in range(warmup):
        r.step()
    ctx.sync()
    kernels = ctx.kernels_per_forward()
    if r.ep is not None:
        n_active = ctx.last_dispatch()[0]  # this rank's experts used by the rows it received
        routing = None
    else:
        routing = ctx.last_routing(T, E, K)
        n_active = int((routing["counts"] > 0).sum())

    # ---- device time: inputs resident in HBM --------------------------------
    # No host synchronisation inside the loop; the 256 MB flush before each
    # step lets the host enqueue the step's kernels ahead of the GPU.
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    r.barrier()
    torch.cuda.synchronize()
    if clocks:
        clocks.__enter__()
    with torch.cuda.stream(r.stream):
        for i in range(steps):
            r.flush.fill_(i & 0xFF)
            starts[i].record(r.stream)
            r.step()
            ends[i].record(r.stream)
    torch.cuda.synchronize()
    if clocks:
        clocks.__exit__(None, None, None)
    r.barrier()
    total_ms = r.max_over_ranks(sum(s.elapsed_time(e) for s, e in zip(starts, ends)))
    ms_per_step = total_ms / steps
    value = T_all * steps / (total_ms / 1e3)
    device_out = r.out_dev.cpu().numpy()

    # ---- per-kernel durations for the roofline (events around each stage on
    # the launching stream; a separate pass) ----------------------------------
    ctx.set_stage_timing(True)
    stage_ms = []
    for i in range(steps):
        r.do_flush(i)
        r.step()
        stage_ms.append(ctx.stage_times())
    ctx.set_stage_timing(False)
    stages = {k: sum(s[k] for s in stage_ms) / len(stage_ms) for k in stage_ms[0]} if stage_ms else {}

    # ---- e2e: the host call on the host clock --------------------------------
    for _ in range(max(1, warmup)):
        r.host_call()
    e2e_s = 0.0
    for i in range(steps):
        r.do_flush(i)
        torch.cuda.synchronize()
        r.barrier()
        t0 = time.perf_counter()
        r.host_call()
        e2e_s += time.perf_counter() - t0
    e2e_s = r.max_over_ranks(e2e_s)
    host_out = r.out_pin.numpy().copy()
    same = bool(np.array_equal(host_out.view(np.uint32), device_out.view(np.uint32)) or
                np.array_equal(np.nan_to_num(host_out), np.nan_to_num(device_out)))

    # ---- roofline of the dominant kernel (gate/up + SwiGLU) ------------------
    peak_gbs, peak_bf16, peak_src = load_peaks()
    gu_ms, dn_ms = stages.get("gate_up", float("nan")), stages.get("down", float("nan"))
    gu_bytes, dn_bytes = n_active * 2 * MATRIX_BYTES, n_active * MATRIX_BYTES
    achieved = gu_bytes / (gu_ms / 1e3) / 1e9
    step_bytes = layers * (ROUTER_BYTES + 3 * n_active * MATRIX_BYTES)  # n_active of the last layer
    dispatched = T * K if r.ep is None else ctx.last_dispatch()[1]
    gu_flops = 2.0 * (2 * D) * H * dispatched
    path, bn = ctx.last_expert_path()
    kind = ("kind::mxf8f6f4, 3 e4m3 activation terms" if bn > 16 and ctx.get_option(spt.OPT_PREFILL_FP8)
            else "kind::mxf4, 4 e2m1 activation terms")
    kernel = {"gemv16": "k_gemv16<0> gate/up (e2m1 -> f16 in registers, mma.sync f16 -> f32, fused SwiGLU)",
              "tcgen05": f"k_mma_gemm<{bn}> gate/up (tcgen05 {kind}, fused SwiGLU)",
              "exact": "k_gemv gate/up (bit-exact CUDA-core MXFP4 GEMV, fused SwiGLU)"}[path]
    roof = {"bound": "hbm", "achieved": achieved, "peak": peak_gbs, "unit": "GB/s", "frac": achieved / peak_gbs,
            "traffic": load_traffic(f"{name}:{path}:gate_up_dram_bytes"), "kernel": kernel,
            "algorithmic_bytes": gu_bytes, "avg_ms": gu_ms, "peak_source": peak_src,
            "tflops": gu_flops / (gu_ms / 1e3) / 1e12,
            "down_kernel": {"achieved": dn_bytes / (dn_ms / 1e3) / 1e9, "avg_ms": dn_ms, "algorithmic_bytes": dn_bytes},
            "step_hbm_fraction": step_bytes / (ms_per_step / 1e3) / 1e9 / peak_gbs}

    # ---- parity (outside the timed regions) ----------------------------------
    parity = None
    if rank == 0 and not args.no_parity:
        if layers > 1:
            parity = parity_stack(name, r, device_out) if r.ep is None else None
        else:
            parity = parity_block(name, r.x_host, T, device_out, routing)
    r.close()
    return {"value": value, "unit": "tokens/s", "ms_per_step": ms_per_step, "tokens_per_step": T_all,
            "expert_path": path, "active_experts": n_active, "kernels_per_step": kernels,
            "gpu_launches": steps * kernels, "stages_ms": {k: round(v, 5) for k, v in stages.items()},
            "roofline": roof,
            "e2e": {"value": T_all * steps / e2e_s, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 4,
                    "d2h_bytes_per_step": T * H * 4, "ms_per_step": 1e3 * e2e_s / steps,
                    "clock": "host (perf_counter) around the C-ABI call, after a synchronised L2 flush",
                    "matches_device_path": same},
            "parity": parity}


DTYPES = {"gemv16": "mxfp4 weights (f16 in registers) x 2-term f16 activations -> f32 (mma.sync)",
          "tcgen05": "mxfp4 weights x block-scaled activation terms -> f32 (tcgen05)",
          "exact": "f32 (mxfp4 weights), the reference's AVX2 order"}


def run_ours(args):
    import torch

    rank, world, local = dist_info()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    spt = importlib.import_module("stream-pt_b200")
    ctx = spt.Context(local)
    ctx.set_path({"mma": spt.PATH_MMA, "exact": spt.PATH_EXACT, "auto": spt.PATH_AUTO,
                  "gemv16": spt.PATH_GEMV16}[args.path])
    clocks = ClockSampler(local)
    main = measure(spt, torch, ctx, args.config, args, rank, world, local, args.steps, args.warmup, clocks)
    extras = {}
    if not args.no_extras:
        names = ["c0", "c2", "c3", "c4"] if world == 1 else ["c3", "c4"]
        for n in names:
            if n == args.config:
                continue
            extras[n] = measure(spt, torch, ctx, n, args, rank, world, local, min(args.steps, 10),
                                max(3, min(args.warmup, 5)))
            extras[n]["workload"] = workload_config(n, world, ep_mode(n))["workload"]
            extras[n]["scaling"] = "strong" if CONFIGS[n].get("strong") else "weak"
    line = {"metric": "moe_block_tokens_per_s", "value": main["value"], "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": main["ms_per_step"],
            "higher_is_better": True, "scaling": "strong" if CONFIGS[args.config].get("strong") else "weak",
            "vs_baseline": None, "dtype": DTYPES[main["expert_path"]], "data": "synthetic",
            "config": workload_config(args.config, world, ep_mode(args.config)),
            "expert_path": main["expert_path"], "active_experts": main["active_experts"],
            "roofline": main["roofline"], "stages_ms": main["stages_ms"], "e2e": main["e2e"],
            "parity": main["parity"], "gpu_launches": main["gpu_launches"]}
    if extras:
        line["configs"] = extras
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tps, cores, sample = cpu_baseline(args.config)
        line["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}
    if rank == 0:
        line["clocks"] = clocks.summary()
        line["native_so_loaded"] = native_libraries()
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


Q80_ROWS, Q80_IN = 201088, 2880  # GPT-OSS output head (vocabulary x hidden)


def run_q80(args):
    """--config q80: the Q8_0 LM head (MulQ80Argmax, forward/q80.go:22-105),
    one token per step: argmax over W x for a 201,088 x 2,880 Q8_0 matrix
    resident in HBM.  Synthetic bytes (uniform int8, float16 scales
    N(0, 0.01)); 615 MB per step, larger than L2."""
    import torch
    rank, world, local = dist_info()
    torch.cuda.set_device(local)
    spt = importlib.import_module("stream-pt_b200")
    rng = np.random.default_rng(80)
    nb = Q80_IN // 32
    data = rng.integers(0, 256, size=(Q80_ROWS, nb, 34), dtype=np.uint8)
    data[:, :, :2] = (rng.standard_normal((Q80_ROWS, nb)) * 0.01).astype(np.float16).view(np.uint8).reshape(
        Q80_ROWS, nb, 2)
    data = data.reshape(-1)
    ctx = spt.Context(local)
    m = ctx.q80_matrix(data, Q80_IN, Q80_ROWS)
    x_host = spt.synth_normal_host(80, 1, Q80_IN)
    x_dev = torch.from_numpy(x_host).to(f"cuda:{local}")
    res = torch.zeros(2, dtype=torch.int64, device=f"cuda:{local}")
    stream = torch.cuda.ExternalStream(ctx.stream)

    def step():
        m.mul_device(x_dev.data_ptr(), 0, res.data_ptr(), res.data_ptr() + 8)

    for _ in range(args.warmup):
        step()
    ctx.sync()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                starts[i].record(stream)
                step()
                ends[i].record(stream)
        torch.cuda.synchronize()
    ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
    # e2e: the public host call (host x -> device -> head -> argmax and logit
    # back), synchronous, on the host clock
    e_ms = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        _, idx, logit = m.mul(x_host, want_y=False)
        if i >= args.warmup:
            e_ms.append((time.perf_counter() - t0) * 1e3)
    e2e_ms = sum(e_ms) / len(e_ms)
    # parity of the whole head against the oracle (outside the timed regions):
    # every logit bit for bit, the argmax row and its logit
    from oracle import oracle
    y_got, idx_got, logit_got = m.mul(x_host, want_y=True)
    y_want, idx_want, logit_want = oracle.mul_q80(data, Q80_IN, Q80_ROWS, x_host, os.cpu_count() or 1)
    logits_exact = bool(np.array_equal(y_got.view(np.uint32), y_want.view(np.uint32)))
    parity = {"rows_checked": Q80_ROWS, "logits_bit_exact": logits_exact,
              "argmax_equal": int(idx_got) == int(idx_want) == int(idx),
              "logit_bit_exact": np.float32(logit_got).view(np.uint32) == np.float32(logit_want).view(np.uint32)}
    parity["logit_bit_exact"] = bool(parity["logit_bit_exact"])
    parity["ok"] = bool(logits_exact and parity["argmax_equal"] and parity["logit_bit_exact"])
    peak, _, peak_src = load_peaks()
    nbytes = Q80_ROWS * nb * 34
    line = {"metric": "lm_head_tokens_per_s", "value": 1e3 / ms, "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q8_0 weights x f32 -> f32 (CUDA cores, bit-exact)",
            "data": "synthetic",
            "config": {"workload": "q80: Q8_0 LM head argmax, 201088 x 2880 (north_star q80.go)",
                       "rows": Q80_ROWS, "input": Q80_IN, "l2": "615 MB matrix > L2"},
            "roofline": {"bound": "hbm", "achieved": nbytes / (ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": nbytes / (ms / 1e3) / 1e9 / peak,
                         "traffic": load_traffic("q80:gemv:dram_bytes"), "kernel": "k_q80_gemv",
                         "algorithmic_bytes": nbytes, "avg_ms": ms, "peak_source": peak_src},
            "e2e": {"value": 1e3 / e2e_ms, "unit": "tokens/s", "h2d_bytes_per_step": Q80_IN * 4,
                    "d2h_bytes_per_step": 20, "ms_per_step": e2e_ms,
                    "clock": "host (perf_counter) around the synchronous host call"},
            "parity": parity, "gpu_launches": args.steps * 3, "argmax": int(idx), "clocks": clocks.summary()}
    if not args.no_cpu_baseline:
        from oracle import oracle
        workers = os.cpu_count() or 1
        oracle.mul_q80(data, Q80_IN, Q80_ROWS, x_host, workers)
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 10.0 and reps < 100:
            oracle.mul_q80(data, Q80_IN, Q80_ROWS, x_host, workers)
            reps += 1
        el = time.perf_counter() - t0
        line["cpu_baseline"] = {"value": reps / el, "unit": "tokens/s", "cores": workers, "kind": "port",
                                "sample": f"{reps} full passes over the head ({el:.1f} s)"}
    print(json.dumps(line), flush=True)
    m.close()
    ctx.close()


Q40_LAYERS, Q40_QKV, Q40_QD = 36, 5120, 4096  # GPT-OSS-120B: 36 layers, Q/K/V = 4096 + 512 + 512 rows, O input 4096


def _q40_bytes(rows, input_, seed):
    rng = np.random.default_rng(seed)
    nb = input_ // 32
    data = rng.integers(0, 256, size=(rows, nb, 18), dtype=np.uint8)
    data[:, :, :2] = (rng.standard_normal((rows, nb)) * 0.01).astype(np.float16).view(np.uint8).reshape(rows, nb, 2)
    return data.reshape(-1)


def _q40_traffic(prefix):
    qkv, o = load_traffic(prefix + ":qkv_dram_bytes"), load_traffic(prefix + ":o_dram_bytes")
    return None if qkv is None or o is None else Q40_LAYERS * (qkv + o)


def run_q40(args):
    """--config q40 / q40b: the Q4_0 attention projections of GPT-OSS-120B
    (MulQ40Into / MulQ40BatchInto, forward/q40.go:35-101): per layer the
    Q, K and V rows fused in one 5,120 x 2,880 matrix (the three tensors
    share their input; rows are independent, so the fused product equals the
    three) and O, 2,880 x 4,096; 36 layers resident in HBM (537 MB, larger
    than L2).  q40: one decode token per step (batch 1, the one-input
    order); q40b: 128 tokens per step (the batched order).  Synthetic bytes
    (uniform nibbles, float16 scales N(0, 0.01)), N(0, 1) inputs.  The step's
    72 launches are captured once into a CUDA graph and replayed."""
    import torch
    rank, world, local = dist_info()
    torch.cuda.set_device(local)
    spt = importlib.import_module("stream-pt_b200")
    batch = 1 if args.config == "q40" else 128
    ctx = spt.Context(local)
    mats = []
    host = {}
    for l in range(Q40_LAYERS):
        for kind, rows, inp in (("qkv", Q40_QKV, H), ("o", H, Q40_QD)):
            data = _q40_bytes(rows, inp, 4000 + 2 * l + (kind == "o"))
            if l == 0:
                host[kind] = data
            r, t = spt.q40_tensor(data, inp, rows, name=f"blk.{l}.attn_{kind}.weight")
            mats.append((ctx.q40_matrix(r, t), inp, rows))
    x_h = spt.synth_normal_host(40, 1, batch * H)
    a_h = spt.synth_normal_host(41, 1, batch * Q40_QD)
    dev = f"cuda:{local}"
    x_d, a_d = torch.from_numpy(x_h).to(dev), torch.from_numpy(a_h).to(dev)
    y_qkv = torch.empty(batch * Q40_QKV, dtype=torch.float32, device=dev)
    y_o = torch.empty(batch * H, dtype=torch.float32, device=dev)
    stream = torch.cuda.ExternalStream(ctx.stream)

    def step():
        for m, inp, rows in mats:
            if inp == H:
                m.mul_device(x_d.data_ptr(), y_qkv.data_ptr(), batch)
            else:
                m.mul_device(a_d.data_ptr(), y_o.data_ptr(), batch)

    for _ in range(args.warmup):
        step()
    ctx.sync()
    launch = "CUDA graph of the step's 72 launches"
    graph = None
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream, capture_error_mode="thread_local"):
            step()
        torch.cuda.synchronize()
    except Exception as exc:  # capture refused: time the direct launches
        graph, launch = None, f"direct launches (graph capture failed: {type(exc).__name__})"
        torch.cuda.synchronize()
    run = graph.replay if graph is not None else step
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                starts[i].record(stream)
                run()
                ends[i].record(stream)
        torch.cuda.synchronize()
    ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, ends)) / args.steps
    # parity of the timed step's first layer against the oracle (outside the timed region)
    from oracle import oracle
    workers = os.cpu_count() or 1
    got_q = torch.empty_like(y_qkv)
    got_o = torch.empty_like(y_o)
    mats[0][0].mul_device(x_d.data_ptr(), got_q.data_ptr(), batch)
    mats[1][0].mul_device(a_d.data_ptr(), got_o.data_ptr(), batch)
    ctx.sync()
    items = min(batch, 8)
    want_q = oracle.mul_q40(host["qkv"], H, Q40_QKV, x_h[:items * H] if batch > 1 else x_h, items if batch > 1 else 1,
                            workers)
    want_o = oracle.mul_q40(host["o"], Q40_QD, H, a_h[:items * Q40_QD] if batch > 1 else a_h,
                            items if batch > 1 else 1, workers)
    gq = got_q.cpu().numpy().reshape(batch, Q40_QKV)[:items]
    go = got_o.cpu().numpy().reshape(batch, H)[:items]
    bit_exact = bool(np.array_equal(gq.view(np.uint32), want_q.view(np.uint32)) and
                     np.array_equal(go.view(np.uint32), want_o.view(np.uint32)))
    # e2e: the public host call per matrix (host x -> device -> product -> host y)
    e_ms = []
    xq_host, xo_host = x_h, a_h
    yq_host = np.empty(batch * Q40_QKV, np.float32)
    yo_host = np.empty(batch * H, np.float32)
    for i in range(args.warmup + max(2, args.steps // 4)):
        t0 = time.perf_counter()
        for m, inp, rows in mats:
            if inp == H:
                m.mul(xq_host, batch, yq_host)
            else:
                m.mul(xo_host, batch, yo_host)
        if i >= args.warmup:
            e_ms.append((time.perf_counter() - t0) * 1e3)
    e2e_ms = sum(e_ms) / len(e_ms)
    peak, _, peak_src = load_peaks()
    nbytes = Q40_LAYERS * (Q40_QKV * (H // 32) * 18 + H * (Q40_QD // 32) * 18)
    fmas = Q40_LAYERS * (Q40_QKV * H + H * Q40_QD) * batch
    line = {"metric": "attn_proj_tokens_per_s", "value": batch * 1e3 / ms, "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "q4_0 weights x f32 -> f32 (CUDA cores, bit-exact)", "data": "synthetic",
            "config": {"workload": f"{args.config}: Q4_0 attention projections (fused QKV 5120x2880 + O 2880x4096) "
                                   f"of 36 layers, batch {batch} (north_star q40.go)",
                       "batch": batch, "layers": Q40_LAYERS, "launch": launch,
                       "l2": "537 MB of matrices per step > L2"},
            "parity": {"bit_exact": bit_exact, "items_checked": items, "matrices_checked": 2},
            "e2e": {"value": batch * 1e3 / e2e_ms, "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": Q40_LAYERS * batch * (H + Q40_QD) * 4,
                    "d2h_bytes_per_step": Q40_LAYERS * batch * (Q40_QKV + H) * 4 + Q40_LAYERS * 2 * 4,
                    "clock": "host (perf_counter) around the 72 synchronous host calls"},
            "gpu_launches": args.steps * 2 * Q40_LAYERS, "clocks": clocks.summary()}
    if batch == 1:
        line["roofline"] = {"bound": "hbm", "achieved": nbytes / (ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                            "frac": nbytes / (ms / 1e3) / 1e9 / peak, "traffic": _q40_traffic("q40:gemv"),
                            "traffic_scope": "per step: 36 x the fused-QKV and O launches ncu captured",
                            "kernel": "k_q40_gemv",
                            "algorithmic_bytes": nbytes, "avg_ms": ms, "peak_source": peak_src}
    else:
        nominal = 148 * 128 * 2 * 1.965e9 / 1e12  # fp32 FMA on CUDA cores at the max SM clock
        tf = 2 * fmas / (ms / 1e3) / 1e12
        line["roofline"] = {"bound": "fp32-fma", "achieved": tf, "peak": nominal, "unit": "TFLOP/s",
                            "frac": tf / nominal, "traffic": _q40_traffic("q40b:batch"),
                            "traffic_scope": "per step: 36 x the fused-QKV and O launches ncu captured",
                            "kernel": "k_q40_batch",
                            "algorithmic_flops": 2 * fmas, "algorithmic_bytes": nbytes, "avg_ms": ms,
                            "peak_source": "nominal fp32 CUDA-core rate (148 SMs x 128 FMA/clk x 1965 MHz); "
                                           "no measured fp32 figure"}
    if not args.no_cpu_baseline:
        xs_ = x_h[:H * min(batch, 8)] if batch > 1 else x_h
        nb_ = min(batch, 8) if batch > 1 else 1
        oracle.mul_q40(host["qkv"], H, Q40_QKV, xs_, nb_, workers)
        reps, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < 10.0:
            oracle.mul_q40(host["qkv"], H, Q40_QKV, xs_, nb_, workers)
            reps += 1
        el = time.perf_counter() - t0
        per_tok = el / reps / nb_ * (Q40_QKV * H + H * Q40_QD) / (Q40_QKV * H) * Q40_LAYERS
        line["cpu_baseline"] = {"value": 1.0 / per_tok, "unit": "tokens/s", "cores": workers, "kind": "port",
                                "sample": f"{reps} products of one fused QKV matrix x {nb_} token(s) ({el:.1f} s), "
                                          "scaled by FMA count to the 72 matrices of a step"}
    print(json.dumps(line), flush=True)
    if graph is not None:
        del graph
    for m, _, _ in mats:
        m.close()
    ctx.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c1", choices=sorted(CONFIGS) + ["q80", "q40", "q40b"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--path", default="auto", choices=["auto", "mma", "gemv16", "exact"],
                    help="expert products: the library's choice (auto), tcgen05 (mma), the decode GEMV "
                         "(gemv16) or the bit-exact CUDA-core GEMV (exact)")
    ap.add_argument("--no-extras", action="store_true", help="only the --config workload")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.config == "q80":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the q80 mode times the LM head only through "
                              "its cpu_baseline (the oracle port) in the same line"}), flush=True)
        else:
            run_q80(args)
    elif args.config in ("q40", "q40b"):
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the q40 modes time the oracle port only "
                              "through the cpu_baseline of the same line"}), flush=True)
        else:
            run_q40(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
