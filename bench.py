"""Benchmark of the B200 MoE FFN block (GPT-OSS-120B shapes).

python bench.py [--gpus N] [--steps K] [--warmup W] [--config c1] [--impl ours|reference]

Prints ONE JSON line (rank 0).  A step is one forward of the MoE block over
one batch of synthetic tokens (seeded Philox weights generated on the device,
N(0,1) activations).  `value` times the device path with inputs resident in
HBM; `e2e` times the C-ABI host call (pinned host x -> H2D -> block -> D2H).
The L2 (126 MB) is flushed between timed steps by writing a 256 MB buffer.

--impl reference times the CPU restatement of the reference's AVX2 path
(oracle/, all host threads) on the same config; rank 0 only.

Configs (BASELINE.json configs[i]): c0 T=1 decode, c1 T=32 prefill batch
(default: the headline workload), c2 T=2048 Zipf-skewed routing.  Under
torchrun (N > 1) the block runs expert-parallel: rank r holds experts
[r*128/N, (r+1)*128/N), routes its own batch of the config's T tokens and
exchanges token and result rows with the other ranks over NCCL (the layout
of configs[3]); per-rank tokens are fixed, so scaling is weak.
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

CONFIGS = {
    "c0": dict(T=1, seed=0, zipf_s=0.0, zipf_beta=0.0, router_bias=True,
               desc="decode, 1 token (BASELINE configs[0])"),
    "c1": dict(T=32, seed=1, zipf_s=0.0, zipf_beta=0.0, router_bias=True,
               desc="prefill batch T=32 (BASELINE configs[1])"),
    "c2": dict(T=2048, seed=2, zipf_s=1.1, zipf_beta=0.9, router_bias=True,
               desc="prefill T=2048, Zipf(1.1)-skewed router bias (BASELINE configs[2])"),
    "c4": dict(T=64, seed=4, zipf_s=0.0, zipf_beta=0.0, router_bias=True, layers=36,
               desc="36-layer stack, RMSNorm + MoE + residual per layer, 64 token rows (BASELINE configs[4])"),
}
EPS = 1e-5


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    return 6650.0, "fallback (6.65 TB/s)"


def load_traffic(config, key="gate_up_dram_bytes"):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if not os.path.exists(p):
        return None
    d = json.load(open(p))
    return d.get(config, {}).get(key)


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


def mma_fp4(T):
    """Token tiles of <= 16 (T*top_k <= 8*experts) run the kind::mxf4 GEMM."""
    return T * K <= 8 * E


def mma_kind(T):
    return "kind::mxf4" if mma_fp4(T) else "kind::mxf8f6f4"


def mma_dtype(T):
    if mma_fp4(T):
        return "mxfp4 weights x 4-term e2m1 activations -> f32 (tcgen05 kind::mxf4)"
    return "mxfp4 weights x 3-term e4m3 activations -> f32 (tcgen05 kind::mxf8f6f4)"


def dist_info():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def cpu_baseline(cfg_name, seconds=12.0, workers=None):
    """The oracle (C restatement of the reference's AVX2 path) on the same
    workload, all host threads.  Returns (tokens/s, cores, sample text)."""
    from oracle import oracle
    spt = importlib.import_module("stream-pt_b200")
    c = CONFIGS[cfg_name]
    cfg = spt.Config(H, D, E, K)
    params = spt.SynthParams(seed=c["seed"], zipf_s=c["zipf_s"], zipf_beta=c["zipf_beta"],
                             router_bias=c["router_bias"])
    host = spt.synth_layer_host(cfg, params)
    w = oracle.Weights(H, D, E, K, host["router"], host["router_bias"], host["gate"], host["up"],
                       host["down"], host["gate_bias"], host["up_bias"], host["down_bias"])
    norm = spt.synth_norm_host(params, 0, H)
    layers = c.get("layers", 1)
    workers = workers or os.cpu_count() or 1
    T = c["T"]
    # bounded sample: at most 64 tokens of the workload per repetition, one
    # layer (a stack's time is the per-layer time times its depth)
    Ts = min(T, 64)
    x = spt.synth_normal_host(c["seed"], 1000, Ts * H)

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
    return tps, workers, f"{what} of {cfg_name} ({el:.1f} s, memory-resident weights)"


def run_reference(args):
    rank, world, _ = dist_info()
    if rank != 0:
        return
    tps, cores, sample = cpu_baseline(args.config, seconds=max(3.0, 2.0 * args.steps))
    line = {"metric": "moe_block_tokens_per_s", "value": tps, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * CONFIGS[args.config]["T"] / tps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (mxfp4 weights)",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": f"{args.config}: {CONFIGS[args.config]['desc']}",
                       "tokens_per_step": CONFIGS[args.config]["T"], "hidden": H, "experts": E, "top_k": K},
            "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch

    rank, world, local = dist_info()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120))
    spt = importlib.import_module("stream-pt_b200")
    c = CONFIGS[args.config]
    T = c["T"]
    cfg = spt.Config(H, D, E, K)
    params = spt.SynthParams(seed=c["seed"], zipf_s=c["zipf_s"], zipf_beta=c["zipf_beta"],
                             router_bias=c["router_bias"])
    ctx = spt.Context(local)
    flags = spt.ARENA_GEMV if args.path == "exact" else spt.ARENA_MMA
    layers = c.get("layers", 1)
    ep = None
    if world > 1:
        # expert parallelism: this rank holds experts [r*E/N, (r+1)*E/N) and
        # the whole router; token rows cross NVLink through the library's NCCL
        # exchange (the id of its communicator comes from rank 0)
        experts = spt.ep_expert_range(E, world, rank)
        arena = ctx.synthetic_arena(cfg, params, n_layers=layers, flags=flags, experts=experts)
        uid = [spt.ep_unique_id() if rank == 0 else None]
        torch.distributed.broadcast_object_list(uid, src=0)
        ep = spt.ExpertParallel(ctx, uid[0], rank, world)
        ep.set_capacity(T)  # fixed-capacity exchange: no host synchronisation per step
    else:
        arena = ctx.synthetic_arena(cfg, params, n_layers=layers, flags=flags)
    ctx.set_path({"mma": spt.PATH_MMA, "exact": spt.PATH_EXACT, "auto": spt.PATH_AUTO, "gemv16": spt.PATH_GEMV16}[args.path])
    stream = torch.cuda.ExternalStream(ctx.stream)
    x_host = spt.synth_normal_host(c["seed"] + 7919 * rank, 1000, T * H)
    x_dev = torch.from_numpy(x_host).to(f"cuda:{local}")
    out_dev = torch.empty_like(x_dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{local}")

    def step():
        if layers > 1:
            # the stack updates the residual stream in place: every step starts
            # from the same input rows (a 737 KB device copy, part of the step)
            with torch.cuda.stream(stream):
                out_dev.copy_(x_dev)
            ctx.forward_stack_device(arena, out_dev.data_ptr(), T, eps=EPS, ep=ep)
        elif ep is not None:
            ctx.forward_moe_batch_ep_device(ep, arena, x_dev.data_ptr(), out_dev.data_ptr(), T)
        else:
            ctx.forward_moe_batch_device(arena, x_dev.data_ptr(), out_dev.data_ptr(), T)

    def host_call(xn, on):
        if layers > 1:
            ctx.forward_stack(arena, xn, T, eps=EPS, ep=ep, out=on)
        elif ep is not None:
            ctx.forward_moe_batch_ep(ep, arena, xn, T, out=on)
        else:
            ctx.forward_moe_batch(arena, xn, T, out=on)

    torch.cuda.synchronize()
    for _ in range(args.warmup):
        step()
    ctx.sync()
    if ep is not None:
        n_active = ctx.last_dispatch()[0]  # this rank's experts used by the rows it received
    else:
        routing = ctx.last_routing(T, E, K)
        n_active = int((routing["counts"] > 0).sum())

    # ---- timed region: device-resident inputs ------------------------------
    # No host synchronisation inside the loop; the 256 MB L2 flush before each
    # step also lets the host enqueue the step's kernels ahead of the GPU.
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                flush.fill_(i & 0xFF)
                starts[i].record(stream)
                step()
                ends[i].record(stream)
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
    total_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    if world > 1:
        t = torch.tensor([total_ms], device=f"cuda:{local}")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = world * T * args.steps / (total_ms / 1e3)
    kernels_per_step = ctx.kernels_per_forward()
    # one launch per step: the single-launch decode kernel is the whole block
    decode_kernel = kernels_per_step == 1 and layers == 1 and ep is None

    # ---- per-kernel durations (same workload, CUDA events around each stage
    # on the launching stream; per-stage timing runs the separate kernels)
    # for the roofline ------------------------------------------------------
    ctx.set_stage_timing(True)
    stage_ms = []
    for i in range(args.steps):
        with torch.cuda.stream(stream):
            flush.fill_(i & 0xFF)
        step()
        stage_ms.append(ctx.stage_times())
    ctx.set_stage_timing(False)

    # ---- e2e through the C ABI with pinned host buffers --------------------
    x_pin = torch.from_numpy(x_host).pin_memory()
    out_pin = torch.empty_like(x_pin).pin_memory()
    xn, on = x_pin.numpy(), out_pin.numpy()
    for _ in range(max(1, args.warmup)):
        host_call(xn, on)
    e_st = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e_en = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if world > 1:
        torch.distributed.barrier()
    for i in range(args.steps):
        with torch.cuda.stream(stream):
            flush.fill_(i & 0xFF)
        e_st[i].record(stream)
        host_call(xn, on)
        e_en[i].record(stream)
    torch.cuda.synchronize()
    e2e_ms = sum(s.elapsed_time(e) for s, e in zip(e_st, e_en))
    if world > 1:
        t = torch.tensor([e2e_ms], device=f"cuda:{local}")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * T * args.steps / (e2e_ms / 1e3)
    ok = bool(np.array_equal(on.view(np.uint32), out_dev.cpu().numpy().view(np.uint32)) or
              np.array_equal(np.nan_to_num(on), np.nan_to_num(out_dev.cpu().numpy())))

    # ---- roofline of the dominant kernel (gate/up GEMV + SwiGLU) -----------
    peak, peak_src = load_peaks()
    gu = [s["gate_up"] for s in stage_ms if s]
    dn = [s["down"] for s in stage_ms if s]
    gu_ms = sum(gu) / len(gu) if gu else float("nan")
    dn_ms = sum(dn) / len(dn) if dn else float("nan")
    gu_bytes = n_active * 2 * MATRIX_BYTES
    dn_bytes = n_active * MATRIX_BYTES
    achieved = gu_bytes / (gu_ms / 1e3) / 1e9
    stages_avg = {k: round(sum(s[k] for s in stage_ms) / len(stage_ms), 5) for k in stage_ms[0]} if stage_ms else {}
    step_bytes = layers * (ROUTER_BYTES + 3 * n_active * MATRIX_BYTES)  # n_active of the last layer
    line = {
        "metric": "moe_block_tokens_per_s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": mma_dtype(T) if args.path == "mma" else "f32 (mxfp4 weights)",
        "data": "synthetic",
        "config": {"workload": f"{args.config}: {c['desc']}", "tokens_per_step": T, "hidden": H, "layers": layers,
                   "expert_path": args.path,
                   "expert_dim": D, "experts": E, "top_k": K, "seed": c["seed"],
                   "parallelism": (f"ep{world}: {E // world} experts per GPU, {T} tokens per rank, NCCL "
                                   "all-to-all dispatch/combine (fixed capacity)" if world > 1 else "single GPU"),
                   "l2": "256 MB buffer written between timed steps",
                   "active_experts": n_active},
        "roofline": ({"bound": "hbm", "achieved": step_bytes / (ms_per_step / 1e3) / 1e9, "peak": peak,
                      "unit": "GB/s", "frac": step_bytes / (ms_per_step / 1e3) / 1e9 / peak,
                      "traffic": load_traffic(args.config, "decode_dram_bytes"),
                      "kernel": "k_moe_decode (whole block in one cooperative launch, tcgen05 kind::mxf4)",
                      "algorithmic_bytes": step_bytes, "avg_ms": ms_per_step, "peak_source": peak_src,
                      "separate_kernels": {"gate_up_achieved": achieved, "gate_up_ms": gu_ms,
                                           "down_ms": dn_ms}}
                     if decode_kernel else
                     {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                      "frac": achieved / peak, "traffic": load_traffic(args.config),
                      "kernel": (f"k_mma_gemm gate/up (tcgen05 {mma_kind(T)}, fused SwiGLU)" if args.path == "mma"
                                 else "k_gemv<gate_up> (fused gate+up MXFP4 GEMV + SwiGLU)"),
                      "algorithmic_bytes": gu_bytes, "avg_ms": gu_ms, "peak_source": peak_src,
                      "down_kernel": {"achieved": dn_bytes / (dn_ms / 1e3) / 1e9, "avg_ms": dn_ms,
                                      "algorithmic_bytes": dn_bytes},
                      "step_hbm_fraction": step_bytes / (ms_per_step / 1e3) / 1e9 / peak}),
        "stages_ms": stages_avg,
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": T * H * 4,
                "d2h_bytes_per_step": T * H * 4, "ms_per_step": e2e_ms / args.steps,
                "matches_device_path": ok},
        "gpu_launches": args.steps * kernels_per_step,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tps, cores, sample = cpu_baseline(args.config)
        line["cpu_baseline"] = {"value": tps, "unit": "tokens/s", "cores": cores, "kind": "port",
                                "sample": sample}
    if rank == 0:
        line["clocks"] = clocks.summary()
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
    if ep is not None:
        ep.close()
    arena.close()
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
    e_ms = []
    for i in range(args.warmup + args.steps):
        st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.record(stream)
        _, idx, logit = m.mul(x_host, want_y=False)
        en.record(stream)
        torch.cuda.synchronize()
        if i >= args.warmup:
            e_ms.append(st.elapsed_time(en))
    e2e_ms = sum(e_ms) / len(e_ms)
    peak, peak_src = load_peaks()
    nbytes = Q80_ROWS * nb * 34
    line = {"metric": "lm_head_tokens_per_s", "value": 1e3 / ms, "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q8_0 weights x f32 -> f32 (CUDA cores, bit-exact)",
            "data": "synthetic",
            "config": {"workload": "q80: Q8_0 LM head argmax, 201088 x 2880 (north_star q80.go)",
                       "rows": Q80_ROWS, "input": Q80_IN, "l2": "615 MB matrix > L2"},
            "roofline": {"bound": "hbm", "achieved": nbytes / (ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": nbytes / (ms / 1e3) / 1e9 / peak, "traffic": None, "kernel": "k_q80_gemv",
                         "algorithmic_bytes": nbytes, "avg_ms": ms, "peak_source": peak_src},
            "e2e": {"value": 1e3 / e2e_ms, "unit": "tokens/s", "h2d_bytes_per_step": Q80_IN * 4,
                    "d2h_bytes_per_step": 16, "ms_per_step": e2e_ms},
            "gpu_launches": args.steps * 3, "argmax": int(idx), "clocks": clocks.summary()}
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c1", choices=sorted(CONFIGS) + ["q80"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--path", default="auto", choices=["auto", "mma", "gemv16", "exact"],
                    help="expert GEMMs on tcgen05 (mma) or the bit-exact CUDA-core GEMV (exact)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.config == "q80":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the q80 mode times the LM head only through "
                              "its cpu_baseline (the oracle port) in the same line"}), flush=True)
        else:
            run_q80(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
