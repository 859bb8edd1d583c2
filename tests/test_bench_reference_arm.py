"""bench.py's reference arm on the host, launched as a benchmark harness does
(``bench.py --impl reference``): one JSON line with the base contract's keys,
the same metric and ``config`` as the B200 arm's line, a ``cpu_baseline`` that
describes the run, zero-byte ``e2e`` copies, and no product library loaded in
the process (the oracle generates its inputs and is what it times).  The
modes with no reference arm print their ``unavailable`` line and exit 0."""
import json
import os
import socket
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402  (imports no GPU code at module level)


def run_bench(*args, timeout=240, launcher=()):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run([sys.executable, *launcher, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=env,
                         capture_output=True, text=True, timeout=timeout)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_reference_arm_line():
    line = run_bench("--impl", "reference", "--steps", "1", "--warmup", "3")
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["metric"] == "moe_block_tokens_per_s" and line["unit"] == "tokens/s"
    assert line["higher_is_better"] is True and line["n_gpus"] == 1
    assert line["steps"] == 1 and line["warmup"] == 3
    # the B200 arm's config for the same workload, key for key
    assert line["config"] == bench.workload_config("c1", 1, bench.ep_mode("c1"))
    assert line["value"] > 0
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["value"] == line["value"] and cb["cores"] >= 1 and cb["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    loaded = line["native_so_loaded"]
    assert not any("libspt_moe" in p for p in loaded), loaded
    assert any("libspt_oracle" in p for p in loaded), loaded


def test_modes_without_a_reference_arm():
    for config in ("q80", "q40", "q40b"):
        line = run_bench("--config", config, "--impl", "reference", "--steps", "1", "--warmup", "3", timeout=60)
        assert line["impl"] == "reference" and line["unavailable"], line


def test_reference_arm_under_torchrun():
    """Two ranks as the scaling runs launch them: rank 0 alone prints one line
    (the N-rank workload's config), the other rank exits 0 without work."""
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    launcher = ("-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
                "127.0.0.1", "--master-port", str(port))
    line = run_bench("--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "3", launcher=launcher)
    assert line["impl"] == "reference" and line["n_gpus"] == 2
    assert line["config"] == bench.workload_config("c1", 2, bench.ep_mode("c1"))
    assert not any("libspt_moe" in p for p in line["native_so_loaded"])

