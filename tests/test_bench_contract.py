"""The bench's reference arm on the CPU (no GPU): `bench.py --impl reference` times the C
restatement of the reference's attention (oracle/attn_ref.c) on the host cores and prints
one JSON line with the keys the benchmark driver reads: the same metric, unit and direction
as the GPU arm, `impl: reference`, a cpu_baseline describing the run, and an e2e object
with no host/device copies."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "whisper_small_en_encoder_attention_windows_per_s"
    assert d["unit"] == "windows/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] >= 3
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["cores"] >= 1 and cb["kind"] in ("port", "reference") and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"]


def test_reference_arm_two_ranks_prints_once():
    """Launched the way the driver launches N > 1 (torchrun, 127.0.0.1): rank 0 alone runs
    and prints the reference line; the other rank exits 0 without work."""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", "29561", "bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1",
           "--warmup", "3"]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout[-2000:]
    assert json.loads(lines[0])["impl"] == "reference"
