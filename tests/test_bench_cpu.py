"""bench.py's reference arm (the oracle timed on host cores) runs without a GPU: its
one JSON line carries the fields the bench contract names."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    p = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", "norm", "--steps", "2", "--warmup", "1"],
        capture_output=True, text=True, timeout=600, cwd=ROOT,
    )
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, p.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "add+RMSNorm fwd+bwd HBM GB/s" and d["unit"] == "GB/s"
    assert d["n_gpus"] == 1 and d["higher_is_better"] is True and d["scaling"] == "weak"
    assert d["warmup"] >= 3  # the timing rule's minimum is enforced
    assert d["value"] > 0 and d["ms_per_step"] > 0
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"] == "add_rmsnorm_fwd_bwd_bf16_8192x4096"
    assert d["config"]["rows_per_gpu"] == 8192 and d["config"]["dim"] == 4096  # the same keys as the GPU arm's config


def test_default_reference_arm_is_the_long_attention_config():
    """The default workload is the north star's primary target; its reference arm times
    the oracle on one (b, h) slice per host core in spawned processes."""
    p = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "1"],
        capture_output=True, text=True, timeout=900, cwd=ROOT,
    )
    assert p.returncode == 0, p.stderr[-2000:]
    d = json.loads([ln for ln in p.stdout.splitlines() if ln.startswith("{")][-1])
    assert d["impl"] == "reference" and d["metric"] == "causal flash-attn fwd+bwd TFLOP/s" and d["unit"] == "TFLOP/s"
    assert d["scaling"] == "strong" and d["value"] > 0
    cfg = d["config"]
    assert cfg["workload"] == "flash_attention_causal_fwd_bwd_b8_h32_s8192_d128_bf16"
    assert (cfg["batch"], cfg["heads"], cfg["seq_len"], cfg["head_dim"]) == (8, 32, 8192, 128)
    assert d["cpu_baseline"]["cores"] >= 1 and "spawned processes" in d["cpu_baseline"]["sample"]


def test_help_lists_the_workloads():
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--help"], capture_output=True, text=True, timeout=120, cwd=ROOT)
    assert p.returncode == 0
    for w in ("norm", "attn", "attn_small", "gemm", "gemm_ragged", "gemm_f32", "gpt", "prefill", "decode"):
        assert w in p.stdout


def test_decode_reference_arm_json_line():
    p = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", "decode", "--steps", "1", "--warmup", "1"],
        capture_output=True, text=True, timeout=600, cwd=ROOT,
    )
    assert p.returncode == 0, p.stderr[-2000:]
    d = json.loads([ln for ln in p.stdout.splitlines() if ln.startswith("{")][-1])
    assert d["impl"] == "reference" and d["metric"] == "decode attention HBM GB/s" and d["unit"] == "GB/s"
    assert d["value"] > 0 and d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["config"]["workload"] == "gpt_decode_attention_kv_24x8x16x1024x64_pos1023_bf16"
