"""bench.py's driver contract on the host: the reference arm's JSON line, rank != 0 printing nothing, and the
algorithmic-byte / FLOP tables the roofline fields are computed from."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(env_extra, *args):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=600)


def test_reference_arm_json_line():
    p = _run({}, "--impl", "reference", "--steps", "1", "--warmup", "1", "--layers", "1")
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in d, key
    assert d["value"] > 0 and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["cores"] >= 1 and d["cpu_baseline"]["sample"]
    assert d["scaling"] == "strong" and d["config"]["global_batch"] == 32 and d["config"]["seq_len"] == 2048


def test_reference_arm_other_ranks_print_nothing():
    p = _run({"RANK": "1", "WORLD_SIZE": "2"}, "--impl", "reference", "--steps", "1", "--warmup", "1",
             "--layers", "1")
    assert p.returncode == 0, p.stderr[-2000:]
    assert p.stdout.strip() == ""


def test_roofline_from_profile_groups():
    """The roofline fields follow from the profiled pass's per-launch times and the FLOP tables."""
    sys.path.insert(0, ROOT)
    import bench as B
    pk = {"hbm_gbs": 6500.0, "bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0}
    rows = 65536
    groups = [("gemm_tc", "rt_proj", 12, 2.8), ("gemm_tc", "ts_q", 12, 0.4), ("gemm_tc", "ts_wo", 12, 1.8),
              ("gemm_tc", "head_ce", 1, 3.8), ("rt_scan", "", 12, 8.0)]
    roof, by_kernel, by_site, breakdown = B.roofline_tables(groups, rows, 1, pk, "measured")
    fl = rows * (12 * (B.gemm_flops("rt_proj", 1) + B.gemm_flops("ts_q", 1) + B.gemm_flops("ts_wo", 1))
                 + B.gemm_flops("head_ce", 1))
    ach = fl / (8.8e-3) / 1e12
    assert roof["bound"] == "tensor" and abs(roof["achieved"] - ach) < 0.1
    assert abs(roof["frac"] - ach / 1400.0) < 1e-4
    assert abs(by_site["ts_wo"]["achieved"] - 12 * rows * 2 * 768 * 768 / 1.8e-3 / 1e12) < 0.1
    assert breakdown["gemm_tc"]["launches_per_step"] == 37


def test_roofline_tables():
    sys.path.insert(0, ROOT)
    import bench as B
    # projection columns [wk; wq; wv; wg] = 2 * 12 * 32 + 768 + 12
    assert B.gemm_flops("rt_proj", 1, 12) == 2 * 768 * 1548
    assert B.gemm_flops("head_ce", 10, 12) == 10 * 2 * 768 * 32768
    assert B.gemm_flops("unknown", 10, 12) == 0
    # TrainedSdm: the query (d -> 4 heads x 32) and wo (d -> d) launches are separate call sites, each counted once
    assert B.gemm_flops("ts_q", 1) == 2 * 768 * 128 and B.gemm_flops("ts_wo", 1) == 2 * 768 * 768
    assert B.gemm_flops("swiglu_gu", 1) == 2 * 768 * 4096 and B.gemm_flops("swiglu_down", 1) == 2 * 2048 * 768
    # FULL: the call sites of one token sum to the algorithmic 109.5 MFLOP/token
    full = 12 * sum(B.gemm_flops(t, 1) for t in ("rt_proj", "rt_out", "ts_q", "ts_wo")) + B.gemm_flops("head_ce", 1)
    assert full == 12 * (2 * 768 * 1548 + 2 * 768 ** 2 + 2 * 768 * 128 + 2 * 768 ** 2) + 2 * 32768 * 768
    assert abs(full / 1e6 - 109.5) < 0.1
    # PARTIAL: 206.3 MFLOP/token
    part = 12 * sum(B.gemm_flops(t, 1) for t in ("rt_proj", "rt_out", "swiglu_gu", "swiglu_down")) + \
        B.gemm_flops("head_logits", 1)
    assert abs(part / 1e6 - 206.3) < 0.1
    # every GEMM call site with a measured DRAM figure has a FLOP figure
    for (k, tag) in B.NCU_DRAM_PER_TOKEN:
        if k == "gemm_tc":
            assert B.gemm_flops(tag, 1) > 0, tag
    # decode state bytes per (stream-step, layer, head): k rows of dh + 1 floats read + k read-modified-written
    assert B.DECODE_STATE_BYTES_PER_HEAD == 4160 + 8320
    # bf16 row in + row out
    assert B.kernel_bytes("rmsnorm", "", 3) == 3 * 768 * 4
    # num (64 fp32) + den per head in, bf16 hi/lo row out
    assert B.kernel_bytes("rt_finish", "rt_out", 1) == 12 * (64 * 4 + 4) + 768 * 4
    # every kernel with a measured DRAM figure also has an algorithmic figure
    for (k, tag) in B.NCU_DRAM_PER_TOKEN:
        if k != "gemm_tc":
            assert B.kernel_bytes(k, tag, 1) > 0, (k, tag)
    # the scan's reference-algorithm bytes per (token, head): state re-read + re-written once per 128-token chunk
    assert B.SCAN_BYTES_PER_TOKEN_HEAD == 4804


if __name__ == "__main__":
    sys.exit(pytest.main([__file__, "-q"]))
