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


def test_reference_arm_other_ranks_print_nothing():
    p = _run({"RANK": "1", "WORLD_SIZE": "2"}, "--impl", "reference", "--steps", "1", "--warmup", "1",
             "--layers", "1")
    assert p.returncode == 0, p.stderr[-2000:]
    assert p.stdout.strip() == ""


def test_roofline_tables():
    sys.path.insert(0, ROOT)
    import bench as B
    # projection columns [wk; wq; wv; wg] = 2 * 12 * 32 + 768 + 12
    assert B.gemm_flops("rt_proj", 1, 12) == 2 * 768 * 1548
    assert B.gemm_flops("head_ce", 10, 12) == 10 * 2 * 768 * 32768
    assert B.gemm_flops("unknown", 10, 12) == 0
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
