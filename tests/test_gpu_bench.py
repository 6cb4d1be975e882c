"""bench.py's JSON line on a B200, at a small configuration: every key the benchmark contract asks for is present
and consistent, and the loss the timed steps computed equals the CPU oracle's loss on the same ids and weights."""
import json
import math
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ROWS, SEQ, LAYERS = 2, 512, 2


@pytest.mark.gpu
def test_bench_json_line_and_loss(cuda_ok):
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--global-rows", str(ROWS), "--seq", str(SEQ),
                        "--layers", str(LAYERS), "--steps", "3", "--warmup", "3", "--decode-streams", "4",
                        "--decode-steps", "4", "--decode-prompt", "64", "--no-scaled"], cwd=ROOT, capture_output=True,
                       text=True, timeout=900)
    assert p.returncode == 0, p.stderr[-3000:]
    d = json.loads(p.stdout.strip().splitlines()[-1])

    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in d, key
    assert d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3 and d["value"] > 0
    # throughput = tokens of the step / device time of the step
    assert d["value"] == pytest.approx(ROWS * SEQ / (d["ms_per_step"] / 1e3), rel=2e-3)

    e2e = d["e2e"]
    assert e2e["value"] > 0 and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 2 * ROWS * SEQ * 4  # int32 ids + int32 targets
    assert e2e["d2h_bytes_per_step"] > 0
    assert d["gpu_launches"] > 0

    roof = d["roofline"]
    for key in ("kernel", "bound", "achieved", "peak", "unit", "frac", "traffic"):
        assert key in roof, key
    assert roof["bound"] in ("hbm", "tensor") and roof["achieved"] > 0 and roof["peak"] > 0
    assert roof["frac"] == pytest.approx(roof["achieved"] / roof["peak"], rel=1e-2)
    for k, v in d["roofline_by_kernel"].items():
        assert v["achieved"] > 0, k

    cpu = d["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["value"] > 0 and cpu["cores"] >= 1 and cpu["sample"]
    clk = d["clocks"]
    assert "sm_mhz" in clk and "sm_max_mhz" in clk and isinstance(clk["reasons"], list)
    assert d["decode"]["value"] > 0 and d["decode"]["cuda_graph"] is True
    assert d["decode"]["roofline"]["achieved"] > 0 and d["decode"]["steps"] == 4
    assert d["scaling"] == "strong" and d["config"]["global_batch"] == ROWS
    for tag, site in d["roofline_by_call_site"].items():  # every GEMM call site has its own FLOP figure
        assert site["achieved"] > 0, tag
    assert {"rt_proj", "rt_out", "ts_q", "ts_wo", "head_ce"} <= set(d["roofline_by_call_site"])
    part = d["partial"]
    assert part["value"] > 0 and part["roofline_gemm"]["achieved"] > 0
    assert {"swiglu_gu", "swiglu_down", "head_logits"} <= set(part["roofline_by_call_site"])

    # the timed steps' loss against the oracle on the bench's own ids (rank 0 seed) and weights
    sys.path.insert(0, ROOT)
    import bench as B
    from oracle import sdm_oracle as O
    P = B.oracle_params(LAYERS)
    ids = B.zipf_ids(1000, ROWS, SEQ + 1)
    lg = O.lm_forward(P, ids[:, :-1], bf16_stream=True, margins=False)
    want = O.ce_sum(lg, ids[:, 1:]) / (ROWS * SEQ)
    assert math.isfinite(d["loss_mean"])
    # bf16 activations: logits agree to ~1e-3 relative, the mean CE to well within this
    assert d["loss_mean"] == pytest.approx(want, rel=2e-3), (d["loss_mean"], want)
    assert np.isfinite(want)
