"""Test infrastructure: times the UNMODIFIED SDMCHAT reference module (torch, CPU, all host threads) beside this
directory's numpy port on the same machine, model and tokens, and writes the ratio to port_vs_reference.json.

The GPU box cannot import the reference (it does not travel), so bench.py's CPU legs time the port there; this
factor, measured where both run, says how the port's CPU speed compares with the reference's own CPU forward.

    python oracle/time_port_vs_reference.py --ref PATH_TO_SDMCHAT_CHECKOUT [--tokens 2048]

Model: FULL onesdm_allsdm d768 L12 (the benchmark's), built with the reference's own build_onesdm
(experiments/track4/sdmllm/track4_onesdm_models.py:617-625) from the same seed and perturbation as bench.py;
one row of Zipf(1.1) tokens; the reference's forward with logits (OneSdmLM.forward, :550-555) in float32 under
torch.no_grad, and the port's lm_forward + CE sum with the same weights."""
import argparse
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("SDMCHAT_REF"), help="SDMCHAT checkout (or SDMCHAT_REF)")
    ap.add_argument("--tokens", type=int, default=2048)
    a = ap.parse_args()
    if not a.ref:
        ap.error("--ref (or SDMCHAT_REF) is required")
    sys.path.insert(0, os.path.join(a.ref, "experiments", "track4", "sdmllm"))
    import track4_onesdm_models as OM  # noqa: E402
    import bench  # noqa: E402

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    torch.manual_seed(0)
    ref = OM.build_onesdm("onesdm_allsdm", bench.V, bench.model_cfg(12)).eval()
    bench.perturb(ref)
    ids = bench.zipf_ids(99, 1, a.tokens + 1)
    x = torch.from_numpy(ids[:, :-1].astype(np.int64))
    with torch.no_grad():
        ref(x[:, :17])  # warm
        t0 = time.perf_counter()
        ref(x)
        t_ref = time.perf_counter() - t0

    P = bench.oracle_params(12)
    bench.oracle_step(P, ids[:, :17])  # warm
    t0 = time.perf_counter()
    bench.oracle_step(P, ids)
    t_port = time.perf_counter() - t0

    out = {"tokens": a.tokens, "rows": 1, "host_threads": threads,
           "reference_torch_cpu_tok_s": round(a.tokens / t_ref, 1),
           "port_numpy_tok_s": round(a.tokens / t_port, 1),
           "port_over_reference": round(t_ref / t_port, 4),
           "model": "FULL onesdm_allsdm d768 L12 (bench weights), forward with logits",
           "script": "oracle/time_port_vs_reference.py"}
    with open(os.path.join(HERE, "port_vs_reference.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(json.dumps(out))


if __name__ == "__main__":
    main()
