#!/usr/bin/env python
"""Benchmark of the SDMCHAT FULL arm (onesdm_allsdm) d768 L12 T2048 on B200: prefill + tied-head loss tokens/s.

    python bench.py [--gpus N --steps K --warmup W]              this build (libsdm_b200, sm_100a)
    python bench.py --impl reference [...]                        the reference algorithm on the host CPU cores
    torchrun --nproc-per-node N bench.py --gpus N ...             one process per GPU (NCCL)

Workload (the reference's headline case, FULL prefill): OneSdmLM FULL arm, d 768, 12 layers, 12 run-time memory
heads x 64, 1,024 slots per head (32 x 32 product keys), k 16, fades (0, .8, .99, 1) x 3, TrainedSdm body at the
reference defaults (4 heads, n_sub 72, k 32, value width 192), tied 32,768-row token table; bf16 weights and
activations, float32 memory state.  Weights: random init of that architecture (seed 0) with the zero-initialised
output maps / value tables perturbed (std 0.02) so no module is a no-op.  Data: synthetic Zipf(1.1) token ids (numpy
default_rng, ids = min(rank-1, 32767)) of shape [32, 2048], batch-sharded 32/N rows per GPU (strong scaling: the
global batch is fixed).  A step = forward of every row + the tied-head cross-entropy sum against the next token
(replayed as one CUDA graph), then an NCCL all-reduce of (loss sum, token count) when N > 1.  Every step's working set
(activations, 0.4 GB per layer at 32 rows) is larger than the 126 MB L2, so no L2 flush is added.

The JSON line adds: e2e (the same step through the public API from pinned host ids, H2D + D2H inside the timed
region); roofline of the dominant kernel and roofline_by_call_site / roofline_by_kernel (measured live with CUDA events
around every launch of a profiled pass of the same K steps on one row stream, right after the timed region);
weak (N > 1: 32 rows per GPU); decode (256 streams sharded over the GPUs, 2,048-token prompts, 512 carried-state greedy
steps, with its HBM roofline); partial (N = 1: the PARTIAL arm, [8, 2048], forward + tied logits); scaled (the scaled
FULL arm d1536 L24, 64 rows x 16,384 tokens sharded over the GPUs, and the same at 2,048 tokens for the per-token
flatness); cpu_baseline (the CPU oracle port of the reference algorithm, 1 row x 2,048 tokens, rank 0 at N = 1);
clocks sampled during the timed region.
"""
import argparse
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

V, D, LAYERS, HEADS, T_SEQ, GLOBAL_ROWS = 32768, 768, 12, 12, 2048, 32
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC = "tokens/sec FULL d768 L12 T2048 prefill (forward + tied-head CE sum)"
ROW_STREAMS = 2  # rows split over two CUDA streams in the timed steps (OneSdmLM.loss_sum row_streams)
REF_TOKENS = 512  # tokens of one reference-arm step (1 row; four 128-token chunks, so the state carries across)
CPU_TOKENS = 2048  # the CPU baseline's sample: 1 row at the full window


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--global-rows", type=int, default=GLOBAL_ROWS, help="rows of T_SEQ tokens over all GPUs")
    ap.add_argument("--seq", type=int, default=T_SEQ)
    ap.add_argument("--layers", type=int, default=LAYERS)
    ap.add_argument("--decode-streams", type=int, default=256, help="decode streams over all GPUs")
    ap.add_argument("--decode-steps", type=int, default=512)
    ap.add_argument("--decode-prompt", type=int, default=T_SEQ)
    ap.add_argument("--scaled-rows", type=int, default=64, help="scaled FULL rows over all GPUs")
    ap.add_argument("--scaled-seq", type=int, default=16384)
    ap.add_argument("--scaled-steps", type=int, default=3)
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-partial", action="store_true")
    ap.add_argument("--no-scaled", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="timed steps launched eagerly instead of a CUDA graph")
    ap.add_argument("--row-streams", type=int, default=ROW_STREAMS, help="CUDA streams the rows are split over")
    return ap.parse_args(argv)


def zipf_ids(seed, rows, T):
    rng = np.random.default_rng(seed)
    return np.minimum(rng.zipf(1.1, size=(rows, T)) - 1, V - 1).astype(np.int64)


def model_cfg(layers, d=D, heads=HEADS, mlp_f=2048):
    return dict(d=d, layers=layers, mlp_f=mlp_f, heads=heads, n_sub=32, d_a=32, k=16,
                decays=(0.0, 0.8, 0.99, 1.0) * (heads // 4))


def workload(layers, rows_total, T):
    return (f"FULL onesdm_allsdm d768 L{layers} h12x64 M1024 k16, TrainedSdm n_sub72 k32, V32768, "
            f"{rows_total} rows x {T} tokens (batch-sharded over the GPUs)")


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            js = json.load(f)
        return {k: float(js[k]) for k in FALLBACK_PEAKS}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ------------------------------------------------------------------------------------------- reference (CPU)
def oracle_params(layers, seed=0):
    """The benchmark model's weights (same seed and perturbation as the GPU arm) as oracle parameter objects."""
    import torch
    import sdmchat_b200 as S
    from oracle import sdm_oracle as O
    torch.manual_seed(seed)
    model = S.build_onesdm("onesdm_allsdm", V, model_cfg(layers))
    perturb(model)
    sd = {k: v.to(torch.bfloat16).float().numpy() if v.dim() >= 1 and not k.endswith(
        ("keys1", "keys2", "addr_b", "log_scale", "onorm_w", "wg.bias", "decays_fixed")) else v.float().numpy()
          for k, v in model.state_dict().items()}
    P = {"emb": sd["emb.weight"], "nf_w": sd["nf.w"], "layers": []}
    for i in range(layers):
        msd = {k[len(f"mems.{i}."):]: v for k, v in sd.items() if k.startswith(f"mems.{i}.")}
        ssd = {k[len(f"sdms.{i}."):]: v for k, v in sd.items() if k.startswith(f"sdms.{i}.")}
        P["layers"].append({"mem": O.RunTimeSdmParams(msd, HEADS, 32, 32, 16),
                            "sdm": O.TrainedSdmParams(ssd, 4, model.sdm_n_sub, model.sdm_d_a, 32)})
    return P


def cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        return max([i.get("num_threads", 1) for i in threadpool_info()] + [1])
    except Exception:
        return os.cpu_count() or 1


def oracle_step(P, ids):
    """One CPU step: the oracle forward + CE sum over ids (1, n + 1)."""
    from oracle import sdm_oracle as O
    lg = O.lm_forward(P, ids[:, :-1], bf16_stream=True, margins=False)
    return O.ce_sum(lg, ids[:, 1:])


def time_oracle(P, tokens):
    """Wall time of the oracle forward + CE sum on one row of `tokens` ids after a short warm run (cost_bench's
    method, track4_onesdm_puzzles.py:342-377, with one rep: the sample is 10-30 s of CPU work)."""
    ids = zipf_ids(99, 1, tokens + 1)
    oracle_step(P, ids[:, :17])  # warm
    t0 = time.perf_counter()
    oracle_step(P, ids)
    return tokens / (time.perf_counter() - t0)


def all_host_threads():
    """Let the CPU baseline's BLAS use every host core (torchrun sets OMP_NUM_THREADS=1 for its workers)."""
    try:
        from threadpoolctl import threadpool_limits
        return threadpool_limits(limits=os.cpu_count() or 1)
    except Exception:
        return None


def port_vs_reference():
    """The port's CPU speed against the unmodified reference module's torch CPU forward, both timed on one host
    (oracle/time_port_vs_reference.py writes the figures; the reference itself cannot run on the GPU box)."""
    p = os.path.join(ROOT, "oracle", "port_vs_reference.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        r = json.load(f)
    return {"reference_torch_cpu_tok_s": r["reference_torch_cpu_tok_s"], "port_tok_s": r["port_numpy_tok_s"],
            "port_over_reference": r["port_over_reference"], "host_threads": r["host_threads"],
            "sample": f"1 row x {r['tokens']} tokens, FULL d768 L12, both on the build host", "source": r["script"]}


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    _limits = all_host_threads()  # noqa: F841 (kept alive for the whole run)
    P = oracle_params(a.layers)
    ids = zipf_ids(99, 1, REF_TOKENS + 1)
    for _ in range(a.warmup):
        oracle_step(P, ids[:, :65])  # warm-up steps on a 64-token sample: the timed steps carry the full sample
    t0 = time.perf_counter()
    for _ in range(a.steps):
        oracle_step(P, ids)
    dt = time.perf_counter() - t0
    val = REF_TOKENS * a.steps / dt
    cores = cpu_threads()
    sample = (f"1 row x {REF_TOKENS} tokens per step (four 128-token chunks, state carried between them) of the "
              f"FULL d768 L{a.layers} forward + tied-head CE sum; numpy float32 port of the reference algorithm")
    out = {"metric": METRIC, "impl": "reference", "value": round(val, 3), "unit": "tokens/s", "n_gpus": a.gpus,
           "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(1e3 * dt / a.steps, 3),
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic Zipf(1.1) token ids; random-init weights (seed 0, output maps perturbed)",
           "config": {"workload": workload(a.layers, a.global_rows, a.seq), "global_batch": a.global_rows,
                      "seq_len": a.seq, "parallelism": "host CPU"},
           "cpu_baseline": {"value": round(val, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
                            "sample": sample, "port_vs_reference": port_vs_reference()},
           "e2e": {"value": round(val, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


# ------------------------------------------------------------------------------------------------- ours (GPU)
def perturb(model):
    import torch
    with torch.no_grad():
        for m in model.mems:
            torch.nn.init.normal_(m.wo.weight, std=0.02)
            torch.nn.init.normal_(m.wg.weight, std=0.5 / m.d ** 0.5)
        for s in getattr(model, "sdms", []):
            torch.nn.init.normal_(s.values, std=0.02)


class Clocks:
    """nvidia-smi samples of this GPU's clocks and throttle reasons while the timed region runs."""
    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, dev_index):
        self.proc = None
        self.lines = []
        try:
            import torch
            uuid = "GPU-" + str(torch.cuda.get_device_properties(dev_index).uuid)
            self.cmd = ["nvidia-smi", "-i", uuid, f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                        "-lms", "100"]
        except Exception:
            self.cmd = ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "100"]

    def start(self):
        try:
            self.proc = subprocess.Popen(self.cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=lambda: self.lines.extend(self.proc.stdout), daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx.append(float(f[1]))
            except ValueError:
                continue
            for n, v in zip(names, f[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def gemm_flops_per_row(tag, d=D, heads=HEADS, mlp_f=2048, vocab=V):
    """Algorithmic FLOPs per row of one tensor-core GEMM launch, by call site (2 * K * N of the reference's matmul;
    the float32-accurate hi/lo split of the wo inputs is not counted)."""
    C = 2 * heads * 32 + d + heads  # [wk; wq; wv; wg] columns: 1,548 at d 768
    return {"rt_proj": 2 * d * C, "rt_out": 2 * d * d, "ts_q": 2 * d * (4 * 32), "ts_wo": 2 * d * d,
            "swiglu_gu": 2 * d * 2 * mlp_f, "swiglu_down": 2 * mlp_f * d,
            "head_ce": 2 * d * vocab, "head_logits": 2 * d * vocab, "head_argmax": 2 * d * vocab,
            "head_project": 2 * d * vocab}.get(tag, 0)


def gemm_flops(tag, rows, layers=None):
    """Algorithmic FLOPs of one GEMM launch of `rows` rows at call site `tag` (FULL d768 shapes)."""
    return gemm_flops_per_row(tag) * rows


# DRAM bytes (read + write) per token of one launch, from the ncu captures summarised in
# profiles/{pk_fast_kernel,rt_lists_rt_scan,ts_gather_rt_finish}_lm_d768_L12_B4_T2048.md (8,192 tokens, layer 6),
# scaled by tokens: the bench's 65,536-token launches are too large to capture with every metric.
NCU_DRAM_PER_TOKEN = {
    ("pk_address", "rt_address"): (26652160 + 49920) / 8192,
    ("pk_address", "ts"): 4578816 / 8192,
    ("rt_lists", ""): (51309056 + 4100608) / 8192,
    ("rt_scan", ""): (64075264 + 2735616) / 8192,
    ("ts_gather", "ts"): 15511808 / 8192,
    ("rt_finish", "rt_out"): (25603840 + 92160) / 8192,
    # tensor-core GEMMs, from a one-pass capture of one full bench step (65,536 rows per launch), averaged over the
    # 12 layers of each call site (profiles/gemm_tc_dram_full_prefill_d768_L12_B32_T2048.md); the TrainedSdm
    # figure covers its query and wo launches together, half each
    ("gemm_tc", "rt_proj"): 6893.9,
    ("gemm_tc", "rt_out"): 5772.4,
    ("gemm_tc", "ts_q"): 3687.0 / 2,
    ("gemm_tc", "ts_wo"): 3687.0 / 2,
    ("gemm_tc", "head_ce"): 4475.6,
}


# Algorithmic HBM bytes of the SDM scan per (token, head), the per-unit figure of the reference's chunked form
# (chunk L = 128, M = 1024 slots, dh = 64, k = 16): the state in and out once per chunk 2*M*(dh+1)*4/L = 4,160,
# slot ids + weights of the writes and reads 2k*(4+4) = 256, the bf16 value row 2*dh = 128, num/den
# 4*(dh+1) = 260.  This design keeps the state on chip, so its own traffic is far below this figure.
SCAN_BYTES_PER_TOKEN_HEAD = 2 * 1024 * 65 * 4 // 128 + 2 * 16 * 8 + 2 * 64 + 4 * 65
# Decode: per stream-step and (layer, head) the k rows of (dh + 1) floats read, and k rows read-modified-written:
# k (dh + 1) 4 = 4,160 B + 8,320 B = 12,480 B (the lazy decay keeps the rest of the state untouched).
DECODE_STATE_BYTES_PER_HEAD = 16 * 65 * 4 * 3


def kernel_bytes(kernel, tag, tokens):
    """Algorithmic HBM bytes of one launch of a memory-bound kernel of the step: its inputs read once and its
    outputs written once, per (token, head) of the call site (k slot ids + weights are 8 B per pair)."""
    dh, k, ts_h, ts_dh, ts_k = D // HEADS, 16, 4, D // 4, 32
    per = {
        # product-key addressing: z (d_a float32) [+ gate] in, k (id, weight) pairs out; one RunTimeSdm launch
        # covers the write keys (gated) and the read queries
        ("pk_address", "rt_address"): HEADS * (2 * (32 * 4 + k * 8) + 4),
        ("pk_address", "ts"): ts_h * (32 * 4 + ts_k * 8),
        # chunk lists + intra reads: write/read selections and the value row in; num, den and the chunk record out
        ("rt_lists", ""): HEADS * (4 * k * 4 + dh * 4 + dh * 4 + 4 + 2 * k * 8),
        # state scan: read selections, value row, intra num/den and the chunk record in; num, den out
        ("rt_scan", ""): HEADS * (2 * k * 4 + dh * 4 + dh * 4 + 4 + 2 * k * 8 + dh * 4 + 4),
        # TrainedSdm gather: k (id, weight) pairs in, the bf16 hi/lo read out (the value table is L2-resident)
        ("ts_gather", "ts"): ts_h * (ts_k * 8 + ts_dh * 4),
        # finish: num, den in; bf16 hi/lo read out
        ("rt_finish", "rt_out"): HEADS * (dh * 4 + 4) + D * 4,
        # RMSNorm of the bf16 stream (per layer, and the final norm before the tied head): the row in, the row out
        ("rmsnorm", ""): D * 2 * 2,
        ("rmsnorm", "head_ce"): D * 2 * 2,
        ("rmsnorm", "swiglu"): D * 2 * 2,
        ("rmsnorm", "head_logits"): D * 2 * 2,
        # embedding: the id in, the table row in, the stream row out
        ("embed", ""): 4 + D * 2 * 2,
        # CE combine: the head's (max, sum) partial per 128 columns, the target logit and the target in
        ("ce_combine", "head_ce"): (V // 128) * 8 + 4 + 4,
    }
    return per.get((kernel, tag), 0) * tokens


def roofline_tables(groups, rows_tokens, steps, pk, how, flops_per_row=gemm_flops_per_row):
    """From the profiled pass's (kernel, tag, launches, ms) groups: the dominant kernel's roofline, every kernel
    against its own roof, every GEMM call site against the tensor peak, and the per-kernel breakdown."""
    per_kernel = {}
    for k, tag, n, ms in groups:
        d = per_kernel.setdefault(k, {"launches": 0, "ms": 0.0, "tags": {}})
        d["launches"] += n
        d["ms"] += ms
        d["tags"][tag] = d["tags"].get(tag, 0.0) + ms
    if not per_kernel:
        return None, {}, {}, {}
    tens = pk["bf16_tflops_sustained"]
    dom = max(per_kernel, key=lambda k: per_kernel[k]["ms"])
    nl = per_kernel[dom]["launches"]
    if dom == "gemm_tc":
        flops = sum(flops_per_row(tag) * rows_tokens * n for k, tag, n, ms in groups if k == dom)
        ach = flops / (per_kernel[dom]["ms"] / 1e3) / 1e12
        traffic = None
        if all((k, tag) in NCU_DRAM_PER_TOKEN for k, tag, n, ms in groups if k == dom):
            traffic = round(sum(NCU_DRAM_PER_TOKEN[(k, tag)] * rows_tokens * n
                                for k, tag, n, ms in groups if k == dom) / nl)
        roof = {"kernel": "gemm_tc (tcgen05 bf16 GEMM, all call sites)", "bound": "tensor",
                "achieved": round(ach, 1), "peak": tens, "unit": "TFLOP/s", "frac": round(ach / tens, 4),
                "traffic": traffic, "traffic_unit": "bytes per launch (DRAM read + write)",
                "traffic_source": "ncu dram bytes per row of one-pass full-size captures, scaled to the launch",
                "algorithmic_flops_per_launch": round(flops / nl), "peak_source": f"{how} bf16_tflops_sustained",
                "avg_launch_ms": round(per_kernel[dom]["ms"] / nl, 4)}
    else:
        byts = sum(kernel_bytes(k, tag, rows_tokens) * n for k, tag, n, ms in groups if k == dom)
        ach = byts / (per_kernel[dom]["ms"] / 1e3) / 1e9
        traffic = None
        if all((k, tag) in NCU_DRAM_PER_TOKEN for k, tag, n, ms in groups if k == dom):
            traffic = round(sum(NCU_DRAM_PER_TOKEN[(k, tag)] * rows_tokens * n
                                for k, tag, n, ms in groups if k == dom) / nl)
        roof = {"kernel": dom, "bound": "hbm", "achieved": round(ach, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": round(ach / pk["hbm_gbs"], 4), "traffic": traffic,
                "traffic_source": "ncu dram bytes per token of a 8,192-token capture, scaled to the launch",
                "algorithmic_bytes_per_launch": round(byts / nl), "peak_source": f"{how} hbm_gbs",
                "avg_launch_ms": round(per_kernel[dom]["ms"] / nl, 4)}
    by_kernel, by_site = {}, {}
    for k, v in per_kernel.items():
        if k == "gemm_tc":
            fl = sum(flops_per_row(tag) * rows_tokens * n for kk, tag, n, ms in groups if kk == k)
            ach = fl / (v["ms"] / 1e3) / 1e12
            by_kernel[k] = {"bound": "tensor", "achieved": round(ach, 1), "unit": "TFLOP/s",
                            "frac": round(ach / tens, 4)}
            for kk, tag, n, ms in groups:
                if kk == k and ms > 0:
                    f = flops_per_row(tag) * rows_tokens * n / (ms / 1e3) / 1e12
                    by_site[tag] = {"ms_per_step": round(ms / steps, 3), "launches_per_step": n / steps,
                                    "achieved": round(f, 1), "unit": "TFLOP/s", "frac": round(f / tens, 4)}
        else:
            byts = sum(kernel_bytes(k, tag, rows_tokens) * n for kk, tag, n, ms in groups if kk == k)
            if byts:
                ach = byts / (v["ms"] / 1e3) / 1e9
                by_kernel[k] = {"bound": "hbm", "achieved": round(ach, 1), "unit": "GB/s",
                                "frac": round(ach / pk["hbm_gbs"], 4)}
    breakdown = {k: {"ms_per_step": round(v["ms"] / steps, 3), "launches_per_step": v["launches"] / steps,
                     "by_call_site_ms": {t: round(ms / steps, 3) for t, ms in v["tags"].items()}}
                 for k, v in sorted(per_kernel.items(), key=lambda kv: -kv[1]["ms"])}
    return roof, by_kernel, by_site, breakdown


def scan_roofline(groups, token_heads, pk):
    """The SDM scan (rt_lists + rt_scan) at the reference chunked form's bytes per (token, head)."""
    ms = sum(m for k, tag, n, m in groups if k in ("rt_lists", "rt_scan"))
    if ms <= 0:
        return None
    alg = token_heads * SCAN_BYTES_PER_TOKEN_HEAD
    ach = alg / (ms / 1e3) / 1e9
    own = token_heads * (kernel_bytes("rt_lists", "", 1) + kernel_bytes("rt_scan", "", 1)) / HEADS
    dram = token_heads * (NCU_DRAM_PER_TOKEN[("rt_lists", "")] + NCU_DRAM_PER_TOKEN[("rt_scan", "")]) / HEADS
    return {"kernels": "rt_lists + rt_scan", "bound": "hbm", "achieved": round(ach, 1), "unit": "GB/s",
            "peak": pk["hbm_gbs"], "frac": round(ach / pk["hbm_gbs"], 4),
            "algorithmic_bytes_per_token_head": SCAN_BYTES_PER_TOKEN_HEAD,
            "algorithmic_basis": "the reference's chunked scan (L=128): state in + out per chunk "
                                 "2*M*(dh+1)*4/L + ids/weights 2k*8 + V 2*dh + num/den 4*(dh+1)",
            "own_bytes_per_token_head": round(own / token_heads, 1),
            "own_frac": round(own / (ms / 1e3) / 1e9 / pk["hbm_gbs"], 4),
            "traffic_per_token_head": round(dram / token_heads, 1), "ms": round(ms, 3)}


def param_bytes(model):
    return sum(p.numel() * p.element_size() for p in model.parameters())


def run_ours(a):
    import torch
    import sdmchat_b200 as S
    from sdmchat_b200 import _lib
    from sdmchat_b200 import dist as D_

    rank, world = D_.env_world()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        D_.init("nccl", timeout_s=300, device=dev)
    lib = _lib.lib()
    pk, how = peaks()

    torch.manual_seed(0)
    model = S.build_onesdm("onesdm_allsdm", V, model_cfg(a.layers))
    perturb(model)
    model = model.to_bf16_stream().to(dev)
    r0, r1 = D_.shard_rows(a.global_rows, rank, world)
    B, T = r1 - r0, a.seq
    ids_np = zipf_ids(1000, a.global_rows, T + 1)[r0:r1]  # the global batch, this rank's rows
    ids_host = torch.from_numpy(ids_np[:, :-1].astype(np.int32)).pin_memory()
    tgt_host = torch.from_numpy(ids_np[:, 1:].astype(np.int32)).pin_memory()
    ids = ids_host.to(dev)
    tgt = tgt_host.to(dev)
    loss_buf = torch.zeros(2, dtype=torch.float64, device=dev)  # (loss sum, token count)
    st = torch.cuda.current_stream()

    def sync():
        D_.barrier()
        torch.cuda.synchronize()

    def events():
        return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    # the step: forward + CE sum of this rank's rows (one CUDA graph replay), then the (loss, count) all-reduce
    n0 = lib.sdm_kernel_launch_count()
    graph_step = None if a.no_graph else model.loss_graph(B, T, row_streams=a.row_streams)
    launches_per_step = None
    if graph_step is not None:  # launches recorded into the graph: two warm-up passes and the capture
        launches_per_step = (lib.sdm_kernel_launch_count() - n0) // 3

    def step(idx, tg):
        if graph_step is not None:
            loss = graph_step(idx, tg)
            loss_buf[0].copy_(loss[0])
        else:
            if not idx.is_cuda:  # host ids (the e2e pass): copied in as the graph step does
                ids.copy_(idx, non_blocking=True)
                tgt.copy_(tg, non_blocking=True)
                idx, tg = ids, tgt
            loss_buf.zero_()
            with torch.no_grad():
                model.loss_sum(idx, tg, out=loss_buf[:1], row_streams=a.row_streams)
        loss_buf[1] = float(B * T)
        D_.all_reduce_(loss_buf)
        return loss_buf

    for _ in range(a.warmup):
        step(ids, tgt)
    sync()
    clocks = Clocks(local)
    clocks.start()
    e0, e1 = events()
    n0 = lib.sdm_kernel_launch_count()
    e0.record(st)
    for _ in range(a.steps):
        step(ids, tgt)
    e1.record(st)
    torch.cuda.synchronize()
    launches = (launches_per_step * a.steps) if graph_step is not None else lib.sdm_kernel_launch_count() - n0
    sync()
    clk = clocks.stop()
    t_dev = D_.max_over_ranks(e0.elapsed_time(e1) / 1e3, dev)
    loss_mean = float(loss_buf[0].item() / loss_buf[1].item())
    tokens = a.global_rows * T * a.steps
    value = tokens / t_dev

    # e2e: the same graph step through the public API from pinned host ids, the loss read back every step
    host_loss = torch.zeros(2, dtype=torch.float64).pin_memory()
    for _ in range(2):
        host_loss.copy_(step(ids_host, tgt_host), non_blocking=True)
    sync()
    e2, e3 = events()
    e2.record(st)
    for _ in range(a.steps):
        host_loss.copy_(step(ids_host, tgt_host), non_blocking=True)
    e3.record(st)
    torch.cuda.synchronize()
    sync()
    t_e2e = D_.max_over_ranks(e2.elapsed_time(e3) / 1e3, dev)
    e2e = {"value": round(tokens / t_e2e, 1), "unit": "tokens/s",
           "h2d_bytes_per_step": int(ids_host.numel() * 4 + tgt_host.numel() * 4), "d2h_bytes_per_step": 16,
           "api": "OneSdmLM.loss_graph step (pinned host ids/targets in, loss sum out)"}

    # per-kernel CUDA events around every launch, in an eager pass of the same K steps on one row stream (events
    # inside the graph or across two streams would overlap and share their time)
    lib.sdm_profile_begin()
    for _ in range(a.steps):
        loss_buf.zero_()
        with torch.no_grad():
            model.loss_sum(ids, tgt, out=loss_buf[:1], row_streams=1)
    torch.cuda.synchronize()
    groups = _lib.profile_groups()
    sync()
    rows_tokens = B * T
    roof, by_kernel, by_site, breakdown = roofline_tables(groups, rows_tokens, a.steps, pk, how)
    roof_scan = scan_roofline(groups, rows_tokens * HEADS * a.layers * a.steps, pk)
    if roof_scan:
        roof_scan["ms_per_step"] = round(roof_scan.pop("ms") / a.steps, 3)
    del graph_step
    torch.cuda.synchronize()

    # weak scaling beside the strong headline (N > 1): the full 32 rows on every GPU
    weak = None
    if world > 1:
        wB = a.global_rows
        w_ids = torch.from_numpy(zipf_ids(3000 + rank, wB, T + 1)).to(dev)
        wstep = model.loss_graph(wB, T, row_streams=a.row_streams)
        for _ in range(a.warmup):
            wstep(w_ids[:, :-1], w_ids[:, 1:])
        sync()
        e4, e5 = events()
        e4.record(st)
        for _ in range(a.steps):
            wl = wstep(w_ids[:, :-1], w_ids[:, 1:])
            loss_buf[0].copy_(wl[0])
            D_.all_reduce_(loss_buf)
        e5.record(st)
        torch.cuda.synchronize()
        sync()
        t_w = D_.max_over_ranks(e4.elapsed_time(e5) / 1e3, dev)
        weak = {"value": round(world * wB * T * a.steps / t_w, 1), "unit": "tokens/s", "rows_per_gpu": wB,
                "ms_per_step": round(1e3 * t_w / a.steps, 3), "scaling": "weak"}
        del wstep, w_ids
        torch.cuda.synchronize()

    decode = run_decode(a, model, rank, world, dev, pk, how, D_) if not a.no_decode else None
    partial = run_partial(a, rank, world, dev, pk, how) if (not a.no_partial and world == 1) else None
    del model
    torch.cuda.empty_cache()
    scaled = run_scaled(a, rank, world, dev, D_) if not a.no_scaled else None

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        _limits = all_host_threads()  # noqa: F841
        P = oracle_params(a.layers)
        v = time_oracle(P, CPU_TOKENS)
        cpu = {"value": round(v, 2), "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
               "sample": f"1 row x {CPU_TOKENS} tokens (sixteen 128-token chunks) of the same FULL d768 "
                         f"L{a.layers} model, forward + tied-head CE sum, numpy float32 port of the reference "
                         "algorithm (one run after a 16-token warm run)",
               "port_vs_reference": port_vs_reference()}

    if rank == 0:
        out = {"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": a.steps,
               "warmup": a.warmup, "ms_per_step": round(1e3 * t_dev / a.steps, 3), "higher_is_better": True,
               "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
               "data": "synthetic Zipf(1.1) token ids; random-init weights (seed 0, output maps perturbed)",
               "config": {"workload": workload(a.layers, a.global_rows, T), "global_batch": a.global_rows,
                          "seq_len": T, "rows_per_gpu": B, "parallelism": f"dp{world} (batch shards)",
                          "row_streams": a.row_streams, "cuda_graph": not a.no_graph,
                          "l2": "per-step working set > 126 MB L2 (no flush)"},
               "e2e": e2e, "gpu_launches": int(launches), "roofline": roof, "roofline_scan": roof_scan,
               "roofline_by_call_site": by_site, "roofline_by_kernel": by_kernel, "cpu_baseline": cpu,
               "profiled_pass": f"{a.steps} steps eager, one row stream, CUDA events around every launch",
               "clocks": clk, "weak": weak, "decode": decode, "partial": partial, "scaled": scaled,
               "loss_mean": round(loss_mean, 5), "kernels": breakdown}
        print(json.dumps(out), flush=True)
    D_.finalize()


def run_decode(a, model, rank, world, dev, pk, how, D_):
    """Config 4: the global streams sharded over the GPUs, each prefilled with a prompt, then carried-state greedy
    steps replayed as one CUDA graph per step.  Roofline: per stream-step the state rows the lazy-decay step must
    move (k rows of dh + 1 floats read, k read-modified-written, per layer-head) plus every weight once per step."""
    import torch
    s0, s1 = D_.shard_rows(a.decode_streams, rank, world)
    Sd = s1 - s0
    prompt = torch.from_numpy(zipf_ids(2000, a.decode_streams, a.decode_prompt)[s0:s1]).to(dev)
    st = torch.cuda.current_stream()
    with torch.no_grad():
        state = model.init_decode(Sd, dev)
        nxt = torch.empty(Sd, dtype=torch.int32, device=dev)
        group = 32  # prompts prefilled 32 streams at a time (bounded workspace), each into its slice of the state
        for g0 in range(0, Sd, group):
            g1 = min(Sd, g0 + group)
            sub = [{k: v[g0:g1] for k, v in s.items()} for s in state]  # views: prefill writes into the state
            nxt[g0:g1] = model.prefill(prompt[g0:g1], sub)
        step_fn = model.decode_graph(state)
        for _ in range(3):
            nxt = step_fn(nxt)
        D_.barrier()
        torch.cuda.synchronize()
        e4, e5 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e4.record(st)
        for _ in range(a.decode_steps):
            nxt = step_fn(nxt)
        e5.record(st)
        torch.cuda.synchronize()
    D_.barrier()
    t_dec = D_.max_over_ranks(e4.elapsed_time(e5) / 1e3, dev)
    ms_step = 1e3 * t_dec / a.decode_steps
    wbytes = param_bytes(model)
    m = model.mems[0]
    state_bytes = Sd * model.n_layers * m.h * DECODE_STATE_BYTES_PER_HEAD
    step_bytes = state_bytes + wbytes
    ach = step_bytes / (ms_step / 1e3) / 1e9
    del step_fn, state
    torch.cuda.synchronize()
    return {"value": round(a.decode_streams * a.decode_steps / t_dec, 1), "unit": "tokens/s",
            "streams_total": a.decode_streams, "streams_per_gpu": Sd, "prompt": a.decode_prompt,
            "steps": a.decode_steps, "ms_per_step": round(ms_step, 4), "cuda_graph": True,
            "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(ach / pk["hbm_gbs"], 4), "bytes_per_gpu_step": int(step_bytes),
                         "basis": f"{Sd} streams x 1.80 MB of state rows (12 layers x 12 heads x 12,480 B) + "
                                  f"{wbytes / 1e6:.1f} MB of bf16 weights, per GPU-step",
                         "peak_source": f"{how} hbm_gbs"}}


def run_partial(a, rank, world, dev, pk, how):
    """Config 2: the PARTIAL arm (onesdm: RunTimeSdm then SwiGLU(RMSNorm) per layer, f 2048), ids [8, 2048],
    prefill forward + the tied logits (materialised, bf16), on one GPU, with its GEMM roofline."""
    import torch
    import sdmchat_b200 as S
    from sdmchat_b200 import _lib
    lib = _lib.lib()
    torch.manual_seed(0)
    model = S.build_onesdm("onesdm", V, model_cfg(a.layers))
    perturb(model)
    model = model.to_bf16_stream().to(dev)
    Bp, T = 8, a.seq
    ids = torch.from_numpy(zipf_ids(4000, Bp, T)).to(dev)
    st = torch.cuda.current_stream()
    with torch.no_grad():
        for _ in range(a.warmup):
            lg = model(ids)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(a.steps):
            lg = model(ids)
        e1.record(st)
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / 1e3
        lib.sdm_profile_begin()
        for _ in range(a.steps):
            lg = model(ids)
        torch.cuda.synchronize()
        groups = _lib.profile_groups()
    del lg
    rows = Bp * T
    gemm_ms = sum(ms for k, tag, n, ms in groups if k == "gemm_tc")
    gemm_fl = sum(gemm_flops_per_row(tag) * rows * n for k, tag, n, ms in groups if k == "gemm_tc")
    alg_per_token = (a.layers * (gemm_flops_per_row("rt_proj") + gemm_flops_per_row("rt_out")
                                 + gemm_flops_per_row("swiglu_gu") + gemm_flops_per_row("swiglu_down"))
                     + gemm_flops_per_row("head_logits"))
    tens = pk["bf16_tflops_sustained"]
    roof, by_kernel, by_site, breakdown = roofline_tables(groups, rows, a.steps, pk, how)
    gemm = {"bound": "tensor", "achieved": round(gemm_fl / (gemm_ms / 1e3) / 1e12, 1) if gemm_ms else None,
            "peak": tens, "unit": "TFLOP/s",
            "frac": round(gemm_fl / (gemm_ms / 1e3) / 1e12 / tens, 4) if gemm_ms else None,
            "algorithmic_flops_per_token": alg_per_token, "peak_source": f"{how} bf16_tflops_sustained"}
    del model
    torch.cuda.empty_cache()
    return {"value": round(Bp * T * a.steps / t, 1), "unit": "tokens/s", "metric": "tokens/sec PARTIAL d768 L12 "
            "T2048 prefill (forward + tied logits)", "config": {"workload": f"PARTIAL onesdm d768 L{a.layers} h12x64 "
            "M1024 k16, SwiGLU f2048, V32768, 8 rows x 2048 tokens", "global_batch": Bp, "seq_len": T},
            "ms_per_step": round(1e3 * t / a.steps, 3), "steps": a.steps, "roofline_gemm": gemm,
            "roofline_dominant": roof, "roofline_by_call_site": by_site, "roofline_by_kernel": by_kernel,
            "kernels": breakdown}


def run_scaled(a, rank, world, dev, D_):
    """Config 5: the scaled FULL arm (d1536, 24 layers, 24 heads x 64, 1,024 slots, k16, TrainedSdm n_sub 103 at
    mlp_f 4096), 64 Zipf rows x 16,384 tokens sharded over the GPUs, forward + tied CE sum; and the same rows at
    2,048 tokens, so the per-token cost can be compared across window lengths."""
    import torch
    import sdmchat_b200 as S
    torch.manual_seed(0)
    model = S.build_onesdm("onesdm_allsdm", V, model_cfg(24, d=1536, heads=24, mlp_f=4096))
    perturb(model)
    model = model.to_bf16_stream().to(dev)
    r0, r1 = D_.shard_rows(a.scaled_rows, rank, world)
    Bs = r1 - r0
    st = torch.cuda.current_stream()
    res = {"workload": f"scaled FULL onesdm_allsdm d1536 L24 h24x64 M1024 k16, TrainedSdm n_sub{model.sdm_n_sub} "
                       f"k32, V32768, {a.scaled_rows} rows (batch-sharded)", "rows_per_gpu": Bs, "by_seq": {}}
    for T in (2048, a.scaled_seq):
        ids = torch.from_numpy(zipf_ids(5000, a.scaled_rows, T + 1)[r0:r1]).to(dev)
        idx, tgt = ids[:, :-1].contiguous(), ids[:, 1:].contiguous()
        out = torch.zeros(1, dtype=torch.float64, device=dev)
        with torch.no_grad():
            for _ in range(max(1, min(a.warmup, 3))):
                model.loss_sum(idx, tgt, out=out, row_streams=a.row_streams)
            D_.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            for _ in range(a.scaled_steps):
                model.loss_sum(idx, tgt, out=out, row_streams=a.row_streams)
            e1.record(st)
            torch.cuda.synchronize()
        D_.barrier()
        t = D_.max_over_ranks(e0.elapsed_time(e1) / 1e3, dev)
        res["by_seq"][str(T)] = {"value": round(a.scaled_rows * T * a.scaled_steps / t, 1), "unit": "tokens/s",
                                 "ms_per_step": round(1e3 * t / a.scaled_steps, 2), "steps": a.scaled_steps}
        del ids, idx, tgt
        torch.cuda.empty_cache()
    lo, hi = res["by_seq"]["2048"]["value"], res["by_seq"][str(a.scaled_seq)]["value"]
    res["per_token_cost_ratio"] = round(lo / hi, 4)  # cost per token at the long window / at 2,048 tokens
    del model
    torch.cuda.empty_cache()
    return res


def main():
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
