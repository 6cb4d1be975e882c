"""Small, fixed workloads for profiling one kernel at a time (ncu / compute-sanitizer friendly sizes).

    python -m sdmchat_b200.profile_cases scan     # one RunTimeSdm d768 layer forward, 8 x 2048 tokens (bf16)
    python -m sdmchat_b200.profile_cases gemm     # the layer's projection GEMM alone, 16384 x 768 x 1548
    python -m sdmchat_b200.profile_cases pk       # product-key addressing of 16384 tokens x 12 heads
    python -m sdmchat_b200.profile_cases decode   # 32 streams x 12 layers FULL decode steps
    python -m sdmchat_b200.profile_cases lm       # FULL d768 L12 forward + CE sum, 4 x 2048 Zipf(1.1) tokens
    python -m sdmchat_b200.profile_cases scaled   # scaled FULL d1536 L24 forward + CE sum at T = 2K / 8K / 16K

Each case runs its workload once untimed and then `--reps` times (default 2), and prints one line of CUDA-event
timings; nothing else runs on the GPU, so `ncu -k regex:<kernel> -c N` captures exactly the launches of interest.
"""
import argparse
import json

import torch

import sdmchat_b200 as S
from sdmchat_b200 import _lib


def _layer(dev):
    torch.manual_seed(0)
    m = S.RunTimeSdm(768, heads=12, n_sub=32, d_a=32, k=16, decays=S.readme_fades(12))
    with torch.no_grad():
        torch.nn.init.normal_(m.wo.weight, std=0.02)
        torch.nn.init.normal_(m.wg.weight, std=0.5 / 768 ** 0.5)
    return m.to(dev).to(torch.bfloat16)


def _full_model(dev):
    """The benchmark's FULL d768 L12 model: seed-0 init with the zero-initialised output maps perturbed."""
    torch.manual_seed(0)
    model = S.build_onesdm("onesdm_allsdm", 32768, dict(d=768, layers=12, mlp_f=2048, heads=12,
                                                         decays=S.readme_fades(12)))
    with torch.no_grad():
        for m in model.mems:
            torch.nn.init.normal_(m.wo.weight, std=0.02)
            torch.nn.init.normal_(m.wg.weight, std=0.5 / 768 ** 0.5)
        for s in model.sdms:
            torch.nn.init.normal_(s.values, std=0.02)
    return model.to_bf16_stream().to(dev)


def _scaled_model(dev):
    """Scaled FULL (d1536, 24 layers, 24 heads x 64, 1,024 slots, k16; TrainedSdm 4 heads, n_sub 103, dh 384, k32;
    tied 32,768-row table): seed-0 init with the zero-initialised output maps perturbed."""
    torch.manual_seed(0)
    model = S.build_onesdm("onesdm_allsdm", 32768, dict(d=1536, layers=24, mlp_f=4096, heads=24,
                                                         decays=S.readme_fades(24)))
    with torch.no_grad():
        for m in model.mems:
            torch.nn.init.normal_(m.wo.weight, std=0.02)
            torch.nn.init.normal_(m.wg.weight, std=0.5 / 1536 ** 0.5)
        for s in model.sdms:
            torch.nn.init.normal_(s.values, std=0.02)
    return model.to_bf16_stream().to(dev)


def _timed(fn, reps):
    fn()  # first call: module load and attribute setup stay out of the timing
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for _ in range(reps):
        fn()
    b.record(st)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["scan", "gemm", "pk", "decode", "lm", "scaled"])
    ap.add_argument("--reps", type=int, default=2)
    ap.add_argument("--rows", type=int, default=4, help="scaled: batch rows per window length")
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    with torch.no_grad():
        if a.case == "scan":
            m = _layer(dev)
            x = (torch.randn(8, 2048, 768, device=dev, generator=g) * 0.02).to(torch.bfloat16)
            ms = _timed(lambda: m(x), a.reps)
            out = {"case": "scan", "tokens": 8 * 2048, "ms_per_layer_forward": ms}
        elif a.case == "gemm":
            x = torch.randn(16384, 768, device=dev, generator=g).to(torch.bfloat16)
            w = torch.randn(1548, 768, device=dev, generator=g).to(torch.bfloat16)
            y = torch.empty(16384, 1548, device=dev)
            lib = _lib.lib()

            def run():
                _lib.check(lib.sdm_gemm(_lib.ptr(x), _lib.ptr(w), 16384, 768, 1548, _lib.SDM_BF16, _lib.ptr(y),
                                        _lib.stream_ptr(dev)), "sdm_gemm")
            ms = _timed(run, a.reps)
            out = {"case": "gemm", "shape": [16384, 768, 1548], "ms": ms,
                   "tflops": 2 * 16384 * 768 * 1548 / (ms / 1e3) / 1e12}
        elif a.case == "pk":
            z = torch.randn(16384, 12, 32, device=dev, generator=g)
            k1 = torch.randn(12, 32, 16, device=dev, generator=g)
            k2 = torch.randn(12, 32, 16, device=dev, generator=g)
            ms = _timed(lambda: S.pk_address(z, k1, k2, 16), a.reps)
            out = {"case": "pk", "addresses": 16384 * 12, "ms": ms}
        elif a.case == "lm":
            import numpy as np
            model = _full_model(dev)
            rng = np.random.default_rng(1000)
            ids_np = np.minimum(rng.zipf(1.1, size=(4, 2049)) - 1, 32767)
            ids = torch.from_numpy(ids_np[:, :-1].astype(np.int32)).to(dev)
            tgt = torch.from_numpy(ids_np[:, 1:].astype(np.int32)).to(dev)
            ms = _timed(lambda: model.loss_sum(ids, tgt), a.reps)
            out = {"case": "lm", "tokens": 4 * 2048, "ms_per_forward": ms, "tok_per_s": 8192 / (ms / 1e3)}
        elif a.case == "scaled":
            import numpy as np
            model = _scaled_model(dev)
            rng = np.random.default_rng(1001)
            per_t = {}
            for T in (2048, 8192, 16384):
                ids_np = np.minimum(rng.zipf(1.1, size=(a.rows, T + 1)) - 1, 32767)
                ids = torch.from_numpy(ids_np[:, :-1].astype(np.int32)).to(dev)
                tgt = torch.from_numpy(ids_np[:, 1:].astype(np.int32)).to(dev)
                ms = _timed(lambda: model.loss_sum(ids, tgt), a.reps)
                per_t[T] = {"ms_per_forward": round(ms, 3), "tok_per_s": round(a.rows * T / (ms / 1e3), 1)}
            out = {"case": "scaled", "model": "FULL d1536 L24 h24x64 M1024 k16, TrainedSdm n_sub 103", "rows": a.rows,
                   "by_window": per_t}
        else:
            model = _full_model(dev)
            state = model.init_decode(32, dev)
            ids = torch.randint(0, 32768, (32,), device=dev, generator=g)
            ms = _timed(lambda: model.decode_step(ids, state), a.reps)
            out = {"case": "decode", "streams": 32, "ms_per_step": ms}
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
