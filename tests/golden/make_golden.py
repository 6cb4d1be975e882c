"""Write the golden fixtures of this directory from the UNMODIFIED SDMCHAT reference module.

Run from the repository root, where the reference checkout is readable:
    python tests/golden/make_golden.py --ref PATH_TO_SDMCHAT_CHECKOUT   (or SDMCHAT_REF=PATH in the environment)

It imports experiments/track4/sdmllm/track4_onesdm_models.py (the reference's own RunTimeSdm, TrainedSdm,
pk_address and OneSdmLM) on the CPU in float32, builds seeded modules exactly as the reference's constructors and
self-test do, runs them, and saves inputs, weights and outputs as small .npz files.  The tests read only these
files; nothing at test time (here or on a GPU box) touches the reference checkout.

Cases (reference lines are in track4_onesdm_models.py unless noted):
  pk_selftest     the self-test's brute-force product-key case (:694-702): z (30,2,12), keys (2,9,6), k 5
  pk_k4 / pk_k16  z (256, 4, 32), keys (4, 32, 16): the run-time memory's addressing at k 4 and k 16
  pk_ns72_k32     z (128, 4, 32), keys (4, 72, 16), k 32: the FULL arm's trained-table addressing (n_sub 72)
  rt_config1      the reference's CPU-runnable benchmark case: RunTimeSdm(256, heads 4, n_sub 32, d_a 32, k 4) with Uniform[0.90, 0.999]
                  fades, x (2, 256, 256) N(0,1); prepare outputs, forward, num/den, last_state, forward_sequential
  rt_small_*      the self-test's tiny memory (d 32, 4 heads, n_sub 6, d_a 8, k 5, fades 0/0.7/0.95/1, chunk 7)
                  with perturbed wo/wg (:713-718): plain, reset at BOS, learned fades, sum read without out-norm,
                  no write gate
  rt_prevtok      the fade-0 previous-token known answer (:773-785)
  ts_selftest     TrainedSdm(32, n_sub 12, heads 2, d_a 8, k 7) with N(0,1) values (:855-871)
  lm_partial / lm_full / lm_partial_bos
                  tiny OneSdmLM arms (d 64, 2 layers, 4 heads, n_sub 8, d_a 8, k 4, V 256, chunk 16, T 40) run with a
                  bfloat16 residual stream: token table, every RMSNorm and the SwiGLU in bfloat16; the memory's and
                  the trained table's matrices bfloat16-rounded, kept float32.  Weights perturbed as the self-test does.
"""
import argparse
import os
import sys

import numpy as np
import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(path):
    sys.path.insert(0, os.path.join(path, "experiments", "track4", "sdmllm"))
    import track4_onesdm_models as OM  # noqa: E402
    return OM


def npd(t):
    t = t.detach()
    if t.dtype in (torch.int64, torch.int32, torch.bool):
        return t.to(torch.int32).numpy() if t.dtype != torch.bool else t.numpy()
    return t.float().numpy()


def sd_np(module, prefix=""):
    return {prefix + k: npd(v) for k, v in module.state_dict().items()}


def save(name, **arrs):
    path = os.path.join(HERE, name + ".npz")
    np.savez_compressed(path, **arrs)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


def capture_rt(OM, m, x, reset=None):
    """Run RunTimeSdm.forward and capture prepare outputs and the (num, den) handed to finish."""
    got = {}
    orig_prep, orig_fin = m.prepare, m.finish

    def prep(xx):
        r = orig_prep(xx)
        got["prep"] = r
        return r

    def fin(num, den, B, T, dtype):
        got["num"], got["den"] = num, den
        return orig_fin(num, den, B, T, dtype)
    m.prepare, m.finish = prep, fin
    try:
        out = m(x, reset)
    finally:
        del m.prepare, m.finish
    siw, ww, sir, wr, V = got["prep"]
    mem, cnt = m.last_state
    return dict(out=npd(out), siw=npd(siw), ww=npd(ww), sir=npd(sir), wr=npd(wr), V=npd(V), num=npd(got["num"]),
                den=npd(got["den"]), mem=npd(mem), cnt=npd(cnt), gate=npd(m.last_gate))


def pk_cases(OM):
    torch.manual_seed(0)
    k1, k2 = torch.randn(2, 9, 6), torch.randn(2, 9, 6)
    z = torch.randn(30, 2, 12)
    sv, si = OM.pk_address(z, k1, k2, 5)
    save("pk_selftest", z=npd(z), keys1=npd(k1), keys2=npd(k2), k=5, sv=npd(sv), si=npd(si))
    g = torch.Generator().manual_seed(11)
    keys1, keys2 = torch.randn(4, 32, 16, generator=g), torch.randn(4, 32, 16, generator=g)
    z = torch.randn(256, 4, 32, generator=g)
    for k in (4, 16):
        sv, si = OM.pk_address(z, keys1, keys2, k)
        save(f"pk_k{k}", z=npd(z), keys1=npd(keys1), keys2=npd(keys2), k=k, sv=npd(sv), si=npd(si))
    keys1, keys2 = torch.randn(4, 72, 16, generator=g), torch.randn(4, 72, 16, generator=g)
    z = torch.randn(128, 4, 32, generator=g)
    sv, si = OM.pk_address(z, keys1, keys2, 32)
    save("pk_ns72_k32", z=npd(z), keys1=npd(keys1), keys2=npd(keys2), k=32, sv=npd(sv), si=npd(si))


def rt_config1(OM):
    torch.manual_seed(0)
    decays = torch.empty(4).uniform_(0.90, 0.999)
    m = OM.RunTimeSdm(256, heads=4, n_sub=32, d_a=32, k=4, decays=tuple(decays.tolist()))
    x = torch.randn(2, 256, 256)
    with torch.no_grad():
        r = capture_rt(OM, m, x)
        seq = m.forward_sequential(x)
    save("rt_config1", x=npd(x), seq_out=npd(seq), heads=4, n_sub=32, d_a=32, k=4, chunk=128,
         **{"p." + k: v for k, v in sd_np(m).items()}, **r)


def perturb_rt(m):
    nn.init.normal_(m.wo.weight, std=0.3)
    nn.init.normal_(m.wg.weight, std=0.5)


def rt_small(OM):
    base = dict(heads=4, n_sub=6, d_a=8, k=5, decays=(0.0, 0.7, 0.95, 1.0), chunk=7)
    variants = {
        "plain": {},
        "learned": {"learn_decay": True},
        "sumread": {"read_mode": "sum", "out_norm": False},
        "nogate": {"write_gate": False},
    }
    for tag, extra in variants.items():
        torch.manual_seed(5)
        m = OM.RunTimeSdm(32, **{**base, **extra})
        perturb_rt(m)
        x = torch.randn(2, 23, 32)
        with torch.no_grad():
            r = capture_rt(OM, m, x)
            seq = m.forward_sequential(x)
        save(f"rt_small_{tag}", x=npd(x), seq_out=npd(seq), **{k: v for k, v in base.items() if k != "decays"},
             write_gate=int(m.write_gate), read_mode=m.read_mode, out_norm=int(m.out_norm),
             **{"p." + k: v for k, v in sd_np(m).items()}, **r)
    torch.manual_seed(6)
    m = OM.RunTimeSdm(32, **base)
    perturb_rt(m)
    x = torch.randn(2, 23, 32)
    reset = torch.zeros(2, 23, dtype=torch.bool)
    reset[0, [0, 4, 9, 15]] = True
    reset[1, [7, 8, 21]] = True
    with torch.no_grad():
        r = capture_rt(OM, m, x, reset)
        seq = m.forward_sequential(x, reset)
    save("rt_small_bos", x=npd(x), reset=npd(reset), seq_out=npd(seq),
         **{k: v for k, v in base.items() if k != "decays"}, write_gate=1, read_mode="mean", out_norm=1,
         **{"p." + k: v for k, v in sd_np(m).items()}, **r)


def rt_prevtok(OM):
    torch.manual_seed(7)
    with torch.no_grad():
        r = OM.RunTimeSdm(8, heads=1, n_sub=4, d_a=4, k=4, decays=(0.0,), write_gate=False, out_norm=False, chunk=3)
        nn.init.zeros_(r.wq.weight)
        nn.init.zeros_(r.wk.weight)
        nn.init.eye_(r.wo.weight)
        x = torch.randn(1, 9, 8)
        got = capture_rt(OM, r, x)
    save("rt_prevtok", x=npd(x), heads=1, n_sub=4, d_a=4, k=4, chunk=3, write_gate=0, read_mode="mean", out_norm=0,
         **{"p." + k: v for k, v in sd_np(r).items()}, **got)


def ts_selftest(OM):
    torch.manual_seed(8)
    ts = OM.TrainedSdm(32, n_sub=12, heads=2, d_a=8, k=7)
    with torch.no_grad():
        nn.init.normal_(ts.values, std=1.0)
        xt = torch.randn(3, 11, 32)
        out = ts(xt)
    save("ts_selftest", x=npd(xt), out=npd(out), si=npd(ts.last_si), heads=2, n_sub=12, d_a=8, k=7,
         **{"p." + k: v for k, v in sd_np(ts).items()})


def to_bf16_stream(model):
    """Put a OneSdmLM in the bf16-residual-stream form used by the tiny LM fixtures."""
    model.emb.to(torch.bfloat16)
    model.nf.to(torch.bfloat16)
    for mn in getattr(model, "mnorms", []):
        mn.to(torch.bfloat16)
    for ml in getattr(model, "mlps", []):
        ml.to(torch.bfloat16)
    for m in model.mems:
        m.norm.to(torch.bfloat16)
        for lin in (m.wk, m.wq, m.wv, m.wg, m.wo):
            lin.weight.data = lin.weight.data.bfloat16().float()
    for s in getattr(model, "sdms", []):
        s.norm.to(torch.bfloat16)
        s.wq.weight.data = s.wq.weight.data.bfloat16().float()
        s.wo.weight.data = s.wo.weight.data.bfloat16().float()
        s.values.data = s.values.data.bfloat16().float()


def lm_case(OM, name, arm, reset_at_bos=False):
    V = 256
    cfg = dict(d=64, layers=2, mlp_f=176, heads=4, n_sub=8, d_a=8, k=4, chunk=16, reset_at_bos=reset_at_bos, bos_id=0)
    torch.manual_seed(21)
    model = OM.build_onesdm(arm, V, cfg)
    with torch.no_grad():
        for m in model.mems:
            perturb_rt(m)
        for s in getattr(model, "sdms", []):
            nn.init.normal_(s.values, std=0.3)
    to_bf16_stream(model)
    g = torch.Generator().manual_seed(22)
    idx = torch.randint(0, V, (2, 40), generator=g)
    if reset_at_bos:
        idx[0, [3, 17]] = 0
        idx[1, [0, 25, 26]] = 0
    caps = []
    for li, m in enumerate(model.mems):
        orig = m.prepare

        def prep(xx, _orig=orig, _li=li):
            r = _orig(xx)
            caps.append((_li, xx.detach().float().numpy(), [npd(t) for t in r]))
            return r
        m.prepare = prep
    with torch.no_grad():
        logits = model(idx)
    for m in model.mems:
        del m.prepare
    out = dict(idx=npd(idx), logits=npd(logits), arm=arm, V=V, reset_at_bos=int(reset_at_bos),
               **{k: v for k, v in cfg.items() if k not in ("reset_at_bos",)},
               **{"p." + k: npd(v) for k, v in model.state_dict().items()})
    for li, xin, (siw, ww, sir, wr, Vv) in caps:
        out[f"L{li}.x_in"] = xin
        out[f"L{li}.siw"], out[f"L{li}.sir"] = siw, sir
        out[f"L{li}.ww"], out[f"L{li}.wr"] = ww, wr
    if arm == "onesdm_allsdm":
        out["sdm_n_sub"], out["sdm_heads"], out["sdm_d_a"], out["sdm_k"] = model.sdm_n_sub, 4, model.sdm_d_a, 32
    save(name, **out)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("SDMCHAT_REF"),
                    help="path of an SDMCHAT checkout (required; or set SDMCHAT_REF)")
    a = ap.parse_args()
    if not a.ref:
        ap.error("--ref (or SDMCHAT_REF) must name an SDMCHAT checkout")
    OM = load_reference(a.ref)
    torch.set_num_threads(1)  # bit-reproducible CPU reductions, as the reference's trainer self-test does
    pk_cases(OM)
    rt_config1(OM)
    rt_small(OM)
    rt_prevtok(OM)
    ts_selftest(OM)
    lm_case(OM, "lm_partial", "onesdm")
    lm_case(OM, "lm_full", "onesdm_allsdm")
    lm_case(OM, "lm_partial_bos", "onesdm", reset_at_bos=True)


if __name__ == "__main__":
    main()
