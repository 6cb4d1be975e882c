"""Parity of the whole benchmarked stacks against the CPU oracle at full depth: FULL d768 L12 (the headline model,
RunTimeSdm + TrainedSdm per layer) and PARTIAL d768 L12 f2048 (RunTimeSdm + SwiGLU(RMSNorm) per layer), one row of
256 Zipf tokens (two 128-token chunks), bf16 weights as the benchmark builds them.

Two comparisons, following the index-exactness protocol of the reference's pk_address (track4_onesdm_models.py:
134-148; exact slot ids wherever the oracle's k-th / (k+1)-th score margin exceeds 1e-6):

* layer by layer (teacher forcing): every layer's GPU input is fed to the oracle layer.  The GPU's slot ids must equal
  the oracle's own wherever the margin exceeds 1e-6 (every differing selection below it is reported with its
  margin), and with the GPU's ids forced into the oracle the layer's outputs must agree within 2e-3 (`rel_bf16`);
  the tied logits and the CE sum likewise on the final stream;
* free running: the oracle's own 12-layer forward against the GPU's.  The first position where any layer's
  selection differs must be a near-tie (margin below 1e-6); every earlier position's logits agree within 2e-3.

The flip report (layer, module, position, head, margin) is written as JSON to $SDM_PARITY_REPORT when it is set."""
import json
import os

import numpy as np
import pytest
import torch

import sdmchat_b200 as S
from goldens import rel_bf16
from oracle import sdm_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
MARGIN = 1e-6
V = 32768


def zipf_ids(seed, shape):
    rng = np.random.default_rng(seed)
    return np.minimum(rng.zipf(1.1, size=shape) - 1, V - 1).astype(np.int64)


def build(arm, seed=0):
    torch.manual_seed(seed)
    model = S.build_onesdm(arm, V, dict(d=768, layers=12, mlp_f=2048, heads=12, decays=S.readme_fades(12)))
    with torch.no_grad():
        for m in model.mems:
            torch.nn.init.normal_(m.wo.weight, std=0.02)
            torch.nn.init.normal_(m.wg.weight, std=0.5 / 768 ** 0.5)
        for s in getattr(model, "sdms", []):
            torch.nn.init.normal_(s.values, std=0.02)
    model = model.to_bf16_stream().to(DEV)
    sd = {k: v.detach().float().cpu().numpy() for k, v in model.state_dict().items()}  # bf16 values, exact
    P = {"emb": sd["emb.weight"], "nf_w": sd["nf.w"], "layers": []}
    for i in range(12):
        msd = {k[len(f"mems.{i}."):]: v for k, v in sd.items() if k.startswith(f"mems.{i}.")}
        lay = {"mem": O.RunTimeSdmParams(msd, 12, 32, 32, 16)}
        if arm == "onesdm":
            lay["mlp"] = (sd[f"mnorms.{i}.w"], sd[f"mlps.{i}.gate.weight"], sd[f"mlps.{i}.up.weight"],
                          sd[f"mlps.{i}.down.weight"])
        else:
            ssd = {k[len(f"sdms.{i}."):]: v for k, v in sd.items() if k.startswith(f"sdms.{i}.")}
            lay["sdm"] = O.TrainedSdmParams(ssd, 4, model.sdm_n_sub, model.sdm_d_a, 32)
        P["layers"].append(lay)
    return model, P


def np32(t):
    return t.detach().float().cpu().numpy()


def flips(got, want, margin, where):
    """Selections whose slot sets differ: (positions as tuples, margins); fails on one above MARGIN."""
    bad = (np.sort(got, -1) != np.sort(want, -1)).any(-1)
    above = bad & (margin > MARGIN)
    assert not above.any(), f"{where}: {int(above.sum())} selections differ above margin {MARGIN}: " \
                            f"{[(tuple(int(i) for i in ix), float(margin[tuple(ix)])) for ix in np.argwhere(above)[:5]]}"
    return [(tuple(int(i) for i in ix), float(margin[tuple(ix)])) for ix in np.argwhere(bad)]


def report(name, rec):
    path = os.environ.get("SDM_PARITY_REPORT")
    if not path:
        return
    data = {}
    if os.path.exists(path):
        with open(path) as f:
            data = json.load(f)
    data[name] = rec
    with open(path, "w") as f:
        json.dump(data, f, indent=1)


def teacher_forced(model, P, idx, arm):
    trace = []
    with torch.no_grad():
        xf = model.residual(idx, trace=trace)
        logits = model._head(xf, "logits")
        tgt = torch.roll(idx, -1, 1)
        tgt[:, -1] = -1
        loss = float(model.loss_sum(idx, tgt).item())
    B, T = idx.shape
    out = {"flips": [], "min_margin": float("inf"), "selections": 0, "max_rel": 0.0}
    for i, rec in enumerate(trace):
        lay = P["layers"][i]
        x_in = np32(rec["x_in"])
        _, own = O.rt_forward(lay["mem"], x_in, bf16_stream=True)
        for key, mk in (("siw", "margin_w"), ("sir", "margin_r")):
            f = flips(rec[key].cpu().numpy(), own[key], own[mk], f"layer {i} {key}")
            out["flips"] += [{"layer": i, "module": key, "index_bht": ix, "margin": m} for ix, m in f]
            out["min_margin"] = min(out["min_margin"], float(own[mk].min()))
            out["selections"] += int(own[mk].size)
        forced, _ = O.rt_forward(lay["mem"], x_in, bf16_stream=True, margins=False,
                                 force={"siw": rec["siw"].cpu().numpy(), "sir": rec["sir"].cpu().numpy()})
        want_mid = O.add_stream(x_in, forced, True)
        e = rel_bf16(np32(rec["x_mid"]), want_mid)
        assert e < 2e-3, f"layer {i}: memory output rel {e:.3g}"
        out["max_rel"] = max(out["max_rel"], e)
        x_mid = np32(rec["x_mid"])
        if arm == "onesdm":
            nw, wg, wu, wd = lay["mlp"]
            want_out = O.add_stream(x_mid, O.swiglu(O.rmsnorm(x_mid, nw, bf16_stream=True), wg, wu, wd, True), True)
        else:
            _, si_o, margin = O.trained_sdm(lay["sdm"], x_mid, True)
            gsi = rec["sdm_si"].cpu().numpy()
            f = flips(gsi.reshape(si_o.shape), si_o, margin, f"layer {i} TrainedSdm")
            out["flips"] += [{"layer": i, "module": "ts", "index_nh": ix, "margin": m} for ix, m in f]
            out["min_margin"] = min(out["min_margin"], float(margin.min()))
            out["selections"] += int(margin.size)
            s_forced = O.trained_sdm(lay["sdm"], x_mid, True, margins=False, force_si=gsi.reshape(si_o.shape))[0]
            want_out = O.add_stream(x_mid, s_forced, True)
        got_out = np32(trace[i + 1]["x_in"]) if i + 1 < len(trace) else np32(xf)
        e = rel_bf16(got_out, want_out)
        assert e < 2e-3, f"layer {i}: body output rel {e:.3g}"
        out["max_rel"] = max(out["max_rel"], e)
    want_lg = O.linear(O.rmsnorm(np32(xf), P["nf_w"], bf16_stream=True), P["emb"], bf16_out=True)
    e = rel_bf16(np32(logits), want_lg)
    assert e < 2e-3, f"logits rel {e:.3g}"
    want_loss = O.ce_sum(want_lg[:, :-1], idx.cpu().numpy()[:, 1:])
    assert abs(loss - want_loss) / abs(want_loss) < 1e-4, (loss, want_loss)
    out.update(logits_rel=e, loss=loss, loss_oracle=want_loss, n_flips=len(out["flips"]))
    return out, trace, logits


def free_running(model, P, idx, trace, logits):
    """The oracle's own forward against the GPU's: positions before the first divergence must agree."""
    lg_o, _, tr_o = O.lm_forward(P, idx.cpu().numpy(), bf16_stream=True, collect=True)
    B, T = idx.shape
    cands = []  # (position, layer, module order, module, margins of the differing selections there)
    for i, (g, o) in enumerate(zip(trace, tr_o)):
        for name, want, margin, got in (("siw", o["prep"]["siw"], o["prep"]["margin_w"], g["siw"]),
                                        ("sir", o["prep"]["sir"], o["prep"]["margin_r"], g["sir"])):
            bad = (np.sort(got.cpu().numpy(), -1) != np.sort(want, -1)).any(-1)  # (B, h, T)
            if bad.any():
                p = int(np.argwhere(bad)[:, 2].min())
                cands.append((p, i, 0, name, [float(m) for m in margin[..., p][bad[..., p]]]))
        if "sdm_si" in o:
            got = g["sdm_si"].cpu().numpy().reshape(o["sdm_si"].shape)  # (B*T, h, k)
            bad = (np.sort(got, -1) != np.sort(o["sdm_si"], -1)).any(-1).reshape(B, T, -1)
            if bad.any():
                p = int(np.argwhere(bad)[:, 1].min())
                m = o["sdm_margin"].reshape(B, T, -1)
                cands.append((p, i, 1, "ts", [float(x) for x in m[:, p][bad[:, p]]]))
    first = min(cands) if cands else None
    p = first[0] if first else T
    res = {"first_divergence": p, "positions": T}
    if first is not None:
        _, i, _, name, margins = first
        res.update(layer=i, module=name, margins=margins)
        assert max(margins) < MARGIN, f"first divergence at position {p} (layer {i} {name}) is not a near-tie: {margins}"
    if p > 0:
        e = rel_bf16(np32(logits)[:, :p], lg_o[:, :p])
        res["logits_rel_before"] = e
        assert e < 2e-3, f"free-running logits rel {e:.3g} before position {p}"
    return res


@pytest.mark.parametrize("arm", ["onesdm_allsdm", "onesdm"])
def test_full_depth_against_oracle(cuda_ok, arm):
    model, P = build(arm)
    idx = torch.from_numpy(zipf_ids(11, (1, 256))).to(DEV)
    forced, trace, logits = teacher_forced(model, P, idx, arm)
    free = free_running(model, P, idx, trace, logits)
    report(f"{arm}_d768_L12_1x256", {"teacher_forced": forced, "free_running": free})
    print(f"{arm}: {forced['selections']} selections, {forced['n_flips']} near-tie flips "
          f"(min oracle margin {forced['min_margin']:.3g}); logits rel {forced['logits_rel']:.3g}; "
          f"free run first divergence at {free['first_divergence']} of {free['positions']}")
