"""Parity of the whole benchmarked stacks against the CPU oracle at full depth: FULL d768 L12 (the headline model,
RunTimeSdm + TrainedSdm per layer) and PARTIAL d768 L12 f2048 (RunTimeSdm + SwiGLU(RMSNorm) per layer), one row of
256 Zipf tokens (two 128-token chunks), bf16 weights as the benchmark builds them.

The index-exactness protocol of the reference's pk_address (track4_onesdm_models.py:134-148): slot ids are compared on
identical addresses, and must be equal wherever the oracle's k-th / (k+1)-th score margin exceeds 1e-6.

* Layer by layer (teacher forcing), at every one of the 12 layers, on the GPU's own layer input:
  - the GPU's slot ids against the oracle's pk_address on the GPU's addresses z (write keys, read queries, TrainedSdm
    queries): equal above margin 1e-6, every differing selection reported with its margin;
  - the GPU's addresses against the oracle's (same input, projection computed by the oracle): within 2e-3;
  - with the GPU's slot ids forced into the oracle, the layer's memory and body outputs within 2e-3 (`rel_bf16`);
  - the oracle's own selections (from its own z) are reported against the GPU's with their margins: RMSNorm rounds its
    output to bfloat16, so a float32-level difference in its sum of squares can move one element by a bfloat16 step
    (2^-8 relative) and a score by up to ~1e-4; selections closer than that can differ between any two correct
    implementations, the reference's own CPU and GPU runs included.
* The tied logits and the CE sum on the final stream within 2e-3 / 1e-4.
* Free running, the oracle's own 12-layer forward against the GPU's: the first (position, layer) where a selection
  differs must be such a near-tie (margin below 1e-3), and every earlier position's logits agree within 2e-3.

The report (selection counts, every flip with its margin, errors) is written as JSON to $SDM_PARITY_REPORT when set."""
import json
import os

import numpy as np
import pytest
import torch

import sdmchat_b200 as S
from goldens import rel, rel_bf16
from oracle import sdm_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
MARGIN = 1e-6
V = 32768


def zipf_ids(seed, shape):
    rng = np.random.default_rng(seed)
    return np.minimum(rng.zipf(1.1, size=shape) - 1, V - 1).astype(np.int64)


def build(arm, seed=0, bf16=True):
    torch.manual_seed(seed)
    model = S.build_onesdm(arm, V, dict(d=768, layers=12, mlp_f=2048, heads=12, decays=S.readme_fades(12)))
    with torch.no_grad():
        for m in model.mems:
            torch.nn.init.normal_(m.wo.weight, std=0.02)
            torch.nn.init.normal_(m.wg.weight, std=0.5 / 768 ** 0.5)
        for s in getattr(model, "sdms", []):
            torch.nn.init.normal_(s.values, std=0.02)
    model = (model.to_bf16_stream() if bf16 else model).to(DEV)
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
    out = {"selections": 0, "pk_flips": [], "pk_min_margin": float("inf"), "own_z_flips": [], "max_rel": 0.0,
           "max_z_rel": 0.0}

    def check_pk(gpu_z, gpu_si, keys1, keys2, k, where, own_si, own_margin):
        """gpu_z (N, h, d_a), gpu_si / own_si (N, h, k), own_margin (N, h)."""
        _, si_z, m_z = O.pk_address(gpu_z, keys1, keys2, k, return_margin=True)
        f = flips(gpu_si, si_z, m_z, where)
        out["pk_flips"] += [{"where": where, "index_nh": ix, "margin": m} for ix, m in f]
        out["pk_min_margin"] = min(out["pk_min_margin"], float(m_z.min()))
        out["selections"] += int(m_z.size)
        bad = (np.sort(gpu_si, -1) != np.sort(own_si, -1)).any(-1)
        out["own_z_flips"] += [{"where": where, "index_nh": tuple(int(i) for i in ix),
                                "margin": float(own_margin[tuple(ix)])} for ix in np.argwhere(bad)]

    def tok(t):  # (B, h, T, k) -> (B*T, h, k)
        return np.asarray(t).transpose(0, 2, 1, 3).reshape(B * T, t.shape[1], -1)

    for i, rec in enumerate(trace):
        lay = P["layers"][i]
        mp = lay["mem"]
        x_in = np32(rec["x_in"])
        _, own = O.rt_forward(mp, x_in, bf16_stream=True)
        z = np32(rec["z"]).reshape(B * T, 2, mp.h, mp.d_a)
        e = max(rel(z[:, 0], own["kz"]), rel(z[:, 1], own["qz"]))
        assert e < 2e-3, f"layer {i}: addresses rel {e:.3g}"
        out["max_z_rel"] = max(out["max_z_rel"], e)
        for j, (key, mk) in enumerate((("siw", "margin_w"), ("sir", "margin_r"))):
            check_pk(z[:, j], tok(rec[key].cpu().numpy()), mp.keys1, mp.keys2, mp.k, f"layer {i} {key}",
                     tok(own[key]), own[mk].transpose(0, 2, 1).reshape(B * T, mp.h))
        forced, _ = O.rt_forward(mp, x_in, bf16_stream=True, margins=False,
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
            sp = lay["sdm"]
            _, si_o, margin = O.trained_sdm(sp, x_mid, True)
            gsi = rec["sdm_si"].cpu().numpy().reshape(si_o.shape)
            q = np32(rec["sdm_q"]).reshape(B * T, sp.h, sp.d_a)
            q_o = O.linear(O.rmsnorm(x_mid, sp.norm_w, bf16_stream=True).reshape(B * T, sp.d), sp.wq)
            e = rel(q, q_o.reshape(q.shape))
            assert e < 2e-3, f"layer {i}: TrainedSdm queries rel {e:.3g}"
            out["max_z_rel"] = max(out["max_z_rel"], e)
            check_pk(q, gsi, sp.keys1, sp.keys2, sp.k, f"layer {i} ts", si_o, margin)
            s_forced = O.trained_sdm(sp, x_mid, True, margins=False, force_si=gsi)[0]
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
    out.update(logits_rel=e, loss=loss, loss_oracle=want_loss, n_pk_flips=len(out["pk_flips"]),
               n_own_z_flips=len(out["own_z_flips"]),
               own_z_flip_max_margin=max([f["margin"] for f in out["own_z_flips"]], default=0.0))
    return out, trace, logits


def free_running(model, P, idx, trace, logits, bf16=True, first_margin=1e-3, tol=2e-3):
    """The oracle's own forward against the GPU's: the first divergence is a near-tie (margin < first_margin) and
    positions before it agree within tol."""
    lg_o, _, tr_o = O.lm_forward(P, idx.cpu().numpy(), bf16_stream=bf16, collect=True)
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
    measure = rel_bf16 if bf16 else rel
    lg = np32(logits)
    res = {"first_divergence": p, "positions": T, "logits_rel_all": measure(lg, lg_o),
           "ce_sum": O.ce_sum(lg[:, :-1], idx.cpu().numpy()[:, 1:]),
           "ce_sum_oracle": O.ce_sum(lg_o[:, :-1], idx.cpu().numpy()[:, 1:])}
    if first is not None:
        _, i, _, name, margins = first
        res.update(layer=i, module=name, margins=margins)
        assert max(margins) < first_margin, f"first divergence at position {p} (layer {i} {name}) is not a near-tie: " \
                                            f"{margins}"
    if p > 0:
        e = measure(lg[:, :p], lg_o[:, :p])
        res["logits_rel_before"] = e
        assert e < tol, f"free-running logits rel {e:.3g} before position {p}"
    return res


@pytest.mark.parametrize("arm", ["onesdm_allsdm", "onesdm"])
def test_full_depth_against_oracle(cuda_ok, arm):
    model, P = build(arm)
    idx = torch.from_numpy(zipf_ids(11, (1, 256))).to(DEV)
    forced, trace, logits = teacher_forced(model, P, idx, arm)
    free = free_running(model, P, idx, trace, logits)
    report(f"{arm}_d768_L12_1x256", {"teacher_forced": forced, "free_running": free})
    print(f"{arm}: {forced['selections']} selections on identical addresses, {forced['n_pk_flips']} near-tie flips "
          f"(min oracle margin {forced['pk_min_margin']:.3g}); {forced['n_own_z_flips']} differ from the oracle's own "
          f"addresses (largest margin {forced['own_z_flip_max_margin']:.3g}); logits rel {forced['logits_rel']:.3g}; "
          f"free run first divergence at {free['first_divergence']} of {free['positions']}")


@pytest.mark.parametrize("arm", ["onesdm_allsdm", "onesdm"])
def test_full_depth_float32_free_running(cuda_ok, arm):
    """The same stacks with float32 weights and activations (the library's float32 mode, the precision of the
    reference's CPU forward): no bfloat16 rounding amplifies float32 summation-order differences, so the free-running
    12-layer forwards must agree at every selection whose margin exceeds 1e-6, and the logits before any divergence
    within 1e-4 (max-norm relative)."""
    model, P = build(arm, bf16=False)
    idx = torch.from_numpy(zipf_ids(12, (1, 256))).to(DEV)
    trace = []
    with torch.no_grad():
        xf = model.residual(idx, trace=trace)
        logits = model._head(xf, "logits")
    free = free_running(model, P, idx, trace, logits, bf16=False, first_margin=MARGIN, tol=1e-4)
    report(f"{arm}_d768_L12_1x256_float32", {"free_running": free})
    print(f"{arm} float32: first divergence at {free['first_divergence']} of {free['positions']}; logits rel "
          f"{free['logits_rel_all']:.3g}; CE sum {free['ce_sum']:.6f} vs oracle {free['ce_sum_oracle']:.6f}")
