"""Load the golden fixtures written by tests/golden/make_golden.py and rebuild oracle parameter objects."""
import os

import numpy as np

from oracle import sdm_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    return {k: z[k] for k in z.files}


def params(g, prefix="p."):
    return {k[len(prefix):]: v for k, v in g.items() if k.startswith(prefix)}


def rt_params(g, prefix="p."):
    sd = params(g, prefix)
    return O.RunTimeSdmParams(sd, int(g["heads"]), int(g["n_sub"]), int(g["d_a"]), int(g["k"]),
                              write_gate=bool(int(g.get("write_gate", 1))), read_mode=str(g.get("read_mode", "mean")),
                              out_norm=bool(int(g.get("out_norm", 1))))


def lm_params(g):
    """Oracle parameter dict of a tiny LM fixture (OneSdmLM state_dict keys)."""
    sd = params(g)
    L = int(g["layers"])
    P = {"emb": sd["emb.weight"], "nf_w": sd["nf.w"], "layers": []}
    for i in range(L):
        msd = {k[len(f"mems.{i}."):]: v for k, v in sd.items() if k.startswith(f"mems.{i}.")}
        lay = {"mem": O.RunTimeSdmParams(msd, int(g["heads"]), int(g["n_sub"]), int(g["d_a"]), int(g["k"]))}
        if f"mlps.{i}.gate.weight" in sd:
            lay["mlp"] = (sd[f"mnorms.{i}.w"], sd[f"mlps.{i}.gate.weight"], sd[f"mlps.{i}.up.weight"],
                          sd[f"mlps.{i}.down.weight"])
        else:
            ssd = {k[len(f"sdms.{i}."):]: v for k, v in sd.items() if k.startswith(f"sdms.{i}.")}
            lay["sdm"] = O.TrainedSdmParams(ssd, int(g["sdm_heads"]), int(g["sdm_n_sub"]), int(g["sdm_d_a"]),
                                            int(g["sdm_k"]))
        P["layers"].append(lay)
    return P


def rel(a, b):
    """The reference self-test's relative error: max |a - b| / max |b| (track4_onesdm_models.py:688-689)."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / (np.abs(b).max() + 1e-12))


def rel_bf16(a, b):
    """`rel` for bfloat16-stored outputs: each element may first differ by one bfloat16 rounding step (at most
    2^-7 |b|, when the float32 accumulations on either side straddle a rounding boundary); the remainder is
    measured like `rel`.  Tests bound it by the same 2e-3."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    excess = np.maximum(np.abs(a - b) - np.abs(b) * 2.0 ** -7, 0.0)
    return float(excess.max() / (np.abs(b).max() + 1e-12))


def same_selection(si_a, si_b, margin, min_margin=0.0):
    """Sorted slot sets equal wherever the selection margin exceeds min_margin; returns (ok, n_checked, n_bad)."""
    a = np.sort(si_a, -1)
    b = np.sort(si_b, -1)
    bad = (a != b).any(-1)
    live = margin > min_margin
    return not bool((bad & live).any()), int(live.sum()), int((bad & live).sum())
