"""Pin the CPU oracle (oracle/sdm_oracle.py) against golden vectors written by the unmodified reference.

Every case here was produced by tests/golden/make_golden.py from the reference's own modules; the oracle must
reproduce them: slot ids exactly (wherever the selection margin is non-zero), floats to float32 rounding.
"""
import numpy as np
import pytest

from goldens import load, lm_params, params, rel, rt_params, same_selection
from oracle import sdm_oracle as O


@pytest.mark.parametrize("name", ["pk_selftest", "pk_k4", "pk_k16", "pk_ns72_k32"])
def test_pk_address_matches_reference(name):
    g = load(name)
    sv, si, margin = O.pk_address(g["z"], g["keys1"], g["keys2"], int(g["k"]), return_margin=True)
    assert sv.shape == g["sv"].shape and si.shape == g["si"].shape
    np.testing.assert_allclose(sv, g["sv"], atol=2e-7, rtol=0)
    ok, n, bad = same_selection(si, g["si"], margin, 0.0)
    assert ok, f"{bad} of {n} selections differ"
    # scores descending, slot ids in range and distinct per (token, head)
    assert (np.diff(sv, axis=-1) <= 0).all()
    n_sub = g["keys1"].shape[1]
    assert si.min() >= 0 and si.max() < n_sub * n_sub
    assert all(len(set(r)) == len(r) for r in si.reshape(-1, si.shape[-1]).tolist())


def test_pk_address_equals_brute_force():
    """The reference self-test (track4_onesdm_models.py:694-702): top-k of the c1 x c1 combine = brute force."""
    rng = np.random.default_rng(3)
    k1, k2 = rng.standard_normal((3, 20, 8)).astype(np.float32), rng.standard_normal((3, 20, 8)).astype(np.float32)
    z = rng.standard_normal((50, 3, 16)).astype(np.float32)
    for k in (1, 4, 16, 20, 32):
        sv, si, margin = O.pk_address(z, k1, k2, k, return_margin=True)
        full = ((np.einsum("nhd,hsd->nhs", O.l2_normalize(z[..., :8]), O.l2_normalize(k1))[..., :, None]
                 + np.einsum("nhd,hsd->nhs", O.l2_normalize(z[..., 8:]), O.l2_normalize(k2))[..., None, :])
                * np.float32(0.5)).reshape(50, 3, 400)
        bv, bi = O.topk_desc(full, min(k, 400))
        np.testing.assert_allclose(sv, bv, atol=1e-6)
        ok, _, _ = same_selection(si, bi, margin, 0.0)
        assert ok


RT_CASES = ["rt_config1", "rt_small_plain", "rt_small_learned", "rt_small_sumread", "rt_small_nogate",
            "rt_small_bos", "rt_prevtok"]


@pytest.mark.parametrize("name", RT_CASES)
def test_runtime_sdm_matches_reference(name):
    g = load(name)
    p = rt_params(g)
    reset = g["reset"] if "reset" in g else None
    out, st = O.rt_forward(p, g["x"], chunk=int(g["chunk"]), reset=reset)
    for key in ("siw", "sir"):
        margin = st["margin_w" if key == "siw" else "margin_r"]
        ok, n, bad = same_selection(st[key], g[key], margin, 0.0)
        assert ok, f"{key}: {bad} of {n} differ"
    for key in ("ww", "wr", "V", "gate"):
        assert rel(np.sort(st[key], -1) if key in ("ww", "wr") else st[key],
                   np.sort(g[key], -1) if key in ("ww", "wr") else g[key]) < 1e-5, key
    assert rel(st["num"], g["num"]) < 1e-5
    assert rel(st["den"], g["den"]) < 1e-5
    if (st["margin_w"] > 0).all():
        assert rel(st["mem"], g["mem"]) < 1e-5
        assert rel(st["cnt"], g["cnt"]) < 1e-5
    else:
        # exact ties (a zero address): which slots win is aten::topk's order, outside the contract; the state
        # then agrees up to a permutation of the locations
        assert rel(np.sort(st["mem"], 2), np.sort(g["mem"], 2)) < 1e-5
        assert rel(np.sort(st["cnt"], 2), np.sort(g["cnt"], 2)) < 1e-5
    assert rel(out, g["out"]) < 1e-5
    if "seq_out" in g:
        # the reference's chunked = sequential claim (track4_onesdm_models.py:728-744), and the oracle's recurrence
        out_s, _ = O.rt_forward(p, g["x"], reset=reset, sequential=True)
        assert rel(out_s, g["seq_out"]) < 1e-5
        np.testing.assert_allclose(out_s, out, atol=1e-5, rtol=1e-4)


def test_previous_token_known_answer():
    """Fade 0 with one shared address reads exactly the value written at t-1 (track4_onesdm_models.py:773-785)."""
    g = load("rt_prevtok")
    p = rt_params(g)
    out, st = O.rt_forward(p, g["x"], chunk=int(g["chunk"]))
    den = 1.0 / p.k
    want = st["V"][0, 0, :-1] * den / (den + float(p.read_eps))
    np.testing.assert_allclose(out[0, 1:], want, atol=1e-5)
    assert float(np.abs(out[0, 0]).max()) == 0.0


def test_chunk_sizes_agree_with_sequential():
    """chunks 1, 5, 23, 64 all equal the sequential recurrence (track4_onesdm_models.py:745-755)."""
    g = load("rt_small_plain")
    p = rt_params(g)
    ref, _ = O.rt_forward(p, g["x"], sequential=True)
    for ch in (1, 5, 23, 64):
        out, _ = O.rt_forward(p, g["x"], chunk=ch)
        np.testing.assert_allclose(out, ref, atol=1e-5, rtol=1e-4)


def test_trained_sdm_matches_reference():
    g = load("ts_selftest")
    p = O.TrainedSdmParams(params(g), int(g["heads"]), int(g["n_sub"]), int(g["d_a"]), int(g["k"]))
    out, si, margin = O.trained_sdm(p, g["x"])
    ok, n, bad = same_selection(si, g["si"], margin, 0.0)
    assert ok, f"{bad} of {n}"
    assert rel(out, g["out"]) < 1e-5


@pytest.mark.parametrize("name", ["lm_partial", "lm_full", "lm_partial_bos"])
def test_bf16_stream_lm_matches_reference(name):
    g = load(name)
    P = lm_params(g)
    logits, h, trace = O.lm_forward(P, g["idx"], bf16_stream=True, chunk=int(g["chunk"]),
                                    reset_at_bos=bool(int(g["reset_at_bos"])), collect=True)
    for li, rec in enumerate(trace):
        # the oracle's own residual input equals the reference's layer input
        assert rel(rec["x_in"], g[f"L{li}.x_in"]) < 1e-2, li
        for key, mk in (("siw", "margin_w"), ("sir", "margin_r")):
            ok, n, bad = same_selection(rec["prep"][key], g[f"L{li}.{key}"], rec["prep"][mk], 1e-6)
            assert ok, f"layer {li} {key}: {bad} of {n}"
    assert rel(logits, g["logits"]) < 2e-3


def test_matched_sdm_n_sub():
    """matched_sdm_n_sub at the FULL arm's d768 / mlp_f 2048 / 4 heads / d_a 32 gives 72 slots per half."""
    assert O.matched_sdm_n_sub(768, 2048, 4, 32) == 72
    assert O.matched_sdm_n_sub(1536, 4096, 4, 32) == 103


def test_bf16_rounding_matches_torch():
    import torch
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(10000) * 10.0 ** rng.integers(-8, 8, 10000)).astype(np.float32)
    want = torch.from_numpy(x).bfloat16().float().numpy()
    np.testing.assert_array_equal(O.bf16(x), want)


def test_teacher_forcing_with_own_selection_is_identity():
    """Forcing the oracle's own slot ids (as the full-depth GPU parity test forces the GPU's) changes nothing."""
    g = load("rt_config1")
    p = rt_params(g)
    x = g["x"]
    out, prep = O.rt_forward(p, x)
    out2, prep2 = O.rt_forward(p, x, force={"siw": prep["siw"], "sir": prep["sir"]})
    np.testing.assert_array_equal(prep2["siw"], prep["siw"])
    np.testing.assert_array_equal(prep2["ww"], prep["ww"])
    np.testing.assert_array_equal(out2, out)
    gt = load("ts_selftest")
    sd = params(gt)
    pt = O.TrainedSdmParams(sd, int(gt["heads"]), int(gt["n_sub"]), int(gt["d_a"]), int(gt["k"]))
    o1, si, _ = O.trained_sdm(pt, gt["x"])
    o2, si2, _ = O.trained_sdm(pt, gt["x"], force_si=si)
    np.testing.assert_array_equal(si2, si)
    np.testing.assert_array_equal(o2, o1)
