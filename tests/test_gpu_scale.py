"""GPU parity at the benchmark's shapes: the d768 / 12 heads x 64 / k16 / 1,024-slot layer against the CPU oracle on
identical inputs, and size-independent properties of the full FULL d768 L12 T2048 stack (determinism, causality,
loss = CE of its own logits, decode = recurrence across a state renormalisation)."""
import numpy as np
import pytest
import torch

import sdmchat_b200 as S
from goldens import rel, rel_bf16, same_selection
from oracle import sdm_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def zipf_ids(rng, shape, V=32768, s=1.1):
    return np.minimum(rng.zipf(s, size=shape) - 1, V - 1).astype(np.int64)


def d768_layer(seed=0, k=16, fades=None):
    torch.manual_seed(seed)
    m = S.RunTimeSdm(768, heads=12, n_sub=32, d_a=32, k=k, decays=fades or S.readme_fades(12))
    with torch.no_grad():
        for lin in (m.wk, m.wq, m.wv):
            torch.nn.init.normal_(lin.weight, std=0.02)
        torch.nn.init.normal_(m.wo.weight, std=0.02)
        torch.nn.init.normal_(m.wg.weight, std=0.5 / 768 ** 0.5)
    return m


def oracle_params(m):
    sd = {k: v.detach().float().cpu().numpy() for k, v in m.state_dict().items()}
    return O.RunTimeSdmParams(sd, m.h, m.n_sub, m.d_a, m.k)


def test_d768_layer_bf16_against_oracle(cuda_ok):
    rng = np.random.default_rng(1)
    m = d768_layer()
    m = m.to(DEV).to(torch.bfloat16)
    emb = (rng.standard_normal((32768, 768)) * 0.02).astype(np.float32)
    ids = zipf_ids(rng, (2, 512))
    x = O.bf16(emb[ids])
    with torch.no_grad():
        out, o = m.forward_with(torch.from_numpy(x).to(DEV).bfloat16())
    p = oracle_params(m)
    want, st = O.rt_forward(p, x, bf16_stream=True)
    flips = 0
    for key, mk in (("siw", "margin_w"), ("sir", "margin_r")):
        got = o[key].cpu().numpy()
        bad = (np.sort(got, -1) != np.sort(st[key], -1)).any(-1)
        live = st[mk] > 1e-6
        assert not (bad & live).any(), f"{key}: {(bad & live).sum()} flips above margin 1e-6"
        flips += int(bad.sum())
    assert flips <= 0.001 * 2 * 2 * 12 * 512  # near-tie flips only
    num = o["num"].cpu().numpy().transpose(0, 2, 1, 3)
    assert rel(num, st["num"]) < 2e-3
    assert rel(m.last_state[0].cpu().numpy(), st["mem"]) < 2e-3
    assert rel(m.last_state[1].cpu().numpy(), st["cnt"]) < 2e-3
    assert rel_bf16(out.float().cpu().numpy(), want) < 2e-3


def test_state_renormalisation_in_decode(cuda_ok):
    """fade 0.8 over 400 tokens drives the lazy scale below 2^-60 (0.8^187): the decode path folds it into the
    state and still equals the chunked form; fade 0 exercises the cleared previous rows."""
    torch.manual_seed(3)
    m = S.RunTimeSdm(128, heads=4, n_sub=16, d_a=16, k=8, decays=(0.8, 0.0, 0.5, 0.97)).to(DEV)
    with torch.no_grad():
        torch.nn.init.normal_(m.wo.weight, std=0.3)
        torch.nn.init.normal_(m.wg.weight, std=0.5)
        x = torch.randn(3, 400, 128, device=DEV)
        a = m(x)
        mem_a = m.last_state[0].clone()
        b = m.forward_sequential(x)
        mem_b = m.last_state[0]
    torch.testing.assert_close(b, a, atol=1e-5, rtol=1e-4)
    assert float((mem_b - mem_a).abs().max() / mem_a.abs().max()) < 1e-4


def full_model(layers=12, seed=0):
    torch.manual_seed(seed)
    model = S.build_onesdm("onesdm_allsdm", 32768, dict(d=768, layers=layers, mlp_f=2048, heads=12,
                                                         decays=S.readme_fades(12)))
    with torch.no_grad():
        for m in model.mems:
            torch.nn.init.normal_(m.wo.weight, std=0.02)
            torch.nn.init.normal_(m.wg.weight, std=0.5 / 768 ** 0.5)
        for s in model.sdms:
            torch.nn.init.normal_(s.values, std=0.02)
    return model.to_bf16_stream().to(DEV)


def test_full_d768_L12_T2048_properties(cuda_ok):
    rng = np.random.default_rng(2)
    model = full_model()
    idx = torch.from_numpy(zipf_ids(rng, (2, 2048))).to(DEV)
    with torch.no_grad():
        a = model(idx)
        b = model(idx)
        assert torch.isfinite(a.float()).all()
        assert torch.equal(a, b), "forward is not bit-reproducible"
        idx2 = idx.clone()
        p = 1500
        idx2[:, p] = (idx2[:, p] + 5) % 32768
        c = model(idx2)
        assert torch.equal(a[:, :p], c[:, :p]), "a later token changed an earlier position (causality)"
        assert not torch.equal(a[:, p:], c[:, p:])
        tgt = torch.roll(idx, -1, 1)
        tgt[:, -1] = -1
        loss = float(model.loss_sum(idx, tgt).item())
        lg = a.double()[:, :-1]
        want = float((torch.logsumexp(lg, -1) - lg.gather(-1, idx[:, 1:, None])[..., 0]).sum())
    assert abs(loss - want) / abs(want) < 1e-4


def test_decode_graph_equals_eager(cuda_ok):
    """The CUDA-graph decode step replays exactly the eager step: same ids, same carried state, bit for bit."""
    rng = np.random.default_rng(5)
    model = full_model(layers=2, seed=2)
    idx = torch.from_numpy(zipf_ids(rng, (3, 64))).to(DEV)
    with torch.no_grad():
        st1, st2 = model.init_decode(3), model.init_decode(3)
        a, b = model.prefill(idx, st1), model.prefill(idx, st2)
        step = model.decode_graph(st2)
        for _ in range(5):
            a = model.decode_step(a, st1)
            b = step(b).clone()
            assert torch.equal(a, b)
    for i in range(2):
        for key in st1[i]:
            assert torch.equal(st1[i][key], st2[i][key]), key


def test_full_decode_matches_prefill(cuda_ok):
    """Greedy decode on the carried state = argmax of the chunked forward on the whole prefix."""
    rng = np.random.default_rng(4)
    model = full_model(layers=2, seed=1)
    idx = torch.from_numpy(zipf_ids(rng, (4, 300))).to(DEV)
    with torch.no_grad():
        gen = model.generate(idx, 8)
        seq = torch.cat([idx, gen], 1)
        lg = model(seq[:, :-1]).float()[:, 299:]
    top = torch.topk(lg, 2, -1).values
    clear = (top[..., 0] - top[..., 1]) > 1e-2
    assert (lg.argmax(-1) == gen)[clear].all()
    assert clear.float().mean() > 0.5


def test_loss_sum_row_streams_equal(cuda_ok):
    """Rows split over two CUDA streams give the same CE sum (up to the order of float64 additions)."""
    rng = np.random.default_rng(6)
    model = full_model(layers=2, seed=3)
    idx = torch.from_numpy(zipf_ids(rng, (4, 512))).to(DEV)
    tgt = torch.roll(idx, -1, 1)
    with torch.no_grad():
        a = float(model.loss_sum(idx, tgt).item())
        b = float(model.loss_sum(idx, tgt, row_streams=2).item())
        c = float(model.loss_sum(idx, tgt, row_streams=2).item())
    assert abs(a - b) <= 1e-12 * abs(a) and abs(b - c) <= 1e-12 * abs(a)


def test_scaled_full_d1536_window16k_state_carry(cuda_ok):
    """Scaled FULL shapes (d1536, 24 heads x 64, 1,024 slots, k16, window 16,384): the chunked scan carries the
    state through 256 chunks; the prefix's chunked forward followed by 64 carried-state decode steps (the token
    recurrence) gives the chunked forward's last 64 outputs and its final memory."""
    torch.manual_seed(7)
    m = S.RunTimeSdm(1536, heads=24, n_sub=32, d_a=32, k=16, decays=S.readme_fades(24))
    with torch.no_grad():
        for lin in (m.wk, m.wq, m.wv):
            torch.nn.init.normal_(lin.weight, std=0.02)
        torch.nn.init.normal_(m.wo.weight, std=0.02)
        torch.nn.init.normal_(m.wg.weight, std=0.5 / 1536 ** 0.5)
    m = m.to(DEV)
    T, tail = 16384, 64
    g = torch.Generator(device=DEV).manual_seed(8)
    x = torch.randn(1, T, 1536, device=DEV, generator=g)
    with torch.no_grad():
        full = m(x)
        mem_full, cnt_full = (t.clone() for t in m.last_state)
        _, o = m.forward_with(x[:, :T - tail], want=("sel",))
        st = m.init_state(1, DEV)
        st["mem"].copy_(m.last_state[0])
        st["cnt"].copy_(m.last_state[1])
        st["last_w"].copy_(o["siw"][:, :, -1, :])
        steps = torch.stack([m.decode_step(x[:, t], st) for t in range(T - tail, T)], 1)
    assert torch.isfinite(full).all()
    torch.testing.assert_close(steps, full[:, T - tail:], atol=1e-5, rtol=1e-4)
    mem_dec = st["mem"] * st["scale"][..., None, None]
    cnt_dec = st["cnt"] * st["scale"][..., None]
    assert float((mem_dec - mem_full).abs().max() / mem_full.abs().max()) < 1e-4
    assert float((cnt_dec - cnt_full).abs().max() / cnt_full.abs().max()) < 1e-4


def test_scaled_trained_sdm_d1536_against_oracle(cuda_ok):
    """Scaled FULL's TrainedSdm body (d1536: 4 heads, d_a 32, n_sub 103 -> 10,609 slots, dh 384, k 32) against the
    CPU oracle: selections exact wherever the margin exceeds 1e-6, outputs within 2e-3."""
    rng = np.random.default_rng(9)
    torch.manual_seed(9)
    n_sub = O.matched_sdm_n_sub(1536, 4096, 4, 32)
    ts = S.TrainedSdm(1536, n_sub=n_sub, heads=4, d_a=32, k=32)
    with torch.no_grad():
        torch.nn.init.normal_(ts.values, std=0.02)
        torch.nn.init.normal_(ts.wo.weight, std=0.02)
    sd = {k: v.detach().float().numpy() for k, v in ts.state_dict().items()}
    ts = ts.to(DEV)
    x = rng.standard_normal((2, 300, 1536)).astype(np.float32)
    p = O.TrainedSdmParams(sd, 4, n_sub, 32, 32)
    want, si_o, margin = O.trained_sdm(p, x)
    with torch.no_grad():
        out = ts(torch.from_numpy(x).to(DEV)).cpu().numpy()
    ok, n, bad = same_selection(ts.last_si.cpu().numpy().reshape(si_o.shape), si_o, margin, 1e-6)
    assert ok, f"{bad} of {n}"
    assert rel(out, want) < 2e-3


def test_scaled_trained_sdm_bf16_dense_gather_equals_small_calls(cuda_ok):
    """The bf16 value gather of scaled FULL's TrainedSdm (dh 384): a large call (2,400 (token, head) items: the
    dense-lane gather) against calls of 40 tokens (160 items: the per-warp gather), both summing each column over the
    32 picked rows in slot order with fused multiply-adds.  Selections identical, outputs to the output GEMM's
    rounding (the two call sizes take different GEMM kernels)."""
    rng = np.random.default_rng(23)
    torch.manual_seed(23)
    n_sub = O.matched_sdm_n_sub(1536, 4096, 4, 32)
    ts = S.TrainedSdm(1536, n_sub=n_sub, heads=4, d_a=32, k=32)
    with torch.no_grad():
        torch.nn.init.normal_(ts.values, std=0.02)
        torch.nn.init.normal_(ts.wo.weight, std=0.02)
    ts = ts.to(DEV).to(torch.bfloat16)
    x = torch.from_numpy(rng.standard_normal((1, 600, 1536)).astype(np.float32)).to(DEV).bfloat16()
    with torch.no_grad():
        big = ts(x)
        si_big = ts.last_si.clone().reshape(600, 4, 32)
        for c0 in (0, 280, 560):
            small = ts(x[:, c0:c0 + 40])
            assert torch.equal(si_big[c0:c0 + 40], ts.last_si.reshape(40, 4, 32)), c0
            assert rel_bf16(small.float().cpu().numpy(), big[:, c0:c0 + 40].float().cpu().numpy()) < 1e-4, c0
