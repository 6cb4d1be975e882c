"""The module methods of the drop-in boundary beside forward(), each on the library against the CPU oracle:
SwiGLU.forward (track4_sdmllm_models.py:96-97) at the PARTIAL arm's d768 / f2048 in bf16 (the fused gate|up tensor-core
GEMM) and float32, SwiGLU.block, RunTimeSdm._chunk with a carried state and BOS segments (track4_onesdm_models.py:
215-241), RunTimeSdm.finish (:243-247), OneSdmLM.project (:528-529) and OneSdmLM.set_leak (:560-564)."""
import numpy as np
import pytest
import torch

import sdmchat_b200 as S
from goldens import rel, rel_bf16
from oracle import sdm_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def np32(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_swiglu_forward_d768_f2048(cuda_ok, dt):
    torch.manual_seed(0)
    m = S.SwiGLU(768, 2048)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 300, 768, generator=g)
    nw = 1.0 + 0.1 * torch.randn(768, generator=g)
    m = m.to(DEV).to(dt)
    xd = x.to(DEV).to(dt)
    with torch.no_grad():
        out = m(xd)
        blk = m.block(xd, nw.to(DEV))
    bf = dt == torch.bfloat16
    wg, wu, wd = (np32(w) for w in (m.gate.weight, m.up.weight, m.down.weight))
    xs = np32(xd)
    want = O.swiglu(xs, wg, wu, wd, bf16_stream=bf)
    nwv = np32(nw.to(dt))
    want_blk = O.add_stream(xs, O.swiglu(O.rmsnorm(xs, nwv, bf16_stream=bf), wg, wu, wd, bf), bf)
    if bf:
        assert rel_bf16(np32(out), want) < 2e-3
        assert rel_bf16(np32(blk), want_blk) < 2e-3
    else:
        np.testing.assert_allclose(np32(out), want, atol=1e-5, rtol=1e-4)
        np.testing.assert_allclose(np32(blk), want_blk, atol=1e-5, rtol=1e-4)
    # the packed weight is reused until a weight changes
    p1 = m._packed(dt, xd.device)[0]
    with torch.no_grad():
        m.up.weight.mul_(2)
        out2 = m(xd)
    assert m._packed(dt, xd.device)[0] is not p1
    want2 = O.swiglu(xs, wg, np32(m.up.weight), wd, bf16_stream=bf)
    assert (rel_bf16 if bf else rel)(np32(out2), want2) < (2e-3 if bf else 1e-5)


def rt_small(seed, fades, k=4):
    torch.manual_seed(seed)
    m = S.RunTimeSdm(256, heads=4, n_sub=32, d_a=32, k=k, decays=fades)
    return m.to(DEV)


@pytest.mark.parametrize("fades,bos", [((0.9, 0.95, 0.999, 0.97), False), ((0.0, 0.8, 0.99, 1.0), True)])
def test_chunk_with_carried_state(cuda_ok, fades, bos):
    """_chunk from a non-empty state equals the reference's chunk formula (the oracle's rt_chunk), float32."""
    m = rt_small(2, fades)
    g = torch.Generator(device=DEV).manual_seed(3)
    B, L = 2, 128
    x = torch.randn(B, L, 256, device=DEV, generator=g)
    with torch.no_grad():
        siw, ww, sir, wr, V = m.prepare(x)
    mem = torch.randn(B, 4, m.M, 64, device=DEV, generator=g) * 0.3
    cnt = torch.rand(B, 4, m.M, device=DEV, generator=g)
    lam = m.decay()
    seg = seg_prev = None
    if bos:
        seg = torch.zeros(B, L, dtype=torch.long, device=DEV)
        seg[0, 40:] = 1
        seg[0, 97:] = 2
        seg[1, :] = 5
        seg_prev = torch.tensor([0, 4], device=DEV)  # row 1: a new segment from the chunk's first position
    with torch.no_grad():
        num, den, mem2, cnt2 = m._chunk(siw, ww, sir, wr, V, mem, cnt, lam, seg, seg_prev)
    args = [np32(t) for t in (siw, ww, sir, wr, V, mem, cnt)]
    args[0], args[2] = args[0].astype(np.int64), args[2].astype(np.int64)
    kw = {} if seg is None else dict(seg=seg.cpu().numpy(), seg_prev=seg_prev.cpu().numpy())
    wn, wd, wm, wc = O.rt_chunk(*args, np32(lam), m.M, **kw)
    assert num.shape == wn.shape and den.shape == wd.shape
    assert rel(np32(num), wn) < 1e-5
    assert rel(np32(den), wd) < 1e-5
    assert rel(np32(mem2), wm) < 1e-5
    assert rel(np32(cnt2), wc) < 1e-5


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_finish(cuda_ok, dt):
    m = rt_small(4, (0.9, 0.95, 0.999, 0.97))
    with torch.no_grad():
        torch.nn.init.normal_(m.onorm_w, mean=1.0, std=0.1)
    m = m.to(dt)
    g = torch.Generator(device=DEV).manual_seed(5)
    B, T = 2, 70
    num = torch.randn(B, 4, T, 64, device=DEV, generator=g)
    den = torch.rand(B, 4, T, 1, device=DEV, generator=g) * 3
    with torch.no_grad():
        out = m.finish(num, den, B, T, dt)
    sd = {k: np32(v) for k, v in m.state_dict().items()}
    p = O.RunTimeSdmParams(sd, 4, 32, 32, 4)
    want = O.rt_finish(p, np32(num), np32(den), bf16_out=dt == torch.bfloat16)
    assert out.dtype == dt and out.shape == (B, T, 256)
    if dt == torch.bfloat16:
        assert rel_bf16(np32(out), want) < 2e-3
    else:
        np.testing.assert_allclose(np32(out), want, atol=1e-5, rtol=1e-4)


def test_project_and_set_leak(cuda_ok):
    torch.manual_seed(6)
    model = S.build_onesdm("onesdm", 1000, dict(d=128, layers=1, mlp_f=352, heads=4))
    model = model.to_bf16_stream().to(DEV)
    h = torch.randn(3, 50, 128, device=DEV).to(torch.bfloat16)
    with torch.no_grad():
        lg = model.project(h)
    want = O.linear(np32(h), np32(model.emb.weight), bf16_out=True)
    assert lg.shape == (3, 50, 1000) and lg.dtype == torch.bfloat16
    assert rel_bf16(np32(lg), want) < 2e-3
    idx = torch.randint(0, 1000, (1, 20), device=DEV)
    model.set_leak(True)
    assert all(m._leak for m in model.mems)
    with pytest.raises(NotImplementedError), torch.no_grad():
        model(idx)
    model.set_leak(False)
    with torch.no_grad():
        model(idx)
