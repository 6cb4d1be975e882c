"""The drop-in modules construct exactly as the reference's: same state_dict keys, shapes and seeded weights."""
import numpy as np
import torch

import sdmchat_b200 as S
from goldens import load, params


def test_runtime_sdm_constructor_reproduces_reference_weights():
    """The CPU-runnable benchmark case (RunTimeSdm 256, 4 heads, k 4) built the reference's way
    (torch.manual_seed(0), Uniform[0.90, 0.999] fades drawn first) gives the reference module's exact weights (tests/golden/rt_config1.npz holds its state_dict)."""
    g = load("rt_config1")
    torch.manual_seed(0)
    decays = torch.empty(4).uniform_(0.90, 0.999)
    m = S.RunTimeSdm(256, heads=4, n_sub=32, d_a=32, k=4, decays=tuple(decays.tolist()))
    ref = params(g)
    sd = m.state_dict()
    assert sorted(sd) == sorted(ref)
    for k, v in sd.items():
        np.testing.assert_array_equal(v.numpy(), ref[k], err_msg=k)


def test_trained_sdm_and_lm_state_dict_layout():
    for name in ("lm_partial", "lm_full"):
        g = load(name)
        ref = params(g)
        arm = str(g["arm"])
        cfg = dict(d=64, layers=2, mlp_f=176, heads=4, n_sub=8, d_a=8, k=4, chunk=16)
        model = S.build_onesdm(arm, int(g["V"]), cfg)
        sd = model.state_dict()
        assert sorted(sd) == sorted(ref), name
        for k, v in sd.items():
            assert tuple(v.shape) == ref[k].shape, k


def test_lm_init_matches_reference_seeded():
    """OneSdmLM's init order equals the reference's: with the same seed, the unperturbed tensors agree."""
    g = load("lm_partial")
    torch.manual_seed(21)
    model = S.build_onesdm("onesdm", 256, dict(d=64, layers=2, mlp_f=176, heads=4, n_sub=8, d_a=8, k=4, chunk=16))
    ref = params(g)
    for k in ("mems.0.wk.weight", "mems.1.wq.weight", "mlps.0.gate.weight", "mems.0.keys1", "mems.1.addr_b"):
        want = ref[k]
        got = model.state_dict()[k].float().numpy()
        # the fixture stores these bf16-rounded; compare at bf16 precision
        np.testing.assert_allclose(got, want, rtol=1e-2, atol=1e-6, err_msg=k)


def test_defaults_and_helpers():
    assert S.matched_sdm_n_sub(768, 2048, 4, 32) == 72
    assert S.mlp_width(768) == 2048 and S.mlp_width(256) == 688
    assert S.readme_fades(12) == (0.0, 0.8, 0.99, 1.0) * 3
    m = S.build_onesdm("onesdm_allsdm", 512, dict(d=768, layers=1, mlp_f=2048, heads=12, decays=S.readme_fades(12)))
    assert m.sdm_n_sub == 72 and m.sdms[0].dh == 192 and m.sdms[0].d_a == 32
    assert S.decode_state_bytes(m) == 1 * 12 * 1024 * 65 * 4
