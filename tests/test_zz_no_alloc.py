"""The allocation-free decode step, sdm_rt_decode_step_noalloc, against the workspace decode step.

Some callers cannot allocate device memory on their decode path: a serving loop that owns every byte of the GPU in
a fixed pool, or a host runtime behind an FFI with no device allocator to provide a workspace.  For them the library
runs the decode step on a fixed scratch array of its own.  This test calls that entry point through the C ABI and
checks that two consecutive calls, and a third that empties some streams through its reset mask, reproduce
sdm_rt_decode_step bit for bit (the same kernels on the same inputs: output and carried state identical), and that a
request larger than the fixed scratch is refused before any launch.
It is collected last and passes alone in a fresh process as well as after the other tests.
"""
import numpy as np
import pytest
import torch

import sdmchat_b200 as S
from sdmchat_b200 import _lib

pytestmark = pytest.mark.gpu


def layer():
    torch.manual_seed(0)
    m = S.RunTimeSdm(768, heads=12, n_sub=32, d_a=32, k=16, decays=S.readme_fades(12))
    with torch.no_grad():
        torch.nn.init.normal_(m.wo.weight, std=0.02)
        torch.nn.init.normal_(m.wg.weight, std=0.5 / 768 ** 0.5)
    return m.to("cuda").to(torch.bfloat16)


def test_noalloc_decode_matches_workspace_decode(cuda_ok):
    m = layer()
    n = 8
    ref_state = m.init_state(n, "cuda")
    state = {k: v.clone() for k, v in ref_state.items()}
    p, _ = m._params(torch.bfloat16)
    lib = _lib.lib()
    g = torch.Generator(device="cuda").manual_seed(1)
    # two calls in a row (the second reads the state the first wrote), then a third that empties streams 1 and 5
    resets = [None, None, torch.tensor([0, 1, 0, 0, 0, 1, 0, 0], dtype=torch.uint8, device="cuda")]
    with torch.no_grad():
        for call, rs in enumerate(resets):
            x = (torch.randn(n, 768, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
            want = m.decode_step(x, ref_state, reset=rs, add_residual=True)
            out = torch.empty_like(x)
            rc = lib.sdm_rt_decode_step_noalloc(p, _lib.ptr(x), n, _lib.ptr(rs), 1, _lib.ptr(out),
                                                _lib.ptr(state["mem"]), _lib.ptr(state["cnt"]),
                                                _lib.ptr(state["scale"]), _lib.ptr(state["last_w"]),
                                                _lib.stream_ptr())
            assert rc == 0, lib.sdm_status_string(rc)
            torch.cuda.synchronize()
            # the same kernels on the same inputs: bit-identical output and carried state
            assert torch.equal(out, want), call
            for key in ("mem", "cnt", "scale", "last_w"):
                assert torch.equal(state[key], ref_state[key]), (call, key)
            assert float(state["cnt"].abs().sum()) > 0
        # the reset streams hold only the third token's writes: one write per selected slot
        cnt = state["cnt"] * state["scale"][..., None]
        assert torch.count_nonzero(cnt[1]) <= 12 * 16 and torch.count_nonzero(cnt[0]) > 12 * 16


def test_noalloc_rejects_requests_beyond_its_scratch(cuda_ok):
    m = layer()
    p, _ = m._params(torch.bfloat16)
    lib = _lib.lib()
    cap = lib.sdm_rt_decode_noalloc_scratch_bytes()
    assert cap == 8 << 20
    n = 1
    while lib.sdm_rt_decode_workspace_size(p, n) <= cap:
        n *= 2
    fake = torch.empty(1, device="cuda")  # never touched: the call is refused on the host
    rc = lib.sdm_rt_decode_step_noalloc(p, _lib.ptr(fake), n, None, 0, _lib.ptr(fake), _lib.ptr(fake),
                                        _lib.ptr(fake), _lib.ptr(fake), _lib.ptr(fake), _lib.stream_ptr())
    assert rc == 6  # SDM_ERR_WORKSPACE
    assert lib.sdm_rt_decode_workspace_size(p, 256) <= cap  # the benchmark's decode: 32 streams per GPU fit easily
    np.testing.assert_equal(int(lib.sdm_rt_decode_workspace_size(p, 32)) > 0, True)
