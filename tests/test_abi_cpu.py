"""The C ABI library without a GPU: it loads, exports every symbol include/sdm_b200.h declares, and rejects bad
arguments on the host (before anything is launched) with the documented status codes."""
import ctypes
import os
import re

import pytest
import torch

import sdmchat_b200 as S
from sdmchat_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "sdm_b200.h")


def header_functions():
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(sdm_\w+)\s*\(", txt)))


def test_library_exports_every_declared_function():
    lib = _lib.lib()
    declared = header_functions()
    assert len(declared) >= 19
    for name in declared:
        assert hasattr(lib, name), name
    assert sorted(_lib.exported_symbols()) == declared


def test_abi_version_and_status_strings():
    lib = _lib.lib()
    assert lib.sdm_abi_version() == _lib.ABI_VERSION
    for code in range(7):
        assert lib.sdm_status_string(code)
    assert b"unknown" in lib.sdm_status_string(99)


def test_host_side_argument_errors():
    lib = _lib.lib()
    fake = ctypes.c_void_p(0x10000)  # never dereferenced: every call below is rejected before a launch
    # null pointers
    assert lib.sdm_pk_address(None, fake, fake, 4, 1, 32, 32, 16, None, fake, None) == 1
    # d_a not supported / odd, k out of range, n_sub out of range
    assert lib.sdm_pk_address(fake, fake, fake, 4, 1, 5, 32, 16, None, fake, None) == 2
    assert lib.sdm_pk_address(fake, fake, fake, 4, 1, 32, 32, 33, None, fake, None) == 2
    assert lib.sdm_pk_address(fake, fake, fake, 4, 1, 32, 129, 16, None, fake, None) == 2
    assert lib.sdm_rmsnorm(fake, fake, 4, 16, 1e-6, 7, fake, None) == 1
    assert lib.sdm_gemm(fake, fake, 4, 0, 8, 1, fake, None) == 2
    # the scan: too many slots for the shared-memory state
    assert lib.sdm_rt_scan(fake, fake, fake, fake, fake, 64, fake, None, 1, 8, 1, 128, 64, 16, None, None, fake, fake,
                           None, None, fake, 1 << 20, None) == 2
    # a carried state needs both mem and cnt
    assert lib.sdm_rt_scan(fake, fake, fake, fake, fake, 64, fake, None, 1, 8, 1, 32, 64, 16, fake, None, fake, fake,
                           None, None, fake, 1 << 20, None) == 1
    # the scan's chunk lists need their workspace
    need = lib.sdm_rt_scan_workspace_size(2, 2048, 12, 16)
    assert need == 2 * 12 * 32 * lib.sdm_rt_scan_workspace_size(1, 64, 1, 16)
    assert lib.sdm_rt_scan(fake, fake, fake, fake, fake, 768, fake, None, 2, 2048, 12, 32, 64, 16, None, None, fake,
                           fake, None, None, fake, need - 1, None) == 6


def rt_params(d=768, heads=12, n_sub=32, d_a=32, k=16, dtype=_lib.SDM_BF16):
    return _lib.RtParams(d=d, heads=heads, n_sub=n_sub, d_a=d_a, k=k, write_gate=1, read_sum=0, out_norm=1,
                         read_eps=1e-3, out_norm_eps=1e-2, norm_eps=1e-6, dtype=dtype,
                         **{n: 0x10000 for n in ("norm_w", "w_proj", "wg_bias", "wo", "keys1", "keys2", "addr_b",
                                                 "log_scale", "decay", "onorm_w")})


def test_workspace_queries_and_too_small_workspace():
    lib = _lib.lib()
    p = rt_params()
    need = lib.sdm_rt_forward_workspace_size(p, 2, 256)
    # hx (bf16) + projection (fp32, 1548 cols) + 4 selection arrays + num/den + r (bf16)
    N = 512
    assert need >= N * 768 * 2 + N * 1548 * 4 + 4 * N * 12 * 16 * 4 + N * 768 * 4 + N * 768 * 2
    fake = ctypes.c_void_p(0x10000)
    st = lib.sdm_rt_forward(p, fake, 2, 256, None, 0, fake, None, None, None, None, None, None, None, None, None,
                            None, None, fake, need - 1, None)
    assert st == 6
    bad = rt_params(heads=7)
    assert lib.sdm_rt_forward_workspace_size(bad, 2, 256) == 0
    assert lib.sdm_rt_forward(bad, fake, 2, 256, None, 0, fake, None, None, None, None, None, None, None, None, None,
                              None, None, fake, 1 << 30, None) == 2
    assert lib.sdm_rt_decode_workspace_size(p, 32) > 0
    assert lib.sdm_tied_head_workspace_size(65536, 768, 32768, 1) > 4096 * 32768 * 4


def test_modules_need_device_tensors():
    m = S.RunTimeSdm(32, heads=4, n_sub=6, d_a=8, k=5, decays=(0.0, 0.7, 0.95, 1.0))
    with torch.no_grad(), pytest.raises(ValueError):
        m(torch.randn(1, 4, 32))


def test_forward_only_guard():
    m = S.RunTimeSdm(32, heads=4, n_sub=6, d_a=8, k=5, decays=(0.0, 0.7, 0.95, 1.0))
    with pytest.raises(NotImplementedError):
        m(torch.randn(1, 4, 32, requires_grad=True))
