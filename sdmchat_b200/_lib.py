"""ctypes binding of libsdm_b200.so (the C ABI declared in include/sdm_b200.h).

The library is loaded from this package directory.  There is no fallback: if it is missing or was built for
another architecture, every operation raises.  torch is used only for device memory, the current stream and
workspace buffers (from its caching allocator, so repeated calls do not cudaMalloc).
"""
import ctypes
import os

import torch

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libsdm_b200.so")

SDM_F32, SDM_BF16 = 0, 1
ABI_VERSION = 3

c_int, c_int64, c_float, c_size_t, c_void_p, c_double = (ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t,
                                                          ctypes.c_void_p, ctypes.c_double)


class RtParams(ctypes.Structure):
    """sdm_rt_params (include/sdm_b200.h)."""
    _fields_ = [("d", c_int), ("heads", c_int), ("n_sub", c_int), ("d_a", c_int), ("k", c_int),
                ("write_gate", c_int), ("read_sum", c_int), ("out_norm", c_int),
                ("read_eps", c_float), ("out_norm_eps", c_float), ("norm_eps", c_float), ("dtype", c_int),
                ("norm_w", c_void_p), ("w_proj", c_void_p), ("wg_bias", c_void_p), ("wo", c_void_p),
                ("keys1", c_void_p), ("keys2", c_void_p), ("addr_b", c_void_p), ("log_scale", c_void_p),
                ("decay", c_void_p), ("onorm_w", c_void_p)]


class TsParams(ctypes.Structure):
    """sdm_ts_params (include/sdm_b200.h)."""
    _fields_ = [("d", c_int), ("heads", c_int), ("n_sub", c_int), ("d_a", c_int), ("k", c_int),
                ("norm_eps", c_float), ("dtype", c_int),
                ("norm_w", c_void_p), ("wq", c_void_p), ("keys1", c_void_p), ("keys2", c_void_p),
                ("values", c_void_p), ("log_scale", c_void_p), ("wo", c_void_p)]


P = c_void_p
_SIGS = {
    "sdm_abi_version": (c_int, []),
    "sdm_status_string": (ctypes.c_char_p, [c_int]),
    "sdm_kernel_launch_count": (c_int64, []),
    "sdm_profile_begin": (c_int, []),
    "sdm_profile_end": (c_int, []),
    "sdm_profile_group": (c_int, [c_int, ctypes.c_char_p, ctypes.c_char_p, c_int, ctypes.POINTER(c_int),
                                  ctypes.POINTER(c_double)]),
    "sdm_device_status": (c_int, [P]),
    "sdm_set_wait_limit_ns": (c_int, [ctypes.c_uint64]),
    "sdm_wait_probe": (c_int, [P, P]),
    "sdm_pk_address": (c_int, [P, P, P, c_int64, c_int, c_int, c_int, c_int, P, P, P]),
    "sdm_rmsnorm": (c_int, [P, P, c_int64, c_int, c_float, c_int, P, P]),
    "sdm_rt_forward_workspace_size": (c_size_t, [ctypes.POINTER(RtParams), c_int, c_int]),
    "sdm_rt_forward": (c_int, [ctypes.POINTER(RtParams), P, c_int, c_int, P, c_int, P, P, P, P, P, P, P, P, P, P, P, P,
                               P, c_size_t, P]),
    "sdm_rt_scan_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int]),
    "sdm_rt_scan": (c_int, [P, P, P, P, P, c_int64, P, P, c_int, c_int, c_int, c_int, c_int, c_int, P, P, P, P, P,
                            P, P, c_size_t, P]),
    "sdm_rt_finish_workspace_size": (c_size_t, [ctypes.POINTER(RtParams), c_int64]),
    "sdm_rt_finish": (c_int, [ctypes.POINTER(RtParams), P, P, c_int64, P, P, P, c_size_t, P]),
    "sdm_rt_decode_workspace_size": (c_size_t, [ctypes.POINTER(RtParams), c_int]),
    "sdm_rt_decode_step": (c_int, [ctypes.POINTER(RtParams), P, c_int, P, c_int, P, P, P, P, P, P, c_size_t, P]),
    "sdm_rt_decode_noalloc_scratch_bytes": (c_size_t, []),
    "sdm_rt_decode_step_noalloc": (c_int, [ctypes.POINTER(RtParams), P, c_int, P, c_int, P, P, P, P, P, P]),
    "sdm_ts_forward_workspace_size": (c_size_t, [ctypes.POINTER(TsParams), c_int64]),
    "sdm_ts_forward": (c_int, [ctypes.POINTER(TsParams), P, c_int64, c_int, P, P, P, P, P, c_size_t, P]),
    "sdm_swiglu_pack": (c_int, [P, P, c_int, c_int, c_int, P, P]),
    "sdm_swiglu_forward_workspace_size": (c_size_t, [c_int64, c_int, c_int, c_int]),
    "sdm_swiglu_forward": (c_int, [P, P, P, P, c_int64, c_int, c_int, c_float, c_int, c_int, P, P, c_size_t, P]),
    "sdm_swiglu_workspace_size": (c_size_t, [c_int64, c_int, c_int, c_int]),
    "sdm_swiglu_block": (c_int, [P, P, P, P, P, c_int64, c_int, c_int, c_float, c_int, P, P, c_size_t, P]),
    "sdm_tied_head_workspace_size": (c_size_t, [c_int64, c_int, c_int, c_int]),
    "sdm_tied_logits": (c_int, [P, P, P, c_int64, c_int, c_int, c_float, c_int, P, P, c_size_t, P]),
    "sdm_tied_ce_sum": (c_int, [P, P, P, P, c_int64, c_int, c_int, c_float, c_int, P, P, c_size_t, P]),
    "sdm_tied_argmax": (c_int, [P, P, P, c_int64, c_int, c_int, c_float, c_int, P, P, c_size_t, P]),
    "sdm_tied_project": (c_int, [P, P, c_int64, c_int, c_int, c_int, P, P]),
    "sdm_embed": (c_int, [P, P, c_int64, c_int, c_int, c_int, P, P, P]),
    "sdm_gemm": (c_int, [P, P, c_int64, c_int, c_int, c_int, P, P]),
}

_lib = None


def lib():
    """Load libsdm_b200.so once; raise if it is absent or its ABI version differs."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m sdmchat_b200.build` "
                               "(there is no CPU or PyTorch fallback for this path)")
        h = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        if h.sdm_abi_version() != ABI_VERSION:
            raise RuntimeError(f"libsdm_b200 ABI {h.sdm_abi_version()} != {ABI_VERSION}: rebuild the library")
        _lib = h
    return _lib


def exported_symbols():
    """Names of every function the header declares (checked against the library by the CPU tests)."""
    return list(_SIGS)


def check(status, what):
    if status != 0:
        msg = lib().sdm_status_string(status).decode()
        raise RuntimeError(f"{what} failed: {msg} (status {status})")


def ptr(t):
    """Device pointer of a CUDA tensor (None -> NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("libsdm_b200 takes device tensors only")
    return ctypes.c_void_p(t.data_ptr())


def stream_ptr(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def workspace(nbytes, device):
    """A workspace buffer from torch's caching allocator (no cudaMalloc once warm)."""
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def dtype_code(dt):
    if dt == torch.float32:
        return SDM_F32
    if dt == torch.bfloat16:
        return SDM_BF16
    raise TypeError(f"libsdm_b200 computes in float32 or bfloat16, not {dt}")


def profile_groups():
    """After sdm_profile_end(): list of (kernel, tag, launches, total_ms)."""
    n = lib().sdm_profile_end()
    if n < 0:
        raise RuntimeError("sdm_profile_end: CUDA error while reading launch events")
    out = []
    for i in range(n):
        k, t = ctypes.create_string_buffer(64), ctypes.create_string_buffer(64)
        cnt, ms = c_int(0), c_double(0.0)
        check(lib().sdm_profile_group(i, k, t, 64, ctypes.byref(cnt), ctypes.byref(ms)), "sdm_profile_group")
        out.append((k.value.decode(), t.value.decode(), cnt.value, ms.value))
    return out
