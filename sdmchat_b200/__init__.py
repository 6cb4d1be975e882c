"""sdmchat_b200: the SDMCHAT run-time sparse-distributed-memory path on NVIDIA B200 (sm_100a).

The compute is libsdm_b200.so (hand-written CUDA, C ABI in include/sdm_b200.h); this package holds the drop-in
PyTorch modules that call it (same constructors and state_dict keys as the reference's) and its ctypes binding.
"""
from .modules import RMSNorm, RunTimeSdm, SwiGLU, TrainedSdm, matched_sdm_n_sub, pk_address, trained_sdm_params
from .lm import (ALLSDM_ARMS, DEFAULTS, OneSdmLM, allsdm_n_sub, build_onesdm, decode_state_bytes, lm_kwargs,
                 mlp_width, readme_fades)

__all__ = ["RMSNorm", "RunTimeSdm", "SwiGLU", "TrainedSdm", "matched_sdm_n_sub", "pk_address", "trained_sdm_params",
           "ALLSDM_ARMS", "DEFAULTS", "OneSdmLM", "allsdm_n_sub", "build_onesdm", "decode_state_bytes", "lm_kwargs",
           "mlp_width", "readme_fades"]
