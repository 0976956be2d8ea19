"""ctypes bindings for libboa_b200.so (declared in include/boa_b200.h).

The library is built in-tree by ``boa_b200.build.build()`` (nvcc, sm_100a).
There is no CPU fallback: if the library or a GPU is missing, every entry point
raises ``RuntimeError`` (mirroring the reference, whose extension is required
at import time, gpu_range_coder.py:381).
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
# BOA_B200_LIB overrides the library path (e.g. a build with BOA_PHASE_PROFILE)
LIB_PATH = os.environ.get("BOA_B200_LIB") or os.path.join(_HERE, "libboa_b200.so")

BOA_OK = 0
BOA_ERR_ARG = 1
BOA_ERR_CUDA = 2
BOA_ERR_OVERFLOW = 3
BOA_ERR_TIMEOUT = 4
BOA_ERR_UNSUPPORTED = 5
BOA_ERR_RANGE = 6

BOA_QUANT_REF = 0
BOA_QUANT_BQ = 1

BOA_WEIGHTS_TF32 = 0
BOA_WEIGHTS_BF16 = 1
BOA_WEIGHTS_F16 = 2
BOA_WEIGHTS_TF32X3 = 3
BOA_WEIGHTS_F16X2 = 4

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t

# name -> argtypes (restype int unless listed in _RESTYPES)
SIGNATURES = {
    "boa_last_error": [],
    "boa_abi_version": [],
    "boa_rc_create": [_P, _I, _I, _I, _I, _I, _I],
    "boa_rc_destroy": [_P],
    "boa_rc_info": [_P, _P, _P, _P, _P, _P],
    "boa_rc_load": [_P, _P, _P, _P],
    "boa_rc_set_sizes": [_P, _P, _P],
    "boa_rc_get_sizes": [_P, _P, _P],
    "boa_rc_get_words": [_P, _P, _P],
    "boa_rc_device_buffers": [_P, _P, _P],
    "boa_rc_encode_step": [_P, _P, _P, _P, _P],
    "boa_rc_finalize": [_P, _P],
    "boa_rc_init_decoder": [_P, _P],
    "boa_rc_decode_step": [_P, _P, _P, _P, _P],
    "boa_rc_encode_steps": [_P, _I, _I, _P, _I64, _P, _I64, _P, _I64, _P],
    "boa_rc_decode_steps": [_P, _I, _I, _P, _I64, _P, _I64, _P, _I64, _P],
    "boa_rc_encode_noalloc": [_I, _I, _I, _I, _P, _P, _P, _P, _I, _P, _P],
    "boa_model_create": [_P, _I, _I, _I, _P, _SZ, _I, _I],
    "boa_model_destroy": [_P],
    "boa_model_workspace_bytes": [_P, _I],
    "boa_model_info": [_P, _P, _P, _P, _P, _P],
    "boa_model_set_time_block": [_P, _I],
    "boa_model_time_block": [_P, _I, _I, _P],
    "boa_model_status": [_P, _P],
    "boa_diag_timeout": [_I64, _I],
    "boa_diag_gemm": [_I, _I, _I, _P, _P, _P, _I],
    "boa_model_step": [_P, _I, _P, _P, _P, _SZ, _P],
    "boa_model_logits": [_P, _I, _I, _P, _P, _P, _SZ, _P],
    "boa_codec_encode": [_P, _I, _P, _I64, _P, _P, _I, _P, _I, _P, _SZ, _P],
    "boa_codec_decode": [_P, _I, _P, _I, _P, _P, _P, _P, _I64, _I, _P, _SZ, _P],
    "boa_codec_encode_range": [_P, _I, _P, _I64, _P, _I, _I, _P, _I, _P, _I, _P, _SZ, _P],
    "boa_codec_decode_range": [_P, _I, _P, _I, _P, _P, _I, _I, _P, _P, _I64, _I, _P, _SZ, _P],
}
_RESTYPES = {
    "boa_last_error": ctypes.c_char_p,
    "boa_model_workspace_bytes": ctypes.c_size_t,
}

_lib = None
_lock = threading.Lock()


class BoaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[boa_b200 error {code}] {msg}")
        self.code = code


def load():
    """Load libboa_b200.so (raises if it was not built)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libboa_b200.so not found at {LIB_PATH}; run __graft_entry__.build() "
                "(nvcc, sm_100a). This build has no CPU fallback.")
        lib = ctypes.CDLL(LIB_PATH)
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name, None)
            if fn is None:
                continue
            fn.argtypes = argtypes
            fn.restype = _RESTYPES.get(name, ctypes.c_int)
        _lib = lib
        return lib


def exported_symbols():
    lib = load()
    return {n for n in SIGNATURES if getattr(lib, n, None) is not None}


def check(rc: int, what: str = ""):
    if rc != BOA_OK:
        msg = load().boa_last_error()
        msg = msg.decode() if msg else ""
        raise BoaError(rc, f"{what}: {msg}" if what else msg)


def call(name: str, *args):
    fn = getattr(load(), name)
    rc = fn(*args)
    check(rc, name)
    return rc


def require_cuda(device=None):
    import torch
    if not torch.cuda.is_available():
        raise RuntimeError("boa_b200 requires a CUDA GPU (sm_100a); no CPU fallback exists")
    load()


def stream_ptr(device=None) -> int:
    import torch
    return int(torch.cuda.current_stream(device).cuda_stream)
