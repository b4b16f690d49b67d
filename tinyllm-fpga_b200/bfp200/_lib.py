"""ctypes binding of libbfp200.so (C ABI declared in include/bfp200.h).

The library is built in-tree (bfp200/lib/libbfp200.so, see bfp200.build).  There
is no fallback: if the library cannot be loaded, or no sm_100 GPU is present,
every compute call raises ``BfpError``.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

LIB_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib")
LIB_PATH = os.path.join(LIB_DIR, "libbfp200.so")

# error codes (bfp200.h)
OK, EINVAL, ENODEV, ECUDA, EIMAGE, ESTATE, ETIMEOUT, ENOMEM = 0, -1, -2, -3, -4, -5, -6, -7
NSTAGES = 12


class BfpError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"bfp200 error {code}: {msg}")
        self.code = code


class Cfg(C.Structure):
    _fields_ = [("D", C.c_int), ("H_Q", C.c_int), ("H_KV", C.c_int), ("HD", C.c_int), ("FFN", C.c_int),
                ("NL", C.c_int), ("VOCAB", C.c_int), ("MAX_CTX", C.c_int), ("NPROMPT_MAX", C.c_int),
                ("max_seqs", C.c_int), ("rope_base", C.c_double), ("eps", C.c_double)]


_P = C.c_void_p
_I = C.c_int
_Z = C.c_size_t
_D = C.c_double

# name -> argtypes (all return int)
SIGNATURES = {
    "bfp200_last_error": [C.c_char_p, _Z],
    "bfp200_open": [C.POINTER(Cfg), _I, C.POINTER(_P)],
    "bfp200_close": [_P],
    "bfp200_load_image": [_P, _P, _Z],
    "bfp200_load_rom": [_P, _I, _P, _Z],
    "bfp200_generate": [_P, _P, _P, _I, _I, _I, _P],
    "bfp200_generate_multi": [_P, _I, _P, _P, _I, _I, _I, _P],
    "bfp200_uncertified_steps": [_P, C.POINTER(C.c_longlong)],
    "bfp200_last_timing": [_P, C.POINTER(_D), C.POINTER(_D)],
    "bfp200_last_launches": [_P, C.POINTER(C.c_longlong)],
    "bfp200_tile_quantize": [_P, _P, _Z, _P, _P],
    "bfp200_tile_decode": [_P, _P, _P, _Z, _P],
    "bfp200_matvec": [_P, _P, _P, _P, _P, _I, _I, _I, _P, _P],
    "bfp200_rmsnorm_fp": [_P, _P, _P, _I, _I, _D, _P],
    "bfp200_silu_fp": [_P, _P, _Z, _P],
    "bfp200_softmax_fp": [_P, _P, _I, _I, _P],
    "bfp200_rope_fp": [_P, _P, _P, _I, _I, _D, _P],
    "bfp200_pairwise_sum": [_P, _P, _I, _I, _P],
    "bfp200_rope_table": [_P, _I, _I, _D],
    "bfp200_fwd_layer": [_P, _I, _P, _P, _P, _I, _P, _P, _I, _P, _P],
    "bfp200_fwd_layer_decode": [_P, _I, _P, _P, _P, _I, _P, _P, _I, _P, _P],
    "bfp200_wait_probe": [_P, _I],
    "bfp200_stage_dims": [_P, _P],
    "bfp200_time_matmuls": [_P, _I, _I, C.POINTER(_D), C.POINTER(_I)],
    "bfp200_profile_forward": [_P, _I, _I, _P, _P],
    "bfp200_matvec_noalloc": [_P, _P, _P, _P, _I, _I, _I, _P, _P, _P],
    "bfp200_generate_sampled": [_P, _P, _P, _I, _I, _D, _I, C.c_uint32, _P],
    "bfp200_sample_uniforms": [C.c_uint32, _I, _P],
    "bfp200_matvec_timed": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _P, _P, C.POINTER(_D)],
    "bfp200_rtl_matvec": [_P, _P, _P, _P, _P, _I, _I, _I, _P, _P],
    "bfp200_rtl_rmsnorm": [_P, _P, _P, _P, _P, _I, _I, _P, _P],
    "bfp200_rtl_rope": [_P, _P, _P, _P, _I, _I, _P, _P, _P],
    "bfp200_rtl_softmax": [_P, _P, _P, _I, _I, _P, _P, _P],
    "bfp200_rtl_swiglu": [_P, _P, _P, _P, _P, _Z, _P, _P, _P],
    "bfp200_rtl_residual": [_P, _P, _P, _P, _P, _Z, _P, _P],
    "bfp200_nccl_unique_id": [_P],
    "bfp200_head_shard": [_P, _P, _I, _I],
    "bfp200_head_shard_group": [_P, _I],
    "bfp200_generate_sharded": [_P, _I, _P, _P, _I, _I, _I, _P],
}
NCCL_ID_BYTES = 128


def _nccl_hint():
    """Points the library's run-time NCCL loader at the NCCL that torch
    ships (nvidia-nccl wheel) unless the caller chose one."""
    if "BFP200_NCCL_LIB" in os.environ:
        return
    try:
        import importlib.util
        spec = importlib.util.find_spec("nvidia.nccl")
    except (ImportError, ValueError):
        return
    for d in (spec.submodule_search_locations or []) if spec else []:
        cand = os.path.join(d, "lib", "libnccl.so.2")
        if os.path.exists(cand):
            os.environ["BFP200_NCCL_LIB"] = cand
            return

_lib = None


def lib():
    """Loads libbfp200.so (once).  Raises BfpError if it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise BfpError(ENODEV, f"{LIB_PATH} not built (run bfp200.build.build())")
        _nccl_hint()
        L = C.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = C.c_int
        L.bfp200_default_cfg.argtypes = [C.POINTER(Cfg)]
        L.bfp200_default_cfg.restype = None
        _lib = L
    return _lib


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    lib().bfp200_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc):
    if rc != OK:
        raise BfpError(rc, last_error())


def ptr(a):
    """Address of a C-contiguous numpy array (None -> NULL)."""
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "array must be C-contiguous"
    return a.ctypes.data


def arr(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)
