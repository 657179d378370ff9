"""ctypes binding of the C ABI (include/attention_lab_b200.h).

The library is built in-tree by `attention_lab_b200.build`. There is no fallback: if the shared object is missing or
cannot be loaded, importing the operators raises, so a silent CPU or eager path can never stand in for the kernels.
"""
from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_uint, c_void_p, POINTER
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libattention_lab_b200.so"

AL_OK, AL_EINVAL, AL_ESTATE, AL_ECUDA, AL_EUNSUPPORTED = 0, 1, 2, 3, 4
AL_F32, AL_BF16 = 0, 1

P64 = POINTER(c_int64)

# name -> argtypes, in the order of include/attention_lab_b200.h
SIGNATURES = {
    "al_last_error": [],
    "al_version": [],
    "al_device_status": [POINTER(c_uint)],
    "al_sparse_decode_step": [c_void_p, c_int64, c_int64, c_int64,
                              c_void_p, c_int64, c_int64, c_int64,
                              c_void_p, c_void_p, c_int,
                              c_void_p, c_void_p, c_void_p, c_int,
                              c_void_p, c_int64, c_int64,
                              c_void_p, c_void_p,
                              c_int, c_int, c_int, c_int, c_int, c_int,
                              c_int, c_int, c_int, c_int, c_int, c_int,
                              c_float, c_int,
                              c_void_p, c_void_p, c_void_p, c_int, c_void_p],
    "al_select_rows": [c_void_p, c_int64, c_int64, c_void_p, c_int,
                       c_void_p, c_void_p,
                       c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                       c_int, c_void_p, c_void_p, c_int, c_void_p],
    "al_gathered_attend": [c_void_p, c_int64, c_int64, c_int64,
                           c_void_p, c_void_p, c_int, c_void_p,
                           c_int, c_int, c_int, c_int, c_int, c_int, c_float,
                           c_void_p, c_int, c_void_p],
    "al_dense_decode": [c_void_p, c_int64, c_int64, c_int64,
                        c_void_p, c_void_p, c_int,
                        c_int, c_int, c_int, c_int, c_int, c_int, c_float,
                        c_void_p, c_int, c_void_p],
    "al_append_kvz": [c_void_p, c_void_p, c_int,
                      c_void_p, P64, c_void_p, P64,
                      c_int, c_void_p, c_int, c_void_p, P64,
                      c_void_p, P64, c_void_p,
                      c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p],
    "al_project_keys": [c_void_p, P64, c_void_p, c_int,
                        c_int, c_int, c_int, c_int, c_int, c_void_p, c_int, c_int, c_void_p],
    "al_project_queries": [c_void_p, P64, c_void_p, c_int,
                           c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_int, c_void_p],
    "al_candidate_scores": [c_void_p, P64, c_void_p, c_int,
                            c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p, c_int, c_void_p],
    "al_context_local_topk": [c_void_p, c_int64, c_int64, c_int64,
                              c_void_p, c_void_p, c_void_p, c_int,
                              c_void_p, c_int64, c_int64,
                              c_void_p, c_void_p,
                              c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                              c_int64, c_int, c_void_p, c_void_p, c_int, c_void_p],
    "al_context_threshold": [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                             c_int, c_int, c_void_p, c_void_p, c_void_p],
    "al_gathered_attend_partial": [c_void_p, c_int64, c_int64, c_int64,
                                   c_void_p, c_void_p, c_int, c_void_p,
                                   c_int, c_int, c_int, c_int, c_int, c_int, c_float,
                                   c_void_p, c_int, c_void_p],
    "al_lse_merge": [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_int, c_void_p],
    "al_xchg_create": [ctypes.c_size_t, POINTER(c_void_p), c_void_p],
    "al_xchg_open": [c_void_p, POINTER(c_void_p)],
    "al_xchg_close": [c_void_p],
    "al_xchg_destroy": [c_void_p],
    "al_xchg_push": [c_void_p, ctypes.c_size_t, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p],
    "al_context_threshold_peer": [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                                  c_int, c_int, c_void_p, c_void_p, c_void_p],
    "al_lse_merge_peer": [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
                          c_int, c_void_p],
    "al_context_threshold_noalloc": [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
                                     c_void_p, c_void_p],
    "al_prefill_score_topk": [c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_int, c_int, c_int,
                              c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p],
}

_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and return the library with every entry point's signature set."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH.name} is not built: run `python -m attention_lab_b200.build` "
                               "(the sparse-decode operators have no CPU fallback)")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, args in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_char_p if name == "al_last_error" else c_int
        _lib = lib
    return _lib


def check(rc: int) -> None:
    """Map a status code to the exception the reference raises for the same condition."""
    if rc == AL_OK:
        return
    msg = load().al_last_error().decode(errors="replace")
    if rc in (AL_EINVAL, AL_EUNSUPPORTED):
        raise ValueError(msg)
    raise RuntimeError(msg)


def strides(t, n: int):
    """First n element strides of a tensor as a ctypes int64 array."""
    arr = (c_int64 * n)(*[int(s) for s in t.stride()[:n]])
    return arr


def device_status() -> int:
    """Synchronise the current device and return (and clear) the kernels' error bits."""
    v = c_uint(0)
    check(load().al_device_status(ctypes.byref(v)))
    return int(v.value)
