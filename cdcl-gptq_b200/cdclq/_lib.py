"""Loader of the sm_100a CUDA library (libcdclq_cuda.so, built in-tree by cdcl-gptq_b200/build.py).

There is deliberately no fallback: if the shared library is missing or cannot be loaded, every compute call
raises.  Loading the library does not need a GPU; computing does (the C ABI returns CDCLQ_ERR_CUDA).
"""
import ctypes
import os

from .abi import CBatchInput, CBatchLayer, CConfig, CLayerStats, CModelOpts, CModelReport, CRunProfile

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcdclq_cuda.so")

_lib = None

P = ctypes.c_void_p
SZ = ctypes.c_size_t
I32 = ctypes.c_int
CFG = ctypes.POINTER(CConfig)

# name -> (restype, argtypes); every symbol declared in include/cdclq.h
SIGNATURES = {
    "cdclq_config_default": (None, [CFG]),
    "cdclq_effective_group": (SZ, [CFG, SZ]),
    "cdclq_num_groups": (SZ, [CFG, SZ]),
    "cdclq_validate": (I32, [CFG, SZ]),
    "cdclq_last_error": (ctypes.c_char_p, []),
    "cdclq_prep_cache_new": (P, []),
    "cdclq_prep_cache_free": (None, [P]),
    "cdclq_quantize_layer": (I32, [P, SZ, SZ, P, P, ctypes.c_char_p, CFG, P, P, P, P, P, P,
                                   ctypes.POINTER(CLayerStats)]),
    "cdclq_quantize_layer_ex": (I32, [P, SZ, SZ, P, P, ctypes.c_char_p, CFG, P, P, P, P, P, P,
                                      ctypes.POINTER(CLayerStats), P]),
    "cdclq_row_chunk": (SZ, [CFG, SZ]),
    "cdclq_quantize_batch": (I32, [ctypes.POINTER(CBatchInput), SZ, ctypes.POINTER(CBatchLayer), SZ, CFG, I32, P]),
    "cdclq_widen_to_f32_device": (I32, [P, I32, SZ, P, P]),
    "cdclq_first_non_finite_device": (I32, [P, SZ, P, P]),
    "cdclq_check_matrix_device": (I32, [P, SZ, ctypes.c_char_p, P]),
    "cdclq_pack_device": (I32, [P, SZ, SZ, SZ, P, P, P]),
    "cdclq_encode_groups_device": (I32, [P, P, SZ, P, P, P]),
    "cdclq_prepare_factors": (I32, [ctypes.POINTER(CBatchInput), SZ, P, SZ, CFG, P, I32, P]),
    "cdclq_quantize_batch_prepared": (I32, [ctypes.POINTER(CBatchInput), SZ, P, ctypes.POINTER(CBatchLayer), SZ, CFG,
                                            I32, P]),
    "cdclq_cholesky_lower": (I32, [P, SZ]),
    "cdclq_tri_inverse_lower": (I32, [P, SZ, P]),
    "cdclq_upper_chol_of_inverse": (I32, [P, SZ, P]),
    "cdclq_gram_accumulate": (I32, [P, P, SZ, SZ, P]),
    "cdclq_gram_accumulate_bf16_device": (I32, [P, SZ, SZ, P, I32, P]),
    "cdclq_gram_accumulate_half_device": (I32, [P, I32, SZ, SZ, P, I32, P]),
    "cdclq_column_scores_device": (I32, [P, SZ, SZ, P, P, P]),
    "cdclq_prepare_layer_factors": (I32, [ctypes.POINTER(CBatchInput), SZ, ctypes.POINTER(CBatchLayer), SZ, P, SZ, CFG,
                                          P, I32, P]),
    "cdclq_gram_accumulate_device": (I32, [P, P, SZ, SZ, P, P]),
    "cdclq_gram_accumulate_device_noalloc": (I32, [P, P, SZ, SZ, P, P]),
    "cdclq_proxy_loss": (I32, [P, P, SZ, SZ, P, P]),
    "cdclq_rtn_layer": (I32, [P, SZ, SZ, CFG, P]),
    "cdclq_find_params": (I32, [P, SZ, SZ, ctypes.c_uint32, I32, P, P]),
    "cdclq_row_bytes": (SZ, [SZ, SZ, P]),
    "cdclq_pack": (I32, [P, SZ, SZ, SZ, P, P]),
    "cdclq_unpack_dequant": (I32, [P, SZ, SZ, SZ, P, P, P, P, P]),
    "cdclq_runtime_unique_id": (I32, [P]),
    "cdclq_runtime_create": (I32, [I32, I32, I32, P, ctypes.c_double, ctypes.POINTER(P)]),
    "cdclq_runtime_destroy": (None, [P]),
    "cdclq_runtime_stream": (P, [P]),
    "cdclq_runtime_quantize_batch": (I32, [P, ctypes.POINTER(CBatchInput), SZ, ctypes.POINTER(CBatchLayer), SZ, CFG, I32,
                                           I32]),
    "cdclq_shard_rows": (None, [SZ, SZ, I32, I32, SZ, ctypes.POINTER(SZ), ctypes.POINTER(SZ)]),
    "cdclq_assign_owners": (None, [P, SZ, I32, I32, P]),
    "cdclq_quantize_model": (I32, [P, ctypes.POINTER(CModelOpts), ctypes.POINTER(CModelReport)]),
    "cdclq_dequantize_packed": (I32, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p,
                                      ctypes.POINTER(ctypes.c_uint64)]),
    "cdclq_launch_count": (ctypes.c_uint64, []),
    "cdclq_last_run_profile": (I32, [ctypes.POINTER(CRunProfile)]),
    "cdclq_version": (ctypes.c_char_p, []),
}


class CdclqError(RuntimeError):
    """A failed library call; `.code` is the CDCLQ_ERR_* status."""

    def __init__(self, code, msg):
        super().__init__(msg)
        self.code = code


def lib():
    """The loaded library (loaded once).  Raises if libcdclq_cuda.so is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                "libcdclq_cuda.so is not built (expected at %s); run `python cdcl-gptq_b200/build.py`" % LIB_PATH)
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_run_profile():
    p = CRunProfile()
    check(lib().cdclq_last_run_profile(ctypes.byref(p)))
    return p.as_dict()


def check(rc):
    if rc != 0:
        msg = lib().cdclq_last_error().decode("utf-8", "replace")
        raise CdclqError(rc, msg)
    return rc
