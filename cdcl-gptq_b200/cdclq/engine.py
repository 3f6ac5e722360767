"""`engine.rs` surface over the CUDA library: quantize_layer, PrepCache, proxy_loss, rtn_layer.

Mirrors src/engine.rs:690-838: same names, same argument meaning, same error texts (raised as CdclqError,
whose `.code` is the CDCLQ_ERR_* status).  All arithmetic runs in libcdclq_cuda.so on the GPU.
"""
import ctypes

import numpy as np

from ._lib import CdclqError, check, lib
from .abi import CLayerStats, Config, LayerStats, effective_group, num_groups
from .quant import QLayer


def _p(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


class PrepCache:
    """One-entry memo of the prepared factors (src/engine.rs:220-223): keyed by (hessian key, permutation)."""

    def __init__(self):
        self._h = lib().cdclq_prep_cache_new()

    def close(self):
        if self._h:
            lib().cdclq_prep_cache_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h


def validate(cfg: Config, n: int):
    """src/engine.rs:240-258."""
    c = cfg.to_c()
    check(lib().cdclq_validate(ctypes.byref(c), n))


def row_chunk(cfg: Config, d_out: int) -> int:
    """src/engine.rs:768-770."""
    c = cfg.to_c()
    return int(lib().cdclq_row_chunk(ctypes.byref(c), d_out))


def quantize_layer(w, d_out, d_in, h, m=None, hkey="", cfg: Config = None, cache: PrepCache = None,
                   return_chunk_passes=False):
    """engine::quantize_layer (src/engine.rs:690-799).

    w: d_out x d_in f32 (original order); h: d_in x d_in f32; m: optional d_in x d_in f32.
    Returns (QLayer, LayerStats) [, chunk_passes].
    """
    cfg = cfg or Config()
    w = np.ascontiguousarray(np.asarray(w, dtype=np.float32).reshape(-1))
    h = np.ascontiguousarray(np.asarray(h, dtype=np.float32).reshape(-1))
    if w.size != d_out * d_in:
        raise CdclqError(-3, "assertion failed: w.len() == d_out * n")
    if h.size != d_in * d_in:
        raise CdclqError(-3, "assertion failed: h.len() == n * n")
    mm = None
    if m is not None:
        mm = np.ascontiguousarray(np.asarray(m, dtype=np.float32).reshape(-1))
        if mm.size != d_in * d_in:
            raise CdclqError(-3, "assertion failed: mm.len() == n * n")
    c = cfg.to_c()
    ng = num_groups(cfg, d_in)
    perm = np.zeros(d_in, np.uint32)
    gbits = np.zeros(ng, np.uint8)
    codes = np.zeros((d_out, d_in), np.uint8)
    scales = np.zeros((d_out, ng), np.float32)
    zeros = np.zeros((d_out, ng), np.float32)
    st = CLayerStats()
    rc = row_chunk(cfg, d_out)
    passes = np.zeros((d_out + rc - 1) // rc, np.uint32)
    check(lib().cdclq_quantize_layer_ex(_p(w), d_out, d_in, _p(h), _p(mm), (hkey or "").encode(), ctypes.byref(c),
                                        cache.handle if cache is not None else None, _p(perm), _p(gbits), _p(codes),
                                        _p(scales), _p(zeros), ctypes.byref(st), _p(passes)))
    ql = QLayer(d_out, d_in, effective_group(cfg, d_in), perm, gbits, codes, scales, zeros)
    stats = LayerStats.from_c(st)
    if return_chunk_passes:
        return ql, stats, passes
    return ql, stats


def proxy_loss(w_t, w_hat, rows, n, h):
    """src/engine.rs:808-815: sum_r e_r (E H)_r with E = w_t - w_hat."""
    a = np.ascontiguousarray(np.asarray(w_t, np.float32).reshape(-1))
    b = np.ascontiguousarray(np.asarray(w_hat, np.float32).reshape(-1))
    hh = np.ascontiguousarray(np.asarray(h, np.float32).reshape(-1))
    out = ctypes.c_double(0.0)
    check(lib().cdclq_proxy_loss(_p(a), _p(b), rows, n, _p(hh), ctypes.byref(out)))
    return out.value


def rtn_layer(w, d_out, n, cfg: Config):
    """src/engine.rs:822-838."""
    a = np.ascontiguousarray(np.asarray(w, np.float32).reshape(-1))
    out = np.zeros((d_out, n), np.float32)
    c = cfg.to_c()
    check(lib().cdclq_rtn_layer(_p(a), d_out, n, ctypes.byref(c), _p(out)))
    return out
