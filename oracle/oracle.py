"""ctypes binding of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and
`--impl reference` legs, never by the product package.  Function names and argument meaning mirror the
reference crate (src/engine.rs, src/linalg.rs, src/quant.rs) and the product binding (cdclq.*), so a parity
test reads the same on both sides.
"""
import ctypes
import os
import subprocess
import sys
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_ROOT = os.path.dirname(_HERE)
sys.path.insert(0, os.path.join(_ROOT, "cdcl-gptq_b200"))
from cdclq.abi import CConfig, CLayerStats, Config, LayerStats, effective_group, num_groups  # noqa: E402

LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

P = ctypes.c_void_p
SZ = ctypes.c_size_t
CFG = ctypes.POINTER(CConfig)


def build(force=False):
    src = os.path.join(_HERE, "oracle.cpp")
    hdr = os.path.join(_ROOT, "include", "cdclq.h")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < max(os.path.getmtime(src),
                                                                                  os.path.getmtime(hdr)):
        subprocess.run(["make", "-C", _HERE, "-s"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        sig = {
            "oracle_last_error": (ctypes.c_char_p, []),
            "oracle_set_threads": (None, [ctypes.c_int]),
            "oracle_max_threads": (ctypes.c_int, []),
            "oracle_prep_cache_new": (P, []),
            "oracle_prep_cache_free": (None, [P]),
            "oracle_effective_group": (SZ, [CFG, SZ]),
            "oracle_validate": (ctypes.c_int, [CFG, SZ]),
            "oracle_row_chunk": (SZ, [CFG, SZ]),
            "oracle_round_f16": (ctypes.c_float, [ctypes.c_float]),
            "oracle_round_f16_array": (None, [P, SZ, P]),
            "oracle_find_params": (None, [P, SZ, SZ, ctypes.c_uint32, ctypes.c_int, P, P]),
            "oracle_cholesky_lower": (ctypes.c_int, [P, SZ]),
            "oracle_tri_inverse_lower": (None, [P, SZ, P]),
            "oracle_upper_chol_of_inverse": (ctypes.c_int, [P, SZ, P]),
            "oracle_gram_accumulate": (None, [P, P, SZ, SZ, P]),
            "oracle_compute_perm": (ctypes.c_int, [P, P, SZ, SZ, CFG, P, ctypes.POINTER(SZ)]),
            "oracle_build_prepared": (ctypes.c_int, [P, SZ, P, CFG, P, P, ctypes.POINTER(ctypes.c_double)]),
            "oracle_quantize_layer_ex": (ctypes.c_int, [P, SZ, SZ, P, P, ctypes.c_char_p, CFG, P, P, P, P, P, P,
                                                        ctypes.POINTER(CLayerStats), P]),
            "oracle_proxy_loss": (ctypes.c_double, [P, P, SZ, SZ, P]),
            "oracle_rtn_layer": (None, [P, SZ, SZ, CFG, P]),
            "oracle_row_bytes": (SZ, [SZ, SZ, P]),
            "oracle_pack_row": (None, [P, SZ, SZ, P, P]),
            "oracle_unpack_row": (None, [P, SZ, SZ, P, P]),
            "oracle_dequantize": (None, [SZ, SZ, SZ, P, P, P, P, P]),
            "oracle_rng_normal": (None, [ctypes.c_uint64, SZ, ctypes.c_float, P]),
            "oracle_problem": (None, [SZ, SZ, SZ, ctypes.c_uint64, P, P]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _p(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


class OracleError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(msg)
        self.code = code


def _check(rc):
    if rc != 0:
        raise OracleError(rc, lib().oracle_last_error().decode())


def set_threads(t):
    lib().oracle_set_threads(int(t))


def max_threads():
    return int(lib().oracle_max_threads())


@dataclass
class OQLayer:
    """Same fields as the reference's QLayer (src/quant.rs:161-175)."""

    d_out: int
    d_in: int
    group: int
    perm: np.ndarray
    gbits: np.ndarray
    codes: np.ndarray
    scales: np.ndarray
    zeros: np.ndarray

    def dequantize(self):
        out = np.zeros((self.d_out, self.d_in), np.float32)
        lib().oracle_dequantize(self.d_out, self.d_in, self.group, _p(self.perm), _p(self.codes), _p(self.scales),
                                _p(self.zeros), _p(out))
        return out

    def bits_codes(self):
        bits = sum(int(self.gbits[j // self.group]) for j in range(self.d_in))
        return bits / self.d_in

    def bits_total(self):
        return self.bits_codes() + 24.0 / self.group


class PrepCache:
    def __init__(self):
        self.handle = lib().oracle_prep_cache_new()

    def __del__(self):
        try:
            lib().oracle_prep_cache_free(self.handle)
        except Exception:
            pass


def row_chunk(cfg: Config, d_out):
    c = cfg.to_c()
    return int(lib().oracle_row_chunk(ctypes.byref(c), d_out))


def validate(cfg: Config, n):
    c = cfg.to_c()
    _check(lib().oracle_validate(ctypes.byref(c), n))


def quantize_layer(w, d_out, d_in, h, m=None, hkey="", cfg: Config = None, cache: PrepCache = None,
                   return_chunk_passes=False):
    """src/engine.rs:690-799 (CPU restatement)."""
    cfg = cfg or Config()
    w = np.ascontiguousarray(np.asarray(w, np.float32).reshape(-1))
    h = np.ascontiguousarray(np.asarray(h, np.float32).reshape(-1))
    mm = None if m is None else np.ascontiguousarray(np.asarray(m, np.float32).reshape(-1))
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
    _check(lib().oracle_quantize_layer_ex(_p(w), d_out, d_in, _p(h), _p(mm), (hkey or "").encode(), ctypes.byref(c),
                                          cache.handle if cache is not None else None, _p(perm), _p(gbits), _p(codes),
                                          _p(scales), _p(zeros), ctypes.byref(st), _p(passes)))
    ql = OQLayer(d_out, d_in, effective_group(cfg, d_in), perm, gbits, codes, scales, zeros)
    stats = LayerStats.from_c(st)
    return (ql, stats, passes) if return_chunk_passes else (ql, stats)


def round_f16(x):
    x = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1))
    out = np.zeros_like(x)
    lib().oracle_round_f16_array(_p(x), x.size, _p(out))
    return out


def find_params(vals, bits, mse=False):
    v = np.ascontiguousarray(np.atleast_2d(vals), dtype=np.float32)
    s = np.zeros(v.shape[0], np.float32)
    z = np.zeros(v.shape[0], np.float32)
    lib().oracle_find_params(_p(v), v.shape[0], v.shape[1], bits, 1 if mse else 0, _p(s), _p(z))
    return s, z


def cholesky_lower(a, n):
    _check(lib().oracle_cholesky_lower(_p(a), n))
    return a


def tri_inverse_lower(l, n):
    l = np.ascontiguousarray(l, np.float64)
    y = np.zeros((n, n), np.float64)
    lib().oracle_tri_inverse_lower(_p(l), n, _p(y))
    return y


def upper_chol_of_inverse(h, n):
    h = np.ascontiguousarray(h, np.float64)
    u = np.zeros((n, n), np.float32)
    _check(lib().oracle_upper_chol_of_inverse(_p(h), n, _p(u)))
    return u


def gram_accumulate(x, y, t, n, h):
    x = np.ascontiguousarray(x, np.float32)
    y = x if y is x else np.ascontiguousarray(y, np.float32)
    lib().oracle_gram_accumulate(_p(x), _p(y), t, n, _p(h))
    return h


def compute_perm(h, w, d_out, n, cfg: Config):
    h = np.ascontiguousarray(h, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    perm = np.zeros(n, np.uint32)
    nskel = SZ(0)
    c = cfg.to_c()
    _check(lib().oracle_compute_perm(_p(h), _p(w), d_out, n, ctypes.byref(c), _p(perm), ctypes.byref(nskel)))
    return perm, nskel.value


def build_prepared(h, n, perm, cfg: Config):
    h = np.ascontiguousarray(h, np.float32)
    perm = np.ascontiguousarray(perm, np.uint32)
    u = np.zeros((n, n), np.float32)
    h32 = np.zeros((n, n), np.float32)
    d = ctypes.c_double(0)
    c = cfg.to_c()
    _check(lib().oracle_build_prepared(_p(h), n, _p(perm), ctypes.byref(c), _p(u), _p(h32), ctypes.byref(d)))
    return u, h32, d.value


def proxy_loss(w_t, w_hat, rows, n, h):
    a = np.ascontiguousarray(w_t, np.float32)
    b = np.ascontiguousarray(w_hat, np.float32)
    hh = np.ascontiguousarray(h, np.float32)
    return float(lib().oracle_proxy_loss(_p(a), _p(b), rows, n, _p(hh)))


def rtn_layer(w, d_out, n, cfg: Config):
    a = np.ascontiguousarray(w, np.float32)
    out = np.zeros((d_out, n), np.float32)
    c = cfg.to_c()
    lib().oracle_rtn_layer(_p(a), d_out, n, ctypes.byref(c), _p(out))
    return out


def row_bytes(n, g, gbits):
    gb = np.ascontiguousarray(gbits, np.uint8)
    return int(lib().oracle_row_bytes(n, g, _p(gb)))


def pack(codes, d_out, n, g, gbits):
    gb = np.ascontiguousarray(gbits, np.uint8)
    rb = row_bytes(n, g, gb)
    out = np.zeros((d_out, rb), np.uint8)
    codes = np.ascontiguousarray(codes, np.uint8).reshape(d_out, n)
    for r in range(d_out):
        row = np.ascontiguousarray(codes[r])
        buf = np.zeros(rb, np.uint8)
        lib().oracle_pack_row(_p(row), n, g, _p(gb), _p(buf))
        out[r] = buf
    return out, rb


def unpack(packed, d_out, n, g, gbits):
    gb = np.ascontiguousarray(gbits, np.uint8)
    codes = np.zeros((d_out, n), np.uint8)
    for r in range(d_out):
        row = np.ascontiguousarray(packed[r])
        out = np.zeros(n, np.uint8)
        lib().oracle_unpack_row(_p(row), n, g, _p(gb), _p(out))
        codes[r] = out
    return codes


def rng_normal(seed, count, scale=1.0):
    out = np.zeros(count, np.float32)
    lib().oracle_rng_normal(seed, count, scale, _p(out))
    return out


def problem(d_out, n, tokens, seed):
    """src/engine.rs:850-869: (w, h) of the reference's engine tests."""
    w = np.zeros((d_out, n), np.float32)
    h = np.zeros((n, n), np.float32)
    lib().oracle_problem(d_out, n, tokens, seed, _p(w), _p(h))
    return w, h


def damped(h, n, damp):
    """src/engine.rs:873-880."""
    mean = 0.0
    for x in np.diag(np.asarray(h, np.float32).reshape(n, n)):
        mean += float(x)  # sequential f64 sum, as the reference's iterator sum
    mean /= n
    d = np.array(h, np.float32, copy=True)
    idx = np.arange(n)
    d[idx, idx] += np.float32(damp * mean)
    return d
