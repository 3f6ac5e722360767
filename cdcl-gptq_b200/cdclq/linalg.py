"""`linalg.rs` surface over the CUDA library (src/linalg.rs:200-418)."""
import ctypes

import numpy as np

from ._lib import check, lib


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


def cholesky_lower(a, n):
    """src/linalg.rs:200-276: in place on an n x n f64 array; lower triangle = L."""
    assert a.dtype == np.float64 and a.flags.c_contiguous and a.size == n * n
    check(lib().cdclq_cholesky_lower(_p(a), n))
    return a


def tri_inverse_lower(l, n):
    """src/linalg.rs:284-347."""
    l = np.ascontiguousarray(l, np.float64)
    y = np.zeros((n, n), np.float64)
    check(lib().cdclq_tri_inverse_lower(_p(l), n, _p(y)))
    return y


def upper_chol_of_inverse(h, n):
    """src/linalg.rs:362-375: U (f32, upper) with H^-1 = U^T U."""
    h = np.ascontiguousarray(h, np.float64)
    u = np.zeros((n, n), np.float32)
    check(lib().cdclq_upper_chol_of_inverse(_p(h), n, _p(u)))
    return u


def gram_accumulate(x, y, t, n, h):
    """src/linalg.rs:388-418: h (f64, in place) += x^T y over t tokens."""
    x = np.ascontiguousarray(x, np.float32)
    y = x if y is x else np.ascontiguousarray(y, np.float32)
    assert h.dtype == np.float64 and h.flags.c_contiguous
    check(lib().cdclq_gram_accumulate(_p(x), _p(y), t, n, _p(h)))
    return h


def gram_accumulate_device(x, h, stream=0):
    """H (f64, device tensor, in place) += X^T X for X a (t, n) f32 device tensor: the bit-exact f32 path
    (src/linalg.rs:388-418: token chunks of 2048, f32 sums in increasing token order, widened into H), both
    triangles."""
    t, n = int(x.shape[0]), int(x.shape[1])
    assert h.shape == (n, n) and h.is_contiguous() and x.is_contiguous()
    check(lib().cdclq_gram_accumulate_device(ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(x.data_ptr()), t, n,
                                             ctypes.c_void_p(h.data_ptr()), ctypes.c_void_p(stream)))
    return h


def gram_accumulate_half_device(x, h, lower_only=False, stream=0):
    """H (f64, device tensor, in place) += X^T X for X a (t, n) bf16 or f16 device tensor on the tcgen05 tensor
    cores (token chunks of 2048 accumulated in f32, then widened into H; src/linalg.rs:392-416)."""
    import torch

    t, n = int(x.shape[0]), int(x.shape[1])
    assert h.shape == (n, n) and h.is_contiguous() and x.is_contiguous()
    code = {torch.bfloat16: 2, torch.float16: 1}.get(x.dtype)
    if code is None:
        raise TypeError("half Gram: x must be bf16 or f16, got %s" % x.dtype)
    check(lib().cdclq_gram_accumulate_half_device(ctypes.c_void_p(x.data_ptr()), code, t, n,
                                                  ctypes.c_void_p(h.data_ptr()), 1 if lower_only else 0,
                                                  ctypes.c_void_p(stream)))
    return h


def gram_accumulate_bf16_device(x_bf16, h, lower_only=False, stream=0):
    """H (f64, device tensor, in place) += X^T X for X a (t, n) bf16 device tensor, on the tcgen05 tensor cores:
    the token chunks of 2048 of src/linalg.rs:392 are accumulated in f32 inside the tensor core, then widened
    into H.  With lower_only only the lower triangle of H is updated."""
    t, n = int(x_bf16.shape[0]), int(x_bf16.shape[1])
    assert h.shape == (n, n) and h.is_contiguous() and x_bf16.is_contiguous()
    check(lib().cdclq_gram_accumulate_bf16_device(ctypes.c_void_p(x_bf16.data_ptr()), t, n,
                                                  ctypes.c_void_p(h.data_ptr()), 1 if lower_only else 0,
                                                  ctypes.c_void_p(stream)))
    return h
