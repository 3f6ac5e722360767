"""`io.rs` surface: safetensors weights and calibration Hessians onto the device, and the packed output format.

    to_device_f32      tensor_to_f32 (src/io.rs:37-45): the raw bytes go to the device, the bf16/f16 -> f32
                       widening (lossless) runs there (cdclq_widen_to_f32_device)
    HessianStore       src/io.rs:136-226: files indexed by `<layer>.H`, `aliases` metadata resolving layers that
                       share an input, the square-shape check and the load-time non-finite refusal (the scan runs on
                       the device: cdclq_check_matrix_device), messages as the reference's
    packed_tensors     src/io.rs:244-270: the six tensors of a packed layer; codes packed and scales/zero points
                       encoded on the device (cdclq_pack_device, cdclq_encode_groups_device)
    read_packed_layer  src/io.rs:276-296, its exact inverse
    save_packed        one safetensors file of packed layers

torch is the plumbing for device memory here (tensors, streams); the conversions are the library's kernels.
"""
import ctypes
import json

import numpy as np

from ._lib import CdclqError, check, lib
from .abi import CDCLQ_ERR_ARG
from .quant import QLayer, row_bytes

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2


def _dtype_code(torch, dt):
    m = {torch.float32: DTYPE_F32, torch.float16: DTYPE_F16, torch.bfloat16: DTYPE_BF16}
    if dt not in m:
        raise CdclqError(CDCLQ_ERR_ARG, "unsupported weight dtype %s (need F32/F16/BF16)" % dt)
    return m[dt]


def to_device_f32(t, stream=0):
    """A host tensor of f32/f16/bf16 as a contiguous f32 device tensor: raw copy, then widening on the device."""
    import torch

    code = _dtype_code(torch, t.dtype)
    raw = t.contiguous().to("cuda", non_blocking=False)
    out = torch.empty(raw.shape, dtype=torch.float32, device="cuda")
    check(lib().cdclq_widen_to_f32_device(ctypes.c_void_p(raw.data_ptr()), code, raw.numel(),
                                          ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(stream)))
    return out


class HessianStore:
    """Calibration Hessians: `<layer>.H` (f32 d_in x d_in), optional `<layer>.M`, and an `aliases` metadata
    entry (JSON {layer: owner}) for layers that share an input (src/io.rs:124-188).  Later files override
    earlier ones for the same layer name."""

    def __init__(self, paths):
        from safetensors import safe_open

        self.paths = list(paths)
        self.index = {}
        self.aliases = {}
        for fi, p in enumerate(self.paths):
            with safe_open(p, framework="pt") as f:
                for name in f.keys():
                    if name.endswith(".H"):
                        self.index[name[:-2]] = fi
                md = f.metadata() or {}
                if "aliases" in md:
                    self.aliases.update(json.loads(md["aliases"]))

    def resolve(self, layer):
        """The layer whose `.H` serves `layer` (itself or its alias target), or None."""
        if layer in self.index:
            return layer
        o = self.aliases.get(layer)
        return o if o is not None and o in self.index else None

    def _tensor(self, owner, suffix, stream=0):
        from safetensors import safe_open

        if owner not in self.index:
            raise CdclqError(CDCLQ_ERR_ARG, "no Hessian for %s" % owner)
        key = "%s.%s" % (owner, suffix)
        with safe_open(self.paths[self.index[owner]], framework="pt") as f:
            if key not in f.keys():
                return None
            t = f.get_tensor(key)
        sh = list(t.shape)
        if len(sh) != 2 or sh[0] != sh[1]:
            raise CdclqError(CDCLQ_ERR_ARG, "%s: expected a square matrix, got %s" % (key, "[" + ", ".join(map(str, sh)) + "]"))
        d = to_device_f32(t, stream)
        check(lib().cdclq_check_matrix_device(ctypes.c_void_p(d.data_ptr()), sh[0], key.encode(), ctypes.c_void_p(stream)))
        return d, sh[0]

    def get_h(self, owner, stream=0):
        """(device f32 tensor, n) of `<owner>.H` (src/io.rs:217-219)."""
        r = self._tensor(owner, "H", stream)
        if r is None:
            raise CdclqError(CDCLQ_ERR_ARG, "missing %s.H" % owner)
        return r

    def get_m(self, owner, stream=0):
        """The optional cross-covariance `<owner>.M` as a device tensor, or None (src/io.rs:222-224)."""
        r = self._tensor(owner, "M", stream)
        return None if r is None else r[0]


def packed_tensors(layer, ql, stream=0):
    """The six tensors of one packed layer (src/io.rs:244-270) as numpy arrays:
    `.qweight` u8 [d_out, row_bytes], `.scales` f16 [d_out, ng], `.qzeros` u8 [d_out, ng], `.perm` i32 [d_in],
    `.gbits` u8 [ng], `.gsize` i32 [1]."""
    import torch

    ng = ql.ngroups()
    gb = np.ascontiguousarray(ql.gbits, np.uint8)
    rb = row_bytes(ql.d_in, ql.group, gb)
    codes = torch.from_numpy(np.ascontiguousarray(ql.codes, np.uint8)).cuda()
    sc = torch.from_numpy(np.ascontiguousarray(ql.scales, np.float32).reshape(-1)).cuda()
    zr = torch.from_numpy(np.ascontiguousarray(ql.zeros, np.float32).reshape(-1)).cuda()
    qw = torch.empty((ql.d_out, rb), dtype=torch.uint8, device="cuda")
    s16 = torch.empty(ql.d_out * ng, dtype=torch.int16, device="cuda")
    qz = torch.empty(ql.d_out * ng, dtype=torch.uint8, device="cuda")
    s = ctypes.c_void_p(stream)
    check(lib().cdclq_pack_device(ctypes.c_void_p(codes.data_ptr()), ql.d_out, ql.d_in, ql.group,
                                  ctypes.c_void_p(gb.ctypes.data), ctypes.c_void_p(qw.data_ptr()), s))
    check(lib().cdclq_encode_groups_device(ctypes.c_void_p(sc.data_ptr()), ctypes.c_void_p(zr.data_ptr()),
                                           ql.d_out * ng, ctypes.c_void_p(s16.data_ptr()),
                                           ctypes.c_void_p(qz.data_ptr()), s))
    torch.cuda.synchronize()
    return {
        layer + ".qweight": qw.cpu().numpy(),
        layer + ".scales": s16.cpu().numpy().view(np.float16).reshape(ql.d_out, ng),
        layer + ".qzeros": qz.cpu().numpy().reshape(ql.d_out, ng),
        layer + ".perm": np.asarray(ql.perm, dtype=np.uint32).astype(np.int32),
        layer + ".gbits": gb.copy(),
        layer + ".gsize": np.array([ql.group], dtype=np.int32),
    }


def read_packed_layer(tensors, layer):
    """Rebuild a QLayer from the tensors written by packed_tensors (src/io.rs:276-296); a missing companion
    tensor is an error naming it."""

    def get(suffix):
        k = "%s.%s" % (layer, suffix)
        if k not in tensors:
            raise CdclqError(CDCLQ_ERR_ARG, "%s: tensor not found" % k)
        return tensors[k]

    qw, sc, qz, pm, gb, gs = (get(x) for x in ("qweight", "scales", "qzeros", "perm", "gbits", "gsize"))
    d_out, d_in, group = int(qw.shape[0]), int(pm.shape[0]), int(np.asarray(gs).reshape(-1)[0])
    perm = np.asarray(pm).astype(np.int32).astype(np.uint32)
    scales = np.asarray(sc, dtype=np.float16).astype(np.float32)
    zeros = np.asarray(qz, dtype=np.uint8).astype(np.float32)
    return QLayer.from_packed(d_out, d_in, group, perm, np.asarray(gb, np.uint8), np.asarray(qw, np.uint8), scales,
                              zeros)


def save_packed(path, tensors, metadata=None):
    """Write packed-layer tensors (dicts from packed_tensors) to one safetensors file."""
    from safetensors.numpy import save_file

    save_file({k: np.ascontiguousarray(v) for k, v in tensors.items()}, path, metadata=metadata)
