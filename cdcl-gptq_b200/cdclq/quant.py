"""`quant.rs` surface: the quantized-layer container and the grid helpers (src/quant.rs).

`QLayer` holds one layer in the PERMUTED column order, exactly like the reference's struct
(src/quant.rs:153-175).  Its pack/dequantize run on the GPU through the C ABI.
"""
import ctypes
from dataclasses import dataclass

import numpy as np

from ._lib import check, lib

F16_MIN_NORMAL = np.float32(6.1035156e-5)  # src/quant.rs:20


def _p(a):
    return ctypes.c_void_p(a.ctypes.data)


def row_bits(n, g, gbits):
    """src/quant.rs:98-100."""
    gb = np.asarray(gbits, dtype=np.int64)
    return int(sum(int(gb[j // g]) for j in range(n))) if n < 64 else int(
        np.bincount(np.arange(n) // g, minlength=len(gb)).astype(np.int64) @ gb)


def row_bytes(n, g, gbits):
    """src/quant.rs:102-104."""
    return (row_bits(n, g, gbits) + 7) // 8


@dataclass
class QLayer:
    d_out: int
    d_in: int
    group: int
    perm: np.ndarray    # u32 [d_in]: permuted position -> original column
    gbits: np.ndarray   # u8 [ngroups]
    codes: np.ndarray   # u8 [d_out, d_in] permuted order
    scales: np.ndarray  # f32 [d_out, ngroups]
    zeros: np.ndarray   # f32 [d_out, ngroups]

    def ngroups(self):
        return len(self.gbits)

    def dequantize(self):
        """Dequantized weights in the ORIGINAL column order (src/quant.rs:189-202), computed on the GPU."""
        packed, _ = self.pack()
        return dequantize_packed_layer(packed, self.d_out, self.d_in, self.group, self.perm, self.gbits, self.scales,
                                       self.zeros)

    def pack(self):
        """LSB-first mixed-width bit stream (src/quant.rs:207-214): (uint8 [d_out, row_bytes], row_bytes)."""
        rb = int(lib().cdclq_row_bytes(self.d_in, self.group, _p(np.ascontiguousarray(self.gbits, np.uint8))))
        out = np.zeros((self.d_out, rb), dtype=np.uint8)
        codes = np.ascontiguousarray(self.codes, dtype=np.uint8)
        gb = np.ascontiguousarray(self.gbits, dtype=np.uint8)
        check(lib().cdclq_pack(_p(codes), self.d_out, self.d_in, self.group, _p(gb), _p(out)))
        return out, rb

    @staticmethod
    def from_packed(d_out, d_in, group, perm, gbits, packed, scales, zeros):
        """src/quant.rs:219-235; codes are recovered with the GPU unpacker through a dequantization probe."""
        codes = unpack_codes(packed, d_out, d_in, group, gbits)
        return QLayer(d_out, d_in, group, np.asarray(perm, np.uint32), np.asarray(gbits, np.uint8), codes,
                      np.asarray(scales, np.float32).reshape(d_out, -1), np.asarray(zeros, np.float32).reshape(d_out, -1))

    def bits_codes(self):
        """src/quant.rs:239-241."""
        return row_bits(self.d_in, self.group, self.gbits) / self.d_in

    def bits_total(self):
        """src/quant.rs:248-250."""
        return self.bits_codes() + 24.0 / self.group


def dequantize_packed_layer(packed, d_out, d_in, group, perm, gbits, scales, zeros):
    out = np.zeros((d_out, d_in), dtype=np.float32)
    args = [np.ascontiguousarray(packed, np.uint8), np.ascontiguousarray(gbits, np.uint8),
            np.ascontiguousarray(perm, np.uint32), np.ascontiguousarray(scales, np.float32),
            np.ascontiguousarray(zeros, np.float32)]
    check(lib().cdclq_unpack_dequant(_p(args[0]), d_out, d_in, group, _p(args[1]), _p(args[2]), _p(args[3]),
                                     _p(args[4]), _p(out)))
    return out


def unpack_codes(packed, d_out, d_in, group, gbits):
    """src/quant.rs:133-151 on the GPU: dequantize with scale 1, zero 0 and the identity permutation."""
    ng = (d_in + group - 1) // group
    ones = np.ones((d_out, ng), np.float32)
    zs = np.zeros((d_out, ng), np.float32)
    ident = np.arange(d_in, dtype=np.uint32)
    vals = dequantize_packed_layer(packed, d_out, d_in, group, ident, gbits, ones, zs)
    return vals.astype(np.uint8)


def find_params(vals, bits, mse=False):
    """src/quant.rs:40-83 for each row of `vals` (rows are independent groups); returns (scales, zeros)."""
    v = np.ascontiguousarray(np.atleast_2d(vals), dtype=np.float32)
    s = np.zeros(v.shape[0], np.float32)
    z = np.zeros(v.shape[0], np.float32)
    check(lib().cdclq_find_params(_p(v), v.shape[0], v.shape[1], bits, 1 if mse else 0, _p(s), _p(z)))
    return s, z
