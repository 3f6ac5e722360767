"""The multi-GPU runtime and the model-level pipeline of the C ABI (cdclq_runtime_*, cdclq_quantize_model).

    Runtime            one rank of a job: its device, stream and NCCL communicator, all owned by the library
                       (one process per GPU; rank 0 makes the unique id, the caller hands it to every rank)
    Runtime.quantize_batch
                       cdclq_quantize_batch over the ranks: rows sharded in whole row chunks, factors computed by
                       their owner and broadcast over NVLink, statistics all-reduced, outputs gathered on rank 0
    QuantOpts, quantize_model
                       pipeline::quantize_model (src/pipeline.rs:26-227): safetensors shards in, packed and
                       dequantized shards plus report.json out
    dequantize_packed  pipeline::dequantize_packed (src/pipeline.rs:239-275)
    shard_rows, assign_owners
                       the row sharding and the factorisation owners the runtime uses (host logic, no GPU)

Everything here is a thin binding: the sharding, the collectives, the file I/O and the kernels are the library's.
"""
import ctypes
import json
import os
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np

from ._lib import check, lib
from .abi import CBatchInput, CBatchLayer, CModelOpts, CModelReport, Config

UNIQUE_ID_BYTES = 128


def _prefer_framework_nccl():
    """Points the library at the NCCL that torch loads (the pip package nvidia-nccl), unless the caller chose one:
    the library opens NCCL at its first runtime, and a process that creates a runtime before importing torch would
    otherwise hold the system's libnccl.so.2 under the soname torch needs for its own, newer copy."""
    if os.environ.get("CDCLQ_NCCL_LIBRARY"):
        return
    try:
        import importlib.util

        spec = importlib.util.find_spec("nvidia.nccl")
        for d in (spec.submodule_search_locations or []) if spec else []:
            p = os.path.join(d, "lib", "libnccl.so.2")
            if os.path.exists(p):
                os.environ["CDCLQ_NCCL_LIBRARY"] = p
                return
    except Exception:
        pass


_prefer_framework_nccl()


def shard_rows(d_out, row_chunk, rank, nranks, rotate=0):
    """[r0, r1) of `rank`: whole row chunks, contiguous, rotated by `rotate` (cdclq_shard_rows)."""
    r0, r1 = ctypes.c_size_t(0), ctypes.c_size_t(0)
    lib().cdclq_shard_rows(d_out, row_chunk, rank, nranks, rotate, ctypes.byref(r0), ctypes.byref(r1))
    return r0.value, r1.value


def assign_owners(ns, nranks, power=3):
    """Owner rank per item by longest processing time on n^power (cdclq_assign_owners)."""
    a = (ctypes.c_size_t * max(1, len(ns)))(*ns)
    o = (ctypes.c_int * max(1, len(ns)))()
    lib().cdclq_assign_owners(a, len(ns), nranks, power, o)
    return list(o)[:len(ns)]


def unique_id():
    """A new NCCL unique id (rank 0 makes it and sends it to the other ranks)."""
    buf = (ctypes.c_uint8 * UNIQUE_ID_BYTES)()
    check(lib().cdclq_runtime_unique_id(buf))
    return bytes(buf)


def shared_unique_id():
    """Rank 0's unique id on every rank of torch.distributed's default group (made by rank 0, sent through the
    group); the host side of joining a runtime, no GPU needed."""
    import torch.distributed as dist

    obj = [unique_id() if dist.get_rank() == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]


class Runtime:
    """One rank: `device`, `nranks`, `rank`, and (nranks > 1) the unique id every rank shares.  Every wait is
    bounded by `timeout_s`; calls are collective (all ranks, same order)."""

    def __init__(self, device=0, nranks=1, rank=0, uid: Optional[bytes] = None, timeout_s=600.0):
        self.nranks, self.rank, self.device = nranks, rank, device
        h = ctypes.c_void_p()
        idb = None if uid is None else (ctypes.c_uint8 * UNIQUE_ID_BYTES).from_buffer_copy(uid)
        check(lib().cdclq_runtime_create(device, nranks, rank, idb, float(timeout_s), ctypes.byref(h)))
        self.handle = h

    @classmethod
    def from_process_group(cls, device=None, timeout_s=600.0):
        """Joins a runtime over the ranks of torch.distributed's default group (any backend): rank 0's unique id
        travels through the group, the library's own communicator does the work."""
        import torch.distributed as dist

        uid = shared_unique_id()
        if device is None:
            device = int(os.environ.get("LOCAL_RANK", dist.get_rank()))
        return cls(device, dist.get_world_size(), dist.get_rank(), uid, timeout_s)

    @property
    def stream_handle(self):
        """The runtime's CUDA stream (an int handle for torch.cuda.ExternalStream)."""
        return lib().cdclq_runtime_stream(self.handle) or 0

    def close(self):
        if getattr(self, "handle", None):
            lib().cdclq_runtime_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def quantize_batch(self, inputs, layers, cfg: Config, on_device, gather=True):
        """cdclq_runtime_quantize_batch: `inputs` a ctypes array of CBatchInput, `layers` of CBatchLayer, each
        describing a FULL layer (every rank quantizes its rows)."""
        c = cfg.to_c()
        check(lib().cdclq_runtime_quantize_batch(self.handle, inputs, len(inputs), layers, len(layers), ctypes.byref(c),
                                                 1 if on_device else 0, 1 if gather else 0))


@dataclass
class QuantOpts:
    """pipeline::QuantOpts (src/pipeline.rs:26-41)."""

    weights: List[str]
    hessians: List[str]
    out_dir: str
    cfg: Config = field(default_factory=Config)
    only: List[str] = field(default_factory=list)
    skip: List[str] = field(default_factory=list)
    emit_packed: bool = True
    emit_dequant: bool = True
    verbose: bool = False


def _cstrs(xs):
    arr = (ctypes.c_char_p * max(1, len(xs)))(*[x.encode() for x in xs])
    return arr, len(xs)


def quantize_model(opts: QuantOpts, runtime: Optional[Runtime] = None):
    """pipeline::quantize_model (src/pipeline.rs:79-227) on the GPU(s).  Returns the report (report.json's
    content: config, per-layer records, totals) read back from out_dir."""
    o = CModelOpts()
    keep = []
    for name in ("weights", "hessians", "only", "skip"):
        arr, n = _cstrs(getattr(opts, name))
        keep.append(arr)
        setattr(o, name, ctypes.cast(arr, ctypes.POINTER(ctypes.c_char_p)))
        setattr(o, "n_" + name, n)
    o.out_dir = opts.out_dir.encode()
    o.emit_packed = 1 if opts.emit_packed else 0
    o.emit_dequant = 1 if opts.emit_dequant else 0
    o.verbose = 1 if opts.verbose else 0
    o.cfg = opts.cfg.to_c()
    rep = CModelReport()
    check(lib().cdclq_quantize_model(runtime.handle if runtime else None, ctypes.byref(o), ctypes.byref(rep)))
    with open(os.path.join(opts.out_dir, "report.json")) as f:
        report = json.load(f)
    report["_totals"] = {"layers": int(rep.layers), "total_loss_gptq": rep.total_loss_gptq,
                         "total_loss_final": rep.total_loss_final, "total_gain_pct": rep.total_gain_pct,
                         "total_secs": rep.total_secs}
    return report


def dequantize_packed(input_path, output_path, dtype=None):
    """pipeline::dequantize_packed (src/pipeline.rs:239-275); returns the number of layers expanded."""
    n = ctypes.c_uint64(0)
    check(lib().cdclq_dequantize_packed(input_path.encode(), output_path.encode(),
                                        None if dtype is None else dtype.encode(), ctypes.byref(n)))
    return int(n.value)


def batch_tables(inputs_h, layers, cfg: Config):
    """Descriptor tables for Runtime.quantize_batch over host numpy arrays: inputs_h [n x n f32], layers
    [(input index, W d_out x n f32)].  Returns (inputs, layers, outputs, stats, keep-alive list)."""
    from .abi import CLayerStats, num_groups

    ins = (CBatchInput * len(inputs_h))()
    keep = []
    for i, h in enumerate(inputs_h):
        hh = np.ascontiguousarray(h, np.float32)
        keep.append(hh)
        ins[i].h = hh.ctypes.data
        ins[i].n = hh.shape[0]
    lys = (CBatchLayer * len(layers))()
    outs, stats = [], [CLayerStats() for _ in layers]
    for k, (inp, w) in enumerate(layers):
        ww = np.ascontiguousarray(w, np.float32)
        keep.append(ww)
        d, n = ww.shape
        ng = num_groups(cfg, n)
        o = dict(perm=np.zeros(n, np.uint32), gbits=np.zeros(ng, np.uint8), codes=np.zeros((d, n), np.uint8),
                 scales=np.zeros((d, ng), np.float32), zeros=np.zeros((d, ng), np.float32))
        outs.append(o)
        L = lys[k]
        L.w = ww.ctypes.data
        L.d_out = d
        L.input = inp
        for key in ("perm", "gbits", "codes", "scales", "zeros"):
            setattr(L, key, o[key].ctypes.data)
        L.stats = ctypes.pointer(stats[k])
    return ins, lys, outs, stats, keep
