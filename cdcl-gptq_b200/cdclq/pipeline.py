"""`pipeline.rs` counterpart: a model's layers quantized as one batch, optionally over several GPUs.

The reference quantizes layer after layer on one host, its jobs sorted by Hessian owner so that consecutive
layers reuse one factorisation (src/pipeline.rs:92-175).  Here all layers of a model go through one
cdclq_quantize_batch call (every distinct input factorised once), and with several GPUs - one process per
GPU, torch.distributed over NCCL as the plumbing - the work is split along the independence structure of the
algorithm:

  * rows: every layer's rows are split in whole row chunks, a contiguous range per rank (rows are
    independent, src/engine.rs:9-15; conflict selection and the tol stop are per row chunk,
    src/engine.rs:480-511, 660-665, so chunk boundaries must not move); the assignment of ranges to ranks
    rotates from layer to layer, so that leftover chunks spread over the ranks;
  * factorisations: the distinct inputs are assigned to ranks by longest-processing-time on n^3 (Cholesky +
    triangular inverse), each rank factorises its share (cdclq_prepare_factors) and every factor U is then
    broadcast from its owner, so no rank repeats another's factorisation;
  * statistics: the per-layer sums of the row shards are additive (the caller all-reduces them).

Results are bit-identical to a single-GPU run: the factorisation is deterministic, and a row's computation
does not depend on which rank holds it.
"""
import ctypes

import numpy as np

from ._lib import check, lib
from .abi import CBatchInput, CBatchLayer, CLayerStats, num_groups


def shard_rows(d_out, row_chunk, rank, world, rotate=0):
    """Contiguous row range [r0, r1) of `rank`, in whole row chunks of `row_chunk` rows.  `rotate` shifts which
    rank takes which range, so that the layers of a model hand their leftover chunks to different ranks."""
    chunks = (d_out + row_chunk - 1) // row_chunk
    v = (rank + rotate) % world
    c0 = chunks * v // world
    c1 = chunks * (v + 1) // world
    return min(c0 * row_chunk, d_out), min(c1 * row_chunk, d_out)


def assign_factorisations(ns, world, power=3):
    """Owner rank of each distinct input: longest-processing-time scheduling on the n^power cost of its work
    (n^3: Cholesky + triangular inverse; n^2: a Hessian accumulation over a fixed token count), largest first,
    ties by index, each to the least-loaded rank (ties to the lowest rank)."""
    owner = [0] * len(ns)
    load = [0.0] * world
    for i in sorted(range(len(ns)), key=lambda i: (-ns[i], i)):
        r = min(range(world), key=lambda r: (load[r], r))
        owner[i] = r
        load[r] += float(ns[i]) ** power
    return owner


def exchange_factors(factors, owner, stream_handle=None):
    """Broadcast every factor from its owner rank, inputs in index order (every rank takes the same collective
    steps in the same order).  `factors` are tensors on the process group's device.

    The collectives are ordered after torch's current stream.  When the factors were written on another stream
    (`stream_handle`, the library's stream: 0 = the legacy default stream), the current stream first waits for
    that stream, and afterwards that stream waits for the broadcasts, so the library reads every factor only
    once it has landed."""
    import torch
    import torch.distributed as dist

    cur = torch.cuda.current_stream() if stream_handle is not None else None
    other = None
    if cur is not None and stream_handle != cur.cuda_stream:
        other = torch.cuda.ExternalStream(stream_handle) if stream_handle else torch.cuda.default_stream()
        ev = torch.cuda.Event()
        ev.record(other)
        cur.wait_event(ev)
    for i, u in enumerate(factors):
        dist.broadcast(u, src=owner[i])
    if other is not None:
        ev = torch.cuda.Event()
        ev.record(cur)
        other.wait_event(ev)


class ModelBatch:
    """Descriptor tables and caller-allocated outputs for one model on one rank.

    layers: [(name, d_out, d_in, input index)]; inputs: [(name, n)]; H: per input an n x n f32 tensor; W: per
    layer a d_out x d_in f32 tensor (original column order).  All tensors on the device (on_device=True) or
    all in (pinned) host memory (on_device=False, copies inside the library).  With world > 1 the rank keeps
    the rows shard_rows() gives it, and `run` needs torch.distributed initialised (NCCL).  With w_sharded=True
    each W entry holds only this rank's rows (shard_rows(d_out, cfg.row_chunk, rank, world, rotate=layer index))
    and layers without rows on this rank may be None.

    With a skeleton (cfg.skeleton_pct > 0) the column permutation ranks columns by H_jj * ||W_:j||^2 over ALL
    rows of the layer (src/engine.rs:271-304); a row-sharded rank therefore computes those scores from the full
    W (cdclq_column_scores_device, the same row-ordered f64 sums as a single-GPU run) and hands them to the
    library, which needs the full W on every rank (w_sharded=False).  The permutation then differs from layer to
    layer, so the factorisations are spread per layer (cdclq_prepare_layer_factors, owners by LPT on n^3) and
    each layer's U is broadcast from its owner.
    """

    def __init__(self, torch, layers, inputs, H, W, cfg, rank=0, world=1, on_device=True, distribute_factors=True,
                 w_sharded=False):
        self.torch = torch
        self.cfg = cfg
        self.rank, self.world = rank, world
        self.on_device = on_device
        skel_scores = world > 1 and cfg.skeleton_pct > 0.0
        if skel_scores and w_sharded:
            raise ValueError("a skeleton ranks columns by the whole weight matrix: every rank needs the full W "
                             "(w_sharded=False) to compute the column scores")
        self.keep = []
        self.ins = (CBatchInput * len(inputs))()
        for i, (_, n) in enumerate(inputs):
            self.keep.append(H[i])
            self.ins[i].h = H[i].data_ptr()
            self.ins[i].n = n
        rc = cfg.row_chunk
        if rc <= 0 and world > 1:
            raise ValueError("multi-GPU row sharding needs a pinned row_chunk (row chunks must not move)")
        colsq = [self._column_scores(w, H[inp], d_out, d_in) for ((_, d_out, d_in, inp), w) in zip(layers, W)] \
            if skel_scores else [None] * len(layers)
        rows = []
        for li, ((name, d_out, d_in, inp), w) in enumerate(zip(layers, W)):
            r0, r1 = shard_rows(d_out, rc, rank, world, rotate=li) if world > 1 else (0, d_out)
            if r1 > r0:
                rows.append((name, d_out, d_in, inp, w, r0, r1, li))
        self.layer_index = [r[7] for r in rows]
        self.names = [r[0] for r in rows]
        self.shards = [(r[5], r[6]) for r in rows]
        self.lys = (CBatchLayer * len(rows))()
        self.stats = [CLayerStats() for _ in rows]
        self.outs = []
        self.h2d_bytes = sum(int(h.numel()) * 4 for h in H)
        self.d2h_bytes = 0
        dev = "cuda" if on_device else "cpu"
        for i, (name, d_out, d_in, inp, w, r0, r1, li) in enumerate(rows):
            ng = num_groups(cfg, d_in)
            rs = r1 - r0
            wv = w if w_sharded else w[r0:r1]
            if tuple(wv.shape) != (rs, d_in):
                raise ValueError("%s: weight rows %s, expected %s" % (name, tuple(wv.shape), (rs, d_in)))
            self.keep.append(wv)
            o = dict(perm=np.zeros(d_in, np.uint32), gbits=np.zeros(ng, np.uint8),
                     codes=torch.empty(rs, d_in, dtype=torch.uint8, device=dev, pin_memory=not on_device),
                     scales=torch.empty(rs, ng, dtype=torch.float32, device=dev, pin_memory=not on_device),
                     zeros=torch.empty(rs, ng, dtype=torch.float32, device=dev, pin_memory=not on_device))
            self.outs.append(o)
            L = self.lys[i]
            L.w = wv.data_ptr()
            L.d_out = rs
            L.input = inp
            L.perm = o["perm"].ctypes.data
            L.gbits = o["gbits"].ctypes.data
            L.codes = o["codes"].data_ptr()
            L.scales = o["scales"].data_ptr()
            L.zeros = o["zeros"].data_ptr()
            L.stats = ctypes.pointer(self.stats[i])
            if skel_scores:
                L.colsq = colsq[li]
            self.h2d_bytes += rs * d_in * 4
            self.d2h_bytes += rs * d_in + 2 * rs * ng * 4 + d_in * 4 + ng
        self.weights = sum((r1 - r0) * d_in for (_, _, d_in, _, _, r0, r1, _) in rows)

        # skeleton: a factor per layer (its own permutation), spread over the ranks by LPT on n^3
        self.layer_factors = skel_scores and distribute_factors
        if self.layer_factors:
            self.all_lys = (CBatchLayer * len(layers))()  # every layer, full rows: what the factor depends on
            for li, ((_, d_out, d_in, inp), w) in enumerate(zip(layers, W)):
                A = self.all_lys[li]
                A.w = w.data_ptr()
                A.d_out = d_out
                A.input = inp
                A.colsq = colsq[li]
            ns = [d_in for (_, _, d_in, _) in layers]
            self.lowner = assign_factorisations(ns, world)
            self.lu = [torch.empty(n, n, dtype=torch.float32, device="cuda") for n in ns]
            self.lmine = [li for li in range(len(layers)) if self.lowner[li] == rank]
            self._lwhich = (ctypes.c_size_t * max(1, len(self.lmine)))(*self.lmine)
            self._lu_out = (ctypes.c_void_p * max(1, len(self.lmine)))(*[self.lu[li].data_ptr() for li in self.lmine])
            for i, li in enumerate(self.layer_index):
                self.lys[i].u = self.lu[li].data_ptr()

        # factorisations spread over the ranks: factor buffers for every input, owners by LPT on n^3
        self.distributed = world > 1 and distribute_factors and cfg.skeleton_pct <= 0.0
        if self.distributed:
            ns = [n for (_, n) in inputs]
            self.owner = assign_factorisations(ns, world)
            self.u = [torch.empty(n, n, dtype=torch.float32, device="cuda") for n in ns]
            self.mine = [i for i in range(len(ns)) if self.owner[i] == rank]
            self._which = (ctypes.c_size_t * max(1, len(self.mine)))(*self.mine)
            self._u_out = (ctypes.c_void_p * max(1, len(self.mine)))(*[self.u[i].data_ptr() for i in self.mine])
            self._u_in = (ctypes.c_void_p * len(ns))(*[u.data_ptr() for u in self.u])
            self.which = ctypes.cast(self._which, ctypes.c_void_p)
            self.u_out = ctypes.cast(self._u_out, ctypes.c_void_p)
            self.u_in = ctypes.cast(self._u_in, ctypes.c_void_p)

    def _column_scores(self, w, h, d_out, n):
        """Skeleton column scores of the full W (device f64, or pinned host f64 when on_device=False)."""
        torch = self.torch
        wd = w if w.is_cuda else w.cuda()
        hd = h if h.is_cuda else h.cuda()
        cs = torch.empty(n, dtype=torch.float64, device="cuda")
        check(lib().cdclq_column_scores_device(ctypes.c_void_p(wd.data_ptr()), d_out, n, ctypes.c_void_p(hd.data_ptr()),
                                               ctypes.c_void_p(cs.data_ptr()), None))
        if not self.on_device:
            cs = cs.cpu().pin_memory()
        self.keep.append(cs)
        return cs.data_ptr()

    def run(self, stream_handle):
        c = self.cfg.to_c()
        dev = 1 if self.on_device else 0
        if self.layer_factors:
            check(lib().cdclq_prepare_layer_factors(self.ins, len(self.ins), self.all_lys, len(self.all_lys),
                                                    ctypes.cast(self._lwhich, ctypes.c_void_p), len(self.lmine),
                                                    ctypes.byref(c), ctypes.cast(self._lu_out, ctypes.c_void_p), dev,
                                                    ctypes.c_void_p(stream_handle)))
            exchange_factors(self.lu, self.lowner, stream_handle)
            check(lib().cdclq_quantize_batch(self.ins, len(self.ins), self.lys, len(self.lys), ctypes.byref(c), dev,
                                             ctypes.c_void_p(stream_handle)))
            return
        if not self.distributed:
            check(lib().cdclq_quantize_batch(self.ins, len(self.ins), self.lys, len(self.lys), ctypes.byref(c), dev,
                                             ctypes.c_void_p(stream_handle)))
            return
        check(lib().cdclq_prepare_factors(self.ins, len(self.ins), self.which, len(self.mine), ctypes.byref(c),
                                          self.u_out, dev, ctypes.c_void_p(stream_handle)))
        exchange_factors(self.u, self.owner, stream_handle)
        check(lib().cdclq_quantize_batch_prepared(self.ins, len(self.ins), self.u_in, self.lys, len(self.lys),
                                                  ctypes.byref(c), dev, ctypes.c_void_p(stream_handle)))
