"""ctypes mirror of include/cdclq.h and the Python form of the reference's `engine::Config`.

Shared by the product binding (`cdclq._lib`) and by the test-only oracle binding (`oracle/oracle.py`); it
defines data layouts only and performs no computation.
"""
import ctypes
from dataclasses import dataclass, fields

CDCLQ_OK = 0
CDCLQ_ERR_CONFIG = -1
CDCLQ_ERR_NOT_PD = -2
CDCLQ_ERR_ARG = -3
CDCLQ_ERR_CUDA = -4
CDCLQ_ERR_NONFINITE = -5

METHOD_GPTQ = 0
METHOD_CDCL = 1


class CConfig(ctypes.Structure):
    """`cdclq_config` (include/cdclq.h), field for field."""

    _fields_ = [
        ("group", ctypes.c_uint64),
        ("block", ctypes.c_uint64),
        ("sub_block", ctypes.c_uint64),
        ("cd_sweeps", ctypes.c_uint64),
        ("passes", ctypes.c_uint64),
        ("row_chunk", ctypes.c_uint64),
        ("threads", ctypes.c_uint64),
        ("damp", ctypes.c_double),
        ("skeleton_pct", ctypes.c_double),
        ("refine_frac", ctypes.c_double),
        ("tol", ctypes.c_double),
        ("bits", ctypes.c_uint32),
        ("skeleton_bits", ctypes.c_uint32),
        ("act_order", ctypes.c_int32),
        ("mse_grid", ctypes.c_int32),
        ("method", ctypes.c_int32),
        ("refit_scales", ctypes.c_int32),
    ]


class CLayerStats(ctypes.Structure):
    """`cdclq_layer_stats` (include/cdclq.h)."""

    _fields_ = [
        ("loss_gptq", ctypes.c_double),
        ("loss_final", ctypes.c_double),
        ("subblocks_total", ctypes.c_uint64),
        ("subblocks_refined", ctypes.c_uint64),
        ("code_updates", ctypes.c_uint64),
        ("skeleton_groups", ctypes.c_uint64),
        ("bits_codes", ctypes.c_double),
        ("bits_total", ctypes.c_double),
        ("secs_prepare", ctypes.c_double),
        ("secs_quant", ctypes.c_double),
        ("passes_max", ctypes.c_uint64),
    ]


class CBatchInput(ctypes.Structure):
    _fields_ = [("h", ctypes.c_void_p), ("n", ctypes.c_size_t)]


class CBatchLayer(ctypes.Structure):
    _fields_ = [
        ("w", ctypes.c_void_p),
        ("d_out", ctypes.c_size_t),
        ("input", ctypes.c_size_t),
        ("perm", ctypes.c_void_p),
        ("gbits", ctypes.c_void_p),
        ("codes", ctypes.c_void_p),
        ("scales", ctypes.c_void_p),
        ("zeros", ctypes.c_void_p),
        ("stats", ctypes.POINTER(CLayerStats)),
        ("colsq", ctypes.c_void_p),
        ("u", ctypes.c_void_p),
    ]


class CModelOpts(ctypes.Structure):
    """`cdclq_model_opts` (include/cdclq.h)."""

    _fields_ = [
        ("weights", ctypes.POINTER(ctypes.c_char_p)),
        ("n_weights", ctypes.c_size_t),
        ("hessians", ctypes.POINTER(ctypes.c_char_p)),
        ("n_hessians", ctypes.c_size_t),
        ("out_dir", ctypes.c_char_p),
        ("only", ctypes.POINTER(ctypes.c_char_p)),
        ("n_only", ctypes.c_size_t),
        ("skip", ctypes.POINTER(ctypes.c_char_p)),
        ("n_skip", ctypes.c_size_t),
        ("emit_packed", ctypes.c_int32),
        ("emit_dequant", ctypes.c_int32),
        ("verbose", ctypes.c_int32),
        ("pad", ctypes.c_int32),
        ("cfg", CConfig),
    ]


class CModelReport(ctypes.Structure):
    """`cdclq_model_report` (include/cdclq.h)."""

    _fields_ = [
        ("layers", ctypes.c_uint64),
        ("total_loss_gptq", ctypes.c_double),
        ("total_loss_final", ctypes.c_double),
        ("total_gain_pct", ctypes.c_double),
        ("total_secs", ctypes.c_double),
    ]


class CRunProfile(ctypes.Structure):
    """`cdclq_run_profile` (include/cdclq.h)."""

    _fields_ = [
        ("ms_prepare", ctypes.c_double),
        ("ms_phase1", ctypes.c_double),
        ("ms_stats", ctypes.c_double),
        ("ms_repair", ctypes.c_double),
        ("ms_final", ctypes.c_double),
        ("flops_phase1", ctypes.c_double),
        ("flops_repair", ctypes.c_double),
        ("flops_final", ctypes.c_double),
        ("flops_factor", ctypes.c_double),
        ("repair_launches", ctypes.c_uint64),
        ("factorisations", ctypes.c_uint64),
        ("weights", ctypes.c_uint64),
        ("launches", ctypes.c_uint64),
        ("factor_batches", ctypes.c_uint64),
        ("ms_host", ctypes.c_double),
        ("repair_layout", ctypes.c_uint64),
    ]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


@dataclass
class Config:
    """`engine::Config` (src/engine.rs:93-167) with the reference's defaults.

    `method` is "gptq" or "cdcl" (`engine::Method`, src/engine.rs:82-88).  `threads` is the CLI's global
    `--threads` (src/main.rs:22): it only fixes the automatic row chunk (src/engine.rs:768-770).
    """

    bits: int = 3
    group: int = 128
    block: int = 128
    damp: float = 0.01
    act_order: bool = True
    skeleton_pct: float = 0.0
    skeleton_bits: int = 8
    mse_grid: bool = False
    method: str = "cdcl"
    refine_frac: float = 1.0
    sub_block: int = 64
    cd_sweeps: int = 1
    passes: int = 10
    tol: float = 1e-3
    refit_scales: bool = True
    row_chunk: int = 0
    threads: int = 0

    def to_c(self) -> CConfig:
        if self.method not in ("gptq", "cdcl"):
            raise ValueError("method must be 'gptq' or 'cdcl'")
        c = CConfig()
        c.group = int(self.group)
        c.block = int(self.block)
        c.sub_block = int(self.sub_block)
        c.cd_sweeps = int(self.cd_sweeps)
        c.passes = int(self.passes)
        c.row_chunk = int(self.row_chunk)
        c.threads = int(self.threads)
        c.damp = float(self.damp)
        c.skeleton_pct = float(self.skeleton_pct)
        c.refine_frac = float(self.refine_frac)
        c.tol = float(self.tol)
        c.bits = int(self.bits)
        c.skeleton_bits = int(self.skeleton_bits)
        c.act_order = 1 if self.act_order else 0
        c.mse_grid = 1 if self.mse_grid else 0
        c.method = METHOD_CDCL if self.method == "cdcl" else METHOD_GPTQ
        c.refit_scales = 1 if self.refit_scales else 0
        return c

    def replace(self, **kw) -> "Config":
        d = {f.name: getattr(self, f.name) for f in fields(self)}
        d.update(kw)
        return Config(**d)

    def debug_string(self) -> str:
        """The `{:?}` rendering of the reference's Config, as stored in report.json (src/pipeline.rs:217)."""
        m = "Cdcl" if self.method == "cdcl" else "Gptq"

        def f(x):
            r = repr(float(x))
            return r

        return (
            "Config { bits: %d, group: %d, block: %d, damp: %s, act_order: %s, skeleton_pct: %s, skeleton_bits: %d, "
            "mse_grid: %s, method: %s, refine_frac: %s, sub_block: %d, cd_sweeps: %d, passes: %d, tol: %s, "
            "refit_scales: %s, row_chunk: %d }"
            % (self.bits, self.group, self.block, f(self.damp), str(self.act_order).lower(), f(self.skeleton_pct),
               self.skeleton_bits, str(self.mse_grid).lower(), m, f(self.refine_frac), self.sub_block,
               self.cd_sweeps, self.passes, f(self.tol), str(self.refit_scales).lower(), self.row_chunk)
        )


@dataclass
class LayerStats:
    """`engine::LayerStats` (src/engine.rs:173-199) plus `passes_max`."""

    loss_gptq: float = 0.0
    loss_final: float = 0.0
    subblocks_total: int = 0
    subblocks_refined: int = 0
    code_updates: int = 0
    skeleton_groups: int = 0
    bits_codes: float = 0.0
    bits_total: float = 0.0
    secs_prepare: float = 0.0
    secs_quant: float = 0.0
    passes_max: int = 0

    @staticmethod
    def from_c(s: CLayerStats) -> "LayerStats":
        return LayerStats(**{f.name: getattr(s, f.name) for f in fields(LayerStats)})


def effective_group(cfg: Config, n: int) -> int:
    """src/engine.rs:227-233."""
    return n if (cfg.group == 0 or cfg.group >= n) else cfg.group


def num_groups(cfg: Config, n: int) -> int:
    g = effective_group(cfg, n)
    return (n + g - 1) // g
