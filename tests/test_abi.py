"""The C-ABI libraries load and export every symbol include/cdclq.h declares (no GPU needed, no compute)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "cdclq.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(cdclq_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_reference_entry_points():
    syms = declared_symbols()
    for s in ["cdclq_quantize_layer", "cdclq_upper_chol_of_inverse", "cdclq_gram_accumulate", "cdclq_cholesky_lower",
              "cdclq_tri_inverse_lower", "cdclq_quantize_batch", "cdclq_prep_cache_new", "cdclq_last_error"]:
        assert s in syms


def test_cuda_library_exports_every_declared_symbol():
    import cdclq

    L = cdclq.lib()
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, missing
    from cdclq._lib import SIGNATURES

    assert set(SIGNATURES) == set(declared_symbols())


def test_cuda_library_is_sm100a():
    """The shipped library carries sm_100a code (cuobjdump is not used: the fatbin is only listed by nvcc's
    own ELF section name)."""
    import cdclq

    data = open(cdclq.LIB_PATH, "rb").read()
    assert b".nv_fatbin" in data


def test_host_logic_without_gpu():
    """Configuration helpers are host code and work without a device."""
    import cdclq
    from cdclq.abi import Config

    L = cdclq.lib()
    c = cdclq.abi.CConfig()
    L.cdclq_config_default(ctypes.byref(c))
    d = Config()
    for f, v in [("bits", 3), ("group", 128), ("block", 128), ("sub_block", 64), ("passes", 10), ("cd_sweeps", 1)]:
        assert getattr(c, f) == v == getattr(d, f)
    assert abs(c.tol - 1e-3) < 1e-15 and abs(c.damp - 0.01) < 1e-15 and c.refine_frac == 1.0
    assert c.act_order == 1 and c.refit_scales == 1 and c.mse_grid == 0 and c.method == 1
    assert cdclq.effective_group(Config(group=0), 100) == 100
    assert cdclq.effective_group(Config(group=128), 100) == 100
    assert cdclq.effective_group(Config(group=32), 100) == 32
    assert L.cdclq_num_groups(ctypes.byref(Config(group=32).to_c()), 100) == 4
    for cfg, msg in [(Config(bits=1), "bits and skeleton_bits must be in 2..=8"),
                     (Config(sub_block=0), "block and sub_block must be > 0"),
                     (Config(group=96, block=64), "group size 96 must divide the block size 64 (or be a multiple of it)"),
                     (Config(refine_frac=-0.1), "refine_frac must be in [0, 1]")]:
        with pytest.raises(cdclq.CdclqError) as ei:
            cdclq.validate(cfg, 512)
        assert str(ei.value) == msg and ei.value.code == -1
    cdclq.validate(Config(group=256, block=128), 512)
    assert cdclq.row_chunk(Config(row_chunk=128), 1000) == 128
    assert cdclq.row_chunk(Config(row_chunk=0, threads=24), 2048) == 86
    assert cdclq.row_chunk(Config(row_chunk=0, threads=24), 256) == 32
    assert cdclq.row_chunk(Config(row_chunk=0, threads=24), 5632) == 235
    assert cdclq.row_chunk(Config(row_chunk=0, threads=1), 5632) == 256
    assert cdclq.row_chunk(Config(row_chunk=500), 100) == 100


def test_row_chunk_matches_oracle():
    import cdclq
    import oracle as orc
    from cdclq.abi import Config

    for cfg in [Config(row_chunk=0, threads=t) for t in (1, 3, 8, 24, 96)] + [Config(row_chunk=r) for r in (1, 7, 128)]:
        for d in (1, 31, 256, 2048, 5632):
            assert cdclq.row_chunk(cfg, d) == orc.row_chunk(cfg, d)
