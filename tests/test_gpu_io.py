"""Device ingest and packed output (cdclq.io) against the reference's rules: lossless widening, the load-time
non-finite refusal with its message, and the packed layer format (byte-exact with the oracle's packer, exact
round trip through a safetensors file)."""
import numpy as np
import pytest

import oracle as orc
from cdclq.abi import Config

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt", ["float32", "float16", "bfloat16"])
def test_widen_on_device_is_lossless(gpu, dt):
    import torch

    from cdclq.io import to_device_f32

    g = torch.Generator().manual_seed(3)
    x = (torch.randn(257, 129, generator=g) * 100).to(getattr(torch, dt))
    x[0, 0] = float("inf")
    x[1, 1] = float("-inf")
    y = to_device_f32(x)
    torch.cuda.synchronize()
    assert torch.equal(y.cpu(), x.float())


def test_non_finite_hessian_is_refused_with_the_reference_message(gpu, tmp_path):
    import torch
    from safetensors.numpy import save_file

    import cdclq
    from cdclq.io import HessianStore

    n = 64
    h = np.eye(n, dtype=np.float32)
    h[7, 9] = np.inf
    h[3, 5] = np.nan  # the first in row-major order
    p = tmp_path / "h.safetensors"
    save_file({"m.layers.0.mlp.H": h, "m.layers.0.attn.H": np.eye(n, dtype=np.float32)}, str(p))
    st = HessianStore([str(p)])
    with pytest.raises(cdclq.CdclqError) as ei:
        st.get_h("m.layers.0.mlp")
    assert ei.value.code == -5
    assert str(ei.value) == ("m.layers.0.mlp.H: 64 x 64 matrix has a non-finite entry (NaN) at [ 3, 5 ]; the "
                             "calibration data or the captured forward is corrupt, refusing to quantize")
    d, nn = st.get_h("m.layers.0.attn")
    torch.cuda.synchronize()
    assert nn == n and torch.equal(d.cpu(), torch.eye(n))
    with pytest.raises(cdclq.CdclqError) as ei:
        st.get_h("m.layers.9.mlp")
    assert str(ei.value) == "no Hessian for m.layers.9.mlp"


def test_packed_layer_roundtrip_and_bytes(gpu, tmp_path):
    import cdclq
    from safetensors.numpy import load_file

    from cdclq.io import packed_tensors, read_packed_layer, save_packed

    d_out, n = 48, 256
    w, h = orc.problem(d_out, n, 900, 61)
    cfg = Config(bits=4, group=32, block=32, skeleton_pct=10.0, row_chunk=16)  # mixed widths (skeleton groups)
    ql, _ = cdclq.quantize_layer(w, d_out, n, h, None, "x", cfg)
    t = packed_tensors("model.layers.0.mlp.down_proj", ql)
    assert t["model.layers.0.mlp.down_proj.qweight"].dtype == np.uint8
    assert np.array_equal(t["model.layers.0.mlp.down_proj.qweight"], orc.pack(ql.codes, d_out, n, ql.group, ql.gbits)[0])
    assert np.array_equal(t["model.layers.0.mlp.down_proj.scales"].astype(np.float32), ql.scales)
    assert np.array_equal(t["model.layers.0.mlp.down_proj.qzeros"].astype(np.float32), ql.zeros)
    p = tmp_path / "packed.safetensors"
    save_packed(str(p), t)
    back = read_packed_layer(load_file(str(p)), "model.layers.0.mlp.down_proj")
    for k in ("perm", "gbits", "codes", "scales", "zeros"):
        assert np.array_equal(getattr(back, k), getattr(ql, k)), k
    assert back.group == ql.group and back.d_in == n and back.d_out == d_out
    assert np.array_equal(back.dequantize(), ql.dequantize())
