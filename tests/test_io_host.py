"""Host logic of cdclq.io without a GPU: the Hessian store's index, aliases and later-file override
(src/io.rs:136-188), and the packed reader's missing-tensor error."""
import json

import numpy as np
import pytest


def _write(path, tensors, aliases=None):
    from safetensors.numpy import save_file

    save_file(tensors, str(path), metadata={"aliases": json.dumps(aliases)} if aliases else None)


def test_hessian_store_index_aliases_and_override(tmp_path):
    from cdclq.io import HessianStore

    a, b = tmp_path / "a.safetensors", tmp_path / "b.safetensors"
    eye = np.eye(4, dtype=np.float32)
    _write(a, {"m.l0.q_proj.H": eye, "m.l0.o_proj.H": eye, "m.l0.o_proj.M": eye},
           aliases={"m.l0.k_proj": "m.l0.q_proj", "m.l0.v_proj": "m.l0.q_proj", "m.l0.ghost": "m.l9.none"})
    _write(b, {"m.l0.o_proj.H": 2 * eye})
    st = HessianStore([str(a), str(b)])
    assert st.resolve("m.l0.q_proj") == "m.l0.q_proj"
    assert st.resolve("m.l0.k_proj") == "m.l0.q_proj" and st.resolve("m.l0.v_proj") == "m.l0.q_proj"
    assert st.resolve("m.l0.ghost") is None  # alias to a layer without a Hessian
    assert st.resolve("m.l0.up_proj") is None
    assert st.index["m.l0.o_proj"] == 1  # the later file wins


def test_read_packed_layer_names_a_missing_tensor():
    import cdclq
    from cdclq.io import read_packed_layer

    t = {"x.qweight": np.zeros((2, 3), np.uint8), "x.scales": np.zeros((2, 1), np.float16)}
    with pytest.raises(cdclq.CdclqError) as ei:
        read_packed_layer(t, "x")
    assert str(ei.value) == "x.qzeros: tensor not found"
