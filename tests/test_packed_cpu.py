"""The on-disk super-block format (safetensors): round trips of oracle-packed streams,
metadata, and the error cases. No GPU."""

import json

import numpy as np
import pytest

from oracle import int4 as O


def _streams():
    a = O.quantize_pack_matrix(O.make_weights(256, 512, 1))
    b = O.quantize_pack_matrix(O.make_weights(512, 256, 2))
    return {"model.layers.0.self_attn.q_proj": {"superblocks": a, "original_shape": (256, 512), "n_elements": 256 * 512},
            "lm_head": {"superblocks": b, "original_shape": (512, 256), "n_elements": 512 * 256,
                        "variant": "toplevel"}}


def test_round_trip_bytes_and_metadata(tmp_path):
    from moat_b200.packed import FORMAT, load_packed, save_packed
    layers = _streams()
    p = str(tmp_path / "w.safetensors")
    save_packed(p, layers)
    got = load_packed(p)
    assert set(got) == set(layers)
    for name, layer in layers.items():
        np.testing.assert_array_equal(got[name]["superblocks"], layer["superblocks"])
        assert got[name]["original_shape"] == layer["original_shape"]
        assert got[name]["n_elements"] == layer["n_elements"]
        assert got[name]["variant"] == layer.get("variant", "engine")
        assert got[name]["group_size"] == 32
    # a plain safetensors reader sees uint8 streams and the metadata records
    from safetensors import safe_open
    with safe_open(p, framework="numpy") as f:
        meta = f.metadata()
        assert meta["format"] == FORMAT
        rec = json.loads(meta["lm_head"])
        assert rec["shape"] == [512, 256] and rec["variant"] == "toplevel"
        t = f.get_tensor("model.layers.0.self_attn.q_proj")
        assert t.dtype == np.uint8 and t.shape == (256 * 512 // 256 * 144,)


def test_dequant_of_loaded_stream_matches_oracle(tmp_path):
    from moat_b200.packed import load_packed, save_packed
    w = O.make_weights(64, 256, 3)
    st = O.quantize_pack_matrix(w)
    p = str(tmp_path / "w.safetensors")
    save_packed(p, {"w": {"superblocks": st, "original_shape": (64, 256), "n_elements": 64 * 256}})
    got = load_packed(p)["w"]["superblocks"]
    np.testing.assert_array_equal(O.unpack_superblock_weights(got).view(np.uint16),
                                  O.unpack_superblock_weights(st).view(np.uint16))


def test_rejects_bad_inputs(tmp_path):
    from moat_b200.packed import load_packed, save_packed
    with pytest.raises(ValueError):
        save_packed(str(tmp_path / "a.safetensors"), {"x": {"superblocks": np.zeros(100, np.uint8)}})
    with pytest.raises(ValueError):
        save_packed(str(tmp_path / "b.safetensors"),
                    {"x": {"superblocks": np.zeros(144, np.uint8), "n_elements": 257}})
    from safetensors.numpy import save_file
    other = str(tmp_path / "other.safetensors")
    save_file({"x": np.zeros(144, np.uint8)}, other, metadata={"format": "something-else"})
    with pytest.raises(ValueError):
        load_packed(other)
