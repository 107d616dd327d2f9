"""GGUF loader: layers written in the model file's naming and layout read
back byte for byte (CPU), and a layer loaded from the file decodes exactly
like the same layer uploaded directly (GPU)."""
from __future__ import annotations

import numpy as np
import pytest

from flash_moe_b200 import gguf_store, synth
from flash_moe_b200.formats import Q3_K, Q4_K, Q5_K, Q6_K, Q8_0


def _layers():
    a = synth.make_layer(seed=81, hidden=512, inter=256, n_experts=8, top_k=2, gate_type=Q4_K,
                         up_type=Q4_K, down_type=Q8_0, shared_inter=256,
                         shared_types=(Q6_K, Q6_K, Q5_K))
    b = synth.make_layer(seed=82, hidden=512, inter=256, n_experts=8, top_k=2, gate_type=Q3_K,
                         up_type=Q3_K, down_type=Q6_K, shared_inter=0)
    return {0: a, 3: b}


def test_write_read_round_trip(tmp_path):
    layers = _layers()
    path = gguf_store.write_layers(tmp_path / "m.gguf", layers)
    assert gguf_store.moe_layers(path) == [0, 3]
    assert gguf_store.expert_tensor_types(path) == {l: lw.kinds for l, lw in layers.items()}
    for l, lw in layers.items():
        got = gguf_store.layer_weights(path, l, top_k=lw.top_k)
        assert (got.hidden, got.inter, got.n_experts) == (lw.hidden, lw.inter, lw.n_experts)
        assert got.kinds == lw.kinds
        for role in ("gate", "up", "down"):
            np.testing.assert_array_equal(getattr(got, role), getattr(lw, role))
        np.testing.assert_array_equal(got.router, lw.router)
        assert got.shared_inter == lw.shared_inter
        if lw.shared_inter:
            assert got.shared_types == lw.shared_types
            for role in ("gate", "up", "down"):
                np.testing.assert_array_equal(getattr(got, f"shared_{role}"),
                                              getattr(lw, f"shared_{role}"))
            np.testing.assert_array_equal(got.shared_gate_inp, lw.shared_gate_inp)
        for e in (0, lw.n_experts - 1):
            for role, arr in got.expert(e).items():
                np.testing.assert_array_equal(arr, lw.expert(e)[role])


def test_missing_layer_and_bad_type(tmp_path):
    import gguf
    path = gguf_store.write_layers(tmp_path / "m.gguf", _layers())
    with pytest.raises(KeyError):
        gguf_store.layer_weights(path, 1)
    w = gguf.GGUFWriter(str(tmp_path / "f16.gguf"), "qwen35moe")
    for role, shape in (("gate", (4, 8, 256)), ("up", (4, 8, 256)), ("down", (4, 256, 8))):
        w.add_tensor(f"blk.0.ffn_{role}_exps.weight", np.zeros(shape, np.float16))
    w.add_tensor("blk.0.ffn_gate_inp.weight", np.zeros((4, 256), np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pytest.raises(ValueError, match="supported block formats"):
        gguf_store.layer_weights(tmp_path / "f16.gguf", 0)


@pytest.mark.gpu
def test_gguf_layer_decodes_like_direct_upload(tmp_path):
    import torch
    from flash_moe_b200.backend import B200ExpertBackend
    from flash_moe_b200.store import ExpertArena
    layers = _layers()
    path = gguf_store.write_layers(tmp_path / "m.gguf", layers)
    from_file = B200ExpertBackend(gguf_store.load_arena(path, top_k=2))
    direct_arena = ExpertArena()
    for l, lw in layers.items():
        direct_arena.add_layer(l, lw)
    direct = B200ExpertBackend(direct_arena)
    xs = synth.make_tokens(83, 3, 512)
    for l in layers:
        a = from_file.forward_layer(l, xs)
        b = direct.forward_layer(l, xs)
        np.testing.assert_array_equal(a, b)
