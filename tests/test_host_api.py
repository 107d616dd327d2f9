"""Host-side logic of the reference-facing Python API, on the CPU: the
checks ``run_moe_layer`` / ``run_moe_sequence`` make before the single
device call, and the selection policy of ``load_native_expert``."""
from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest

from flash_moe_b200 import native_expert as NE
from flash_moe_b200.moe_layer import run_moe_layer, run_moe_sequence


class _Backend:
    """A backend whose layer call returns a recognisable value."""

    def __init__(self, hidden=8, inter=4, experts=6, top_k=2):
        w = SimpleNamespace(hidden=hidden, inter=inter, n_experts=experts, top_k=top_k)
        self.store = SimpleNamespace(layer=lambda l: SimpleNamespace(weights=w))
        self.calls = []

    def forward_layer(self, layer, x):
        self.calls.append((layer, np.array(x)))
        return np.asarray(x, np.float32) * 2


def _router(**kw):
    base = dict(top_k=2, num_experts=6, hidden_size=8, gate_dtype=np.dtype(np.float32))
    base.update(kw)
    return SimpleNamespace(**base)


def test_layer_call_goes_to_forward_layer():
    be = _Backend()
    x = np.arange(8, dtype=np.float32)
    np.testing.assert_array_equal(run_moe_layer(3, x, _router(), be, 8, 4), x * 2)
    xs = np.ones((5, 8), np.float32)
    np.testing.assert_array_equal(run_moe_sequence(3, xs, _router(), be, 8, 4), xs * 2)
    assert [c[0] for c in be.calls] == [3, 3]


@pytest.mark.parametrize("bad", [dict(gate_dtype=np.dtype(np.float16)), dict(top_k=3),
                                 dict(num_experts=7), dict(hidden_size=16)])
def test_router_that_differs_from_the_resident_layer_is_rejected(bad):
    with pytest.raises(ValueError):
        run_moe_layer(0, np.zeros(8, np.float32), _router(**bad), _Backend(), 8, 4)


def test_shape_checks():
    be = _Backend()
    with pytest.raises(ValueError):
        run_moe_layer(0, np.zeros(8, np.float32), _router(), be, 8, 8)
    with pytest.raises(ValueError):
        run_moe_layer(0, np.zeros(9, np.float32), _router(), be, 8, 4)
    with pytest.raises(ValueError):
        run_moe_sequence(0, np.zeros((2, 9), np.float32), _router(), be, 8, 4)
    assert not be.calls


def test_per_expert_backend_is_refused():
    with pytest.raises(TypeError):
        run_moe_layer(0, np.zeros(8, np.float32), _router(), SimpleNamespace(), 8, 4)


def test_load_native_expert_policy(monkeypatch, capsys):
    types = {0: {"gate": 11, "up": 11, "down": 12}}
    with pytest.raises(ValueError):
        NE.load_native_expert("fast", None, "CUDA", types)
    assert NE.load_native_expert("openvino", None, "CUDA", types) is None
    # a CPU device is never served, whatever the GPUs
    monkeypatch.setattr(NE, "cuda_device_count", lambda: 1)
    assert NE.load_native_expert("auto", None, "CPU", types) is None
    assert "CUDA device" in capsys.readouterr().out
    with pytest.raises(RuntimeError, match="CUDA device"):
        NE.load_native_expert("native", None, "CPU", types)
    # unsupported formats
    with pytest.raises(RuntimeError, match="unsupported"):
        NE.load_native_expert("native", None, "cuda:0", {0: {"gate": 2, "up": 11, "down": 12}})
    # no visible GPU
    monkeypatch.setattr(NE, "cuda_device_count", lambda: 0)
    with pytest.raises(RuntimeError, match="no CUDA device"):
        NE.load_native_expert("native", None, "GPU", types)
    assert NE.load_native_expert("auto", None, "GPU", types) is None
