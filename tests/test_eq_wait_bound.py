"""The EQ kernels' bounded waits, run out on healthy copies (no fault, trap or hang): with the wait
bound at 0 polls every wait on a weight copy or a tensor-core completion gives up at once, the
blocks let their copies in flight land and return, and the call raises the engine's error; the
CUDA context stays usable, and with the default bound restored the next call reproduces the
earlier result bit for bit. Both edge-product forms are covered: the SIMT ring of bulk copies and
the tcgen05 path (RUNE_EQ_TENSOR_CORES=1)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.helpers import GOLDEN, load_params, load_state

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _tiny_eq():
    from rune_b200.mobius.plugin import build_model

    g = np.load(GOLDEN / "tiny_equivariant.npz")
    model = build_model(load_params(g))
    model.load_state_dict({k: torch.as_tensor(v, dtype=torch.float32)
                           for k, v in load_state(g).items()}, strict=True)
    return model.to(DEV).eval(), g


def _run(model, g):
    pos = torch.as_tensor(g["tri:positions"], dtype=torch.float64, device=DEV)
    types = torch.as_tensor(g["tri:types"], dtype=torch.int32, device=DEV)
    res = model.evaluate(pos, np.asarray(g["tri:cell"]).reshape(1, 9), np.ones((1, 3), bool),
                         types)
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in res.items()}


@pytest.mark.parametrize("tensor_cores", [False, True])
def test_wait_bound_runs_out_and_recovers(monkeypatch, tensor_cores):
    from rune_b200.runtime.library import DEFAULT_WAIT_POLLS

    if tensor_cores:
        monkeypatch.setenv("RUNE_EQ_TENSOR_CORES", "1")
    else:
        monkeypatch.delenv("RUNE_EQ_TENSOR_CORES", raising=False)
    model, g = _tiny_eq()
    base = _run(model, g)
    engine = model.engine()
    assert engine.stats()["tensor_core_layers"] == (model.message_layers if tensor_cores else 0)
    engine.set_wait_polls(0)
    with pytest.raises(RuntimeError, match="did not complete in time"):
        _run(model, g)
    # the context is intact: other device work runs, and the engine recovers
    assert float(torch.ones(1024, device=DEV).sum()) == 1024.0
    engine.set_wait_polls(DEFAULT_WAIT_POLLS)
    again = _run(model, g)
    for key in base:
        np.testing.assert_array_equal(again[key], base[key])
