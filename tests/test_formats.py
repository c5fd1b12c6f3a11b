"""On-disk model formats against the reference's own reader and exporter: GPUMD nep.txt
(rune/nep/model.py:284-489) and the native mobius1 file (rune/mobius/export.py:120-146,
rune/mobius/src/mobius.cu:26-151). Fixtures: tests/golden/make_formats.py."""

from __future__ import annotations

import ast

import numpy as np
import pytest
import torch

from rune_b200.mobius.native import load_mobius1
from rune_b200.nep.plugin import load_model as load_nep

from .helpers import GOLDEN

NEP = np.load(GOLDEN / "nep_txt.npz")
MOB = np.load(GOLDEN / "mobius1.npz")


def _cases(store):
    return sorted({k.split(":")[0] for k in store.files})


def _state(store, case):
    pre = f"{case}:param:"
    return {k[len(pre):]: store[k] for k in store.files if k.startswith(pre)}


@pytest.mark.parametrize("case", _cases(NEP))
def test_nep_txt_matches_reference_reader(case, tmp_path):
    path = tmp_path / "nep.txt"
    path.write_text(str(NEP[f"{case}:text"]))
    model = load_nep(path)
    ref_params = ast.literal_eval(str(NEP[f"{case}:params"]))
    for key, value in ref_params.items():
        assert model.params[key] == value, key
    ref_state = _state(NEP, case)
    state = model.state_dict()
    assert set(state) == set(ref_state)
    for key, value in ref_state.items():
        np.testing.assert_array_equal(state[key].double().numpy(), value, err_msg=key)


def test_nep_txt_errors(tmp_path):
    text = str(NEP["plain:text"])
    path = tmp_path / "nep.txt"
    path.write_text(text.replace("nep4", "nap4", 1))
    with pytest.raises(ValueError, match="first line should start with nep4 or nep5"):
        load_nep(path)
    path.write_text(text.replace("nep4", "nep5", 1))
    with pytest.raises(NotImplementedError, match="Only nep4"):
        load_nep(path)
    lines = text.splitlines()
    ann = next(i for i, line in enumerate(lines) if line.startswith("ANN"))
    lines[ann] = lines[ann].replace("ANN 7 0", "ANN 7 3")
    path.write_text("\n".join(lines))
    with pytest.raises(ValueError, match="single-hidden-layer"):
        load_nep(path)
    per_type = str(NEP["pertype:text"]).splitlines()
    tokens = per_type[1].split()
    tokens[3] = "4.5"  # a different radial cutoff for the second type
    per_type[1] = " ".join(tokens)
    path.write_text("\n".join(per_type))
    with pytest.raises(NotImplementedError, match="Per-type cutoffs"):
        load_nep(path)
    path.write_text("\n".join(text.splitlines()[:9]))
    with pytest.raises(ValueError, match="too short"):
        load_nep(path)


@pytest.mark.parametrize("case", _cases(MOB))
def test_mobius1_matches_reference_export(case, tmp_path):
    path = tmp_path / "mobius.txt"
    path.write_text(str(MOB[f"{case}:text"]))
    model = load_mobius1(path)
    ref_params = ast.literal_eval(str(MOB[f"{case}:params"]))
    for key in ("elements", "n_desc_radial", "n_desc_angular", "k_max_radial", "k_max_angular",
                "l_max", "hidden_dim", "blocks", "ffn_dim", "message_layers", "message_dim",
                "pair_dim", "message_groups", "vector_channels", "message_basis_size",
                "rcut_radial", "rcut_angular", "message_cutoff", "activation", "has_q_222",
                "has_q_1111", "has_q_112", "has_q_123", "has_q_233", "has_q_134"):
        assert model.params[key] == ref_params[key], key
    assert model.params.get("message_mode", "scalar") == ref_params.get("message_mode",
                                                                         "scalar")
    ref_state = _state(MOB, case)
    state = model.state_dict()
    assert set(state) == set(ref_state)
    for key, value in ref_state.items():
        np.testing.assert_array_equal(state[key].double().numpy(),
                                      value.astype(np.float32).astype(np.float64), err_msg=key)


def test_mobius1_errors(tmp_path):
    text = str(MOB["local:text"])
    path = tmp_path / "mobius.txt"
    path.write_text(text.replace("mobius1", "mobius2", 1))
    with pytest.raises(ValueError, match="expected 'mobius1' in model file"):
        load_mobius1(path)
    path.write_text(text.replace("schema 1", "schema 2", 1))
    with pytest.raises(ValueError, match="unsupported native schema"):
        load_mobius1(path)
    path.write_text(text.replace("END", "", 1))
    with pytest.raises(ValueError, match="expected 'END' in model file"):
        load_mobius1(path)
    path.write_text(text + "extra\n")
    with pytest.raises(ValueError, match="unexpected data after END"):
        load_mobius1(path)
    lines = text.splitlines()
    cut = next(i for i, line in enumerate(lines) if line.startswith("tensors"))
    path.write_text("\n".join(lines[:cut + 3]))
    with pytest.raises(ValueError, match="missing or nonfinite tensor values"):
        load_mobius1(path)


def test_plugins_dispatch_text_formats(tmp_path):
    from rune_b200.mobius.plugin import load_model as load_mobius

    path = tmp_path / "mobius.txt"
    path.write_text(str(MOB["scalar:text"]))
    model = load_mobius(path)
    assert model.message_layers == 2
    path = tmp_path / "nep.txt"
    path.write_text(str(NEP["zbl:text"]))
    nep = load_nep(path)
    assert nep.zbl is not None and not nep.zbl.flexible
    assert isinstance(nep.shared_bias, torch.nn.Parameter)
