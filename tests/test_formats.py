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


@pytest.mark.parametrize("case", _cases(NEP))
def test_nep_export_matches_reference_exporter(case, tmp_path):
    """export_model of the model read from the fixture writes the reference exporter's text
    (rune/nep/plugin.py:84-91, rune/nep/model.py:491-579), and reading it back gives the same
    state_dict bit for bit."""
    from rune_b200.nep.plugin import export_model

    path = tmp_path / "nep.txt"
    path.write_text(str(NEP[f"{case}:text"]))
    model = load_nep(path)
    (tmp_path / "out").mkdir()
    out = export_model(model, tmp_path / "out" / "model")
    assert out.name == str(NEP[f"{case}:export_name"]) == "nep.txt"
    assert out.read_text() == str(NEP[f"{case}:export"])
    again = load_nep(out)
    for key, value in model.state_dict().items():
        assert torch.equal(again.state_dict()[key], value), key


def test_export_paths(tmp_path):
    from rune_b200.mobius.export import export_path
    from rune_b200.nep.plugin import export_model

    assert export_path(tmp_path / "model").name == "mobius.txt"
    assert export_path(tmp_path / "model_epoch_12").name == "mobius_epoch_12.txt"
    assert export_path(tmp_path / "custom.txt").name == "custom.txt"
    path = tmp_path / "nep.txt"
    path.write_text(str(NEP["plain:text"]))
    model = load_nep(path)
    assert export_model(model, tmp_path / "model_epoch_3").name == "nep_epoch_3.txt"


@pytest.mark.parametrize("case", _cases(MOB))
def test_mobius1_export_matches_reference_exporter(case, tmp_path):
    """The fixture texts are the reference exporter's output (rune/mobius/export.py:120-146) for
    float32 models; exporting the model read from them writes the same bytes, and the
    plugin's export_model names a trainer's ``model`` ``mobius.txt``."""
    from rune_b200.mobius.plugin import export_model

    text = str(MOB[f"{case}:text"])
    path = tmp_path / "in.txt"
    path.write_text(text)
    model = load_mobius1(path)
    out = export_model(model, tmp_path / "model")
    assert out.name == "mobius.txt"
    assert out.read_text() == text
    again = load_mobius1(out)
    for key, value in model.state_dict().items():
        assert torch.equal(again.state_dict()[key], value), key


def test_mobius1_export_of_a_checkpoint_model(tmp_path):
    """A seeded float32 model (not read from a file) exports and reads back bit for bit."""
    from rune_b200.mobius.plugin import build_model, export_model, resolve_params

    params = resolve_params(dict(elements=["Si", "O"], rcut_radial=4.0, rcut_angular=3.5,
                                 n_max_radial=2, n_max_angular=2, basis_size_radial=3,
                                 basis_size_angular=3, l_max=4, l_max_4body=2, l_max_5body=1,
                                 has_q_112=1, has_q_123=1, has_q_233=1, has_q_134=1,
                                 hidden_dim=8, ffn_dim=12, blocks=1, message_layers=1,
                                 message_dim=8, pair_dim=3, message_groups=2,
                                 message_mode="equivariant", equivariant_channels=3,
                                 zbl=[0.7, 2.0]))
    torch.manual_seed(3)
    model = build_model(params)
    out = export_model(model, tmp_path / "m.txt")
    again = load_mobius1(out)
    for key, value in model.state_dict().items():
        assert torch.equal(again.state_dict()[key], value.float()), key
    assert export_model(again, tmp_path / "m2.txt").read_text() == out.read_text()
