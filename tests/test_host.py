"""CPU-only checks of the host side: the C-ABI library and its exports, the C struct layout,
the derived tables, parameter resolution and checkpoint loading. No GPU compute here."""

from __future__ import annotations

import ctypes
import re
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest

from oracle import descriptor as odesc
from rune_b200 import tables
from rune_b200.runtime import library as L
from tests.helpers import GOLDEN, ROOT, load_params, oam_checkpoint

HEADER = ROOT / "include" / "rune_b200.h"


def header_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^(?:int|void|const char\*)\s+(rune_\w+)\(", text, re.M)))


def test_library_exports_every_header_symbol():
    lib = L.load_library()
    names = header_functions()
    assert names, "no functions parsed from the header"
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(L.EXPORTED)


def test_struct_layout_matches_header(tmp_path):
    src = tmp_path / "layout.c"
    src.write_text(textwrap.dedent(f"""
        #include <stddef.h>
        #include <stdio.h>
        #include "{HEADER}"
        int main(void) {{
            printf("%zu %zu %zu %zu %zu\\n", sizeof(rune_model_config), sizeof(rune_stats),
                   offsetof(rune_model_config, message_cutoff),
                   offsetof(rune_model_config, zbl_rc_outer),
                   offsetof(rune_stats, tensor_core_layers));
            return 0;
        }}"""))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    want = [ctypes.sizeof(L.ModelConfig), ctypes.sizeof(L.Stats),
             L.ModelConfig.message_cutoff.offset, L.ModelConfig.zbl_rc_outer.offset,
             L.Stats.tensor_core_layers.offset]
    assert got == want


def test_status_codes_and_constants_match_header():
    text = HEADER.read_text()
    for name in ("RUNE_OK", "RUNE_ERR_INVALID", "RUNE_ERR_CUDA", "RUNE_ERR_NEIGHBOR_OVERFLOW",
                 "RUNE_ERR_TYPE", "RUNE_ERR_OOM", "RUNE_ERR_STATE", "RUNE_ERR_RETRY"):
        value = re.search(rf"#define {name} (\d+)", text)
        assert value and int(value.group(1)) == getattr(L, name), name
    polls = re.search(r"#define RUNE_DEFAULT_WAIT_POLLS (\d+)u", text)
    assert polls and int(polls.group(1)) == L.DEFAULT_WAIT_POLLS


def test_z_tables_are_legendre_derivatives():
    for order in range(1, 9):
        np.testing.assert_array_equal(np.array(tables.legendre_z_coefficients(order)),
                                      np.array(odesc.ZCOEF[order], float))


def test_invariant_term_table_matches_oracle():
    rng = np.random.default_rng(3)
    s = rng.normal(size=(7, 24))
    flags = (1, 1, 1, 1, 1, 1)
    t = tables.invariant_terms(4, flags, tables.C3B_VALUES, tables.C4B_VALUES,
                               tables.C5B_VALUES, tables.C4B2_VALUES)
    q = np.zeros((7, 10))
    for coef, out, *idx in t:
        v = np.full(7, coef, np.float64)
        for i in idx:
            if i >= 0:
                v = v * s[:, int(i)]
        q[:, int(out)] += v
    np.testing.assert_allclose(q, odesc.invariants(s, 4, flags), rtol=1e-6, atol=1e-9)


def test_random_init_matches_reference_seed():
    import torch

    from rune_b200.nep.plugin import build_model

    g = np.load(GOLDEN / "nep_fcc108.npz")
    torch.manual_seed(20261201)
    model = build_model(load_params(g))
    for key, value in model.state_dict().items():
        np.testing.assert_array_equal(value.numpy(), g[f"param:{key}"], err_msg=key)


@pytest.mark.parametrize("name", ["local", "scalar", "equivariant", "equivariant_flexzbl"])
def test_state_dict_layout_matches_reference(name):
    import torch

    from rune_b200.mobius.plugin import build_model

    g = np.load(GOLDEN / f"tiny_{name}.npz")
    model = build_model(load_params(g))
    ref = {k[len("param:"):]: g[k] for k in g.files if k.startswith("param:")}
    assert set(model.state_dict()) == set(ref)
    model.load_state_dict({k: torch.as_tensor(v) for k, v in ref.items()}, strict=True)


def test_checkpoints_load_strict():
    for variant in ("loc", "mp", "eq"):
        if oam_checkpoint(variant) is None:
            pytest.skip("repository weights not present")
        from rune_b200.mobius.plugin import load_model

        model = load_model(ROOT / "weights" / f"mobius-oam-{variant}.pt")
        assert model.params["n_types"] == 89


def test_resolve_params_errors():
    from rune_b200.mobius.plugin import resolve_params as mob
    from rune_b200.nep.plugin import resolve_params as nep

    with pytest.raises(ValueError, match="Unknown model parameter"):
        nep({"elements": ["Cu"], "bogus": 1})
    with pytest.raises(ValueError, match="hidden_dims"):
        nep({"elements": ["Cu"], "hidden_dims": [10, 10]})
    with pytest.raises(ValueError, match="cutoffs"):
        nep({"elements": ["Cu"], "rcut_radial": 4.0, "rcut_angular": 5.0})
    with pytest.raises(ValueError, match="divisible"):
        mob({"elements": ["Cu"], "hidden_dim": 10, "message_groups": 3})
    with pytest.raises(ValueError, match="Equivariant parameters"):
        mob({"elements": ["Cu"], "equivariant_channels": 4})
    p = mob({"elements": ["Fe", "C"], "message_mode": "equivariant"})
    assert p["equivariant_l_max"] == p["l_max"]


def test_checkpoint_identity_is_checked(tmp_path):
    import torch

    from rune_b200.mobius.plugin import load_model

    path = tmp_path / "bad.pt"
    torch.save({"plugin": {"name": "other"}, "model_params": {}}, path)
    with pytest.raises(ValueError, match="Checkpoint is not a mobius-force-field model"):
        load_model(path)


def test_calculator_host_errors():
    import torch

    from rune_b200.interface import EngineCalculator, PropertyNotImplementedError
    from rune_b200.mobius.plugin import build_model

    g = np.load(GOLDEN / "tiny_local.npz")
    params = load_params(g)

    class Calc(EngineCalculator):
        @staticmethod
        def _load(artifact, device):
            return build_model(params)

    class Atoms:
        positions = np.zeros((2, 3))
        cell = np.eye(3) * 5.0
        pbc = np.array([True, True, True])
        numbers = np.array([26, 1])

        def get_volume(self):
            return 125.0

    calc = Calc("unused", device="cpu", compute_stress=False)
    with pytest.raises(ValueError, match="not supported"):
        calc.calculate(Atoms(), ["energy"])
    Atoms.numbers = np.array([26, 6])
    with pytest.raises(PropertyNotImplementedError):
        calc.calculate(Atoms(), ["stress"])
    with pytest.raises(RuntimeError, match="CUDA"):
        calc.calculate(Atoms(), ["energy"])
    del torch


def test_no_cpu_fallback_in_product():
    """The product package never imports the oracle."""
    for path in (ROOT / "rune_b200").rglob("*.py"):
        text = path.read_text()
        assert "import oracle" not in text and "from oracle" not in text, path


def test_engine_requires_cuda_model():
    import torch

    from rune_b200.mobius.plugin import build_model

    g = np.load(GOLDEN / "tiny_local.npz")
    model = build_model(load_params(g))
    batch = {"types": torch.zeros(1, dtype=torch.long), "positions": torch.zeros(1, 3),
             "radial_neighbors": torch.full((1, 1), -1), "angular_neighbors": torch.full((1, 1), -1),
             "radial_offsets": torch.zeros(1, 1, 3), "angular_offsets": torch.zeros(1, 1, 3),
             "n_atoms_per_structure": torch.tensor([1])}
    with pytest.raises(RuntimeError, match="CUDA devices only"):
        model(batch)
