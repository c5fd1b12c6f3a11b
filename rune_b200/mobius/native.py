"""Reader of the ``mobius1`` text format (the native GPUMD evaluator's model file).

The reference writes it with ``rune.mobius.export.export_model`` (rune/mobius/export.py:79-146)
and reads it in C++ (rune/mobius/src/mobius.cu:26-151). This reader applies the same structure
checks, with the native reader's messages (as ``ValueError``), and rebuilds a Möbius model whose
parameters are the file's tensors, rounded to float32, so a GPUMD-style user can evaluate a
native model file on the engine without the torch checkpoint.
"""

from __future__ import annotations

import itertools
import math
from pathlib import Path

import numpy as np
import torch

from .. import tables

_ACTIVATIONS = {0: "tanh", 1: "silu", 2: "gelu"}
_FLAGS = ("has_q_222", "has_q_1111", "has_q_112", "has_q_123", "has_q_233", "has_q_134")


def _require(condition, message):
    if not condition:
        raise ValueError(message)


def read_mobius1(path):
    """(elements, ints, reals, tensors) of a mobius1 file; tensors as float64 arrays."""
    tokens = Path(path).read_text().split()
    pos = 0

    def word(message):
        nonlocal pos
        _require(pos < len(tokens), message)
        pos += 1
        return tokens[pos - 1]

    def integer(message):
        try:
            return int(word(message))
        except ValueError:
            raise ValueError(message) from None

    def real(message):
        try:
            value = float(word(message))
        except ValueError:
            raise ValueError(message) from None
        _require(math.isfinite(value), message)
        return value

    def expect(name):
        _require(pos < len(tokens) and word("") == name, f"expected '{name}' in model file")

    expect("mobius1")
    count = integer("invalid element count")
    _require(0 < count <= 118, "invalid element count")
    elements = [word("missing element") for _ in range(count)]
    _require(len(set(elements)) == len(elements), "duplicate elements")
    expect("schema")
    _require(integer("unsupported native schema") == 1, "unsupported native schema")
    expect("ints")
    count = integer("invalid integer metadata count")
    _require(0 < count < 1000, "invalid integer metadata count")
    ints = {}
    for _ in range(count):
        key = word("invalid integer metadata")
        value = integer("invalid integer metadata")
        _require(key not in ints, "duplicate integer metadata")
        ints[key] = value
    expect("reals")
    count = integer("invalid real metadata count")
    _require(0 < count < 1000, "invalid real metadata count")
    reals = {}
    for _ in range(count):
        key = word("invalid real metadata")
        value = real("invalid real metadata")
        _require(key not in reals, "duplicate real metadata")
        reals[key] = value
    expect("tensors")
    count = integer("invalid tensor count")
    _require(0 < count < 100000, "invalid tensor count")
    tensors = {}
    for _ in range(count):
        key = word("invalid tensor rank")
        rank = integer("invalid tensor rank")
        _require(0 <= rank <= 8, "invalid tensor rank")
        shape = []
        for _ in range(rank):
            dim = integer("invalid tensor dimension")
            _require(dim >= 0, "invalid tensor dimension")
            shape.append(dim)
        size = int(np.prod(shape)) if shape else 1
        _require(pos + size <= len(tokens), "missing or nonfinite tensor values")
        try:
            values = np.array(tokens[pos:pos + size], dtype=np.float64)
        except ValueError:
            raise ValueError("missing or nonfinite tensor values") from None
        _require(bool(np.isfinite(values).all()), "missing or nonfinite tensor values")
        pos += size
        _require(key not in tensors, "duplicate tensor name")
        tensors[key] = values.reshape(shape)
    expect("END")
    _require(pos == len(tokens), "unexpected data after END")
    return elements, ints, reals, tensors


def _check(elements, ints, reals, tensors):
    """The native reader's consistency checks (mobius.cu:77-150)."""
    i, r = ints.get, reals.get
    _require(i("n_types") == len(elements), "element count mismatch")
    for key in ("n_desc_radial", "n_desc_angular", "k_max_radial", "k_max_angular", "num_L",
                "input_dim", "hidden_dim", "ffn_dim", "message_dim", "pair_dim",
                "message_groups", "message_basis_size"):
        _require((i(key) or 0) > 0, f"invalid {key}")
    _require(i("message_layers", -1) >= 0 and i("blocks", -1) >= 0, "negative layer count")
    _require(i("activation") in _ACTIVATIONS, "unsupported activation")
    _require(i("message_mode") in (0, 1), "unsupported message mode")
    _require(1 <= (i("l_max") or 0) <= 8, "unsupported angular order")
    _require(not i("message_layers") or i("hidden_dim") % i("message_groups") == 0,
             "invalid message groups")
    _require(all((r(k) or 0) > 0 for k in ("rcut_radial", "rcut_angular", "message_cutoff",
                                            "norm_eps")),
             "cutoffs and normalization epsilon must be positive")
    _require(r("message_cutoff") <= r("rcut_radial"), "message cutoff exceeds radial cutoff")
    _require(i("max_neighbors_radial", 0) > 0 and i("max_neighbors_angular", 0) > 0 and
             i("vector_channels", -1) >= 0, "invalid neighbor/channel capacity")
    _require(i("input_dim") == i("n_desc_radial") + i("n_desc_angular") * i("num_L"),
             "descriptor dimension mismatch")
    eq = i("message_mode") == 1
    _require(not eq or (i("equivariant_channels", 0) > 0 and
                        1 <= i("equivariant_l_max", 0) <= i("l_max") and i("message_layers") > 0),
             "invalid equivariant dimensions")


def _invariant_flags(l_max, num_l, table):
    """The invariant flags whose terms reproduce the file's invariant table."""
    for flags in itertools.product((0, 1), repeat=6):
        if l_max + sum(flags) != num_l:
            continue
        terms = tables.invariant_terms(l_max, flags, tables.C3B_VALUES, tables.C4B_VALUES,
                                       tables.C5B_VALUES, tables.C4B2_VALUES)
        if len(terms) != len(table):
            continue
        idx = table[:, 3:7].astype(int)
        if np.array_equal(terms[:, 2:6].astype(int), idx) and np.array_equal(
                terms[:, 1].astype(int), table[:, 0].astype(int)):
            return dict(zip(_FLAGS, flags))
    raise ValueError("invalid descriptor polynomial tables")


def load_mobius1(path, device=None):
    """Möbius model from a mobius1 file (engine-evaluated)."""
    from .model import Mobius

    elements, ints, reals, tensors = read_mobius1(path)
    _check(elements, ints, reals, tensors)
    _require(tensors.get("desc.invariant_terms") is not None and
             tensors["desc.invariant_terms"].shape[-1] == 7,
             "invalid descriptor polynomial tables")
    flags = _invariant_flags(ints["l_max"], ints["num_L"], tensors["desc.invariant_terms"])
    params = {name: ints[name] for name in (
        "n_desc_radial", "n_desc_angular", "k_max_radial", "k_max_angular", "l_max",
        "hidden_dim", "blocks", "ffn_dim", "message_layers", "message_dim", "pair_dim",
        "message_groups", "vector_channels", "message_basis_size", "max_neighbors_radial",
        "max_neighbors_angular")}
    params.update({name: reals[name] for name in ("rcut_radial", "rcut_angular",
                                                   "message_cutoff", "norm_eps")})
    params.update(flags)
    params["l_max_4body"] = 2 if flags["has_q_222"] else 0
    params["l_max_5body"] = 1 if flags["has_q_1111"] else 0
    params["elements"] = list(elements)
    params["n_types"] = len(elements)
    params["activation"] = _ACTIVATIONS[ints["activation"]]
    if ints["message_mode"] == 1:
        params["message_mode"] = "equivariant"
        params["equivariant_channels"] = ints["equivariant_channels"]
        params["equivariant_l_max"] = ints["equivariant_l_max"]
    if ints.get("zbl_enabled"):
        if ints.get("zbl_flexible"):
            pairs = tensors.get("zbl.pair_parameters")
            _require(pairs is not None, "missing or incorrectly shaped tensor "
                                        "'zbl.pair_parameters'")
            params["zbl"] = {"rc_inner": 0.0, "rc_outer": 0.0, "flexible": True,
                             "parameters": pairs.astype(np.float32).reshape(-1).tolist()}
        else:
            params["zbl"] = [reals["zbl_rc_inner"], reals["zbl_rc_outer"]]
    else:
        params["zbl"] = None
    model = Mobius(params)
    state = model.state_dict()
    new_state = {}
    for name, value in state.items():
        _require(name in tensors, f"missing or incorrectly shaped tensor '{name}'")
        data = torch.as_tensor(tensors[name], dtype=value.dtype)
        _require(data.numel() == value.numel(), f"missing or incorrectly shaped tensor '{name}'")
        new_state[name] = data.reshape(value.shape)
    model.load_state_dict(new_state, strict=True)
    if device is not None:
        model.to(device)
    return model
