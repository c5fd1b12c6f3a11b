"""Writer of the ``mobius1`` text format, the model file of the native GPUMD Möbius evaluator.

The file layout is the reference's (rune/mobius/export.py:79-146): a header line with the
elements, ``schema 1``, integer metadata, real metadata (17 significant digits), every
state_dict tensor promoted to float64 in state_dict order, then the descriptor's sparse
polynomial tables (harmonic basis monomials, invariant monomials, their offsets) and the
orthonormal metric of the direction states. Values are written with 17 significant digits, so
a float32 model round-trips exactly through ``rune_b200.mobius.native.load_mobius1``.
"""

from __future__ import annotations

import math
from math import comb
from pathlib import Path

import numpy as np
import torch

from .. import tables

_ACTIVATION_CODES = {"tanh": 0, "silu": 1, "swish": 1, "gelu": 2}
_INT_NAMES = ("n_desc_radial", "n_desc_angular", "k_max_radial", "k_max_angular", "l_max",
              "hidden_dim", "blocks", "ffn_dim", "message_layers", "message_dim", "pair_dim",
              "message_groups", "vector_channels", "message_basis_size",
              "max_neighbors_radial", "max_neighbors_angular")


def _xy_terms(power: int, imaginary: bool):
    """Monomials x^a y^b of Re or Im (x + i y)^power: (coefficient, a, b) by ascending b."""
    out = []
    for b in range(power + 1):
        if (b % 2 == 1) != imaginary:
            continue
        quarter = (b - 1) // 2 if imaginary else b // 2
        out.append(((-1.0 if quarter % 2 else 1.0) * comb(power, b), power - b, b))
    return out


def basis_terms(angular):
    """Sparse real harmonic basis (rune/mobius/export.py:20-36): rows (component, coefficient,
    x power, y power, z power) and the row offset of every component. Components run over
    orders 1..L_max, then |m| = 0..L, the real part before the imaginary one."""
    rows, offsets = [], [0]
    component = 0
    for order in range(1, int(angular.L_max) + 1):
        z = getattr(angular, f"Z{order}").detach().cpu().double().numpy()
        for m in range(order + 1):
            for imaginary in ((False,) if m == 0 else (False, True)):
                for coef, xp, yp in _xy_terms(m, imaginary):
                    for zp in range((order + m) % 2, order - m + 1, 2):
                        value = coef * float(z[m, zp])
                        if value:
                            rows.append([component, value, xp, yp, zp])
                component += 1
                offsets.append(len(rows))
    return (torch.tensor(rows, dtype=torch.float64),
            torch.tensor(offsets, dtype=torch.float64))


def invariant_terms(angular):
    """Sparse invariant polynomials (rune/mobius/export.py:39-76): rows (output, coefficient,
    degree, four moment indices padded with -1) per enabled invariant in the descriptor's
    order, coefficients in float64 from the model's float32 coefficient buffers."""
    channels = []
    c3 = angular.C3B.detach().cpu().double().tolist()
    for order in range(1, int(angular.L_max) + 1):
        start, stop = order * order - 1, (order + 1) ** 2 - 1
        channels.append([(c3[k] * (1 if k == start else 2), (k, k)) for k in range(start, stop)])
    if angular.has_q_222:
        c = angular.C4B.detach().cpu().double().tolist()
        channels.append([(c[0], (3, 3, 3)), (c[1], (3, 4, 4)), (c[1], (3, 5, 5)),
                         (c[2], (3, 6, 6)), (c[2], (3, 7, 7)), (c[3], (6, 5, 5)),
                         (-c[3], (6, 4, 4)), (c[4], (4, 5, 7))])
    if angular.has_q_1111:
        c = angular.C5B.detach().cpu().double().tolist()
        channels.append([(c[0], (0, 0, 0, 0)), (c[1], (0, 0, 1, 1)), (c[1], (0, 0, 2, 2)),
                         (c[2], (1, 1, 1, 1)), (2 * c[2], (1, 1, 2, 2)), (c[2], (2, 2, 2, 2))])
    if angular.has_q_112:
        c = angular.C4B2.detach().cpu().double().tolist()
        channels.append([(c[0], (0, 0, 3)), (c[1], (0, 1, 4)), (c[1], (0, 2, 5)),
                         (c[2], (3, 1, 1)), (c[2], (3, 2, 2)), (c[3], (6, 1, 1)),
                         (-c[3], (6, 2, 2)), (c[4], (1, 2, 7))])
    for enabled, terms, coefs in ((angular.has_q_123, tables.Q123, tables.C4B_123_VALUES),
                                  (angular.has_q_233, tables.Q233, tables.C4B_233_VALUES),
                                  (angular.has_q_134, tables.Q134, tables.C4B_134_VALUES)):
        if enabled:
            channels.append([(sign * coefs[k], idx) for k, sign, idx in terms])
    rows, offsets = [], [0]
    for output, terms in enumerate(channels):
        for coef, idx in terms:
            rows.append([output, coef, len(idx), *idx, *([-1] * (4 - len(idx)))])
        offsets.append(len(rows))
    return (torch.tensor(rows, dtype=torch.float64),
            torch.tensor(offsets, dtype=torch.float64))


def export_data(model):
    """(ints, reals, tensors) of the mobius1 schema; the model is not modified."""
    state = model.state_dict()
    if any(v.dtype not in (torch.float32, torch.float64) for v in state.values()):
        raise ValueError("Native Möbius export requires float32 or float64 weights and buffers.")
    p = model.params
    ints = {name: int(p[name]) for name in _INT_NAMES}
    zbl = model.zbl
    ints.update(n_types=model.n_elements, num_L=model.num_L, input_dim=model.input_dim,
                message_mode=int(model.message_mode == "equivariant"),
                equivariant_channels=model.equivariant_channels,
                equivariant_l_max=model.equivariant_l_max,
                activation=_ACTIVATION_CODES[model.activation.strip().lower()],
                zbl_enabled=int(zbl is not None),
                zbl_flexible=int(zbl is not None and zbl.flexible))
    reals = {name: float(p[name]) for name in ("rcut_radial", "rcut_angular", "message_cutoff",
                                                "norm_eps")}
    reals.update(zbl_rc_inner=zbl.rc_inner if zbl else 0.0,
                 zbl_rc_outer=zbl.rc_outer if zbl else 0.0)
    if not all(math.isfinite(v) for v in reals.values()):
        raise ValueError("Cannot export nonfinite Möbius configuration values.")
    tensors = {name: v.detach().cpu().double().contiguous() for name, v in state.items()}
    angular = model.descriptor.angular
    tensors["desc.basis_terms"], tensors["desc.basis_offsets"] = basis_terms(angular)
    tensors["desc.invariant_terms"], tensors["desc.invariant_offsets"] = invariant_terms(angular)
    tensors["desc.orthonormal_scale"] = torch.as_tensor(
        tables.orthonormal_scale(int(angular.L_max)), dtype=torch.float64)
    if not all(bool(torch.isfinite(v).all()) for v in tensors.values()):
        raise ValueError("Cannot export a Möbius model containing nonfinite values.")
    return ints, reals, tensors


def export_path(path) -> Path:
    """Output name of ``export_model``: a trainer's ``model`` becomes ``mobius.txt`` and
    ``model_epoch_<k>`` becomes ``mobius_epoch_<k>.txt`` (rune/mobius/export.py:123-127)."""
    path = Path(path)
    if path.name == "model":
        return path.with_name("mobius.txt")
    if path.name.startswith("model_epoch_"):
        return path.with_name(path.name.replace("model_", "mobius_", 1) + ".txt")
    return path


def export_model(model, path) -> Path:
    """Write `model` as a mobius1 file and return the path written."""
    path = export_path(path)
    ints, reals, tensors = export_data(model)
    lines = [f"mobius1 {model.n_elements} {' '.join(model.elements)}", "schema 1",
             f"ints {len(ints)}"]
    lines += [f"{name} {value}" for name, value in ints.items()]
    lines.append(f"reals {len(reals)}")
    lines += [f"{name} {value:.17g}" for name, value in reals.items()]
    lines.append(f"tensors {len(tensors)}")
    for name, value in tensors.items():
        lines.append(f"{name} {value.ndim} {' '.join(str(s) for s in value.shape)}".rstrip()
                     if value.ndim else f"{name} 0 ")
        flat = np.asarray(value.reshape(-1).numpy(), np.float64).tolist()
        for start in range(0, len(flat), 8):
            lines.append(" ".join(format(x, ".17g") for x in flat[start:start + 8]))
    lines.append("END")
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("w", encoding="utf-8", newline="\n") as handle:
        handle.write("\n".join(lines) + "\n")
    return path
