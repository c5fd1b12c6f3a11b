"""NEP4 model container (parameter layout of rune/nep/model.py:48-85); forward on the engine."""

from __future__ import annotations

import re

import numpy as np
import torch
import torch.nn as nn

from .._modules import Descriptor, EngineModel, ZBLRepulsion


class NEP(EngineModel):
    family = "nep"

    def __init__(self, params):
        super().__init__()
        self.params = dict(params)
        self.descriptor = Descriptor(self.params)
        self.n_desc_radial = self.params["n_desc_radial"]
        self.n_desc_angular = self.params["n_desc_angular"]
        self.L_max = self.params["l_max"]
        self.num_L = self.descriptor.angular.num_L
        self.elements = list(self.params["elements"])
        self.n_elements = len(self.elements)
        input_dim = self.n_desc_radial + self.n_desc_angular * self.num_L
        self.input_dim = input_dim
        hidden_dims = list(self.params["hidden_dims"])
        if len(hidden_dims) != 1:
            raise ValueError("rune_b200 evaluates single-hidden-layer NEP models.")
        self.element_mlps = nn.ModuleDict()
        for element in self.elements:
            self.element_mlps[element] = nn.Sequential(
                nn.Linear(input_dim, hidden_dims[0]), nn.Tanh(),
                nn.Linear(hidden_dims[-1], 1, bias=False))
        self.register_buffer("q_scaler", torch.ones(input_dim, dtype=torch.float32))
        self._configure_zbl()
        self.shared_bias = nn.Parameter(torch.zeros(1))

    @classmethod
    def from_nep_txt(cls, filepath, device=None):
        """A GPUMD ``nep.txt`` NEP4 model (rune/nep/model.py:284-489): header, optional zbl line,
        cutoffs, n_max, basis_size, l_max, ANN, then per element W0 (neurons x dim, row
        major), b0 (stored with the opposite sign), w1; the shared bias; the radial and angular
        c-tables in (n, k, t1, t2) order; q_scaler; flexible ZBL parameters to the end."""
        with open(filepath, "r") as handle:
            lines = [line.strip() for line in handle if line.strip() != ""]
        pos = 0

        def next_line():
            nonlocal pos
            tokens = lines[pos].split()
            pos += 1
            return tokens

        tokens = next_line()
        match = re.fullmatch(r"nep(\d+)(?:_(.*))?", tokens[0].lower())
        if match is None:
            raise ValueError("Invalid nep.txt: first line should start with nep4 or nep5.")
        if int(match.group(1)) != 4:
            raise NotImplementedError("Only nep4 is supported by the RUNE loader.")
        has_zbl = "zbl" in (match.group(2) or "").split("_")
        num_types = int(tokens[1])
        elements = tokens[2:]
        if len(elements) != num_types:
            raise ValueError("Invalid nep.txt: element count mismatch.")
        zbl = None
        if has_zbl:
            tokens = next_line()
            if tokens[0] != "zbl" or len(tokens) not in (3, 4):
                raise ValueError("Invalid nep.txt: zbl line not found after nep4_zbl header.")
            inner, outer = float(tokens[1]), float(tokens[2])
            zbl = {"rc_inner": inner, "rc_outer": outer,
                   "flexible": inner == 0.0 and outer == 0.0}
            if len(tokens) == 4:
                raise NotImplementedError("Typewise ZBL cutoffs are not supported in RUNE.")
        tokens = next_line()
        if tokens[0] != "cutoff":
            raise ValueError("Invalid nep.txt: cutoff line not found.")
        if len(tokens) == 5:
            rcut_radial, rcut_angular = float(tokens[1]), float(tokens[2])
        else:
            if len(tokens) != 2 * num_types + 3:
                raise ValueError("Invalid nep.txt: cutoff line length mismatch.")
            radial = {float(tokens[1 + 2 * t]) for t in range(num_types)}
            angular = {float(tokens[2 + 2 * t]) for t in range(num_types)}
            if len(radial) != 1 or len(angular) != 1:
                raise NotImplementedError("Per-type cutoffs are not supported in RUNE.")
            rcut_radial, rcut_angular = radial.pop(), angular.pop()
        max_radial, max_angular = int(tokens[-2]), int(tokens[-1])
        header = {}
        for key in ("n_max", "basis_size"):
            tokens = next_line()
            if tokens[0] != key:
                raise ValueError(f"Invalid nep.txt: {key} line not found.")
            header[key] = (int(tokens[1]), int(tokens[2]))
        tokens = next_line()
        if tokens[0] != "l_max":
            raise ValueError("Invalid nep.txt: l_max line not found.")
        lmax = [int(v) for v in tokens[1:]]
        if not 1 <= len(lmax) <= 7:
            raise ValueError("Invalid nep.txt: l_max should contain 1 to 7 values.")
        lmax += [1, 0, 0, 0, 0, 0][len(lmax) - 1:]
        l_max, q222, q1111, q112, q123, q233, q134 = lmax
        tokens = next_line()
        if tokens[0] != "ANN" or len(tokens) != 3:
            raise ValueError("Invalid nep.txt: expected ANN width 0.")
        neurons = int(tokens[1])
        if not 1 <= neurons <= 200:
            raise ValueError("Invalid nep.txt: ANN width must be in [1, 200].")
        if int(tokens[2]) != 0:
            raise ValueError(
                "RUNE only supports single-hidden-layer NEP text models (ANN width 0).")
        nr, na = header["n_max"][0] + 1, header["n_max"][1] + 1
        kr, ka = header["basis_size"][0] + 1, header["basis_size"][1] + 1
        params = {
            "elements": elements, "rcut_radial": rcut_radial, "rcut_angular": rcut_angular,
            "n_desc_radial": nr, "n_desc_angular": na, "k_max_radial": kr, "k_max_angular": ka,
            "l_max": l_max, "l_max_4body": 2 if q222 > 0 else 0,
            "l_max_5body": 1 if q1111 > 0 else 0,
            "has_q_222": int(q222 > 0), "has_q_1111": int(q1111 > 0), "has_q_112": int(q112 > 0),
            "has_q_123": int(q123 > 0), "has_q_233": int(q233 > 0), "has_q_134": int(q134 > 0),
            "max_neighbors_radial": max_radial, "max_neighbors_angular": max_angular,
            "hidden_dims": [neurons], "n_types": num_types,
        }
        if zbl is not None and not zbl["flexible"]:
            params["zbl"] = zbl
        model = cls(params)
        dim = nr + na * model.num_L
        values = np.array([float(t) for line in lines[pos:] for t in line.split()], np.float64)
        off = 0

        def take(count):
            nonlocal off
            if off + count > len(values):
                raise ValueError("Invalid nep.txt: the parameter section is too short.")
            chunk = values[off:off + count]
            off += count
            return torch.as_tensor(chunk, dtype=torch.float32)

        with torch.no_grad():
            for element in elements:
                w0 = take(neurons * dim).reshape(neurons, dim)
                b0 = take(neurons)
                w1 = take(neurons)
                mlp = model.element_mlps[element]
                mlp[0].weight.copy_(w0)
                mlp[0].bias.copy_(-b0)
                mlp[-1].weight.copy_(w1.view(1, -1))
            model.shared_bias.copy_(take(1))
            for table, nn_, kk in ((model.descriptor.radial.c_table, nr, kr),
                                   (model.descriptor.angular.c_table, na, ka)):
                flat = take(nn_ * kk * num_types * num_types).reshape(nn_, kk, num_types,
                                                                      num_types)
                table.copy_(flat.permute(2, 3, 0, 1))
            model.q_scaler.copy_(take(dim))
            if zbl is not None and zbl["flexible"]:
                zbl["parameters"] = values[off:].astype(np.float32).tolist()
                model.params["zbl"] = zbl
                model._configure_zbl()
        if device is not None:
            model.to(device)
        return model

    def save_nep_txt(self, filepath):
        """Write the model as a GPUMD nep.txt (rune/nep/model.py:491-579): the header, the zbl
        line, cutoffs, n_max, basis_size, the l_max line without trailing zero flags beyond the
        third value, ``ANN <neurons> 0``, per element W0, -b0 and w1, the shared bias, the
        radial and angular c-tables in (n, k, t1, t2) order, q_scaler and, for flexible ZBL, its
        pair parameters; one value per line as ``%18.10e``."""
        p = self.params
        if len(p["hidden_dims"]) != 1:
            raise ValueError("RUNE nep.txt export requires exactly one NEP hidden layer.")
        if p["max_neighbors_radial"] > 819:
            raise ValueError("GPUMD nep.txt export requires max_neighbors_radial <= 819.")
        angular = self.descriptor.angular
        zbl = self.zbl
        lines = [f"{'nep4_zbl' if zbl is not None else 'nep4'} {len(self.elements)} "
                 + " ".join(self.elements)]
        if zbl is not None:
            lines.append(f"zbl {zbl.rc_inner} {zbl.rc_outer}")
        lines.append(f"cutoff {p['rcut_radial']} {p['rcut_angular']} "
                     f"{p['max_neighbors_radial']} {p['max_neighbors_angular']}")
        lines.append(f"n_max {int(p['n_desc_radial']) - 1} {int(p['n_desc_angular']) - 1}")
        lines.append(f"basis_size {int(p['k_max_radial']) - 1} {int(p['k_max_angular']) - 1}")
        flags = [int(self.L_max), 2 if angular.has_q_222 else 0, angular.has_q_1111,
                 angular.has_q_112, angular.has_q_123, angular.has_q_233, angular.has_q_134]
        while len(flags) > 3 and flags[-1] == 0:
            flags.pop()
        lines.append("l_max " + " ".join(str(v) for v in flags))
        lines.append(f"ANN {int(p['hidden_dims'][0])} 0")
        values = []
        for element in self.elements:
            mlp = self.element_mlps[element]
            values += mlp[0].weight.detach().cpu().reshape(-1).tolist()
            values += (-mlp[0].bias.detach().cpu()).reshape(-1).tolist()
            values += mlp[-1].weight.detach().cpu().reshape(-1).tolist()
        values.append(self.shared_bias.detach().cpu().reshape(-1)[0].item())
        for table in (self.descriptor.radial.c_table, angular.c_table):
            values += table.detach().cpu().permute(2, 3, 0, 1).reshape(-1).tolist()
        values += self.q_scaler.detach().cpu().reshape(-1).tolist()
        if zbl is not None and zbl.flexible:
            values += zbl.pair_parameters.detach().cpu().reshape(-1).tolist()
        lines += [f"{v:18.10e}" for v in values]
        with open(filepath, "w") as handle:
            handle.write("\n".join(lines) + "\n")

    def _configure_zbl(self):
        zbl = self.params.get("zbl")
        self.zbl = ZBLRepulsion(self.elements, zbl, max_pairs=55) if zbl is not None else None
        if self.zbl is not None and not self.zbl.max_rc_outer <= self.params["rcut_angular"]:
            raise ValueError(
                "ZBL rc_outer cannot exceed rcut_angular because NEP evaluates ZBL on the "
                "angular neighbor list.")
