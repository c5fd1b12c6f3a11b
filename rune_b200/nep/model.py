"""NEP4 model container (parameter layout of rune/nep/model.py:48-85); forward on the engine."""

from __future__ import annotations

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

    def _configure_zbl(self):
        zbl = self.params.get("zbl")
        self.zbl = ZBLRepulsion(self.elements, zbl, max_pairs=55) if zbl is not None else None
        if self.zbl is not None and not self.zbl.max_rc_outer <= self.params["rcut_angular"]:
            raise ValueError(
                "ZBL rc_outer cannot exceed rcut_angular because NEP evaluates ZBL on the "
                "angular neighbor list.")
