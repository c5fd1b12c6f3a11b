"""Möbius model container (parameter layout and initialisation order of
rune/mobius/model.py:78-254, layers.py, message.py, equivariant.py); forward on the engine."""

from __future__ import annotations

import torch
import torch.nn as nn

from .._modules import Descriptor, EngineModel, ZBLRepulsion
from ..elements import atomic_numbers

_ACTIVATIONS = {"tanh": nn.Tanh, "silu": nn.SiLU, "swish": nn.SiLU, "gelu": nn.GELU}


def activation_factory(name: str):
    """rune/mobius/layers.py:11-23."""
    key = str(name).strip().lower()
    if key not in _ACTIVATIONS:
        choices = ", ".join(sorted(_ACTIVATIONS))
        raise ValueError(f"Unsupported Mobius activation {name!r}; choose one of {choices}.")
    return _ACTIVATIONS[key]


class RMSNorm(nn.Module):
    def __init__(self, dimension: int, eps: float = 1.0e-8):
        super().__init__()
        if dimension <= 0:
            raise ValueError("RMSNorm dimension must be positive.")
        self.dimension = int(dimension)
        self.eps = float(eps)
        self.weight = nn.Parameter(torch.ones(self.dimension))


class ResidualBlock(nn.Module):
    def __init__(self, hidden_dim, ffn_dim, activation, norm_eps=1.0e-8):
        super().__init__()
        self.norm = RMSNorm(hidden_dim, eps=norm_eps)
        self.ffn = nn.Sequential(nn.Linear(hidden_dim, ffn_dim), activation_factory(activation)(),
                                 nn.Linear(ffn_dim, hidden_dim))


class ElementwiseLinearHead(nn.Module):
    def __init__(self, n_elements: int, hidden_dim: int):
        super().__init__()
        if n_elements <= 0:
            raise ValueError("ElementwiseLinearHead requires at least one element.")
        self.weight = nn.Parameter(torch.empty(n_elements, hidden_dim))
        self.bias = nn.Parameter(torch.zeros(n_elements))
        nn.init.xavier_uniform_(self.weight)


class MessageBlock(nn.Module):
    """rune/mobius/message.py:12-98 (parameters only)."""

    def __init__(self, *, hidden_dim, message_dim, pair_dim, message_groups, vector_channels,
                 n_elements, basis_size, cutoff, activation, norm_eps=1.0e-8):
        super().__init__()
        if message_groups <= 0:
            raise ValueError("message_groups must be positive.")
        if hidden_dim % message_groups != 0:
            raise ValueError(f"hidden_dim ({hidden_dim}) must be divisible by "
                             f"message_groups ({message_groups}).")
        if vector_channels < 0:
            raise ValueError("vector_channels cannot be negative.")
        if basis_size <= 0:
            raise ValueError("message basis_size must be positive.")
        if cutoff <= 0.0:
            raise ValueError("message cutoff must be positive.")
        self.vector_channels = int(vector_channels)
        make = activation_factory(activation)
        self.input_norm = RMSNorm(hidden_dim, eps=norm_eps)
        self.pair_embedding = nn.Embedding(n_elements * n_elements, pair_dim)
        self.edge_mlp = nn.Sequential(nn.Linear(basis_size + pair_dim, message_dim), make())
        self.group_gate = nn.Linear(message_dim, message_groups)
        self.value_projection = nn.Linear(hidden_dim, hidden_dim, bias=False)
        if self.vector_channels:
            self.vector_gate = nn.Linear(message_dim, vector_channels)
            self.vector_source = nn.Linear(hidden_dim, vector_channels, bias=False)
            self.vector_mix = nn.Linear(vector_channels, vector_channels, bias=False)
        else:
            self.vector_gate = self.vector_source = self.vector_mix = None
        self.message_norm = RMSNorm(hidden_dim, eps=norm_eps)
        self.update = nn.Sequential(nn.Linear(hidden_dim + vector_channels, message_dim), make(),
                                    nn.Linear(message_dim, hidden_dim))


class DirectionEncoder(nn.Module):
    """rune/mobius/equivariant.py:12-39 (parameters only)."""

    def __init__(self, n_desc, channels, l_max):
        super().__init__()
        if n_desc <= 0 or channels <= 0 or l_max <= 0:
            raise ValueError("DirectionEncoder dimensions must be positive.")
        self.projections = nn.ModuleList(nn.Linear(n_desc, channels, bias=False)
                                         for _ in range(l_max))


class EquivariantBlock(nn.Module):
    """rune/mobius/equivariant.py:42-122 (parameters only)."""

    def __init__(self, *, hidden_dim, message_dim, pair_dim, message_groups,
                 equivariant_channels, l_max, n_elements, basis_size, cutoff, activation,
                 norm_eps=1.0e-8):
        super().__init__()
        if hidden_dim <= 0 or message_dim <= 0 or pair_dim <= 0:
            raise ValueError("Equivariant block dimensions must be positive.")
        if message_groups <= 0 or hidden_dim % message_groups != 0:
            raise ValueError("message_groups must be positive and divide hidden_dim.")
        if equivariant_channels <= 0 or l_max <= 0:
            raise ValueError("Angular channels and l_max must be positive.")
        if n_elements <= 0 or basis_size <= 0 or cutoff <= 0.0:
            raise ValueError("Elements, radial basis size and cutoff must be positive.")
        make = activation_factory(activation)
        angular_width = l_max * equivariant_channels
        self.input_norm = RMSNorm(hidden_dim, eps=norm_eps)
        self.center_context = nn.Linear(hidden_dim, message_dim, bias=False)
        self.neighbor_context = nn.Linear(hidden_dim, message_dim, bias=False)
        self.pair_embedding = nn.Embedding(n_elements * n_elements, pair_dim)
        edge_input_dim = basis_size + pair_dim + 2 * message_dim + 2 * angular_width
        self.edge_mlp = nn.Sequential(nn.Linear(edge_input_dim, message_dim), make())
        self.group_gate = nn.Linear(message_dim, message_groups)
        self.direction_gates = nn.Linear(message_dim, 2 * angular_width)
        self.value_projection = nn.Linear(hidden_dim, hidden_dim, bias=False)
        self.direction_mix = nn.ModuleList(
            nn.Linear(equivariant_channels, equivariant_channels, bias=False)
            for _ in range(l_max))
        self.message_norm = RMSNorm(hidden_dim, eps=norm_eps)
        self.update = nn.Sequential(nn.Linear(hidden_dim + angular_width, message_dim), make(),
                                    nn.Linear(message_dim, hidden_dim))


class Mobius(EngineModel):
    """Möbius potential; outputs follow the RUNE model contract (rune/mobius/model.py:47-74)."""

    model_family = "mobius"
    family = "mobius"

    def __init__(self, params: dict):
        super().__init__()
        self.params = dict(params)
        self.elements = list(self.params["elements"])
        if not self.elements:
            raise ValueError("Mobius requires a non-empty elements list.")
        if len(set(self.elements)) != len(self.elements):
            raise ValueError("Mobius elements must not contain duplicates.")
        invalid = [e for e in self.elements if e not in atomic_numbers]
        if invalid:
            raise ValueError(f"Unknown chemical element symbols: {invalid}.")
        self.n_elements = len(self.elements)
        if int(self.params.get("n_types", self.n_elements)) != self.n_elements:
            raise ValueError("params['n_types'] must match the number of entries in "
                             "params['elements'].")
        self.params["n_types"] = self.n_elements
        p = self.params
        self.hidden_dim = int(p.get("hidden_dim", 96))
        self.blocks = int(p.get("blocks", 3))
        self.ffn_dim = int(p.get("ffn_dim", 2 * self.hidden_dim))
        self.activation = str(p.get("activation", "silu"))
        self.message_layers = int(p.get("message_layers", 2))
        self.message_mode = p.get("message_mode", "scalar")
        if self.message_mode not in ("scalar", "equivariant"):
            raise ValueError("message_mode must be 'scalar' or 'equivariant'.")
        self.equivariant_channels = int(p.get("equivariant_channels", 8))
        self.equivariant_l_max = p.get("equivariant_l_max")
        if self.equivariant_l_max is None:
            self.equivariant_l_max = int(p["l_max"])
        if self.message_mode == "equivariant":
            if self.message_layers < 1 or self.equivariant_channels < 1:
                raise ValueError("Equivariant messages require positive layers and channels.")
            if not 1 <= self.equivariant_l_max <= min(int(p["l_max"]), 8):
                raise ValueError("equivariant_l_max must be in 1..min(l_max, 8).")
            p.update(message_mode=self.message_mode,
                     equivariant_channels=self.equivariant_channels,
                     equivariant_l_max=self.equivariant_l_max)
        self.message_dim = int(p.get("message_dim", self.hidden_dim))
        self.pair_dim = int(p.get("pair_dim", 16))
        self.message_groups = int(p.get("message_groups", 8))
        self.vector_channels = int(p.get("vector_channels", 8))
        self.norm_eps = float(p.get("norm_eps", 1.0e-8))
        if min(self.hidden_dim, self.ffn_dim, self.message_dim, self.pair_dim) <= 0:
            raise ValueError("Mobius hidden, FFN, message, and pair dimensions must be positive.")
        if self.blocks < 0 or self.message_layers < 0:
            raise ValueError("Mobius blocks and message_layers cannot be negative.")
        if self.message_layers and self.hidden_dim % self.message_groups != 0:
            raise ValueError("hidden_dim must be divisible by message_groups.")
        p.update({"model": "mobius", "hidden_dim": self.hidden_dim, "blocks": self.blocks,
                  "ffn_dim": self.ffn_dim, "activation": self.activation,
                  "message_layers": self.message_layers, "message_dim": self.message_dim,
                  "pair_dim": self.pair_dim, "message_groups": self.message_groups,
                  "vector_channels": self.vector_channels, "norm_eps": self.norm_eps})
        self.descriptor = Descriptor(p)
        self.n_desc_radial = int(p["n_desc_radial"])
        self.n_desc_angular = int(p["n_desc_angular"])
        self.num_L = int(self.descriptor.angular.num_L)
        self.input_dim = self.n_desc_radial + self.n_desc_angular * self.num_L
        scaler = p.get("descriptor_scaler")
        if scaler is None:
            scaler_tensor = torch.ones(self.input_dim, dtype=torch.float32)
        else:
            scaler_tensor = torch.as_tensor(scaler, dtype=torch.float32).reshape(-1)
            if scaler_tensor.numel() != self.input_dim:
                raise ValueError(f"descriptor_scaler has {scaler_tensor.numel()} values; "
                                 f"Mobius expects {self.input_dim}.")
        self.register_buffer("q_scaler", scaler_tensor.clone())
        p["descriptor_scaler"] = scaler_tensor.tolist()
        self.input_projection = nn.Linear(self.input_dim, self.hidden_dim)
        self.element_embedding = nn.Embedding(self.n_elements, self.hidden_dim)
        self.residual_blocks = nn.ModuleList(
            ResidualBlock(self.hidden_dim, self.ffn_dim, self.activation, norm_eps=self.norm_eps)
            for _ in range(self.blocks))
        output_norm = RMSNorm(self.hidden_dim, eps=self.norm_eps)
        energy_heads = ElementwiseLinearHead(self.n_elements, self.hidden_dim)
        basis = int(p.get("message_basis_size", p["k_max_radial"]))
        cutoff = float(p.get("message_cutoff", p["rcut_radial"]))
        if cutoff > float(p["rcut_radial"]):
            raise ValueError("message_cutoff cannot exceed rcut_radial because Mobius uses "
                             "the radial neighbor list for message edges.")
        p["message_basis_size"] = basis
        p["message_cutoff"] = cutoff
        mparams = dict(hidden_dim=self.hidden_dim, message_dim=self.message_dim,
                       pair_dim=self.pair_dim, message_groups=self.message_groups,
                       n_elements=self.n_elements, basis_size=basis, cutoff=cutoff,
                       activation=self.activation, norm_eps=self.norm_eps)
        if self.message_mode == "equivariant":
            self.direction_encoder = DirectionEncoder(self.n_desc_angular,
                                                      self.equivariant_channels,
                                                      self.equivariant_l_max)
            self.message_blocks = nn.ModuleList(
                EquivariantBlock(**mparams, equivariant_channels=self.equivariant_channels,
                                 l_max=self.equivariant_l_max)
                for _ in range(self.message_layers))
        else:
            self.message_blocks = nn.ModuleList(
                MessageBlock(**mparams, vector_channels=self.vector_channels)
                for _ in range(self.message_layers))
        self.output_norm = output_norm
        self.energy_heads = energy_heads
        self.zbl = ZBLRepulsion(self.elements, p["zbl"]) if p.get("zbl") is not None else None
        if self.zbl is not None and self.zbl.max_rc_outer > float(p["rcut_radial"]):
            raise ValueError("ZBL rc_outer cannot exceed rcut_radial because Mobius "
                             "evaluates ZBL on the radial neighbor list.")

    def set_descriptor_scaler(self, scaler) -> torch.Tensor:
        """rune/mobius/model.py:467-479."""
        scaler = torch.as_tensor(scaler, device=self.q_scaler.device,
                                 dtype=self.q_scaler.dtype).reshape(-1)
        if scaler.numel() != self.input_dim:
            raise ValueError(f"Descriptor scaler must contain {self.input_dim} values.")
        if not torch.isfinite(scaler).all():
            raise ValueError("Descriptor scaler must contain only finite values.")
        with torch.no_grad():
            self.q_scaler.copy_(scaler)
        self.params["descriptor_scaler"] = scaler.detach().cpu().tolist()
        return self.q_scaler.detach().cpu().clone()
