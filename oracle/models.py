"""float64 restatement of the NEP4 and Möbius (Local / MP / EQ) energy, force and virial.

Test infrastructure only (see ``oracle/__init__.py``). Forward passes follow the reference
modules cited per function; the backward passes are the analytic adjoints of those forward
passes (the reference obtains them with ``torch.autograd.grad``, ``rune/mobius/model.py:338``),
written out so that each transposed sum is explicit. Parameters are a ``state_dict``-style
mapping of numpy arrays keyed exactly as the reference modules name them.
"""

from __future__ import annotations

import numpy as np
from scipy.special import erf

from . import descriptor as desc
from .descriptor import EdgeList

K_C_SP = 14.399645  # rune/mobius/zbl.py:10
ZBL_A_INV_FACTOR = 2.134563
# float32 buffers in the reference (zbl.py:38-63), hence float32-rounded even in a float64 model
UNIVERSAL_ZBL = np.array([[0.18175, 3.1998], [0.50986, 0.94229], [0.28022, 0.4029],
                          [0.02817, 0.20162]]).astype(np.float32).astype(np.float64)


# --------------------------------------------------------------------------- helpers
def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def act(name, x):
    """Activation and its derivative (rune/mobius/layers.py:11-23)."""
    name = name.lower()
    if name == "tanh":
        t = np.tanh(x)
        return t, 1.0 - t * t
    if name in ("silu", "swish"):
        s = sigmoid(x)
        return x * s, s * (1.0 + x * (1.0 - s))
    if name == "gelu":
        cdf = 0.5 * (1.0 + erf(x / np.sqrt(2.0)))
        return x * cdf, cdf + x * np.exp(-0.5 * x * x) / np.sqrt(2.0 * np.pi)
    raise ValueError(name)


def rmsnorm(h, weight, eps):
    """RMSNorm without centring (rune/mobius/layers.py:26-44); returns y and 1/rms."""
    rho = 1.0 / np.sqrt(np.mean(h * h, -1, keepdims=True) + eps)
    return h * rho * weight, rho


def rmsnorm_back(h, rho, weight, dy):
    gw = dy * weight
    return rho * gw - (rho ** 3 / h.shape[-1]) * h * np.sum(gw * h, -1, keepdims=True)


def segment_sum(values, index, n):
    out = np.zeros((n,) + values.shape[1:])
    np.add.at(out, index, values)
    return out


# --------------------------------------------------------------------------- ZBL
def zbl(config, z_of_type, types, edges: EdgeList):
    """Per-centre ZBL energy and per-edge dE/dr (rune/mobius/zbl.py:92-141)."""
    n = len(types)
    if config is None or len(edges.center) == 0:
        return np.zeros(n), np.zeros((len(edges.center), 3))
    d = np.maximum(edges.dist, 1e-12)
    ti, tj = types[edges.center], types[edges.neighbor]
    zi, zj = z_of_type[ti], z_of_type[tj]
    a_inv = (zi ** 0.23 + zj ** 0.23) * ZBL_A_INV_FACTOR
    pref = K_C_SP * zi * zj
    if config["flexible"]:
        t_count = len(z_of_type)
        lo, hi = np.minimum(ti, tj), np.maximum(ti, tj)
        idx = lo * t_count - lo * (lo - 1) // 2 + hi - lo
        par = np.asarray(config["parameters"], dtype=np.float32).astype(np.float64)
        par = par.reshape(-1, 10)[idx]
        rin, rout = par[:, 0], par[:, 1]
        coef = par[:, 2:].reshape(-1, 4, 2)
    else:
        rin = np.full_like(d, config["rc_inner"])
        rout = np.full_like(d, config["rc_outer"])
        coef = np.broadcast_to(UNIVERSAL_ZBL, (len(d), 4, 2))
    ex = np.exp(-coef[:, :, 1] * (d * a_inv)[:, None])
    phi = np.sum(coef[:, :, 0] * ex, -1)
    dphi = np.sum(-coef[:, :, 0] * coef[:, :, 1] * a_inv[:, None] * ex, -1)
    scr = pref * phi / d
    dscr = pref * (dphi / d - phi / (d * d))
    width = np.maximum(rout - rin, 1e-12)
    arg = np.pi * (d - rin) / width
    cut = np.where(d < rin, 1.0, np.where(d < rout, 0.5 * np.cos(arg) + 0.5, 0.0))
    dcut = np.where((d >= rin) & (d < rout), -0.5 * np.pi / width * np.sin(arg), 0.0)
    energy = segment_sum(0.5 * scr * cut, edges.center, n)
    grad = (0.5 * (dscr * cut + scr * dcut))[:, None] * edges.unit
    return energy, grad


def normalize_zbl(config):
    """Universal ([rc_inner, rc_outer]) or flexible mapping (rune/mobius/zbl.py:68-90)."""
    if config is None:
        return None
    if isinstance(config, dict):
        inner, outer = float(config["rc_inner"]), float(config["rc_outer"])
        flexible = bool(config.get("flexible", inner == 0.0 and outer == 0.0))
        return dict(rc_inner=inner, rc_outer=outer, flexible=flexible,
                    parameters=config.get("parameters"))
    inner, outer = map(float, config)
    return dict(rc_inner=inner, rc_outer=outer, flexible=inner == 0.0 and outer == 0.0,
                parameters=None)


# --------------------------------------------------------------------------- inputs
def edges_from_pairs(positions, cell, pairs, dtype=np.float64):
    """Directed edges from (i, j, S) triples: r = (R_j + S @ cell) - R_i in ``dtype``.

    With ``dtype=np.float32`` the rounding matches the reference ``BatchBuilder``, which casts
    positions and float64 offsets to the model dtype and then forms ``R_j + off - R_i``
    (``rune/mobius/descriptor.py:813-817``).
    """
    pairs = np.asarray(pairs, dtype=np.int64).reshape(-1, 5)
    i, j = pairs[:, 0], pairs[:, 1]
    off = (pairs[:, 2:5].astype(np.float64) @ np.asarray(cell, np.float64)).astype(dtype)
    pos = np.asarray(positions, np.float64).astype(dtype)
    vec = (pos[j] + off) - pos[i]
    return EdgeList(i, j, vec.astype(np.float64))


def descriptor_params(params):
    return dict(rc_r=float(params["rcut_radial"]), rc_a=float(params["rcut_angular"]),
                l_max=int(params["l_max"]),
                flags=tuple(int(params.get(k, 0)) for k in
                            ("has_q_222", "has_q_1111", "has_q_112", "has_q_123",
                             "has_q_233", "has_q_134")))


def _finish(energies, forces, atomic_virial, structure_sizes):
    sid = np.repeat(np.arange(len(structure_sizes)), structure_sizes)
    nb = len(structure_sizes)
    return dict(energies=energies, energy=segment_sum(energies, sid, nb), forces=forces,
                virial=segment_sum(atomic_virial, sid, nb))


# --------------------------------------------------------------------------- NEP4
def nep_forward(params, w, types, radial: EdgeList, angular: EdgeList, structure_sizes,
                z_of_type=None):
    """NEP energy, forces, virial (rune/nep/model.py:87-170, rune/nep/force.py:165-235)."""
    types = np.asarray(types)
    n = len(types)
    p = descriptor_params(params)
    cr = w["descriptor.radial.c_table"]
    ca = w["descriptor.angular.c_table"]
    q, s = desc.descriptor_forward(p, cr, ca, types, n, radial, angular)
    x = q * w["q_scaler"]
    energies = np.zeros(n)
    dx = np.zeros_like(x)
    for t, element in enumerate(params["elements"]):
        m = types == t
        if not m.any():
            continue
        w1 = w[f"element_mlps.{element}.0.weight"]
        b1 = w[f"element_mlps.{element}.0.bias"]
        w2 = w[f"element_mlps.{element}.2.weight"]
        a = x[m] @ w1.T + b1
        z = np.tanh(a)
        energies[m] = (z @ w2.T)[:, 0] - w["shared_bias"][0]
        dx[m] = ((1.0 - z * z) * w2[0]) @ w1
    dq = dx * w["q_scaler"]
    zcfg = normalize_zbl(params.get("zbl"))
    ez, gz = zbl(zcfg, z_of_type, types, angular) if zcfg else (np.zeros(n), None)
    energies = energies + ez
    g_r, g_a = desc.descriptor_edge_gradients(p, cr, ca, types, dq, s, radial, angular)
    f1, v1 = desc.accumulate(n, radial, g_r)
    f2, v2 = desc.accumulate(n, angular, g_a + (gz if gz is not None else 0.0))
    return _finish(energies, f1 + f2, v1 + v2, structure_sizes)


# --------------------------------------------------------------------------- Möbius
class _MobiusParams:
    def __init__(self, params):
        self.H = int(params["hidden_dim"])
        self.blocks = int(params["blocks"])
        self.activation = str(params.get("activation", "silu"))
        self.eps = float(params.get("norm_eps", 1e-8))
        self.layers = int(params.get("message_layers", 0))
        self.mode = params.get("message_mode", "scalar")
        self.G = int(params.get("message_groups", 8))
        self.V = int(params.get("vector_channels", 0))
        self.Km = int(params.get("message_basis_size", params["k_max_radial"]))
        self.rc_m = float(params.get("message_cutoff", params["rcut_radial"]))
        self.Ce = int(params.get("equivariant_channels", 0) or 0)
        self.Le = int(params.get("equivariant_l_max", 0) or 0)
        self.T = len(params["elements"])


def _mp_forward(mp, w, pre, h, types, e: EdgeList):
    n, H = h.shape
    c, j = e.center, e.neighbor
    u, rho_in = rmsnorm(h, w[pre + "input_norm.weight"], mp.eps)
    cache = dict(h=h, u=u, rho_in=rho_in)
    b, db = desc.chebyshev_masked(e.dist, mp.rc_m, mp.Km)
    pair = w[pre + "pair_embedding.weight"][types[c] * mp.T + types[j]]
    ein = np.concatenate([b, pair], 1)
    a_e = ein @ w[pre + "edge_mlp.0.weight"].T + w[pre + "edge_mlp.0.bias"]
    z, dz_da = act(mp.activation, a_e)
    fc, dfc = desc.cutoff_fn(e.dist, mp.rc_m)
    inside = e.dist < mp.rc_m
    cut, dcut = np.where(inside, fc, 0.0), np.where(inside, dfc, 0.0)
    sg = sigmoid(z @ w[pre + "group_gate.weight"].T + w[pre + "group_gate.bias"])
    gate = sg * cut[:, None]
    v = u @ w[pre + "value_projection.weight"].T
    gw = H // mp.G
    ev = (v[j].reshape(-1, mp.G, gw) * gate[:, :, None]).reshape(-1, H)
    msg = segment_sum(ev, c, n)
    cache.update(db=db, z=z, dz_da=dz_da, cut=cut, dcut=dcut, sg=sg, gate=gate, v=v, msg=msg)
    if mp.V:
        sv = sigmoid(z @ w[pre + "vector_gate.weight"].T + w[pre + "vector_gate.bias"])
        vg = sv * cut[:, None]
        src = u @ w[pre + "vector_source.weight"].T
        evec = (vg * src[j])[:, :, None] * e.unit[:, None, :]
        vec = segment_sum(evec, c, n)
        mixed = np.einsum("ba,nax->nbx", w[pre + "vector_mix.weight"], vec)
        t = np.sum(mixed * mixed, -1)
        cache.update(sv=sv, vg=vg, src=src, mixed=mixed)
    else:
        t = np.zeros((n, 0))
    un, rho_m = rmsnorm(msg, w[pre + "message_norm.weight"], mp.eps)
    uin = np.concatenate([un, t], 1)
    au = uin @ w[pre + "update.0.weight"].T + w[pre + "update.0.bias"]
    zu, dzu = act(mp.activation, au)
    h_new = h + zu @ w[pre + "update.2.weight"].T + w[pre + "update.2.bias"]
    cache.update(rho_m=rho_m, dzu=dzu)
    return h_new, cache


def _mp_backward(mp, w, pre, cache, dh_out, types, e: EdgeList):
    """Adjoint of MessageBlock.forward (rune/mobius/message.py:125-193) w.r.t. h and r."""
    h, u = cache["h"], cache["u"]
    n, H = h.shape
    c, j = e.center, e.neighbor
    gw = H // mp.G
    dau = (dh_out @ w[pre + "update.2.weight"]) * cache["dzu"]
    duin = dau @ w[pre + "update.0.weight"]
    dmsg = rmsnorm_back(cache["msg"], cache["rho_m"], w[pre + "message_norm.weight"],
                        duin[:, :H])
    dmi = dmsg[c].reshape(-1, mp.G, gw)
    v = cache["v"]
    dgate = np.sum(dmi * v[j].reshape(-1, mp.G, gw), -1)
    dv = segment_sum((cache["gate"][:, :, None] * dmi).reshape(-1, H), j, n)
    sg = cache["sg"]
    cut = cache["cut"]
    dlg = dgate * cut[:, None] * sg * (1.0 - sg)
    dcut_e = np.sum(dgate * sg, 1)
    dz = dlg @ w[pre + "group_gate.weight"]
    dunit = np.zeros((len(c), 3))
    du = dv @ w[pre + "value_projection.weight"]
    if mp.V:
        dt = duin[:, H:]
        mixed = cache["mixed"]
        dmixed = 2.0 * dt[:, :, None] * mixed
        dvec = np.einsum("ba,nbx->nax", w[pre + "vector_mix.weight"], dmixed)
        dvi = dvec[c]
        proj = np.sum(dvi * e.unit[:, None, :], -1)
        src, vg, sv = cache["src"], cache["vg"], cache["sv"]
        dvg = src[j] * proj
        dsrc = segment_sum(vg * proj, j, n)
        dunit += np.sum((vg * src[j])[:, :, None] * dvi, 1)
        dlv = dvg * cut[:, None] * sv * (1.0 - sv)
        dcut_e += np.sum(dvg * sv, 1)
        dz += dlv @ w[pre + "vector_gate.weight"]
        du += dsrc @ w[pre + "vector_source.weight"]
    dpre = dz * cache["dz_da"]
    dein = dpre @ w[pre + "edge_mlp.0.weight"]
    dd = np.sum(dein[:, :mp.Km] * cache["db"], 1) + dcut_e * cache["dcut"]
    dh = dh_out + rmsnorm_back(h, cache["rho_in"], w[pre + "input_norm.weight"], du)
    return dh, dd, dunit


def _eq_blocks(mp):
    return [slice(l * l - 1, (l + 1) * (l + 1) - 1) for l in range(1, mp.Le + 1)]


def _eq_forward(mp, w, pre, h, D, Yn, types, e: EdgeList):
    """EquivariantBlock.forward (rune/mobius/equivariant.py:124-223)."""
    n, H = h.shape
    c, j = e.center, e.neighbor
    E = len(c)
    Ce, Le = mp.Ce, mp.Le
    blocks = _eq_blocks(mp)
    u, rho_in = rmsnorm(h, w[pre + "input_norm.weight"], mp.eps)
    mixed = np.zeros_like(D)
    pc = np.zeros((E, Le, Ce))
    pn = np.zeros((E, Le, Ce))
    for l, blk in enumerate(blocks, start=1):
        mixed[:, :, blk] = np.einsum("dc,ncm->ndm", w[pre + f"direction_mix.{l - 1}.weight"],
                                     D[:, :, blk])
        pc[:, l - 1] = np.sum(D[c][:, :, blk] * Yn[:, None, blk], -1)
        pn[:, l - 1] = (-1) ** l * np.sum(D[j][:, :, blk] * Yn[:, None, blk], -1)
    b, db = desc.chebyshev_masked(e.dist, mp.rc_m, mp.Km)
    pair = w[pre + "pair_embedding.weight"][types[c] * mp.T + types[j]]
    ctx_c = u @ w[pre + "center_context.weight"].T
    ctx_n = u @ w[pre + "neighbor_context.weight"].T
    ein = np.concatenate([b, pair, ctx_c[c], ctx_n[j], pc.reshape(E, Le * Ce), pn.reshape(E, Le * Ce)],
                         1)
    a_e = ein @ w[pre + "edge_mlp.0.weight"].T + w[pre + "edge_mlp.0.bias"]
    z, dz_da = act(mp.activation, a_e)
    fc, dfc = desc.cutoff_fn(e.dist, mp.rc_m)
    inside = e.dist < mp.rc_m
    cut, dcut = np.where(inside, fc, 0.0), np.where(inside, dfc, 0.0)
    sg = sigmoid(z @ w[pre + "group_gate.weight"].T + w[pre + "group_gate.bias"])
    gate = sg * cut[:, None]
    v = u @ w[pre + "value_projection.weight"].T
    gw = H // mp.G
    msg = segment_sum((v[j].reshape(-1, mp.G, gw) * gate[:, :, None]).reshape(-1, H), c, n)
    ag = np.tanh(z @ w[pre + "direction_gates.weight"].T + w[pre + "direction_gates.bias"])
    ag = ag.reshape(E, 2, Le, Ce)
    Dn = D.copy()
    for l, blk in enumerate(blocks, start=1):
        ed = cut[:, None, None] * (ag[:, 0, l - 1, :, None] * mixed[j][:, :, blk]
                                   + ag[:, 1, l - 1, :, None] * Yn[:, None, blk])
        Dn[:, :, blk] += segment_sum(ed, c, n)
    inv = np.concatenate([np.sum(Dn[:, :, blk] ** 2, -1) for blk in blocks], 1)
    un, rho_m = rmsnorm(msg, w[pre + "message_norm.weight"], mp.eps)
    uin = np.concatenate([un, inv], 1)
    au = uin @ w[pre + "update.0.weight"].T + w[pre + "update.0.bias"]
    zu, dzu = act(mp.activation, au)
    h_new = h + zu @ w[pre + "update.2.weight"].T + w[pre + "update.2.bias"]
    cache = dict(h=h, u=u, rho_in=rho_in, D=D, Dn=Dn, mixed=mixed, db=db, dz_da=dz_da,
                 cut=cut, dcut=dcut, sg=sg, gate=gate, v=v, msg=msg, ag=ag, rho_m=rho_m,
                 dzu=dzu)
    return h_new, Dn, cache


def _eq_backward(mp, w, pre, cache, dh_out, dDn, Yn, types, e: EdgeList):
    """Adjoint of EquivariantBlock.forward w.r.t. h, the direction state and the edges."""
    h = cache["h"]
    n, H = h.shape
    c, j = e.center, e.neighbor
    E = len(c)
    Ce, Le = mp.Ce, mp.Le
    blocks = _eq_blocks(mp)
    gw = H // mp.G
    dau = (dh_out @ w[pre + "update.2.weight"]) * cache["dzu"]
    duin = dau @ w[pre + "update.0.weight"]
    dmsg = rmsnorm_back(cache["msg"], cache["rho_m"], w[pre + "message_norm.weight"],
                        duin[:, :H])
    dinv = duin[:, H:].reshape(n, Le, Ce)
    Dn, D, mixed, ag, cut = cache["Dn"], cache["D"], cache["mixed"], cache["ag"], cache["cut"]
    dDp = dDn.copy()
    for l, blk in enumerate(blocks):
        dDp[:, :, blk] += 2.0 * dinv[:, l, :, None] * Dn[:, :, blk]
    dD = dDp.copy()
    dDpi = dDp[c]
    S1 = np.zeros((E, Le, Ce))
    S2 = np.zeros((E, Le, Ce))
    dmixed = np.zeros_like(D)
    dYn = np.zeros_like(Yn)
    for l, blk in enumerate(blocks):
        S1[:, l] = np.sum(dDpi[:, :, blk] * mixed[j][:, :, blk], -1)
        S2[:, l] = np.sum(dDpi[:, :, blk] * Yn[:, None, blk], -1)
        dmixed[:, :, blk] += segment_sum(
            cut[:, None, None] * ag[:, 0, l, :, None] * dDpi[:, :, blk], j, n)
        dYn[:, blk] += cut[:, None] * np.sum(ag[:, 1, l, :, None] * dDpi[:, :, blk], 1)
    dcut_e = np.sum(ag[:, 0] * S1 + ag[:, 1] * S2, (1, 2))
    dag = np.stack([cut[:, None, None] * S1, cut[:, None, None] * S2], 1)
    dld = (dag * (1.0 - ag * ag)).reshape(E, 2 * mp.Le * mp.Ce)
    dmi = dmsg[c].reshape(-1, mp.G, gw)
    v = cache["v"]
    dgate = np.sum(dmi * v[j].reshape(-1, mp.G, gw), -1)
    dv = segment_sum((cache["gate"][:, :, None] * dmi).reshape(-1, H), j, n)
    sg = cache["sg"]
    dlg = dgate * cut[:, None] * sg * (1.0 - sg)
    dcut_e += np.sum(dgate * sg, 1)
    dz = dlg @ w[pre + "group_gate.weight"] + dld @ w[pre + "direction_gates.weight"]
    dein = (dz * cache["dz_da"]) @ w[pre + "edge_mlp.0.weight"]
    K, P = mp.Km, w[pre + "pair_embedding.weight"].shape[1]
    M = w[pre + "center_context.weight"].shape[0]
    o = K + P
    dctx_c = segment_sum(dein[:, o:o + M], c, n)
    dctx_n = segment_sum(dein[:, o + M:o + 2 * M], j, n)
    o += 2 * M
    dpc = dein[:, o:o + Le * Ce].reshape(E, Le, Ce)
    dpn = dein[:, o + Le * Ce:o + 2 * Le * Ce].reshape(E, Le, Ce)
    for l, blk in enumerate(blocks, start=1):
        sign = (-1) ** l
        dD[:, :, blk] += segment_sum(dpc[:, l - 1, :, None] * Yn[:, None, blk], c, n)
        dD[:, :, blk] += segment_sum(sign * dpn[:, l - 1, :, None] * Yn[:, None, blk], j, n)
        dYn[:, blk] += np.sum(dpc[:, l - 1, :, None] * D[c][:, :, blk]
                              + sign * dpn[:, l - 1, :, None] * D[j][:, :, blk], 1)
        dD[:, :, blk] += np.einsum("dc,ndm->ncm", w[pre + f"direction_mix.{l - 1}.weight"],
                                   dmixed[:, :, blk])
    dd = np.sum(dein[:, :K] * cache["db"], 1) + dcut_e * cache["dcut"]
    du = (dctx_c @ w[pre + "center_context.weight"]
          + dctx_n @ w[pre + "neighbor_context.weight"]
          + dv @ w[pre + "value_projection.weight"])
    dh = dh_out + rmsnorm_back(h, cache["rho_in"], w[pre + "input_norm.weight"], du)
    return dh, dD, dd, dYn


def mobius_forward(params, w, types, radial: EdgeList, angular: EdgeList, structure_sizes,
                   z_of_type=None):
    """Möbius energy, forces, virial (rune/mobius/model.py:256-393)."""
    types = np.asarray(types)
    n = len(types)
    mp = _MobiusParams(params)
    p = descriptor_params(params)
    cr = w["descriptor.radial.c_table"]
    ca = w["descriptor.angular.c_table"]
    q, s = desc.descriptor_forward(p, cr, ca, types, n, radial, angular)
    # encode: input projection, embedding, residual blocks (model.py:267-270)
    x = q * w["q_scaler"]
    h = x @ w["input_projection.weight"].T + w["input_projection.bias"]
    h = h + w["element_embedding.weight"][types]
    res = []
    for b in range(mp.blocks):
        pre = f"residual_blocks.{b}."
        u, rho = rmsnorm(h, w[pre + "norm.weight"], mp.eps)
        a = u @ w[pre + "ffn.0.weight"].T + w[pre + "ffn.0.bias"]
        z, dz = act(mp.activation, a)
        res.append((h, rho, dz))
        h = h + z @ w[pre + "ffn.2.weight"].T + w[pre + "ffn.2.bias"]
    caches = []
    if mp.layers and mp.mode == "equivariant":
        Cl = mp.Le * (mp.Le + 2)
        scale = desc.orthonormal_scale(mp.Le)
        sn = s[:, :, :Cl] * scale
        D = np.zeros((n, mp.Ce, Cl))
        for l, blk in enumerate(_eq_blocks(mp)):
            D[:, :, blk] = np.einsum("dn,inm->idm",
                                     w[f"direction_encoder.projections.{l}.weight"],
                                     sn[:, :, blk])
        y, dy = desc.angular_basis(radial.unit, mp.Le)
        Yn = y[:, :Cl] * scale
        for layer in range(mp.layers):
            h, D, cache = _eq_forward(mp, w, f"message_blocks.{layer}.", h, D, Yn, types,
                                      radial)
            caches.append(cache)
    elif mp.layers:
        for layer in range(mp.layers):
            h, cache = _mp_forward(mp, w, f"message_blocks.{layer}.", h, types, radial)
            caches.append(cache)
    y_out, rho_out = rmsnorm(h, w["output_norm.weight"], mp.eps)
    head_w = w["energy_heads.weight"][types]
    energies = np.sum(y_out * head_w, -1) + w["energy_heads.bias"][types]
    zcfg = normalize_zbl(params.get("zbl"))
    ez, gz = zbl(zcfg, z_of_type, types, radial) if zcfg else (np.zeros(n), None)
    energies = energies + ez

    # ---- analytic backward
    dh = rmsnorm_back(h, rho_out, w["output_norm.weight"], head_w)
    edge_dd = np.zeros(len(radial.center))
    edge_dunit = np.zeros((len(radial.center), 3))
    moment_gradient = None
    if mp.layers and mp.mode == "equivariant":
        dD = np.zeros_like(D)
        dYn = np.zeros_like(Yn)
        for layer in reversed(range(mp.layers)):
            dh, dD, dd, dYl = _eq_backward(mp, w, f"message_blocks.{layer}.", caches[layer],
                                           dh, dD, Yn, types, radial)
            edge_dd += dd
            dYn += dYl
        edge_dunit += np.einsum("em,emx->ex", dYn * scale, dy[:, :Cl])
        dsn = np.zeros_like(sn)
        for l, blk in enumerate(_eq_blocks(mp)):
            dsn[:, :, blk] = np.einsum("dn,idm->inm",
                                       w[f"direction_encoder.projections.{l}.weight"],
                                       dD[:, :, blk])
        moment_gradient = np.zeros_like(s)
        moment_gradient[:, :, :Cl] = dsn * scale
    elif mp.layers:
        for layer in reversed(range(mp.layers)):
            dh, dd, du_e = _mp_backward(mp, w, f"message_blocks.{layer}.", caches[layer], dh,
                                        types, radial)
            edge_dd += dd
            edge_dunit += du_e
    for b in reversed(range(mp.blocks)):
        pre = f"residual_blocks.{b}."
        h_in, rho, dz = res[b]
        da = (dh @ w[pre + "ffn.2.weight"]) * dz
        du = da @ w[pre + "ffn.0.weight"]
        dh = dh + rmsnorm_back(h_in, rho, w[pre + "norm.weight"], du)
    dq = (dh @ w["input_projection.weight"]) * w["q_scaler"]
    g_r, g_a = desc.descriptor_edge_gradients(p, cr, ca, types, dq, s, radial, angular,
                                              moment_gradient)
    proj = np.sum(edge_dunit * radial.unit, 1)
    g_edge = edge_dd[:, None] * radial.unit + (edge_dunit - proj[:, None] * radial.unit) \
        * radial.inv[:, None]
    if gz is not None:
        g_edge = g_edge + gz
    f1, v1 = desc.accumulate(n, radial, g_r + g_edge)
    f2, v2 = desc.accumulate(n, angular, g_a)
    return _finish(energies, f1 + f2, v1 + v2, structure_sizes)
