"""float64 restatement of the NEP / Möbius descriptor and its analytic force contraction.

Test infrastructure only (see ``oracle/__init__.py``). Follows
``rune/mobius/descriptor.py`` (identical mathematics in ``rune/nep/descriptor.py``) and
``rune/mobius/force.py`` (``rune/nep/force.py``).
"""

from __future__ import annotations

import numpy as np

# Coefficient tables of the reference (rune/mobius/descriptor.py:10-139). They are part of the
# model definition (trained weights depend on them), so they are restated value for value.
C3B = np.array([
    0.238732414637843, 0.119366207318922, 0.119366207318922, 0.099471839432435,
    0.596831036594608, 0.596831036594608, 0.149207759148652, 0.149207759148652,
    0.139260575205408, 0.104445431404056, 0.104445431404056, 1.044454314040563,
    1.044454314040563, 0.174075719006761, 0.174075719006761, 0.011190581936149,
    0.223811638722978, 0.223811638722978, 0.111905819361489, 0.111905819361489,
    1.566681471060845, 1.566681471060845, 0.195835183882606, 0.195835183882606,
    0.01367737792196, 0.102580334414698, 0.102580334414698, 2.872249363611549,
    2.872249363611549, 0.119677056817148, 0.119677056817148, 2.154187022708661,
    2.154187022708661, 0.215418702270866, 0.215418702270866, 0.004041043476943,
    0.169723826031592, 0.169723826031592, 0.106077391269745, 0.106077391269745,
    0.424309565078979, 0.424309565078979, 0.127292869523694, 0.127292869523694,
    2.80044312952126, 2.80044312952126, 0.233370260793438, 0.233370260793438,
    0.004662742473395, 0.004079899664221, 0.004079899664221, 0.024479397985326,
    0.024479397985326, 0.012239698992663, 0.012239698992663, 0.538546755677165,
    0.538546755677165, 0.134636688919291, 0.134636688919291, 3.500553911901575,
    3.500553911901575, 0.250039565135827, 0.250039565135827, 8.2569397966e-05,
    0.005944996653579, 0.005944996653579, 0.104037441437634, 0.104037441437634,
    0.762941237209318, 0.762941237209318, 0.114441185581398, 0.114441185581398,
    5.950941650232678, 5.950941650232678, 0.141689086910302, 0.141689086910302,
    4.250672607309055, 4.250672607309055, 0.265667037956816, 0.265667037956816,
])
C4B = np.array([-0.007499480826664, -0.134990654879954, 0.067495327439977,
                0.404971964639861, -0.809943929279723])
C5B = np.array([0.026596810706114, 0.053193621412227, 0.026596810706114])
C4B2 = np.array([0.027493550848847, 0.164961305093080, -0.013746775424423,
                 0.041240326273270, 0.082480652546540])
C4B_123 = np.array([-0.008418146349617, -0.016836292699234, -0.033672585398469,
                    -0.042090731748086, -0.067345170796937, -0.084181463496172,
                    -0.168362926992344])
C4B_233 = np.array([0.008572620635186, 0.009644198214584, 0.019288396429168,
                    0.025717861905558, 0.026789439484956, 0.032147327381947,
                    0.038576792858337, 0.128589309527790, 0.192883964291685,
                    0.321473273819474])
C4B_134 = np.array([0.003645164295772, 0.004860219061029, 0.006075273826286,
                    0.018225821478859, 0.024301095305146, 0.036451642957719,
                    0.042526916784005, 0.072903285915437, 0.085053833568010,
                    0.255161500704030])
# (coefficient index, sign, (a, b, c)) cubic terms, rune/mobius/descriptor.py:141-196
Q123 = [(6, 1, (12, 2, 4)), (6, -1, (11, 2, 5)), (6, 1, (1, 11, 4)), (6, 1, (1, 12, 5)),
        (5, 1, (0, 11, 6)), (5, 1, (0, 12, 7)),
        (3, 1, (14, 2, 6)), (3, -1, (13, 2, 7)), (3, 1, (1, 13, 6)), (3, 1, (1, 14, 7)),
        (4, 1, (10, 0, 5)), (4, 1, (0, 4, 9)),
        (1, 1, (10, 2, 3)), (1, 1, (0, 3, 8)), (1, 1, (1, 3, 9)),
        (0, 1, (10, 2, 6)), (0, -1, (10, 1, 7)), (0, -1, (2, 7, 9)), (0, -1, (1, 6, 9)),
        (2, -1, (2, 5, 8)), (2, -1, (1, 4, 8))]
Q233 = [(0, 1, (3, 8, 8)), (1, 1, (10, 10, 3)), (1, 1, (3, 9, 9)),
        (2, -1, (10, 10, 6)), (2, 1, (6, 9, 9)), (3, 1, (4, 8, 9)), (3, 1, (10, 5, 8)),
        (4, -1, (13, 13, 3)), (4, -1, (14, 14, 3)),
        (5, -1, (14, 7, 9)), (5, -1, (13, 6, 9)), (5, -1, (10, 14, 6)), (5, 1, (10, 13, 7)),
        (6, 1, (10, 7, 9)), (7, -1, (11, 6, 8)), (7, -1, (12, 7, 8)),
        (8, 1, (11, 4, 9)), (8, 1, (12, 5, 9)), (8, 1, (10, 12, 4)), (8, -1, (10, 11, 5)),
        (9, 1, (12, 14, 4)), (9, 1, (11, 14, 5)), (9, 1, (13, 11, 4)), (9, -1, (13, 12, 5))]
Q134 = [(0, -1, (10, 15, 2)), (0, -1, (1, 15, 9)), (1, 1, (0, 15, 8)),
        (2, -1, (1, 13, 18)), (2, -1, (1, 14, 19)), (2, -1, (2, 14, 18)), (2, 1, (2, 13, 19)),
        (3, -1, (10, 18, 2)), (3, 1, (1, 10, 19)), (3, 1, (1, 18, 9)), (3, 1, (2, 19, 9)),
        (4, 1, (1, 16, 8)), (4, 1, (2, 17, 8)),
        (5, 1, (0, 10, 17)), (5, 1, (0, 16, 9)), (5, -1, (1, 11, 16)), (5, -1, (1, 12, 17)),
        (5, -1, (2, 12, 16)), (5, 1, (2, 11, 17)),
        (6, 1, (1, 13, 22)), (6, 1, (1, 14, 23)), (6, -1, (2, 14, 22)), (6, 1, (2, 13, 23)),
        (7, 1, (0, 11, 18)), (7, 1, (0, 12, 19)), (8, 1, (0, 13, 20)), (8, 1, (0, 14, 21)),
        (9, 1, (1, 11, 20)), (9, 1, (1, 12, 21)), (9, -1, (2, 12, 20)), (9, 1, (2, 11, 21))]
# z-polynomial coefficients of the real angular basis (rune/mobius/descriptor.py:197-251)
ZCOEF = {
    1: [[0, 1], [1, 0]],
    2: [[-1, 0, 3], [0, 1, 0], [1, 0, 0]],
    3: [[0, -3, 0, 5], [-1, 0, 5, 0], [0, 1, 0, 0], [1, 0, 0, 0]],
    4: [[3, 0, -30, 0, 35], [0, -3, 0, 7, 0], [-1, 0, 7, 0, 0], [0, 1, 0, 0, 0],
        [1, 0, 0, 0, 0]],
    5: [[0, 15, 0, -70, 0, 63], [1, 0, -14, 0, 21, 0], [0, -1, 0, 3, 0, 0],
        [-1, 0, 9, 0, 0, 0], [0, 1, 0, 0, 0, 0], [1, 0, 0, 0, 0, 0]],
    6: [[-5, 0, 105, 0, -315, 0, 231], [0, 5, 0, -30, 0, 33, 0], [1, 0, -18, 0, 33, 0, 0],
        [0, -3, 0, 11, 0, 0, 0], [-1, 0, 11, 0, 0, 0, 0], [0, 1, 0, 0, 0, 0, 0],
        [1, 0, 0, 0, 0, 0, 0]],
    7: [[0, -35, 0, 315, 0, -693, 0, 429], [-5, 0, 135, 0, -495, 0, 429, 0],
        [0, 15, 0, -110, 0, 143, 0, 0], [3, 0, -66, 0, 143, 0, 0, 0],
        [0, -3, 0, 13, 0, 0, 0, 0], [-1, 0, 13, 0, 0, 0, 0, 0], [0, 1, 0, 0, 0, 0, 0, 0],
        [1, 0, 0, 0, 0, 0, 0, 0]],
    8: [[35, 0, -1260, 0, 6930, 0, -12012, 0, 6435], [0, -35, 0, 385, 0, -1001, 0, 715, 0],
        [-1, 0, 33, 0, -143, 0, 143, 0, 0], [0, 3, 0, -26, 0, 39, 0, 0, 0],
        [1, 0, -26, 0, 65, 0, 0, 0, 0], [0, -1, 0, 5, 0, 0, 0, 0, 0],
        [-1, 0, 15, 0, 0, 0, 0, 0, 0], [0, 1, 0, 0, 0, 0, 0, 0, 0],
        [1, 0, 0, 0, 0, 0, 0, 0, 0]],
}


# The reference registers C3B/C4B/C5B/C4B2 as float32 buffers (descriptor.py:520-523), so a
# float64 model still sees float32-rounded values; the q123/q233/q134 coefficients and the
# orthonormal scale use the full-precision Python floats (descriptor.py:186-196, 626-637).
C3B_BUF = C3B.astype(np.float32).astype(np.float64)
C4B_BUF = C4B.astype(np.float32).astype(np.float64)
C5B_BUF = C5B.astype(np.float32).astype(np.float64)
C4B2_BUF = C4B2.astype(np.float32).astype(np.float64)


def cutoff_fn(d, rc):
    """Cosine cutoff and its derivative, unmasked (descriptor.py:379-382)."""
    arg = np.pi * d / rc
    return 0.5 * np.cos(arg) + 0.5, -0.5 * np.pi / rc * np.sin(arg)


def chebyshev_with_derivative(d, rc, k_max):
    """f_k(d) and df_k/dd (rune/mobius/descriptor.py:377-414)."""
    d = np.asarray(d, dtype=np.float64)
    fc, fcp = cutoff_fn(d, rc)
    rs = d / rc - 1.0
    x = 2.0 * rs * rs - 1.0
    dxdr = 4.0 * rs / rc
    basis = np.zeros(d.shape + (k_max,))
    deriv = np.zeros_like(basis)
    if k_max == 0:
        return basis, deriv
    basis[..., 0] = fc
    deriv[..., 0] = fcp
    if k_max == 1:
        return basis, deriv
    t2, t1 = np.ones_like(d), x
    u2, u1 = np.ones_like(d), 2.0 * x
    core = 0.5 * (x + 1.0)
    basis[..., 1] = core * fc
    deriv[..., 1] = 0.5 * dxdr * fc + core * fcp
    for k in range(2, k_max):
        tn = 2.0 * x * t1 - t2
        un = 2.0 * x * u1 - u2
        core = 0.5 * (tn + 1.0)
        basis[..., k] = core * fc
        deriv[..., k] = 0.5 * k * u1 * dxdr * fc + core * fcp
        t2, t1 = t1, tn
        u2, u1 = u1, un
    return basis, deriv


def chebyshev_masked(d, rc, k_max):
    """Message-edge basis: zero at and beyond the cutoff (descriptor.py:357-374)."""
    b, db = chebyshev_with_derivative(d, rc, k_max)
    inside = (np.asarray(d) < rc)[..., None]
    return np.where(inside, b, 0.0), np.where(inside, db, 0.0)


def angular_basis(unit, l_max):
    """Real polynomial angular basis Y_c and dY_c/d(x,y,z) (descriptor.py:574-624).

    Returns ``basis [E, C]`` and ``grad [E, C, 3]`` with ``C = l_max (l_max + 2)``.
    """
    unit = np.asarray(unit, dtype=np.float64)
    x, y, z = unit[:, 0], unit[:, 1], unit[:, 2]
    e = unit.shape[0]
    count = l_max * (l_max + 2)
    basis = np.zeros((e, count))
    grad = np.zeros((e, count, 3))
    # powers of w = x + i y
    wre = [np.ones(e)]
    wim = [np.zeros(e)]
    for _ in range(l_max):
        wre.append(wre[-1] * x - wim[-1] * y)
        wim.append(wre[-2] * y + wim[-1] * x)
    for order in range(1, l_max + 1):
        idx = order * order - 1
        coef = ZCOEF[order]
        for n1 in range(order + 1):
            zf = np.zeros(e)
            dzf = np.zeros(e)
            start = 0 if (order + n1) % 2 == 0 else 1
            for n2 in range(start, order - n1 + 1, 2):
                zf += coef[n1][n2] * z ** n2
                if n2:
                    dzf += coef[n1][n2] * n2 * z ** (n2 - 1)
            if n1 == 0:
                basis[:, idx] = zf
                grad[:, idx, 2] = dzf
                idx += 1
            else:
                re, im = wre[n1], wim[n1]
                pre, pim = n1 * wre[n1 - 1], n1 * wim[n1 - 1]
                basis[:, idx] = zf * re
                basis[:, idx + 1] = zf * im
                # d(w^n)/dx = n w^(n-1); d(w^n)/dy = i n w^(n-1)
                grad[:, idx, 0] = zf * pre
                grad[:, idx, 1] = -zf * pim
                grad[:, idx, 2] = dzf * re
                grad[:, idx + 1, 0] = zf * pim
                grad[:, idx + 1, 1] = zf * pre
                grad[:, idx + 1, 2] = dzf * im
                idx += 2
    return basis, grad


def num_invariants(l_max, flags):
    return l_max + int(sum(bool(f) for f in flags))


def _cubic(s, terms, coefs):
    out = np.zeros(s.shape[:-1])
    for k, sign, (a, b, c) in terms:
        out = out + sign * coefs[k] * s[..., a] * s[..., b] * s[..., c]
    return out


def invariants(s, l_max, flags):
    """q[..., L] from moments s[..., C] (rune/mobius/descriptor.py:650-733).

    ``flags`` = (q222, q1111, q112, q123, q233, q134).
    """
    q = []
    for order in range(1, l_max + 1):
        start = order * order - 1
        c = C3B_BUF[start:start + 2 * order + 1]
        comp = s[..., start:start + 2 * order + 1]
        q.append(c[0] * comp[..., 0] ** 2 + 2.0 * np.sum(c[1:] * comp[..., 1:] ** 2, -1))
    f222, f1111, f112, f123, f233, f134 = flags
    if f222:
        s3, s4, s5, s6, s7 = (s[..., k] for k in range(3, 8))
        q.append(C4B_BUF[0] * s3 ** 3 + C4B_BUF[1] * s3 * (s4 ** 2 + s5 ** 2)
                 + C4B_BUF[2] * s3 * (s6 ** 2 + s7 ** 2) + C4B_BUF[3] * s6 * (s5 ** 2 - s4 ** 2)
                 + C4B_BUF[4] * s4 * s5 * s7)
    if f1111:
        s0, s1, s2 = s[..., 0], s[..., 1], s[..., 2]
        a, b = s0 * s0, s1 * s1 + s2 * s2
        q.append(C5B_BUF[0] * a * a + C5B_BUF[1] * a * b + C5B_BUF[2] * b * b)
    if f112:
        s10, s11r, s11i, s20, s21r, s21i, s22r, s22i = (s[..., k] for k in range(8))
        q.append(C4B2_BUF[0] * s10 * s10 * s20 + C4B2_BUF[1] * s10 * (s11r * s21r + s11i * s21i)
                 + C4B2_BUF[2] * s20 * (s11r ** 2 + s11i ** 2)
                 + C4B2_BUF[3] * s22r * (s11r ** 2 - s11i ** 2) + C4B2_BUF[4] * s11r * s11i * s22i)
    if f123:
        q.append(_cubic(s, Q123, C4B_123))
    if f233:
        q.append(_cubic(s, Q233, C4B_233))
    if f134:
        q.append(_cubic(s, Q134, C4B_134))
    return np.stack(q, -1)


def invariant_weight(dq_ang, s, l_max, flags):
    """w[..., C] = sum_L dq_ang[..., L] dq_L/ds (rune/mobius/force.py:28-133).

    ``dq_ang`` has shape ``s.shape[:-1] + (num_L,)``. The cubic q123/q233/q134 parts use the
    product rule on the same term lists (force.py:18-25 with descriptor.py:254-277).
    """
    w = np.zeros_like(s)
    col = 0
    for order in range(1, l_max + 1):
        start = order * order - 1
        n = 2 * order + 1
        fac = np.full(n, 4.0)
        fac[0] = 2.0
        w[..., start:start + n] += dq_ang[..., col, None] * fac * C3B_BUF[start:start + n] \
            * s[..., start:start + n]
        col += 1
    f222, f1111, f112, f123, f233, f134 = flags
    s10, s11r, s11i = s[..., 0], s[..., 1], s[..., 2]
    if s.shape[-1] >= 8:
        s20, s21r, s21i, s22r, s22i = (s[..., k] for k in range(3, 8))
    if f222:
        g = dq_ang[..., col]
        col += 1
        c = C4B_BUF
        w[..., 3] += g * (3 * c[0] * s20 ** 2 + c[1] * (s21r ** 2 + s21i ** 2)
                          + c[2] * (s22r ** 2 + s22i ** 2))
        w[..., 4] += g * (2 * c[1] * s20 * s21r - 2 * c[3] * s22r * s21r + c[4] * s21i * s22i)
        w[..., 5] += g * (2 * c[1] * s20 * s21i + 2 * c[3] * s22r * s21i + c[4] * s21r * s22i)
        w[..., 6] += g * (2 * c[2] * s20 * s22r + c[3] * (s21i ** 2 - s21r ** 2))
        w[..., 7] += g * (2 * c[2] * s20 * s22i + c[4] * s21r * s21i)
    if f1111:
        g = dq_ang[..., col]
        col += 1
        c = C5B_BUF
        a, b = s10 ** 2, s11r ** 2 + s11i ** 2
        factor = c[1] * a + 2 * c[2] * b
        w[..., 0] += g * 2 * s10 * (2 * c[0] * a + c[1] * b)
        w[..., 1] += g * 2 * s11r * factor
        w[..., 2] += g * 2 * s11i * factor
    if f112:
        g = dq_ang[..., col]
        col += 1
        c = C4B2_BUF
        a, b, cc, d, e, f, gg, h = s10, s11r, s11i, s20, s21r, s21i, s22r, s22i
        w[..., 0] += g * (2 * c[0] * a * d + c[1] * (b * e + cc * f))
        w[..., 1] += g * (c[1] * a * e + 2 * c[2] * d * b + 2 * c[3] * gg * b + c[4] * cc * h)
        w[..., 2] += g * (c[1] * a * f + 2 * c[2] * d * cc - 2 * c[3] * gg * cc + c[4] * b * h)
        w[..., 3] += g * (c[0] * a * a + c[2] * (b * b + cc * cc))
        w[..., 4] += g * c[1] * a * b
        w[..., 5] += g * c[1] * a * cc
        w[..., 6] += g * c[3] * (b * b - cc * cc)
        w[..., 7] += g * c[4] * b * cc
    for enabled, terms, coefs in ((f123, Q123, C4B_123), (f233, Q233, C4B_233),
                                  (f134, Q134, C4B_134)):
        if not enabled:
            continue
        g = dq_ang[..., col]
        col += 1
        for k, sign, idx in terms:
            coef = sign * coefs[k]
            for pos in range(3):
                rest = [idx[p] for p in range(3) if p != pos]
                w[..., idx[pos]] += g * coef * s[..., rest[0]] * s[..., rest[1]]
    return w


def orthonormal_scale(l_max):
    """sqrt of the descriptor metric (rune/mobius/descriptor.py:626-637)."""
    size = l_max * (l_max + 2)
    metric = C3B[:size] * 2.0
    for order in range(1, l_max + 1):
        metric[order * order - 1] *= 0.5
    return np.sqrt(metric)


class EdgeList:
    """Flat directed edge list: centre i, neighbour j, vector r_ij = R_j + shift - R_i."""

    def __init__(self, center, neighbor, vectors):
        self.center = np.asarray(center, dtype=np.int64)
        self.neighbor = np.asarray(neighbor, dtype=np.int64)
        self.vectors = np.asarray(vectors, dtype=np.float64).reshape(-1, 3)
        self.dist = np.linalg.norm(self.vectors, axis=1)
        self.inv = 1.0 / np.maximum(self.dist, 1e-12)
        self.unit = self.vectors * self.inv[:, None]


def descriptor_forward(p, c_radial, c_angular, types, n_atoms, radial: EdgeList,
                       angular: EdgeList):
    """q [N, D] and moments s [N, na, C] (rune/mobius/descriptor.py:822-911).

    ``p`` holds ``rc_r, rc_a, l_max, flags``; c tables are [T, T, n, K].
    """
    nr, kr = c_radial.shape[2:]
    na, ka = c_angular.shape[2:]
    cnt = p["l_max"] * (p["l_max"] + 2)
    fr, _ = chebyshev_with_derivative(radial.dist, p["rc_r"], kr)
    cr = c_radial[types[radial.center], types[radial.neighbor]]
    q_r = np.zeros((n_atoms, nr))
    np.add.at(q_r, radial.center, np.einsum("enk,ek->en", cr, fr))
    fa, _ = chebyshev_with_derivative(angular.dist, p["rc_a"], ka)
    ca = c_angular[types[angular.center], types[angular.neighbor]]
    gn = np.einsum("enk,ek->en", ca, fa)
    y, _ = angular_basis(angular.unit, p["l_max"])
    s = np.zeros((n_atoms, na, cnt))
    np.add.at(s, angular.center, gn[:, :, None] * y[:, None, :])
    q_a = invariants(s, p["l_max"], p["flags"])  # [N, na, L]
    q = np.concatenate([q_r, q_a.transpose(0, 2, 1).reshape(n_atoms, -1)], 1)
    return q, s


def descriptor_edge_gradients(p, c_radial, c_angular, types, dq, s, radial: EdgeList,
                              angular: EdgeList, moment_gradient=None):
    """dE/dr_e for every radial and angular edge (rune/mobius/force.py:165-243)."""
    nr, kr = c_radial.shape[2:]
    na, ka = c_angular.shape[2:]
    n_atoms = dq.shape[0]
    _, fpr = chebyshev_with_derivative(radial.dist, p["rc_r"], kr)
    cr = c_radial[types[radial.center], types[radial.neighbor]]
    rad = np.einsum("en,enk,ek->e", dq[radial.center, :nr], cr, fpr)
    g_radial = (rad * radial.inv)[:, None] * radial.vectors

    n_l = num_invariants(p["l_max"], p["flags"])
    dq_ang = dq[:, nr:].reshape(n_atoms, n_l, na).transpose(0, 2, 1)
    w = invariant_weight(dq_ang, s, p["l_max"], p["flags"])
    if moment_gradient is not None:
        w = w + moment_gradient
    fa, fpa = chebyshev_with_derivative(angular.dist, p["rc_a"], ka)
    ca = c_angular[types[angular.center], types[angular.neighbor]]
    gn = np.einsum("enk,ek->en", ca, fa)
    gnp = np.einsum("enk,ek->en", ca, fpa)
    y, dy = angular_basis(angular.unit, p["l_max"])
    we = w[angular.center]  # [E, na, C]
    radial_scalar = np.einsum("enc,en,ec->e", we, gnp, y)
    wr = np.einsum("enc,en->ec", we, gn)
    dir_vec = np.einsum("ec,ecx->ex", wr, dy)
    proj = np.einsum("ex,ex->e", dir_vec, angular.unit)
    g_angular = (radial_scalar[:, None] * angular.unit
                 + (dir_vec - proj[:, None] * angular.unit) * angular.inv[:, None])
    return g_radial, g_angular


def accumulate(n_atoms, edges: EdgeList, gradient):
    """Forces and atomic virial from per-edge dE/dr (rune/mobius/model.py:23-44)."""
    forces = np.zeros((n_atoms, 3))
    virial = np.zeros((n_atoms, 9))
    np.add.at(forces, edges.center, gradient)
    np.add.at(forces, edges.neighbor, -gradient)
    pv = -(gradient[:, :, None] * edges.vectors[:, None, :]).reshape(-1, 9)
    np.add.at(virial, edges.neighbor, pv)
    return forces, virial
