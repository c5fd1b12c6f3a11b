"""Constant tables of the NEP / Möbius angular descriptor and the invariant term table.

The numeric tables are part of the model definition (trained weights depend on them) and are
restated from the reference ``rune/mobius/descriptor.py`` (identical in
``rune/nep/descriptor.py``):

* ``C3B`` / ``C4B`` / ``C5B`` / ``C4B2`` (descriptor.py:10-106) and the z-polynomial
  coefficients ``Z1``..``Z8`` (:197-251) are registered as float32 buffers by the model modules,
  exactly as the reference registers them (:520-526), so checkpoints round-trip.
* The cubic invariants q123 / q233 / q134 (:107-196) are restated as
  (coefficient index, sign, moment indices) lists.

``invariant_terms`` flattens every invariant into monomials ``coef * prod s[idx]`` — the single
table the CUDA kernels evaluate (and differentiate by the product rule).
"""

from __future__ import annotations

import numpy as np

C3B_VALUES = [
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
]
C4B_VALUES = [-0.007499480826664, -0.134990654879954, 0.067495327439977, 0.404971964639861,
              -0.809943929279723]
C5B_VALUES = [0.026596810706114, 0.053193621412227, 0.026596810706114]
C4B2_VALUES = [0.027493550848847, 0.164961305093080, -0.013746775424423, 0.041240326273270,
               0.082480652546540]
C4B_123_VALUES = [-0.008418146349617, -0.016836292699234, -0.033672585398469,
                  -0.042090731748086, -0.067345170796937, -0.084181463496172,
                  -0.168362926992344]
C4B_233_VALUES = [0.008572620635186, 0.009644198214584, 0.019288396429168, 0.025717861905558,
                  0.026789439484956, 0.032147327381947, 0.038576792858337, 0.128589309527790,
                  0.192883964291685, 0.321473273819474]
C4B_134_VALUES = [0.003645164295772, 0.004860219061029, 0.006075273826286, 0.018225821478859,
                  0.024301095305146, 0.036451642957719, 0.042526916784005, 0.072903285915437,
                  0.085053833568010, 0.255161500704030]

# (coefficient index, sign, moment indices)
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


def legendre_z_coefficients(order: int) -> list[list[float]]:
    """Z_L[m][p]: coefficients of the z-polynomial of the order-L, |m| basis component.

    Row m is d^m P_L / dz^m (P_L the Legendre polynomial) scaled to the primitive integer
    polynomial with positive leading coefficient; with (x + i y)^m this spans the reference's
    real polynomial basis (descriptor.py:197-251 lists the same integers).
    """
    from fractions import Fraction
    from math import comb, gcd

    # P_L(z) = 2^-L sum_k (-1)^k C(L,k) C(2L-2k, L) z^(L-2k)
    poly = [Fraction(0)] * (order + 1)
    for k in range(order // 2 + 1):
        poly[order - 2 * k] += Fraction((-1) ** k * comb(order, k) * comb(2 * order - 2 * k, order),
                                        2 ** order)
    rows = []
    cur = poly
    for m in range(order + 1):
        nums = [c for c in cur if c != 0]
        lead = [c for c in cur if c != 0][-1]
        scale = Fraction(1)
        dens = 1
        for c in nums:
            dens = dens * c.denominator // gcd(dens, c.denominator)
        ints = [int(c * dens) for c in cur]
        g = 0
        for v in ints:
            g = gcd(g, abs(v))
        ints = [v // g for v in ints]
        if lead < 0:
            ints = [-v for v in ints]
        del scale
        rows.append([float(v) for v in ints] + [0.0] * (order + 1 - len(ints)))
        cur = [cur[p + 1] * (p + 1) for p in range(len(cur) - 1)] + [Fraction(0)]
    return rows


def z_tables() -> dict[int, np.ndarray]:
    return {order: np.array(legendre_z_coefficients(order), dtype=np.float32)
            for order in range(1, 9)}


def invariant_terms(l_max, flags, c3b, c4b, c5b, c4b2) -> np.ndarray:
    """Monomial table [n_terms, 6] = (coef, output L, i0, i1, i2, i3 or -1).

    ``flags`` = (q222, q1111, q112, q123, q233, q134); output L counts the enabled invariants in
    the reference order (descriptor.py:650-723). ``c3b``.. are the model's float32 buffers.
    """
    c3b = np.asarray(c3b, np.float32)
    c4b = np.asarray(c4b, np.float32)
    c5b = np.asarray(c5b, np.float32)
    c4b2 = np.asarray(c4b2, np.float32)
    rows = []

    def add(coef, out, *idx):
        idx = list(idx) + [-1] * (4 - len(idx))
        rows.append([float(np.float32(coef)), out] + idx)

    out = 0
    for order in range(1, l_max + 1):
        start = order * order - 1
        add(c3b[start], out, start, start)
        for m in range(1, 2 * order + 1):
            add(np.float32(2.0) * c3b[start + m], out, start + m, start + m)
        out += 1
    f222, f1111, f112, f123, f233, f134 = (int(bool(f)) for f in flags)
    if f222:
        add(c4b[0], out, 3, 3, 3)
        add(c4b[1], out, 3, 4, 4)
        add(c4b[1], out, 3, 5, 5)
        add(c4b[2], out, 3, 6, 6)
        add(c4b[2], out, 3, 7, 7)
        add(c4b[3], out, 6, 5, 5)
        add(-c4b[3], out, 6, 4, 4)
        add(c4b[4], out, 4, 5, 7)
        out += 1
    if f1111:
        add(c5b[0], out, 0, 0, 0, 0)
        add(c5b[1], out, 0, 0, 1, 1)
        add(c5b[1], out, 0, 0, 2, 2)
        add(c5b[2], out, 1, 1, 1, 1)
        add(np.float32(2.0) * c5b[2], out, 1, 1, 2, 2)
        add(c5b[2], out, 2, 2, 2, 2)
        out += 1
    if f112:
        add(c4b2[0], out, 0, 0, 3)
        add(c4b2[1], out, 0, 1, 4)
        add(c4b2[1], out, 0, 2, 5)
        add(c4b2[2], out, 3, 1, 1)
        add(c4b2[2], out, 3, 2, 2)
        add(c4b2[3], out, 6, 1, 1)
        add(-c4b2[3], out, 6, 2, 2)
        add(c4b2[4], out, 1, 2, 7)
        out += 1
    for enabled, terms, coefs in ((f123, Q123, C4B_123_VALUES), (f233, Q233, C4B_233_VALUES),
                                  (f134, Q134, C4B_134_VALUES)):
        if not enabled:
            continue
        for k, sign, idx in terms:
            add(sign * coefs[k], out, *idx)
        out += 1
    return np.array(rows, dtype=np.float32).reshape(-1, 6)


def orthonormal_scale(l_max: int) -> np.ndarray:
    """sqrt of the descriptor metric diag(C3B * (1 if m = 0 else 2)) (descriptor.py:626-637)."""
    size = l_max * (l_max + 2)
    metric = np.array(C3B_VALUES[:size], dtype=np.float64) * 2.0
    for order in range(1, l_max + 1):
        metric[order * order - 1] *= 0.5
    return np.sqrt(metric)
