"""O(N) numpy cell-list neighbour builder — TEST INFRASTRUCTURE ONLY.

Produces the same pair set as the reference builders: ASE ``neighbor_list("ijS")`` at
``max(rc)`` filtered by ``|r|^2 < rc^2`` (``rune/mobius/interface/batch.py:42-102``) and the
training builder ``rune/datasets/neighbor.py:36-134``. Pairs are returned as integer
``(i, j, S0, S1, S2)`` rows sorted by (i, j, S), with ``r_ij = R_j + S @ cell - R_i``.
"""

from __future__ import annotations

import itertools

import numpy as np


def _thickness(cell):
    a, b, c = cell
    volume = abs(np.dot(a, np.cross(b, c)))
    areas = np.array([np.linalg.norm(np.cross(b, c)), np.linalg.norm(np.cross(c, a)),
                      np.linalg.norm(np.cross(a, b))])
    if volume < 1e-12 or np.any(areas < 1e-12):
        raise ValueError("Degenerate cell is not supported for neighbour construction.")
    return volume / areas


def neighbor_pairs(positions, cell, pbc, cutoffs):
    """Return one (i, j, S) array per cutoff in ``cutoffs``."""
    pos = np.asarray(positions, dtype=np.float64).reshape(-1, 3)
    cell = np.asarray(cell, dtype=np.float64).reshape(3, 3)
    pbc = np.asarray(pbc, dtype=bool).reshape(3)
    n = len(pos)
    rc = float(max(cutoffs))
    empty = [np.zeros((0, 5), np.int64) for _ in cutoffs]
    if n == 0:
        return empty
    if not pbc.any() and np.abs(np.linalg.det(cell)) < 1e-12:
        cell = np.eye(3)
    h = _thickness(cell)
    frac = pos @ np.linalg.inv(cell)
    wrap = np.where(pbc, np.floor(frac), 0.0).astype(np.int64)
    fw = frac - wrap
    lo = np.where(pbc, 0.0, fw.min(0))
    span = np.where(pbc, 1.0, np.maximum(fw.max(0) - lo, 1e-9) * (1 + 1e-12) + 1e-12)
    nb = np.maximum(1, np.floor(h * span / rc)).astype(np.int64)
    width = span / nb
    reach = np.ceil(rc / (h * width)).astype(np.int64)
    b = np.minimum(np.floor((fw - lo) / width).astype(np.int64), nb - 1)
    key = (b[:, 0] * nb[1] + b[:, 1]) * nb[2] + b[:, 2]
    order = np.argsort(key, kind="stable")
    counts = np.bincount(key, minlength=int(np.prod(nb)))
    starts = np.concatenate([[0], np.cumsum(counts)[:-1]])
    out_i, out_j, out_s = [], [], []
    ranges = [range(-reach[a], reach[a] + 1) for a in range(3)]
    for off in itertools.product(*ranges):
        t = b + np.array(off)
        img = np.where(pbc, np.floor_divide(t, nb), 0)
        tw = np.where(pbc, t - img * nb, t)
        valid = np.all((tw >= 0) & (tw < nb), 1)
        ii = np.nonzero(valid)[0]
        if ii.size == 0:
            continue
        tk = (tw[ii, 0] * nb[1] + tw[ii, 1]) * nb[2] + tw[ii, 2]
        cnt = counts[tk]
        ci = np.repeat(ii, cnt)
        first = np.repeat(starts[tk], cnt)
        local = np.arange(cnt.sum()) - np.repeat(np.cumsum(cnt) - cnt, cnt)
        cj = order[first + local]
        shift = np.repeat(img[ii], cnt, 0) - wrap[cj] + wrap[ci]
        d = (pos[cj] - pos[ci]) + shift @ cell
        keep = np.einsum("ij,ij->i", d, d) < rc * rc
        keep &= ~((ci == cj) & np.all(shift == 0, 1))
        out_i.append(ci[keep])
        out_j.append(cj[keep])
        out_s.append(shift[keep])
    if not out_i:
        return empty
    i = np.concatenate(out_i)
    j = np.concatenate(out_j)
    s = np.concatenate(out_s)
    d = (pos[j] - pos[i]) + s @ cell
    d2 = np.einsum("ij,ij->i", d, d)
    res = []
    for cutoff in cutoffs:
        m = d2 < float(cutoff) ** 2
        rows = np.concatenate([i[m, None], j[m, None], s[m]], 1)
        k = np.lexsort((rows[:, 4], rows[:, 3], rows[:, 2], rows[:, 1], rows[:, 0]))
        res.append(rows[k])
    return res
