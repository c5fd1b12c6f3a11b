// Periodic cell-list neighbour build on the device.
//
// Pair-set contract: every (i, j, S) with |R_j + S.cell - R_i| < max(rc_radial, rc_angular),
// excluding (i, i, 0) — the ASE neighbor_list("ijS") semantics used by the reference
// BatchBuilder (rune/mobius/interface/batch.py:42-102) and the training builder
// (rune/datasets/neighbor.py:36-134). Membership is decided in float64 from the caller's
// positions; the stored edge vector is then formed in float32 exactly as the reference model
// does (positions and S.cell cast to float32, r = (R_j + off) - R_i; descriptor.py:813-817).
//
// Layout: one fixed-stride row per centre atom (row i starts at i * stride). A row holds the
// edges inside the larger cutoff only ("long"), followed by the edges inside the smaller
// cutoff ("short"); the list with the larger cutoff is the whole row and the other one its
// suffix, so the radial and angular lists share one array. The stride comes from the previous
// call (or a density estimate); a row that does not fit sets an overflow flag, and the call
// is repeated with the stride raised to the largest count.
//
// Binning: per structure, bins along each axis = floor(thickness / rc) (>= 1); the stencil
// reaches ceil(rc / bin thickness) bins, on periodic axes wrapping with an integer image shift,
// so cells thinner than the cutoff produce every periodic image (the small-box case of
// rune/mobius/src/mobius.cu:170-201). A non-periodic axis has no images; atoms outside the
// cell along it fall into its first or last bin.
// Bin contents are sorted by atom index, so the edge order is deterministic.

#include <cub/cub.cuh>

#include "engine.cuh"

namespace rune {

namespace {

__device__ __forceinline__ int floordiv(int a, int b) {
    int q = a / b;
    if ((a % b != 0) && ((a < 0) != (b < 0))) --q;
    return q;
}

// Bin every atom; record its structure, integer wrap (floor of the fractional coordinate on
// periodic axes, so that shifts refer to the caller's unwrapped positions) and bin.
__global__ void k_bin_atoms(int n_atoms, int n_types, int n_structures,
                            const int* __restrict__ atom_ptr, const double* __restrict__ pos,
                            const int* __restrict__ types, const StructGeom* __restrict__ geom,
                            int* __restrict__ tsafe, int* __restrict__ sid_out, int4* __restrict__ binc,
                            int4* __restrict__ wrap, int* __restrict__ bin_count,
                            unsigned int* __restrict__ flags) {
    int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= n_atoms) return;
    int lo = 0, hi = n_structures - 1;
    while (lo < hi) {  // last structure whose first atom <= a
        int mid = (lo + hi + 1) >> 1;
        if (atom_ptr[mid] <= a) lo = mid; else hi = mid - 1;
    }
    sid_out[a] = lo;
    const StructGeom& g = geom[lo];
    double p[3] = {pos[3 * a], pos[3 * a + 1], pos[3 * a + 2]};
    int t = types[a];
    if (t < 0 || t >= n_types) {
        atomicOr(flags, 1u);
        t = 0;  // keep every table read in bounds; the call reports the error at its end
    }
    tsafe[a] = t;
    int b[3], w[3];
    bool finite = isfinite(p[0]) && isfinite(p[1]) && isfinite(p[2]);
    if (!finite) atomicOr(flags, 2u);
    for (int k = 0; k < 3; ++k) {
        double f = p[0] * g.inv[0 * 3 + k] + p[1] * g.inv[1 * 3 + k] + p[2] * g.inv[2 * 3 + k];
        if (!finite) f = 0.0;
        if (g.pbc[k]) {
            double fl = floor(f);
            if (fabs(fl) > 1.0e5) { atomicOr(flags, 2u); fl = 0.0; }
            w[k] = (int)fl;
            double fw = f - fl;
            int bk = (int)(fw * g.nb[k]);
            b[k] = min(max(bk, 0), g.nb[k] - 1);
        } else {
            // non-periodic: bins over the cell's extent, atoms outside it clamped into the
            // edge bins (clamping keeps neighbours within the stencil reach)
            w[k] = 0;
            double fc = fmin(fmax(f, -1.0), 2.0);
            b[k] = min(max((int)floor(fc * g.nb[k]), 0), g.nb[k] - 1);
        }
    }
    int bin = g.bin_offset + (b[0] * g.nb[1] + b[1]) * g.nb[2] + b[2];
    binc[a] = make_int4(b[0], b[1], b[2], bin);
    wrap[a] = make_int4(w[0], w[1], w[2], 0);
    atomicAdd(&bin_count[bin], 1);
}

__global__ void k_fill_bins(int n_atoms, const int4* __restrict__ binc,
                            const int* __restrict__ bin_start, int* __restrict__ bin_fill,
                            int* __restrict__ bin_atoms) {
    int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= n_atoms) return;
    int bin = binc[a].w;
    int slot = atomicAdd(&bin_fill[bin], 1);
    bin_atoms[bin_start[bin] + slot] = a;
}

// Candidate record in bin order: float64 position and the packed integer wrap.
__device__ __forceinline__ double pack_wrap(int4 w) {
    unsigned long long u = ((unsigned long long)(w.x & 0x1fffff)) |
                           ((unsigned long long)(w.y & 0x1fffff) << 21) |
                           ((unsigned long long)(w.z & 0x1fffff) << 42);
    return __longlong_as_double((long long)u);
}
__device__ __forceinline__ int3 unpack_wrap(double d) {
    unsigned long long u = (unsigned long long)__double_as_longlong(d);
    auto ext = [](unsigned long long v) { int x = (int)(v & 0x1fffff); return x >= (1 << 20) ? x - (1 << 21) : x; };
    return make_int3(ext(u), ext(u >> 21), ext(u >> 42));
}

// Wrapped float64 position P = R - w.cell of atom a: pair vectors are formed as
// (P_j - P_i) + I.cell with I the integer image of the bin stencil, exactly antisymmetric
// under i <-> j, I -> -I, so the two directions of a pair always agree on membership.
__device__ __forceinline__ double3 wrapped(const double* __restrict__ pos, int a, int4 w,
                                           const StructGeom& g) {
    return make_double3(pos[3 * a] - (w.x * g.cell[0] + w.y * g.cell[3] + w.z * g.cell[6]),
                        pos[3 * a + 1] - (w.x * g.cell[1] + w.y * g.cell[4] + w.z * g.cell[7]),
                        pos[3 * a + 2] - (w.x * g.cell[2] + w.y * g.cell[5] + w.z * g.cell[8]));
}

// Sort each bin's atom list ascending (rank sort; atom indices are unique), warp per bin, and
// write the bin-ordered candidate arrays (atom index; wrapped position and wrap).
__global__ void k_sort_bins(int n_bins, const int* __restrict__ bin_start,
                            const int* __restrict__ bin_count, const int* __restrict__ unsorted,
                            const double* __restrict__ pos, const int4* __restrict__ wrap,
                            const int* __restrict__ sid, const StructGeom* __restrict__ geom,
                            int* __restrict__ batom, double4* __restrict__ bpos) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (warp >= n_bins) return;
    int start = bin_start[warp], n = bin_count[warp];
    for (int base = 0; base < n; base += 32) {
        int k = base + lane;
        int v = k < n ? unsorted[start + k] : 0;
        int rank = 0;
        for (int m = 0; m < n; ++m) rank += unsorted[start + m] < v;
        if (k < n) {
            int4 w = wrap[v];
            double3 P = wrapped(pos, v, w, geom[sid[v]]);
            batom[start + rank] = v;
            bpos[start + rank] = make_double4(P.x, P.y, P.z, pack_wrap(w));
        }
    }
}

struct Traverse {
    const StructGeom* geom;
    const int* sid;
    const int* bin_start;
    const int* bin_count;
    const int* batom;
    const double4* bpos;  // wrapped float64 position, packed wrap in .w
    double rc_max2, rc_min2;
};

constexpr int kBuildWarps = 4;

// Neighbour rows of the atoms of one bin, warp per bin, lane per atom (bins with more than 32
// atoms are processed 32 at a time). The stencil of a bin is common to its atoms: its bins are
// visited in a fixed order (x, y, then the z range of one image, whose bins are consecutive),
// each range's candidates staged in shared memory by the warp and tested by every lane against
// its own atom. Pair vectors are (P_j - (P_i - I.cell)), I the integer image of the range:
// exactly antisymmetric under i <-> j, I -> -I, so both directions agree on membership.
//
// Row layout: long edges (inside the larger cutoff only) from the front of the atom's row,
// short ones from the back in reverse order; afterwards a partial in-place reversal puts the
// short block, in traversal order, right behind the long one. Rows that do not fit set flag 16
// and are left empty (the call is repeated with a larger stride). Per warp, the largest counts
// of both lists (packed count << 32 | ~atom, so the first atom wins) and their sums go to
// `summary`.
__global__ void __launch_bounds__(kBuildWarps * 32)
k_nbr_build(int n_bins, Traverse tv, int stride, bool radial_is_full,
            float4* __restrict__ edges, int* __restrict__ shifts, int* __restrict__ rp_full,
            int* __restrict__ cnt_full, int* __restrict__ rp_short, int* __restrict__ cnt_short,
            unsigned long long* __restrict__ summary, unsigned int* __restrict__ flags) {
    __shared__ int s_j[kBuildWarps][32];
    __shared__ double4 s_p[kBuildWarps][32];
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int b = blockIdx.x * kBuildWarps + warp;
    if (b >= n_bins) return;
    int start = tv.bin_start[b], count = tv.bin_count[b];
    if (count == 0) return;
    const StructGeom& g = tv.geom[tv.sid[tv.batom[start]]];
    int local = b - g.bin_offset;
    int bz = local % g.nb[2], by = (local / g.nb[2]) % g.nb[1], bx = local / (g.nb[2] * g.nb[1]);
    unsigned long long m_r = 0, m_a = 0, s_r = 0, s_a = 0;
    for (int chunk = 0; chunk < count; chunk += 32) {
        int k = start + chunk + lane;
        bool active = chunk + lane < count;
        int i = active ? tv.batom[k] : 0;
        double4 pi = active ? tv.bpos[k] : make_double4(0, 0, 0, 0);
        int3 wi = unpack_wrap(pi.w);
        long long base = (long long)i * stride;
        int nl = 0, ns = 0;
        for (int dx = -g.reach[0]; dx <= g.reach[0]; ++dx) {
            int tx = bx + dx, ix = 0;
            if (g.pbc[0]) { ix = floordiv(tx, g.nb[0]); tx -= ix * g.nb[0]; }
            else if (tx < 0 || tx >= g.nb[0]) continue;
            for (int dy = -g.reach[1]; dy <= g.reach[1]; ++dy) {
                int ty = by + dy, iy = 0;
                if (g.pbc[1]) { iy = floordiv(ty, g.nb[1]); ty -= iy * g.nb[1]; }
                else if (ty < 0 || ty >= g.nb[1]) continue;
                int column = g.bin_offset + (tx * g.nb[1] + ty) * g.nb[2];
                int z = bz - g.reach[2], zend = bz + g.reach[2];
                while (z <= zend) {
                    int iz = 0, tz0, seg_end;
                    if (g.pbc[2]) {
                        iz = floordiv(z, g.nb[2]);
                        tz0 = z - iz * g.nb[2];
                        seg_end = min(zend, (iz + 1) * g.nb[2] - 1);
                    } else {
                        tz0 = z;
                        seg_end = zend;
                        if (z < 0) { z = 0; continue; }
                        if (z >= g.nb[2]) break;
                        seg_end = min(seg_end, g.nb[2] - 1);
                    }
                    int tz1 = tz0 + (seg_end - z);
                    int a0 = tv.bin_start[column + tz0], a1 = tv.bin_start[column + tz1 + 1];
                    double o0 = pi.x - (ix * g.cell[0] + iy * g.cell[3] + iz * g.cell[6]);
                    double o1 = pi.y - (ix * g.cell[1] + iy * g.cell[4] + iz * g.cell[7]);
                    double o2 = pi.z - (ix * g.cell[2] + iy * g.cell[5] + iz * g.cell[8]);
                    bool home = ix == 0 && iy == 0 && iz == 0;
                    for (int c0 = a0; c0 < a1; c0 += 32) {
                        __syncwarp();
                        if (c0 + lane < a1) {
                            s_j[warp][lane] = tv.batom[c0 + lane];
                            s_p[warp][lane] = tv.bpos[c0 + lane];
                        }
                        __syncwarp();
                        int nv = min(32, a1 - c0);
                        // distances of four candidates at a time (independent float64
                        // chains), then the members among them in order
                        for (int t0 = 0; t0 < nv; t0 += 4) {
                            double r2v[4];
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                double4 pj = s_p[warp][min(t0 + u, nv - 1)];
                                double d0 = pj.x - o0, d1 = pj.y - o1, d2 = pj.z - o2;
                                r2v[u] = d0 * d0 + d1 * d1 + d2 * d2;
                            }
#pragma unroll
                            for (int u = 0; u < 4; ++u) {
                                int t = t0 + u;
                                if (t >= nv) break;
                                int j = s_j[warp][t];
                                double r2 = r2v[u];
                                if (!active || !(r2 < tv.rc_max2) || (home && j == i)) continue;
                                bool is_short = r2 < tv.rc_min2;
                                int slot = is_short ? stride - 1 - ns : nl;
                                if (is_short) ++ns; else ++nl;
                                if (slot < 0 || slot >= stride || nl + ns > stride) continue;
                                double4 pj = s_p[warp][t];
                                double d0 = pj.x - o0, d1 = pj.y - o1, d2 = pj.z - o2;
                                int3 wj = unpack_wrap(pj.w);
                                int s0 = ix - wj.x + wi.x, s1 = iy - wj.y + wi.y;
                                int s2 = iz - wj.z + wi.z;
                                // the float64 pair vector rounded once to float32: its error is
                                // relative to |r|, not to the magnitude of the positions
                                edges[base + slot] = make_float4((float)d0, (float)d1, (float)d2,
                                                                 __int_as_float(j));
                                shifts[base + slot] =
                                    (s0 & 1023) | ((s1 & 1023) << 10) | ((s2 & 1023) << 20);
                            }
                        }
                    }
                    z = seg_end + 1;
                }
            }
        }
        if (active) {
            bool fits = nl + ns <= stride;
            if (!fits) atomicOr(flags, 16u);
            if (fits) {
                // reverse [nl, stride) as far as the short block needs: pair t swaps nl + t and
                // stride - 1 - t, which puts short edge t (written at stride - 1 - t) at nl + t
                int pairs = min(ns, (stride - nl) / 2);
                for (int t0 = 0; t0 < pairs; t0 += 4) {  // four swaps in flight
                    float4 ex[4], ey[4];
                    int sx[4], sy[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        if (t0 + u < pairs) {
                            long long x = base + nl + t0 + u, y = base + stride - 1 - t0 - u;
                            ex[u] = edges[x];
                            ey[u] = edges[y];
                            sx[u] = shifts[x];
                            sy[u] = shifts[y];
                        }
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        if (t0 + u < pairs) {
                            long long x = base + nl + t0 + u, y = base + stride - 1 - t0 - u;
                            edges[x] = ey[u];
                            shifts[x] = sy[u];
                            edges[y] = ex[u];
                            shifts[y] = sx[u];
                        }
                }
            }
            rp_full[i] = (int)base;
            cnt_full[i] = fits ? nl + ns : 0;
            rp_short[i] = (int)base + (fits ? nl : 0);
            cnt_short[i] = fits ? ns : 0;
            int nt = nl + ns;
            unsigned long long nr = radial_is_full ? nt : ns, na = radial_is_full ? ns : nt;
            unsigned long long inv = 0xffffffffull - (unsigned long long)i;
            m_r = max(m_r, (nr << 32) | inv);
            m_a = max(m_a, (na << 32) | inv);
            s_r += nr;
            s_a += na;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        m_r = max(m_r, __shfl_xor_sync(0xffffffffu, m_r, o));
        m_a = max(m_a, __shfl_xor_sync(0xffffffffu, m_a, o));
        s_r += __shfl_xor_sync(0xffffffffu, s_r, o);
        s_a += __shfl_xor_sync(0xffffffffu, s_a, o);
    }
    if (lane == 0) {
        atomicMax(&summary[0], m_r);
        atomicMax(&summary[1], m_a);
        atomicAdd(&summary[2], s_r);
        atomicAdd(&summary[3], s_a);
    }
}

// Exact lists from candidate lists (the Verlet-skin cache), warp per atom, lanes over the
// candidates of its row: the pair vector is re-formed in float64 from the current positions and
// the candidate's image shift, (R_j - R_i) + S.cell (exactly antisymmetric), and classified
// against the two cutoffs. A first pass counts, a second writes the long edges from the front of
// the row and the short ones behind them, both in candidate order. Count summary as in
// k_nbr_build.
__global__ void k_filter_candidates(int n_atoms, EdgeList cand, const int* __restrict__ cshifts,
                                    const double* __restrict__ pos,
                                    const StructGeom* __restrict__ geom,
                                    const int* __restrict__ sid, double rc_max2, double rc_min2,
                                    bool radial_is_full, float4* __restrict__ edges,
                                    int* __restrict__ shifts, int* __restrict__ rp_full,
                                    int* __restrict__ cnt_full, int* __restrict__ rp_short,
                                    int* __restrict__ cnt_short,
                                    unsigned long long* __restrict__ summary) {
    int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (i >= n_atoms) return;
    const StructGeom& g = geom[sid[i]];
    int b = cand.row_ptr[i], nc = cand.cnt[i];
    double pi0 = pos[3 * i], pi1 = pos[3 * i + 1], pi2 = pos[3 * i + 2];
    unsigned lt = (1u << lane) - 1u;
    int nl_total = 0;
    for (int pass = 0; pass < 2; ++pass) {
        int nl = 0, ns = 0;
        for (int k0 = 0; k0 < nc; k0 += 32) {
            int k = k0 + lane;
            bool in_max = false, in_min = false;
            double d0 = 0, d1 = 0, d2 = 0;
            int j = 0, sh = 0;
            if (k < nc) {
                j = edge_j(cand.e[b + k]);
                sh = cshifts[b + k];
                int s0 = ((sh & 1023) ^ 512) - 512, s1 = (((sh >> 10) & 1023) ^ 512) - 512;
                int s2 = (((sh >> 20) & 1023) ^ 512) - 512;
                d0 = (pos[3 * j] - pi0) + (s0 * g.cell[0] + s1 * g.cell[3] + s2 * g.cell[6]);
                d1 = (pos[3 * j + 1] - pi1) + (s0 * g.cell[1] + s1 * g.cell[4] + s2 * g.cell[7]);
                d2 = (pos[3 * j + 2] - pi2) + (s0 * g.cell[2] + s1 * g.cell[5] + s2 * g.cell[8]);
                double r2 = d0 * d0 + d1 * d1 + d2 * d2;
                in_max = r2 < rc_max2;
                in_min = r2 < rc_min2;
            }
            bool is_long = in_max && !in_min;
            unsigned ml = __ballot_sync(0xffffffffu, is_long);
            unsigned ms = __ballot_sync(0xffffffffu, in_min);
            if (pass == 1 && (is_long || in_min)) {
                int slot = is_long ? b + nl + __popc(ml & lt) : b + nl_total + ns + __popc(ms & lt);
                edges[slot] = make_float4((float)d0, (float)d1, (float)d2, __int_as_float(j));
                shifts[slot] = sh;
            }
            nl += __popc(ml);
            ns += __popc(ms);
        }
        if (pass == 0) {
            nl_total = nl;
            if (lane == 0) {
                rp_full[i] = b;
                cnt_full[i] = nl + ns;
                rp_short[i] = b + nl;
                cnt_short[i] = ns;
                int nt = nl + ns;
                unsigned long long nr = radial_is_full ? nt : ns, na = radial_is_full ? ns : nt;
                unsigned long long inv = 0xffffffffull - (unsigned long long)i;
                atomicMax(&summary[0], (nr << 32) | inv);
                atomicMax(&summary[1], (na << 32) | inv);
                atomicAdd(&summary[2], nr);
                atomicAdd(&summary[3], na);
            }
        }
    }
}

// Padded reference rows -> CSR. Entries equal to -1 are skipped wherever they sit in a row.
__global__ void k_padded_count(int n_atoms, int width, const int64_t* __restrict__ nbr,
                               int n_atoms_check, const int* __restrict__ types, int n_types,
                               int* __restrict__ cnt, unsigned int* __restrict__ flags) {
    int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= n_atoms) return;
    if (types[a] < 0 || types[a] >= n_types) atomicOr(flags, 1u);
    int c = 0;
    for (int k = 0; k < width; ++k) {
        int64_t j = nbr[(int64_t)a * width + k];
        if (j == -1) continue;
        if (j < 0 || j >= n_atoms_check) atomicOr(flags, 4u);
        ++c;
    }
    cnt[a] = c;
}

__global__ void k_padded_fill(int n_atoms, int width, const int64_t* __restrict__ nbr,
                              const float* __restrict__ off, const float* __restrict__ pos,
                              const int* __restrict__ row_ptr, float4* __restrict__ edges) {
    int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= n_atoms) return;
    int o = row_ptr[a];
    for (int k = 0; k < width; ++k) {
        int64_t jj = nbr[(int64_t)a * width + k];
        if (jj < 0 || jj >= n_atoms) continue;
        int j = (int)jj;
        const float* of = off + ((int64_t)a * width + k) * 3;
        // (R_j - R_i) + off formed exactly in float64 from the float32 inputs, rounded once, so
        // the error is relative to |r| (the reference's float32 (R_j + off) - R_i rounds at |R|)
        float r0 = (float)(((double)pos[3 * j] - (double)pos[3 * a]) + (double)of[0]);
        float r1 = (float)(((double)pos[3 * j + 1] - (double)pos[3 * a + 1]) + (double)of[1]);
        float r2 = (float)(((double)pos[3 * j + 2] - (double)pos[3 * a + 2]) + (double)of[2]);
        edges[o++] = make_float4(r0, r1, r2, __int_as_float(j));
    }
}

// Reverse-edge index: for edge e = (i -> j, r) find (j -> i, ~-r) in row j. Distinct periodic
// images of one atom differ by a lattice vector, so a 1e-4 A match is unambiguous.
__global__ void k_rev_index(int n_atoms, EdgeList L, int* __restrict__ rev,
                            unsigned int* __restrict__ flags) {
    int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    if (i >= n_atoms) return;
    int b = L.row_ptr[i], n = L.cnt[i];
    for (int k = lane; k < n; k += 32) {
        float4 e = L.e[b + k];
        int j = edge_j(e);
        int bj = L.row_ptr[j], nj = L.cnt[j];
        int found = -1;
        // four candidates per step, their loads in flight together
        for (int m = 0; m < nj && found < 0; m += 4) {
            float4 f[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) f[u] = L.e[bj + min(m + u, nj - 1)];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float x = e.x + f[u].x, y = e.y + f[u].y, z = e.z + f[u].z;
                if (found < 0 && m + u < nj && edge_j(f[u]) == i &&
                    x * x + y * y + z * z < 1.0e-8f)
                    found = bj + m + u;
            }
        }
        if (found < 0) atomicOr(flags, 8u);
        rev[b + k] = found < 0 ? b + k : found;
    }
}

// Neighbour limit of the list with the larger cutoff (a full row never needs more slots).
inline int cfg_full_limit(const rune_model_config& c) {
    return c.rc_radial >= c.rc_angular ? c.max_neighbors_radial : c.max_neighbors_angular;
}

inline int blocks_for(long long n, int per) { return (int)((n + per - 1) / per); }

}  // namespace

// ----------------------------------------------------------------------------- host side
static void structure_geometry(const double* cells, const uint8_t* pbc, int n_structures,
                               double rc, std::vector<StructGeom>& out, int& total_bins) {
    out.resize(n_structures);
    total_bins = 0;
    for (int s = 0; s < n_structures; ++s) {
        StructGeom& g = out[s];
        const double* c = cells + 9 * s;
        bool any = pbc[3 * s] || pbc[3 * s + 1] || pbc[3 * s + 2];
        double m[9];
        for (int k = 0; k < 9; ++k) m[k] = c[k];
        double det = m[0] * (m[4] * m[8] - m[5] * m[7]) - m[1] * (m[3] * m[8] - m[5] * m[6]) +
                     m[2] * (m[3] * m[7] - m[4] * m[6]);
        if (!any && std::fabs(det) < 1e-12) {
            for (int k = 0; k < 9; ++k) m[k] = (k % 4 == 0) ? 1.0 : 0.0;
            det = 1.0;
        }
        if (std::fabs(det) < 1e-12)
            throw Error(RUNE_ERR_INVALID,
                        "Degenerate cell is not supported for periodic neighbor construction.");
        for (int k = 0; k < 9; ++k) g.cell[k] = m[k];
        // inverse (frac = pos @ inv)
        double id = 1.0 / det;
        g.inv[0] = (m[4] * m[8] - m[5] * m[7]) * id;
        g.inv[1] = (m[2] * m[7] - m[1] * m[8]) * id;
        g.inv[2] = (m[1] * m[5] - m[2] * m[4]) * id;
        g.inv[3] = (m[5] * m[6] - m[3] * m[8]) * id;
        g.inv[4] = (m[0] * m[8] - m[2] * m[6]) * id;
        g.inv[5] = (m[2] * m[3] - m[0] * m[5]) * id;
        g.inv[6] = (m[3] * m[7] - m[4] * m[6]) * id;
        g.inv[7] = (m[1] * m[6] - m[0] * m[7]) * id;
        g.inv[8] = (m[0] * m[4] - m[1] * m[3]) * id;
        // plane spacings: volume / |b x c| etc.
        auto cross_norm = [&](int u, int v) {
            double x = m[3 * u + 1] * m[3 * v + 2] - m[3 * u + 2] * m[3 * v + 1];
            double y = m[3 * u + 2] * m[3 * v + 0] - m[3 * u + 0] * m[3 * v + 2];
            double z = m[3 * u + 0] * m[3 * v + 1] - m[3 * u + 1] * m[3 * v + 0];
            return std::sqrt(x * x + y * y + z * z);
        };
        double vol = std::fabs(det);
        double h[3] = {vol / cross_norm(1, 2), vol / cross_norm(2, 0), vol / cross_norm(0, 1)};
        int bins = 1;
        for (int k = 0; k < 3; ++k) {
            g.pbc[k] = pbc[3 * s + k] ? 1 : 0;
            if (g.pbc[k]) {
                long long nb = (long long)std::floor(h[k] / rc);
                nb = std::max(1LL, std::min(nb, 1024LL));
                g.nb[k] = (int)nb;
                g.reach[k] = (int)std::ceil(rc * nb / h[k] - 1e-12);
                if (g.reach[k] < 1) g.reach[k] = 1;
                if (g.reach[k] > 400)
                    throw Error(RUNE_ERR_INVALID, "Periodic cell is too thin for the cutoff.");
            } else {
                // no images; bins of at least rc across the cell when it is a real one (a
                // structure without periodic axes and without a cell has the unit cell here)
                long long nb = (long long)std::floor(h[k] / rc);
                nb = std::max(1LL, std::min(nb, 1024LL));
                g.nb[k] = (int)nb;
                g.reach[k] = nb == 1 ? 0 : (int)std::min<long long>(
                                                nb - 1, (long long)std::ceil(rc * nb / h[k] - 1e-12));
            }
            bins *= g.nb[k];
        }
        g.bin_offset = total_bins;
        total_bins += bins;
    }
}

template <typename T>
static void exclusive_scan(Engine& eng, const T* in, T* out, int n, cudaStream_t stream) {
    size_t bytes = 0;
    RUNE_CUDA_TRY(cub::DeviceScan::ExclusiveSum(nullptr, bytes, in, out, n, stream));
    void* tmp = eng.ws.take(bytes + 256);
    KernelScope ks("cub_exclusive_scan", stream, 2);
    RUNE_CUDA_TRY(cub::DeviceScan::ExclusiveSum(tmp, bytes, in, out, n, stream));
}

// Row stride of the edge slab: the previous call's (kept while it fits), else a density
// estimate per structure (atoms per cell volume x sphere volume, with 50% headroom; a
// structure without a cell volume holds at most its own atom count), rounded up to 8.
static int row_stride(Engine& eng, const BatchInput& in, double rc, bool candidates) {
    const double pi = 3.14159265358979323846;
    double sphere = 4.0 / 3.0 * pi * rc * rc * rc;
    double est = 16.0;
    for (int s = 0; s < in.n_structures; ++s) {
        int ns = in.atom_ptr[s + 1] - in.atom_ptr[s];
        const double* c = in.cells + 9 * s;
        double vol = std::fabs(c[0] * (c[4] * c[8] - c[5] * c[7]) -
                               c[1] * (c[3] * c[8] - c[5] * c[6]) +
                               c[2] * (c[3] * c[7] - c[4] * c[6]));
        // without periodic axes the cell only bins (atoms may lie outside it): an estimate
        // that proves too small costs one repeat of the call with the stride raised
        double e = vol > 1e-6 ? 1.5 * ns / vol * sphere + 16.0 : (double)ns + 8.0;
        est = std::max(est, e);
    }
    // a full row never needs more than max_neighbors slots (larger counts are an error), except
    // a candidate row, which also holds the skin shell
    int cap = std::max(cfg_full_limit(eng.cfg), 8) + 8;
    if (candidates) cap = 4 * cap + 64;
    long long v = std::min<long long>((long long)std::ceil(est), cap);
    return (int)((v + 7) & ~7LL);
}

void build_neighbors(Engine& eng, const BatchInput& in, const int* d_atom_ptr, NeighborData& nd,
                     cudaStream_t stream, double skin, int* stride_state) {
    const rune_model_config& cfg = eng.cfg;
    int n = in.n_atoms;
    // With a skin the rows are candidate lists: every pair within max(rc) + skin, none split off
    // as short (rc_min < 0), in rows of their own persistent stride.
    double rc_max = std::max(cfg.rc_radial, cfg.rc_angular) + skin;
    double rc_min = skin > 0.0 ? -1.0 : std::min(cfg.rc_radial, cfg.rc_angular);
    int& stride_ref = stride_state ? *stride_state : eng.row_stride;
    std::vector<StructGeom> geom;
    int total_bins = 0;
    structure_geometry(in.cells, in.pbc, in.n_structures, rc_max, geom, total_bins);

    const StructGeom* d_geom = static_cast<const StructGeom*>(
        eng.stage_upload(geom.data(), sizeof(StructGeom) * geom.size(), stream));
    eng.flush_uploads(stream);  // one copy for this call's host tables
    int* sid = eng.ws.take_n<int>(n);
    int* tsafe = eng.ws.take_n<int>(n);
    int4* binc = eng.ws.take_n<int4>(n);
    int4* wrap = eng.ws.take_n<int4>(n);
    int* bin_count = eng.ws.take_n<int>(total_bins + 1);
    int* bin_start = eng.ws.take_n<int>(total_bins + 1);
    int* bin_fill = eng.ws.take_n<int>(total_bins + 1);
    int* bin_tmp = eng.ws.take_n<int>(n);
    int* batom = eng.ws.take_n<int>(n);
    double4* bpos = eng.ws.take_n<double4>(n);
    int* cnt_short = eng.ws.take_n<int>(n + 1);
    int* cnt_full = eng.ws.take_n<int>(n + 1);
    int* rp_short = eng.ws.take_n<int>(n + 1);
    int* rp_full = eng.ws.take_n<int>(n + 1);
    unsigned long long* summary = eng.ws.take_n<unsigned long long>(4);
    int stride = stride_ref > 0 ? stride_ref : row_stride(eng, in, rc_max, skin > 0.0);
    long long slab = (long long)n * stride;
    if (slab + 1 > INT32_MAX)
        throw Error(RUNE_ERR_INVALID, "batch too large: " + std::to_string(n) + " atoms x " +
                                          std::to_string(stride) +
                                          " edge slots exceed 2^31 edges per call");
    float4* edges = eng.ws.take_n<float4>((size_t)slab + 1);
    int* shifts = eng.ws.take_n<int>((size_t)slab + 1);
    RUNE_CUDA_TRY(cudaMemsetAsync(bin_count, 0, sizeof(int) * (total_bins + 1), stream));
    RUNE_CUDA_TRY(cudaMemsetAsync(bin_fill, 0, sizeof(int) * (total_bins + 1), stream));
    RUNE_CUDA_TRY(cudaMemsetAsync(summary, 0, sizeof(unsigned long long) * 4, stream));

    const int tpb = 256;
    if (n > 0) {
        RUNE_KERNEL("k_bin_atoms", stream,
                    k_bin_atoms<<<blocks_for(n, tpb), tpb, 0, stream>>>(
                        n, cfg.n_types, in.n_structures, d_atom_ptr, in.positions, in.types,
                        d_geom, tsafe, sid, binc, wrap, bin_count, eng.d_flags));
        RUNE_LAUNCH_CHECK();
    }
    exclusive_scan(eng, bin_count, bin_start, total_bins + 1, stream);
    if (n > 0) {
        RUNE_KERNEL("k_fill_bins", stream,
                    k_fill_bins<<<blocks_for(n, tpb), tpb, 0, stream>>>(n, binc, bin_start,
                                                                          bin_fill, bin_tmp));
        RUNE_KERNEL("k_sort_bins", stream,
                    k_sort_bins<<<blocks_for((long long)total_bins * 32, tpb), tpb, 0, stream>>>(
                        total_bins, bin_start, bin_count, bin_tmp, in.positions, wrap, sid,
                        d_geom, batom, bpos));
        RUNE_LAUNCH_CHECK();
    }
    Traverse tv{d_geom, sid, bin_start, bin_count, batom, bpos, rc_max * rc_max,
                rc_min < 0.0 ? -1.0 : rc_min * rc_min};
    bool radial_is_full = cfg.rc_radial >= cfg.rc_angular;
    if (n > 0) {
        RUNE_KERNEL("k_nbr_build", stream,
                    k_nbr_build<<<blocks_for(total_bins, kBuildWarps), kBuildWarps * 32, 0,
                                  stream>>>(total_bins, tv, stride, radial_is_full, edges,
                                            shifts, rp_full, cnt_full, rp_short, cnt_short,
                                            summary, eng.d_flags));
        RUNE_LAUNCH_CHECK();
    }
    EdgeList full{edges, rp_full, cnt_full, nullptr};
    EdgeList shrt{edges, rp_short, cnt_short, nullptr};
    nd.n_atoms = n;
    nd.total_edges = (int)slab;
    nd.edges = edges;
    nd.shifts = shifts;
    nd.radial = radial_is_full ? full : shrt;
    nd.angular = radial_is_full ? shrt : full;
    nd.cnt_r = nd.radial.cnt;
    nd.cnt_a = nd.angular.cnt;
    nd.positions64 = in.positions;
    nd.sid = sid;
    nd.geom = d_geom;
    nd.summary = summary;
    nd.capacity = slab;
    nd.types = tsafe;
    eng.stats.neighbor_builds++;
}

void filter_candidates(Engine& eng, const NeighborData& cand, const double* positions,
                       NeighborData& nd, cudaStream_t stream) {
    const rune_model_config& cfg = eng.cfg;
    int n = cand.n_atoms;
    double rc_max = std::max(cfg.rc_radial, cfg.rc_angular);
    double rc_min = std::min(cfg.rc_radial, cfg.rc_angular);
    bool radial_is_full = cfg.rc_radial >= cfg.rc_angular;
    long long slab = cand.capacity;
    float4* edges = eng.ws.take_n<float4>((size_t)slab + 1);
    int* shifts = eng.ws.take_n<int>((size_t)slab + 1);
    int* rp_full = eng.ws.take_n<int>(n + 1);
    int* cnt_full = eng.ws.take_n<int>(n + 1);
    int* rp_short = eng.ws.take_n<int>(n + 1);
    int* cnt_short = eng.ws.take_n<int>(n + 1);
    unsigned long long* summary = eng.ws.take_n<unsigned long long>(4);
    RUNE_CUDA_TRY(cudaMemsetAsync(summary, 0, sizeof(unsigned long long) * 4, stream));
    const int tpb = 256;
    if (n > 0) {
        EdgeList c = cand.radial;  // the candidate rows (one class)
        RUNE_KERNEL("k_filter_candidates", stream,
                    k_filter_candidates<<<blocks_for((long long)n * 32, tpb), tpb, 0, stream>>>(
                        n, c, cand.shifts, positions, cand.geom, cand.sid, rc_max * rc_max,
                        rc_min * rc_min, radial_is_full, edges, shifts, rp_full, cnt_full,
                        rp_short, cnt_short, summary));
        RUNE_LAUNCH_CHECK();
    }
    EdgeList full{edges, rp_full, cnt_full, nullptr};
    EdgeList shrt{edges, rp_short, cnt_short, nullptr};
    nd = cand;
    nd.total_edges = (int)slab;
    nd.edges = edges;
    nd.shifts = shifts;
    nd.radial = radial_is_full ? full : shrt;
    nd.angular = radial_is_full ? shrt : full;
    nd.cnt_r = nd.radial.cnt;
    nd.cnt_a = nd.angular.cnt;
    nd.positions64 = positions;
    nd.summary = summary;
}

// End-of-call checks of a device-built list (after the stream synchronisation): neighbour
// limits, row overflow (returns false: rerun with the stride raised to the largest count);
// records the statistics.
bool finish_neighbors(Engine& eng, const NeighborData& nd, const HostSync& hs) {
    const rune_model_config& cfg = eng.cfg;
    int largest = 0;
    for (int which = 0; which < 2; ++which) {
        unsigned long long v = hs.maxc[which];
        int count = (int)(v >> 32);
        int atom = (int)(0xffffffffull - (v & 0xffffffffull));
        int limit = which == 0 ? cfg.max_neighbors_radial : cfg.max_neighbors_angular;
        largest = std::max(largest, count);
        if (nd.n_atoms > 0 && count > limit) {
            throw Error(RUNE_ERR_NEIGHBOR_OVERFLOW,
                        "Neighbor count " + std::to_string(count) + " for atom " +
                            std::to_string(atom) + " exceeds max_neighbors=" +
                            std::to_string(limit) +
                            ". Increase max_neighbors_radial or max_neighbors_angular.");
        }
    }
    if (hs.flags & 16u) {
        eng.row_stride = (largest + largest / 8 + 8 + 7) & ~7;
        return false;
    }
    eng.stats.last_radial_edges = (int64_t)hs.maxc[2];
    eng.stats.last_angular_edges = (int64_t)hs.maxc[3];
    eng.stats.last_edges = std::max(eng.stats.last_radial_edges, eng.stats.last_angular_edges);
    return true;
}

void build_padded(Engine& eng, const PaddedInput& in, NeighborData& nd, cudaStream_t stream) {
    int n = in.n_atoms;
    const int tpb = 256;
    EdgeList lists[2];
    int totals[2] = {0, 0};
    const int64_t* nbr[2] = {in.radial_neighbors, in.angular_neighbors};
    const float* off[2] = {in.radial_offsets, in.angular_offsets};
    int width[2] = {in.radial_width, in.angular_width};
    int* cnt[2];
    int* rp[2];
    for (int w = 0; w < 2; ++w) {
        cnt[w] = eng.ws.take_n<int>(n + 1);
        rp[w] = eng.ws.take_n<int>(n + 1);
        RUNE_CUDA_TRY(cudaMemsetAsync(cnt[w] + n, 0, sizeof(int), stream));
        if (n > 0 && width[w] > 0) {
            RUNE_KERNEL("k_padded_count", stream, k_padded_count<<<blocks_for(n, tpb), tpb, 0, stream>>>(n, width[w], nbr[w], n,
                                                                     in.types, eng.cfg.n_types,
                                                                     cnt[w], eng.d_flags));
            RUNE_LAUNCH_CHECK();
        } else if (n > 0) {
            RUNE_CUDA_TRY(cudaMemsetAsync(cnt[w], 0, sizeof(int) * n, stream));
        }
        exclusive_scan(eng, cnt[w], rp[w], n + 1, stream);
    }
    HostSync* hs = eng.host_sync;
    RUNE_CUDA_TRY(cudaMemcpyAsync(&hs->total, rp[0] + n, sizeof(int), cudaMemcpyDeviceToHost,
                                  stream));
    RUNE_CUDA_TRY(cudaMemcpyAsync(&hs->total2, rp[1] + n, sizeof(int), cudaMemcpyDeviceToHost,
                                  stream));
    RUNE_CUDA_TRY(cudaMemcpyAsync(&hs->flags, eng.d_flags, sizeof(unsigned int),
                                  cudaMemcpyDeviceToHost, stream));
    RUNE_CUDA_TRY(cudaStreamSynchronize(stream));
    eng.check_flags(hs->flags, stream);
    totals[0] = hs->total;
    totals[1] = hs->total2;
    for (int w = 0; w < 2; ++w) {
        float4* e = eng.ws.take_n<float4>(totals[w] + 1);
        if (n > 0 && totals[w] > 0) {
            RUNE_KERNEL("k_padded_fill", stream, k_padded_fill<<<blocks_for(n, tpb), tpb, 0, stream>>>(n, width[w], nbr[w], off[w],
                                                                    in.positions, rp[w], e));
            RUNE_LAUNCH_CHECK();
        }
        lists[w] = EdgeList{e, rp[w], cnt[w], nullptr};
    }
    nd.n_atoms = n;
    nd.total_edges = totals[0];
    nd.total_angular = totals[1];
    nd.edges = nullptr;
    nd.shifts = nullptr;
    nd.radial = lists[0];
    nd.angular = lists[1];
    nd.cnt_r = cnt[0];
    nd.cnt_a = cnt[1];
    eng.stats.last_edges = totals[0];
    eng.stats.last_radial_edges = totals[0];
    eng.stats.last_angular_edges = totals[1];
}

void build_reverse(Engine& eng, NeighborData& nd, EdgeList& list, int n_edges,
                   cudaStream_t stream) {
    int* rev = eng.ws.take_n<int>(n_edges + 1);
    if (nd.n_atoms > 0 && n_edges > 0) {
        RUNE_KERNEL("k_rev_index", stream, k_rev_index<<<blocks_for((long long)nd.n_atoms * 32, 256), 256, 0, stream>>>(
            nd.n_atoms, list, rev, eng.d_flags));
        RUNE_LAUNCH_CHECK();
    }
    list.rev = rev;
}

}  // namespace rune
