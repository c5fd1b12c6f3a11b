// Descriptor forward, NEP per-element network, invariant adjoint and the analytic force /
// virial kernel.
//
// Mathematics (reference rune/mobius/descriptor.py, identical in rune/nep/descriptor.py):
//   f_k(r)      = 0.5 (T_k(x) + 1) fc(r),  x = 2 (r/rc - 1)^2 - 1, fc = 0.5 cos(pi r/rc) + 0.5
//                 (descriptor.py:377-414, derivative through U_{k-1})
//   q_r[i, n]   = sum_j sum_k c_r[t_i, t_j, n, k] f_k(r_ij)                     (:839-851)
//   s[i, n, c]  = sum_j g_n(r_ij) Y_c(r_ij / r_ij),  g_n = sum_k c_a[t_i, t_j, n, k] f_k (:853-880)
//   q_ang[i, n, L] = polynomial invariants of s[i, n, :]                         (:650-733)
//   q[i] = [q_r, q_ang permuted L-major]                                         (:882-888)
// Forces follow rune/mobius/force.py:165-243 with the per-edge gradient g_e = dE/dr_e added
// to the centre and subtracted from the neighbour.
//
// Thread mapping: one warp per atom. Edge-parallel work (basis functions, harmonics) has one
// lane per edge; contractions switch to one lane per output channel so that the c-table rows
// of a type pair are read contiguously. All sums run in a fixed order: results are
// deterministic and no floating-point atomics are used.
//
// Force assembly is "pull" style: the neighbour lists are symmetric, so the transposed sum
// F_j -= g_e over edges e = (i -> j) equals, for atom j, a sum over its own row of the reverse
// edge's gradient, which the warp of atom j evaluates from atom i's adjoints (gathered) and
// r_rev = -r_e. Parity gives Y_L(-u) = (-1)^L Y_L(u), so harmonics are evaluated once per
// edge for both directions.

#include <type_traits>

#include "basis.cuh"
#include "engine.cuh"

namespace rune {

namespace {

constexpr int kWarpsPerBlock = 4;
constexpr unsigned kNoFactor = 0xffu;
constexpr int kTile = 64;  // atoms per tile of the NEP tiled layouts

// Shared-memory copies of the transposed c-tables for small type counts (float offsets into the
// kernel's dynamic shared memory, -1 = read from global memory).
struct Stage {
    int r = -1, a = -1;
};

__host__ __device__ inline int c_table_float4s(const DescParams& p, bool radial) {
    return p.T * p.T * (radial ? p.kr * p.npr : p.ka * p.npa);
}

// Copies the staged tables (all threads of the block) and points p at them; ends with a block
// barrier, so every thread of the block must call it before any early return.
__device__ __forceinline__ void stage_tables(DescParams& p, Stage st, float* smem) {
    if (st.r >= 0) {
        float4* dst = reinterpret_cast<float4*>(smem + st.r);
        for (int k = threadIdx.x; k < c_table_float4s(p, true); k += blockDim.x)
            dst[k] = __ldg(p.c_rt + k);
        p.c_rt = dst;
    }
    if (st.a >= 0) {
        float4* dst = reinterpret_cast<float4*>(smem + st.a);
        for (int k = threadIdx.x; k < c_table_float4s(p, false); k += blockDim.x)
            dst[k] = __ldg(p.c_at + k);
        p.c_at = dst;
    }
    __syncthreads();
}

// acc[n] += f * c[n] for the npr (or npa) float4 of one basis function k.
template <int NMAX>
__device__ __forceinline__ void axpy_row(float* acc, const float4* ck, int np,
                                         float f) {
#pragma unroll
    for (int q = 0; q < NMAX / 4; ++q)
        if (q < np) {
            float4 c = ck[q];  // generic load: the table may be staged in shared memory
            acc[4 * q] += c.x * f;
            acc[4 * q + 1] += c.y * f;
            acc[4 * q + 2] += c.z * f;
            acc[4 * q + 3] += c.w * f;
        }
}

// q_ang[L][n] of one atom from its moments s[n][c] (row stride cs), lanes over (L, n); the
// terms of output L are term_ptr[L] .. term_ptr[L + 1] of the packed monomial table.
__device__ __forceinline__ void invariants(const DescParams& p, const float* sacc, int cs,
                                           float* qang, int lane) {
    for (int o = lane; o < p.na * p.nL; o += 32) {
        int L = o / p.na, n = o - L * p.na;
        const float* sn = sacc + n * cs;
        int t0 = __ldg(p.term_ptr + L), t1 = __ldg(p.term_ptr + L + 1);
        float v = 0.0f;
        for (int k = t0; k < t1; ++k) {
            int4 t = __ldg(p.terms + k);
            unsigned f = (unsigned)t.z;
            float x = __int_as_float(t.x) * sn[f & 0xffu] * sn[(f >> 8) & 0xffu];
            unsigned i2 = (f >> 16) & 0xffu, i3 = f >> 24;
            if (i2 != kNoFactor) x *= sn[i2];
            if (i3 != kNoFactor) x *= sn[i3];
            v += x;
        }
        qang[o] = v;
    }
}

// Angular adjoint w[c][n] = mg[n][c] + sum_L dq[L][n] d q_L[n] / d s[n][c], lanes over (c, n):
// the product rule applied through the derivative table, whose entries for harmonic c hold
// (coef, L, the other factors) of every occurrence of c in a term (rune/mobius/force.py:28-133).
__device__ __forceinline__ void invariant_adjoint(const DescParams& p, const float* sacc, int cs,
                                                  const float* dqang /* [L][na] */,
                                                  const float* mg /* [na][C] or null */,
                                                  float* w /* [C][na] */, int lane) {
    for (int o = lane; o < p.na * p.C; o += 32) {
        int c = o / p.na, n = o - c * p.na;
        const float* sn = sacc + n * cs;
        float v = mg ? mg[n * p.C + c] : 0.0f;
        int d0 = __ldg(p.dterm_ptr + c), d1 = __ldg(p.dterm_ptr + c + 1);
        for (int k = d0; k < d1; ++k) {
            int4 t = __ldg(p.dterms + k);
            unsigned f = (unsigned)t.z;
            float x = __int_as_float(t.x) * dqang[t.y * p.na + n];
            unsigned o0 = f & 0xffu, o1 = (f >> 8) & 0xffu, o2 = (f >> 16) & 0xffu;
            if (o0 != kNoFactor) x *= sn[o0];
            if (o1 != kNoFactor) x *= sn[o1];
            if (o2 != kNoFactor) x *= sn[o2];
            v += x;
        }
        w[o] = v;
    }
}

// Centre-side gradient dE/dr_e of every angular edge of atom a (rune/mobius/force.py:195-241):
//   g_e = rs u + (dir - (dir . u) u) / r,   rs = sum_nc w[c][n] g'_n Y_c,
//   dir = sum_c (sum_n w[c][n] g_n) grad Y_c
// with the adjoint w [C][na] of atom a in shared memory; lane per edge, g_n and g'_n in
// registers (NMAX >= na).
template <int NMAX, int LMAX, bool F32 = false, int NA = 0>
__device__ __forceinline__ void angular_edge_grads(const DescParams& p, const EdgeList& ang,
                                                   const int* __restrict__ types, int a, int ta,
                                                   const float* sw, int lane,
                                                   float4* __restrict__ grad) {
    // channel count: exact at compile time when NA > 0 (the unrolled channel loops then hold
    // no predicated padding channels), else the table's
    const int na = NA > 0 ? NA : p.na;
    const int npa = NA > 0 ? (NA + 3) / 4 : p.npa;
    int b = ang.row_ptr[a], cnt = ang.cnt[a];
    for (int k = lane; k < cnt; k += 32) {
        float4 e = ang.e[b + k];
        float r = edge_len<F32>(e);
        float inv = 1.0f / fmaxf(r, 1.0e-12f);
        float ux = e.x * inv, uy = e.y * inv, uz = e.z * inv;
        const float4* crow = p.c_at + (size_t)(ta * p.T + types[edge_j(e)]) * p.ka * p.npa;
        float g[NMAX], gp[NMAX];
#pragma unroll
        for (int n = 0; n < NMAX; ++n) g[n] = gp[n] = 0.0f;
        basis_visit<F32, true>(r, p.rc_a, p.ka, [&](int kk, float f, float df) {
            const float4* ck = crow + kk * p.npa;
#pragma unroll
            for (int q = 0; q < NMAX / 4; ++q)
                if (q < npa) {
                    float4 c = ck[q];  // generic load: the table may be staged in shared memory
                    g[4 * q] += c.x * f;      gp[4 * q] += c.x * df;
                    g[4 * q + 1] += c.y * f;  gp[4 * q + 1] += c.y * df;
                    g[4 * q + 2] += c.z * f;  gp[4 * q + 2] += c.z * df;
                    g[4 * q + 3] += c.w * f;  gp[4 * q + 3] += c.w * df;
                }
        });
        float rs = 0.f, d0 = 0.f, d1 = 0.f, d2 = 0.f;
        angular_components<true, LMAX>(ux, uy, uz, p.lmax, p.zc,
                                       [&](int c, int, float Y, float dx, float dy, float dz) {
            const float* wc = sw + c * na;
            float a1 = 0.f, a2 = 0.f;
            if constexpr (NMAX <= 32) {
#pragma unroll
                for (int n = 0; n < NMAX; ++n)
                    if (n < na) {
                        a1 += wc[n] * gp[n];
                        a2 += wc[n] * g[n];
                    }
            } else {  // more than 32 channels: rolled loop (g, gp in local memory)
                for (int n = 0; n < na; ++n) {
                    a1 += wc[n] * gp[n];
                    a2 += wc[n] * g[n];
                }
            }
            rs += Y * a1;
            d0 += a2 * dx; d1 += a2 * dy; d2 += a2 * dz;
        });
        float pu = d0 * ux + d1 * uy + d2 * uz;
        grad[b + k] = make_float4(rs * ux + (d0 - pu * ux) * inv, rs * uy + (d1 - pu * uy) * inv,
                                  rs * uz + (d2 - pu * uz) * inv, 0.0f);
    }
}

// The radial adjoint dq[0 .. nr) as npr float4 per atom (zero padded), for the force kernel.
__device__ __forceinline__ void store_dqr(const DescParams& p, const float* sdq,
                                          float4* __restrict__ dqr, int i, int lane) {
    for (int q = lane; q < p.npr; q += 32) {
        int n = 4 * q;
        dqr[(size_t)i * p.npr + q] =
            make_float4(n < p.nr ? sdq[n] : 0.f, n + 1 < p.nr ? sdq[n + 1] : 0.f,
                        n + 2 < p.nr ? sdq[n + 2] : 0.f, n + 3 < p.nr ? sdq[n + 3] : 0.f);
    }
}

struct ForwardSmem {
    // per-warp float offsets; rows padded to an odd stride (no bank conflicts)
    int ys, gs, cs, sy, sg, sacc, sq, total;
    __host__ __device__ explicit ForwardSmem(const DescParams& p) {
        ys = p.C | 1;
        gs = p.na | 1;
        cs = p.C | 1;
        sy = 0;
        sg = sy + 32 * ys;
        sacc = sg + 32 * gs;
        sq = sacc + p.na * cs;
        total = sq + p.D;
        total = (total + 3) & ~3;
    }
};

struct NepHead {
    int H;
    const float* w1;      // [T][H][Dp], rows padded to a multiple of 4
    const float* w1t;     // [T][D][Hp]
    const float* b1;      // [T][H]
    const float* w2;      // [T][H]
    const float* scaler;  // [Dp]
    float bias;
};

// Descriptor forward, warp per atom, lane per edge. Row layout (Möbius): q [N, D] with the
// invariants, s [N, na, C]. Tiled layout (NEP): the radial channels and the moments only, in
// 128-atom tiles (element e of atom a at tile(a) + e * 128 + a % 128), for the thread-per-atom
// kernel that finishes the descriptor and runs the element network.
template <bool TILED, int NMAX, int LMAX>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
k_desc_forward(int n_atoms, DescParams p, EdgeList rad, EdgeList ang,
               const int* __restrict__ types, float* __restrict__ q_out,
               float* __restrict__ s_out, Stage st) {
    extern __shared__ float4 smem_f4[];
    float* smem = reinterpret_cast<float*>(smem_f4);
    stage_tables(p, st, smem);
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int i = blockIdx.x * kWarpsPerBlock + warp;
    ForwardSmem L(p);
    float* sm = smem + warp * L.total;
    float* sy = sm + L.sy;
    float* sg = sm + L.sg;
    float* sacc = sm + L.sacc;
    float* sq = sm + L.sq;
    if (i >= n_atoms) return;
    int ti = types[i];

    // ---- radial channels q_r[n]: lane per edge, channel sums in registers
    {
        float acc[NMAX];
#pragma unroll
        for (int n = 0; n < NMAX; ++n) acc[n] = 0.0f;
        int b = rad.row_ptr[i], cnt = rad.cnt[i];
        for (int k = lane; k < cnt; k += 32) {
            float4 e = rad.e[b + k];
            float r = edge_len<TILED>(e);
            const float4* crow = p.c_rt + (size_t)(ti * p.T + types[edge_j(e)]) * p.kr * p.npr;
            basis_visit<TILED, false>(r, p.rc_r, p.kr, [&](int kk, float f, float) {
                axpy_row<NMAX>(acc, crow + kk * p.npr, p.npr, f);
            });
        }
#pragma unroll
        for (int n = 0; n < NMAX; ++n)
            if (n < p.nr) {
                float v = warp_sum(acc[n]);
                if (lane == 0) sq[n] = v;
            }
    }

    // ---- angular moments s[n][c]: lane per edge for g_n and Y_c, lanes over (n, c) for the sum
    for (int o = lane; o < p.na * L.cs; o += 32) sacc[o] = 0.0f;
    {
        int b = ang.row_ptr[i], cnt = ang.cnt[i];
        for (int base = 0; base < cnt; base += 32) {
            int k = base + lane;
            if (k < cnt) {
                float4 e = ang.e[b + k];
                float r = edge_len<TILED>(e);
                float inv = 1.0f / fmaxf(r, 1.0e-12f);
                float* yrow = sy + lane * L.ys;
                angular_components<false, LMAX>(e.x * inv, e.y * inv, e.z * inv, p.lmax, p.zc,
                                                [&](int c, int, float Y, float, float, float) {
                                                    yrow[c] = Y;
                                                });
                const float4* crow =
                    p.c_at + (size_t)(ti * p.T + types[edge_j(e)]) * p.ka * p.npa;
                float g[NMAX];
#pragma unroll
                for (int n = 0; n < NMAX; ++n) g[n] = 0.0f;
                basis_visit<TILED, false>(r, p.rc_a, p.ka, [&](int kk, float f, float) {
                    axpy_row<NMAX>(g, crow + kk * p.npa, p.npa, f);
                });
                float* grow = sg + lane * L.gs;
#pragma unroll
                for (int n = 0; n < NMAX; ++n)
                    if (n < p.na) grow[n] = g[n];
            }
            __syncwarp();
            int nv = min(32, cnt - base);
            for (int o = lane; o < p.na * p.C; o += 32) {
                int n = o / p.C, c = o - n * p.C;
                float s = sacc[n * L.cs + c];
                for (int ee = 0; ee < nv; ++ee) s += sg[ee * L.gs + n] * sy[ee * L.ys + c];
                sacc[n * L.cs + c] = s;
            }
            __syncwarp();
        }
    }

    if constexpr (TILED) {
        __syncwarp();
        size_t tq = (size_t)(i / kTile) * p.nr * kTile + (i % kTile);
        for (int n = lane; n < p.nr; n += 32) q_out[tq + (size_t)n * kTile] = sq[n];
        size_t ts = (size_t)(i / kTile) * p.na * p.C * kTile + (i % kTile);
        for (int o = lane; o < p.na * p.C; o += 32) {
            int n = o / p.C, c = o - n * p.C;
            s_out[ts + (size_t)o * kTile] = sacc[n * L.cs + c];
        }
        return;
    }
    // ---- invariants and descriptor row
    invariants(p, sacc, L.cs, sq + p.nr, lane);
    __syncwarp();
    if (q_out)
        for (int d = lane; d < p.D; d += 32) q_out[(size_t)i * p.D + d] = sq[d];
    if (s_out)
        for (int o = lane; o < p.na * p.C; o += 32) {
            int n = o / p.C, c = o - n * p.C;
            s_out[(size_t)i * p.na * p.C + o] = sacc[n * L.cs + c];
        }
}

// NEP per-atom work, four lanes per atom (a quad), 32 atoms per block: the invariants from the
// tiled moments, the element network E = w2 . tanh(W1 (q * scaler) + b1) - bias
// (rune/nep/model.py:157-170) and its adjoint dq, then — when forces are wanted — the radial
// adjoint (padded float4 rows) and the angular adjoint w [C][na] (tiled) for the edge kernels.
// The outputs of every stage (invariants, hidden units, dq entries, adjoint entries) are dealt
// round-robin to the quad's lanes. Per atom, shared memory holds the moments, q, the hidden
// derivatives and dq as rows; float4 rows have a stride of an odd number of float4 so that
// the eight quads of a warp hit distinct banks. The monomial and derivative tables are copied
// to shared memory once per block. Weights are float4 rows padded to multiples of 4
// (w1 [T][H][Dp], w1t [T][D][Hp]).
constexpr int kQuadAtoms = 32;  // atoms per block (128 threads)

__host__ __device__ inline int odd_float4_stride(int n) {
    int s = (n + 3) / 4;  // float4 per row
    return 4 * (s | 1);
}

struct NepAtomSmem {
    int dp4, hp4;                    // float4 per padded row of q (Dp / 4) and hidden (Hp / 4)
    int qs, zs, ss, ds;              // row strides (floats) of q, hidden, moments, dq
    int q, z, s, dq, terms, dterms, tptr, dptr, total;  // float offsets
    __host__ __device__ NepAtomSmem(const DescParams& p, int H) {
        dp4 = (p.D + 3) / 4;
        hp4 = (H + 3) / 4;
        qs = odd_float4_stride(p.D);
        zs = odd_float4_stride(H);
        ss = (p.na * p.C) | 1;
        ds = p.D | 1;
        q = 0;
        z = q + qs * kQuadAtoms;
        s = z + zs * kQuadAtoms;
        dq = s + ss * kQuadAtoms;
        terms = (dq + ds * kQuadAtoms + 3) & ~3;
        dterms = terms + 4 * p.n_terms;
        tptr = dterms + 4 * p.n_dterms;
        dptr = tptr + p.nL + 1;
        total = dptr + p.C + 1;
    }
};

__global__ void __launch_bounds__(4 * kQuadAtoms)
k_nep_atoms(int n_atoms, int n_owned, DescParams p, NepHead head, const int* __restrict__ types,
            const float* __restrict__ qr_t, const float* __restrict__ s_t,
            double* __restrict__ e_model, float4* __restrict__ dqr, float* __restrict__ w_t,
            float* __restrict__ gtab) {
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    const int H = head.H, D = p.D, nr = p.nr, na = p.na, C = p.C, NC = p.na * p.C;
    NepAtomSmem L(p, H);
    int4* TERMS = reinterpret_cast<int4*>(smem + L.terms);
    int4* DTERMS = reinterpret_cast<int4*>(smem + L.dterms);
    int* TPTR = reinterpret_cast<int*>(smem + L.tptr);
    int* DPTR = reinterpret_cast<int*>(smem + L.dptr);
    const int tid = threadIdx.x;
    const int a0 = blockIdx.x * kQuadAtoms;
    const int n_here = min(kQuadAtoms, n_atoms - a0);
    for (int k = tid; k < p.n_terms; k += blockDim.x) TERMS[k] = __ldg(p.terms + k);
    for (int k = tid; k < p.n_dterms; k += blockDim.x) DTERMS[k] = __ldg(p.dterms + k);
    for (int k = tid; k <= p.nL; k += blockDim.x) TPTR[k] = __ldg(p.term_ptr + k);
    for (int k = tid; k <= C; k += blockDim.x) DPTR[k] = __ldg(p.dterm_ptr + k);
    // moments and radial channels of the block's atoms, coalesced from the tiled layout
    for (int k = tid; k < kQuadAtoms * NC; k += blockDim.x) {
        int e = k / kQuadAtoms, j = k - e * kQuadAtoms;
        int a = a0 + j;
        if (j < n_here)
            smem[L.s + j * L.ss + e] =
                s_t[(size_t)(a / kTile) * NC * kTile + (size_t)e * kTile + (a % kTile)];
    }
    for (int k = tid; k < kQuadAtoms * L.qs; k += blockDim.x) {
        int e = k / kQuadAtoms, j = k - e * kQuadAtoms;
        int a = a0 + j;
        float v = 0.0f;
        if (j < n_here && e < nr)
            v = qr_t[(size_t)(a / kTile) * nr * kTile + (size_t)e * kTile + (a % kTile)];
        smem[L.q + j * L.qs + e] = v;  // invariants fill nr .. D below; padding stays 0
    }
    __syncthreads();
    const int j = tid >> 2, r = tid & 3;  // atom of this quad, lane within the quad
    const int a = a0 + j;
    if (j >= n_here) return;  // whole quads leave together; no block barrier below
    const unsigned qmask = 0xfu << (tid & 28);
    float* Q = smem + L.q + j * L.qs;
    float* Z = smem + L.z + j * L.zs;
    float* S = smem + L.s + j * L.ss;
    float* DQ = smem + L.dq + j * L.ds;
    int ti = types[a];
    // atoms >= n_owned are ghosts of a domain call: no energy, hence no adjoint
    const float own = a < n_owned ? 1.0f : 0.0f;
    // ---- invariants q_ang[L][n] (outputs dealt to the quad's lanes)
    for (int o = r; o < na * p.nL; o += 4) {
        int l = o / na, n = o - l * na;
        const float* sn = S + n * C;
        float v = 0.0f;
        for (int k = TPTR[l]; k < TPTR[l + 1]; ++k) {
            int4 tm = TERMS[k];
            unsigned f = (unsigned)tm.z;
            float x = __int_as_float(tm.x) * sn[f & 0xffu] * sn[(f >> 8) & 0xffu];
            unsigned i2 = (f >> 16) & 0xffu, i3 = f >> 24;
            if (i2 != kNoFactor) x *= sn[i2];
            if (i3 != kNoFactor) x *= sn[i3];
            v += x;
        }
        Q[nr + l * na + n] = v;
    }
    __syncwarp(qmask);
    // ---- element network
    for (int d = r; d < D; d += 4) Q[d] *= __ldg(head.scaler + d);
    __syncwarp(qmask);
    const float4* Q4 = reinterpret_cast<const float4*>(Q);
    const float4* w1 = reinterpret_cast<const float4*>(head.w1) + (size_t)ti * H * L.dp4;
    const float4* w1t = reinterpret_cast<const float4*>(head.w1t) + (size_t)ti * D * L.hp4;
    const float* b1 = head.b1 + (size_t)ti * H;
    const float* w2 = head.w2 + (size_t)ti * H;
    float e = 0.0f;
    for (int h = r; h < 4 * L.hp4; h += 4) {
        if (h >= H) {
            Z[h] = 0.0f;
            continue;
        }
        const float4* row = w1 + (size_t)h * L.dp4;
        float s0 = __ldg(b1 + h), s1 = 0.f, s2 = 0.f, s3 = 0.f;
        for (int d4 = 0; d4 < L.dp4; ++d4) {
            float4 w = __ldg(row + d4), q = Q4[d4];
            s0 += w.x * q.x; s1 += w.y * q.y; s2 += w.z * q.z; s3 += w.w * q.w;
        }
        float z = tanhf((s0 + s1) + (s2 + s3));
        float wv = own * __ldg(w2 + h);
        e += wv * z;
        Z[h] = wv * (1.0f - z * z);
    }
    e += __shfl_xor_sync(qmask, e, 1);
    e += __shfl_xor_sync(qmask, e, 2);
    if (r == 0) e_model[a] = own * (double)(e - head.bias);
    if (!w_t) return;  // energy only
    __syncwarp(qmask);
    const float4* Z4 = reinterpret_cast<const float4*>(Z);
    for (int d = r; d < D; d += 4) {
        const float4* col = w1t + (size_t)d * L.hp4;
        float g0 = 0.f, g1 = 0.f, g2 = 0.f, g3 = 0.f;
        for (int h4 = 0; h4 < L.hp4; ++h4) {
            float4 w = __ldg(col + h4), z = Z4[h4];
            g0 += w.x * z.x; g1 += w.y * z.y; g2 += w.z * z.z; g3 += w.w * z.w;
        }
        DQ[d] = ((g0 + g1) + (g2 + g3)) * __ldg(head.scaler + d);
    }
    __syncwarp(qmask);
    // ---- radial adjoint contracted with the c-table per neighbour type (when requested):
    //      G[a][t][k] = sum_n dq[n] c_r[t_a][t][n][k], rows of kr padded to 4
    if (gtab) {
        int kp = (p.kr + 3) & ~3;
        for (int o = r; o < p.T * kp; o += 4) {
            int t = o / kp, k = o - t * kp;
            float v = 0.0f;
            if (k < p.kr) {
                const float* cc = p.c_r + (size_t)(ti * p.T + t) * nr * p.kr + k;
                for (int n = 0; n < nr; ++n) v += DQ[n] * __ldg(cc + (size_t)n * p.kr);
            }
            gtab[((size_t)a * p.T + t) * kp + k] = v;
        }
    }
    // ---- adjoints: radial (padded float4 rows) and angular w[c][n] (tiled)
    for (int q = r; q < p.npr; q += 4) {
        int n = 4 * q;
        dqr[(size_t)a * p.npr + q] =
            make_float4(n < nr ? DQ[n] : 0.f, n + 1 < nr ? DQ[n + 1] : 0.f,
                        n + 2 < nr ? DQ[n + 2] : 0.f, n + 3 < nr ? DQ[n + 3] : 0.f);
    }
    // w[c][n]: each derivative term of harmonic c is decoded once and applied to up to eight
    // channels n (the same products, in the same order per output, as one output at a time)
    float* wb = w_t + (size_t)(a / kTile) * NC * kTile + (a % kTile);
    for (int c = r; c < C; c += 4) {
        for (int n0 = 0; n0 < na; n0 += 8) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = 0.0f;
            for (int k = DPTR[c]; k < DPTR[c + 1]; ++k) {
                int4 tm = DTERMS[k];
                unsigned f = (unsigned)tm.z;
                float coef = __int_as_float(tm.x);
                const float* dql = DQ + nr + tm.y * na;
                unsigned o0 = f & 0xffu, o1 = (f >> 8) & 0xffu, o2 = (f >> 16) & 0xffu;
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    int n = n0 + u;
                    if (n >= na) break;
                    const float* sn = S + n * C;
                    float x = coef * dql[n];
                    if (o0 != kNoFactor) x *= sn[o0];
                    if (o1 != kNoFactor) x *= sn[o1];
                    if (o2 != kNoFactor) x *= sn[o2];
                    v[u] += x;
                }
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                int n = n0 + u;
                if (n >= na) break;
                wb[(size_t)(c * na + n) * kTile] = v[u];
            }
        }
    }
}

// Centre-side angular edge gradients from the tiled angular adjoint (NEP), warp per atom;
// NA > 0: the angular channel count, fixed at compile time.
template <int NMAX, int LMAX, int NA>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
k_angular_grad(int n_atoms, DescParams p, EdgeList ang, const int* __restrict__ types,
               const float* __restrict__ w_t, float4* __restrict__ ang_grad, Stage st) {
    extern __shared__ float4 smem_f4[];
    float* smem = reinterpret_cast<float*>(smem_f4);
    stage_tables(p, st, smem);
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int i = blockIdx.x * kWarpsPerBlock + warp;
    float* sw = smem + warp * p.C * p.na;
    if (i >= n_atoms) return;
    const float* wb = w_t + (size_t)(i / kTile) * p.C * p.na * kTile + (i % kTile);
    for (int o = lane; o < p.C * p.na; o += 32) sw[o] = wb[(size_t)o * kTile];
    __syncwarp();
    angular_edge_grads<NMAX, LMAX, true, NA>(p, ang, types, i, types[i], sw, lane, ang_grad);
}

// Backward of the descriptor for Möbius: the radial adjoint (padded copy for the force kernel),
// the angular adjoint w from dq [N, D] and s [N, na, C] (+ the direct moment gradient
// mg [N, na, C] of the equivariant blocks, rune/mobius/force.py:200-201), then the centre-side
// angular edge gradients; warp per atom.
template <int NMAX, int LMAX>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
k_desc_backward(int n_atoms, DescParams p, EdgeList ang, const int* __restrict__ types,
                const float* __restrict__ dq, const float* __restrict__ s,
                const float* __restrict__ mg, float4* __restrict__ dqr,
                float4* __restrict__ ang_grad, Stage st) {
    extern __shared__ float4 smem_f4[];
    float* smem = reinterpret_cast<float*>(smem_f4);
    stage_tables(p, st, smem);
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int i = blockIdx.x * kWarpsPerBlock + warp;
    int cs = p.C | 1;
    int per = p.na * cs + p.na * p.C + p.D;
    float* ss = smem + warp * per;
    float* sw = ss + p.na * cs;
    float* sdq = sw + p.na * p.C;
    if (i >= n_atoms) return;
    for (int o = lane; o < p.na * p.C; o += 32) {
        int n = o / p.C, c = o - n * p.C;
        ss[n * cs + c] = s[(size_t)i * p.na * p.C + o];
    }
    for (int d = lane; d < p.D; d += 32) sdq[d] = dq[(size_t)i * p.D + d];
    __syncwarp();
    store_dqr(p, sdq, dqr, i, lane);
    invariant_adjoint(p, ss, cs, sdq + p.nr, mg ? mg + (size_t)i * p.na * p.C : nullptr, sw,
                      lane);
    __syncwarp();
    angular_edge_grads<NMAX, LMAX>(p, ang, types, i, types[i], sw, lane, ang_grad);
}

}  // namespace

// ----------------------------------------------------------------------------- ZBL
struct ZblParams {
    int mode;  // RUNE_ZBL_*
    double rc_inner, rc_outer;
    const float* zpow;   // [T] Z^0.23
    const float* z;      // [T] Z
    const float* coef;   // [4][2] universal
    const float* pairs;  // [T(T+1)/2][10] flexible
    int T;
};

// Screened pair energy (halved per directed edge) and its radial derivative, in float64
// (rune/mobius/zbl.py:92-141; rune/nep/zbl.py:102-163). Pairs at or beyond rc_outer return 0
// without evaluating the exponentials.
__device__ __forceinline__ void zbl_edge(const ZblParams& zp, int ti, int tj, double d,
                                         double& e, double& de) {
    e = 0.0;
    de = 0.0;
    d = fmax(d, 1.0e-12);
    double rin = zp.rc_inner, rout = zp.rc_outer;
    const float* cf = zp.coef;
    if (zp.mode == RUNE_ZBL_FLEXIBLE) {
        int lo = min(ti, tj), hi = max(ti, tj);
        int idx = lo * zp.T - lo * (lo - 1) / 2 + hi - lo;
        const float* pr = zp.pairs + (size_t)idx * 10;
        rin = __ldg(pr);
        rout = __ldg(pr + 1);
        cf = pr + 2;
    }
    if (d >= rout) return;
    double zi = __ldg(zp.z + ti), zj = __ldg(zp.z + tj);
    double a_inv = (pow(zi, 0.23) + pow(zj, 0.23)) * 2.134563;
    double pref = 14.399645 * zi * zj;
    double phi = 0.0, dphi = 0.0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        double c = __ldg(cf + 2 * k), a = __ldg(cf + 2 * k + 1);
        double ex = exp(-a * d * a_inv);
        phi += c * ex;
        dphi -= c * a * a_inv * ex;
    }
    double scr = pref * phi / d;
    double dscr = pref * (dphi / d - phi / (d * d));
    double width = fmax(rout - rin, 1.0e-12);
    double cut, dcut;
    if (d < rin) {
        cut = 1.0;
        dcut = 0.0;
    } else {
        const double pi = 3.14159265358979323846;
        double arg = pi * (d - rin) / width;
        cut = 0.5 * cos(arg) + 0.5;
        dcut = -0.5 * pi / width * sin(arg);
    }
    e = 0.5 * scr * cut;
    de = 0.5 * (dscr * cut + scr * dcut);
}

namespace {

struct ForceArgs {
    DescParams p;
    EdgeList rad, ang, zbl_list;
    const int* types;
    const float4* dqr;        // [N][npr] radial adjoint, zero padded
    const float* gtab;        // [N][T][gkp] radial adjoint contracted per neighbour type, or null
    int gkp;
    const float4* ang_grad;   // [angular edges] centre-side gradients; ang.rev pairs them
    ZblParams zbl;
    const float4* edge_grad;  // [E_radial] direct dE/dr on the radial list (messages), or null
    const double* positions64;  // float64 positions (device path) or null
    const int* sid;             // structure of each atom (device path)
    const StructGeom* geom;     // per-structure cells (device path)
    const int* shifts;          // packed image shift per edge (device path)
    double zbl_max_outer;       // largest ZBL outer cutoff
    int n_owned;                // atoms >= n_owned are ghosts of a domain call (no ZBL energy)
    bool descriptor;          // evaluate descriptor derivatives (false: ZBL energy only)
    double* e_zbl;            // [N]
    float* forces;            // [N, 3] or null
    double* virial_atom;      // [N, 9] (centre-attributed) or null
};

// Force and centre-attributed virial of every atom, warp per atom, lane per edge of its rows:
//   radial:  F_a += (sigma_a(e) + sigma_i(rev e)) u_e, both scalars evaluated here from the two
//            atoms' radial adjoints (sigma = sum_nk dq_n c_nk f'_k);
//   angular: F_a += G_e - G_rev(e) from the stored centre-side gradients;
//   messages (Möbius MP / EQ): the same pull over the radial list's edge gradients;
//   ZBL:     pair-symmetric, F_a += 2 g_e (in a domain call, (own(a) + own(j)) g_e with the
//            energy and virial of the pair's half counted at owned centres only).
// Virial: W -= g_e (x) r_e for the centre-side gradient of every edge of atom a.
// With the contracted radial adjoint (GTAB) the kernel fits 80 registers: six blocks per SM hide
// more of its gather latency; the channel-contraction form keeps 128 (four blocks).
template <int NMAX, bool ZBL, bool GTAB>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, GTAB ? 6 : 4)
k_forces(int n_atoms, ForceArgs A) {
    const DescParams& p = A.p;
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int a = blockIdx.x * kWarpsPerBlock + warp;
    if (a >= n_atoms) return;
    int ta = A.types[a];
    double F0 = 0.0, F1 = 0.0, F2 = 0.0, ez = 0.0;
    double W[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
    auto add_virial = [&](float g0, float g1, float g2, const float4& r) {
        // W_ab -= g_a r_b (rune/mobius/model.py:40)
        W[0] -= (double)g0 * r.x; W[1] -= (double)g0 * r.y; W[2] -= (double)g0 * r.z;
        W[3] -= (double)g1 * r.x; W[4] -= (double)g1 * r.y; W[5] -= (double)g1 * r.z;
        W[6] -= (double)g2 * r.x; W[7] -= (double)g2 * r.y; W[8] -= (double)g2 * r.z;
    };
    // With the contracted radial adjoint (the NEP form) a lane's few edges are summed in
    // float32 and the lane's partials enter the float64 warp sums once: the float64 form spends
    // the kernel's issue budget on conversions. The basis is evaluated in float32 as well.
    float f0 = 0.f, f1 = 0.f, f2 = 0.f;
    float w[9] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    auto add_lane = [&](float g0, float g1, float g2, const float4& r) {
        w[0] -= g0 * r.x; w[1] -= g0 * r.y; w[2] -= g0 * r.z;
        w[3] -= g1 * r.x; w[4] -= g1 * r.y; w[5] -= g1 * r.z;
        w[6] -= g2 * r.x; w[7] -= g2 * r.y; w[8] -= g2 * r.z;
    };

    if (A.descriptor) {
        float4 dqa[NMAX / 4];
#pragma unroll
        for (int q = 0; q < NMAX / 4; ++q)
            dqa[q] = !GTAB && q < p.npr ? __ldg(A.dqr + (size_t)a * p.npr + q)
                                         : make_float4(0, 0, 0, 0);
        // ---- radial descriptor
        int b = A.rad.row_ptr[a], cnt = A.rad.cnt[a];
        for (int k = lane; k < cnt; k += 32) {
            float4 e = A.rad.e[b + k];
            int i = edge_j(e);
            int ti = A.types[i];
            float r = edge_len<GTAB>(e);
            float inv = 1.0f / fmaxf(r, 1.0e-12f);
            float sa = 0.0f, si = 0.0f;
            if (GTAB) {
                const float* ga = A.gtab + ((size_t)a * p.T + ti) * A.gkp;
                const float* gi = A.gtab + ((size_t)i * p.T + ta) * A.gkp;
                basis_visit<true, true>(r, p.rc_r, p.kr, [&](int kk, float, float df) {
                    sa += __ldg(ga + kk) * df;
                    si += __ldg(gi + kk) * df;
                });
            } else {
            const float4* ca = p.c_rt + (size_t)(ta * p.T + ti) * p.kr * p.npr;
            const float4* ci = p.c_rt + (size_t)(ti * p.T + ta) * p.kr * p.npr;
            float4 dqi[NMAX / 4];
#pragma unroll
            for (int q = 0; q < NMAX / 4; ++q)
                dqi[q] = q < p.npr ? __ldg(A.dqr + (size_t)i * p.npr + q)
                                   : make_float4(0, 0, 0, 0);
            chebyshev_visit<true>(r, p.rc_r, p.kr, [&](int kk, float, float df) {
                float va = 0.0f, vi = 0.0f;
#pragma unroll
                for (int q = 0; q < NMAX / 4; ++q)
                    if (q < p.npr) {
                        float4 x = __ldg(ca + kk * p.npr + q), y = __ldg(ci + kk * p.npr + q);
                        va += dqa[q].x * x.x + dqa[q].y * x.y + dqa[q].z * x.z + dqa[q].w * x.w;
                        vi += dqi[q].x * y.x + dqi[q].y * y.y + dqi[q].z * y.z + dqi[q].w * y.w;
                    }
                sa += va * df;
                si += vi * df;
            });
            }
            float ux = e.x * inv, uy = e.y * inv, uz = e.z * inv;
            float st = sa + si;
            if (GTAB) {
                f0 += st * ux; f1 += st * uy; f2 += st * uz;
                add_lane(sa * ux, sa * uy, sa * uz, e);
            } else {
                F0 += (double)(st * ux); F1 += (double)(st * uy); F2 += (double)(st * uz);
                add_virial(sa * ux, sa * uy, sa * uz, e);
            }
        }
        // ---- angular descriptor: stored centre-side gradients, reverse edges gathered
        b = A.ang.row_ptr[a];
        cnt = A.ang.cnt[a];
        for (int k = lane; k < cnt; k += 32) {
            float4 e = A.ang.e[b + k];
            float4 g = A.ang_grad[b + k];
            float4 gr = A.ang_grad[A.ang.rev[b + k]];
            if (GTAB) {
                f0 += g.x - gr.x; f1 += g.y - gr.y; f2 += g.z - gr.z;
                add_lane(g.x, g.y, g.z, e);
            } else {
                F0 += (double)g.x - (double)gr.x;
                F1 += (double)g.y - (double)gr.y;
                F2 += (double)g.z - (double)gr.z;
                add_virial(g.x, g.y, g.z, e);
            }
        }
        if (GTAB) {
            F0 += (double)f0; F1 += (double)f1; F2 += (double)f2;
#pragma unroll
            for (int q = 0; q < 9; ++q) W[q] += (double)w[q];
        }
        // ---- direct edge gradients from message blocks (radial list, reverse index)
        if (A.edge_grad) {
            b = A.rad.row_ptr[a];
            cnt = A.rad.cnt[a];
            for (int k = lane; k < cnt; k += 32) {
                float4 e = A.rad.e[b + k];
                float4 g = A.edge_grad[b + k];
                float4 gr = A.edge_grad[A.rad.rev[b + k]];
                F0 += (double)g.x - (double)gr.x;
                F1 += (double)g.y - (double)gr.y;
                F2 += (double)g.z - (double)gr.z;
                add_virial(g.x, g.y, g.z, e);
            }
        }
    }
    // ---- ZBL (pair-symmetric: the reverse edge carries -g, so the pull adds 2 g). Close pairs
    // dominate and their energy is steep, so the pair vector is re-formed in float64 when the
    // caller's float64 positions are available.
    if (ZBL) {
        int b = A.zbl_list.row_ptr[a], cnt = A.zbl_list.cnt[a];
        const StructGeom* g = A.geom ? A.geom + A.sid[a] : nullptr;
        for (int k = lane; k < cnt; k += 32) {
            float4 e = A.zbl_list.e[b + k];
            int i = edge_j(e);
            double x = e.x, y = e.y, z = e.z;
            double r = sqrt(x * x + y * y + z * z);
            if (r >= A.zbl_max_outer) continue;
            if (g) {
                int sh = A.shifts[b + k];
                int s0 = ((sh & 1023) ^ 512) - 512, s1 = (((sh >> 10) & 1023) ^ 512) - 512;
                int s2 = (((sh >> 20) & 1023) ^ 512) - 512;
                x = (A.positions64[3 * i] - A.positions64[3 * a]) +
                    (s0 * g->cell[0] + s1 * g->cell[3] + s2 * g->cell[6]);
                y = (A.positions64[3 * i + 1] - A.positions64[3 * a + 1]) +
                    (s0 * g->cell[1] + s1 * g->cell[4] + s2 * g->cell[7]);
                z = (A.positions64[3 * i + 2] - A.positions64[3 * a + 2]) +
                    (s0 * g->cell[2] + s1 * g->cell[5] + s2 * g->cell[8]);
                r = sqrt(x * x + y * y + z * z);
            }
            double own_a = a < A.n_owned ? 1.0 : 0.0;
            double wf = own_a + (i < A.n_owned ? 1.0 : 0.0);
            if (wf == 0.0) continue;
            double en, de;
            zbl_edge(A.zbl, ta, A.types[i], r, en, de);
            ez += own_a * en;
            if (A.descriptor) {
                double inv = 1.0 / fmax(r, 1.0e-12);
                double g0 = de * x * inv, g1 = de * y * inv, g2 = de * z * inv;
                F0 += wf * g0; F1 += wf * g1; F2 += wf * g2;
                g0 *= own_a; g1 *= own_a; g2 *= own_a;
                W[0] -= g0 * x; W[1] -= g0 * y; W[2] -= g0 * z;
                W[3] -= g1 * x; W[4] -= g1 * y; W[5] -= g1 * z;
                W[6] -= g2 * x; W[7] -= g2 * y; W[8] -= g2 * z;
            }
        }
    }
    F0 = warp_sum(F0); F1 = warp_sum(F1); F2 = warp_sum(F2);
    ez = warp_sum(ez);
#pragma unroll
    for (int k = 0; k < 9; ++k) W[k] = warp_sum(W[k]);
    if (lane == 0) {
        A.e_zbl[a] = ez;
        if (A.forces) {
            A.forces[3 * a] = (float)F0;
            A.forces[3 * a + 1] = (float)F1;
            A.forces[3 * a + 2] = (float)F2;
        }
        if (A.virial_atom)
            for (int k = 0; k < 9; ++k) A.virial_atom[(size_t)a * 9 + k] = W[k];
    }
}

}  // namespace

// ----------------------------------------------------------------------------- launchers
// Channel counts up to 64 are supported; the kernels keep per-channel sums in registers sized
// by the smallest of 8 / 16 / 32 / 64 that holds max(nr, na), and unroll the harmonics up to
// order 4 or 8.
int channel_bound(const DescParams& p) {
    int n = std::max(p.nr, p.na);
    return n <= 8 ? 8 : n <= 16 ? 16 : n <= 32 ? 32 : 64;
}

template <int N, int L>
struct Shape {
    static constexpr int nmax = N;
    static constexpr int lmax = L;
};

template <typename F>
static void dispatch_shape(const DescParams& p, F&& f) {
    bool small = p.lmax <= 4;
    switch (channel_bound(p)) {
        case 8: small ? f(Shape<8, 4>{}) : f(Shape<8, 8>{}); break;
        case 16: small ? f(Shape<16, 4>{}) : f(Shape<16, 8>{}); break;
        case 32: small ? f(Shape<32, 4>{}) : f(Shape<32, 8>{}); break;
        default: small ? f(Shape<64, 4>{}) : f(Shape<64, 8>{}); break;
    }
}

// Plans the staged c-tables behind `base_floats` of other dynamic shared memory: each table
// is staged when the whole request stays within 64 KB. Returns the total bytes.
static size_t plan_stage(const DescParams& p, size_t base_floats, bool radial, bool angular,
                         Stage& st) {
    size_t off = (base_floats + 3) & ~size_t(3);
    const size_t limit = 64 * 1024 / sizeof(float);
    if (radial && off + 4 * (size_t)c_table_float4s(p, true) <= limit) {
        st.r = (int)off;
        off += 4 * (size_t)c_table_float4s(p, true);
    }
    if (angular && off + 4 * (size_t)c_table_float4s(p, false) <= limit) {
        st.a = (int)off;
        off += 4 * (size_t)c_table_float4s(p, false);
    }
    return sizeof(float) * std::max(off, base_floats);
}

size_t forward_smem_bytes(const DescParams& p) {
    ForwardSmem L(p);
    return sizeof(float) * L.total * kWarpsPerBlock;
}

static void set_smem(const void* fn, size_t bytes) {
    if (bytes > 48 * 1024)
        RUNE_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)bytes));
}

size_t nep_tiled_floats(int n_atoms, int per_atom) {
    return (size_t)((n_atoms + kTile - 1) / kTile) * per_atom * kTile;
}

void launch_desc_forward(const DescParams& p, int n_atoms, const EdgeList& rad,
                         const EdgeList& ang, const int* types, float* q, float* s, bool tiled,
                         cudaStream_t stream) {
    if (n_atoms == 0) return;
    int blocks = (n_atoms + kWarpsPerBlock - 1) / kWarpsPerBlock;
    Stage st;
    size_t bytes = plan_stage(p, forward_smem_bytes(p) / sizeof(float), true, true, st);
    dispatch_shape(p, [&](auto shape) {
        constexpr int NM = decltype(shape)::nmax, LM = decltype(shape)::lmax;
        if (tiled) {
            set_smem((const void*)k_desc_forward<true, NM, LM>, bytes);
            RUNE_KERNEL("k_desc_forward", stream,
                        k_desc_forward<true, NM, LM>
                        <<<blocks, kWarpsPerBlock * 32, bytes, stream>>>(n_atoms, p, rad, ang,
                                                                          types, q, s, st));
        } else {
            set_smem((const void*)k_desc_forward<false, NM, LM>, bytes);
            RUNE_KERNEL("k_desc_forward", stream,
                        k_desc_forward<false, NM, LM>
                        <<<blocks, kWarpsPerBlock * 32, bytes, stream>>>(n_atoms, p, rad, ang,
                                                                          types, q, s, st));
        }
    });
    RUNE_LAUNCH_CHECK();
}

void launch_nep_atoms(const DescParams& p, int n_atoms, int n_owned, const NepHeadArgs& nep,
                      const int* types, const float* qr_t, const float* s_t, double* e_model,
                      float4* dqr, float* w_t, float* gtab, cudaStream_t stream) {
    if (n_atoms == 0) return;
    NepHead h{nep.H, nep.w1, nep.w1t, nep.b1, nep.w2, nep.scaler, nep.bias};
    size_t bytes = sizeof(float) * NepAtomSmem(p, nep.H).total;
    set_smem((const void*)k_nep_atoms, bytes);
    int blocks = (n_atoms + kQuadAtoms - 1) / kQuadAtoms;
    RUNE_KERNEL("k_nep_atoms", stream,
                k_nep_atoms<<<blocks, 4 * kQuadAtoms, bytes, stream>>>(
                    n_atoms, n_owned, p, h, types, qr_t, s_t, e_model, dqr, w_t, gtab));
    RUNE_LAUNCH_CHECK();
}

void launch_angular_grad(const DescParams& p, int n_atoms, const EdgeList& ang,
                         const int* types, const float* w_t, float4* ang_grad,
                         cudaStream_t stream) {
    if (n_atoms == 0) return;
    int blocks = (n_atoms + kWarpsPerBlock - 1) / kWarpsPerBlock;
    Stage st;
    size_t bytes = plan_stage(p, (size_t)p.C * p.na * kWarpsPerBlock, false, true, st);
    auto launch = [&](auto kernel) {
        set_smem((const void*)kernel, bytes);
        RUNE_KERNEL("k_angular_grad", stream,
                    kernel<<<blocks, kWarpsPerBlock * 32, bytes, stream>>>(n_atoms, p, ang, types,
                                                                           w_t, ang_grad, st));
    };
    if (channel_bound(p) == 8 && p.lmax <= 4) {
        // the usual NEP shapes: exact angular channel counts
        switch (p.na) {
            case 4: launch(k_angular_grad<8, 4, 4>); break;
            case 5: launch(k_angular_grad<8, 4, 5>); break;
            case 6: launch(k_angular_grad<8, 4, 6>); break;
            case 8: launch(k_angular_grad<8, 4, 8>); break;
            default: launch(k_angular_grad<8, 4, 0>); break;
        }
    } else {
        dispatch_shape(p, [&](auto shape) {
            constexpr int NM = decltype(shape)::nmax, LM = decltype(shape)::lmax;
            launch(k_angular_grad<NM, LM, 0>);
        });
    }
    RUNE_LAUNCH_CHECK();
}

void launch_desc_backward(const DescParams& p, int n_atoms, const EdgeList& ang,
                          const int* types, const float* dq, const float* s, const float* mg,
                          float4* dqr, float4* ang_grad, cudaStream_t stream) {
    if (n_atoms == 0) return;
    int blocks = (n_atoms + kWarpsPerBlock - 1) / kWarpsPerBlock;
    Stage st;
    size_t bytes = plan_stage(p, (size_t)(p.na * (p.C | 1) + p.na * p.C + p.D) * kWarpsPerBlock,
                              false, true, st);
    dispatch_shape(p, [&](auto shape) {
        constexpr int NM = decltype(shape)::nmax, LM = decltype(shape)::lmax;
        set_smem((const void*)k_desc_backward<NM, LM>, bytes);
        RUNE_KERNEL("k_desc_backward", stream,
                    k_desc_backward<NM, LM><<<blocks, kWarpsPerBlock * 32, bytes, stream>>>(
                        n_atoms, p, ang, types, dq, s, mg, dqr, ang_grad, st));
    });
    RUNE_LAUNCH_CHECK();
}

void launch_forces(const ForceLaunch& f, cudaStream_t stream) {
    if (f.n_atoms == 0) return;
    ForceArgs A;
    A.p = f.p;
    A.rad = f.rad;
    A.ang = f.ang;
    A.zbl_list = f.zbl_list;
    A.types = f.types;
    A.dqr = f.dqr;
    A.gtab = f.gtab;
    A.gkp = f.gkp;
    A.ang_grad = f.ang_grad;
    A.zbl = ZblParams{f.zbl_mode, f.zbl_rc_inner, f.zbl_rc_outer, f.zbl_zpow, f.zbl_z,
                      f.zbl_coef, f.zbl_pairs, f.p.T};
    A.edge_grad = f.edge_grad;
    A.positions64 = f.positions64;
    A.sid = f.sid;
    A.geom = f.geom;
    A.shifts = f.shifts;
    A.zbl_max_outer = f.zbl_max_outer;
    A.n_owned = f.n_owned;
    A.descriptor = f.descriptor;
    A.e_zbl = f.e_zbl;
    A.forces = f.forces;
    A.virial_atom = f.virial_atom;
    int blocks = (f.n_atoms + kWarpsPerBlock - 1) / kWarpsPerBlock;
    bool zbl = f.zbl_mode != RUNE_ZBL_NONE;
    auto launch = [&](auto nm) {
        constexpr int NM = decltype(nm)::value;
        auto go = [&](auto kernel) {
            RUNE_KERNEL("k_forces", stream,
                        kernel<<<blocks, kWarpsPerBlock * 32, 0, stream>>>(f.n_atoms, A));
        };
        if (f.gtab)
            zbl ? go(k_forces<NM, true, true>) : go(k_forces<NM, false, true>);
        else
            zbl ? go(k_forces<NM, true, false>) : go(k_forces<NM, false, false>);
    };
    switch (channel_bound(f.p)) {
        case 8: launch(std::integral_constant<int, 8>{}); break;
        case 16: launch(std::integral_constant<int, 16>{}); break;
        case 32: launch(std::integral_constant<int, 32>{}); break;
        default: launch(std::integral_constant<int, 64>{}); break;
    }
    RUNE_LAUNCH_CHECK();
}

}  // namespace rune
