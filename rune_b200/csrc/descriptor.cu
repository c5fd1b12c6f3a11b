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

// q_ang[L][n] of one atom from its moments s[n][c], lanes over (n, L); the terms of output L
// are term_ptr[L] .. term_ptr[L + 1] of the monomial table.
__device__ __forceinline__ void invariants(const DescParams& p, const float* sacc, float* qang,
                                           int lane) {
    for (int o = lane; o < p.na * p.nL; o += 32) {
        int n = o / p.nL, L = o - n * p.nL;
        const float* sn = sacc + n * p.C;
        int t0 = (int)__ldg(p.term_ptr + L), t1 = (int)__ldg(p.term_ptr + L + 1);
        float v = 0.0f;
        for (int k = t0; k < t1; ++k) {
            const float* t = p.terms + 6 * k;
            float x = __ldg(t) * sn[(int)__ldg(t + 2)] * sn[(int)__ldg(t + 3)];
            int i2 = (int)__ldg(t + 4), i3 = (int)__ldg(t + 5);
            if (i2 >= 0) x *= sn[i2];
            if (i3 >= 0) x *= sn[i3];
            v += x;
        }
        qang[L * p.na + n] = v;
    }
}

// Angular adjoint w[c][n] = mg[n][c] + sum_L dq[L][n] d q_L[n] / d s[n][c], lanes over (n, c):
// the product rule applied through the derivative table, whose entries for harmonic c hold
// (coef, L, the other factors) of every occurrence of c in a term (rune/mobius/force.py:28-133).
__device__ __forceinline__ void invariant_adjoint(const DescParams& p, const float* sacc,
                                                  const float* dqang /* [L][na] */,
                                                  const float* mg /* [na][C] or null */,
                                                  float* w /* [C][na] */, int lane) {
    for (int o = lane; o < p.na * p.C; o += 32) {
        int n = o / p.C, c = o - n * p.C;
        const float* sn = sacc + n * p.C;
        float v = mg ? mg[o] : 0.0f;
        int d0 = (int)__ldg(p.dterm_ptr + c), d1 = (int)__ldg(p.dterm_ptr + c + 1);
        for (int k = d0; k < d1; ++k) {
            const float* t = p.dterms + 6 * k;
            float x = __ldg(t) * dqang[(int)__ldg(t + 1) * p.na + n];
            int o0 = (int)__ldg(t + 2), o1 = (int)__ldg(t + 3), o2 = (int)__ldg(t + 4);
            if (o0 >= 0) x *= sn[o0];
            if (o1 >= 0) x *= sn[o1];
            if (o2 >= 0) x *= sn[o2];
            v += x;
        }
        w[c * p.na + n] = v;
    }
}

// Centre-side gradient dE/dr_e of every angular edge of atom a (rune/mobius/force.py:195-241):
//   g_e = rs u + (dir - (dir . u) u) / r,   rs = sum_nc w[c][n] g'_n Y_c,
//   dir = sum_c (sum_n w[c][n] g_n) grad Y_c
// with the adjoint w [C][na] of atom a in shared memory; lane per edge, g_n and g'_n in
// registers (NMAX >= na).
template <int NMAX, int LMAX>
__device__ __forceinline__ void angular_edge_grads(const DescParams& p, const EdgeList& ang,
                                                   const int* __restrict__ types, int a, int ta,
                                                   const float* sw, int lane,
                                                   float4* __restrict__ grad) {
    int b = ang.row_ptr[a], cnt = ang.cnt[a];
    for (int k = lane; k < cnt; k += 32) {
        float4 e = ang.e[b + k];
        float r = (float)sqrt((double)e.x * e.x + (double)e.y * e.y + (double)e.z * e.z);
        float inv = 1.0f / fmaxf(r, 1.0e-12f);
        float ux = e.x * inv, uy = e.y * inv, uz = e.z * inv;
        const float* crow = p.c_a + (size_t)(ta * p.T + types[edge_j(e)]) * p.na * p.ka;
        float g[NMAX], gp[NMAX];
#pragma unroll
        for (int n = 0; n < NMAX; ++n) g[n] = gp[n] = 0.0f;
        chebyshev_visit<true>(r, p.rc_a, p.ka, [&](int kk, float f, float df) {
#pragma unroll
            for (int n = 0; n < NMAX; ++n)
                if (n < p.na) {
                    float cv = __ldg(crow + n * p.ka + kk);
                    g[n] += cv * f;
                    gp[n] += cv * df;
                }
        });
        float rs = 0.f, d0 = 0.f, d1 = 0.f, d2 = 0.f;
        angular_components<true, LMAX>(ux, uy, uz, p.lmax, p.zc,
                                       [&](int c, int, float Y, float dx, float dy, float dz) {
            const float* wc = sw + c * p.na;
            float a1 = 0.f, a2 = 0.f;
#pragma unroll
            for (int n = 0; n < NMAX; ++n)
                if (n < p.na) {
                    a1 += wc[n] * gp[n];
                    a2 += wc[n] * g[n];
                }
            rs += Y * a1;
            d0 += a2 * dx; d1 += a2 * dy; d2 += a2 * dz;
        });
        float pu = d0 * ux + d1 * uy + d2 * uz;
        grad[b + k] = make_float4(rs * ux + (d0 - pu * ux) * inv, rs * uy + (d1 - pu * uy) * inv,
                                  rs * uz + (d2 - pu * uz) * inv, 0.0f);
    }
}

struct ForwardSmem {
    // per-warp float offsets; per-lane rows padded to an odd stride (no bank conflicts)
    int ys, gs, sy, sg, sacc, sq, sz, sw, total;
    __host__ __device__ ForwardSmem(const DescParams& p, int nep_hidden) {
        ys = p.C | 1;
        gs = p.na | 1;
        sy = 0;
        sg = sy + 32 * ys;
        sacc = sg + 32 * gs;
        sq = sacc + p.na * p.C;
        sz = sq + 2 * p.D;              // q and dq
        sw = sz + (nep_hidden > 0 ? nep_hidden : 0);
        total = sw + (nep_hidden > 0 ? p.na * p.C : 0);
        total = (total + 3) & ~3;
    }
};

struct NepHead {
    int H;
    const float* w1;      // [T][H][D]
    const float* b1;      // [T][H]
    const float* w2;      // [T][H]
    const float* scaler;  // [D]
    float bias;
};

// Descriptor forward, warp per atom. Writes q [N, D] and s [N, na, C]. With NEP, also runs the
// element network (rune/nep/model.py:157-170) and writes the energy, dq_r and the centre-side
// angular edge gradients used by the force kernel.
template <bool NEP, int NMAX, int LMAX>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
k_desc_forward(int n_atoms, DescParams p, EdgeList rad, EdgeList ang,
               const int* __restrict__ types, float* __restrict__ q_out,
               float* __restrict__ s_out, NepHead head, double* __restrict__ e_model,
               float* __restrict__ dq_out, float4* __restrict__ ang_grad) {
    extern __shared__ float smem[];
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int i = blockIdx.x * kWarpsPerBlock + warp;
    ForwardSmem L(p, NEP ? head.H : 0);
    float* sm = smem + warp * L.total;
    float* sy = sm + L.sy;
    float* sg = sm + L.sg;
    float* sacc = sm + L.sacc;
    float* sq = sm + L.sq;
    float* sdq = sq + p.D;
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
            float r = (float)sqrt((double)e.x * e.x + (double)e.y * e.y + (double)e.z * e.z);
            const float* crow = p.c_r + (size_t)(ti * p.T + types[edge_j(e)]) * p.nr * p.kr;
            chebyshev_visit<false>(r, p.rc_r, p.kr, [&](int kk, float f, float) {
#pragma unroll
                for (int n = 0; n < NMAX; ++n)
                    if (n < p.nr) acc[n] += __ldg(crow + n * p.kr + kk) * f;
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
    for (int o = lane; o < p.na * p.C; o += 32) sacc[o] = 0.0f;
    {
        int b = ang.row_ptr[i], cnt = ang.cnt[i];
        for (int base = 0; base < cnt; base += 32) {
            int k = base + lane;
            if (k < cnt) {
                float4 e = ang.e[b + k];
                float r = (float)sqrt((double)e.x * e.x + (double)e.y * e.y + (double)e.z * e.z);
                float inv = 1.0f / fmaxf(r, 1.0e-12f);
                float* yrow = sy + lane * L.ys;
                angular_components<false, LMAX>(e.x * inv, e.y * inv, e.z * inv, p.lmax, p.zc,
                                                [&](int c, int, float Y, float, float, float) {
                                                    yrow[c] = Y;
                                                });
                const float* crow = p.c_a + (size_t)(ti * p.T + types[edge_j(e)]) * p.na * p.ka;
                float g[NMAX];
#pragma unroll
                for (int n = 0; n < NMAX; ++n) g[n] = 0.0f;
                chebyshev_visit<false>(r, p.rc_a, p.ka, [&](int kk, float f, float) {
#pragma unroll
                    for (int n = 0; n < NMAX; ++n)
                        if (n < p.na) g[n] += __ldg(crow + n * p.ka + kk) * f;
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
                float s = sacc[o];
                for (int ee = 0; ee < nv; ++ee) s += sg[ee * L.gs + n] * sy[ee * L.ys + c];
                sacc[o] = s;
            }
            __syncwarp();
        }
    }

    // ---- invariants and descriptor row
    invariants(p, sacc, sq + p.nr, lane);
    __syncwarp();
    if (q_out)
        for (int d = lane; d < p.D; d += 32) q_out[(size_t)i * p.D + d] = sq[d];
    if (s_out)
        for (int o = lane; o < p.na * p.C; o += 32) s_out[(size_t)i * p.na * p.C + o] = sacc[o];

    if constexpr (NEP) {
        // ---- element network: E = w2 . tanh(W1 (q * scaler) + b1) - bias
        float* sz = sm + L.sz;
        const float* w1 = head.w1 + (size_t)ti * head.H * p.D;
        const float* b1 = head.b1 + (size_t)ti * head.H;
        const float* w2 = head.w2 + (size_t)ti * head.H;
        for (int d = lane; d < p.D; d += 32) sdq[d] = sq[d] * __ldg(head.scaler + d);
        __syncwarp();
        float e = 0.0f;
        for (int h = lane; h < head.H; h += 32) {
            const float* row = w1 + (size_t)h * p.D;
            float a = __ldg(b1 + h);
            for (int d = 0; d < p.D; ++d) a += __ldg(row + d) * sdq[d];
            float z = tanhf(a);
            float wv = __ldg(w2 + h);
            e += wv * z;
            sz[h] = wv * (1.0f - z * z);
        }
        e = warp_sum(e);
        __syncwarp();
        for (int d = lane; d < p.D; d += 32) {
            float g = 0.0f;
            for (int h = 0; h < head.H; ++h) g += sz[h] * __ldg(w1 + (size_t)h * p.D + d);
            sdq[d] = g * __ldg(head.scaler + d);
        }
        __syncwarp();
        if (lane == 0) e_model[i] = (double)(e - head.bias);
        // ---- adjoints for the force kernel (when forces or virial are wanted): dq_r and the
        // angular edge gradients
        if (ang_grad) {
            for (int n = lane; n < p.nr; n += 32) dq_out[(size_t)i * p.D + n] = sdq[n];
            float* sw = sm + L.sw;  // [C][na]
            invariant_adjoint(p, sacc, sdq + p.nr, nullptr, sw, lane);
            __syncwarp();
            angular_edge_grads<NMAX, LMAX>(p, ang, types, i, ti, sw, lane, ang_grad);
        }
    }
}

// Backward of the descriptor for Möbius: the angular adjoint w from dq [N, D] and s [N, na, C]
// (+ the direct moment gradient mg [N, na, C] of the equivariant blocks,
// rune/mobius/force.py:200-201), then the centre-side angular edge gradients; warp per atom.
template <int NMAX, int LMAX>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
k_desc_backward(int n_atoms, DescParams p, EdgeList ang, const int* __restrict__ types,
                const float* __restrict__ dq, const float* __restrict__ s,
                const float* __restrict__ mg, float4* __restrict__ ang_grad) {
    extern __shared__ float smem[];
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int i = blockIdx.x * kWarpsPerBlock + warp;
    int per = 2 * p.na * p.C + p.D;
    float* ss = smem + warp * per;
    float* sw = ss + p.na * p.C;
    float* sdq = sw + p.na * p.C;
    if (i >= n_atoms) return;
    for (int o = lane; o < p.na * p.C; o += 32) ss[o] = s[(size_t)i * p.na * p.C + o];
    for (int d = lane; d < p.D; d += 32) sdq[d] = dq[(size_t)i * p.D + d];
    __syncwarp();
    invariant_adjoint(p, ss, sdq + p.nr, mg ? mg + (size_t)i * p.na * p.C : nullptr, sw, lane);
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
    const float* dq;  // [N, dq_stride]; first nr entries are the radial adjoint
    int dq_stride;
    const float4* ang_grad;   // [angular edges] centre-side gradients; ang.rev pairs them
    ZblParams zbl;
    const float4* edge_grad;  // [E_radial] direct dE/dr on the radial list (messages), or null
    const double* positions64;  // float64 positions (device path) or null
    const int* sid;             // structure of each atom (device path)
    const StructGeom* geom;     // per-structure cells (device path)
    const int* shifts;          // packed image shift per edge (device path)
    double zbl_max_outer;       // largest ZBL outer cutoff
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
//   ZBL:     pair-symmetric, F_a += 2 g_e.
// Virial: W -= g_e (x) r_e for the centre-side gradient of every edge of atom a.
template <int NMAX, bool ZBL>
__global__ void __launch_bounds__(kWarpsPerBlock * 32, 4) k_forces(int n_atoms, ForceArgs A) {
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

    if (A.descriptor) {
        float dqa[NMAX];
#pragma unroll
        for (int n = 0; n < NMAX; ++n)
            dqa[n] = n < p.nr ? __ldg(A.dq + (size_t)a * A.dq_stride + n) : 0.0f;
        // ---- radial descriptor
        int b = A.rad.row_ptr[a], cnt = A.rad.cnt[a];
        for (int k = lane; k < cnt; k += 32) {
            float4 e = A.rad.e[b + k];
            int i = edge_j(e);
            int ti = A.types[i];
            float r = (float)sqrt((double)e.x * e.x + (double)e.y * e.y + (double)e.z * e.z);
            float inv = 1.0f / fmaxf(r, 1.0e-12f);
            const float* ca = p.c_r + (size_t)(ta * p.T + ti) * p.nr * p.kr;
            const float* ci = p.c_r + (size_t)(ti * p.T + ta) * p.nr * p.kr;
            float dqi[NMAX];
#pragma unroll
            for (int n = 0; n < NMAX; ++n)
                dqi[n] = n < p.nr ? __ldg(A.dq + (size_t)i * A.dq_stride + n) : 0.0f;
            float sa = 0.0f, si = 0.0f;
            chebyshev_visit<true>(r, p.rc_r, p.kr, [&](int kk, float, float df) {
                float va = 0.0f, vi = 0.0f;
#pragma unroll
                for (int n = 0; n < NMAX; ++n)
                    if (n < p.nr) {
                        va += dqa[n] * __ldg(ca + n * p.kr + kk);
                        vi += dqi[n] * __ldg(ci + n * p.kr + kk);
                    }
                sa += va * df;
                si += vi * df;
            });
            float ux = e.x * inv, uy = e.y * inv, uz = e.z * inv;
            float st = sa + si;
            F0 += (double)(st * ux); F1 += (double)(st * uy); F2 += (double)(st * uz);
            add_virial(sa * ux, sa * uy, sa * uz, e);
        }
        // ---- angular descriptor: stored centre-side gradients, reverse edges gathered
        b = A.ang.row_ptr[a];
        cnt = A.ang.cnt[a];
        for (int k = lane; k < cnt; k += 32) {
            float4 e = A.ang.e[b + k];
            float4 g = A.ang_grad[b + k];
            float4 gr = A.ang_grad[A.ang.rev[b + k]];
            F0 += (double)g.x - (double)gr.x;
            F1 += (double)g.y - (double)gr.y;
            F2 += (double)g.z - (double)gr.z;
            add_virial(g.x, g.y, g.z, e);
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
            double en, de;
            zbl_edge(A.zbl, ta, A.types[i], r, en, de);
            ez += en;
            if (A.descriptor) {
                double inv = 1.0 / fmax(r, 1.0e-12);
                double g0 = de * x * inv, g1 = de * y * inv, g2 = de * z * inv;
                F0 += 2.0 * g0; F1 += 2.0 * g1; F2 += 2.0 * g2;
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
// Channel counts up to 32 are supported; the kernels keep per-channel sums in registers sized
// by the smallest of 8 / 16 / 32 that holds max(nr, na), and unroll the harmonics up to order
// 4 or 8.
int channel_bound(const DescParams& p) {
    int n = std::max(p.nr, p.na);
    return n <= 8 ? 8 : n <= 16 ? 16 : 32;
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
        default: small ? f(Shape<32, 4>{}) : f(Shape<32, 8>{}); break;
    }
}

size_t forward_smem_bytes(const DescParams& p, int nep_hidden) {
    ForwardSmem L(p, nep_hidden);
    return sizeof(float) * L.total * kWarpsPerBlock;
}

static void set_smem(const void* fn, size_t bytes) {
    if (bytes > 48 * 1024)
        RUNE_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)bytes));
}

void launch_desc_forward(const DescParams& p, int n_atoms, const EdgeList& rad,
                         const EdgeList& ang, const int* types, float* q, float* s,
                         const NepHeadArgs* nep, double* e_model, float* dq, float4* ang_grad,
                         cudaStream_t stream) {
    if (n_atoms == 0) return;
    int blocks = (n_atoms + kWarpsPerBlock - 1) / kWarpsPerBlock;
    size_t bytes = forward_smem_bytes(p, nep ? nep->H : 0);
    dispatch_shape(p, [&](auto shape) {
        constexpr int NM = decltype(shape)::nmax, LM = decltype(shape)::lmax;
        if (nep) {
            NepHead h{nep->H, nep->w1, nep->b1, nep->w2, nep->scaler, nep->bias};
            set_smem((const void*)k_desc_forward<true, NM, LM>, bytes);
            RUNE_KERNEL("k_desc_forward", stream,
                        k_desc_forward<true, NM, LM>
                        <<<blocks, kWarpsPerBlock * 32, bytes, stream>>>(
                            n_atoms, p, rad, ang, types, q, s, h, e_model, dq, ang_grad));
        } else {
            NepHead h{0, nullptr, nullptr, nullptr, nullptr, 0.f};
            set_smem((const void*)k_desc_forward<false, NM, LM>, bytes);
            RUNE_KERNEL("k_desc_forward", stream,
                        k_desc_forward<false, NM, LM>
                        <<<blocks, kWarpsPerBlock * 32, bytes, stream>>>(
                            n_atoms, p, rad, ang, types, q, s, h, nullptr, nullptr, nullptr));
        }
    });
    RUNE_LAUNCH_CHECK();
}

void launch_desc_backward(const DescParams& p, int n_atoms, const EdgeList& ang,
                          const int* types, const float* dq, const float* s, const float* mg,
                          float4* ang_grad, cudaStream_t stream) {
    if (n_atoms == 0) return;
    int blocks = (n_atoms + kWarpsPerBlock - 1) / kWarpsPerBlock;
    size_t bytes = sizeof(float) * (2 * p.na * p.C + p.D) * kWarpsPerBlock;
    dispatch_shape(p, [&](auto shape) {
        constexpr int NM = decltype(shape)::nmax, LM = decltype(shape)::lmax;
        set_smem((const void*)k_desc_backward<NM, LM>, bytes);
        RUNE_KERNEL("k_desc_backward", stream,
                    k_desc_backward<NM, LM><<<blocks, kWarpsPerBlock * 32, bytes, stream>>>(
                        n_atoms, p, ang, types, dq, s, mg, ang_grad));
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
    A.dq = f.dq;
    A.dq_stride = f.dq_stride;
    A.ang_grad = f.ang_grad;
    A.zbl = ZblParams{f.zbl_mode, f.zbl_rc_inner, f.zbl_rc_outer, f.zbl_zpow, f.zbl_z,
                      f.zbl_coef, f.zbl_pairs, f.p.T};
    A.edge_grad = f.edge_grad;
    A.positions64 = f.positions64;
    A.sid = f.sid;
    A.geom = f.geom;
    A.shifts = f.shifts;
    A.zbl_max_outer = f.zbl_max_outer;
    A.descriptor = f.descriptor;
    A.e_zbl = f.e_zbl;
    A.forces = f.forces;
    A.virial_atom = f.virial_atom;
    int blocks = (f.n_atoms + kWarpsPerBlock - 1) / kWarpsPerBlock;
    bool zbl = f.zbl_mode != RUNE_ZBL_NONE;
    auto launch = [&](auto nm) {
        constexpr int NM = decltype(nm)::value;
        if (zbl)
            RUNE_KERNEL("k_forces", stream,
                        k_forces<NM, true><<<blocks, kWarpsPerBlock * 32, 0, stream>>>(
                            f.n_atoms, A));
        else
            RUNE_KERNEL("k_forces", stream,
                        k_forces<NM, false><<<blocks, kWarpsPerBlock * 32, 0, stream>>>(
                            f.n_atoms, A));
    };
    switch (channel_bound(f.p)) {
        case 8: launch(std::integral_constant<int, 8>{}); break;
        case 16: launch(std::integral_constant<int, 16>{}); break;
        default: launch(std::integral_constant<int, 32>{}); break;
    }
    RUNE_LAUNCH_CHECK();
}

}  // namespace rune
