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

#include "basis.cuh"
#include "engine.cuh"

namespace rune {

namespace {

constexpr int kWarpsPerBlock = 4;

struct Term {
    float coef;
    int L;
    int i0, i1, i2, i3;
};

__device__ __forceinline__ Term load_term(const float* __restrict__ t, int k) {
    Term r;
    r.coef = __ldg(t + 6 * k);
    r.L = (int)__ldg(t + 6 * k + 1);
    r.i0 = (int)__ldg(t + 6 * k + 2);
    r.i1 = (int)__ldg(t + 6 * k + 3);
    r.i2 = (int)__ldg(t + 6 * k + 4);
    r.i3 = (int)__ldg(t + 6 * k + 5);
    return r;
}

// q_ang[n][L] of one channel n from its moments sn[c] (stride 1), written into q (+= form).
__device__ __forceinline__ void invariants_channel(const DescParams& p, const float* sn,
                                                   float* qout /* [nL] stride qstride */,
                                                   int qstride) {
    for (int k = 0; k < p.n_terms; ++k) {
        Term t = load_term(p.terms, k);
        float v = t.coef * sn[t.i0] * sn[t.i1];
        if (t.i2 >= 0) v *= sn[t.i2];
        if (t.i3 >= 0) v *= sn[t.i3];
        qout[t.L * qstride] += v;
    }
}

// w[c * na + n] += sum_L dq[L] d q_L / d s_c for one channel n (product rule over the term
// table; rune/mobius/force.py:28-133).
__device__ __forceinline__ void invariant_adjoint_channel(const DescParams& p, const float* sn,
                                                          const float* dqn /* stride na */,
                                                          float* w, int n) {
    for (int k = 0; k < p.n_terms; ++k) {
        Term t = load_term(p.terms, k);
        float g = dqn[t.L * p.na] * t.coef;
        int idx[4] = {t.i0, t.i1, t.i2, t.i3};
        float v[4] = {sn[t.i0], sn[t.i1], t.i2 >= 0 ? sn[t.i2] : 1.0f,
                      t.i3 >= 0 ? sn[t.i3] : 1.0f};
#pragma unroll
        for (int f = 0; f < 4; ++f) {
            if (idx[f] < 0) continue;
            float prod = g;
#pragma unroll
            for (int o = 0; o < 4; ++o)
                if (o != f) prod *= v[o];
            w[idx[f] * p.na + n] += prod;
        }
    }
}

struct ForwardSmem {
    // per-warp float offsets
    int sf, sy, sg, stj, sacc, sq, sz, sw, total;
    __host__ __device__ ForwardSmem(const DescParams& p, int nep_hidden) {
        int kmax = p.kr > p.ka ? p.kr : p.ka;
        sf = 0;
        sy = sf + 32 * kmax;
        sg = sy + 32 * p.C;
        stj = sg + 32 * p.na;
        sacc = stj + 32;
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
// element network (rune/nep/model.py:157-170) and writes the energy, dq_r and the angular
// adjoint w [N, C, na] used by the force kernel.
template <bool NEP>
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
k_desc_forward(int n_atoms, DescParams p, EdgeList rad, EdgeList ang,
               const int* __restrict__ types, float* __restrict__ q_out,
               float* __restrict__ s_out, NepHead head, double* __restrict__ e_model,
               float* __restrict__ dq_out, float* __restrict__ w_out) {
    extern __shared__ float smem[];
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int i = blockIdx.x * kWarpsPerBlock + warp;
    ForwardSmem L(p, NEP ? head.H : 0);
    float* sm = smem + warp * L.total;
    float* sf = sm + L.sf;
    float* sy = sm + L.sy;
    float* sg = sm + L.sg;
    int* stj = reinterpret_cast<int*>(sm + L.stj);
    float* sacc = sm + L.sacc;
    float* sq = sm + L.sq;
    float* sdq = sq + p.D;
    if (i >= n_atoms) return;
    int ti = types[i];

    // ---- radial channels: q_r[n]
    float acc0 = 0.0f, acc1 = 0.0f;
    {
        int b = rad.row_ptr[i], cnt = rad.cnt[i];
        for (int base = 0; base < cnt; base += 32) {
            int k = base + lane;
            if (k < cnt) {
                float4 e = rad.e[b + k];
                float r = (float)sqrt((double)e.x * e.x + (double)e.y * e.y + (double)e.z * e.z);
                chebyshev(r, p.rc_r, p.kr, sf + lane * p.kr, nullptr);
                stj[lane] = types[edge_j(e)];
            }
            __syncwarp();
            int nv = min(32, cnt - base);
            for (int ee = 0; ee < nv; ++ee) {
                const float* crow = p.c_r + (size_t)(ti * p.T + stj[ee]) * p.nr * p.kr;
                const float* fe = sf + ee * p.kr;
                if (lane < p.nr) {
                    const float* cr = crow + lane * p.kr;
                    float s = 0.0f;
                    for (int kk = 0; kk < p.kr; ++kk) s += __ldg(cr + kk) * fe[kk];
                    acc0 += s;
                }
                if (lane + 32 < p.nr) {
                    const float* cr = crow + (lane + 32) * p.kr;
                    float s = 0.0f;
                    for (int kk = 0; kk < p.kr; ++kk) s += __ldg(cr + kk) * fe[kk];
                    acc1 += s;
                }
            }
            __syncwarp();
        }
    }

    // ---- angular moments s[n][c]
    for (int o = lane; o < p.na * p.C; o += 32) sacc[o] = 0.0f;
    {
        int b = ang.row_ptr[i], cnt = ang.cnt[i];
        for (int base = 0; base < cnt; base += 32) {
            int k = base + lane;
            if (k < cnt) {
                float4 e = ang.e[b + k];
                float r = (float)sqrt((double)e.x * e.x + (double)e.y * e.y + (double)e.z * e.z);
                float inv = 1.0f / fmaxf(r, 1.0e-12f);
                chebyshev(r, p.rc_a, p.ka, sf + lane * p.ka, nullptr);
                float* yrow = sy + lane * p.C;
                angular_components<false>(e.x * inv, e.y * inv, e.z * inv, p.lmax, p.zc,
                                          [&](int c, int, float Y, float, float, float) {
                                              yrow[c] = Y;
                                          });
                stj[lane] = types[edge_j(e)];
            }
            __syncwarp();
            int nv = min(32, cnt - base);
            for (int o = lane; o < nv * p.na; o += 32) {
                int ee = o / p.na, n = o - ee * p.na;
                const float* cr = p.c_a + ((size_t)(ti * p.T + stj[ee]) * p.na + n) * p.ka;
                const float* fe = sf + ee * p.ka;
                float s = 0.0f;
                for (int kk = 0; kk < p.ka; ++kk) s += __ldg(cr + kk) * fe[kk];
                sg[ee * p.na + n] = s;
            }
            __syncwarp();
            for (int o = lane; o < p.na * p.C; o += 32) {
                int n = o / p.C, c = o - n * p.C;
                float s = sacc[o];
                for (int ee = 0; ee < nv; ++ee) s += sg[ee * p.na + n] * sy[ee * p.C + c];
                sacc[o] = s;
            }
            __syncwarp();
        }
    }

    // ---- invariants and descriptor row
    for (int d = lane; d < p.D; d += 32) sq[d] = 0.0f;
    __syncwarp();
    if (lane < p.nr) sq[lane] = acc0;
    if (lane + 32 < p.nr) sq[lane + 32] = acc1;
    for (int n = lane; n < p.na; n += 32)
        invariants_channel(p, sacc + n * p.C, sq + p.nr + n, p.na);
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
        // ---- adjoints for the force kernel: dq_r and w[c][n]
        for (int n = lane; n < p.nr; n += 32) dq_out[(size_t)i * p.D + n] = sdq[n];
        float* sw = sm + L.sw;  // [C][na]
        for (int o = lane; o < p.na * p.C; o += 32) sw[o] = 0.0f;
        __syncwarp();
        for (int n = lane; n < p.na; n += 32)
            invariant_adjoint_channel(p, sacc + n * p.C, sdq + p.nr + n, sw, n);
        __syncwarp();
        for (int o = lane; o < p.na * p.C; o += 32) w_out[(size_t)i * p.na * p.C + o] = sw[o];
    }
}

// Angular adjoint w[i][c][n] from dq [N, D] and s [N, na, C] (+ optional direct moment
// gradient mg [N, na, C], rune/mobius/force.py:200-201), warp per atom.
__global__ void __launch_bounds__(kWarpsPerBlock * 32)
k_desc_weights(int n_atoms, DescParams p, const float* __restrict__ dq,
               const float* __restrict__ s, const float* __restrict__ mg,
               float* __restrict__ w_out) {
    extern __shared__ float smem[];
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int i = blockIdx.x * kWarpsPerBlock + warp;
    int per = 2 * p.na * p.C + p.D;
    float* ss = smem + warp * per;
    float* sw = ss + p.na * p.C;
    float* sdq = sw + p.na * p.C;
    if (i >= n_atoms) return;
    for (int o = lane; o < p.na * p.C; o += 32) {
        ss[o] = s[(size_t)i * p.na * p.C + o];
        int n = o / p.C, c = o - n * p.C;
        sw[c * p.na + n] = mg ? mg[(size_t)i * p.na * p.C + o] : 0.0f;
    }
    for (int d = lane; d < p.D; d += 32) sdq[d] = dq[(size_t)i * p.D + d];
    __syncwarp();
    for (int n = lane; n < p.na; n += 32)
        invariant_adjoint_channel(p, ss + n * p.C, sdq + p.nr + n, sw, n);
    __syncwarp();
    for (int o = lane; o < p.na * p.C; o += 32) w_out[(size_t)i * p.na * p.C + o] = sw[o];
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
    const float* w;   // [N, C, na]
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

__global__ void __launch_bounds__(kWarpsPerBlock * 32) k_forces(int n_atoms, ForceArgs A) {
    extern __shared__ float smem[];
    const DescParams& p = A.p;
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int a = blockIdx.x * kWarpsPerBlock + warp;
    int kmax = max(p.kr, p.ka);
    int per_lane = 2 * kmax + 4 * p.na;
    int per_warp = p.C * p.na + p.nr + 32 * per_lane;
    float* sm = smem + warp * per_warp;
    float* sw = sm;                     // [C][na] adjoint of atom a
    float* sdq = sw + p.C * p.na;       // [nr]
    float* lane_sm = sdq + p.nr + lane * per_lane;
    float* fk = lane_sm;                // [kmax]
    float* fpk = fk + kmax;             // [kmax]
    float* ga = fpk + kmax;             // [na] g_n (centre a)
    float* gpa = ga + p.na;             // [na] g'_n (centre a)
    float* gi = gpa + p.na;             // [na] g_n (centre i, reverse edge)
    float* gpi = gi + p.na;             // [na] g'_n (centre i)
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
        for (int o = lane; o < p.C * p.na; o += 32) sw[o] = A.w[(size_t)a * p.C * p.na + o];
        for (int n = lane; n < p.nr; n += 32) sdq[n] = A.dq[(size_t)a * A.dq_stride + n];
        __syncwarp();
        // ---- radial descriptor: F_a += (sigma_a + sigma_i) u, sigma = sum_nk dq c f'
        int b = A.rad.row_ptr[a], cnt = A.rad.cnt[a];
        for (int k = lane; k < cnt; k += 32) {
            float4 e = A.rad.e[b + k];
            int i = edge_j(e);
            int ti = A.types[i];
            float r = (float)sqrt((double)e.x * e.x + (double)e.y * e.y + (double)e.z * e.z);
            float inv = 1.0f / fmaxf(r, 1.0e-12f);
            chebyshev(r, p.rc_r, p.kr, fk, fpk);
            const float* ca = p.c_r + (size_t)(ta * p.T + ti) * p.nr * p.kr;
            const float* ci = p.c_r + (size_t)(ti * p.T + ta) * p.nr * p.kr;
            const float* dqi = A.dq + (size_t)i * A.dq_stride;
            float sa = 0.0f, si = 0.0f;
            for (int n = 0; n < p.nr; ++n) {
                float va = 0.0f, vi = 0.0f;
                const float* ra = ca + n * p.kr;
                const float* ri = ci + n * p.kr;
                for (int kk = 0; kk < p.kr; ++kk) {
                    va += __ldg(ra + kk) * fpk[kk];
                    vi += __ldg(ri + kk) * fpk[kk];
                }
                sa += sdq[n] * va;
                si += __ldg(dqi + n) * vi;
            }
            float ux = e.x * inv, uy = e.y * inv, uz = e.z * inv;
            float st = sa + si;
            F0 += (double)(st * ux); F1 += (double)(st * uy); F2 += (double)(st * uz);
            add_virial(sa * ux, sa * uy, sa * uz, e);
        }
        // ---- angular descriptor
        b = A.ang.row_ptr[a];
        cnt = A.ang.cnt[a];
        for (int k = lane; k < cnt; k += 32) {
            float4 e = A.ang.e[b + k];
            int i = edge_j(e);
            int ti = A.types[i];
            float r = (float)sqrt((double)e.x * e.x + (double)e.y * e.y + (double)e.z * e.z);
            float inv = 1.0f / fmaxf(r, 1.0e-12f);
            float ux = e.x * inv, uy = e.y * inv, uz = e.z * inv;
            chebyshev(r, p.rc_a, p.ka, fk, fpk);
            const float* ca = p.c_a + (size_t)(ta * p.T + ti) * p.na * p.ka;
            const float* ci = p.c_a + (size_t)(ti * p.T + ta) * p.na * p.ka;
            for (int n = 0; n < p.na; ++n) {
                float v0 = 0.f, v1 = 0.f, v2 = 0.f, v3 = 0.f;
                for (int kk = 0; kk < p.ka; ++kk) {
                    float xa = __ldg(ca + n * p.ka + kk), xi = __ldg(ci + n * p.ka + kk);
                    v0 += xa * fk[kk];
                    v1 += xa * fpk[kk];
                    v2 += xi * fk[kk];
                    v3 += xi * fpk[kk];
                }
                ga[n] = v0; gpa[n] = v1; gi[n] = v2; gpi[n] = v3;
            }
            const float* wi = A.w + (size_t)i * p.C * p.na;
            float rs_a = 0.f, rs_i = 0.f;
            float da0 = 0.f, da1 = 0.f, da2 = 0.f, di0 = 0.f, di1 = 0.f, di2 = 0.f;
            angular_components<true>(ux, uy, uz, p.lmax, p.zc,
                                     [&](int c, int L, float Y, float dx, float dy, float dz) {
                const float* wa = sw + c * p.na;
                const float* wic = wi + c * p.na;
                float a1 = 0.f, a2 = 0.f, b1 = 0.f, b2 = 0.f;
                for (int n = 0; n < p.na; ++n) {
                    float x = wa[n], y = __ldg(wic + n);
                    a1 += x * gpa[n];
                    a2 += x * ga[n];
                    b1 += y * gpi[n];
                    b2 += y * gi[n];
                }
                float par = (L & 1) ? -1.0f : 1.0f;  // Y_L(-u) = (-1)^L Y_L(u)
                rs_a += Y * a1;
                rs_i += par * Y * b1;
                da0 += a2 * dx; da1 += a2 * dy; da2 += a2 * dz;
                float nb2 = -par * b2;  // grad Y_L at -u = -(-1)^L grad Y_L(u)
                di0 += nb2 * dx; di1 += nb2 * dy; di2 += nb2 * dz;
            });
            float pa = da0 * ux + da1 * uy + da2 * uz;
            float pi = di0 * ux + di1 * uy + di2 * uz;
            // centre gradient (force.py:215-240) and reverse-edge gradient at r_rev = -r
            float gc0 = rs_a * ux + (da0 - pa * ux) * inv;
            float gc1 = rs_a * uy + (da1 - pa * uy) * inv;
            float gc2 = rs_a * uz + (da2 - pa * uz) * inv;
            float gr0 = -rs_i * ux + (di0 - pi * ux) * inv;
            float gr1 = -rs_i * uy + (di1 - pi * uy) * inv;
            float gr2 = -rs_i * uz + (di2 - pi * uz) * inv;
            F0 += (double)gc0 - (double)gr0;
            F1 += (double)gc1 - (double)gr1;
            F2 += (double)gc2 - (double)gr2;
            add_virial(gc0, gc1, gc2, e);
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
    if (A.zbl.mode != RUNE_ZBL_NONE) {
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
size_t forward_smem_bytes(const DescParams& p, int nep_hidden) {
    ForwardSmem L(p, nep_hidden);
    return sizeof(float) * L.total * kWarpsPerBlock;
}

void launch_desc_forward(const DescParams& p, int n_atoms, const EdgeList& rad,
                         const EdgeList& ang, const int* types, float* q, float* s,
                         const NepHeadArgs* nep, double* e_model, float* dq, float* w,
                         cudaStream_t stream) {
    if (n_atoms == 0) return;
    int blocks = (n_atoms + kWarpsPerBlock - 1) / kWarpsPerBlock;
    size_t bytes = forward_smem_bytes(p, nep ? nep->H : 0);
    if (nep) {
        NepHead h{nep->H, nep->w1, nep->b1, nep->w2, nep->scaler, nep->bias};
        if (bytes > 48 * 1024)
            RUNE_CUDA_TRY(cudaFuncSetAttribute(k_desc_forward<true>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)bytes));
        RUNE_KERNEL("k_desc_forward", stream, k_desc_forward<true><<<blocks, kWarpsPerBlock * 32, bytes, stream>>>(
            n_atoms, p, rad, ang, types, q, s, h, e_model, dq, w));
    } else {
        NepHead h{0, nullptr, nullptr, nullptr, nullptr, 0.f};
        if (bytes > 48 * 1024)
            RUNE_CUDA_TRY(cudaFuncSetAttribute(k_desc_forward<false>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)bytes));
        RUNE_KERNEL("k_desc_forward", stream, k_desc_forward<false><<<blocks, kWarpsPerBlock * 32, bytes, stream>>>(
            n_atoms, p, rad, ang, types, q, s, h, nullptr, nullptr, nullptr));
    }
    RUNE_LAUNCH_CHECK();
}

void launch_desc_weights(const DescParams& p, int n_atoms, const float* dq, const float* s,
                         const float* mg, float* w, cudaStream_t stream) {
    if (n_atoms == 0) return;
    int blocks = (n_atoms + kWarpsPerBlock - 1) / kWarpsPerBlock;
    size_t bytes = sizeof(float) * (2 * p.na * p.C + p.D) * kWarpsPerBlock;
    if (bytes > 48 * 1024)
        RUNE_CUDA_TRY(cudaFuncSetAttribute(k_desc_weights,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)bytes));
    RUNE_KERNEL("k_desc_weights", stream, k_desc_weights<<<blocks, kWarpsPerBlock * 32, bytes, stream>>>(n_atoms, p, dq, s, mg, w));
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
    A.w = f.w;
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
    int kmax = std::max(f.p.kr, f.p.ka);
    size_t per_warp = f.p.C * f.p.na + f.p.nr + 32 * (2 * kmax + 4 * f.p.na);
    size_t bytes = sizeof(float) * per_warp * kWarpsPerBlock;
    if (bytes > 48 * 1024)
        RUNE_CUDA_TRY(cudaFuncSetAttribute(k_forces, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)bytes));
    int blocks = (f.n_atoms + kWarpsPerBlock - 1) / kWarpsPerBlock;
    RUNE_KERNEL("k_forces", stream, k_forces<<<blocks, kWarpsPerBlock * 32, bytes, stream>>>(f.n_atoms, A));
    RUNE_LAUNCH_CHECK();
}

}  // namespace rune
