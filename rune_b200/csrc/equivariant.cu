// Möbius EQ blocks (rune/mobius/equivariant.py): direction encoder, equivariant message block,
// and their analytic adjoints with respect to node states, direction states and edge vectors.
//
// Forward of one block for the directed edge e = (i <- j), u = r / |r| (equivariant.py:124-223):
//   Y       = normalised real harmonics of u, orders 1..Le           (descriptor.py:643-648)
//   pc[l,c] = D_i[c, l] . Y_l,  pn[l,c] = (-1)^l D_j[c, l] . Y_l       probes
//   z       = act(W_x [b ; pc ; pn] + pb[t_i t_j] + A_i + B_j)         edge MLP; the context
//             columns are folded into per-atom A = W_e,c W_c RMSNorm(h), B = W_e,n W_n RMSNorm(h)
//   gate    = sigmoid(W_g z + b_g) cut;   (a, b) = tanh(W_d z + b_d)    per (order, channel)
//   msg_i   = sum_e gate[g(c)] v_j[c];    D'_i = D_i + sum_e cut (a mixed_j + b Y)
//   h'      = h + W_u2 act(W_u1 [RMSNorm(msg) ; |D'_l|^2] + b_u1) + b_u2
// The backward is split into a centre-side pass (per-edge adjoints, dE/dr_e, centre sums) and a
// pull pass in which atom j gathers the transposed sums (dv_j, dmixed_j, dD_j, dB_j) from the
// reverse edges of its own row. All sums run in a fixed order; no atomics.

#include "basis.cuh"
#include "engine.cuh"

namespace rune {

namespace {

constexpr int kWarps = 2;
constexpr int CH = 8;  // edges per chunk

__device__ __forceinline__ int order_of(int m) {  // component m of the packed basis -> l
    int l = 1;
    while ((l + 1) * (l + 1) - 1 <= m) ++l;
    return l;
}

// out[ee][o] = bias[o] + sum_k WT[k][o] x[ee][k] for ee < ne, lanes over o. k runs in steps of 4
// (x rows padded with zeros to a multiple of 4, WT padded with zero rows).
__device__ __forceinline__ void chunk_gemv(int ne, int n_out, int n_in4, const float* __restrict__ WT,
                                           const float* __restrict__ bias, const float* x, int ldx,
                                           float* out, int ldo, int lane) {
    for (int o = lane; o < n_out; o += 32) {
        float acc[CH];
        float b0 = bias ? __ldg(bias + o) : 0.0f;
#pragma unroll
        for (int ee = 0; ee < CH; ++ee) acc[ee] = b0;
        for (int k = 0; k < n_in4; k += 4) {
            float w0 = __ldg(WT + (size_t)(k + 0) * n_out + o);
            float w1 = __ldg(WT + (size_t)(k + 1) * n_out + o);
            float w2 = __ldg(WT + (size_t)(k + 2) * n_out + o);
            float w3 = __ldg(WT + (size_t)(k + 3) * n_out + o);
#pragma unroll
            for (int ee = 0; ee < CH; ++ee) {
                float4 xv = *reinterpret_cast<const float4*>(x + ee * ldx + k);
                acc[ee] += w0 * xv.x + w1 * xv.y + w2 * xv.z + w3 * xv.w;
            }
        }
        for (int ee = 0; ee < ne; ++ee) out[ee * ldo + o] = acc[ee];
    }
}

struct EqDims {
    int XP;   // padded edge-MLP input width (basis + probes), multiple of 4
    int GD;   // group gates + direction gates
    int GDP;  // GD padded to 4
    int MP;   // M padded to 4
    int LC;   // Le * Ce
    int DC;   // Ce * Cl
    __host__ __device__ EqDims(const EqLayerArgs& L) {
        LC = L.Le * L.Ce;
        XP = (L.K + 2 * LC + 3) & ~3;
        GD = L.G + 2 * LC;
        GDP = (GD + 3) & ~3;
        MP = (L.M + 3) & ~3;
        DC = L.Ce * L.Cl;
    }
};

// geometry, basis and scaled harmonics of a chunk (lane = edge)
__device__ __forceinline__ void chunk_geometry(const EqLayerArgs& L, const EdgeList& rad,
                                               const int* types, int ti, int e0, int ne, int lane,
                                               float* sx, int ldx, float* sdb, float* sgeo,
                                               int* sidx, float* sY, float* sdY) {
    if (lane < ne) {
        float4 e = rad.e[e0 + lane];
        int j = edge_j(e);
        float r = (float)sqrt((double)e.x * e.x + (double)e.y * e.y + (double)e.z * e.z);
        float inv = 1.0f / fmaxf(r, 1.0e-12f);
        float cut, dcut;
        cheb_masked(r, L.rc, L.K, sx + lane * ldx, sdb ? sdb + lane * L.K : nullptr, cut, dcut);
        float* g = sgeo + lane * 8;
        g[0] = e.x * inv; g[1] = e.y * inv; g[2] = e.z * inv;
        g[3] = cut; g[4] = dcut; g[5] = inv; g[6] = r;
        sidx[2 * lane] = j;
        sidx[2 * lane + 1] = ti * L.T + types[j];
        float* y = sY + lane * L.Cl;
        float* dy = sdY ? sdY + lane * L.Cl * 3 : nullptr;
        if (dy) {
            angular_components<true>(g[0], g[1], g[2], L.Le, L.zc,
                                     [&](int c, int, float Y, float dx, float ddy, float dz) {
                                         float s = __ldg(L.scale + c);
                                         y[c] = Y * s;
                                         dy[3 * c] = dx * s;
                                         dy[3 * c + 1] = ddy * s;
                                         dy[3 * c + 2] = dz * s;
                                     });
        } else {
            angular_components<false>(g[0], g[1], g[2], L.Le, L.zc,
                                      [&](int c, int, float Y, float, float, float) {
                                          y[c] = Y * __ldg(L.scale + c);
                                      });
        }
    }
    __syncwarp();
}

// probes into x[ee][K + l Ce + c] (centre) and x[ee][K + LC + l Ce + c] (neighbour), zero pad
__device__ __forceinline__ void chunk_probes(const EqLayerArgs& L, const EqDims& d, int ne, int lane,
                                             const float* sDi, const float* __restrict__ D,
                                             const int* sidx, const float* sY, float* sx) {
    for (int o = lane; o < ne * L.Ce; o += 32) {
        int ee = o / L.Ce, c = o - ee * L.Ce;
        const float* Dj = D + (size_t)sidx[2 * ee] * d.DC + (size_t)c * L.Cl;
        const float* Di = sDi + c * L.Cl;
        const float* y = sY + ee * L.Cl;
        float* x = sx + ee * d.XP + L.K;
        for (int l = 1; l <= L.Le; ++l) {
            float pc = 0.0f, pn = 0.0f;
            for (int m = l * l - 1; m < (l + 1) * (l + 1) - 1; ++m) {
                pc += Di[m] * y[m];
                pn += __ldg(Dj + m) * y[m];
            }
            x[(l - 1) * L.Ce + c] = pc;
            x[d.LC + (l - 1) * L.Ce + c] = (l & 1) ? -pn : pn;
        }
    }
    for (int o = lane; o < ne * (d.XP - L.K - 2 * d.LC); o += 32) {
        int w = d.XP - L.K - 2 * d.LC;
        int ee = o / w, k = o - ee * w;
        sx[ee * d.XP + L.K + 2 * d.LC + k] = 0.0f;
    }
    __syncwarp();
}

// z = act(pre), pre = W_x x + pb[pair] + A_i + B_j; optionally keeps act'
__device__ __forceinline__ void chunk_edge_mlp(const EqLayerArgs& L, const EqDims& d, int ne, int lane,
                                               const float* sx, const int* sidx,
                                               const float* __restrict__ abv, int ldabv,
                                               const float* sA, float* sz, float* sdz) {
    chunk_gemv(ne, L.M, d.XP, L.wxT, nullptr, sx, d.XP, sz, d.MP, lane);
    __syncwarp();
    for (int o = lane; o < ne * L.M; o += 32) {
        int ee = o / L.M, m = o - ee * L.M;
        float pre = sz[ee * d.MP + m] + __ldg(L.pb + (size_t)sidx[2 * ee + 1] * L.M + m) + sA[m] +
                    __ldg(abv + (size_t)sidx[2 * ee] * ldabv + L.M + m);
        float y, dy;
        activation(L.act, pre, y, dy);
        sz[ee * d.MP + m] = y;
        if (sdz) sdz[ee * d.MP + m] = dy;
    }
    // zero the pad columns so padded GEMVs read zeros
    for (int o = lane; o < ne * (d.MP - L.M); o += 32) {
        int w = d.MP - L.M;
        int ee = o / w, k = o - ee * w;
        sz[ee * d.MP + L.M + k] = 0.0f;
        if (sdz) sdz[ee * d.MP + L.M + k] = 0.0f;
    }
    __syncwarp();
}

// gates: sg[ee][o] = sigmoid (o < G) or tanh (o >= G) of W_gd z + b_gd
__device__ __forceinline__ void chunk_gates(const EqLayerArgs& L, const EqDims& d, int ne, int lane,
                                            const float* sz, float* sg) {
    chunk_gemv(ne, d.GD, d.MP, L.wgdT, L.bgd, sz, d.MP, sg, d.GDP, lane);
    __syncwarp();
    for (int o = lane; o < ne * d.GD; o += 32) {
        int ee = o / d.GD, q = o - ee * d.GD;
        float v = sg[ee * d.GDP + q];
        sg[ee * d.GDP + q] = q < L.G ? sigmoidf_(v) : tanhf(v);
    }
    __syncwarp();
}

struct FwdSmem {
    int sx, sz, sgeo, sidx, sY, sDi, sA, smsg, sinc, total;
    __host__ __device__ FwdSmem(const EqLayerArgs& L) {
        EqDims d(L);
        int xs = d.XP > d.GDP ? d.XP : d.GDP;
        sx = 0;
        sz = sx + CH * xs;
        sgeo = sz + CH * d.MP;
        sidx = sgeo + CH * 8;
        sY = sidx + CH * 2;
        sDi = sY + CH * L.Cl;
        sA = sDi + d.DC;
        smsg = sA + L.M;
        sinc = smsg + L.H;
        total = (sinc + d.DC + 3) & ~3;
    }
};

__global__ void __launch_bounds__(kWarps * 32)
k_eq_forward_edges(int n_atoms, EqLayerArgs L, EdgeList rad, const int* __restrict__ types,
                   const float* __restrict__ abv, const float* __restrict__ D,
                   const float* __restrict__ mixed, float* __restrict__ msg_out,
                   float* __restrict__ dn_out, float* __restrict__ gva_out) {
    extern __shared__ __align__(16) float smem[];
    EqDims d(L);
    FwdSmem S(L);
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int i = blockIdx.x * kWarps + warp;
    float* sm = smem + warp * S.total;
    float* sx = sm + S.sx;
    float* sz = sm + S.sz;
    float* sgeo = sm + S.sgeo;
    int* sidx = reinterpret_cast<int*>(sm + S.sidx);
    float* sY = sm + S.sY;
    float* sDi = sm + S.sDi;
    float* sA = sm + S.sA;
    float* smsg = sm + S.smsg;
    float* sinc = sm + S.sinc;
    if (i >= n_atoms) return;
    int ti = types[i];
    int ldabv = 2 * L.M + L.H;
    int gw = L.H / L.G;
    int GVA = L.G + d.LC;
    for (int o = lane; o < d.DC; o += 32) {
        sDi[o] = D[(size_t)i * d.DC + o];
        sinc[o] = 0.0f;
    }
    for (int m = lane; m < L.M; m += 32) sA[m] = abv[(size_t)i * ldabv + m];
    for (int c = lane; c < L.H; c += 32) smsg[c] = 0.0f;
    __syncwarp();
    int row = rad.row_ptr[i], cnt = rad.cnt[i];
    for (int base = 0; base < cnt; base += CH) {
        int ne = min(CH, cnt - base);
        int e0 = row + base;
        chunk_geometry(L, rad, types, ti, e0, ne, lane, sx, d.XP, nullptr, sgeo, sidx, sY, nullptr);
        chunk_probes(L, d, ne, lane, sDi, D, sidx, sY, sx);
        chunk_edge_mlp(L, d, ne, lane, sx, sidx, abv, ldabv, sA, sz, nullptr);
        float* sg = sx;  // x is no longer needed
        chunk_gates(L, d, ne, lane, sz, sg);
        // store gate*cut and cut*transport for the backward pull
        for (int o = lane; o < ne * GVA; o += 32) {
            int ee = o / GVA, q = o - ee * GVA;
            gva_out[(size_t)(e0 + ee) * GVA + q] = sg[ee * d.GDP + q] * sgeo[ee * 8 + 3];
        }
        // scalar messages
        for (int c = lane; c < L.H; c += 32) {
            int g = c / gw;
            float acc = smsg[c];
            for (int ee = 0; ee < ne; ++ee)
                acc += sg[ee * d.GDP + g] * sgeo[ee * 8 + 3] *
                       __ldg(abv + (size_t)sidx[2 * ee] * ldabv + 2 * L.M + c);
            smsg[c] = acc;
        }
        // direction updates: lanes over (c, m)
        for (int o = lane; o < d.DC; o += 32) {
            int c = o / L.Cl, m = o - c * L.Cl;
            int l = order_of(m);
            float acc = sinc[o];
            for (int ee = 0; ee < ne; ++ee) {
                const float* g = sg + ee * d.GDP + L.G;
                float a = g[(l - 1) * L.Ce + c], b = g[d.LC + (l - 1) * L.Ce + c];
                float mj = __ldg(mixed + (size_t)sidx[2 * ee] * d.DC + o);
                acc += sgeo[ee * 8 + 3] * (a * mj + b * sY[ee * L.Cl + m]);
            }
            sinc[o] = acc;
        }
        __syncwarp();
    }
    for (int c = lane; c < L.H; c += 32) msg_out[(size_t)i * L.H + c] = smsg[c];
    for (int o = lane; o < d.DC; o += 32) dn_out[(size_t)i * d.DC + o] = sDi[o] + sinc[o];
}

// mixed[c', m] = sum_c W_mix,l(m)[c', c] D[c, m]   (equivariant.py:148-158)
__global__ void k_eq_mix(int n_atoms, EqLayerArgs L, const float* __restrict__ D,
                         float* __restrict__ mixed) {
    int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (i >= n_atoms) return;
    int DC = L.Ce * L.Cl;
    const float* Di = D + (size_t)i * DC;
    for (int o = lane; o < DC; o += 32) {
        int cp = o / L.Cl, m = o - cp * L.Cl;
        int l = order_of(m);
        const float* w = L.wmix + ((size_t)(l - 1) * L.Ce + cp) * L.Ce;
        float s = 0.0f;
        for (int c = 0; c < L.Ce; ++c) s += __ldg(w + c) * Di[c * L.Cl + m];
        mixed[(size_t)i * DC + o] = s;
    }
}

// uin = [RMSNorm_msg(msg), |D'_l[c]|^2]
__global__ void k_eq_node_forward(int n_atoms, EqLayerArgs L, const float* __restrict__ msg,
                                  const float* __restrict__ dn, float* __restrict__ uin,
                                  float* __restrict__ rho_m) {
    int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (i >= n_atoms) return;
    int LC = L.Le * L.Ce, DC = L.Ce * L.Cl, HU = L.H + LC;
    const float* m = msg + (size_t)i * L.H;
    double ss = 0.0;
    for (int c = lane; c < L.H; c += 32) ss += (double)m[c] * m[c];
    ss = warp_sum(ss);
    float rho = (float)(1.0 / sqrt(ss / L.H + (double)L.eps));
    if (lane == 0) rho_m[i] = rho;
    for (int c = lane; c < L.H; c += 32) uin[(size_t)i * HU + c] = m[c] * rho * __ldg(L.g_msg + c);
    const float* Dn = dn + (size_t)i * DC;
    for (int o = lane; o < LC; o += 32) {
        int l = o / L.Ce + 1, c = o - (l - 1) * L.Ce;
        float s = 0.0f;
        for (int mm = l * l - 1; mm < (l + 1) * (l + 1) - 1; ++mm) {
            float v = Dn[c * L.Cl + mm];
            s += v * v;
        }
        uin[(size_t)i * HU + L.H + o] = s;
    }
}

// dmsg = RMSNorm^T(duin[:H]);  dDp = dDn_next + 2 duin[H + l Ce + c] D'[c, m]
__global__ void k_eq_node_backward(int n_atoms, EqLayerArgs L, const float* __restrict__ msg,
                                   const float* __restrict__ rho_m, const float* __restrict__ dn,
                                   const float* __restrict__ duin, const float* __restrict__ ddn_next,
                                   float* __restrict__ dmsg, float* __restrict__ ddp) {
    int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (i >= n_atoms) return;
    int LC = L.Le * L.Ce, DC = L.Ce * L.Cl, HU = L.H + LC;
    const float* m = msg + (size_t)i * L.H;
    const float* du = duin + (size_t)i * HU;
    double dot = 0.0;
    for (int c = lane; c < L.H; c += 32) dot += (double)(du[c] * __ldg(L.g_msg + c)) * m[c];
    dot = warp_sum(dot);
    float rho = rho_m[i];
    float coef = (float)((double)rho * rho * rho * dot / L.H);
    for (int c = lane; c < L.H; c += 32)
        dmsg[(size_t)i * L.H + c] = rho * du[c] * __ldg(L.g_msg + c) - coef * m[c];
    for (int o = lane; o < DC; o += 32) {
        int c = o / L.Cl, mm = o - c * L.Cl;
        int l = order_of(mm);
        float v = 2.0f * du[L.H + (l - 1) * L.Ce + c] * dn[(size_t)i * DC + o];
        if (ddn_next) v += ddn_next[(size_t)i * DC + o];
        ddp[(size_t)i * DC + o] = v;
    }
}

struct BwdSmem {
    int sx, sdb, sz, sdz, sg, sdl, sgeo, sidx, sY, sdY, sDi, sdDp, sdmsg, sdA, sdDc, sdYn,
        spart, total;
    __host__ __device__ BwdSmem(const EqLayerArgs& L) {
        EqDims d(L);
        int xs = d.XP > d.GDP ? d.XP : d.GDP;
        sx = 0;
        sdb = sx + CH * xs;
        sz = sdb + CH * L.K;
        sdz = sz + CH * d.MP;
        sg = sdz + CH * d.MP;
        sdl = sg + CH * d.GDP;
        sgeo = sdl + CH * d.GDP;
        sidx = sgeo + CH * 8;
        sY = sidx + CH * 2;
        sdY = sY + CH * L.Cl;
        sDi = sdY + CH * L.Cl * 3;
        sdDp = sDi + d.DC;
        sdmsg = sdDp + d.DC;
        sdA = sdmsg + L.H;
        sdDc = sdA + L.M;
        sdYn = sdDc + d.DC;
        spart = sdYn + CH * L.Cl;
        total = (spart + CH * (L.Ce + L.G) + 3) & ~3;
        sx = (sx + 3) & ~3;
    }
};

// Centre side: per-edge adjoints; stores dpre_e and dpn_e, adds dE/dr_e, and writes the centre
// sums dA_i and the probe part of dD_i.
__global__ void __launch_bounds__(kWarps * 32)
k_eq_backward_centre(int n_atoms, EqLayerArgs L, EdgeList rad, const int* __restrict__ types,
                     const float* __restrict__ abv, const float* __restrict__ D,
                     const float* __restrict__ mixed, const float* __restrict__ dmsg,
                     const float* __restrict__ ddp, float* __restrict__ dpre_out,
                     float* __restrict__ dpn_out, float4* __restrict__ edge_grad,
                     float* __restrict__ dabv, float* __restrict__ ddc) {
    extern __shared__ __align__(16) float smem[];
    EqDims d(L);
    BwdSmem S(L);
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int i = blockIdx.x * kWarps + warp;
    float* sm = smem + warp * S.total;
    float* sx = sm + S.sx;
    float* sdb = sm + S.sdb;
    float* sz = sm + S.sz;
    float* sdz = sm + S.sdz;
    float* sg = sm + S.sg;
    float* sdl = sm + S.sdl;
    float* sgeo = sm + S.sgeo;
    int* sidx = reinterpret_cast<int*>(sm + S.sidx);
    float* sY = sm + S.sY;
    float* sdY = sm + S.sdY;
    float* sDi = sm + S.sDi;
    float* sdDp = sm + S.sdDp;
    float* sdmsg = sm + S.sdmsg;
    float* sdA = sm + S.sdA;
    float* sdDc = sm + S.sdDc;
    float* sdYn = sm + S.sdYn;
    float* spart = sm + S.spart;
    if (i >= n_atoms) return;
    int ti = types[i];
    int ldabv = 2 * L.M + L.H;
    int gw = L.H / L.G;
    for (int o = lane; o < d.DC; o += 32) {
        sDi[o] = D[(size_t)i * d.DC + o];
        sdDp[o] = ddp[(size_t)i * d.DC + o];
        sdDc[o] = 0.0f;
    }
    for (int m = lane; m < L.M; m += 32) sdA[m] = 0.0f;
    for (int c = lane; c < L.H; c += 32) sdmsg[c] = dmsg[(size_t)i * L.H + c];
    __syncwarp();
    // the recomputed pre-activation reads A_i directly from abv[i][0..M)
    int row = rad.row_ptr[i], cnt = rad.cnt[i];
    for (int base = 0; base < cnt; base += CH) {
        int ne = min(CH, cnt - base);
        int e0 = row + base;
        chunk_geometry(L, rad, types, ti, e0, ne, lane, sx, d.XP, sdb, sgeo, sidx, sY, sdY);
        chunk_probes(L, d, ne, lane, sDi, D, sidx, sY, sx);
        chunk_edge_mlp(L, d, ne, lane, sx, sidx, abv, ldabv, abv + (size_t)i * ldabv, sz, sdz);
        chunk_gates(L, d, ne, lane, sz, sg);
        // direction-gate adjoints (lanes over (ee, c))
        for (int o = lane; o < ne * L.Ce; o += 32) {
            int ee = o / L.Ce, c = o - ee * L.Ce;
            const float* mj = mixed + (size_t)sidx[2 * ee] * d.DC + (size_t)c * L.Cl;
            const float* dd = sdDp + c * L.Cl;
            const float* y = sY + ee * L.Cl;
            float cut = sgeo[ee * 8 + 3];
            const float* g = sg + ee * d.GDP + L.G;
            float* dl = sdl + ee * d.GDP + L.G;
            float part = 0.0f;
            for (int l = 1; l <= L.Le; ++l) {
                float s1 = 0.0f, s2 = 0.0f;
                for (int m = l * l - 1; m < (l + 1) * (l + 1) - 1; ++m) {
                    s1 += dd[m] * __ldg(mj + m);
                    s2 += dd[m] * y[m];
                }
                int qa = (l - 1) * L.Ce + c, qb = d.LC + (l - 1) * L.Ce + c;
                float a = g[qa], b = g[qb];
                dl[qa] = cut * s1 * (1.0f - a * a);
                dl[qb] = cut * s2 * (1.0f - b * b);
                part += a * s1 + b * s2;
            }
            spart[ee * (L.Ce + L.G) + c] = part;
        }
        // group-gate adjoints (lanes over (ee, g))
        for (int o = lane; o < ne * L.G; o += 32) {
            int ee = o / L.G, g = o - ee * L.G;
            const float* vj = abv + (size_t)sidx[2 * ee] * ldabv + 2 * L.M + g * gw;
            float dg = 0.0f;
            for (int c = 0; c < gw; ++c) dg += sdmsg[g * gw + c] * __ldg(vj + c);
            float s = sg[ee * d.GDP + g];
            sdl[ee * d.GDP + g] = dg * sgeo[ee * 8 + 3] * s * (1.0f - s);
            spart[ee * (L.Ce + L.G) + L.Ce + g] = dg * s;
        }
        // injection part of dY (lanes over (ee, m))
        for (int o = lane; o < ne * L.Cl; o += 32) {
            int ee = o / L.Cl, m = o - ee * L.Cl;
            int l = order_of(m);
            const float* gb = sg + ee * d.GDP + L.G + d.LC + (l - 1) * L.Ce;
            float s = 0.0f;
            for (int c = 0; c < L.Ce; ++c) s += gb[c] * sdDp[c * L.Cl + m];
            sdYn[ee * L.Cl + m] = sgeo[ee * 8 + 3] * s;
        }
        for (int o = lane; o < ne * (d.GDP - d.GD); o += 32) {
            int w = d.GDP - d.GD;
            int ee = o / w, k = o - ee * w;
            sdl[ee * d.GDP + d.GD + k] = 0.0f;
        }
        __syncwarp();
        // dz = W_gd^T dl ; dpre = dz * act'
        chunk_gemv(ne, L.M, d.GDP, L.wgd, nullptr, sdl, d.GDP, sz, d.MP, lane);
        __syncwarp();
        for (int o = lane; o < ne * d.MP; o += 32) {
            int ee = o / d.MP, m = o - ee * d.MP;
            float v = m < L.M ? sz[ee * d.MP + m] * sdz[ee * d.MP + m] : 0.0f;
            sz[ee * d.MP + m] = v;
            if (m < L.M) dpre_out[(size_t)(e0 + ee) * L.M + m] = v;
        }
        __syncwarp();
        for (int m = lane; m < L.M; m += 32) {
            float acc = sdA[m];
            for (int ee = 0; ee < ne; ++ee) acc += sz[ee * d.MP + m];
            sdA[m] = acc;
        }
        // dx = W_x^T dpre (basis and probe adjoints)
        chunk_gemv(ne, d.XP, d.MP, L.wx, nullptr, sz, d.MP, sx, d.XP, lane);
        __syncwarp();
        // neighbour-probe adjoints are stored for the pull; centre-probe adjoints go into dD_i
        for (int o = lane; o < ne * d.LC; o += 32) {
            int ee = o / d.LC, q = o - ee * d.LC;
            dpn_out[(size_t)(e0 + ee) * d.LC + q] = sx[ee * d.XP + L.K + d.LC + q];
        }
        for (int c = lane; c < L.Ce; c += 32) {
            for (int ee = 0; ee < ne; ++ee) {
                const float* y = sY + ee * L.Cl;
                for (int l = 1; l <= L.Le; ++l) {
                    float dpc = sx[ee * d.XP + L.K + (l - 1) * L.Ce + c];
                    for (int m = l * l - 1; m < (l + 1) * (l + 1) - 1; ++m)
                        sdDc[c * L.Cl + m] += dpc * y[m];
                }
            }
        }
        // probe parts of dY (lanes over (ee, m))
        for (int o = lane; o < ne * L.Cl; o += 32) {
            int ee = o / L.Cl, m = o - ee * L.Cl;
            int l = order_of(m);
            const float* dpc = sx + ee * d.XP + L.K + (l - 1) * L.Ce;
            const float* dpn = sx + ee * d.XP + L.K + d.LC + (l - 1) * L.Ce;
            const float* Dj = D + (size_t)sidx[2 * ee] * d.DC;
            float s = 0.0f, t = 0.0f;
            for (int c = 0; c < L.Ce; ++c) {
                s += dpc[c] * sDi[c * L.Cl + m];
                t += dpn[c] * __ldg(Dj + c * L.Cl + m);
            }
            sdYn[ee * L.Cl + m] += s + ((l & 1) ? -t : t);
        }
        __syncwarp();
        // edge-vector gradient (lane = edge)
        if (lane < ne) {
            int ee = lane;
            const float* g = sgeo + ee * 8;
            float dcut_e = 0.0f;
            for (int q = 0; q < L.Ce + L.G; ++q) dcut_e += spart[ee * (L.Ce + L.G) + q];
            float dd = dcut_e * g[4];
            for (int k = 0; k < L.K; ++k) dd += sx[ee * d.XP + k] * sdb[ee * L.K + k];
            float du0 = 0.f, du1 = 0.f, du2 = 0.f;
            for (int m = 0; m < L.Cl; ++m) {
                float w = sdYn[ee * L.Cl + m];
                const float* dy = sdY + (ee * L.Cl + m) * 3;
                du0 += w * dy[0];
                du1 += w * dy[1];
                du2 += w * dy[2];
            }
            float pu = du0 * g[0] + du1 * g[1] + du2 * g[2];
            float inv = g[5];
            float4 G = edge_grad[e0 + ee];
            G.x += dd * g[0] + (du0 - pu * g[0]) * inv;
            G.y += dd * g[1] + (du1 - pu * g[1]) * inv;
            G.z += dd * g[2] + (du2 - pu * g[2]) * inv;
            edge_grad[e0 + ee] = G;
        }
        __syncwarp();
    }
    for (int m = lane; m < L.M; m += 32) dabv[(size_t)i * ldabv + m] = sdA[m];
    for (int o = lane; o < d.DC; o += 32) ddc[(size_t)i * d.DC + o] = sdDc[o];
}

// Pull side for atom i over the reverse edges of its row: dB_i, dv_i (into dabv), and
// dD_prev = dDp_i + dD_probe,centre + dD_probe,neighbour + W_mix^T dmixed_i.
__global__ void k_eq_backward_pull(int n_atoms, EqLayerArgs L, EdgeList rad,
                                   const float* __restrict__ gva, const float* __restrict__ dpre,
                                   const float* __restrict__ dpn, const float* __restrict__ dmsg,
                                   const float* __restrict__ ddp, const float* __restrict__ ddc,
                                   float* __restrict__ dabv, float* __restrict__ dd_prev) {
    extern __shared__ __align__(16) float smem[];
    EqDims d(L);
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int i = blockIdx.x * kWarps + warp;
    int per = (L.M + L.H + 2 * d.DC + CH * (L.Cl + 2) + 3) & ~3;
    float* sm = smem + warp * per;
    float* sdB = sm;
    float* sdv = sdB + L.M;
    float* sdmix = sdv + L.H;
    float* sdDn = sdmix + d.DC;
    float* sY = sdDn + d.DC;
    int* sidx = reinterpret_cast<int*>(sY + CH * L.Cl);
    if (i >= n_atoms) return;
    int ldabv = 2 * L.M + L.H;
    int gw = L.H / L.G;
    int GVA = L.G + d.LC;
    for (int m = lane; m < L.M; m += 32) sdB[m] = 0.0f;
    for (int c = lane; c < L.H; c += 32) sdv[c] = 0.0f;
    for (int o = lane; o < d.DC; o += 32) {
        sdmix[o] = 0.0f;
        sdDn[o] = 0.0f;
    }
    int row = rad.row_ptr[i], cnt = rad.cnt[i];
    for (int base = 0; base < cnt; base += CH) {
        int ne = min(CH, cnt - base);
        int e0 = row + base;
        if (lane < ne) {
            float4 e = rad.e[e0 + lane];
            sidx[2 * lane] = edge_j(e);
            sidx[2 * lane + 1] = rad.rev[e0 + lane];
            float r = (float)sqrt((double)e.x * e.x + (double)e.y * e.y + (double)e.z * e.z);
            float inv = 1.0f / fmaxf(r, 1.0e-12f);
            float* y = sY + lane * L.Cl;
            angular_components<false>(e.x * inv, e.y * inv, e.z * inv, L.Le, L.zc,
                                      [&](int c, int, float Y, float, float, float) {
                                          y[c] = Y * __ldg(L.scale + c);
                                      });
        }
        __syncwarp();
        for (int m = lane; m < L.M; m += 32) {
            float acc = sdB[m];
            for (int ee = 0; ee < ne; ++ee) acc += __ldg(dpre + (size_t)sidx[2 * ee + 1] * L.M + m);
            sdB[m] = acc;
        }
        for (int c = lane; c < L.H; c += 32) {
            int g = c / gw;
            float acc = sdv[c];
            for (int ee = 0; ee < ne; ++ee)
                acc += __ldg(gva + (size_t)sidx[2 * ee + 1] * GVA + g) *
                       __ldg(dmsg + (size_t)sidx[2 * ee] * L.H + c);
            sdv[c] = acc;
        }
        for (int o = lane; o < d.DC; o += 32) {
            int c = o / L.Cl, m = o - c * L.Cl;
            int l = order_of(m);
            int q = (l - 1) * L.Ce + c;
            float am = sdmix[o], an = sdDn[o];
            for (int ee = 0; ee < ne; ++ee) {
                int e = sidx[2 * ee + 1], j = sidx[2 * ee];
                am += __ldg(gva + (size_t)e * GVA + L.G + q) * __ldg(ddp + (size_t)j * d.DC + o);
                an += __ldg(dpn + (size_t)e * d.LC + q) * sY[ee * L.Cl + m];
            }
            sdmix[o] = am;
            sdDn[o] = an;
        }
        __syncwarp();
    }
    for (int m = lane; m < L.M; m += 32) dabv[(size_t)i * ldabv + L.M + m] = sdB[m];
    for (int c = lane; c < L.H; c += 32) dabv[(size_t)i * ldabv + 2 * L.M + c] = sdv[c];
    for (int o = lane; o < d.DC; o += 32) {
        int c = o / L.Cl, m = o - c * L.Cl;
        int l = order_of(m);
        float s = ddp[(size_t)i * d.DC + o] + ddc[(size_t)i * d.DC + o] + sdDn[o];
        const float* w = L.wmix + (size_t)(l - 1) * L.Ce * L.Ce;
        for (int cp = 0; cp < L.Ce; ++cp) s += __ldg(w + cp * L.Ce + c) * sdmix[cp * L.Cl + m];
        dd_prev[(size_t)i * d.DC + o] = s;
    }
}

// D0[c, m] = sum_n P_l(m)[c, n] s[n, m] scale[m]  (equivariant.py:12-39, descriptor.py:639-641)
__global__ void k_eq_encode(int n_atoms, EqLayerArgs L, int na, int C,
                            const float* __restrict__ proj, const float* __restrict__ s,
                            float* __restrict__ D0) {
    int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (i >= n_atoms) return;
    int DC = L.Ce * L.Cl;
    for (int o = lane; o < DC; o += 32) {
        int c = o / L.Cl, m = o - c * L.Cl;
        int l = order_of(m);
        const float* p = proj + ((size_t)(l - 1) * L.Ce + c) * na;
        float acc = 0.0f;
        for (int n = 0; n < na; ++n) acc += __ldg(p + n) * s[((size_t)i * na + n) * C + m];
        D0[(size_t)i * DC + o] = acc * __ldg(L.scale + m);
    }
}

// moment gradient mg[n, m] = scale[m] sum_c P_l(m)[c, n] dD0[c, m]  (zero for m >= Cl)
__global__ void k_eq_encode_backward(int n_atoms, EqLayerArgs L, int na, int C,
                                     const float* __restrict__ proj, const float* __restrict__ dd0,
                                     float* __restrict__ mg) {
    int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (i >= n_atoms) return;
    int DC = L.Ce * L.Cl;
    for (int o = lane; o < na * C; o += 32) {
        int n = o / C, m = o - n * C;
        float acc = 0.0f;
        if (m < L.Cl) {
            int l = order_of(m);
            for (int c = 0; c < L.Ce; ++c)
                acc += __ldg(proj + ((size_t)(l - 1) * L.Ce + c) * na + n) *
                       dd0[(size_t)i * DC + c * L.Cl + m];
            acc *= __ldg(L.scale + m);
        }
        mg[(size_t)i * na * C + o] = acc;
    }
}

}  // namespace

size_t eq_forward_smem(const EqLayerArgs& L) { return sizeof(float) * FwdSmem(L).total * kWarps; }
size_t eq_backward_smem(const EqLayerArgs& L) { return sizeof(float) * BwdSmem(L).total * kWarps; }

static void set_smem(const void* fn, size_t bytes) {
    if (bytes > 48 * 1024)
        RUNE_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)bytes));
}

void eq_mix(const EqLayerArgs& L, int n, const float* D, float* mixed, cudaStream_t stream) {
    if (n == 0) return;
    RUNE_KERNEL("k_eq_mix", stream,
                k_eq_mix<<<(n * 32 + 255) / 256, 256, 0, stream>>>(n, L, D, mixed));
    RUNE_LAUNCH_CHECK();
}

void eq_forward_edges(const EqLayerArgs& L, int n, const EdgeList& rad, const int* types,
                      const float* abv, const float* D, const float* mixed, float* msg,
                      float* dn, float* gva, cudaStream_t stream) {
    if (n == 0) return;
    size_t bytes = eq_forward_smem(L);
    set_smem((const void*)k_eq_forward_edges, bytes);
    RUNE_KERNEL("k_eq_forward_edges", stream,
                k_eq_forward_edges<<<(n + kWarps - 1) / kWarps, kWarps * 32, bytes, stream>>>(
                    n, L, rad, types, abv, D, mixed, msg, dn, gva));
    RUNE_LAUNCH_CHECK();
}

void eq_node_forward(const EqLayerArgs& L, int n, const float* msg, const float* dn, float* uin,
                     float* rho_m, cudaStream_t stream) {
    if (n == 0) return;
    RUNE_KERNEL("k_eq_node_forward", stream,
                k_eq_node_forward<<<(n * 32 + 255) / 256, 256, 0, stream>>>(n, L, msg, dn, uin,
                                                                              rho_m));
    RUNE_LAUNCH_CHECK();
}

void eq_node_backward(const EqLayerArgs& L, int n, const float* msg, const float* rho_m,
                      const float* dn, const float* duin, const float* ddn_next, float* dmsg,
                      float* ddp, cudaStream_t stream) {
    if (n == 0) return;
    RUNE_KERNEL("k_eq_node_backward", stream,
                k_eq_node_backward<<<(n * 32 + 255) / 256, 256, 0, stream>>>(
                    n, L, msg, rho_m, dn, duin, ddn_next, dmsg, ddp));
    RUNE_LAUNCH_CHECK();
}

void eq_backward_edges(const EqLayerArgs& L, int n, const EdgeList& rad, const int* types,
                       const float* abv, const float* D, const float* mixed, const float* dmsg,
                       const float* ddp, const float* gva, float* dpre, float* dpn,
                       float4* edge_grad, float* dabv, float* ddc, float* dd_prev,
                       cudaStream_t stream) {
    if (n == 0) return;
    size_t bytes = eq_backward_smem(L);
    set_smem((const void*)k_eq_backward_centre, bytes);
    RUNE_KERNEL("k_eq_backward_centre", stream,
                k_eq_backward_centre<<<(n + kWarps - 1) / kWarps, kWarps * 32, bytes, stream>>>(
                    n, L, rad, types, abv, D, mixed, dmsg, ddp, dpre, dpn, edge_grad, dabv, ddc));
    RUNE_LAUNCH_CHECK();
    EqDims d(L);
    size_t pbytes = sizeof(float) * kWarps * ((L.M + L.H + 2 * d.DC + CH * (L.Cl + 2) + 3) & ~3);
    set_smem((const void*)k_eq_backward_pull, pbytes);
    RUNE_KERNEL("k_eq_backward_pull", stream,
                k_eq_backward_pull<<<(n + kWarps - 1) / kWarps, kWarps * 32, pbytes, stream>>>(
                    n, L, rad, gva, dpre, dpn, dmsg, ddp, ddc, dabv, dd_prev));
    RUNE_LAUNCH_CHECK();
}

void eq_encode(const EqLayerArgs& L, int n, int na, int C, const float* proj, const float* s,
               float* D0, cudaStream_t stream) {
    if (n == 0) return;
    RUNE_KERNEL("k_eq_encode", stream,
                k_eq_encode<<<(n * 32 + 255) / 256, 256, 0, stream>>>(n, L, na, C, proj, s, D0));
    RUNE_LAUNCH_CHECK();
}

void eq_encode_backward(const EqLayerArgs& L, int n, int na, int C, const float* proj,
                        const float* dd0, float* mg, cudaStream_t stream) {
    if (n == 0) return;
    RUNE_KERNEL("k_eq_encode_backward", stream,
                k_eq_encode_backward<<<(n * 32 + 255) / 256, 256, 0, stream>>>(n, L, na, C, proj,
                                                                                 dd0, mg));
    RUNE_LAUNCH_CHECK();
}

}  // namespace rune
