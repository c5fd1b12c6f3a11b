// Möbius MP message block (rune/mobius/message.py:125-193): forward edge and node kernels and
// their analytic adjoints with respect to the node states and the edge vectors.
//
// Per directed edge e = (i <- j) on the radial list (message cutoff rc_m):
//   b_k   = Chebyshev basis masked at rc_m (descriptor.py:357-374), cut = fc masked
//   z     = act(W_e [b ; P[t_i t_j]] + b_e)            edge MLP (the pair part is a per-pair
//                                                        table pb = W_e,pair P + b_e built at load)
//   gate  = sigmoid(W_g z + b_g) * cut                   [G]   grouped scalar gates
//   vg    = sigmoid(W_vg z + b_vg) * cut                 [V]   vector gates
//   msg_i = sum_e gate[g(c)] v_j[c]                      v = W_v RMSNorm(h)
//   vec_i = sum_e vg[k] src_j[k] u_e                     src = W_src RMSNorm(h), u = r / |r|
// Node: t = |W_mix vec|^2, h' = h + W_u2 act(W_u1 [RMSNorm(msg) ; t] + b_u1) + b_u2.
//
// The forward stores gate and vg per edge, with and without the cutoff. The backward evaluates,
// for each centre i, the adjoint of every edge of its row (the stored sigmoids, then z once more
// for dpre) and the edge-vector gradient dE/dr_e; the
// transposed sums into neighbours (dv_j, dsrc_j) are pulled by atom j's warp through the
// reverse-edge index, reading the stored gates of the reverse edges. No atomics.
//
// Thread mapping: one warp per centre atom; edges in chunks of 32 (one lane per edge for
// geometry), contractions with lanes over output channels.

#include <type_traits>

#include "basis.cuh"
#include "engine.cuh"

namespace rune {

namespace {

constexpr int kWarps = 4;

// Message basis b_k, b'_k (descriptor.py:357-374) into registers: zero at and beyond rc and for
// k >= K (the padding of the KMAX-wide arrays); float64 inside like the descriptor basis.
template <int KMAX>
__device__ __forceinline__ void message_basis(float rf, float rcf, int K, float (&b)[KMAX],
                                              float (&db)[KMAX], float& cut, float& dcut) {
    const double pi = 3.14159265358979323846;
    double r = rf, rc = rcf;
    double xr = r / rc;
    bool inside = rf < rcf;
    double sv = 0.0, cv = -1.0;
    if (inside) sincospi(xr, &sv, &cv);
    double fc = inside ? 0.5 * cv + 0.5 : 0.0;
    double fcp = inside ? -0.5 * pi / rc * sv : 0.0;
    cut = (float)fc;
    dcut = (float)fcp;
    double rs = xr - 1.0;
    double x = 2.0 * rs * rs - 1.0;
    double dxdr = 4.0 * rs / rc;
    double t2 = 1.0, t1 = x, u2 = 1.0, u1 = 2.0 * x;
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
        double f, df;
        if (k == 0) {
            f = fc;
            df = fcp;
        } else if (k == 1) {
            double core = 0.5 * (x + 1.0);
            f = core * fc;
            df = 0.5 * dxdr * fc + core * fcp;
        } else {
            double tn = 2.0 * x * t1 - t2;
            double core = 0.5 * (tn + 1.0);
            f = core * fc;
            df = 0.5 * k * u1 * dxdr * fc + core * fcp;
            double un = 2.0 * x * u1 - u2;
            t2 = t1; t1 = tn;
            u2 = u1; u1 = un;
        }
        b[k] = k < K ? (float)f : 0.0f;
        db[k] = k < K ? (float)df : 0.0f;
    }
}

// Block-shared weights: W_e basis part transposed [K][M], [W_g; W_vg] [GV][M], [b_g; b_vg].
struct MpWeights {
    int wk, wgv, bgv, total;  // float offsets
    __host__ __device__ explicit MpWeights(const MpLayerArgs& L) {
        wk = 0;
        wgv = wk + L.K * L.Mp;
        bgv = wgv + (L.G + L.V) * L.Mp;
        total = (bgv + L.G + L.V + 3) & ~3;
    }
};

__device__ __forceinline__ void load_mp_weights(const MpLayerArgs& L, float* sm) {
    MpWeights W(L);
    for (int o = threadIdx.x; o < L.K * L.Mp; o += blockDim.x) {
        int k = o / L.Mp, m = o - k * L.Mp;
        sm[W.wk + o] = L.we_k[m * L.K + k];
    }
    for (int o = threadIdx.x; o < (L.G + L.V) * L.Mp; o += blockDim.x) sm[W.wgv + o] = L.wgv[o];
    for (int o = threadIdx.x; o < L.G + L.V; o += blockDim.x) sm[W.bgv + o] = L.bgv[o];
}

// Gate logits of one edge (lane): z = act(pb[pair] + W_e b) is streamed four hidden units at a
// time into lg[q] = b_q + sum_m W_gv[q, m] z_m; the hidden units are never stored. All lanes
// read the same weights (shared-memory broadcast), float4 along m.
template <int KMAX, int GMAX>
__device__ __forceinline__ void edge_logits(const MpLayerArgs& L, const float* sw,
                                            const float (&b)[KMAX], const float* pbrow,
                                            float (&lg)[GMAX]) {
    MpWeights W(L);
    const int GV = L.G + L.V;
#pragma unroll
    for (int q = 0; q < GMAX; ++q) lg[q] = q < GV ? sw[W.bgv + q] : 0.0f;
    for (int m0 = 0; m0 < L.Mp; m0 += 4) {
        float4 a = __ldg(reinterpret_cast<const float4*>(pbrow + m0));
#pragma unroll
        for (int k = 0; k < KMAX; ++k)
            if (k < L.K) {
                float4 w = *reinterpret_cast<const float4*>(sw + W.wk + k * L.Mp + m0);
                a.x += w.x * b[k]; a.y += w.y * b[k]; a.z += w.z * b[k]; a.w += w.w * b[k];
            }
        float z0, z1, z2, z3, d;
        activation(L.act, a.x, z0, d);
        activation(L.act, a.y, z1, d);
        activation(L.act, a.z, z2, d);
        activation(L.act, a.w, z3, d);
#pragma unroll
        for (int q = 0; q < GMAX; ++q)
            if (q < GV) {
                float4 w = *reinterpret_cast<const float4*>(sw + W.wgv + q * L.Mp + m0);
                lg[q] += w.x * z0 + w.y * z1 + w.z * z2 + w.w * z3;
            }
    }
}

// Forward edge kernel, warp per centre atom i, lane per edge (chunks of 32): gates
// sigmoid(logits) * cut stored per edge, then the message and vector sums of the chunk with
// lanes over channels.
template <int KMAX, int GMAX>
__global__ void __launch_bounds__(kWarps * 32)
k_mp_forward_edges(int n_atoms, MpLayerArgs L, EdgeList rad, const int* __restrict__ types,
                   const float* __restrict__ vs, float* __restrict__ msg_out,
                   float* __restrict__ vec_out, float* __restrict__ gv_out,
                   float* __restrict__ sg_out) {
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    MpWeights W(L);
    load_mp_weights(L, smem);
    __syncthreads();
    const int GV = L.G + L.V, HV = L.H + L.V, GS = GV | 1;
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int i = blockIdx.x * kWarps + warp;
    float* sgate = smem + W.total + warp * (32 * GS + 32 * 4 + 32);  // [32][GS]
    float* sgeo = sgate + 32 * GS;                                    // [32][4] unit vector
    int* sj = reinterpret_cast<int*>(sgeo + 32 * 4);                  // [32]
    if (i >= n_atoms) return;
    int ti = types[i];
    int gw = L.H / L.G;
    float accm[8], accv = 0.0f;  // channels lane + 32 t (H <= 256); vector entry `lane` (3V <= 32)
#pragma unroll
    for (int t = 0; t < 8; ++t) accm[t] = 0.0f;
    int row = rad.row_ptr[i], cnt = rad.cnt[i];
    for (int base = 0; base < cnt; base += 32) {
        int nv = min(32, cnt - base);
        if (lane < nv) {
            int e = row + base + lane;
            float4 ed = rad.e[e];
            int j = edge_j(ed);
            float r = (float)sqrt((double)ed.x * ed.x + (double)ed.y * ed.y + (double)ed.z * ed.z);
            float inv = 1.0f / fmaxf(r, 1.0e-12f);
            float b[KMAX], db[KMAX], cut, dcut;
            message_basis<KMAX>(r, L.rc, L.K, b, db, cut, dcut);
            float lg[GMAX];
            edge_logits<KMAX, GMAX>(L, smem, b, L.pb + (size_t)(ti * L.T + types[j]) * L.Mp, lg);
#pragma unroll
            for (int q = 0; q < GMAX; ++q)
                if (q < GV) {
                    float sgq = sigmoidf_(lg[q]);
                    float g = sgq * cut;
                    sgate[lane * GS + q] = g;
                    gv_out[(size_t)e * GV + q] = g;
                    sg_out[(size_t)e * GV + q] = sgq;
                }
            sgeo[lane * 4] = ed.x * inv;
            sgeo[lane * 4 + 1] = ed.y * inv;
            sgeo[lane * 4 + 2] = ed.z * inv;
            sj[lane] = j;
        }
        __syncwarp();
        for (int ee = 0; ee < nv; ++ee) {
            const float* vj = vs + (size_t)sj[ee] * HV;
            const float* ge = sgate + ee * GS;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                int c = lane + 32 * t;
                if (c < L.H) accm[t] += ge[c / gw] * __ldg(vj + c);
            }
            if (lane < 3 * L.V) {
                int k = lane / 3, x = lane - 3 * k;
                accv += ge[L.G + k] * __ldg(vj + L.H + k) * sgeo[ee * 4 + x];
            }
        }
        __syncwarp();
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        int c = lane + 32 * t;
        if (c < L.H) msg_out[(size_t)i * L.H + c] = accm[t];
    }
    if (lane < 3 * L.V) vec_out[(size_t)i * 3 * L.V + lane] = accv;
}

// uin = [RMSNorm_msg(msg), |W_mix vec|^2]; keeps 1/rms and the mixed vectors for the adjoint.
__global__ void k_mp_node_forward(int n_atoms, MpLayerArgs L, const float* __restrict__ msg,
                                  const float* __restrict__ vec, float* __restrict__ uin,
                                  float* __restrict__ rho_m, float* __restrict__ mixed) {
    int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (i >= n_atoms) return;
    int HV = L.H + L.V;
    const float* m = msg + (size_t)i * L.H;
    double ss = 0.0;
    for (int c = lane; c < L.H; c += 32) ss += (double)m[c] * m[c];
    ss = warp_sum(ss);
    float rho = (float)(1.0 / sqrt(ss / L.H + (double)L.eps));
    if (lane == 0) rho_m[i] = rho;
    for (int c = lane; c < L.H; c += 32) uin[(size_t)i * HV + c] = m[c] * rho * __ldg(L.g_msg + c);
    const float* v = vec + (size_t)i * 3 * L.V;
    for (int b = lane; b < L.V; b += 32) {
        float t = 0.0f;
        for (int x = 0; x < 3; ++x) {
            float s = 0.0f;
            for (int a = 0; a < L.V; ++a) s += __ldg(L.wmix + b * L.V + a) * v[3 * a + x];
            mixed[(size_t)i * 3 * L.V + 3 * b + x] = s;
            t += s * s;
        }
        uin[(size_t)i * HV + L.H + b] = t;
    }
}

// dmsg = RMSNorm_msg^T(duin[:H]), dvec = W_mix^T (2 duin[H:] * mixed).
__global__ void k_mp_node_backward(int n_atoms, MpLayerArgs L, const float* __restrict__ msg,
                                   const float* __restrict__ rho_m,
                                   const float* __restrict__ mixed,
                                   const float* __restrict__ duin, float* __restrict__ dmsg,
                                   float* __restrict__ dvec) {
    int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (i >= n_atoms) return;
    int HV = L.H + L.V;
    const float* m = msg + (size_t)i * L.H;
    const float* d = duin + (size_t)i * HV;
    double dot = 0.0;
    for (int c = lane; c < L.H; c += 32) dot += (double)(d[c] * __ldg(L.g_msg + c)) * m[c];
    dot = warp_sum(dot);
    float rho = rho_m[i];
    float coef = (float)((double)rho * rho * rho * dot / L.H);
    for (int c = lane; c < L.H; c += 32)
        dmsg[(size_t)i * L.H + c] = rho * d[c] * __ldg(L.g_msg + c) - coef * m[c];
    const float* mx = mixed + (size_t)i * 3 * L.V;
    for (int o = lane; o < 3 * L.V; o += 32) {
        int a = o / 3, x = o - 3 * a;
        float s = 0.0f;
        for (int b = 0; b < L.V; ++b) s += __ldg(L.wmix + b * L.V + a) * 2.0f * d[L.H + b] * mx[3 * b + x];
        dvec[(size_t)i * 3 * L.V + o] = s;
    }
}

// Adjoint of the edge part, warp per centre atom i, lane per edge of its row.
// Centre side: the gate adjoints (dmsg_i . v_j over the group, dvec_i . u v_src,j), then the
// hidden units are streamed again, four at a time, to form dpre = act' (W_gv^T dlogits) and the
// basis adjoint db_k = sum_m W_e[m, k] dpre_m; dE/dr_e is added to edge_grad[e].
// Neighbour side (pull): dv_i and dsrc_i from the reverse edges of row i (stored gates).
template <int KMAX, int GMAX>
__global__ void __launch_bounds__(kWarps * 32)
k_mp_backward_edges(int n_atoms, MpLayerArgs L, EdgeList rad, const int* __restrict__ types,
                    const float* __restrict__ vs, const float* __restrict__ dmsg,
                    const float* __restrict__ dvec, const float* __restrict__ gv,
                    const float* __restrict__ sgv, float4* __restrict__ edge_grad,
                    float* __restrict__ dvs) {
    extern __shared__ float4 smem4[];
    float* smem = reinterpret_cast<float*>(smem4);
    MpWeights W(L);
    load_mp_weights(L, smem);
    __syncthreads();
    const int GV = L.G + L.V, HV = L.H + L.V;
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int i = blockIdx.x * kWarps + warp;
    int per_warp = ((L.H + 3) & ~3) + 4 * 12 + 32 * 4 + 2 * 32;
    float* sdm = smem + W.total + warp * per_warp;  // dmsg_i [H]
    float* sdvec = sdm + ((L.H + 3) & ~3);          // dvec_i [3V] (room for 48)
    float* sgeo = sdvec + 4 * 12;                   // [32][4] reverse unit vectors
    int* sj = reinterpret_cast<int*>(sgeo + 32 * 4);
    int* srev = sj + 32;
    if (i >= n_atoms) return;
    int ti = types[i];
    int gw = L.H / L.G;
    const bool vec4 = (HV % 4 == 0) && (gw % 4 == 0);  // float4 gathers of v_j are aligned
    for (int c = lane; c < L.H; c += 32) sdm[c] = dmsg[(size_t)i * L.H + c];
    for (int o = lane; o < 3 * L.V; o += 32) sdvec[o] = dvec[(size_t)i * 3 * L.V + o];
    __syncwarp();
    int row = rad.row_ptr[i], cnt = rad.cnt[i];
    // ---- centre side, lane per edge
    for (int k0 = lane; k0 < cnt; k0 += 32) {
        int e = row + k0;
        float4 ed = rad.e[e];
        int j = edge_j(ed);
        float r = (float)sqrt((double)ed.x * ed.x + (double)ed.y * ed.y + (double)ed.z * ed.z);
        float inv = 1.0f / fmaxf(r, 1.0e-12f);
        float u0 = ed.x * inv, u1 = ed.y * inv, u2 = ed.z * inv;
        float b[KMAX], db[KMAX], cut, dcut;
        message_basis<KMAX>(r, L.rc, L.K, b, db, cut, dcut);
        const float* pbrow = L.pb + (size_t)(ti * L.T + types[j]) * L.Mp;
        float lg[GMAX];  // becomes d logits below
        const float* sge = sgv + (size_t)e * GV;  // the forward's sigmoids of this edge
        // gate adjoints -> d logits; cutoff and unit-vector adjoints
        const float* vj = vs + (size_t)j * HV;
        float dcut_e = 0.0f, du0 = 0.0f, du1 = 0.0f, du2 = 0.0f;
#pragma unroll
        for (int q = 0; q < GMAX; ++q) {
            if (q >= GV) continue;
            float sg = __ldg(sge + q);
            float dg;
            if (q < L.G) {
                dg = 0.0f;
                if (vec4) {
                    for (int c = 0; c < gw; c += 4) {
                        float4 v = __ldg(reinterpret_cast<const float4*>(vj + q * gw + c));
                        float4 d = *reinterpret_cast<const float4*>(sdm + q * gw + c);
                        dg += v.x * d.x + v.y * d.y + v.z * d.z + v.w * d.w;
                    }
                } else {
                    for (int c = 0; c < gw; ++c) dg += __ldg(vj + q * gw + c) * sdm[q * gw + c];
                }
            } else {
                int k = q - L.G;
                float src = __ldg(vj + L.H + k);
                float d0 = sdvec[3 * k], d1 = sdvec[3 * k + 1], d2 = sdvec[3 * k + 2];
                dg = src * (d0 * u0 + d1 * u1 + d2 * u2);
                float a = sg * cut * src;
                du0 += a * d0; du1 += a * d1; du2 += a * d2;
            }
            dcut_e += dg * sg;
            lg[q] = dg * cut * sg * (1.0f - sg);  // now d logits
        }
        // hidden units again: dpre = act'(pre) * (W_gv^T dl); db_k += W_e[m, k] dpre_m
        float dbk[KMAX];
#pragma unroll
        for (int k = 0; k < KMAX; ++k) dbk[k] = 0.0f;
        for (int m0 = 0; m0 < L.Mp; m0 += 4) {
            float4 a = __ldg(reinterpret_cast<const float4*>(pbrow + m0));
#pragma unroll
            for (int k = 0; k < KMAX; ++k)
                if (k < L.K) {
                    float4 w = *reinterpret_cast<const float4*>(smem + W.wk + k * L.Mp + m0);
                    a.x += w.x * b[k]; a.y += w.y * b[k]; a.z += w.z * b[k]; a.w += w.w * b[k];
                }
            float dz0 = 0.f, dz1 = 0.f, dz2 = 0.f, dz3 = 0.f;
#pragma unroll
            for (int q = 0; q < GMAX; ++q)
                if (q < GV) {
                    float4 w = *reinterpret_cast<const float4*>(smem + W.wgv + q * L.Mp + m0);
                    dz0 += w.x * lg[q]; dz1 += w.y * lg[q]; dz2 += w.z * lg[q]; dz3 += w.w * lg[q];
                }
            float y, d0, d1, d2, d3;
            activation(L.act, a.x, y, d0);
            activation(L.act, a.y, y, d1);
            activation(L.act, a.z, y, d2);
            activation(L.act, a.w, y, d3);
            dz0 *= d0; dz1 *= d1; dz2 *= d2; dz3 *= d3;
#pragma unroll
            for (int k = 0; k < KMAX; ++k)
                if (k < L.K) {
                    float4 w = *reinterpret_cast<const float4*>(smem + W.wk + k * L.Mp + m0);
                    dbk[k] += w.x * dz0 + w.y * dz1 + w.z * dz2 + w.w * dz3;
                }
        }
        float dd = dcut_e * dcut;
#pragma unroll
        for (int k = 0; k < KMAX; ++k) dd += dbk[k] * db[k];
        float pu = du0 * u0 + du1 * u1 + du2 * u2;
        float4 G = edge_grad[e];
        G.x += dd * u0 + (du0 - pu * u0) * inv;
        G.y += dd * u1 + (du1 - pu * u1) * inv;
        G.z += dd * u2 + (du2 - pu * u2) * inv;
        edge_grad[e] = G;
    }
    // ---- neighbour side: pull the reverse edges' contributions into dv_i and dsrc_i
    float accm[8], accs = 0.0f;
#pragma unroll
    for (int t = 0; t < 8; ++t) accm[t] = 0.0f;
    for (int base = 0; base < cnt; base += 32) {
        int nv = min(32, cnt - base);
        __syncwarp();
        if (lane < nv) {
            int e = row + base + lane;
            float4 ed = rad.e[e];
            float r = (float)sqrt((double)ed.x * ed.x + (double)ed.y * ed.y + (double)ed.z * ed.z);
            float inv = 1.0f / fmaxf(r, 1.0e-12f);
            float* g = sgeo + lane * 4;
            g[0] = -ed.x * inv; g[1] = -ed.y * inv; g[2] = -ed.z * inv;  // unit of the reverse edge
            sj[lane] = edge_j(ed);
            srev[lane] = rad.rev[e];
        }
        __syncwarp();
        for (int ee = 0; ee < nv; ++ee) {
            const float* gr = gv + (size_t)srev[ee] * GV;
            const float* dmj = dmsg + (size_t)sj[ee] * L.H;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                int c = lane + 32 * t;
                if (c < L.H) accm[t] += __ldg(gr + c / gw) * __ldg(dmj + c);
            }
            if (lane < L.V) {
                const float* dvj = dvec + (size_t)sj[ee] * 3 * L.V + 3 * lane;
                const float* u = sgeo + ee * 4;
                float proj = __ldg(dvj) * u[0] + __ldg(dvj + 1) * u[1] + __ldg(dvj + 2) * u[2];
                accs += __ldg(gr + L.G + lane) * proj;
            }
        }
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        int c = lane + 32 * t;
        if (c < L.H) dvs[(size_t)i * HV + c] = accm[t];
    }
    if (lane < L.V) dvs[(size_t)i * HV + L.H + lane] = accs;
}

size_t mp_smem_bytes(const MpLayerArgs& L, bool backward) {
    MpWeights W(L);
    int GS = (L.G + L.V) | 1;
    int per_warp = backward ? ((L.H + 3) & ~3) + 4 * 12 + 32 * 4 + 2 * 32
                            : 32 * GS + 32 * 4 + 32;
    return sizeof(float) * (W.total + kWarps * per_warp);
}

template <typename F>
void dispatch_mp(const MpLayerArgs& L, F&& f) {
    int GV = L.G + L.V;
    if (L.K <= 17 && GV <= 16) f(std::integral_constant<int, 17>{}, std::integral_constant<int, 16>{});
    else if (L.K <= 17) f(std::integral_constant<int, 17>{}, std::integral_constant<int, 32>{});
    else f(std::integral_constant<int, 33>{}, std::integral_constant<int, 32>{});
}

}  // namespace

void mp_forward_edges(const MpLayerArgs& L, int n_atoms, const EdgeList& rad, const int* types,
                      const float* vs, float* msg, float* vec, float* gv, float* sg,
                      cudaStream_t stream) {
    if (n_atoms == 0) return;
    size_t bytes = mp_smem_bytes(L, false);
    int blocks = (n_atoms + kWarps - 1) / kWarps;
    dispatch_mp(L, [&](auto km, auto gm) {
        constexpr int KM = decltype(km)::value, GM = decltype(gm)::value;
        if (bytes > 48 * 1024)
            RUNE_CUDA_TRY(cudaFuncSetAttribute(k_mp_forward_edges<KM, GM>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)bytes));
        RUNE_KERNEL("k_mp_forward_edges", stream,
                    k_mp_forward_edges<KM, GM><<<blocks, kWarps * 32, bytes, stream>>>(
                        n_atoms, L, rad, types, vs, msg, vec, gv, sg));
    });
    RUNE_LAUNCH_CHECK();
}

void mp_node_forward(const MpLayerArgs& L, int n_atoms, const float* msg, const float* vec,
                     float* uin, float* rho_m, float* mixed, cudaStream_t stream) {
    if (n_atoms == 0) return;
    RUNE_KERNEL("k_mp_node_forward", stream,
                k_mp_node_forward<<<(n_atoms * 32 + 255) / 256, 256, 0, stream>>>(
                    n_atoms, L, msg, vec, uin, rho_m, mixed));
    RUNE_LAUNCH_CHECK();
}

void mp_node_backward(const MpLayerArgs& L, int n_atoms, const float* msg, const float* rho_m,
                      const float* mixed, const float* duin, float* dmsg, float* dvec,
                      cudaStream_t stream) {
    if (n_atoms == 0) return;
    RUNE_KERNEL("k_mp_node_backward", stream,
                k_mp_node_backward<<<(n_atoms * 32 + 255) / 256, 256, 0, stream>>>(
                    n_atoms, L, msg, rho_m, mixed, duin, dmsg, dvec));
    RUNE_LAUNCH_CHECK();
}

void mp_backward_edges(const MpLayerArgs& L, int n_atoms, const EdgeList& rad, const int* types,
                       const float* vs, const float* dmsg, const float* dvec, const float* gv,
                       const float* sg, float4* edge_grad, float* dvs, cudaStream_t stream) {
    if (n_atoms == 0) return;
    size_t bytes = mp_smem_bytes(L, true);
    int blocks = (n_atoms + kWarps - 1) / kWarps;
    dispatch_mp(L, [&](auto km, auto gm) {
        constexpr int KM = decltype(km)::value, GM = decltype(gm)::value;
        if (bytes > 48 * 1024)
            RUNE_CUDA_TRY(cudaFuncSetAttribute(k_mp_backward_edges<KM, GM>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)bytes));
        RUNE_KERNEL("k_mp_backward_edges", stream,
                    k_mp_backward_edges<KM, GM><<<blocks, kWarps * 32, bytes, stream>>>(
                        n_atoms, L, rad, types, vs, dmsg, dvec, gv, sg, edge_grad, dvs));
    });
    RUNE_LAUNCH_CHECK();
}

}  // namespace rune
