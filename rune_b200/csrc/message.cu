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
// The forward stores gate and vg per edge. The backward evaluates, for each centre i, the
// adjoint of every edge of its row (recomputing z) and the edge-vector gradient dE/dr_e; the
// transposed sums into neighbours (dv_j, dsrc_j) are pulled by atom j's warp through the
// reverse-edge index, reading the stored gates of the reverse edges. No atomics.
//
// Thread mapping: one warp per centre atom; edges in chunks of 32 (one lane per edge for
// geometry), contractions with lanes over output channels.

#include "basis.cuh"
#include "engine.cuh"

namespace rune {

namespace {

constexpr int kWarps = 4;

struct MpSmem {
    int sb, sdb, sz, sdz, sgv, sgate, sgeo, sidx, smsg, svec, total;
    __host__ __device__ MpSmem(const MpLayerArgs& L, bool backward) {
        int GV = L.G + L.V;
        sb = 0;
        sdb = sb + 32 * L.K;
        sz = sdb + (backward ? 32 * L.K : 0);
        sdz = sz + 32 * L.M;
        sgv = sdz + (backward ? 32 * L.M : 0);
        sgate = sgv + 32 * GV;             // backward: d(logits)
        sgeo = sgate + (backward ? 32 * GV : 0);
        sidx = sgeo + 32 * 8;              // ux uy uz cut dcut inv r
        smsg = sidx + 32 * 2;              // j, pair (as int)
        svec = smsg + L.H + (backward ? L.H : 0);
        total = svec + 2 * 3 * (L.V > 0 ? L.V : 1);
        total = (total + 3) & ~3;
    }
};

__device__ __forceinline__ int block_weights_floats(const MpLayerArgs& L) {
    return L.M * L.K + (L.G + L.V) * L.M + (L.G + L.V);
}

// Load the per-block copies of W_e (basis columns), [W_g; W_vg] and [b_g; b_vg].
__device__ __forceinline__ void load_block_weights(const MpLayerArgs& L, float* wk, float* wgv,
                                                   float* bgv) {
    for (int o = threadIdx.x; o < L.M * L.K; o += blockDim.x) wk[o] = L.we_k[o];
    for (int o = threadIdx.x; o < (L.G + L.V) * L.M; o += blockDim.x) wgv[o] = L.wgv[o];
    for (int o = threadIdx.x; o < L.G + L.V; o += blockDim.x) bgv[o] = L.bgv[o];
}

// Phase shared by forward and backward: geometry, basis and the edge MLP for one chunk.
__device__ __forceinline__ void edge_chunk_mlp(const MpLayerArgs& L, const EdgeList& rad,
                                               const int* types, int ti, int row, int base,
                                               int nv, int lane, const float* wk, float* sb,
                                               float* sdb, float* sz, float* sdz, float* sgeo,
                                               int* sidx) {
    if (lane < nv) {
        float4 e = rad.e[row + base + lane];
        int j = edge_j(e);
        float r = (float)sqrt((double)e.x * e.x + (double)e.y * e.y + (double)e.z * e.z);
        float inv = 1.0f / fmaxf(r, 1.0e-12f);
        float cut, dcut;
        cheb_masked(r, L.rc, L.K, sb + lane * L.K, sdb ? sdb + lane * L.K : nullptr, cut, dcut);
        float* g = sgeo + lane * 8;
        g[0] = e.x * inv; g[1] = e.y * inv; g[2] = e.z * inv;
        g[3] = cut; g[4] = dcut; g[5] = inv; g[6] = r;
        sidx[2 * lane] = j;
        sidx[2 * lane + 1] = ti * L.T + types[j];
    }
    __syncwarp();
    for (int o = lane; o < nv * L.M; o += 32) {
        int ee = o / L.M, m = o - ee * L.M;
        const float* bb = sb + ee * L.K;
        const float* w = wk + m * L.K;
        float pre = __ldg(L.pb + (size_t)sidx[2 * ee + 1] * L.M + m);
        for (int k = 0; k < L.K; ++k) pre += w[k] * bb[k];
        float y, dy;
        activation(L.act, pre, y, dy);
        sz[ee * L.M + m] = y;
        if (sdz) sdz[ee * L.M + m] = dy;
    }
    __syncwarp();
}

__global__ void __launch_bounds__(kWarps * 32)
k_mp_forward_edges(int n_atoms, MpLayerArgs L, EdgeList rad, const int* __restrict__ types,
                   const float* __restrict__ vs, float* __restrict__ msg_out,
                   float* __restrict__ vec_out, float* __restrict__ gv_out) {
    extern __shared__ float smem[];
    int GV = L.G + L.V, HV = L.H + L.V;
    float* wk = smem;
    float* wgv = wk + L.M * L.K;
    float* bgv = wgv + GV * L.M;
    int wfl = (block_weights_floats(L) + 3) & ~3;
    load_block_weights(L, wk, wgv, bgv);
    __syncthreads();
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int i = blockIdx.x * kWarps + warp;
    MpSmem S(L, false);
    float* sm = smem + wfl + warp * S.total;
    float* sb = sm + S.sb;
    float* sz = sm + S.sz;
    float* sgv = sm + S.sgv;
    float* sgeo = sm + S.sgeo;
    int* sidx = reinterpret_cast<int*>(sm + S.sidx);
    float* smsg = sm + S.smsg;
    float* svec = sm + S.svec;
    if (i >= n_atoms) return;
    int ti = types[i];
    int gw = L.H / L.G;
    for (int c = lane; c < L.H; c += 32) smsg[c] = 0.0f;
    for (int c = lane; c < 3 * L.V; c += 32) svec[c] = 0.0f;
    int row = rad.row_ptr[i], cnt = rad.cnt[i];
    for (int base = 0; base < cnt; base += 32) {
        int nv = min(32, cnt - base);
        edge_chunk_mlp(L, rad, types, ti, row, base, nv, lane, wk, sb, nullptr, sz, nullptr,
                       sgeo, sidx);
        // gates: sigmoid(W z + b) * cut
        for (int o = lane; o < nv * GV; o += 32) {
            int ee = o / GV, q = o - ee * GV;
            const float* w = wgv + q * L.M;
            const float* zz = sz + ee * L.M;
            float lg = bgv[q];
            for (int m = 0; m < L.M; ++m) lg += w[m] * zz[m];
            float g = sigmoidf_(lg) * sgeo[ee * 8 + 3];
            sgv[ee * GV + q] = g;
            gv_out[(size_t)(row + base + ee) * GV + q] = g;
        }
        __syncwarp();
        // scalar messages: lanes over channels, neighbour values gathered (coalesced)
        for (int c = lane; c < L.H; c += 32) {
            int g = c / gw;
            float acc = smsg[c];
            for (int ee = 0; ee < nv; ++ee)
                acc += sgv[ee * GV + g] * __ldg(vs + (size_t)sidx[2 * ee] * HV + c);
            smsg[c] = acc;
        }
        // vector branch: lanes over (channel, axis)
        for (int o = lane; o < 3 * L.V; o += 32) {
            int k = o / 3, x = o - 3 * k;
            float acc = svec[o];
            for (int ee = 0; ee < nv; ++ee)
                acc += sgv[ee * GV + L.G + k] * __ldg(vs + (size_t)sidx[2 * ee] * HV + L.H + k) *
                       sgeo[ee * 8 + x];
            svec[o] = acc;
        }
        __syncwarp();
    }
    for (int c = lane; c < L.H; c += 32) msg_out[(size_t)i * L.H + c] = smsg[c];
    for (int o = lane; o < 3 * L.V; o += 32) vec_out[(size_t)i * 3 * L.V + o] = svec[o];
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

// Adjoint of the edge part. Centre side: for each edge e = (i <- j) of row i, dE/dr_e is added
// to edge_grad[e]. Neighbour side (pull): dv_i, dsrc_i from the reverse edges of row i.
__global__ void __launch_bounds__(kWarps * 32)
k_mp_backward_edges(int n_atoms, MpLayerArgs L, EdgeList rad, const int* __restrict__ types,
                    const float* __restrict__ vs, const float* __restrict__ dmsg,
                    const float* __restrict__ dvec, const float* __restrict__ gv,
                    float4* __restrict__ edge_grad, float* __restrict__ dvs) {
    extern __shared__ float smem[];
    int GV = L.G + L.V, HV = L.H + L.V;
    float* wk = smem;
    float* wgv = wk + L.M * L.K;
    float* bgv = wgv + GV * L.M;
    int wfl = (block_weights_floats(L) + 3) & ~3;
    load_block_weights(L, wk, wgv, bgv);
    __syncthreads();
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int i = blockIdx.x * kWarps + warp;
    MpSmem S(L, true);
    float* sm = smem + wfl + warp * S.total;
    float* sb = sm + S.sb;
    float* sdb = sm + S.sdb;
    float* sz = sm + S.sz;
    float* sdz = sm + S.sdz;
    float* ssg = sm + S.sgv;    // sigmoid values (no cut)
    float* sdl = sm + S.sgate;  // d logits
    float* sgeo = sm + S.sgeo;
    int* sidx = reinterpret_cast<int*>(sm + S.sidx);
    float* sdm = sm + S.smsg;   // dmsg of atom i [H]
    float* sdv = sdm + L.H;     // dv accumulator [H]
    float* sdvec = sm + S.svec; // dvec of atom i [3V]
    float* sdsrc = sdvec + 3 * (L.V > 0 ? L.V : 1);  // dsrc accumulator [V] (3V room)
    if (i >= n_atoms) return;
    int ti = types[i];
    int gw = L.H / L.G;
    for (int c = lane; c < L.H; c += 32) {
        sdm[c] = dmsg[(size_t)i * L.H + c];
        sdv[c] = 0.0f;
    }
    for (int o = lane; o < 3 * L.V; o += 32) {
        sdvec[o] = dvec[(size_t)i * 3 * L.V + o];
        sdsrc[o] = 0.0f;
    }
    __syncwarp();
    int row = rad.row_ptr[i], cnt = rad.cnt[i];
    for (int base = 0; base < cnt; base += 32) {
        int nv = min(32, cnt - base);
        edge_chunk_mlp(L, rad, types, ti, row, base, nv, lane, wk, sb, sdb, sz, sdz, sgeo, sidx);
        // sigmoids
        for (int o = lane; o < nv * GV; o += 32) {
            int ee = o / GV, q = o - ee * GV;
            const float* w = wgv + q * L.M;
            const float* zz = sz + ee * L.M;
            float lg = bgv[q];
            for (int m = 0; m < L.M; ++m) lg += w[m] * zz[m];
            ssg[ee * GV + q] = sigmoidf_(lg);
        }
        __syncwarp();
        // d gate (groups) and d vector-gate; d logits = d gate * cut * s (1 - s)
        for (int o = lane; o < nv * GV; o += 32) {
            int ee = o / GV, q = o - ee * GV;
            int j = sidx[2 * ee];
            float dg;
            if (q < L.G) {
                dg = 0.0f;
                const float* vj = vs + (size_t)j * HV + q * gw;
                for (int c = 0; c < gw; ++c) dg += sdm[q * gw + c] * __ldg(vj + c);
            } else {
                int k = q - L.G;
                const float* u = sgeo + ee * 8;
                float proj = sdvec[3 * k] * u[0] + sdvec[3 * k + 1] * u[1] + sdvec[3 * k + 2] * u[2];
                dg = __ldg(vs + (size_t)j * HV + L.H + k) * proj;
            }
            sdl[ee * GV + q] = dg;  // the gate adjoint; turned into d logits below
        }
        __syncwarp();
        // per edge (lane = edge): cutoff adjoint, unit-vector adjoint, d logits in place
        float dcut_e = 0.0f, du0 = 0.0f, du1 = 0.0f, du2 = 0.0f;
        if (lane < nv) {
            int ee = lane;
            int j = sidx[2 * ee];
            float cut = sgeo[ee * 8 + 3];
            for (int q = 0; q < GV; ++q) {
                float s = ssg[ee * GV + q];
                float dg = sdl[ee * GV + q];
                dcut_e += dg * s;
                sdl[ee * GV + q] = dg * cut * s * (1.0f - s);
            }
            for (int k = 0; k < L.V; ++k) {
                float a = ssg[ee * GV + L.G + k] * cut * __ldg(vs + (size_t)j * HV + L.H + k);
                du0 += a * sdvec[3 * k];
                du1 += a * sdvec[3 * k + 1];
                du2 += a * sdvec[3 * k + 2];
            }
        }
        __syncwarp();
        // dz = W_gv^T dl ; dpre = dz * act'
        for (int o = lane; o < nv * L.M; o += 32) {
            int ee = o / L.M, m = o - ee * L.M;
            float s = 0.0f;
            for (int q = 0; q < GV; ++q) s += wgv[q * L.M + m] * sdl[ee * GV + q];
            sdz[ee * L.M + m] *= s;  // now d pre-activation
        }
        __syncwarp();
        // d basis: db_k = sum_m W_e[m, k] dpre[m]; then dd = sum_k db_k b'_k + dcut * cut'
        if (lane < nv) {
            int ee = lane;
            const float* dp = sdz + ee * L.M;
            const float* dbk = sdb + ee * L.K;
            float dd = 0.0f;
            for (int k = 0; k < L.K; ++k) {
                float s = 0.0f;
                for (int m = 0; m < L.M; ++m) s += wk[m * L.K + k] * dp[m];
                dd += s * dbk[k];
            }
            const float* g = sgeo + ee * 8;
            dd += dcut_e * g[4];
            float pu = du0 * g[0] + du1 * g[1] + du2 * g[2];
            float inv = g[5];
            float4 G = edge_grad[row + base + ee];
            G.x += dd * g[0] + (du0 - pu * g[0]) * inv;
            G.y += dd * g[1] + (du1 - pu * g[1]) * inv;
            G.z += dd * g[2] + (du2 - pu * g[2]) * inv;
            edge_grad[row + base + ee] = G;
        }
        __syncwarp();
    }
    // ---- neighbour side: pull the reverse edges' contributions into dv_i and dsrc_i
    for (int base = 0; base < cnt; base += 32) {
        int nv = min(32, cnt - base);
        if (lane < nv) {
            int e = row + base + lane;
            float4 ed = rad.e[e];
            float r = (float)sqrt((double)ed.x * ed.x + (double)ed.y * ed.y + (double)ed.z * ed.z);
            float inv = 1.0f / fmaxf(r, 1.0e-12f);
            float* g = sgeo + lane * 8;
            g[0] = -ed.x * inv; g[1] = -ed.y * inv; g[2] = -ed.z * inv;  // unit of the reverse edge
            sidx[2 * lane] = edge_j(ed);
            sidx[2 * lane + 1] = rad.rev[e];
        }
        __syncwarp();
        for (int c = lane; c < L.H; c += 32) {
            int g = c / gw;
            float acc = sdv[c];
            for (int ee = 0; ee < nv; ++ee)
                acc += __ldg(gv + (size_t)sidx[2 * ee + 1] * GV + g) *
                       __ldg(dmsg + (size_t)sidx[2 * ee] * L.H + c);
            sdv[c] = acc;
        }
        for (int k = lane; k < L.V; k += 32) {
            float acc = sdsrc[k];
            for (int ee = 0; ee < nv; ++ee) {
                int j = sidx[2 * ee];
                const float* dvj = dvec + (size_t)j * 3 * L.V + 3 * k;
                const float* u = sgeo + ee * 8;
                float proj = __ldg(dvj) * u[0] + __ldg(dvj + 1) * u[1] + __ldg(dvj + 2) * u[2];
                acc += __ldg(gv + (size_t)sidx[2 * ee + 1] * GV + L.G + k) * proj;
            }
            sdsrc[k] = acc;
        }
        __syncwarp();
    }
    for (int c = lane; c < L.H; c += 32) dvs[(size_t)i * HV + c] = sdv[c];
    for (int k = lane; k < L.V; k += 32) dvs[(size_t)i * HV + L.H + k] = sdsrc[k];
}

size_t mp_smem_bytes(const MpLayerArgs& L, bool backward) {
    MpSmem S(L, backward);
    int wfl = (L.M * L.K + (L.G + L.V) * L.M + (L.G + L.V) + 3) & ~3;
    return sizeof(float) * (wfl + kWarps * S.total);
}

}  // namespace

void mp_forward_edges(const MpLayerArgs& L, int n_atoms, const EdgeList& rad, const int* types,
                      const float* vs, float* msg, float* vec, float* gv, cudaStream_t stream) {
    if (n_atoms == 0) return;
    size_t bytes = mp_smem_bytes(L, false);
    if (bytes > 48 * 1024)
        RUNE_CUDA_TRY(cudaFuncSetAttribute(k_mp_forward_edges,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    int blocks = (n_atoms + kWarps - 1) / kWarps;
    RUNE_KERNEL("k_mp_forward_edges", stream,
                k_mp_forward_edges<<<blocks, kWarps * 32, bytes, stream>>>(n_atoms, L, rad, types,
                                                                           vs, msg, vec, gv));
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
                       float4* edge_grad, float* dvs, cudaStream_t stream) {
    if (n_atoms == 0) return;
    size_t bytes = mp_smem_bytes(L, true);
    if (bytes > 48 * 1024)
        RUNE_CUDA_TRY(cudaFuncSetAttribute(k_mp_backward_edges,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    int blocks = (n_atoms + kWarps - 1) / kWarps;
    RUNE_KERNEL("k_mp_backward_edges", stream,
                k_mp_backward_edges<<<blocks, kWarps * 32, bytes, stream>>>(
                    n_atoms, L, rad, types, vs, dmsg, dvec, gv, edge_grad, dvs));
    RUNE_LAUNCH_CHECK();
}

}  // namespace rune
