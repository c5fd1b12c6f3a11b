// C ABI of the rune_b200 engine: model set-up, workspace, and the evaluation pipeline.
//
// Pipeline of one evaluation (rune/mobius/model.py:307-393, rune/nep/model.py:87-155):
//   neighbour list (device cell list, or the caller's padded lists)
//   -> descriptor forward (+ NEP element network, fused)
//   -> Möbius: per-atom dense network forward and analytic backward (dense.cu)
//   -> angular adjoints -> force / virial kernel (pull form, no atomics)
//   -> per-structure energy and virial sums in float64 (fixed-order, deterministic).

#include <cstdlib>
#include <cstring>
#include <memory>
#include <cstdio>
#include <mutex>

#include "engine.cuh"

namespace rune {

namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string& message) { g_last_error = message; }

const float* Engine::tensor(const std::string& name) const {
    auto it = offsets.find(name);
    if (it == offsets.end()) throw Error(RUNE_ERR_INVALID, "missing tensor: " + name);
    return blob + it->second;
}

void Engine::check_flags(unsigned int flags, cudaStream_t stream) {
    if (!flags) return;
    RUNE_CUDA_TRY(cudaMemsetAsync(d_flags, 0, sizeof(unsigned int), stream));
    RUNE_CUDA_TRY(cudaStreamSynchronize(stream));
    if (flags & 1u)
        throw Error(RUNE_ERR_TYPE, "Atom type index outside the model's element list.");
    if (flags & 2u) throw Error(RUNE_ERR_INVALID, "Positions must be finite.");
    if (flags & 4u) throw Error(RUNE_ERR_INVALID, "Neighbor index out of range.");
    if (flags & 8u)
        throw Error(RUNE_ERR_INVALID,
                    "Neighbor lists must be symmetric: every (i, j, offset) needs (j, i, -offset).");
    if (flags & 32u)
        throw Error(RUNE_ERR_CUDA, "A device-side copy did not complete in time; the results "
                                   "of this call are invalid.");
}

void* Engine::stage_upload(const void* src, size_t bytes, cudaStream_t stream) {
    size_t at = (staging.off + 63) & ~size_t(63);
    if (staging.base && d_mirror && at + bytes <= staging.cap) {
        std::memcpy(staging.base + at, src, bytes);
        staging.off = at + bytes;
        stage_first = std::min(stage_first, at);
        return d_mirror + at;
    }
    // no room: a pageable copy into the workspace (it synchronises the stream); remember the
    // size so the staging buffer grows after this call
    staging_want = std::max(staging_want, at + bytes);
    void* dst = ws.take(bytes);
    RUNE_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, stream));
    return dst;
}

void Engine::flush_uploads(cudaStream_t stream) {
    if (stage_first >= staging.off) return;
    RUNE_CUDA_TRY(cudaMemcpyAsync(d_mirror + stage_first, staging.base + stage_first,
                                  staging.off - stage_first, cudaMemcpyHostToDevice, stream));
    stage_first = ~size_t(0);
}

namespace {

// ----------------------------------------------------------------------------- reductions
// Per-atom energies (model + ZBL) and partial sums (energy + 9 virial) over fixed chunks of
// each structure's atoms; block c is chunk c, found in chunk_ptr by binary search.
// Per-chunk sums (fixed order: each thread strides its atoms, then a fixed shuffle tree per
// warp and the warps in order) of the per-atom energy and virial; per-atom energies written.
constexpr int kSumThreads = 256;
__global__ void __launch_bounds__(kSumThreads)
k_chunk_partials(int n_structures, const int* __restrict__ chunk_ptr,
                 const int* __restrict__ atom_ptr, int chunk, const double* __restrict__ e_model,
                 const double* __restrict__ e_zbl, float* __restrict__ energies,
                 const double* __restrict__ vir, double* __restrict__ part) {
    __shared__ double red[kSumThreads / 32][10];
    int c = blockIdx.x;
    int lo = 0, hi = n_structures - 1;
    while (lo < hi) {  // last structure whose first chunk <= c
        int mid = (lo + hi + 1) >> 1;
        if (chunk_ptr[mid] <= c) lo = mid; else hi = mid - 1;
    }
    int a0 = atom_ptr[lo] + (c - chunk_ptr[lo]) * chunk;
    int a1 = min(a0 + chunk, atom_ptr[lo + 1]);
    double acc[10];
#pragma unroll
    for (int k = 0; k < 10; ++k) acc[k] = 0.0;
    for (int a = a0 + threadIdx.x; a < a1; a += blockDim.x) {
        double e = e_model[a] + e_zbl[a];
        if (energies) energies[a] = (float)e;
        acc[0] += e;
        if (vir)
#pragma unroll
            for (int k = 0; k < 9; ++k) acc[1 + k] += vir[(size_t)a * 9 + k];
    }
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int k = 0; k < 10; ++k) acc[k] = warp_sum(acc[k]);
    if (lane == 0)
#pragma unroll
        for (int k = 0; k < 10; ++k) red[warp][k] = acc[k];
    __syncthreads();
    if (threadIdx.x < 10) {
        double v = 0.0;
        for (int w = 0; w < kSumThreads / 32; ++w) v += red[w][threadIdx.x];
        part[(size_t)c * 10 + threadIdx.x] = v;
    }
}

// Per-structure totals from the chunk partials: a warp per structure, lanes over its chunks
// (fixed order: lane-strided sums, then a fixed shuffle tree).
__global__ void k_structure_sum(int n_structures, const int* __restrict__ chunk_ptr,
                                const double* __restrict__ part, double* __restrict__ energy,
                                double* __restrict__ virial) {
    int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (s >= n_structures) return;
    double acc[10];
#pragma unroll
    for (int k = 0; k < 10; ++k) acc[k] = 0.0;
    for (int c = chunk_ptr[s] + lane; c < chunk_ptr[s + 1]; c += 32)
#pragma unroll
        for (int k = 0; k < 10; ++k) acc[k] += part[(size_t)c * 10 + k];
#pragma unroll
    for (int k = 0; k < 10; ++k) acc[k] = warp_sum(acc[k]);
    if (lane == 0) {
        if (energy) energy[s] = acc[0];
        if (virial)
            for (int k = 0; k < 9; ++k) virial[(size_t)s * 9 + k] = acc[1 + k];
    }
}

constexpr int kChunk = 1024;

}  // namespace

// ----------------------------------------------------------------------------- Möbius dense
struct MlpBuffers {
    float* h0;      // [N, H] after input projection
    float* hb;      // [blocks + 1][N, H] residual stream (hb[b] = input of block b)
    float* rho;     // [blocks][N]
    float* z;       // [N, F]
    float* dz;      // [blocks][N, F] activation derivative
    float* dh;      // [N, H]
    float* tmp;     // [N, max(H, F)]
};

// One halo exchange of a domain call (nothing in a rehearsal or outside halo mode). Before the
// first exchange of an attempt the workspace must hold everything the attempt will take (the
// rehearsal measured it): growing it restarts the attempt, which is safe only while no
// exchange has been issued.
static void halo_exchange(Engine& eng, const DomainCall* dom, int op, float* rows, int width,
                          cudaStream_t stream) {
    if (!dom || !dom->halo || dom->rehearsal) return;
    if (dom->exchanges == 0 && eng.ws.cap < eng.halo_bytes) {
        eng.ws.want = eng.halo_bytes;
        throw Error(-1, "workspace");
    }
    ++dom->exchanges;
    int rc = dom->halo(dom->halo_ctx, op, rows, width, stream);
    if (rc != 0)
        throw Error(RUNE_ERR_STATE, "halo exchange hook failed (status " + std::to_string(rc) +
                                        ")");
}

// Forward and dX-only backward of the Möbius network: input projection, residual blocks,
// message blocks (MP), readout. Returns dq [N, D] (descriptor scaler applied) and accumulates
// the message blocks' edge-vector gradients into edge_grad (radial list).
//
// In a domain call only owned atoms have energies (the readout runs over them, the other rows
// of e_model and of the energy adjoint are zero), and EQ layer l runs its centre kernels over
// the prefix of atoms whose outputs later layers read (DomainCall::layer_centres); the rows it
// does not compute are zero, and its per-edge arrays cover only that prefix's rows (rows have
// a fixed stride on the device path).
static void mobius_network(Engine& eng, int N, const float* q, const float* moments,
                           const int* types, const NeighborData& nd, double* e_model, float* dq,
                           float4* edge_grad, float* moment_grad, cudaStream_t stream,
                           const DomainCall* dom) {
    const rune_model_config& c = eng.cfg;
    int H = c.hidden_dim, F = c.ffn_dim, B = c.blocks, D = eng.D;
    int NL = (int)eng.mp.size();
    float eps = (float)c.norm_eps;
    // Rows the dense stem (input projection, residual blocks) must produce: in a domain call
    // without MP blocks, the atoms within the message shells (owned atoms for Local); the
    // descriptor adjoint of the other rows is zero.
    int R0 = N;
    const bool halo = dom && dom->halo;
    if (halo)
        R0 = dom->n_owned;  // the owners of ghost rows compute them; the halo brings them
    else if (dom && NL == 0)
        R0 = dom->shell_end[std::min<size_t>(eng.eq.size(), dom->shell_end.size() - 1)];
    // residual stream: hb[0..B] residual blocks, then hb[B+1..B+NL] message blocks
    float* hb = eng.ws.take_n<float>((size_t)(B + NL + (int)eng.eq.size() + 1) * N * H);
    float* rho = eng.ws.take_n<float>((size_t)(B > 0 ? B : 1) * N);
    float* z = eng.ws.take_n<float>((size_t)N * F);
    float* dz = eng.ws.take_n<float>((size_t)(B > 0 ? B : 1) * N * F);
    float* dh = eng.ws.take_n<float>((size_t)N * H);
    float* tmp = eng.ws.take_n<float>((size_t)N * std::max(H, F));
    float* dup = eng.ws.take_n<float>((size_t)N * H);
    // few rows (small structures): split-K scratch for the dense layers (not in static calls,
    // whose scratch is fixed)
    struct SplitScope {
        ~SplitScope() { set_gemm_split_scratch(nullptr, 0); }
    } split_scope;
    if (!eng.static_call && N > 0 && N <= 64 * 74) {
        size_t cap = (size_t)N * 4096;
        set_gemm_split_scratch(eng.ws.take_n<double>(cap), cap);
    }
    // h0 = q @ (scaler * W_in^T) + b + emb[t]
    {
        GemmEpilogue ep;
        ep.bias = eng.input_projection.b;
        ep.emb = eng.embedding;
        ep.types = types;
        gemm(R0, H, D, q, D, eng.input_projection.wt, H, hb, H, ep, stream);
    }
    for (int b = 0; b < B; ++b) {
        float* h = hb + (size_t)b * N * H;
        float* hn = hb + (size_t)(b + 1) * N * H;
        row_rms(R0, H, h, H, eps, rho + (size_t)b * N, stream);
        GemmEpilogue e1;
        e1.row_scale = rho + (size_t)b * N;
        e1.bias = eng.ffn1[b].b;
        e1.act = c.activation;
        e1.dact = dz + (size_t)b * N * F;
        gemm(R0, F, H, h, H, eng.ffn1[b].wt, F, z, F, e1, stream);
        GemmEpilogue e2;
        e2.bias = eng.ffn2[b].b;
        e2.residual = h;
        gemm(R0, H, F, z, F, eng.ffn2[b].wt, H, hn, H, e2, stream);
    }
    // ---- MP message blocks
    struct MpSaved {
        float *rho_in, *vs, *msg, *rho_m, *mixed, *gv, *sg, *dact;
    };
    std::vector<MpSaved> saved(NL);
    int E = nd.total_edges;
    for (int l = 0; l < NL; ++l) {
        const MpLayer& L = eng.mp[l];
        const MpLayerArgs& a = L.args;
        int HV = a.H + a.V, GV = a.G + a.V;
        float* h = hb + (size_t)(B + l) * N * H;
        float* hn = hb + (size_t)(B + l + 1) * N * H;
        MpSaved& sv = saved[l];
        sv.rho_in = eng.ws.take_n<float>(N);
        sv.vs = eng.ws.take_n<float>((size_t)N * HV);
        sv.msg = eng.ws.take_n<float>((size_t)N * H);
        sv.rho_m = eng.ws.take_n<float>(N);
        sv.mixed = eng.ws.take_n<float>((size_t)N * 3 * std::max(a.V, 1));
        sv.gv = eng.ws.take_n<float>((size_t)(E + 1) * GV);
        sv.sg = eng.ws.take_n<float>((size_t)(E + 1) * GV);
        sv.dact = eng.ws.take_n<float>((size_t)N * a.M);
        float* vec = eng.ws.take_n<float>((size_t)N * 3 * std::max(a.V, 1));
        float* uin = eng.ws.take_n<float>((size_t)N * HV);
        float* zu = eng.ws.take_n<float>((size_t)N * a.M);
        row_rms(N, H, h, H, eps, sv.rho_in, stream);
        GemmEpilogue ev;
        ev.row_scale = sv.rho_in;
        gemm(N, HV, H, h, H, L.vs.wt, HV, sv.vs, HV, ev, stream);
        mp_forward_edges(a, N, nd.radial, types, sv.vs, sv.msg, vec, sv.gv, sv.sg, stream);
        mp_node_forward(a, N, sv.msg, vec, uin, sv.rho_m, sv.mixed, stream);
        GemmEpilogue e1;
        e1.bias = L.upd1.b;
        e1.act = c.activation;
        e1.dact = sv.dact;
        gemm(N, a.M, HV, uin, HV, L.upd1.wt, a.M, zu, a.M, e1, stream);
        GemmEpilogue e2;
        e2.bias = L.upd2.b;
        e2.residual = h;
        gemm(N, H, a.M, zu, a.M, L.upd2.wt, H, hn, H, e2, stream);
    }
    // ---- EQ blocks
    int NQ = (int)eng.eq.size();
    struct EqSaved {
        float *rho_in, *abv, *D, *mixed, *msg, *rho_m, *dn, *gva, *dact;
        int centres;  // atoms whose layer outputs are read later (centre kernels)
        int rows;     // atoms whose layer inputs are read (the centres' neighbours)
    };
    std::vector<EqSaved> qs(NQ);
    // edge slots of the rows of the first `a` atoms
    auto prefix_edges = [&](int a) -> size_t {
        return a == N ? (size_t)E : (size_t)a * (size_t)(E / std::max(N, 1));
    };
    int max_centres = 0;
    for (int l = 0; l < NQ; ++l) {
        qs[l].centres = dom ? dom->layer_centres(l, NQ) : N;
        // halo mode: every row of a layer's input is present (ghost rows by exchange)
        qs[l].rows = halo ? N : l == 0 ? R0 : qs[l - 1].centres;
        max_centres = std::max(max_centres, qs[l].centres);
    }
    if (NQ) {
        const EqLayerArgs& a0 = eng.eq[0].args;
        int DC = a0.Ce * a0.Cl;
        float* D = eng.ws.take_n<float>((size_t)N * DC);
        eq_encode(a0, R0, eng.desc.na, eng.desc.C, eng.eq_proj, moments, D, stream);
        if (halo) {
            halo_exchange(eng, dom, RUNE_HALO_FILL, hb + (size_t)(B + NL) * N * H, H, stream);
            halo_exchange(eng, dom, RUNE_HALO_FILL, D, DC, stream);
        }
        for (int l = 0; l < NQ; ++l) {
            const EqLayer& L = eng.eq[l];
            const EqLayerArgs& a = L.args;
            int LC = a.Le * a.Ce, HU = H + LC, W3 = 2 * a.M + H;
            float* h = hb + (size_t)(B + NL + l) * N * H;
            float* hn = hb + (size_t)(B + NL + l + 1) * N * H;
            EqSaved& sv = qs[l];
            sv.D = D;
            sv.rho_in = eng.ws.take_n<float>(N);
            sv.abv = eng.ws.take_n<float>((size_t)N * W3);
            sv.mixed = eng.ws.take_n<float>((size_t)N * DC);
            sv.msg = eng.ws.take_n<float>((size_t)N * H);
            sv.rho_m = eng.ws.take_n<float>(N);
            sv.dn = eng.ws.take_n<float>((size_t)N * DC);
            sv.gva = eng.ws.take_n<float>((prefix_edges(sv.centres) + 1) * (a.G + LC));
            sv.dact = eng.ws.take_n<float>((size_t)N * a.M);
            float* uin = eng.ws.take_n<float>((size_t)N * HU);
            float* zu = eng.ws.take_n<float>((size_t)N * a.M);
            row_rms(sv.rows, H, h, H, eps, sv.rho_in, stream);
            GemmEpilogue ev;
            ev.row_scale = sv.rho_in;
            gemm(sv.rows, W3, H, h, H, L.nodes.wt, W3, sv.abv, W3, ev, stream);
            eq_mix(a, sv.rows, D, sv.mixed, stream);
            eq_forward_edges(a, sv.centres, nd.radial, types, sv.abv, D, sv.mixed, sv.msg, sv.dn,
                             sv.gva, eng.d_flags, stream);
            if (sv.centres < N) {
                size_t rows = (size_t)(N - sv.centres);
                RUNE_CUDA_TRY(cudaMemsetAsync(sv.msg + (size_t)sv.centres * H, 0,
                                              sizeof(float) * rows * H, stream));
                RUNE_CUDA_TRY(cudaMemsetAsync(sv.dn + (size_t)sv.centres * DC, 0,
                                              sizeof(float) * rows * DC, stream));
            }
            eq_node_forward(a, sv.centres, sv.msg, sv.dn, uin, sv.rho_m, stream);
            GemmEpilogue e1;
            e1.bias = L.upd1.b;
            e1.act = c.activation;
            e1.dact = sv.dact;
            gemm(sv.centres, a.M, HU, uin, HU, L.upd1.wt, a.M, zu, a.M, e1, stream);
            GemmEpilogue e2;
            e2.bias = L.upd2.b;
            e2.residual = h;
            gemm(sv.centres, H, a.M, zu, a.M, L.upd2.wt, H, hn, H, e2, stream);
            D = sv.dn;
            if (halo && l + 1 < NQ) {
                halo_exchange(eng, dom, RUNE_HALO_FILL, hn, H, stream);
                halo_exchange(eng, dom, RUNE_HALO_FILL, sv.dn, DC, stream);
            }
        }
    }
    float* hout = hb + (size_t)(B + NL + NQ) * N * H;
    int n_owned = dom ? dom->n_owned : N;
    readout(n_owned, H, hout, types, eng.out_norm, eng.head_w, eng.head_b, eps, e_model, dh,
            stream);
    if (n_owned < N) {
        RUNE_CUDA_TRY(cudaMemsetAsync(e_model + n_owned, 0, sizeof(double) * (N - n_owned),
                                      stream));
        RUNE_CUDA_TRY(cudaMemsetAsync(dh + (size_t)n_owned * H, 0,
                                      sizeof(float) * (size_t)(N - n_owned) * H, stream));
    }
    if (NQ) {
        const EqLayerArgs& a0 = eng.eq[0].args;
        int DC = a0.Ce * a0.Cl;
        float* ddn = nullptr;  // adjoint of the last block's output direction state: zero
        float* dpre = eng.ws.take_n<float>((prefix_edges(max_centres) + 1) * a0.M);
        float* dpn = eng.ws.take_n<float>((prefix_edges(max_centres) + 1) * a0.Le * a0.Ce);
        for (int l = NQ - 1; l >= 0; --l) {
            const EqLayer& L = eng.eq[l];
            const EqLayerArgs& a = L.args;
            int LC = a.Le * a.Ce, HU = H + LC, W3 = 2 * a.M + H;
            float* h = hb + (size_t)(B + NL + l) * N * H;
            EqSaved& sv = qs[l];
            float* dzu = eng.ws.take_n<float>((size_t)N * a.M);
            float* duin = eng.ws.take_n<float>((size_t)N * HU);
            float* dmsg = eng.ws.take_n<float>((size_t)N * H);
            float* ddp = eng.ws.take_n<float>((size_t)N * DC);
            float* dabv = eng.ws.take_n<float>((size_t)N * W3);
            float* ddc = eng.ws.take_n<float>((size_t)N * DC);
            float* ddprev = eng.ws.take_n<float>((size_t)N * DC);
            GemmEpilogue e2;
            e2.mul = sv.dact;
            gemm(sv.centres, a.M, H, dh, H, L.upd2.w, a.M, dzu, a.M, e2, stream);
            GemmEpilogue e1;
            gemm(sv.centres, HU, a.M, dzu, a.M, L.upd1.w, HU, duin, HU, e1, stream);
            eq_node_backward(a, sv.centres, sv.msg, sv.rho_m, sv.dn, duin, ddn, dmsg, ddp,
                             stream);
            eq_backward_edges(a, sv.rows, sv.centres, nd.radial, types, sv.abv, sv.D, sv.mixed,
                              dmsg, ddp, sv.gva, dpre, dpn, edge_grad, dabv, ddc, ddprev,
                              eng.d_flags, stream);
            GemmEpilogue ev;
            gemm(sv.rows, H, W3, dabv, W3, L.nodes.w, H, dup, H, ev, stream);
            rms_backward_add(sv.rows, H, h, sv.rho_in, dup, dh, stream);
            ddn = ddprev;
            if (halo) {  // ghost rows' partial adjoints go to their owners
                halo_exchange(eng, dom, RUNE_HALO_REDUCE, dh, H, stream);
                halo_exchange(eng, dom, RUNE_HALO_REDUCE, ddprev, DC, stream);
            }
        }
        eq_encode_backward(a0, R0, eng.desc.na, eng.desc.C, eng.eq_proj, ddn, moment_grad,
                           stream);
        if (R0 < N)
            RUNE_CUDA_TRY(cudaMemsetAsync(moment_grad + (size_t)R0 * eng.desc.na * eng.desc.C,
                                          0,
                                          sizeof(float) * (size_t)(N - R0) * eng.desc.na *
                                              eng.desc.C,
                                          stream));
    }
    for (int l = NL - 1; l >= 0; --l) {
        const MpLayer& L = eng.mp[l];
        const MpLayerArgs& a = L.args;
        int HV = a.H + a.V;
        float* h = hb + (size_t)(B + l) * N * H;
        MpSaved& sv = saved[l];
        float* dzu = eng.ws.take_n<float>((size_t)N * a.M);
        float* duin = eng.ws.take_n<float>((size_t)N * HV);
        float* dmsg = eng.ws.take_n<float>((size_t)N * H);
        float* dvec = eng.ws.take_n<float>((size_t)N * 3 * std::max(a.V, 1));
        float* dvs = eng.ws.take_n<float>((size_t)N * HV);
        GemmEpilogue e2;
        e2.mul = sv.dact;
        gemm(N, a.M, H, dh, H, L.upd2.w, a.M, dzu, a.M, e2, stream);
        GemmEpilogue e1;
        gemm(N, HV, a.M, dzu, a.M, L.upd1.w, HV, duin, HV, e1, stream);
        mp_node_backward(a, N, sv.msg, sv.rho_m, sv.mixed, duin, dmsg, dvec, stream);
        mp_backward_edges(a, N, nd.radial, types, sv.vs, dmsg, dvec, sv.gv, sv.sg, edge_grad,
                          dvs, stream);
        GemmEpilogue ev;
        gemm(N, H, HV, dvs, HV, L.vs.w, H, dup, H, ev, stream);
        rms_backward_add(N, H, h, sv.rho_in, dup, dh, stream);
    }
    for (int b = B - 1; b >= 0; --b) {
        float* h = hb + (size_t)b * N * H;
        // dz = (dh @ W2) * act'
        GemmEpilogue e2;
        e2.mul = dz + (size_t)b * N * F;
        gemm(R0, F, H, dh, H, eng.ffn2[b].w, F, tmp, F, e2, stream);
        // du' = dz @ (W1 diag(gamma)) ; dh += RMSNorm^T(du')
        GemmEpilogue e1;
        gemm(R0, H, F, tmp, F, eng.ffn1[b].w, H, dup, H, e1, stream);
        rms_backward_add(R0, H, h, rho + (size_t)b * N, dup, dh, stream);
    }
    GemmEpilogue e0;
    gemm(R0, D, H, dh, H, eng.input_projection.w, D, dq, D, e0, stream);
    if (R0 < N)
        RUNE_CUDA_TRY(cudaMemsetAsync(dq + (size_t)R0 * D, 0, sizeof(float) * (size_t)(N - R0) * D,
                                      stream));
}

CallTables stage_call_tables(Engine& eng, int n_structures, const int* atom_ptr_host,
                             cudaStream_t stream) {
    std::vector<int> chunk_ptr(n_structures + 1, 0);
    for (int s = 0; s < n_structures; ++s) {
        int n = atom_ptr_host[s + 1] - atom_ptr_host[s];
        chunk_ptr[s + 1] = chunk_ptr[s] + (n + kChunk - 1) / kChunk;
    }
    CallTables ct;
    ct.n_chunks = chunk_ptr[n_structures];
    ct.atom_ptr = static_cast<const int*>(
        eng.stage_upload(atom_ptr_host, sizeof(int) * (n_structures + 1), stream));
    ct.chunk_ptr = static_cast<const int*>(
        eng.stage_upload(chunk_ptr.data(), sizeof(int) * (n_structures + 1), stream));
    return ct;
}

void evaluate(Engine& eng, NeighborData& nd, int n_atoms, int n_structures, const int* types,
              const CallTables& ct, const Outputs& out, cudaStream_t stream,
              const DomainCall* dom) {
    const rune_model_config& c = eng.cfg;
    if (nd.types) types = nd.types;
    const DescParams& p = eng.desc;
    int N = n_atoms;
    int n_owned = dom ? dom->n_owned : N;
    bool derivs = (out.flags & (RUNE_FORCES | RUNE_VIRIAL)) != 0;
    double* e_model = eng.ws.take_n<double>(N);
    double* e_zbl = eng.ws.take_n<double>(N);
    float4* dqr = eng.ws.take_n<float4>((size_t)N * p.npr);
    // Centre-side angular edge gradients, indexed like the angular list's edges (on the device
    // path the lists share one edge array, so it is sized by that array).
    float4* ang_grad = nullptr;
    if (derivs) {
        size_t n_ang = nd.edges ? (size_t)nd.total_edges : (size_t)nd.total_angular;
        ang_grad = eng.ws.take_n<float4>(n_ang + 1);
    }
    float4* edge_grad = nullptr;
    float* gtab = nullptr;
    int gkp = 0;
    if (c.kind == RUNE_NEP) {
        NepHeadArgs h{c.nep_hidden, eng.nep_w1, eng.nep_w1t, eng.nep_b1, eng.nep_w2,
                      eng.tensor("@q_scaler.p"), eng.nep_bias};
        float* qr_t = eng.ws.take_n<float>(nep_tiled_floats(N, p.nr));
        float* s_t = eng.ws.take_n<float>(nep_tiled_floats(N, p.na * p.C));
        float* w_t = derivs ? eng.ws.take_n<float>(nep_tiled_floats(N, p.na * p.C)) : nullptr;
        // with few types the force kernel reads the radial adjoint pre-contracted with the
        // c-table per neighbour type (two loads per basis function instead of a channel sum)
        gkp = (p.kr + 3) & ~3;
        if (derivs && p.T * gkp <= 256) gtab = eng.ws.take_n<float>((size_t)N * p.T * gkp);
        launch_desc_forward(p, N, nd.radial, nd.angular, types, qr_t, s_t, true, stream);
        launch_nep_atoms(p, N, n_owned, h, types, qr_t, s_t, e_model, dqr, w_t, gtab, stream);
        if (derivs) launch_angular_grad(p, N, nd.angular, types, w_t, ang_grad, stream);
    } else {
        float* q = eng.ws.take_n<float>((size_t)N * p.D);
        float* dq = eng.ws.take_n<float>((size_t)N * p.D);
        float* s = eng.ws.take_n<float>((size_t)N * p.na * p.C);
        launch_desc_forward(p, N, nd.radial, nd.angular, types, q, s, false, stream);
        float* mg = nullptr;
        if (!eng.eq.empty()) mg = eng.ws.take_n<float>((size_t)N * p.na * p.C);
        if (!eng.mp.empty() || !eng.eq.empty()) {
            if (!nd.radial.rev)
                build_reverse(eng, nd, nd.radial, nd.total_edges, stream);
            edge_grad = eng.ws.take_n<float4>((size_t)nd.total_edges + 1);
            RUNE_CUDA_TRY(cudaMemsetAsync(edge_grad, 0, sizeof(float4) * (nd.total_edges + 1),
                                          stream));
        }
        mobius_network(eng, N, q, s, types, nd, e_model, dq, edge_grad, mg, stream, dom);
        if (derivs) launch_desc_backward(p, N, nd.angular, types, dq, s, mg, dqr, ang_grad, stream);
    }
    if (derivs && !nd.angular.rev) {
        // On the device path the angular rows are prefixes of the radial rows when the radial
        // cutoff is the larger one, and the reverse of a short edge is short: the radial
        // reverse index then serves both lists.
        if (nd.edges && nd.radial.rev && eng.cfg.rc_radial >= eng.cfg.rc_angular)
            nd.angular.rev = nd.radial.rev;
        else
            build_reverse(eng, nd, nd.angular,
                          nd.edges ? nd.total_edges : nd.total_angular, stream);
    }
    double* vir_atom = (out.flags & RUNE_VIRIAL) ? eng.ws.take_n<double>((size_t)N * 9) : nullptr;
    float* forces = out.forces;
    if (derivs && !forces) forces = eng.ws.take_n<float>((size_t)N * 3);
    ForceLaunch f{};
    f.n_atoms = N;
    f.p = p;
    f.rad = nd.radial;
    f.ang = nd.angular;
    f.zbl_list = c.kind == RUNE_NEP ? nd.angular : nd.radial;
    f.types = types;
    f.dqr = dqr;
    f.gtab = gtab;
    f.gkp = gkp;
    f.ang_grad = ang_grad;
    f.zbl_mode = c.zbl_mode;
    f.zbl_rc_inner = c.zbl_rc_inner;
    f.zbl_rc_outer = c.zbl_rc_outer;
    if (c.zbl_mode != RUNE_ZBL_NONE) {
        f.zbl_zpow = eng.tensor("@zbl.zpow");
        f.zbl_z = eng.tensor("zbl.atomic_numbers");
        f.zbl_coef = eng.tensor("zbl.universal_coefficients");
        f.zbl_pairs = c.zbl_mode == RUNE_ZBL_FLEXIBLE ? eng.tensor("zbl.pair_parameters")
                                                      : nullptr;
    }
    f.edge_grad = edge_grad;
    f.positions64 = nd.positions64;
    f.sid = nd.sid;
    f.geom = nd.geom;
    f.shifts = nd.shifts;
    f.zbl_max_outer = eng.zbl_max_outer;
    f.n_owned = n_owned;
    f.descriptor = derivs;
    f.e_zbl = e_zbl;
    f.forces = derivs ? forces : nullptr;
    f.virial_atom = vir_atom;
    launch_forces(f, stream);

    // per-atom energies and per-structure sums (fixed chunks, fixed order)
    double* part = eng.ws.take_n<double>((size_t)std::max(ct.n_chunks, 1) * 10);
    if (ct.n_chunks > 0) {
        RUNE_KERNEL("k_chunk_partials", stream,
                    k_chunk_partials<<<ct.n_chunks, kSumThreads, 0, stream>>>(
                        n_structures, ct.chunk_ptr, ct.atom_ptr, kChunk, e_model, e_zbl,
                        out.energies, vir_atom, part));
        RUNE_LAUNCH_CHECK();
    }
    if (n_structures > 0) {
        RUNE_KERNEL("k_structure_sum", stream,
                    k_structure_sum<<<(n_structures * 32 + 255) / 256, 256, 0, stream>>>(
                        n_structures, ct.chunk_ptr, part, out.energy,
                        (out.flags & RUNE_VIRIAL) ? out.virial : nullptr));
        RUNE_LAUNCH_CHECK();
    }
    eng.stats.calls++;
}

// ----------------------------------------------------------------------------- finalize
namespace {

struct BlobBuilder {
    std::vector<float> data;
    std::map<std::string, size_t> off;
    void add(const std::string& name, const std::vector<float>& v) {
        size_t o = (data.size() + 63) & ~size_t(63);  // 256-byte alignment
        data.resize(o + v.size());
        std::memcpy(data.data() + o, v.data(), v.size() * sizeof(float));
        off[name] = o;
    }
};

const std::vector<float>& need(Engine& e, const std::string& name, size_t count) {
    auto it = e.host.find(name);
    if (it == e.host.end()) throw Error(RUNE_ERR_INVALID, "missing tensor: " + name);
    if (count && it->second.size() != count)
        throw Error(RUNE_ERR_INVALID, "tensor " + name + " has " +
                                          std::to_string(it->second.size()) + " values, expected " +
                                          std::to_string(count));
    return it->second;
}

std::vector<float> transpose(const std::vector<float>& w, int rows, int cols) {
    std::vector<float> t((size_t)rows * cols);
    for (int r = 0; r < rows; ++r)
        for (int c = 0; c < cols; ++c) t[(size_t)c * rows + r] = w[(size_t)r * cols + c];
    return t;
}

}  // namespace

static void finalize(Engine& e) {
    rune_model_config& c = e.cfg;
    int T = c.n_types;
    if (T < 1) throw Error(RUNE_ERR_INVALID, "n_types must be positive");
    if (c.l_max < 1 || c.l_max > 8) throw Error(RUNE_ERR_INVALID, "l_max must be in 1..8");
    e.C = c.l_max * (c.l_max + 2);
    e.nL = c.l_max + (c.has_q222 > 0) + (c.has_q1111 > 0) + (c.has_q112 > 0) +
           (c.has_q123 > 0) + (c.has_q233 > 0) + (c.has_q134 > 0);
    e.D = c.n_desc_radial + c.n_desc_angular * e.nL;
    if (c.n_desc_radial < 1 || c.n_desc_radial > 64 || c.n_desc_angular < 1 ||
        c.n_desc_angular > 64)
        throw Error(RUNE_ERR_INVALID, "n_desc_radial and n_desc_angular must be in 1..64");
    if (c.k_max_radial < 1 || c.k_max_angular < 1)
        throw Error(RUNE_ERR_INVALID, "k_max_radial and k_max_angular must be positive");
    BlobBuilder bb;
    int nr = c.n_desc_radial, na = c.n_desc_angular, kr = c.k_max_radial, ka = c.k_max_angular;
    bb.add("descriptor.radial.c_table", need(e, "descriptor.radial.c_table", (size_t)T * T * nr * kr));
    bb.add("descriptor.angular.c_table",
           need(e, "descriptor.angular.c_table", (size_t)T * T * na * ka));
    // z-polynomial table zc[L][m][p] from the Z{L} buffers ([L+1, L+1])
    std::vector<float> zc(9 * 9 * 9, 0.0f);
    for (int L = 1; L <= c.l_max; ++L) {
        const auto& z = need(e, "descriptor.angular.Z" + std::to_string(L), (size_t)(L + 1) * (L + 1));
        for (int m = 0; m <= L; ++m)
            for (int p = 0; p <= L; ++p) zc[(L * 9 + m) * 9 + p] = z[(size_t)m * (L + 1) + p];
    }
    bb.add("@zc", zc);
    const auto& terms = need(e, "invariant_terms", 0);
    if (terms.size() % 6 != 0) throw Error(RUNE_ERR_INVALID, "invariant_terms must be [n, 6]");
    e.n_terms = (int)(terms.size() / 6);
    for (int k = 0; k < e.n_terms; ++k) {
        int L = (int)terms[6 * k + 1];
        if (L < 0 || L >= e.nL) throw Error(RUNE_ERR_INVALID, "invariant term with bad output");
        for (int f = 2; f < 6; ++f)
            if ((int)terms[6 * k + f] >= e.C)
                throw Error(RUNE_ERR_INVALID, "invariant term with bad moment index");
    }
    {
        // Device tables (layout in DescParams): terms grouped by output L, each packed into
        // 16 bytes with its factor indices as bytes; the derivative table holds, for every
        // occurrence of harmonic c in a term, the coefficient and the other factors.
        auto bits = [](int v) {
            float f;
            std::memcpy(&f, &v, sizeof(f));
            return f;
        };
        auto pack = [](const int* idx, int n) {
            unsigned v = 0xffffffffu;
            for (int k = 0; k < n; ++k)
                if (idx[k] >= 0) v = (v & ~(0xffu << (8 * k))) | ((unsigned)idx[k] << (8 * k));
            return (int)v;
        };
        int prev = 0;
        for (int k = 0; k < e.n_terms; ++k) {
            int L = (int)terms[6 * k + 1];
            if (L < prev) throw Error(RUNE_ERR_INVALID, "invariant_terms must be grouped by output");
            prev = L;
        }
        std::vector<float> packed, term_ptr(e.nL + 1);
        for (int k = 0; k < e.n_terms; ++k) {
            const float* t = terms.data() + 6 * k;
            int idx[4] = {(int)t[2], (int)t[3], (int)t[4], (int)t[5]};
            packed.insert(packed.end(), {t[0], bits((int)t[1]), bits(pack(idx, 4)), 0.0f});
        }
        for (int L = 0; L <= e.nL; ++L) {
            int k = 0;
            while (k < e.n_terms && (int)terms[6 * k + 1] < L) ++k;
            term_ptr[L] = bits(k);
        }
        std::vector<std::vector<float>> by_c(e.C);
        for (int k = 0; k < e.n_terms; ++k) {
            const float* t = terms.data() + 6 * k;
            for (int f = 2; f < 6; ++f) {
                int c = (int)t[f];
                if (c < 0) continue;
                int other[3] = {-1, -1, -1}, o = 0;
                for (int g = 2; g < 6; ++g)
                    if (g != f && (int)t[g] >= 0) other[o++] = (int)t[g];
                by_c[c].insert(by_c[c].end(),
                               {t[0], bits((int)t[1]), bits(pack(other, 3)), bits(c)});
            }
        }
        std::vector<float> dterms, dterm_ptr(e.C + 1);
        for (int c = 0; c < e.C; ++c) {
            dterm_ptr[c] = bits((int)(dterms.size() / 4));
            dterms.insert(dterms.end(), by_c[c].begin(), by_c[c].end());
        }
        dterm_ptr[e.C] = bits((int)(dterms.size() / 4));
        e.n_dterms = (int)(dterms.size() / 4);
        if (packed.empty()) packed.assign(4, 0.0f);
        if (dterms.empty()) dterms.assign(4, 0.0f);
        bb.add("@terms", packed);
        bb.add("@term_ptr", term_ptr);
        bb.add("@dterms", dterms);
        bb.add("@dterm_ptr", dterm_ptr);
        // c-tables transposed to [T][T][k][n], n padded to a multiple of 4
        auto transpose_c = [&](const std::vector<float>& ct, int nn, int kk) {
            int np = (nn + 3) / 4 * 4;
            std::vector<float> out((size_t)T * T * kk * np, 0.0f);
            for (size_t pr = 0; pr < (size_t)T * T; ++pr)
                for (int n = 0; n < nn; ++n)
                    for (int k = 0; k < kk; ++k)
                        out[(pr * kk + k) * np + n] = ct[(pr * nn + n) * kk + k];
            return out;
        };
        bb.add("@c_r.t", transpose_c(need(e, "descriptor.radial.c_table", 0), nr, kr));
        bb.add("@c_a.t", transpose_c(need(e, "descriptor.angular.c_table", 0), na, ka));
    }
    const auto& scaler = need(e, "q_scaler", (size_t)e.D);
    bb.add("q_scaler", scaler);

    if (c.kind == RUNE_NEP) {
        int H = c.nep_hidden;
        if (H < 1) throw Error(RUNE_ERR_INVALID, "NEP hidden size must be positive");
        std::vector<float> w1, b1, w2;
        for (int t = 0; t < T; ++t) {
            std::string pre = "element_mlps." + std::to_string(t) + ".";
            const auto& a = need(e, pre + "0.weight", (size_t)H * e.D);
            const auto& b = need(e, pre + "0.bias", (size_t)H);
            const auto& d = need(e, pre + "2.weight", (size_t)H);
            w1.insert(w1.end(), a.begin(), a.end());
            b1.insert(b1.end(), b.begin(), b.end());
            w2.insert(w2.end(), d.begin(), d.end());
        }
        // W1 as float4 rows: [T][H][Dp] and transposed [T][D][Hp], zero padded to multiples
        // of 4 (Dp, Hp); the scaler padded alike
        int Dp = (e.D + 3) / 4 * 4, Hp = (H + 3) / 4 * 4;
        std::vector<float> w1p((size_t)T * H * Dp, 0.0f), w1tp((size_t)T * e.D * Hp, 0.0f);
        for (int t = 0; t < T; ++t)
            for (int h = 0; h < H; ++h)
                for (int d = 0; d < e.D; ++d) {
                    float v = w1[((size_t)t * H + h) * e.D + d];
                    w1p[((size_t)t * H + h) * Dp + d] = v;
                    w1tp[((size_t)t * e.D + d) * Hp + h] = v;
                }
        bb.add("@nep.w1", w1p);
        bb.add("@nep.w1t", w1tp);
        std::vector<float> scp(scaler);
        scp.resize(Dp, 0.0f);
        bb.add("@q_scaler.p", scp);
        bb.add("@nep.b1", b1);
        bb.add("@nep.w2", w2);
        e.nep_bias = need(e, "shared_bias", 1)[0];
    } else {
        int H = c.hidden_dim, F = c.ffn_dim, D = e.D;
        if (c.kind != RUNE_MOBIUS_LOCAL && c.message_layers > 0 && c.kind != RUNE_MOBIUS_MP &&
            c.kind != RUNE_MOBIUS_EQ)
            throw Error(RUNE_ERR_INVALID, "unknown model kind");
        const auto& win = need(e, "input_projection.weight", (size_t)H * D);
        std::vector<float> ws(win);
        for (int o = 0; o < H; ++o)
            for (int d = 0; d < D; ++d) ws[(size_t)o * D + d] *= scaler[d];
        bb.add("@in.w", ws);
        bb.add("@in.wt", transpose(ws, H, D));
        bb.add("input_projection.bias", need(e, "input_projection.bias", (size_t)H));
        bb.add("element_embedding.weight", need(e, "element_embedding.weight", (size_t)T * H));
        for (int b = 0; b < c.blocks; ++b) {
            std::string pre = "residual_blocks." + std::to_string(b) + ".";
            const auto& g = need(e, pre + "norm.weight", (size_t)H);
            std::vector<float> w1(need(e, pre + "ffn.0.weight", (size_t)F * H));
            for (int o = 0; o < F; ++o)
                for (int k = 0; k < H; ++k) w1[(size_t)o * H + k] *= g[k];
            bb.add(pre + "@w1", w1);
            bb.add(pre + "@w1t", transpose(w1, F, H));
            bb.add(pre + "ffn.0.bias", need(e, pre + "ffn.0.bias", (size_t)F));
            const auto& w2 = need(e, pre + "ffn.2.weight", (size_t)H * F);
            bb.add(pre + "@w2", w2);
            bb.add(pre + "@w2t", transpose(w2, H, F));
            bb.add(pre + "ffn.2.bias", need(e, pre + "ffn.2.bias", (size_t)H));
        }
        if (c.kind == RUNE_MOBIUS_MP) {
            int M = c.message_dim, P = c.pair_dim, G = c.message_groups, V = c.vector_channels;
            int K = c.message_basis_size;
            if (G < 1 || H % G != 0) throw Error(RUNE_ERR_INVALID, "message_groups must divide hidden_dim");
            for (int l = 0; l < c.message_layers; ++l) {
                std::string pre = "message_blocks." + std::to_string(l) + ".";
                const auto& pe = need(e, pre + "pair_embedding.weight", (size_t)T * T * P);
                const auto& we = need(e, pre + "edge_mlp.0.weight", (size_t)M * (K + P));
                const auto& be = need(e, pre + "edge_mlp.0.bias", (size_t)M);
                // edge-MLP tables with the hidden size padded to Mp (a multiple of 4; the
                // padded units have zero weights and bias, so act(0) = 0 adds nothing)
                int Mp = (M + 3) / 4 * 4;
                std::vector<float> pb((size_t)T * T * Mp, 0.0f), wk((size_t)Mp * K, 0.0f);
                for (int m = 0; m < M; ++m)
                    for (int k = 0; k < K; ++k) wk[(size_t)m * K + k] = we[(size_t)m * (K + P) + k];
                for (int pr = 0; pr < T * T; ++pr)
                    for (int m = 0; m < M; ++m) {
                        double acc = be[m];
                        for (int k = 0; k < P; ++k)
                            acc += (double)we[(size_t)m * (K + P) + K + k] * pe[(size_t)pr * P + k];
                        pb[(size_t)pr * Mp + m] = (float)acc;
                    }
                bb.add(pre + "@pb", pb);
                bb.add(pre + "@wk", wk);
                std::vector<float> wg(need(e, pre + "group_gate.weight", (size_t)G * M));
                std::vector<float> bgv(need(e, pre + "group_gate.bias", (size_t)G));
                const auto& gin = need(e, pre + "input_norm.weight", (size_t)H);
                std::vector<float> wvs(need(e, pre + "value_projection.weight", (size_t)H * H));
                std::vector<float> wgv((size_t)(G + V) * Mp, 0.0f);
                for (int q = 0; q < G; ++q)
                    for (int m = 0; m < M; ++m) wgv[(size_t)q * Mp + m] = wg[(size_t)q * M + m];
                if (V > 0) {
                    const auto& vg = need(e, pre + "vector_gate.weight", (size_t)V * M);
                    const auto& vb = need(e, pre + "vector_gate.bias", (size_t)V);
                    for (int q = 0; q < V; ++q)
                        for (int m = 0; m < M; ++m)
                            wgv[(size_t)(G + q) * Mp + m] = vg[(size_t)q * M + m];
                    bgv.insert(bgv.end(), vb.begin(), vb.end());
                    const auto& vsrc = need(e, pre + "vector_source.weight", (size_t)V * H);
                    wvs.insert(wvs.end(), vsrc.begin(), vsrc.end());
                    bb.add(pre + "@wmix", need(e, pre + "vector_mix.weight", (size_t)V * V));
                } else {
                    bb.add(pre + "@wmix", std::vector<float>(1, 0.0f));
                }
                for (int o = 0; o < H + V; ++o)
                    for (int k = 0; k < H; ++k) wvs[(size_t)o * H + k] *= gin[k];
                bb.add(pre + "@wgv", wgv);
                bb.add(pre + "@bgv", bgv);
                bb.add(pre + "@vs.w", wvs);
                bb.add(pre + "@vs.wt", transpose(wvs, H + V, H));
                bb.add(pre + "message_norm.weight", need(e, pre + "message_norm.weight", (size_t)H));
                const auto& u1 = need(e, pre + "update.0.weight", (size_t)M * (H + V));
                bb.add(pre + "@u1.w", u1);
                bb.add(pre + "@u1.wt", transpose(u1, M, H + V));
                bb.add(pre + "update.0.bias", need(e, pre + "update.0.bias", (size_t)M));
                const auto& u2 = need(e, pre + "update.2.weight", (size_t)H * M);
                bb.add(pre + "@u2.w", u2);
                bb.add(pre + "@u2.wt", transpose(u2, H, M));
                bb.add(pre + "update.2.bias", need(e, pre + "update.2.bias", (size_t)H));
            }
        }
        if (c.kind == RUNE_MOBIUS_EQ) {
            int M = c.message_dim, P = c.pair_dim, G = c.message_groups, K = c.message_basis_size;
            int Ce = c.equivariant_channels, Le = c.equivariant_l_max, Cl = Le * (Le + 2);
            int LC = Le * Ce, na = c.n_desc_angular;
            if (G < 1 || H % G != 0) throw Error(RUNE_ERR_INVALID, "message_groups must divide hidden_dim");
            if (Le < 1 || Le > c.l_max || Ce < 1)
                throw Error(RUNE_ERR_INVALID, "invalid equivariant_l_max / equivariant_channels");
            int XP = (K + 2 * LC + 3) & ~3, GD = G + 2 * LC, GDP = (GD + 3) & ~3, MP = (M + 3) & ~3;
            int IN = K + P + 2 * M + 2 * LC;
            std::vector<float> proj;
            for (int l = 0; l < Le; ++l) {
                const auto& w = need(e, "direction_encoder.projections." + std::to_string(l) + ".weight",
                                     (size_t)Ce * na);
                proj.insert(proj.end(), w.begin(), w.end());
            }
            bb.add("@eq.proj", proj);
            // orthonormal harmonic scale sqrt(C3B (1 if m = 0 else 2)) (descriptor.py:626-637),
            // computed by the host from the full-precision constants
            const auto& sc = need(e, "eq_scale", 0);
            if ((int)sc.size() < Cl) throw Error(RUNE_ERR_INVALID, "eq_scale is too short");
            std::vector<float> scale(sc.begin(), sc.begin() + Cl);
            bb.add("@eq.scale", scale);
            for (int l = 0; l < c.message_layers; ++l) {
                std::string pre = "message_blocks." + std::to_string(l) + ".";
                const auto& pe = need(e, pre + "pair_embedding.weight", (size_t)T * T * P);
                const auto& we = need(e, pre + "edge_mlp.0.weight", (size_t)M * IN);
                const auto& be = need(e, pre + "edge_mlp.0.bias", (size_t)M);
                std::vector<float> pb((size_t)T * T * M);
                for (int pr = 0; pr < T * T; ++pr)
                    for (int m = 0; m < M; ++m) {
                        double acc = be[m];
                        for (int k = 0; k < P; ++k)
                            acc += (double)we[(size_t)m * IN + K + k] * pe[(size_t)pr * P + k];
                        pb[(size_t)pr * M + m] = (float)acc;
                    }
                bb.add(pre + "@pb", pb);
                // basis + probe columns: x = [b (K) ; pc (LC) ; pn (LC)], in the tile-padded
                // shapes of the edge kernels
                EqTileDims td(K + 2 * LC, M, GD);
                auto xcol = [&](int q) { return q < K ? q : K + P + 2 * M + (q - K); };
                std::vector<float> wxT((size_t)td.XK * td.MN, 0.0f), wx((size_t)td.MK * td.XN, 0.0f);
                for (int q = 0; q < K + 2 * LC; ++q)
                    for (int m = 0; m < M; ++m) {
                        float v = we[(size_t)m * IN + xcol(q)];
                        wxT[(size_t)q * td.MN + m] = v;
                        wx[(size_t)m * td.XN + q] = v;
                    }
                bb.add(pre + "@wxT", wxT);
                bb.add(pre + "@wx", wx);
                // per-atom contexts: A = W_e[:, ctx_c] W_c, B = W_e[:, ctx_n] W_n, then W_v
                const auto& wc = need(e, pre + "center_context.weight", (size_t)M * H);
                const auto& wn = need(e, pre + "neighbor_context.weight", (size_t)M * H);
                const auto& wv = need(e, pre + "value_projection.weight", (size_t)H * H);
                const auto& gin = need(e, pre + "input_norm.weight", (size_t)H);
                std::vector<float> nodes((size_t)(2 * M + H) * H);
                for (int part = 0; part < 2; ++part) {
                    const auto& wctx = part == 0 ? wc : wn;
                    int off = K + P + part * M;
                    for (int m = 0; m < M; ++m)
                        for (int h = 0; h < H; ++h) {
                            double acc = 0.0;
                            for (int k = 0; k < M; ++k)
                                acc += (double)we[(size_t)m * IN + off + k] * wctx[(size_t)k * H + h];
                            nodes[((size_t)part * M + m) * H + h] = (float)(acc * gin[h]);
                        }
                }
                for (int o = 0; o < H; ++o)
                    for (int h = 0; h < H; ++h)
                        nodes[((size_t)2 * M + o) * H + h] = wv[(size_t)o * H + h] * gin[h];
                bb.add(pre + "@nodes.w", nodes);
                bb.add(pre + "@nodes.wt", transpose(nodes, 2 * M + H, H));
                // gates
                const auto& wg = need(e, pre + "group_gate.weight", (size_t)G * M);
                const auto& bg = need(e, pre + "group_gate.bias", (size_t)G);
                const auto& wd = need(e, pre + "direction_gates.weight", (size_t)2 * LC * M);
                const auto& bd = need(e, pre + "direction_gates.bias", (size_t)2 * LC);
                std::vector<float> wgd((size_t)td.GK * td.MN, 0.0f),
                    wgdT((size_t)td.MK * td.GN, 0.0f), bgd(GD);
                for (int o = 0; o < GD; ++o) {
                    bgd[o] = o < G ? bg[o] : bd[o - G];
                    for (int m = 0; m < M; ++m) {
                        float v = o < G ? wg[(size_t)o * M + m] : wd[(size_t)(o - G) * M + m];
                        wgd[(size_t)o * td.MN + m] = v;
                        wgdT[(size_t)m * td.GN + o] = v;
                    }
                }
                bb.add(pre + "@wgd", wgd);
                bb.add(pre + "@wgdT", wgdT);
                bb.add(pre + "@bgd", bgd);

                std::vector<float> wmix;
                for (int q = 0; q < Le; ++q) {
                    const auto& w = need(e, pre + "direction_mix." + std::to_string(q) + ".weight",
                                         (size_t)Ce * Ce);
                    wmix.insert(wmix.end(), w.begin(), w.end());
                }
                bb.add(pre + "@wmix", wmix);
                bb.add(pre + "message_norm.weight", need(e, pre + "message_norm.weight", (size_t)H));
                const auto& u1 = need(e, pre + "update.0.weight", (size_t)M * (H + LC));
                bb.add(pre + "@u1.w", u1);
                bb.add(pre + "@u1.wt", transpose(u1, M, H + LC));
                bb.add(pre + "update.0.bias", need(e, pre + "update.0.bias", (size_t)M));
                const auto& u2 = need(e, pre + "update.2.weight", (size_t)H * M);
                bb.add(pre + "@u2.w", u2);
                bb.add(pre + "@u2.wt", transpose(u2, H, M));
                bb.add(pre + "update.2.bias", need(e, pre + "update.2.bias", (size_t)H));
            }
        }
        bb.add("output_norm.weight", need(e, "output_norm.weight", (size_t)H));
        bb.add("energy_heads.weight", need(e, "energy_heads.weight", (size_t)T * H));
        bb.add("energy_heads.bias", need(e, "energy_heads.bias", (size_t)T));
    }
    if (c.zbl_mode != RUNE_ZBL_NONE) {
        const auto& z = need(e, "zbl.atomic_numbers", (size_t)T);
        std::vector<float> zp(T);
        for (int t = 0; t < T; ++t) zp[t] = (float)std::pow((double)z[t], 0.23);
        bb.add("zbl.atomic_numbers", z);
        bb.add("@zbl.zpow", zp);
        bb.add("zbl.universal_coefficients", need(e, "zbl.universal_coefficients", 8));
        e.zbl_max_outer = c.zbl_rc_outer;
        if (c.zbl_mode == RUNE_ZBL_FLEXIBLE) {
            const auto& pp = need(e, "zbl.pair_parameters", (size_t)T * (T + 1) / 2 * 10);
            bb.add("zbl.pair_parameters", pp);
            e.zbl_max_outer = 0.0;
            for (size_t k = 0; k < pp.size() / 10; ++k)
                e.zbl_max_outer = std::max(e.zbl_max_outer, (double)pp[10 * k + 1]);
        }
    }

    RUNE_CUDA_TRY(cudaSetDevice(e.device));
    RUNE_CUDA_TRY(cudaMalloc(&e.blob, bb.data.size() * sizeof(float)));
    RUNE_CUDA_TRY(cudaMemcpy(e.blob, bb.data.data(), bb.data.size() * sizeof(float),
                             cudaMemcpyHostToDevice));
    e.blob_floats = bb.data.size();
    e.offsets = bb.off;
    DescParams& p = e.desc;
    p.nr = nr; p.na = na; p.kr = kr; p.ka = ka; p.lmax = c.l_max; p.C = e.C; p.nL = e.nL;
    p.D = e.D; p.T = T;
    p.rc_r = (float)c.rc_radial;
    p.rc_a = (float)c.rc_angular;
    p.c_r = e.tensor("descriptor.radial.c_table");
    p.c_a = e.tensor("descriptor.angular.c_table");
    p.zc = e.tensor("@zc");
    p.c_rt = reinterpret_cast<const float4*>(e.tensor("@c_r.t"));
    p.c_at = reinterpret_cast<const float4*>(e.tensor("@c_a.t"));
    p.npr = (nr + 3) / 4;
    p.npa = (na + 3) / 4;
    p.n_terms = e.n_terms;
    p.terms = reinterpret_cast<const int4*>(e.tensor("@terms"));
    p.term_ptr = reinterpret_cast<const int*>(e.tensor("@term_ptr"));
    p.dterms = reinterpret_cast<const int4*>(e.tensor("@dterms"));
    p.dterm_ptr = reinterpret_cast<const int*>(e.tensor("@dterm_ptr"));
    p.n_dterms = e.n_dterms;
    e.q_scaler = e.tensor("q_scaler");
    if (c.kind == RUNE_NEP) {
        e.nep_w1 = e.tensor("@nep.w1");
        e.nep_w1t = e.tensor("@nep.w1t");
        e.nep_b1 = e.tensor("@nep.b1");
        e.nep_w2 = e.tensor("@nep.w2");
    } else {
        int H = c.hidden_dim, F = c.ffn_dim;
        e.input_projection = Dense{e.D, H, e.tensor("@in.wt"), e.tensor("@in.w"),
                                   e.tensor("input_projection.bias")};
        e.embedding = e.tensor("element_embedding.weight");
        e.ffn1.clear();
        e.ffn2.clear();
        for (int b = 0; b < c.blocks; ++b) {
            std::string pre = "residual_blocks." + std::to_string(b) + ".";
            e.ffn1.push_back(Dense{H, F, e.tensor(pre + "@w1t"), e.tensor(pre + "@w1"),
                                   e.tensor(pre + "ffn.0.bias")});
            e.ffn2.push_back(Dense{F, H, e.tensor(pre + "@w2t"), e.tensor(pre + "@w2"),
                                   e.tensor(pre + "ffn.2.bias")});
        }
        e.mp.clear();
        if (c.kind == RUNE_MOBIUS_MP) {
            int M = c.message_dim, G = c.message_groups, V = c.vector_channels;
            for (int l = 0; l < c.message_layers; ++l) {
                std::string pre = "message_blocks." + std::to_string(l) + ".";
                MpLayer L;
                L.args = MpLayerArgs{H, M, G, V, c.message_basis_size, T, c.activation,
                                     (float)c.message_cutoff, (float)c.norm_eps,
                                     e.tensor(pre + "@pb"), e.tensor(pre + "@wk"),
                                     e.tensor(pre + "@wgv"), e.tensor(pre + "@bgv"),
                                     e.tensor(pre + "message_norm.weight"),
                                     e.tensor(pre + "@wmix")};
                L.args.Mp = (M + 3) / 4 * 4;
                if (H > 256 || 3 * V > 32 || G + V > 32 || c.message_basis_size > 33)
                    throw Error(RUNE_ERR_INVALID,
                                "MP message blocks support hidden_dim <= 256, vector_channels "
                                "<= 10, message_groups + vector_channels <= 32 and "
                                "message_basis_size <= 33");
                L.vs = Dense{H, H + V, e.tensor(pre + "@vs.wt"), e.tensor(pre + "@vs.w"), nullptr};
                L.upd1 = Dense{H + V, M, e.tensor(pre + "@u1.wt"), e.tensor(pre + "@u1.w"),
                               e.tensor(pre + "update.0.bias")};
                L.upd2 = Dense{M, H, e.tensor(pre + "@u2.wt"), e.tensor(pre + "@u2.w"),
                               e.tensor(pre + "update.2.bias")};
                e.mp.push_back(L);
            }
        }
        e.eq.clear();
        if (c.kind == RUNE_MOBIUS_EQ) {
            int M = c.message_dim, G = c.message_groups;
            int Ce = c.equivariant_channels, Le = c.equivariant_l_max, LC = Le * Ce;
            e.eq_proj = e.tensor("@eq.proj");
            for (int l = 0; l < c.message_layers; ++l) {
                std::string pre = "message_blocks." + std::to_string(l) + ".";
                EqLayer L;
                L.args = EqLayerArgs{H, M, G, Ce, Le, Le * (Le + 2), c.message_basis_size, T,
                                     c.activation, (float)c.message_cutoff, (float)c.norm_eps,
                                     e.tensor(pre + "@pb"), e.tensor(pre + "@wxT"),
                                     e.tensor(pre + "@wx"), e.tensor(pre + "@wgdT"),
                                     e.tensor(pre + "@wgd"), e.tensor(pre + "@bgd"),
                                     e.tensor(pre + "@wmix"), e.tensor(pre + "message_norm.weight"),
                                     e.tensor("@eq.scale"), e.tensor("@zc")};
                EqTileDims td(c.message_basis_size + 2 * LC, M, G + 2 * LC);
                L.args.XK = td.XK; L.args.XN = td.XN; L.args.MK = td.MK;
                L.args.MN = td.MN; L.args.GK = td.GK; L.args.GN = td.GN;
                L.args.wait_polls = e.wait_polls;

                if (td.XN > 320 || td.MN > 320 || td.GN > 320 || H > 1024 ||
                    c.message_basis_size > 64)
                    throw Error(RUNE_ERR_INVALID,
                                "EQ blocks support message_basis_size <= 64 and "
                                "message_basis_size + 2 (l_max Ce), message_dim and "
                                "message_groups + 2 (l_max Ce) up to 320");
                L.nodes = Dense{H, 2 * M + H, e.tensor(pre + "@nodes.wt"),
                                e.tensor(pre + "@nodes.w"), nullptr};
                L.upd1 = Dense{H + LC, M, e.tensor(pre + "@u1.wt"), e.tensor(pre + "@u1.w"),
                               e.tensor(pre + "update.0.bias")};
                L.upd2 = Dense{M, H, e.tensor(pre + "@u2.wt"), e.tensor(pre + "@u2.w"),
                               e.tensor(pre + "update.2.bias")};
                e.eq.push_back(L);
            }
            // tensor-core forms of the four edge-product weights of every layer (K <= 320),
            // when RUNE_EQ_TENSOR_CORES=1 at finalize: the edge products then run on tcgen05
            // (exact-integer digits, parity-equal to the SIMT products). Not the default: on
            // B200 the SIMT kernels are faster (OAM-EQ on MgO 36^3: 1.30e5 against 1.13e5
            // atoms/s), because the tiles' neighbour gathers, not the products, bound them.
            const char* want_tc = std::getenv("RUNE_EQ_TENSOR_CORES");
            bool tc = !e.eq.empty() && want_tc && std::string(want_tc) == "1";
            size_t bytes = 0;
            for (auto& L : e.eq) {
                const EqLayerArgs& a = L.args;
                tc = tc && a.XK <= 320 && a.MK <= 320 && a.GK <= 320;
                bytes += ((eq_tc_bytes(a.XK, a.MN) + 255) & ~size_t(255)) +
                         ((eq_tc_bytes(a.MK, a.GN) + 255) & ~size_t(255)) +
                         ((eq_tc_bytes(a.GK, a.MN) + 255) & ~size_t(255)) +
                         ((eq_tc_bytes(a.MK, a.XN) + 255) & ~size_t(255));
            }
            if (tc) {
                RUNE_CUDA_TRY(cudaMalloc(&e.eq_tc_buf, bytes));
                char* p = static_cast<char*>(e.eq_tc_buf);
                auto pack = [&](const float* W, int K, int N) {
                    EqTcW t = eq_tc_pack(W, K, N, p, nullptr);
                    p += (eq_tc_bytes(K, N) + 255) & ~size_t(255);
                    return t;
                };
                for (auto& L : e.eq) {
                    EqLayerArgs& a = L.args;
                    a.tx = pack(a.wxT, a.XK, a.MN);
                    a.tgd = pack(a.wgdT, a.MK, a.GN);
                    a.tgdT = pack(a.wgd, a.GK, a.MN);
                    a.txT = pack(a.wx, a.MK, a.XN);
                    a.tc = true;
                    ++e.stats.tensor_core_layers;
                }
                RUNE_CUDA_TRY(cudaDeviceSynchronize());
            }
        }
        e.out_norm = e.tensor("output_norm.weight");
        e.head_w = e.tensor("energy_heads.weight");
        e.head_b = e.tensor("energy_heads.bias");
    }
    RUNE_CUDA_TRY(cudaMalloc(&e.d_flags, sizeof(unsigned int)));
    RUNE_CUDA_TRY(cudaMemset(e.d_flags, 0, sizeof(unsigned int)));
    RUNE_CUDA_TRY(cudaMallocHost(&e.host_sync, sizeof(HostSync)));
    e.staging.cap = 1u << 20;
    RUNE_CUDA_TRY(cudaMallocHost(&e.staging.base, e.staging.cap));
    RUNE_CUDA_TRY(cudaMalloc(&e.d_mirror, e.staging.cap));
    e.host.clear();
    e.finalized = true;
}

void grow_workspace(Engine& e, size_t want, cudaStream_t stream) {
    RUNE_CUDA_TRY(cudaStreamSynchronize(stream));
    // the failing request is only the first one past the end: grow geometrically from both
    size_t cap = std::max(2 * want + (64u << 20), e.ws.cap * 2);
    if (e.ws.base) RUNE_CUDA_TRY(cudaFree(e.ws.base));
    e.ws.base = nullptr;
    e.ws.cap = 0;
    // the geometric margin never takes the last 8 GiB of the device (communication libraries
    // and the caller's own allocations need room next to a large workspace)
    size_t free_b = 0, total_b = 0;
    if (cudaMemGetInfo(&free_b, &total_b) == cudaSuccess) {
        const size_t reserve = size_t(8) << 30;
        size_t room = free_b > reserve ? free_b - reserve : 0;
        if (cap > room) cap = std::max(room, want + (64u << 20));
    } else {
        cudaGetLastError();
    }
    cudaError_t err = cudaMalloc(&e.ws.base, cap);
    if (err != cudaSuccess && cap > want + (64u << 20)) {
        // the geometric margin does not fit: the request itself (plus 64 MiB) may
        cudaGetLastError();
        cap = want + (64u << 20);
        err = cudaMalloc(&e.ws.base, cap);
    }
    if (err != cudaSuccess) {
        cudaGetLastError();
        e.ws.base = nullptr;
        throw Error(RUNE_ERR_OOM, "device workspace allocation of " + std::to_string(cap) +
                                      " bytes failed");
    }
    e.ws.cap = cap;
    e.stats.workspace_grows++;
    e.stats.workspace_bytes = (int64_t)cap;
}

template <typename Fn>
static int guarded(Fn&& fn) {
    try {
        fn();
        return RUNE_OK;
    } catch (const Error& err) {
        set_error(err.message);
        return err.code < 0 ? RUNE_ERR_STATE : err.code;
    } catch (const std::exception& ex) {
        set_error(ex.what());
        return RUNE_ERR_INVALID;
    }
}

struct ProfilerInstall {
    Engine& e;
    explicit ProfilerInstall(Engine& eng) : e(eng) { set_current_profiler(&e.prof); }
    ~ProfilerInstall() {
        set_current_profiler(nullptr);
        e.stats.kernel_launches = e.prof.launches;
    }
};

static void grow_staging(Engine& e) {
    if (e.staging_want <= e.staging.cap) return;
    size_t cap = std::max(e.staging_want * 2, e.staging.cap * 2);
    char* p = nullptr;
    if (cudaMallocHost(&p, cap) != cudaSuccess) {
        cudaGetLastError();
        return;  // keep the old buffer; large uploads stay pageable
    }
    char* d = nullptr;
    if (cudaMalloc(&d, cap) != cudaSuccess) {
        cudaGetLastError();
        cudaFreeHost(p);
        return;
    }
    if (e.staging.base) cudaFreeHost(e.staging.base);
    if (e.d_mirror) cudaFree(e.d_mirror);
    e.staging.base = p;
    e.d_mirror = d;
    e.staging.cap = cap;
}

template <typename Fn>
static void with_workspace(Engine& e, cudaStream_t stream, Fn&& fn) {
    ProfilerInstall install(e);
    for (int attempt = 0; attempt < 40; ++attempt) {
        e.ws.reset();
        e.staging.off = 0;
        e.stage_first = ~size_t(0);
        try {
            fn();
            // every call ends with a stream synchronisation: the timing events are complete
            e.prof.resolve();
            grow_staging(e);
            return;
        } catch (const Error& err) {
            cudaStreamSynchronize(stream);
            e.prof.resolve();
            if (err.code == -2) continue;  // edge buffer regrown: repeat the call
            if (err.code != -1) throw;
            grow_workspace(e, e.ws.want, stream);
        }
    }
    throw Error(RUNE_ERR_OOM, "workspace sizing did not converge");
}

}  // namespace rune

// ============================================================================= C ABI
using rune::Engine;
using rune::Error;

struct rune_engine {
    Engine impl;
};

extern "C" {

int rune_engine_create(const rune_model_config* config, int device, rune_engine** out) {
    return rune::guarded([&] {
        if (!config || !out) throw Error(RUNE_ERR_INVALID, "null argument");
        int count = 0;
        RUNE_CUDA_TRY(cudaGetDeviceCount(&count));
        if (device < 0 || device >= count)
            throw Error(RUNE_ERR_INVALID, "CUDA device " + std::to_string(device) +
                                              " is not available");
        std::unique_ptr<rune_engine> e(new rune_engine());
        e->impl.cfg = *config;
        e->impl.device = device;
        *out = e.release();
    });
}

int rune_engine_set_tensor(rune_engine* engine, const char* name, const float* host_data,
                           int64_t count) {
    return rune::guarded([&] {
        if (!engine || !name || (count > 0 && !host_data))
            throw Error(RUNE_ERR_INVALID, "null argument");
        if (engine->impl.finalized) throw Error(RUNE_ERR_STATE, "engine already finalized");
        engine->impl.host[name] = std::vector<float>(host_data, host_data + count);
    });
}

int rune_engine_finalize(rune_engine* engine) {
    return rune::guarded([&] {
        if (!engine) throw Error(RUNE_ERR_INVALID, "null engine");
        if (engine->impl.finalized) throw Error(RUNE_ERR_STATE, "engine already finalized");
        rune::finalize(engine->impl);
    });
}

namespace rune {
namespace {

// Device-path call body: neighbour build, evaluation, one synchronisation for the count summary
// and error flags (a row overflow raises the stride and asks for a repeat).
void device_body(Engine& e, const BatchInput& in, const Outputs& o, cudaStream_t stream,
                 const DomainCall* dom) {
    CallTables ct = stage_call_tables(e, in.n_structures, in.atom_ptr, stream);
    NeighborData nd;
    build_neighbors(e, in, ct.atom_ptr, nd, stream);  // flushes the uploads
    evaluate(e, nd, in.n_atoms, in.n_structures, in.types, ct, o, stream, dom);
    HostSync* hs = e.host_sync;
    RUNE_CUDA_TRY(cudaMemcpyAsync(hs->maxc, nd.summary, sizeof(unsigned long long) * 4,
                                  cudaMemcpyDeviceToHost, stream));
    RUNE_CUDA_TRY(cudaMemcpyAsync(&hs->flags, e.d_flags, sizeof(unsigned int),
                                  cudaMemcpyDeviceToHost, stream));
    RUNE_CUDA_TRY(cudaStreamSynchronize(stream));
    unsigned int f = hs->flags;
    if (f & 16u) {
        RUNE_CUDA_TRY(cudaMemsetAsync(e.d_flags, 0, sizeof(unsigned int), stream));
        finish_neighbors(e, nd, *hs);  // raises the row stride
        if (dom && dom->exchanges > 0)  // other ranks took part: the caller repeats on all
            throw Error(RUNE_ERR_RETRY, "neighbour rows regrown: repeat the halo call");
        throw Error(-2, "edge rows regrown");
    }
    e.check_flags(f, stream);
    finish_neighbors(e, nd, *hs);
    e.last = nd;
    e.last_valid = true;
}

void compute_device(Engine& e, const BatchInput& in, int32_t flags, const Outputs& o,
                    cudaStream_t stream, const DomainCall* dom) {
    (void)flags;
    with_workspace(e, stream, [&] { device_body(e, in, o, stream, dom); });
}

// The exchanging attempt of a halo call: like with_workspace, but an attempt that has issued an
// exchange is never repeated here (the other ranks would not repeat theirs).
void compute_halo_attempt(Engine& e, const BatchInput& in, const Outputs& o, cudaStream_t stream,
                          DomainCall& dom) {
    ProfilerInstall install(e);
    for (int attempt = 0; attempt < 40; ++attempt) {
        e.ws.reset();
        e.staging.off = 0;
        e.stage_first = ~size_t(0);
        dom.exchanges = 0;
        try {
            device_body(e, in, o, stream, &dom);
            e.prof.resolve();
            grow_staging(e);
            return;
        } catch (const Error& err) {
            cudaStreamSynchronize(stream);
            e.prof.resolve();
            if (dom.exchanges > 0) throw;
            if (err.code == -2) continue;
            if (err.code != -1) throw;
            grow_workspace(e, e.ws.want, stream);
        }
    }
    throw Error(RUNE_ERR_OOM, "workspace sizing did not converge");
}

void check_outputs(float* forces_dev, double* energy_dev, double* virial_dev, int32_t flags) {
    if (!energy_dev) throw Error(RUNE_ERR_INVALID, "energy output is required");
    if ((flags & RUNE_FORCES) && !forces_dev)
        throw Error(RUNE_ERR_INVALID, "forces requested without an output buffer");
    if ((flags & RUNE_VIRIAL) && !virial_dev)
        throw Error(RUNE_ERR_INVALID, "virial requested without an output buffer");
}

}  // namespace
}  // namespace rune

int rune_engine_compute(rune_engine* engine, int32_t n_atoms, int32_t n_structures,
                        const int32_t* types_dev, const double* positions_dev,
                        const double* cells_host, const uint8_t* pbc_host,
                        const int32_t* atom_ptr_host, int32_t flags, float* energies_dev,
                        double* energy_dev, float* forces_dev, double* virial_dev,
                        void* stream_ptr) {
    return rune::guarded([&] {
        if (!engine) throw Error(RUNE_ERR_INVALID, "null engine");
        Engine& e = engine->impl;
        if (!e.finalized) throw Error(RUNE_ERR_STATE, "rune_engine_finalize was not called");
        if (n_atoms < 0 || n_structures < 1 || !atom_ptr_host || !cells_host || !pbc_host)
            throw Error(RUNE_ERR_INVALID, "invalid batch description");
        if (atom_ptr_host[0] != 0 || atom_ptr_host[n_structures] != n_atoms)
            throw Error(RUNE_ERR_INVALID, "atom_ptr must start at 0 and end at n_atoms");
        for (int s = 0; s < n_structures; ++s)
            if (atom_ptr_host[s + 1] < atom_ptr_host[s])
                throw Error(RUNE_ERR_INVALID, "atom_ptr must be non-decreasing");
        rune::check_outputs(forces_dev, energy_dev, virial_dev, flags);
        RUNE_CUDA_TRY(cudaSetDevice(e.device));
        rune::BatchInput in{n_atoms, n_structures, types_dev, positions_dev,
                            cells_host, pbc_host, atom_ptr_host};
        rune::Outputs o{energies_dev, energy_dev, forces_dev, virial_dev, flags};
        rune::compute_device(e, in, flags, o, static_cast<cudaStream_t>(stream_ptr), nullptr);
    });
}

int rune_engine_compute_domain(rune_engine* engine, int32_t n_atoms, int32_t n_shells,
                               const int32_t* shell_end_host, const int32_t* types_dev,
                               const double* positions_dev, const double* cell_host,
                               int32_t flags, float* energies_dev, double* energy_dev,
                               float* forces_dev, double* virial_dev, void* stream_ptr) {
    return rune::guarded([&] {
        if (!engine) throw Error(RUNE_ERR_INVALID, "null engine");
        Engine& e = engine->impl;
        if (!e.finalized) throw Error(RUNE_ERR_STATE, "rune_engine_finalize was not called");
        int layers = (int)(e.mp.size() + e.eq.size());
        if (n_shells != layers + 1)
            throw Error(RUNE_ERR_INVALID,
                        "a domain call of this model needs " + std::to_string(layers + 1) +
                            " ghost shells (one per message layer plus the descriptor shell)");
        if (n_atoms < 0 || !shell_end_host || !cell_host)
            throw Error(RUNE_ERR_INVALID, "invalid domain description");
        if (shell_end_host[0] < 0 || shell_end_host[n_shells] != n_atoms)
            throw Error(RUNE_ERR_INVALID, "shell_end must start at n_owned >= 0 and end at n_atoms");
        for (int k = 0; k < n_shells; ++k)
            if (shell_end_host[k + 1] < shell_end_host[k])
                throw Error(RUNE_ERR_INVALID, "shell_end must be non-decreasing");
        rune::check_outputs(forces_dev, energy_dev, virial_dev, flags);
        RUNE_CUDA_TRY(cudaSetDevice(e.device));
        rune::DomainCall dom;
        dom.n_owned = shell_end_host[0];
        dom.shell_end.assign(shell_end_host, shell_end_host + n_shells + 1);
        const uint8_t pbc[3] = {0, 0, 0};
        const int32_t atom_ptr[2] = {0, n_atoms};
        rune::BatchInput in{n_atoms, 1, types_dev, positions_dev, cell_host, pbc, atom_ptr};
        rune::Outputs o{energies_dev, energy_dev, forces_dev, virial_dev, flags};
        rune::compute_device(e, in, flags, o, static_cast<cudaStream_t>(stream_ptr), &dom);
    });
}

int rune_engine_compute_halo(rune_engine* engine, int32_t n_atoms, int32_t n_owned,
                             const int32_t* types_dev, const double* positions_dev,
                             const double* cell_host, int32_t flags, rune_halo_fn halo,
                             void* halo_ctx, float* energies_dev, double* energy_dev,
                             float* forces_dev, double* virial_dev, void* stream_ptr) {
    return rune::guarded([&] {
        if (!engine) throw Error(RUNE_ERR_INVALID, "null engine");
        Engine& e = engine->impl;
        if (!e.finalized) throw Error(RUNE_ERR_STATE, "rune_engine_finalize was not called");
        if (!e.mp.empty() || e.cfg.kind == RUNE_NEP)
            throw Error(RUNE_ERR_INVALID,
                        "halo exchange serves the Local and EQ Möbius models; use "
                        "rune_engine_compute_domain for this model");
        if (!halo) throw Error(RUNE_ERR_INVALID, "a halo call needs an exchange hook");
        if (n_atoms < 0 || n_owned < 0 || n_owned > n_atoms || !cell_host)
            throw Error(RUNE_ERR_INVALID, "invalid domain description");
        rune::check_outputs(forces_dev, energy_dev, virial_dev, flags);
        RUNE_CUDA_TRY(cudaSetDevice(e.device));
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        rune::DomainCall dom;
        dom.n_owned = n_owned;
        dom.shell_end = {n_owned, n_atoms};
        dom.halo = halo;
        dom.halo_ctx = halo_ctx;
        const uint8_t pbc[3] = {0, 0, 0};
        const int32_t atom_ptr[2] = {0, n_atoms};
        rune::BatchInput in{n_atoms, 1, types_dev, positions_dev, cell_host, pbc, atom_ptr};
        rune::Outputs o{energies_dev, energy_dev, forces_dev, virial_dev, flags};
        auto key = [&] {
            std::vector<double> k{(double)n_atoms, (double)n_owned, (double)e.row_stride,
                                  (double)flags};
            k.insert(k.end(), cell_host, cell_host + 9);
            return k;
        };
        if (key() != e.halo_key) {
            // rehearsal: the same work without exchanges, which settles the workspace and the
            // row stride (its repeats are local: no other rank takes part)
            dom.rehearsal = true;
            rune::compute_device(e, in, flags, o, stream, &dom);
            dom.rehearsal = false;
            e.halo_bytes = e.ws.off;
            e.halo_key = key();
        }
        try {
            rune::compute_halo_attempt(e, in, o, stream, dom);
        } catch (...) {
            e.halo_key.clear();  // sizes changed (or the call failed): rehearse next time
            throw;
        }
    });
}

int rune_engine_compute_padded(rune_engine* engine, int32_t n_atoms, int32_t n_structures,
                               const int32_t* types_dev, const float* positions_dev,
                               const int64_t* radial_neighbors_dev, int32_t radial_width,
                               const float* radial_offsets_dev,
                               const int64_t* angular_neighbors_dev, int32_t angular_width,
                               const float* angular_offsets_dev, const int32_t* atom_ptr_host,
                               int32_t flags, float* energies_dev, double* energy_dev,
                               float* forces_dev, double* virial_dev, void* stream_ptr) {
    return rune::guarded([&] {
        if (!engine) throw Error(RUNE_ERR_INVALID, "null engine");
        Engine& e = engine->impl;
        if (!e.finalized) throw Error(RUNE_ERR_STATE, "rune_engine_finalize was not called");
        if (n_atoms < 0 || n_structures < 1 || !atom_ptr_host)
            throw Error(RUNE_ERR_INVALID, "invalid batch description");
        if (atom_ptr_host[0] != 0 || atom_ptr_host[n_structures] != n_atoms)
            throw Error(RUNE_ERR_INVALID, "atom_ptr must start at 0 and end at n_atoms");
        for (int s = 0; s < n_structures; ++s)
            if (atom_ptr_host[s + 1] < atom_ptr_host[s])
                throw Error(RUNE_ERR_INVALID, "atom_ptr must be non-decreasing");
        if (!energy_dev) throw Error(RUNE_ERR_INVALID, "energy output is required");
        if ((flags & RUNE_FORCES) && !forces_dev)
            throw Error(RUNE_ERR_INVALID, "forces requested without an output buffer");
        if ((flags & RUNE_VIRIAL) && !virial_dev)
            throw Error(RUNE_ERR_INVALID, "virial requested without an output buffer");
        RUNE_CUDA_TRY(cudaSetDevice(e.device));
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        rune::with_workspace(e, stream, [&] {
            rune::PaddedInput in{n_atoms, n_structures, types_dev, positions_dev,
                                 radial_neighbors_dev, radial_width, radial_offsets_dev,
                                 angular_neighbors_dev, angular_width, angular_offsets_dev,
                                 atom_ptr_host};
            rune::CallTables ct = rune::stage_call_tables(e, n_structures, atom_ptr_host, stream);
            e.flush_uploads(stream);
            rune::NeighborData nd;
            rune::build_padded(e, in, nd, stream);
            // the pull-form force kernel needs symmetric lists: verify once per call
            rune::build_reverse(e, nd, nd.radial, nd.total_edges, stream);
            rune::build_reverse(e, nd, nd.angular, nd.total_angular, stream);
            rune::Outputs o{energies_dev, energy_dev, forces_dev, virial_dev, flags};
            rune::evaluate(e, nd, n_atoms, n_structures, types_dev, ct, o, stream);
            unsigned int flags_h = 0;
            RUNE_CUDA_TRY(cudaMemcpyAsync(&flags_h, e.d_flags, sizeof(unsigned int),
                                          cudaMemcpyDeviceToHost, stream));
            RUNE_CUDA_TRY(cudaStreamSynchronize(stream));
            e.check_flags(flags_h, stream);
            e.last_valid = false;
        });
    });
}

int rune_engine_neighbor_pairs(rune_engine* engine, int32_t which, int32_t* pairs_host,
                               int64_t capacity, int64_t* count) {
    return rune::guarded([&] {
        if (!engine || !count) throw Error(RUNE_ERR_INVALID, "null argument");
        Engine& e = engine->impl;
        if (!e.last_valid || !e.last.edges)
            throw Error(RUNE_ERR_STATE, "no device-built neighbour list available");
        RUNE_CUDA_TRY(cudaSetDevice(e.device));
        int n = e.last.n_atoms, total = e.last.total_edges;
        std::vector<int> row(n + 1), cnt(n + 1), shifts(total);
        std::vector<float4> edges(total);
        const rune::EdgeList& list = which == 0 ? e.last.radial : e.last.angular;
        const int* dcnt = list.cnt;
        RUNE_CUDA_TRY(cudaMemcpy(row.data(), list.row_ptr, sizeof(int) * (n > 0 ? n : 1),
                                 cudaMemcpyDeviceToHost));
        RUNE_CUDA_TRY(cudaMemcpy(cnt.data(), dcnt, sizeof(int) * (n > 0 ? n : 1),
                                 cudaMemcpyDeviceToHost));
        if (total > 0) {
            RUNE_CUDA_TRY(cudaMemcpy(edges.data(), e.last.edges, sizeof(float4) * total,
                                     cudaMemcpyDeviceToHost));
            RUNE_CUDA_TRY(cudaMemcpy(shifts.data(), e.last.shifts, sizeof(int) * total,
                                     cudaMemcpyDeviceToHost));
        }
        int64_t k = 0;
        auto sx = [](int v, int sh) {
            int x = (v >> sh) & 1023;
            return x >= 512 ? x - 1024 : x;
        };
        for (int i = 0; i < n; ++i)
            for (int m = 0; m < cnt[i]; ++m) {
                int idx = row[i] + m;
                if (pairs_host && k < capacity) {
                    int32_t* r = pairs_host + 5 * k;
                    float4 ed = edges[idx];
                    int j;
                    std::memcpy(&j, &ed.w, sizeof(int));
                    r[0] = i;
                    r[1] = j;
                    r[2] = sx(shifts[idx], 0);
                    r[3] = sx(shifts[idx], 10);
                    r[4] = sx(shifts[idx], 20);
                }
                ++k;
            }
        *count = k;
    });
}

int rune_md_nve(rune_engine* engine, int32_t n_atoms, const int32_t* types_dev,
                double* positions_dev, double* velocities_dev, const double* masses_dev,
                const double* cell_host, const uint8_t* pbc_host, double dt_fs, int32_t n_steps,
                double skin, double* energies_host, float* forces_dev, int64_t* rebuilds_host,
                void* stream_ptr) {
    return rune::guarded([&] {
        if (!engine) throw Error(RUNE_ERR_INVALID, "null engine");
        Engine& e = engine->impl;
        if (!e.finalized) throw Error(RUNE_ERR_STATE, "rune_engine_finalize was not called");
        if (n_atoms < 0 || n_steps < 0 || !cell_host || !pbc_host)
            throw Error(RUNE_ERR_INVALID, "invalid MD arguments");
        if (n_atoms > 0 && (!types_dev || !positions_dev || !velocities_dev || !masses_dev))
            throw Error(RUNE_ERR_INVALID, "MD state buffers are required");
        if (!(dt_fs > 0.0) || !(skin >= 0.0))
            throw Error(RUNE_ERR_INVALID, "dt must be positive and skin non-negative");
        RUNE_CUDA_TRY(cudaSetDevice(e.device));
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        rune::ProfilerInstall install(e);
        rune::MdArgs a{n_atoms, types_dev, positions_dev, velocities_dev, masses_dev, cell_host,
                       pbc_host, dt_fs, n_steps, skin, energies_host, forces_dev, rebuilds_host};
        rune::md_nve(e, a, stream);
        e.last_valid = false;
        rune::grow_staging(e);
    });
}

int rune_engine_stats(const rune_engine* engine, rune_stats* out) {
    return rune::guarded([&] {
        if (!engine || !out) throw Error(RUNE_ERR_INVALID, "null argument");
        *out = engine->impl.stats;
    });
}

void rune_engine_destroy(rune_engine* engine) {
    if (!engine) return;
    Engine& e = engine->impl;
    cudaSetDevice(e.device);
    if (e.blob) cudaFree(e.blob);
    if (e.eq_tc_buf) cudaFree(e.eq_tc_buf);
    if (e.ws.base) cudaFree(e.ws.base);
    if (e.d_flags) cudaFree(e.d_flags);
    if (e.host_sync) cudaFreeHost(e.host_sync);
    if (e.staging.base) cudaFreeHost(e.staging.base);
    if (e.d_mirror) cudaFree(e.d_mirror);
    e.prof.release();
    delete engine;
}

const char* rune_last_error(void) { return rune::g_last_error.c_str(); }

}  // extern "C"

// ============================================================================= profiling
namespace rune {

namespace {
thread_local Profiler* g_profiler = nullptr;
}

Profiler* current_profiler() { return g_profiler; }
void set_current_profiler(Profiler* p) { g_profiler = p; }

cudaEvent_t Profiler::event() {
    if (!pool.empty()) {
        cudaEvent_t e = pool.back();
        pool.pop_back();
        return e;
    }
    cudaEvent_t e;
    RUNE_CUDA_TRY(cudaEventCreate(&e));
    return e;
}

void Profiler::resolve() {
    for (auto& p : pending) {
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, p.start, p.stop) != cudaSuccess) {
            cudaGetLastError();
            ms = 0.f;
        }
        auto it = totals.find(p.name);
        if (it == totals.end()) {
            order.push_back(p.name);
            totals[p.name] = {ms, 1};
        } else {
            it->second.first += ms;
            it->second.second += 1;
        }
        pool.push_back(p.start);
        pool.push_back(p.stop);
    }
    pending.clear();
}

void Profiler::release() {
    for (auto& p : pending) {
        cudaEventDestroy(p.start);
        cudaEventDestroy(p.stop);
    }
    pending.clear();
    for (auto e : pool) cudaEventDestroy(e);
    pool.clear();
}

KernelScope::KernelScope(const char* kernel, cudaStream_t s, int n_launches)
    : prof(g_profiler), stream(s), name(kernel) {
    if (!prof) return;
    prof->launches += n_launches;
    if (!prof->timing) return;
    cudaEvent_t start = prof->event();
    stop = prof->event();
    RUNE_CUDA_TRY(cudaEventRecord(start, stream));
    prof->pending.push_back(Profiler::Pending{name, start, stop});
}

KernelScope::~KernelScope() {
    if (prof && prof->timing && stop) cudaEventRecord(stop, stream);
}

}  // namespace rune

extern "C" {

int rune_engine_set_profiling(rune_engine* engine, int32_t enabled) {
    return rune::guarded([&] {
        if (!engine) throw Error(RUNE_ERR_INVALID, "null engine");
        engine->impl.prof.timing = enabled != 0;
    });
}

static_assert(RUNE_DEFAULT_WAIT_POLLS == rune::kEqWaitPolls, "default wait bound");

int rune_engine_set_wait_polls(rune_engine* engine, uint32_t polls) {
    return rune::guarded([&] {
        if (!engine) throw Error(RUNE_ERR_INVALID, "null engine");
        engine->impl.wait_polls = polls;
        for (auto& L : engine->impl.eq) L.args.wait_polls = polls;
    });
}

int rune_engine_kernel_stat(const rune_engine* engine, int32_t index, char* name_buf,
                            int32_t name_capacity, double* total_ms, int64_t* launches) {
    return rune::guarded([&] {
        if (!engine) throw Error(RUNE_ERR_INVALID, "null engine");
        const auto& prof = engine->impl.prof;
        if (index < 0 || index >= (int32_t)prof.order.size())
            throw Error(RUNE_ERR_INVALID, "kernel stat index out of range");
        const std::string& name = prof.order[index];
        const auto& t = prof.totals.at(name);
        if (name_buf && name_capacity > 0) {
            std::snprintf(name_buf, name_capacity, "%s", name.c_str());
        }
        if (total_ms) *total_ms = t.first;
        if (launches) *launches = t.second;
    });
}

int rune_tc_selftest(int32_t M, int32_t N, int32_t K, const float* a_host, const float* b_host,
                     float* c_host, int32_t device) {
    return rune::guarded([&] {
        if (!a_host || !b_host || !c_host) throw Error(RUNE_ERR_INVALID, "null argument");
        rune::tc_selftest(M, N, K, a_host, b_host, c_host, device);
    });
}

int rune_engine_reset_kernel_stats(rune_engine* engine) {
    return rune::guarded([&] {
        if (!engine) throw Error(RUNE_ERR_INVALID, "null engine");
        engine->impl.prof.totals.clear();
        engine->impl.prof.order.clear();
    });
}

}  // extern "C"

// ============================================================================= static scratch
// Scratch for rune_engine_compute_padded_static: one fixed device array, so the call allocates
// nothing. Host code cannot use the symbol itself as a device address; the address is looked
// up once per device (cudaGetSymbolAddress, with that device current) and cached.
namespace rune {
namespace {

constexpr size_t kStaticScratchBytes = RUNE_STATIC_SCRATCH_BYTES;
__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_static_mutex;
void* g_static_ptr[kMaxDevices] = {};

void* static_scratch_for(int device) {
    if (device < 0 || device >= kMaxDevices)
        throw Error(RUNE_ERR_INVALID, "device index out of range for the static scratch");
    std::lock_guard<std::mutex> lock(g_static_mutex);
    if (!g_static_ptr[device]) {
        void* ptr = nullptr;
        cudaError_t err = cudaGetSymbolAddress(&ptr, g_static_scratch);
        if (err != cudaSuccess || !ptr)
            throw Error(RUNE_ERR_CUDA, std::string("cudaGetSymbolAddress(static scratch): ") +
                                           cudaGetErrorString(err));
        g_static_ptr[device] = ptr;
    }
    return g_static_ptr[device];
}

}  // namespace
}  // namespace rune

extern "C" int rune_engine_compute_padded_static(
    rune_engine* engine, int32_t n_atoms, int32_t n_structures, const int32_t* types_dev,
    const float* positions_dev, const int64_t* radial_neighbors_dev, int32_t radial_width,
    const float* radial_offsets_dev, const int64_t* angular_neighbors_dev, int32_t angular_width,
    const float* angular_offsets_dev, const int32_t* atom_ptr_host, int32_t flags,
    float* energies_dev, double* energy_dev, float* forces_dev, double* virial_dev,
    void* stream_ptr) {
    return rune::guarded([&] {
        if (!engine) throw Error(RUNE_ERR_INVALID, "null engine");
        Engine& e = engine->impl;
        if (!e.finalized) throw Error(RUNE_ERR_STATE, "rune_engine_finalize was not called");
        if (n_atoms < 0 || n_structures < 1 || !atom_ptr_host)
            throw Error(RUNE_ERR_INVALID, "invalid batch description");
        if (atom_ptr_host[0] != 0 || atom_ptr_host[n_structures] != n_atoms)
            throw Error(RUNE_ERR_INVALID, "atom_ptr must start at 0 and end at n_atoms");
        for (int s = 0; s < n_structures; ++s)
            if (atom_ptr_host[s + 1] < atom_ptr_host[s])
                throw Error(RUNE_ERR_INVALID, "atom_ptr must be non-decreasing");
        if (!energy_dev) throw Error(RUNE_ERR_INVALID, "energy output is required");
        if ((flags & RUNE_FORCES) && !forces_dev)
            throw Error(RUNE_ERR_INVALID, "forces requested without an output buffer");
        if ((flags & RUNE_VIRIAL) && !virial_dev)
            throw Error(RUNE_ERR_INVALID, "virial requested without an output buffer");
        RUNE_CUDA_TRY(cudaSetDevice(e.device));
        void* scratch = rune::static_scratch_for(e.device);
        cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
        // carve this call's arrays from the static array instead of the engine's workspace
        rune::Arena saved = e.ws;
        e.ws.base = static_cast<char*>(scratch);
        e.ws.cap = rune::kStaticScratchBytes;
        e.ws.reset();
        e.static_call = true;
        e.staging.off = 0;
        e.stage_first = ~size_t(0);
        rune::ProfilerInstall install(e);
        try {
            rune::PaddedInput in{n_atoms, n_structures, types_dev, positions_dev,
                                 radial_neighbors_dev, radial_width, radial_offsets_dev,
                                 angular_neighbors_dev, angular_width, angular_offsets_dev,
                                 atom_ptr_host};
            rune::CallTables ct = rune::stage_call_tables(e, n_structures, atom_ptr_host, stream);
            e.flush_uploads(stream);
            rune::NeighborData nd;
            rune::build_padded(e, in, nd, stream);
            rune::build_reverse(e, nd, nd.radial, nd.total_edges, stream);
            rune::build_reverse(e, nd, nd.angular, nd.total_angular, stream);
            rune::Outputs o{energies_dev, energy_dev, forces_dev, virial_dev, flags};
            rune::evaluate(e, nd, n_atoms, n_structures, types_dev, ct, o, stream);
            unsigned int flags_h = 0;
            RUNE_CUDA_TRY(cudaMemcpyAsync(&flags_h, e.d_flags, sizeof(unsigned int),
                                          cudaMemcpyDeviceToHost, stream));
            RUNE_CUDA_TRY(cudaStreamSynchronize(stream));
            e.check_flags(flags_h, stream);
            e.prof.resolve();
        } catch (const Error& err) {
            cudaStreamSynchronize(stream);
            e.prof.resolve();
            size_t want = e.ws.want;
            e.ws = saved;
            e.static_call = false;
            e.last_valid = false;
            if (err.code == -1)
                throw Error(RUNE_ERR_INVALID,
                            "rune_engine_compute_padded_static: this batch needs at least " +
                                std::to_string(want) + " bytes of scratch; the static scratch "
                                "holds " + std::to_string(rune::kStaticScratchBytes) +
                                " bytes. Use rune_engine_compute_padded for larger batches.");
            throw;
        }
        e.ws = saved;
        e.static_call = false;
        e.last_valid = false;
    });
}
