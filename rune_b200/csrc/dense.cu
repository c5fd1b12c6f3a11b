// Dense per-atom layers of the Möbius network: a tiled fp32 GEMM with fused epilogues and the
// row-wise RMSNorm / readout kernels.
//
// Forward and backward of rune/mobius/layers.py (RMSNorm :26-44, ResidualBlock :47-67,
// ElementwiseLinearHead :70-89) and the input projection of rune/mobius/model.py:267-268.
// RMSNorm weights are folded into the following layer's matrix at load time, so a normalised
// GEMM is C = rho[m] * (h @ (diag(gamma) W^T)) and needs only the per-row 1/rms.

#include "engine.cuh"

namespace rune {

namespace {

constexpr int BM = 64, BN = 64, BK = 16, TM = 4, TN = 4;

// Scratch for split-K products (float64 partials), set by the caller for the calls of one
// evaluation on this thread; null: no split.
thread_local double* g_split_ws = nullptr;
thread_local size_t g_split_cap = 0;

// Epilogue of one output element from its float64 dot product.
__device__ __forceinline__ void gemm_store(const GemmEpilogue& ep, int m, int n, int N, int ldc,
                                           double acc, float* __restrict__ C) {
    float rs = ep.row_scale ? ep.row_scale[m] : 1.0f;
    float v = (float)(acc * (double)rs);
    if (ep.bias) v += __ldg(ep.bias + n);
    if (ep.emb) v += __ldg(ep.emb + (size_t)ep.types[m] * N + n);
    size_t o = (size_t)m * ldc + n;
    if (ep.act >= 0) {
        float y, dy;
        activation(ep.act, v, y, dy);
        v = y;
        if (ep.dact) ep.dact[o] = dy;
    }
    if (ep.residual) v += ep.residual[o];
    if (ep.mul) v *= ep.mul[o];
    C[o] = v;
}

// Acc = double: fp32 operands; each BK-wide slice of the dot product is summed in float32 and
// the slice sums are accumulated in float64 (the residual stream of the Möbius network reaches
// magnitudes where a float32 sum over the whole of K costs ~1e-6 eV/atom; a 16-term float32
// partial keeps the FP32 pipes busy and the error at the level of float32 products).
// Split-K: block z covers k in [z ks, (z + 1) ks) and, with `part`, writes its float64 dot
// products to part[z][M][N] instead of applying the epilogue.
template <typename Acc>
__global__ void __launch_bounds__(256)
k_gemm(int M, int N, int K, const float* __restrict__ A, int lda, const float* __restrict__ B,
       int ldb, float* __restrict__ C, int ldc, GemmEpilogue ep, int ks,
       double* __restrict__ part) {
    const int kb = blockIdx.z * ks, ke = min(K, kb + ks);
    __shared__ float As[2][BK][BM + 4];
    __shared__ float Bs[2][BK][BN];
    int tid = threadIdx.x;
    int tx = tid & 15, ty = tid >> 4;
    int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    Acc acc[TM][TN];
#pragma unroll
    for (int a = 0; a < TM; ++a)
#pragma unroll
        for (int b = 0; b < TN; ++b) acc[a][b] = Acc(0);

    // loaders: A tile 64x16 (4 per thread), B tile 16x64 (4 per thread)
    int a_row = tid >> 2, a_k = (tid & 3) * 4;
    int b_k = tid >> 4, b_col = (tid & 15) * 4;
    float ra[4], rb[4];
    auto load = [&](int k0) {
        int m = m0 + a_row;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            int k = k0 + a_k + q;
            ra[q] = (m < M && k < ke) ? __ldg(A + (size_t)m * lda + k) : 0.0f;
        }
        int k = k0 + b_k;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            int n = n0 + b_col + q;
            rb[q] = (k < ke && n < N) ? __ldg(B + (size_t)k * ldb + n) : 0.0f;
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int q = 0; q < 4; ++q) As[buf][a_k + q][a_row] = ra[q];
#pragma unroll
        for (int q = 0; q < 4; ++q) Bs[buf][b_k][b_col + q] = rb[q];
    };
    int tiles = (ke - kb + BK - 1) / BK;
    load(kb);
    store(0);
    __syncthreads();
    for (int t = 0; t < tiles; ++t) {
        int buf = t & 1;
        if (t + 1 < tiles) load(kb + (t + 1) * BK);
        float part[TM][TN];
#pragma unroll
        for (int a = 0; a < TM; ++a)
#pragma unroll
            for (int b = 0; b < TN; ++b) part[a][b] = 0.0f;
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            float av[TM], bv[TN];
#pragma unroll
            for (int a = 0; a < TM; ++a) av[a] = As[buf][k][ty * TM + a];
#pragma unroll
            for (int b = 0; b < TN; ++b) bv[b] = Bs[buf][k][tx * TN + b];
#pragma unroll
            for (int a = 0; a < TM; ++a)
#pragma unroll
                for (int b = 0; b < TN; ++b) part[a][b] = fmaf(av[a], bv[b], part[a][b]);
        }
#pragma unroll
        for (int a = 0; a < TM; ++a)
#pragma unroll
            for (int b = 0; b < TN; ++b) acc[a][b] += (Acc)part[a][b];
        if (t + 1 < tiles) store(buf ^ 1);
        __syncthreads();
    }
#pragma unroll
    for (int a = 0; a < TM; ++a) {
        int m = m0 + ty * TM + a;
        if (m >= M) continue;
#pragma unroll
        for (int b = 0; b < TN; ++b) {
            int n = n0 + tx * TN + b;
            if (n >= N) continue;
            if (part)
                part[((size_t)blockIdx.z * M + m) * N + n] = (double)acc[a][b];
            else
                gemm_store(ep, m, n, N, ldc, (double)acc[a][b], C);
        }
    }
}

// Sum of the split-K partials in split order, then the epilogue.
__global__ void k_gemm_finish(int M, int N, int splits, const double* __restrict__ part,
                              float* __restrict__ C, int ldc, GemmEpilogue ep) {
    long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long long)M * N) return;
    int m = (int)(idx / N), n = (int)(idx % N);
    double acc = 0.0;
    for (int z = 0; z < splits; ++z) acc += part[(size_t)z * M * N + idx];
    gemm_store(ep, m, n, N, ldc, acc, C);
}

// 1 / sqrt(mean(h^2) + eps) per row, warp per row, accumulated in float64.
__global__ void k_row_rms(int M, int H, const float* __restrict__ h, int ld, float eps,
                          float* __restrict__ rho) {
    int m = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (m >= M) return;
    double s = 0.0;
    for (int k = lane; k < H; k += 32) {
        double v = h[(size_t)m * ld + k];
        s += v * v;
    }
    s = warp_sum(s);
    if (lane == 0) rho[m] = (float)(1.0 / sqrt(s / H + (double)eps));
}

// dh += rho * dup - rho^3 / H * (dup . h) h, where dup = gamma * (dL/d normalised).
__global__ void k_rms_back(int M, int H, const float* __restrict__ h,
                           const float* __restrict__ rho, const float* __restrict__ dup,
                           float* __restrict__ dh) {
    int m = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (m >= M) return;
    const float* hr = h + (size_t)m * H;
    const float* dr = dup + (size_t)m * H;
    double dot = 0.0;
    for (int k = lane; k < H; k += 32) dot += (double)dr[k] * hr[k];
    dot = warp_sum(dot);
    float r = rho[m];
    float c = (float)((double)r * r * r * dot / H);
    float* out = dh + (size_t)m * H;
    for (int k = lane; k < H; k += 32) out[k] += r * dr[k] - c * hr[k];
}

// E = w[t] . RMSNorm(h) + b[t] and dE/dh (rune/mobius/layers.py:70-89, model.py:302).
__global__ void k_readout(int M, int H, const float* __restrict__ h, const int* __restrict__ types,
                          const float* __restrict__ gamma, const float* __restrict__ head_w,
                          const float* __restrict__ head_b, float eps, double* __restrict__ e,
                          float* __restrict__ dh) {
    int m = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (m >= M) return;
    int t = types[m];
    const float* hr = h + (size_t)m * H;
    const float* wr = head_w + (size_t)t * H;
    double ss = 0.0, dot = 0.0;
    for (int k = lane; k < H; k += 32) {
        double v = hr[k];
        ss += v * v;
        dot += v * ((double)gamma[k] * wr[k]);
    }
    ss = warp_sum(ss);
    dot = warp_sum(dot);
    double rho = 1.0 / sqrt(ss / H + (double)eps);
    if (lane == 0) e[m] = rho * dot + (double)head_b[t];
    if (dh) {
        float r = (float)rho;
        float c = (float)(rho * rho * rho * dot / H);
        for (int k = lane; k < H; k += 32) dh[(size_t)m * H + k] = r * gamma[k] * wr[k] - c * hr[k];
    }
}

}  // namespace

void set_gemm_split_scratch(double* ws, size_t cap) {
    g_split_ws = ws;
    g_split_cap = cap;
}

// Grids of fewer blocks than SMs (few rows) split K so that about two blocks per SM run, each
// over a shorter dependent chain of K tiles, when split scratch is available.
void gemm(int M, int N, int K, const float* A, int lda, const float* B, int ldb, float* C,
          int ldc, const GemmEpilogue& ep, cudaStream_t stream) {
    if (M == 0 || N == 0) return;
    int gx = (N + BN - 1) / BN, gy = (M + BM - 1) / BM;
    int tiles = (K + BK - 1) / BK;
    int splits = 1;
    constexpr int kSms = 148;
    if (g_split_ws && gx * gy < kSms && tiles >= 4) {
        splits = std::min(tiles / 2, (2 * kSms + gx * gy - 1) / (gx * gy));
        while (splits > 1 && (size_t)splits * M * N > g_split_cap) --splits;
    }
    if (splits > 1) {
        int tps = (tiles + splits - 1) / splits;  // K tiles per split
        splits = (tiles + tps - 1) / tps;
        RUNE_KERNEL("k_gemm", stream,
                    k_gemm<double><<<dim3(gx, gy, splits), 256, 0, stream>>>(
                        M, N, K, A, lda, B, ldb, C, ldc, ep, tps * BK, g_split_ws));
        RUNE_LAUNCH_CHECK();
        long long total = (long long)M * N;
        RUNE_KERNEL("k_gemm_finish", stream,
                    k_gemm_finish<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(
                        M, N, splits, g_split_ws, C, ldc, ep));
        RUNE_LAUNCH_CHECK();
        return;
    }
    RUNE_KERNEL("k_gemm", stream,
                k_gemm<double><<<dim3(gx, gy, 1), 256, 0, stream>>>(M, N, K, A, lda, B, ldb, C,
                                                                   ldc, ep, K, nullptr));
    RUNE_LAUNCH_CHECK();
}

void row_rms(int M, int H, const float* h, int ld, float eps, float* rho, cudaStream_t stream) {
    if (M == 0) return;
    RUNE_KERNEL("k_row_rms", stream, k_row_rms<<<(M * 32 + 255) / 256, 256, 0, stream>>>(M, H, h, ld, eps, rho));
    RUNE_LAUNCH_CHECK();
}

void rms_backward_add(int M, int H, const float* h, const float* rho, const float* dup,
                      float* dh, cudaStream_t stream) {
    if (M == 0) return;
    RUNE_KERNEL("k_rms_back", stream, k_rms_back<<<(M * 32 + 255) / 256, 256, 0, stream>>>(M, H, h, rho, dup, dh));
    RUNE_LAUNCH_CHECK();
}

void readout(int M, int H, const float* h, const int* types, const float* gamma,
             const float* head_w, const float* head_b, float eps, double* e_model, float* dh,
             cudaStream_t stream) {
    if (M == 0) return;
    RUNE_KERNEL("k_readout", stream, k_readout<<<(M * 32 + 255) / 256, 256, 0, stream>>>(M, H, h, types, gamma, head_w, head_b,
                                                         eps, e_model, dh));
    RUNE_LAUNCH_CHECK();
}

}  // namespace rune
