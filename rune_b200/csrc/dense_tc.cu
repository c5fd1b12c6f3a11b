// Tensor-core (tcgen05, kind::i8) GEMM with float32-level, unbiased results:
//
//   C[M, N] = epilogue(A[M, K] @ B[K, N]),  A = activations (row-major, float32),
//                                           B = a weight matrix (packed once, tc_pack)
//
// Exact-integer products (the Ozaki scheme on integer tensor cores). Every row of A and every
// column of B gets a power-of-two scale 2^e with all its |x| < 2^e; each value then splits
// exactly into four signed 7-bit digits (tc::split_digits),
//   x = 2^(e - 6) (d0 + d1 2^-7 + d2 2^-14 + d3 2^-21) + r,   |r| <= 2^(e - 28),
// and the dot product is 2^(ea + eb - 12) sum_t 2^(-7 t) D_t with
//   D_t = sum_{p + q = t} A_p . B_q   (t = 0 .. 3: ten int8 products per K step).
// The tensor core accumulates the D_t exactly in int32 (|D_t| <= 4 * 64 * 64 * K < 2^31 for
// K <= 8192), so the only roundings are the digit truncation (2^-28 of the row's / column's
// largest entry) and one rounding of the float64 combination to float32: no accumulation
// rounding, hence no bias (a tf32 split accumulated in the tensor core's float32 accumulator
// rounds every step toward zero, which the residual Möbius networks compound).
//
// The engine's dense layers do not route to this kernel: measured on B200 it is slower than the
// SIMT kernel of dense.cu on the OAM layer shapes (each block splits its A tile into digits
// again for every 64 output columns), and one scale per row of A keeps only 2^-28 of the row's
// largest entry, which the descriptor input of the config-3 structures (entries spread over
// many orders) does not tolerate (forces 2e-4 eV/A off). rune_tc_selftest checks it.
//
// One block computes a 128 x 64 tile of C (tcgen05.mma.cta_group::1.kind::i8, M = 128,
// N = 64, K = 32 per instruction) with the four D_t in TMEM (4 x 64 = 256 columns, two blocks
// per SM). Operands are K-major "core matrices" of 8 rows x 16 bytes, no swizzle: in a K step
// of 32, element (r, k) of a digit plane sits at byte (r / 8) 256 + (k / 16) 128 + (r % 8) 16 +
// k % 16 (leading byte offset 128, stride byte offset 256).
//
// Roles in the 256-thread block:
//   all threads     first the exponent of each of the tile's 128 rows of A (warp per 16 rows);
//   thread 0        issues the MMAs (10 per K step) and the commits;
//   thread 32       streams B by bulk copies (units of 8 KB: four digit planes of 64 x 32);
//   warps 2 .. 7    load the A slice of each K step (128 rows x 32 k), split it into digits and
//                   store the four planes (16 KB);
//   all threads     the epilogue: D_t from TMEM (warp w reads lanes 32 (w % 4) .., columns
//                   32 (w / 4) ..), combined in float64, scaled, epilogue functions, stored.
// A ring of kStages slots carries one K step each; every wait is bounded (error flag 32 on
// give-up, after which the block drains what it issued and stores nothing).

#include <cstring>

#include "engine.cuh"
#include "umma.cuh"

namespace rune {

namespace {

constexpr int kBM = 128, kBN = 64, kBK = 32;
constexpr int kStages = 4;
constexpr int kDigits = 4;
constexpr uint32_t kAPlane = kBM * kBK;              // bytes of one digit plane of A
constexpr uint32_t kBPlane = kBN * kBK;              // bytes of one digit plane of B
constexpr uint32_t kAUnit = kDigits * kAPlane;       // 16 KB per K step
constexpr uint32_t kBUnit = kDigits * kBPlane;       // 8 KB per K step
constexpr uint32_t kTmemCols = kDigits * kBN;        // 256
constexpr int kProducers = 192;                      // warps 2 .. 7

struct GemmShared {
    unsigned long long full_a[kStages];  // A slice stored (kProducers arrivals)
    unsigned long long full_b[kStages];  // B unit landed (bulk-copy bytes)
    unsigned long long empty[kStages];   // MMAs of the slot complete
    unsigned long long done;
    uint32_t tmem;
    int fail;
    int issued_b;  // B units whose copy was issued
    int row_exp[kBM];
};

struct GemmSmem {
    size_t ring, shared, total;  // byte offsets
    __host__ __device__ GemmSmem() {
        ring = 0;
        shared = ring + (size_t)kStages * (kAUnit + kBUnit);
        total = shared + sizeof(GemmShared);
    }
};

// Byte offset of element (r, k) (k < 32) inside one K-major digit plane.
__device__ __forceinline__ uint32_t plane_offset(int r, int k) {
    return (uint32_t)((r >> 3) * 256 + (k >> 4) * 128 + (r & 7) * 16 + (k & 15));
}

// Epilogue of one output element from its float64 dot product (as the SIMT kernel's).
__device__ __forceinline__ void tc_store(const GemmEpilogue& ep, int m, int n, int N, int ldc,
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

__global__ void __launch_bounds__(256, 1)
k_gemm_tc(int M, int N, int K, const float* __restrict__ A, int lda,
          const signed char* __restrict__ Bq, const int* __restrict__ col_exp, int nblocks_n,
          float* __restrict__ C, int ldc, GemmEpilogue ep, unsigned* __restrict__ err) {
    using namespace tc;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    GemmSmem L;
    unsigned char* ring = smem_raw + L.ring;
    auto* sh = reinterpret_cast<GemmShared*>(smem_raw + L.shared);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nb = blockIdx.x, m0 = blockIdx.y * kBM, n0 = nb * kBN;
    const int ns = (K + kBK - 1) / kBK;
    auto slot_a = [&](int st) { return ring + (size_t)st * (kAUnit + kBUnit); };
    auto slot_b = [&](int st) { return slot_a(st) + kAUnit; };

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&sh->full_a[s]), kProducers);
            mbar_init(smem_u32(&sh->full_b[s]), 1);
            mbar_init(smem_u32(&sh->empty[s]), 1);
        }
        mbar_init(smem_u32(&sh->done), 1);
        sh->issued_b = 0;
        sh->fail = 0;
        asm volatile("fence.mbarrier_init.release.cluster;");
    }
    // exponent of every row of the tile: a warp per 16 rows, lanes along K
    for (int rr = 0; rr < kBM / 8; ++rr) {
        int r = warp * (kBM / 8) + rr, m = m0 + r;
        float amax = 0.0f;
        if (m < M)
            for (int k = lane; k < K; k += 32) amax = fmaxf(amax, fabsf(A[(size_t)m * lda + k]));
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (lane == 0) sh->row_exp[r] = digit_exponent(amax);
    }
    if (warp == 0) tmem_alloc(&sh->tmem, kTmemCols);
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = sh->tmem;

    if (tid == 32) {
        // B producer: unit (s, nb) of the packed weights into slot s % kStages
        for (int s = 0; s < ns; ++s) {
            int st = s % kStages, use = s / kStages;
            if (use > 0 && !mbar_wait(smem_u32(&sh->empty[st]), (use - 1) & 1)) {
                atomicOr(err, 32u);
                sh->fail = 1;
                break;
            }
            if (*(volatile int*)&sh->fail) break;
            uint32_t bar = smem_u32(&sh->full_b[st]);
            mbar_expect_tx(bar, kBUnit);
            bulk_g2s(smem_u32(slot_b(st)), Bq + ((size_t)s * nblocks_n + nb) * kBUnit, kBUnit,
                     bar);
            *(volatile int*)&sh->issued_b = s + 1;
        }
    } else if (warp >= 2) {
        // A producers: 128 rows x 32 k per step; a thread takes four consecutive k of a row
        const int t = tid - 64;  // 0 .. 191
        for (int s = 0; s < ns; ++s) {
            int st = s % kStages, use = s / kStages;
            if (use > 0 && !mbar_wait(smem_u32(&sh->empty[st]), (use - 1) & 1)) {
                atomicOr(err, 32u);
                sh->fail = 1;
                break;
            }
            if (*(volatile int*)&sh->fail) break;
            unsigned char* planes = slot_a(st);
            for (int u = t; u < kBM * (kBK / 4); u += kProducers) {
                int r = u >> 3, kq = (u & 7) * 4, m = m0 + r;
                int e = sh->row_exp[r];
                uint32_t w[kDigits] = {0u, 0u, 0u, 0u};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    int k = s * kBK + kq + j;
                    float x = (m < M && k < K) ? __ldg(A + (size_t)m * lda + k) : 0.0f;
                    int d[kDigits];
                    split_digits(x, e, d);
#pragma unroll
                    for (int p = 0; p < kDigits; ++p) w[p] |= (uint32_t)(d[p] & 0xff) << (8 * j);
                }
                uint32_t off = plane_offset(r, kq);
#pragma unroll
                for (int p = 0; p < kDigits; ++p)
                    *reinterpret_cast<uint32_t*>(planes + p * kAPlane + off) = w[p];
            }
            fence_async_smem();
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];"
                         ::"r"(smem_u32(&sh->full_a[st])) : "memory");
        }
    } else if (tid == 0) {
        // MMA issuer: D_t += A_p . B_q for p + q = t <= 3
        const uint32_t idesc = idesc_i8(kBM, kBN);
        for (int s = 0; s < ns; ++s) {
            int st = s % kStages, use = s / kStages;
            if (!mbar_wait(smem_u32(&sh->full_b[st]), use & 1) ||
                !mbar_wait(smem_u32(&sh->full_a[st]), use & 1) || *(volatile int*)&sh->fail) {
                atomicOr(err, 32u);
                sh->fail = 1;
                break;
            }
            fence_after_sync();
            uint32_t a0 = smem_u32(slot_a(st)), b0 = smem_u32(slot_b(st));
#pragma unroll
            for (int tt = 0; tt < kDigits; ++tt) {
#pragma unroll
                for (int p = 0; p <= tt; ++p) {
                    int q = tt - p;
                    uint64_t ad = smem_desc(a0 + p * kAPlane, kALbo, kASbo);
                    uint64_t bd = smem_desc(b0 + q * kBPlane, kALbo, kASbo);
                    mma_i8(tmem + (uint32_t)(tt * kBN), ad, bd, idesc,
                           (s > 0 || p > 0) ? 1u : 0u);
                }
            }
            mma_commit(smem_u32(&sh->empty[st]));
        }
        mma_commit(smem_u32(&sh->done));
    }
    // everyone: wait for the last MMAs, then the epilogue
    __syncthreads();
    bool ok = !sh->fail;
    if (ok && !mbar_wait(smem_u32(&sh->done), 0)) {
        if (tid == 0) atomicOr(err, 32u);
        ok = false;
    }
    ok = __syncthreads_and(ok);
    if (!ok && tid == 0) {
        // drain (bounded): the last copy issued into each slot lands before the block exits
        int issued = sh->issued_b;
        for (int s = issued - kStages > 0 ? issued - kStages : 0; s < issued; ++s)
            mbar_wait(smem_u32(&sh->full_b[s % kStages]), (s / kStages) & 1);
    }
    fence_after_sync();
    if (ok) {
        const int q = warp & 3, half = warp >> 2;
        const int r = 32 * q + lane, m = m0 + r;
        const int c0 = 32 * half;
        double acc[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = 0.0;
#pragma unroll
        for (int tt = kDigits - 1; tt >= 0; --tt) {
            float v[32];
            tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(tt * kBN + c0), v);
#pragma unroll
            for (int j = 0; j < 32; ++j)
                acc[j] = acc[j] * 0.0078125 + (double)__float_as_int(v[j]);
        }
        // acc = sum_t 2^(-7 t) D_t (exact in float64: Horner from the last digit)
        if (m < M) {
            int ea = sh->row_exp[r];
#pragma unroll 4
            for (int j = 0; j < 32; ++j) {
                int n = n0 + c0 + j;
                if (n < N) {
                    double val = ldexp(acc[j], ea + __ldg(col_exp + n) - 12);
                    tc_store(ep, m, n, N, ldc, val, C);
                }
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        fence_after_sync();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// Packs B [K][N] (row-major: W^T or W of a layer) into tensor-core units: unit (s, b) = K step
// s (k in [32 s, 32 s + 32)) x column block b (n in [64 b, 64 b + 64)) at byte
// (s * NB + b) * 8192, digit planes 0 .. 3 of 2048 bytes each; element (n, k) of a plane at
// ((n % 64) / 8) 256 + ((k % 32) / 16) 128 + (n % 8) 16 + k % 16. One thread per (unit, n)
// reads the column exponent computed by k_tc_col_exp.
__global__ void k_tc_col_exp(const float* __restrict__ B, int K, int N, int NB,
                             int* __restrict__ col_exp) {
    int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= NB * kBN) return;
    float amax = 0.0f;
    if (n < N)
        for (int k = 0; k < K; ++k) amax = fmaxf(amax, fabsf(B[(size_t)k * N + n]));
    col_exp[n] = tc::digit_exponent(amax);
}

__global__ void k_tc_pack(const float* __restrict__ B, int K, int N, int NB,
                          const int* __restrict__ col_exp, signed char* __restrict__ out) {
    long long total = (long long)((K + kBK - 1) / kBK * kBK) * NB * kBN;
    for (long long o = blockIdx.x * (long long)blockDim.x + threadIdx.x; o < total;
         o += (long long)gridDim.x * blockDim.x) {
        int n = (int)(o % (NB * kBN)), k = (int)(o / (NB * kBN));
        float x = (k < K && n < N) ? B[(size_t)k * N + n] : 0.0f;
        int d[kDigits];
        tc::split_digits(x, col_exp[n], d);
        int s = k / kBK, b = n / kBN, nn = n % kBN, kk = k % kBK;
        size_t unit = ((size_t)s * NB + b) * kBUnit;
        uint32_t at = (uint32_t)((nn >> 3) * 256 + (kk >> 4) * 128 + (nn & 7) * 16 + (kk & 15));
#pragma unroll
        for (int p = 0; p < kDigits; ++p) out[unit + p * kBPlane + at] = (signed char)d[p];
    }
}

}  // namespace

size_t gemm_tc_smem() { return GemmSmem().total; }

// bytes of a packed operand: the digit units, then the column exponents (int32, padded)
size_t tc_packed_bytes(int K, int N) {
    size_t ns = (size_t)((K + kBK - 1) / kBK), nb = (size_t)((N + kBN - 1) / kBN);
    return ns * nb * kBUnit + nb * kBN * sizeof(int);
}

void tc_pack(const float* B, int K, int N, void* out, cudaStream_t stream) {
    int NB = (N + kBN - 1) / kBN;
    size_t ns = (size_t)((K + kBK - 1) / kBK);
    signed char* q = static_cast<signed char*>(out);
    int* col_exp = reinterpret_cast<int*>(q + ns * NB * kBUnit);
    k_tc_col_exp<<<(NB * kBN + 127) / 128, 128, 0, stream>>>(B, K, N, NB, col_exp);
    long long total = (long long)ns * kBK * NB * kBN;
    int blocks = (int)std::min<long long>((total + 255) / 256, 4096);
    k_tc_pack<<<blocks, 256, 0, stream>>>(B, K, N, NB, col_exp, q);
    RUNE_CUDA_TRY(cudaGetLastError());
}

void gemm_tc(int M, int N, int K, const float* A, int lda, const TcMatrix& B, float* C, int ldc,
             const GemmEpilogue& ep, unsigned* err, cudaStream_t stream) {
    if (M == 0 || N == 0) return;
    if (B.K != K || B.N != N) throw Error(RUNE_ERR_INVALID, "tensor-core operand shape mismatch");
    if (K > 8192) throw Error(RUNE_ERR_INVALID, "tensor-core GEMM: K above 8192");
    size_t bytes = gemm_tc_smem();
    RUNE_CUDA_TRY(cudaFuncSetAttribute((const void*)k_gemm_tc,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    int nblocks_n = (N + kBN - 1) / kBN;
    size_t ns = (size_t)((K + kBK - 1) / kBK);
    const signed char* q = static_cast<const signed char*>(B.w);
    const int* col_exp = reinterpret_cast<const int*>(q + ns * nblocks_n * kBUnit);
    dim3 grid(nblocks_n, (M + kBM - 1) / kBM);
    RUNE_KERNEL("k_gemm_tc", stream,
                k_gemm_tc<<<grid, 256, bytes, stream>>>(M, N, K, A, lda, q, col_exp, nblocks_n,
                                                         C, ldc, ep, err));
    RUNE_LAUNCH_CHECK();
}

void tc_selftest(int M, int N, int K, const float* a_host, const float* b_host, float* c_host,
                 int device) {
    if (M < 1 || N < 1 || K < 1 || M > 65536 || N > 4096 || K > 4096)
        throw Error(RUNE_ERR_INVALID,
                    "tc self-test sizes: 1 <= M <= 65536, 1 <= N <= 4096, 1 <= K <= 4096");
    RUNE_CUDA_TRY(cudaSetDevice(device));
    size_t fa = (size_t)M * K, fb = (size_t)K * N, fc = (size_t)M * N;
    size_t pb = tc_packed_bytes(K, N);
    size_t off_b = fa * 4, off_c = off_b + fb * 4;
    size_t off_p = (off_c + fc * 4 + 255) & ~size_t(255);
    size_t off_e = (off_p + pb + 255) & ~size_t(255);
    char* buf = nullptr;
    RUNE_CUDA_TRY(cudaMalloc(&buf, off_e + 256));
    struct Free {
        char* p;
        ~Free() { cudaFree(p); }
    } guard{buf};
    float* da = reinterpret_cast<float*>(buf);
    float* db = reinterpret_cast<float*>(buf + off_b);
    float* dc = reinterpret_cast<float*>(buf + off_c);
    void* dp = buf + off_p;
    unsigned* derr = reinterpret_cast<unsigned*>(buf + off_e);
    RUNE_CUDA_TRY(cudaMemcpy(da, a_host, sizeof(float) * fa, cudaMemcpyHostToDevice));
    RUNE_CUDA_TRY(cudaMemcpy(db, b_host, sizeof(float) * fb, cudaMemcpyHostToDevice));
    RUNE_CUDA_TRY(cudaMemset(derr, 0, sizeof(unsigned)));
    tc_pack(db, K, N, dp, nullptr);
    GemmEpilogue ep;
    gemm_tc(M, N, K, da, K, TcMatrix{dp, K, N}, dc, N, ep, derr, nullptr);
    RUNE_CUDA_TRY(cudaDeviceSynchronize());
    unsigned flag = 0;
    RUNE_CUDA_TRY(cudaMemcpy(&flag, derr, sizeof(unsigned), cudaMemcpyDeviceToHost));
    if (flag) throw Error(RUNE_ERR_CUDA, "tc self-test: a bounded wait gave up (flag 32)");
    RUNE_CUDA_TRY(cudaMemcpy(c_host, dc, sizeof(float) * fc, cudaMemcpyDeviceToHost));
}

}  // namespace rune
