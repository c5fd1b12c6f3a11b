// Tensor-core (tcgen05) GEMM for the shape of the dense per-atom layers of the Möbius network:
//
//   C[M, N] = epilogue(A[M, K] @ B[K, N]),  A = activations (row-major, float32),
//                                           B = a weight matrix (packed once, tc_pack)
//
// One block computes a 128 x 128 tile of C with M = 128 rows per MMA (tcgen05.mma.cta_group::1
// .kind::tf32, N = 128, K = 8 per instruction). Float32-level products come from a three-term
// tf32 split, x = hi + lo (hi = x rounded to tf32, lo = x - hi rounded to tf32):
// a.b ~= hi.hi + hi.lo + lo.hi. The tensor core adds each MMA into its float32 accumulator
// rounding toward zero, so the K loop is cut into chunks of kChunk steps held in two alternating
// TMEM buffers, and the chunk sums are added in float64 (shared memory).
//
// Measured on B200 (tests/test_tc.py and the engine's parity tests): outputs within 2-6e-7 of
// sum |a b|, but every chunk sum keeps a bias toward zero of a few float32 ulps, which
// the residual Möbius network compounds (config-3 energies 3.5e-6 eV/atom off, against 4e-9 with
// the float32 SIMT kernel) while the 128 x 128 tiles of these layers run no faster than the SIMT
// kernel. The engine's dense layers therefore use dense.cu; this kernel is reached through
// rune_tc_selftest only.
//
// Roles in the 256-thread block:
//   thread 0        issues the MMAs (3 per K step) and the commits;
//   thread 32       streams B by bulk copies (8 KB units, tf32 hi and lo planes);
//   warps 2, 3      load the A slice of each K step (128 rows x 8 k), split it into hi / lo and
//                   store it as K-major 8 x 4 core matrices;
//   warps 4 .. 7    read each finished chunk from TMEM (warp 4 + q owns TMEM lanes 32 q ..) and
//                   add it into the float64 tile; at the end all threads apply the epilogue.
// A ring of kStages slots carries one K step each (A slice + B unit); every wait is bounded
// (error flag 32 on give-up, after which the block drains what it issued and stores nothing).

#include <cstring>

#include "engine.cuh"
#include "umma.cuh"

namespace rune {

namespace {

constexpr int kBM = 128, kBN = 128;
constexpr int kStages = 4;
constexpr int kChunk = 4;                           // K steps per accumulator chunk
constexpr uint32_t kUnitFloats = 2u * 8u * kBN;     // B unit: hi + lo planes, 8 KB
constexpr uint32_t kASliceFloats = 2u * 8u * kBM;   // A slice: hi + lo planes, 8 KB
constexpr int kAccLd = kBN + 1;                     // float64 tile row stride (odd: 2-way banks)
constexpr uint32_t kTmemCols = 2 * kBN;

struct GemmShared {
    unsigned long long full_a[kStages];  // A slice stored (64 loader arrivals)
    unsigned long long full_b[kStages];  // B unit landed (bulk-copy bytes)
    unsigned long long empty[kStages];   // MMAs of the slot complete
    unsigned long long chunk_full[2];
    unsigned long long chunk_empty[2];  // 128 reader arrivals
    unsigned long long done;
    uint32_t tmem;
    int fail;
    int issued_b;  // B units whose copy was issued
};

struct GemmSmem {
    size_t ring, shared, acc, total;  // byte offsets
    __host__ __device__ GemmSmem() {
        ring = 0;
        shared = ring + (size_t)kStages * (kUnitFloats + kASliceFloats) * 4;
        acc = (shared + sizeof(GemmShared) + 15) & ~size_t(15);
        total = acc + (size_t)kBM * kAccLd * 8;
    }
};

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
k_gemm_tc(int M, int N, int K, const float* __restrict__ A, int lda, const float* __restrict__ Bp,
          int nblocks_n, float* __restrict__ C, int ldc, GemmEpilogue ep,
          unsigned* __restrict__ err) {
    using namespace tc;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    GemmSmem L;
    float* ring = reinterpret_cast<float*>(smem_raw + L.ring);
    auto* sh = reinterpret_cast<GemmShared*>(smem_raw + L.shared);
    double* acc = reinterpret_cast<double*>(smem_raw + L.acc);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nb = blockIdx.x, m0 = blockIdx.y * kBM, n0 = nb * kBN;
    const int ns = (K + 7) / 8;
    const int nch = (ns + kChunk - 1) / kChunk;
    auto slot_b = [&](int st) { return ring + (size_t)st * (kUnitFloats + kASliceFloats); };
    auto slot_a = [&](int st) { return slot_b(st) + kUnitFloats; };

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&sh->full_a[s]), 64);
            mbar_init(smem_u32(&sh->full_b[s]), 1);
            mbar_init(smem_u32(&sh->empty[s]), 1);
        }
        sh->issued_b = 0;
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&sh->chunk_full[b]), 1);
            mbar_init(smem_u32(&sh->chunk_empty[b]), 128);
        }
        mbar_init(smem_u32(&sh->done), 1);
        sh->fail = 0;
        asm volatile("fence.mbarrier_init.release.cluster;");
    }
    if (warp == 0) tmem_alloc(&sh->tmem, kTmemCols);
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = sh->tmem;

    if (tid == 32) {
        // B producer: unit (s, nb) of the packed weights into slot s % kStages
        const uint32_t bytes = kUnitFloats * 4u;
        for (int s = 0; s < ns; ++s) {
            int st = s % kStages, use = s / kStages;
            if (use > 0 && !mbar_wait(smem_u32(&sh->empty[st]), (use - 1) & 1)) {
                atomicOr(err, 32u);
                sh->fail = 1;
                break;
            }
            if (*(volatile int*)&sh->fail) break;
            uint32_t bar = smem_u32(&sh->full_b[st]);
            mbar_expect_tx(bar, bytes);
            bulk_g2s(smem_u32(slot_b(st)), Bp + ((size_t)s * nblocks_n + nb) * kUnitFloats, bytes,
                     bar);
            *(volatile int*)&sh->issued_b = s + 1;
        }
    } else if (warp == 2 || warp == 3) {
        // A producers: 128 rows x 8 k per step, two rows per thread, split into hi / lo
        const int t = tid - 64;  // 0 .. 63
        for (int s = 0; s < ns; ++s) {
            int st = s % kStages, use = s / kStages;
            if (use > 0 && !mbar_wait(smem_u32(&sh->empty[st]), (use - 1) & 1)) {
                atomicOr(err, 32u);
                sh->fail = 1;
                break;
            }
            if (*(volatile int*)&sh->fail) break;
            float* hi = slot_a(st);
            float* lo = hi + 8 * kBM;
            for (int rr = 0; rr < 2; ++rr) {
                int r = 2 * t + rr, m = m0 + r;
                float x[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    int k = 8 * s + q;
                    x[q] = (m < M && k < K) ? __ldg(A + (size_t)m * lda + k) : 0.0f;
                }
                // element (r, k) at float (r / 8) * 64 + (k / 4) * 32 + (r % 8) * 4 + k % 4
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    float4 vh, vl;
                    tf32_split(x[4 * h], vh.x, vl.x);
                    tf32_split(x[4 * h + 1], vh.y, vl.y);
                    tf32_split(x[4 * h + 2], vh.z, vl.z);
                    tf32_split(x[4 * h + 3], vh.w, vl.w);
                    int off = (r >> 3) * 64 + h * 32 + (r & 7) * 4;
                    *reinterpret_cast<float4*>(hi + off) = vh;
                    *reinterpret_cast<float4*>(lo + off) = vl;
                }
            }
            fence_async_smem();
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];"
                         ::"r"(smem_u32(&sh->full_a[st])) : "memory");
        }
    } else if (tid == 0) {
        // MMA issuer
        const uint32_t idesc = idesc_tf32(kBM, kBN);
        int s = 0;
        for (; s < ns; ++s) {
            int st = s % kStages, use = s / kStages;
            int c = s / kChunk;
            bool first = (s % kChunk) == 0;
            if (first && c >= 2 &&
                !mbar_wait(smem_u32(&sh->chunk_empty[c & 1]), ((c >> 1) - 1) & 1)) {
                atomicOr(err, 32u);
                sh->fail = 1;
                break;
            }
            if (!mbar_wait(smem_u32(&sh->full_b[st]), use & 1) ||
                !mbar_wait(smem_u32(&sh->full_a[st]), use & 1) || *(volatile int*)&sh->fail) {
                atomicOr(err, 32u);
                sh->fail = 1;
                break;
            }
            fence_after_sync();
            uint32_t b_hi = smem_u32(slot_b(st)), b_lo = b_hi + kUnitFloats * 2u;
            uint32_t a_hi = smem_u32(slot_a(st)), a_lo = a_hi + kASliceFloats * 2u;
            uint64_t adh = smem_desc(a_hi, kALbo, kASbo), adl = smem_desc(a_lo, kALbo, kASbo);
            uint64_t bdh = smem_desc(b_hi, kALbo, kASbo), bdl = smem_desc(b_lo, kALbo, kASbo);
            uint32_t d = tmem + (uint32_t)((c & 1) * kBN);
            mma_tf32(d, adh, bdh, idesc, first ? 0u : 1u);
            mma_tf32(d, adh, bdl, idesc, 1u);
            mma_tf32(d, adl, bdh, idesc, 1u);
            mma_commit(smem_u32(&sh->empty[st]));
            if ((s + 1) % kChunk == 0 || s + 1 == ns) mma_commit(smem_u32(&sh->chunk_full[c & 1]));
        }
        mma_commit(smem_u32(&sh->done));
        if (!mbar_wait(smem_u32(&sh->done), 0)) {
            atomicOr(err, 32u);
            sh->fail = 1;
        }
        fence_before_sync();
    } else if (warp >= 4) {
        // readers: TMEM lane = tile row 32 q + lane; chunk sums into the float64 tile
        const int q = warp - 4, r = 32 * q + lane;
        double* row = acc + (size_t)r * kAccLd;
        for (int c = 0; c < nch; ++c) {
            if (!mbar_wait(smem_u32(&sh->chunk_full[c & 1]), (c >> 1) & 1) ||
                *(volatile int*)&sh->fail) {
                atomicOr(err, 32u);
                sh->fail = 1;
                break;
            }
            fence_after_sync();
#pragma unroll 1
            for (int g = 0; g < kBN / 32; ++g) {
                float v[32];
                tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)((c & 1) * kBN + 32 * g),
                          v);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    double a = c ? row[32 * g + j] : 0.0;
                    row[32 * g + j] = a + (double)v[j];
                }
            }
            fence_before_sync();
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];"
                         ::"r"(smem_u32(&sh->chunk_empty[c & 1])) : "memory");
        }
    }
    __syncthreads();
    bool ok = !sh->fail;
    if (!ok && tid == 0) {
        // drain (bounded): the last copy issued into each slot lands before the block exits
        int issued = sh->issued_b;
        for (int s = issued - kStages > 0 ? issued - kStages : 0; s < issued; ++s)
            mbar_wait(smem_u32(&sh->full_b[s % kStages]), (s / kStages) & 1);
    }
    if (ok) {
        // epilogue: consecutive threads take consecutive columns (coalesced rows of C)
        for (int o = tid; o < kBM * kBN; o += blockDim.x) {
            int r = o / kBN, cc = o - r * kBN;
            int m = m0 + r, n = n0 + cc;
            if (m < M && n < N) tc_store(ep, m, n, N, ldc, acc[(size_t)r * kAccLd + cc], C);
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) {
        fence_after_sync();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace

// Packs B [K][N] (row-major: W^T or W of a layer) into tensor-core units: unit (s, b) = K step
// s (k in [8 s, 8 s + 8)) x column block b (n in [128 b, 128 b + 128)) at float
// (s * Np / 128 + b) * 2048, hi plane then lo plane; in a plane, element (n, k) sits at
// ((n % 128) / 8) 64 + ((k % 8) / 4) 32 + (n % 8) 4 + k % 4 (K-major 8 x 4 core matrices).
__global__ void k_tc_pack(const float* __restrict__ B, int K, int N, int NB,
                          float* __restrict__ out) {
    long long total = (long long)((K + 7) / 8 * 8) * NB * kBN;
    for (long long o = blockIdx.x * (long long)blockDim.x + threadIdx.x; o < total;
         o += (long long)gridDim.x * blockDim.x) {
        int n = (int)(o % (NB * kBN)), k = (int)(o / (NB * kBN));
        float x = (k < K && n < N) ? B[(size_t)k * N + n] : 0.0f;
        float hi, lo;
        tc::tf32_split(x, hi, lo);
        int s = k / 8, b = n / kBN, nn = n % kBN, kk = k % 8;
        size_t unit = ((size_t)s * NB + b) * kUnitFloats;
        size_t at = (size_t)(nn / 8) * 64 + (kk / 4) * 32 + (nn % 8) * 4 + kk % 4;
        out[unit + at] = hi;
        out[unit + 8 * kBN + at] = lo;
    }
}

size_t gemm_tc_smem() { return GemmSmem().total; }

size_t tc_packed_floats(int K, int N) {
    return (size_t)((K + 7) / 8) * ((N + kBN - 1) / kBN) * kUnitFloats;
}

void tc_pack(const float* B, int K, int N, float* out, cudaStream_t stream) {
    int NB = (N + kBN - 1) / kBN;
    long long total = (long long)((K + 7) / 8 * 8) * NB * kBN;
    int blocks = (int)std::min<long long>((total + 255) / 256, 4096);
    k_tc_pack<<<blocks, 256, 0, stream>>>(B, K, N, NB, out);
    RUNE_CUDA_TRY(cudaGetLastError());
}

void gemm_tc(int M, int N, int K, const float* A, int lda, const TcMatrix& B, float* C, int ldc,
             const GemmEpilogue& ep, unsigned* err, cudaStream_t stream) {
    if (M == 0 || N == 0) return;
    if (B.K != K || B.N != N) throw Error(RUNE_ERR_INVALID, "tensor-core operand shape mismatch");
    size_t bytes = gemm_tc_smem();
    RUNE_CUDA_TRY(cudaFuncSetAttribute((const void*)k_gemm_tc,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    int nblocks_n = (N + kBN - 1) / kBN;
    dim3 grid(nblocks_n, (M + kBM - 1) / kBM);
    RUNE_KERNEL("k_gemm_tc", stream,
                k_gemm_tc<<<grid, 256, bytes, stream>>>(M, N, K, A, lda, B.w, nblocks_n, C, ldc,
                                                         ep, err));
    RUNE_LAUNCH_CHECK();
}

void tc_selftest(int M, int N, int K, const float* a_host, const float* b_host, float* c_host,
                 int device) {
    if (M < 1 || N < 1 || K < 1 || M > 65536 || N > 4096 || K > 4096)
        throw Error(RUNE_ERR_INVALID,
                    "tc self-test sizes: 1 <= M <= 65536, 1 <= N <= 4096, 1 <= K <= 4096");
    RUNE_CUDA_TRY(cudaSetDevice(device));
    size_t fa = (size_t)M * K, fb = (size_t)K * N, fc = (size_t)M * N, fp = tc_packed_floats(K, N);
    float* buf = nullptr;
    RUNE_CUDA_TRY(cudaMalloc(&buf, sizeof(float) * (fa + fb + fc + fp + 256)));
    struct Free {
        float* p;
        ~Free() { cudaFree(p); }
    } guard{buf};
    float* da = buf;
    float* db = da + fa;
    float* dc = db + fb;
    float* dp = dc + fc + (64 - (fa + fb + fc) % 64) % 64;  // 256-byte aligned
    unsigned* derr = reinterpret_cast<unsigned*>(dp + fp + 64);
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
