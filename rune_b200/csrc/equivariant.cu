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
#include "umma.cuh"

namespace rune {

namespace {

constexpr int kWarps = 2;
constexpr int CH = 8;  // edges per chunk

__device__ __forceinline__ int order_of(int m) {  // component m of the packed basis -> l
    int l = 1;
    while ((l + 1) * (l + 1) - 1 <= m) ++l;
    return l;
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

// ----------------------------------------------------------------------------- edge tiles
// The edge kernels run one block per centre atom and process its row in tiles of 32 edges.
// Per tile, the edge-MLP inputs, hidden units and gates live in shared memory as k-major
// tiles ([feature][edge], row stride kLd), and every matrix product is a block-wide GEMM: warp w
// computes edges 4w .. 4w+3, lane l the output columns l + 32 t, with the weights streamed
// through shared memory 16 rows at a time (all warps share a slice; each weight is read once
// from L2 per tile of 32 edges).
constexpr int kTe = 32;         // edges per tile
constexpr int kLd = 36;         // row stride of the k-major tiles
constexpr int kTThreads = 256;  // 8 warps
// Weight rows per staged slice: 8 in both kernels, whose shared memory then fits two blocks per
// SM.
constexpr int kKsForward = 8;
constexpr int kKsBackward = 8;
__host__ __device__ constexpr int slice_rows(bool bwd) { return bwd ? kKsBackward : kKsForward; }
constexpr int kMaxK = 64;       // message basis size bound of the per-edge basis arrays

// Weight slices arrive by TMA bulk copies (cp.async.bulk, one thread issues, an mbarrier per
// buffer counts the bytes) into two shared-memory buffers: slice s + 1 is in flight while slice s
// is consumed. Waits are bounded: after L.wait_polls polls the block sets error flag 32 in
// `err`, lets the copies it issued land (a wait with the full bound kEqWaitPolls), skips the rest
// of its work and returns normally (the host reports the failure).

struct SliceRing {
    float* buf[2];
    unsigned mbar[2];   // shared-memory addresses of the two mbarriers
    unsigned phase[2];  // completed uses of each buffer (parity of the next wait)
    unsigned* err;
    unsigned polls;     // bound of ring_wait
    bool failed;
};

__device__ __forceinline__ unsigned smem_addr(const void* p) {
    return (unsigned)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void ring_init(SliceRing& R, float* buf0, float* buf1,
                                          unsigned long long* bars, unsigned* err,
                                          unsigned polls) {
    R.buf[0] = buf0;
    R.buf[1] = buf1;
    R.mbar[0] = smem_addr(bars);
    R.mbar[1] = smem_addr(bars + 1);
    R.phase[0] = R.phase[1] = 0;
    R.err = err;
    R.polls = polls;
    R.failed = false;
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(R.mbar[0]));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(R.mbar[1]));
        asm volatile("fence.mbarrier_init.release.cluster;");
    }
    __syncthreads();
}

// Thread 0: bulk-copy `bytes` (a multiple of 16, 16-byte aligned) from global src into buffer b.
__device__ __forceinline__ void ring_issue(const SliceRing& R, int b, const float* src,
                                           unsigned bytes) {
    if (threadIdx.x != 0) return;
    // earlier generic-proxy reads of the buffer happen before the async-proxy write
    asm volatile("fence.proxy.async.shared::cta;");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(R.mbar[b]),
                 "r"(bytes));
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_addr(R.buf[b])), "l"(src), "r"(bytes), "r"(R.mbar[b])
        : "memory");
}

// All threads: wait for the pending copy into buffer b (at most `polls` polls).
__device__ __forceinline__ bool ring_wait_polls(SliceRing& R, int b, unsigned polls) {
    unsigned parity = R.phase[b] & 1u;
    for (unsigned it = 0; it < polls; ++it) {
        unsigned ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(R.mbar[b]), "r"(parity)
            : "memory");
        if (ok) {
            ++R.phase[b];
            return true;
        }
    }
    if (threadIdx.x == 0) atomicOr(R.err, 32u);
    return false;
}

__device__ __forceinline__ bool ring_wait(SliceRing& R, int b) {
    return ring_wait_polls(R, b, R.polls);
}

// Thread tile of the block GEMM: warp w owns output columns [w N/8, (w+1) N/8) for all 32 edges;
// lane (rg = lane % 8, cg = lane / 8) owns edges 4 rg .. 4 rg + 3 and the NT = N/32 contiguous
// columns starting at w N/8 + cg NT. Per k a warp reads 32 A values (one 128-byte wavefront) and
// N/8 B values, so every weight is read from shared memory once per k.
struct TileCoords {
    int e0;  // first edge (row) of the thread tile
    int c0;  // first output column of the thread tile
    __device__ explicit TileCoords(int N) {
        int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        e0 = 4 * (lane & 7);
        c0 = warp * (N / 8) + (lane >> 3) * (N / 32);
    }
};

// Epilogue store of a thread tile into a k-major tile T [col][kLd]: the thread's four edges of
// one column are contiguous, so each column is one 16-byte store (no bank conflicts). Columns
// from `ncap` on (padding of a wider product that nothing reads) are not stored.
template <int NT>
__device__ __forceinline__ void store_tile(float* T, int te0, int tc0, const float (&v)[4][NT],
                                           int ncap) {
#pragma unroll
    for (int t = 0; t < NT; ++t)
        if (tc0 + t < ncap)
            *reinterpret_cast<float4*>(T + (tc0 + t) * kLd + te0) =
                make_float4(v[0][t], v[1][t], v[2][t], v[3][t]);
}

// acc[r][t] = init + sum_k A[k][e0 + r] B[k][c0 + t] for k < K (a multiple of KS). B is [K][32 NT]
// row-major in global memory. init(acc, e0, c0) adds the epilogue's per-output terms to the zeroed
// accumulators after the block barrier that opens the product, so their global loads are in
// flight while the first weight slices arrive. Every thread of the block calls it (block barriers
// inside); on return no copy is in flight and A may be overwritten.
template <int NT, int KS, typename Init>
__device__ __forceinline__ void tile_gemm(int K, const float* A, const float* __restrict__ B,
                                          SliceRing& R, float (&acc)[4][NT], Init&& init) {
    constexpr int N = 32 * NT;
    constexpr unsigned kBytes = KS * N * sizeof(float);
    TileCoords tc(N);
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[r][t] = 0.0f;
    const int ns = K / KS;
    __syncthreads();  // both buffers free
    ring_issue(R, 0, B, kBytes);
    if (ns > 1) ring_issue(R, 1, B + (size_t)KS * N, kBytes);
    init(acc, tc.e0, tc.c0);
    for (int s = 0; s < ns; ++s) {
        int b = s & 1;
        bool ok = ring_wait(R, b);
        // one block barrier per slice: every thread's wait result, and every thread is done with
        // slice s - 1, whose buffer then takes slice s + 1
        if (__syncthreads_or(!ok)) {  // uniform across the block
            R.failed = true;
            // the copies still in flight land before the block moves on: this slice's, when
            // this thread's wait gave up, and at s = 0 slice 1 (later slices are issued after
            // this barrier)
            if (!ok) ring_wait_polls(R, b, kEqWaitPolls);
            if (s == 0 && ns > 1) ring_wait_polls(R, b ^ 1, kEqWaitPolls);
            __syncthreads();
            break;
        }
        if (s >= 1 && s + 1 < ns) ring_issue(R, b ^ 1, B + (size_t)(s + 1) * KS * N, kBytes);
        const float* Bs = R.buf[b] + tc.c0;
        const float* As = A + s * KS * kLd + tc.e0;
#pragma unroll 4
        for (int kk = 0; kk < KS; ++kk) {
            float4 a = *reinterpret_cast<const float4*>(As + kk * kLd);
            float bv[NT];
            if constexpr (NT % 2 == 0) {
#pragma unroll
                for (int t = 0; t < NT; t += 2) {
                    float2 v = *reinterpret_cast<const float2*>(Bs + kk * N + t);
                    bv[t] = v.x;
                    bv[t + 1] = v.y;
                }
            } else {
#pragma unroll
                for (int t = 0; t < NT; ++t) bv[t] = Bs[kk * N + t];
            }
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                acc[0][t] += a.x * bv[t];
                acc[1][t] += a.y * bv[t];
                acc[2][t] += a.z * bv[t];
                acc[3][t] += a.w * bv[t];
            }
        }
    }
    __syncthreads();
}

// tile_gemm with NT = N / 32 chosen at run time; init(acc, e0, c0) as in tile_gemm, epi(acc, e0,
// c0) receives the accumulators and the thread tile's first edge and column.
template <int KS, typename Init, typename Epi>
__device__ __forceinline__ void tile_gemm_n(int N, int K, const float* A,
                                            const float* __restrict__ B, SliceRing& R,
                                            Init&& init, Epi&& epi) {
    TileCoords tc(N);
    auto run = [&](auto& acc) {
        constexpr int NT = sizeof(acc[0]) / sizeof(float);
        tile_gemm<NT, KS>(K, A, B, R, acc, init);
        epi(acc, tc.e0, tc.c0);
    };
    switch (N / 32) {
        case 1: { float acc[4][1]; run(acc); break; }
        case 2: { float acc[4][2]; run(acc); break; }
        case 3: { float acc[4][3]; run(acc); break; }
        case 4: { float acc[4][4]; run(acc); break; }
        case 6: { float acc[4][6]; run(acc); break; }
        case 8: { float acc[4][8]; run(acc); break; }
        default: { float acc[4][10]; run(acc); break; }
    }
}

template <int KS, typename Epi>
__device__ __forceinline__ void tile_gemm_n(int N, int K, const float* A,
                                            const float* __restrict__ B, SliceRing& R, Epi&& epi) {
    tile_gemm_n<KS>(N, K, A, B, R, [](auto&, int, int) {}, epi);
}

// ----------------------------------------------------------------- tensor-core edge GEMMs
// The four edge products of a tile run on the tensor cores (tcgen05.mma kind::i8) with
// exact-integer digits, the scheme of dense_tc.cu: every edge (a column of the input tile) and
// every output feature (a column of W) gets a power-of-two scale 2^e above its largest |x|,
// each value splits exactly into four signed 7-bit digits, and the ten digit products with
// shift t = p + q <= 3 accumulate exactly in int32 in TMEM (D_t, t = 0 .. 3); the result is
// 2^(e_f + e_e - 12) sum_t 2^(-7 t) D_t, the D_t combined exactly in int32 and rounded once to
// float32 before an exact power-of-two scale. No accumulation rounding, so no bias; the
// truncation is 2^-28 of an edge's largest input.
//
// Shapes: M = 128 output features per MMA (W^T as the A operand, K-major units packed once),
// N = the tile's 32 edges (B operand: the tile's digits, made once per product and reused by
// every feature chunk), K = 32 per MMA step. TMEM holds the four D_t (4 x 32 columns).
// Thread 0 streams the weight units through two 16 KB shared-memory slots by bulk copies (no
// multicast) and issues the MMAs; warps 0 .. 3 read TMEM (warp w: features 32 w .. of the
// chunk) and write the raw products into the output tile [feature][edge], whose existing
// epilogues then run unchanged. Every wait is bounded (error flag 32, the call returns false).
constexpr int kTcChunk = 128;                      // output features per MMA
constexpr int kTcK = 32;                           // k per MMA step
constexpr uint32_t kTcWPlane = kTcChunk * kTcK;    // 4 KB
constexpr uint32_t kTcWUnit = 4 * kTcWPlane;       // 16 KB
constexpr uint32_t kTcXPlane = kTe * kTcK;         // 1 KB: 32 edges x 32 k
constexpr uint32_t kTcXUnit = 4 * kTcXPlane;       // 4 KB
constexpr int kTcMaxSteps = 10;                    // K up to 320
constexpr uint32_t kTcCols = 128;                  // TMEM columns: 4 accumulators x 32 edges
// shared-memory floats of the tensor-core region: one weight slot, exponents (32 + 8 x 32
// partials), mbarriers and the TMEM address. The tile's digits take the place of the product's
// own float32 input tile (dead after the split): K step s occupies bytes [4096 s, 4096 s +
// 4096) of it, below the float32 rows of every later step (32 rows x 144 bytes per step).
constexpr uint32_t kTcHalf = kTcWUnit / 2;        // digit planes 0-1 or 2-3 of a unit
constexpr int kTcFloats = (int)(2 * kTcHalf) / 4 + 288 + 12;

struct TcCtx {
    unsigned char* wbuf[2];
    int* eexp;
    uint32_t full[2], empty[2], done;  // mbarrier addresses
    uint32_t tmem;
    unsigned fills[2], uses[2], dones;  // completed phases (thread 0's copies drive the ring)
    unsigned* err;
    unsigned polls;  // bound of a wait before the block gives up
};

__device__ __forceinline__ uint32_t tc_plane_offset(int r, int k) {
    return (uint32_t)((r >> 3) * 256 + (k >> 4) * 128 + (r & 7) * 16 + (k & 15));
}

// Region layout and barrier initialisation (thread 0), TMEM allocation (warp 0); all threads
// call it, with a block barrier at the end.
__device__ void tc_init(TcCtx& C, float* region, unsigned* err, unsigned polls) {
    using namespace tc;
    unsigned char* base = reinterpret_cast<unsigned char*>(region);
    C.wbuf[0] = base;
    C.wbuf[1] = base + kTcHalf;
    C.eexp = reinterpret_cast<int*>(base + 2 * kTcHalf);
    unsigned long long* bars = reinterpret_cast<unsigned long long*>(C.eexp + 288);
    C.full[0] = smem_u32(bars);
    C.full[1] = smem_u32(bars + 1);
    C.empty[0] = smem_u32(bars + 2);
    C.empty[1] = smem_u32(bars + 3);
    C.done = smem_u32(bars + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 5);
    C.fills[0] = C.fills[1] = C.uses[0] = C.uses[1] = C.dones = 0;
    C.err = err;
    C.polls = polls;
    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; ++b) {
            mbar_init(C.full[b], 1);
            mbar_init(C.empty[b], 1);
        }
        mbar_init(C.done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;");
    }
    if (threadIdx.x < 32) tmem_alloc(tmem_slot, kTcCols);
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    C.tmem = *tmem_slot;
}

__device__ void tc_release(TcCtx& C) {
    using namespace tc;
    fence_before_sync();
    __syncthreads();
    if (threadIdx.x < 32) {
        fence_after_sync();
        tmem_dealloc(C.tmem, kTcCols);
    }
}

// out[f * kLd + e] = sum_k W[k][f] A[k * kLd + e] for f < n_out and the 32 edges of the tile
// (A: [W.K][kLd], rows beyond W.K read as zero). A is consumed: its storage receives the
// tile's digits. Every thread of the block calls it (block barriers inside); false (uniform)
// when a bounded wait gave up.
__device__ bool tc_tile_gemm(TcCtx& C, const EqTcW& W, int n_out, float* A, float* out) {
    using namespace tc;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int* partial = C.eexp + 32;
    __syncthreads();
    {  // largest |x| of every edge: eight threads per edge, then a combination per edge
        int e = tid & 31, part = tid >> 5;
        float amax = 0.0f;
        for (int k = part; k < W.K; k += blockDim.x >> 5) amax = fmaxf(amax, fabsf(A[k * kLd + e]));
        partial[part * 32 + e] = __float_as_int(amax);
    }
    __syncthreads();
    if (tid < 32) {
        float amax = 0.0f;
        for (int p = 0; p < (int)(blockDim.x >> 5); ++p)
            amax = fmaxf(amax, __int_as_float(partial[p * 32 + tid]));
        C.eexp[tid] = digit_exponent(amax);
    }
    __syncthreads();
    // the tile's digit planes, written over the input tile one K step at a time: every thread
    // reads its four values of step s (one edge, four consecutive k; 256 threads = 32 edges x 32
    // k), the block synchronises, then the digits of step s go to bytes [4096 s, 4096 s + 4096),
    // which hold only float32 rows of steps <= s (already read)
    unsigned char* digits = reinterpret_cast<unsigned char*>(const_cast<float*>(A));
    for (int s = 0; s < W.steps; ++s) {
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        int e = tid & 31, kk = 4 * (tid >> 5);
        if (tid < 256) {
            int ee = C.eexp[e];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                int k = s * kTcK + kk + j;
                float x = k < W.K ? A[k * kLd + e] : 0.0f;
                int d[4];
                split_digits_fixed(x, ee, d);
#pragma unroll
                for (int p = 0; p < 4; ++p) w[p] |= (uint32_t)(d[p] & 0xff) << (8 * j);
            }
        }
        __syncthreads();
        if (tid < 256) {
            unsigned char* dst = digits + s * kTcXUnit + tc_plane_offset(e, kk);
#pragma unroll
            for (int p = 0; p < 4; ++p) *reinterpret_cast<uint32_t*>(dst + p * kTcXPlane) = w[p];
        }
    }
    fence_async_smem();
    __syncthreads();
    const uint32_t idesc = idesc_i8(kTcChunk, kTe);
    bool ok = true;
    for (int c = 0; c < W.chunks && c * kTcChunk < n_out; ++c) {
        if (tid == 0) {
            // weight half-units of this chunk (digit planes 0-1, then 2-3, of every K step)
            // through the two slots: the MMAs of one half while the next half is in flight
            const int n_half = 2 * W.steps;
            auto fill = [&](int u) -> bool {
                int b = (int)(C.fills[0] + C.fills[1]) & 1;
                // the slot's previous half must be consumed: wait for the MMAs that read it
                // (their commit completed phase fills - 1 of the slot's empty barrier)
                if (C.fills[b] > 0 && !mbar_wait(C.empty[b], (C.fills[b] - 1) & 1, C.polls))
                    return false;
                mbar_expect_tx(C.full[b], kTcHalf);
                bulk_g2s(smem_u32(C.wbuf[b]),
                         W.q + ((size_t)c * W.steps + (u >> 1)) * kTcWUnit + (u & 1) * kTcHalf,
                         kTcHalf, C.full[b]);
                ++C.fills[b];
                return true;
            };
            bool go = fill(0);
            for (int u = 0; u < n_half && go; ++u) {
                if (u + 1 < n_half) go = fill(u + 1);
                int b = (int)(C.uses[0] + C.uses[1]) & 1;
                if (!mbar_wait(C.full[b], C.uses[b] & 1, C.polls)) go = false;
                if (!go) break;
                fence_after_sync();
                const int s = u >> 1, h = u & 1;
                uint32_t w0 = smem_u32(C.wbuf[b]), x0 = smem_u32(digits + s * kTcXUnit);
                // D_t += W_p X_(t - p) for the two weight planes p = 2 h, 2 h + 1 in the slot
#pragma unroll
                for (int t = 0; t < 4; ++t) {
#pragma unroll
                    for (int pp = 0; pp < 2; ++pp) {
                        int p = 2 * h + pp;
                        if (p > t) continue;
                        uint64_t ad = smem_desc(w0 + pp * kTcWPlane, kALbo, kASbo);
                        uint64_t bd = smem_desc(x0 + (t - p) * kTcXPlane, kALbo, kASbo);
                        mma_i8(C.tmem + (uint32_t)(t * kTe), ad, bd, idesc,
                               (s > 0 || p > 0) ? 1u : 0u);
                    }
                }
                mma_commit(C.empty[b]);
                ++C.uses[b];
            }
            if (!go) {
                atomicOr(C.err, 32u);
                // let every copy issued into a slot land before anything reuses the block
                for (int bb = 0; bb < 2; ++bb)
                    while (C.uses[bb] < C.fills[bb]) {
                        mbar_wait(C.full[bb], C.uses[bb] & 1);
                        ++C.uses[bb];
                    }
            }
            mma_commit(C.done);
            // thread 0 alone waits for the chunk's MMAs (the other threads wait at the block
            // barrier instead of polling the mbarrier)
            bool fine = mbar_wait(C.done, C.dones & 1, C.polls);
            if (!fine) {
                // the MMAs in flight finish before TMEM is read again or freed
                atomicOr(C.err, 32u);
                mbar_wait(C.done, C.dones & 1);
            }
            partial[0] = (go && fine) ? 1 : 0;
            fence_before_sync();
        }
        ++C.dones;
        __syncthreads();
        if (partial[0] == 0) {  // the same shared value for every thread: uniform
            ok = false;
            break;
        }
        fence_after_sync();
        if (warp < 4) {
            // warp w: TMEM lanes (features) 32 w .. 32 w + 31; 16 edges at a time. The four
            // accumulators combine exactly in int32 (|D_0| <= 320 * 64 * 64, so 128 D_0 + D_1 and
            // 128 D_2 + D_3 stay below 2^31); value = (hi + lo 2^-14) 2^(e_f + e_e - 19), two
            // conversions and one rounding of the sum before the exact power-of-two scale
            int f = c * kTcChunk + 32 * warp + lane;
            int ef = f < n_out ? __ldg(W.fexp + f) - 19 : 0;
            float* row = out + f * kLd;
#pragma unroll 1
            for (int h = 0; h < 2; ++h) {
                float v[4][16];
#pragma unroll
                for (int t = 0; t < 4; ++t)
                    tmem_ld16(C.tmem + ((uint32_t)(32 * warp) << 16) +
                                  (uint32_t)(t * kTe + 16 * h), v[t]);
                if (f < n_out) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4) {
                        float r[4];
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            int hi = __float_as_int(v[0][j + q]) * 128 + __float_as_int(v[1][j + q]);
                            int lo = __float_as_int(v[2][j + q]) * 128 + __float_as_int(v[3][j + q]);
                            float val = fmaf((float)lo, 0x1p-14f, (float)hi);
                            r[q] = scale_pow2(val, ef + C.eexp[16 * h + j + q]);
                        }
                        *reinterpret_cast<float4*>(row + 16 * h + j) =
                            make_float4(r[0], r[1], r[2], r[3]);
                    }
                }
            }
        }
        fence_before_sync();
        __syncthreads();
    }
    return ok;
}

// The SIMT epilogue of a tile product read back from the tensor-core output tile T
// ([rows][kLd], rows >= `written` read as zero): the same thread tile and the same epilogue.
template <typename Epi>
__device__ __forceinline__ void tile_epilogue_from(int N, const float* T, int written,
                                                   Epi&& epi) {
    TileCoords tcd(N);
    auto run = [&](auto& acc) {
        constexpr int NT = sizeof(acc[0]) / sizeof(float);
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                int c = tcd.c0 + t;
                acc[r][t] = c < written ? T[c * kLd + tcd.e0 + r] : 0.0f;
            }
        epi(acc, tcd.e0, tcd.c0);
    };
    switch (N / 32) {
        case 1: { float acc[4][1]; run(acc); break; }
        case 2: { float acc[4][2]; run(acc); break; }
        case 3: { float acc[4][3]; run(acc); break; }
        case 4: { float acc[4][4]; run(acc); break; }
        case 6: { float acc[4][6]; run(acc); break; }
        case 8: { float acc[4][8]; run(acc); break; }
        default: { float acc[4][10]; run(acc); break; }
    }
}

// Per-edge rows in shared memory are read with one edge per lane: their strides are odd
// (geometry kGeo, harmonics and their adjoints ys, cutoff partials ps) so that the 32
// lanes of a warp hit 32 different banks.
constexpr int kGeo = 9;

struct EqTileSmem {
    int bs, bar, t1, t3, geo, idx, Y, dYn, part, Di, ddp, dmsg, accH, accM, accDC, total;
    int ys, ps;
    int r1;  // rows of T1: the X input and the gate rows (wider products store no padding)
    __host__ __device__ EqTileSmem(const EqLayerArgs& L, bool bwd) {
        auto up4 = [](int x) { return (x + 3) & ~3; };
        int DC = L.Ce * L.Cl;
        int nmax = L.XN > L.MN ? L.XN : L.MN;
        nmax = nmax > L.GN ? nmax : L.GN;
        r1 = L.XK > L.GK ? L.XK : L.GK;
        int r3 = L.MK > L.MN ? L.MK : L.MN;
        ys = L.Cl | 1;
        ps = (L.Ce + L.G) | 1;
        bs = 0;  // two slice buffers (SIMT products) or the tensor-core region
        bar = bs + (L.tc ? kTcFloats : 2 * slice_rows(bwd) * nmax);  // two mbarriers
        t1 = bar + 4;
        t3 = t1 + r1 * kLd;
        geo = t3 + r3 * kLd;
        idx = up4(geo + kTe * kGeo);
        Y = idx + kTe * 2;
        dYn = up4(Y + kTe * ys);
        part = dYn + (bwd ? kTe * ys : 0);
        Di = up4(part + (bwd ? kTe * ps : 0));
        ddp = Di + DC;
        dmsg = ddp + (bwd ? DC : 0);
        accH = dmsg + (bwd ? L.H : 0);
        accM = accH + (bwd ? 0 : L.H);
        accDC = accM + (bwd ? L.M : 0);
        total = up4(accDC + DC);
    }
};

// Geometry of the tile's edges (thread e < 32): unit vector, cutoff and its derivative, 1/r,
// the message basis into rows 0 .. K of T1 (column e) and the scaled harmonics. Columns
// e >= ne are zero with j = i. (The backward recomputes basis derivatives and harmonic
// gradients where it needs them, once per edge.)
__device__ __forceinline__ void tile_geometry(const EqLayerArgs& L, const EqTileSmem& S,
                                              float* sm, const EdgeList& rad, const int* types,
                                              int i, int ti, int e0, int ne) {
    int e = threadIdx.x;
    if (e >= kTe) return;
    float* T1 = sm + S.t1;
    float* g = sm + S.geo + e * kGeo;
    int* idx = reinterpret_cast<int*>(sm + S.idx) + 2 * e;
    float* y = sm + S.Y + e * S.ys;
    if (e >= ne) {
        for (int k = 0; k < L.K; ++k) T1[k * kLd + e] = 0.0f;
        for (int q = 0; q < 8; ++q) g[q] = 0.0f;
        idx[0] = i;
        idx[1] = 0;
        for (int m = 0; m < L.Cl; ++m) y[m] = 0.0f;
        return;
    }
    float4 ed = rad.e[e0 + e];
    int j = edge_j(ed);
    float r = (float)sqrt((double)ed.x * ed.x + (double)ed.y * ed.y + (double)ed.z * ed.z);
    float inv = 1.0f / fmaxf(r, 1.0e-12f);
    float b[kMaxK], cut, dcut;
    cheb_masked(r, L.rc, L.K, b, nullptr, cut, dcut);
    for (int k = 0; k < L.K; ++k) T1[k * kLd + e] = b[k];
    g[0] = ed.x * inv; g[1] = ed.y * inv; g[2] = ed.z * inv;
    g[3] = cut; g[4] = dcut; g[5] = inv; g[6] = r;
    idx[0] = j;
    idx[1] = ti * L.T + types[j];
    angular_components<false>(g[0], g[1], g[2], L.Le, L.zc,
                              [&](int c, int, float Y, float, float, float) {
                                  y[c] = Y * __ldg(L.scale + c);
                              });
}

// The 24 harmonic components of orders 1..4 (a row of D, mixed: 16-byte aligned, the arena
// aligns every array to 256 bytes and rows are multiples of 24 floats) as six 16-byte loads.
__device__ __forceinline__ void load_row24(const float* __restrict__ p, float (&v)[24]) {
#pragma unroll
    for (int q = 0; q < 6; ++q) {
        float4 t = __ldg(reinterpret_cast<const float4*>(p) + q);
        v[4 * q] = t.x;
        v[4 * q + 1] = t.y;
        v[4 * q + 2] = t.z;
        v[4 * q + 3] = t.w;
    }
}

// Order (0-based) of harmonic component m < 24 (compile-time m after unrolling).
__device__ __forceinline__ constexpr int order24(int m) {
    return m < 3 ? 0 : m < 8 ? 1 : m < 15 ? 2 : 3;
}

// Probes into T1: pc[l][c] (rows K + (l-1) Ce + c) and pn[l][c] (rows K + LC + ...), and zero
// rows up to XK. With orders up to 4 the neighbour's row is read with 16-byte loads (same sums,
// same order).
__device__ __forceinline__ void tile_probes(const EqLayerArgs& L, const EqTileSmem& S, float* sm,
                                            const float* __restrict__ D) {
    const int LC = L.Le * L.Ce, DC = L.Ce * L.Cl;
    float* T1 = sm + S.t1;
    const float* Di = sm + S.Di;
    const int* idx = reinterpret_cast<const int*>(sm + S.idx);
    if (L.Cl == 24) {
        for (int o = threadIdx.x; o < kTe * L.Ce; o += blockDim.x) {
            int e = o % kTe, c = o / kTe;
            float dj[24];
            load_row24(D + (size_t)idx[2 * e] * DC + (size_t)c * 24, dj);
            const float* Dic = Di + c * 24;
            const float* y = sm + S.Y + e * S.ys;
            float pc[4] = {0.0f, 0.0f, 0.0f, 0.0f}, pn[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int m = 0; m < 24; ++m) {
                float ym = y[m];
                pc[order24(m)] += Dic[m] * ym;
                pn[order24(m)] += dj[m] * ym;
            }
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                T1[(L.K + l * L.Ce + c) * kLd + e] = pc[l];
                T1[(L.K + LC + l * L.Ce + c) * kLd + e] = (l & 1) ? pn[l] : -pn[l];
            }
        }
    } else
    for (int o = threadIdx.x; o < kTe * L.Ce; o += blockDim.x) {
        int e = o % kTe, c = o / kTe;
        const float* Dj = D + (size_t)idx[2 * e] * DC + (size_t)c * L.Cl;
        const float* Dic = Di + c * L.Cl;
        const float* y = sm + S.Y + e * S.ys;
        for (int l = 1; l <= L.Le; ++l) {
            float pc = 0.0f, pn = 0.0f;
            for (int m = l * l - 1; m < (l + 1) * (l + 1) - 1; ++m) {
                pc += Dic[m] * y[m];
                pn += __ldg(Dj + m) * y[m];
            }
            T1[(L.K + (l - 1) * L.Ce + c) * kLd + e] = pc;
            T1[(L.K + LC + (l - 1) * L.Ce + c) * kLd + e] = (l & 1) ? -pn : pn;
        }
    }
    for (int o = threadIdx.x; o < kTe * (L.XK - L.K - 2 * LC); o += blockDim.x) {
        int e = o % kTe, k = L.K + 2 * LC + o / kTe;
        T1[k * kLd + e] = 0.0f;
    }
}

// Forward of one EQ block over the edges of centre atom i (one block per atom): gates stored per
// edge (gate * cut and transport * cut, for the backward pull), the scalar message and the
// direction update D'_i = D_i + sum_e cut (a mixed_j + b Y).
template <bool TC>
__global__ void __launch_bounds__(kTThreads)
k_eq_forward_edges(int n_atoms, EqLayerArgs L, EdgeList rad, const int* __restrict__ types,
                   const float* __restrict__ abv, const float* __restrict__ D,
                   const float* __restrict__ mixed, float* __restrict__ msg_out,
                   float* __restrict__ dn_out, float* __restrict__ gva_out,
                   unsigned* __restrict__ err) {
    extern __shared__ float4 smem4[];
    float* sm = reinterpret_cast<float*>(smem4);
    EqTileSmem S(L, false);
    const int i = blockIdx.x;
    if (i >= n_atoms) return;  // uniform per block
    const int tid = threadIdx.x;
    const int DC = L.Ce * L.Cl, LC = L.Le * L.Ce, ldabv = 2 * L.M + L.H, gw = L.H / L.G;
    const int GVA = L.G + LC, GD = L.G + 2 * LC;
    float* T1 = sm + S.t1;
    float* T3 = sm + S.t3;
    const float* geo = sm + S.geo;
    const int* idx = reinterpret_cast<const int*>(sm + S.idx);
    float* Di = sm + S.Di;
    float* msg = sm + S.accH;
    float* inc = sm + S.accDC;
    SliceRing R;
    TcCtx C;
    if constexpr (TC) {
        tc_init(C, sm + S.bs, err, L.wait_polls);
    } else {
        int nmax = max(max(L.XN, L.MN), L.GN);
        ring_init(R, sm + S.bs, sm + S.bs + kKsForward * nmax,
                  reinterpret_cast<unsigned long long*>(sm + S.bar), err, L.wait_polls);
    }
    bool failed = false;
    int ti = types[i];
    for (int o = tid; o < DC; o += blockDim.x) {
        Di[o] = D[(size_t)i * DC + o];
        inc[o] = 0.0f;
    }
    for (int c = tid; c < L.H; c += blockDim.x) msg[c] = 0.0f;
    const float* Ai = abv + (size_t)i * ldabv;
    int row = rad.row_ptr[i], cnt = rad.cnt[i];
    for (int base = 0; base < cnt; base += kTe) {
        int ne = min(kTe, cnt - base);
        int e0 = row + base;
        __syncthreads();
        tile_geometry(L, S, sm, rad, types, i, ti, e0, ne);
        __syncthreads();
        tile_probes(L, S, sm, D);
        // pre = W_x x + pb[pair] + A_i + B_j ; z = act(pre)  -> T3 [m][e]
        // pre-activation terms of the edge MLP: pair bias, centre and neighbour node terms
        auto pre_z = [&](auto& acc, int te0, int tc0) {
            constexpr int NT = sizeof(acc[0]) / sizeof(float);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                int e = te0 + r;
                int j = idx[2 * e], pr = idx[2 * e + 1];
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    int m = tc0 + t;
                    if (m < L.M)
                        acc[r][t] += __ldg(L.pb + (size_t)pr * L.M + m) + __ldg(Ai + m) +
                                     __ldg(abv + (size_t)j * ldabv + L.M + m);
                }
            }
        };
        auto epi_z = [&](auto& acc, int te0, int tc0) {
            constexpr int NT = sizeof(acc[0]) / sizeof(float);
            float zv[4][NT];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    int m = tc0 + t;
                    float z = 0.0f;
                    if (m < L.M) {
                        float dz;
                        activation(L.act, acc[r][t], z, dz);
                    }
                    zv[r][t] = z;
                }
            }
            store_tile(T3, te0, tc0, zv, L.MN);
        };
        if constexpr (TC) {
            if (!tc_tile_gemm(C, L.tx, L.M, T1, T3)) { failed = true; break; }
            tile_epilogue_from(L.MN, T3, L.M, [&](auto& acc, int te0, int tc0) {
                pre_z(acc, te0, tc0);
                epi_z(acc, te0, tc0);
            });
        } else {
            tile_gemm_n<kKsForward>(L.MN, L.XK, T1, L.wxT, R, pre_z, epi_z);
            if (R.failed) break;
        }
        // gates: sigmoid (groups) and tanh (transport a, injection b) -> T1 [q][e]
        auto epi_g = [&](auto& acc, int te0, int tc0) {
            constexpr int NT = sizeof(acc[0]) / sizeof(float);
            float gv[4][NT];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    int q = tc0 + t;
                    float v = 0.0f;
                    if (q < GD) {
                        float x = acc[r][t] + __ldg(L.bgd + q);
                        v = q < L.G ? sigmoidf_(x) : tanhf(x);
                    }
                    gv[r][t] = v;
                }
            }
            store_tile(T1, te0, tc0, gv, S.r1);
        };
        if constexpr (TC) {
            if (!tc_tile_gemm(C, L.tgd, GD, T3, T1)) { failed = true; break; }
            tile_epilogue_from(L.GN, T1, GD, epi_g);
        } else {
            tile_gemm_n<kKsForward>(L.GN, L.MK, T3, L.wgdT, R, epi_g);
            if (R.failed) break;
        }
        __syncthreads();
        for (int o = tid; o < ne * GVA; o += blockDim.x) {
            int e = o / GVA, q = o - e * GVA;
            gva_out[(size_t)(e0 + e) * GVA + q] = T1[q * kLd + e] * geo[e * kGeo + 3];
        }
        for (int c = tid; c < L.H; c += blockDim.x) {
            const float* gr = T1 + (c / gw) * kLd;
            float acc = msg[c];
#pragma unroll 8
            for (int e = 0; e < ne; ++e)
                acc += gr[e] * geo[e * kGeo + 3] * __ldg(abv + (size_t)idx[2 * e] * ldabv + 2 * L.M + c);
            msg[c] = acc;
        }
        for (int o = tid; o < DC; o += blockDim.x) {
            int c = o / L.Cl, m = o - c * L.Cl;
            int l = order_of(m);
            const float* ga = T1 + (L.G + (l - 1) * L.Ce + c) * kLd;
            const float* gb = T1 + (L.G + LC + (l - 1) * L.Ce + c) * kLd;
            float acc = inc[o];
#pragma unroll 8
            for (int e = 0; e < ne; ++e)
                acc += geo[e * kGeo + 3] * (ga[e] * __ldg(mixed + (size_t)idx[2 * e] * DC + o) +
                                         gb[e] * sm[S.Y + e * S.ys + m]);
            inc[o] = acc;
        }
    }
    __syncthreads();
    (void)failed;
    for (int c = tid; c < L.H; c += blockDim.x) msg_out[(size_t)i * L.H + c] = msg[c];
    for (int o = tid; o < DC; o += blockDim.x) dn_out[(size_t)i * DC + o] = Di[o] + inc[o];
    if constexpr (TC) tc_release(C);
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

// Centre side of the backward of one EQ block, one block per centre atom, tiles of 32 edges:
// per edge the gate adjoints, dpre (stored for the pull, summed into dA_i), the input adjoint
// dx = W_x^T dpre (basis part -> dE/dr, centre probes -> dD_i, neighbour probes stored for the
// pull), the harmonic adjoint and the edge-vector gradient added to edge_grad.
template <bool TC>
__global__ void __launch_bounds__(kTThreads, 2)
k_eq_backward_centre(int n_atoms, EqLayerArgs L, EdgeList rad, const int* __restrict__ types,
                     const float* __restrict__ abv, const float* __restrict__ D,
                     const float* __restrict__ mixed, const float* __restrict__ dmsg,
                     const float* __restrict__ ddp, float* __restrict__ dpre_out,
                     float* __restrict__ dpn_out, float4* __restrict__ edge_grad,
                     float* __restrict__ dabv, float* __restrict__ ddc,
                     unsigned* __restrict__ err) {
    extern __shared__ float4 smem4[];
    float* sm = reinterpret_cast<float*>(smem4);
    EqTileSmem S(L, true);
    const int i = blockIdx.x;
    if (i >= n_atoms) return;  // uniform per block
    const int tid = threadIdx.x;
    const int DC = L.Ce * L.Cl, LC = L.Le * L.Ce, ldabv = 2 * L.M + L.H, gw = L.H / L.G;
    const int GD = L.G + 2 * LC, NP = L.Ce + L.G;
    float* T1 = sm + S.t1;
    float* T3 = sm + S.t3;
    const float* geo = sm + S.geo;
    const int* idx = reinterpret_cast<const int*>(sm + S.idx);
    float* Di = sm + S.Di;
    float* dDp = sm + S.ddp;
    float* dmi = sm + S.dmsg;
    float* dA = sm + S.accM;
    float* dDc = sm + S.accDC;
    float* dYn = sm + S.dYn;
    float* part = sm + S.part;
    SliceRing R;
    TcCtx C;
    if constexpr (TC) {
        tc_init(C, sm + S.bs, err, L.wait_polls);
    } else {
        int nmax = max(max(L.XN, L.MN), L.GN);
        ring_init(R, sm + S.bs, sm + S.bs + kKsBackward * nmax,
                  reinterpret_cast<unsigned long long*>(sm + S.bar), err, L.wait_polls);
    }
    int ti = types[i];
    for (int o = tid; o < DC; o += blockDim.x) {
        Di[o] = D[(size_t)i * DC + o];
        dDp[o] = ddp[(size_t)i * DC + o];
        dDc[o] = 0.0f;
    }
    for (int m = tid; m < L.M; m += blockDim.x) dA[m] = 0.0f;
    for (int c = tid; c < L.H; c += blockDim.x) dmi[c] = dmsg[(size_t)i * L.H + c];
    const float* Ai = abv + (size_t)i * ldabv;
    int row = rad.row_ptr[i], cnt = rad.cnt[i];
    for (int base = 0; base < cnt; base += kTe) {
        int ne = min(kTe, cnt - base);
        int e0 = row + base;
        __syncthreads();
        tile_geometry(L, S, sm, rad, types, i, ti, e0, ne);
        __syncthreads();
        tile_probes(L, S, sm, D);
        // recompute pre: z -> T3; act' -> this edge's dpre record (read back by the same thread
        // in the dz epilogue, which has the same thread tile)
        auto pre_z = [&](auto& acc, int te0, int tc0) {
            constexpr int NT = sizeof(acc[0]) / sizeof(float);
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                int e = te0 + r;
                int j = idx[2 * e], pr = idx[2 * e + 1];
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    int m = tc0 + t;
                    if (m < L.M)
                        acc[r][t] += __ldg(L.pb + (size_t)pr * L.M + m) + __ldg(Ai + m) +
                                     __ldg(abv + (size_t)j * ldabv + L.M + m);
                }
            }
        };
        auto epi_z = [&](auto& acc, int te0, int tc0) {
            constexpr int NT = sizeof(acc[0]) / sizeof(float);
            float zv[4][NT];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                int e = te0 + r;
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    int m = tc0 + t;
                    float z = 0.0f, dz = 0.0f;
                    if (m < L.M) activation(L.act, acc[r][t], z, dz);
                    zv[r][t] = z;
                    if (m < L.M && e < ne) dpre_out[(size_t)(e0 + e) * L.M + m] = dz;
                }
            }
            store_tile(T3, te0, tc0, zv, L.MN);
        };
        if constexpr (TC) {
            if (!tc_tile_gemm(C, L.tx, L.M, T1, T3)) break;
            tile_epilogue_from(L.MN, T3, L.M, [&](auto& acc, int te0, int tc0) {
                pre_z(acc, te0, tc0);
                epi_z(acc, te0, tc0);
            });
        } else {
            tile_gemm_n<kKsBackward>(L.MN, L.XK, T1, L.wxT, R, pre_z, epi_z);
            if (R.failed) break;
        }
        // gate values -> T1 [q][e]
        auto epi_g = [&](auto& acc, int te0, int tc0) {
            constexpr int NT = sizeof(acc[0]) / sizeof(float);
            float gv[4][NT];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    int q = tc0 + t;
                    float v = 0.0f;
                    if (q < GD) {
                        float x = acc[r][t] + __ldg(L.bgd + q);
                        v = q < L.G ? sigmoidf_(x) : tanhf(x);
                    }
                    gv[r][t] = v;
                }
            }
            store_tile(T1, te0, tc0, gv, S.r1);
        };
        if constexpr (TC) {
            if (!tc_tile_gemm(C, L.tgd, GD, T3, T1)) break;
            tile_epilogue_from(L.GN, T1, GD, epi_g);
        } else {
            tile_gemm_n<kKsBackward>(L.GN, L.MK, T3, L.wgdT, R, epi_g);
            if (R.failed) break;
        }
        __syncthreads();
        // injection part of the harmonic adjoint (reads b before it becomes d logits)
        for (int o = tid; o < kTe * L.Cl; o += blockDim.x) {
            int e = o % kTe, m = o / kTe;  // lanes over edges: one T1 row per warp
            int l = order_of(m);
            const float* gb = T1 + (L.G + LC + (l - 1) * L.Ce) * kLd + e;
            float s = 0.0f;
            for (int c = 0; c < L.Ce; ++c) s += gb[c * kLd] * dDp[c * L.Cl + m];
            dYn[e * S.ys + m] = geo[e * kGeo + 3] * s;
        }
        __syncthreads();
        // direction-gate adjoints -> d logits (rows of a and b), cutoff partials
        if (L.Cl == 24) {
            for (int o = tid; o < kTe * L.Ce; o += blockDim.x) {
                int e = o % kTe, c = o / kTe;
                float mj[24];
                load_row24(mixed + (size_t)idx[2 * e] * DC + (size_t)c * 24, mj);
                const float* dd = dDp + c * 24;
                const float* y = sm + S.Y + e * S.ys;
                float cut = geo[e * kGeo + 3];
                float s1[4] = {0.0f, 0.0f, 0.0f, 0.0f}, s2[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
                for (int m = 0; m < 24; ++m) {
                    float dm = dd[m];
                    s1[order24(m)] += dm * mj[m];
                    s2[order24(m)] += dm * y[m];
                }
                float p = 0.0f;
#pragma unroll
                for (int l = 0; l < 4; ++l) {
                    int qa = L.G + l * L.Ce + c, qb = qa + LC;
                    float a = T1[qa * kLd + e], b = T1[qb * kLd + e];
                    T1[qa * kLd + e] = cut * s1[l] * (1.0f - a * a);
                    T1[qb * kLd + e] = cut * s2[l] * (1.0f - b * b);
                    p += a * s1[l] + b * s2[l];
                }
                part[e * S.ps + c] = p;
            }
        } else
        for (int o = tid; o < kTe * L.Ce; o += blockDim.x) {
            int e = o % kTe, c = o / kTe;
            const float* mj = mixed + (size_t)idx[2 * e] * DC + (size_t)c * L.Cl;
            const float* dd = dDp + c * L.Cl;
            const float* y = sm + S.Y + e * S.ys;
            float cut = geo[e * kGeo + 3];
            float p = 0.0f;
            for (int l = 1; l <= L.Le; ++l) {
                float s1 = 0.0f, s2 = 0.0f;
                for (int m = l * l - 1; m < (l + 1) * (l + 1) - 1; ++m) {
                    s1 += dd[m] * __ldg(mj + m);
                    s2 += dd[m] * y[m];
                }
                int qa = L.G + (l - 1) * L.Ce + c, qb = qa + LC;
                float a = T1[qa * kLd + e], b = T1[qb * kLd + e];
                T1[qa * kLd + e] = cut * s1 * (1.0f - a * a);
                T1[qb * kLd + e] = cut * s2 * (1.0f - b * b);
                p += a * s1 + b * s2;
            }
            part[e * S.ps + c] = p;
        }
        // group-gate adjoints
        for (int o = tid; o < kTe * L.G; o += blockDim.x) {
            int e = o % kTe, g = o / kTe;
            const float* vj = abv + (size_t)idx[2 * e] * ldabv + 2 * L.M + g * gw;
            float dg = 0.0f;
            if (((gw | ldabv | (2 * L.M)) & 3) == 0) {  // 16-byte rows: four values per load
                for (int c = 0; c < gw; c += 4) {
                    float4 v = __ldg(reinterpret_cast<const float4*>(vj + c));
                    dg += dmi[g * gw + c] * v.x;
                    dg += dmi[g * gw + c + 1] * v.y;
                    dg += dmi[g * gw + c + 2] * v.z;
                    dg += dmi[g * gw + c + 3] * v.w;
                }
            } else {
                for (int c = 0; c < gw; ++c) dg += dmi[g * gw + c] * __ldg(vj + c);
            }
            float s = T1[g * kLd + e];
            T1[g * kLd + e] = dg * geo[e * kGeo + 3] * s * (1.0f - s);
            part[e * S.ps + L.Ce + g] = dg * s;
        }
        for (int o = tid; o < kTe * (L.GK - GD); o += blockDim.x) {
            int e = o % kTe, q = GD + o / kTe;
            T1[q * kLd + e] = 0.0f;
        }
        // dz = W_gd^T dl ; dpre = dz act'  -> T3 [m][e], stored per edge
        auto epi_dz = [&](auto& acc, int te0, int tc0) {
            constexpr int NT = sizeof(acc[0]) / sizeof(float);
            float dv[4][NT];
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                int m = tc0 + t;
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    int e = te0 + r;
                    float v = 0.0f;  // padding edges: their gate adjoints are zero
                    if (m < L.M && e < ne) {
                        float* rec = dpre_out + (size_t)(e0 + e) * L.M + m;
                        v = acc[r][t] * *rec;
                        *rec = v;
                    }
                    dv[r][t] = v;
                }
            }
            store_tile(T3, te0, tc0, dv, L.MN);
        };
        if constexpr (TC) {
            if (!tc_tile_gemm(C, L.tgdT, L.M, T1, T3)) break;
            tile_epilogue_from(L.MN, T3, L.M, epi_dz);
        } else {
            tile_gemm_n<kKsBackward>(L.MN, L.GK, T1, L.wgd, R, epi_dz);
            if (R.failed) break;
        }
        __syncthreads();
        for (int m = tid; m < L.M; m += blockDim.x) {
            float acc = dA[m];
            for (int e = 0; e < ne; ++e) acc += T3[m * kLd + e];
            dA[m] = acc;
        }
        // dx = W_x^T dpre -> T1 [k][e]
        if constexpr (TC) {
            // the raw products are the result (rows K + 2 LC .. r1 are not read)
            if (!tc_tile_gemm(C, L.txT, L.K + 2 * LC, T3, T1)) break;
        } else {
            tile_gemm_n<kKsBackward>(L.XN, L.MK, T3, L.wx, R, [&](auto& acc, int te0, int tc0) {
                store_tile(T1, te0, tc0, acc, S.r1);
            });
            if (R.failed) break;
        }
        __syncthreads();
        for (int o = tid; o < ne * LC; o += blockDim.x) {
            int e = o / LC, q = o - e * LC;
            dpn_out[(size_t)(e0 + e) * LC + q] = T1[(L.K + LC + q) * kLd + e];
        }
        for (int o = tid; o < DC; o += blockDim.x) {
            int c = o / L.Cl, m = o - c * L.Cl;
            int l = order_of(m);
            const float* dpc = T1 + (L.K + (l - 1) * L.Ce + c) * kLd;
            float acc = dDc[o];
            for (int e = 0; e < ne; ++e) acc += dpc[e] * sm[S.Y + e * S.ys + m];
            dDc[o] = acc;
        }
        for (int o = tid; o < ne * L.Cl; o += blockDim.x) {
            int e = o / L.Cl, m = o - e * L.Cl;
            int l = order_of(m);
            const float* dpc = T1 + (L.K + (l - 1) * L.Ce) * kLd + e;
            const float* dpn = T1 + (L.K + LC + (l - 1) * L.Ce) * kLd + e;
            const float* Dj = D + (size_t)idx[2 * e] * DC + m;
            float s = 0.0f, t = 0.0f;
#pragma unroll 8
            for (int c = 0; c < L.Ce; ++c) {
                s += dpc[c * kLd] * Di[c * L.Cl + m];
                t += dpn[c * kLd] * __ldg(Dj + c * L.Cl);
            }
            dYn[e * S.ys + m] += s + ((l & 1) ? -t : t);
        }
        __syncthreads();
        if (tid < ne) {
            int e = tid;
            const float* g = geo + e * kGeo;
            float dcut_e = 0.0f;
            for (int q = 0; q < NP; ++q) dcut_e += part[e * S.ps + q];
            float dd = dcut_e * g[4];
            {
                float b[kMaxK], db[kMaxK], c_, dc_;
                cheb_masked(g[6], L.rc, L.K, b, db, c_, dc_);
                for (int k = 0; k < L.K; ++k) dd += T1[k * kLd + e] * db[k];
            }
            float du0 = 0.f, du1 = 0.f, du2 = 0.f;
            const float* w = dYn + e * S.ys;
            angular_components<true>(g[0], g[1], g[2], L.Le, L.zc,
                                     [&](int c, int, float, float dx, float ddy, float dz) {
                                         float wc = w[c] * __ldg(L.scale + c);
                                         du0 += wc * dx;
                                         du1 += wc * ddy;
                                         du2 += wc * dz;
                                     });
            float pu = du0 * g[0] + du1 * g[1] + du2 * g[2];
            float inv = g[5];
            float4 G = edge_grad[e0 + e];
            G.x += dd * g[0] + (du0 - pu * g[0]) * inv;
            G.y += dd * g[1] + (du1 - pu * g[1]) * inv;
            G.z += dd * g[2] + (du2 - pu * g[2]) * inv;
            edge_grad[e0 + e] = G;
        }
    }
    __syncthreads();
    for (int m = tid; m < L.M; m += blockDim.x) dabv[(size_t)i * ldabv + m] = dA[m];
    for (int o = tid; o < DC; o += blockDim.x) ddc[(size_t)i * DC + o] = dDc[o];
    if constexpr (TC) tc_release(C);
}

// Pull side for atom i over the reverse edges of its row: dB_i, dv_i (into dabv), and
// dD_prev = dDp_i + dD_probe,centre + dD_probe,neighbour + W_mix^T dmixed_i.
// Only atoms below n_centres ran the centre kernel and the node backward (a domain call's
// active prefix): reverse edges from other centres are skipped, and the centre-side parts of
// atoms >= n_centres (dA in dabv, dD_p, dD_probe,centre) are zero.
__global__ void k_eq_backward_pull(int n_atoms, int n_centres, EqLayerArgs L, EdgeList rad,
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
        int e0 = row + base;
        // this chunk's edges whose reverse edge belongs to an active centre, compacted
        bool take = false;
        float4 e;
        int j = 0;
        if (lane < min(CH, cnt - base)) {
            e = rad.e[e0 + lane];
            j = edge_j(e);
            take = j < n_centres;
        }
        unsigned ballot = __ballot_sync(0xffffffffu, take);
        int ne = __popc(ballot);
        int slot = __popc(ballot & ((1u << lane) - 1u));
        __syncwarp();
        if (take) {
            sidx[2 * slot] = j;
            sidx[2 * slot + 1] = rad.rev[e0 + lane];
            float r = (float)sqrt((double)e.x * e.x + (double)e.y * e.y + (double)e.z * e.z);
            float inv = 1.0f / fmaxf(r, 1.0e-12f);
            float* y = sY + slot * L.Cl;
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
    bool centre = i < n_centres;
    if (!centre)
        for (int m = lane; m < L.M; m += 32) dabv[(size_t)i * ldabv + m] = 0.0f;
    for (int m = lane; m < L.M; m += 32) dabv[(size_t)i * ldabv + L.M + m] = sdB[m];
    for (int c = lane; c < L.H; c += 32) dabv[(size_t)i * ldabv + 2 * L.M + c] = sdv[c];
    for (int o = lane; o < d.DC; o += 32) {
        int c = o / L.Cl, m = o - c * L.Cl;
        int l = order_of(m);
        float s = (centre ? ddp[(size_t)i * d.DC + o] + ddc[(size_t)i * d.DC + o] : 0.0f) +
                  sdDn[o];
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

namespace {

// Exponent of every output feature f of W [K][N] (its column): all |W[k][f]| < 2^e.
__global__ void k_eq_tc_fexp(const float* __restrict__ W, int K, int N, int rows,
                             int* __restrict__ fexp) {
    int f = blockIdx.x * blockDim.x + threadIdx.x;
    if (f >= rows) return;
    float amax = 0.0f;
    if (f < N)
        for (int k = 0; k < K; ++k) amax = fmaxf(amax, fabsf(W[(size_t)k * N + f]));
    fexp[f] = tc::digit_exponent(amax);
}

// Digit units of W: unit (chunk c, step s) holds features c * 128 .. + 127 and k in
// [32 s, 32 s + 32), four planes of 128 x 32 bytes, K-major core matrices.
__global__ void k_eq_tc_pack(const float* __restrict__ W, int K, int N, int chunks, int steps,
                             const int* __restrict__ fexp, signed char* __restrict__ out) {
    long long total = (long long)chunks * kTcChunk * steps * kTcK;
    for (long long o = blockIdx.x * (long long)blockDim.x + threadIdx.x; o < total;
         o += (long long)gridDim.x * blockDim.x) {
        int f = (int)(o % (chunks * kTcChunk)), k = (int)(o / (chunks * kTcChunk));
        float x = (k < K && f < N) ? W[(size_t)k * N + f] : 0.0f;
        int d[4];
        tc::split_digits(x, fexp[f], d);
        int c = f / kTcChunk, r = f % kTcChunk, s = k / kTcK, kk = k % kTcK;
        size_t unit = ((size_t)c * steps + s) * kTcWUnit;
        uint32_t at = tc_plane_offset(r, kk);
#pragma unroll
        for (int p = 0; p < 4; ++p) out[unit + p * kTcWPlane + at] = (signed char)d[p];
    }
}

}  // namespace

size_t eq_tc_bytes(int K, int N) {
    size_t chunks = (size_t)((N + kTcChunk - 1) / kTcChunk), steps = (size_t)((K + kTcK - 1) / kTcK);
    return chunks * steps * kTcWUnit + chunks * kTcChunk * sizeof(int);
}

EqTcW eq_tc_pack(const float* W, int K, int N, void* out, cudaStream_t stream) {
    EqTcW t;
    t.K = K;
    t.N = N;
    t.chunks = (N + kTcChunk - 1) / kTcChunk;
    t.steps = (K + kTcK - 1) / kTcK;
    if (t.steps > kTcMaxSteps)
        throw Error(RUNE_ERR_INVALID, "EQ tensor-core products support K <= 320");
    signed char* q = static_cast<signed char*>(out);
    int* fexp = reinterpret_cast<int*>(q + (size_t)t.chunks * t.steps * kTcWUnit);
    int rows = t.chunks * kTcChunk;
    k_eq_tc_fexp<<<(rows + 127) / 128, 128, 0, stream>>>(W, K, N, rows, fexp);
    long long total = (long long)rows * t.steps * kTcK;
    int blocks = (int)std::min<long long>((total + 255) / 256, 4096);
    k_eq_tc_pack<<<blocks, 256, 0, stream>>>(W, K, N, t.chunks, t.steps, fexp, q);
    RUNE_CUDA_TRY(cudaGetLastError());
    t.q = q;
    t.fexp = fexp;
    return t;
}

size_t eq_forward_smem(const EqLayerArgs& L) { return sizeof(float) * EqTileSmem(L, false).total; }
size_t eq_backward_smem(const EqLayerArgs& L) { return sizeof(float) * EqTileSmem(L, true).total; }

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
                      float* dn, float* gva, unsigned* err, cudaStream_t stream) {
    if (n == 0) return;
    size_t bytes = eq_forward_smem(L);
    // the SIMT and tensor-core forms are separate instantiations, so that the SIMT kernel keeps
    // its own register allocation
    auto kernel = L.tc ? k_eq_forward_edges<true> : k_eq_forward_edges<false>;
    set_smem((const void*)kernel, bytes);
    RUNE_KERNEL("k_eq_forward_edges", stream,
                kernel<<<n, kTThreads, bytes, stream>>>(n, L, rad, types, abv, D, mixed, msg, dn,
                                                        gva, err));
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

void eq_backward_edges(const EqLayerArgs& L, int n, int n_centres, const EdgeList& rad,
                       const int* types, const float* abv, const float* D, const float* mixed, const float* dmsg,
                       const float* ddp, const float* gva, float* dpre, float* dpn,
                       float4* edge_grad, float* dabv, float* ddc, float* dd_prev,
                       unsigned* err, cudaStream_t stream) {
    if (n == 0) return;
    size_t bytes = eq_backward_smem(L);
    auto centre = L.tc ? k_eq_backward_centre<true> : k_eq_backward_centre<false>;
    set_smem((const void*)centre, bytes);
    if (n_centres > 0) {
        RUNE_KERNEL("k_eq_backward_centre", stream,
                    centre<<<n_centres, kTThreads, bytes, stream>>>(
                        n_centres, L, rad, types, abv, D, mixed, dmsg, ddp, dpre, dpn, edge_grad,
                        dabv, ddc, err));
        RUNE_LAUNCH_CHECK();
    }
    EqDims d(L);
    size_t pbytes = sizeof(float) * kWarps * ((L.M + L.H + 2 * d.DC + CH * (L.Cl + 2) + 3) & ~3);
    set_smem((const void*)k_eq_backward_pull, pbytes);
    RUNE_KERNEL("k_eq_backward_pull", stream,
                k_eq_backward_pull<<<(n + kWarps - 1) / kWarps, kWarps * 32, pbytes, stream>>>(
                    n, n_centres, L, rad, gva, dpre, dpn, dmsg, ddp, ddc, dabv, dd_prev));
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
