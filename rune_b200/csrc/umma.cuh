// Blackwell (sm_100a) tensor-core building blocks: shared-memory matrix descriptors, the tf32
// and i8 instruction descriptors, TMEM allocation, tcgen05.mma / commit / ld, bounded mbarrier
// waits, and the exact digit split of the integer products.
//
// Operand layout (no swizzle, K-major "core matrices" of 8 rows x 16 bytes): leading byte
// offset (between the two core matrices along K) 128 and stride byte offset (between 8-row
// groups) 256, the same for A (rows = M) and B (rows = N). A tf32 step holds 8 k (element
// (r, k) at (r / 8) 256 + (k / 4) 128 + (r % 8) 16 + (k % 4) 4), an i8 step 32 k (element (r, k)
// at (r / 8) 256 + (k / 16) 128 + (r % 8) 16 + k % 16).
#pragma once

#include <cstdint>

namespace rune {
namespace tc {

constexpr uint32_t kALbo = 128, kASbo = 256;  // K-major core-matrix offsets (bytes)
constexpr unsigned kWaitLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// Shared-memory matrix descriptor (no swizzle): start address, leading and stride byte offsets
// in 16-byte units, descriptor version 1 (bits 46-47), base offset 0, layout type 0.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

// Instruction descriptor of tcgen05.mma.kind::tf32: float32 accumulator (bits 4-5 = 1), A and
// B tf32 (bits 7-9 and 10-12 = 2), A and B K-major (bits 15, 16 = 0), N / 8 in bits 17-22,
// M / 16 in bits 24-28.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}

// Instruction descriptor of tcgen05.mma.kind::i8: signed 32-bit accumulator (bits 4-5 = 2), A
// and B signed 8-bit (bits 7-9 and 10-12 = 1), both K-major, N / 8 in bits 17-22, M / 16 in
// bits 24-28.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}

// D[tmem] (+)= A[desc] * B[desc] on signed 8-bit operands with exact int32 accumulation
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Exact split of x (|x| <= 2^e) into four signed digits of 7 bits:
// x = 2^(e - 6) (d0 + d1 2^-7 + d2 2^-14 + d3 2^-21) + r, |r| <= 2^(e - 28), |d_k| <= 64.
// Every step is exact in float32: the scaling is a power of two and each residual is the
// difference of a value and its nearest integer.
__device__ __forceinline__ void split_digits(float x, int e, int (&d)[4]) {
    float y = ldexpf(x, 6 - e);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        float q = rintf(y);
        d[k] = (int)q;
        y = (y - q) * 128.0f;
    }
}

// The same four digits from one rounding to a 27-bit fixed-point integer: q = round(x 2^(27 - e))
// (|q| < 2^27), then balanced base-128 digits by integer shifts, q = d0 2^21 + d1 2^14 + d2 2^7 +
// d3, |d_k| <= 64. x = 2^(e - 6) (d0 + d1 2^-7 + d2 2^-14 + d3 2^-21) + r, |r| <= 2^(e - 28), as
// above (only exact ties may pick other digits).
__device__ __forceinline__ void split_digits_fixed(float x, int e, int (&d)[4]) {
    int q = __float2int_rn(ldexpf(x, 27 - e));
    int d0 = (q + (1 << 20)) >> 21;
    int r = q - (d0 << 21);
    int d1 = (r + (1 << 13)) >> 14;
    r -= d1 << 14;
    int d2 = (r + (1 << 6)) >> 7;
    d[0] = d0;
    d[1] = d1;
    d[2] = d2;
    d[3] = r - (d2 << 7);
}

// x 2^s for the power-of-two scales of the digit products: one multiplication while 2^s is a
// normal float, ldexpf otherwise.
__device__ __forceinline__ float scale_pow2(float x, int s) {
    return (s >= -126 && s <= 127) ? x * __int_as_float((s + 127) << 23) : ldexpf(x, s);
}

// Exponent e with |x| < 2^e for every |x| <= amax (0 for amax = 0).
__device__ __forceinline__ int digit_exponent(float amax) {
    int e = 0;
    if (amax > 0.0f) frexpf(amax, &e);
    return e;
}

__device__ __forceinline__ uint32_t tf32_hi(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

// x -> (hi, lo): hi = x rounded to tf32, lo = (x - hi) rounded to tf32 (the tensor core would
// otherwise truncate lo's low mantissa bits when it reads the 32-bit container)
__device__ __forceinline__ void tf32_split(float x, float& hi, float& lo) {
    hi = __uint_as_float(tf32_hi(x));
    lo = __uint_as_float(tf32_hi(x - hi));
}

// ---------------------------------------------------------------------------- TMEM
// One full warp allocates `cols` columns (a power of two >= 32) and writes the TMEM address
// to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(dst)), "r"(cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols));
}

__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// generic-proxy shared-memory writes -> visible to the tensor core / bulk-copy (async) proxy
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// D[tmem] (+)= A[desc] * B[desc]; one thread issues
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// the mbarrier at `bar` receives one arrival when every MMA issued so far by this thread is
// complete
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(bar) : "memory");
}

// 32 consecutive columns of this thread's TMEM lane (warp w reads lanes 32 (w % 4) .. + 31);
// the load and its wait are one asm statement, so no use of the registers precedes the wait
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive columns of this thread's TMEM lane (as tmem_ld32)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------------------- mbarriers
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

// bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) global -> shared,
// completion counted on `bar` (no multicast)
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// wait until the phase of parity `parity` of `bar` has completed; false after `polls` polls
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity,
                                          unsigned polls = kWaitLimit) {
    for (unsigned it = 0; it < polls; ++it) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}

}  // namespace tc
}  // namespace rune
