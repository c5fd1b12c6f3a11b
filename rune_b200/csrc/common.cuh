// Shared device helpers and engine-internal declarations for the rune_b200 CUDA engine.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

#include "../../include/rune_b200.h"

namespace rune {

constexpr int kWarp = 32;

// ----------------------------------------------------------------------------- errors
void set_error(const std::string& message);

struct Status {
    int code = RUNE_OK;
    std::string message;
};

#define RUNE_CUDA_TRY(expr)                                                              \
    do {                                                                                 \
        cudaError_t _e = (expr);                                                         \
        if (_e != cudaSuccess) {                                                         \
            throw ::rune::Error(RUNE_ERR_CUDA, std::string(#expr) + ": " +               \
                                                   cudaGetErrorString(_e));              \
        }                                                                                \
    } while (0)

#define RUNE_LAUNCH_CHECK() RUNE_CUDA_TRY(cudaGetLastError())

struct Error {
    int code;
    std::string message;
    Error(int c, std::string m) : code(c), message(std::move(m)) {}
};

// ----------------------------------------------------------------------------- profiling
// Kernel launch accounting. The engine installs its profiler as the thread's current one for
// the duration of a call; every launch site opens a KernelScope, which counts the launch and,
// when timing is on, brackets it with CUDA events on the launching stream.
struct Profiler {
    bool timing = false;
    int64_t launches = 0;
    struct Pending {
        std::string name;
        cudaEvent_t start, stop;
    };
    std::vector<Pending> pending;
    std::vector<cudaEvent_t> pool;
    std::map<std::string, std::pair<double, int64_t>> totals;
    std::vector<std::string> order;

    cudaEvent_t event();
    void resolve();  // after the stream is synchronised
    void release();
};

Profiler* current_profiler();
void set_current_profiler(Profiler* p);

struct KernelScope {
    Profiler* prof;
    cudaStream_t stream;
    std::string name;
    cudaEvent_t stop = nullptr;
    KernelScope(const char* kernel, cudaStream_t s, int n_launches = 1);
    ~KernelScope();
};

#define RUNE_KERNEL(name, stream, ...)              \
    do {                                            \
        ::rune::KernelScope _rune_ks(name, stream); \
        __VA_ARGS__;                                \
    } while (0)

// ----------------------------------------------------------------------------- device math
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Activation value and derivative (rune/mobius/layers.py:11-23: tanh, SiLU, exact-erf GELU).
__device__ __forceinline__ void activation(int kind, float x, float& y, float& dy) {
    if (kind == RUNE_ACT_TANH) {
        float t = tanhf(x);
        y = t;
        dy = 1.0f - t * t;
    } else if (kind == RUNE_ACT_SILU) {
        float s = 1.0f / (1.0f + expf(-x));
        y = x * s;
        dy = s * (1.0f + x * (1.0f - s));
    } else {
        const float inv_sqrt2 = 0.70710678118654752f;
        const float inv_sqrt2pi = 0.39894228040143268f;
        float cdf = 0.5f * (1.0f + erff(x * inv_sqrt2));
        y = x * cdf;
        dy = cdf + x * inv_sqrt2pi * expf(-0.5f * x * x);
    }
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// Edge record: r_ij (x, y, z) in float32 and the neighbour index j in the w slot.
__device__ __forceinline__ int edge_j(const float4& e) { return __float_as_int(e.w); }

// ----------------------------------------------------------------------------- edge lists
// Row i of a list owns e[row_ptr[i] .. row_ptr[i] + cnt[i]).
struct EdgeList {
    const float4* e = nullptr;
    const int* row_ptr = nullptr;
    const int* cnt = nullptr;
    const int* rev = nullptr;  // index of the reverse edge (j -> i, -S), when built
};

// ----------------------------------------------------------------------------- descriptor
struct DescParams {
    int nr, na, kr, ka, lmax, C, nL, D, T;
    float rc_r, rc_a;
    const float* c_r;    // [T, T, nr, kr]
    const float* c_a;    // [T, T, na, ka]
    // The c-tables transposed to [T, T, k, n] with n padded to a multiple of 4 (npr, npa
    // float4 per k), so that one lane reads all channels of one basis function as float4.
    const float4* c_rt;
    const float4* c_at;
    int npr, npa;        // float4 per (type pair, k)
    const float* zc;     // [9][9][9] z-polynomial coefficients, zc[L][m][power]
    int n_terms;
    // Invariant monomials, grouped by output L: {coef (float bits), L, factors packed 8 bits
    // each (0xff unused), 0}; term_ptr[L] .. term_ptr[L + 1] are the terms of output L.
    const int4* terms;
    const int* term_ptr;  // [nL + 1]
    // Derivative table: one entry per occurrence of harmonic c in a term,
    // {coef (float bits), L, the other factors packed (0xff unused), c}; entries of harmonic c
    // are dterm_ptr[c] .. dterm_ptr[c + 1].
    const int4* dterms;
    const int* dterm_ptr;  // [C + 1]
    int n_dterms;
};

}  // namespace rune
