// Velocity-Verlet NVE on the device with a Verlet-skin neighbour cache.
//
// Candidate lists hold every pair within max(rc) + skin (the cluster neighbour build with the
// larger cutoff); each step re-forms the pair vectors from the current positions and keeps the
// pairs inside the cutoffs (filter_candidates). The candidates are rebuilt when an atom has moved
// more than skin / 2 since the last build — the rebuild rule of the reference's native cache
// (rune/mobius/src/mobius.cu:334-402, rune/mobius/mobius_neighbor_check.py:24-83).
//
// Units: positions in A, velocities in A/fs, masses in amu, forces in eV/A, time step in fs;
// a = F / m * 9.64853321e-3 A/fs^2 and the kinetic energy is 1/2 m v^2 * 103.642697 eV.

#include <algorithm>
#include <cstring>

#include "engine.cuh"

namespace rune {

namespace {

constexpr double kAccel = 9.64853321e-3;  // (eV / A / amu) -> A / fs^2
constexpr double kKinetic = 103.642697;   // amu A^2 / fs^2 -> eV

// First half of a step: v += dt/2 a, x += dt v; the largest squared displacement from the
// reference positions of the candidate build (atomicMax on the bits: non-negative doubles order
// like their bit patterns).
__global__ void k_vv_drift(int n, double dt, const float* __restrict__ F,
                           const double* __restrict__ m, double* __restrict__ x,
                           double* __restrict__ v, const double* __restrict__ x_ref,
                           unsigned long long* __restrict__ max_d2) {
    __shared__ double red[256];
    int a = blockIdx.x * blockDim.x + threadIdx.x;
    double d2 = 0.0;
    if (a < n) {
        double s = 0.5 * dt * kAccel / m[a];
        for (int k = 0; k < 3; ++k) {
            double vk = v[3 * a + k] + s * (double)F[3 * a + k];
            double xk = x[3 * a + k] + dt * vk;
            v[3 * a + k] = vk;
            x[3 * a + k] = xk;
            double d = xk - x_ref[3 * a + k];
            d2 += d * d;
        }
    }
    red[threadIdx.x] = d2;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) red[threadIdx.x] = fmax(red[threadIdx.x], red[threadIdx.x + s]);
        __syncthreads();
    }
    if (threadIdx.x == 0) atomicMax(max_d2, (unsigned long long)__double_as_longlong(red[0]));
}

// Second half: v += dt/2 a and the per-atom kinetic energy.
__global__ void k_vv_kick(int n, double dt, const float* __restrict__ F,
                          const double* __restrict__ m, double* __restrict__ v,
                          double* __restrict__ ke) {
    int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= n) return;
    double s = 0.5 * dt * kAccel / m[a];
    double e = 0.0;
    for (int k = 0; k < 3; ++k) {
        double vk = v[3 * a + k] + s * (double)F[3 * a + k];
        v[3 * a + k] = vk;
        e += vk * vk;
    }
    ke[a] = 0.5 * m[a] * e * kKinetic;
}

// Kinetic energy of the initial velocities.
__global__ void k_kinetic(int n, const double* __restrict__ m, const double* __restrict__ v,
                          double* __restrict__ ke) {
    int a = blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= n) return;
    double e = v[3 * a] * v[3 * a] + v[3 * a + 1] * v[3 * a + 1] + v[3 * a + 2] * v[3 * a + 2];
    ke[a] = 0.5 * m[a] * e * kKinetic;
}

// Deterministic sum (one block, fixed order) of x[0..n) into *out.
__global__ void k_sum(int n, const double* __restrict__ x, double* __restrict__ out) {
    __shared__ double red[256];
    double s = 0.0;
    for (int a = threadIdx.x; a < n; a += blockDim.x) s += x[a];
    red[threadIdx.x] = s;
    __syncthreads();
    for (int k = blockDim.x / 2; k > 0; k >>= 1) {
        if (threadIdx.x < k) red[threadIdx.x] += red[threadIdx.x + k];
        __syncthreads();
    }
    if (threadIdx.x == 0) *out = red[0];
}

struct DeviceBuffer {
    void* p = nullptr;
    explicit DeviceBuffer(size_t bytes) {
        RUNE_CUDA_TRY(cudaMalloc(&p, bytes ? bytes : 1));
    }
    ~DeviceBuffer() {
        if (p) cudaFree(p);
    }
    template <typename T>
    T* as() const { return static_cast<T*>(p); }
};

struct PinnedScalars {
    double* p = nullptr;
    PinnedScalars() { RUNE_CUDA_TRY(cudaMallocHost(&p, 8 * sizeof(double))); }
    ~PinnedScalars() {
        if (p) cudaFreeHost(p);
    }
};

}  // namespace

void md_nve(Engine& e, const MdArgs& a, cudaStream_t stream) {
    const int n = a.n_atoms;
    const int tpb = 256;
    const int blocks = std::max(1, (n + tpb - 1) / tpb);
    DeviceBuffer x_ref(sizeof(double) * 3 * std::max(n, 1));
    DeviceBuffer ke(sizeof(double) * std::max(n, 1));
    DeviceBuffer scal(sizeof(double) * 8);  // [0] max d2 bits, [1] kinetic, [2] potential
    DeviceBuffer fbuf(sizeof(float) * 3 * std::max(n, 1));
    float* F = a.forces ? a.forces : fbuf.as<float>();
    double* d_scal = scal.as<double>();
    PinnedScalars host;
    int atom_ptr[2] = {0, n};
    BatchInput in{n, 1, a.types, a.positions, a.cell, a.pbc, atom_ptr};
    const double half_skin2 = 0.25 * a.skin * a.skin;

    Arena cand_ws;  // candidate lists persist across steps until the next rebuild
    // frees the candidate arena on every exit, including a failed rebuild or evaluation
    struct ArenaGuard {
        Arena& a;
        ~ArenaGuard() {
            if (a.base) cudaFree(a.base);
            a.base = nullptr;
        }
    } cand_guard{cand_ws};
    NeighborData cand;
    int cand_stride = 0;
    int64_t rebuilds = 0;

    auto rebuild = [&]() {
        RUNE_CUDA_TRY(cudaMemcpyAsync(x_ref.p, a.positions, sizeof(double) * 3 * n,
                                      cudaMemcpyDeviceToDevice, stream));
        for (int attempt = 0; attempt < 40; ++attempt) {
            std::swap(e.ws, cand_ws);
            e.staging.off = 0;
            e.stage_first = ~size_t(0);
            bool grow = false;
            try {
                e.ws.reset();
                CallTables ct = stage_call_tables(e, 1, atom_ptr, stream);
                build_neighbors(e, in, ct.atom_ptr, cand, stream, a.skin, &cand_stride);
            } catch (const Error& err) {
                if (err.code != -1) {
                    std::swap(e.ws, cand_ws);
                    throw;
                }
                grow = true;
            }
            std::swap(e.ws, cand_ws);
            if (grow) {
                RUNE_CUDA_TRY(cudaStreamSynchronize(stream));
                size_t cap = std::max(2 * cand_ws.want + (64u << 20), cand_ws.cap * 2);
                if (cand_ws.base) RUNE_CUDA_TRY(cudaFree(cand_ws.base));
                cand_ws.base = nullptr;
                cand_ws.cap = 0;
                if (cudaMalloc(&cand_ws.base, cap) != cudaSuccess) {
                    cudaGetLastError();
                    throw Error(RUNE_ERR_OOM, "candidate list allocation failed");
                }
                cand_ws.cap = cap;
                continue;
            }
            // candidate rows that did not fit: raise the stride and build again
            unsigned long long maxc[4];
            unsigned int flags = 0;
            RUNE_CUDA_TRY(cudaMemcpyAsync(maxc, cand.summary, sizeof(maxc),
                                          cudaMemcpyDeviceToHost, stream));
            RUNE_CUDA_TRY(cudaMemcpyAsync(&flags, e.d_flags, sizeof(flags),
                                          cudaMemcpyDeviceToHost, stream));
            RUNE_CUDA_TRY(cudaStreamSynchronize(stream));
            if (flags & 16u) {
                RUNE_CUDA_TRY(cudaMemsetAsync(e.d_flags, 0, sizeof(unsigned int), stream));
                int largest = (int)(std::max(maxc[0], maxc[1]) >> 32);
                cand_stride = (largest + largest / 8 + 8 + 7) & ~7;
                continue;
            }
            e.check_flags(flags, stream);
            ++rebuilds;
            return;
        }
        throw Error(RUNE_ERR_OOM, "candidate list sizing did not converge");
    };

    // forces and potential energy at the current positions, from the candidate lists
    auto forces = [&]() {
        for (int attempt = 0; attempt < 40; ++attempt) {
            e.ws.reset();
            e.staging.off = 0;
            e.stage_first = ~size_t(0);
            try {
                CallTables ct = stage_call_tables(e, 1, atom_ptr, stream);
                e.flush_uploads(stream);
                NeighborData nd;
                filter_candidates(e, cand, a.positions, nd, stream);
                Outputs o{nullptr, d_scal + 2, F, nullptr, RUNE_FORCES};
                evaluate(e, nd, n, 1, a.types, ct, o, stream);
                unsigned long long maxc[4];
                unsigned int flags = 0;
                RUNE_CUDA_TRY(cudaMemcpyAsync(maxc, nd.summary, sizeof(maxc),
                                              cudaMemcpyDeviceToHost, stream));
                RUNE_CUDA_TRY(cudaMemcpyAsync(&flags, e.d_flags, sizeof(flags),
                                              cudaMemcpyDeviceToHost, stream));
                RUNE_CUDA_TRY(cudaStreamSynchronize(stream));
                e.check_flags(flags, stream);
                HostSync hs{};
                std::memcpy(hs.maxc, maxc, sizeof(maxc));
                finish_neighbors(e, nd, hs);  // neighbour limits and statistics
                return;
            } catch (const Error& err) {
                if (err.code != -1) throw;
                grow_workspace(e, e.ws.want, stream);
            }
        }
        throw Error(RUNE_ERR_OOM, "workspace sizing did not converge");
    };

    auto record = [&](int step) {
        RUNE_KERNEL("k_sum", stream, k_sum<<<1, tpb, 0, stream>>>(n, ke.as<double>(), d_scal + 1));
        RUNE_CUDA_TRY(cudaMemcpyAsync(host.p, d_scal, sizeof(double) * 3, cudaMemcpyDeviceToHost,
                                      stream));
        RUNE_CUDA_TRY(cudaStreamSynchronize(stream));
        if (a.energies) {
            a.energies[2 * step] = host.p[2];
            a.energies[2 * step + 1] = host.p[1];
        }
    };

    rebuild();
    forces();
    if (n > 0)
        RUNE_KERNEL("k_kinetic", stream,
                    k_kinetic<<<blocks, tpb, 0, stream>>>(n, a.masses, a.velocities,
                                                          ke.as<double>()));
    record(0);
    for (int step = 1; step <= a.n_steps; ++step) {
        RUNE_CUDA_TRY(cudaMemsetAsync(d_scal, 0, sizeof(double), stream));
        if (n > 0)
            RUNE_KERNEL("k_vv_drift", stream,
                        k_vv_drift<<<blocks, tpb, 0, stream>>>(
                            n, a.dt, F, a.masses, a.positions, a.velocities, x_ref.as<double>(),
                            reinterpret_cast<unsigned long long*>(d_scal)));
        RUNE_CUDA_TRY(cudaMemcpyAsync(host.p, d_scal, sizeof(double), cudaMemcpyDeviceToHost,
                                      stream));
        RUNE_CUDA_TRY(cudaStreamSynchronize(stream));
        double max_d2;
        std::memcpy(&max_d2, host.p, sizeof(double));
        if (max_d2 > half_skin2) rebuild();
        forces();
        if (n > 0)
            RUNE_KERNEL("k_vv_kick", stream,
                        k_vv_kick<<<blocks, tpb, 0, stream>>>(n, a.dt, F, a.masses, a.velocities,
                                                              ke.as<double>()));
        record(step);
    }
    if (a.rebuilds) *a.rebuilds = rebuilds;
}

}  // namespace rune
