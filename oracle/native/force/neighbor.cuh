// Test infrastructure (checker only): stand-ins for the GPUMD cell-list helpers that the
// reference's native Möbius evaluator calls (rune/mobius/src/mobius.cu:205-270, 375):
//
//   apply_mic      minimum-image displacement through fractional coordinates (periodic axes);
//   find_cell_id   bin of a wrapped position: floor(fractional coordinate x bins) per axis,
//                  flattened as cx + nx (cy + ny cz), the order mobius.cu's stencil uses;
//   find_cell_list per-bin counts, their exclusive sum and the atoms of every bin, sorted by
//                  index within a bin.
//
// Bins are at least half a cutoff thick along each cell vector (Box::get_num_bins), so the
// evaluator's five-bin stencil covers every pair inside the cutoff.
#pragma once

#include <thrust/device_ptr.h>
#include <thrust/scan.h>

#include "potential.cuh"

__device__ __forceinline__ void apply_mic(const Box& box, double& x, double& y, double& z) {
    const double* h = box.cpu_h;
    const double* g = box.cpu_h + 9;
    double sx = g[0] * x + g[1] * y + g[2] * z;
    double sy = g[3] * x + g[4] * y + g[5] * z;
    double sz = g[6] * x + g[7] * y + g[8] * z;
    if (box.pbc_x) sx -= nearbyint(sx);
    if (box.pbc_y) sy -= nearbyint(sy);
    if (box.pbc_z) sz -= nearbyint(sz);
    x = h[0] * sx + h[1] * sy + h[2] * sz;
    y = h[3] * sx + h[4] * sy + h[5] * sz;
    z = h[6] * sx + h[7] * sy + h[8] * sz;
}

__device__ __forceinline__ int standin_bin(double s, int n) {
    int c = (int)floor(s * n);
    c %= n;
    if (c < 0) c += n;
    return c;
}

__device__ __forceinline__ void find_cell_id(const Box& box, double x, double y, double z,
                                             double /*rc_inv: bins come from the box*/, int nx,
                                             int ny, int nz, int& cx, int& cy, int& cz,
                                             int& cell) {
    const double* g = box.cpu_h + 9;
    cx = standin_bin(g[0] * x + g[1] * y + g[2] * z, nx);
    cy = standin_bin(g[3] * x + g[4] * y + g[5] * z, ny);
    cz = standin_bin(g[6] * x + g[7] * y + g[8] * z, nz);
    cell = cx + nx * (cy + ny * cz);
}

namespace gpumd_standin {

__global__ void k_cell_of(Box box, int n, const double* pos, int nx, int ny, int nz,
                          int* cell_of, int* count) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    int cx, cy, cz, cell;
    find_cell_id(box, pos[i], pos[n + i], pos[2 * n + i], 0.0, nx, ny, nz, cx, cy, cz, cell);
    cell_of[i] = cell;
    atomicAdd(count + cell, 1);
}

__global__ void k_cell_fill(int n, const int* cell_of, const int* sum, int* cursor,
                            int* contents) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    int c = cell_of[i];
    contents[sum[c] + atomicAdd(cursor + c, 1)] = i;
}

__global__ void k_cell_sort(int cells, const int* count, const int* sum, int* contents) {
    int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cells) return;
    int* a = contents + sum[c];
    for (int k = 1; k < count[c]; ++k) {  // insertion sort: bins hold a few atoms
        int v = a[k], m = k - 1;
        while (m >= 0 && a[m] > v) {
            a[m + 1] = a[m];
            --m;
        }
        a[m + 1] = v;
    }
}

}  // namespace gpumd_standin

inline void find_cell_list(double /*cell size: bins already fixed*/, const int* bins, Box& box,
                           const GPU_Vector<double>& position, GPU_Vector<int>& cell_count,
                           GPU_Vector<int>& cell_count_sum, GPU_Vector<int>& cell_contents) {
    using namespace gpumd_standin;
    const int n = (int)(position.size() / 3);
    const int cells = bins[0] * bins[1] * bins[2];
    cell_count.resize(cells);
    cell_count_sum.resize(cells);
    if ((int)cell_contents.size() != n) cell_contents.resize(n);
    GPU_Vector<int> cell_of(n > 0 ? n : 1), cursor(cells);
    cell_count.fill_zero();
    cursor.fill_zero();
    const int t = 128;
    if (n > 0)
        k_cell_of<<<(n + t - 1) / t, t>>>(box, n, position.data(), bins[0], bins[1], bins[2],
                                          cell_of.data(), cell_count.data());
    thrust::exclusive_scan(thrust::device_ptr<int>(cell_count.data()),
                           thrust::device_ptr<int>(cell_count.data() + cells),
                           thrust::device_ptr<int>(cell_count_sum.data()));
    if (n > 0) {
        k_cell_fill<<<(n + t - 1) / t, t>>>(n, cell_of.data(), cell_count_sum.data(),
                                            cursor.data(), cell_contents.data());
        k_cell_sort<<<(cells + t - 1) / t, t>>>(cells, cell_count.data(), cell_count_sum.data(),
                                                cell_contents.data());
    }
    if (cudaGetLastError() != cudaSuccess)
        throw std::runtime_error("find_cell_list: kernel launch failed");
}
