// Test infrastructure (checker only, never linked into rune_b200): minimal stand-ins for the
// three GPUMD types that the reference's native Möbius evaluator (rune/mobius/src/mobius.cu,
// pinned to GPUMD fd805e1b) is written against, so that its own sources compile unchanged:
//
//   Box           the simulation cell: cpu_h[0..8] the matrix whose columns are the three cell
//                 vectors (row-major, so x = cpu_h[0] s0 + cpu_h[1] s1 + cpu_h[2] s2), cpu_h[9..17]
//                 its inverse, periodic flags and the perpendicular thickness along each cell
//                 vector (mobius.cu:183-196, 272-284, 330-349);
//   GPU_Vector<T> a device array with size(), data() and resize() (mobius.cuh:26-31);
//   Potential     the base class whose compute() the evaluator overrides, with the cutoff rc
//                 and the atom range [N1, N2) (mobius.cuh:8-17, mobius.cu:303-305, 323).
//
// Written from how mobius.cu uses them; GPUMD itself is not vendored in the reference.
#pragma once

#include <cuda_runtime.h>

#include <cmath>
#include <cstddef>
#include <stdexcept>

struct Box {
    double cpu_h[18] = {};
    int pbc_x = 1, pbc_y = 1, pbc_z = 1;
    double thickness_x = 0, thickness_y = 0, thickness_z = 0;

    // Cell from three row vectors a, b, c (cell[3 v + d] = component d of vector v).
    void set_from_rows(const double* cell, const int* pbc) {
        for (int r = 0; r < 3; ++r)
            for (int c = 0; c < 3; ++c) cpu_h[3 * r + c] = cell[3 * c + r];
        pbc_x = pbc[0];
        pbc_y = pbc[1];
        pbc_z = pbc[2];
        get_inverse();
    }
    double get_volume() const {
        const double* h = cpu_h;
        return std::fabs(h[0] * (h[4] * h[8] - h[5] * h[7]) - h[1] * (h[3] * h[8] - h[5] * h[6]) +
                         h[2] * (h[3] * h[7] - h[4] * h[6]));
    }
    // inverse (adjugate / determinant) and the thickness along each cell vector: volume over
    // the area spanned by the other two
    void get_inverse() {
        const double* h = cpu_h;
        double det = h[0] * (h[4] * h[8] - h[5] * h[7]) - h[1] * (h[3] * h[8] - h[5] * h[6]) +
                     h[2] * (h[3] * h[7] - h[4] * h[6]);
        double* g = cpu_h + 9;
        g[0] = (h[4] * h[8] - h[5] * h[7]) / det;
        g[1] = (h[2] * h[7] - h[1] * h[8]) / det;
        g[2] = (h[1] * h[5] - h[2] * h[4]) / det;
        g[3] = (h[5] * h[6] - h[3] * h[8]) / det;
        g[4] = (h[0] * h[8] - h[2] * h[6]) / det;
        g[5] = (h[2] * h[3] - h[0] * h[5]) / det;
        g[6] = (h[3] * h[7] - h[4] * h[6]) / det;
        g[7] = (h[1] * h[6] - h[0] * h[7]) / det;
        g[8] = (h[0] * h[4] - h[1] * h[3]) / det;
        double v = std::fabs(det);
        auto area = [&](int p, int q) {  // |column p x column q|
            double ax = h[p], ay = h[3 + p], az = h[6 + p];
            double bx = h[q], by = h[3 + q], bz = h[6 + q];
            double cx = ay * bz - az * by, cy = az * bx - ax * bz, cz = ax * by - ay * bx;
            return std::sqrt(cx * cx + cy * cy + cz * cz);
        };
        thickness_x = v / area(1, 2);
        thickness_y = v / area(0, 2);
        thickness_z = v / area(0, 1);
    }
    void set_is_orthogonal() {}  // the stand-in treats every cell as general (triclinic)
    // bins along each cell vector at least `size` thick; one bin along open directions
    void get_num_bins(double size, int* bins) const {
        const double t[3] = {thickness_x, thickness_y, thickness_z};
        const int p[3] = {pbc_x, pbc_y, pbc_z};
        for (int d = 0; d < 3; ++d) {
            int n = p[d] ? (int)std::floor(t[d] / size) : 1;
            bins[d] = n < 1 ? 1 : n;
        }
    }
};

template <typename T>
class GPU_Vector {
public:
    GPU_Vector() = default;
    explicit GPU_Vector(size_t n) { resize(n); }
    GPU_Vector(const GPU_Vector&) = delete;
    GPU_Vector& operator=(const GPU_Vector&) = delete;
    ~GPU_Vector() { cudaFree(ptr_); }
    // contents are not kept across a change of size
    void resize(size_t n) {
        if (n == n_ && ptr_) return;
        cudaFree(ptr_);
        ptr_ = nullptr;
        n_ = n;
        if (n && cudaMalloc(&ptr_, n * sizeof(T)) != cudaSuccess)
            throw std::runtime_error("GPU_Vector: cudaMalloc failed");
    }
    size_t size() const { return n_; }
    T* data() { return ptr_; }
    const T* data() const { return ptr_; }
    void fill_zero() {
        if (n_) cudaMemset(ptr_, 0, n_ * sizeof(T));
    }
    void copy_from_host(const T* h) {
        if (n_) cudaMemcpy(ptr_, h, n_ * sizeof(T), cudaMemcpyHostToDevice);
    }
    void copy_to_host(T* h) const {
        if (n_) cudaMemcpy(h, ptr_, n_ * sizeof(T), cudaMemcpyDeviceToHost);
    }

private:
    T* ptr_ = nullptr;
    size_t n_ = 0;
};

class Potential {
public:
    double rc = 0.0;
    int N1 = 0, N2 = 0;
    virtual ~Potential() = default;
    virtual void compute(Box& box, const GPU_Vector<int>& type,
                         const GPU_Vector<double>& position, GPU_Vector<double>& potential,
                         GPU_Vector<double>& force, GPU_Vector<double>& virial) = 0;
};
