// Test infrastructure (checker only, never linked into rune_b200): a C ABI around the
// reference's native FP64 Möbius evaluator (class Mobius, rune/mobius/src/mobius.cu:300-483),
// compiled from the reference's own sources against the GPUMD stand-ins in force/. It is what a
// GPUMD run of the reference would execute for one force evaluation (Mobius::compute on the
// default stream), driven with one structure:
//
//   rn_create   Mobius(model_path, n_atoms)      the `mobius1` file written by export_model
//   rn_compute  Mobius::compute, `reps` times on device-resident inputs (the first call is not
//               timed), returning the last call's per-atom energies, forces [n][3] and the
//               virial W_ab = -sum_e g_a r_b (row-major), and the mean device time per call
//
// GPUMD's conventions are translated here: positions and forces are [3][n] device arrays,
// the per-atom virial is nine [n] arrays xx yy zz xy xz yz yx zx zy of -r_a g_b
// (force.cu:59-63), and potential / force / virial are accumulated, so they are zeroed before
// every call.
#include <cstring>
#include <string>
#include <vector>

#include "mobius.cuh"

namespace {
thread_local std::string g_error;
}

extern "C" {

const char* rn_last_error() { return g_error.c_str(); }

int rn_create(const char* model_path, int n_atoms, void** handle) {
    try {
        *handle = new Mobius(model_path, n_atoms);
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return 1;
    }
}

void rn_destroy(void* handle) { delete static_cast<Mobius*>(handle); }

int rn_compute(void* handle, int n, const int* types, const double* pos, const double* cell,
               const int* pbc, double* energies, double* forces, double* virial, int reps,
               float* ms_per_call) {
    try {
        Mobius& m = *static_cast<Mobius*>(handle);
        Box box;
        box.set_from_rows(cell, pbc);
        GPU_Vector<int> t(n);
        GPU_Vector<double> p(3 * (size_t)n), pe(n), f(3 * (size_t)n), w(9 * (size_t)n);
        t.copy_from_host(types);
        std::vector<double> soa(3 * (size_t)n);
        for (int i = 0; i < n; ++i)
            for (int d = 0; d < 3; ++d) soa[(size_t)d * n + i] = pos[3 * (size_t)i + d];
        p.copy_from_host(soa.data());
        auto once = [&]() {
            pe.fill_zero();
            f.fill_zero();
            w.fill_zero();
            m.compute(box, t, p, pe, f, w);
        };
        once();
        cudaEvent_t a, b;
        cudaEventCreate(&a);
        cudaEventCreate(&b);
        cudaEventRecord(a, 0);
        for (int r = 0; r < reps; ++r) once();
        cudaEventRecord(b, 0);
        cudaEventSynchronize(b);
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, a, b);
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        if (ms_per_call) *ms_per_call = reps > 0 ? ms / reps : 0.0f;
        cudaError_t st = cudaDeviceSynchronize();
        if (st != cudaSuccess) throw std::runtime_error(cudaGetErrorString(st));
        pe.copy_to_host(energies);
        f.copy_to_host(soa.data());
        for (int i = 0; i < n; ++i)
            for (int d = 0; d < 3; ++d) forces[3 * (size_t)i + d] = soa[(size_t)d * n + i];
        std::vector<double> wa(9 * (size_t)n);
        w.copy_to_host(wa.data());
        const int ca[9] = {0, 1, 2, 0, 0, 1, 1, 2, 2}, cb[9] = {0, 1, 2, 1, 2, 2, 0, 0, 1};
        for (int k = 0; k < 9; ++k) virial[k] = 0.0;
        for (int k = 0; k < 9; ++k) {
            double s = 0.0;
            for (int i = 0; i < n; ++i) s += wa[(size_t)k * n + i];
            virial[3 * cb[k] + ca[k]] += s;  // GPUMD (a, b) = -sum r_a g_b = W_ba
        }
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return 1;
    }
}

}  // extern "C"
