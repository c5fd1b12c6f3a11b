// Radial and angular basis functions shared by the descriptor, MP and EQ kernels.
#pragma once

#include <cuda_runtime.h>

namespace rune {

// f_k (and df_k/dr with DERIV) for k < K, handed to visit(k, f_k, df_k) in increasing k.
// Evaluated in float64 from r / rc with cospi / sinpi: a float32 pi (rounded up) and 1/rc
// would bias every basis function the same way, which adds up over edges and atoms. Each value
// is rounded to float32 once.
template <bool DERIV, typename Visit>
__device__ __forceinline__ void chebyshev_visit(float rf, float rcf, int K, Visit&& visit) {
    const double pi = 3.14159265358979323846;
    double r = rf, rc = rcf;
    double xr = r / rc;
    double fc, fcp = 0.0;
    if (DERIV) {
        double sv, cv;
        sincospi(xr, &sv, &cv);
        fc = 0.5 * cv + 0.5;
        fcp = -0.5 * pi / rc * sv;
    } else {
        fc = 0.5 * cospi(xr) + 0.5;
    }
    double rs = xr - 1.0;
    double x = 2.0 * rs * rs - 1.0;
    double dxdr = 4.0 * rs / rc;
    if (K <= 0) return;
    visit(0, (float)fc, (float)fcp);
    if (K == 1) return;
    double t2 = 1.0, t1 = x, u2 = 1.0, u1 = 2.0 * x;
    double core = 0.5 * (x + 1.0);
    visit(1, (float)(core * fc), DERIV ? (float)(0.5 * dxdr * fc + core * fcp) : 0.0f);
    for (int k = 2; k < K; ++k) {
        double tn = 2.0 * x * t1 - t2;
        core = 0.5 * (tn + 1.0);
        float d = 0.0f;
        if (DERIV) d = (float)(0.5 * k * u1 * dxdr * fc + core * fcp);
        visit(k, (float)(core * fc), d);
        t2 = t1; t1 = tn;
        if (DERIV) {
            double un = 2.0 * x * u1 - u2;
            u2 = u1; u1 = un;
        }
    }
}

// f_k and df_k/dr for k < K into out[k], dout[k] (either may be null).
__device__ __forceinline__ void chebyshev(float rf, float rcf, int K, float* out, float* dout) {
    if (dout)
        chebyshev_visit<true>(rf, rcf, K, [&](int k, float f, float df) {
            if (out) out[k] = f;
            dout[k] = df;
        });
    else
        chebyshev_visit<false>(rf, rcf, K, [&](int k, float f, float) { out[k] = f; });
}

// Real polynomial angular basis (descriptor.py:574-624): for order L and m = 0..L the
// component is zf_{L,m}(z) (m = 0) or zf_{L,m}(z) * {Re, Im}((x + i y)^m), zf a polynomial in
// z with coefficients zc[L][m][p]. `visit(c, L, Y, dYx, dYy, dYz)` gets every component in
// the reference order; derivatives are with respect to the unnormalised (x, y, z).
template <bool GRAD, int LMAX = 8, typename Visit>
__device__ __forceinline__ void angular_components(float x, float y, float z, int lmax,
                                                   const float* __restrict__ zc, Visit&& visit) {
    static_assert(LMAX >= 1 && LMAX <= 8, "LMAX must be in 1..8");
    float zp[LMAX + 1], wr[LMAX + 1], wi[LMAX + 1];
    zp[0] = 1.0f; wr[0] = 1.0f; wi[0] = 0.0f;
#pragma unroll
    for (int p = 1; p <= LMAX; ++p) {
        zp[p] = zp[p - 1] * z;
        wr[p] = wr[p - 1] * x - wi[p - 1] * y;
        wi[p] = wr[p - 1] * y + wi[p - 1] * x;
    }
#pragma unroll
    for (int L = 1; L <= LMAX; ++L) {
        if (L > lmax) break;
        int c = L * L - 1;
#pragma unroll
        for (int m = 0; m <= L; ++m) {
            float zf = 0.0f, dzf = 0.0f;
            const float* coef = zc + (L * 9 + m) * 9;
#pragma unroll
            for (int p = (L + m) & 1; p <= L - m; p += 2) {
                float a = __ldg(coef + p);
                zf += a * zp[p];
                if (GRAD && p > 0) dzf += a * (float)p * zp[p - 1];
            }
            if (m == 0) {
                visit(c, L, zf, 0.0f, 0.0f, dzf);
                ++c;
            } else {
                float mre = (float)m * wr[m - 1], mim = (float)m * wi[m - 1];
                visit(c, L, zf * wr[m], zf * mre, -zf * mim, dzf * wr[m]);
                visit(c + 1, L, zf * wi[m], zf * mim, zf * mre, dzf * wi[m]);
                c += 2;
            }
        }
    }
}

// Message-edge basis (descriptor.py:357-374), zero at and beyond rc; float64 internally for
// the same reason as the descriptor basis.
__device__ __forceinline__ void cheb_masked(float rf, float rcf, int K, float* b, float* db,
                                            float& cut, float& dcut) {
    const double pi = 3.14159265358979323846;
    double r = rf, rc = rcf;
    double xr = r / rc;
    bool inside = rf < rcf;
    double fc = inside ? 0.5 * cospi(xr) + 0.5 : 0.0;
    double fcp = inside ? -0.5 * pi / rc * sinpi(xr) : 0.0;
    cut = (float)fc;
    dcut = (float)fcp;
    double rs = xr - 1.0;
    double x = 2.0 * rs * rs - 1.0;
    double dxdr = 4.0 * rs / rc;
    b[0] = (float)fc;
    if (db) db[0] = (float)fcp;
    if (K == 1) return;
    double t2 = 1.0, t1 = x, u2 = 1.0, u1 = 2.0 * x;
    double core = 0.5 * (x + 1.0);
    b[1] = (float)(core * fc);
    if (db) db[1] = (float)(0.5 * dxdr * fc + core * fcp);
    for (int k = 2; k < K; ++k) {
        double tn = 2.0 * x * t1 - t2;
        double un = 2.0 * x * u1 - u2;
        core = 0.5 * (tn + 1.0);
        b[k] = (float)(core * fc);
        if (db) db[k] = (float)(0.5 * k * u1 * dxdr * fc + core * fcp);
        t2 = t1; t1 = tn;
        u2 = u1; u1 = un;
    }
}

}  // namespace rune
