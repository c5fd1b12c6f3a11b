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

// The same basis evaluated in float32 throughout, for the NEP kernels, whose issue budget goes
// to conversions between float32 and float64 in the form above. What biased the earlier float32
// form is avoided: r / rc is a correctly rounded division (no rounded 1/rc), and the cosine
// cutoff comes from sincospif / cospif (cos(pi x) without a rounded pi), so every rounding is
// to nearest and none is shared by all basis functions. The Chebyshev recurrences run in
// float32 (errors of a few ulps that grow linearly with k, both signs). Only the derivative
// factors pi / rc and 4 / rc are rounded constants (relative 6e-8 on df, never on f).
template <bool DERIV, typename Visit>
__device__ __forceinline__ void chebyshev_visit_f32(float r, float rc, int K, Visit&& visit) {
    float xr = __fdiv_rn(r, rc);
    float fc, fcp = 0.0f;
    if (DERIV) {
        float sv, cv;
        sincospif(xr, &sv, &cv);
        fc = 0.5f * cv + 0.5f;
        fcp = (-0.5f * 3.14159265358979323846f / rc) * sv;
    } else {
        fc = 0.5f * cospif(xr) + 0.5f;
    }
    float rs = xr - 1.0f;
    float x = fmaf(2.0f * rs, rs, -1.0f);
    float dxdr = (4.0f / rc) * rs;
    if (K <= 0) return;
    visit(0, fc, fcp);
    if (K == 1) return;
    float t2 = 1.0f, t1 = x, u2 = 1.0f, u1 = 2.0f * x;
    float core = 0.5f * (x + 1.0f);
    visit(1, core * fc, DERIV ? 0.5f * dxdr * fc + core * fcp : 0.0f);
    for (int k = 2; k < K; ++k) {
        float tn = fmaf(2.0f * x, t1, -t2);
        core = 0.5f * (tn + 1.0f);
        float d = 0.0f;
        if (DERIV) d = 0.5f * (float)k * u1 * dxdr * fc + core * fcp;
        visit(k, core * fc, d);
        t2 = t1; t1 = tn;
        if (DERIV) {
            float un = fmaf(2.0f * x, u1, -u2);
            u2 = u1; u1 = un;
        }
    }
}

// |r| of an edge vector in float32 (the float64 form converts four times per edge).
__device__ __forceinline__ float edge_len_f32(float x, float y, float z) {
    return sqrtf(fmaf(x, x, fmaf(y, y, z * z)));
}

// The float64 (F32 = false) or float32 (F32 = true) form of the basis and of |r|.
template <bool F32, bool DERIV, typename Visit>
__device__ __forceinline__ void basis_visit(float r, float rc, int K, Visit&& visit) {
    if constexpr (F32)
        chebyshev_visit_f32<DERIV>(r, rc, K, visit);
    else
        chebyshev_visit<DERIV>(r, rc, K, visit);
}

template <bool F32>
__device__ __forceinline__ float edge_len(const float4& e) {
    if constexpr (F32)
        return edge_len_f32(e.x, e.y, e.z);
    else
        return (float)sqrt((double)e.x * e.x + (double)e.y * e.y + (double)e.z * e.z);
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
