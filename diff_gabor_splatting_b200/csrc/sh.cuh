// Real spherical-harmonic basis (Inria ordering) through degree 3 and its
// direction derivatives: the basis and constants of spherical_harmonics.cu:11-42
// (the same real-SH table as the reference's polynomial test oracle,
// tests/test_spherical_harmonics.py:20-68).
#pragma once

namespace gs {

template <int Degree>
__device__ __forceinline__ void sh_basis(float x, float y, float z, float* b) {
    b[0] = 0.28209479177387814f;
    if constexpr (Degree > 0) {
        constexpr float c1 = 0.4886025119029199f;
        b[1] = -c1 * y;
        b[2] = c1 * z;
        b[3] = -c1 * x;
    }
    if constexpr (Degree > 1) {
        constexpr float a = 1.0925484305920792f, c = 0.31539156525252005f,
                        d = 0.5462742152960396f;
        b[4] = a * x * y;
        b[5] = -a * y * z;
        b[6] = c * (2 * z * z - x * x - y * y);
        b[7] = -a * x * z;
        b[8] = d * (x * x - y * y);
    }
    if constexpr (Degree > 2) {
        constexpr float a = -0.5900435899266435f, b1 = 2.890611442640554f,
                        c = -0.4570457994644658f, d = 0.3731763325901154f,
                        e = 1.445305721320277f;
        b[9] = a * y * (3 * x * x - y * y);
        b[10] = b1 * x * y * z;
        b[11] = c * y * (4 * z * z - x * x - y * y);
        b[12] = d * z * (2 * z * z - 3 * x * x - 3 * y * y);
        b[13] = c * x * (4 * z * z - x * x - y * y);
        b[14] = e * z * (x * x - y * y);
        b[15] = a * x * (x * x - 3 * y * y);
    }
}

// gdir += sum_k h_k grad(basis_k)(x, y, z): the basis derivatives of the table above
// contracted with per-coefficient weights h as they are formed, so the 3K derivatives
// are never held at once.
template <int Degree>
__device__ __forceinline__ void sh_basis_grad_dot(float x, float y, float z, const float* h,
                                                  float* gdir) {
    float gx = 0.f, gy = 0.f, gz = 0.f;
    if constexpr (Degree > 0) {
        constexpr float c1 = 0.4886025119029199f;
        gy -= c1 * h[1];
        gz += c1 * h[2];
        gx -= c1 * h[3];
    }
    if constexpr (Degree > 1) {
        constexpr float a = 1.0925484305920792f, c = 0.31539156525252005f,
                        d = 0.5462742152960396f;
        gx += a * y * h[4] - a * z * h[7] - 2 * c * x * h[6] + 2 * d * x * h[8];
        gy += a * x * h[4] - a * z * h[5] - 2 * c * y * h[6] - 2 * d * y * h[8];
        gz += -a * y * h[5] + 4 * c * z * h[6] - a * x * h[7];
    }
    if constexpr (Degree > 2) {
        constexpr float a = -0.5900435899266435f, b1 = 2.890611442640554f,
                        c = -0.4570457994644658f, d = 0.3731763325901154f,
                        e = 1.445305721320277f;
        const float xx = x * x, yy = y * y, zz = z * z;
        gx += 6 * a * x * y * h[9] + b1 * y * z * h[10] - 2 * c * x * y * h[11] -
              6 * d * x * z * h[12] + c * (4 * zz - 3 * xx - yy) * h[13] + 2 * e * x * z * h[14] +
              3 * a * (xx - yy) * h[15];
        gy += 3 * a * (xx - yy) * h[9] + b1 * x * z * h[10] + c * (4 * zz - xx - 3 * yy) * h[11] -
              6 * d * y * z * h[12] - 2 * c * x * y * h[13] - 2 * e * y * z * h[14] -
              6 * a * x * y * h[15];
        gz += b1 * x * y * h[10] + 8 * c * y * z * h[11] + d * (6 * zz - 3 * xx - 3 * yy) * h[12] +
              8 * c * x * z * h[13] + e * (xx - yy) * h[14];
    }
    gdir[0] += gx;
    gdir[1] += gy;
    gdir[2] += gz;
}

// Clamped colour raw = 0.5 + sum_k basis_k coef_k (spherical_harmonics.cu:62-64).
template <int Degree>
__device__ __forceinline__ float sh_raw(const float* basis, const float* coeffs, int ch) {
    constexpr int K = (Degree + 1) * (Degree + 1);
    float raw = 0.5f;
#pragma unroll
    for (int k = 0; k < K; ++k) raw += basis[k] * __ldg(coeffs + k * 3 + ch);
    return raw;
}

// Add to gdir the direction gradient of both clamped colour sets given their
// gradients gcol[6] (first rgb, second rgb); spherical_harmonics.cu:65-75.
template <int Degree>
__device__ __forceinline__ void sh_direction_grad(const float* dir, const float* first,
                                                  const float* second, const float* gcol,
                                                  float* gdir) {
    constexpr int K = (Degree + 1) * (Degree + 1);
    bool any = false;
#pragma unroll
    for (int i = 0; i < 6; ++i) any = any || gcol[i] != 0.f;
    if (!any) return;
    // Each clamped channel that passes weights its coefficients: h_k = sum over (set,
    // channel) of g * coef_k, and d/ddir sum_k basis_k coef_k g = sum_k h_k grad(basis_k).
    // One (set, channel) at a time, so only its K coefficients are live.
    float basis[K], h[K];
    sh_basis<Degree>(dir[0], dir[1], dir[2], basis);
#pragma unroll
    for (int k = 0; k < K; ++k) h[k] = 0.f;
#pragma unroll 1
    for (int sc = 0; sc < 6; ++sc) {
        float g = gcol[0];
#pragma unroll
        for (int i = 1; i < 6; ++i) g = sc == i ? gcol[i] : g;
        if (g == 0.f) continue;
        const float* coeffs = (sc < 3 ? first : second) + (sc < 3 ? sc : sc - 3);
        float coef[K];
        float raw = 0.5f;
#pragma unroll
        for (int k = 0; k < K; ++k) {
            coef[k] = __ldg(coeffs + k * 3);
            raw += basis[k] * coef[k];
        }
        if (!(raw >= 0.f)) continue;   // clamped: adds nothing
#pragma unroll
        for (int k = 0; k < K; ++k) h[k] = fmaf(g, coef[k], h[k]);
    }
    sh_basis_grad_dot<Degree>(dir[0], dir[1], dir[2], h, gdir);
}

}  // namespace gs
