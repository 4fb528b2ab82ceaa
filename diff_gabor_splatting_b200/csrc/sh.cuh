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

template <int Degree>
__device__ __forceinline__ void sh_basis_grad(float x, float y, float z, float* dx, float* dy,
                                              float* dz) {
    constexpr int K = (Degree + 1) * (Degree + 1);
#pragma unroll
    for (int k = 0; k < K; ++k) dx[k] = dy[k] = dz[k] = 0.f;
    if constexpr (Degree > 0) {
        constexpr float c1 = 0.4886025119029199f;
        dy[1] = -c1;
        dz[2] = c1;
        dx[3] = -c1;
    }
    if constexpr (Degree > 1) {
        constexpr float a = 1.0925484305920792f, c = 0.31539156525252005f,
                        d = 0.5462742152960396f;
        dx[4] = a * y; dy[4] = a * x;
        dy[5] = -a * z; dz[5] = -a * y;
        dx[6] = -2 * c * x; dy[6] = -2 * c * y; dz[6] = 4 * c * z;
        dx[7] = -a * z; dz[7] = -a * x;
        dx[8] = 2 * d * x; dy[8] = -2 * d * y;
    }
    if constexpr (Degree > 2) {
        constexpr float a = -0.5900435899266435f, b1 = 2.890611442640554f,
                        c = -0.4570457994644658f, d = 0.3731763325901154f,
                        e = 1.445305721320277f;
        dx[9] = 6 * a * x * y; dy[9] = 3 * a * (x * x - y * y);
        dx[10] = b1 * y * z; dy[10] = b1 * x * z; dz[10] = b1 * x * y;
        dx[11] = -2 * c * x * y; dy[11] = c * (4 * z * z - x * x - 3 * y * y); dz[11] = 8 * c * y * z;
        dx[12] = -6 * d * x * z; dy[12] = -6 * d * y * z; dz[12] = d * (6 * z * z - 3 * x * x - 3 * y * y);
        dx[13] = c * (4 * z * z - 3 * x * x - y * y); dy[13] = -2 * c * x * y; dz[13] = 8 * c * x * z;
        dx[14] = 2 * e * x * z; dy[14] = -2 * e * y * z; dz[14] = e * (x * x - y * y);
        dx[15] = 3 * a * (x * x - y * y); dy[15] = -6 * a * x * y;
    }
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
    float basis[K], dx[K], dy[K], dz[K];
    sh_basis<Degree>(dir[0], dir[1], dir[2], basis);
    sh_basis_grad<Degree>(dir[0], dir[1], dir[2], dx, dy, dz);
#pragma unroll
    for (int set = 0; set < 2; ++set) {
        const float* coeffs = set == 0 ? first : second;
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) {
            const float raw = sh_raw<Degree>(basis, coeffs, ch);
            const float g = raw >= 0.f ? gcol[set * 3 + ch] : 0.f;
            if (g == 0.f) continue;
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const float cf = __ldg(coeffs + k * 3 + ch);
                gdir[0] += g * cf * dx[k];
                gdir[1] += g * cf * dy[k];
                gdir[2] += g * cf * dz[k];
            }
        }
    }
}

}  // namespace gs
