// Stand-alone SH colour entry points behind the SHColors autograd bridge
// (rendering.py:221-238 -> spherical_harmonics.cu:45-150).  One thread per
// (scene, surfel); the thread loops over the scene's cameras, so the backward
// sums the coefficient gradients over cameras in registers instead of issuing the
// reference's per-pair atomics (spherical_harmonics.cu:70-71).
#include "common.cuh"
#include "sh.cuh"

namespace gs {
namespace {

constexpr int kShThreads = 256;

template <int Degree>
__global__ __launch_bounds__(kShThreads) void sh_forward_kernel(
    const float* __restrict__ first, const float* __restrict__ second,
    const float* __restrict__ dirs, int64_t C, int64_t N, float* __restrict__ colors) {
    constexpr int K = (Degree + 1) * (Degree + 1);
    const int64_t n = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t s = blockIdx.y;
    if (n >= N) return;
    const int64_t sn = s * N + n;
    for (int64_t c = 0; c < C; ++c) {
        const int64_t p = (s * C + c) * N + n;
        float basis[K];
        sh_basis<Degree>(dirs[p * 3], dirs[p * 3 + 1], dirs[p * 3 + 2], basis);
#pragma unroll
        for (int set = 0; set < 2; ++set)
#pragma unroll
            for (int ch = 0; ch < 3; ++ch)
                colors[p * 6 + set * 3 + ch] =
                    fmaxf(sh_raw<Degree>(basis, (set ? second : first) + sn * K * 3, ch), 0.f);
    }
}

template <int Degree>
__global__ __launch_bounds__(kShThreads) void sh_backward_kernel(
    const float* __restrict__ first, const float* __restrict__ second,
    const float* __restrict__ dirs, const float* __restrict__ gcolors, int64_t C, int64_t N,
    float* __restrict__ gfirst, float* __restrict__ gsecond, float* __restrict__ gdirs) {
    constexpr int K = (Degree + 1) * (Degree + 1);
    const int64_t n = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t s = blockIdx.y;
    if (n >= N) return;
    const int64_t sn = s * N + n;
    for (int64_t c = 0; c < C; ++c) {
        const int64_t p = (s * C + c) * N + n;
        float d[3] = {dirs[p * 3], dirs[p * 3 + 1], dirs[p * 3 + 2]};
        float g[6], gd[3] = {0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 6; ++i) g[i] = gcolors[p * 6 + i];
        sh_direction_grad<Degree>(d, first + sn * K * 3, second + sn * K * 3, g, gd);
#pragma unroll
        for (int i = 0; i < 3; ++i) gdirs[p * 3 + i] = gd[i];
    }
#pragma unroll 1
    for (int sc = 0; sc < 6; ++sc) {
        const int set = sc / 3, ch = sc % 3;
        const float* cf = (set ? second : first) + sn * K * 3;
        float coef[K], acc[K];
#pragma unroll
        for (int k = 0; k < K; ++k) { coef[k] = cf[k * 3 + ch]; acc[k] = 0.f; }
        for (int64_t c = 0; c < C; ++c) {
            const int64_t p = (s * C + c) * N + n;
            const float g = gcolors[p * 6 + sc];
            float basis[K];
            sh_basis<Degree>(dirs[p * 3], dirs[p * 3 + 1], dirs[p * 3 + 2], basis);
            float raw = 0.5f;
#pragma unroll
            for (int k = 0; k < K; ++k) raw += basis[k] * coef[k];
            if (raw >= 0.f) {
#pragma unroll
                for (int k = 0; k < K; ++k) acc[k] += g * basis[k];
            }
        }
        float* out = (set ? gsecond : gfirst) + sn * K * 3;
#pragma unroll
        for (int k = 0; k < K; ++k) out[k * 3 + ch] = acc[k];
    }
}

}  // namespace
}  // namespace gs

using namespace gs;

extern "C" int gs_sh_forward(const float* first, const float* second, const float* directions,
                             int degree, int64_t scenes, int64_t cameras, int64_t surfels,
                             float* colors, void* stream) {
    if (degree < 0 || degree > 3) return fail(GS_ERR_ARGUMENT, "SH degree must be 0 through 3");
    if (scenes < 0 || cameras < 0 || surfels < 0) return fail(GS_ERR_ARGUMENT, "gs_sh_forward: invalid sizes");
    if (scenes > 65535) return fail(GS_ERR_LIMIT, "gs_sh_forward: more than 65535 scenes");
    if (scenes == 0 || cameras == 0 || surfels == 0) return GS_OK;
    dim3 grid(unsigned((surfels + kShThreads - 1) / kShThreads), unsigned(scenes));
    auto s = as_stream(stream);
    switch (degree) {
        case 0: sh_forward_kernel<0><<<grid, kShThreads, 0, s>>>(first, second, directions, cameras, surfels, colors); break;
        case 1: sh_forward_kernel<1><<<grid, kShThreads, 0, s>>>(first, second, directions, cameras, surfels, colors); break;
        case 2: sh_forward_kernel<2><<<grid, kShThreads, 0, s>>>(first, second, directions, cameras, surfels, colors); break;
        default: sh_forward_kernel<3><<<grid, kShThreads, 0, s>>>(first, second, directions, cameras, surfels, colors); break;
    }
    GS_CHECK_LAUNCH("sh_forward_kernel");
    return GS_OK;
}

extern "C" int gs_sh_backward(const float* first, const float* second, const float* directions,
                              const float* grad_colors, int degree, int64_t scenes, int64_t cameras,
                              int64_t surfels, float* grad_first, float* grad_second,
                              float* grad_directions, void* stream) {
    if (degree < 0 || degree > 3) return fail(GS_ERR_ARGUMENT, "SH degree must be 0 through 3");
    if (scenes < 0 || cameras < 0 || surfels < 0) return fail(GS_ERR_ARGUMENT, "gs_sh_backward: invalid sizes");
    if (scenes > 65535) return fail(GS_ERR_LIMIT, "gs_sh_backward: more than 65535 scenes");
    auto s = as_stream(stream);
    const int64_t K = int64_t(degree + 1) * (degree + 1);
    if (scenes == 0 || surfels == 0) return GS_OK;
    if (cameras == 0) {
        GS_CUDA(cudaMemsetAsync(grad_first, 0, sizeof(float) * scenes * surfels * K * 3, s));
        GS_CUDA(cudaMemsetAsync(grad_second, 0, sizeof(float) * scenes * surfels * K * 3, s));
        return GS_OK;
    }
    dim3 grid(unsigned((surfels + kShThreads - 1) / kShThreads), unsigned(scenes));
#define GS_SHB(D) sh_backward_kernel<D><<<grid, kShThreads, 0, s>>>(first, second, directions, grad_colors, cameras, surfels, grad_first, grad_second, grad_directions)
    switch (degree) {
        case 0: GS_SHB(0); break;
        case 1: GS_SHB(1); break;
        case 2: GS_SHB(2); break;
        default: GS_SHB(3); break;
    }
#undef GS_SHB
    GS_CHECK_LAUNCH("sh_backward_kernel");
    return GS_OK;
}
