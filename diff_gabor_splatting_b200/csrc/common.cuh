// Shared constants, error plumbing and small device helpers of libgabor_b200.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/gabor_b200.h"

namespace gs {

constexpr int kTile = 16;                 // tile edge in pixels (rasterize.cu:16)
constexpr int kBlock = kTile * kTile;     // one thread per tile pixel
constexpr int kRec = GS_RECORD_FLOATS;    // 20-float splat record
constexpr int kMaps = 9;                  // rgb, alpha, depth, normal(3), distortion
constexpr float kPi = 3.14159265358979323846f;

// Per-thread error message set by the C entry points.
void set_error(const std::string& message);
int fail(int code, const std::string& message);
int cuda_status(cudaError_t error, const char* what);

#define GS_CHECK_LAUNCH(what)                                              \
    do {                                                                   \
        cudaError_t e_ = cudaGetLastError();                               \
        if (e_ != cudaSuccess) return ::gs::cuda_status(e_, what);         \
    } while (0)

#define GS_CUDA(call)                                                      \
    do {                                                                   \
        cudaError_t e_ = (call);                                           \
        if (e_ != cudaSuccess) return ::gs::cuda_status(e_, #call);        \
    } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

__device__ __forceinline__ void cross3(const float* a, const float* b, float* c) {
    c[0] = a[1] * b[2] - a[2] * b[1];
    c[1] = a[2] * b[0] - a[0] * b[2];
    c[2] = a[0] * b[1] - a[1] * b[0];
}

// Tile rectangle [x0, y0, x1, y1) of a record: the reference's integer bounds
// (rasterize.cu:24-30): float (x - r)/16 and (x + r + 15)/16, truncated, clamped.
__device__ __forceinline__ int4 tile_rect(float x, float y, int radius, int tw, int th) {
    return make_int4(max(0, min(tw, int((x - radius) / kTile))),
                     max(0, min(th, int((y - radius) / kTile))),
                     max(0, min(tw, int((x + radius + kTile - 1) / kTile))),
                     max(0, min(th, int((y + radius + kTile - 1) / kTile))));
}

// Warp reduce-scatter of NV (power of two, <= 32) per-lane values: afterwards lane
// l holds the warp-wide sum of value (l >> (5 - log2 NV)) in v[0].  Costs
// NV - 1 + (5 - log2 NV) shuffles instead of 5 * NV for NV separate reductions.
template <int NV>
__device__ __forceinline__ void warp_reduce_scatter(float* v, int lane) {
    static_assert(NV >= 1 && NV <= 32 && (NV & (NV - 1)) == 0, "NV must be a power of two");
    int bit = 16;
#pragma unroll
    for (int half = NV / 2; half >= 1; half /= 2) {
        bool upper = lane & bit;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            float send = upper ? v[i] : v[i + half];
            float keep = upper ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
        }
        bit >>= 1;
    }
    for (; bit >= 1; bit >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], bit);
}

}  // namespace gs
