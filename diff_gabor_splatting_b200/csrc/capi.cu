// Error plumbing, version, and the layout converters used by the reference-layout
// (`_C`-style) entry points.
#include <string>

#include "common.cuh"

namespace gs {

namespace {
thread_local std::string g_last_error;
constexpr int kPackThreads = 256;
unsigned blocks_for(int64_t n) { return unsigned((n + kPackThreads - 1) / kPackThreads); }

// geometry[Q][17] + opacity of the record's primitive -> 20-float record
__global__ void pack_geometry_kernel(int64_t Q, const float* __restrict__ geometry,
                                     const float* __restrict__ opacities,
                                     const int64_t* __restrict__ prim_ids,
                                     float* __restrict__ records) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= Q * kRec) return;
    const int64_t q = i / kRec;
    const int k = int(i % kRec);
    float v = 0.f;
    if (k < 17) v = geometry[q * 17 + k];
    else if (k == 17) v = opacities[prim_ids[q]];
    records[i] = v;
}

__global__ void pack_rows_kernel(int64_t A, int width, int padded, const float* __restrict__ in,
                                 float* __restrict__ out) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= A * padded) return;
    const int64_t a = i / padded;
    const int k = int(i % padded);
    out[i] = k < width ? in[a * width + k] : 0.f;
}

__global__ void unpack_rows_kernel(int64_t A, int width, int padded, const float* __restrict__ in,
                                   float* __restrict__ out) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= A * width) return;
    out[i] = in[(i / width) * padded + i % width];
}

__global__ void unpack_geometry_kernel(int64_t Q, const float* __restrict__ grad_records,
                                       const int64_t* __restrict__ prim_ids,
                                       float* __restrict__ grad_geometry,
                                       float* __restrict__ grad_opacities) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= Q * 18) return;
    const int64_t q = i / 18;
    const int k = int(i % 18);
    const float v = grad_records[q * kRec + k];
    if (k < 17) grad_geometry[q * 17 + k] = v;
    else if (v != 0.f) atomicAdd(grad_opacities + prim_ids[q], v);
}
// Scene, camera and surfel of each reported pair p = (s C + c) N + n.  Unsigned 32-bit
// division when the pair index and the divisors fit (the usual case), 64-bit otherwise.
__global__ void pair_ids_kernel(int64_t count, const int64_t* __restrict__ pairs, int64_t C,
                                int64_t N, bool narrow, int64_t* __restrict__ scene_ids,
                                int64_t* __restrict__ camera_ids,
                                int64_t* __restrict__ primitive_ids) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= count) return;
    const int64_t p = pairs ? pairs[i] : i;
    int64_t image, n;
    narrow = narrow && p >= 0 && p <= 0xffffffffLL;
    if (narrow) {
        const unsigned q = unsigned(p) / unsigned(N);
        image = q;
        n = int64_t(unsigned(p) - q * unsigned(N));
    } else {
        image = p / N;
        n = p - image * N;
    }
    const int64_t s = narrow ? int64_t(unsigned(image) / unsigned(C)) : image / C;
    if (scene_ids) scene_ids[i] = s;
    if (camera_ids) camera_ids[i] = image - s * C;
    if (primitive_ids) primitive_ids[i] = n;
}
// Per-surfel appearance rows from the separate appearance tensors (classic: colour 3,
// secondary colour 3, weights 4, magnitudes 4, phases 4 -> 20-float rows; neural: W1 30,
// b1 6, W2 18, b2 3 -> 60-float rows), and the reverse for their gradients.  One thread
// per row slot; the pad slots are written zero.
struct SurfelRowTable {
    const float* in[5];
    float* out[5];
    int width[5], first[6], parts, padded;
};

__global__ void pack_surfel_rows_kernel(int64_t A, SurfelRowTable t, float* __restrict__ rows) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= A * t.padded) return;
    const int64_t a = i / t.padded;
    const int k = int(i % t.padded);
    float v = 0.f;
#pragma unroll
    for (int p = 0; p < 5; ++p)
        if (p < t.parts && k >= t.first[p] && k < t.first[p + 1])
            v = t.in[p][a * t.width[p] + (k - t.first[p])];
    rows[i] = v;
}

__global__ void unpack_surfel_rows_kernel(int64_t A, SurfelRowTable t,
                                          const float* __restrict__ rows) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int used = t.first[t.parts];
    if (i >= A * used) return;
    const int64_t a = i / used;
    const int k = int(i % used);
    const float v = rows[a * t.padded + k];
#pragma unroll
    for (int p = 0; p < 5; ++p)
        if (p < t.parts && k >= t.first[p] && k < t.first[p + 1])
            t.out[p][a * t.width[p] + (k - t.first[p])] = v;
}

SurfelRowTable surfel_row_table(int neural) {
    SurfelRowTable t{};
    static const int classic[5] = {3, 3, 4, 4, 4}, siren[4] = {30, 6, 18, 3};
    t.parts = neural ? 4 : 5;
    t.padded = neural ? GS_NEURAL_ROW_FLOATS : GS_CLASSIC_ROW_FLOATS;
    t.first[0] = 0;
    for (int p = 0; p < t.parts; ++p) {
        t.width[p] = neural ? siren[p] : classic[p];
        t.first[p + 1] = t.first[p] + t.width[p];
    }
    return t;
}

// FP32 throughput probe: every thread runs eight independent multiply-add chains (or
// eight float2 chains issued as paired FFMA2), so the FMA pipes, not latency, bound it.
template <bool Paired>
__global__ __launch_bounds__(256) void fp32_probe_kernel(int iterations, float seed,
                                                         float* __restrict__ out) {
    constexpr int kChains = 8;
    const float b = 0.999f, c = 1e-3f * seed;
    float result = 0.f;
    if constexpr (Paired) {
        float2 acc[kChains];
#pragma unroll
        for (int k = 0; k < kChains; ++k) acc[k] = make_float2(threadIdx.x + k, blockIdx.x - k);
        const float2 b2 = make_float2(b, b), c2 = make_float2(c, c);
        for (int i = 0; i < iterations; ++i) {
#pragma unroll
            for (int k = 0; k < kChains; ++k) acc[k] = __ffma2_rn(acc[k], b2, c2);
        }
#pragma unroll
        for (int k = 0; k < kChains; ++k) result += acc[k].x + acc[k].y;
    } else {
        float acc[kChains];
#pragma unroll
        for (int k = 0; k < kChains; ++k) acc[k] = float(threadIdx.x + k);
        for (int i = 0; i < iterations; ++i) {
#pragma unroll
            for (int k = 0; k < kChains; ++k) acc[k] = fmaf(acc[k], b, c);
        }
#pragma unroll
        for (int k = 0; k < kChains; ++k) result += acc[k];
    }
    if (result == 12345.f) out[blockIdx.x] = result;   // keeps the chains live
}
}  // namespace

void set_error(const std::string& message) { g_last_error = message; }

int fail(int code, const std::string& message) {
    set_error(message);
    return code;
}

int cuda_status(cudaError_t error, const char* what) {
    return fail(GS_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(error));
}

}  // namespace gs

using namespace gs;

extern "C" int gs_version(void) { return 1; }

extern "C" const char* gs_last_error(void) { return g_last_error.c_str(); }

extern "C" int gs_pack_geometry(const float* geometry, const float* opacities,
                                const int64_t* primitive_ids, int64_t Q, int64_t opacity_count,
                                float* records, void* stream) {
    if (Q < 0 || opacity_count < 0) return fail(GS_ERR_ARGUMENT, "gs_pack_geometry: invalid sizes");
    if (Q == 0) return GS_OK;
    pack_geometry_kernel<<<blocks_for(Q * kRec), kPackThreads, 0, as_stream(stream)>>>(
        Q, geometry, opacities, primitive_ids, records);
    GS_CHECK_LAUNCH("pack_geometry_kernel");
    return GS_OK;
}

extern "C" int gs_pack_rows(const float* appearance, int64_t A, int width, float* rows, void* stream) {
    if (A < 0 || (width != 18 && width != 57)) return fail(GS_ERR_ARGUMENT, "gs_pack_rows: invalid sizes");
    if (A == 0) return GS_OK;
    const int padded = width == 18 ? GS_CLASSIC_ROW_FLOATS : GS_NEURAL_ROW_FLOATS;
    pack_rows_kernel<<<blocks_for(A * padded), kPackThreads, 0, as_stream(stream)>>>(
        A, width, padded, appearance, rows);
    GS_CHECK_LAUNCH("pack_rows_kernel");
    return GS_OK;
}

extern "C" int gs_unpack_geometry_grads(const float* grad_records, const int64_t* primitive_ids,
                                        int64_t Q, int64_t opacity_count, float* grad_geometry,
                                        float* grad_opacities, void* stream) {
    if (Q < 0 || opacity_count < 0) return fail(GS_ERR_ARGUMENT, "gs_unpack_geometry_grads: invalid sizes");
    auto s = as_stream(stream);
    if (opacity_count) GS_CUDA(cudaMemsetAsync(grad_opacities, 0, sizeof(float) * opacity_count, s));
    if (Q == 0) return GS_OK;
    unpack_geometry_kernel<<<blocks_for(Q * 18), kPackThreads, 0, s>>>(Q, grad_records, primitive_ids,
                                                                        grad_geometry, grad_opacities);
    GS_CHECK_LAUNCH("unpack_geometry_kernel");
    return GS_OK;
}

extern "C" int gs_unpack_rows(const float* rows, int64_t A, int width, float* appearance, void* stream) {
    if (A < 0 || (width != 18 && width != 57)) return fail(GS_ERR_ARGUMENT, "gs_unpack_rows: invalid sizes");
    if (A == 0) return GS_OK;
    const int padded = width == 18 ? GS_CLASSIC_ROW_FLOATS : GS_NEURAL_ROW_FLOATS;
    unpack_rows_kernel<<<blocks_for(A * width), kPackThreads, 0, as_stream(stream)>>>(
        A, width, padded, rows, appearance);
    GS_CHECK_LAUNCH("unpack_rows_kernel");
    return GS_OK;
}

extern "C" int gs_pair_ids(const int64_t* pairs, int64_t count, int64_t cameras, int64_t surfels,
                           int64_t* scene_ids, int64_t* camera_ids, int64_t* primitive_ids,
                           void* stream) {
    if (count < 0 || cameras < 1 || surfels < 1)
        return fail(GS_ERR_ARGUMENT, "gs_pair_ids: invalid sizes");
    if (count == 0) return GS_OK;
    const bool narrow = cameras <= 0xffffffffLL && surfels <= 0xffffffffLL;
    pair_ids_kernel<<<blocks_for(count), kPackThreads, 0, as_stream(stream)>>>(
        count, pairs, cameras, surfels, narrow, scene_ids, camera_ids, primitive_ids);
    GS_CHECK_LAUNCH("pair_ids_kernel");
    return GS_OK;
}

extern "C" int gs_fp32_probe(int blocks, int iterations, int paired, float* out, void* stream) {
    if (blocks < 1 || iterations < 1 || !out)
        return fail(GS_ERR_ARGUMENT, "gs_fp32_probe: invalid arguments");
    auto s = as_stream(stream);
    if (paired)
        fp32_probe_kernel<true><<<unsigned(blocks), 256, 0, s>>>(iterations, 1.f, out);
    else
        fp32_probe_kernel<false><<<unsigned(blocks), 256, 0, s>>>(iterations, 1.f, out);
    GS_CHECK_LAUNCH("fp32_probe_kernel");
    return GS_OK;
}

extern "C" int gs_pack_surfel_rows(int neural, const float* const* appearance, int64_t count,
                                   float* rows, void* stream) {
    if (count < 0 || !appearance || (count > 0 && !rows))
        return fail(GS_ERR_ARGUMENT, "gs_pack_surfel_rows: invalid arguments");
    if (count == 0) return GS_OK;
    SurfelRowTable t = surfel_row_table(neural);
    for (int p = 0; p < t.parts; ++p) {
        if (!appearance[p]) return fail(GS_ERR_ARGUMENT, "gs_pack_surfel_rows: NULL input");
        t.in[p] = appearance[p];
    }
    pack_surfel_rows_kernel<<<blocks_for(count * t.padded), kPackThreads, 0, as_stream(stream)>>>(
        count, t, rows);
    GS_CHECK_LAUNCH("pack_surfel_rows_kernel");
    return GS_OK;
}

extern "C" int gs_unpack_surfel_rows(int neural, const float* rows, int64_t count,
                                     float* const* grad_appearance, void* stream) {
    if (count < 0 || !grad_appearance || (count > 0 && !rows))
        return fail(GS_ERR_ARGUMENT, "gs_unpack_surfel_rows: invalid arguments");
    if (count == 0) return GS_OK;
    SurfelRowTable t = surfel_row_table(neural);
    for (int p = 0; p < t.parts; ++p) {
        if (!grad_appearance[p]) return fail(GS_ERR_ARGUMENT, "gs_unpack_surfel_rows: NULL output");
        t.out[p] = grad_appearance[p];
    }
    unpack_surfel_rows_kernel<<<blocks_for(count * t.first[t.parts]), kPackThreads, 0,
                                as_stream(stream)>>>(count, t, rows);
    GS_CHECK_LAUNCH("unpack_surfel_rows_kernel");
    return GS_OK;
}
