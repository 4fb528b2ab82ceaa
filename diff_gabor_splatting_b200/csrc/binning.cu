// Tile binning: per-tile, depth-ordered record lists.
//
// The reference (rasterize.cu:32-69, 454-493) counts tiles per record, scans,
// emits one 64-bit key (image*tw*th + tile) << 32 | depth_bits per (record, tile)
// in record order, and radix-sorts all I keys over 64 bits (8 passes over 12-byte
// pairs).  The stable sort makes the order within a tile (depth bits, record
// index).
//
// Here the same order is produced with far less traffic:
//   1. stable radix sort of the R records by their 32-bit depth bits (R << I);
//   2. tile counts gathered in that order, inclusive scan, one host read of I
//      (the reference's one synchronisation, rasterize.cu:466-468);
//   3. expansion of every (record, tile) slot in depth order, writing a 32-bit
//      tile id and the record index (8 bytes per slot, coalesced);
//   4. stable radix sort of the slots by tile id over only ceil(log2(tiles)) bits
//      (2 passes for up to 65536 tiles), which keeps the depth order inside each
//      tile;
//   5. tile ranges from the sorted tile ids.
// Result: point_list and ranges identical to the reference's.
#include <cub/cub.cuh>

#include <mutex>

#include "common.cuh"

namespace gs {
namespace {

constexpr int kBinThreads = 256;

inline size_t align_up(size_t v) { return (v + 255) & ~size_t(255); }

struct CountLayout {
    size_t keys_in, keys_out, idx_in, idx_out, counts, offsets, temp, temp_bytes, total;
};

CountLayout count_layout(int64_t R) {
    CountLayout L{};
    size_t sort_bytes = 0, scan_bytes = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, (const uint32_t*)nullptr, (uint32_t*)nullptr,
                                    (const int*)nullptr, (int*)nullptr, int(R), 0, 32);
    cub::DeviceScan::InclusiveSum(nullptr, scan_bytes, (const int64_t*)nullptr, (int64_t*)nullptr,
                                  int(R));
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t at = off; off += align_up(bytes); return at; };
    L.keys_in = take(sizeof(uint32_t) * R);
    L.keys_out = take(sizeof(uint32_t) * R);
    L.idx_in = take(sizeof(int) * R);
    L.idx_out = take(sizeof(int) * R);
    L.counts = take(sizeof(int64_t) * R);
    L.offsets = take(sizeof(int64_t) * R);
    L.temp_bytes = std::max(sort_bytes, scan_bytes);
    L.temp = take(L.temp_bytes);
    L.total = off;
    return L;
}

struct SortLayout {
    size_t keys_in, keys_out, vals_in, owners, temp, temp_bytes, total;
};

int tile_bits(int64_t n_tiles) {
    int bits = 1;
    while ((int64_t(1) << bits) < n_tiles) ++bits;
    return bits;
}

SortLayout sort_layout(int64_t I, int64_t n_tiles) {
    SortLayout L{};
    size_t sort_bytes = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, (const uint32_t*)nullptr, (uint32_t*)nullptr,
                                    (const int*)nullptr, (int*)nullptr, int(I), 0, tile_bits(n_tiles));
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t at = off; off += align_up(bytes); return at; };
    L.keys_in = take(sizeof(uint32_t) * I);
    L.keys_out = take(sizeof(uint32_t) * I);
    L.vals_in = take(sizeof(int) * I);
    L.owners = take(sizeof(int64_t) * ((I + 1023) / 1024 + 1));
    L.temp_bytes = sort_bytes;
    L.temp = take(sort_bytes);
    L.total = off;
    return L;
}

// Tile rectangle of a record.  Plain: the reference's square bounds (tile_rect).
// Tight (GS_BIN_TIGHT, records carrying opacity in slot 17): additionally clipped to the
// tiles that can hold a sample with alpha >= 1/255.  Such a sample has
// o exp(-min(rho3, rho2)/2) >= 1/255, so min(rho3, rho2) <= thr = 2 ln(255 o): it lies
// in the image of the local disc u^2 + v^2 <= thr (an ellipse, bounded by the same
// conic formula the reference uses for its 3-sigma disc, rendering.py:189-196, with 9
// replaced by thr) or within sqrt(thr/2) pixels of the centre (the rho2 branch).  The
// level is widened by 5% + 0.05 and the box by 2 pixels so float rounding of the
// per-pixel test cannot reach outside it; records whose conic is not a bounded ellipse
// keep the plain rectangle.  Images are unchanged; only tiles no sample of the record
// can reach are dropped.
__device__ __forceinline__ int4 bin_rect(const float* g, int radius, int tw, int th, bool tight) {
    const int4 b = tile_rect(g[9], g[10], radius, tw, th);
    if (!tight || b.z <= b.x || b.w <= b.y) return b;
    const double o = g[17];
    if (!(o * 255.0 >= 1.0 - 1e-6)) return make_int4(b.x, b.y, b.x, b.y);   // never accepted
    const double thr = (2.0 * log(255.0 * o)) * 1.05 + 0.05;
    const double t6 = g[6], t7 = g[7], t8 = g[8];
    const double den = thr * (t6 * t6 + t7 * t7) - t8 * t8;
    if (!(den < 0.0)) return b;
    const double fa = thr / den, fc = -1.0 / den;
    const double cx = fa * (g[0] * t6 + g[1] * t7) + fc * g[2] * t8;
    const double cy = fa * (g[3] * t6 + g[4] * t7) + fc * g[5] * t8;
    const double ex2 = cx * cx - (fa * (double(g[0]) * g[0] + double(g[1]) * g[1]) + fc * double(g[2]) * g[2]);
    const double ey2 = cy * cy - (fa * (double(g[3]) * g[3] + double(g[4]) * g[4]) + fc * double(g[5]) * g[5]);
    if (!(ex2 >= 0.0 && ey2 >= 0.0)) return b;
    const double ex = sqrt(ex2), ey = sqrt(ey2), rd = sqrt(fmax(thr * 0.5, 0.0));
    const double x0 = fmin(cx - ex, g[9] - rd) - 2.0, x1 = fmax(cx + ex, g[9] + rd) + 2.0;
    const double y0 = fmin(cy - ey, g[10] - rd) - 2.0, y1 = fmax(cy + ey, g[10] + rd) + 2.0;
    if (!(isfinite(x0) && isfinite(x1) && isfinite(y0) && isfinite(y1))) return b;
    const double lim = 1e9;   // far outside any image; keeps the int conversion defined
    const int tx0 = int(floor(fmin(fmax(x0, -lim), lim) / kTile));
    const int tx1 = int(floor(fmin(fmax(x1, -lim), lim) / kTile)) + 1;
    const int ty0 = int(floor(fmin(fmax(y0, -lim), lim) / kTile));
    const int ty1 = int(floor(fmin(fmax(y1, -lim), lim) / kTile)) + 1;
    int4 c = make_int4(max(b.x, tx0), max(b.y, ty0), min(b.z, tx1), min(b.w, ty1));
    if (c.z <= c.x || c.w <= c.y) c = make_int4(b.x, b.y, b.x, b.y);
    return c;
}

// Depth sort keys: the 32 bits of the record's centre depth T[2][2] (record slot 8),
// the low half of the reference's key (rasterize.cu:52-53).
__global__ void depth_keys_kernel(int64_t R, const float* __restrict__ records, int stride,
                                  const int* __restrict__ radii, uint32_t* __restrict__ keys,
                                  int* __restrict__ idx) {
    const int64_t r = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (r >= R) return;
    keys[r] = radii[r] > 0 ? __float_as_uint(records[r * stride + 8]) : 0xffffffffu;
    idx[r] = int(r);
}

__global__ void tile_counts_kernel(int64_t R, const float* __restrict__ records, int stride,
                                   const int* __restrict__ radii, const int* __restrict__ order,
                                   int tw, int th, bool tight, int64_t* __restrict__ counts) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= R) return;
    const int r = order[i];
    const int radius = radii[r];
    if (radius <= 0) { counts[i] = 0; return; }
    const int4 b = bin_rect(records + int64_t(r) * stride, radius, tw, th, tight);
    counts[i] = int64_t(b.z - b.x) * (b.w - b.y);
}

// Expansion of (record, tile) slots in depth order.  A block owns 1024 consecutive
// slots: two threads find the first and last owning record (binary search of the
// inclusive offsets in global memory), the block stages those records' offsets and
// tile rectangles in shared memory, and each slot finds its owner there (10 shared
// steps instead of ~21 dependent global loads per slot).  Writes are coalesced.
constexpr int kExpandItems = 4;
constexpr int kExpandSlots = kBinThreads * kExpandItems;

__device__ __forceinline__ int64_t first_above(const int64_t* __restrict__ offsets, int64_t n,
                                               int64_t value) {
    int64_t lo = 0, hi = n - 1;   // first j with offsets[j] > value (offsets[n-1] > value)
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (offsets[mid] > value) hi = mid; else lo = mid + 1;
    }
    return lo;
}

// first_owner[b] = the record (in depth order) owning slot b * kExpandSlots: each
// record writes the entries of the blocks whose first slot falls in its slot range.
__global__ void first_owner_kernel(int64_t R, int64_t blocks, const int64_t* __restrict__ offsets,
                                   int64_t* __restrict__ first_owner) {
    const int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (j >= R) return;
    const int64_t begin = j ? offsets[j - 1] : 0, end = offsets[j];
    for (int64_t b = (begin + kExpandSlots - 1) / kExpandSlots; b * kExpandSlots < end && b < blocks;
         ++b)
        first_owner[b] = j;
}

__global__ __launch_bounds__(kBinThreads) void expand_kernel(
    int64_t I, int64_t R, const int64_t* __restrict__ offsets, const int* __restrict__ order,
    const float* __restrict__ records, int stride, const int* __restrict__ radii,
    const int64_t* __restrict__ image_ids, int64_t per_image, int tw, int th, bool tight,
    const int64_t* __restrict__ first_owner, uint32_t* __restrict__ tile_keys,
    int* __restrict__ values) {
    __shared__ int64_t s_end[kExpandSlots];
    __shared__ int4 s_rect[kExpandSlots];    // x0, y0, width, record
    __shared__ uint32_t s_base[kExpandSlots];   // image * tw * th
    __shared__ int64_t s_first, s_last;
    const int64_t i0 = int64_t(blockIdx.x) * kExpandSlots;
    const int64_t i1 = min(i0 + kExpandSlots, I) - 1;
    if (threadIdx.x == 0) s_first = first_owner[blockIdx.x];
    if (threadIdx.x == 32) {
        // an upper bound on the owner of the block's last slot, from the next block's
        // first owner (extra empty records in the range are harmless to the search)
        if (i1 + 1 < I) {
            const int64_t next = first_owner[blockIdx.x + 1];
            s_last = next > 0 && offsets[next - 1] > i1 ? next - 1 : next;
        } else {
            s_last = first_above(offsets, R, i1);
        }
    }
    __syncthreads();
    const int64_t first = s_first;
    const int64_t owners = s_last - first + 1;
    if (owners <= kExpandSlots) {
        for (int t = threadIdx.x; t < owners; t += blockDim.x) {
            const int64_t j = first + t;
            s_end[t] = offsets[j];
            const int r = order[j];
            const int4 b = bin_rect(records + int64_t(r) * stride, radii[r], tw, th, tight);
            s_rect[t] = make_int4(b.x, b.y, max(b.z - b.x, 1), r);
            const int64_t image = image_ids ? image_ids[r] : r / per_image;
            s_base[t] = uint32_t(image * tw * th);
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kExpandItems; ++k) {
            const int64_t i = i0 + k * kBinThreads + threadIdx.x;
            if (i > i1) break;
            int lo = 0, hi = int(owners) - 1;
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                if (s_end[mid] > i) hi = mid; else lo = mid + 1;
            }
            const int64_t start = lo ? s_end[lo - 1] : (first ? offsets[first - 1] : 0);
            const int local = int(i - start);
            const int4 b = s_rect[lo];
            tile_keys[i] = s_base[lo] + uint32_t((b.y + local / b.z) * tw + b.x + local % b.z);
            values[i] = b.w;
        }
        return;
    }
    // many empty owners in range (only possible with caller-made records whose
    // radius is positive but whose tile rectangle is empty): per-slot global search
#pragma unroll 1
    for (int k = 0; k < kExpandItems; ++k) {
        const int64_t i = i0 + k * kBinThreads + threadIdx.x;
        if (i > i1) break;
        const int64_t j = first_above(offsets, R, i);
        const int r = order[j];
        const int64_t start = j ? offsets[j - 1] : 0;
        const int64_t local = i - start;
        const int4 b = bin_rect(records + int64_t(r) * stride, radii[r], tw, th, tight);
        const int w = b.z - b.x;
        const int64_t image = image_ids ? image_ids[r] : r / per_image;
        tile_keys[i] = uint32_t(image * tw * th + int64_t(b.y + int(local / w)) * tw + b.x +
                                int(local % w));
        values[i] = r;
    }
}

// Tile ranges from the sorted tile ids: a range starts where the id changes.  Each
// thread reads four consecutive ids with one 16-byte load plus the id before them.
constexpr int kRangeItems = 4;

__global__ void ranges_kernel(int64_t I, const uint32_t* __restrict__ keys, int2* __restrict__ ranges) {
    const int64_t i0 = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * kRangeItems;
    if (i0 >= I) return;
    uint32_t t[kRangeItems + 1];
    t[0] = i0 ? keys[i0 - 1] : 0xffffffffu;
    if (i0 + kRangeItems <= I) {
        const uint4 v = *reinterpret_cast<const uint4*>(keys + i0);
        t[1] = v.x; t[2] = v.y; t[3] = v.z; t[4] = v.w;
    } else {
#pragma unroll
        for (int k = 0; k < kRangeItems; ++k) t[k + 1] = i0 + k < I ? keys[i0 + k] : 0xffffffffu;
    }
#pragma unroll
    for (int k = 0; k < kRangeItems; ++k) {
        const int64_t i = i0 + k;
        if (i >= I) break;
        if (t[k + 1] != t[k]) {
            ranges[t[k + 1]].x = int(i);
            if (i0 + k > 0) ranges[t[k]].y = int(i);
        }
    }
    if (i0 + kRangeItems >= I) {   // the thread holding the last id closes its range
        const int64_t last = I - 1;
        ranges[keys[last]].y = int(I);
    }
}

unsigned blocks_for(int64_t n) { return unsigned((n + kBinThreads - 1) / kBinThreads); }

int check_common(const char* fn, const float* records, int stride, const int32_t* radii,
                 int64_t R, int64_t per_image, int64_t images, int width, int height) {
    if (!records && R > 0) return fail(GS_ERR_ARGUMENT, std::string(fn) + ": records is NULL");
    if (!radii && R > 0) return fail(GS_ERR_ARGUMENT, std::string(fn) + ": radii is NULL");
    if (stride < 11) return fail(GS_ERR_ARGUMENT, std::string(fn) + ": record stride below 11");
    if (R < 0 || images < 1 || width < 1 || height < 1 || per_image < 0)
        return fail(GS_ERR_ARGUMENT, std::string(fn) + ": invalid sizes");
    if (R > INT_MAX) return fail(GS_ERR_LIMIT, std::string(fn) + ": too many projected primitives");
    const int64_t tw = (width + kTile - 1) / kTile, th = (height + kTile - 1) / kTile;
    if (images * tw * th > INT_MAX)
        return fail(GS_ERR_LIMIT, std::string(fn) + ": image tile count exceeds int32");
    return GS_OK;
}

}  // namespace
}  // namespace gs

using namespace gs;

extern "C" int gs_bin_count_workspace(int64_t records, size_t* bytes) {
    if (records < 0 || !bytes) return fail(GS_ERR_ARGUMENT, "gs_bin_count_workspace: invalid arguments");
    if (records > INT_MAX) return fail(GS_ERR_LIMIT, "gs_bin_count_workspace: too many projected primitives");
    *bytes = records ? count_layout(records).total : 0;
    return GS_OK;
}

extern "C" int gs_bin_count(const float* records, int record_stride, const int32_t* radii,
                            const int64_t* image_ids, int64_t R, int64_t records_per_image,
                            int64_t images, int width, int height, int flags, void* workspace1,
                            size_t workspace1_bytes, int64_t* intersections, void* stream) {
    int st = check_common("gs_bin_count", records, record_stride, radii, R, records_per_image,
                          images, width, height);
    if (st) return st;
    const bool tight = flags & GS_BIN_TIGHT;
    if (tight && record_stride < 18)
        return fail(GS_ERR_ARGUMENT, "gs_bin_count: GS_BIN_TIGHT needs opacity in record slot 17");
    if (!intersections) return fail(GS_ERR_ARGUMENT, "gs_bin_count: intersections is NULL");
    *intersections = 0;
    if (R == 0) return GS_OK;
    if (!image_ids && records_per_image < 1)
        return fail(GS_ERR_ARGUMENT, "gs_bin_count: records_per_image must be positive without image_ids");
    const CountLayout L = count_layout(R);
    if (!workspace1 || workspace1_bytes < L.total)
        return fail(GS_ERR_WORKSPACE, "gs_bin_count: workspace too small");
    auto* base = static_cast<char*>(workspace1);
    auto* keys_in = reinterpret_cast<uint32_t*>(base + L.keys_in);
    auto* keys_out = reinterpret_cast<uint32_t*>(base + L.keys_out);
    auto* idx_in = reinterpret_cast<int*>(base + L.idx_in);
    auto* idx_out = reinterpret_cast<int*>(base + L.idx_out);
    auto* counts = reinterpret_cast<int64_t*>(base + L.counts);
    auto* offsets = reinterpret_cast<int64_t*>(base + L.offsets);
    void* temp = base + L.temp;
    auto s = as_stream(stream);
    const int tw = (width + kTile - 1) / kTile, th = (height + kTile - 1) / kTile;
    depth_keys_kernel<<<blocks_for(R), kBinThreads, 0, s>>>(R, records, record_stride, radii,
                                                            keys_in, idx_in);
    GS_CHECK_LAUNCH("depth_keys_kernel");
    size_t temp_bytes = L.temp_bytes;
    GS_CUDA(cub::DeviceRadixSort::SortPairs(temp, temp_bytes, keys_in, keys_out, idx_in, idx_out,
                                            int(R), 0, 32, s));
    tile_counts_kernel<<<blocks_for(R), kBinThreads, 0, s>>>(R, records, record_stride, radii,
                                                             idx_out, tw, th, tight, counts);
    GS_CHECK_LAUNCH("tile_counts_kernel");
    temp_bytes = L.temp_bytes;
    GS_CUDA(cub::DeviceScan::InclusiveSum(temp, temp_bytes, counts, offsets, int(R), s));
    int64_t total = 0;
    GS_CUDA(cudaMemcpyAsync(&total, offsets + R - 1, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
    GS_CUDA(cudaStreamSynchronize(s));
    *intersections = total;
    if (total > INT_MAX)
        return fail(GS_ERR_LIMIT, "gs_bin_count: tile intersection count exceeds int32");
    return GS_OK;
}

extern "C" int gs_bin_sort_workspace(int64_t records, int64_t intersections, int64_t images,
                                     int width, int height, size_t* bytes) {
    if (!bytes || records < 0 || intersections < 0 || images < 1 || width < 1 || height < 1)
        return fail(GS_ERR_ARGUMENT, "gs_bin_sort_workspace: invalid arguments");
    if (intersections > INT_MAX)
        return fail(GS_ERR_LIMIT, "gs_bin_sort_workspace: tile intersection count exceeds int32");
    const int64_t tw = (width + kTile - 1) / kTile, th = (height + kTile - 1) / kTile;
    *bytes = intersections ? sort_layout(intersections, images * tw * th).total : 0;
    return GS_OK;
}

extern "C" int gs_bin_sort(const float* records, int record_stride, const int32_t* radii,
                           const int64_t* image_ids, int64_t R, int64_t records_per_image,
                           int64_t images, int width, int height, int flags, const void* workspace1,
                           size_t workspace1_bytes, void* workspace2, size_t workspace2_bytes,
                           int64_t I, int32_t* point_list, int32_t* ranges, void* stream) {
    int st = check_common("gs_bin_sort", records, record_stride, radii, R, records_per_image,
                          images, width, height);
    if (st) return st;
    const bool tight = flags & GS_BIN_TIGHT;
    if (tight && record_stride < 18)
        return fail(GS_ERR_ARGUMENT, "gs_bin_sort: GS_BIN_TIGHT needs opacity in record slot 17");
    if (I < 0 || I > INT_MAX) return fail(GS_ERR_LIMIT, "gs_bin_sort: tile intersection count exceeds int32");
    if (!ranges) return fail(GS_ERR_ARGUMENT, "gs_bin_sort: ranges is NULL");
    const int tw = (width + kTile - 1) / kTile, th = (height + kTile - 1) / kTile;
    const int64_t n_tiles = images * tw * th;
    auto s = as_stream(stream);
    GS_CUDA(cudaMemsetAsync(ranges, 0, sizeof(int2) * n_tiles, s));
    if (I == 0 || R == 0) return GS_OK;
    if (!point_list) return fail(GS_ERR_ARGUMENT, "gs_bin_sort: point_list is NULL");
    const CountLayout C = count_layout(R);
    if (!workspace1 || workspace1_bytes < C.total)
        return fail(GS_ERR_WORKSPACE, "gs_bin_sort: workspace 1 too small");
    const SortLayout L = sort_layout(I, n_tiles);
    if (!workspace2 || workspace2_bytes < L.total)
        return fail(GS_ERR_WORKSPACE, "gs_bin_sort: workspace 2 too small");
    const auto* base1 = static_cast<const char*>(workspace1);
    const auto* order = reinterpret_cast<const int*>(base1 + C.idx_out);
    const auto* offsets = reinterpret_cast<const int64_t*>(base1 + C.offsets);
    auto* base = static_cast<char*>(workspace2);
    auto* keys_in = reinterpret_cast<uint32_t*>(base + L.keys_in);
    auto* keys_out = reinterpret_cast<uint32_t*>(base + L.keys_out);
    auto* vals_in = reinterpret_cast<int*>(base + L.vals_in);
    auto* owners = reinterpret_cast<int64_t*>(base + L.owners);
    void* temp = base + L.temp;
    const int64_t expand_blocks = (I + kExpandSlots - 1) / kExpandSlots;
    first_owner_kernel<<<blocks_for(R), kBinThreads, 0, s>>>(R, expand_blocks, offsets, owners);
    GS_CHECK_LAUNCH("first_owner_kernel");
    expand_kernel<<<unsigned(expand_blocks), kBinThreads, 0, s>>>(
        I, R, offsets, order, records, record_stride, radii, image_ids, records_per_image, tw, th,
        tight, owners, keys_in, vals_in);
    GS_CHECK_LAUNCH("expand_kernel");
    size_t temp_bytes = L.temp_bytes;
    GS_CUDA(cub::DeviceRadixSort::SortPairs(temp, temp_bytes, keys_in, keys_out, vals_in, point_list,
                                            int(I), 0, tile_bits(n_tiles), s));
    ranges_kernel<<<blocks_for((I + kRangeItems - 1) / kRangeItems), kBinThreads, 0, s>>>(
        I, keys_out, reinterpret_cast<int2*>(ranges));
    GS_CHECK_LAUNCH("ranges_kernel");
    return GS_OK;
}

// ------------------------------------------------------------------------------
// gs_bin_static: binning without any allocation.
//
// Some callers cannot allocate device memory at the moment they need binning: a
// renderer embedded in a host application whose allocator owns every device byte
// (game-engine or DCC plugins with a fixed memory budget), code that runs while a
// CUDA stream is being captured into a graph (cudaMalloc is not permitted during
// capture), or real-time loops that forbid allocation after start-up.  For them the
// two workspaces of gs_bin_count/gs_bin_sort live in one file-scope device array,
// which every GPU that loads this library holds (32 MiB) until the process exits.
// ------------------------------------------------------------------------------
namespace gs {
namespace {

constexpr int64_t kStaticMaxRecords = 65536;
constexpr int64_t kStaticMaxIntersections = int64_t(1) << 20;
constexpr size_t kStaticScratchBytes = size_t(32) << 20;

static __device__ __align__(256) unsigned char g_bin_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_address[kMaxDevices] = {};

// Device address of g_bin_scratch on the current device, looked up once per device.
int static_scratch(void** out) {
    int device = 0;
    GS_CUDA(cudaGetDevice(&device));
    if (device < 0 || device >= kMaxDevices)
        return fail(GS_ERR_LIMIT, "gs_bin_static: device ordinal beyond 63");
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_address[device]) {
        void* address = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&address, g_bin_scratch);
        if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(g_bin_scratch)");
        g_scratch_address[device] = address;
    }
    *out = g_scratch_address[device];
    return GS_OK;
}

}  // namespace
}  // namespace gs

extern "C" int gs_bin_static(const float* records, int record_stride, const int32_t* radii,
                             const int64_t* image_ids, int64_t records_count,
                             int64_t records_per_image, int64_t images, int width, int height,
                             int32_t* point_list, int64_t point_list_capacity, int32_t* ranges,
                             int64_t* intersections, void* stream) {
    if (!intersections) return fail(GS_ERR_ARGUMENT, "gs_bin_static: intersections is NULL");
    *intersections = 0;
    if (records_count > kStaticMaxRecords)
        return fail(GS_ERR_LIMIT, "gs_bin_static: more than 65536 records (the static scratch "
                                  "limit); use gs_bin_count/gs_bin_sort with caller workspaces");
    int st = check_common("gs_bin_static", records, record_stride, radii, records_count,
                          records_per_image, images, width, height);
    if (st) return st;
    void* scratch = nullptr;
    st = static_scratch(&scratch);
    if (st) return st;
    size_t bytes1 = 0;
    st = gs_bin_count_workspace(records_count, &bytes1);
    if (st) return st;
    bytes1 = align_up(bytes1);
    if (bytes1 > kStaticScratchBytes)
        return fail(GS_ERR_LIMIT, "gs_bin_static: count workspace exceeds the static scratch");
    int64_t total = 0;
    st = gs_bin_count(records, record_stride, radii, image_ids, records_count, records_per_image,
                      images, width, height, 0, scratch, bytes1, &total, stream);
    if (st) return st;
    *intersections = total;
    if (total > kStaticMaxIntersections)
        return fail(GS_ERR_LIMIT, "gs_bin_static: more than 1048576 tile intersections (the "
                                  "static scratch limit)");
    if (total > point_list_capacity)
        return fail(GS_ERR_ARGUMENT, "gs_bin_static: point_list capacity is below the "
                                     "intersection count returned in *intersections");
    size_t bytes2 = 0;
    st = gs_bin_sort_workspace(records_count, total, images, width, height, &bytes2);
    if (st) return st;
    if (bytes1 + bytes2 > kStaticScratchBytes)
        return fail(GS_ERR_LIMIT, "gs_bin_static: sort workspace exceeds the static scratch");
    return gs_bin_sort(records, record_stride, radii, image_ids, records_count, records_per_image,
                       images, width, height, 0, scratch, bytes1,
                       static_cast<char*>(scratch) + bytes1, bytes2, total, point_list, ranges,
                       stream);
}
