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
//   2. per record, in that order, its tiles as row spans (one span per tile row it
//      reaches) and their counts; inclusive scans of slots and spans; one host read
//      of the totals (the reference's one synchronisation, rasterize.cu:466-468);
//   3. images up to kRowMaxColumns tiles wide (the row path): the spans written out as
//      (tile row, packed span) pairs, stably sorted by tile row, and the tile lists
//      assembled per chunk of a row's spans (counts per column, a scan over the row's
//      chunks, ranked writes straight to the point list) -- no per-slot sort at all;
//   4. wider images and arena mode (the slot path): the spans written with their
//      first slot and first tile, every (record, tile) slot expanded in depth order
//      (32-bit tile id + record), stably sorted by tile id over only
//      ceil(log2(tiles)) bits, which keeps the depth order inside each tile, and tile
//      ranges from the sorted ids.
// With the reference's rectangles (flags 0) point_list and ranges are identical to
// the reference's.  GS_BIN_TIGHT keeps, per tile row, only the tiles a sample with
// alpha >= 1/255 can reach (see record_region): same images, shorter lists.
#include <cub/cub.cuh>

#include <mutex>

#include "common.cuh"

namespace gs {
namespace {

constexpr int kBinThreads = 256;

inline size_t align_up(size_t v) { return (v + 255) & ~size_t(255); }

struct CountLayout {
    size_t keys_in, keys_out, idx_in, idx_out, slots, slot_end, spans, span_end, temp, temp_bytes,
        total;
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
    L.slots = take(sizeof(int64_t) * R);
    L.slot_end = take(sizeof(int64_t) * R);
    L.spans = take(sizeof(int64_t) * R);
    L.span_end = take(sizeof(int64_t) * R);
    L.temp_bytes = std::max(sort_bytes, scan_bytes);
    L.temp = take(L.temp_bytes);
    L.total = off;
    return L;
}

struct SortLayout {
    size_t item_end, item_tile, item_record, owners, keys_in, keys_out, vals_in, temp, temp_bytes,
        total;
};

int tile_bits(int64_t n_tiles) {
    int bits = 1;
    while ((int64_t(1) << bits) < n_tiles) ++bits;
    return bits;
}

constexpr int kExpandItems = 4;
constexpr int kExpandSlots = kBinThreads * kExpandItems;

SortLayout sort_layout(int64_t I, int64_t spans, int64_t n_tiles) {
    SortLayout L{};
    size_t sort_bytes = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, (const uint32_t*)nullptr, (uint32_t*)nullptr,
                                    (const int*)nullptr, (int*)nullptr, int(I), 0, tile_bits(n_tiles));
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t at = off; off += align_up(bytes); return at; };
    L.item_end = take(sizeof(int64_t) * spans);
    L.item_tile = take(sizeof(uint32_t) * spans);
    L.item_record = take(sizeof(int) * spans);
    L.owners = take(sizeof(int64_t) * ((I + kExpandSlots - 1) / kExpandSlots + 1));
    L.keys_in = take(sizeof(uint32_t) * I);
    L.keys_out = take(sizeof(uint32_t) * I);
    L.vals_in = take(sizeof(int) * I);
    L.temp_bytes = sort_bytes;
    L.temp = take(sort_bytes);
    L.total = off;
    return L;
}

// The tiles of one record, row by row.  rect is the reference's square tile bounds
// (tile_rect).  Tight regions (GS_BIN_TIGHT; opacity in record slot 17) keep per tile
// row only the tiles a sample with alpha >= 1/255 can reach.  Such a sample has
// o exp(-min(rho3, rho2)/2) >= 1/255, so min(rho3, rho2) <= thr = 2 ln(255 o): it lies in
// the image of the local disc u^2 + v^2 <= thr -- an ellipse, the same conic the
// reference bounds for its 3-sigma disc (rendering.py:189-196) with 9 replaced by thr
// -- or within sqrt(thr/2) pixels of the centre (the rho2 branch).  The level is widened
// by 5% + 0.05, so float rounding in the per-pixel test cannot reach a dropped tile.
//
// The conic is set up per record in double (its adjugate cancels badly in float) and
// reduced to centred form: with Y = y - cy, the boundary is x = cx + a Y -/+ sqrt(p Y^2
// + q) (p < 0 < q), its leftmost point at Y = yl and its rightmost at -yl, its height
// |Y| <= ey.  Per row band, the x-range of the convex region is taken where its
// boundary is extreme: at yl (or -yl) clamped into the band.  The rows evaluate that in
// single precision with every operation's rounding explicit (no contraction), so the
// counting and writing passes get identical rows; each range is widened by `margin` =
// 2 pixels plus a bound on the float error of that evaluation (and each band by a bound
// on the error of Y, so no row the double evaluation keeps is lost).  Records whose conic is
// not a bounded ellipse, or whose centred form does not fit float, keep full rows.
struct Region {
    int4 rect;            // [x0, y0, x1, y1) tiles
    int exact;            // per-row spans from the ellipse and disc
    float cx, cy;         // ellipse centre
    float a, p, q;        // boundary x = cx + a Y -/+ sqrt(p Y^2 + q)
    float yl, ey;         // Y of the leftmost point; half height
    float margin;         // pixels added on both sides of each row's range
    float dcx, dcy, rd;   // low-pass disc
    float yerr;           // bound on the float error of Y, added to both band edges
};   // 72 bytes: a warp reading the fields of different records spreads over the banks

// Reads the record's T (slots 0-8), centre (9-10) and, for tight regions, opacity (17).
// Records come in depth order, one scattered 80-byte row per lane: rows of at least 20
// floats on 16-byte boundaries are read with four 16-byte loads (each one L2 sector)
// instead of twelve 4-byte ones (one sector each, the L1 keeping few of them).
__device__ __noinline__ void record_region(const float* records, int64_t r, int stride,
                                           int radius, int tw, int th, bool tight,
                                           Region* out) {
    float g[18];
    const float* row = records + r * stride;
    const bool vector_rows =
        stride >= 20 && stride % 4 == 0 && (reinterpret_cast<uintptr_t>(records) & 15u) == 0;
    if (vector_rows) {
        const float4* q = reinterpret_cast<const float4*>(row);
        const float4 a = __ldg(q), b = __ldg(q + 1), c = __ldg(q + 2), d = __ldg(q + 4);
        g[0] = a.x; g[1] = a.y; g[2] = a.z; g[3] = a.w;
        g[4] = b.x; g[5] = b.y; g[6] = b.z; g[7] = b.w;
        g[8] = c.x; g[9] = c.y; g[10] = c.z;
        g[17] = d.y;
    } else {
#pragma unroll
        for (int k = 0; k < 11; ++k) g[k] = row[k];
    }
    Region R;
    R.rect = tile_rect(g[9], g[10], radius, tw, th);
    R.exact = 0;
    const int4 b = R.rect;
    if (!tight || b.z <= b.x || b.w <= b.y) { *out = R; return; }
    if (!vector_rows) g[17] = row[17];   // the opacity, read only for tight regions
    const double o = g[17];
    if (!(o * 255.0 >= 1.0 - 1e-6)) {   // alpha <= o < 1/255: never accepted
        R.rect = make_int4(b.x, b.y, b.x, b.y);
        *out = R;
        return;
    }
    // the level's 5% widening dwarfs the single-precision logarithm's error
    const double thr = double(2.f * __logf(255.f * g[17])) * 1.05 + 0.05;
    double T[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) T[k] = g[k];
    // dual conic C = T diag(thr, thr, -1) T^T
    auto dual = [&](int i, int j) {
        return thr * (T[3 * i] * T[3 * j] + T[3 * i + 1] * T[3 * j + 1]) - T[3 * i + 2] * T[3 * j + 2];
    };
    const double c00 = dual(0, 0), c01 = dual(0, 1), c02 = dual(0, 2), c11 = dual(1, 1),
                 c12 = dual(1, 2), c22 = dual(2, 2);
    *out = R;
    if (!(c22 < 0.0)) return;   // not a bounded ellipse in front of the camera
    const double inv22 = 1.0 / c22;
    const double cx = c02 * inv22, cy = c12 * inv22;   // centre: pole of the line at infinity
    // primal conic: adjugate of the dual, signed so the interior is negative
    double m00 = c11 * c22 - c12 * c12, m01 = c02 * c12 - c01 * c22, m02 = c01 * c12 - c02 * c11;
    double m11 = c00 * c22 - c02 * c02, m12 = c01 * c02 - c00 * c12, m22 = c00 * c11 - c01 * c01;
    double k = m00 * cx * cx + 2 * m01 * cx * cy + 2 * m02 * cx + m11 * cy * cy + 2 * m12 * cy + m22;
    if (k > 0) { m00 = -m00; m01 = -m01; m11 = -m11; k = -k; }
    if (!(m00 > 0.0)) return;
    // m00 X^2 + 2 m01 X Y + m11 Y^2 + k = 0 solved for X
    const double inv00 = 1.0 / m00;
    const double a = -m01 * inv00;
    const double pd = (m01 * m01 - m00 * m11) * (inv00 * inv00), qd = -k * inv00;
    if (!(pd < 0.0 && qd > 0.0)) return;
    const double inv_p = 1.0 / pd;
    const double ey = sqrt(-qd * inv_p);
    const double yl = -a * sqrt(qd * inv_p / (pd - a * a));
    // Float error of a row's evaluation, each term at least twice its bound: Y = y - cy
    // is off by at most 2^-24 (|cy| + |Y|) < ey_err; D = p Y^2 + q by 2^-22 q from the
    // roundings of p, q, p Y and the fma, plus 2 |p Y| ey_err <= 2 (q / ey) ey_err, and
    // near the tips (D ~ 0) sqrt(D) inherits sqrt of that whole; a Y + cx and the final
    // sums add relative errors of their magnitudes.
    const double ey_err = 0x1p-23 * (fabs(cy) + ey + 64.0);
    const double margin = 2.0 + 0x1p-10 * sqrt(qd) + sqrt(4.0 * (qd / ey) * ey_err) +
                          2.0 * fabs(a) * ey_err + 0x1p-20 * (fabs(cx) + fabs(a) * (fabs(cy) + ey));
    R.cx = float(cx); R.cy = float(cy);
    R.a = float(a); R.p = float(pd); R.q = float(qd);
    R.yl = float(yl); R.ey = float(ey);
    R.margin = float(margin);
    R.yerr = float(2.0 * ey_err);
    R.dcx = g[9]; R.dcy = g[10]; R.rd = float(sqrt(fmax(thr * 0.5, 0.0)));
    const float all = R.cx + R.cy + R.a + R.p + R.q + R.yl + R.ey + R.margin + R.rd + R.yerr;
    if (!isfinite(all) || !(R.p < 0.f) || !(R.q > 0.f)) return;
    R.exact = 1;
    *out = R;
}

// Tiles [x0, x1) of tile row ty (x1 <= x0: none).
__device__ __forceinline__ int2 row_span(const Region& R, int ty) {
    if (!R.exact) return make_int2(R.rect.x, R.rect.z);
    const float y0 = float(ty * kTile - 2), y1 = float(ty * kTile + kTile + 1);
    float lo = INFINITY, hi = -INFINITY;
    const float ya = fmaxf(__fsub_rn(__fsub_rn(y0, R.cy), R.yerr), -R.ey);
    const float yb = fminf(__fadd_rn(__fsub_rn(y1, R.cy), R.yerr), R.ey);
    if (ya <= yb) {
        float y = fminf(fmaxf(R.yl, ya), yb);
        float d = fmaxf(__fmaf_rn(__fmul_rn(R.p, y), y, R.q), 0.f);
        lo = __fsub_rn(__fmaf_rn(R.a, y, R.cx), __fsqrt_rn(d));
        y = fminf(fmaxf(-R.yl, ya), yb);
        d = fmaxf(__fmaf_rn(__fmul_rn(R.p, y), y, R.q), 0.f);
        hi = __fadd_rn(__fmaf_rn(R.a, y, R.cx), __fsqrt_rn(d));
    }
    const float dy = fmaxf(fmaxf(__fsub_rn(y0, R.dcy), __fsub_rn(R.dcy, y1)), 0.f);
    if (dy <= R.rd) {
        const float hw = __fsqrt_rn(__fmaf_rn(-dy, dy, __fmul_rn(R.rd, R.rd)));
        lo = fminf(lo, __fsub_rn(R.dcx, hw));
        hi = fmaxf(hi, __fadd_rn(R.dcx, hw));
    }
    if (!(lo <= hi)) return make_int2(R.rect.x, R.rect.x);
    const float lim = 1e9f;
    const int x0 = int(floorf(__fmul_rn(fminf(fmaxf(__fsub_rn(lo, R.margin), -lim), lim), 1.f / kTile)));
    const int x1 = int(floorf(__fmul_rn(fminf(fmaxf(__fadd_rn(hi, R.margin), -lim), lim), 1.f / kTile))) + 1;
    return make_int2(max(R.rect.x, x0), min(R.rect.z, x1));
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

// Write each record's spans (depth order) with their end slot (inclusive scan value),
// first tile id and record (the slot path).
__global__ void spans_kernel(int64_t R, const float* __restrict__ records, int stride,
                             const int* __restrict__ radii, const int* __restrict__ order,
                             const int64_t* __restrict__ slot_end,
                             const int64_t* __restrict__ span_end,
                             const int64_t* __restrict__ image_ids, int64_t per_image, int tw,
                             int th, bool tight, const int64_t* __restrict__ limits,
                             int64_t* __restrict__ item_end, uint32_t* __restrict__ item_tile,
                             int* __restrict__ item_record) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= R || (limits && limits[1] == 0)) return;   // arena overflow: no spans
    const int64_t first_span = i ? span_end[i - 1] : 0;
    if (span_end[i] == first_span) return;
    const int r = order[i];
    int64_t slot = i ? slot_end[i - 1] : 0;
    int64_t k = first_span;
    Region G;
    record_region(records, r, stride, radii[r], tw, th, tight, &G);
    const int64_t image = image_ids ? image_ids[r] : r / per_image;
    const uint32_t base = uint32_t(image * tw * th);
    for (int ty = G.rect.y; ty < G.rect.w; ++ty) {
        const int2 sp = row_span(G, ty);
        if (sp.y <= sp.x) continue;
        slot += sp.y - sp.x;
        item_end[k] = slot;
        item_tile[k] = base + uint32_t(ty * tw + sp.x);
        item_record[k] = r;
        ++k;
    }
}

// A span packed for the row sort: first column (16 bits), tile count (16 bits), record.
__device__ __forceinline__ uint64_t pack_span(int x0, int len, int record) {
    return uint64_t(uint32_t(x0) | uint32_t(len) << 16) | uint64_t(uint32_t(record)) << 32;
}

// Per record (depth order): tiles (slots) and non-empty tile rows (spans), and the row
// path's span writer, load-balanced for tight regions, whose rows each cost an exact
// double-precision evaluation: a warp takes 32
// consecutive records (depth order), each lane sets up its record's region and parks it
// in shared memory, and the warp's lanes then evaluate the 32 records' tile rows as one
// list, 32 rows at a time, so a record with many rows no longer idles the other lanes.
// A row's record is the last lane whose first row index is not past it.
constexpr int kBalancedWarps = kBinThreads / 32;

struct BalancedShared {
    Region region[kBalancedWarps][32];
    int first[kBalancedWarps][33];      // exclusive prefix of the lanes' row counts
    int slots[kBalancedWarps][32];      // per record: tiles, non-empty rows (counting)
    int spans[kBalancedWarps][32];
    int64_t out[kBalancedWarps][32];    // per record: next span index (writing)
    int64_t end[kBalancedWarps][32];    // per record: end of its span range
    uint32_t row_base[kBalancedWarps][32];   // per record: image * th
    int record[kBalancedWarps][32];
};

__device__ __forceinline__ int owner_lane(const int* first, int t) {
    int lo = 0;
#pragma unroll
    for (int step = 16; step >= 1; step >>= 1)
        if (first[lo + step] <= t) lo += step;
    return lo;
}

__global__ __launch_bounds__(kBinThreads, 4) void tile_counts_balanced_kernel(
    int64_t R, const float* __restrict__ records, int stride, const int* __restrict__ radii,
    const int* __restrict__ order, int tw, int th, bool tight, int64_t* __restrict__ slots,
    int64_t* __restrict__ spans) {
    __shared__ BalancedShared sh;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    int rows = 0;
    int64_t n_slots = 0, n_spans = 0;
    if (i < R) {
        const int r = order[i];
        const int radius = radii[r];
        if (radius > 0) {
            Region& G = sh.region[warp][lane];
            record_region(records, r, stride, radius, tw, th, tight, &G);
            if (G.rect.z > G.rect.x) {
                if (G.exact) {
                    rows = max(G.rect.w - G.rect.y, 0);
                } else {
                    n_spans = G.rect.w - G.rect.y;
                    n_slots = n_spans * (G.rect.z - G.rect.x);
                }
            }
        }
    }
    int incl = rows;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    int* first = sh.first[warp];
    first[lane] = incl - rows;
    if (lane == 31) first[32] = incl;
    sh.slots[warp][lane] = 0;
    sh.spans[warp][lane] = 0;
    __syncwarp();
    const int total = first[32];
    for (int t = lane; t < total; t += 32) {
        const int o = owner_lane(first, t);
        const Region& G = sh.region[warp][o];
        const int2 sp = row_span(G, G.rect.y + (t - first[o]));
        if (sp.y > sp.x) {
            atomicAdd(&sh.slots[warp][o], sp.y - sp.x);
            atomicAdd(&sh.spans[warp][o], 1);
        }
    }
    __syncwarp();
    if (i >= R) return;
    if (rows) {
        n_slots = sh.slots[warp][lane];
        n_spans = sh.spans[warp][lane];
    }
    slots[i] = n_slots;
    spans[i] = n_spans;
}

// Row-path spans (as spans_kernel<true>), balanced: a row's output index is its record's
// first span plus the non-empty rows before it, counted across passes per record and
// within a pass with a ballot over the lanes holding rows of the same record.
__global__ __launch_bounds__(kBinThreads, 4) void spans_rows_balanced_kernel(
    int64_t R, const float* __restrict__ records, int stride, const int* __restrict__ radii,
    const int* __restrict__ order, const int64_t* __restrict__ span_end,
    const int64_t* __restrict__ image_ids, int64_t per_image, int tw, int th, bool tight,
    uint32_t* __restrict__ row_keys, uint64_t* __restrict__ row_spans) {
    __shared__ BalancedShared sh;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    int rows = 0;
    if (i < R) {
        const int64_t first_span = i ? span_end[i - 1] : 0;
        if (span_end[i] != first_span) {
            const int r = order[i];
            Region& G = sh.region[warp][lane];
            record_region(records, r, stride, radii[r], tw, th, tight, &G);
            rows = max(G.rect.w - G.rect.y, 0);
            sh.out[warp][lane] = first_span;
            sh.end[warp][lane] = span_end[i];
            const int64_t image = image_ids ? image_ids[r] : r / per_image;
            sh.row_base[warp][lane] = uint32_t(image * th);
            sh.record[warp][lane] = r;
        }
    }
    int incl = rows;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    int* first = sh.first[warp];
    first[lane] = incl - rows;
    if (lane == 31) first[32] = incl;
    __syncwarp();
    const int total = first[32];
    const unsigned below = (1u << lane) - 1u;
    for (int t0 = 0; t0 < total; t0 += 32) {
        const int t = t0 + lane;
        const bool live = t < total;
        int o = 0;
        int2 sp = make_int2(0, 0);
        if (live) {
            o = owner_lane(first, t);
            const Region& G = sh.region[warp][o];
            sp = row_span(G, G.rect.y + (t - first[o]));
        }
        const bool keep = live && sp.y > sp.x;
        const unsigned same = __match_any_sync(0xffffffffu, live ? o : -1);
        const unsigned kept = __ballot_sync(0xffffffffu, keep) & same;
        const int64_t k = keep ? sh.out[warp][o] + __popc(kept & below) : 0;
        if (keep && k < sh.end[warp][o]) {   // the count pass's range, which the rows match
            const int ty = sh.region[warp][o].rect.y + (t - first[o]);
            row_keys[k] = sh.row_base[warp][o] + uint32_t(ty);
            row_spans[k] = pack_span(sp.x, sp.y - sp.x, sh.record[warp][o]);
        }
        __syncwarp();
        // the group's highest lane moves its record's next index past this pass's rows
        if (live && (same >> lane) == 1u) sh.out[warp][o] += __popc(kept);
        __syncwarp();
    }
}

// first_owner[b] = the span owning slot b * kExpandSlots: each span writes the entries
// of the blocks whose first slot falls in its slot range.
// limits (arena mode, else NULL): device [intersections, spans] of this binning, zero
// when they exceed the arena; I and S are then the arena capacities.
__global__ void first_owner_kernel(int64_t S, int64_t blocks, const int64_t* __restrict__ limits,
                                   const int64_t* __restrict__ item_end,
                                   int64_t* __restrict__ first_owner) {
    const int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (limits) {
        S = limits[1];
        blocks = (limits[0] + kExpandSlots - 1) / kExpandSlots;
    }
    if (j >= S) return;
    const int64_t begin = j ? item_end[j - 1] : 0, end = item_end[j];
    for (int64_t b = (begin + kExpandSlots - 1) / kExpandSlots; b * kExpandSlots < end && b < blocks;
         ++b)
        first_owner[b] = j;
}

// Expansion of (record, tile) slots in depth order.  A block owns 1024 consecutive
// slots and the spans covering them (at most 1024: every span holds a slot); it stages
// their end slots, first tiles and records in shared memory, and each slot finds its
// span by a shared binary search.  Writes are coalesced.
// Arena mode (limits non-NULL): I is the arena capacity; slots from the live count up to
// it get the last tile's id as a pad key, which the stable tile sort keeps behind every
// real entry of that tile, past the live count the ranges are built from.
__global__ __launch_bounds__(kBinThreads) void expand_kernel(
    int64_t I, int64_t S, const int64_t* __restrict__ limits, uint32_t pad_key,
    const int64_t* __restrict__ item_end, const uint32_t* __restrict__ item_tile,
    const int* __restrict__ item_record, const int64_t* __restrict__ first_owner,
    uint32_t* __restrict__ tile_keys, int* __restrict__ values) {
    __shared__ int64_t s_end[kExpandSlots];
    __shared__ uint32_t s_tile[kExpandSlots];
    __shared__ int s_record[kExpandSlots];
    __shared__ int64_t s_first, s_last;
    const int64_t i0 = int64_t(blockIdx.x) * kExpandSlots;
    if (limits) {
        const int64_t capacity = I;
        I = limits[0];
        S = limits[1];
        for (int64_t i = max(i0, I) + threadIdx.x; i < min(i0 + kExpandSlots, capacity);
             i += kBinThreads) {
            tile_keys[i] = pad_key;
            values[i] = -1;
        }
        if (i0 >= I) return;
    }
    const int64_t i1 = min(i0 + kExpandSlots, I) - 1;
    if (threadIdx.x == 0) s_first = first_owner[blockIdx.x];
    if (threadIdx.x == 32) {
        if (i1 + 1 < I) {   // owner of the last slot, from the next block's first owner
            const int64_t next = first_owner[blockIdx.x + 1];
            s_last = next > 0 && item_end[next - 1] > i1 ? next - 1 : next;
        } else {
            s_last = S - 1;
        }
    }
    __syncthreads();
    const int64_t first = s_first;
    const int owners = int(s_last - first + 1);
    for (int t = threadIdx.x; t < owners; t += blockDim.x) {
        s_end[t] = item_end[first + t];
        s_tile[t] = item_tile[first + t];
        s_record[t] = item_record[first + t];
    }
    const int64_t first_start = first ? item_end[first - 1] : 0;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kExpandItems; ++k) {
        const int64_t i = i0 + k * kBinThreads + threadIdx.x;
        if (i > i1) break;
        int lo = 0, hi = owners - 1;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (s_end[mid] > i) hi = mid; else lo = mid + 1;
        }
        const int64_t start = lo ? s_end[lo - 1] : first_start;
        tile_keys[i] = s_tile[lo] + uint32_t(i - start);
        values[i] = s_record[lo];
    }
}

// Tile ranges from the sorted tile ids: a range starts where the id changes.  Each
// thread reads four consecutive ids with one 16-byte load plus the id before them.
constexpr int kRangeItems = 4;

__global__ void ranges_kernel(int64_t I, const int64_t* __restrict__ limits,
                              const uint32_t* __restrict__ keys, int2* __restrict__ ranges) {
    if (limits) I = limits[0];   // arena: the live entries lead the sorted keys
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

// ------------------------------------------------------------------------------
// Tile lists from row spans, without sorting the slots.
//
// Every (record, tile) slot belongs to one row span (a record's tiles in one tile row),
// and the spans come out of spans_kernel in depth order.  A stable sort of the S spans
// by tile row (S is several times smaller than the slot count I) leaves each row's
// spans in depth order; then, per chunk of kRowChunk consecutive spans of one row, a
// warp counts the spans covering each tile column, an exclusive scan over a row's
// chunks gives every chunk its starting position in each tile, and the warp writes its
// spans' records at those positions with ranks taken in span order.  The lists are the
// stable tile sort's lists exactly: within a tile, records in depth order.
// ------------------------------------------------------------------------------
constexpr int kRowChunk = 64;         // spans per chunk (one warp)
constexpr int kRowWarps = 4;          // warps (chunks) per block
constexpr int kRowMaxColumns = 1024;  // tile columns this path handles (wider: slot sort)

inline bool rows_path(int tw) { return tw <= kRowMaxColumns; }

struct RowLayout {
    size_t keys_in, keys_out, idx_in, idx_out, row_first, row_end, chunk_base, chunk_row,
        chunk_counts, chunk_prefix, tile_count, tile_start, temp, temp_bytes, total;
    int64_t rows, chunks_cap;
};

RowLayout row_layout(int64_t spans, int64_t images, int tw, int th) {
    RowLayout L{};
    L.rows = images * th;
    L.chunks_cap = spans / kRowChunk + L.rows + 1;
    const int64_t n_tiles = images * tw * th;
    size_t sort_bytes = 0, scan_rows = 0, scan_tiles = 0;
    cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, (const uint32_t*)nullptr, (uint32_t*)nullptr,
                                    (const uint64_t*)nullptr, (uint64_t*)nullptr, int(spans), 0,
                                    tile_bits(L.rows));
    cub::DeviceScan::InclusiveSum(nullptr, scan_rows, (const int*)nullptr, (int*)nullptr,
                                  int(L.rows));
    cub::DeviceScan::ExclusiveSum(nullptr, scan_tiles, (const int*)nullptr, (int*)nullptr,
                                  int(n_tiles));
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t at = off; off += align_up(bytes); return at; };
    L.keys_in = take(sizeof(uint32_t) * spans);
    L.keys_out = take(sizeof(uint32_t) * spans);
    L.idx_in = take(sizeof(uint64_t) * spans);
    L.idx_out = take(sizeof(uint64_t) * spans);
    L.row_first = take(sizeof(int) * L.rows);
    L.row_end = take(sizeof(int) * L.rows);
    L.chunk_base = take(sizeof(int) * (L.rows + 1));
    L.chunk_row = take(sizeof(int) * L.chunks_cap);
    L.chunk_counts = take(sizeof(int) * L.chunks_cap * tw);
    L.chunk_prefix = take(sizeof(int) * L.chunks_cap * tw);
    L.tile_count = take(sizeof(int) * n_tiles);
    L.tile_start = take(sizeof(int) * n_tiles);
    L.temp_bytes = std::max(sort_bytes, std::max(scan_rows, scan_tiles));
    L.temp = take(L.temp_bytes);
    L.total = off;
    return L;
}

__device__ __forceinline__ void unpack_span(uint64_t v, int& x0, int& x1, int& record) {
    x0 = int(v & 0xffffu);
    x1 = x0 + int((v >> 16) & 0xffffu);
    record = int(v >> 32);
}

// [row_first, row_end) of each tile row in the row-sorted span list (both zeroed first).
// Four keys per thread, read with one 16-byte load when the key array is 16-byte
// aligned (it starts 256 bytes into the caller's workspace; scalar loads otherwise),
// plus its two neighbours; each bound is written by the one thread whose keys hold the
// row change.
constexpr int kBoundKeys = 4;

__global__ void row_bounds_kernel(int64_t S, const uint32_t* __restrict__ rows,
                                  int* __restrict__ row_first, int* __restrict__ row_end) {
    const int64_t k0 = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * kBoundKeys;
    if (k0 >= S) return;
    uint32_t r[kBoundKeys + 2];   // keys k0-1 .. k0+4 (0xffffffff outside the list)
    if (k0 + kBoundKeys <= S && (reinterpret_cast<uintptr_t>(rows) & 15u) == 0u) {
        const uint4 q = *reinterpret_cast<const uint4*>(rows + k0);
        r[1] = q.x; r[2] = q.y; r[3] = q.z; r[4] = q.w;
    } else {
#pragma unroll
        for (int i = 0; i < kBoundKeys; ++i) r[1 + i] = k0 + i < S ? rows[k0 + i] : 0xffffffffu;
    }
    r[0] = k0 > 0 ? rows[k0 - 1] : 0xffffffffu;
    r[kBoundKeys + 1] = k0 + kBoundKeys < S ? rows[k0 + kBoundKeys] : 0xffffffffu;
#pragma unroll
    for (int i = 0; i < kBoundKeys; ++i) {
        const int64_t k = k0 + i;
        if (k >= S) break;
        if (r[i] != r[i + 1]) row_first[r[i + 1]] = int(k);
        if (r[i + 2] != r[i + 1]) row_end[r[i + 1]] = int(k + 1);
    }
}

// chunks of each row, into chunk_base[1 + row] (inclusive-scanned afterwards)
__global__ void row_chunks_kernel(int64_t rows, const int* __restrict__ row_first,
                                  const int* __restrict__ row_end, int* __restrict__ chunks) {
    const int64_t r = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    chunks[r] = (row_end[r] - row_first[r] + kRowChunk - 1) / kRowChunk;
}

// chunk_row[c] = the row of chunk c, one warp per row writing its chunks' entries
__global__ void chunk_rows_kernel(int64_t rows, const int* __restrict__ chunk_base,
                                  int* __restrict__ chunk_row) {
    const int64_t r = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    for (int c = chunk_base[r] + lane; c < chunk_base[r + 1]; c += 32) chunk_row[c] = int(r);
}

struct RowChunk {
    int row, begin, end;   // spans [begin, end) of the row-sorted list
};

// The chunk of a global chunk id (false past the last chunk).
__device__ __forceinline__ bool row_chunk(int64_t chunk, int64_t rows,
                                          const int* __restrict__ chunk_base,
                                          const int* __restrict__ chunk_row,
                                          const int* __restrict__ row_first,
                                          const int* __restrict__ row_end, RowChunk& c) {
    if (chunk >= chunk_base[rows]) return false;
    const int row = chunk_row[chunk];
    c.row = row;
    c.begin = row_first[row] + int(chunk - chunk_base[row]) * kRowChunk;
    c.end = min(c.begin + kRowChunk, row_end[row]);
    return true;
}

// Per chunk: how many of its spans cover each tile column (warp-private counters).
__global__ __launch_bounds__(kRowWarps * 32) void row_count_kernel(
    int64_t rows, int tw, const int* __restrict__ chunk_base, const int* __restrict__ chunk_row,
    const int* __restrict__ row_first, const int* __restrict__ row_end,
    const uint64_t* __restrict__ spans_by_row, int* __restrict__ chunk_counts) {
    extern __shared__ int row_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int* count = row_smem + warp * tw;
    RowChunk c;
    const int64_t chunk = int64_t(blockIdx.x) * kRowWarps + warp;
    if (!row_chunk(chunk, rows, chunk_base, chunk_row, row_first, row_end, c)) return;
    for (int x = lane; x < tw; x += 32) count[x] = 0;
    __syncwarp();
    for (int g = c.begin + lane; g < c.end; g += 32) {
        int x0, x1, record;
        unpack_span(spans_by_row[g], x0, x1, record);
        for (int x = x0; x < x1; ++x) atomicAdd(count + x, 1);
    }
    __syncwarp();
    for (int x = lane; x < tw; x += 32) chunk_counts[chunk * tw + x] = count[x];
}

// Per (row, column): exclusive scan of the chunk counts over the row's chunks; the
// total is the tile's entry count.
__global__ void row_scan_kernel(int64_t rows, int tw, const int* __restrict__ chunk_base,
                                const int* __restrict__ chunk_counts,
                                int* __restrict__ chunk_prefix, int* __restrict__ tile_count) {
    const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= rows * tw) return;
    const int64_t row = t / tw, x = t % tw;
    int sum = 0;
    const int64_t end = chunk_base[row + 1];
    int64_t c = chunk_base[row];
    // eight chunks' counts loaded at once, so the walk waits on memory once per eight
    for (; c + 8 <= end; c += 8) {
        int n[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) n[k] = chunk_counts[(c + k) * tw + x];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            chunk_prefix[(c + k) * tw + x] = sum;
            sum += n[k];
        }
    }
    for (; c < end; ++c) {
        chunk_prefix[c * tw + x] = sum;
        sum += chunk_counts[c * tw + x];
    }
    tile_count[t] = sum;
}

__global__ void tile_ranges_kernel(int64_t n_tiles, const int* __restrict__ tile_count,
                                   const int* __restrict__ tile_start, int2* __restrict__ ranges) {
    const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= n_tiles) return;
    const int n = tile_count[t];
    ranges[t] = n ? make_int2(tile_start[t], tile_start[t] + n) : make_int2(0, 0);
}

// Per chunk: write each span's record into every tile it covers.  Lanes take 32 spans
// at a time in list (depth) order; a tile's rank among them is the number of lower
// lanes covering it (a per-column lane mask built with shared atomics), so the order
// within a tile follows the list whatever the lanes' timing.  Each slot is written
// straight to the point list (a column's slots of one chunk are adjacent there); with
// only two tile-wide arrays of shared memory per warp the kernel keeps most of an SM's
// warps resident, which hides the latency of its scattered writes.
__device__ __forceinline__ void rank_group(int x0, int x1, unsigned* lanes, int lane) {
    for (int x = x0; x < x1; ++x) atomicOr(lanes + x, 1u << lane);
    __syncwarp();
}

__device__ __forceinline__ void advance_group(int x0, int x1, unsigned* lanes, int* cursor,
                                              unsigned below) {
    __syncwarp();
    for (int x = x0; x < x1; ++x)   // the lowest covering lane advances the column
        if ((lanes[x] & below) == 0u) cursor[x] += __popc(lanes[x]);
    __syncwarp();
    for (int x = x0; x < x1; ++x) lanes[x] = 0u;
    __syncwarp();
}

__global__ __launch_bounds__(kRowWarps * 32) void row_write_kernel(
    int64_t rows, int tw, const int* __restrict__ chunk_base, const int* __restrict__ chunk_row,
    const int* __restrict__ row_first, const int* __restrict__ row_end,
    const uint64_t* __restrict__ spans_by_row, const int* __restrict__ chunk_prefix,
    const int* __restrict__ tile_start, int* __restrict__ point_list) {
    extern __shared__ int row_smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int* cursor = row_smem + warp * 2 * tw;   // next point-list position of each column
    unsigned* lanes = reinterpret_cast<unsigned*>(cursor + tw);
    RowChunk c;
    const int64_t chunk = int64_t(blockIdx.x) * kRowWarps + warp;
    if (!row_chunk(chunk, rows, chunk_base, chunk_row, row_first, row_end, c)) return;
    const unsigned below = (1u << lane) - 1u;
    for (int x = lane; x < tw; x += 32) {
        cursor[x] = tile_start[int64_t(c.row) * tw + x] + chunk_prefix[chunk * tw + x];
        lanes[x] = 0u;
    }
    __syncwarp();
    for (int g0 = c.begin; g0 < c.end; g0 += 32) {
        const int g = g0 + lane;
        int x0 = 0, x1 = 0, record = 0;
        if (g < c.end) unpack_span(spans_by_row[g], x0, x1, record);
        rank_group(x0, x1, lanes, lane);
        for (int x = x0; x < x1; ++x) point_list[cursor[x] + __popc(lanes[x] & below)] = record;
        advance_group(x0, x1, lanes, cursor, below);
    }
}

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

namespace gs {
namespace {

// Depth pre-sort, per-record tile and span counts, and their inclusive scans, into
// workspace 1 (asynchronous: the totals stay on the device at slot_end/span_end[R-1]).
int count_phase(const char* fn, const float* records, int record_stride, const int32_t* radii,
                int64_t R, bool tight, int width, int height, void* workspace1,
                size_t workspace1_bytes, cudaStream_t s) {
    const CountLayout L = count_layout(R);
    if (!workspace1 || workspace1_bytes < L.total)
        return fail(GS_ERR_WORKSPACE, std::string(fn) + ": workspace too small");
    auto* base = static_cast<char*>(workspace1);
    auto* keys_in = reinterpret_cast<uint32_t*>(base + L.keys_in);
    auto* keys_out = reinterpret_cast<uint32_t*>(base + L.keys_out);
    auto* idx_in = reinterpret_cast<int*>(base + L.idx_in);
    auto* idx_out = reinterpret_cast<int*>(base + L.idx_out);
    auto* slots = reinterpret_cast<int64_t*>(base + L.slots);
    auto* slot_end = reinterpret_cast<int64_t*>(base + L.slot_end);
    auto* n_spans = reinterpret_cast<int64_t*>(base + L.spans);
    auto* span_end = reinterpret_cast<int64_t*>(base + L.span_end);
    void* temp = base + L.temp;
    const int tw = (width + kTile - 1) / kTile, th = (height + kTile - 1) / kTile;
    depth_keys_kernel<<<blocks_for(R), kBinThreads, 0, s>>>(R, records, record_stride, radii,
                                                            keys_in, idx_in);
    GS_CHECK_LAUNCH("depth_keys_kernel");
    size_t temp_bytes = L.temp_bytes;
    GS_CUDA(cub::DeviceRadixSort::SortPairs(temp, temp_bytes, keys_in, keys_out, idx_in, idx_out,
                                            int(R), 0, 32, s));
    tile_counts_balanced_kernel<<<blocks_for(R), kBinThreads, 0, s>>>(
        R, records, record_stride, radii, idx_out, tw, th, tight, slots, n_spans);
    GS_CHECK_LAUNCH("tile_counts_balanced_kernel");
    temp_bytes = L.temp_bytes;
    GS_CUDA(cub::DeviceScan::InclusiveSum(temp, temp_bytes, slots, slot_end, int(R), s));
    temp_bytes = L.temp_bytes;
    GS_CUDA(cub::DeviceScan::InclusiveSum(temp, temp_bytes, n_spans, span_end, int(R), s));
    return GS_OK;
}

// Spans, first-owner table, expansion, tile sort and ranges into workspace 2,
// point_list and ranges.  I and S are the intersection and span counts, or with
// `limits` (arena mode) the arena capacities, the live counts being read on the device.
int sort_phase(const float* records, int record_stride, const int32_t* radii,
               const int64_t* image_ids, int64_t R, int64_t records_per_image, int64_t images,
               int width, int height, bool tight, const void* workspace1, void* workspace2,
               int64_t I, int64_t spans, const int64_t* limits, int32_t* point_list,
               int32_t* ranges, cudaStream_t s) {
    const int tw = (width + kTile - 1) / kTile, th = (height + kTile - 1) / kTile;
    const int64_t n_tiles = images * tw * th;
    const CountLayout C = count_layout(R);
    const SortLayout L = sort_layout(I, spans, n_tiles);
    const auto* base1 = static_cast<const char*>(workspace1);
    const auto* order = reinterpret_cast<const int*>(base1 + C.idx_out);
    const auto* slot_end = reinterpret_cast<const int64_t*>(base1 + C.slot_end);
    const auto* span_end = reinterpret_cast<const int64_t*>(base1 + C.span_end);
    auto* base = static_cast<char*>(workspace2);
    auto* item_end = reinterpret_cast<int64_t*>(base + L.item_end);
    auto* item_tile = reinterpret_cast<uint32_t*>(base + L.item_tile);
    auto* item_record = reinterpret_cast<int*>(base + L.item_record);
    auto* owners = reinterpret_cast<int64_t*>(base + L.owners);
    auto* keys_in = reinterpret_cast<uint32_t*>(base + L.keys_in);
    auto* keys_out = reinterpret_cast<uint32_t*>(base + L.keys_out);
    auto* vals_in = reinterpret_cast<int*>(base + L.vals_in);
    void* temp = base + L.temp;
    spans_kernel<<<blocks_for(R), kBinThreads, 0, s>>>(R, records, record_stride, radii, order,
                                                       slot_end, span_end, image_ids,
                                                       records_per_image, tw, th, tight, limits,
                                                       item_end, item_tile, item_record);
    GS_CHECK_LAUNCH("spans_kernel");
    const int64_t expand_blocks = (I + kExpandSlots - 1) / kExpandSlots;
    first_owner_kernel<<<blocks_for(spans), kBinThreads, 0, s>>>(spans, expand_blocks, limits,
                                                                 item_end, owners);
    GS_CHECK_LAUNCH("first_owner_kernel");
    expand_kernel<<<unsigned(expand_blocks), kBinThreads, 0, s>>>(
        I, spans, limits, uint32_t(n_tiles - 1), item_end, item_tile, item_record, owners, keys_in,
        vals_in);
    GS_CHECK_LAUNCH("expand_kernel");
    size_t temp_bytes = L.temp_bytes;
    GS_CUDA(cub::DeviceRadixSort::SortPairs(temp, temp_bytes, keys_in, keys_out, vals_in, point_list,
                                            int(I), 0, tile_bits(n_tiles), s));
    ranges_kernel<<<blocks_for((I + kRangeItems - 1) / kRangeItems), kBinThreads, 0, s>>>(
        I, limits, keys_out, reinterpret_cast<int2*>(ranges));
    GS_CHECK_LAUNCH("ranges_kernel");
    return GS_OK;
}

// gs_bin_sort's path for images up to kRowMaxColumns tiles wide: spans, then tile lists
// from the row-sorted spans (row_count / row_scan / row_write) instead of the slot
// expansion and the slot sort.
int sort_phase_rows(const float* records, int record_stride, const int32_t* radii,
                    const int64_t* image_ids, int64_t R, int64_t records_per_image,
                    int64_t images, int width, int height, bool tight, const void* workspace1,
                    void* workspace2, int64_t I, int64_t S, int32_t* point_list, int32_t* ranges,
                    cudaStream_t s) {
    const int tw = (width + kTile - 1) / kTile, th = (height + kTile - 1) / kTile;
    const int64_t n_tiles = images * tw * th;
    const CountLayout C = count_layout(R);
    const RowLayout L = row_layout(S, images, tw, th);
    const auto* base1 = static_cast<const char*>(workspace1);
    const auto* order = reinterpret_cast<const int*>(base1 + C.idx_out);
    const auto* span_end = reinterpret_cast<const int64_t*>(base1 + C.span_end);
    auto* base = static_cast<char*>(workspace2);
    auto* keys_in = reinterpret_cast<uint32_t*>(base + L.keys_in);
    auto* keys_out = reinterpret_cast<uint32_t*>(base + L.keys_out);
    auto* idx_in = reinterpret_cast<uint64_t*>(base + L.idx_in);
    auto* idx_out = reinterpret_cast<uint64_t*>(base + L.idx_out);
    auto* row_first = reinterpret_cast<int*>(base + L.row_first);
    auto* row_end = reinterpret_cast<int*>(base + L.row_end);
    auto* chunk_base = reinterpret_cast<int*>(base + L.chunk_base);
    auto* chunk_counts = reinterpret_cast<int*>(base + L.chunk_counts);
    auto* tile_count = reinterpret_cast<int*>(base + L.tile_count);
    auto* tile_start = reinterpret_cast<int*>(base + L.tile_start);
    void* temp = base + L.temp;
    spans_rows_balanced_kernel<<<blocks_for(R), kBinThreads, 0, s>>>(
        R, records, record_stride, radii, order, span_end, image_ids, records_per_image, tw, th,
        tight, keys_in, idx_in);
    GS_CHECK_LAUNCH("spans_rows_balanced_kernel");
    size_t temp_bytes = L.temp_bytes;
    GS_CUDA(cub::DeviceRadixSort::SortPairs(temp, temp_bytes, keys_in, keys_out, idx_in, idx_out,
                                            int(S), 0, tile_bits(L.rows), s));
    GS_CUDA(cudaMemsetAsync(row_first, 0, sizeof(int) * L.rows, s));
    GS_CUDA(cudaMemsetAsync(row_end, 0, sizeof(int) * L.rows, s));
    row_bounds_kernel<<<blocks_for((S + kBoundKeys - 1) / kBoundKeys), kBinThreads, 0, s>>>(
        S, keys_out, row_first, row_end);
    GS_CHECK_LAUNCH("row_bounds_kernel");
    // chunks per row (staged in tile_count), inclusive-scanned into chunk_base[1..rows]
    row_chunks_kernel<<<blocks_for(L.rows), kBinThreads, 0, s>>>(L.rows, row_first, row_end,
                                                                 tile_count);
    GS_CHECK_LAUNCH("row_chunks_kernel");
    GS_CUDA(cudaMemsetAsync(chunk_base, 0, sizeof(int), s));
    temp_bytes = L.temp_bytes;
    GS_CUDA(cub::DeviceScan::InclusiveSum(temp, temp_bytes, tile_count, chunk_base + 1,
                                          int(L.rows), s));
    const unsigned chunk_blocks = unsigned((L.chunks_cap + kRowWarps - 1) / kRowWarps);
    const size_t count_smem = sizeof(int) * kRowWarps * tw;
    auto* chunk_row = reinterpret_cast<int*>(base + L.chunk_row);
    chunk_rows_kernel<<<blocks_for(L.rows * 32), kBinThreads, 0, s>>>(L.rows, chunk_base, chunk_row);
    GS_CHECK_LAUNCH("chunk_rows_kernel");
    row_count_kernel<<<chunk_blocks, kRowWarps * 32, count_smem, s>>>(
        L.rows, tw, chunk_base, chunk_row, row_first, row_end, idx_out, chunk_counts);
    GS_CHECK_LAUNCH("row_count_kernel");
    auto* chunk_prefix = reinterpret_cast<int*>(base + L.chunk_prefix);
    row_scan_kernel<<<blocks_for(L.rows * tw), kBinThreads, 0, s>>>(
        L.rows, tw, chunk_base, chunk_counts, chunk_prefix, tile_count);
    GS_CHECK_LAUNCH("row_scan_kernel");
    temp_bytes = L.temp_bytes;
    GS_CUDA(cub::DeviceScan::ExclusiveSum(temp, temp_bytes, tile_count, tile_start, int(n_tiles), s));
    tile_ranges_kernel<<<blocks_for(n_tiles), kBinThreads, 0, s>>>(
        n_tiles, tile_count, tile_start, reinterpret_cast<int2*>(ranges));
    GS_CHECK_LAUNCH("tile_ranges_kernel");
    const size_t write_smem = sizeof(int) * kRowWarps * 2 * tw;   // <= 32 KB (tw <= 1024)
    row_write_kernel<<<chunk_blocks, kRowWarps * 32, write_smem, s>>>(
        L.rows, tw, chunk_base, chunk_row, row_first, row_end, idx_out, chunk_prefix, tile_start,
        point_list);
    GS_CHECK_LAUNCH("row_write_kernel");
    (void)I;
    return GS_OK;
}

// Arena mode: report the live counts and zero them when they exceed the arena.
__global__ void arena_limits_kernel(int64_t R, const int64_t* __restrict__ slot_end,
                                    const int64_t* __restrict__ span_end, int64_t max_slots,
                                    int64_t max_spans, int64_t* __restrict__ totals,
                                    int64_t* __restrict__ limits) {
    const int64_t I = R ? slot_end[R - 1] : 0, S = R ? span_end[R - 1] : 0;
    if (totals) {
        totals[0] = I;
        totals[1] = S;
    }
    const bool fits = I <= max_slots && S <= max_spans;
    limits[0] = fits ? I : 0;
    limits[1] = fits ? S : 0;
}

}  // namespace
}  // namespace gs

extern "C" int gs_bin_count(const float* records, int record_stride, const int32_t* radii,
                            const int64_t* image_ids, int64_t R, int64_t records_per_image,
                            int64_t images, int width, int height, int flags, void* workspace1,
                            size_t workspace1_bytes, int64_t* intersections, int64_t* spans,
                            void* stream) {
    int st = check_common("gs_bin_count", records, record_stride, radii, R, records_per_image,
                          images, width, height);
    if (st) return st;
    const bool tight = flags & GS_BIN_TIGHT;
    if (tight && record_stride < 18)
        return fail(GS_ERR_ARGUMENT, "gs_bin_count: GS_BIN_TIGHT needs opacity in record slot 17");
    if (!intersections || !spans) return fail(GS_ERR_ARGUMENT, "gs_bin_count: NULL output");
    *intersections = 0;
    *spans = 0;
    if (R == 0) return GS_OK;
    if (!image_ids && records_per_image < 1)
        return fail(GS_ERR_ARGUMENT, "gs_bin_count: records_per_image must be positive without image_ids");
    auto s = as_stream(stream);
    st = count_phase("gs_bin_count", records, record_stride, radii, R, tight, width, height,
                     workspace1, workspace1_bytes, s);
    if (st) return st;
    const CountLayout L = count_layout(R);
    const auto* base = static_cast<const char*>(workspace1);
    const auto* slot_end = reinterpret_cast<const int64_t*>(base + L.slot_end);
    const auto* span_end = reinterpret_cast<const int64_t*>(base + L.span_end);
    int64_t totals[2] = {0, 0};
    GS_CUDA(cudaMemcpyAsync(&totals[0], slot_end + R - 1, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
    GS_CUDA(cudaMemcpyAsync(&totals[1], span_end + R - 1, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
    GS_CUDA(cudaStreamSynchronize(s));
    *intersections = totals[0];
    *spans = totals[1];
    if (totals[0] > INT_MAX)
        return fail(GS_ERR_LIMIT, "gs_bin_count: tile intersection count exceeds int32");
    return GS_OK;
}

extern "C" int gs_bin_sort_workspace(int64_t records, int64_t intersections, int64_t spans,
                                     int64_t images, int width, int height, size_t* bytes) {
    if (!bytes || records < 0 || intersections < 0 || spans < 0 || spans > intersections ||
        images < 1 || width < 1 || height < 1)
        return fail(GS_ERR_ARGUMENT, "gs_bin_sort_workspace: invalid arguments");
    if (intersections > INT_MAX)
        return fail(GS_ERR_LIMIT, "gs_bin_sort_workspace: tile intersection count exceeds int32");
    const int64_t tw = (width + kTile - 1) / kTile, th = (height + kTile - 1) / kTile;
    if (!intersections)
        *bytes = 0;
    else if (rows_path(int(tw)))
        *bytes = row_layout(spans, images, int(tw), int(th)).total;
    else
        *bytes = sort_layout(intersections, spans, images * tw * th).total;
    return GS_OK;
}

extern "C" int gs_bin_sort(const float* records, int record_stride, const int32_t* radii,
                           const int64_t* image_ids, int64_t R, int64_t records_per_image,
                           int64_t images, int width, int height, int flags, const void* workspace1,
                           size_t workspace1_bytes, void* workspace2, size_t workspace2_bytes,
                           int64_t I, int64_t spans, int32_t* point_list, int32_t* ranges,
                           void* stream) {
    int st = check_common("gs_bin_sort", records, record_stride, radii, R, records_per_image,
                          images, width, height);
    if (st) return st;
    const bool tight = flags & GS_BIN_TIGHT;
    if (tight && record_stride < 18)
        return fail(GS_ERR_ARGUMENT, "gs_bin_sort: GS_BIN_TIGHT needs opacity in record slot 17");
    if (I < 0 || I > INT_MAX) return fail(GS_ERR_LIMIT, "gs_bin_sort: tile intersection count exceeds int32");
    if (spans < 0 || spans > I || (I > 0 && spans == 0))
        return fail(GS_ERR_ARGUMENT, "gs_bin_sort: span count inconsistent with the intersections");
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
    const size_t needed = rows_path(tw) ? row_layout(spans, images, tw, th).total
                                        : sort_layout(I, spans, n_tiles).total;
    if (!workspace2 || workspace2_bytes < needed)
        return fail(GS_ERR_WORKSPACE, "gs_bin_sort: workspace 2 too small");
    if (rows_path(tw))
        return sort_phase_rows(records, record_stride, radii, image_ids, R, records_per_image,
                               images, width, height, tight, workspace1, workspace2, I, spans,
                               point_list, ranges, s);
    return sort_phase(records, record_stride, radii, image_ids, R, records_per_image, images, width,
                      height, tight, workspace1, workspace2, I, spans, nullptr, point_list, ranges,
                      s);
}

// ------------------------------------------------------------------------------
// gs_bin_arena: binning without a host synchronisation.
//
// gs_bin_count reads the intersection and span counts back to the host to size the
// sort (the reference does the same, rasterize.cu:466-468), which stalls the host and
// keeps a render step out of CUDA graph capture.  Here the caller provides an arena
// sized for at most max_intersections slots and max_spans row spans; every launch is
// sized by those capacities and reads the live counts on the device.  Slots past the
// live count carry a pad key the stable sort keeps at the end.  When a count exceeds
// the arena nothing is binned (all tile ranges empty) and `totals` reports the counts
// needed, for the caller to check after the fact and grow the arena.
// ------------------------------------------------------------------------------
namespace {

struct ArenaLayout {
    size_t count, sort, limits, total;
};

ArenaLayout arena_layout(int64_t R, int64_t max_slots, int64_t max_spans, int64_t n_tiles) {
    ArenaLayout A{};
    A.count = align_up(count_layout(R).total);
    A.sort = align_up(sort_layout(max_slots, max_spans, n_tiles).total);
    A.limits = A.count + A.sort;
    A.total = A.limits + align_up(2 * sizeof(int64_t));
    return A;
}

}  // namespace

extern "C" int gs_bin_arena_workspace(int64_t records, int64_t max_intersections,
                                      int64_t max_spans, int64_t images, int width, int height,
                                      size_t* bytes) {
    if (!bytes || records < 0 || max_intersections < 1 || max_spans < 1 ||
        max_spans > max_intersections || images < 1 || width < 1 || height < 1)
        return fail(GS_ERR_ARGUMENT, "gs_bin_arena_workspace: invalid arguments");
    if (records > INT_MAX) return fail(GS_ERR_LIMIT, "gs_bin_arena_workspace: too many records");
    if (max_intersections > INT_MAX)
        return fail(GS_ERR_LIMIT, "gs_bin_arena_workspace: arena beyond int32 intersections");
    const int64_t tw = (width + kTile - 1) / kTile, th = (height + kTile - 1) / kTile;
    *bytes = arena_layout(records, max_intersections, max_spans, images * tw * th).total;
    return GS_OK;
}

extern "C" int gs_bin_arena(const float* records, int record_stride, const int32_t* radii,
                            const int64_t* image_ids, int64_t R, int64_t records_per_image,
                            int64_t images, int width, int height, int flags, void* workspace,
                            size_t workspace_bytes, int64_t max_intersections, int64_t max_spans,
                            int32_t* point_list, int32_t* ranges, int64_t* totals, void* stream) {
    int st = check_common("gs_bin_arena", records, record_stride, radii, R, records_per_image,
                          images, width, height);
    if (st) return st;
    const bool tight = flags & GS_BIN_TIGHT;
    if (tight && record_stride < 18)
        return fail(GS_ERR_ARGUMENT, "gs_bin_arena: GS_BIN_TIGHT needs opacity in record slot 17");
    if (max_intersections < 1 || max_spans < 1 || max_spans > max_intersections)
        return fail(GS_ERR_ARGUMENT, "gs_bin_arena: invalid arena capacities");
    if (max_intersections > INT_MAX)
        return fail(GS_ERR_LIMIT, "gs_bin_arena: arena beyond int32 intersections");
    if (!ranges || !point_list) return fail(GS_ERR_ARGUMENT, "gs_bin_arena: NULL output");
    if (!image_ids && records_per_image < 1 && R > 0)
        return fail(GS_ERR_ARGUMENT, "gs_bin_arena: records_per_image must be positive without image_ids");
    const int tw = (width + kTile - 1) / kTile, th = (height + kTile - 1) / kTile;
    const int64_t n_tiles = images * tw * th;
    const ArenaLayout A = arena_layout(R, max_intersections, max_spans, n_tiles);
    if (!workspace || workspace_bytes < A.total)
        return fail(GS_ERR_WORKSPACE, "gs_bin_arena: workspace too small");
    auto s = as_stream(stream);
    GS_CUDA(cudaMemsetAsync(ranges, 0, sizeof(int2) * n_tiles, s));
    if (R == 0) {
        if (totals) GS_CUDA(cudaMemsetAsync(totals, 0, 2 * sizeof(int64_t), s));
        return GS_OK;
    }
    char* base = static_cast<char*>(workspace);
    st = count_phase("gs_bin_arena", records, record_stride, radii, R, tight, width, height, base,
                     A.count, s);
    if (st) return st;
    const CountLayout C = count_layout(R);
    auto* limits = reinterpret_cast<int64_t*>(base + A.limits);
    arena_limits_kernel<<<1, 1, 0, s>>>(R, reinterpret_cast<const int64_t*>(base + C.slot_end),
                                        reinterpret_cast<const int64_t*>(base + C.span_end),
                                        max_intersections, max_spans, totals, limits);
    GS_CHECK_LAUNCH("arena_limits_kernel");
    return sort_phase(records, record_stride, radii, image_ids, R, records_per_image, images, width,
                      height, tight, base, base + A.count, max_intersections, max_spans, limits,
                      point_list, ranges, s);
}

// ------------------------------------------------------------------------------
// gs_bin_static: binning without any allocation.
//
// Some callers cannot allocate device memory at the moment they need binning: a
// renderer embedded in a host application whose allocator owns every device byte
// (game-engine or DCC plugins with a fixed memory budget), or a real-time loop that
// forbids allocation after start-up.  For them the two workspaces of
// gs_bin_count/gs_bin_sort live in one file-scope device array, which every GPU that
// loads this library holds (80 MiB) until the process exits.
//
// Limits.  The workspaces grow with the records (count phase), the row spans, the
// tile columns and the tiles (sort phase).  Within kStaticMaxRecords records,
// kStaticMaxIntersections intersections (spans never exceed intersections),
// kStaticMaxColumns tile columns and kStaticMaxTiles tiles over all images, the two
// together stay below kStaticScratchBytes (the sort phase's largest case, 2^20 spans
// over 128 columns, needs about 61 MiB with CUB's temporary storage; the count phase
// 3.5 MiB).  The entry point checks each limit before any work and checks the
// computed workspace sizes again before using the array.
// ------------------------------------------------------------------------------
namespace gs {
namespace {

constexpr int64_t kStaticMaxRecords = 65536;
constexpr int64_t kStaticMaxIntersections = int64_t(1) << 20;
constexpr int64_t kStaticMaxColumns = 128;                 // images up to 2048 px wide
constexpr int64_t kStaticMaxTiles = int64_t(1) << 18;      // 16x16 tiles, all images
constexpr size_t kStaticScratchBytes = size_t(80) << 20;

static __device__ __align__(256) unsigned char g_bin_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_address[kMaxDevices] = {};

// Device address of g_bin_scratch on the current device.  Host code only knows the
// array's host-side stand-in; the device address is looked up once per device (the
// first gs_bin_static call made with that device current) and kept for the process.
// A device reset (cudaDeviceReset) would invalidate the kept address: processes that
// reset a device after using this entry point are not supported.
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
    const int64_t tw = (width + kTile - 1) / kTile, th = (height + kTile - 1) / kTile;
    if (tw > kStaticMaxColumns)
        return fail(GS_ERR_LIMIT, "gs_bin_static: image wider than 2048 pixels (128 tile "
                                  "columns, the static scratch limit)");
    if (images > kStaticMaxTiles / (tw * th) ||
        images * tw * th > kStaticMaxTiles)
        return fail(GS_ERR_LIMIT, "gs_bin_static: more than 262144 tiles over all images "
                                  "(the static scratch limit)");
    void* scratch = nullptr;
    st = static_scratch(&scratch);
    if (st) return st;
    size_t bytes1 = 0;
    st = gs_bin_count_workspace(records_count, &bytes1);
    if (st) return st;
    bytes1 = align_up(bytes1);
    if (bytes1 > kStaticScratchBytes)
        return fail(GS_ERR_LIMIT, "gs_bin_static: count workspace exceeds the static scratch");
    int64_t total = 0, spans = 0;
    st = gs_bin_count(records, record_stride, radii, image_ids, records_count, records_per_image,
                      images, width, height, 0, scratch, bytes1, &total, &spans, stream);
    if (st) return st;
    *intersections = total;
    if (total > kStaticMaxIntersections)
        return fail(GS_ERR_LIMIT, "gs_bin_static: more than 1048576 tile intersections (the "
                                  "static scratch limit)");
    if (total > point_list_capacity)
        return fail(GS_ERR_ARGUMENT, "gs_bin_static: point_list capacity is below the "
                                     "intersection count returned in *intersections");
    size_t bytes2 = 0;
    st = gs_bin_sort_workspace(records_count, total, spans, images, width, height, &bytes2);
    if (st) return st;
    if (bytes1 + bytes2 > kStaticScratchBytes)
        return fail(GS_ERR_LIMIT, "gs_bin_static: sort workspace exceeds the static scratch");
    return gs_bin_sort(records, record_stride, radii, image_ids, records_count, records_per_image,
                       images, width, height, 0, scratch, bytes1,
                       static_cast<char*>(scratch) + bytes1, bytes2, total, spans, point_list,
                       ranges, stream);
}
