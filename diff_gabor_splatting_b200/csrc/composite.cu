// Tile compositor: front-to-back forward and reverse-order backward.
//
// One CTA of 16x16 threads per image tile, one thread per pixel, the tile's
// depth-sorted record list walked in batches staged in shared memory.
//   forward  restates renderForward  (rasterize.cu:229-281) with sampleSurface
//            (:84-103) and appearanceForward (:105-138);
//   backward restates renderBackward (rasterize.cu:283-399) with
//            appearanceBackward (:146-197).
// Per-pixel arithmetic follows the reference expression by expression (same
// operation order, full-precision expf/sinf/cosf), so images agree to rounding.
//
// Differences, all in data movement and in where sums are formed:
//   * records and appearance rows are 80/240-byte aligned rows staged with 16-byte
//     cp.async copies, double-buffered (the next batch lands while the current one is
//     composited; the reference gathers scalars through two levels of indirection,
//     :219-226, between two barriers per batch);
//   * opacity travels inside the record, so no per-primitive opacity gather;
//   * backward gradients of one record are summed across the warp with a
//     shared-memory transpose (every lane stores its fields as a row, every lane sums
//     a column), across the CTA's 8 warps at the flush, and added to global memory
//     once per (tile, record): 8x fewer global atomics than one per warp, and for
//     classic rows one 16-byte vector atomic per four fields;
//   * neural: the gradients of the direction inputs' weights and of the direction
//     are per-record constants times the b1 sums, formed once per (tile, record).
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"

namespace gs {
namespace {

constexpr int kBatch = 64;
constexpr int kClassicRow = GS_CLASSIC_ROW_FLOATS;
constexpr int kNeuralRow = GS_NEURAL_ROW_FLOATS;

struct Params {
    const float4* records;
    const float4* rows;
    int row_mode;
    const int64_t* prim_ids;
    int64_t cameras, surfels;
    const float* backgrounds;
    const int* point_list;
    const int2* ranges;
    int width, height, tw, th;
    float near_plane, far_plane;
    // forward outputs / backward inputs.  The nine maps as five planes: rgb (3
    // channels), alpha, depth, normals (3), distortion; plane g of pixel p starts at
    // out[g] + p * out_px[g] (channels adjacent).  Gradients likewise with a channel
    // stride (0 for a broadcast gradient); a NULL plane is a zero gradient.
    float* out[5];
    int64_t out_px[5];
    float* state;
    int* contributors;
    const float* gin[5];
    int64_t gin_px[5], gin_ch[5];
    // optional median depth (2DGS convention: the depth of the last contribution made
    // while the transmittance before it exceeds 0.5), its list position (1-based within
    // the tile range, 0 for none) and its gradient; NULL when not requested
    float* median;
    int64_t median_px;
    int* median_index;
    const float* gin_median;
    int64_t gin_median_px;
    // selected-pixel mode (NULL groups: whole tiles): one CTA per group of up to 256
    // selected pixels of one tile, groups[b] = (tile, first, count, -); selected pixel
    // i = (x, y, output index, -); outputs and gradients are indexed by output index
    const int4* groups;
    const int4* selected;
    // backward outputs
    float* grad_records;
    float* grad_xy;
    float* grad_rows;
    float* grad_backgrounds;
    // optional work counters: [0] samples tested, [1] contributions accepted
    unsigned long long* counters;
    // optional warp accept masks (NULL: none): plane w of warp_mask_words words holds,
    // for warp w of a tile's CTA, bit p & 31 of word p >> 5 set when a pixel of that
    // warp accepted the record at point-list position p (written by the forward, read
    // by the backward, which skips the records its warp accepted nowhere)
    unsigned* warp_mask;
    int64_t warp_mask_words;
};

constexpr int kMaskWarps = 8;   // warps of a 256-thread tile CTA: planes of a warp mask

// OR the forward's accepted bits of one warp for list positions [p0, p0 + 64) into its
// plane: up to three words, each only when it has a bit set and lies inside the plane.
__device__ __forceinline__ void or_accepted(const Params& P, int warp, int64_t p0,
                                            unsigned lo, unsigned hi) {
    unsigned* plane = P.warp_mask + int64_t(warp) * P.warp_mask_words;
    const uint64_t bits = (uint64_t(hi) << 32) | lo;
    const int64_t w0 = p0 >> 5;
    const int o = int(p0 & 31);
    const unsigned word[3] = {unsigned(bits << o), unsigned((bits << o) >> 32),
                              o ? unsigned(bits >> (64 - o)) : 0u};
#pragma unroll
    for (int k = 0; k < 3; ++k)
        if (word[k] && w0 + k < P.warp_mask_words) atomicOr(plane + w0 + k, word[k]);
}

// Each warp of a tile CTA composites an 8x4 block of the 16x16 tile (warps 0-1 the top
// two blocks, and so on).  A splat covers a compact patch of a tile, which touches fewer
// 8x4 blocks than 16x2 rows: fewer warps run a record's accept path with most lanes
// idle (measured: config 3 compositors 61.6 -> 56.8 ms, config 1 19.0 -> 18.3 ms).
constexpr int kWarpW = 8, kWarpH = 4, kWarpBlocksX = kTile / kWarpW;

// The pixel a thread composites: in tile mode pixel (x, y) of tile blockIdx.x from the
// warp's block and the lane's place in it, output index (image H + y) W + x; in
// selected-pixel mode the rank-th pixel of group blockIdx.x (threads past the group's
// count are outside).
struct PixelSlot {
    int tile, image, x, y;
    int64_t pixel;
    bool inside;
};

__device__ __forceinline__ PixelSlot pixel_slot(const Params& P, int rank) {
    PixelSlot q;
    const int tiles_per_image = P.tw * P.th;
    if (P.groups) {
        const int4 group = P.groups[blockIdx.x];
        q.tile = group.x;
        q.image = q.tile / tiles_per_image;
        q.inside = rank < group.z;
        const int4 sel = P.selected[group.y + (q.inside ? rank : 0)];
        q.x = sel.x;
        q.y = sel.y;
        q.pixel = sel.z;
    } else {
        q.tile = blockIdx.x;
        q.image = q.tile / tiles_per_image;
        const int local = q.tile % tiles_per_image;
        const int lane = rank & 31, warp = rank >> 5;
        q.x = (local % P.tw) * kTile + (warp % kWarpBlocksX) * kWarpW + lane % kWarpW;
        q.y = (local / P.tw) * kTile + (warp / kWarpBlocksX) * kWarpH + lane / kWarpW;
        q.inside = q.x < P.width && q.y < P.height;
        q.pixel = (int64_t(q.image) * P.height + q.y) * P.width + q.x;
    }
    return q;
}

// First map channel and channel count of plane g (rgb, alpha, depth, normals, distortion).
__host__ __device__ constexpr int plane_first(int g) {
    return g == 0 ? 0 : g == 1 ? 3 : g == 2 ? 4 : g == 3 ? 5 : 8;
}
__host__ __device__ constexpr int plane_size(int g) { return g == 0 || g == 3 ? 3 : 1; }

// Add this thread's counts into the block total and then into counters[0..1].
__device__ __forceinline__ void add_counts(unsigned long long* counters, unsigned tests,
                                           unsigned accepts) {
    __shared__ unsigned long long block_counts[2];
    const int rank = threadIdx.y * blockDim.x + threadIdx.x;
    if (rank < 2) block_counts[rank] = 0;
    __syncthreads();
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        tests += __shfl_xor_sync(0xffffffffu, tests, o);
        accepts += __shfl_xor_sync(0xffffffffu, accepts, o);
    }
    if ((rank & 31) == 0) {
        atomicAdd(block_counts, (unsigned long long)tests);
        atomicAdd(block_counts + 1, (unsigned long long)accepts);
    }
    __syncthreads();
    if (rank < 2) atomicAdd(counters + rank, block_counts[rank]);
}

__device__ __forceinline__ int64_t row_of(const Params& P, int r) {
    if (P.row_mode == GS_ROWS_PER_RECORD) return r;
    if (P.row_mode == GS_ROWS_EXPLICIT) return P.prim_ids[r];
    // r < 2^31 (int32 point lists), so 32-bit unsigned division suffices whenever the
    // divisors fit; a scene (surfels x cameras) beyond 2^32 records takes the 64-bit path
    const int64_t per_scene = P.surfels * P.cameras;
    if (per_scene <= 0xffffffffLL) {
        const unsigned u = unsigned(r), n = u % unsigned(P.surfels);
        const unsigned s = u / unsigned(per_scene);
        return int64_t(s) * P.surfels + n;
    }
    return (r / per_scene) * P.surfels + r % P.surfels;
}

// Squared local radius beyond which a sample of opacity o is certainly below the
// alpha acceptance threshold: o * exp(-rho/2) < 1/255 for every rho > 2 ln(255 o).
// The 1e-4 margin covers the rounding of expf, of the product and of this logf
// (each a few 1e-7 relative), so the exact test would reject every sample the early
// test rejects.  o <= 0 gives -inf (always rejected, as the exact test does).
__device__ __forceinline__ float reject_threshold(float opacity) {
    return 2.f * logf(255.f * opacity) + 1e-4f;
}

template <bool Neural, int kSize = kBatch>
struct Batch {
    static constexpr int kRow = Neural ? kNeuralRow : kClassicRow;
    static constexpr bool kNeural = Neural;
    static constexpr int kCapacity = kSize;
    int ids[kSize];
    int64_t rows[kSize];
    float4 geo[kSize][kRec / 4];
    float4 app[kSize][kRow / 4];
    float half_weight[Neural ? 1 : kSize];   // classic: half the sum of the 4 wave weights
};

// Batch staging, double-buffered: `issue_batch` stages `count` records (list positions
// first + stride*e) and their appearance rows with one 16-byte cp.async (LDGSTS) per
// element, issued while the previous batch is composited; `finish_batch` waits for this
// thread's own copies and fixes up the elements it copied: record slot 18 (pad in
// memory) gets the early-rejection threshold of the record's opacity, and classic rows
// get 2*pi*magnitude in place of each magnitude (the factor every wave argument uses,
// computed once per record instead of once per sample: the same float product the
// per-sample expression 2 * pi * magnitude rounds to) and the half sum of the four wave
// weights (the thread copying weights 2-3 also copies weights 0-1 into a scratch slot).
// The caller's next barrier makes the batch visible to all threads.  Each loading
// thread reads its record id (L1-cached); the part-0 thread keeps it for the kernels'
// gradient writes.
__device__ __forceinline__ void copy16_async(void* smem, const void* gmem) {
    const unsigned dst = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(gmem) : "memory");
}

template <class B>
__device__ __forceinline__ void issue_batch(B& b, float4* weights01, const Params& P, int first,
                                            int stride, int count, int rank) {
    constexpr int kRow = B::kRow;
    constexpr int kPer = kRec / 4 + kRow / 4;
    for (int i = rank; i < count * kPer; i += kBlock) {
        const int e = i / kPer, part = i % kPer;
        const int id = __ldg(P.point_list + first + stride * e);
        if (part < kRec / 4) {
            if (part == 0) b.ids[e] = id;
            copy16_async(&b.geo[e][part], P.records + int64_t(id) * (kRec / 4) + part);
        } else {
            const int q = part - kRec / 4;
            const int64_t row = row_of(P, id);
            if (q == 0) b.rows[e] = row;
            copy16_async(&b.app[e][q], P.rows + row * (kRow / 4) + q);
            if (!B::kNeural && q == 2) copy16_async(&weights01[e], P.rows + row * (kRow / 4) + 1);
        }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}

template <class B>
__device__ __forceinline__ void finish_batch(B& b, const float4* weights01, int count, int rank) {
    constexpr int kRow = B::kRow;
    constexpr int kPer = kRec / 4 + kRow / 4;
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    for (int i = rank; i < count * kPer; i += kBlock) {
        const int e = i / kPer, part = i % kPer;
        if (part == 4) {   // slot 18 (pad in memory) <- rejection threshold of the opacity
            float4& v = b.geo[e][4];
            v.z = reject_threshold(v.y);
        }
        if constexpr (!B::kNeural) {
            constexpr float kTwoPi = 2 * kPi;
            const int q = part - kRec / 4;
            if (q == 2) {   // weights 2-3, magnitudes 0-1
                float4& v = b.app[e][2];
                const float4 w01 = weights01[e];
                b.half_weight[e] = 0.5f * ((w01.z + w01.w) + (v.x + v.y));
                v.z = kTwoPi * v.z;
                v.w = kTwoPi * v.w;
            }
            if (q == 3) {   // magnitudes 2-3
                float4& v = b.app[e][3];
                v.x = kTwoPi * v.x;
                v.y = kTwoPi * v.y;
            }
        }
    }
}

struct Sample {
    float k[3], l[3], p[3], s[2], depth, expo, alpha;
    bool surface;
};

// Ray/plane intersection and filtered opacity: rasterize.cu:84-103.
__device__ __forceinline__ bool sample_surface(const float* g, int x, int y, bool neural,
                                               float near_plane, Sample& v) {
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        v.k[k] = x * g[6 + k] - g[k];
        v.l[k] = y * g[6 + k] - g[3 + k];
    }
    cross3(v.k, v.l, v.p);
    if (v.p[2] == 0) return false;
    const float dx = g[9] - x, dy = g[10] - y;
    const float rho2 = 2 * (dx * dx + dy * dy);
    // Early rejection (same decision as the exact test below, fewer instructions):
    // alpha = o exp(-min(rho3, rho2)/2) < 1/255 once both radii exceed g[18].  rho3 is
    // bounded from below by (p0^2 + p1^2)/p2^2 with a fast divide, shrunk by 1e-5 to
    // cover its few-ulp error; NaN or an out-of-range p2^2 falls through.
    if (rho2 > g[18]) {
        const float q = v.p[2] * v.p[2];
        if (q >= 1.17549435e-38f && q <= 1e37f &&
            __fdividef(fmaf(v.p[1], v.p[1], v.p[0] * v.p[0]), q) * (1.f - 1e-5f) > g[18])
            return false;
    }
    v.s[0] = v.p[0] / v.p[2];
    v.s[1] = v.p[1] / v.p[2];
    const float rho3 = v.s[0] * v.s[0] + v.s[1] * v.s[1];
    v.surface = rho3 <= rho2;
    v.depth = (neural || v.surface) ? v.s[0] * g[6] + v.s[1] * g[7] + g[8] : g[8];
    if (v.depth < near_plane || !isfinite(v.depth)) return false;
    v.expo = expf(-0.5f * fminf(rho3, rho2));
    v.alpha = fminf(0.99f, g[17] * v.expo);
    return v.alpha >= 1.0f / 255.0f;
}

// Frequency directions d_f = (cos(pi f/4), sin(pi f/4)) evaluated like the reference
// (cosf/sinf of the float angle, rasterize.cu:128, 176).
struct Directions {
    float c[4], s[4];
    __device__ __forceinline__ Directions() {
#pragma unroll
        for (int f = 0; f < 4; ++f) {
            c[f] = cosf(kPi * f / 4);
            s[f] = sinf(kPi * f / 4);
        }
    }
};

// Sine and cosine for gradient arithmetic only (images use the exact cosf/sinf):
// Cody-Waite reduction of x by 2*pi with a two-term constant (2*pi = hi + lo,
// hi = float(2*pi)), then the SFU approximations on [-pi, pi].  Absolute error below
// 1e-6 for |x| < 1e4, far inside the gradients' 1e-4 tolerance.
__device__ __forceinline__ void grad_sincos(float x, float* s, float* c) {
    const float k = rintf(x * 0.159154943091895336f);
    float r = fmaf(-k, 6.28318548202514648f, x);
    r = fmaf(-k, -1.74845553e-07f, r);
    __sincosf(r, s, c);
}

// Fast forms for the appearance, used unless exact appearance is requested:
// Cody-Waite reduction by 2*pi as in grad_sincos, then the SFU approximations
// (|error| < 4e-7 for the waves, so an image moves by less than 1e-6), and the SFU
// exponential with a fast divide for the sigmoid.
constexpr float kThird = 1.f / 3;   // fast and gradient-only forms multiply instead of divide

__device__ __forceinline__ float fast_cos(float x) {
    const float k = rintf(x * 0.159154943091895336f);
    float r = fmaf(-k, 6.28318548202514648f, x);
    r = fmaf(-k, -1.74845553e-07f, r);
    return __cosf(r);
}
__device__ __forceinline__ float fast_sin(float x) {
    const float k = rintf(x * 0.159154943091895336f);
    float r = fmaf(-k, 6.28318548202514648f, x);
    r = fmaf(-k, -1.74845553e-07f, r);
    return __sinf(r);
}

// Appearance: rasterize.cu:105-138.  Exact: the reference's expressions with
// full-precision cosf/sinf/expf (images bit-identical to the reference's); otherwise
// the fast forms above.
template <bool Neural, bool Exact>
__device__ __forceinline__ void appearance_forward(const float* a, const float* g, const Sample& v,
                                                   const Directions& dirs, float half_weight,
                                                   float* color, float* hidden, float* pre) {
    if constexpr (Neural) {
        const float input[5] = {Exact ? v.s[0] / 3 : v.s[0] * kThird,
                                Exact ? v.s[1] / 3 : v.s[1] * kThird, g[14], g[15], g[16]};
#pragma unroll
        for (int h = 0; h < 6; ++h) {
            float z = a[30 + h];
#pragma unroll
            for (int k = 0; k < 5; ++k) z += a[h * 5 + k] * input[k];
            pre[h] = z;
            hidden[h] = Exact ? sinf(30 * z) : fast_sin(30 * z);
        }
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            float z = a[54 + c];
#pragma unroll
            for (int h = 0; h < 6; ++h) z += a[36 + c * 6 + h] * hidden[h];
            color[c] = Exact ? 1 / (1 + expf(-z)) : __fdividef(1.f, 1.f + __expf(-z));
        }
    } else if constexpr (Exact) {
        float h1 = 0, h2 = 0;
#pragma unroll
        for (int f = 0; f < 4; ++f) {
            const float dot = dirs.c[f] * v.s[0] + dirs.s[f] * v.s[1];
            const float arg = a[10 + f] * dot + a[14 + f];   // a[10+f] = 2 pi mag_f
            const float wave = cosf(arg);
            h1 += a[6 + f] * 0.5f * (1 + wave);
            h2 += a[6 + f] * 0.5f * (1 - wave);
        }
#pragma unroll
        for (int c = 0; c < 3; ++c) color[c] = h1 * a[c] + h2 * a[3 + c];
    } else {
        // h1 = sum w_f (1 + wave_f) / 2 = W/2 + hw/2 and h2 = W/2 - hw/2 with
        // hw = sum w_f wave_f and W/2 staged per record: one FMA per wave.
        float hw = 0;
#pragma unroll
        for (int f = 0; f < 4; ++f) {
            const float dot = dirs.c[f] * v.s[0] + dirs.s[f] * v.s[1];
            hw = fmaf(a[6 + f], fast_cos(a[10 + f] * dot + a[14 + f]), hw);
        }
        const float h1 = fmaf(0.5f, hw, half_weight), h2 = fmaf(-0.5f, hw, half_weight);
#pragma unroll
        for (int c = 0; c < 3; ++c) color[c] = h1 * a[c] + h2 * a[3 + c];
    }
}

template <bool Neural, bool Count, bool Exact, bool Median, bool Mask>
__global__ __launch_bounds__(kBlock, 4) void composite_forward_kernel(const Params P) {
    static_assert(kBatch == 64 && kBlock / 32 == kMaskWarps, "accepted bits: two words a batch");
    unsigned tests = 0, accepts = 0;
    __shared__ Batch<Neural> batches[2];
    __shared__ float4 weights01[2][Neural ? 1 : kBatch];
    const int rank = threadIdx.y * kTile + threadIdx.x;
    const int warp = rank >> 5, lane = rank & 31;
    // Mask: which of the current batch's records this pixel accepted (bit j of records
    // 0-31, then 32-63), OR-reduced over the warp after each batch
    unsigned accepted_lo = 0, accepted_hi = 0;
    const PixelSlot slot = pixel_slot(P, rank);
    const int tile = slot.tile, image = slot.image, x = slot.x, y = slot.y;
    const bool inside = slot.inside;
    const int64_t pixel = slot.pixel;
    bool done = !inside;
    float out[kMaps] = {}, T = 1, m1 = 0, m2 = 0, median = 0;
    int median_at = 0;
    int last = 0;
    const int2 range = P.ranges[tile];
    const Directions dirs;
    const float mscale = P.far_plane / (P.far_plane - P.near_plane);
    const float mscale_near = mscale * P.near_plane;
    // Double-buffered batches: batch b+1's copies are in flight while batch b is
    // composited; one barrier per batch (after this thread's copies of batch b landed and
    // were fixed up) makes batch b visible and retires batch b-1's buffer.
    if (range.x < range.y)
        issue_batch(batches[0], weights01[0], P, range.x, 1, min(kBatch, range.y - range.x), rank);
    for (int start = range.x, b = 0; start < range.y; start += kBatch, ++b) {
        auto& batch = batches[b & 1];
        const int count = min(kBatch, range.y - start);
        finish_batch(batch, weights01[b & 1], count, rank);
        if (__syncthreads_count(done) == kBlock) break;
        if (start + kBatch < range.y)
            issue_batch(batches[(b + 1) & 1], weights01[(b + 1) & 1], P, start + kBatch, 1,
                        min(kBatch, range.y - start - kBatch), rank);
        for (int j = 0; j < count && !done; ++j) {
            const float* g = reinterpret_cast<const float*>(batch.geo[j]);
            Sample v;
            if constexpr (Count) ++tests;
            if (!sample_surface(g, x, y, Neural, P.near_plane, v)) continue;
            const float next = T * (1 - v.alpha);
            if (next < 0.0001f) { done = true; break; }
            if constexpr (Count) ++accepts;
            if constexpr (Mask) {
                if (j < 32) accepted_lo |= 1u << j;
                else accepted_hi |= 1u << (j - 32);
            }
            float color[3], hidden[6], pre[6];
            appearance_forward<Neural, Exact>(reinterpret_cast<const float*>(batch.app[j]), g, v, dirs,
                                              batch.half_weight[Neural ? 0 : j], color, hidden,
                                              pre);
            const float w = T * v.alpha;
            const float m = Exact ? mscale * (1 - P.near_plane / v.depth)
                                  : fmaf(-mscale_near, __fdividef(1.f, v.depth), mscale);
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                out[c] += w * color[c];
                out[5 + c] += w * g[11 + c];
            }
            out[4] += w * v.depth;
            out[8] += w * (m * m * (1 - T) + m2 - 2 * m * m1);
            m1 += w * m;
            m2 += w * m * m;
            last = start + j - range.x + 1;
            if (Median && T > 0.5f) {   // transmittance before this contribution
                median = v.depth;
                median_at = last;
            }
            T = next;
        }
        if constexpr (Mask) {   // the warp's accepted records of this batch, as bits
            const unsigned lo = __reduce_or_sync(0xffffffffu, accepted_lo);
            const unsigned hi = __reduce_or_sync(0xffffffffu, accepted_hi);
            accepted_lo = accepted_hi = 0;
            if (lane == 0 && (lo | hi)) or_accepted(P, warp, start, lo, hi);
        }
    }
    if (inside) {
#pragma unroll
        for (int c = 0; c < 3; ++c) out[c] += T * P.backgrounds[image * 3 + c];
        out[3] = 1 - T;
#pragma unroll
        for (int g = 0; g < 5; ++g) {
            float* o = P.out[g] + pixel * P.out_px[g];
#pragma unroll
            for (int k = 0; k < plane_size(g); ++k) o[k] = out[plane_first(g) + k];
        }
        P.state[pixel * 3] = T;
        P.state[pixel * 3 + 1] = m1;
        P.state[pixel * 3 + 2] = m2;
        P.contributors[pixel] = last;
        if constexpr (Median) {
            P.median[pixel * P.median_px] = median;
            P.median_index[pixel] = median_at;
        }
    }
    if constexpr (Count) add_counts(P.counters, tests, accepts);
}

// ------------------------------------------------------------------------------
// backward
// ------------------------------------------------------------------------------

// Per-record gradient fields, packed: record slots (T 0-8, xy 9-10, normal 11-13,
// [dir 14-16 neural]), opacity (record slot 17), then the appearance row.
template <bool Neural, bool Normals>
struct Fields {
    // Packed per-record gradient fields summed over a warp's pixels: record slots 0-13
    // (T, xy, normal), the opacity, then the appearance row.  Classic: the 18-float row.
    // Neural: 39 of the 57 row floats -- per hidden unit the weights of the (u, v) inputs,
    // then b1, W2, b2.  The weights of the three direction inputs and the direction
    // gradient (record slots 14-16) are per-record constants (the direction, the input
    // weights) times the b1 sums, so the flush forms them (21 values per record).
    // Without a normal-map gradient (Normals false: its plane is NULL, every pixel's
    // normal gradient zero) the normal slots 11-13 have no field: the classic row then
    // has 30 fields, one 32-column pass of the warp reduction with nothing left over.
    static constexpr int kGeo = Normals ? 14 : 11;
    static constexpr int kRow = Neural ? 39 : 18;
    static constexpr int kCount = kGeo + 1 + kRow;   // classic 33 / 30, neural 54 / 51
    static constexpr int kB1 = kGeo + 1 + 12;                  // neural: field of b1[0]
    // classic: packed field of record slot s / appearance-row slot q (-1: no field)
    static __device__ __forceinline__ int record_field(int s) {
        return s < kGeo ? s : (s == 17 ? kGeo : -1);
    }
    static __device__ __forceinline__ int row_field(int q) { return q < kRow ? kGeo + 1 + q : -1; }
    // neural: row slot of packed row field p (W1 (u, v) columns, b1, W2, b2)
    static __device__ __forceinline__ int neural_row_slot(int p) {
        return p < 12 ? (p >> 1) * 5 + (p & 1) : p < 18 ? 30 + (p - 12) : p < 36 ? 36 + (p - 18)
                                                                          : 54 + (p - 36);
    }
};

constexpr int kBackBatch = 24;
constexpr int kWarps = kBlock / 32;

constexpr int kLaneStride = 36;   // 32 fields + 4 pad: a lane's 16-byte stores hit 4 new banks

template <bool Neural, bool Normals>
struct BackShared {
    using F = Fields<Neural, Normals>;
    // per (warp, record) row of field sums.  Classic: 33 (31) floats, an odd stride, so
    // the flush's reads (thread i: record i / 10, fields 4 (i % 10) + k) spread over the
    // banks instead of four-way conflicts with a stride of 36.  Neural: 56 (52).
    static constexpr int kStride = Neural ? (F::kCount + 3) / 4 * 4 : (F::kCount | 1);
    Batch<Neural, kBackBatch> batch[2];        // double-buffered: batch b+1 lands during b
    float4 weights01[2][Neural ? 1 : kBackBatch];
    float rows[kWarps][kBackBatch][kStride];   // per (warp, record) field sums
    float lanes[kWarps][32][kLaneStride];      // per-warp transpose scratch, 32 fields a pass
    unsigned mask[2][kBackBatch];              // warps that stored a row for the record
    int warp_max[kWarps];
    float bg[3];
};

// Sum `vals` over the warp's 32 lanes into the warp's row for the record, 32 fields a
// pass: every lane stores its fields as one row of the warp's scratch (16-byte stores,
// conflict-free).  Lane (quad q = lane % 8, group g = lane / 8) then adds columns
// 4q..4q+3 over rows 8g..8g+7 with eight 16-byte loads (each quarter-warp reads one
// whole row: conflict-free), and the four groups' partial sums are scattered with two
// shuffle steps, after which the lane holds the full sum of column 4q + g: 8 loads +
// 28 adds + 3 shuffles, 3 adds and 6 selects, where one column per lane costs 32 loads
// and 31 adds and a shuffle butterfly 31 shuffles, 62 selects and 31 adds.  One or two
// fields left over past the passes are summed with a plain butterfly.  Plain stores, no
// shared atomics: the CTA's eight rows are summed at the flush; `mask` records which
// warps stored.
template <bool Neural, bool Normals>
__device__ __forceinline__ void warp_store(const float* vals, float (*scratch)[kLaneStride],
                                           float* row, unsigned* mask, int warp, int lane) {
    using F = Fields<Neural, Normals>;
    constexpr int kPasses = F::kCount / 32 + (F::kCount % 32 > 2 ? 1 : 0);
    const int quad = lane & 7, group = lane >> 3;
    const bool high = group & 2, odd = group & 1;
#pragma unroll
    for (int pass = 0; pass < kPasses; ++pass) {
        if (pass) __syncwarp();
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int f = pass * 32 + 4 * k;
            float4 q;
            q.x = f + 0 < F::kCount ? vals[f + 0] : 0.f;
            q.y = f + 1 < F::kCount ? vals[f + 1] : 0.f;
            q.z = f + 2 < F::kCount ? vals[f + 2] : 0.f;
            q.w = f + 3 < F::kCount ? vals[f + 3] : 0.f;
            *reinterpret_cast<float4*>(&scratch[lane][4 * k]) = q;
        }
        __syncwarp();
        float4 s = *reinterpret_cast<const float4*>(&scratch[8 * group][4 * quad]);
#pragma unroll
        for (int r = 1; r < 8; ++r) {
            const float4 t = *reinterpret_cast<const float4*>(&scratch[8 * group + r][4 * quad]);
            s.x += t.x;
            s.y += t.y;
            s.z += t.z;
            s.w += t.w;
        }
        // groups g and g ^ 2: the high pair keeps columns 2-3, the low pair 0-1
        float k0 = high ? s.z : s.x, k1 = high ? s.w : s.y;
        k0 += __shfl_xor_sync(0xffffffffu, high ? s.x : s.z, 16);
        k1 += __shfl_xor_sync(0xffffffffu, high ? s.y : s.w, 16);
        // groups g and g ^ 1: the odd one keeps the second column
        float sum = odd ? k1 : k0;
        sum += __shfl_xor_sync(0xffffffffu, odd ? k0 : k1, 8);
        const int column = pass * 32 + 4 * quad + group;
        if (column < F::kCount) row[column] = sum;
    }
#pragma unroll
    for (int f = kPasses * 32; f < F::kCount; ++f) {
        float v = vals[f];
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) row[f] = v;
    }
    __syncwarp();   // column reads done before the next record's stores
    if (lane == 0) atomicOr(mask, 1u << warp);
}

template <bool Neural, bool Count, bool Normals, bool Mask>
__global__ __launch_bounds__(kBlock, Neural ? 2 : 3) void composite_backward_kernel(const Params P) {
    unsigned tests = 0, accepts = 0;
    using F = Fields<Neural, Normals>;
    using S = BackShared<Neural, Normals>;
    constexpr int kRow = Batch<Neural>::kRow;
    extern __shared__ float4 dynamic_smem[];
    S& sh = *reinterpret_cast<S*>(dynamic_smem);
    int* warp_max = sh.warp_max;
    float* bg_acc = sh.bg;
    const int lane = (threadIdx.y * kTile + threadIdx.x) & 31;
    const int warp = (threadIdx.y * kTile + threadIdx.x) >> 5;
    const int rank = threadIdx.y * kTile + threadIdx.x;
    const PixelSlot slot = pixel_slot(P, rank);
    const int tile = slot.tile, image = slot.image, x = slot.x, y = slot.y;
    const bool inside = slot.inside;
    const int64_t pixel = slot.pixel;
    const int last = inside ? P.contributors[pixel] : 0;
    // median depth gradient goes to the depth of the median contribution
    const int median_at = inside && P.gin_median ? P.median_index[pixel] : 0;
    const float go_median = median_at ? P.gin_median[pixel * P.gin_median_px] : 0.f;
    if (rank < 3) bg_acc[rank] = 0.f;
    if (rank < 2 * kBackBatch) sh.mask[rank / kBackBatch][rank % kBackBatch] = 0u;
    int wmax = last;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) wmax = max(wmax, __shfl_xor_sync(0xffffffffu, wmax, o));
    if (lane == 0) warp_max[warp] = wmax;
    float go[kMaps] = {};
    if (inside) {
#pragma unroll
        for (int g = 0; g < 5; ++g) {
            if (!P.gin[g]) continue;
            const float* gi = P.gin[g] + pixel * P.gin_px[g];
#pragma unroll
            for (int k = 0; k < plane_size(g); ++k) go[plane_first(g) + k] = gi[k * P.gin_ch[g]];
        }
    }
    const float final_t = inside ? P.state[pixel * 3] : 0;
    const float total_a = 1 - final_t;
    const float m1 = inside ? P.state[pixel * 3 + 1] : 0, m2 = inside ? P.state[pixel * 3 + 2] : 0;
    float T = final_t, suffix = 0, background_dot = 0;
    {
        float bgv[4] = {};
#pragma unroll
        for (int c = 0; c < 3; ++c) {
            background_dot += go[c] * P.backgrounds[image * 3 + c];
            bgv[c] = final_t * go[c];
        }
        warp_reduce_scatter<4>(bgv, lane);
        __syncthreads();   // bg_acc initialised
        if ((lane & 7) == 0 && (lane >> 3) < 3 && bgv[0] != 0.f) atomicAdd(bg_acc + (lane >> 3), bgv[0]);
    }
    int block_last = 0;
#pragma unroll
    for (int w = 0; w < kBlock / 32; ++w) block_last = max(block_last, warp_max[w]);
    const int2 range = P.ranges[tile];
    const Directions dirs;
    const float mscale = P.far_plane / (P.far_plane - P.near_plane);
    // per-pixel constants of the gradient expressions
    const float mscale_near = mscale * P.near_plane;
    const float depth_term = go[8] * 2 * mscale_near;                // d distortion / d depth
    const float background_term = final_t * (go[3] - background_dot);  // galpha's T-independent part
    constexpr int kRecQuads = kRec / 4, kQuads = kRecQuads + kRow / 4;
    // 16-byte vector atomics need 16-byte aligned gradient rows (records and rows are
    // 80/240-byte rows, so aligned bases suffice)
    const bool vector_atomics =
        ((reinterpret_cast<uintptr_t>(P.grad_records) | reinterpret_cast<uintptr_t>(P.grad_rows)) &
         15u) == 0u;
    // Double-buffered batches in reverse list order: batch b+1's copies are in flight
    // while batch b is replayed and flushed.  The barrier after this thread's copies of
    // batch b landed also orders batch b-1's flush (its ids, rows and masks) before batch
    // b+1's copies and mask reset reuse that buffer.
    if (block_last > 0)
        issue_batch(sh.batch[0], sh.weights01[0], P, range.x + block_last - 1, -1,
                    min(kBackBatch, block_last), rank);
    for (int start = block_last, b = 0; start > 0; start -= kBackBatch, ++b) {
        const int count = min(kBackBatch, start);
        auto& batch = sh.batch[b & 1];
        unsigned* mask = sh.mask[b & 1];
        finish_batch(batch, sh.weights01[b & 1], count, rank);
        __syncthreads();
        if (start > kBackBatch) {
            issue_batch(sh.batch[(b + 1) & 1], sh.weights01[(b + 1) & 1], P,
                        range.x + start - kBackBatch - 1, -1, min(kBackBatch, start - kBackBatch),
                        rank);
            if (rank < kBackBatch) sh.mask[(b + 1) & 1][rank] = 0u;
        }
        // Mask: bit k of `accepted` = whether a pixel of this warp accepted the record at
        // list position low + k in the forward (positions past the plane: assumed so)
        uint64_t accepted = ~uint64_t(0);
        if constexpr (Mask) {
            const int64_t high = int64_t(range.x) + start - 1, low = high - (count - 1);
            const unsigned* plane = P.warp_mask + int64_t(warp) * P.warp_mask_words;
            const int64_t w0 = low >> 5, w1 = high >> 5;
            const unsigned a0 = w0 < P.warp_mask_words ? plane[w0] : ~0u;
            const unsigned a1 = w1 == w0 ? 0u : (w1 < P.warp_mask_words ? plane[w1] : ~0u);
            accepted = ((uint64_t(a1) << 32) | a0) >> (low & 31);
        }
        for (int j = 0; j < count; ++j) {
            // a record no pixel of the warp accepted in the forward adds no gradient here
            if (Mask && !((accepted >> (count - 1 - j)) & 1u)) continue;
            const float* g = reinterpret_cast<const float*>(batch.geo[j]);
            const float* a = reinterpret_cast<const float*>(batch.app[j]);
            Sample v;
            bool active = inside && start - j <= last;
            if constexpr (Count) tests += active;
            if (active) active = sample_surface(g, x, y, Neural, P.near_plane, v);
            if constexpr (Count) accepts += active;
            if (!__any_sync(0xffffffffu, active)) continue;
            float vals[F::kCount];
#pragma unroll
            for (int i = 0; i < F::kCount; ++i) vals[i] = 0.f;
            float* gg = vals;                  // record fields 0..kGeo-1
            float& gopacity = vals[F::kGeo];
            float* ga = vals + F::kGeo + 1;    // appearance row fields
            if (active) {
                float color[3], hidden[6], pre[6], gc[3], gs[2] = {0.f, 0.f};
                float waves[4], sines[4];
                // T before this sample: one correctly rounded reciprocal, shared with galpha
                const float inv_transmit = __frcp_rn(1 - v.alpha);
                T *= inv_transmit;
                const float w = T * v.alpha;
                // colour replay: feeds only gradients, so the waves, the SIREN's sines
                // and its sigmoid use the fast forms (cosines kept for the adjoint)
                float coss[6], dots[4], h1, h2;
                if constexpr (Neural) {
                    const float input[5] = {v.s[0] * kThird, v.s[1] * kThird, g[14], g[15], g[16]};
#pragma unroll
                    for (int h = 0; h < 6; ++h) {
                        float z = a[30 + h];
#pragma unroll
                        for (int k = 0; k < 5; ++k) z += a[h * 5 + k] * input[k];
                        pre[h] = z;
                        grad_sincos(30 * z, &hidden[h], &coss[h]);
                    }
#pragma unroll
                    for (int c = 0; c < 3; ++c) {
                        float z = a[54 + c];
#pragma unroll
                        for (int h = 0; h < 6; ++h) z += a[36 + c * 6 + h] * hidden[h];
                        color[c] = __fdividef(1.f, 1.f + __expf(-z));
                    }
                } else {
                    float hw = 0;
#pragma unroll
                    for (int f = 0; f < 4; ++f) {
                        dots[f] = dirs.c[f] * v.s[0] + dirs.s[f] * v.s[1];
                        grad_sincos(a[10 + f] * dots[f] + a[14 + f], &sines[f], &waves[f]);
                        hw = fmaf(a[6 + f], waves[f], hw);
                    }
                    h1 = fmaf(0.5f, hw, batch.half_weight[Neural ? 0 : j]);
                    h2 = fmaf(-0.5f, hw, batch.half_weight[Neural ? 0 : j]);
#pragma unroll
                    for (int c = 0; c < 3; ++c) color[c] = h1 * a[c] + h2 * a[3 + c];
                }
                const float inv_depth = __fdividef(1.f, v.depth);
                const float m = fmaf(-mscale_near, inv_depth, mscale);
                float gw = go[4] * v.depth + go[8] * (m * m * total_a + m2 - 2 * m * m1);
#pragma unroll
                for (int c = 0; c < 3; ++c) {
                    if constexpr (Normals) {
                        gw += go[c] * color[c] + go[5 + c] * g[11 + c];
                        gg[11 + c] += w * go[5 + c];
                    } else {   // the same value with a zero normal gradient
                        gw = __fadd_rn(gw, __fmul_rn(go[c], color[c]));
                    }
                    gc[c] = w * go[c];
                }
                const float galpha = fmaf(T, gw, (background_term - suffix) * inv_transmit);
                suffix += w * gw;
                // appearance backward: rasterize.cu:146-197
                if constexpr (Neural) {
                    // packed row fields: W1 (u, v) columns 0-11, b1 12-17, W2 18-35, b2 36-38;
                    // the direction columns and the direction gradient come from the b1
                    // sums at the flush
                    const float input[2] = {v.s[0] * kThird, v.s[1] * kThird};
                    float gh[6] = {}, gi[2] = {};
#pragma unroll
                    for (int c = 0; c < 3; ++c) {
                        const float gz = gc[c] * color[c] * (1 - color[c]);
                        ga[36 + c] += gz;
#pragma unroll
                        for (int h = 0; h < 6; ++h) {
                            ga[18 + c * 6 + h] += gz * hidden[h];
                            gh[h] += gz * a[36 + c * 6 + h];
                        }
                    }
#pragma unroll
                    for (int h = 0; h < 6; ++h) {
                        const float gz = gh[h] * 30 * coss[h];
                        ga[12 + h] += gz;
#pragma unroll
                        for (int k = 0; k < 2; ++k) {
                            ga[2 * h + k] += gz * input[k];
                            gi[k] += gz * a[h * 5 + k];
                        }
                    }
                    gs[0] += gi[0] * kThird;
                    gs[1] += gi[1] * kThird;
                } else {
                    // The reference's per-wave loop (rasterize.cu:173-195) factored: summed
                    // over waves, d colour / d c1 = h1 and d colour / d c2 = h2; every
                    // wave's weight and phase terms go through S1 = sum gc (c1 + c2) / 2 and
                    // S2 = sum gc (c1 - c2) / 2.  The magnitude field holds gt * dot; the
                    // flush multiplies its per-tile sum by 2 pi.
                    float S1 = 0, S2 = 0;
#pragma unroll
                    for (int c = 0; c < 3; ++c) {
                        ga[c] = gc[c] * h1;
                        ga[3 + c] = gc[c] * h2;
                        S1 = fmaf(gc[c], a[c] + a[3 + c], S1);
                        S2 = fmaf(gc[c], a[c] - a[3 + c], S2);
                    }
                    S1 *= 0.5f;
                    S2 *= 0.5f;
#pragma unroll
                    for (int f = 0; f < 4; ++f) {
                        const float gt = -(a[6 + f] * sines[f]) * S2;
                        ga[6 + f] = fmaf(waves[f], S2, S1);
                        ga[10 + f] = gt * dots[f];
                        ga[14 + f] = gt;
                        const float u = gt * a[10 + f];   // a[10+f] = 2 pi mag_f
                        gs[0] = fmaf(u, dirs.c[f], gs[0]);
                        gs[1] = fmaf(u, dirs.s[f], gs[1]);
                    }
                }
                // geometry: rasterize.cu:359-385
                float gz = w * fmaf(depth_term * fmaf(m, total_a, -m1), inv_depth * inv_depth,
                                    go[4]);
                if (start - j == median_at) gz += go_median;
                if (Neural || v.surface) {
                    gs[0] += gz * g[6];
                    gs[1] += gz * g[7];
                    gg[6] += gz * v.s[0];
                    gg[7] += gz * v.s[1];
                }
                gg[8] += gz;
                float grho = 0;
                if (g[17] * v.expo < 0.99f) {
                    gopacity = galpha * v.expo;
                    grho = -0.5f * galpha * g[17] * v.expo;
                }
                if (v.surface) {
                    gs[0] += 2 * v.s[0] * grho;
                    gs[1] += 2 * v.s[1] * grho;
                } else {
                    gg[9] += 4 * (g[9] - x) * grho;
                    gg[10] += 4 * (g[10] - y) * grho;
                }
                const float inv_p2 = __frcp_rn(v.p[2]);
                const float gp[3] = {gs[0] * inv_p2, gs[1] * inv_p2,
                                     -(gs[0] * v.s[0] + gs[1] * v.s[1]) * inv_p2};
                float gk[3], gl[3];
                cross3(v.l, gp, gk);
                cross3(gp, v.k, gl);
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    gg[k] -= gk[k];
                    gg[3 + k] -= gl[k];
                    gg[6 + k] += x * gk[k] + y * gl[k];
                }
            }
            warp_store<Neural, Normals>(vals, sh.lanes[warp], sh.rows[warp][j], &mask[j], warp,
                                        lane);
        }
        // flush: sum the warps' rows of each record in warp order and add them to global
        // memory.  Classic: one 16-byte vector atomic per (tile, record, 4-slot quad) of
        // the record and its appearance row (slots without a field add zero).  Neural: one
        // atomic per (tile, record, field) (its 57-field rows gain nothing from quads).
        __syncthreads();
        if constexpr (Neural) {
            constexpr int kItems = F::kCount + 21;   // fields, then the formed values
            for (int i = rank; i < count * kItems; i += kBlock) {
                const int e = i / kItems, item = i % kItems;
                const unsigned stored = mask[e];
                auto field_sum = [&](int field) {
                    float sum = 0.f;
#pragma unroll
                    for (int w = 0; w < kWarps; ++w)
                        if (stored & (1u << w)) sum += sh.rows[w][e][field];
                    return sum;
                };
                const int64_t r = batch.ids[e];
                float* grad_row = P.grad_rows + batch.rows[e] * kRow;
                if (item < F::kCount) {
                    const float val = field_sum(item);
                    if (val == 0.f) continue;
                    if (item < F::kGeo) {
                        if (P.grad_xy && (item == 9 || item == 10))
                            atomicAdd(P.grad_xy + r * 2 + (item - 9), val);
                        else
                            atomicAdd(P.grad_records + r * kRec + item, val);
                    } else if (item == F::kGeo) {
                        atomicAdd(P.grad_records + r * kRec + 17, val);   // opacity
                    } else {
                        atomicAdd(grad_row + F::neural_row_slot(item - F::kGeo - 1), val);
                    }
                    continue;
                }
                const int d = item - F::kCount;
                const float* geo = reinterpret_cast<const float*>(batch.geo[e]);
                if (d < 18) {   // W1[h][2 + k] = dir_k * sum of b1[h]
                    const int h = d / 3, k = d % 3;
                    const float val = geo[14 + k] * field_sum(F::kB1 + h);
                    if (val != 0.f) atomicAdd(grad_row + h * 5 + 2 + k, val);
                } else {        // direction_k = sum_h W1[h][2 + k] * sum of b1[h]
                    const int k = d - 18;
                    const float* app = reinterpret_cast<const float*>(batch.app[e]);
                    float val = 0.f;
#pragma unroll
                    for (int h = 0; h < 6; ++h) val = fmaf(app[h * 5 + 2 + k], field_sum(F::kB1 + h), val);
                    if (val != 0.f) atomicAdd(P.grad_records + r * kRec + 14 + k, val);
                }
            }
            continue;
        }
        for (int i = rank; i < count * kQuads; i += kBlock) {
            const int e = i / kQuads, quad = i % kQuads;
            const unsigned stored = mask[e];
            float v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int field = quad < kRecQuads ? F::record_field(4 * quad + k)
                                                   : F::row_field(4 * (quad - kRecQuads) + k);
                float val = 0.f;
                if (field >= 0) {
#pragma unroll
                    for (int w = 0; w < kWarps; ++w)
                        if (stored & (1u << w)) val += sh.rows[w][e][field];
                }
                v[k] = val;
            }
            if (v[0] == 0.f && v[1] == 0.f && v[2] == 0.f && v[3] == 0.f) continue;
            float* dst;
            if (quad < kRecQuads) {
                const int64_t r = batch.ids[e];
                dst = P.grad_records + r * kRec + 4 * quad;
                if (P.grad_xy && quad == 2) {   // slots 9-10 (xy) go to their own array
                    if (v[0] != 0.f) atomicAdd(dst, v[0]);
                    if (v[1] != 0.f) atomicAdd(P.grad_xy + r * 2, v[1]);
                    if (v[2] != 0.f) atomicAdd(P.grad_xy + r * 2 + 1, v[2]);
                    if (v[3] != 0.f) atomicAdd(dst + 3, v[3]);
                    continue;
                }
            } else {
                const int q = 4 * (quad - kRecQuads);
                if constexpr (!Neural) {   // magnitudes (row slots 10-13) take their 2 pi
                    if (q == 8) { v[2] *= 2 * kPi; v[3] *= 2 * kPi; }
                    if (q == 12) { v[0] *= 2 * kPi; v[1] *= 2 * kPi; }
                }
                dst = P.grad_rows + batch.rows[e] * kRow + q;
            }
            if (vector_atomics) {
                atomicAdd(reinterpret_cast<float4*>(dst), make_float4(v[0], v[1], v[2], v[3]));
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (v[k] != 0.f) atomicAdd(dst + k, v[k]);
            }
        }
    }
    __syncthreads();
    if (rank < 3 && bg_acc[rank] != 0.f) atomicAdd(P.grad_backgrounds + image * 3 + rank, bg_acc[rank]);
    if constexpr (Count) add_counts(P.counters, tests, accepts);
}

int check_composite(const char* fn, const float* records, const float* rows, int row_mode,
                    const int64_t* prim_ids, int64_t cameras, int64_t surfels, int64_t R,
                    const float* backgrounds, const int32_t* ranges, int64_t images, int width,
                    int height) {
    if (images < 1 || width < 1 || height < 1 || R < 0)
        return fail(GS_ERR_ARGUMENT, std::string(fn) + ": invalid sizes");
    const int64_t tw = (width + kTile - 1) / kTile, th = (height + kTile - 1) / kTile;
    if (images * tw * th > INT_MAX)
        return fail(GS_ERR_LIMIT, std::string(fn) + ": image tile count exceeds int32");
    if (int64_t(width) * height * images * kMaps > (int64_t(1) << 62))
        return fail(GS_ERR_LIMIT, std::string(fn) + ": image too large");
    if (!backgrounds || !ranges) return fail(GS_ERR_ARGUMENT, std::string(fn) + ": NULL buffer");
    if (R > 0 && (!records || !rows)) return fail(GS_ERR_ARGUMENT, std::string(fn) + ": NULL records");
    if (reinterpret_cast<uintptr_t>(records) % 16 || reinterpret_cast<uintptr_t>(rows) % 16)
        return fail(GS_ERR_ARGUMENT, std::string(fn) + ": records and rows must be 16-byte aligned");
    if (row_mode == GS_ROWS_EXPLICIT && R > 0 && !prim_ids)
        return fail(GS_ERR_ARGUMENT, std::string(fn) + ": primitive_ids is NULL");
    if (row_mode == GS_ROWS_PER_SURFEL && R > 0 && (cameras < 1 || surfels < 1))
        return fail(GS_ERR_ARGUMENT, std::string(fn) + ": cameras and surfels must be positive");
    if (row_mode < 0 || row_mode > 2) return fail(GS_ERR_ARGUMENT, std::string(fn) + ": bad row mode");
    return GS_OK;
}

}  // namespace
}  // namespace gs

using namespace gs;

namespace gs {
namespace {

Params common_params(const float* records, const float* rows, int row_mode,
                     const int64_t* primitive_ids, int64_t cameras, int64_t surfels,
                     const float* backgrounds, const int32_t* point_list, const int32_t* ranges,
                     int width, int height, float near_plane, float far_plane) {
    Params P{};
    P.records = reinterpret_cast<const float4*>(records);
    P.rows = reinterpret_cast<const float4*>(rows);
    P.row_mode = row_mode;
    P.prim_ids = primitive_ids;
    P.cameras = cameras;
    P.surfels = surfels;
    P.backgrounds = backgrounds;
    P.point_list = point_list;
    P.ranges = reinterpret_cast<const int2*>(ranges);
    P.width = width;
    P.height = height;
    P.tw = (width + kTile - 1) / kTile;
    P.th = (height + kTile - 1) / kTile;
    P.near_plane = near_plane;
    P.far_plane = far_plane;
    return P;
}

int launch_forward(Params& P, int64_t images, int neural, int flags, uint64_t* counters,
                   void* stream, int64_t group_count = -1) {
    const int64_t tiles = group_count >= 0 ? group_count : images * P.tw * P.th;
    if (tiles == 0) return GS_OK;
    auto s = as_stream(stream);
    P.counters = reinterpret_cast<unsigned long long*>(counters);
    const dim3 block(kTile, kTile);
    const bool exact = flags & GS_COMPOSITE_EXACT;
    const unsigned grid = unsigned(tiles);
#define GS_FWD_M(N, C, E, M)                                                               \
    (P.warp_mask ? composite_forward_kernel<N, C, E, M, true><<<grid, block, 0, s>>>(P)       \
                 : composite_forward_kernel<N, C, E, M, false><<<grid, block, 0, s>>>(P))
#define GS_FWD(N, C, E) (P.median ? GS_FWD_M(N, C, E, true) : GS_FWD_M(N, C, E, false))
    if (neural) {
        if (counters) { if (exact) GS_FWD(true, true, true); else GS_FWD(true, true, false); }
        else { if (exact) GS_FWD(true, false, true); else GS_FWD(true, false, false); }
    } else {
        if (counters) { if (exact) GS_FWD(false, true, true); else GS_FWD(false, true, false); }
        else { if (exact) GS_FWD(false, false, true); else GS_FWD(false, false, false); }
    }
#undef GS_FWD
#undef GS_FWD_M
    GS_CHECK_LAUNCH("composite_forward_kernel");
    return GS_OK;
}

int launch_backward(Params& P, int64_t images, int neural, uint64_t* counters, void* stream,
                    int64_t group_count = -1) {
    auto s = as_stream(stream);
    const int64_t tiles = group_count >= 0 ? group_count : images * P.tw * P.th;
    if (tiles == 0) return GS_OK;
    P.counters = reinterpret_cast<unsigned long long*>(counters);
    const dim3 block(kTile, kTile);
    auto launch = [&](auto kernel, size_t smem) -> int {
        // the shared-memory opt-in is set once per kernel and device, so launches under
        // CUDA graph capture make no attribute calls
        int device = 0;
        GS_CUDA(cudaGetDevice(&device));
        static std::mutex mutex;
        static std::set<std::pair<const void*, int>> configured;
        {
            std::lock_guard<std::mutex> lock(mutex);
            const auto key = std::make_pair(reinterpret_cast<const void*>(kernel), device);
            if (!configured.count(key)) {
                GS_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             int(smem)));
                configured.insert(key);
            }
        }
        kernel<<<unsigned(tiles), block, smem, s>>>(P);
        return GS_OK;
    };
    // a NULL normal-map gradient plane drops the normal fields from the kernel
#define GS_BWD(N, C, M)                                                                    \
    (P.warp_mask ? launch(composite_backward_kernel<N, C, M, true>, sizeof(BackShared<N, M>)) \
                 : launch(composite_backward_kernel<N, C, M, false>, sizeof(BackShared<N, M>)))
    const bool normals = P.gin[3] != nullptr;
    int st;
    if (neural && counters)
        st = normals ? GS_BWD(true, true, true) : GS_BWD(true, true, false);
    else if (neural)
        st = normals ? GS_BWD(true, false, true) : GS_BWD(true, false, false);
    else if (counters)
        st = normals ? GS_BWD(false, true, true) : GS_BWD(false, true, false);
    else
        st = normals ? GS_BWD(false, false, true) : GS_BWD(false, false, false);
#undef GS_BWD
    if (st) return st;
    GS_CHECK_LAUNCH("composite_backward_kernel");
    return GS_OK;
}

int check_backward_buffers(const char* fn, const float* state, const int32_t* contributors,
                           const float* grad_backgrounds, int64_t records_count,
                           const float* grad_records, const float* grad_rows) {
    if (!state || !contributors || !grad_backgrounds ||
        (records_count > 0 && (!grad_records || !grad_rows)))
        return fail(GS_ERR_ARGUMENT, std::string(fn) + ": NULL buffer");
    return GS_OK;
}

}  // namespace
}  // namespace gs

extern "C" int gs_composite_forward(const float* records, const float* rows, int row_mode,
                                    const int64_t* primitive_ids, int64_t cameras, int64_t surfels,
                                    int64_t records_count, int64_t rows_count,
                                    const float* backgrounds, const int32_t* point_list,
                                    const int32_t* ranges, int64_t images, int width, int height,
                                    int neural, int flags, float near_plane, float far_plane,
                                    float* maps, float* state, int32_t* contributors,
                                    uint64_t* counters, void* stream) {
    int st = check_composite("gs_composite_forward", records, rows, row_mode, primitive_ids, cameras,
                             surfels, records_count, backgrounds, ranges, images, width, height);
    if (st) return st;
    (void)rows_count;
    if (!maps || !state || !contributors) return fail(GS_ERR_ARGUMENT, "gs_composite_forward: NULL output");
    Params P = common_params(records, rows, row_mode, primitive_ids, cameras, surfels, backgrounds,
                             point_list, ranges, width, height, near_plane, far_plane);
    for (int g = 0; g < 5; ++g) {
        P.out[g] = maps + plane_first(g);
        P.out_px[g] = kMaps;
    }
    P.state = state;
    P.contributors = contributors;
    return launch_forward(P, images, neural, flags, counters, stream);
}

extern "C" int gs_composite_forward_split(const float* records, const float* rows, int row_mode,
                                          const int64_t* primitive_ids, int64_t cameras,
                                          int64_t surfels, int64_t records_count,
                                          int64_t rows_count, const float* backgrounds,
                                          const int32_t* point_list, const int32_t* ranges,
                                          int64_t images, int width, int height, int neural,
                                          int flags, float near_plane, float far_plane,
                                          float* const* planes, const int64_t* plane_strides,
                                          float* median_depth, int64_t median_stride,
                                          int32_t* median_index, const int32_t* selected,
                                          const int32_t* groups, int64_t group_count,
                                          float* state, int32_t* contributors,
                                          uint32_t* warp_masks, int64_t warp_mask_words,
                                          uint64_t* counters, void* stream) {
    int st = check_composite("gs_composite_forward_split", records, rows, row_mode, primitive_ids,
                             cameras, surfels, records_count, backgrounds, ranges, images, width,
                             height);
    if (st) return st;
    (void)rows_count;
    if (!planes || !plane_strides || !state || !contributors)
        return fail(GS_ERR_ARGUMENT, "gs_composite_forward_split: NULL output");
    Params P = common_params(records, rows, row_mode, primitive_ids, cameras, surfels, backgrounds,
                             point_list, ranges, width, height, near_plane, far_plane);
    for (int g = 0; g < 5; ++g) {
        if (!planes[g] || plane_strides[g] < plane_size(g))
            return fail(GS_ERR_ARGUMENT, "gs_composite_forward_split: bad plane " + std::to_string(g));
        P.out[g] = planes[g];
        P.out_px[g] = plane_strides[g];
    }
    if (median_depth && (!median_index || median_stride < 1))
        return fail(GS_ERR_ARGUMENT, "gs_composite_forward_split: median depth needs its index buffer");
    P.median = median_depth;
    P.median_px = median_stride;
    P.median_index = median_index;
    P.state = state;
    P.contributors = contributors;
    if (bool(selected) != bool(groups) || (groups && group_count < 0) || group_count > INT_MAX)
        return fail(GS_ERR_ARGUMENT, "gs_composite_forward_split: bad selected-pixel groups");
    P.selected = reinterpret_cast<const int4*>(selected);
    P.groups = reinterpret_cast<const int4*>(groups);
    if (warp_masks && warp_mask_words < 1)
        return fail(GS_ERR_ARGUMENT, "gs_composite_forward_split: warp masks need a positive plane size");
    P.warp_mask = warp_masks;
    P.warp_mask_words = warp_mask_words;
    return launch_forward(P, images, neural, flags, counters, stream, groups ? group_count : -1);
}

extern "C" int gs_composite_backward(const float* records, const float* rows, int row_mode,
                                     const int64_t* primitive_ids, int64_t cameras, int64_t surfels,
                                     int64_t records_count, int64_t rows_count,
                                     const float* backgrounds, const int32_t* point_list,
                                     const int32_t* ranges, const float* state,
                                     const int32_t* contributors, const float* grad_maps,
                                     int64_t images, int width, int height, int neural,
                                     float near_plane, float far_plane, float* grad_records,
                                     float* grad_xy, float* grad_rows, float* grad_backgrounds,
                                     uint64_t* counters, void* stream) {
    int st = check_composite("gs_composite_backward", records, rows, row_mode, primitive_ids,
                             cameras, surfels, records_count, backgrounds, ranges, images, width,
                             height);
    if (st) return st;
    (void)rows_count;
    if (!grad_maps) return fail(GS_ERR_ARGUMENT, "gs_composite_backward: NULL buffer");
    st = check_backward_buffers("gs_composite_backward", state, contributors, grad_backgrounds,
                                records_count, grad_records, grad_rows);
    if (st) return st;
    Params P = common_params(records, rows, row_mode, primitive_ids, cameras, surfels, backgrounds,
                             point_list, ranges, width, height, near_plane, far_plane);
    P.state = const_cast<float*>(state);
    P.contributors = const_cast<int*>(contributors);
    for (int g = 0; g < 5; ++g) {
        P.gin[g] = grad_maps + plane_first(g);
        P.gin_px[g] = kMaps;
        P.gin_ch[g] = 1;
    }
    P.grad_records = grad_records;
    P.grad_xy = grad_xy;
    P.grad_rows = grad_rows;
    P.grad_backgrounds = grad_backgrounds;
    return launch_backward(P, images, neural, counters, stream);
}

extern "C" int gs_composite_backward_split(const float* records, const float* rows, int row_mode,
                                           const int64_t* primitive_ids, int64_t cameras,
                                           int64_t surfels, int64_t records_count,
                                           int64_t rows_count, const float* backgrounds,
                                           const int32_t* point_list, const int32_t* ranges,
                                           const float* state, const int32_t* contributors,
                                           const float* const* grad_planes,
                                           const int64_t* grad_strides,
                                           const int32_t* median_index,
                                           const float* grad_median, int64_t grad_median_stride,
                                           const int32_t* selected, const int32_t* groups,
                                           int64_t group_count, int64_t images,
                                           int width, int height, int neural, float near_plane,
                                           float far_plane, float* grad_records, float* grad_xy,
                                           float* grad_rows, float* grad_backgrounds,
                                           const uint32_t* warp_masks, int64_t warp_mask_words,
                                           uint64_t* counters, void* stream) {
    int st = check_composite("gs_composite_backward_split", records, rows, row_mode, primitive_ids,
                             cameras, surfels, records_count, backgrounds, ranges, images, width,
                             height);
    if (st) return st;
    (void)rows_count;
    if (!grad_planes || !grad_strides)
        return fail(GS_ERR_ARGUMENT, "gs_composite_backward_split: NULL buffer");
    st = check_backward_buffers("gs_composite_backward_split", state, contributors,
                                grad_backgrounds, records_count, grad_records, grad_rows);
    if (st) return st;
    Params P = common_params(records, rows, row_mode, primitive_ids, cameras, surfels, backgrounds,
                             point_list, ranges, width, height, near_plane, far_plane);
    P.state = const_cast<float*>(state);
    P.contributors = const_cast<int*>(contributors);
    for (int g = 0; g < 5; ++g) {
        if (grad_strides[2 * g] < 0 || grad_strides[2 * g + 1] < 0)
            return fail(GS_ERR_ARGUMENT, "gs_composite_backward_split: negative stride");
        P.gin[g] = grad_planes[g];
        P.gin_px[g] = grad_strides[2 * g];
        P.gin_ch[g] = grad_strides[2 * g + 1];
    }
    if (grad_median && (!median_index || grad_median_stride < 0))
        return fail(GS_ERR_ARGUMENT, "gs_composite_backward_split: median gradient needs its index buffer");
    P.median_index = const_cast<int*>(median_index);
    P.gin_median = grad_median;
    P.gin_median_px = grad_median_stride;
    if (bool(selected) != bool(groups) || (groups && group_count < 0) || group_count > INT_MAX)
        return fail(GS_ERR_ARGUMENT, "gs_composite_backward_split: bad selected-pixel groups");
    P.selected = reinterpret_cast<const int4*>(selected);
    P.groups = reinterpret_cast<const int4*>(groups);
    P.grad_records = grad_records;
    P.grad_xy = grad_xy;
    P.grad_rows = grad_rows;
    P.grad_backgrounds = grad_backgrounds;
    if (warp_masks && warp_mask_words < 1)
        return fail(GS_ERR_ARGUMENT, "gs_composite_backward_split: warp masks need a positive plane size");
    P.warp_mask = const_cast<unsigned*>(warp_masks);
    P.warp_mask_words = warp_mask_words;
    return launch_backward(P, images, neural, counters, stream, groups ? group_count : -1);
}
