// Fused per-(scene, surfel) projection: splat setup, culling, SH colours and
// record packing (forward), and its hand-derived reverse pass (backward).
//
// Forward restates src/gabor_splatting/rendering.py:156-218 (quaternion_matrix,
// project_surfaces), rendering.py:334-374 (colour evaluation and record packing)
// and spherical_harmonics.cu:45-85.  The reference runs ~30 PyTorch launches over
// [S, C, N] for this and lets autograd build the reverse graph; here one thread
// owns one surfel of one scene, loops over the scene's cameras, and reads the
// surfel's parameters once.  The element-wise parts use explicitly rounded
// multiplies/adds in the order PyTorch's separate element-wise kernels round them,
// so screen radii and tile bounds (hard ceil/trunc decisions) agree with the
// reference's projection.
//
// Backward replaces the autograd graph of those ops: surfel gradients (mean,
// quaternion, scales, opacity, SH coefficients, wave parameters) are summed over
// the cameras in registers, camera gradients (view rotation/translation,
// intrinsics) are reduced per block in shared memory and added with one atomic per
// value per block.
#include "common.cuh"
#include "sh.cuh"

namespace gs {
namespace {

constexpr int kProjThreads = 256;
constexpr float kMinRadius = 3 * 0.707106f;   // rendering.py:208

// Sums in the order PyTorch's CUDA reduction over a last dimension of 3 or 4 uses:
// (a0 + a2) + a1 and (a0 + a2) + (a1 + a3), each add rounded.
__device__ __forceinline__ float sum3(float a0, float a1, float a2) {
    return __fadd_rn(__fadd_rn(a0, a2), a1);
}
__device__ __forceinline__ float sum4(float a0, float a1, float a2, float a3) {
    return __fadd_rn(__fadd_rn(a0, a2), __fadd_rn(a1, a3));
}

struct Surfel {
    float mean[3], q[4], qn[4], qnorm, scale[2], R[3][3], tangent[3][2];
};

struct Camera {
    float Rc[3][3], tc[3], K[3][3];
};

__device__ __forceinline__ void load_surfel(Surfel& v, const float* means, const float* quats,
                                            const float* scales, int64_t sn) {
#pragma unroll
    for (int i = 0; i < 3; ++i) v.mean[i] = means[sn * 3 + i];
    float4 q = reinterpret_cast<const float4*>(quats)[sn];
    v.q[0] = q.x; v.q[1] = q.y; v.q[2] = q.z; v.q[3] = q.w;
    float2 sc = reinterpret_cast<const float2*>(scales)[sn];
    v.scale[0] = sc.x; v.scale[1] = sc.y;
    // q / ||q|| (rendering.py:158)
    float ss = sum4(__fmul_rn(q.x, q.x), __fmul_rn(q.y, q.y), __fmul_rn(q.z, q.z),
                    __fmul_rn(q.w, q.w));
    v.qnorm = sqrtf(ss);
#pragma unroll
    for (int i = 0; i < 4; ++i) v.qn[i] = __fdiv_rn(v.q[i], v.qnorm);
    const float w = v.qn[0], x = v.qn[1], y = v.qn[2], z = v.qn[3];
    // rendering.py:160-172, each product and sum rounded like the element-wise ops
    v.R[0][0] = __fsub_rn(1.f, __fmul_rn(2.f, __fadd_rn(__fmul_rn(y, y), __fmul_rn(z, z))));
    v.R[0][1] = __fmul_rn(2.f, __fsub_rn(__fmul_rn(x, y), __fmul_rn(w, z)));
    v.R[0][2] = __fmul_rn(2.f, __fadd_rn(__fmul_rn(x, z), __fmul_rn(w, y)));
    v.R[1][0] = __fmul_rn(2.f, __fadd_rn(__fmul_rn(x, y), __fmul_rn(w, z)));
    v.R[1][1] = __fsub_rn(1.f, __fmul_rn(2.f, __fadd_rn(__fmul_rn(x, x), __fmul_rn(z, z))));
    v.R[1][2] = __fmul_rn(2.f, __fsub_rn(__fmul_rn(y, z), __fmul_rn(w, x)));
    v.R[2][0] = __fmul_rn(2.f, __fsub_rn(__fmul_rn(x, z), __fmul_rn(w, y)));
    v.R[2][1] = __fmul_rn(2.f, __fadd_rn(__fmul_rn(y, z), __fmul_rn(w, x)));
    v.R[2][2] = __fsub_rn(1.f, __fmul_rn(2.f, __fadd_rn(__fmul_rn(x, x), __fmul_rn(y, y))));
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j) v.tangent[i][j] = __fmul_rn(v.R[i][j], v.scale[j]);
}

__device__ __forceinline__ void load_camera(Camera& cam, const float* views, const float* intr,
                                            int64_t sc) {
    const float* V = views + sc * 16;
    const float* K = intr + sc * 9;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            cam.Rc[i][j] = __ldg(V + i * 4 + j);
            cam.K[i][j] = __ldg(K + i * 3 + j);
        }
        cam.tc[i] = __ldg(V + i * 4 + 3);
    }
}

// Three-term inner product accumulated as a fused multiply-add chain.
__device__ __forceinline__ float dot3(float a0, float b0, float a1, float b1, float a2, float b2) {
    return __fmaf_rn(a2, b2, __fmaf_rn(a1, b1, __fmul_rn(a0, b0)));
}

struct Pair {
    float cm[3], plane[3][3], T[3][3], denom, f[3], xy[2], normal[3], sign, dvec[3], dnorm,
        dir[3];
    bool valid;
};

// Forward splat setup of one (camera, surfel) pair: rendering.py:180-206.
__device__ __forceinline__ void setup_pair(Pair& p, const Surfel& v, const Camera& c) {
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        p.cm[i] = __fadd_rn(dot3(c.Rc[i][0], v.mean[0], c.Rc[i][1], v.mean[1], c.Rc[i][2], v.mean[2]),
                            c.tc[i]);
#pragma unroll
        for (int j = 0; j < 2; ++j)
            p.plane[i][j] = dot3(c.Rc[i][0], v.tangent[0][j], c.Rc[i][1], v.tangent[1][j],
                                 c.Rc[i][2], v.tangent[2][j]);
        p.plane[i][2] = p.cm[i];
    }
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j)
            p.T[i][j] = dot3(c.K[i][0], p.plane[0][j], c.K[i][1], p.plane[1][j], c.K[i][2],
                             p.plane[2][j]);
    const float t[3] = {9.f, 9.f, -1.f};
    float dt[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) dt[j] = __fmul_rn(t[j], __fmul_rn(p.T[2][j], p.T[2][j]));
    const float d = sum3(dt[0], dt[1], dt[2]);
    p.denom = d;
    p.valid = d != 0.f;
    float safe = p.valid ? d : 1.f;
#pragma unroll
    for (int j = 0; j < 3; ++j) p.f[j] = __fdiv_rn(t[j], safe);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        float term[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) term[j] = __fmul_rn(__fmul_rn(p.f[j], p.T[i][j]), p.T[2][j]);
        p.xy[i] = sum3(term[0], term[1], term[2]);
    }
    float n[3];
#pragma unroll
    for (int i = 0; i < 3; ++i)
        n[i] = dot3(c.Rc[i][0], v.R[0][2], c.Rc[i][1], v.R[1][2], c.Rc[i][2], v.R[2][2]);
    float facing = -sum3(__fmul_rn(p.cm[0], n[0]), __fmul_rn(p.cm[1], n[1]),
                         __fmul_rn(p.cm[2], n[2]));
    p.sign = facing > 0.f ? 1.f : -1.f;
#pragma unroll
    for (int i = 0; i < 3; ++i) p.normal[i] = __fmul_rn(n[i], p.sign);
    // camera centre -Rc^T t and the unit world direction centre -> mean
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        float center = -dot3(c.Rc[0][i], c.tc[0], c.Rc[1][i], c.tc[1], c.Rc[2][i], c.tc[2]);
        p.dvec[i] = __fsub_rn(v.mean[i], center);
    }
    p.dnorm = fmaxf(sqrtf(sum3(__fmul_rn(p.dvec[0], p.dvec[0]), __fmul_rn(p.dvec[1], p.dvec[1]),
                               __fmul_rn(p.dvec[2], p.dvec[2]))), 1e-12f);
#pragma unroll
    for (int i = 0; i < 3; ++i) p.dir[i] = __fdiv_rn(p.dvec[i], p.dnorm);
    // facing is kept in sign; culling needs it non-zero
    p.sign = facing == 0.f ? 0.f : p.sign;
}

// Unit world direction from the camera centre -Rc^T t to the surfel mean
// (rendering.py:202-206), rounded like setup_pair.
__device__ __forceinline__ void view_direction(const Surfel& v, const Camera& c, float* dir) {
    float d[3];
#pragma unroll
    for (int i = 0; i < 3; ++i) {
        float center = -dot3(c.Rc[0][i], c.tc[0], c.Rc[1][i], c.tc[1], c.Rc[2][i], c.tc[2]);
        d[i] = __fsub_rn(v.mean[i], center);
    }
    const float norm = fmaxf(sqrtf(sum3(__fmul_rn(d[0], d[0]), __fmul_rn(d[1], d[1]),
                                        __fmul_rn(d[2], d[2]))), 1e-12f);
#pragma unroll
    for (int i = 0; i < 3; ++i) dir[i] = __fdiv_rn(d[i], norm);
}

// Screen radius and visibility: rendering.py:194-217.
__device__ __forceinline__ int pair_radius(const Pair& p, int tw, int th, float near_plane,
                                           float far_plane) {
    float extent[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        float term[3];
#pragma unroll
        for (int j = 0; j < 3; ++j) term[j] = __fmul_rn(p.f[j], __fmul_rn(p.T[i][j], p.T[i][j]));
        float e2 = __fsub_rn(__fmul_rn(p.xy[i], p.xy[i]), sum3(term[0], term[1], term[2]));
        extent[i] = sqrtf(fmaxf(e2, 1e-4f));
    }
    float radius = ceilf(fmaxf(fmaxf(extent[0], extent[1]), kMinRadius));
    bool visible = p.valid && p.sign != 0.f && p.cm[2] > near_plane && p.cm[2] < far_plane;
    visible = visible && isfinite(radius) && radius < 1073741824.f && isfinite(p.xy[0]) &&
              isfinite(p.xy[1]);
    if (!visible) return 0;
    // x / 16 is exact in binary floating point: the product with 1/16 rounds to the same
    // value as the division, without a division sequence
    constexpr float kInvTile = 1.f / kTile;
    const float lim[2] = {float(tw), float(th)};
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        float lower = fmaxf(truncf(__fmul_rn(__fsub_rn(p.xy[i], radius), kInvTile)), 0.f);
        float upper =
            fmaxf(truncf(__fmul_rn(__fadd_rn(__fadd_rn(p.xy[i], radius), float(kTile - 1)), kInvTile)),
                  0.f);
        if (!(fminf(upper, lim[i]) > fminf(lower, lim[i]))) return 0;
    }
    return int(radius);
}

template <int Degree>
__global__ __launch_bounds__(kProjThreads) void project_forward_kernel(
    const float* __restrict__ means, const float* __restrict__ quats,
    const float* __restrict__ scales, const float* __restrict__ opacities,
    const float* __restrict__ views, const float* __restrict__ intr,
    const float* __restrict__ sh_first, const float* __restrict__ sh_second,
    const float* __restrict__ fweights, const float* __restrict__ fmags,
    const float* __restrict__ fphases, int64_t C, int64_t N, const int64_t* __restrict__ offsets,
    int tw, int th, float near_plane, float far_plane, float4* __restrict__ records,
    float2* __restrict__ xy_out, float4* __restrict__ app_rows, int* __restrict__ radii) {
    const int64_t n = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t s = blockIdx.y;
    // ragged batches: scene s owns surfels [offsets[s], offsets[s+1]) and its pairs
    // start at C * offsets[s], camera-major like the dense layout
    const int64_t base = offsets ? offsets[s] : s * N;
    if (offsets) N = offsets[s + 1] - base;
    if (n >= N) return;
    const int64_t sn = base + n;
    Surfel v;
    load_surfel(v, means, quats, scales, sn);
    const float opacity = opacities[sn];
    constexpr int K = Degree >= 0 ? (Degree + 1) * (Degree + 1) : 1;
    float4 wv, mv, pv;
    if constexpr (Degree >= 0) {
        wv = reinterpret_cast<const float4*>(fweights)[sn];
        mv = reinterpret_cast<const float4*>(fmags)[sn];
        pv = reinterpret_cast<const float4*>(fphases)[sn];
    }
    // Appearance rows with SH colours: both colour sets' coefficients are loaded once
    // into registers, both colours are evaluated inside the camera loop and each
    // 80-byte row is written at once (five 16-byte stores, no partially written
    // sectors).  Re-reading the coefficient sets per camera from L1/L2 instead made the
    // kernel wait on those loads, and more so the more threads an SM held (their sets
    // no longer fitting L1).
    float coef[Degree >= 0 ? 2 : 1][K * 3];
    if constexpr (Degree >= 0) {
#pragma unroll
        for (int set = 0; set < 2; ++set) {
            const float4* src = reinterpret_cast<const float4*>(
                (set == 0 ? sh_first : sh_second) + sn * K * 3);
            if constexpr ((K * 3) % 4 == 0) {
                // 12 or 48 floats per set: every set starts 16-byte aligned
#pragma unroll
                for (int i = 0; i < K * 3 / 4; ++i) {
                    const float4 q = __ldg(src + i);
                    coef[set][4 * i] = q.x; coef[set][4 * i + 1] = q.y;
                    coef[set][4 * i + 2] = q.z; coef[set][4 * i + 3] = q.w;
                }
            } else {
                // 3 or 27 floats per set: sets start 4-byte aligned only
#pragma unroll
                for (int i = 0; i < K * 3; ++i)
                    coef[set][i] = __ldg(reinterpret_cast<const float*>(src) + i);
            }
        }
    }
    for (int64_t c = 0; c < C; ++c) {
        Camera cam;
        load_camera(cam, views, intr, s * C + c);
        Pair p;
        setup_pair(p, v, cam);
        const int64_t pid = C * base + c * N + n;
        float4* rec = records + pid * (kRec / 4);
        rec[0] = make_float4(p.T[0][0], p.T[0][1], p.T[0][2], p.T[1][0]);
        rec[1] = make_float4(p.T[1][1], p.T[1][2], p.T[2][0], p.T[2][1]);
        rec[2] = make_float4(p.T[2][2], p.xy[0], p.xy[1], p.normal[0]);
        rec[3] = make_float4(p.normal[1], p.normal[2], p.dir[0], p.dir[1]);
        rec[4] = make_float4(p.dir[2], opacity, 0.f, 0.f);
        xy_out[pid] = make_float2(p.xy[0], p.xy[1]);
        radii[pid] = pair_radius(p, tw, th, near_plane, far_plane);
        if constexpr (Degree >= 0) {
            float4* row = app_rows + pid * (GS_CLASSIC_ROW_FLOATS / 4);
            {
                // both clamped SH colours of the pair's view direction (the direction
                // spherical_harmonics.cu evaluates)
                float basis[K], col[6];
                sh_basis<Degree>(p.dir[0], p.dir[1], p.dir[2], basis);
#pragma unroll
                for (int set = 0; set < 2; ++set) {
#pragma unroll
                    for (int ch = 0; ch < 3; ++ch) {
                        float raw = 0.5f;
#pragma unroll
                        for (int k = 0; k < K; ++k) raw += basis[k] * coef[set][k * 3 + ch];
                        col[set * 3 + ch] = fmaxf(raw, 0.f);
                    }
                }
                row[0] = make_float4(col[0], col[1], col[2], col[3]);
                row[1] = make_float4(col[4], col[5], wv.x, wv.y);
            }
            row[2] = make_float4(wv.z, wv.w, mv.x, mv.y);
            row[3] = make_float4(mv.z, mv.w, pv.x, pv.y);
            row[4] = make_float4(pv.z, pv.w, 0.f, 0.f);
        }
    }
}

// ------------------------------------------------------------------------------
// backward
// ------------------------------------------------------------------------------
constexpr int kCamGrads = 21;   // Rc (9), t (3), K (9)

template <int Degree>
// Two blocks per SM (128 registers, a few spilled): the per-pair gathers need the
// extra warps in flight more than the registers.
__global__ __launch_bounds__(kProjThreads, 2) void project_backward_kernel(
    const float* __restrict__ means, const float* __restrict__ quats,
    const float* __restrict__ scales, const float* __restrict__ views,
    const float* __restrict__ intr, const float* __restrict__ sh_first,
    const float* __restrict__ sh_second, int64_t C, int64_t N,
    const float* __restrict__ grad_records, const float* __restrict__ grad_xy,
    const float* __restrict__ grad_rows, float* __restrict__ g_means,
    float* __restrict__ g_quats, float* __restrict__ g_scales, float* __restrict__ g_opac,
    float* __restrict__ g_views, float* __restrict__ g_intr, float* __restrict__ g_sh1,
    float* __restrict__ g_sh2, float* __restrict__ g_w, float* __restrict__ g_m,
    float* __restrict__ g_p, int64_t chunks, const int64_t* __restrict__ offsets) {
    extern __shared__ float cam_acc[];   // [C][kCamGrads], C <= kMaxSharedCameras
    const int lane = threadIdx.x & 31;
    const int64_t s = blockIdx.y;
    const bool shared_cams = C * kCamGrads * sizeof(float) <= 32768;
    if (shared_cams) {
        for (int i = threadIdx.x; i < C * kCamGrads; i += blockDim.x) cam_acc[i] = 0.f;
        __syncthreads();
    }
    constexpr int K = Degree >= 0 ? (Degree + 1) * (Degree + 1) : 1;
    const int64_t base = offsets ? offsets[s] : s * N;   // ragged batches as in the forward
    if (offsets) N = offsets[s + 1] - base;
    for (int64_t chunk = blockIdx.x; chunk < chunks; chunk += gridDim.x) {
        const int64_t n = chunk * blockDim.x + threadIdx.x;
        const bool live = n < N;
        const int64_t sn = base + (live ? n : 0);
        Surfel v;
        load_surfel(v, means, quats, scales, sn);
        float gR[3][3] = {}, gmean[3] = {}, gscale[2] = {}, gop = 0.f;
        float gw[4] = {}, gm[4] = {}, gph[4] = {};
        for (int64_t c = 0; c < C; ++c) {
            const int64_t pid = C * base + c * N + (live ? n : 0);
            float gr[kRec], gxy[2], gcol[6] = {};
            if (live) {
                const float4* g4 = reinterpret_cast<const float4*>(grad_records) + pid * (kRec / 4);
#pragma unroll
                for (int i = 0; i < kRec / 4; ++i) {
                    float4 t = g4[i];
                    gr[4 * i] = t.x; gr[4 * i + 1] = t.y; gr[4 * i + 2] = t.z; gr[4 * i + 3] = t.w;
                }
                float2 t = reinterpret_cast<const float2*>(grad_xy)[pid];
                gxy[0] = t.x; gxy[1] = t.y;
                if constexpr (Degree >= 0) {
                    // the row's 18 gradients as five 16-byte loads (rows are 80 bytes)
                    const float4* row4 = reinterpret_cast<const float4*>(grad_rows) +
                                         pid * (GS_CLASSIC_ROW_FLOATS / 4);
                    float row[20];
#pragma unroll
                    for (int i = 0; i < 5; ++i) {
                        const float4 q = row4[i];
                        row[4 * i] = q.x; row[4 * i + 1] = q.y;
                        row[4 * i + 2] = q.z; row[4 * i + 3] = q.w;
                    }
#pragma unroll
                    for (int i = 0; i < 6; ++i) gcol[i] = row[i];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        gw[i] += row[6 + i];
                        gm[i] += row[10 + i];
                        gph[i] += row[14 + i];
                    }
                }
            } else {
#pragma unroll
                for (int i = 0; i < kRec; ++i) gr[i] = 0.f;
                gxy[0] = gxy[1] = 0.f;
            }
            gop += gr[17];
            bool any = gxy[0] != 0.f || gxy[1] != 0.f;
#pragma unroll
            for (int i = 0; i < 17; ++i) any = any || (i != 9 && i != 10 && gr[i] != 0.f);
#pragma unroll
            for (int i = 0; i < 6; ++i) any = any || gcol[i] != 0.f;
            float gcam[kCamGrads] = {};
            if (any) {
                Camera cam;
                load_camera(cam, views, intr, s * C + c);
                Pair p;
                setup_pair(p, v, cam);
                float gdir[3] = {gr[14], gr[15], gr[16]};
                if constexpr (Degree >= 0) {
                    // direction gradient of both clamped SH colours
                    // (spherical_harmonics.cu:65-75); coefficient gradients are
                    // accumulated after the camera loop.
                    sh_direction_grad<Degree>(p.dir, sh_first + sn * K * 3, sh_second + sn * K * 3,
                                              gcol, gdir);
                }
                // T = K plane: gT from the record, plus the conic-centre path xy(T).
                float gT[3][3];
#pragma unroll
                for (int i = 0; i < 3; ++i)
#pragma unroll
                    for (int j = 0; j < 3; ++j) gT[i][j] = gr[i * 3 + j];
                {
                    // xy_i = sum_j f_j T_ij T_2j, f_j = t_j / denom, denom = sum_j t_j T_2j^2
                    const float t[3] = {9.f, 9.f, -1.f};
                    float gf[3];
#pragma unroll
                    for (int j = 0; j < 3; ++j) {
                        gf[j] = 0.f;
#pragma unroll
                        for (int i = 0; i < 2; ++i) {
                            gT[i][j] += gxy[i] * p.f[j] * p.T[2][j];
                            gT[2][j] += gxy[i] * p.f[j] * p.T[i][j];
                            gf[j] += gxy[i] * p.T[i][j] * p.T[2][j];
                        }
                    }
                    if (p.valid) {
                        float gden = 0.f;
                        const float inv_denom = 1.f / p.denom;
#pragma unroll
                        for (int j = 0; j < 3; ++j) gden -= gf[j] * p.f[j] * inv_denom;
#pragma unroll
                        for (int j = 0; j < 3; ++j) gT[2][j] += gden * 2.f * t[j] * p.T[2][j];
                    }
                }
                // K and plane
                float gplane[3][3];
#pragma unroll
                for (int i = 0; i < 3; ++i)
#pragma unroll
                    for (int k = 0; k < 3; ++k) {
                        float acc = 0.f, accp = 0.f;
#pragma unroll
                        for (int j = 0; j < 3; ++j) {
                            acc += gT[i][j] * p.plane[k][j];
                            accp += cam.K[j][i] * gT[j][k];
                        }
                        gcam[12 + i * 3 + k] = acc;
                        gplane[i][k] = accp;
                    }
                // normal n = sign * Rc R[:,2]
                float gn[3] = {gr[11] * p.sign, gr[12] * p.sign, gr[13] * p.sign};
                // direction: dir = dvec / max(|dvec|, 1e-12), dvec = mean + Rc^T t
                float gd[3];
                {
                    const float inv = 1.f / p.dnorm;
                    const float dd = gdir[0] * p.dir[0] + gdir[1] * p.dir[1] + gdir[2] * p.dir[2];
                    const bool clamped = !(p.dnorm > 1e-12f);
#pragma unroll
                    for (int i = 0; i < 3; ++i)
                        gd[i] = clamped ? gdir[i] * inv : (gdir[i] - p.dir[i] * dd) * inv;
                }
#pragma unroll
                for (int i = 0; i < 3; ++i) {
                    gmean[i] += gd[i];
                    // dvec_i = mean_i + sum_j Rc_ji t_j
#pragma unroll
                    for (int j = 0; j < 3; ++j) {
                        gcam[j * 3 + i] += gd[i] * cam.tc[j];
                    }
                }
#pragma unroll
                for (int j = 0; j < 3; ++j)
                    gcam[9 + j] += cam.Rc[j][0] * gd[0] + cam.Rc[j][1] * gd[1] + cam.Rc[j][2] * gd[2];
                // plane = [Rc tangent | Rc mean + t]
#pragma unroll
                for (int i = 0; i < 3; ++i) {
                    gcam[9 + i] += gplane[i][2];
#pragma unroll
                    for (int k = 0; k < 3; ++k) {
                        gcam[i * 3 + k] += gplane[i][0] * v.tangent[k][0] +
                                           gplane[i][1] * v.tangent[k][1] +
                                           gplane[i][2] * v.mean[k] + gn[i] * v.R[k][2];
                    }
                }
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    float gt0 = 0.f, gt1 = 0.f, gmk = 0.f, gr2 = 0.f;
#pragma unroll
                    for (int i = 0; i < 3; ++i) {
                        gt0 += cam.Rc[i][k] * gplane[i][0];
                        gt1 += cam.Rc[i][k] * gplane[i][1];
                        gmk += cam.Rc[i][k] * gplane[i][2];
                        gr2 += cam.Rc[i][k] * gn[i];
                    }
                    gmean[k] += gmk;
                    gR[k][0] += gt0 * v.scale[0];
                    gR[k][1] += gt1 * v.scale[1];
                    gR[k][2] += gr2;
                    gscale[0] += gt0 * v.R[k][0];
                    gscale[1] += gt1 * v.R[k][1];
                }
            }
            // camera gradients: reduce over the warp, then over the block
            unsigned any_mask = __ballot_sync(0xffffffffu, any);
            if (any_mask) {
                float red[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) red[i] = i < kCamGrads ? gcam[i] : 0.f;
                warp_reduce_scatter<32>(red, lane);
                if (lane < kCamGrads && red[0] != 0.f) {
                    if (shared_cams) {
                        atomicAdd(cam_acc + c * kCamGrads + lane, red[0]);
                    } else {
                        const int64_t sc = s * C + c;
                        float* dst = lane < 12 ? g_views + sc * 16 + (lane < 9 ? (lane / 3) * 4 + lane % 3
                                                                               : (lane - 9) * 4 + 3)
                                               : g_intr + sc * 9 + (lane - 12);
                        atomicAdd(dst, red[0]);
                    }
                }
            }
        }
        if constexpr (Degree >= 0 && Degree <= 1) {
            if (live) {
                // SH coefficient gradients, degrees 0-1 (degrees 2-3:
                // sh_coefficient_grad_kernel): the sum over the scene's cameras of
                // g * basis(dir) where the clamp passes, per (colour set, channel), both
                // sets in one pass after the camera loop (6K accumulators), each camera's
                // direction and basis evaluated once and its six colour gradients read with
                // two vector loads.  Per accumulator the cameras add in order.
                constexpr int kSets = 2;
#pragma unroll 1
                for (int pass = 0; pass < 2 / kSets; ++pass) {
                    float acc[kSets][3][K];
#pragma unroll
                    for (int t = 0; t < kSets; ++t)
#pragma unroll
                        for (int ch = 0; ch < 3; ++ch)
#pragma unroll
                            for (int k = 0; k < K; ++k) acc[t][ch][k] = 0.f;
                    for (int64_t c = 0; c < C; ++c) {
                        const int64_t pid = C * base + c * N + n;
                        const float4* grow =
                            reinterpret_cast<const float4*>(grad_rows) + pid * (GS_CLASSIC_ROW_FLOATS / 4);
                        const float4 q0 = grow[0], q1 = grow[1];
                        const float gall[6] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y};
                        bool any = false;
#pragma unroll
                        for (int t = 0; t < kSets; ++t)
#pragma unroll
                            for (int ch = 0; ch < 3; ++ch)
                                any = any || gall[(pass * kSets + t) * 3 + ch] != 0.f;
                        if (!any) continue;
                        Camera cam;
                        load_camera(cam, views, intr, s * C + c);
                        float dir[3], basis[K];
                        view_direction(v, cam, dir);
                        sh_basis<Degree>(dir[0], dir[1], dir[2], basis);
#pragma unroll
                        for (int t = 0; t < kSets; ++t) {
                            const int set = pass * kSets + t;
                            const float* cf = (set == 0 ? sh_first : sh_second) + sn * K * 3;
#pragma unroll
                            for (int ch = 0; ch < 3; ++ch) {
                                const float g = gall[set * 3 + ch];
                                if (g == 0.f) continue;
                                float raw = 0.5f;
#pragma unroll
                                for (int k = 0; k < K; ++k) raw += basis[k] * __ldg(cf + k * 3 + ch);
                                if (raw >= 0.f) {
#pragma unroll
                                    for (int k = 0; k < K; ++k) acc[t][ch][k] += g * basis[k];
                                }
                            }
                        }
                    }
#pragma unroll
                    for (int t = 0; t < kSets; ++t) {
                        const int set = pass * kSets + t;
                        float* gco = (set == 0 ? g_sh1 : g_sh2) + sn * K * 3;
#pragma unroll
                        for (int ch = 0; ch < 3; ++ch)
#pragma unroll
                            for (int k = 0; k < K; ++k) gco[k * 3 + ch] = acc[t][ch][k];
                    }
                }
            }
        }
        if (live) {
            // quaternion_matrix backward through the normalisation (rendering.py:156-173)
            const float w = v.qn[0], x = v.qn[1], y = v.qn[2], z = v.qn[3];
            float gq[4];
            gq[0] = 2.f * (-z * gR[0][1] + y * gR[0][2] + z * gR[1][0] - x * gR[1][2] -
                           y * gR[2][0] + x * gR[2][1]);
            gq[1] = 2.f * (y * gR[0][1] + z * gR[0][2] + y * gR[1][0] - w * gR[1][2] +
                           z * gR[2][0] + w * gR[2][1]) -
                    4.f * x * (gR[1][1] + gR[2][2]);
            gq[2] = 2.f * (x * gR[0][1] + w * gR[0][2] + x * gR[1][0] + z * gR[1][2] -
                           w * gR[2][0] + z * gR[2][1]) -
                    4.f * y * (gR[0][0] + gR[2][2]);
            gq[3] = 2.f * (-w * gR[0][1] + x * gR[0][2] + w * gR[1][0] + y * gR[1][2] +
                           x * gR[2][0] + y * gR[2][1]) -
                    4.f * z * (gR[0][0] + gR[1][1]);
            const float dq = gq[0] * w + gq[1] * x + gq[2] * y + gq[3] * z;
            float4 out;
            out.x = (gq[0] - w * dq) / v.qnorm;
            out.y = (gq[1] - x * dq) / v.qnorm;
            out.z = (gq[2] - y * dq) / v.qnorm;
            out.w = (gq[3] - z * dq) / v.qnorm;
            reinterpret_cast<float4*>(g_quats)[sn] = out;
#pragma unroll
            for (int i = 0; i < 3; ++i) g_means[sn * 3 + i] = gmean[i];
            reinterpret_cast<float2*>(g_scales)[sn] = make_float2(gscale[0], gscale[1]);
            g_opac[sn] = gop;
            if constexpr (Degree >= 0) {
                reinterpret_cast<float4*>(g_w)[sn] = make_float4(gw[0], gw[1], gw[2], gw[3]);
                reinterpret_cast<float4*>(g_m)[sn] = make_float4(gm[0], gm[1], gm[2], gm[3]);
                reinterpret_cast<float4*>(g_p)[sn] = make_float4(gph[0], gph[1], gph[2], gph[3]);
            }
        }
    }
    if (shared_cams) {
        __syncthreads();
        for (int i = threadIdx.x; i < C * kCamGrads; i += blockDim.x) {
            float val = cam_acc[i];
            if (val == 0.f) continue;
            const int64_t sc = s * C + i / kCamGrads;
            const int k = i % kCamGrads;
            float* dst = k < 12 ? g_views + sc * 16 + (k < 9 ? (k / 3) * 4 + k % 3 : (k - 9) * 4 + 3)
                                : g_intr + sc * 9 + (k - 12);
            atomicAdd(dst, val);
        }
    }
}

// SH coefficient gradients of degrees 2-3 (spherical_harmonics.cu:128-150 under the
// clamp of its forward, :80-85): per (surfel, colour set, channel), the sum over the
// scene's cameras, in camera order, of g * basis(dir) for the cameras whose unclamped
// colour is >= 0.  Eight lanes per surfel, six of them busy: each holds its channel's K
// coefficients and K accumulators, reads its one colour gradient per camera (a surfel's
// six lanes read the first 24 bytes of the pair's gradient row together) and recomputes
// the pair's direction and basis.  Inside project_backward_kernel the 6K accumulators
// of these degrees did not fit, and one pass per colour set after the camera loop
// re-read every pair's gradient row from DRAM (config 4: 3.19 -> 2.71 ms, config 1
// 0.46 -> 0.33 ms).  Every coefficient gradient of the launch is written.
constexpr int kShLanes = 8;

template <int Degree>
__global__ __launch_bounds__(kProjThreads) void sh_coefficient_grad_kernel(
    const float* __restrict__ means, const float* __restrict__ views,
    const float* __restrict__ intr, const float* __restrict__ sh_first,
    const float* __restrict__ sh_second, int64_t C, int64_t N,
    const int64_t* __restrict__ offsets, const float* __restrict__ grad_rows,
    float* __restrict__ g_sh1, float* __restrict__ g_sh2) {
    constexpr int K = (Degree + 1) * (Degree + 1);
    const int64_t s = blockIdx.y;
    const int64_t base = offsets ? offsets[s] : s * N;   // ragged batches as in the forward
    if (offsets) N = offsets[s + 1] - base;
    const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t n = t / kShLanes;
    const int sub = int(t % kShLanes);   // colour set sub / 3, channel sub % 3
    if (n >= N || sub >= 6) return;
    const int64_t sn = base + n;
    Surfel v;   // view_direction reads the mean only
#pragma unroll
    for (int i = 0; i < 3; ++i) v.mean[i] = means[sn * 3 + i];
    const int64_t at = sn * K * 3 + sub % 3;
    const float* cf = (sub < 3 ? sh_first : sh_second) + at;
    float coef[K], acc[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
        coef[k] = __ldg(cf + k * 3);
        acc[k] = 0.f;
    }
    for (int64_t c = 0; c < C; ++c) {
        const float g = grad_rows[(C * base + c * N + n) * GS_CLASSIC_ROW_FLOATS + sub];
        if (g == 0.f) continue;
        Camera cam;
        load_camera(cam, views, intr, s * C + c);
        float dir[3], basis[K];
        view_direction(v, cam, dir);
        sh_basis<Degree>(dir[0], dir[1], dir[2], basis);
        float raw = 0.5f;
#pragma unroll
        for (int k = 0; k < K; ++k) raw += basis[k] * coef[k];
        if (raw >= 0.f) {
#pragma unroll
            for (int k = 0; k < K; ++k) acc[k] += g * basis[k];
        }
    }
    float* out = (sub < 3 ? g_sh1 : g_sh2) + at;
#pragma unroll
    for (int k = 0; k < K; ++k) out[k * 3] = acc[k];
}

}  // namespace
}  // namespace gs

using namespace gs;

// The kernels move quaternions, records, appearance rows, wave parameters and their
// gradients as 16-byte vectors and scales and screen centres as 8-byte vectors: their
// buffers must start on those boundaries (every row then does too).
static bool misaligned(const void* p, uintptr_t bytes) {
    return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) != 0;
}

static int project_forward_impl(const char* fn, const int64_t* offsets, const float* means,
                                const float* quaternions, const float* scales,
                                  const float* opacities, const float* view_matrices,
                                  const float* intrinsics, const float* sh_first,
                                  const float* sh_second, const float* frequency_weights,
                                  const float* frequency_magnitudes, const float* phases,
                                  int sh_degree, int64_t scenes, int64_t cameras, int64_t surfels,
                                  int width, int height, float near_plane, float far_plane,
                                  float* records, float* xy, float* app_rows, int32_t* radii,
                                  void* stream) {
    if (scenes < 1 || cameras < 1 || surfels < 0 || width < 1 || height < 1)
        return fail(GS_ERR_ARGUMENT, std::string(fn) + ": invalid sizes");
    if (sh_degree > 3) return fail(GS_ERR_ARGUMENT, std::string(fn) + ": SH degree must be 0-3");
    if (scenes > 65535) return fail(GS_ERR_LIMIT, std::string(fn) + ": more than 65535 scenes");
    if (surfels == 0) return GS_OK;
    if (sh_degree >= 0 && (!sh_first || !sh_second || !frequency_weights || !frequency_magnitudes ||
                           !phases || !app_rows))
        return fail(GS_ERR_ARGUMENT, std::string(fn) + ": SH mode needs coefficient and row buffers");
    if (misaligned(quaternions, 16) || misaligned(records, 16) || misaligned(scales, 8) ||
        misaligned(xy, 8) ||
        (sh_degree >= 0 && (misaligned(frequency_weights, 16) ||
                            misaligned(frequency_magnitudes, 16) || misaligned(phases, 16) ||
                            misaligned(app_rows, 16))))
        return fail(GS_ERR_ARGUMENT, std::string(fn) + ": quaternions, records, rows and wave "
                                                       "parameters must be 16-byte aligned, "
                                                       "scales and xy 8-byte aligned");
    const int tw = (width + kTile - 1) / kTile, th = (height + kTile - 1) / kTile;
    dim3 grid(unsigned((surfels + kProjThreads - 1) / kProjThreads), unsigned(scenes));
    auto s = as_stream(stream);
    auto* rec = reinterpret_cast<float4*>(records);
    auto* xy2 = reinterpret_cast<float2*>(xy);
    auto* rows = reinterpret_cast<float4*>(app_rows);
#define GS_PROJ(D)                                                                            \
    project_forward_kernel<D><<<grid, kProjThreads, 0, s>>>(                                  \
        means, quaternions, scales, opacities, view_matrices, intrinsics, sh_first, sh_second, \
        frequency_weights, frequency_magnitudes, phases, cameras, surfels, offsets, tw, th,     \
        near_plane, far_plane, rec, xy2, rows, radii)
    switch (sh_degree) {
        case 0: GS_PROJ(0); break;
        case 1: GS_PROJ(1); break;
        case 2: GS_PROJ(2); break;
        case 3: GS_PROJ(3); break;
        default: GS_PROJ(-1); break;
    }
#undef GS_PROJ
    GS_CHECK_LAUNCH("project_forward_kernel");
    return GS_OK;
}

extern "C" int gs_project_forward(const float* means, const float* quaternions, const float* scales,
                                  const float* opacities, const float* view_matrices,
                                  const float* intrinsics, const float* sh_first,
                                  const float* sh_second, const float* frequency_weights,
                                  const float* frequency_magnitudes, const float* phases,
                                  int sh_degree, int64_t scenes, int64_t cameras, int64_t surfels,
                                  int width, int height, float near_plane, float far_plane,
                                  float* records, float* xy, float* app_rows, int32_t* radii,
                                  void* stream) {
    return project_forward_impl("gs_project_forward", nullptr, means, quaternions, scales,
                                opacities, view_matrices, intrinsics, sh_first, sh_second,
                                frequency_weights, frequency_magnitudes, phases, sh_degree, scenes,
                                cameras, surfels, width, height, near_plane, far_plane, records, xy,
                                app_rows, radii, stream);
}

extern "C" int gs_project_forward_ragged(const float* means, const float* quaternions,
                                         const float* scales, const float* opacities,
                                         const float* view_matrices, const float* intrinsics,
                                         const float* sh_first, const float* sh_second,
                                         const float* frequency_weights,
                                         const float* frequency_magnitudes, const float* phases,
                                         int sh_degree, int64_t scenes, int64_t cameras,
                                         const int64_t* scene_offsets, int64_t max_surfels,
                                         int width, int height, float near_plane,
                                         float far_plane, float* records, float* xy,
                                         float* app_rows, int32_t* radii, void* stream) {
    if (!scene_offsets) return fail(GS_ERR_ARGUMENT, "gs_project_forward_ragged: NULL offsets");
    return project_forward_impl("gs_project_forward_ragged", scene_offsets, means, quaternions,
                                scales, opacities, view_matrices, intrinsics, sh_first, sh_second,
                                frequency_weights, frequency_magnitudes, phases, sh_degree, scenes,
                                cameras, max_surfels, width, height, near_plane, far_plane, records,
                                xy, app_rows, radii, stream);
}

static int project_backward_impl(const char* fn, const int64_t* offsets, int64_t total_surfels,
                                 const float* means, const float* quaternions, const float* scales,
                                   const float* view_matrices, const float* intrinsics,
                                   const float* sh_first, const float* sh_second, int sh_degree,
                                   int64_t scenes, int64_t cameras, int64_t surfels,
                                   const float* grad_records, const float* grad_xy,
                                   const float* grad_app_rows, float* grad_means,
                                   float* grad_quaternions, float* grad_scales,
                                   float* grad_opacities, float* grad_view_matrices,
                                   float* grad_intrinsics, float* grad_sh_first,
                                   float* grad_sh_second, float* grad_frequency_weights,
                                   float* grad_frequency_magnitudes, float* grad_phases,
                                   void* stream) {
    if (scenes < 1 || cameras < 1 || surfels < 0)
        return fail(GS_ERR_ARGUMENT, std::string(fn) + ": invalid sizes");
    if (sh_degree > 3) return fail(GS_ERR_ARGUMENT, std::string(fn) + ": SH degree must be 0-3");
    if (scenes > 65535) return fail(GS_ERR_LIMIT, std::string(fn) + ": more than 65535 scenes");
    if (misaligned(quaternions, 16) || misaligned(grad_records, 16) ||
        misaligned(grad_quaternions, 16) || misaligned(scales, 8) || misaligned(grad_xy, 8) ||
        misaligned(grad_scales, 8) ||
        (sh_degree >= 0 && (misaligned(grad_app_rows, 16) ||
                            misaligned(grad_frequency_weights, 16) ||
                            misaligned(grad_frequency_magnitudes, 16) ||
                            misaligned(grad_phases, 16))))
        return fail(GS_ERR_ARGUMENT, std::string(fn) + ": quaternions, record and row gradients "
                                                       "and their 4-vector gradients must be "
                                                       "16-byte aligned, scales and xy 8-byte "
                                                       "aligned");
    auto s = as_stream(stream);
    GS_CUDA(cudaMemsetAsync(grad_view_matrices, 0, sizeof(float) * 16 * scenes * cameras, s));
    GS_CUDA(cudaMemsetAsync(grad_intrinsics, 0, sizeof(float) * 9 * scenes * cameras, s));
    if (sh_degree >= 0 && sh_degree <= 1) {   // degrees 2-3: every one written below
        const int64_t sn = offsets ? total_surfels : scenes * surfels;
        const int64_t K = int64_t(sh_degree + 1) * (sh_degree + 1);
        GS_CUDA(cudaMemsetAsync(grad_sh_first, 0, sizeof(float) * sn * K * 3, s));
        GS_CUDA(cudaMemsetAsync(grad_sh_second, 0, sizeof(float) * sn * K * 3, s));
    }
    if (surfels == 0) return GS_OK;
    const int64_t chunks = (surfels + kProjThreads - 1) / kProjThreads;
    // enough blocks to fill the GPU a few times over, each looping over chunks
    int64_t per_scene = (148 * 8 + scenes - 1) / scenes;
    if (per_scene > chunks) per_scene = chunks;
    if (per_scene < 1) per_scene = 1;
    dim3 grid{unsigned(per_scene), unsigned(scenes)};
    const size_t smem = cameras * kCamGrads * sizeof(float) <= 32768
                            ? size_t(cameras) * kCamGrads * sizeof(float)
                            : 0;
#define GS_PROJ_BWD(D)                                                                          \
    project_backward_kernel<D><<<grid, kProjThreads, smem, s>>>(                                \
        means, quaternions, scales, view_matrices, intrinsics, sh_first, sh_second, cameras,   \
        surfels, grad_records, grad_xy, grad_app_rows, grad_means, grad_quaternions,           \
        grad_scales, grad_opacities, grad_view_matrices, grad_intrinsics, grad_sh_first,       \
        grad_sh_second, grad_frequency_weights, grad_frequency_magnitudes, grad_phases, chunks, \
        offsets)
    switch (sh_degree) {
        case 0: GS_PROJ_BWD(0); break;
        case 1: GS_PROJ_BWD(1); break;
        case 2: GS_PROJ_BWD(2); break;
        case 3: GS_PROJ_BWD(3); break;
        default: GS_PROJ_BWD(-1); break;
    }
#undef GS_PROJ_BWD
    GS_CHECK_LAUNCH("project_backward_kernel");
    if (sh_degree >= 2) {
        const dim3 sh_grid{unsigned((surfels * kShLanes + kProjThreads - 1) / kProjThreads),
                           unsigned(scenes)};
#define GS_SH_GRAD(D)                                                                           \
    sh_coefficient_grad_kernel<D><<<sh_grid, kProjThreads, 0, s>>>(                              \
        means, view_matrices, intrinsics, sh_first, sh_second, cameras, surfels, offsets,      \
        grad_app_rows, grad_sh_first, grad_sh_second)
        if (sh_degree == 2) GS_SH_GRAD(2);
        else GS_SH_GRAD(3);
#undef GS_SH_GRAD
        GS_CHECK_LAUNCH("sh_coefficient_grad_kernel");
    }
    return GS_OK;
}

extern "C" int gs_project_backward(const float* means, const float* quaternions, const float* scales,
                                   const float* view_matrices, const float* intrinsics,
                                   const float* sh_first, const float* sh_second, int sh_degree,
                                   int64_t scenes, int64_t cameras, int64_t surfels,
                                   const float* grad_records, const float* grad_xy,
                                   const float* grad_app_rows, float* grad_means,
                                   float* grad_quaternions, float* grad_scales,
                                   float* grad_opacities, float* grad_view_matrices,
                                   float* grad_intrinsics, float* grad_sh_first,
                                   float* grad_sh_second, float* grad_frequency_weights,
                                   float* grad_frequency_magnitudes, float* grad_phases,
                                   void* stream) {
    return project_backward_impl("gs_project_backward", nullptr, 0, means, quaternions, scales,
                                 view_matrices, intrinsics, sh_first, sh_second, sh_degree, scenes,
                                 cameras, surfels, grad_records, grad_xy, grad_app_rows, grad_means,
                                 grad_quaternions, grad_scales, grad_opacities, grad_view_matrices,
                                 grad_intrinsics, grad_sh_first, grad_sh_second,
                                 grad_frequency_weights, grad_frequency_magnitudes, grad_phases,
                                 stream);
}

extern "C" int gs_project_backward_ragged(
    const float* means, const float* quaternions, const float* scales, const float* view_matrices,
    const float* intrinsics, const float* sh_first, const float* sh_second, int sh_degree,
    int64_t scenes, int64_t cameras, const int64_t* scene_offsets, int64_t max_surfels,
    int64_t total_surfels, const float* grad_records, const float* grad_xy,
    const float* grad_app_rows, float* grad_means, float* grad_quaternions, float* grad_scales,
    float* grad_opacities, float* grad_view_matrices, float* grad_intrinsics,
    float* grad_sh_first, float* grad_sh_second, float* grad_frequency_weights,
    float* grad_frequency_magnitudes, float* grad_phases, void* stream) {
    if (!scene_offsets || total_surfels < 0)
        return fail(GS_ERR_ARGUMENT, "gs_project_backward_ragged: invalid offsets");
    return project_backward_impl("gs_project_backward_ragged", scene_offsets, total_surfels, means,
                                 quaternions, scales, view_matrices, intrinsics, sh_first,
                                 sh_second, sh_degree, scenes, cameras, max_surfels, grad_records,
                                 grad_xy, grad_app_rows, grad_means, grad_quaternions, grad_scales,
                                 grad_opacities, grad_view_matrices, grad_intrinsics,
                                 grad_sh_first, grad_sh_second, grad_frequency_weights,
                                 grad_frequency_magnitudes, grad_phases, stream);
}
