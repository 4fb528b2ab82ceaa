/*
 * gabor_b200.h -- C ABI of the B200-native Gabor surface-splatting render path.
 *
 * One shared library (diff_gabor_splatting_b200/libgabor_b200.so, sm_100a).
 * Every entry point takes plain device pointers, sizes and a cudaStream_t passed
 * as void*, launches asynchronously on that stream, allocates nothing, and returns
 * an int status: 0 on success, otherwise one of GS_ERR_* with a message readable
 * through gs_last_error() (per calling thread).  The only entry point that waits
 * on the stream is gs_bin_count (it returns the number of tile intersections to
 * the host, exactly as the reference does after its CUB scan).
 *
 * Reference interfaces replaced (luisrodolfo10/diff_gabor_splatting v0.1.1):
 *   _C.rasterize_forward   src/gabor_splatting/csrc/rasterize.h:5-9,  rasterize.cu:425-503
 *   _C.rasterize_backward  src/gabor_splatting/csrc/rasterize.h:10-15, rasterize.cu:505-529
 *   _C.evaluate_sh_forward  rasterize.h:18-19, spherical_harmonics.cu:106-126
 *   _C.evaluate_sh_backward rasterize.h:20-21, spherical_harmonics.cu:128-150
 *   PyTorch projection/packing ops  src/gabor_splatting/rendering.py:156-218, 334-374
 *
 * Layouts (all row-major, float32 unless stated):
 *   record  [R][20]  splat record per projected pair: T (3x3 homogeneous plane
 *                    transform, 9), xy (conic centre, 2), normal (3), view dir (3),
 *                    opacity (1), 2 zero pad.  80 bytes, 16-byte aligned.
 *   classic appearance row [A][20]: colour (3), secondary colour (3), frequency
 *                    weights (4), magnitudes (4), phases (4), 2 zero pad.
 *   neural appearance row  [A][60]: W1 (6x5), b1 (6), W2 (3x6), b2 (3), 3 zero pad.
 *   maps   [images][H][W][9]: rgb, alpha, accumulated depth, normal (3), distortion.
 *   state  [images][H][W][3]: final transmittance, m1, m2.
 *   ranges [images*tw*th][2] int32: [start, end) of each 16x16 tile's list.
 */
#ifndef GABOR_B200_H
#define GABOR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GS_OK 0
#define GS_ERR_ARGUMENT 1   /* invalid size, pointer or option */
#define GS_ERR_LIMIT 2      /* a count exceeds an index range the kernels support */
#define GS_ERR_CUDA 3       /* a CUDA runtime call or launch failed */
#define GS_ERR_WORKSPACE 4  /* the workspace passed is smaller than required */

#define GS_RECORD_FLOATS 20
#define GS_CLASSIC_ROW_FLOATS 20
#define GS_NEURAL_ROW_FLOATS 60

/* Appearance-row addressing of a record r (gs_composite_*). */
#define GS_ROWS_PER_RECORD 0   /* row = r */
#define GS_ROWS_PER_SURFEL 1   /* r = (s*C + c)*N + n  ->  row = s*N + n */
#define GS_ROWS_EXPLICIT 2     /* row = primitive_ids[r] (int64) */

int gs_version(void);
const char* gs_last_error(void);

/* ---------------------------------------------------------------------------
 * Fused projection.  Replaces rendering.py:156-218 (quaternion_matrix,
 * project_surfaces), the SH colour launch rendering.py:334-340 and the record
 * packing rendering.py:341-374 with one launch over (scene, surfel) threads that
 * loop over the scene's cameras.  Pair index p = (s*C + c)*N + n.
 *   sh_degree < 0: no SH; app_rows may be NULL.
 *   sh_degree 0..3: both colours are evaluated per pair (spherical_harmonics.cu:
 *   45-85) and written with the surfel's weights/magnitudes/phases into
 *   app_rows[p] (classic appearance row layout).
 * Outputs: records[P][20], xy[P][2], radii[P] (int32, 0 = culled).
 * Alignment (GS_ERR_ARGUMENT otherwise): quaternions, records, app_rows and the three
 * wave-parameter arrays start on 16 bytes, scales and xy on 8 (the kernels move their
 * rows as vectors).
 */
int gs_project_forward(const float* means, const float* quaternions, const float* scales,
                       const float* opacities, const float* view_matrices,
                       const float* intrinsics, const float* sh_first,
                       const float* sh_second, const float* frequency_weights,
                       const float* frequency_magnitudes, const float* phases,
                       int sh_degree, int64_t scenes, int64_t cameras, int64_t surfels,
                       int width, int height, float near_plane, float far_plane,
                       float* records, float* xy, float* app_rows, int32_t* radii,
                       void* stream);

/* Reverse of gs_project_forward (the PyTorch autograd of rendering.py:156-218,
 * 334-374 and spherical_harmonics.cu:128-150).  grad_records[P][20] (slots 9-10
 * ignored), grad_xy[P][2], grad_app_rows[P][20] (SH mode).  Surfel gradients are
 * summed over cameras in registers; camera gradients are reduced per block and
 * added with atomics.  Every output is overwritten (zeroed first on the stream).
 * Alignment as in gs_project_forward, for the inputs and for the matching gradients
 * (grad_records, grad_app_rows, grad_quaternions and the wave-parameter gradients on 16
 * bytes, grad_xy and grad_scales on 8). */
int gs_project_backward(const float* means, const float* quaternions, const float* scales,
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
                        void* stream);

/* Ragged scene batches (no counterpart in the reference, which lists them outside its
 * release): scene s owns surfels [scene_offsets[s], scene_offsets[s+1]) of the
 * concatenated per-surfel arrays (scene_offsets: device int64[S+1], starting at 0);
 * its pairs are records [C * scene_offsets[s], C * scene_offsets[s+1]), camera-major
 * (pair C*o_s + c*N_s + n).  max_surfels is the largest N_s, total_surfels
 * scene_offsets[S].  Otherwise as gs_project_forward / gs_project_backward. */
int gs_project_forward_ragged(const float* means, const float* quaternions, const float* scales,
                              const float* opacities, const float* view_matrices,
                              const float* intrinsics, const float* sh_first,
                              const float* sh_second, const float* frequency_weights,
                              const float* frequency_magnitudes, const float* phases,
                              int sh_degree, int64_t scenes, int64_t cameras,
                              const int64_t* scene_offsets, int64_t max_surfels, int width,
                              int height, float near_plane, float far_plane, float* records,
                              float* xy, float* app_rows, int32_t* radii, void* stream);
int gs_project_backward_ragged(const float* means, const float* quaternions,
                               const float* scales, const float* view_matrices,
                               const float* intrinsics, const float* sh_first,
                               const float* sh_second, int sh_degree, int64_t scenes,
                               int64_t cameras, const int64_t* scene_offsets,
                               int64_t max_surfels, int64_t total_surfels,
                               const float* grad_records, const float* grad_xy,
                               const float* grad_app_rows, float* grad_means,
                               float* grad_quaternions, float* grad_scales,
                               float* grad_opacities, float* grad_view_matrices,
                               float* grad_intrinsics, float* grad_sh_first,
                               float* grad_sh_second, float* grad_frequency_weights,
                               float* grad_frequency_magnitudes, float* grad_phases, void* stream);

/* ---------------------------------------------------------------------------
 * Tile binning (rasterize.cu:23-69, 454-493).  Two phases around the one host
 * synchronisation the reference also has (rasterize.cu:466-468):
 *   gs_bin_count : depth-sort the records, count each record's tiles as row spans
 *                  (one span per tile row it reaches), scan; returns the intersection
 *                  count I and the span count to the host (waits on the stream).
 *   gs_bin_sort  : write the spans, expand (tile, record) slots in depth order,
 *                  stable-sort by tile, write point_list[I] (record indices) and ranges.
 * With flags 0 the result is identical to the reference's stable 64-bit
 * (tile << 32 | depth bits) sort of its square 3-sigma tile bounds: within a tile,
 * records are ordered by depth bits, then index.  GS_BIN_TIGHT keeps, per tile row,
 * only the tiles a sample with alpha >= 1/255 can reach (the projected ellipse of the
 * opacity's alpha level and the low-pass disc, widened for rounding): images are
 * unchanged, lists shorter.  It needs opacity in record slot 17 (record_stride >= 18)
 * and must be given to both calls.
 * records: float rows of `record_stride` floats (x, y at 9-10, depth at 8);
 * image_ids: int64 per record, or NULL for image = r / records_per_image.
 * Workspace 1 must stay untouched between the two calls.
 */
#define GS_BIN_TIGHT 1
int gs_bin_count_workspace(int64_t records, size_t* bytes);
int gs_bin_count(const float* records, int record_stride, const int32_t* radii,
                 const int64_t* image_ids, int64_t records_count, int64_t records_per_image,
                 int64_t images, int width, int height, int flags, void* workspace1,
                 size_t workspace1_bytes, int64_t* intersections, int64_t* spans, void* stream);
int gs_bin_sort_workspace(int64_t records, int64_t intersections, int64_t spans, int64_t images,
                          int width, int height, size_t* bytes);
int gs_bin_sort(const float* records, int record_stride, const int32_t* radii,
                const int64_t* image_ids, int64_t records_count, int64_t records_per_image,
                int64_t images, int width, int height, int flags, const void* workspace1,
                size_t workspace1_bytes, void* workspace2, size_t workspace2_bytes,
                int64_t intersections, int64_t spans, int32_t* point_list, int32_t* ranges,
                void* stream);

/* Binning without a host synchronisation (so a render step can be captured in a CUDA
 * graph): the caller sizes an arena for at most max_intersections (record, tile) slots
 * and max_spans row spans (gs_bin_arena_workspace); every launch is sized by those
 * capacities and the live counts stay on the device.  point_list holds
 * max_intersections entries (those past the live count are padding); ranges as for
 * gs_bin_sort.  totals (device int64[2], nullable) receives the live intersection and
 * span counts; when either exceeds its capacity nothing is binned (every tile range
 * empty) and totals says how large the arena must be.  Same order and flags as
 * gs_bin_count + gs_bin_sort.  No counterpart in the reference, whose binning reads the
 * count on the host (rasterize.cu:466-468). */
int gs_bin_arena_workspace(int64_t records, int64_t max_intersections, int64_t max_spans,
                           int64_t images, int width, int height, size_t* bytes);
int gs_bin_arena(const float* records, int record_stride, const int32_t* radii,
                 const int64_t* image_ids, int64_t records_count, int64_t records_per_image,
                 int64_t images, int width, int height, int flags, void* workspace,
                 size_t workspace_bytes, int64_t max_intersections, int64_t max_spans,
                 int32_t* point_list, int32_t* ranges, int64_t* totals, void* stream);

/* No-allocation binning: gs_bin_count followed by gs_bin_sort with both workspaces
 * taken from an 80 MiB array compiled into the library (one per GPU that loads it,
 * held until the process exits), for callers that cannot allocate device memory when
 * they bin: a host application whose own allocator owns every device byte, or a
 * real-time loop that forbids allocation after start-up.  No counterpart in the
 * reference.  Square (reference) bins, flags 0.  Limits, each checked before any
 * work (GS_ERR_LIMIT beyond; *intersections still reports the count when that is
 * the cause): at most 65536 records, 1048576 tile intersections, images up to 2048
 * pixels wide (128 tile columns) and 262144 16x16 tiles over all images; within them
 * the workspaces always fit the array.  point_list must hold point_list_capacity
 * entries.  The first call on a device looks the array's device address up with that
 * device current (cudaGetSymbolAddress) and keeps it for the process: make that
 * first call before any stream capture, and do not reset the device afterwards.
 * Every call uses the same array: calls that overlap on the GPU race and corrupt each
 * other's lists, so serialise them (one stream, or events).  Waits on the stream
 * once, like gs_bin_count. */
int gs_bin_static(const float* records, int record_stride, const int32_t* radii,
                  const int64_t* image_ids, int64_t records_count, int64_t records_per_image,
                  int64_t images, int width, int height, int32_t* point_list,
                  int64_t point_list_capacity, int32_t* ranges, int64_t* intersections,
                  void* stream);

/* ---------------------------------------------------------------------------
 * Tile compositor.  Forward: renderForward (rasterize.cu:229-281); backward:
 * renderBackward (rasterize.cu:283-399).  One CTA per 16x16 tile.
 * row_mode selects the appearance row of a record (GS_ROWS_*); `cameras`,
 * `surfels` are used by GS_ROWS_PER_SURFEL, primitive_ids by GS_ROWS_EXPLICIT.
 * Backward adds into grad_records / grad_rows / grad_backgrounds (the caller
 * zeroes them, so several calls over image chunks can accumulate into shared
 * appearance rows); grad_xy (nullable, [R][2]) receives the slot 9-10
 * (screen-centre) gradients instead of grad_records when given.
 * Forward flags: 0 evaluates the Gabor waves, SIREN sines and sigmoid with the SFU
 * (wave error < 4e-7, images within 1e-6 of the exact evaluation); GS_COMPOSITE_EXACT
 * uses full-precision cosf/sinf/expf in the reference's expression order, which makes
 * images bit-identical to the reference's.
 * counters (nullable, uint64[2], zeroed by the caller) receives the work done:
 * [0] ray/splat samples tested, [1] contributions accepted (blended forward,
 * differentiated backward).  A NULL pointer selects kernels without counting.
 */
#define GS_COMPOSITE_EXACT 1   /* forward flags: full-precision cosf/sinf/expf appearance */
int gs_composite_forward(const float* records, const float* rows, int row_mode,
                         const int64_t* primitive_ids, int64_t cameras, int64_t surfels,
                         int64_t records_count, int64_t rows_count,
                         const float* backgrounds, const int32_t* point_list,
                         const int32_t* ranges, int64_t images, int width, int height,
                         int neural, int flags, float near_plane, float far_plane, float* maps,
                         float* state, int32_t* contributors, uint64_t* counters,
                         void* stream);
int gs_composite_backward(const float* records, const float* rows, int row_mode,
                          const int64_t* primitive_ids, int64_t cameras, int64_t surfels,
                          int64_t records_count, int64_t rows_count,
                          const float* backgrounds, const int32_t* point_list,
                          const int32_t* ranges, const float* state,
                          const int32_t* contributors, const float* grad_maps,
                          int64_t images, int width, int height, int neural,
                          float near_plane, float far_plane, float* grad_records,
                          float* grad_xy, float* grad_rows, float* grad_backgrounds,
                          uint64_t* counters, void* stream);

/* The same compositor with the nine maps as five planes -- rgb (3 channels), alpha,
 * depth, normals (3), distortion -- each at its own address: plane g of pixel p
 * starts at planes[g] + p * plane_strides[g] (floats, channels adjacent).  The
 * backward reads each plane's gradient at grad_planes[g] + p * grad_strides[2g] +
 * k * grad_strides[2g+1] (a stride of 0 reads a broadcast value; a NULL plane is a
 * zero gradient, and a NULL normal-map plane also drops the normal terms from the
 * backward's per-record sums).  `planes`, `plane_strides`, `grad_planes` and `grad_strides` are
 * host arrays.  No counterpart in the reference, which writes one [..][9] array and
 * slices it: with separate planes a framework hands each output's gradient to the
 * kernel as it is, without assembling a full [..][9] gradient.
 * Median depth (optional, no counterpart in the reference, which lists it outside its
 * release): with median_depth non-NULL the forward also writes, per pixel, the depth of
 * the last contribution made while the transmittance before it exceeds 0.5 (the 2DGS
 * convention; 0 without contributions) at median_depth + p * median_stride, and its
 * 1-based position in the tile's list (0: none) in median_index[p]; the backward adds
 * grad_median[p * grad_median_stride] (nullable; stride 0 broadcasts) to that
 * contribution's depth gradient.
 * Selected pixels (optional; no counterpart in the reference, which lists
 * selected-pixel rendering outside its release): with groups non-NULL only listed
 * pixels are composited, one CTA per group: groups[4g..4g+3] = (tile, first, count, 0)
 * with count <= 256, every listed pixel of the group inside that tile, and
 * selected[4i..4i+3] = (x, y, output index, 0) for i in [first, first + count).  All
 * per-pixel arrays (planes, state, contributors, median, gradients) are then indexed by
 * output index instead of (image H + y) W + x.
 * Warp accept masks (optional; no counterpart in the reference): with warp_masks
 * non-NULL (8 planes of warp_mask_words 32-bit words, zeroed by the caller before the
 * forward; warp_mask_words >= ceil(point-list length / 32)) the forward sets, for each
 * of a CTA's eight warps, bit p % 32 of word p / 32 of that warp's plane when a pixel
 * of the warp accepted the record at point-list position p, and the backward, given
 * the same masks, skips the records its warp accepted nowhere -- records that add no
 * gradient there.  Images and gradients are the same with or without masks; they pay
 * when most records of a tile reach few of its 8x4-pixel warp blocks (splats small
 * against the tile).  Positions past the planes are treated as accepted. */
int gs_composite_forward_split(const float* records, const float* rows, int row_mode,
                               const int64_t* primitive_ids, int64_t cameras, int64_t surfels,
                               int64_t records_count, int64_t rows_count,
                               const float* backgrounds, const int32_t* point_list,
                               const int32_t* ranges, int64_t images, int width, int height,
                               int neural, int flags, float near_plane, float far_plane,
                               float* const* planes, const int64_t* plane_strides,
                               float* median_depth, int64_t median_stride,
                               int32_t* median_index, const int32_t* selected,
                               const int32_t* groups, int64_t group_count, float* state,
                               int32_t* contributors, uint32_t* warp_masks,
                               int64_t warp_mask_words, uint64_t* counters, void* stream);
int gs_composite_backward_split(const float* records, const float* rows, int row_mode,
                                const int64_t* primitive_ids, int64_t cameras, int64_t surfels,
                                int64_t records_count, int64_t rows_count,
                                const float* backgrounds, const int32_t* point_list,
                                const int32_t* ranges, const float* state,
                                const int32_t* contributors, const float* const* grad_planes,
                                const int64_t* grad_strides, const int32_t* median_index,
                                const float* grad_median, int64_t grad_median_stride,
                                const int32_t* selected, const int32_t* groups,
                                int64_t group_count, int64_t images, int width,
                                int height, int neural, float near_plane, float far_plane,
                                float* grad_records, float* grad_xy, float* grad_rows,
                                float* grad_backgrounds, const uint32_t* warp_masks,
                                int64_t warp_mask_words, uint64_t* counters, void* stream);

/* ---------------------------------------------------------------------------
 * Fused Adam step.  Replaces torch.optim.Adam.step() in the reference's optimisation
 * loop (examples/fit_texture.py:50-61; torch/optim/adam.py _multi_tensor_adam):
 * for every tensor t with sizes[t] float32 elements, p += -(lr / (1 - beta1^step)) *
 * m / (sqrt(v) / sqrt(1 - beta2^step) + eps) after m = lerp(m, g + wd p, 1 - beta1) and
 * v = beta2 v + (1 - beta2) (g + wd p)^2, in one launch per 48 tensors.  The pointer
 * arrays and sizes are host arrays; all device arrays are contiguous.  `step` is the
 * step number after this update (1 for the first).  No counterpart in the reference's
 * native module.
 */
int gs_adam_step(int tensors, float* const* params, const float* const* grads,
                 float* const* exp_avgs, float* const* exp_avg_sqs, const int64_t* sizes,
                 double lr, double beta1, double beta2, double eps, double weight_decay,
                 int64_t step, void* stream);

/* Capturable form of gs_adam_step, the counterpart of torch.optim.Adam(capturable=True)
 * (torch/optim/adam.py, _multi_tensor_adam with device step tensors): `steps` is a host
 * array of device pointers, one float32 step count per tensor (its own, not shared),
 * which this call increments by one on the device before the update computes its bias
 * corrections from it (in double).  Nothing is read back to the host, so the call can
 * be recorded in a CUDA graph and replayed.  `skip` (nullable) is a device int32 flag
 * read when the kernels run: nonzero leaves every parameter, moment and step count as
 * it was (a recorded training step whose render overflowed its binning arena must not
 * move the parameters).  No counterpart in the reference's native module.
 */
int gs_adam_step_capturable(int tensors, float* const* params, const float* const* grads,
                            float* const* exp_avgs, float* const* exp_avg_sqs,
                            const int64_t* sizes, float* const* steps, double lr, double beta1,
                            double beta2, double eps, double weight_decay, const int32_t* skip,
                            void* stream);

/* ---------------------------------------------------------------------------
 * Layout converters for the reference-layout entry points (the `_C` mirror).
 * gs_pack_geometry: geometry[Q][17] + opacities[primitive_ids[q]] -> records[Q][20].
 * gs_pack_rows:     appearance[A][width] (18 or 57) -> rows[A][20 or 60].
 * gs_unpack_geometry_grads: grad_records[Q][20] -> grad_geometry[Q][17] and
 *                   grad_opacities[primitive_ids[q]] += slot 17 (zeroed first).
 * gs_unpack_rows:   rows[A][20 or 60] -> appearance[A][width].
 */
int gs_pack_geometry(const float* geometry, const float* opacities,
                     const int64_t* primitive_ids, int64_t records_count,
                     int64_t opacity_count, float* records, void* stream);
int gs_pack_rows(const float* appearance, int64_t rows_count, int width, float* rows,
                 void* stream);
int gs_unpack_geometry_grads(const float* grad_records, const int64_t* primitive_ids,
                             int64_t records_count, int64_t opacity_count,
                             float* grad_geometry, float* grad_opacities, void* stream);
int gs_unpack_rows(const float* rows, int64_t rows_count, int width, float* appearance,
                   void* stream);

/* Per-surfel appearance rows of the renderers without SH (the reference concatenates the
 * appearance tensors, rendering.py:347-356): `appearance` is a host array of device
 * pointers -- classic (neural == 0): colors [A][3], secondary_colors [A][3],
 * frequency_weights, frequency_magnitudes, phases [A][4]; neural: input_weights [A][30],
 * input_biases [A][6], output_weights [A][18], output_biases [A][3] -- packed into
 * rows[A][20] (classic) or rows[A][60] (neural), pad slots zero.  The unpack form
 * writes each row's fields back to the separate tensors (their gradients). */
int gs_pack_surfel_rows(int neural, const float* const* appearance, int64_t count, float* rows,
                        void* stream);
int gs_unpack_surfel_rows(int neural, const float* rows, int64_t count,
                          float* const* grad_appearance, void* stream);

/* Metadata ids of reported pairs (rendering.py:389-399: scene_ids, camera_ids,
 * primitive_ids = pair // (C N), pair // N % C, pair % N) in one pass: for i < count the
 * pair p = pairs[i] (pairs NULL: p = i) of the dense (scene, camera, surfel) layout
 * p = (s C + c) N + n gives scene_ids[i] = s, camera_ids[i] = c, primitive_ids[i] = n
 * (int64 outputs, each nullable). */
int gs_pair_ids(const int64_t* pairs, int64_t count, int64_t cameras, int64_t surfels,
                int64_t* scene_ids, int64_t* camera_ids, int64_t* primitive_ids, void* stream);

/* Measurement: FP32 multiply-add throughput of this GPU, the denominator of the
 * compositors' FP32 roofline (no counterpart in the reference).  blocks x 256 threads
 * each run `iterations` steps of eight independent fused multiply-add chains (2 flops
 * each; paired != 0: eight float2 chains as FFMA2, 4 flops each).  `out` (device, one
 * float per block) is written only on an impossible value; time the launch with
 * events on `stream`. */
int gs_fp32_probe(int blocks, int iterations, int paired, float* out, void* stream);

/* ---------------------------------------------------------------------------
 * Spherical-harmonic colours (spherical_harmonics.cu:45-150) for the
 * SHColors entry points.  first/second [B][N][K][3], directions [B][C][N][3],
 * colors [B][C][N][6].  Backward overwrites its three outputs; coefficient
 * gradients are summed over cameras in registers (no atomics).
 */
int gs_sh_forward(const float* first, const float* second, const float* directions,
                  int degree, int64_t scenes, int64_t cameras, int64_t surfels,
                  float* colors, void* stream);
int gs_sh_backward(const float* first, const float* second, const float* directions,
                   const float* grad_colors, int degree, int64_t scenes, int64_t cameras,
                   int64_t surfels, float* grad_first, float* grad_second,
                   float* grad_directions, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* GABOR_B200_H */
