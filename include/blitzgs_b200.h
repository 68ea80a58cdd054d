/*
 * blitzgs_b200 -- C ABI of the B200 (sm_100a) Gaussian-splatting training path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (passed as void*; NULL = legacy default stream), launches asynchronously on
 * that stream and returns an int status: 0 on success, otherwise a CUDA error
 * code or one of the BLITZ_E* codes below.  blitz_last_error() returns a
 * description of the last failure on the calling thread.  The library never
 * allocates or frees device memory: the caller provides every output and
 * scratch buffer (sizes are queried with the *_bytes functions).  Nothing
 * traps: conditions the reference turns into a device __trap() set bits in a
 * caller-provided device error word instead.
 *
 * Tensor layouts are the reference's (row-major, fp32 unless stated):
 *   means3D [P,3], scales [P,3] (activated), rotations [P,4] (r,x,y,z;
 *   normalised by the caller; 16-byte aligned rows), opacities [P] (activated),
 *   SH coefficients addressed as (dc + i*dc_stride, rest + i*rest_stride) in
 *   floats so both a contiguous [P,16,3] tensor (dc_stride = rest_stride = 48,
 *   rest = dc + 3) and split [P,1,3] / [P,15,3] tensors are accepted,
 *   viewmatrix / projmatrix: device float[16] (the transposed world-to-view
 *   and full projection matrices of the reference Camera), campos float[3].
 *
 * Images are [3,H,W]; tiles are 16x16 pixels, grid_x = ceil(W/16),
 * grid_y = ceil(H/16), tile t = ty*grid_x + tx.
 */
#ifndef BLITZGS_B200_H_
#define BLITZGS_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BLITZ_OK 0
#define BLITZ_EINVAL 10001      /* bad argument (size, alignment, null pointer) */
#define BLITZ_ESCRATCH 10002    /* scratch buffer smaller than *_bytes() asked for */
#define BLITZ_ESCAN 10003       /* an ordered list scan gave up waiting (results of that launch are unordered) */

/* Device error-word bits (see blitz_preprocess_forward). */
#define BLITZ_ERRBIT_PREFILTERED_CULLED 1u /* a Gaussian failed the near test with prefiltered=1 */

/* Library version string (no reference counterpart). */
const char* blitz_version(void);
/* Message for the last non-zero status returned on this host thread; the
 * reference raises these as Python exceptions from its pybind11 modules. */
const char* blitz_last_error(void);

/*
 * EWA preprocess of P Gaussians for one camera.
 * Replaces _C.preprocess_gaussians / PreprocessGaussiansCUDA
 * (submodule/diff-gaussian-rasterization_f/rasterize_points.cu:834-923 and
 * cuda_rasterizer/rasterizer_impl.cu:982-1067).
 * Outputs (all written, zeros for culled Gaussians): means2D [P,2] (pixels),
 * depths [P] (view z), radii int32 [P], conic_opacity [P,4], rgb [P,3];
 * optional (may be NULL): cov3D [P,6], clamped uint8 [P,3], rects [P,2] (the
 * float half-extents of each Gaussian's screen rectangle, which the full
 * rasterizer bins over: forward.cu:253-262).
 * culling (uint8 [P], may be NULL): Gaussians with a non-zero entry are
 * skipped, as _C.rasterize_gaussians skips them (forward.cu:196-203).
 * error_word: device uint32 OR-ed with BLITZ_ERRBIT_* (may be NULL).
 * M = SH coefficients beyond DC per Gaussian (0..15), D = active degree (0..3).
 */
int blitz_preprocess_forward(int64_t P, int D, int M, const float* means3D, const float* scales,
                             const float* rotations, const float* sh_dc, int64_t dc_stride,
                             const float* sh_rest, int64_t rest_stride, const float* opacities,
                             float scale_modifier, const float* viewmatrix, const float* projmatrix,
                             const float* campos, float tanfovx, float tanfovy, int image_height,
                             int image_width, int prefiltered, float* means2D, float* depths,
                             int32_t* radii, float* cov3D, float* conic_opacity, float* rgb,
                             uint8_t* clamped, const uint8_t* culling, float* rects, uint32_t* error_word,
                             void* stream);

/*
 * Backward of blitz_preprocess_forward.
 * Replaces _C.preprocess_gaussians_backward / PreprocessGaussiansBackwardCUDA
 * (submodule/diff-gaussian-rasterization_f/rasterize_points.cu:926-1029 and
 * cuda_rasterizer/backward.cu:146-400).
 * Upstream gradients are addressed with per-Gaussian strides (floats):
 *   dL_dmeans2D (x,y) at g_means2D + i*g_means2D_stride  (NDC-scaled, as the
 *     reference's render backward produces),
 *   dL_dconic_opacity float4 at g_conic_opacity + i*g_conic_stride (16-byte aligned),
 *   dL_dcolors (r,g,b) at g_colors + i*g_colors_stride.
 * Outputs: dL_dmeans3D [P,3], dL_dscales [P,3], dL_drotations [P,4]
 * (w.r.t. the rotation as passed in), dL_dopacity [P] (may be NULL), SH grads
 * at (g_dc + i*g_dc_stride, g_rest + i*g_rest_stride).
 * accumulate = 0 overwrites the outputs (zeros for radii <= 0), 1 adds.
 */
int blitz_preprocess_backward(int64_t P, int D, int M, const int32_t* radii, const float* means3D,
                              const float* scales, const float* rotations, const float* sh_dc,
                              int64_t dc_stride, const float* sh_rest, int64_t rest_stride,
                              float scale_modifier, const float* viewmatrix, const float* projmatrix,
                              const float* campos, float tanfovx, float tanfovy, int image_height,
                              int image_width, const float* g_means2D, int64_t g_means2D_stride,
                              const float* g_conic_opacity, int64_t g_conic_stride,
                              const float* g_colors, int64_t g_colors_stride, float* dL_dmeans3D,
                              float* dL_dscales, float* dL_drotations, float* dL_dopacity,
                              float* g_dc, int64_t g_dc_stride, float* g_rest, int64_t g_rest_stride,
                              int accumulate, void* stream);

/*
 * Preprocess from the model's RAW parameters (fused training path).
 * Same outputs as blitz_preprocess_forward, but scaling_raw / rotation_raw /
 * opacity_raw are GaussianModel's _scaling / _rotation / _opacity and the
 * kernel applies exp, normalize and sigmoid itself (scene/gaussian_model.py:
 * 248-276) with PyTorch's float arithmetic; rotation_norm (device [P], may be
 * NULL = computed in the kernel) is ||_rotation|| per Gaussian.
 * Optional fused extras (each may be NULL):
 *   reg_sums  device double[2] += {sum of the smallest activated scale, count}
 *             over Gaussians with radius > 0 and a non-empty tile rect (the
 *             min-scale regulariser of gaussian_renderer/loss_distribution.py:314-322);
 *   vis_list  device uint32 [P] receives the indices of Gaussians with
 *             radius > 0 (unordered), vis_count (device int32, zero on entry)
 *             their number -- the work list of blitz_preprocess_backward_raw.
 *             With a list, only the rows of listed Gaussians are guaranteed to
 *             be written in means2D / depths / conic_opacity / rgb (radii is
 *             always written for every Gaussian): a training view touches a
 *             few percent of the model, and the other rows are never read;
 *   counts    device uint32 [P]: tile count of each Gaussian under the
 *             compute_locally mask (uint8 [tiles], NULL = all tiles), and
 *             totals (device uint64 [2]) = {tile instances R, Gaussians with
 *             at least one tile}: the output of blitz_render_count, fused
 *             (counts and totals must be both given or both NULL);
 *   slot_of   device uint32 [P] (with a list): slot_of[i] = position of
 *             listed Gaussian i in vis_list (other entries untouched);
 *   exchange  host pointer to a blitz_exchange_out (with a list and the
 *             scratch; NULL = none).  With it the visible list is in
 *             ascending index order (the exchange keeps one order on every
 *             run); without it the list's order is unspecified;
 *   scratch   device buffer of blitz_preprocess_scratch_bytes(P) bytes: runs
 *             the cull and the full computation as two kernels (faster when
 *             most Gaussians are off-screen); NULL runs one kernel.
 * Replaces the activation kernels + preprocess of the reference training step
 * (gaussian_renderer/__init__.py:260-324); no reference op is a single match.
 */
/* Size of the optional scratch of blitz_preprocess_forward_raw (no reference
 * counterpart: the reference allocates its temporaries per call).  Its first
 * 4 bytes are a status word of the ordered list scans: zero a new buffer
 * once, then check it with blitz_read_totals; the launches never clear it. */
size_t blitz_preprocess_scratch_bytes(int64_t P);

/*
 * Optional exchange outputs of blitz_preprocess_forward_raw for the
 * multi-GPU step (they need vis_list).  They replace the record packing and
 * the getTouchedIdsBool routing of all_to_all_communication_final
 * (gaussian_renderer/__init__.py:22-189, f/rasterize_points.cu:212-256) for
 * the listed Gaussians only, inside the preprocess kernel.  Row j belongs to
 * the j-th listed Gaussian (vis_list[j]):
 *   records   [P,12] float, 16-byte aligned: conic00 conic01 conic11 opacity |
 *             means2D x y | r g b | depth | radius (int32 bits) | smallest
 *             activated scale;
 *   dest_mask [P] uint32: bit r set when the Gaussian's square tile rect,
 *             flattened to the tile-id interval [ymin*gx+xmin,
 *             (ymax-1)*gx+xmax-1], overlaps rank r's interval
 *             [tile_lo[r], tile_hi[r]) (an empty interval sends nothing);
 *   dest_counts [n_ranks] int32, zero on entry: rows per destination rank.
 * tile_lo / tile_hi: device int32 [n_ranks] (n_ranks <= 32); a rank that
 * renders none of this camera gets lo = hi = 0.
 */
typedef struct blitz_exchange_out {
  int n_ranks;
  const int32_t* tile_lo;
  const int32_t* tile_hi;
  float* records;
  uint32_t* dest_mask;
  int32_t* dest_counts;
} blitz_exchange_out;
int blitz_preprocess_forward_raw(int64_t P, int D, int M, const float* xyz, const float* scaling_raw,
                                 const float* rotation_raw, const float* rotation_norm,
                                 const float* opacity_raw, const float* sh_dc, int64_t dc_stride,
                                 const float* sh_rest, int64_t rest_stride, float scale_modifier,
                                 const float* viewmatrix, const float* projmatrix, const float* campos,
                                 float tanfovx, float tanfovy, int image_height, int image_width,
                                 float* means2D, float* depths, int32_t* radii, float* conic_opacity,
                                 float* rgb, double* reg_sums, uint32_t* vis_list, int32_t* vis_count,
                                 const uint8_t* compute_locally, uint32_t* counts, uint64_t* totals,
                                 uint32_t* slot_of, const blitz_exchange_out* exchange, void* scratch,
                                 size_t scratch_bytes, void* stream);

/*
 * Backward of blitz_preprocess_forward_raw: gradients with respect to the
 * RAW parameters (xyz, _scaling, _rotation, _opacity, SH), chained through
 * the activations in the kernel.  reg_scale (device float, may be NULL) is
 * dLoss/d(reg_sums[0]).  With vis_list/vis_count from the forward only those
 * Gaussians are processed: the caller zero-fills the outputs first, and
 * `accumulate` selects whether their rows are stored (0) or added onto (1);
 * with NULL lists every Gaussian is processed and `accumulate` selects
 * overwrite (0) or add (1).
 * rows (with a list only; 0 otherwise): BLITZ_ROWS_UPSTREAM_BY_SLOT reads the
 * upstream gradients of the j-th listed Gaussian at row j (the compact record
 * of blitz_render_backward with record_rows), BLITZ_ROWS_OUTPUT_BY_SLOT writes
 * its gradients at row j of [vis_count, ...] outputs (every row written: no
 * zero-fill; the gradient as sparse rows, indices = vis_list).
 * g_minscale (may be NULL): per-row d(loss)/d(smallest activated scale) at
 * g_minscale + row*g_minscale_stride (row as for the upstream gradients),
 * added to the first smallest axis -- the multi-GPU regulariser gradient.
 */
#define BLITZ_ROWS_UPSTREAM_BY_SLOT 1
#define BLITZ_ROWS_OUTPUT_BY_SLOT 2
int blitz_preprocess_backward_raw(int64_t P, int D, int M, const int32_t* radii, const float* means2D,
                                  const float* xyz, const float* scaling_raw, const float* rotation_raw,
                                  const float* rotation_norm, const float* opacity_raw, const float* sh_dc,
                                  int64_t dc_stride, const float* sh_rest, int64_t rest_stride,
                                  float scale_modifier, const float* viewmatrix, const float* projmatrix,
                                  const float* campos, float tanfovx, float tanfovy, int image_height,
                                  int image_width, const float* g_means2D, int64_t g_means2D_stride,
                                  const float* g_conic_opacity, int64_t g_conic_stride,
                                  const float* g_colors, int64_t g_colors_stride, const float* reg_scale,
                                  const float* g_minscale, int64_t g_minscale_stride,
                                  const uint32_t* vis_list, const int32_t* vis_count, float* g_xyz,
                                  float* g_scaling_raw, float* g_rotation_raw, float* g_opacity_raw,
                                  float* g_dc, int64_t g_dc_stride, float* g_rest, int64_t g_rest_stride,
                                  int accumulate, int rows, void* stream);

/*
 * Render forward, phase 1 of 2: per-Gaussian tile-touch counts under the
 * compute_locally mask (bool [grid_y*grid_x], NULL = every tile), and the
 * device totals {R = tile instances, n_vis = Gaussians with count > 0}
 * (uint64 [2]).  Replaces the updateTileTouched + scan + blocking readback
 * of renderForward (submodule/diff-gaussian-rasterization_r/cuda_rasterizer/
 * rasterizer_impl.cu:602-621); the caller reads the two totals back (one
 * small device-to-host copy) to size phase 2.
 */
int blitz_render_count(int64_t P, int image_height, int image_width, const float* means2D,
                       const int32_t* radii, const uint8_t* compute_locally, uint32_t* counts,
                       uint64_t* totals, void* stream);

/* Scratch bytes blitz_render_forward needs for the given totals. */
size_t blitz_render_scratch_bytes(int64_t P, int64_t n_vis, int64_t R, int image_height,
                                  int image_width);

/*
 * Render forward, phase 2 of 2: binning (depth sort + stable tile sort) and
 * front-to-back alpha blending.
 * Replaces _C.render_gaussians / RenderGaussiansCUDA
 * (submodule/diff-gaussian-rasterization_r/rasterize_points.cu:274-361,
 * rasterizer_impl.cu:556-723, forward.cu:263-413).
 * State kept for the backward (caller-owned): point_list uint32 [R],
 * ranges uint32 [n_tiles,2], final_T [H*W], n_contrib uint32 [H*W].
 * Outputs: out_color [3,H,W] (zero outside compute_locally tiles),
 * n_render / n_consider / n_contrib_tile int32 [n_tiles], out_observe int32 [P]
 * (must be zero on entry).
 */
int blitz_render_forward(int64_t P, int64_t n_vis, int64_t R, int image_height, int image_width,
                         const float* means2D, const float* depths, const int32_t* radii,
                         const float* conic_opacity, const float* rgb, const float* bg,
                         const uint8_t* compute_locally, const uint32_t* counts, void* scratch,
                         size_t scratch_bytes, uint32_t* point_list, uint32_t* ranges,
                         float* final_T, uint32_t* n_contrib, float* out_color, int32_t* n_render,
                         int32_t* n_consider, int32_t* n_contrib_tile, int32_t* out_observe,
                         void* stream);

/*
 * The two halves of blitz_render_forward, for callers that schedule or time
 * them separately: binning (point_list, ranges) and blending (everything
 * else).  Same arguments and contracts as blitz_render_forward.
 * n_vis and R may also be capacities above the totals (the kernels read the
 * exact counts on the device), so the binning can be issued before the
 * totals are read back; if the true totals exceed them, the tile lists are
 * clipped to the R instances the buffers hold -- no access goes beyond them
 * -- and the caller bins again with the exact totals.
 * blitz_render_blend may also record, for blitz_render_backward, the
 * Gaussians that contributed to each warp strip (8 strips of 8x4 pixels per
 * tile): strip_ids / strip_pos int32 [8*R] (Gaussian id and 0-based tile-list
 * position, strip s of tile t at [8*ranges[t].begin + s*n_t + e], n_t the
 * tile's list length) and strip_counts int32 [n_tiles*8].  All three or none
 * (NULL); no counterpart in the reference.
 */
int blitz_render_bin(int64_t P, int64_t n_vis, int64_t R, int image_height, int image_width, const float* means2D,
                     const float* depths, const int32_t* radii, const uint8_t* compute_locally, const uint32_t* counts,
                     void* scratch, size_t scratch_bytes, uint32_t* point_list, uint32_t* ranges, void* stream);
int blitz_render_blend(int64_t P, int image_height, int image_width, const float* means2D, const float* conic_opacity,
                       const float* rgb, const float* bg, const uint8_t* compute_locally, const uint32_t* point_list,
                       const uint32_t* ranges, float* final_T, uint32_t* n_contrib, float* out_color,
                       int32_t* n_render, int32_t* n_consider, int32_t* n_contrib_tile, int32_t* out_observe,
                       int32_t* strip_ids, int32_t* strip_pos, int32_t* strip_counts, void* stream);

/*
 * Binning for callers that cannot allocate device memory at call time (no
 * counterpart in the reference).  Same arguments and results as
 * blitz_render_bin minus the scratch buffer: the scratch is a fixed
 * BLITZ_NOALLOC_SCRATCH_BYTES array inside this library, held by every GPU
 * that loads it until the process exits.  Requests whose
 * blitz_render_scratch_bytes() exceed it fail with BLITZ_ESCRATCH.  All calls
 * on a device share the array: calls that overlap on the GPU race.  The first
 * call on a device resolves the array's address (make it before any stream
 * capture) and caches it for the process: it is the address in the device's
 * primary context (the CUDA runtime's and PyTorch's), so callers that use a
 * context of their own, or reset the device within the process, must not use
 * this entry point.  Allocates nothing.
 */
#define BLITZ_NOALLOC_SCRATCH_BYTES (64u << 20)
int blitz_render_bin_noalloc(int64_t P, int64_t n_vis, int64_t R, int image_height, int image_width,
                             const float* means2D, const float* depths, const int32_t* radii,
                             const uint8_t* compute_locally, const uint32_t* counts, uint32_t* point_list,
                             uint32_t* ranges, void* stream);

/*
 * Render backward.
 * Replaces _C.render_gaussians_backward / RenderGaussiansBackwardCUDA
 * (submodule/diff-gaussian-rasterization_r/rasterize_points.cu:364-436,
 * rasterizer_impl.cu:727-804, backward.cu:324-530).
 * grad_accum: float [rows,16], zero on entry; per Gaussian the kernel adds
 *   [0:2]  dL/dmeans2D (x,y)          [4:6]  sum |dL/dmeans2D| (x,y)
 *   [8:12] dL/dconic_opacity (c00, c01, c11, opacity)
 *   [12:15] dL/dcolors (r,g,b); other slots stay zero.
 * (The c01 entry keeps the reference's convention: half the derivative with
 * respect to the stored off-diagonal conic entry.)
 * record_rows (may be NULL): row of Gaussian i's record, e.g. the slot_of map
 * of blitz_preprocess_forward_raw, so the record has one row per listed
 * Gaussian instead of P rows; NULL uses row i.
 * strip_ids / strip_pos / strip_counts (all three or NULL): the strip lists
 * blitz_render_blend recorded for this render; with them each strip replays
 * only the Gaussians that contributed to it (same result, less work).
 */
int blitz_render_backward(int64_t P, int image_height, int image_width, const uint32_t* point_list,
                          const uint32_t* ranges, const float* final_T, const uint32_t* n_contrib,
                          const float* means2D, const float* conic_opacity, const float* rgb,
                          const float* bg, const uint8_t* compute_locally, const float* dL_dpix,
                          const uint32_t* record_rows, const int32_t* strip_ids, const int32_t* strip_pos,
                          const int32_t* strip_counts, float* grad_accum, void* stream);

/*
 * Full (non-distributed) rasterizer.  Replaces _C.rasterize_gaussians,
 * _C.rasterize_gaussians_simp, _C.rasterize_gaussians_depth and
 * _C.mark_visible (submodule/diff-gaussian-rasterization_f/rasterize_points.cu:
 * 372-784, cuda_rasterizer/rasterizer_impl.cu:100-114, 119-191, 336-853,
 * forward.cu:292-845).  A forward is: blitz_preprocess_forward with culling
 * and rects -> blitz_rasterize_count -> (read the totals) ->
 * blitz_rasterize_bin -> blitz_render_blend (colour, no mask) or
 * blitz_rasterize_blend (with flag_max_count / simp statistics) or
 * blitz_rasterize_depth; its backward is blitz_render_backward over the same
 * lists, then blitz_preprocess_backward.
 *
 * blitz_rasterize_count: per-Gaussian tile counts over each Gaussian's float
 * half-extent rectangle (rects [P,2]) keeping only the tiles that pass the
 * exact tile test on conic_opacity (the Gaussian reaches alpha >= 1/255 at
 * the point of the tile's pixel-centre rectangle the test picks), and the
 * device totals {R, n_vis} (uint64 [2]).
 * blitz_rasterize_bin: the per-tile lists of those instances in (depth,
 * index) order -- point_list uint32 [R], ranges uint32 [n_tiles,2]; scratch
 * of blitz_render_scratch_bytes bytes.
 * blitz_rasterize_blend: the colour blend (as blitz_render_blend without a
 * tile mask) plus, each optional: max_count float [P] += 1 for the Gaussian
 * of largest weight alpha*T of every pixel (flag_max_count, and simp);
 * accum_w float [P] += alpha*T and accum_n int32 [P] += 1 over every
 * (pixel, Gaussian) blend (simp; together).  At least one must be given;
 * the arrays accumulate (zero them first).
 * blitz_rasterize_depth: the colour blend of rasterize_gaussians_depth with,
 * per pixel, the Gaussian of largest weight among those whose ray-ellipsoid
 * depth (3-sigma ellipsoid, rotations and scales as given) is >= 0: out_pts
 * [3,H,W] its closest ray point, out_depth [H,W], discriminants [H,W], gidx
 * int32 [H,W] (0 where none), accum_alpha [H,W] the final transmittance.
 * blitz_mark_visible: present uint8 [P] = view depth > 0.2 (projmatrix is
 * accepted for the reference's signature and not read).
 */
int blitz_rasterize_count(int64_t P, int image_height, int image_width, const float* means2D, const int32_t* radii,
                          const float* rects, const float* conic_opacity, uint32_t* counts, uint64_t* totals,
                          void* stream);
int blitz_rasterize_bin(int64_t P, int64_t n_vis, int64_t R, int image_height, int image_width, const float* means2D,
                        const float* depths, const int32_t* radii, const float* rects, const float* conic_opacity,
                        const uint32_t* counts, void* scratch, size_t scratch_bytes, uint32_t* point_list,
                        uint32_t* ranges, void* stream);
int blitz_rasterize_blend(int64_t P, int image_height, int image_width, const float* means2D,
                          const float* conic_opacity, const float* rgb, const float* bg, const uint32_t* point_list,
                          const uint32_t* ranges, float* final_T, uint32_t* n_contrib, float* out_color,
                          float* max_count, float* accum_w, int32_t* accum_n, void* stream);
int blitz_rasterize_depth(int64_t P, int image_height, int image_width, const float* means2D,
                          const float* conic_opacity, const float* rgb, const float* bg, const uint32_t* point_list,
                          const uint32_t* ranges, const float* means3D, const float* scales, const float* rotations,
                          const float* projmatrix, const float* campos, float* out_color, float* out_pts,
                          float* out_depth, float* accum_alpha, int32_t* gidx, float* discriminants, void* stream);
int blitz_mark_visible(int64_t P, const float* means3D, const float* viewmatrix, const float* projmatrix,
                       uint8_t* present, void* stream);

/*
 * Fused L1 + SSIM over a band [C,Hb,W] (forward).
 * Replaces pixelwise_l1_with_mask + pixelwise_ssim_with_mask and their sums
 * (utils/loss_utils.py:83-124, gaussian_renderer/loss_distribution.py:250-257).
 * gt: uint8 (divided by 255 and clamped, as the reference does) or fp32;
 * exactly one of gt_u8 / gt_f32 is non-NULL.  window11: HOST float[11], the
 * normalised 1D Gaussian window.  sums: device double[2] {sum |img-gt|,
 * sum SSIM}, zero on entry.  partials: device float [C,Hb,W,3] scratch kept
 * for the backward.
 */
int blitz_loss_forward(int C, int Hb, int W, const float* img, const uint8_t* gt_u8,
                       const float* gt_f32, const float* window11, float* partials, double* sums,
                       void* stream);

/* Backward: scale = device float[2] {dL/d(sum L1), dL/d(sum SSIM)};
 * writes dL_dimg [C,Hb,W]. */
int blitz_loss_backward(int C, int Hb, int W, const float* img, const uint8_t* gt_u8,
                        const float* gt_f32, const float* window11, const float* partials,
                        const float* scale, float* dL_dimg, void* stream);

/*
 * Multi-GPU exchange, receiving side (no counterpart in the reference, whose
 * all_to_all_communication_final splits the received tensors with PyTorch,
 * gaussian_renderer/__init__.py:22-189): the rows of one camera are the
 * n_segments runs [seg_start[s], seg_start[s] + seg_count[s]) of records
 * ([*,12] floats: c00 c01 c11 opacity | x y | r g b | depth radius-bits
 * min-axis-scale; 16-byte aligned), in order.  Writes conic [n,4] (16-byte
 * aligned), means2D [n,2], rgb [n,3], depths [n], radii int32 [n]; with reg
 * (device double[2], caller-zeroed) adds the sum of the min-axis scales of
 * the rows with radius > 0 and their count.  n_segments <= 32.
 */
int blitz_exchange_unpack(int n_segments, const int64_t* seg_start, const int64_t* seg_count, const float* records,
                          float* conic, float* means2D, float* rgb, float* depths, int32_t* radii, double* reg,
                          void* stream);

/*
 * Multi-GPU exchange, backward send side (no counterpart in the reference):
 * row r of the camera's render-backward record rec16 [n,16] (see
 * blitz_render_backward) becomes the 12-float gradient record
 * {dconic c00 c01 c11, dopacity | dx dy | dr dg db | |dx| |dy| | dmin-scale}
 * at send row seg_start[s] + (r - rows before run s); dmin-scale =
 * *reg_scale for rows with radius > 0 (reg_scale may be NULL: 0).
 * n = sum of seg_count; n_segments <= 32.
 */
int blitz_grad_records_pack(int n_segments, const int64_t* seg_start, const int64_t* seg_count, const float* rec16,
                            const int32_t* radii, const float* reg_scale, float* send, void* stream);

/*
 * Per-camera loss of the training step, on the device (no counterpart in
 * the reference, which forms it with PyTorch scalar ops in
 * gaussian_renderer/loss_distribution.py:307-322):
 *   loss = (1 - l) * (L1 / N3) + l * (1 - SSIM / N3) + w * reg / max(cnt, 1)
 * sums: device double[2] from blitz_loss_forward; reg: device double[2]
 * {sum of min-axis scales, count} from blitz_preprocess_forward_raw, or NULL
 * for no regulariser.  Rounded step by step in float32 as PyTorch's CUDA
 * kernels evaluate that expression on 0-dim float32 tensors (division by
 * the number N3 as multiplication by its float32 reciprocal).
 * out: device float[5] {loss, L1, SSIM, reg, cnt}.
 */
int blitz_loss_combine(const double* sums, const double* reg, float one_minus_lambda, float lambda, float n3,
                       float reg_weight, float* out, void* stream);

/*
 * Backward of blitz_loss_combine: from the upstream gradients of loss, L1
 * and SSIM (device floats; NULL counts as 0) and the forward's out, writes
 * scales = device float[3] {dLoss/d(sum L1), dLoss/d(sum SSIM), dLoss/d reg}
 * as PyTorch's autograd forms them; scales[0..1] is blitz_loss_backward's
 * scale, scales[2] the reg_scale of blitz_preprocess_backward_raw.
 */
int blitz_loss_combine_backward(const float* g_loss, const float* g_l1, const float* g_ss, const float* fwd_out,
                                float one_minus_lambda, float lambda, float n3, float reg_weight, float* scales,
                                void* stream);

/*
 * Binning totals to the host (no counterpart in the reference, whose
 * renderForward reads num_rendered back with a blocking cudaMemcpy,
 * r/cuda_rasterizer/rasterizer_impl.cu:621): copies totals (device int64[2]
 * {R, V}) and, when both are non-NULL, vis_count (device int32) to the host
 * and waits for the stream.  host_totals / host_vis should be pinned.
 * status / host_status (both NULL, or both given): a device status word of
 * the ordered scans (the first 4 bytes of a blitz_preprocess_forward_raw
 * scratch, or of a blitz_exchange_pack scratch) read in the same wait; when
 * it is non-zero it is cleared and the call returns BLITZ_ESCAN.
 */
int blitz_read_totals(const int64_t* totals, const int32_t* vis_count, const uint32_t* status, int64_t* host_totals,
                      int32_t* host_vis, uint32_t* host_status, void* stream);

/*
 * Zero n device buffers on a side stream, after the work already queued on
 * `stream` (no counterpart in the reference).  The library keeps one side
 * stream and two events per device.  blitz_zero_fill_wait(stream) makes
 * `stream` wait for the last fill issued on this device; call it before
 * `stream` touches the buffers.  Not re-entrant across host threads.
 */
int blitz_zero_fill_async(int n, void* const* ptrs, const size_t* bytes, void* stream);

/*
 * Zero the listed rows of up to 8 dense row-major arrays in one launch on
 * `stream` (no counterpart in the reference): row rows[i] of array a, i.e.
 * row_bytes[a] bytes (a multiple of 4) at arrays[a] + rows[i] * row_bytes[a].
 * rows: device uint32 [n_rows].  Used to reset the rows of a reused dense
 * gradient buffer that an earlier view wrote, instead of the whole buffer.
 */
int blitz_zero_rows(int n_arrays, void* const* arrays, const size_t* row_bytes, const uint32_t* rows, int64_t n_rows,
                    void* stream);
int blitz_zero_fill_wait(void* stream);

/*
 * Routing mask bool [P, mp_world_size] against per-rank tile rectangles:
 * rectangles int32 [mp_world_size, 4] = {tile row begin, row end, column
 * begin, column end} (widened by one tile with avoid_pixel_all2all; the
 * begin bounds only while positive).  As in the reference, the square tile
 * rect is tested without first rejecting an empty one.
 * Replaces _C.get_local2j_ids_bool_adjust_mode6 / GetLocal2jIdsBoolAdjustMode6CUDA
 * (submodule/diff-gaussian-rasterization_f/rasterize_points.cu:291-368).
 */
int blitz_get_local2j_ids_bool_adjust_mode6(int image_height, int image_width, int mp_rank, int mp_world_size,
                                            int64_t P, const float* means2D, const int32_t* radii,
                                            const int32_t* rectangles, int avoid_pixel_all2all, uint8_t* out,
                                            void* stream);

/*
 * Sparse Adam step of one parameter tensor [N, M] (M floats per Gaussian):
 * for every element of a Gaussian with visible[g] != 0,
 *   m = b1 m + (1-b1) g;  v = b2 v + (1-b2) g^2;  param -= lr m / (sqrt(v) + eps)
 * with the bias corrections folded into lr by the caller; invisible
 * Gaussians keep their parameter and moments.
 * Replaces _C.adamUpdate / ADAM::adamUpdate
 * (submodule/diff-gaussian-rasterization_f/rasterize_points.cu:807-833,
 * cuda_rasterizer/adam.cu:10-38), bit for bit.
 */
int blitz_adam_update(float* param, const float* param_grad, float* exp_avg, float* exp_avg_sq,
                      const uint8_t* visible, float lr, float b1, float b2, float eps, int64_t N, int64_t M,
                      void* stream);

/*
 * The same step for listed Gaussians only (no reference counterpart: the
 * reference always passes a dense gradient): grad_rows [n_rows, M] holds the
 * gradient of Gaussian rows[j] (int64, distinct) in row j -- the sparse
 * gradient of the fused step -- so nothing is read or written for the others.
 * grad_scale multiplies each gradient element first: the trainer's
 * `param.grad /= bsz` (train_internal.py:504-515) fused into the step, bit
 * for bit when grad_scale is the float32 reciprocal of bsz (how PyTorch
 * divides a float tensor by a host scalar); 1 leaves the gradient as given.
 */
int blitz_adam_update_rows(float* param, const float* grad_rows, float* exp_avg, float* exp_avg_sq,
                           const int64_t* rows, int64_t n_rows, float grad_scale, float lr, float b1, float b2,
                           float eps, int64_t N, int64_t M, void* stream);

/*
 * Send-buffer packing of one camera's exchange records (no reference
 * counterpart: the reference gathers with torch index_select per rank).
 * Row j < n_rows of records/dest_mask goes to every rank r with bit r set,
 * at row dest_offset[r] + k of send [*,12] (16-byte aligned), k counting
 * that rank's rows of this call in row order: each rank's segment keeps the
 * order of the rows (with the index-ordered list of the two-kernel
 * preprocess, ascending index order, the same on every run).  send_row
 * receives row_base + j there.  dest_offset: HOST int64 array [n_ranks]
 * (n_ranks <= 32).  scratch: device buffer of
 * blitz_exchange_pack_scratch_bytes(n_rows, n_ranks) bytes whose first 4
 * bytes are a status word (zero it once when allocated; check it with
 * blitz_read_totals); calls on one stream may share it.
 */
size_t blitz_exchange_pack_scratch_bytes(int64_t n_rows, int n_ranks);
int blitz_exchange_pack(int64_t n_rows, int n_ranks, const float* records, const uint32_t* dest_mask,
                        const int64_t* dest_offset, float* send, int32_t* send_row, int32_t row_base, void* scratch,
                        size_t scratch_bytes, void* stream);

/*
 * Batched forms for the multi-GPU step, which preprocesses, packs and
 * back-propagates every camera of a batch on every rank (no reference
 * counterpart: the reference calls its preprocess once per camera from
 * Python, gaussian_renderer/__init__.py:260-324).  Each call loops over the
 * cameras inside the library, so a batch costs one call instead of one per
 * camera.  Camera k's output rows start at row k*cam_stride of every output
 * (means2D + 2*k*cam_stride, records + 12*k*cam_stride, ...).
 *
 * blitz_preprocess_forward_raw_batch: blitz_preprocess_forward_raw with a
 * visible list (ascending index order) and the exchange outputs, for
 * n_cams cameras.  viewmatrices / projmatrices: device [n_cams][16];
 * campos: device [n_cams][3]; tanfov: HOST float [n_cams][2] (x, y).
 * counts: device int32 [n_cams][1 + n_ranks], zero on entry: [k][0] = list
 * length, [k][1 + r] = rows for rank r.  tile_bounds: device int32
 * [n_cams][2][n_ranks] (tile_lo row, then tile_hi row); n_ranks = 0 skips
 * the exchange outputs (records / dest_mask / tile_bounds may be NULL).
 * The cameras run side by side on up to 8 side streams the library keeps
 * per device, ordered after the work already on `stream`; `stream` waits for
 * all of them before the call returns.  scratch:
 * blitz_preprocess_batch_scratch_bytes(n_cams, P) bytes (a slice per
 * camera); its first 4 bytes are the status word of blitz_read_totals.
 */
size_t blitz_preprocess_batch_scratch_bytes(int n_cams, int64_t P);
int blitz_preprocess_forward_raw_batch(int n_cams, int64_t P, int D, int M, const float* xyz,
                                       const float* scaling_raw, const float* rotation_raw, const float* opacity_raw,
                                       const float* sh_dc, int64_t dc_stride, const float* sh_rest,
                                       int64_t rest_stride, float scale_modifier, const float* viewmatrices,
                                       const float* projmatrices, const float* campos, const float* tanfov,
                                       int image_height, int image_width, int64_t cam_stride, float* means2D,
                                       float* depths, int32_t* radii, float* conic_opacity, float* rgb,
                                       uint32_t* vis_list, int32_t* counts, int n_ranks, const int32_t* tile_bounds,
                                       float* records, uint32_t* dest_mask, void* scratch, size_t scratch_bytes,
                                       void* stream);

/*
 * blitz_exchange_pack_batch: blitz_exchange_pack for n_cams cameras.
 * n_rows, row_base: HOST int64 [n_cams]; dest_offset: HOST int64
 * [n_cams][n_ranks]; records / dest_mask rows of camera k start at row
 * k*cam_stride.  scratch: blitz_exchange_pack_scratch_bytes(max n_rows,
 * n_ranks) bytes.
 */
int blitz_exchange_pack_batch(int n_cams, int n_ranks, const int64_t* n_rows, int64_t cam_stride,
                              const float* records, const uint32_t* dest_mask, const int64_t* dest_offset,
                              const int64_t* row_base, float* send, int32_t* send_row, void* scratch,
                              size_t scratch_bytes, void* stream);

/*
 * blitz_preprocess_backward_raw_batch: the listed backward of every camera,
 * accumulated into the raw-parameter gradients (which the caller has
 * zero-filled or holds earlier contributions).  radii / means2D / vis_list
 * rows of camera k start at row k*cam_stride; counts as in the forward
 * batch (only [k][0] is read, with row stride counts_stride).  upstream:
 * the received 12-float gradient records [c00 c01 c11 op | x y | r g b |
 * |x| |y| d(min scale)], camera k's j-th listed Gaussian at row
 * upstream_row0[k] + j (upstream_row0: HOST int64 [n_cams]).
 */
int blitz_preprocess_backward_raw_batch(int n_cams, int64_t P, int D, int M, const int32_t* radii,
                                        const float* means2D, const uint32_t* vis_list, const int32_t* counts,
                                        int counts_stride, int64_t cam_stride, const float* xyz,
                                        const float* scaling_raw, const float* rotation_raw,
                                        const float* opacity_raw, const float* sh_dc, int64_t dc_stride,
                                        const float* sh_rest, int64_t rest_stride, float scale_modifier,
                                        const float* viewmatrices, const float* projmatrices, const float* campos,
                                        const float* tanfov, int image_height, int image_width,
                                        const float* upstream, const int64_t* upstream_row0, float* g_xyz,
                                        float* g_scaling_raw, float* g_rotation_raw, float* g_opacity_raw,
                                        float* g_dc, int64_t g_dc_stride, float* g_rest, int64_t g_rest_stride,
                                        void* stream);

/*
 * Routing mask bool [P, mp_world_size]: Gaussian i overlaps the tile-id
 * interval [dist_global_strategy[r], dist_global_strategy[r+1]) of rank r.
 * Replaces _C.get_local2j_ids_bool / GetLocal2jIdsBoolCUDA
 * (submodule/diff-gaussian-rasterization_f/rasterize_points.cu:212-288).
 */
int blitz_get_local2j_ids_bool(int image_height, int image_width, int mp_rank, int mp_world_size,
                               int64_t P, const float* means2D, const int32_t* radii,
                               const int32_t* dist_global_strategy, int avoid_pixel_all2all,
                               uint8_t* out, void* stream);

/*
 * MEASUREMENT-ONLY entry (no reference counterpart; not part of the
 * rasterizer's operator surface, and no operator calls it): `blocks` CTAs of 256
 * threads each run 8 independent FMA chains for `iters` iterations
 * (2*8*iters FLOP per thread); timing it gives the FP32 throughput used as
 * the blend kernels' roofline denominator.  sink: device float, never written
 * in practice.
 */
int blitz_fp32_probe(int blocks, int64_t iters, float* sink, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BLITZGS_B200_H_ */
