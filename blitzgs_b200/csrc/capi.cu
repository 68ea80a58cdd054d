// extern "C" entry points (declared in include/blitzgs_b200.h).
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "blitzgs_b200.h"
#include "common.cuh"
#include "kernels.h"

using namespace blitz;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* what) {
  char buf[512];
  if (code > 0 && code < 10000)
    snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString((cudaError_t)code));
  else
    snprintf(buf, sizeof(buf), "%s (status %d)", what, code);
  g_last_error = buf;
  return code;
}

int check(int code, const char* what) { return code == 0 ? 0 : fail(code, what); }

inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

PreprocessParams make_pp(int64_t P, int D, int M, const float* means3D, const float* scales,
                         const float* rotations, const float* dc, int64_t dc_stride,
                         const float* rest, int64_t rest_stride, const float* opacities,
                         float scale_modifier, const float* viewmatrix, const float* projmatrix,
                         const float* campos, float tanfovx, float tanfovy, int H, int W) {
  PreprocessParams p{};
  p.P = P;
  p.D = D;
  p.M = M;
  p.means3D = means3D;
  p.scales = scales;
  p.rotations = rotations;
  p.opacities = opacities;
  p.dc = dc;
  p.dc_stride = dc_stride;
  p.rest = rest;
  p.rest_stride = rest_stride;
  p.sh_packed16 = (M == 15 && dc_stride == 48 && rest_stride == 48 && rest == dc + 3 && aligned16(dc));
  p.scale_modifier = scale_modifier;
  p.viewmatrix = viewmatrix;
  p.projmatrix = projmatrix;
  p.campos = campos;
  p.tanfovx = tanfovx;
  p.tanfovy = tanfovy;
  // focal lengths exactly as the reference host code computes them
  p.focal_y = H / (2.0f * tanfovy);
  p.focal_x = W / (2.0f * tanfovx);
  p.W = W;
  p.H = H;
  p.grid_x = (W + kTileX - 1) / kTileX;
  p.grid_y = (H + kTileY - 1) / kTileY;
  return p;
}

static int preprocess_forward_raw_impl(int64_t P, int D, int M, const float* xyz, const float* scaling_raw,
                                 const float* rotation_raw, const float* rotation_norm,
                                 const float* opacity_raw, const float* sh_dc, int64_t dc_stride,
                                 const float* sh_rest, int64_t rest_stride, float scale_modifier,
                                 const float* viewmatrix, const float* projmatrix, const float* campos,
                                 float tanfovx, float tanfovy, int image_height, int image_width,
                                 float* means2D, float* depths, int32_t* radii, float* conic_opacity,
                                 float* rgb, double* reg_sums, uint32_t* vis_list, int32_t* vis_count,
                                 const uint8_t* compute_locally, uint32_t* counts, uint64_t* totals,
                                 uint32_t* slot_of, const blitz_exchange_out* exchange, void* scratch,
                                 size_t scratch_bytes, void* stream, int grid_share,
                                       unsigned* status) {
  if (P < 0 || D < 0 || D > 3 || M < 0 || M > 15 || image_height <= 0 || image_width <= 0)
    return fail(BLITZ_EINVAL, "blitz_preprocess_forward_raw: bad sizes");
  if (P == 0) return 0;
  if (!xyz || !scaling_raw || !rotation_raw || !opacity_raw || !sh_dc || !viewmatrix || !projmatrix || !campos ||
      !means2D || !depths || !radii || !conic_opacity || !rgb || (M > 0 && !sh_rest) || ((vis_list == nullptr) != (vis_count == nullptr)) ||
      ((counts == nullptr) != (totals == nullptr)))
    return fail(BLITZ_EINVAL, "blitz_preprocess_forward_raw: null pointer");
  if (P >= (int64_t)0xffffffff) return fail(BLITZ_EINVAL, "blitz_preprocess_forward_raw: P must be < 2^32");
  if (!aligned16(rotation_raw) || !aligned16(conic_opacity) || (reinterpret_cast<uintptr_t>(means2D) & 7u))
    return fail(BLITZ_EINVAL, "blitz_preprocess_forward_raw: alignment");
  PreprocessParams p = make_pp(P, D, M, xyz, scaling_raw, rotation_raw, sh_dc, dc_stride, sh_rest, rest_stride,
                               opacity_raw, scale_modifier, viewmatrix, projmatrix, campos, tanfovx, tanfovy,
                               image_height, image_width);
  p.raw = true;
  p.rot_norm = rotation_norm;
  p.reg_sums = reg_sums;
  p.vis_list_out = vis_list;
  p.vis_count_out = vis_count;
  p.listed_rows_only = vis_list != nullptr;
  if (slot_of && !vis_list) return fail(BLITZ_EINVAL, "blitz_preprocess_forward_raw: slot_of needs vis_list");
  p.slot_of_out = slot_of;
  if (exchange && exchange->n_ranks > 0) {
    const blitz_exchange_out& x = *exchange;
    if (!vis_list || x.n_ranks > 32 || !x.tile_lo || !x.tile_hi || !x.records || !x.dest_mask || !x.dest_counts)
      return fail(BLITZ_EINVAL, "blitz_preprocess_forward_raw: exchange outputs need vis_list, n_ranks <= 32 and "
                                "non-null buffers");
    if (!aligned16(x.records)) return fail(BLITZ_EINVAL, "blitz_preprocess_forward_raw: records must be 16-byte aligned");
    // the exchange must keep one order on every run: list in index order
    if (!scratch) return fail(BLITZ_EINVAL, "blitz_preprocess_forward_raw: exchange outputs need the scratch");
    p.ordered_list = true;
    p.x_ranks = x.n_ranks;
    p.x_tile_lo = x.tile_lo;
    p.x_tile_hi = x.tile_hi;
    p.x_records = x.records;
    p.x_mask = x.dest_mask;
    p.x_counts = x.dest_counts;
  }
  p.counts_out = counts;
  p.totals_out = reinterpret_cast<unsigned long long*>(totals);
  p.compute_locally = reinterpret_cast<const bool*>(compute_locally);
  p.out_means2D = means2D;
  p.out_depths = depths;
  p.out_radii = radii;
  p.out_conic_opacity = conic_opacity;
  p.out_rgb = rgb;
  if (scratch && scratch_bytes < preprocess_scratch_bytes(P))
    return fail(BLITZ_ESCRATCH, "blitz_preprocess_forward_raw: scratch smaller than blitz_preprocess_scratch_bytes(P)");
  return check(launch_preprocess_fwd(p, S(stream), scratch, scratch_bytes, grid_share, status),
               "blitz_preprocess_forward_raw");
}

}  // namespace

namespace blitz {
void set_last_error(const char* msg) { g_last_error = msg; }
}  // namespace blitz

extern "C" {

const char* blitz_version(void) { return "blitzgs_b200 0.1 (sm_100a)"; }

const char* blitz_last_error(void) { return g_last_error.c_str(); }

int blitz_preprocess_forward(int64_t P, int D, int M, const float* means3D, const float* scales,
                             const float* rotations, const float* sh_dc, int64_t dc_stride,
                             const float* sh_rest, int64_t rest_stride, const float* opacities,
                             float scale_modifier, const float* viewmatrix, const float* projmatrix,
                             const float* campos, float tanfovx, float tanfovy, int image_height,
                             int image_width, int prefiltered, float* means2D, float* depths,
                             int32_t* radii, float* cov3D, float* conic_opacity, float* rgb,
                             uint8_t* clamped, const uint8_t* culling, float* rects, uint32_t* error_word,
                             void* stream) {
  if (P < 0 || D < 0 || D > 3 || M < 0 || M > 15 || image_height <= 0 || image_width <= 0)
    return fail(BLITZ_EINVAL, "blitz_preprocess_forward: bad sizes");
  if (P == 0) return 0;
  if (!means3D || !scales || !rotations || !sh_dc || !opacities || !viewmatrix || !projmatrix ||
      !campos || !means2D || !depths || !radii || !conic_opacity || !rgb || (M > 0 && !sh_rest))
    return fail(BLITZ_EINVAL, "blitz_preprocess_forward: null pointer");
  if (!aligned16(rotations) || !aligned16(conic_opacity) || (reinterpret_cast<uintptr_t>(means2D) & 7u) ||
      (reinterpret_cast<uintptr_t>(rects) & 7u))
    return fail(BLITZ_EINVAL,
                "blitz_preprocess_forward: rotations/conic_opacity need 16-byte, means2D/rects 8-byte alignment");
  if (prefiltered && !error_word)
    return fail(BLITZ_EINVAL, "blitz_preprocess_forward: prefiltered=1 needs an error word");
  PreprocessParams p = make_pp(P, D, M, means3D, scales, rotations, sh_dc, dc_stride, sh_rest,
                               rest_stride, opacities, scale_modifier, viewmatrix, projmatrix,
                               campos, tanfovx, tanfovy, image_height, image_width);
  p.prefiltered = prefiltered != 0;
  p.out_means2D = means2D;
  p.out_depths = depths;
  p.out_radii = radii;
  p.out_conic_opacity = conic_opacity;
  p.out_rgb = rgb;
  p.out_clamped = reinterpret_cast<bool*>(clamped);
  p.out_cov3D = cov3D;
  p.culling = reinterpret_cast<const bool*>(culling);
  p.out_rects = rects;
  p.error_flag = error_word;
  return check(launch_preprocess_fwd(p, S(stream)), "blitz_preprocess_forward");
}

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
                              int accumulate, void* stream) {
  if (P < 0 || D < 0 || D > 3 || M < 0 || M > 15 || image_height <= 0 || image_width <= 0)
    return fail(BLITZ_EINVAL, "blitz_preprocess_backward: bad sizes");
  if (P == 0) return 0;
  if (!radii || !means3D || !scales || !rotations || !sh_dc || !g_means2D || !g_conic_opacity ||
      !g_colors || !dL_dmeans3D || !dL_dscales || !dL_drotations || !g_dc || (M > 0 && (!sh_rest || !g_rest)))
    return fail(BLITZ_EINVAL, "blitz_preprocess_backward: null pointer");
  if (!aligned16(rotations) || !aligned16(dL_drotations) || !aligned16(g_conic_opacity) ||
      (g_conic_stride & 3))
    return fail(BLITZ_EINVAL, "blitz_preprocess_backward: 16-byte alignment required");
  PreprocessBwdParams b{};
  b.f = make_pp(P, D, M, means3D, scales, rotations, sh_dc, dc_stride, sh_rest, rest_stride, nullptr,
                scale_modifier, viewmatrix, projmatrix, campos, tanfovx, tanfovy, image_height,
                image_width);
  b.radii = radii;
  b.g_means2D = g_means2D;
  b.g_means2D_stride = g_means2D_stride;
  b.g_conic_opacity = g_conic_opacity;
  b.g_conic_stride = g_conic_stride;
  b.g_colors = g_colors;
  b.g_colors_stride = g_colors_stride;
  b.g_means3D = dL_dmeans3D;
  b.g_scales = dL_dscales;
  b.g_rotations = dL_drotations;
  b.g_opacities = dL_dopacity;
  b.g_dc = g_dc;
  b.g_dc_stride = g_dc_stride;
  b.g_rest = g_rest;
  b.g_rest_stride = g_rest_stride;
  return check(launch_preprocess_bwd(b, accumulate != 0, S(stream)), "blitz_preprocess_backward");
}

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
                                 size_t scratch_bytes, void* stream) {
  return preprocess_forward_raw_impl(P, D, M, xyz, scaling_raw, rotation_raw, rotation_norm, opacity_raw, sh_dc,
                                     dc_stride, sh_rest, rest_stride, scale_modifier, viewmatrix, projmatrix, campos,
                                     tanfovx, tanfovy, image_height, image_width, means2D, depths, radii,
                                     conic_opacity, rgb, reg_sums, vis_list, vis_count, compute_locally, counts,
                                     totals, slot_of, exchange, scratch, scratch_bytes, stream, 1, nullptr);
}

size_t blitz_preprocess_scratch_bytes(int64_t P) { return preprocess_scratch_bytes(P); }

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
                                  int accumulate, int rows, void* stream) {
  if (P < 0 || D < 0 || D > 3 || M < 0 || M > 15 || image_height <= 0 || image_width <= 0)
    return fail(BLITZ_EINVAL, "blitz_preprocess_backward_raw: bad sizes");
  if (P == 0) return 0;
  if (!radii || !means2D || !xyz || !scaling_raw || !rotation_raw || !opacity_raw || !sh_dc || !g_means2D ||
      !g_conic_opacity || !g_colors || !g_xyz || !g_scaling_raw || !g_rotation_raw || !g_dc ||
      (M > 0 && (!sh_rest || !g_rest)) || ((vis_list == nullptr) != (vis_count == nullptr)))
    return fail(BLITZ_EINVAL, "blitz_preprocess_backward_raw: null pointer");
  if (!aligned16(rotation_raw) || !aligned16(g_rotation_raw) || !aligned16(g_conic_opacity) || (g_conic_stride & 3))
    return fail(BLITZ_EINVAL, "blitz_preprocess_backward_raw: 16-byte alignment required");
  PreprocessBwdParams b{};
  b.f = make_pp(P, D, M, xyz, scaling_raw, rotation_raw, sh_dc, dc_stride, sh_rest, rest_stride, opacity_raw,
                scale_modifier, viewmatrix, projmatrix, campos, tanfovx, tanfovy, image_height, image_width);
  b.f.raw = true;
  b.f.rot_norm = rotation_norm;
  b.radii = radii;
  b.means2D = means2D;
  b.reg_scale = reg_scale;
  b.vis_list = vis_list;
  b.vis_count = vis_count;
  if ((rows & ~(BLITZ_ROWS_UPSTREAM_BY_SLOT | BLITZ_ROWS_OUTPUT_BY_SLOT)) || (rows && !vis_list))
    return fail(BLITZ_EINVAL, "blitz_preprocess_backward_raw: bad rows flags (slot rows need vis_list)");
  b.g_minscale = g_minscale;
  b.g_minscale_stride = g_minscale_stride;
  b.upstream_by_slot = rows & BLITZ_ROWS_UPSTREAM_BY_SLOT;
  b.out_by_slot = rows & BLITZ_ROWS_OUTPUT_BY_SLOT;
  b.g_means2D = g_means2D;
  b.g_means2D_stride = g_means2D_stride;
  b.g_conic_opacity = g_conic_opacity;
  b.g_conic_stride = g_conic_stride;
  b.g_colors = g_colors;
  b.g_colors_stride = g_colors_stride;
  b.g_means3D = g_xyz;
  b.g_scales = g_scaling_raw;
  b.g_rotations = g_rotation_raw;
  b.g_opacities = g_opacity_raw;
  b.g_dc = g_dc;
  b.g_dc_stride = g_dc_stride;
  b.g_rest = g_rest;
  b.g_rest_stride = g_rest_stride;
  return check(launch_preprocess_bwd(b, accumulate != 0, S(stream)), "blitz_preprocess_backward_raw");
}

int blitz_render_count(int64_t P, int image_height, int image_width, const float* means2D,
                       const int32_t* radii, const uint8_t* compute_locally, uint32_t* counts,
                       uint64_t* totals, void* stream) {
  if (P < 0 || image_height <= 0 || image_width <= 0 || !totals || (P > 0 && (!means2D || !radii || !counts)))
    return fail(BLITZ_EINVAL, "blitz_render_count: bad arguments");
  if (P >= (int64_t)0xffffffff) return fail(BLITZ_EINVAL, "blitz_render_count: P must be < 2^32");
  BinParams b{};
  b.P = P;
  b.W = image_width;
  b.H = image_height;
  b.grid_x = (image_width + kTileX - 1) / kTileX;
  b.grid_y = (image_height + kTileY - 1) / kTileY;
  b.means2D = means2D;
  b.radii = radii;
  b.compute_locally = reinterpret_cast<const bool*>(compute_locally);
  b.counts = counts;
  b.totals = reinterpret_cast<unsigned long long*>(totals);
  return check(launch_bin_count(b, S(stream)), "blitz_render_count");
}

size_t blitz_render_scratch_bytes(int64_t P, int64_t n_vis, int64_t R, int image_height, int image_width) {
  const int gx = (image_width + kTileX - 1) / kTileX, gy = (image_height + kTileY - 1) / kTileY;
  return bin_scratch_bytes(P, n_vis, R, gx * gy);
}

namespace {

int render_bin_impl(int64_t P, int64_t n_vis, int64_t R, int image_height, int image_width, const float* means2D,
                    const float* depths, const int32_t* radii, const uint8_t* compute_locally, const uint32_t* counts,
                    void* scratch, size_t scratch_bytes, uint32_t* point_list, uint32_t* ranges, cudaStream_t st,
                    const float* rects = nullptr, const float* conic_opacity = nullptr) {
  const int gx = (image_width + kTileX - 1) / kTileX, gy = (image_height + kTileY - 1) / kTileY;
  if (R > 0 && scratch_bytes < bin_scratch_bytes(P, n_vis, R, gx * gy))
    return fail(BLITZ_ESCRATCH, "render binning: scratch too small");
  BinSortParams bs{};
  bs.b.P = P;
  bs.b.W = image_width;
  bs.b.H = image_height;
  bs.b.grid_x = gx;
  bs.b.grid_y = gy;
  bs.b.means2D = means2D;
  bs.b.depths = depths;
  bs.b.radii = radii;
  bs.b.compute_locally = reinterpret_cast<const bool*>(compute_locally);
  bs.b.counts = const_cast<uint32_t*>(counts);
  bs.b.rects = rects;
  bs.b.conic_opacity = conic_opacity;
  bs.n_vis = n_vis;
  bs.R = R;
  bs.scratch = scratch;
  bs.scratch_bytes = scratch_bytes;
  bs.point_list = point_list;
  bs.ranges = reinterpret_cast<uint2*>(ranges);
  return check(launch_bin_sort(bs, st), "render binning");
}

int render_blend_impl(int64_t P, int image_height, int image_width, const float* means2D, const float* conic_opacity,
                      const float* rgb, const float* bg, const uint8_t* compute_locally, const uint32_t* point_list,
                      const uint32_t* ranges, float* final_T, uint32_t* n_contrib, float* out_color,
                      int32_t* n_render, int32_t* n_consider, int32_t* n_contrib_tile, int32_t* out_observe,
                      int32_t* strip_ids, int32_t* strip_pos, int32_t* strip_counts, cudaStream_t st) {
  BlendFwdParams f{};
  f.W = image_width;
  f.H = image_height;
  f.grid_x = (image_width + kTileX - 1) / kTileX;
  f.grid_y = (image_height + kTileY - 1) / kTileY;
  f.P = P;
  f.ranges = reinterpret_cast<const uint2*>(ranges);
  f.point_list = point_list;
  f.means2D = means2D;
  f.conic_opacity = conic_opacity;
  f.rgb = rgb;
  f.bg = bg;
  f.compute_locally = reinterpret_cast<const bool*>(compute_locally);
  f.out_color = out_color;
  f.final_T = final_T;
  f.n_contrib = n_contrib;
  f.out_observe = out_observe;
  f.n_render = n_render;
  f.n_consider = n_consider;
  f.n_contrib_tile = n_contrib_tile;
  f.strip_ids = strip_ids;
  f.strip_pos = strip_pos;
  f.strip_counts = strip_counts;
  return check(launch_blend_fwd(f, st), "render blend");
}

bool render_args_ok(int64_t P, int64_t n_vis, int64_t R, int H, int W) {
  return !(P < 0 || n_vis < 0 || R < 0 || R >= (int64_t)0x7fffffff || n_vis > P || H <= 0 || W <= 0);
}

}  // namespace

int blitz_render_forward(int64_t P, int64_t n_vis, int64_t R, int image_height, int image_width,
                         const float* means2D, const float* depths, const int32_t* radii,
                         const float* conic_opacity, const float* rgb, const float* bg,
                         const uint8_t* compute_locally, const uint32_t* counts, void* scratch,
                         size_t scratch_bytes, uint32_t* point_list, uint32_t* ranges,
                         float* final_T, uint32_t* n_contrib, float* out_color, int32_t* n_render,
                         int32_t* n_consider, int32_t* n_contrib_tile, int32_t* out_observe,
                         void* stream) {
  int e = blitz_render_bin(P, n_vis, R, image_height, image_width, means2D, depths, radii, compute_locally, counts,
                           scratch, scratch_bytes, point_list, ranges, stream);
  if (e) return e;
  return blitz_render_blend(P, image_height, image_width, means2D, conic_opacity, rgb, bg, compute_locally,
                            point_list, ranges, final_T, n_contrib, out_color, n_render, n_consider, n_contrib_tile,
                            out_observe, nullptr, nullptr, nullptr, stream);
}

int blitz_render_bin(int64_t P, int64_t n_vis, int64_t R, int image_height, int image_width, const float* means2D,
                     const float* depths, const int32_t* radii, const uint8_t* compute_locally, const uint32_t* counts,
                     void* scratch, size_t scratch_bytes, uint32_t* point_list, uint32_t* ranges, void* stream) {
  if (!render_args_ok(P, n_vis, R, image_height, image_width)) return fail(BLITZ_EINVAL, "blitz_render_bin: bad sizes");
  if (!ranges || (P > 0 && (!means2D || !depths || !radii || !counts)) || (R > 0 && (!point_list || !scratch)))
    return fail(BLITZ_EINVAL, "blitz_render_bin: null pointer");
  if (P > 0 && (reinterpret_cast<uintptr_t>(means2D) & 7u)) return fail(BLITZ_EINVAL, "blitz_render_bin: means2D alignment");
  return render_bin_impl(P, n_vis, R, image_height, image_width, means2D, depths, radii, compute_locally, counts,
                         scratch, scratch_bytes, point_list, ranges, S(stream));
}

int blitz_render_blend(int64_t P, int image_height, int image_width, const float* means2D, const float* conic_opacity,
                       const float* rgb, const float* bg, const uint8_t* compute_locally, const uint32_t* point_list,
                       const uint32_t* ranges, float* final_T, uint32_t* n_contrib, float* out_color,
                       int32_t* n_render, int32_t* n_consider, int32_t* n_contrib_tile, int32_t* out_observe,
                       int32_t* strip_ids, int32_t* strip_pos, int32_t* strip_counts, void* stream) {
  if (!render_args_ok(P, 0, 0, image_height, image_width)) return fail(BLITZ_EINVAL, "blitz_render_blend: bad sizes");
  if ((strip_ids == nullptr) != (strip_pos == nullptr) || (strip_ids == nullptr) != (strip_counts == nullptr))
    return fail(BLITZ_EINVAL, "blitz_render_blend: strip_ids, strip_pos and strip_counts go together");
  if (!bg || !ranges || !final_T || !n_contrib || !out_color || !n_render || !n_consider || !n_contrib_tile ||
      (P > 0 && (!means2D || !conic_opacity || !rgb || !out_observe || !point_list)))
    return fail(BLITZ_EINVAL, "blitz_render_blend: null pointer");
  if (P > 0 && (!aligned16(conic_opacity) || (reinterpret_cast<uintptr_t>(means2D) & 7u)))
    return fail(BLITZ_EINVAL, "blitz_render_blend: conic_opacity needs 16-byte, means2D 8-byte alignment");
  return render_blend_impl(P, image_height, image_width, means2D, conic_opacity, rgb, bg, compute_locally, point_list,
                           ranges, final_T, n_contrib, out_color, n_render, n_consider, n_contrib_tile, out_observe,
                           strip_ids, strip_pos, strip_counts, S(stream));
}

int blitz_render_backward(int64_t P, int image_height, int image_width, const uint32_t* point_list,
                          const uint32_t* ranges, const float* final_T, const uint32_t* n_contrib,
                          const float* means2D, const float* conic_opacity, const float* rgb,
                          const float* bg, const uint8_t* compute_locally, const float* dL_dpix,
                          const uint32_t* record_rows, const int32_t* strip_ids, const int32_t* strip_pos,
                          const int32_t* strip_counts, float* grad_accum, void* stream) {
  if (P < 0 || image_height <= 0 || image_width <= 0)
    return fail(BLITZ_EINVAL, "blitz_render_backward: bad sizes");
  if ((strip_ids == nullptr) != (strip_pos == nullptr) || (strip_ids == nullptr) != (strip_counts == nullptr))
    return fail(BLITZ_EINVAL, "blitz_render_backward: strip_ids, strip_pos and strip_counts go together");
  if (!ranges || !final_T || !n_contrib || !bg || !dL_dpix ||
      (P > 0 && (!means2D || !conic_opacity || !rgb || !grad_accum)))
    return fail(BLITZ_EINVAL, "blitz_render_backward: null pointer");
  if (P > 0 && (!aligned16(conic_opacity) || !aligned16(grad_accum)))
    return fail(BLITZ_EINVAL, "blitz_render_backward: 16-byte alignment required");
  BlendBwdParams b{};
  b.W = image_width;
  b.H = image_height;
  b.grid_x = (image_width + kTileX - 1) / kTileX;
  b.grid_y = (image_height + kTileY - 1) / kTileY;
  b.P = P;
  b.ranges = reinterpret_cast<const uint2*>(ranges);
  b.point_list = point_list;
  b.means2D = means2D;
  b.conic_opacity = conic_opacity;
  b.rgb = rgb;
  b.bg = bg;
  b.compute_locally = reinterpret_cast<const bool*>(compute_locally);
  b.final_T = final_T;
  b.n_contrib = n_contrib;
  b.dL_dpix = dL_dpix;
  b.grad_accum = grad_accum;
  b.record_rows = record_rows;
  b.strip_ids = strip_ids;
  b.strip_pos = strip_pos;
  b.strip_counts = strip_counts;
  return check(launch_blend_bwd(b, S(stream)), "blitz_render_backward");
}

int blitz_loss_forward(int C, int Hb, int W, const float* img, const uint8_t* gt_u8,
                       const float* gt_f32, const float* window11, float* partials, double* sums,
                       void* stream) {
  if (C < 0 || Hb < 0 || W < 0 || !window11 || !sums || ((gt_u8 == nullptr) == (gt_f32 == nullptr)))
    return fail(BLITZ_EINVAL, "blitz_loss_forward: bad arguments");
  if ((int64_t)C * Hb * W > 0 && (!img || !partials)) return fail(BLITZ_EINVAL, "blitz_loss_forward: null pointer");
  LossParams p{C, Hb, W, img, gt_u8, gt_f32, partials};
  return check(launch_loss_fwd(p, window11, sums, S(stream)), "blitz_loss_forward");
}

int blitz_loss_backward(int C, int Hb, int W, const float* img, const uint8_t* gt_u8,
                        const float* gt_f32, const float* window11, const float* partials,
                        const float* scale, float* dL_dimg, void* stream) {
  if (C < 0 || Hb < 0 || W < 0 || !window11 || !scale || ((gt_u8 == nullptr) == (gt_f32 == nullptr)))
    return fail(BLITZ_EINVAL, "blitz_loss_backward: bad arguments");
  if ((int64_t)C * Hb * W > 0 && (!img || !partials || !dL_dimg))
    return fail(BLITZ_EINVAL, "blitz_loss_backward: null pointer");
  LossBwdParams b{};
  b.f = LossParams{C, Hb, W, img, gt_u8, gt_f32, const_cast<float*>(partials)};
  b.scale = scale;
  b.dL_dimg = dL_dimg;
  return check(launch_loss_bwd(b, window11, S(stream)), "blitz_loss_backward");
}

int blitz_get_local2j_ids_bool(int image_height, int image_width, int mp_rank, int mp_world_size,
                               int64_t P, const float* means2D, const int32_t* radii,
                               const int32_t* dist_global_strategy, int avoid_pixel_all2all,
                               uint8_t* out, void* stream) {
  (void)mp_rank;
  if (P < 0 || mp_world_size <= 0 || image_height <= 0 || image_width <= 0)
    return fail(BLITZ_EINVAL, "blitz_get_local2j_ids_bool: bad sizes");
  if (P == 0) return 0;
  if (!means2D || !radii || !dist_global_strategy || !out)
    return fail(BLITZ_EINVAL, "blitz_get_local2j_ids_bool: null pointer");
  RouteParams r{};
  r.P = P;
  r.W = image_width;
  r.H = image_height;
  r.grid_x = (image_width + kTileX - 1) / kTileX;
  r.grid_y = (image_height + kTileY - 1) / kTileY;
  r.world_size = mp_world_size;
  r.means2D = means2D;
  r.radii = radii;
  r.dist_global_strategy = dist_global_strategy;
  r.avoid_pixel_all2all = avoid_pixel_all2all != 0;
  r.out_bool = reinterpret_cast<bool*>(out);
  return check(launch_route_bool(r, S(stream)), "blitz_get_local2j_ids_bool");
}

int blitz_get_local2j_ids_bool_adjust_mode6(int image_height, int image_width, int mp_rank, int mp_world_size,
                                            int64_t P, const float* means2D, const int32_t* radii,
                                            const int32_t* rectangles, int avoid_pixel_all2all, uint8_t* out,
                                            void* stream) {
  (void)mp_rank;
  if (P < 0 || mp_world_size <= 0 || image_height <= 0 || image_width <= 0)
    return fail(BLITZ_EINVAL, "blitz_get_local2j_ids_bool_adjust_mode6: bad sizes");
  if (P == 0) return 0;
  if (!means2D || !radii || !rectangles || !out)
    return fail(BLITZ_EINVAL, "blitz_get_local2j_ids_bool_adjust_mode6: null pointer");
  RouteParams r{};
  r.P = P;
  r.W = image_width;
  r.H = image_height;
  r.grid_x = (image_width + kTileX - 1) / kTileX;
  r.grid_y = (image_height + kTileY - 1) / kTileY;
  r.world_size = mp_world_size;
  r.means2D = means2D;
  r.radii = radii;
  r.avoid_pixel_all2all = avoid_pixel_all2all != 0;
  r.out_bool = reinterpret_cast<bool*>(out);
  return check(launch_route_bool_rect(r, rectangles, S(stream)), "blitz_get_local2j_ids_bool_adjust_mode6");
}

int blitz_adam_update(float* param, const float* param_grad, float* exp_avg, float* exp_avg_sq,
                      const uint8_t* visible, float lr, float b1, float b2, float eps, int64_t N, int64_t M,
                      void* stream) {
  if (N < 0 || M <= 0) return fail(BLITZ_EINVAL, "blitz_adam_update: bad sizes");
  if (N == 0) return 0;
  if (!param || !param_grad || !exp_avg || !exp_avg_sq || !visible)
    return fail(BLITZ_EINVAL, "blitz_adam_update: null pointer");
  AdamParams a{};
  a.param = param;
  a.grad = param_grad;
  a.exp_avg = exp_avg;
  a.exp_avg_sq = exp_avg_sq;
  a.visible = reinterpret_cast<const bool*>(visible);
  a.lr = lr;
  a.b1 = b1;
  a.b2 = b2;
  a.eps = eps;
  a.N = N;
  a.M = M;
  return check(launch_adam(a, S(stream)), "blitz_adam_update");
}

int blitz_adam_update_rows(float* param, const float* grad_rows, float* exp_avg, float* exp_avg_sq,
                           const int64_t* rows, int64_t n_rows, float grad_scale, float lr, float b1, float b2,
                           float eps, int64_t N, int64_t M, void* stream) {
  if (N < 0 || M <= 0 || n_rows < 0) return fail(BLITZ_EINVAL, "blitz_adam_update_rows: bad sizes");
  if (n_rows == 0) return 0;
  if (!param || !grad_rows || !exp_avg || !exp_avg_sq || !rows)
    return fail(BLITZ_EINVAL, "blitz_adam_update_rows: null pointer");
  AdamParams a{};
  a.param = param;
  a.grad = grad_rows;
  a.exp_avg = exp_avg;
  a.exp_avg_sq = exp_avg_sq;
  a.rows = rows;
  a.n_rows = n_rows;
  a.grad_scale = grad_scale;
  a.lr = lr;
  a.b1 = b1;
  a.b2 = b2;
  a.eps = eps;
  a.N = N;
  a.M = M;
  return check(launch_adam(a, S(stream)), "blitz_adam_update_rows");
}

size_t blitz_exchange_pack_scratch_bytes(int64_t n_rows, int n_ranks) {
  return exchange_pack_scratch_bytes(n_rows, n_ranks);
}

int blitz_exchange_pack(int64_t n_rows, int n_ranks, const float* records, const uint32_t* dest_mask,
                        const int64_t* dest_offset, float* send, int32_t* send_row, int32_t row_base, void* scratch,
                        size_t scratch_bytes, void* stream) {
  if (n_rows < 0 || n_ranks <= 0 || n_ranks > 32) return fail(BLITZ_EINVAL, "blitz_exchange_pack: bad sizes");
  if (n_rows == 0) return 0;
  if (!records || !dest_mask || !dest_offset || !send || !send_row || !scratch)
    return fail(BLITZ_EINVAL, "blitz_exchange_pack: null pointer");
  if (!aligned16(records) || !aligned16(send)) return fail(BLITZ_EINVAL, "blitz_exchange_pack: 16-byte alignment");
  if (scratch_bytes < exchange_pack_scratch_bytes(n_rows, n_ranks))
    return fail(BLITZ_ESCRATCH, "blitz_exchange_pack: scratch smaller than blitz_exchange_pack_scratch_bytes");
  PackParams k{};
  k.n_rows = n_rows;
  k.n_ranks = n_ranks;
  for (int r = 0; r < n_ranks; ++r) k.dest_offset[r] = dest_offset[r];
  k.records = records;
  k.mask = dest_mask;
  k.send = send;
  k.send_row = send_row;
  k.row_base = row_base;
  return check(launch_exchange_pack(k, scratch, S(stream)), "blitz_exchange_pack");
}

int blitz_exchange_pack_batch(int n_cams, int n_ranks, const int64_t* n_rows, int64_t cam_stride,
                              const float* records, const uint32_t* dest_mask, const int64_t* dest_offset,
                              const int64_t* row_base, float* send, int32_t* send_row, void* scratch,
                              size_t scratch_bytes, void* stream) {
  if (n_cams < 0 || n_ranks <= 0 || n_ranks > 32 || cam_stride < 0)
    return fail(BLITZ_EINVAL, "blitz_exchange_pack_batch: bad sizes");
  if (n_cams == 0) return 0;
  if (!n_rows || !dest_offset || !row_base) return fail(BLITZ_EINVAL, "blitz_exchange_pack_batch: null pointer");
  for (int c = 0; c < n_cams; ++c) {
    if (n_rows[c] < 0 || n_rows[c] > cam_stride || row_base[c] < 0 || row_base[c] > 0x7fffffff)
      return fail(BLITZ_EINVAL, "blitz_exchange_pack_batch: bad rows");
    const int rc = blitz_exchange_pack(n_rows[c], n_ranks, records ? records + 12 * c * cam_stride : nullptr,
                                       dest_mask ? dest_mask + c * cam_stride : nullptr, dest_offset + c * n_ranks,
                                       send, send_row, (int32_t)row_base[c], scratch, scratch_bytes, stream);
    if (rc) return rc;
  }
  return 0;
}

}  // extern "C"

namespace {

// Side streams on which the batched preprocess runs its cameras side by
// side, per device (created on first use; the library's only other
// resources are the zero fill's stream and events).
constexpr int kBatchStreams = 8;
struct BatchStreams {
  bool ready = false;
  cudaStream_t s[kBatchStreams] = {};
  cudaEvent_t fork = nullptr, join[kBatchStreams] = {};
};
BatchStreams g_batch[64];
std::mutex g_batch_mu;

int batch_streams(BatchStreams** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= 64) return BLITZ_EINVAL;
  BatchStreams& b = g_batch[dev];
  if (!b.ready) {
    std::lock_guard<std::mutex> lock(g_batch_mu);
    if (!b.ready) {
      e = cudaEventCreateWithFlags(&b.fork, cudaEventDisableTiming);
      for (int i = 0; i < kBatchStreams && e == cudaSuccess; ++i) {
        e = cudaStreamCreateWithFlags(&b.s[i], cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&b.join[i], cudaEventDisableTiming);
      }
      if (e != cudaSuccess) return (int)e;
      b.ready = true;
    }
  }
  *out = &b;
  return 0;
}

size_t batch_slice_bytes(int64_t P) { return (preprocess_scratch_bytes(P) + 255) / 256 * 256; }

}  // namespace

extern "C" {

size_t blitz_preprocess_batch_scratch_bytes(int n_cams, int64_t P) {
  return (size_t)std::max(n_cams, 1) * batch_slice_bytes(P);
}

int blitz_preprocess_forward_raw_batch(int n_cams, int64_t P, int D, int M, const float* xyz,
                                       const float* scaling_raw, const float* rotation_raw, const float* opacity_raw,
                                       const float* sh_dc, int64_t dc_stride, const float* sh_rest,
                                       int64_t rest_stride, float scale_modifier, const float* viewmatrices,
                                       const float* projmatrices, const float* campos, const float* tanfov,
                                       int image_height, int image_width, int64_t cam_stride, float* means2D,
                                       float* depths, int32_t* radii, float* conic_opacity, float* rgb,
                                       uint32_t* vis_list, int32_t* counts, int n_ranks, const int32_t* tile_bounds,
                                       float* records, uint32_t* dest_mask, void* scratch, size_t scratch_bytes,
                                       void* stream) {
  if (n_cams < 0 || n_ranks < 0 || n_ranks > 32 || cam_stride < P)
    return fail(BLITZ_EINVAL, "blitz_preprocess_forward_raw_batch: bad sizes");
  if (n_cams == 0 || P == 0) return 0;
  if (!viewmatrices || !projmatrices || !campos || !tanfov || !vis_list || !counts || !scratch)
    return fail(BLITZ_EINVAL, "blitz_preprocess_forward_raw_batch: null pointer");
  if (n_ranks > 0 && (!tile_bounds || !records || !dest_mask))
    return fail(BLITZ_EINVAL, "blitz_preprocess_forward_raw_batch: exchange outputs need tile_bounds, records, "
                              "dest_mask");
  if ((cam_stride & 3) != 0) return fail(BLITZ_EINVAL, "blitz_preprocess_forward_raw_batch: cam_stride % 4");
  const size_t slice = batch_slice_bytes(P);
  if (scratch_bytes < (size_t)n_cams * slice)
    return fail(BLITZ_ESCRATCH, "blitz_preprocess_forward_raw_batch: scratch smaller than "
                                "blitz_preprocess_batch_scratch_bytes(n_cams, P)");
  BatchStreams* bs = nullptr;
  int rc0 = batch_streams(&bs);
  if (rc0) return fail(rc0, "blitz_preprocess_forward_raw_batch: side streams");
  // cameras run side by side on the side streams, each on its own scratch
  // slice; all report into the first slice's status word
  const int ns = std::min(n_cams, kBatchStreams);
  cudaError_t e = cudaEventRecord(bs->fork, S(stream));
  for (int i = 0; i < ns && e == cudaSuccess; ++i) e = cudaStreamWaitEvent(bs->s[i], bs->fork, 0);
  if (e != cudaSuccess) return check((int)e, "blitz_preprocess_forward_raw_batch: fork");
  unsigned* status = reinterpret_cast<unsigned*>(static_cast<char*>(scratch) + kPreStatusOffset);
  const int cs = 1 + n_ranks;
  int rc_all = 0;
  for (int c = 0; c < n_cams && !rc_all; ++c) {
    blitz_exchange_out x{};
    x.n_ranks = n_ranks;
    if (n_ranks > 0) {
      x.tile_lo = tile_bounds + (int64_t)c * 2 * n_ranks;
      x.tile_hi = tile_bounds + (int64_t)c * 2 * n_ranks + n_ranks;
      x.records = records + 12 * c * cam_stride;
      x.dest_mask = dest_mask + c * cam_stride;
      x.dest_counts = counts + (int64_t)c * cs + 1;
    }
    const int64_t o = c * cam_stride;
    rc_all = preprocess_forward_raw_impl(
        P, D, M, xyz, scaling_raw, rotation_raw, nullptr, opacity_raw, sh_dc, dc_stride, sh_rest, rest_stride,
        scale_modifier, viewmatrices + 16 * c, projmatrices + 16 * c, campos + 3 * c, tanfov[2 * c],
        tanfov[2 * c + 1], image_height, image_width, means2D + 2 * o, depths + o, radii + o, conic_opacity + 4 * o,
        rgb + 3 * o, nullptr, vis_list + o, counts + (int64_t)c * cs, nullptr, nullptr, nullptr, nullptr,
        n_ranks > 0 ? &x : nullptr, static_cast<char*>(scratch) + (size_t)c * slice, slice, bs->s[c % ns], 1,
        status);
  }
  // join: the caller's stream waits for every side stream (also after an error)
  for (int i = 0; i < ns; ++i) {
    cudaEventRecord(bs->join[i], bs->s[i]);
    cudaStreamWaitEvent(S(stream), bs->join[i], 0);
  }
  return rc_all;
}

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
                                        void* stream) {
  if (n_cams < 0 || counts_stride < 1 || cam_stride < P)
    return fail(BLITZ_EINVAL, "blitz_preprocess_backward_raw_batch: bad sizes");
  if (n_cams == 0 || P == 0) return 0;
  if (!viewmatrices || !projmatrices || !campos || !tanfov || !vis_list || !counts || !upstream || !upstream_row0)
    return fail(BLITZ_EINVAL, "blitz_preprocess_backward_raw_batch: null pointer");
  if (!aligned16(upstream)) return fail(BLITZ_EINVAL, "blitz_preprocess_backward_raw_batch: upstream alignment");
  for (int c = 0; c < n_cams; ++c) {
    if (upstream_row0[c] < 0) return fail(BLITZ_EINVAL, "blitz_preprocess_backward_raw_batch: bad upstream row");
    const int64_t o = c * cam_stride;
    const float* u = upstream + 12 * upstream_row0[c];
    const int rc = blitz_preprocess_backward_raw(
        P, D, M, radii + o, means2D + 2 * o, xyz, scaling_raw, rotation_raw, nullptr, opacity_raw, sh_dc, dc_stride,
        sh_rest, rest_stride, scale_modifier, viewmatrices + 16 * c, projmatrices + 16 * c, campos + 3 * c,
        tanfov[2 * c], tanfov[2 * c + 1], image_height, image_width, u + 4, 12, u + 0, 12, u + 6, 12, nullptr,
        u + 11, 12, vis_list + o, counts + (int64_t)c * counts_stride, g_xyz, g_scaling_raw, g_rotation_raw,
        g_opacity_raw, g_dc, g_dc_stride, g_rest, g_rest_stride, 1, BLITZ_ROWS_UPSTREAM_BY_SLOT, stream);
    if (rc) return rc;
  }
  return 0;
}

}  // extern "C"

namespace {

int fill_segments(int n_segments, const int64_t* seg_start, const int64_t* seg_count, Segments& sg, int64_t& n) {
  if (n_segments < 0 || n_segments > kMaxSegments || (n_segments > 0 && (!seg_start || !seg_count))) return 1;
  sg.n = n_segments;
  n = 0;
  for (int s = 0; s < n_segments; ++s) {
    if (seg_start[s] < 0 || seg_count[s] < 0) return 1;
    sg.start[s] = seg_start[s];
    sg.count[s] = seg_count[s];
    n += seg_count[s];
  }
  return 0;
}

}  // namespace

extern "C" {

int blitz_exchange_unpack(int n_segments, const int64_t* seg_start, const int64_t* seg_count, const float* records,
                          float* conic, float* means2D, float* rgb, float* depths, int32_t* radii, double* reg,
                          void* stream) {
  UnpackParams p{};
  int64_t n = 0;
  if (fill_segments(n_segments, seg_start, seg_count, p.seg, n))
    return fail(BLITZ_EINVAL, "blitz_exchange_unpack: bad segments");
  if (n == 0) return 0;
  if (!records || !conic || !means2D || !rgb || !depths || !radii)
    return fail(BLITZ_EINVAL, "blitz_exchange_unpack: null pointer");
  if (!aligned16(records) || !aligned16(conic) || (reinterpret_cast<uintptr_t>(means2D) & 7u))
    return fail(BLITZ_EINVAL, "blitz_exchange_unpack: records/conic need 16-byte, means2D 8-byte alignment");
  p.records = records;
  p.conic = conic;
  p.means2D = means2D;
  p.rgb = rgb;
  p.depths = depths;
  p.radii = radii;
  p.reg = reg;
  return check(launch_exchange_unpack(p, n, S(stream)), "blitz_exchange_unpack");
}

int blitz_grad_records_pack(int n_segments, const int64_t* seg_start, const int64_t* seg_count, const float* rec16,
                            const int32_t* radii, const float* reg_scale, float* send, void* stream) {
  GradPackParams p{};
  int64_t n = 0;
  if (fill_segments(n_segments, seg_start, seg_count, p.seg, n))
    return fail(BLITZ_EINVAL, "blitz_grad_records_pack: bad segments");
  if (n == 0) return 0;
  if (!rec16 || !radii || !send) return fail(BLITZ_EINVAL, "blitz_grad_records_pack: null pointer");
  if (!aligned16(rec16) || !aligned16(send))
    return fail(BLITZ_EINVAL, "blitz_grad_records_pack: rec16 and send need 16-byte alignment");
  p.rec16 = rec16;
  p.radii = radii;
  p.reg_scale = reg_scale;
  p.send = send;
  return check(launch_grad_records_pack(p, n, S(stream)), "blitz_grad_records_pack");
}

int blitz_loss_combine(const double* sums, const double* reg, float one_minus_lambda, float lambda, float n3,
                       float reg_weight, float* out, void* stream) {
  if (!sums || !out || !(n3 > 0.f)) return fail(BLITZ_EINVAL, "blitz_loss_combine: bad arguments");
  LossCombineParams p{sums, reg, one_minus_lambda, lambda, n3, reg_weight, out};
  return check(launch_loss_combine(p, S(stream)), "blitz_loss_combine");
}

int blitz_loss_combine_backward(const float* g_loss, const float* g_l1, const float* g_ss, const float* fwd_out,
                                float one_minus_lambda, float lambda, float n3, float reg_weight, float* scales,
                                void* stream) {
  if (!fwd_out || !scales || !(n3 > 0.f)) return fail(BLITZ_EINVAL, "blitz_loss_combine_backward: bad arguments");
  LossCombineParams p{nullptr, nullptr, one_minus_lambda, lambda, n3, reg_weight, const_cast<float*>(fwd_out)};
  return check(launch_loss_combine_bwd(p, g_loss, g_l1, g_ss, scales, S(stream)), "blitz_loss_combine_backward");
}

int blitz_read_totals(const int64_t* totals, const int32_t* vis_count, const uint32_t* status, int64_t* host_totals,
                      int32_t* host_vis, uint32_t* host_status, void* stream) {
  if (!totals || !host_totals || ((vis_count == nullptr) != (host_vis == nullptr)) ||
      ((status == nullptr) != (host_status == nullptr)))
    return fail(BLITZ_EINVAL, "blitz_read_totals: bad arguments");
  cudaError_t e = cudaMemcpyAsync(host_totals, totals, 2 * sizeof(int64_t), cudaMemcpyDeviceToHost, S(stream));
  if (e == cudaSuccess && vis_count)
    e = cudaMemcpyAsync(host_vis, vis_count, sizeof(int32_t), cudaMemcpyDeviceToHost, S(stream));
  if (e == cudaSuccess && status)
    e = cudaMemcpyAsync(host_status, status, sizeof(uint32_t), cudaMemcpyDeviceToHost, S(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(S(stream));
  if (e == cudaSuccess && status && *host_status) {
    const unsigned bits = *host_status;
    e = cudaMemsetAsync(const_cast<uint32_t*>(status), 0, sizeof(uint32_t), S(stream));
    if (e == cudaSuccess) {
      char msg[160];
      snprintf(msg, sizeof(msg), "blitz_read_totals: an ordered scan gave up waiting (status 0x%x)", bits);
      return fail(BLITZ_ESCAN, msg);
    }
  }
  return check((int)e, "blitz_read_totals");
}

}  // extern "C"

namespace {

// Side stream and events of the asynchronous zero fill, per device.
struct FillState {
  bool ready = false;
  cudaStream_t side = nullptr;
  cudaEvent_t queued = nullptr, done = nullptr;
};
constexpr int kMaxDevices = 64;
FillState g_fill[kMaxDevices];
std::mutex g_fill_mu;

int fill_state(FillState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return BLITZ_EINVAL;
  FillState& f = g_fill[dev];
  if (!f.ready) {
    std::lock_guard<std::mutex> lock(g_fill_mu);
    if (!f.ready) {
      e = cudaStreamCreateWithFlags(&f.side, cudaStreamNonBlocking);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&f.queued, cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&f.done, cudaEventDisableTiming);
      if (e != cudaSuccess) return (int)e;
      f.ready = true;
    }
  }
  *out = &f;
  return 0;
}

}  // namespace

extern "C" {

int blitz_zero_fill_async(int n, void* const* ptrs, const size_t* bytes, void* stream) {
  if (n < 0 || (n > 0 && (!ptrs || !bytes))) return fail(BLITZ_EINVAL, "blitz_zero_fill_async: bad arguments");
  FillState* f = nullptr;
  int rc = fill_state(&f);
  if (rc) return fail(rc, "blitz_zero_fill_async: side stream");
  // the side stream starts after everything already queued on `stream`
  cudaError_t e = cudaEventRecord(f->queued, S(stream));
  if (e == cudaSuccess) e = cudaStreamWaitEvent(f->side, f->queued, 0);
  for (int i = 0; e == cudaSuccess && i < n; ++i)
    if (bytes[i]) e = cudaMemsetAsync(ptrs[i], 0, bytes[i], f->side);
  if (e == cudaSuccess) e = cudaEventRecord(f->done, f->side);
  return check((int)e, "blitz_zero_fill_async");
}

int blitz_zero_fill_wait(void* stream) {
  FillState* f = nullptr;
  int rc = fill_state(&f);
  if (rc) return fail(rc, "blitz_zero_fill_wait: side stream");
  return check((int)cudaStreamWaitEvent(S(stream), f->done, 0), "blitz_zero_fill_wait");
}

int blitz_zero_rows(int n_arrays, void* const* arrays, const size_t* row_bytes, const uint32_t* rows, int64_t n_rows,
                    void* stream) {
  if (n_arrays < 0 || n_arrays > kZeroRowsMax || n_rows < 0 || (n_arrays > 0 && (!arrays || !row_bytes)) ||
      (n_rows > 0 && !rows))
    return fail(BLITZ_EINVAL, "blitz_zero_rows: bad arguments");
  ZeroRowsParams p{};
  p.n_arrays = n_arrays;
  p.rows = rows;
  p.n_rows = n_rows;
  for (int a = 0; a < n_arrays; ++a) {
    if (!arrays[a] || row_bytes[a] == 0 || (row_bytes[a] & 3u) || (reinterpret_cast<uintptr_t>(arrays[a]) & 3u))
      return fail(BLITZ_EINVAL, "blitz_zero_rows: arrays need 4-byte aligned rows of whole 32-bit words");
    p.arrays[a] = arrays[a];
    p.row_words[a] = (int64_t)(row_bytes[a] / 4);
  }
  return check(launch_zero_rows(p, S(stream)), "blitz_zero_rows");
}

int blitz_fp32_probe(int blocks, int64_t iters, float* sink, void* stream) {
  if (blocks <= 0 || iters <= 0 || !sink) return fail(BLITZ_EINVAL, "blitz_fp32_probe: bad arguments");
  return check(launch_fma_probe(blocks, iters, sink, S(stream)), "blitz_fp32_probe");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Full (non-distributed) rasterizer: rasterize_gaussians, _simp, _depth and
// mark_visible.

extern "C" {

int blitz_rasterize_count(int64_t P, int image_height, int image_width, const float* means2D, const int32_t* radii,
                          const float* rects, const float* conic_opacity, uint32_t* counts, uint64_t* totals,
                          void* stream) {
  if (P < 0 || P >= (int64_t)0xffffffff || image_height <= 0 || image_width <= 0)
    return fail(BLITZ_EINVAL, "blitz_rasterize_count: bad sizes");
  if (!totals || (P > 0 && (!means2D || !radii || !rects || !conic_opacity || !counts)))
    return fail(BLITZ_EINVAL, "blitz_rasterize_count: null pointer");
  if (P > 0 && ((reinterpret_cast<uintptr_t>(means2D) & 7u) || (reinterpret_cast<uintptr_t>(rects) & 7u) ||
                !aligned16(conic_opacity)))
    return fail(BLITZ_EINVAL, "blitz_rasterize_count: means2D/rects need 8-byte, conic_opacity 16-byte alignment");
  BinParams b{};
  b.P = P;
  b.W = image_width;
  b.H = image_height;
  b.grid_x = (image_width + kTileX - 1) / kTileX;
  b.grid_y = (image_height + kTileY - 1) / kTileY;
  b.means2D = means2D;
  b.radii = radii;
  b.counts = counts;
  b.totals = reinterpret_cast<unsigned long long*>(totals);
  b.rects = rects;
  b.conic_opacity = conic_opacity;
  return check(launch_bin_count(b, S(stream)), "blitz_rasterize_count");
}

int blitz_rasterize_bin(int64_t P, int64_t n_vis, int64_t R, int image_height, int image_width, const float* means2D,
                        const float* depths, const int32_t* radii, const float* rects, const float* conic_opacity,
                        const uint32_t* counts, void* scratch, size_t scratch_bytes, uint32_t* point_list,
                        uint32_t* ranges, void* stream) {
  if (!render_args_ok(P, n_vis, R, image_height, image_width))
    return fail(BLITZ_EINVAL, "blitz_rasterize_bin: bad sizes");
  if (!ranges || (P > 0 && (!means2D || !depths || !radii || !rects || !conic_opacity || !counts)) ||
      (R > 0 && (!point_list || !scratch)))
    return fail(BLITZ_EINVAL, "blitz_rasterize_bin: null pointer");
  if (P > 0 && ((reinterpret_cast<uintptr_t>(means2D) & 7u) || (reinterpret_cast<uintptr_t>(rects) & 7u) ||
                !aligned16(conic_opacity)))
    return fail(BLITZ_EINVAL, "blitz_rasterize_bin: means2D/rects need 8-byte, conic_opacity 16-byte alignment");
  return render_bin_impl(P, n_vis, R, image_height, image_width, means2D, depths, radii, nullptr, counts, scratch,
                         scratch_bytes, point_list, ranges, S(stream), rects, conic_opacity);
}

int blitz_rasterize_blend(int64_t P, int image_height, int image_width, const float* means2D,
                          const float* conic_opacity, const float* rgb, const float* bg, const uint32_t* point_list,
                          const uint32_t* ranges, float* final_T, uint32_t* n_contrib, float* out_color,
                          float* max_count, float* accum_w, int32_t* accum_n, void* stream) {
  if (!render_args_ok(P, 0, 0, image_height, image_width))
    return fail(BLITZ_EINVAL, "blitz_rasterize_blend: bad sizes");
  if ((accum_w == nullptr) != (accum_n == nullptr))
    return fail(BLITZ_EINVAL, "blitz_rasterize_blend: accum_w and accum_n go together");
  if (!bg || !ranges || !final_T || !n_contrib || !out_color ||
      (P > 0 && (!means2D || !conic_opacity || !rgb || !point_list)))
    return fail(BLITZ_EINVAL, "blitz_rasterize_blend: null pointer");
  BlendFwdParams f{};
  f.W = image_width;
  f.H = image_height;
  f.grid_x = (image_width + kTileX - 1) / kTileX;
  f.grid_y = (image_height + kTileY - 1) / kTileY;
  f.P = P;
  f.ranges = reinterpret_cast<const uint2*>(ranges);
  f.point_list = point_list;
  f.means2D = means2D;
  f.conic_opacity = conic_opacity;
  f.rgb = rgb;
  f.bg = bg;
  f.out_color = out_color;
  f.final_T = final_T;
  f.n_contrib = n_contrib;
  f.max_count = max_count;
  f.accum_w = accum_w;
  f.accum_n = accum_n;
  if (!max_count && !accum_w) {
    // plain colour forward: the training blend needs its per-tile outputs
    return fail(BLITZ_EINVAL, "blitz_rasterize_blend: no statistics requested (use blitz_render_blend)");
  }
  return check(launch_blend_fwd(f, S(stream)), "blitz_rasterize_blend");
}

int blitz_rasterize_depth(int64_t P, int image_height, int image_width, const float* means2D,
                          const float* conic_opacity, const float* rgb, const float* bg, const uint32_t* point_list,
                          const uint32_t* ranges, const float* means3D, const float* scales, const float* rotations,
                          const float* projmatrix, const float* campos, float* out_color, float* out_pts,
                          float* out_depth, float* accum_alpha, int32_t* gidx, float* discriminants, void* stream) {
  if (!render_args_ok(P, 0, 0, image_height, image_width))
    return fail(BLITZ_EINVAL, "blitz_rasterize_depth: bad sizes");
  if (!bg || !ranges || !projmatrix || !campos || !out_color || !out_pts || !out_depth || !accum_alpha || !gidx ||
      !discriminants || (P > 0 && (!means2D || !conic_opacity || !rgb || !point_list || !means3D || !scales ||
                                   !rotations)))
    return fail(BLITZ_EINVAL, "blitz_rasterize_depth: null pointer");
  if (P > 0 && (!aligned16(rotations) || !aligned16(conic_opacity)))
    return fail(BLITZ_EINVAL, "blitz_rasterize_depth: rotations and conic_opacity need 16-byte aligned rows");
  DepthParams d{};
  d.W = image_width;
  d.H = image_height;
  d.grid_x = (image_width + kTileX - 1) / kTileX;
  d.grid_y = (image_height + kTileY - 1) / kTileY;
  d.ranges = reinterpret_cast<const uint2*>(ranges);
  d.point_list = point_list;
  d.means2D = means2D;
  d.conic_opacity = conic_opacity;
  d.rgb = rgb;
  d.bg = bg;
  d.means3D = means3D;
  d.scales = scales;
  d.rotations = rotations;
  d.projmatrix = projmatrix;
  d.campos = campos;
  d.out_color = out_color;
  d.out_pts = out_pts;
  d.out_depth = out_depth;
  d.accum_alpha = accum_alpha;
  d.gidx = gidx;
  d.discriminants = discriminants;
  return check(launch_depth_render(d, S(stream)), "blitz_rasterize_depth");
}

int blitz_mark_visible(int64_t P, const float* means3D, const float* viewmatrix, const float* projmatrix,
                       uint8_t* present, void* stream) {
  (void)projmatrix;  // the frustum test reads only the view depth
  if (P < 0) return fail(BLITZ_EINVAL, "blitz_mark_visible: bad sizes");
  if (P > 0 && (!means3D || !viewmatrix || !present)) return fail(BLITZ_EINVAL, "blitz_mark_visible: null pointer");
  return check(launch_mark_visible(P, means3D, viewmatrix, reinterpret_cast<bool*>(present), S(stream)),
               "blitz_mark_visible");
}

}  // extern "C"
