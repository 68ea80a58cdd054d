// Internal launch interface between the C-ABI layer (capi.cu) and the kernels.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace blitz {

enum : unsigned {
  kErrPrefilteredCulled = 1u << 0,  // a Gaussian failed the near test with prefiltered=true
  kErrBinOverflow = 1u << 1,        // more tile instances than the caller sized for
};

struct PreprocessParams {
  int64_t P;
  int D;  // active SH degree
  int M;  // SH coefficients beyond DC held per Gaussian (<= 15)
  const float* means3D;    // [P,3]
  const float* scales;     // [P,3] activated
  const float* rotations;  // [P,4] (r,x,y,z), 16-byte aligned rows
  const float* opacities;  // [P] activated
  const float* dc;         // DC triplet of Gaussian i at dc + i*dc_stride
  int64_t dc_stride;
  const float* rest;       // M triplets of Gaussian i at rest + i*rest_stride
  int64_t rest_stride;
  bool sh_packed16;        // dc/rest are one contiguous 16B-aligned [P,16,3] tensor
  float scale_modifier;
  const float* viewmatrix;  // device [16]
  const float* projmatrix;  // device [16]
  const float* campos;      // device [3]
  float tanfovx, tanfovy, focal_x, focal_y;
  int W, H, grid_x, grid_y;
  bool prefiltered;
  float* out_means2D;        // [P,2]
  float* out_depths;         // [P]
  int* out_radii;            // [P]
  float* out_conic_opacity;  // [P,4]
  float* out_rgb;            // [P,3]
  bool* out_clamped;         // [P,3] or null
  float* out_cov3D;          // [P,6] or null
  // Full-rasterizer extras (both optional): Gaussians with culling[i] set are
  // skipped (radius 0, zero rows), and out_rects receives the float
  // half-extents of each Gaussian's screen rectangle (zeros when culled).
  const bool* culling;       // [P] or null
  float* out_rects;          // [P,2] or null
  unsigned* error_flag;      // device word, OR-ed with kErr* bits
  // Raw-parameter mode: scales/rotations/opacities hold the model's raw
  // _scaling / _rotation / _opacity; the kernel applies exp, normalize and
  // sigmoid itself with the same float arithmetic as PyTorch.
  bool raw;
  const float* rot_norm;     // raw mode: ||_rotation|| per Gaussian, or null = computed here
  double* reg_sums;          // raw mode, optional: {sum min-axis scale, count} over regulariser-visible
  uint32_t* vis_list_out;    // optional [P]: indices of Gaussians with radius > 0
  bool ordered_list;         // two-kernel form: vis_list_out in ascending index order (ordered scans)
  int* vis_count_out;        // device counter for vis_list_out, zero on entry
  // Optional first pass of the binning, fused: per-Gaussian tile counts under
  // the compute_locally mask and the totals {tile instances, Gaussians with a
  // tile} (zeroed by the launcher).
  uint32_t* counts_out;                // [P] or null
  unsigned long long* totals_out;      // [2] or null
  const bool* compute_locally;         // [grid_y*grid_x] or null (all tiles)
  // Gaussians rejected before the full computation get only radii (and
  // counts) written; the caller reads other rows through vis_list_out.
  bool listed_rows_only;
  uint32_t* slot_of_out;  // optional [P]: list position of each listed Gaussian (others untouched)
  // Optional exchange outputs of the multi-GPU step (need vis_list_out): row
  // j = the j-th listed Gaussian's 12-float record and its destination mask
  // (bit r: its square tile rect overlaps rank r's tile interval
  // [x_tile_lo[r], x_tile_hi[r])), x_counts[r] += rows for rank r.
  int x_ranks;              // <= 32; 0 = no exchange outputs
  const int* x_tile_lo;     // device [x_ranks]
  const int* x_tile_hi;     // device [x_ranks]
  float* x_records;         // [P,12]
  uint32_t* x_mask;         // [P]
  int* x_counts;            // [x_ranks], zero on entry
};

struct PreprocessBwdParams {
  PreprocessParams f;      // the forward's inputs (outputs unused)
  const int* radii;        // [P] from the forward
  const float* g_means2D;  // d/d(means2D) of Gaussian i at g_means2D + i*stride (x, y)
  int64_t g_means2D_stride;
  const float* g_conic_opacity;  // float4 at g_conic_opacity + i*stride (conic00, conic01, conic11, opacity)
  int64_t g_conic_stride;
  const float* g_colors;  // rgb grad at g_colors + i*stride
  int64_t g_colors_stride;
  float* g_means3D;    // [P,3]
  float* g_scales;     // [P,3]
  float* g_rotations;  // [P,4]
  float* g_opacities;  // [P] or null
  float* g_dc;         // at g_dc + i*g_dc_stride (3 floats)
  int64_t g_dc_stride;
  float* g_rest;       // at g_rest + i*g_rest_stride (M*3 floats)
  int64_t g_rest_stride;
  // Raw-parameter mode extras (see PreprocessParams::raw): gradients are with
  // respect to the raw parameters.
  const float* means2D;        // forward screen means (regulariser visibility), raw mode
  const float* reg_scale;      // device float: dLoss/d(sum min-axis scale), or null
  const uint32_t* vis_list;    // optional: only these Gaussians are processed; outputs pre-zeroed
  const int* vis_count;        // device count of vis_list
  // With vis_list: upstream gradients are read at row j (the list position)
  // instead of row i, and/or the outputs are written at row j (compact rows).
  bool upstream_by_slot;
  bool out_by_slot;
  // optional: d(loss)/d(smallest activated scale) at g_minscale + row*stride
  // (row = the upstream row), added to the first smallest axis (raw mode)
  const float* g_minscale;
  int64_t g_minscale_stride;
};

// scratch (may be null): preprocess_scratch_bytes(P) bytes select the
// two-kernel form (cull pass + full pass over the candidates), whose visible
// list is in ascending index order when p.ordered_list is set.  The uint32 at byte kPreStatusOffset of
// the scratch collects scan.cuh status bits; the launcher never clears it
// (the caller zeroes a new buffer and reads / clears the word).
constexpr size_t kPreStatusOffset = 0;
size_t preprocess_scratch_bytes(int64_t P);
// grid_share: number of such launches running side by side (each takes that
// share of the device's resident blocks); status: overrides the scratch's
// own status word.
int launch_preprocess_fwd(const PreprocessParams& p, cudaStream_t st, void* scratch = nullptr,
                          size_t scratch_bytes = 0, int grid_share = 1, unsigned* status = nullptr);
int launch_preprocess_bwd(const PreprocessBwdParams& p, bool accumulate, cudaStream_t st);

// ---------------------------------------------------------------------------
// Binning + blending
// ---------------------------------------------------------------------------
struct BinParams {
  int64_t P;
  int W, H, grid_x, grid_y;
  const float* means2D;          // [P,2]
  const float* depths;           // [P]
  const int* radii;              // [P]
  const bool* compute_locally;   // [grid_y*grid_x] or null (= all tiles)
  uint32_t* counts;              // [P] tiles touched under the mask
  unsigned long long* totals;    // device [2]: {instances R, visible Gaussians}
  // Full rasterizer (rasterize_gaussians): with rects, a Gaussian's tiles are
  // those of its float half-extent rectangle that pass the exact tile test on
  // conic_opacity, instead of the square radius rectangle (no mask then).
  const float* rects;            // [P,2] or null
  const float* conic_opacity;    // [P,4], with rects
};

int launch_bin_count(const BinParams& p, cudaStream_t st);

// Scratch needed by bin_sort for the given sizes (bytes).
size_t bin_scratch_bytes(int64_t P, int64_t n_vis, int64_t R, int n_tiles);

struct BinSortParams {
  BinParams b;
  int64_t n_vis;   // visible Gaussians (counts > 0), read back by the host
  int64_t R;       // tile instances, read back by the host
  void* scratch;
  size_t scratch_bytes;
  uint32_t* point_list;  // [R] output: Gaussian index per instance, tile-major, depth order
  uint2* ranges;         // [n_tiles] output: [start, end) per tile
};

int launch_bin_sort(const BinSortParams& p, cudaStream_t st);

struct BlendFwdParams {
  int W, H, grid_x, grid_y;
  int64_t P;
  const uint2* ranges;
  const uint32_t* point_list;
  const float* means2D;
  const float* conic_opacity;
  const float* rgb;
  const float* bg;             // device [3]
  const bool* compute_locally; // or null
  float* out_color;            // [3,H,W]
  float* final_T;              // [H*W]
  uint32_t* n_contrib;         // [H*W] last contributor (1-based position in the tile list)
  int* out_observe;            // [P], zero on entry
  int* n_render;               // [tiles]
  int* n_consider;             // [tiles]
  int* n_contrib_tile;         // [tiles]
  // optional (all or none): per warp strip (8 per tile) the Gaussians that
  // contributed to any of its pixels, in list order -- Gaussian id and
  // 0-based list position at [8 * range.x + strip * n_tile + e] -- and their
  // count at [tile * 8 + strip]; read by the backward
  int* strip_ids;
  int* strip_pos;
  int* strip_counts;
  // Full-rasterizer statistics (rasterize_gaussians with flag_max_count, and
  // rasterize_gaussians_simp), each optional: per pixel, the Gaussian of
  // largest blending weight alpha*T (the first in list order on ties) gets
  // +1 in max_count; every (pixel, Gaussian) blend adds alpha*T to
  // accum_w[id] and 1 to accum_n[id].  With any of them set, n_render /
  // n_consider / n_contrib_tile / out_observe may be null.
  float* max_count;  // [P] or null
  float* accum_w;    // [P] or null
  int* accum_n;      // [P] or null (with accum_w)
};

int launch_blend_fwd(const BlendFwdParams& p, cudaStream_t st);

struct BlendBwdParams {
  int W, H, grid_x, grid_y;
  int64_t P;
  const uint2* ranges;
  const uint32_t* point_list;
  const float* means2D;
  const float* conic_opacity;
  const float* rgb;
  const float* bg;
  const bool* compute_locally;
  const float* final_T;
  const uint32_t* n_contrib;
  const float* dL_dpix;   // [3,H,W]
  float* grad_accum;      // [rows,16], zero on entry; layout in capi docs
  const uint32_t* record_rows;  // optional: record row of Gaussian id (else the id itself)
  const int* strip_ids;         // optional: the forward's strip lists (see BlendFwdParams)
  const int* strip_pos;
  const int* strip_counts;
};

int launch_blend_bwd(const BlendBwdParams& p, cudaStream_t st);

// ---------------------------------------------------------------------------
// Loss
// ---------------------------------------------------------------------------
struct LossParams {
  int C, Hb, W;
  const float* img;        // [C,Hb,W]
  const uint8_t* gt_u8;    // [C,Hb,W] or null
  const float* gt_f32;     // [C,Hb,W] or null
  float* partials;         // [C,Hb,W,3] dSSIM/d(mu1, E[x^2], E[xy]) per pixel (fwd output)
};
// sums: device double[2] {sum |img-gt|, sum SSIM}, zero on entry.
int launch_loss_fwd(const LossParams& p, const float* window11, double* sums, cudaStream_t st);

struct LossBwdParams {
  LossParams f;
  const float* scale;   // device [2]: dLoss/d(sum L1), dLoss/d(sum SSIM)
  float* dL_dimg;       // [C,Hb,W]
};
int launch_loss_bwd(const LossBwdParams& p, const float* window11, cudaStream_t st);

struct LossCombineParams {
  const double* sums;  // {sum L1, sum SSIM}
  const double* reg;   // {sum of min-axis scales, count} or null
  float one_minus_lambda, lambda, n3, reg_weight;
  float* out;          // {loss, L1, SSIM, reg, cnt}; read back by the backward
};
int launch_loss_combine(const LossCombineParams& p, cudaStream_t st);
int launch_loss_combine_bwd(const LossCombineParams& p, const float* g_loss, const float* g_l1, const float* g_ss,
                            float* scales, cudaStream_t st);

// ---------------------------------------------------------------------------
// Routing (which ranks' tile rows a Gaussian overlaps)
// ---------------------------------------------------------------------------
struct RouteParams {
  int64_t P;
  int W, H, grid_x, grid_y;
  int world_size;
  const float* means2D;
  const int* radii;
  const int* dist_global_strategy;  // [world_size+1] tile ids (row starts * grid_x)
  bool avoid_pixel_all2all;
  bool* out_bool;                   // [P, world_size]
};
int launch_route_bool(const RouteParams& p, cudaStream_t st);

// Routing against per-rank tile rectangles [y_l, y_r, x_l, x_r] (the
// reference's getTouchedIdsBoolAdjustMode6).
int launch_route_bool_rect(const RouteParams& p, const int* rectangles, cudaStream_t st);

// Sparse Adam (see adam.cu).  rows == null: dense grad [N,M] and visible [N];
// else grad is [n_rows, M] for Gaussians rows[j].
struct AdamParams {
  float* param;
  const float* grad;
  float* exp_avg;
  float* exp_avg_sq;
  const bool* visible;
  const int64_t* rows;
  int64_t n_rows;
  float lr, b1, b2, eps;
  int64_t N, M;
  float grad_scale;  // rows form: the gradient is multiplied by this first (1 = as given)
};
int launch_adam(const AdamParams& p, cudaStream_t st);

// Pack rows [0, n_rows) of a camera's exchange records into the send buffer:
// row j goes to every rank r whose bit is set in mask[j], at
// dest_offset[r] + (its running position among rank r's rows); send_row
// receives row_base + j there.  cursor: device [n_ranks], zero on entry.
struct PackParams {
  int64_t n_rows;
  int n_ranks;
  int64_t dest_offset[32];
  const float* records;  // [n_rows,12]
  const uint32_t* mask;  // [n_rows]
  float* send;           // [*,12]
  int* send_row;         // [*]
  int row_base;
  // set by the launcher from its scratch
  int* ticket;
  unsigned long long* scan_state;
  unsigned* status;
};
// Scratch of one pack launch: a status word (bytes [0,4), never cleared by
// the launcher), a ticket and the ordered-scan state (cleared per launch).
size_t exchange_pack_scratch_bytes(int64_t n_rows, int n_ranks);
int launch_exchange_pack(PackParams p, void* scratch, cudaStream_t st);

// Received exchange records of one camera: up to kMaxSegments runs of rows
// [seg_start[s], seg_start[s] + seg_count[s]) of a [*,12] buffer, taken in
// order as rows 0..n-1 of the camera.
constexpr int kMaxSegments = 32;
struct Segments {
  int n;
  int64_t start[kMaxSegments];
  int64_t count[kMaxSegments];
};

struct UnpackParams {
  Segments seg;
  const float* records;  // [*,12]
  float* conic;          // [n,4]
  float* means2D;        // [n,2]
  float* rgb;            // [n,3]
  float* depths;         // [n]
  int* radii;            // [n]
  double* reg;           // [2] += {sum of min-axis scales of rows with radius > 0, their count}, or null
};
int launch_exchange_unpack(const UnpackParams& p, int64_t n, cudaStream_t st);

struct GradPackParams {
  Segments seg;          // destination runs in send, in the order of the camera's rows
  const float* rec16;    // [n,16] render-backward record
  const int* radii;      // [n]
  const float* reg_scale;  // device float: dLoss/d(sum of min-axis scales), or null
  float* send;           // [*,12]
};
int launch_grad_records_pack(const GradPackParams& p, int64_t n, cudaStream_t st);

// Full rasterizer, eval outputs (rasterize_gaussians_depth, forward.cu:614-845):
// the colour blend of the tile lists, plus per pixel the Gaussian of largest
// blending weight among those whose ray-ellipsoid depth is >= 0, with that
// depth, the discriminant of the intersection and the 3D point.
struct DepthParams {
  int W, H, grid_x, grid_y;
  const uint2* ranges;
  const uint32_t* point_list;
  const float* means2D;        // [P,2]
  const float* conic_opacity;  // [P,4]
  const float* rgb;            // [P,3]
  const float* bg;             // device [3]
  const float* means3D;        // [P,3]
  const float* scales;         // [P,3] activated
  const float* rotations;      // [P,4] (r,x,y,z), as given
  const float* projmatrix;     // device [16]
  const float* campos;         // device [3]
  float* out_color;            // [3,H,W]
  float* out_pts;              // [3,H,W]
  float* out_depth;            // [H,W]
  float* accum_alpha;          // [H,W] final transmittance
  int* gidx;                   // [H,W]
  float* discriminants;        // [H,W]
};

int launch_depth_render(const DepthParams& p, cudaStream_t st);

// Frustum mark of markVisible (rasterizer_impl.cu:100-114): view depth > 0.2.
int launch_mark_visible(int64_t P, const float* means3D, const float* viewmatrix, bool* present, cudaStream_t st);

// Zero rows[0..n_rows) of up to kZeroRowsMax dense row-major arrays (row i
// of array a: row_words[a] 32-bit words at arrays[a] + i * row_words[a]).
constexpr int kZeroRowsMax = 8;
struct ZeroRowsParams {
  int n_arrays;
  void* arrays[kZeroRowsMax];
  int64_t row_words[kZeroRowsMax];
  const uint32_t* rows;  // device [n_rows]
  int64_t n_rows;
};

int launch_zero_rows(const ZeroRowsParams& p, cudaStream_t st);

int launch_fma_probe(int blocks, int64_t iters, float* sink, cudaStream_t st);

// Records the message blitz_last_error() returns on this thread (capi.cu).
void set_last_error(const char* msg);

}  // namespace blitz
