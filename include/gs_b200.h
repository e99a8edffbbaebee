/*
 * gs_b200.h -- C ABI of the B200 (sm_100a) Gaussian-splat rasterizer.
 *
 * Drop-in kernels for the reference's `gaussian_splats::rasterize` operator
 * (VikaasVarma/gaussian-splats, src/gaussian_splats/kernels/rasterize/
 * interface.py:17-244). Each entry point below replaces one stage that the
 * reference's Python operator launches; the host wrapper (the package's
 * rasterize.py, or any FFI caller) chains them exactly as interface.py does.
 *
 * Conventions shared by every entry point:
 *  - All array arguments are DEVICE pointers to contiguous row-major data on
 *    the current device, except where a name ends in `_host`.
 *  - Nothing here allocates memory. Scratch comes from the caller as
 *    `workspace` buffers (256-byte aligned) of the sizes the matching
 *    `*_workspace_size` queries return. rotation, inverse_covariance,
 *    grad_rotation and bounds rows are read/written as 16-byte vectors and
 *    must be 16-byte aligned; so must color and grad_color when K is 4 or 16.
 *  - Work is enqueued on `stream`; only gs_bin_count() synchronises it.
 *  - Return value: GS_OK (0) or a negative GS_ERR_* code. CUDA launch errors
 *    are reported as GS_ERR_CUDA; gs_last_cuda_error() returns the code.
 *  - Gaussian tensors follow splats/splats.py: mean [N,3], rotation [N,4]
 *    (w,x,y,z, any norm), scale [N,3] (log sigma), opacity [N,1] (logit),
 *    color [N,K,3] (real SH, K = (degree+1)^2 <= 25).
 */
#ifndef GS_B200_H
#define GS_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *gs_stream_t; /* a cudaStream_t; NULL = legacy default stream */

enum {
  GS_OK = 0,
  GS_ERR_INVALID_ARGUMENT = -1, /* sizes, tile size or mode out of range */
  GS_ERR_CUDA = -2,             /* a CUDA runtime call or launch failed */
  GS_ERR_CAPACITY = -3,         /* more intersections than the buffers hold */
  GS_ERR_UNSUPPORTED = -4,      /* SH degree above 4 */
  GS_ERR_MISALIGNED = -5,       /* a buffer misses its required alignment */
  GS_ERR_TIMEOUT = -6           /* a bounded device-side wait gave up (results invalid) */
};

/* Scalars of one render, folded on the host the way the reference folds its
 * Triton constexprs (in double, then rounded to float):
 *   lim_x = 1.3 * tiles_w * tile_size / (2 fx)      project.py:158
 *   lim_y = 1.3 * tiles_h * tile_size / (2 fy)      project.py:159
 *   bwd_lim_x = 1.3 * width / (2 fx)                 project_bwd.py:376
 *   bwd_lim_y = 1.3 * height / (2 fy)                project_bwd.py:377
 *   extent = sqrt(-2 log1p(-confidence)) if ellipsoid else 3    project.py:308
 *   cutoff = -2 log1p(-confidence)                   composite.py:226  */
typedef struct gs_params {
  float fx, fy, cx, cy;
  int32_t width, height, tile_size; /* width, height: multiples of tile_size */
  int32_t gaussian_mode;            /* 1: Gaussian falloff; 0: ellipsoid indicator */
  float near_plane, far_plane;
  float lim_x, lim_y, bwd_lim_x, bwd_lim_y;
  float extent, cutoff, opacity_threshold;
} gs_params;

/* Library version, for load-time checks. */
int32_t gs_version(void);

/* cudaError_t of the last failing CUDA call made by this library. */
int32_t gs_last_cuda_error(void);

/* Projection + SH + tile counting: replaces _project_and_count_kernel and
 * its launcher (project.py:74-345). Writes the four projected op outputs,
 * per-Gaussian tile counts and the tile rectangles
 * bounds [N,4] = (xmin, xmax, ymin, ymax) used by gs_bin_*. When `records`
 * is not NULL it also writes the compositors' staged form of every Gaussian
 * with a non-zero count, records [N,16] float (16-byte aligned): per
 * Gaussian (mean_x, mean_y, conic_xx, 2 conic_xy), (conic_yy, opacity, skip
 * cutoff, conic_xy), (r, g, b, index as float bits) and the bounding box of
 * the pixels where alpha can reach 1/255. gs_composite_fwd/bwd read them. */
int32_t gs_project_fwd(int64_t n, int32_t num_sh, const float *mean, const float *rotation,
                       const float *scale, const float *opacity, const float *color,
                       const float *camera_rotation, const float *camera_translation,
                       const gs_params *params, float *projected_mean,
                       float *inverse_covariance, float *projected_color,
                       float *projected_opacity, int32_t *bounds, int32_t *counts,
                       float *records, gs_stream_t stream);

/* The records gs_project_fwd writes, built from the four projected arrays
 * (the op's outputs) of n Gaussians: for a caller that kept only those, e.g.
 * before a backward pass. No counterpart in the reference, whose compositing
 * kernels gather the four arrays per pixel tile. */
int32_t gs_pack_records(int64_t n, const float *projected_mean, const float *inverse_covariance,
                        const float *projected_color, const float *projected_opacity,
                        const gs_params *params, float *records, gs_stream_t stream);

/* Projection of one scene into `num_views` cameras at once (the batched
 * multi-camera form of gs_project_fwd; no counterpart in the reference, which
 * projects one view per call). Each thread reads its Gaussian's parameters
 * and SH coefficients once, computes the view-independent terms once and
 * projects into every camera; per view the outputs are bit-identical to
 * gs_project_fwd's. Cameras and scalars are HOST arrays:
 * camera_rotations_host [V,3,3], camera_translations_host [V,3],
 * params_host [V]. Outputs are [V, N, ...]: view v starts at v * N rows
 * (records, when not NULL, [V, N, 16]). */
int32_t gs_project_fwd_batch(int64_t n, int32_t num_sh, int32_t num_views, const float *mean,
                             const float *rotation, const float *scale, const float *opacity,
                             const float *color, const float *camera_rotations_host,
                             const float *camera_translations_host, const gs_params *params_host,
                             float *projected_mean, float *inverse_covariance,
                             float *projected_color, float *projected_opacity, int32_t *bounds,
                             int32_t *counts, float *records, gs_stream_t stream);

/* Binning, phase 1: the host sync of emit_intersections
 * (intersections.py:51-52). Orders the Gaussians with counts > 0 by depth
 * (stable: equal depth bits keep index order), prefix-sums their counts in
 * that order, copies the intersection total to *total_host and synchronises
 * `stream`. `workspace` (gs_bin_count_workspace_size(n) bytes) must be passed
 * unchanged to the following gs_bin_sort. Fails with GS_ERR_CAPACITY if the
 * total reaches 2^30. */
int32_t gs_bin_count(int64_t n, const float *projected_mean, const int32_t *counts,
                     void *workspace, uint64_t workspace_bytes, int64_t *total_host,
                     gs_stream_t stream);
uint64_t gs_bin_count_workspace_size(int64_t n);

/* Binning, phase 1 without the host wait (for several views in flight):
 * enqueues what gs_bin_count does and copies the intersection total and the
 * device error word into *total_host and *error_host on `stream` (use pinned
 * memory for a truly asynchronous copy). Read them after synchronising the
 * stream: a non-zero error word means a bounded wait gave up (as
 * GS_ERR_TIMEOUT), and a total of 2^30 or more exceeds the sort's capacity. */
int32_t gs_bin_count_async(int64_t n, const float *projected_mean, const int32_t *counts,
                           void *workspace, uint64_t workspace_bytes, int64_t *total_host,
                           uint32_t *error_host, gs_stream_t stream);

/* Binning, phase 2: emit + sort + tile ranges, replacing _emit_intersections
 * (intersections.py:10-74) and sort_intersections (intersections.py:77-88).
 * gaussian_ids [total] receives the Gaussian index of every (tile, Gaussian)
 * intersection ordered by (tile, depth bits, Gaussian index) -- the order of
 * the reference's stable sort of (tile << 32 | depth bits) keys emitted in
 * Gaussian order; ranges [num_tiles, 2] receives each tile's [start, end).
 * count_workspace is the buffer gs_bin_count (or gs_bin_count_async) filled;
 * sort_workspace holds gs_bin_sort_workspace_size(n, total, params) bytes of
 * scratch. `total` may be any capacity at least the intersection total: the
 * kernels read the true total from count_workspace, so the call can be
 * enqueued before the total reaches the host; gaussian_ids then holds its
 * first (true total) entries. If the true total exceeds the capacity the
 * result is wrong but every access stays inside the buffers -- redo with the
 * true total. */
int32_t gs_bin_sort(int64_t n, int64_t total, const int32_t *bounds, const int32_t *counts,
                    const gs_params *params, const void *count_workspace,
                    uint64_t count_workspace_bytes, void *sort_workspace,
                    uint64_t sort_workspace_bytes, int32_t *gaussian_ids, int64_t *ranges,
                    gs_stream_t stream);
uint64_t gs_bin_sort_workspace_size(int64_t n, int64_t total, const gs_params *params);

/* Binning without any device allocation, for callers that cannot allocate
 * (no counterpart in the reference). Some callers have no workspace to hand
 * over: a plugin or FFI binding inside a host program that owns every device
 * allocation, or a per-frame loop that cannot afford cudaMalloc's implicit
 * device-wide synchronisation. This entry point does what gs_bin_count
 * followed by gs_bin_sort do, with its scratch in a 64 MiB array inside the
 * library (held on every GPU that loads the library until the process exits);
 * it never calls cudaMalloc or cudaFree.
 *  - Limit: the count-phase scratch for n Gaussians plus the sort-phase
 *    scratch for the intersection total must fit in 64 MiB (at 1920x1088
 *    with 16x16 tiles about 18 bytes per Gaussian plus 4.5 bytes per
 *    intersection: e.g. 1M Gaussians with up to 10M intersections; a grid of
 *    more than 256 tile columns or 512 tile rows bins by radix sort, about
 *    16.3 bytes per intersection). Larger inputs return
 *    GS_ERR_CAPACITY, as does a total above ids_capacity; *total_host still
 *    reports the total.
 *  - The first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress), so make that first call before any stream
 *    capture.
 *  - All calls on a device share the array and it keeps the previous call's
 *    contents (every call clears what it needs); calls whose GPU work
 *    overlaps -- other streams, other host threads -- race on it, so
 *    serialise them.
 *  - Synchronises `stream` twice: after the count phase, to read the
 *    intersection total, and at the end, to read the error word of the sort
 *    phase, which lives in the library's array where gs_bin_check cannot
 *    reach it. GS_ERR_TIMEOUT means a bounded wait of either phase gave up
 *    (the ids and ranges are then invalid). */
int32_t gs_bin_noalloc(int64_t n, const float *projected_mean, const int32_t *counts,
                       const int32_t *bounds, const gs_params *params, int32_t *gaussian_ids,
                       int64_t ids_capacity, int64_t *ranges, int64_t *total_host,
                       gs_stream_t stream);

/* The order in which the compositors visit the view's tiles: the tiles by
 * decreasing work (quarter-octave classes), so the longest lists start first
 * instead of whenever their row of tiles comes up. No counterpart in the
 * reference, whose Triton launches take tiles in grid order (composite.py:140,
 * composite_bwd.py:248). Work is each tile's list length (from ranges) for
 * the forward, or with n_contributors [H,W] its largest contributor count
 * (for gs_composite_bwd_deterministic). tile_work is scratch of num_tiles +
 * 128 uint32 words; tile_order receives [num_tiles] int32, a permutation of
 * the tile indices. */
int32_t gs_tile_order(const int64_t *ranges, const int32_t *n_contributors,
                      const gs_params *params, int32_t *tile_order, uint32_t *tile_work,
                      gs_stream_t stream);

/* Front-to-back compositing: replaces _composite_kernel (composite.py:25-162).
 * records: what gs_project_fwd (or gs_pack_records) wrote for the view.
 * image [H,W,3], final_transmittance [H,W], n_contributors [H,W] int32.
 * tile_order: gs_tile_order's permutation, or NULL for row-major order (the
 * results are the same either way). */
int32_t gs_composite_fwd(const float *records, const int32_t *gaussian_ids, const int64_t *ranges,
                         const gs_params *params, float *image, float *final_transmittance,
                         int32_t *n_contributors, const int32_t *tile_order,
                         gs_stream_t stream);

/* Back-to-front compositing gradients: replaces _composite_bwd_kernel and the
 * index_add_ reduction (composite_bwd.py:47-277). Accumulates into
 * grad_projected [N,9] = (d mean_x, d mean_y, d conic_xx, d conic_xy,
 * d conic_yy, d r, d g, d b, d opacity), which this call zeroes first.
 * plan: what gs_composite_bwd_plan built for this render (its tiles heaviest
 * first, the longest ones split), or NULL for whole tiles in row-major order;
 * the gradients agree either way within float rounding (the order of the
 * float atomics differs). */
int32_t gs_composite_bwd(int64_t n, const float *records, const int32_t *gaussian_ids,
                         const int64_t *ranges, const float *grad_image,
                         const float *final_transmittance, const int32_t *n_contributors,
                         const gs_params *params, float *grad_projected, const void *plan,
                         gs_stream_t stream);

/* The backward's work plan of one render (no counterpart in the reference,
 * whose backward takes one tile per program, composite_bwd.py:248): every
 * tile, heaviest first by its walk (list length up to its largest
 * contributor count, composite_bwd.py:81-83), with the tiles whose walk is
 * longer than split_walk entries (0: 2048) cut into parts of at most that
 * many -- one CTA each, which first walks the parts behind its own for the
 * suffix it starts from (the same recurrence, so the same bits) -- so one
 * dense tile no longer sets the kernel's length. Up to 1024 parts beyond the
 * tiles' first ones per view (tiles beyond stay whole). `plan` holds
 * gs_composite_bwd_plan_size(params) bytes, 256-byte aligned. */
uint64_t gs_composite_bwd_plan_size(const gs_params *params);
int32_t gs_composite_bwd_plan(const int64_t *ranges, const int32_t *n_contributors,
                              const gs_params *params, int32_t split_walk, void *plan,
                              uint64_t plan_bytes, gs_stream_t stream);

/* The same gradients, the same bits on every run: the reference's
 * per-intersection form (composite_bwd.py:237-277, its non-atomic default,
 * interface.py:218) made order-fixed. Each tile writes one 9-float row per
 * list position (its warps' contributions added in warp order), the positions
 * are grouped by Gaussian with a stable sort, and each Gaussian's rows are
 * added in list order -- no float addition depends on scheduling. `total` is
 * the length of gaussian_ids (every entry a valid index); the workspace holds
 * gs_composite_bwd_deterministic_workspace_size(n, total) bytes, 256-byte
 * aligned (rows, order, segments and the sort's scratch). Writes
 * grad_projected [N,9] (no zeroing needed). */
uint64_t gs_composite_bwd_deterministic_workspace_size(int64_t n, int64_t total);
int32_t gs_composite_bwd_deterministic(int64_t n, int64_t total, const float *records,
                                       const int32_t *gaussian_ids, const int64_t *ranges,
                                       const float *grad_image, const float *final_transmittance,
                                       const int32_t *n_contributors, const gs_params *params,
                                       void *workspace, uint64_t workspace_bytes,
                                       float *grad_projected, const int32_t *tile_order,
                                       gs_stream_t stream);

/* Parameter gradients: replaces _project_bwd_kernel (project_bwd.py:8-381).
 * SH gradients cover all K coefficients: degree 4 (K = 25) differentiates the
 * forward basis, where the reference's backward stops at 16 (project_bwd.py:33). */
int32_t gs_project_bwd(int64_t n, int32_t num_sh, const float *mean, const float *rotation,
                       const float *scale, const float *opacity, const float *color,
                       const float *camera_rotation, const float *camera_translation,
                       const float *inverse_covariance, const float *grad_projected,
                       const int32_t *counts, const gs_params *params, float *grad_mean,
                       float *grad_rotation, float *grad_scale, float *grad_opacity,
                       float *grad_color, gs_stream_t stream);

/* Projection backward summed over several views (no counterpart in the
 * reference): the parameter gradients of sum_v (rasterize(view v) . grad_v),
 * given each view's screen-space gradient grad_projected [V,N,9] (what
 * gs_composite_bwd writes) and tile counts [V,N]. Each thread reads its
 * Gaussian's parameters once, recomputes each view's conic exactly as
 * gs_project_fwd computed it, and adds the per-view gradients of
 * gs_project_bwd in view order. `views` is a DEVICE array of V records of 29
 * 32-bit words: the view's gs_params (its 17 words as laid out above), the
 * camera rotation (9 floats, row-major) and translation (3 floats) -- so a
 * collective can deliver them without a host round trip. For view-parallel
 * training this replaces all-reducing the parameter gradients (59 floats per
 * Gaussian at SH degree 3) with all-gathering the screen-space ones (9 floats
 * and a count). */
int32_t gs_project_bwd_views(int64_t n, int32_t num_sh, int32_t num_views, const float *mean,
                             const float *rotation, const float *scale, const float *opacity,
                             const float *color, const void *views, const float *grad_projected,
                             const int32_t *counts, float *grad_mean, float *grad_rotation,
                             float *grad_scale, float *grad_opacity, float *grad_color,
                             gs_stream_t stream);

/* ------------------------------------------- view-parallel exchange, peers */

#define GS_MAX_PEERS 8

/* A group of ranks (one process per GPU on one node) exchanging screen-space
 * gradients through peer memory: this rank, the number of ranks, and every
 * rank's exchange arena as mapped in this process (arena[rank] is this GPU's
 * own; each 256-byte aligned, all gs_exchange_layout(n).bytes long, zeroed
 * before first use). */
typedef struct gs_peer_group {
  int32_t rank, world;
  void *arena[GS_MAX_PEERS];
} gs_peer_group;

/* Byte offsets inside an arena for n Gaussians: the screen-space gradient
 * [n, 9] float, tile counts [n] int32, this rank's 29-word view record (as
 * gs_project_bwd_views takes them) and the gathered records of all ranks. */
typedef struct gs_exchange_layout {
  uint64_t grad_projected, counts, record, gathered, bytes;
} gs_exchange_layout;

int32_t gs_exchange_layout_for(int64_t n, int32_t world, gs_exchange_layout *out);

/* One view-parallel backward step, in stream order (all bounded waits; a wait
 * that gives up sets an error bit that gs_exchange_status reports):
 *   gs_exchange_begin     wait until every peer finished reading this rank's
 *                         arena of the previous step;
 *   (compositing backward into the arena's gradient, counts and record
 *    copied into it)
 *   gs_exchange_publish   publish this rank's step, wait for every peer's,
 *                         gather the view records;
 *   gs_exchange_gather    bulk-copy the peers' gradients and counts here;
 *   gs_exchange_finish    tell every peer this rank is done reading (right
 *                         after the gather: nothing reads peer memory later);
 *   gs_project_bwd_peers  projection backward summed over every rank's view.
 * Without the gather, gs_project_bwd_peers reads the peers' arenas directly
 * and gs_exchange_finish must come after it. Step counters live in the
 * arenas, so the sequence replays from a CUDA graph. No counterpart in the
 * reference (it is single-device). */
int32_t gs_exchange_begin(const gs_peer_group *group, gs_stream_t stream);
int32_t gs_exchange_publish(const gs_peer_group *group, int64_t n, gs_stream_t stream);
/* Optional, after gs_exchange_publish: bulk-copy every peer's gradient and
 * counts into this GPU's [world, n, 9] / [world, n] buffers (slot p = rank p;
 * this rank's slot untouched), for gs_project_bwd_peers to read locally. */
int32_t gs_exchange_gather(const gs_peer_group *group, int64_t n, float *grad_projected,
                           int32_t *counts, gs_stream_t stream);
/* Reads each peer's gradient and counts from the gathered buffers when they
 * are given (NULL: straight from peer memory), this rank's from its arena. */
int32_t gs_project_bwd_peers(int64_t n, int32_t num_sh, const gs_peer_group *group,
                             const float *gathered_grad, const int32_t *gathered_counts,
                             const float *mean, const float *rotation, const float *scale,
                             const float *opacity, const float *color, float *grad_mean,
                             float *grad_rotation, float *grad_scale, float *grad_opacity,
                             float *grad_color, gs_stream_t stream);
int32_t gs_exchange_finish(const gs_peer_group *group, gs_stream_t stream);

/* Sharded exchange: the same step with the summed projection backward split
 * over the ranks (no counterpart in the reference). Rank p owns Gaussians
 * [p*rows, min(n, (p+1)*rows)), rows = ceil(n / world). The arena is then
 * gs_shard_layout(...).bytes long (the plain layout followed by this rank's
 * shard of parameter gradients, each array 256-byte aligned). A step is:
 *   gs_exchange_begin, (compositing backward, counts and record into the
 *   arena), gs_exchange_publish as above; then
 *   gs_exchange_gather_rows    copy this rank's shard rows of every rank's
 *                              gradient and counts into [world, rows, 9] /
 *                              [world, rows] buffers on this GPU;
 *   gs_project_bwd_shard       the projection backward of the shard summed
 *                              over every rank's view, into the arena;
 *   gs_exchange_publish_shard  release this rank's shard, wait for every
 *                              peer's (bounded);
 *   gs_exchange_gather_shards  copy every rank's shard into the full gradient
 *                              arrays (grad_color 16-byte aligned);
 *   gs_exchange_finish.
 * Each rank moves rows x 40 B from every peer plus the other ranks' shards of
 * parameter gradients, and computes 1/world of the summed backward. */
typedef struct gs_shard_layout {
  uint64_t rotation, color, mean, scale, opacity; /* byte offsets of the shard's gradients */
  uint64_t bytes;                                 /* arena bytes, shard included */
  int64_t rows;                                   /* Gaussians per shard */
} gs_shard_layout;

int32_t gs_exchange_shard_layout(int64_t n, int32_t world, int32_t num_sh, gs_shard_layout *out);
int32_t gs_exchange_gather_rows(const gs_peer_group *group, int64_t n, float *grad_rows,
                                int32_t *count_rows, gs_stream_t stream);
int32_t gs_project_bwd_shard(int64_t n, int32_t num_sh, const gs_peer_group *group,
                             const float *grad_rows, const int32_t *count_rows,
                             const float *mean, const float *rotation, const float *scale,
                             const float *opacity, const float *color, gs_stream_t stream);
int32_t gs_exchange_publish_shard(const gs_peer_group *group, gs_stream_t stream);
int32_t gs_exchange_gather_shards(const gs_peer_group *group, int64_t n, int32_t num_sh,
                                  float *grad_rotation, float *grad_color, float *grad_mean,
                                  float *grad_scale, float *grad_opacity, gs_stream_t stream);

/* GS_OK, or GS_ERR_TIMEOUT if any wait of this rank's exchanges gave up
 * (sticky). Synchronises `stream`. */
int32_t gs_exchange_status(const gs_peer_group *group, gs_stream_t stream);

/* Binning error word of a count workspace (0 = fine, else some device-side
 * bounded wait in the last gs_bin_count / gs_bin_sort on these workspaces
 * gave up). Synchronises `stream`. */
int32_t gs_bin_check(const void *count_workspace, const void *sort_workspace,
                     gs_stream_t stream);

/* ------------------------------------------------------------ training step */

/* The five parameter arrays of a splat set (or of its gradients or Adam
 * moments), laid out as the Gaussian tensors above. A NULL member in the
 * gradient set skips that parameter (torch.optim.Adam skips params whose
 * .grad is None). */
typedef struct gs_splat_arrays {
  float *mean, *rotation, *scale, *opacity, *color;
} gs_splat_arrays;

/* Step scalars, folded on the host in double and rounded to float the way
 * torch.optim.Adam's foreach path folds them (t = the step number, >= 1):
 *   lerp_weight = 1 - beta1, beta2, sq_weight = 1 - beta2, eps, and per
 *   parameter k (mean, rotation, scale, opacity, color) with its own step t_k:
 *   neg_step_size[k] = -(lr_k / (1 - beta1^t_k)), bias2_sqrt[k] =
 *   sqrt(1 - beta2^t_k); noise_lr and position_lr as noise_splats takes them. */
typedef struct gs_adam_params {
  float lerp_weight, beta2, sq_weight, eps;
  float neg_step_size[5];
  float bias2_sqrt[5];
  float noise_lr, position_lr;
} gs_adam_params;

/* One optimizer step: Adam (torch.optim.Adam as training/train.py:118,151
 * runs it, foreach order) on every parameter with a gradient, updating
 * `params`, `exp_avg` and `exp_avg_sq` in place; then, when `randn` [N,3] is
 * not NULL, the position noise of noise_splats (training/utils.py:50-62)
 * added to the updated means. Replaces optimizer.step() + noise_splats(). The
 * colour arrays must be 16-byte aligned. */
int32_t gs_adam_step(int64_t n, int32_t num_sh, const gs_splat_arrays *params,
                     const gs_splat_arrays *grads, const gs_splat_arrays *exp_avg,
                     const gs_splat_arrays *exp_avg_sq, const gs_adam_params *hyper,
                     const float *randn, gs_stream_t stream);

/* Workspace bytes gs_relocate needs for `n_src` counts (16-byte aligned). */
uint64_t gs_relocate_workspace_size(int64_t n_src);

/* Splat relocation: replaces copy_splats (training/utils.py:120-145) with its
 * normalize_copies (training/utils.py:94-101), and the Adam-moment reset of
 * relocate_splats (training/utils.py:187-193), in one pass. `counts` [n_src]
 * (int64, what sample_counts draws) gives each parent row's number of copies;
 * they must add up to `num_outputs`. Output slot j goes to row
 * output_indices[j] (int64), or output_base + j when output_indices is NULL,
 * and receives a copy of the parent whose run of counts covers j, parents in
 * index order (parents.repeat_interleave(copies)). Each parent and its copies
 * get the renormalised opacity logit and log scale of normalize_copies with
 * copies = count + 1 (clamped to 51), computed in double precision; mean,
 * rotation, colour and `normals` (may be NULL) are copied. Moment rows of the
 * parents and outputs are zeroed in `exp_avg` / `exp_avg_sq` (either set, or
 * any member, may be NULL). Rows are those of `splats` (n_rows >= n_src);
 * output rows must be distinct and not parents (as sampled in the reference:
 * parents have opacity >= 0.005, outputs are dead or new rows). Bad counts or
 * output rows are skipped and recorded; gs_relocate_status reports them.
 * rotation arrays 16-byte aligned. */
int32_t gs_relocate(int64_t n_src, int64_t n_rows, int32_t num_sh, const int64_t *counts,
                    int64_t num_outputs, const int64_t *output_indices, int64_t output_base,
                    const gs_splat_arrays *splats, float *normals, const gs_splat_arrays *exp_avg,
                    const gs_splat_arrays *exp_avg_sq, void *workspace, uint64_t workspace_size,
                    gs_stream_t stream);

/* GS_OK, or GS_ERR_INVALID_ARGUMENT if the last gs_relocate on this
 * workspace met negative counts, counts not adding up to num_outputs, or an
 * output row outside [0, n_rows). Synchronises `stream`. */
int32_t gs_relocate_status(const void *workspace, gs_stream_t stream);

/* ----------------------------------------------------------- training loss */

/* Float words of scratch gs_l1_loss needs (per-block partial sums). */
int64_t gs_l1_loss_scratch_floats(void);

/* L1 photometric loss (training/train.py:140: (image - target).abs().mean())
 * over the target's extent: image [height, width, channels] float32, target
 * [target_height, target_width, channels] covering the image's top-left
 * corner (the rendered image is padded to whole tiles). Writes the mean to
 * the device scalar `loss` (deterministic order; not bit-identical to
 * torch's mean). */
int32_t gs_l1_loss(const float *image, int64_t height, int64_t width, int64_t channels,
                   const float *target, int64_t target_height, int64_t target_width,
                   float *scratch, float *loss, gs_stream_t stream);

/* Its gradient for the whole image, padding included: sign(image - target)
 * times (*grad_loss x the float reciprocal of the element count) inside the
 * target's extent, zero outside -- the values of torch's abs / mean / slice
 * backward chain, bit for bit. */
int32_t gs_l1_loss_backward(const float *image, int64_t height, int64_t width, int64_t channels,
                            const float *target, int64_t target_height, int64_t target_width,
                            const float *grad_loss, float *grad_image, gs_stream_t stream);

/* The deterministic exp / log the kernels use, applied elementwise (test hook
 * for bitwise agreement with the CPU oracle). */
int32_t gs_det_exp(int64_t n, const float *x, float *y, gs_stream_t stream);
int32_t gs_det_log(int64_t n, const float *x, float *y, gs_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GS_B200_H */
