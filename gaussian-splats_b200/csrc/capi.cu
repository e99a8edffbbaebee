// extern "C" entry points declared in include/gs_b200.h: argument checks,
// then the stage launchers.
#include <cstdint>
#include <cstdio>

#include "common.cuh"

namespace gs {

int32_t launch_project_fwd(int64_t, int32_t, const float*, const float*, const float*,
                           const float*, const float*, const float*, const float*,
                           const gs_params&, float*, float*, float*, float*, int32_t*, int32_t*,
                           float*, cudaStream_t);
int32_t launch_project_fwd_batch(int64_t, int32_t, int32_t, const float*, const float*,
                                 const float*, const float*, const float*, const float*,
                                 const float*, const gs_params*, float*, float*, float*, float*,
                                 int32_t*, int32_t*, float*, cudaStream_t);
int32_t launch_pack_records(int64_t, const float*, const float*, const float*, const float*,
                            const gs_params&, float*, cudaStream_t);
int32_t launch_bin_count_async(int64_t, const float*, const int32_t*, void*, int64_t*, uint32_t*,
                               cudaStream_t);
int32_t launch_project_bwd_views(int64_t, int32_t, int32_t, const float*, const float*,
                                 const float*, const float*, const float*, const void*,
                                 const float*, const int32_t*, float*, float*, float*, float*,
                                 float*, cudaStream_t);
int32_t launch_project_bwd(int64_t, int32_t, const float*, const float*, const float*,
                           const float*, const float*, const float*, const float*, const float*,
                           const float*, const int32_t*, const gs_params&, float*, float*, float*,
                           float*, float*, cudaStream_t);
int32_t launch_det_math(int, int64_t, const float*, float*, cudaStream_t);
uint64_t bin_count_workspace_size(int64_t);
uint64_t bin_sort_workspace_size(int64_t, int64_t, const gs_params&);
uint64_t bin_error_word_offset();
int32_t launch_bin_count(int64_t, const float*, const int32_t*, void*, int64_t*, uint32_t*,
                         cudaStream_t);
int32_t launch_bin_sort(int64_t, int64_t, const int32_t*, const int32_t*, const gs_params&,
                        const void*, void*, int32_t*, int64_t*, cudaStream_t);
int32_t launch_composite_fwd(const float*, const int32_t*, const int64_t*, const gs_params&,
                             float*, float*, int32_t*, const int32_t*, cudaStream_t);
int32_t launch_composite_bwd(int64_t, const float*, const int32_t*, const int64_t*, const float*,
                             const float*, const int32_t*, const gs_params&, float*, void*,
                             cudaStream_t);
uint64_t composite_bwd_plan_size(const gs_params&);
int32_t launch_composite_bwd_plan(const int64_t*, const int32_t*, const gs_params&, int, void*,
                                  cudaStream_t);
int32_t launch_tile_order(const int64_t*, const int32_t*, const gs_params&, int32_t*, uint32_t*,
                          cudaStream_t);
uint64_t composite_bwd_deterministic_workspace_size(int64_t, int64_t);
int32_t launch_composite_bwd_deterministic(int64_t, int64_t, const float*, const int32_t*,
                                           const int64_t*, const float*, const float*,
                                           const int32_t*, const gs_params&, void*, float*,
                                           const int32_t*, cudaStream_t);
int32_t launch_adam_step(int64_t, int32_t, const gs_splat_arrays&, const gs_splat_arrays&,
                         const gs_splat_arrays&, const gs_splat_arrays&, const gs_adam_params&,
                         const float*, cudaStream_t);
int32_t launch_project_bwd_peers(int64_t, int32_t, int32_t, const float*, const float*,
                                 const float*, const float*, const float*, const void*,
                                 const float* const*, const int32_t* const*, float*, float*,
                                 float*, float*, float*, cudaStream_t);
int32_t exchange_layout(int64_t, int32_t, gs_exchange_layout*);
int32_t launch_exchange_begin(const gs_peer_group&, cudaStream_t);
int32_t launch_exchange_publish(const gs_peer_group&, int64_t, cudaStream_t);
int32_t launch_exchange_finish(const gs_peer_group&, cudaStream_t);
int32_t exchange_gather(const gs_peer_group&, int64_t, float*, int32_t*, cudaStream_t);
int32_t exchange_status(const gs_peer_group&, cudaStream_t);
int32_t exchange_shard_layout(int64_t, int32_t, int32_t, gs_shard_layout*);
int32_t exchange_gather_rows(const gs_peer_group&, int64_t, float*, int32_t*, cudaStream_t);
int32_t launch_project_bwd_shard(int64_t, int32_t, const gs_peer_group&, const float*,
                                 const int32_t*, const float*, const float*, const float*,
                                 const float*, const float*, cudaStream_t);
int32_t launch_exchange_publish_shard(const gs_peer_group&, cudaStream_t);
int32_t exchange_gather_shards(const gs_peer_group&, int64_t, int32_t, float*, float*, float*,
                               float*, float*, cudaStream_t);
int32_t launch_l1_fwd(const float*, int64_t, int64_t, int64_t, const float*, int64_t, int64_t,
                      float*, float*, cudaStream_t);
int32_t launch_l1_bwd(const float*, int64_t, int64_t, int64_t, const float*, int64_t, int64_t,
                      const float*, float*, cudaStream_t);
int64_t l1_partials();
size_t relocate_workspace_size(int64_t);
int32_t launch_relocate(int64_t, int64_t, int32_t, const int64_t*, int64_t, const int64_t*,
                        int64_t, const gs_splat_arrays&, float*, const gs_splat_arrays*,
                        const gs_splat_arrays*, void*, size_t, cudaStream_t);
int32_t relocate_status(const void*, cudaStream_t);

namespace {
thread_local int32_t g_last_cuda_error = 0;

bool aligned(const void* ptr, uintptr_t bytes) {
  return (reinterpret_cast<uintptr_t>(ptr) % bytes) == 0;
}

bool valid_sh(int32_t num_sh) {
  return num_sh == 1 || num_sh == 4 || num_sh == 9 || num_sh == 16 || num_sh == 25;
}

}  // namespace

void set_cuda_error(cudaError_t err) { g_last_cuda_error = static_cast<int32_t>(err); }

}  // namespace gs

using gs::as_cuda;

extern "C" {

int32_t gs_version(void) { return 100; }

int32_t gs_last_cuda_error(void) { return gs::g_last_cuda_error; }

int32_t gs_project_fwd(int64_t n, int32_t num_sh, const float* mean, const float* rotation,
                       const float* scale, const float* opacity, const float* color,
                       const float* camera_rotation, const float* camera_translation,
                       const gs_params* params, float* projected_mean, float* inverse_covariance,
                       float* projected_color, float* projected_opacity, int32_t* bounds,
                       int32_t* counts, float* records, gs_stream_t stream) {
  GS_TRY(gs::check_params(params));
  if (n < 0 || n >= gs::kMaxGaussians) return GS_ERR_INVALID_ARGUMENT;
  if (!gs::valid_sh(num_sh)) return num_sh > 25 ? GS_ERR_UNSUPPORTED : GS_ERR_INVALID_ARGUMENT;
  if (!gs::aligned(rotation, 16) || !gs::aligned(inverse_covariance, 16) ||
      !gs::aligned(bounds, 16) || !gs::aligned(records, 16) ||
      ((num_sh == 4 || num_sh == 16) && !gs::aligned(color, 16)))
    return GS_ERR_MISALIGNED;
  return gs::launch_project_fwd(n, num_sh, mean, rotation, scale, opacity, color, camera_rotation,
                                camera_translation, *params, projected_mean, inverse_covariance,
                                projected_color, projected_opacity, bounds, counts, records,
                                as_cuda(stream));
}

int32_t gs_project_fwd_batch(int64_t n, int32_t num_sh, int32_t num_views, const float* mean,
                             const float* rotation, const float* scale, const float* opacity,
                             const float* color, const float* camera_rotations_host,
                             const float* camera_translations_host, const gs_params* params_host,
                             float* projected_mean, float* inverse_covariance,
                             float* projected_color, float* projected_opacity, int32_t* bounds,
                             int32_t* counts, float* records, gs_stream_t stream) {
  if (n < 0 || n >= gs::kMaxGaussians || num_views < 0) return GS_ERR_INVALID_ARGUMENT;
  if (num_views > 0 && (!camera_rotations_host || !camera_translations_host || !params_host))
    return GS_ERR_INVALID_ARGUMENT;
  for (int32_t v = 0; v < num_views; ++v) GS_TRY(gs::check_params(params_host + v));
  if (!gs::valid_sh(num_sh)) return num_sh > 25 ? GS_ERR_UNSUPPORTED : GS_ERR_INVALID_ARGUMENT;
  if (!gs::aligned(rotation, 16) || !gs::aligned(inverse_covariance, 16) ||
      !gs::aligned(bounds, 16) || !gs::aligned(records, 16) ||
      ((num_sh == 4 || num_sh == 16) && !gs::aligned(color, 16)))
    return GS_ERR_MISALIGNED;
  return gs::launch_project_fwd_batch(n, num_sh, num_views, mean, rotation, scale, opacity, color,
                                      camera_rotations_host, camera_translations_host,
                                      params_host, projected_mean, inverse_covariance,
                                      projected_color, projected_opacity, bounds, counts, records,
                                      as_cuda(stream));
}

int32_t gs_pack_records(int64_t n, const float* projected_mean, const float* inverse_covariance,
                        const float* projected_color, const float* projected_opacity,
                        const gs_params* params, float* records, gs_stream_t stream) {
  GS_TRY(gs::check_params(params));
  if (n < 0 || n >= gs::kMaxGaussians || (n > 0 && !records)) return GS_ERR_INVALID_ARGUMENT;
  if (!gs::aligned(inverse_covariance, 16) || !gs::aligned(records, 16)) return GS_ERR_MISALIGNED;
  return gs::launch_pack_records(n, projected_mean, inverse_covariance, projected_color,
                                 projected_opacity, *params, records, as_cuda(stream));
}

int32_t gs_bin_count_async(int64_t n, const float* projected_mean, const int32_t* counts,
                           void* workspace, uint64_t workspace_bytes, int64_t* total_host,
                           uint32_t* error_host, gs_stream_t stream) {
  if (n < 0 || n >= gs::kMaxGaussians || !total_host || !error_host)
    return GS_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < gs::bin_count_workspace_size(n)) return GS_ERR_INVALID_ARGUMENT;
  if (!gs::aligned(workspace, 256)) return GS_ERR_MISALIGNED;
  return gs::launch_bin_count_async(n, projected_mean, counts, workspace, total_host, error_host,
                                    as_cuda(stream));
}

uint64_t gs_bin_count_workspace_size(int64_t n) {
  return gs::bin_count_workspace_size(n < 0 ? 0 : n);
}

uint64_t gs_bin_sort_workspace_size(int64_t n, int64_t total, const gs_params* params) {
  if (gs::check_params(params) != GS_OK) return 0;
  return gs::bin_sort_workspace_size(n < 0 ? 0 : n, total < 0 ? 0 : total, *params);
}

int32_t gs_bin_count(int64_t n, const float* projected_mean, const int32_t* counts,
                     void* workspace, uint64_t workspace_bytes, int64_t* total_host,
                     gs_stream_t stream) {
  if (n < 0 || n >= gs::kMaxGaussians || !total_host) return GS_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < gs::bin_count_workspace_size(n)) return GS_ERR_INVALID_ARGUMENT;
  if (!gs::aligned(workspace, 256)) return GS_ERR_MISALIGNED;
  uint32_t error = 0;
  GS_TRY(gs::launch_bin_count(n, projected_mean, counts, workspace, total_host, &error,
                              as_cuda(stream)));
  if (error) return GS_ERR_TIMEOUT;
  if (*total_host >= gs::kMaxIntersections) return GS_ERR_CAPACITY;
  return GS_OK;
}

int32_t gs_bin_sort(int64_t n, int64_t total, const int32_t* bounds, const int32_t* counts,
                    const gs_params* params, const void* count_workspace,
                    uint64_t count_workspace_bytes, void* sort_workspace,
                    uint64_t sort_workspace_bytes, int32_t* gaussian_ids, int64_t* ranges,
                    gs_stream_t stream) {
  GS_TRY(gs::check_params(params));
  if (n < 0 || n >= gs::kMaxGaussians || total < 0) return GS_ERR_INVALID_ARGUMENT;
  if (total >= gs::kMaxIntersections) return GS_ERR_CAPACITY;
  if (count_workspace_bytes < gs::bin_count_workspace_size(n) ||
      sort_workspace_bytes < gs::bin_sort_workspace_size(n, total, *params))
    return GS_ERR_INVALID_ARGUMENT;
  if (!gs::aligned(count_workspace, 256) || !gs::aligned(sort_workspace, 256) ||
      !gs::aligned(bounds, 16))
    return GS_ERR_MISALIGNED;
  return gs::launch_bin_sort(n, total, bounds, counts, *params, count_workspace, sort_workspace,
                             gaussian_ids, ranges, as_cuda(stream));
}

int32_t gs_bin_check(const void* count_workspace, const void* sort_workspace,
                     gs_stream_t stream) {
  uint32_t words[2] = {0, 0};
  const uint64_t off = gs::bin_error_word_offset();
  if (count_workspace)
    GS_CUDA_TRY(cudaMemcpyAsync(&words[0], static_cast<const char*>(count_workspace) + off, 4,
                                cudaMemcpyDeviceToHost, as_cuda(stream)));
  if (sort_workspace)
    GS_CUDA_TRY(cudaMemcpyAsync(&words[1], static_cast<const char*>(sort_workspace) + off, 4,
                                cudaMemcpyDeviceToHost, as_cuda(stream)));
  GS_CUDA_TRY(cudaStreamSynchronize(as_cuda(stream)));
  return (words[0] | words[1]) ? GS_ERR_TIMEOUT : GS_OK;
}

int32_t gs_tile_order(const int64_t* ranges, const int32_t* n_contributors,
                      const gs_params* params, int32_t* tile_order, uint32_t* tile_work,
                      gs_stream_t stream) {
  GS_TRY(gs::check_params(params));
  if (!tile_order || !tile_work || !ranges) return GS_ERR_INVALID_ARGUMENT;
  return gs::launch_tile_order(ranges, n_contributors, *params, tile_order, tile_work,
                               as_cuda(stream));
}

int32_t gs_composite_fwd(const float* records, const int32_t* gaussian_ids,
                         const int64_t* ranges, const gs_params* params, float* image,
                         float* final_transmittance, int32_t* n_contributors,
                         const int32_t* tile_order, gs_stream_t stream) {
  GS_TRY(gs::check_params(params));
  if (!gs::aligned(records, 16)) return GS_ERR_MISALIGNED;
  return gs::launch_composite_fwd(records, gaussian_ids, ranges, *params, image,
                                  final_transmittance, n_contributors, tile_order,
                                  as_cuda(stream));
}

int32_t gs_composite_bwd(int64_t n, const float* records, const int32_t* gaussian_ids,
                         const int64_t* ranges, const float* grad_image,
                         const float* final_transmittance, const int32_t* n_contributors,
                         const gs_params* params, float* grad_projected, const void* plan,
                         gs_stream_t stream) {
  GS_TRY(gs::check_params(params));
  if (n < 0) return GS_ERR_INVALID_ARGUMENT;
  if (!gs::aligned(records, 16) || !gs::aligned(plan, 256)) return GS_ERR_MISALIGNED;
  return gs::launch_composite_bwd(n, records, gaussian_ids, ranges, grad_image,
                                  final_transmittance, n_contributors, *params, grad_projected,
                                  const_cast<void*>(plan), as_cuda(stream));
}

uint64_t gs_composite_bwd_plan_size(const gs_params* params) {
  if (gs::check_params(params) != GS_OK) return 0;
  return gs::composite_bwd_plan_size(*params);
}

int32_t gs_composite_bwd_plan(const int64_t* ranges, const int32_t* n_contributors,
                              const gs_params* params, int32_t split_walk, void* plan,
                              uint64_t plan_bytes, gs_stream_t stream) {
  GS_TRY(gs::check_params(params));
  if (!ranges || !n_contributors || !plan || split_walk < 0) return GS_ERR_INVALID_ARGUMENT;
  if (plan_bytes < gs::composite_bwd_plan_size(*params)) return GS_ERR_INVALID_ARGUMENT;
  if (!gs::aligned(plan, 256)) return GS_ERR_MISALIGNED;
  return gs::launch_composite_bwd_plan(ranges, n_contributors, *params, split_walk, plan,
                                       as_cuda(stream));
}

uint64_t gs_composite_bwd_deterministic_workspace_size(int64_t n, int64_t total) {
  return gs::composite_bwd_deterministic_workspace_size(n < 0 ? 0 : n, total < 0 ? 0 : total);
}

int32_t gs_composite_bwd_deterministic(int64_t n, int64_t total, const float* records,
                                       const int32_t* gaussian_ids, const int64_t* ranges,
                                       const float* grad_image, const float* final_transmittance,
                                       const int32_t* n_contributors, const gs_params* params,
                                       void* workspace, uint64_t workspace_bytes,
                                       float* grad_projected, const int32_t* tile_order,
                                       gs_stream_t stream) {
  GS_TRY(gs::check_params(params));
  if (n < 0 || n >= gs::kMaxGaussians || total < 0 || total >= gs::kMaxIntersections)
    return GS_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < gs::composite_bwd_deterministic_workspace_size(n, total))
    return GS_ERR_INVALID_ARGUMENT;
  if (!gs::aligned(records, 16) || !gs::aligned(workspace, 256) || !gs::aligned(gaussian_ids, 16))
    return GS_ERR_MISALIGNED;
  return gs::launch_composite_bwd_deterministic(n, total, records, gaussian_ids, ranges,
                                                grad_image, final_transmittance, n_contributors,
                                                *params, workspace, grad_projected,
                                                tile_order, as_cuda(stream));
}

int32_t gs_project_bwd(int64_t n, int32_t num_sh, const float* mean, const float* rotation,
                       const float* scale, const float* opacity, const float* color,
                       const float* camera_rotation, const float* camera_translation,
                       const float* inverse_covariance, const float* grad_projected,
                       const int32_t* counts, const gs_params* params, float* grad_mean,
                       float* grad_rotation, float* grad_scale, float* grad_opacity,
                       float* grad_color, gs_stream_t stream) {
  GS_TRY(gs::check_params(params));
  if (n < 0 || n >= gs::kMaxGaussians) return GS_ERR_INVALID_ARGUMENT;
  if (!gs::valid_sh(num_sh)) return num_sh > 25 ? GS_ERR_UNSUPPORTED : GS_ERR_INVALID_ARGUMENT;
  if (!gs::aligned(rotation, 16) || !gs::aligned(inverse_covariance, 16) ||
      !gs::aligned(grad_rotation, 16) ||
      ((num_sh == 4 || num_sh == 16) && (!gs::aligned(color, 16) || !gs::aligned(grad_color, 16))))
    return GS_ERR_MISALIGNED;
  return gs::launch_project_bwd(n, num_sh, mean, rotation, scale, opacity, color,
                                camera_rotation, camera_translation, inverse_covariance,
                                grad_projected, counts, *params, grad_mean, grad_rotation,
                                grad_scale, grad_opacity, grad_color, as_cuda(stream));
}

int32_t gs_adam_step(int64_t n, int32_t num_sh, const gs_splat_arrays* params,
                     const gs_splat_arrays* grads, const gs_splat_arrays* exp_avg,
                     const gs_splat_arrays* exp_avg_sq, const gs_adam_params* hyper,
                     const float* randn, gs_stream_t stream) {
  if (!params || !grads || !exp_avg || !exp_avg_sq || !hyper) return GS_ERR_INVALID_ARGUMENT;
  if (n < 0 || n >= gs::kMaxGaussians) return GS_ERR_INVALID_ARGUMENT;
  if (num_sh < 1 || num_sh > 25) return GS_ERR_INVALID_ARGUMENT;
  const gs_splat_arrays* sets[3] = {params, exp_avg, exp_avg_sq};
  for (const gs_splat_arrays* set : sets) {
    if (!set->mean || !set->rotation || !set->scale || !set->opacity || !set->color)
      return GS_ERR_INVALID_ARGUMENT;
    if (!gs::aligned(set->color, 16)) return GS_ERR_MISALIGNED;
  }
  if (grads->color && !gs::aligned(grads->color, 16)) return GS_ERR_MISALIGNED;
  return gs::launch_adam_step(n, num_sh, *params, *grads, *exp_avg, *exp_avg_sq, *hyper, randn,
                              as_cuda(stream));
}

int32_t gs_project_bwd_views(int64_t n, int32_t num_sh, int32_t num_views, const float* mean,
                             const float* rotation, const float* scale, const float* opacity,
                             const float* color, const void* views, const float* grad_projected,
                             const int32_t* counts, float* grad_mean, float* grad_rotation,
                             float* grad_scale, float* grad_opacity, float* grad_color,
                             gs_stream_t stream) {
  if (n < 0 || n >= gs::kMaxGaussians || num_views < 0 || (num_views > 0 && !views))
    return GS_ERR_INVALID_ARGUMENT;
  if (!gs::valid_sh(num_sh)) return num_sh > 25 ? GS_ERR_UNSUPPORTED : GS_ERR_INVALID_ARGUMENT;
  if (!gs::aligned(rotation, 16) || !gs::aligned(grad_rotation, 16) || !gs::aligned(views, 4) ||
      ((num_sh == 4 || num_sh == 16) && (!gs::aligned(color, 16) || !gs::aligned(grad_color, 16))))
    return GS_ERR_MISALIGNED;
  return gs::launch_project_bwd_views(n, num_sh, num_views, mean, rotation, scale, opacity, color,
                                      views, grad_projected, counts, grad_mean, grad_rotation,
                                      grad_scale, grad_opacity, grad_color, as_cuda(stream));
}

int32_t gs_exchange_layout_for(int64_t n, int32_t world, gs_exchange_layout* out) {
  return gs::exchange_layout(n, world, out);
}

int32_t gs_exchange_begin(const gs_peer_group* group, gs_stream_t stream) {
  if (!group) return GS_ERR_INVALID_ARGUMENT;
  return gs::launch_exchange_begin(*group, as_cuda(stream));
}

int32_t gs_exchange_publish(const gs_peer_group* group, int64_t n, gs_stream_t stream) {
  if (!group || n < 0 || n >= gs::kMaxGaussians) return GS_ERR_INVALID_ARGUMENT;
  return gs::launch_exchange_publish(*group, n, as_cuda(stream));
}

int32_t gs_exchange_gather(const gs_peer_group* group, int64_t n, float* grad_projected,
                           int32_t* counts, gs_stream_t stream) {
  if (!group || n < 0 || n >= gs::kMaxGaussians) return GS_ERR_INVALID_ARGUMENT;
  return gs::exchange_gather(*group, n, grad_projected, counts, as_cuda(stream));
}

int32_t gs_exchange_finish(const gs_peer_group* group, gs_stream_t stream) {
  if (!group) return GS_ERR_INVALID_ARGUMENT;
  return gs::launch_exchange_finish(*group, as_cuda(stream));
}

int32_t gs_exchange_status(const gs_peer_group* group, gs_stream_t stream) {
  if (!group) return GS_ERR_INVALID_ARGUMENT;
  return gs::exchange_status(*group, as_cuda(stream));
}

int32_t gs_project_bwd_peers(int64_t n, int32_t num_sh, const gs_peer_group* group,
                             const float* gathered_grad, const int32_t* gathered_counts,
                             const float* mean, const float* rotation, const float* scale,
                             const float* opacity, const float* color, float* grad_mean,
                             float* grad_rotation, float* grad_scale, float* grad_opacity,
                             float* grad_color, gs_stream_t stream) {
  if (!group || n < 0 || n >= gs::kMaxGaussians) return GS_ERR_INVALID_ARGUMENT;
  if (group->world < 1 || group->world > GS_MAX_PEERS || group->rank < 0 ||
      group->rank >= group->world)
    return GS_ERR_INVALID_ARGUMENT;
  if (!gs::valid_sh(num_sh)) return num_sh > 25 ? GS_ERR_UNSUPPORTED : GS_ERR_INVALID_ARGUMENT;
  if (!gs::aligned(rotation, 16) || !gs::aligned(grad_rotation, 16) ||
      ((num_sh == 4 || num_sh == 16) && (!gs::aligned(color, 16) || !gs::aligned(grad_color, 16))))
    return GS_ERR_MISALIGNED;
  gs_exchange_layout layout;
  GS_TRY(gs::exchange_layout(n, group->world, &layout));
  const float* grads[GS_MAX_PEERS] = {};
  const int32_t* counts[GS_MAX_PEERS] = {};
  for (int p = 0; p < group->world; ++p) {
    if (!group->arena[p] || !gs::aligned(group->arena[p], 256)) return GS_ERR_MISALIGNED;
    const char* base = static_cast<const char*>(group->arena[p]);
    const bool local = p == group->rank || !gathered_grad || !gathered_counts;
    grads[p] = local ? reinterpret_cast<const float*>(base + layout.grad_projected)
                     : gathered_grad + 9 * n * p;
    counts[p] = local ? reinterpret_cast<const int32_t*>(base + layout.counts)
                      : gathered_counts + n * p;
  }
  const void* records = static_cast<const char*>(group->arena[group->rank]) + layout.gathered;
  return gs::launch_project_bwd_peers(n, num_sh, group->world, mean, rotation, scale, opacity,
                                      color, records, grads, counts, grad_mean, grad_rotation,
                                      grad_scale, grad_opacity, grad_color, as_cuda(stream));
}

int32_t gs_exchange_shard_layout(int64_t n, int32_t world, int32_t num_sh,
                                 gs_shard_layout* out) {
  if (!gs::valid_sh(num_sh)) return num_sh > 25 ? GS_ERR_UNSUPPORTED : GS_ERR_INVALID_ARGUMENT;
  return gs::exchange_shard_layout(n, world, num_sh, out);
}

int32_t gs_exchange_gather_rows(const gs_peer_group* group, int64_t n, float* grad_rows,
                                int32_t* count_rows, gs_stream_t stream) {
  if (!group || n < 0 || n >= gs::kMaxGaussians) return GS_ERR_INVALID_ARGUMENT;
  return gs::exchange_gather_rows(*group, n, grad_rows, count_rows, as_cuda(stream));
}

int32_t gs_project_bwd_shard(int64_t n, int32_t num_sh, const gs_peer_group* group,
                             const float* grad_rows, const int32_t* count_rows, const float* mean,
                             const float* rotation, const float* scale, const float* opacity,
                             const float* color, gs_stream_t stream) {
  if (!group || n < 0 || n >= gs::kMaxGaussians) return GS_ERR_INVALID_ARGUMENT;
  if (!gs::valid_sh(num_sh)) return num_sh > 25 ? GS_ERR_UNSUPPORTED : GS_ERR_INVALID_ARGUMENT;
  if (!gs::aligned(rotation, 16) || ((num_sh == 4 || num_sh == 16) && !gs::aligned(color, 16)))
    return GS_ERR_MISALIGNED;
  return gs::launch_project_bwd_shard(n, num_sh, *group, grad_rows, count_rows, mean, rotation,
                                      scale, opacity, color, as_cuda(stream));
}

int32_t gs_exchange_publish_shard(const gs_peer_group* group, gs_stream_t stream) {
  if (!group) return GS_ERR_INVALID_ARGUMENT;
  return gs::launch_exchange_publish_shard(*group, as_cuda(stream));
}

int32_t gs_exchange_gather_shards(const gs_peer_group* group, int64_t n, int32_t num_sh,
                                  float* grad_rotation, float* grad_color, float* grad_mean,
                                  float* grad_scale, float* grad_opacity, gs_stream_t stream) {
  if (!group || n < 0 || n >= gs::kMaxGaussians) return GS_ERR_INVALID_ARGUMENT;
  if (!gs::valid_sh(num_sh)) return num_sh > 25 ? GS_ERR_UNSUPPORTED : GS_ERR_INVALID_ARGUMENT;
  return gs::exchange_gather_shards(*group, n, num_sh, grad_rotation, grad_color, grad_mean,
                                    grad_scale, grad_opacity, as_cuda(stream));
}

uint64_t gs_relocate_workspace_size(int64_t n_src) {
  return n_src < 0 ? 0 : gs::relocate_workspace_size(n_src);
}

int32_t gs_relocate(int64_t n_src, int64_t n_rows, int32_t num_sh, const int64_t* counts,
                    int64_t num_outputs, const int64_t* output_indices, int64_t output_base,
                    const gs_splat_arrays* splats, float* normals, const gs_splat_arrays* exp_avg,
                    const gs_splat_arrays* exp_avg_sq, void* workspace, uint64_t workspace_size,
                    gs_stream_t stream) {
  if (!splats || !workspace || (n_src > 0 && !counts)) return GS_ERR_INVALID_ARGUMENT;
  if (n_src < 0 || n_rows < n_src || n_rows >= gs::kMaxGaussians || num_outputs < 0)
    return GS_ERR_INVALID_ARGUMENT;
  if (!output_indices &&
      (num_outputs > 0 && (output_base < 0 || output_base > n_rows - num_outputs)))
    return GS_ERR_INVALID_ARGUMENT;
  if (!gs::valid_sh(num_sh)) return num_sh > 25 ? GS_ERR_UNSUPPORTED : GS_ERR_INVALID_ARGUMENT;
  if (!splats->mean || !splats->rotation || !splats->scale || !splats->opacity || !splats->color)
    return GS_ERR_INVALID_ARGUMENT;
  if (!gs::aligned(splats->rotation, 16) || !gs::aligned(workspace, 16) ||
      !gs::aligned(counts, 8) || !gs::aligned(output_indices, 8))
    return GS_ERR_MISALIGNED;
  for (const gs_splat_arrays* m : {exp_avg, exp_avg_sq})
    if (m && m->rotation && !gs::aligned(m->rotation, 16)) return GS_ERR_MISALIGNED;
  return gs::launch_relocate(n_src, n_rows, num_sh, counts, num_outputs, output_indices,
                             output_base, *splats, normals, exp_avg, exp_avg_sq, workspace,
                             workspace_size, as_cuda(stream));
}

int32_t gs_relocate_status(const void* workspace, gs_stream_t stream) {
  if (!workspace) return GS_ERR_INVALID_ARGUMENT;
  return gs::relocate_status(workspace, as_cuda(stream));
}

int64_t gs_l1_loss_scratch_floats(void) { return gs::l1_partials(); }

int32_t gs_l1_loss(const float* image, int64_t height, int64_t width, int64_t channels,
                   const float* target, int64_t target_height, int64_t target_width,
                   float* scratch, float* loss, gs_stream_t stream) {
  if (height < 0 || width < 0) return GS_ERR_INVALID_ARGUMENT;
  return gs::launch_l1_fwd(image, height, width, channels, target, target_height, target_width,
                           scratch, loss, as_cuda(stream));
}

int32_t gs_l1_loss_backward(const float* image, int64_t height, int64_t width, int64_t channels,
                            const float* target, int64_t target_height, int64_t target_width,
                            const float* grad_loss, float* grad_image, gs_stream_t stream) {
  if (height < 0 || width < 0) return GS_ERR_INVALID_ARGUMENT;
  return gs::launch_l1_bwd(image, height, width, channels, target, target_height, target_width,
                           grad_loss, grad_image, as_cuda(stream));
}

int32_t gs_det_exp(int64_t n, const float* x, float* y, gs_stream_t stream) {
  if (n < 0) return GS_ERR_INVALID_ARGUMENT;
  return gs::launch_det_math(0, n, x, y, as_cuda(stream));
}

int32_t gs_det_log(int64_t n, const float* x, float* y, gs_stream_t stream) {
  if (n < 0) return GS_ERR_INVALID_ARGUMENT;
  return gs::launch_det_math(1, n, x, y, as_cuda(stream));
}

}  // extern "C"
