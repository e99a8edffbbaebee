// Splat relocation (the MCMC "relocate" step of training/utils.py:83-210):
// copies of sampled parent splats are written over dead or new rows, and the
// parents' and copies' opacity and scale are renormalised so that the copies
// together render like the parent did.
//
// Input is what the reference's sample_counts draws (training/utils.py:104-107):
// counts[i] = how many copies parent i gets, with sum(counts) = the number of
// output rows. Output slot j (0 <= j < num_outputs) goes to row
// output_indices[j] (or output_base + j) and is a copy of the parent whose
// run of counts covers j, in index order -- parents.repeat_interleave(copies)
// of copy_splats (training/utils.py:120-145). Three launches:
//   1. chunk_sum_kernel: the sum of each 4096-count chunk;
//   2. scan_chunks_kernel (one CTA): exclusive offsets of the chunks, and the
//      check that the counts add up to num_outputs;
//   3. relocate_kernel<K>: per thread 16 consecutive counts, a block scan for
//      their output offsets, then per parent normalize_copies
//      (training/utils.py:94-101) and the writes: the parent's new opacity and
//      scale, each copy's mean, rotation, colour, normals, opacity and scale,
//      and zeros in the Adam moments of the parent and copy rows (the
//      optimizer-state reset of training/utils.py:187-193).
// The renormalisation runs in double precision (the binomial series has
// alternating signs) and is rounded to float once per output.

#include "common.cuh"

namespace gs {

size_t relocate_workspace_size(int64_t n_src);
int32_t launch_relocate(int64_t n_src, int64_t n_rows, int32_t num_sh, const int64_t* counts,
                        int64_t num_outputs, const int64_t* output_indices, int64_t output_base,
                        const gs_splat_arrays& splats, float* normals,
                        const gs_splat_arrays* exp_avg, const gs_splat_arrays* exp_avg_sq,
                        void* workspace, size_t workspace_size, cudaStream_t stream);
int32_t relocate_status(const void* workspace, cudaStream_t stream);

namespace {

constexpr int kThreads = 256;
constexpr int kItems = 16;  // consecutive counts per thread
constexpr int64_t kChunk = int64_t{kThreads} * kItems;
constexpr int kMaxCopies = 51;  // normalize_copies clamps copies to [1, 51]

// Error bits in the workspace's first word.
constexpr uint32_t kNegativeCount = 1u;
constexpr uint32_t kTotalMismatch = 2u;
constexpr uint32_t kOutputOutOfRange = 4u;

struct Workspace {
  uint32_t* error;
  int64_t* chunk_offsets;
};

__host__ __device__ inline Workspace carve(void* base) {
  char* p = static_cast<char*>(base);
  return Workspace{reinterpret_cast<uint32_t*>(p), reinterpret_cast<int64_t*>(p + 16)};
}

// Block-wide sum / exclusive scan of one int64 per thread (256 threads).
__device__ __forceinline__ int64_t warp_inclusive_scan(int64_t v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int64_t up = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += up;
  }
  return v;
}

template <int kBlock>
__device__ __forceinline__ int64_t block_exclusive_scan64(int64_t v, int64_t* s_warp,
                                                          int64_t* total) {
  constexpr int kWarps = kBlock / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t inclusive = warp_inclusive_scan(v);
  if (lane == 31) s_warp[warp] = inclusive;
  __syncthreads();
  if (warp == 0) {
    const int64_t w = lane < kWarps ? s_warp[lane] : 0;
    const int64_t wi = warp_inclusive_scan(w);
    if (lane < kWarps) s_warp[lane] = wi - w;
    if (lane == kWarps - 1) s_warp[kWarps] = wi;
  }
  __syncthreads();
  const int64_t out = s_warp[warp] + inclusive - v;
  if (total) *total = s_warp[kWarps];
  __syncthreads();  // s_warp is reused by the caller's next scan
  return out;
}

__global__ void __launch_bounds__(kThreads) chunk_sum_kernel(int64_t n,
                                                             const int64_t* __restrict__ counts,
                                                             Workspace ws) {
  __shared__ int64_t s_warp[kThreads / 32 + 1];
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kChunk + threadIdx.x * kItems;
  int64_t local = 0;
#pragma unroll
  for (int k = 0; k < kItems; ++k) {
    const int64_t i = first + k;
    if (i < n) {
      const int64_t c = counts[i];
      if (c < 0) atomicOr(ws.error, kNegativeCount);
      local += c > 0 ? c : 0;
    }
  }
  int64_t total;
  block_exclusive_scan64<kThreads>(local, s_warp, &total);
  if (threadIdx.x == 0) ws.chunk_offsets[blockIdx.x] = total;
}

// One CTA: chunk sums -> exclusive chunk offsets, in place.
__global__ void __launch_bounds__(1024) scan_chunks_kernel(int64_t num_chunks, int64_t num_outputs,
                                                           Workspace ws) {
  __shared__ int64_t s_warp[1024 / 32 + 1];
  int64_t carry = 0;
  for (int64_t base = 0; base < num_chunks; base += 1024) {
    const int64_t c = base + threadIdx.x;
    const int64_t v = c < num_chunks ? ws.chunk_offsets[c] : 0;
    int64_t tile_total;
    const int64_t prefix = block_exclusive_scan64<1024>(v, s_warp, &tile_total);
    if (c < num_chunks) ws.chunk_offsets[c] = carry + prefix;
    carry += tile_total;
  }
  if (threadIdx.x == 0 && carry != num_outputs) atomicOr(ws.error, kTotalMismatch);
}

// normalize_copies (training/utils.py:94-101) for one parent of opacity
// `logit` with `copies` = its count + 1, clamped to [1, 51]:
//   o' = 1 - (1 - o)^(1 / copies),
//   sum = sum_{d=1..copies} C(copies, d) (-1)^(d-1) o'^d / sqrt(d),
//   scale' = scale * o / sum; opacity' = clamp(o', 0.005, 1 - 1e-6).
// Returns the new opacity logit and writes the factor o / sum.
__device__ __forceinline__ float renormalise(float logit, int copies, double* ratio) {
  const double o = 1.0 / (1.0 + exp(-static_cast<double>(logit)));
  const double new_opacity = 1.0 - pow(1.0 - o, 1.0 / copies);
  double sum = 0.0, binomial = 1.0, power = 1.0;
  for (int d = 1; d <= copies; ++d) {
    binomial = binomial * (copies - d + 1) / d;  // exact: every C(51, d) < 2^53
    power = power * new_opacity;
    const double term = binomial * power / sqrt(static_cast<double>(d));
    sum = (d & 1) ? sum + term : sum - term;
  }
  *ratio = o / sum;
  // the clamp bounds as the float32 tensor sees them
  const double p = fmin(fmax(new_opacity, static_cast<double>(0.005f)),
                        static_cast<double>(static_cast<float>(1.0 - 1e-6)));
  return static_cast<float>(log(p / (1.0 - p)));
}

__device__ __forceinline__ void zero_row(const gs_splat_arrays* m, int64_t row, int num_sh) {
  if (!m) return;
  if (m->mean) {
    m->mean[3 * row] = 0.0f; m->mean[3 * row + 1] = 0.0f; m->mean[3 * row + 2] = 0.0f;
  }
  if (m->rotation) reinterpret_cast<float4*>(m->rotation)[row] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (m->scale) {
    m->scale[3 * row] = 0.0f; m->scale[3 * row + 1] = 0.0f; m->scale[3 * row + 2] = 0.0f;
  }
  if (m->opacity) m->opacity[row] = 0.0f;
  if (m->color) {
    float* c = m->color + row * (3 * num_sh);
    for (int j = 0; j < 3 * num_sh; ++j) c[j] = 0.0f;
  }
}

struct Moments {
  gs_splat_arrays exp_avg, exp_avg_sq;
  bool has_avg, has_avg_sq;
};

template <int K>
__global__ void __launch_bounds__(kThreads) relocate_kernel(
    int64_t n_src, int64_t n_rows, const int64_t* __restrict__ counts, int64_t num_outputs,
    const int64_t* __restrict__ output_indices, int64_t output_base, gs_splat_arrays s,
    float* __restrict__ normals, Moments moments, Workspace ws) {
  __shared__ int64_t s_warp[kThreads / 32 + 1];
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kChunk + threadIdx.x * kItems;
  int64_t c[kItems];
  int64_t local = 0;
#pragma unroll
  for (int k = 0; k < kItems; ++k) {
    const int64_t i = first + k;
    c[k] = i < n_src ? counts[i] : 0;
    c[k] = c[k] > 0 ? c[k] : 0;
    local += c[k];
  }
  int64_t offset = ws.chunk_offsets[blockIdx.x] + block_exclusive_scan64<kThreads>(local, s_warp,
                                                                                   nullptr);
  const gs_splat_arrays* avg = moments.has_avg ? &moments.exp_avg : nullptr;
  const gs_splat_arrays* avg_sq = moments.has_avg_sq ? &moments.exp_avg_sq : nullptr;
  for (int k = 0; k < kItems; ++k) {
    if (c[k] == 0) continue;
    const int64_t parent = first + k;
    const int copies = c[k] + 1 < kMaxCopies ? static_cast<int>(c[k] + 1) : kMaxCopies;
    double ratio;
    const float opacity_logit = renormalise(s.opacity[parent], copies, &ratio);
    float log_scale[3];
#pragma unroll
    for (int a = 0; a < 3; ++a)
      log_scale[a] = static_cast<float>(log(exp(static_cast<double>(s.scale[3 * parent + a])) *
                                            ratio));
    const float m0 = s.mean[3 * parent], m1 = s.mean[3 * parent + 1], m2 = s.mean[3 * parent + 2];
    const float4 q = reinterpret_cast<const float4*>(s.rotation)[parent];
    const float* color = s.color + parent * (3 * K);
    for (int64_t j = offset; j < offset + c[k]; ++j) {
      if (j >= num_outputs) {
        atomicOr(ws.error, kTotalMismatch);
        break;
      }
      const int64_t row = output_indices ? output_indices[j] : output_base + j;
      if (row < 0 || row >= n_rows) {
        atomicOr(ws.error, kOutputOutOfRange);
        continue;
      }
      s.mean[3 * row] = m0; s.mean[3 * row + 1] = m1; s.mean[3 * row + 2] = m2;
      reinterpret_cast<float4*>(s.rotation)[row] = q;
      float* out_color = s.color + row * (3 * K);
#pragma unroll
      for (int e = 0; e < 3 * K; ++e) out_color[e] = color[e];
      if (normals) {
        normals[3 * row] = normals[3 * parent];
        normals[3 * row + 1] = normals[3 * parent + 1];
        normals[3 * row + 2] = normals[3 * parent + 2];
      }
      s.opacity[row] = opacity_logit;
      s.scale[3 * row] = log_scale[0]; s.scale[3 * row + 1] = log_scale[1];
      s.scale[3 * row + 2] = log_scale[2];
      zero_row(avg, row, K);
      zero_row(avg_sq, row, K);
    }
    offset += c[k];
    s.opacity[parent] = opacity_logit;
    s.scale[3 * parent] = log_scale[0]; s.scale[3 * parent + 1] = log_scale[1];
    s.scale[3 * parent + 2] = log_scale[2];
    zero_row(avg, parent, K);
    zero_row(avg_sq, parent, K);
  }
}

}  // namespace

size_t relocate_workspace_size(int64_t n_src) {
  const int64_t chunks = (n_src + kChunk - 1) / kChunk;
  return static_cast<size_t>(16 + 8 * ((chunks + 1) / 2) * 2);
}

int32_t launch_relocate(int64_t n_src, int64_t n_rows, int32_t num_sh, const int64_t* counts,
                        int64_t num_outputs, const int64_t* output_indices, int64_t output_base,
                        const gs_splat_arrays& splats, float* normals,
                        const gs_splat_arrays* exp_avg, const gs_splat_arrays* exp_avg_sq,
                        void* workspace, size_t workspace_size, cudaStream_t stream) {
  if (workspace_size < relocate_workspace_size(n_src)) return GS_ERR_INVALID_ARGUMENT;
  const Workspace ws = carve(workspace);
  const int64_t chunks = (n_src + kChunk - 1) / kChunk;
  Moments moments{};
  moments.has_avg = exp_avg != nullptr;
  moments.has_avg_sq = exp_avg_sq != nullptr;
  if (exp_avg) moments.exp_avg = *exp_avg;
  if (exp_avg_sq) moments.exp_avg_sq = *exp_avg_sq;
  GS_CUDA_TRY(cudaMemsetAsync(ws.error, 0, sizeof(uint32_t), stream));
  if (chunks > 0) {
    chunk_sum_kernel<<<static_cast<unsigned>(chunks), kThreads, 0, stream>>>(n_src, counts, ws);
    GS_TRY(check_launch());
  }
  scan_chunks_kernel<<<1, 1024, 0, stream>>>(chunks, num_outputs, ws);
  GS_TRY(check_launch());
  if (chunks == 0) return GS_OK;
#define GS_LAUNCH(K)                                                                        \
  relocate_kernel<K><<<static_cast<unsigned>(chunks), kThreads, 0, stream>>>(               \
      n_src, n_rows, counts, num_outputs, output_indices, output_base, splats, normals,     \
      moments, ws)
  switch (num_sh) {
    case 1: GS_LAUNCH(1); break;
    case 4: GS_LAUNCH(4); break;
    case 9: GS_LAUNCH(9); break;
    case 16: GS_LAUNCH(16); break;
    case 25: GS_LAUNCH(25); break;
    default: return GS_ERR_UNSUPPORTED;
  }
#undef GS_LAUNCH
  return check_launch();
}

int32_t relocate_status(const void* workspace, cudaStream_t stream) {
  uint32_t error = 0;
  GS_CUDA_TRY(cudaMemcpyAsync(&error, workspace, sizeof(error), cudaMemcpyDeviceToHost, stream));
  GS_CUDA_TRY(cudaStreamSynchronize(stream));
  return error ? GS_ERR_INVALID_ARGUMENT : GS_OK;
}

}  // namespace gs
