// L1 photometric loss of the training step (training/train.py:140:
// (image - target).abs().mean()), fused: the forward reads image and target
// once; the backward writes the whole gradient image, padding included, in one
// pass. Images are [H, W, C] float32, the target [h, w, C] covering the
// image's top-left h x w (the renderer pads to whole tiles; the loss uses the
// unpadded part).
//
// Gradient: d mean|x| / dx = sign(x) * g / count, with sign(0) = 0 and g the
// incoming gradient of the loss -- bit for bit the values of torch's
// abs / mean / slice backward chain. The forward sum is a fixed-order
// two-pass reduction (per-block partial sums in float, their total in double),
// so the loss value is deterministic; it differs from torch's own mean in the
// last bits of its rounding.

#include "common.cuh"

namespace gs {

int32_t launch_l1_fwd(const float* image, int64_t height, int64_t width, int64_t channels,
                      const float* target, int64_t target_height, int64_t target_width,
                      float* partials, float* loss, cudaStream_t stream);
int32_t launch_l1_bwd(const float* image, int64_t height, int64_t width, int64_t channels,
                      const float* target, int64_t target_height, int64_t target_width,
                      const float* grad_loss, float* grad_image, cudaStream_t stream);

namespace {

constexpr int kThreads = 256;
constexpr int kBlocks = 4 * kSmCount;  // partial sums of the forward

// Rows spread over the blocks, a row's elements over the threads (coalesced).
__global__ void __launch_bounds__(kThreads) l1_partial_kernel(
    const float* __restrict__ image, int64_t row_stride, const float* __restrict__ target,
    int64_t rows, int64_t row_length, float* __restrict__ partials) {
  float sum = 0.0f;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* image_row = image + r * row_stride;
    const float* target_row = target + r * row_length;
    for (int64_t c = threadIdx.x; c < row_length; c += kThreads)
      sum += fabsf(__ldg(image_row + c) - __ldg(target_row + c));
  }
  __shared__ float s_warp[kThreads / 32];
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((threadIdx.x & 31) == 0) s_warp[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x < 32) {
    sum = threadIdx.x < kThreads / 32 ? s_warp[threadIdx.x] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (threadIdx.x == 0) partials[blockIdx.x] = sum;
  }
}

__global__ void __launch_bounds__(kThreads) l1_total_kernel(const float* __restrict__ partials,
                                                            int num_partials, int64_t count,
                                                            float* __restrict__ loss) {
  double sum = 0.0;
  for (int k = threadIdx.x; k < num_partials; k += kThreads) sum += partials[k];
  __shared__ double s_warp[kThreads / 32];
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if ((threadIdx.x & 31) == 0) s_warp[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    double total = 0.0;
    for (int w = 0; w < kThreads / 32; ++w) total += s_warp[w];
    *loss = count > 0 ? static_cast<float>(total / static_cast<double>(count)) : 0.0f;
  }
}

// The whole gradient image: rows over the blocks, elements over the threads.
__global__ void __launch_bounds__(kThreads) l1_grad_kernel(
    const float* __restrict__ image, int64_t height, int64_t row_stride,
    const float* __restrict__ target, int64_t rows, int64_t row_length,
    const float* __restrict__ grad_loss, float* __restrict__ grad_image) {
  // g / count as torch's mean backward forms it: g times the float reciprocal
  const float scale = __ldg(grad_loss) * (1.0f / static_cast<float>(rows * row_length));
  for (int64_t r = blockIdx.x; r < height; r += gridDim.x) {
    const float* image_row = image + r * row_stride;
    const float* target_row = target + r * row_length;
    float* grad_row = grad_image + r * row_stride;
    for (int64_t c = threadIdx.x; c < row_stride; c += kThreads) {
      float g = 0.0f;
      if (r < rows && c < row_length) {
        const float d = __ldg(image_row + c) - __ldg(target_row + c);
        g = d > 0.0f ? scale : (d < 0.0f ? -scale : 0.0f * scale);
      }
      grad_row[c] = g;
    }
  }
}

}  // namespace

int32_t launch_l1_fwd(const float* image, int64_t height, int64_t width, int64_t channels,
                      const float* target, int64_t target_height, int64_t target_width,
                      float* partials, float* loss, cudaStream_t stream) {
  if (!image || !target || !partials || !loss || channels < 1 || target_height < 0 ||
      target_width < 0 || target_height > height || target_width > width)
    return GS_ERR_INVALID_ARGUMENT;
  l1_partial_kernel<<<kBlocks, kThreads, 0, stream>>>(image, width * channels, target,
                                                      target_height, target_width * channels,
                                                      partials);
  GS_TRY(check_launch());
  l1_total_kernel<<<1, kThreads, 0, stream>>>(partials, kBlocks,
                                              target_height * target_width * channels, loss);
  return check_launch();
}

int32_t launch_l1_bwd(const float* image, int64_t height, int64_t width, int64_t channels,
                      const float* target, int64_t target_height, int64_t target_width,
                      const float* grad_loss, float* grad_image, cudaStream_t stream) {
  if (!image || !target || !grad_loss || !grad_image || channels < 1 || target_height < 0 ||
      target_width < 0 || target_height > height || target_width > width)
    return GS_ERR_INVALID_ARGUMENT;
  if (height * width == 0) return GS_OK;
  l1_grad_kernel<<<kBlocks, kThreads, 0, stream>>>(image, height, width * channels, target,
                                                   target_height, target_width * channels,
                                                   grad_loss, grad_image);
  return check_launch();
}

int64_t l1_partials() { return kBlocks; }

}  // namespace gs
