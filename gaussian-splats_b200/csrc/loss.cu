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

// Rows spread over the blocks, a row's elements over the threads (coalesced);
// with kVec, four floats per load (rows a multiple of 4 floats, 16-byte
// aligned).
template <bool kVec>
__global__ void __launch_bounds__(kThreads) l1_partial_kernel(
    const float* __restrict__ image, int64_t row_stride, const float* __restrict__ target,
    int64_t rows, int64_t row_length, float* __restrict__ partials) {
  chain_wait();
  float sum = 0.0f;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float* image_row = image + r * row_stride;
    const float* target_row = target + r * row_length;
    if constexpr (kVec) {
      const float4* a = reinterpret_cast<const float4*>(image_row);
      const float4* b = reinterpret_cast<const float4*>(target_row);
      for (int64_t c = threadIdx.x; c < row_length / 4; c += kThreads) {
        const float4 x = __ldg(a + c), y = __ldg(b + c);
        sum += fabsf(x.x - y.x);
        sum += fabsf(x.y - y.y);
        sum += fabsf(x.z - y.z);
        sum += fabsf(x.w - y.w);
      }
    } else {
      for (int64_t c = threadIdx.x; c < row_length; c += kThreads)
        sum += fabsf(__ldg(image_row + c) - __ldg(target_row + c));
    }
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
  chain_wait();
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

__device__ __forceinline__ float l1_grad(float image, float target, float scale) {
  const float d = image - target;
  return d > 0.0f ? scale : (d < 0.0f ? -scale : 0.0f * scale);
}

// The whole gradient image: rows over the blocks, elements over the threads
// (with kVec four at a time; rows and the target's rows a multiple of 4 floats,
// 16-byte aligned).
template <bool kVec>
__global__ void __launch_bounds__(kThreads) l1_grad_kernel(
    const float* __restrict__ image, int64_t height, int64_t row_stride,
    const float* __restrict__ target, int64_t rows, int64_t row_length,
    const float* __restrict__ grad_loss, float* __restrict__ grad_image) {
  chain_wait();
  // g / count as torch's mean backward forms it: g times the float reciprocal
  const float scale = __ldg(grad_loss) * (1.0f / static_cast<float>(rows * row_length));
  for (int64_t r = blockIdx.x; r < height; r += gridDim.x) {
    const float* image_row = image + r * row_stride;
    const float* target_row = target + r * row_length;
    float* grad_row = grad_image + r * row_stride;
    if constexpr (kVec) {
      for (int64_t c = threadIdx.x; c < row_stride / 4; c += kThreads) {
        float4 g = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (r < rows && 4 * c < row_length) {
          const float4 x = __ldg(reinterpret_cast<const float4*>(image_row) + c);
          const float4 y = __ldg(reinterpret_cast<const float4*>(target_row) + c);
          g = make_float4(l1_grad(x.x, y.x, scale), l1_grad(x.y, y.y, scale),
                          l1_grad(x.z, y.z, scale), l1_grad(x.w, y.w, scale));
        }
        reinterpret_cast<float4*>(grad_row)[c] = g;
      }
    } else {
      for (int64_t c = threadIdx.x; c < row_stride; c += kThreads) {
        float g = 0.0f;
        if (r < rows && c < row_length)
          g = l1_grad(__ldg(image_row + c), __ldg(target_row + c), scale);
        grad_row[c] = g;
      }
    }
  }
}

bool vectorisable(const void* image, const void* target, const void* grad, int64_t row_stride,
                  int64_t row_length) {
  const auto aligned16 = [](const void* p) {
    return p == nullptr || reinterpret_cast<uintptr_t>(p) % 16 == 0;
  };
  return row_stride % 4 == 0 && row_length % 4 == 0 && aligned16(image) && aligned16(target) &&
         aligned16(grad);
}

}  // namespace

int32_t launch_l1_fwd(const float* image, int64_t height, int64_t width, int64_t channels,
                      const float* target, int64_t target_height, int64_t target_width,
                      float* partials, float* loss, cudaStream_t stream) {
  if (!image || !target || !partials || !loss || channels < 1 || target_height < 0 ||
      target_width < 0 || target_height > height || target_width > width)
    return GS_ERR_INVALID_ARGUMENT;
  const int64_t row_stride = width * channels, row_length = target_width * channels;
  if (vectorisable(image, target, nullptr, row_stride, row_length))
    launch_chained(l1_partial_kernel<true>, kBlocks, kThreads, stream, image, row_stride, target,
                   target_height, row_length, partials);
  else
    launch_chained(l1_partial_kernel<false>, kBlocks, kThreads, stream, image, row_stride, target,
                   target_height, row_length, partials);
  GS_TRY(check_launch());
  launch_chained(l1_total_kernel, 1, kThreads, stream, partials, kBlocks,
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
  const int64_t row_stride = width * channels, row_length = target_width * channels;
  if (vectorisable(image, target, grad_image, row_stride, row_length))
    launch_chained(l1_grad_kernel<true>, kBlocks, kThreads, stream,
        image, height, row_stride, target, target_height, row_length, grad_loss, grad_image);
  else
    launch_chained(l1_grad_kernel<false>, kBlocks, kThreads, stream,
        image, height, row_stride, target, target_height, row_length, grad_loss, grad_image);
  return check_launch();
}

int64_t l1_partials() { return kBlocks; }

}  // namespace gs
