// Fused optimizer step of the training loop: Adam on every Gaussian
// parameter, then the position noise of the MCMC schedule, in one pass over
// HBM.
//
// The reference runs torch.optim.Adam (eps 1e-15, one group per parameter
// tensor, training/train.py:111-118,151) and then noise_splats
// (training/utils.py:50-62) as ~30 separate elementwise kernels, each
// re-reading its tensors. Here one kernel reads parameter, gradient and both
// moments once and writes parameter and moments once.
//
// Per element, in torch's foreach-Adam order (float32, no fused multiply-add
// unless written, so the CPU oracle reproduces it bit for bit):
//   m = m + (1 - beta1) (g - m)                        _foreach_lerp_
//   v = v beta2;  v = v + (1 - beta2) (g g)             _foreach_mul_, _foreach_addcmul_
//   d = sqrt(v) / sqrt(1 - beta2^t) + eps              _foreach_sqrt/div_/add_
//   p = p + (-(lr / (1 - beta1^t))) (m / d)            _foreach_addcdiv_
// with the step scalars folded on the host in double as torch folds them.
//
// Position noise, on the updated parameters (training/utils.py:50-62):
//   q = rotation / max(|rotation|, 1e-12), R = R(q), s = exp(scale),
//   F = R diag(s), C = F F^T, gate = sigmoid(100 (1 - sigmoid(opacity) - 0.995)),
//   n = ((randn gate) noise_lr) position_lr,  mean += C n
// with `randn` supplied by the caller (the reference draws it with
// torch.randn_like(mean)), so both sides see the same random numbers.
#include "common.cuh"

namespace gs {
namespace {

constexpr int kOptThreads = 256;

struct Moments {
  float w1, beta2, w2, eps;
};

__device__ __forceinline__ float adam_one(float p, float g, float& m, float& v, float neg_step,
                                          float bias2_sqrt, const Moments& c) {
  m = m + c.w1 * (g - m);
  v = v * c.beta2;
  v = v + c.w2 * (g * g);
  const float d = sqrtf(v) / bias2_sqrt + c.eps;
  return p + neg_step * (m / d);
}

__device__ __forceinline__ float sigmoid(float x) { return 1.0f / (1.0f + det_exp(-x)); }

template <bool kNoise>
__global__ void __launch_bounds__(kOptThreads) adam_step_kernel(
    int64_t n, int64_t color_per, gs_splat_arrays p, gs_splat_arrays g, gs_splat_arrays m,
    gs_splat_arrays v, gs_adam_params hp, const float* __restrict__ randn) {
  const Moments c{hp.lerp_weight, hp.beta2, hp.sq_weight, hp.eps};
  const int64_t i = static_cast<int64_t>(blockIdx.x) * kOptThreads + threadIdx.x;
  if (i < n) {
    float mean[3], rot[4], scale[3], opacity;
#pragma unroll
    for (int k = 0; k < 3; ++k) mean[k] = p.mean[3 * i + k];
#pragma unroll
    for (int k = 0; k < 4; ++k) rot[k] = p.rotation[4 * i + k];
#pragma unroll
    for (int k = 0; k < 3; ++k) scale[k] = p.scale[3 * i + k];
    opacity = p.opacity[i];
    if (g.mean) {
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        float mk = m.mean[3 * i + k], vk = v.mean[3 * i + k];
        mean[k] = adam_one(mean[k], g.mean[3 * i + k], mk, vk, hp.neg_step_size[0], hp.bias2_sqrt[0], c);
        m.mean[3 * i + k] = mk;
        v.mean[3 * i + k] = vk;
      }
    }
    if (g.rotation) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float mk = m.rotation[4 * i + k], vk = v.rotation[4 * i + k];
        rot[k] = adam_one(rot[k], g.rotation[4 * i + k], mk, vk, hp.neg_step_size[1], hp.bias2_sqrt[1], c);
        m.rotation[4 * i + k] = mk;
        v.rotation[4 * i + k] = vk;
        p.rotation[4 * i + k] = rot[k];
      }
    }
    if (g.scale) {
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        float mk = m.scale[3 * i + k], vk = v.scale[3 * i + k];
        scale[k] = adam_one(scale[k], g.scale[3 * i + k], mk, vk, hp.neg_step_size[2], hp.bias2_sqrt[2], c);
        m.scale[3 * i + k] = mk;
        v.scale[3 * i + k] = vk;
        p.scale[3 * i + k] = scale[k];
      }
    }
    if (g.opacity) {
      float mk = m.opacity[i], vk = v.opacity[i];
      opacity = adam_one(opacity, g.opacity[i], mk, vk, hp.neg_step_size[3], hp.bias2_sqrt[3], c);
      m.opacity[i] = mk;
      v.opacity[i] = vk;
      p.opacity[i] = opacity;
    }
    if constexpr (kNoise) {
      const float norm = sqrtf(((rot[0] * rot[0] + rot[1] * rot[1]) + rot[2] * rot[2]) +
                               rot[3] * rot[3]);
      const float inv = fmaxf(norm, 1e-12f);
      const float w = rot[0] / inv, x = rot[1] / inv, y = rot[2] / inv, z = rot[3] / inv;
      const float r[3][3] = {
          {1.0f - 2.0f * (y * y + z * z), 2.0f * (x * y - w * z), 2.0f * (x * z + w * y)},
          {2.0f * (x * y + w * z), 1.0f - 2.0f * (x * x + z * z), 2.0f * (y * z - w * x)},
          {2.0f * (x * z - w * y), 2.0f * (y * z + w * x), 1.0f - 2.0f * (x * x + y * y)}};
      const float s[3] = {det_exp(scale[0]), det_exp(scale[1]), det_exp(scale[2])};
      float f[3][3];
#pragma unroll
      for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int b = 0; b < 3; ++b) f[a][b] = r[a][b] * s[b];
      const float gate = sigmoid(100.0f * (1.0f - sigmoid(opacity) - 0.995f));
      float nz[3];
#pragma unroll
      for (int k = 0; k < 3; ++k) nz[k] = ((randn[3 * i + k] * gate) * hp.noise_lr) * hp.position_lr;
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        float shift = 0.0f;
#pragma unroll
        for (int b = 0; b < 3; ++b) {
          const float cov = (f[a][0] * f[b][0] + f[a][1] * f[b][1]) + f[a][2] * f[b][2];
          shift = b == 0 ? cov * nz[0] : shift + cov * nz[b];
        }
        mean[a] = mean[a] + shift;
      }
    }
    if (g.mean || kNoise) {
#pragma unroll
      for (int k = 0; k < 3; ++k) p.mean[3 * i + k] = mean[k];
    }
  }
  // Colour: this CTA's Gaussians own one contiguous run of color_per floats
  // each; the threads stride over it in 16-byte vectors (the run starts on a
  // multiple of 4 floats because kOptThreads is).
  if (!g.color) return;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kOptThreads;
  const int64_t last = first + kOptThreads < n ? first + kOptThreads : n;
  const int64_t c0 = first * color_per, c1 = last * color_per;
  const float ns = hp.neg_step_size[4], bs = hp.bias2_sqrt[4];
  int64_t e = c0 + 4 * static_cast<int64_t>(threadIdx.x);
  for (; e + 3 < c1; e += 4 * kOptThreads) {
    float4 pp = *reinterpret_cast<const float4*>(p.color + e);
    const float4 gg = *reinterpret_cast<const float4*>(g.color + e);
    float4 mm = *reinterpret_cast<const float4*>(m.color + e);
    float4 vv = *reinterpret_cast<const float4*>(v.color + e);
    pp.x = adam_one(pp.x, gg.x, mm.x, vv.x, ns, bs, c);
    pp.y = adam_one(pp.y, gg.y, mm.y, vv.y, ns, bs, c);
    pp.z = adam_one(pp.z, gg.z, mm.z, vv.z, ns, bs, c);
    pp.w = adam_one(pp.w, gg.w, mm.w, vv.w, ns, bs, c);
    *reinterpret_cast<float4*>(p.color + e) = pp;
    *reinterpret_cast<float4*>(m.color + e) = mm;
    *reinterpret_cast<float4*>(v.color + e) = vv;
  }
  for (; e < c1; ++e) {  // the ragged end of the last CTA's run
    float mk = m.color[e], vk = v.color[e];
    p.color[e] = adam_one(p.color[e], g.color[e], mk, vk, ns, bs, c);
    m.color[e] = mk;
    v.color[e] = vk;
  }
}

}  // namespace

int32_t launch_adam_step(int64_t n, int32_t num_sh, const gs_splat_arrays& p,
                         const gs_splat_arrays& g, const gs_splat_arrays& m,
                         const gs_splat_arrays& v, const gs_adam_params& hp, const float* randn,
                         cudaStream_t stream) {
  if (n == 0) return GS_OK;
  const unsigned blocks = ceil_div(n, kOptThreads);
  const int64_t color_per = 3 * static_cast<int64_t>(num_sh);
  if (randn)
    adam_step_kernel<true><<<blocks, kOptThreads, 0, stream>>>(n, color_per, p, g, m, v, hp,
                                                               randn);
  else
    adam_step_kernel<false><<<blocks, kOptThreads, 0, stream>>>(n, color_per, p, g, m, v, hp,
                                                                nullptr);
  return check_launch();
}

}  // namespace gs
