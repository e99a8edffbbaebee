// Projection (forward) and parameter gradients (backward), one thread per
// Gaussian.
//
// Forward follows _project_and_count_kernel (project.py:74-253) and backward
// _project_bwd_kernel (project_bwd.py:8-334) operation for operation in float32
// (the library builds with --fmad=false, so nothing is fused unless written as
// fmaf), which keeps tile bounds and counts bit-identical with the CPU oracle.
//
// Both kernels are HBM-bound: per Gaussian the forward reads 44 + 12K bytes of
// parameters (K = SH coefficients) and writes 64 bytes; the backward reads
// 44 + 12K + 16 + 36 + 4 bytes and writes 44 + 12K bytes. The SH block is the
// bulk (192 B at degree 3); each thread reads its own row with 16-byte
// vector loads when the row is 16-byte aligned (K = 4, 16), scalar otherwise.
#include "common.cuh"

namespace gs {
namespace {

// SH basis function k at unit direction (x, y, z) (project.py:22-61).
__device__ __forceinline__ float sh_basis(int k, float x, float y, float z, float xx, float yy,
                                          float zz) {
  switch (k) {
    case 0: return 0.28209479177387814f;
    case 1: return -0.4886025119029199f * y;
    case 2: return 0.4886025119029199f * z;
    case 3: return -0.4886025119029199f * x;
    case 4: return 1.0925484305920792f * x * y;
    case 5: return -1.0925484305920792f * y * z;
    case 6: return 0.31539156525252005f * (2.0f * zz - xx - yy);
    case 7: return -1.0925484305920792f * x * z;
    case 8: return 0.5462742152960396f * (xx - yy);
    case 9: return -0.5900435899266435f * y * (3.0f * xx - yy);
    case 10: return 2.890611442640554f * x * y * z;
    case 11: return -0.4570457994644658f * y * (4.0f * zz - xx - yy);
    case 12: return 0.3731763325901154f * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
    case 13: return -0.4570457994644658f * x * (4.0f * zz - xx - yy);
    case 14: return 1.445305721320277f * z * (xx - yy);
    case 15: return -0.5900435899266435f * x * (xx - 3.0f * yy);
    case 16: return 2.5033429417967046f * x * y * (xx - yy);
    case 17: return -1.7701307697799304f * y * z * (3.0f * xx - yy);
    case 18: return 0.9461746957575601f * x * y * (7.0f * zz - 1.0f);
    case 19: return -0.6690465435572892f * y * z * (7.0f * zz - 3.0f);
    case 20: return 0.10578554691520431f * (zz * (35.0f * zz - 30.0f) + 3.0f);
    case 21: return -0.6690465435572892f * x * z * (7.0f * zz - 3.0f);
    case 22: return 0.47308734787878004f * (xx - yy) * (7.0f * zz - 1.0f);
    case 23: return -1.7701307697799304f * x * z * (xx - 3.0f * yy);
    default: return 0.6258357354491761f * (xx * (xx - 3.0f * yy) - yy * (3.0f * xx - yy));
  }
}

// Loads the K x 3 SH coefficients of one Gaussian into registers.
template <int K>
__device__ __forceinline__ void load_sh(const float* __restrict__ row, float (&c)[K * 3]) {
  if constexpr ((K * 3) % 4 == 0 && (K * 12) % 16 == 0) {
    const float4* v = reinterpret_cast<const float4*>(row);
#pragma unroll
    for (int j = 0; j < K * 3 / 4; ++j) {
      float4 q = __ldg(v + j);
      c[4 * j] = q.x; c[4 * j + 1] = q.y; c[4 * j + 2] = q.z; c[4 * j + 3] = q.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < K * 3; ++j) c[j] = __ldg(row + j);
  }
}

struct Camera {
  float r00, r01, r02, r10, r11, r12, r20, r21, r22, tx, ty, tz;
};

constexpr int kMaxBatchViews = 16;

__device__ __forceinline__ Camera load_camera(const float* __restrict__ R,
                                              const float* __restrict__ t) {
  return Camera{__ldg(R), __ldg(R + 1), __ldg(R + 2), __ldg(R + 3), __ldg(R + 4), __ldg(R + 5),
                __ldg(R + 6), __ldg(R + 7), __ldg(R + 8), __ldg(t), __ldg(t + 1), __ldg(t + 2)};
}

// Batched projection (several cameras per launch) is built from two parts.
// They evaluate exactly the expressions of project_fwd_kernel below, so with
// no implicit multiply-add fusion every output is bit-identical to it; the
// single-view kernel keeps its own ordering, which holds fewer values live.
//
// The view-independent part of one Gaussian's projection: world mean,
// R(q) diag(exp(scale)) (project.py:144-156,177-199), opacity and the Gaussian
// mode's radius multiplier 2 sqrt(log(255 o)) (project.py:230-236).
struct GaussianTerms {
  float mx, my, mz;
  float a0x, a0y, a0z, a1x, a1y, a1z, a2x, a2y, a2z;
  float o, gaussian_extent;
};

__device__ __forceinline__ GaussianTerms gaussian_terms(int64_t i, const float* __restrict__ mean,
                                                        const float* __restrict__ rotation,
                                                        const float* __restrict__ scale,
                                                        const float* __restrict__ opacity) {
  GaussianTerms g;
  g.mx = __ldg(mean + 3 * i);
  g.my = __ldg(mean + 3 * i + 1);
  g.mz = __ldg(mean + 3 * i + 2);
  // project.py:144-156
  const float4 q4 = __ldg(reinterpret_cast<const float4*>(rotation) + i);
  float qw = q4.x, qx = q4.y, qy = q4.z, qz = q4.w;
  const float inverse_norm = det_rsqrt(qw * qw + qx * qx + qy * qy + qz * qz);
  qw = qw * inverse_norm; qx = qx * inverse_norm; qy = qy * inverse_norm; qz = qz * inverse_norm;
  // project.py:177-199
  const float sx = det_exp(__ldg(scale + 3 * i)), sy = det_exp(__ldg(scale + 3 * i + 1)),
              sz = det_exp(__ldg(scale + 3 * i + 2));
  g.a0x = (1.0f - 2.0f * (qy * qy + qz * qz)) * sx;
  g.a0y = (2.0f * (qx * qy + qw * qz)) * sx;
  g.a0z = (2.0f * (qx * qz - qw * qy)) * sx;
  g.a1x = (2.0f * (qx * qy - qw * qz)) * sy;
  g.a1y = (1.0f - 2.0f * (qx * qx + qz * qz)) * sy;
  g.a1z = (2.0f * (qy * qz + qw * qx)) * sy;
  g.a2x = (2.0f * (qx * qz + qw * qy)) * sz;
  g.a2y = (2.0f * (qy * qz - qw * qx)) * sz;
  g.a2z = (1.0f - 2.0f * (qx * qx + qy * qy)) * sz;
  // project.py:230-236
  g.o = det_sigmoid(__ldg(opacity + i));
  g.gaussian_extent = 2.0f * sqrtf(det_log(g.o * 255.0f));
  return g;
}

// The view-dependent part: camera transform, 2D covariance and conic, SH
// colour along the view direction, tile rectangle and count of Gaussian i
// for one camera (project.py:126-142,158-176,200-253). Output pointers are
// those of this view. The SH row is loaded where it is used, so its 3K
// registers are not live during the covariance (a batched caller's repeated
// loads of the row hit L1).
template <int K>
__device__ __forceinline__ void project_view(
    int64_t i, const GaussianTerms& g, const float* __restrict__ sh_row, const Camera& c,
    const gs_params& p, float* __restrict__ projected_mean, float* __restrict__ inverse_covariance,
    float* __restrict__ projected_color, float* __restrict__ projected_opacity,
    int4* __restrict__ bounds, int32_t* __restrict__ counts, float4* __restrict__ records) {
  const float mx = g.mx, my = g.my, mz = g.mz;
  // project.py:126-142
  const float camera_x = mx * c.r00 + my * c.r01 + mz * c.r02 + c.tx;
  const float camera_y = mx * c.r10 + my * c.r11 + mz * c.r12 + c.ty;
  const float camera_z = mx * c.r20 + my * c.r21 + mz * c.r22 + c.tz;
  const float depth = -camera_z;
  const float safe_z = depth > 0.0f ? fmaxf(1e-4f, depth) : fminf(-1e-4f, depth);
  const float pixel_x = p.fx * camera_x / safe_z + p.cx;
  const float pixel_y = -p.fy * camera_y / safe_z + p.cy;
  projected_mean[3 * i] = pixel_x;
  projected_mean[3 * i + 1] = pixel_y;
  projected_mean[3 * i + 2] = safe_z;
  // project.py:158-176
  const float cov_x = fminf(p.lim_x, fmaxf(-p.lim_x, camera_x / safe_z)) * safe_z;
  const float cov_y = fminf(p.lim_y, fmaxf(-p.lim_y, camera_y / safe_z)) * safe_z;
  const float inverse_z = 1.0f / safe_z;
  const float j00 = p.fx * inverse_z;
  const float j02 = p.fx * cov_x * inverse_z * inverse_z;
  const float j11 = -p.fy * inverse_z;
  const float j12 = -p.fy * cov_y * inverse_z * inverse_z;
  const float jc00 = j00 * c.r00 + j02 * c.r20, jc01 = j00 * c.r01 + j02 * c.r21,
              jc02 = j00 * c.r02 + j02 * c.r22;
  const float jc10 = j11 * c.r10 + j12 * c.r20, jc11 = j11 * c.r11 + j12 * c.r21,
              jc12 = j11 * c.r12 + j12 * c.r22;
  // project.py:200-218
  const float f00 = jc00 * g.a0x + jc01 * g.a0y + jc02 * g.a0z;
  const float f01 = jc00 * g.a1x + jc01 * g.a1y + jc02 * g.a1z;
  const float f02 = jc00 * g.a2x + jc01 * g.a2y + jc02 * g.a2z;
  const float f10 = jc10 * g.a0x + jc11 * g.a0y + jc12 * g.a0z;
  const float f11 = jc10 * g.a1x + jc11 * g.a1y + jc12 * g.a1z;
  const float f12 = jc10 * g.a2x + jc11 * g.a2y + jc12 * g.a2z;
  const float cov00 = f00 * f00 + f01 * f01 + f02 * f02 + 0.03f;
  const float cov01 = f00 * f10 + f01 * f11 + f02 * f12;
  const float cov11 = f10 * f10 + f11 * f11 + f12 * f12 + 0.03f;
  const float determinant = cov00 * cov11 - cov01 * cov01;
  const float conic_xy = -cov01 / determinant;
  const float4 conic = make_float4(cov11 / determinant, conic_xy, conic_xy, cov00 / determinant);
  reinterpret_cast<float4*>(inverse_covariance)[i] = conic;
  // project.py:221-228, _evaluate_sh (project.py:10-71)
  float dx = mx + c.r00 * c.tx + c.r10 * c.ty + c.r20 * c.tz;
  float dy = my + c.r01 * c.tx + c.r11 * c.ty + c.r21 * c.tz;
  float dz = mz + c.r02 * c.tx + c.r12 * c.ty + c.r22 * c.tz;
  const float direction_norm = det_rsqrt(dx * dx + dy * dy + dz * dz);
  dx = dx * direction_norm; dy = dy * direction_norm; dz = dz * direction_norm;
  const float xx = dx * dx, yy = dy * dy, zz = dz * dz;
  float coefficients[K * 3];
  load_sh<K>(sh_row, coefficients);
  float acc_r = 0.0f, acc_g = 0.0f, acc_b = 0.0f;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const float b = sh_basis(k, dx, dy, dz, xx, yy, zz);
    acc_r = fmaf(coefficients[3 * k], b, acc_r);
    acc_g = fmaf(coefficients[3 * k + 1], b, acc_g);
    acc_b = fmaf(coefficients[3 * k + 2], b, acc_b);
  }
  const float red = fmaxf(acc_r + 0.5f, 0.0f), green = fmaxf(acc_g + 0.5f, 0.0f),
              blue = fmaxf(acc_b + 0.5f, 0.0f);
  projected_color[3 * i] = red;
  projected_color[3 * i + 1] = green;
  projected_color[3 * i + 2] = blue;
  // project.py:230-253
  projected_opacity[i] = g.o;
  const float radius_extent = p.gaussian_mode ? g.gaussian_extent : p.extent;
  const float radius_x = radius_extent * sqrtf(cov00);
  const float radius_y = radius_extent * sqrtf(cov11);
  const float ts = static_cast<float>(p.tile_size);
  const float tiles_w = static_cast<float>(p.width / p.tile_size);
  const float tiles_h = static_cast<float>(p.height / p.tile_size);
  // tl.clamp (max then min); a NaN radius clamps to 0.
  const float tmin_x = fminf(fmaxf(floorf((pixel_x - radius_x) / ts), 0.0f), tiles_w);
  const float tmin_y = fminf(fmaxf(floorf((pixel_y - radius_y) / ts), 0.0f), tiles_h);
  const float tmax_x = fminf(fmaxf(floorf((pixel_x + radius_x) / ts) + 1.0f, 0.0f), tiles_w);
  const float tmax_y = fminf(fmaxf(floorf((pixel_y + radius_y) / ts) + 1.0f, 0.0f), tiles_h);
  bounds[i] = make_int4(static_cast<int>(tmin_x), static_cast<int>(tmax_x),
                        static_cast<int>(tmin_y), static_cast<int>(tmax_y));
  const float count = (tmax_x - tmin_x) * (tmax_y - tmin_y);
  const int32_t visible_count =
      (safe_z > p.near_plane && safe_z < p.far_plane) ? static_cast<int32_t>(count) : 0;
  counts[i] = visible_count;
  // the compositors' staged form; Gaussians in no tile are never staged
  if (records != nullptr && visible_count > 0)
    store_record(records, i, make_record(static_cast<int32_t>(i), pixel_x, pixel_y, conic, g.o,
                                         red, green, blue, p));
}

// A CTA's Gaussian rows as project_fwd_kernel stages them in shared memory.
constexpr int kProjectThreads = 128;
template <int K>
struct FwdRows {
  float sh[kProjectThreads * ShPitch<K>::value];
  float4 rotation[kProjectThreads];
  float mean[kProjectThreads * 3];
  float scale[kProjectThreads * 3];
  float opacity[kProjectThreads];
};

// One thread per Gaussian, 128 per CTA. The CTA's rows of the five parameter
// arrays are contiguous ranges, so they are staged into shared memory with
// coalesced asynchronous copies issued all at once -- about 30 KB per CTA
// in flight without holding a register, which a thread's own dependent loads
// could not keep up -- the geometry's rows first (their own copy group, so
// the covariance starts while the SH rows are still arriving), then the SH
// rows.
template <int K>
__global__ void __launch_bounds__(kProjectThreads) project_fwd_kernel(
    int64_t n, const float* __restrict__ mean, const float* __restrict__ rotation,
    const float* __restrict__ scale, const float* __restrict__ opacity,
    const float* __restrict__ color, const float* __restrict__ camera_rotation,
    const float* __restrict__ camera_translation, const gs_params p,
    float* __restrict__ projected_mean, float* __restrict__ inverse_covariance,
    float* __restrict__ projected_color, float* __restrict__ projected_opacity,
    int4* __restrict__ bounds, int32_t* __restrict__ counts, float4* __restrict__ records) {
  chain_wait();
  constexpr int kPitch = ShPitch<K>::value;
  __shared__ __align__(16) FwdRows<K> s;
  const int tid = threadIdx.x;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kProjectThreads;
  const int rows = n - first < kProjectThreads ? static_cast<int>(n - first) : kProjectThreads;
  stage_rows_async<3, 3, kProjectThreads>(s.mean, mean + 3 * first, rows, tid);
  stage_rows_async<4, 4, kProjectThreads>(&s.rotation[0].x, rotation + 4 * first, rows, tid);
  stage_rows_async<3, 3, kProjectThreads>(s.scale, scale + 3 * first, rows, tid);
  stage_rows_async<1, 1, kProjectThreads>(s.opacity, opacity + first, rows, tid);
  cp_async_commit();
  stage_rows_async<3 * K, kPitch, kProjectThreads>(s.sh, color + first * (3 * K), rows, tid);
  cp_async_commit();
  const Camera c = load_camera(camera_rotation, camera_translation);
  cp_async_wait_all_but_last();
  __syncthreads();
  const bool live = tid < rows;  // every thread stays for the second barrier
  const int64_t i = first + tid;
  const float mx = s.mean[3 * tid], my = s.mean[3 * tid + 1], mz = s.mean[3 * tid + 2];
  // project.py:126-142
  const float camera_x = mx * c.r00 + my * c.r01 + mz * c.r02 + c.tx;
  const float camera_y = mx * c.r10 + my * c.r11 + mz * c.r12 + c.ty;
  const float camera_z = mx * c.r20 + my * c.r21 + mz * c.r22 + c.tz;
  const float depth = -camera_z;
  const float safe_z = depth > 0.0f ? fmaxf(1e-4f, depth) : fminf(-1e-4f, depth);
  const float pixel_x = p.fx * camera_x / safe_z + p.cx;
  const float pixel_y = -p.fy * camera_y / safe_z + p.cy;
  if (live) {
    projected_mean[3 * i] = pixel_x;
    projected_mean[3 * i + 1] = pixel_y;
    projected_mean[3 * i + 2] = safe_z;
  }
  // project.py:144-156
  const float4 q4 = s.rotation[tid];
  float qw = q4.x, qx = q4.y, qy = q4.z, qz = q4.w;
  const float inverse_norm = det_rsqrt(qw * qw + qx * qx + qy * qy + qz * qz);
  qw = qw * inverse_norm; qx = qx * inverse_norm; qy = qy * inverse_norm; qz = qz * inverse_norm;
  // project.py:158-176
  const float cov_x = fminf(p.lim_x, fmaxf(-p.lim_x, camera_x / safe_z)) * safe_z;
  const float cov_y = fminf(p.lim_y, fmaxf(-p.lim_y, camera_y / safe_z)) * safe_z;
  const float inverse_z = 1.0f / safe_z;
  const float j00 = p.fx * inverse_z;
  const float j02 = p.fx * cov_x * inverse_z * inverse_z;
  const float j11 = -p.fy * inverse_z;
  const float j12 = -p.fy * cov_y * inverse_z * inverse_z;
  const float jc00 = j00 * c.r00 + j02 * c.r20, jc01 = j00 * c.r01 + j02 * c.r21,
              jc02 = j00 * c.r02 + j02 * c.r22;
  const float jc10 = j11 * c.r10 + j12 * c.r20, jc11 = j11 * c.r11 + j12 * c.r21,
              jc12 = j11 * c.r12 + j12 * c.r22;
  // project.py:177-218
  const float sx = det_exp(s.scale[3 * tid]), sy = det_exp(s.scale[3 * tid + 1]),
              sz = det_exp(s.scale[3 * tid + 2]);
  const float a0x = (1.0f - 2.0f * (qy * qy + qz * qz)) * sx;
  const float a0y = (2.0f * (qx * qy + qw * qz)) * sx;
  const float a0z = (2.0f * (qx * qz - qw * qy)) * sx;
  const float a1x = (2.0f * (qx * qy - qw * qz)) * sy;
  const float a1y = (1.0f - 2.0f * (qx * qx + qz * qz)) * sy;
  const float a1z = (2.0f * (qy * qz + qw * qx)) * sy;
  const float a2x = (2.0f * (qx * qz + qw * qy)) * sz;
  const float a2y = (2.0f * (qy * qz - qw * qx)) * sz;
  const float a2z = (1.0f - 2.0f * (qx * qx + qy * qy)) * sz;
  const float f00 = jc00 * a0x + jc01 * a0y + jc02 * a0z;
  const float f01 = jc00 * a1x + jc01 * a1y + jc02 * a1z;
  const float f02 = jc00 * a2x + jc01 * a2y + jc02 * a2z;
  const float f10 = jc10 * a0x + jc11 * a0y + jc12 * a0z;
  const float f11 = jc10 * a1x + jc11 * a1y + jc12 * a1z;
  const float f12 = jc10 * a2x + jc11 * a2y + jc12 * a2z;
  const float cov00 = f00 * f00 + f01 * f01 + f02 * f02 + 0.03f;
  const float cov01 = f00 * f10 + f01 * f11 + f02 * f12;
  const float cov11 = f10 * f10 + f11 * f11 + f12 * f12 + 0.03f;
  const float determinant = cov00 * cov11 - cov01 * cov01;
  const float conic_xy = -cov01 / determinant;
  const float4 conic = make_float4(cov11 / determinant, conic_xy, conic_xy, cov00 / determinant);
  if (live) reinterpret_cast<float4*>(inverse_covariance)[i] = conic;
  // project.py:230-253
  const float o = det_sigmoid(s.opacity[tid]);
  const float radius_extent = p.gaussian_mode ? 2.0f * sqrtf(det_log(o * 255.0f)) : p.extent;
  const float radius_x = radius_extent * sqrtf(cov00);
  const float radius_y = radius_extent * sqrtf(cov11);
  const float ts = static_cast<float>(p.tile_size);
  const float tiles_w = static_cast<float>(p.width / p.tile_size);
  const float tiles_h = static_cast<float>(p.height / p.tile_size);
  // tl.clamp (max then min); a NaN radius clamps to 0.
  const float tmin_x = fminf(fmaxf(floorf((pixel_x - radius_x) / ts), 0.0f), tiles_w);
  const float tmin_y = fminf(fmaxf(floorf((pixel_y - radius_y) / ts), 0.0f), tiles_h);
  const float tmax_x = fminf(fmaxf(floorf((pixel_x + radius_x) / ts) + 1.0f, 0.0f), tiles_w);
  const float tmax_y = fminf(fmaxf(floorf((pixel_y + radius_y) / ts) + 1.0f, 0.0f), tiles_h);
  const float count = (tmax_x - tmin_x) * (tmax_y - tmin_y);
  const int32_t visible_count =
      (safe_z > p.near_plane && safe_z < p.far_plane) ? static_cast<int32_t>(count) : 0;
  if (live) {
    projected_opacity[i] = o;
    bounds[i] = make_int4(static_cast<int>(tmin_x), static_cast<int>(tmax_x),
                          static_cast<int>(tmin_y), static_cast<int>(tmax_y));
    counts[i] = visible_count;
  }
  // project.py:221-228, _evaluate_sh (project.py:10-71)
  float dx = mx + c.r00 * c.tx + c.r10 * c.ty + c.r20 * c.tz;
  float dy = my + c.r01 * c.tx + c.r11 * c.ty + c.r21 * c.tz;
  float dz = mz + c.r02 * c.tx + c.r12 * c.ty + c.r22 * c.tz;
  const float direction_norm = det_rsqrt(dx * dx + dy * dy + dz * dz);
  dx = dx * direction_norm; dy = dy * direction_norm; dz = dz * direction_norm;
  const float xx = dx * dx, yy = dy * dy, zz = dz * dz;
  cp_async_wait_all();
  __syncthreads();
  if (!live) return;
  float coefficients[K * 3];
  load_sh_shared<K>(s.sh + tid * kPitch, coefficients);
  float acc_r = 0.0f, acc_g = 0.0f, acc_b = 0.0f;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const float b = sh_basis(k, dx, dy, dz, xx, yy, zz);
    acc_r = fmaf(coefficients[3 * k], b, acc_r);
    acc_g = fmaf(coefficients[3 * k + 1], b, acc_g);
    acc_b = fmaf(coefficients[3 * k + 2], b, acc_b);
  }
  const float red = fmaxf(acc_r + 0.5f, 0.0f), green = fmaxf(acc_g + 0.5f, 0.0f),
              blue = fmaxf(acc_b + 0.5f, 0.0f);
  projected_color[3 * i] = red;
  projected_color[3 * i + 1] = green;
  projected_color[3 * i + 2] = blue;
  // the compositors' staged form; Gaussians in no tile are never staged
  if (records != nullptr && visible_count > 0)
    store_record(records, i, make_record(static_cast<int32_t>(i), pixel_x, pixel_y, conic, o,
                                         red, green, blue, p));
}

// One view's conic as the forward computes it (project.py:126-142,158-218):
// the expressions of project_fwd_kernel, so the same bits as the conic the
// forward wrote.
__device__ __forceinline__ float4 view_conic(const GaussianTerms& g, const Camera& c,
                                             const gs_params& p) {
  const float camera_x = g.mx * c.r00 + g.my * c.r01 + g.mz * c.r02 + c.tx;
  const float camera_y = g.mx * c.r10 + g.my * c.r11 + g.mz * c.r12 + c.ty;
  const float camera_z = g.mx * c.r20 + g.my * c.r21 + g.mz * c.r22 + c.tz;
  const float depth = -camera_z;
  const float safe_z = depth > 0.0f ? fmaxf(1e-4f, depth) : fminf(-1e-4f, depth);
  const float cov_x = fminf(p.lim_x, fmaxf(-p.lim_x, camera_x / safe_z)) * safe_z;
  const float cov_y = fminf(p.lim_y, fmaxf(-p.lim_y, camera_y / safe_z)) * safe_z;
  const float inverse_z = 1.0f / safe_z;
  const float j00 = p.fx * inverse_z;
  const float j02 = p.fx * cov_x * inverse_z * inverse_z;
  const float j11 = -p.fy * inverse_z;
  const float j12 = -p.fy * cov_y * inverse_z * inverse_z;
  const float jc00 = j00 * c.r00 + j02 * c.r20, jc01 = j00 * c.r01 + j02 * c.r21,
              jc02 = j00 * c.r02 + j02 * c.r22;
  const float jc10 = j11 * c.r10 + j12 * c.r20, jc11 = j11 * c.r11 + j12 * c.r21,
              jc12 = j11 * c.r12 + j12 * c.r22;
  const float f00 = jc00 * g.a0x + jc01 * g.a0y + jc02 * g.a0z;
  const float f01 = jc00 * g.a1x + jc01 * g.a1y + jc02 * g.a1z;
  const float f02 = jc00 * g.a2x + jc01 * g.a2y + jc02 * g.a2z;
  const float f10 = jc10 * g.a0x + jc11 * g.a0y + jc12 * g.a0z;
  const float f11 = jc10 * g.a1x + jc11 * g.a1y + jc12 * g.a1z;
  const float f12 = jc10 * g.a2x + jc11 * g.a2y + jc12 * g.a2z;
  const float cov00 = f00 * f00 + f01 * f01 + f02 * f02 + 0.03f;
  const float cov01 = f00 * f10 + f01 * f11 + f02 * f12;
  const float cov11 = f10 * f10 + f11 * f11 + f12 * f12 + 0.03f;
  const float determinant = cov00 * cov11 - cov01 * cov01;
  const float conic_xy = -cov01 / determinant;
  return make_float4(cov11 / determinant, conic_xy, conic_xy, cov00 / determinant);
}

// Up to kMaxBatchViews cameras of one batched projection, passed by value.
struct ViewBatch {
  gs_params p[kMaxBatchViews];
  Camera c[kMaxBatchViews];
  int views;
};

// Batched projection: each thread reads its Gaussian's parameters once,
// computes the view-independent terms once, and projects into every view of
// the batch (its SH row comes from HBM once; the later views' loads hit L1).
// View b writes at offset b * n of each output.
template <int K>
__global__ void __launch_bounds__(256) project_fwd_batch_kernel(
    int64_t n, const float* __restrict__ mean, const float* __restrict__ rotation,
    const float* __restrict__ scale, const float* __restrict__ opacity,
    const float* __restrict__ color, const __grid_constant__ ViewBatch batch,
    float* __restrict__ projected_mean, float* __restrict__ inverse_covariance,
    float* __restrict__ projected_color, float* __restrict__ projected_opacity,
    int4* __restrict__ bounds, int32_t* __restrict__ counts, float4* __restrict__ records) {
  chain_wait();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (threadIdx.x == 0) {
    const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x;
    prefetch_gaussian_rows(first, n - first < blockDim.x ? n - first : blockDim.x, K, mean,
                           rotation, scale, opacity, color);
  }
  const GaussianTerms g = gaussian_terms(i, mean, rotation, scale, opacity);
  for (int b = 0; b < batch.views; ++b) {
    const int64_t o = static_cast<int64_t>(b) * n;
    project_view<K>(i, g, color + i * (K * 3), batch.c[b], batch.p[b], projected_mean + 3 * o,
                    inverse_covariance + 4 * o, projected_color + 3 * o, projected_opacity + o,
                    bounds + o, counts + o, records ? records + 4 * o : nullptr);
  }
}

// The view-independent terms of one Gaussian's projection backward
// (project_bwd.py:62-94,320-334): its mean, normalised quaternion and the
// reciprocal of the quaternion's norm, activated scales and opacity. A
// backward over several views computes them once.
struct BwdTerms {
  float mx, my, mz;
  float qw, qx, qy, qz, inverse_qnorm;
  float sx, sy, sz, po;
};

__device__ __forceinline__ BwdTerms bwd_terms_of(float mx, float my, float mz, float4 q4,
                                                 float log_sx, float log_sy, float log_sz,
                                                 float logit) {
  BwdTerms b;
  b.mx = mx;
  b.my = my;
  b.mz = mz;
  const float qnorm = sqrtf(q4.x * q4.x + q4.y * q4.y + q4.z * q4.z + q4.w * q4.w);
  b.inverse_qnorm = 1.0f / qnorm;
  b.qw = q4.x * b.inverse_qnorm;
  b.qx = q4.y * b.inverse_qnorm;
  b.qy = q4.z * b.inverse_qnorm;
  b.qz = q4.w * b.inverse_qnorm;
  b.sx = det_exp(log_sx);
  b.sy = det_exp(log_sy);
  b.sz = det_exp(log_sz);
  b.po = det_sigmoid(logit);
  return b;
}

__device__ __forceinline__ BwdTerms bwd_terms(int64_t i, const float* __restrict__ mean,
                                              const float* __restrict__ rotation,
                                              const float* __restrict__ scale,
                                              const float* __restrict__ opacity) {
  return bwd_terms_of(__ldg(mean + 3 * i), __ldg(mean + 3 * i + 1), __ldg(mean + 3 * i + 2),
                      __ldg(reinterpret_cast<const float4*>(rotation) + i),
                      __ldg(scale + 3 * i), __ldg(scale + 3 * i + 1), __ldg(scale + 3 * i + 2),
                      __ldg(opacity + i));
}

// Gradients of one Gaussian's parameters from its screen-space gradient in
// one view (project_bwd.py:8-334), handed to `sink`: sink.color(g[3K]) with
// the SH coefficient gradients, then sink.rest(mean xyz, rotation, scale xyz,
// opacity). `b` holds the Gaussian's view-independent terms, `sh_row` its
// 3K SH coefficients (global memory, or a staged shared-memory row with
// kShShared), `inv` is the view's conic as the forward computed it and `gp`
// the view's 9-float screen-space gradient of the Gaussian.
// How a view's screen-space gradient is read: through the read-only cache
// (written on this GPU by an earlier kernel), or at L2 only (written by
// another GPU, behind a flag), or from a row staged in shared memory.
struct LoadReadOnly {
  static __device__ __forceinline__ float get(const float* p) { return __ldg(p); }
};
struct LoadShared {
  static __device__ __forceinline__ float get(const float* p) { return *p; }
};
struct LoadPeer {
  static __device__ __forceinline__ float get(const float* p) { return __ldcg(p); }
};

template <int K, class Sink, class Load = LoadReadOnly, bool kShShared = false>
__device__ __forceinline__ void project_bwd_view(
    bool visible, const Camera& c, const gs_params& p, const BwdTerms& b,
    const float* __restrict__ sh_row, float4 inv, const float* __restrict__ gp, Sink& sink) {
  // SH coefficients with a gradient: all K. The reference's backward stops at 16
  // (project_bwd.py:33); degree 4 is carried through here.
  constexpr int KB = K;
  constexpr int KA = K > 16 ? 25 : 16;  // basis / derivative slots
  const float fx = p.fx, fy = p.fy, lim_x = p.bwd_lim_x, lim_y = p.bwd_lim_y;
  const float mx = b.mx, my = b.my, mz = b.mz;
  // project_bwd.py:62-94
  const float camera_x = mx * c.r00 + my * c.r01 + mz * c.r02 + c.tx;
  const float camera_y = mx * c.r10 + my * c.r11 + mz * c.r12 + c.ty;
  const float camera_z = mx * c.r20 + my * c.r21 + mz * c.r22 + c.tz;
  const float qw = b.qw, qx = b.qx, qy = b.qy, qz = b.qz;
  const float r00 = 1.0f - 2.0f * (qy * qy + qz * qz), r01 = 2.0f * (qx * qy - qw * qz),
              r02 = 2.0f * (qx * qz + qw * qy);
  const float r10 = 2.0f * (qx * qy + qw * qz), r11 = 1.0f - 2.0f * (qx * qx + qz * qz),
              r12 = 2.0f * (qy * qz - qw * qx);
  const float r20 = 2.0f * (qx * qz - qw * qy), r21 = 2.0f * (qy * qz + qw * qx),
              r22 = 1.0f - 2.0f * (qx * qx + qy * qy);
  const float depth = -camera_z;
  const float inverse_z = 1.0f / depth;
  const float normalized_x = camera_x * inverse_z, normalized_y = camera_y * inverse_z;
  const float x_grad_mul = (normalized_x >= -lim_x && normalized_x <= lim_x) ? 1.0f : 0.0f;
  const float y_grad_mul = (normalized_y >= -lim_y && normalized_y <= lim_y) ? 1.0f : 0.0f;
  const float covariance_x = fminf(lim_x, fmaxf(-lim_x, normalized_x)) * depth;
  const float covariance_y = fminf(lim_y, fmaxf(-lim_y, normalized_y)) * depth;
  const float j00 = fx * inverse_z, j02 = fx * covariance_x * inverse_z * inverse_z;
  const float j11 = -fy * inverse_z, j12 = -fy * covariance_y * inverse_z * inverse_z;
  // project_bwd.py:96-114
  const float jc00 = j00 * c.r00 + j02 * c.r20, jc01 = j00 * c.r01 + j02 * c.r21,
              jc02 = j00 * c.r02 + j02 * c.r22;
  const float jc10 = j11 * c.r10 + j12 * c.r20, jc11 = j11 * c.r11 + j12 * c.r21,
              jc12 = j11 * c.r12 + j12 * c.r22;
  const float sx = b.sx, sy = b.sy, sz = b.sz;
  const float m0x = jc00 * r00 + jc01 * r10 + jc02 * r20, m0y = jc00 * r01 + jc01 * r11 + jc02 * r21,
              m0z = jc00 * r02 + jc01 * r12 + jc02 * r22;
  const float m1x = jc10 * r00 + jc11 * r10 + jc12 * r20, m1y = jc10 * r01 + jc11 * r11 + jc12 * r21,
              m1z = jc10 * r02 + jc11 * r12 + jc12 * r22;
  const float a00 = m0x * sx, a01 = m0y * sy, a02 = m0z * sz;
  const float a10 = m1x * sx, a11 = m1y * sy, a12 = m1z * sz;
  // project_bwd.py:116-152
  const float inv00 = inv.x, inv01 = inv.y, inv10 = inv01, inv11 = inv.w;
  const float gi00 = Load::get(gp + 2), gi01 = Load::get(gp + 3), gi10 = gi01,
              gi11 = Load::get(gp + 4);
  const float h00 = inv00 * gi00 + inv10 * gi10, h01 = inv00 * gi01 + inv10 * gi11;
  const float h10 = inv01 * gi00 + inv11 * gi10, h11 = inv01 * gi01 + inv11 * gi11;
  const float gcov00 = -(h00 * inv00 + h01 * inv10), gcov01 = -(h00 * inv01 + h01 * inv11);
  const float gcov10 = -(h10 * inv00 + h11 * inv10), gcov11 = -(h10 * inv01 + h11 * inv11);
  const float sym01 = gcov01 + gcov10;
  const float ga00 = 2.0f * gcov00 * a00 + sym01 * a10, ga01 = 2.0f * gcov00 * a01 + sym01 * a11,
              ga02 = 2.0f * gcov00 * a02 + sym01 * a12;
  const float ga10 = sym01 * a00 + 2.0f * gcov11 * a10, ga11 = sym01 * a01 + 2.0f * gcov11 * a11,
              ga12 = sym01 * a02 + 2.0f * gcov11 * a12;
  const float gb00 = ga00 * sx, gb01 = ga01 * sy, gb02 = ga02 * sz;
  const float gb10 = ga10 * sx, gb11 = ga11 * sy, gb12 = ga12 * sz;
  const float grad_sx = ga00 * m0x + ga10 * m1x;
  const float grad_sy = ga01 * m0y + ga11 * m1y;
  const float grad_sz = ga02 * m0z + ga12 * m1z;
  // project_bwd.py:154-189
  const float gr00 = jc00 * gb00 + jc10 * gb10, gr01 = jc00 * gb01 + jc10 * gb11,
              gr02 = jc00 * gb02 + jc10 * gb12;
  const float gr10 = jc01 * gb00 + jc11 * gb10, gr11 = jc01 * gb01 + jc11 * gb11,
              gr12 = jc01 * gb02 + jc11 * gb12;
  const float gr20 = jc02 * gb00 + jc12 * gb10, gr21 = jc02 * gb01 + jc12 * gb11,
              gr22 = jc02 * gb02 + jc12 * gb12;
  float gqw = 2.0f * qz * (gr10 - gr01) + 2.0f * qy * (gr02 - gr20) + 2.0f * qx * (gr21 - gr12);
  float gqx = 2.0f * qy * (gr01 + gr10) + 2.0f * qz * (gr02 + gr20) + 2.0f * qw * (gr21 - gr12) -
              4.0f * qx * (gr11 + gr22);
  float gqy = 2.0f * qx * (gr01 + gr10) + 2.0f * qw * (gr02 - gr20) + 2.0f * qz * (gr12 + gr21) -
              4.0f * qy * (gr00 + gr22);
  float gqz = 2.0f * qw * (gr10 - gr01) + 2.0f * qx * (gr02 + gr20) + 2.0f * qy * (gr12 + gr21) -
              4.0f * qz * (gr00 + gr11);
  const float dot_q = qw * gqw + qx * gqx + qy * gqy + qz * gqz;
  const float gq_scale = b.inverse_qnorm;  // 1 / |q|
  gqw = (gqw - qw * dot_q) * gq_scale;
  gqx = (gqx - qx * dot_q) * gq_scale;
  gqy = (gqy - qy * dot_q) * gq_scale;
  gqz = (gqz - qz * dot_q) * gq_scale;
  // project_bwd.py:191-226
  const float gpx = Load::get(gp), gpy = Load::get(gp + 1);
  float gux = gpx * j00 + gpx * 0.0f;
  float guy = gpy * j11;
  float guz = -0.0f + gpx * j02 + gpy * j12;
  const float mr0 = c.r00 * r00 + c.r01 * r10 + c.r02 * r20,
              mr1 = c.r00 * r01 + c.r01 * r11 + c.r02 * r21,
              mr2 = c.r00 * r02 + c.r01 * r12 + c.r02 * r22;
  const float nr0 = c.r10 * r00 + c.r11 * r10 + c.r12 * r20,
              nr1 = c.r10 * r01 + c.r11 * r11 + c.r12 * r21,
              nr2 = c.r10 * r02 + c.r11 * r12 + c.r12 * r22;
  const float kr0 = c.r20 * r00 + c.r21 * r10 + c.r22 * r20,
              kr1 = c.r20 * r01 + c.r21 * r11 + c.r22 * r21,
              kr2 = c.r20 * r02 + c.r21 * r12 + c.r22 * r22;
  const float gj_j00 = gb00 * mr0 + gb01 * mr1 + gb02 * mr2;
  const float gj_j02 = gb00 * kr0 + gb01 * kr1 + gb02 * kr2;
  const float gj_j11 = gb10 * nr0 + gb11 * nr1 + gb12 * nr2;
  const float gj_j12 = gb10 * kr0 + gb11 * kr1 + gb12 * kr2;
  gux += x_grad_mul * gj_j02 * (fx * inverse_z * inverse_z);
  guy += y_grad_mul * gj_j12 * (-fy * inverse_z * inverse_z);
  const float inverse_z3 = inverse_z * inverse_z * inverse_z;
  guz += gj_j00 * (fx * inverse_z * inverse_z) + gj_j02 * 2.0f * fx * covariance_x * inverse_z3;
  guz += gj_j11 * (-fy * inverse_z * inverse_z) - gj_j12 * 2.0f * fy * covariance_y * inverse_z3;
  float gmx = gux * c.r00 + guy * c.r10 + guz * c.r20;
  float gmy = gux * c.r01 + guy * c.r11 + guz * c.r21;
  float gmz = gux * c.r02 + guy * c.r12 + guz * c.r22;
  // project_bwd.py:228-318: SH VJP for coefficients 0..15 and the view
  // direction's contribution to the mean; degree 4 (coefficients 16..24)
  // differentiates the forward basis (project.py:51-61) the same way.
  const float ddx = mx + c.r00 * c.tx + c.r10 * c.ty + c.r20 * c.tz;
  const float ddy = my + c.r01 * c.tx + c.r11 * c.ty + c.r21 * c.tz;
  const float ddz = mz + c.r02 * c.tx + c.r12 * c.ty + c.r22 * c.tz;
  const float norm = sqrtf(ddx * ddx + ddy * ddy + ddz * ddz);
  const float x = ddx / norm, y = ddy / norm, z = ddz / norm;
  const float xx = x * x, yy = y * y, zz = z * z;
  float basis[KA], dbx[KA], dby[KA], dbz[KA];
#pragma unroll
  for (int k = 0; k < KA; ++k) { dbx[k] = 0.0f; dby[k] = 0.0f; dbz[k] = 0.0f; }
  basis[0] = 0.28209479177387814f;
  basis[1] = -0.4886025119029199f * y;
  basis[2] = 0.4886025119029199f * z;
  basis[3] = -0.4886025119029199f * x;
  basis[4] = 1.0925484305920792f * x * y;
  basis[5] = -1.0925484305920792f * y * z;
  basis[6] = 0.31539156525252005f * (2.0f * zz - xx - yy);
  basis[7] = -1.0925484305920792f * x * z;
  basis[8] = 0.5462742152960396f * (xx - yy);
  basis[9] = -0.5900435899266435f * y * (3.0f * xx - yy);
  basis[10] = 2.890611442640554f * x * y * z;
  basis[11] = -0.4570457994644655f * y * (4.0f * zz - xx - yy);
  basis[12] = 0.3731763325901154f * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
  basis[13] = -0.4570457994644655f * x * (4.0f * zz - xx - yy);
  basis[14] = 1.445305721320277f * z * (xx - yy);
  basis[15] = -0.5900435899266435f * x * (xx - 3.0f * yy);
  dbx[3] = -0.4886025119029199f;
  dby[1] = -0.4886025119029199f;
  dbz[2] = 0.4886025119029199f;
  dbx[4] = 1.0925484305920792f * y;
  dby[4] = 1.0925484305920792f * x;
  dby[5] = -1.0925484305920792f * z;
  dbz[5] = -1.0925484305920792f * y;
  dbx[6] = -0.6307831301050401f * x;
  dby[6] = -0.6307831301050401f * y;
  dbz[6] = 1.2615662610100802f * z;
  dbx[7] = -1.0925484305920792f * z;
  dbz[7] = -1.0925484305920792f * x;
  dbx[8] = 1.0925484305920792f * x;
  dby[8] = -1.0925484305920792f * y;
  dbx[9] = -3.540261539559861f * x * y;
  dby[9] = -1.7701307697799305f * (xx - yy);
  dbx[10] = 2.890611442640554f * y * z;
  dby[10] = 2.890611442640554f * x * z;
  dbz[10] = 2.890611442640554f * x * y;
  dbx[11] = 0.914091599852931f * x * y;
  dby[11] = -0.4570457994644655f * (4.0f * zz - xx - 3.0f * yy);
  dbz[11] = -3.656366399411724f * y * z;
  dbx[12] = -2.2390579955366924f * x * z;
  dby[12] = -2.2390579955366924f * y * z;
  dbz[12] = 0.3731763325901154f * (6.0f * zz - 3.0f * xx - 3.0f * yy);
  dbx[13] = -0.4570457994644655f * (4.0f * zz - 3.0f * xx - yy);
  dby[13] = 0.914091599852931f * x * y;
  dbz[13] = -3.656366399411724f * x * z;
  dbx[14] = 2.890611442640554f * x * z;
  dby[14] = -2.890611442640554f * y * z;
  dbz[14] = 1.445305721320277f * (xx - yy);
  dbx[15] = -1.7701307697799305f * (xx - yy);
  dby[15] = 3.540261539559861f * x * y;
  if constexpr (K > 16) {
    basis[16] = 2.5033429417967046f * x * y * (xx - yy);
    basis[17] = -1.7701307697799304f * y * z * (3.0f * xx - yy);
    basis[18] = 0.9461746957575601f * x * y * (7.0f * zz - 1.0f);
    basis[19] = -0.6690465435572892f * y * z * (7.0f * zz - 3.0f);
    basis[20] = 0.10578554691520431f * (zz * (35.0f * zz - 30.0f) + 3.0f);
    basis[21] = -0.6690465435572892f * x * z * (7.0f * zz - 3.0f);
    basis[22] = 0.47308734787878004f * (xx - yy) * (7.0f * zz - 1.0f);
    basis[23] = -1.7701307697799304f * x * z * (xx - 3.0f * yy);
    basis[24] = 0.6258357354491761f * (xx * (xx - 3.0f * yy) - yy * (3.0f * xx - yy));
    dbx[16] = 2.5033429417967046f * y * (3.0f * xx - yy);
    dby[16] = 2.5033429417967046f * x * (xx - 3.0f * yy);
    dbx[17] = -10.620784618679583f * x * y * z;
    dby[17] = -5.310392309339791f * z * (xx - yy);
    dbz[17] = -1.7701307697799304f * y * (3.0f * xx - yy);
    dbx[18] = 0.9461746957575601f * y * (7.0f * zz - 1.0f);
    dby[18] = 0.9461746957575601f * x * (7.0f * zz - 1.0f);
    dbz[18] = 13.246445740605841f * x * y * z;
    dby[19] = -0.6690465435572892f * z * (7.0f * zz - 3.0f);
    dbz[19] = -0.6690465435572892f * y * (21.0f * zz - 3.0f);
    dbz[20] = 0.10578554691520431f * z * (140.0f * zz - 60.0f);
    dbx[21] = -0.6690465435572892f * z * (7.0f * zz - 3.0f);
    dbz[21] = -0.6690465435572892f * x * (21.0f * zz - 3.0f);
    dbx[22] = 0.9461746957575601f * x * (7.0f * zz - 1.0f);
    dby[22] = -0.9461746957575601f * y * (7.0f * zz - 1.0f);
    dbz[22] = 6.623222870302921f * z * (xx - yy);
    dbx[23] = -5.310392309339791f * z * (xx - yy);
    dby[23] = 10.620784618679583f * x * y * z;
    dbz[23] = -1.7701307697799304f * x * (xx - 3.0f * yy);
    dbx[24] = 2.5033429417967046f * x * (xx - 3.0f * yy);
    dby[24] = 2.5033429417967046f * y * (yy - 3.0f * xx);
  }
  float coefficients[K * 3];
  if constexpr (kShShared)
    load_sh_shared<K>(sh_row, coefficients);
  else
    load_sh<K>(sh_row, coefficients);
  float gc3[3];
  float gdx = 0.0f, gdy = 0.0f, gdz = 0.0f;
#pragma unroll
  for (int ch = 0; ch < 3; ++ch) {
    float raw = 0.0f, sdx = 0.0f, sdy = 0.0f, sdz = 0.0f;
#pragma unroll
    for (int k = 0; k < KB; ++k) {
      const float coef = coefficients[3 * k + ch];
      raw = fmaf(coef, basis[k], raw);
      sdx = fmaf(coef, dbx[k], sdx);
      sdy = fmaf(coef, dby[k], sdy);
      sdz = fmaf(coef, dbz[k], sdz);
    }
    raw = raw + 0.5f;
    const float gc = Load::get(gp + 5 + ch) * (raw > 0.0f ? 1.0f : 0.0f);
    gc3[ch] = visible ? gc : 0.0f;
    gdx += gc * sdx;
    gdy += gc * sdy;
    gdz += gc * sdz;
  }
  float gout[K * 3];
#pragma unroll
  for (int k = 0; k < K; ++k) {
#pragma unroll
    for (int ch = 0; ch < 3; ++ch)
      gout[3 * k + ch] = visible ? gc3[ch] * basis[k] : 0.0f;
  }
  sink.color(gout);
  const float dot_d = x * gdx + y * gdy + z * gdz;
  gdx = (gdx - x * dot_d) / norm;
  gdy = (gdy - y * dot_d) / norm;
  gdz = (gdz - z * dot_d) / norm;
  gmx += gdx; gmy += gdy; gmz += gdz;
  // project_bwd.py:320-334
  const float po = b.po;
  const float go = Load::get(gp + 8) * po * (1.0f - po);
  sink.rest(visible ? gmx : 0.0f, visible ? gmy : 0.0f, visible ? gmz : 0.0f,
            visible ? make_float4(gqw, gqx, gqy, gqz) : make_float4(0.0f, 0.0f, 0.0f, 0.0f),
            visible ? grad_sx * sx : 0.0f, visible ? grad_sy * sy : 0.0f,
            visible ? grad_sz * sz : 0.0f, visible ? go : 0.0f);
}

// Stores one view's gradients (the single-view backward).
template <int K>
struct StoreGradients {
  int64_t i;
  float *grad_mean, *grad_rotation, *grad_scale, *grad_opacity, *grad_color;
  __device__ __forceinline__ void color(const float (&g)[K * 3]) {
    float* gcol = grad_color + i * (K * 3);
    if constexpr ((K * 12) % 16 == 0) {
      float4* v = reinterpret_cast<float4*>(gcol);
#pragma unroll
      for (int j = 0; j < K * 3 / 4; ++j)
        v[j] = make_float4(g[4 * j], g[4 * j + 1], g[4 * j + 2], g[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < K * 3; ++j) gcol[j] = g[j];
    }
  }
  __device__ __forceinline__ void rest(float gmx, float gmy, float gmz, float4 grot, float gsx,
                                       float gsy, float gsz, float go) {
    grad_mean[3 * i] = gmx;
    grad_mean[3 * i + 1] = gmy;
    grad_mean[3 * i + 2] = gmz;
    reinterpret_cast<float4*>(grad_rotation)[i] = grot;
    grad_scale[3 * i] = gsx;
    grad_scale[3 * i + 1] = gsy;
    grad_scale[3 * i + 2] = gsz;
    grad_opacity[i] = go;
  }
};

// Sums the gradients of several views: the 3K colour sums in shared memory
// (one column per thread of a 128-thread block, so a warp's accesses fall in
// distinct banks), the rest in registers. Keeping the colour sums out of
// registers lets four blocks share an SM without spills at K = 16.
template <int K>
struct SharedAccumulateGradients {
  float (*c)[128];
  int t;
  float m[3], s[3], o;
  float4 r;
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int j = 0; j < K * 3; ++j) c[j][t] = 0.0f;
    m[0] = m[1] = m[2] = s[0] = s[1] = s[2] = o = 0.0f;
    r = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  __device__ __forceinline__ void color(const float (&g)[K * 3]) {
#pragma unroll
    for (int j = 0; j < K * 3; ++j) c[j][t] = c[j][t] + g[j];
  }
  __device__ __forceinline__ void rest(float gmx, float gmy, float gmz, float4 grot, float gsx,
                                       float gsy, float gsz, float go) {
    m[0] = m[0] + gmx; m[1] = m[1] + gmy; m[2] = m[2] + gmz;
    r = make_float4(r.x + grot.x, r.y + grot.y, r.z + grot.z, r.w + grot.w);
    s[0] = s[0] + gsx; s[1] = s[1] + gsy; s[2] = s[2] + gsz;
    o = o + go;
  }
};

// One view of gs_project_bwd_views as it lies in device memory: the
// render's gs_params, then the camera rotation (row-major) and translation.
struct ViewRecord {
  gs_params p;
  float R[9];
  float t[3];
};
static_assert(sizeof(ViewRecord) == 29 * 4, "29 32-bit words per view");

// Where the views of gs_project_bwd_views live: [views, n, ...] arrays in this
// GPU's memory.
struct ContiguousViews {
  const float* grad_projected;
  const int32_t* counts;
  int64_t n;
  using Load = LoadReadOnly;
  __device__ __forceinline__ int32_t count(int v, int64_t i) const {
    return __ldg(counts + static_cast<int64_t>(v) * n + i);
  }
  __device__ __forceinline__ const float* grad(int v, int64_t i) const {
    return grad_projected + 9 * (static_cast<int64_t>(v) * n + i);
  }
};

// ... or one [n, 9] gradient and [n] count array per view, each in the memory
// of the GPU that rendered the view (peer-mapped; read at L2 only).
struct PeerViews {
  const float* grad_projected[kMaxPeers];
  const int32_t* counts[kMaxPeers];
  using Load = LoadPeer;
  __device__ __forceinline__ int32_t count(int v, int64_t i) const {
    return __ldcg(counts[v] + i);
  }
  __device__ __forceinline__ const float* grad(int v, int64_t i) const {
    return grad_projected[v] + 9 * i;
  }
};

// Projection backward summed over views: each thread reads its Gaussian's
// parameters once, recomputes each view's conic with the forward's
// expressions, runs the single-view backward per view on that view's
// screen-space gradient and writes the sum over views in view order. The
// views' cameras are read from device memory, so a collective (or a peer
// handshake) can deliver them without a host round trip. A view where the
// Gaussian is not visible contributes zero, as in the single-view backward.
template <int K, class Source>
__global__ void __launch_bounds__(128, K > 16 ? 3 : 4) project_bwd_views_kernel(
    int64_t n, int num_views, const float* __restrict__ mean, const float* __restrict__ rotation,
    const float* __restrict__ scale, const float* __restrict__ opacity,
    const float* __restrict__ color, const ViewRecord* __restrict__ views,
    const __grid_constant__ Source src, float* __restrict__ grad_mean,
    float* __restrict__ grad_rotation, float* __restrict__ grad_scale,
    float* __restrict__ grad_opacity, float* __restrict__ grad_color) {
  chain_wait();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  if (threadIdx.x == 0) {
    const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x;
    prefetch_gaussian_rows(first, n - first < blockDim.x ? n - first : blockDim.x, K, mean,
                           rotation, scale, opacity, color);
  }
  const GaussianTerms g = gaussian_terms(i, mean, rotation, scale, opacity);
  const BwdTerms b = bwd_terms(i, mean, rotation, scale, opacity);
  __shared__ float color_acc[K * 3][128];
  SharedAccumulateGradients<K> acc{color_acc, static_cast<int>(threadIdx.x)};
  acc.zero();
  for (int v = 0; v < num_views; ++v) {
    if (src.count(v, i) == 0) continue;
    const gs_params p = views[v].p;
    const float* R = views[v].R;
    const float* t = views[v].t;
    const Camera c{R[0], R[1], R[2], R[3], R[4], R[5], R[6], R[7], R[8], t[0], t[1], t[2]};
    const float4 inv = view_conic(g, c, p);
    project_bwd_view<K, SharedAccumulateGradients<K>, typename Source::Load>(
        true, c, p, b, color + i * (K * 3), inv, src.grad(v, i), acc);
  }
  float sum[K * 3];
#pragma unroll
  for (int j = 0; j < K * 3; ++j) sum[j] = color_acc[j][threadIdx.x];
  StoreGradients<K> out{i, grad_mean, grad_rotation, grad_scale, grad_opacity, grad_color};
  out.color(sum);
  out.rest(acc.m[0], acc.m[1], acc.m[2], acc.r, acc.s[0], acc.s[1], acc.s[2], acc.o);
}

// Threads (one per Gaussian) of a project_bwd_kernel CTA: its staged rows
// stay within 48 KB of static shared memory at every SH degree. At degree 3
// (96 registers) ten 64-thread CTAs fit an SM where five 128-thread ones did:
// the same resident warps, but CTAs at more staggered phases of their
// stage / compute / write-out cycle, so the copies of some overlap the
// arithmetic of others (0.109 -> 0.103 ms per 1M Gaussians).
constexpr int project_bwd_threads(int) { return 64; }

// A CTA's rows of every input of the single-view backward, staged in shared
// memory; the SH rows are overwritten in place by their gradients.
template <int K, int T>
struct BwdRows {
  float sh[T * ShPitch<K>::value];
  float4 rotation[T];
  float4 conic[T];
  float mean[T * 3];
  float scale[T * 3];
  float grad[T * 9];
  float opacity[T];
  int32_t counts[T];
};

// Sink of the staged backward: the SH gradients replace the thread's own SH
// row in shared memory (the CTA writes them out together, coalesced), the
// rest goes straight to global memory.
template <int K>
struct StagedStoreGradients {
  int64_t i;
  float* row;
  float *grad_mean, *grad_rotation, *grad_scale, *grad_opacity;
  __device__ __forceinline__ void color(const float (&g)[K * 3]) {
    if constexpr ((K * 3) % 4 == 0) {
      float4* v = reinterpret_cast<float4*>(row);
#pragma unroll
      for (int j = 0; j < K * 3 / 4; ++j)
        v[j] = make_float4(g[4 * j], g[4 * j + 1], g[4 * j + 2], g[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < K * 3; ++j) row[j] = g[j];
    }
  }
  __device__ __forceinline__ void rest(float gmx, float gmy, float gmz, float4 grot, float gsx,
                                       float gsy, float gsz, float go) {
    grad_mean[3 * i] = gmx;
    grad_mean[3 * i + 1] = gmy;
    grad_mean[3 * i + 2] = gmz;
    reinterpret_cast<float4*>(grad_rotation)[i] = grot;
    grad_scale[3 * i] = gsx;
    grad_scale[3 * i + 1] = gsy;
    grad_scale[3 * i + 2] = gsz;
    grad_opacity[i] = go;
  }
};

// Writes rows [0, rows) staged at kPitch floats a row back to a row-major
// global array of kRow floats a row, spread over the CTA's threads in global
// address order (16-byte stores where the block allows, as in
// stage_rows_async).
template <int kRow, int kPitch, int kThreads>
__device__ __forceinline__ void store_rows(float* __restrict__ dst, const float* src, int rows,
                                           int tid) {
  const int words = rows * kRow;
  const bool vec = (reinterpret_cast<uint64_t>(dst) & 15) == 0 && (words & 3) == 0 &&
                   (kPitch == kRow || kRow % 4 == 0);
  if (vec) {
    for (int q = tid; q < words / 4; q += kThreads) {
      int d = 4 * q;
      if constexpr (kPitch != kRow) {
        const int r = q / (kRow / 4);
        d = r * kPitch + 4 * (q - r * (kRow / 4));
      }
      reinterpret_cast<float4*>(dst)[q] = *reinterpret_cast<const float4*>(src + d);
    }
  } else {
    for (int w = tid; w < words; w += kThreads) {
      int d = w;
      if constexpr (kPitch != kRow) {
        const int r = w / kRow;
        d = r * kPitch + (w - r * kRow);
      }
      dst[w] = src[d];
    }
  }
}

// Single-view projection backward, one thread per Gaussian. As in the
// forward, the CTA stages its contiguous block of every input (parameters,
// conic, screen-space gradient, count: 292 bytes a Gaussian at SH degree 3)
// into shared memory with coalesced asynchronous copies issued at once, and
// the SH gradients (the bulk of the writes) leave through shared memory as
// coalesced 16-byte stores.
template <int K>
__global__ void __launch_bounds__(project_bwd_threads(K)) project_bwd_kernel(
    int64_t n, const float* __restrict__ mean, const float* __restrict__ rotation,
    const float* __restrict__ scale, const float* __restrict__ opacity,
    const float* __restrict__ color, const float* __restrict__ camera_rotation,
    const float* __restrict__ camera_translation, const float* __restrict__ inverse_covariance,
    const float* __restrict__ grad_projected, const int32_t* __restrict__ counts,
    const gs_params p, float* __restrict__ grad_mean, float* __restrict__ grad_rotation,
    float* __restrict__ grad_scale, float* __restrict__ grad_opacity,
    float* __restrict__ grad_color) {
  chain_wait();
  constexpr int T = project_bwd_threads(K);
  constexpr int kPitch = ShPitch<K>::value;
  __shared__ __align__(16) BwdRows<K, T> s;
  const int tid = threadIdx.x;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * T;
  const int rows = n - first < T ? static_cast<int>(n - first) : T;
  stage_rows_async<3 * K, kPitch, T>(s.sh, color + first * (3 * K), rows, tid);
  stage_rows_async<4, 4, T>(&s.rotation[0].x, rotation + 4 * first, rows, tid);
  stage_rows_async<4, 4, T>(&s.conic[0].x, inverse_covariance + 4 * first, rows, tid);
  stage_rows_async<3, 3, T>(s.mean, mean + 3 * first, rows, tid);
  stage_rows_async<3, 3, T>(s.scale, scale + 3 * first, rows, tid);
  stage_rows_async<9, 9, T>(s.grad, grad_projected + 9 * first, rows, tid);
  stage_rows_async<1, 1, T>(s.opacity, opacity + first, rows, tid);
  stage_rows_async<1, 1, T>(reinterpret_cast<float*>(s.counts),
                            reinterpret_cast<const float*>(counts + first), rows, tid);
  cp_async_commit();
  const Camera c = load_camera(camera_rotation, camera_translation);
  cp_async_wait_all();
  __syncthreads();
  if (tid < rows) {
    const int64_t i = first + tid;
    const BwdTerms b = bwd_terms_of(s.mean[3 * tid], s.mean[3 * tid + 1], s.mean[3 * tid + 2],
                                    s.rotation[tid], s.scale[3 * tid], s.scale[3 * tid + 1],
                                    s.scale[3 * tid + 2], s.opacity[tid]);
    float* row = s.sh + tid * kPitch;
    StagedStoreGradients<K> sink{i, row, grad_mean, grad_rotation, grad_scale, grad_opacity};
    project_bwd_view<K, StagedStoreGradients<K>, LoadShared, true>(
        s.counts[tid] != 0, c, p, b, row, s.conic[tid], s.grad + 9 * tid, sink);
  }
  __syncthreads();
  store_rows<3 * K, kPitch, T>(grad_color + first * (3 * K), s.sh, rows, tid);
}

}  // namespace

#define GS_SH_DISPATCH(num_sh, LAUNCH)        \
  switch (num_sh) {                            \
    case 1: LAUNCH(1); break;                  \
    case 4: LAUNCH(4); break;                  \
    case 9: LAUNCH(9); break;                  \
    case 16: LAUNCH(16); break;                \
    case 25: LAUNCH(25); break;                \
    default: return GS_ERR_UNSUPPORTED;        \
  }

int32_t launch_project_fwd(int64_t n, int32_t num_sh, const float* mean, const float* rotation,
                           const float* scale, const float* opacity, const float* color,
                           const float* camera_rotation, const float* camera_translation,
                           const gs_params& p, float* projected_mean, float* inverse_covariance,
                           float* projected_color, float* projected_opacity, int32_t* bounds,
                           int32_t* counts, float* records, cudaStream_t stream) {
  if (n == 0) return GS_OK;
  const unsigned blocks = ceil_div(n, kProjectThreads);
#define GS_LAUNCH(K)                                                                          \
  launch_chained(project_fwd_kernel<K>, blocks, kProjectThreads, stream,                       \
      n, mean, rotation, scale, opacity, color, camera_rotation, camera_translation, p,       \
      projected_mean, inverse_covariance, projected_color, projected_opacity,                 \
      reinterpret_cast<int4*>(bounds), counts, reinterpret_cast<float4*>(records))
  GS_SH_DISPATCH(num_sh, GS_LAUNCH)
#undef GS_LAUNCH
  return check_launch();
}

int32_t launch_project_fwd_batch(int64_t n, int32_t num_sh, int32_t num_views, const float* mean,
                                 const float* rotation, const float* scale, const float* opacity,
                                 const float* color, const float* camera_rotations_host,
                                 const float* camera_translations_host,
                                 const gs_params* params_host, float* projected_mean,
                                 float* inverse_covariance, float* projected_color,
                                 float* projected_opacity, int32_t* bounds, int32_t* counts,
                                 float* records, cudaStream_t stream) {
  if (n == 0 || num_views == 0) return GS_OK;
  const unsigned blocks = ceil_div(n, 256);
  for (int first = 0; first < num_views; first += kMaxBatchViews) {
    ViewBatch batch{};
    batch.views = num_views - first < kMaxBatchViews ? num_views - first : kMaxBatchViews;
    for (int b = 0; b < batch.views; ++b) {
      const float* R = camera_rotations_host + 9 * (first + b);
      const float* t = camera_translations_host + 3 * (first + b);
      batch.c[b] = Camera{R[0], R[1], R[2], R[3], R[4], R[5], R[6], R[7], R[8], t[0], t[1], t[2]};
      batch.p[b] = params_host[first + b];
    }
    const int64_t o = static_cast<int64_t>(first) * n;
#define GS_LAUNCH(K)                                                                          \
  launch_chained(project_fwd_batch_kernel<K>, blocks, 256, stream,                             \
      n, mean, rotation, scale, opacity, color, batch, projected_mean + 3 * o,                 \
      inverse_covariance + 4 * o, projected_color + 3 * o, projected_opacity + o,              \
      reinterpret_cast<int4*>(bounds) + o, counts + o,                                        \
      records ? reinterpret_cast<float4*>(records) + 4 * o : nullptr)
    GS_SH_DISPATCH(num_sh, GS_LAUNCH)
#undef GS_LAUNCH
    GS_TRY(check_launch());
  }
  return GS_OK;
}

int32_t launch_project_bwd_views(int64_t n, int32_t num_sh, int32_t num_views,
                                 const float* mean, const float* rotation, const float* scale,
                                 const float* opacity, const float* color, const void* views,
                                 const float* grad_projected, const int32_t* counts,
                                 float* grad_mean, float* grad_rotation, float* grad_scale,
                                 float* grad_opacity, float* grad_color, cudaStream_t stream) {
  if (n == 0) return GS_OK;
  const unsigned blocks = ceil_div(n, 128);
  const ContiguousViews src{grad_projected, counts, n};
#define GS_LAUNCH(K)                                                                          \
  launch_chained(project_bwd_views_kernel<K, ContiguousViews>, blocks, 128, stream,            \
      n, num_views, mean, rotation, scale, opacity, color,                                    \
      static_cast<const ViewRecord*>(views), src, grad_mean, grad_rotation, grad_scale,       \
      grad_opacity, grad_color)
  GS_SH_DISPATCH(num_sh, GS_LAUNCH)
#undef GS_LAUNCH
  return check_launch();
}

int32_t launch_project_bwd_peers(int64_t n, int32_t num_sh, int32_t num_views,
                                 const float* mean, const float* rotation, const float* scale,
                                 const float* opacity, const float* color, const void* views,
                                 const float* const* grad_projected, const int32_t* const* counts,
                                 float* grad_mean, float* grad_rotation, float* grad_scale,
                                 float* grad_opacity, float* grad_color, cudaStream_t stream) {
  if (n == 0) return GS_OK;
  if (num_views < 0 || num_views > kMaxPeers) return GS_ERR_INVALID_ARGUMENT;
  PeerViews src{};
  for (int v = 0; v < num_views; ++v) {
    src.grad_projected[v] = grad_projected[v];
    src.counts[v] = counts[v];
  }
  const unsigned blocks = ceil_div(n, 128);
#define GS_LAUNCH(K)                                                                          \
  project_bwd_views_kernel<K, PeerViews><<<blocks, 128, 0, stream>>>(                         \
      n, num_views, mean, rotation, scale, opacity, color,                                    \
      static_cast<const ViewRecord*>(views), src, grad_mean, grad_rotation, grad_scale,       \
      grad_opacity, grad_color)
  GS_SH_DISPATCH(num_sh, GS_LAUNCH)
#undef GS_LAUNCH
  return check_launch();
}

int32_t launch_project_bwd(int64_t n, int32_t num_sh, const float* mean, const float* rotation,
                           const float* scale, const float* opacity, const float* color,
                           const float* camera_rotation, const float* camera_translation,
                           const float* inverse_covariance, const float* grad_projected,
                           const int32_t* counts, const gs_params& p, float* grad_mean,
                           float* grad_rotation, float* grad_scale, float* grad_opacity,
                           float* grad_color, cudaStream_t stream) {
  if (n == 0) return GS_OK;
#define GS_LAUNCH(K)                                                                          \
  launch_chained(project_bwd_kernel<K>, ceil_div(n, project_bwd_threads(K)),                   \
                 project_bwd_threads(K), stream,                                               \
      n, mean, rotation, scale, opacity, color, camera_rotation, camera_translation,           \
      inverse_covariance, grad_projected, counts, p, grad_mean, grad_rotation, grad_scale,    \
      grad_opacity, grad_color)
  GS_SH_DISPATCH(num_sh, GS_LAUNCH)
#undef GS_LAUNCH
  return check_launch();
}

__global__ void det_exp_kernel(int64_t n, const float* __restrict__ x, float* __restrict__ y) {
  chain_wait();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) y[i] = det_exp(x[i]);
}

__global__ void det_log_kernel(int64_t n, const float* __restrict__ x, float* __restrict__ y) {
  chain_wait();
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) y[i] = det_log(x[i]);
}

int32_t launch_det_math(int which, int64_t n, const float* x, float* y, cudaStream_t stream) {
  if (n == 0) return GS_OK;
  if (which == 0)
    launch_chained(det_exp_kernel, ceil_div(n, 256), 256, stream, n, x, y);
  else
    launch_chained(det_log_kernel, ceil_div(n, 256), 256, stream, n, x, y);
  return check_launch();
}

}  // namespace gs
