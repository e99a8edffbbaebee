// Shared definitions for the rasterizer kernels.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/gs_b200.h"
#include "detmath.cuh"

namespace gs {

constexpr float kAlphaMin = 1.0f / 255.0f;  // composite.py:170, composite_bwd.py:121
constexpr float kAlphaMax = 0.99f;           // composite.py:169
constexpr int kSmCount = 148;                // B200: 2 dies x 74 SMs
constexpr int kMaxPeers = GS_MAX_PEERS;      // ranks of a view-parallel exchange

// Records the last CUDA error for gs_last_cuda_error(); defined in capi.cu.
void set_cuda_error(cudaError_t err);

inline int32_t check_launch() {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    set_cuda_error(err);
    return GS_ERR_CUDA;
  }
  return GS_OK;
}

#define GS_CUDA_TRY(expr)                    \
  do {                                       \
    cudaError_t gs_err_ = (expr);            \
    if (gs_err_ != cudaSuccess) {            \
      ::gs::set_cuda_error(gs_err_);         \
      return GS_ERR_CUDA;                    \
    }                                        \
  } while (0)

#define GS_TRY(expr)                         \
  do {                                       \
    int32_t gs_status_ = (expr);             \
    if (gs_status_ != GS_OK) return gs_status_; \
  } while (0)

inline cudaStream_t as_cuda(gs_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Chained launches (programmatic dependent launch). A step is a chain of
// short kernels on one stream. Launched normally, a kernel is set up only
// once the one before has completed and its writes have been flushed;
// launch_chained lets the GPU prepare the launch ahead, so the kernel's CTAs
// start as soon as the previous kernel's last CTA exits, and the flush is
// awaited inside the kernel: every CTA of a kernel in the pipeline first
// executes chain_wait(), which blocks in hardware (no spinning) until the
// previous kernel on the stream has completed and its writes are visible. No
// kernel reads or writes memory before its predecessor is done, so stream
// order holds as before; because every kernel waits before anything else
// (also before an early return), completion stays ordered along the chain:
// k+1 cannot finish before k. After an operation that is not one of these
// kernels (a memset, a copy, another library's kernel) a chained launch is
// ordered as a normal one; chain_wait is a no-op in a kernel launched
// normally. The kernels do not signal their dependents early
// (griddepcontrol.launch_dependents): CTAs of the next kernel parked on the
// SMs while this one still runs cost more than the earlier start saved
// (training step 1.40 -> 1.43 ms on a 1080p view of 1M Gaussians, against
// 1.39 ms without the early signal).
__device__ __forceinline__ void chain_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Launches `kernel` chained (see above). Like a <<<>>> launch, a failed launch
// also leaves its error for cudaGetLastError, which is how the launchers read
// it (check_launch() after each launch).
template <class... Params, class... Args>
inline cudaError_t launch_chained(void (*kernel)(Params...), dim3 grid, dim3 block,
                                  cudaStream_t stream, Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = 0;
  config.stream = stream;
  config.attrs = attr;
  config.numAttrs = 1;
  return cudaLaunchKernelEx(&config, kernel, static_cast<Args&&>(args)...);
}

inline unsigned ceil_div(int64_t a, int64_t b) { return static_cast<unsigned>((a + b - 1) / b); }

// Gaussian index and intersection offsets are 32-bit in the binning kernels.
constexpr int64_t kMaxGaussians = int64_t{1} << 30;
constexpr int64_t kMaxIntersections = int64_t{1} << 30;

// Render scalars every entry point validates the same way: a tile size the
// kernels are instantiated for, and an image of whole tiles.
inline int32_t check_params(const gs_params* p) {
  if (!p) return GS_ERR_INVALID_ARGUMENT;
  const int ts = p->tile_size;
  if (ts != 4 && ts != 8 && ts != 16 && ts != 32) return GS_ERR_INVALID_ARGUMENT;
  if (p->width < 0 || p->height < 0 || p->width % ts || p->height % ts)
    return GS_ERR_INVALID_ARGUMENT;
  return GS_OK;
}

// Starts moving the 16-byte-aligned interior of [ptr, ptr + bytes) from DRAM
// into L2 and returns at once (TMA bulk prefetch: no registers, shared memory
// or barrier, nothing to wait for). One thread of a CTA calls it for the
// CTA's contiguous block of an input array, so the whole block is requested
// at the CTA's start instead of load by load behind the thread's dependent
// arithmetic; the threads' own loads then find it in L2. Only addresses
// inside the range are touched.
__device__ __forceinline__ void prefetch_l2(const void* ptr, uint64_t bytes) {
  constexpr uint64_t kChunk = 1 << 16;  // bytes per instruction
  uint64_t begin = (reinterpret_cast<uint64_t>(ptr) + 15) & ~uint64_t{15};
  const uint64_t end = (reinterpret_cast<uint64_t>(ptr) + bytes) & ~uint64_t{15};
  for (; begin < end; begin += kChunk) {
    const uint64_t size = end - begin < kChunk ? end - begin : kChunk;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(begin),
                 "r"(static_cast<uint32_t>(size))
                 : "memory");
  }
}

// Asynchronous global -> shared copies (cp.async): 16 bytes at L2 only, or 4
// bytes through L1. A thread's copies complete at cp_async_wait_*; a CTA
// barrier after that makes every thread's copies visible.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const uint32_t dst = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}
// Waits for all but the most recently committed group.
__device__ __forceinline__ void cp_async_wait_all_but_last() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
}

// Starts copying rows [0, rows) of a row-major float array (kRow floats a
// row, `src` at row 0) into shared memory at kPitch floats a row (kPitch >
// kRow pads rows so that lanes reading consecutive rows hit distinct banks).
// The copies are spread over the CTA's kThreads threads in address order, so
// each warp's requests are coalesced; a CTA's block of Gaussian rows is one
// contiguous range of every parameter array. 16-byte copies when the source
// block starts on a 16-byte boundary, is a whole number of 16-byte words and
// no word straddles two rows of a padded layout (dst 16-byte aligned, kPitch
// a multiple of 4 when padded); 4-byte copies otherwise (a ragged last block
// or an unaligned caller tensor). Only addresses inside the block are read.
template <int kRow, int kPitch, int kThreads>
__device__ __forceinline__ void stage_rows_async(float* dst, const float* src, int rows, int tid) {
  static_assert(kPitch == kRow || (kRow % 4 == 0 && kPitch % 4 == 0), "padded rows of 16-byte words");
  const int words = rows * kRow;
  const bool vec = (reinterpret_cast<uint64_t>(src) & 15) == 0 && (words & 3) == 0;
  if (vec) {
    for (int q = tid; q < words / 4; q += kThreads) {
      int d = 4 * q;
      if constexpr (kPitch != kRow) {
        const int r = q / (kRow / 4);
        d = r * kPitch + 4 * (q - r * (kRow / 4));
      }
      cp_async16(dst + d, src + 4 * q);
    }
  } else {
    for (int w = tid; w < words; w += kThreads) {
      int d = w;
      if constexpr (kPitch != kRow) {
        const int r = w / kRow;
        d = r * kPitch + (w - r * kRow);
      }
      cp_async4(dst + d, src + w);
    }
  }
}

// Shared-memory pitch (floats) of a CTA's staged SH rows (3K floats each):
// rows of an even number of 16-byte words are padded by one word, so the 8
// lanes of a quarter-warp reading word j of consecutive rows touch 8
// distinct 4-bank groups (an odd word stride); other rows are read as
// scalars at an odd stride or as 16-byte words at an odd word stride already.
template <int K>
struct ShPitch {
  static constexpr int kRow = 3 * K;
  static constexpr int value = (kRow % 4 == 0 && (kRow / 4) % 2 == 0) ? kRow + 4 : kRow;
};

// Loads the 3K SH coefficients of one Gaussian from its staged shared-memory
// row (16-byte words when the row is made of them, scalars otherwise).
template <int K>
__device__ __forceinline__ void load_sh_shared(const float* row, float (&c)[K * 3]) {
  if constexpr ((K * 3) % 4 == 0) {
    const float4* v = reinterpret_cast<const float4*>(row);
#pragma unroll
    for (int j = 0; j < K * 3 / 4; ++j) {
      const float4 q = v[j];
      c[4 * j] = q.x; c[4 * j + 1] = q.y; c[4 * j + 2] = q.z; c[4 * j + 3] = q.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < K * 3; ++j) c[j] = row[j];
  }
}

// Prefetches a CTA's rows [first, first + rows) of the Gaussian parameter
// arrays (mean, rotation, scale, opacity, K SH coefficients) into L2.
__device__ __forceinline__ void prefetch_gaussian_rows(int64_t first, int64_t rows, int k,
                                                       const float* mean, const float* rotation,
                                                       const float* scale, const float* opacity,
                                                       const float* color) {
  const uint64_t r = static_cast<uint64_t>(rows);
  prefetch_l2(color + first * 3 * k, r * 12 * k);
  prefetch_l2(mean + first * 3, r * 12);
  prefetch_l2(rotation + first * 4, r * 16);
  prefetch_l2(scale + first * 3, r * 12);
  prefetch_l2(opacity + first, r * 4);
}

// Pair evaluation shared by the forward and backward compositors:
// d^2 = xx dx^2 + 2 xy dx dy + yy dy^2 with integer pixel coordinates
// (composite.py:159-161), evaluated as fmaf(xx*dx, dx, fmaf((2xy)*dx, dy, (yy*dy)*dy)).
__device__ __forceinline__ float pair_d2(float dx, float dy, float xx, float xy2, float yy) {
  return fmaf(xx * dx, dx, fmaf(xy2 * dx, dy, (yy * dy) * dy));
}

// d^2 above which alpha = min(o e^{-d^2/2}, 0.99) is certainly below 1/255
// (given det_exp's < 1 ulp error): 2 log(255 o) plus a 1e-3 margin that
// dwarfs the rounding of this bound. Pairs beyond it leave T and C unchanged,
// so skipping them is exact. Ellipsoid mode uses its own cutoff directly.
__device__ __forceinline__ float skip_cutoff(float opacity, const gs_params& p) {
  return p.gaussian_mode ? fmaf(2.0f, det_log(opacity * 255.0f), 1e-3f) : p.cutoff;
}

// One Gaussian as the compositors stage it: 64 bytes, written once per view
// by the projection (or gs_pack_records) and gathered per tile with four
// 16-byte asynchronous copies. The skip cutoff and the bounding box of the
// ellipse d2 <= 1.0201 cutoff are derived here once per Gaussian instead of
// once per (tile, list entry).
//   a   = (mean_x, mean_y, conic_xx, 2 conic_xy)
//   b   = (conic_yy, opacity, skip cutoff, conic_xy)
//   c   = (r, g, b, Gaussian index as float bits)
//   box = (xmin, xmax, ymin, ymax) where alpha can reach 1/255: +-inf
//         everywhere for conics whose rounding the box does not bound (condition
//         number above ~1e3), empty when no pixel can reach 1/255.
struct PairRecord {
  float4 a, b, c, box;
};

__device__ __forceinline__ PairRecord make_record(int32_t g, float mx, float my, float4 conic,
                                                  float o, float r, float gg, float b,
                                                  const gs_params& p) {
  const float cutoff = skip_cutoff(o, p);
  const float xx = conic.x, xy = conic.y, yy = conic.w;
  const float det = xx * yy - xy * xy;
  const float inf = __int_as_float(0x7f800000);
  float4 box = make_float4(-inf, inf, -inf, inf);
  if (!(cutoff >= 0.0f)) {
    box = make_float4(inf, -inf, inf, -inf);  // no pixel can reach alpha >= 1/255
  } else if (xx > 0.0f && yy > 0.0f && det > 0.0f && (xx + yy) * (xx + yy) < 4.0e3f * det) {
    const float scaled = 1.0201f * cutoff / det;
    const float hx = sqrtf(scaled * yy) * 1.001f + 0.01f;
    const float hy = sqrtf(scaled * xx) * 1.001f + 0.01f;
    box = make_float4(mx - hx, mx + hx, my - hy, my + hy);
  }
  PairRecord rec;
  rec.a = make_float4(mx, my, xx, 2.0f * xy);
  rec.b = make_float4(yy, o, cutoff, xy);
  rec.c = make_float4(r, gg, b, __int_as_float(g));
  rec.box = box;
  return rec;
}

__device__ __forceinline__ void store_record(float4* records, int64_t g, const PairRecord& rec) {
  float4* dst = records + 4 * g;
  dst[0] = rec.a;
  dst[1] = rec.b;
  dst[2] = rec.c;
  dst[3] = rec.box;
}

}  // namespace gs
