// Per-tile alpha compositing, forward and backward.
//
// One CTA per tile. The tile's list of Gaussians -- ids[start:end), front to
// back -- is staged into shared memory a batch of entries at a time: each
// entry's 64-byte record (projected mean, conic, opacity, colour, skip cutoff
// and box, built once per Gaussian by the projection) arrives by four 16-byte
// asynchronous copies (cp.async, L2 only), double-buffered, so the records of
// batch k+1 are in flight while batch k is composited and each batch costs one
// CTA barrier. Every pixel walks the batch from shared memory. Each warp owns a compact
// block of pixels: in the forward one pixel per thread and an 8 x 4 block
// (4 x 4 tiles: one 4 x 4 block); in the backward, for 8 x 8 and larger
// tiles, two pixels per thread (one column, four rows apart) and an 8 x 8
// block. Two pixels per thread halve the per-pixel cost of everything done
// once per (warp, entry) -- the culling ballot, the loop and shared-memory
// loads and, above all, the warp reduction and atomics of the backward; the
// forward keeps one pixel per thread because its smaller blocks cull more
// and its pixels stop early. The work is FP32 arithmetic per (pixel,
// Gaussian) pair; nothing here is a dense contraction, so tensor cores have
// no role.
//
// Forward (composite.py:25-107). Per pair:
//   d2 = fmaf(xx dx, dx, fmaf(2xy dx, dy, (yy dy) dy)),  p = exp(-d2/2),
//   alpha = min(o p, 0.99), alpha < 1/255 -> 0, C += T alpha c, T *= 1 - alpha
// while the pixel is active ((1 - T) < threshold). Two exact shortcuts skip
// pairs with alpha = 0, which change nothing:
//  * per pixel, d2 > skip_cutoff(o) (given det_exp's < 1 ulp error);
//  * per warp, the staged entry carries the bounding box of the ellipse
//    d2 <= 1.0201 skip_cutoff; each warp ballots the staged entries against
//    its pixel block and walks only the ones whose box meets it (in list
//    order); the backward also drops entries whose ellipse itself misses
//    the block (minimum of the conic's quadratic form over the block). For conics with condition number below ~1e3 the float32 d2 of
//    any pixel outside the box is provably above the cutoff (its relative
//    rounding error is < 2 kappa * 4 ulp < 1e-3); other conics get an
//    infinite box.
// A pixel's contributor count is the number of list entries it saw while
// active, i.e. (index of the entry that ended it) + 1, or the list length if
// it never ended; the tile stops once every pixel has ended
// (composite.py:187-188).
//
// Backward (composite_bwd.py:47-277). Walks the list back to front from
// start + max(n_contributors); a running suffix per pixel (transmittance
// product and composited colour of the entries behind) replaces the
// reference's chunked associative scan; T at an entry is recovered as
// final_T / max(suffix_T (1 - alpha), 1e-4) and the termination test is
// re-evaluated on it, as the reference does. Each thread sums its pixels'
// 9-vectors per entry, each warp reduces them with a butterfly
// reduce-scatter (14 shuffles; skipped when no lane contributes) that leaves
// one component in each of 9 lanes, which add them to grad_projected[g] with
// two atomic instructions.
#include "common.cuh"

namespace gs {

uint64_t radix_sort_workspace_size(int64_t, int64_t);
int32_t launch_sort_positions(int64_t, int64_t, const int32_t*, void*, uint32_t*, int64_t*,
                              cudaStream_t);

namespace {

template <int TS, int PPT>
struct TileShape {
  static constexpr int kPixels = TS * TS;
  static constexpr int kPpt = PPT;                               // pixels per thread
  static constexpr int kThreads = kPixels / kPpt;
  static constexpr int kWarpLanes = kThreads < 32 ? kThreads : 32;
  static constexpr unsigned kWarpMask = kThreads < 32 ? ((1u << kThreads) - 1u) : 0xffffffffu;
  static constexpr int kWarps = kThreads / kWarpLanes;
  static constexpr int kBlockW = TS < 8 ? TS : 8;                // warp block width
  static constexpr int kLaneRows = kWarpLanes / kBlockW;         // rows one pass of lanes covers
  static constexpr int kBlockH = kLaneRows * kPpt;               // warp block height
  static constexpr int kBlocksPerRow = TS / kBlockW;
  static constexpr int kBatch = kPixels < 256 ? kPixels : 256;  // list entries staged at once
};

// This thread's pixels (one column, kLaneRows apart) and its warp's block.
// Resident CTAs of `threads` threads asked of the register allocator for the
// backward: 32 warps per SM (at most 64 registers a thread).
constexpr int min_blocks_for_32_warps(int threads) {
  return 1024 / threads < 16 ? 1024 / threads : 16;
}

// Resident CTAs the forward compositor is compiled for: six 256-thread CTAs
// (48 warps) fit its state in 39 registers without spills, against five at
// its natural 48. Tiles whose six CTAs would not fit an SM's 2048 threads
// (32x32) keep the unconstrained allocation.
constexpr int forward_min_blocks(int threads) { return threads * 6 <= 2048 ? 6 : 1; }

template <int TS, int PPT>
struct PixelMap {
  using S = TileShape<TS, PPT>;
  int px, py0;
  float rx0, rx1, ry0, ry1;
  __device__ __forceinline__ PixelMap(int tile, int tiles_w, int tid) {
    const int warp = tid / S::kWarpLanes, lane = tid % S::kWarpLanes;
    const int bx = (tile % tiles_w) * TS + (warp % S::kBlocksPerRow) * S::kBlockW;
    const int by = (tile / tiles_w) * TS + (warp / S::kBlocksPerRow) * S::kBlockH;
    px = bx + lane % S::kBlockW;
    py0 = by + lane / S::kBlockW;
    rx0 = static_cast<float>(bx);
    rx1 = static_cast<float>(bx + S::kBlockW - 1);
    ry0 = static_cast<float>(by);
    ry1 = static_cast<float>(by + S::kBlockH - 1);
  }
  __device__ __forceinline__ int py(int q) const { return py0 + q * S::kLaneRows; }
  // True if the box (xmin, xmax, ymin, ymax) misses this warp's pixels.
  __device__ __forceinline__ bool misses(const float4& box) const {
    return box.x > rx1 || box.y < rx0 || box.z > ry1 || box.w < ry0;
  }
};

// One buffer of staged list entries: the four float4 of each entry's record
// in separate arrays, so lanes reading consecutive entries' boxes hit
// distinct banks.
template <int NB>
struct StageBuffer {
  float4 a[NB], b[NB], c[NB], box[NB];
};

// The tile this CTA composites: CTA b takes tile_order[b] (the tiles by
// decreasing work, so the longest lists start first instead of whenever their
// row comes up), or tile b without an order. -1 (the CTA exits) for an entry
// that is not a tile of the image.
__device__ __forceinline__ int visit_tile(const int32_t* __restrict__ tile_order,
                                          const gs_params& p) {
  if (tile_order == nullptr) return static_cast<int>(blockIdx.x);
  const int tile = __ldg(tile_order + blockIdx.x);
  const int num_tiles = (p.width / p.tile_size) * (p.height / p.tile_size);
  return tile >= 0 && tile < num_tiles ? tile : -1;
}

// Starts copying Gaussian g's record into `slot` of `buf`.
template <int NB>
__device__ __forceinline__ void stage_async(const float4* __restrict__ records, int32_t g,
                                            StageBuffer<NB>& buf, int slot) {
  const float4* src = records + 4 * static_cast<int64_t>(g);
  cp_async16(&buf.a[slot], src);
  cp_async16(&buf.b[slot], src + 1);
  cp_async16(&buf.c[slot], src + 2);
  cp_async16(&buf.box[slot], src + 3);
}

// True unless the ellipse d2 <= 1.0201 cutoff provably misses the rectangle
// [x0, x1] x [y0, y1] (which holds every pixel of a warp). The minimum of the
// positive definite form q(u, v) = xx u^2 + 2 xy u v + yy v^2 over the
// rectangle (u, v relative to the mean) is 0 when the mean is inside, else it
// lies on an edge, at the edge's critical point clamped to the edge. A
// candidate computed with rounding is still a point of the rectangle, and q
// grows only quadratically away from the true minimiser, so the computed
// minimum exceeds the true one by far less than the 2% margin; conics too
// ill-conditioned for that carry an infinite box and always pass.
__device__ __forceinline__ bool ellipse_meets_rect(const float4& a, const float4& b,
                                                   const float4& box, float x0, float x1,
                                                   float y0, float y1) {
  if (box.x == -__int_as_float(0x7f800000)) return true;  // unconditioned: no exact test
  const float xx = a.z, yy = b.x, xy = b.w;
  const float u0 = x0 - a.x, u1 = x1 - a.x, v0 = y0 - a.y, v1 = y1 - a.y;
  if (u0 <= 0.0f && u1 >= 0.0f && v0 <= 0.0f && v1 >= 0.0f) return true;
  auto q = [&](float u, float v) { return xx * u * u + 2.0f * xy * u * v + yy * v * v; };
  // Critical v per u and u per v (approximate division: any point of the
  // rectangle is a valid candidate).
  const float ru = __fdividef(-xy, yy), rv = __fdividef(-xy, xx);
  float m = q(u0, fminf(fmaxf(ru * u0, v0), v1));
  m = fminf(m, q(u1, fminf(fmaxf(ru * u1, v0), v1)));
  m = fminf(m, q(fminf(fmaxf(rv * v0, u0), u1), v0));
  m = fminf(m, q(fminf(fmaxf(rv * v1, u0), u1), v1));
  return m <= 1.0201f * b.z;
}

// Appends, in order, the batch entries whose box meets this warp's pixel
// block (with kExact, whose ellipse does) and, when `limit` >= 0, whose list
// position is below `limit`, to the warp's list in shared memory; returns how
// many. One ballot per 32 entries replaces a per-entry test inside the pixel
// loop. The exact test pays in the backward, where every selected entry costs
// a warp reduction and atomics; in the forward it costs more than it saves.
template <int TS, int PPT, bool kExact, int NB>
__device__ __forceinline__ int warp_select(const PixelMap<TS, PPT>& pm, const StageBuffer<NB>& buf,
                                           int count, int lane, uint16_t* list,
                                           int64_t position0, int64_t limit) {
  using S = TileShape<TS, PPT>;
  int selected = 0;
  for (int base = 0; base < count; base += S::kWarpLanes) {
    const int j = base + lane;
    bool hit = false;
    if (j < count) {
      const float4 box = buf.box[j];
      hit = !pm.misses(box);
      if (kExact && hit)
        hit = ellipse_meets_rect(buf.a[j], buf.b[j], box, pm.rx0, pm.rx1, pm.ry0, pm.ry1);
    }
    if (limit >= 0) hit = hit && position0 + j < limit;
    const unsigned mask = __ballot_sync(S::kWarpMask, hit);
    if (hit) list[selected + __popc(mask & ((1u << lane) - 1u))] = static_cast<uint16_t>(j);
    selected += __popc(mask);
  }
  __syncwarp(S::kWarpMask);
  return selected;
}

template <int TS, bool kGaussian>
__global__ void __launch_bounds__(TileShape<TS, 1>::kThreads,
                                  forward_min_blocks(TileShape<TS, 1>::kThreads))
    composite_fwd_kernel(const float4* __restrict__ records,
                         const int32_t* __restrict__ gaussian_ids,
                         const int64_t* __restrict__ ranges, const gs_params p,
                         float* __restrict__ image, float* __restrict__ final_transmittance,
                         int32_t* __restrict__ n_contributors,
                         const int32_t* __restrict__ tile_order) {
  chain_wait();
  using S = TileShape<TS, 1>;
  constexpr int NB = S::kBatch;
  constexpr int kWarps = S::kWarps;
  __shared__ StageBuffer<NB> s_buf[2];
  __shared__ uint16_t s_list[kWarps][NB];
  const int tile = visit_tile(tile_order, p);
  if (tile < 0) return;
  const int tid = threadIdx.x;
  const int lane = tid % S::kWarpLanes, warp = tid / S::kWarpLanes;
  const PixelMap<TS, 1> pm(tile, p.width / TS, tid);
  const float fpx = static_cast<float>(pm.px), fpy = static_cast<float>(pm.py0);
  const int64_t start = ranges[2 * tile], end = ranges[2 * tile + 1];
  const float threshold = p.opacity_threshold;
  uint16_t* list = s_list[warp];

  // Thread tid stages entry tid of every batch; the id of its next batch's
  // entry is loaded one batch ahead, so issuing a batch's copies never waits.
  int32_t next_id = 0;
  if (tid < NB) {
    if (start + tid < end) stage_async(records, __ldg(gaussian_ids + start + tid), s_buf[0], tid);
    if (start + NB + tid < end) next_id = __ldg(gaussian_ids + start + NB + tid);
  }
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();

  float T = 1.0f, cr = 0.0f, cg = 0.0f, cb = 0.0f;
  bool done = !((1.0f - T) < threshold);
  int64_t contrib = 0;
  int buf = 0;
  for (int64_t batch = start; batch < end; batch += NB, buf ^= 1) {
    // The next batch's records fill the other buffer while this one is used.
    const int64_t next = batch + NB;
    if (tid < NB && next + tid < end) {
      stage_async(records, next_id, s_buf[buf ^ 1], tid);
      if (next + NB + tid < end) next_id = __ldg(gaussian_ids + next + NB + tid);
    }
    cp_async_commit();
    const StageBuffer<NB>& cur = s_buf[buf];
    if (__any_sync(S::kWarpMask, !done)) {
      const int count = static_cast<int>(end - batch < NB ? end - batch : NB);
      const int selected = warp_select<TS, 1, false>(pm, cur, count, lane, list, 0, -1);
      if (!done) {
        for (int i = 0; i < selected; ++i) {
          const int j = list[i];
          const float4 a = cur.a[j];
          const float4 b = cur.b[j];
          const float dx = fpx - a.x, dy = fpy - a.y;
          const float d2 = pair_d2(dx, dy, a.z, a.w, b.x);
          if (!(d2 <= b.z)) continue;
          float alpha;
          if constexpr (kGaussian) {
            const float prob = d2 >= 0.0f ? det_exp_nonpositive(-0.5f * d2) : det_exp(-0.5f * d2);
            alpha = fminf(b.y * prob, kAlphaMax);
          } else {
            alpha = fminf(b.y, kAlphaMax);
          }
          if (!(alpha >= kAlphaMin)) continue;
          const float4 c = cur.c[j];
          const float weight = T * alpha;
          cr = fmaf(weight, c.x, cr);
          cg = fmaf(weight, c.y, cg);
          cb = fmaf(weight, c.z, cb);
          T = T * (1.0f - alpha);
          if (!((1.0f - T) < threshold)) {
            done = true;
            contrib = batch + j + 1 - start;
            break;
          }
        }
      }
    }
    // This thread's copies of the next batch have landed; the barrier makes
    // every thread's visible and frees the current buffer for refilling.
    cp_async_wait_all();
    if (__syncthreads_count(!done) == 0) break;
  }
  if (!done) contrib = end - start;
  const int64_t pix = static_cast<int64_t>(pm.py0) * p.width + pm.px;
  image[3 * pix] = cr;
  image[3 * pix + 1] = cg;
  image[3 * pix + 2] = cb;
  final_transmittance[pix] = T;
  n_contributors[pix] = static_cast<int32_t>(contrib);
}

// Sums v[0..8] over the 32 lanes of a warp. Values 0..7 go through a
// butterfly reduce-scatter (each exchange halves the values a lane keeps);
// afterwards lane 4k holds the total of value k. Value 8 is reduced plainly
// and lands in every lane. 14 shuffles instead of 45.
__device__ __forceinline__ void warp_reduce_scatter9(const float (&v)[9], int lane,
                                                     float& mine, float& last) {
  const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4;
  float k4[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = h16 ? v[i] : v[4 + i];
    k4[i] = (h16 ? v[4 + i] : v[i]) + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  float k2[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = h8 ? k4[i] : k4[2 + i];
    k2[i] = (h8 ? k4[2 + i] : k4[i]) + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  {
    const float send = h4 ? k2[0] : k2[1];
    mine = (h4 ? k2[1] : k2[0]) + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  mine += __shfl_xor_sync(0xffffffffu, mine, 2);
  mine += __shfl_xor_sync(0xffffffffu, mine, 1);
  last = v[8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) last += __shfl_xor_sync(0xffffffffu, last, o);
}

// Staging of the backward: double-buffered batches of 128 records (the next
// batch in flight while one is used; 17 KB of shared memory, so the eight
// CTAs per SM its register bound allows still fit), or with
// GS_BWD_DOUBLE=0 single-buffered batches of 256 (two barriers per batch).
#ifndef GS_BWD_DOUBLE
#define GS_BWD_DOUBLE 1
#endif
constexpr bool kBackwardDoubleBuffer = GS_BWD_DOUBLE != 0;
template <int TS, int PPT>
struct BackwardBatch {
  static constexpr int kMax = kBackwardDoubleBuffer ? 128 : 256;
  static constexpr int value =
      TileShape<TS, PPT>::kBatch < kMax ? TileShape<TS, PPT>::kBatch : kMax;
};

// Walk tags of the backward kernel (a walk accumulates only the suffix, or
// the gradients too).
struct SuffixPass {
  static constexpr bool value = true;
};
struct GradientPass {
  static constexpr bool value = false;
};

// kRows: the deterministic form. Instead of adding each warp's reduced
// 9-vector into grad_projected[g] with atomics, every warp leaves it in shared
// memory, and after each batch the CTA sums the warps' vectors in warp order
// into one row per list position, rows [position, 9] (positions the tile never
// reaches stay as the caller zeroed them). reduce_rows_kernel then adds each
// Gaussian's rows in list-position order. No float addition depends on
// scheduling, so the gradients are the same bits on every run.
//
// Split tiles. A tile whose walk is long is split into `parts` consecutive
// sub-ranges of its list, each a CTA of its own, so that one dense tile no
// longer sets the kernel's length. Part k needs the transmittance product and
// composited colour of every entry behind it: its CTA first walks the parts
// behind it accumulating only that suffix (the same per-pair decisions and
// the same recurrence, so the same bits as an unsplit walk at that point, at
// about a third of the per-entry cost: no gradients, reductions or atomics),
// then walks its own part with gradients. `items`, when given, lists the work
// of the launch: (tile, part, parts, -), tile -1 for none; else `tile_order`
// (or row-major order) gives whole tiles.
template <int TS, int PPT, bool kGaussian, bool kRows = false>
__global__ void __launch_bounds__(TileShape<TS, PPT>::kThreads,
                                  min_blocks_for_32_warps(TileShape<TS, PPT>::kThreads))
    composite_bwd_kernel(const float4* __restrict__ records,
                         const int32_t* __restrict__ gaussian_ids,
                         const int64_t* __restrict__ ranges, const float* __restrict__ grad_image,
                         const float* __restrict__ final_transmittance,
                         const int32_t* __restrict__ n_contributors, const gs_params p,
                         float* __restrict__ grad_projected,
                         const int32_t* __restrict__ tile_order, const int4* __restrict__ items) {
  chain_wait();
  using S = TileShape<TS, PPT>;
  // (the deterministic form's per-warp vectors of 32 x 32 tiles take smaller batches
  // to stay within 48 KB of shared memory)
  constexpr int NB = kRows && S::kWarps > 8 ? 64 : BackwardBatch<TS, PPT>::value;
  // per (warp, batch entry) reduced vectors of the deterministic form
  __shared__ float s_part[kRows ? S::kWarps : 1][kRows ? NB : 1][9];
  if constexpr (kRows) {
    for (int i = threadIdx.x; i < S::kWarps * NB * 9; i += S::kThreads) (&s_part[0][0][0])[i] = 0.0f;
  }
  constexpr int Q = S::kPpt;
  constexpr int kStage = (NB + S::kThreads - 1) / S::kThreads;  // entries staged per thread
  constexpr unsigned kMask = S::kWarpMask;
  constexpr int kBuffers = kBackwardDoubleBuffer ? 2 : 1;
  __shared__ StageBuffer<NB> s_buf[kBuffers];
  __shared__ uint16_t s_list[S::kWarps][NB];
  __shared__ int s_max_contrib;
  int4 item = make_int4(0, 0, 1, 0);  // (tile, part, parts, -)
  if (items != nullptr)
    item = items[blockIdx.x];
  else
    item.x = visit_tile(tile_order, p);
  const int tile = item.x;
  if (tile < 0) return;
  const int part = item.y, parts = item.z;
  const int tid = threadIdx.x;
  const int lane = tid % S::kWarpLanes, warp = tid / S::kWarpLanes;
  const PixelMap<TS, PPT> pm(tile, p.width / TS, tid);
  const float fpx = static_cast<float>(pm.px);
  const float threshold = p.opacity_threshold;
  float fpy[Q], gr[Q], gg[Q], gb[Q], t_final[Q];
  int contrib[Q];
  int my_max = 0;
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    fpy[q] = static_cast<float>(pm.py(q));
    const int64_t pix = static_cast<int64_t>(pm.py(q)) * p.width + pm.px;
    gr[q] = __ldg(grad_image + 3 * pix);
    gg[q] = __ldg(grad_image + 3 * pix + 1);
    gb[q] = __ldg(grad_image + 3 * pix + 2);
    t_final[q] = __ldg(final_transmittance + pix);
    contrib[q] = __ldg(n_contributors + pix);
    my_max = contrib[q] > my_max ? contrib[q] : my_max;
  }
  if (tid == 0) s_max_contrib = 0;
  __syncthreads();
  const int warp_max_contrib = __reduce_max_sync(kMask, my_max);
  if (lane == 0) atomicMax(&s_max_contrib, warp_max_contrib);
  __syncthreads();
  const int64_t start = ranges[2 * tile];
  int64_t end = ranges[2 * tile + 1];
  if (end > start + s_max_contrib) end = start + s_max_contrib;  // composite_bwd.py:81-83
  // This CTA's part of the walk: [part_lo, part_hi) back to front (the
  // whole walk unless the tile is split; positions stay relative to the
  // tile's start), after the suffix of [part_hi, end).
  int64_t part_lo = start, part_hi = end;
  if (parts > 1) {
    const int64_t chunk = (end - start + parts - 1) / parts;
    part_lo = start + part * chunk < end ? start + part * chunk : end;
    part_hi = part_lo + chunk < end ? part_lo + chunk : end;
  }
  uint16_t* list = s_list[warp];
  float st[Q], sr[Q], sg[Q], sb[Q];  // suffix behind the current entry
#pragma unroll
  for (int q = 0; q < Q; ++q) {
    st[q] = 1.0f;
    sr[q] = sg[q] = sb[q] = 0.0f;
  }
  // One walk over [lo, hi) back to front; with a SuffixPass tag the suffix
  // recurrence only.
  auto walk = [&](auto pass, const int64_t lo, const int64_t hi) {
  constexpr bool kSuffix = decltype(pass)::value;
  const int64_t end = hi;

  // Batches walk back to front: [max(start, batch_end - NB), batch_end). Slot
  // tid + s * kThreads of each batch is this thread's to stage; the ids of its
  // next batch's slots are loaded one batch ahead.
  int32_t next_id[kStage];
  {
    const int64_t first = end - NB > lo ? end - NB : lo;
#pragma unroll
    for (int s = 0; s < kStage; ++s) {
      const int slot = tid + s * S::kThreads;
      if (slot < NB && first + slot < end)
        stage_async(records, __ldg(gaussian_ids + first + slot), s_buf[0], slot);
      const int64_t first2 = first - NB > lo ? first - NB : lo;
      next_id[s] = slot < NB && first2 + slot < first ? __ldg(gaussian_ids + first2 + slot) : 0;
    }
  }
  cp_async_commit();
  cp_async_wait_all();
  __syncthreads();

  int buf = 0;
  for (int64_t batch_end = end; batch_end > lo;
       batch_end -= NB, buf = kBackwardDoubleBuffer ? buf ^ 1 : 0) {
    const int64_t batch_start = batch_end - NB > lo ? batch_end - NB : lo;
    // the next (earlier) batch's records fill the other buffer meanwhile
    if (kBackwardDoubleBuffer && batch_start > lo) {
      const int64_t next_start = batch_start - NB > lo ? batch_start - NB : lo;
      const int64_t after_start = next_start - NB > lo ? next_start - NB : lo;
#pragma unroll
      for (int s = 0; s < kStage; ++s) {
        const int slot = tid + s * S::kThreads;
        if (slot < NB && next_start + slot < batch_start) {
          stage_async(records, next_id[s], s_buf[buf ^ 1], slot);
          if (after_start + slot < next_start)
            next_id[s] = __ldg(gaussian_ids + after_start + slot);
        }
      }
    }
    cp_async_commit();
    const StageBuffer<NB>& cur = s_buf[buf];
    const int count = static_cast<int>(batch_end - batch_start);
    const int selected = warp_select<TS, PPT, true>(pm, cur, count, lane, list,
                                                    batch_start - start, warp_max_contrib);
    for (int i = selected - 1; i >= 0; --i) {
      const int j = list[i];
      const int64_t position = batch_start + j - start;
      float v[9];
#pragma unroll
      for (int k = 0; k < 9; ++k) v[k] = 0.0f;
      bool active = false;
      const float4 a = cur.a[j];
      const float4 b = cur.b[j];
      const float dx = fpx - a.x;
      const float xx = a.z, xy = b.w, yy = b.x, o = b.y;
      (void)xy;  // (not read by the ellipsoid suffix pass)
      const float adx = xx * dx, bdx = a.w * dx;
#pragma unroll
      for (int q = 0; q < Q; ++q) {
        if (!(position < contrib[q])) continue;
        const float dy = fpy[q] - a.y;
        const float d2 = fmaf(adx, dx, fmaf(bdx, dy, (yy * dy) * dy));
        if (!(d2 <= b.z)) continue;
        // Ellipsoid mode: the falloff is the indicator of d2 <= cutoff (the
        // test above), whose derivative is zero, so only colour and opacity
        // get gradients.
        float prob = 1.0f;
        if constexpr (kGaussian)
          prob = d2 >= 0.0f ? det_exp_nonpositive(-0.5f * d2) : det_exp(-0.5f * d2);
        const float alpha_raw = o * prob;
        const float alpha = fminf(alpha_raw, kAlphaMax);
        if (!(alpha >= kAlphaMin)) continue;
        active = true;
        const float4 c = cur.c[j];
        if constexpr (kSuffix) {  // the recurrence only (same expressions as below)
          const float local_t = 1.0f - alpha;
          sr[q] = fmaf(local_t, sr[q], alpha * c.x);
          sg[q] = fmaf(local_t, sg[q], alpha * c.y);
          sb[q] = fmaf(local_t, sb[q], alpha * c.z);
          st[q] = st[q] * local_t;
          continue;
        }
        const float denominator = fmaxf(st[q] * (1.0f - alpha), 1e-4f);
        // T in front of the entry. The quotient only feeds gradients and the
        // termination re-test of the gradient path (tolerance-checked), so it
        // takes the approximate divide (<= 2 ulp, as a Triton fp32 `/` without
        // IEEE rounding does on the reference's GPU path) instead of the
        // IEEE one's ~10 instructions; denominator >= 1e-4 keeps it in range.
        const float forward = __fdividef(t_final[q], denominator);
        const bool still = (1.0f - forward) < threshold;
        // Gradient arithmetic (tolerance-checked, unlike the decisions above)
        // contracts multiply-adds explicitly.
        float weight_grad = gr[q] * (c.x - sr[q]);
        weight_grad = fmaf(gg[q], c.y - sg[q], weight_grad);
        weight_grad = fmaf(gb[q], c.z - sb[q], weight_grad);
        float grad_alpha = still ? forward * weight_grad : 0.0f;
        grad_alpha = alpha_raw < kAlphaMax ? grad_alpha : 0.0f;
        const float grad_color = forward * alpha;
        if constexpr (kGaussian) {
          const float grad_distance = -0.5f * prob * (grad_alpha * o);
          const float gdx = grad_distance * dx, gdy = grad_distance * dy;
          v[0] = fmaf(-2.0f * grad_distance, fmaf(xy, dy, adx), v[0]);
          v[1] = fmaf(-2.0f * grad_distance, fmaf(yy, dy, xy * dx), v[1]);
          v[2] = fmaf(gdx, dx, v[2]);
          v[3] = fmaf(gdx, dy, v[3]);
          v[4] = fmaf(gdy, dy, v[4]);
        }
        v[5] = fmaf(grad_color, gr[q], v[5]);
        v[6] = fmaf(grad_color, gg[q], v[6]);
        v[7] = fmaf(grad_color, gb[q], v[7]);
        v[8] = fmaf(grad_alpha, prob, v[8]);
        const float local_t = 1.0f - alpha;
        sr[q] = fmaf(local_t, sr[q], alpha * c.x);
        sg[q] = fmaf(local_t, sg[q], alpha * c.y);
        sb[q] = fmaf(local_t, sb[q], alpha * c.z);
        st[q] = st[q] * local_t;
      }
      if (!kSuffix && __any_sync(kMask, active)) {
        const int g = __float_as_int(cur.c[j].w);
        float* dst = kRows ? s_part[kRows ? warp : 0][kRows ? j : 0]
                           : grad_projected + 9 * static_cast<int64_t>(g);
        if constexpr (S::kWarpLanes == 32) {
          float mine, last;
          warp_reduce_scatter9(v, lane, mine, last);
          if constexpr (kRows) {
            if ((lane & 3) == 0) dst[lane >> 2] = mine;
            if (lane == 1) dst[8] = last;
          } else {
            if ((lane & 3) == 0) atomicAdd(dst + (lane >> 2), mine);
            if (lane == 1) atomicAdd(dst + 8, last);
          }
        } else {
#pragma unroll
          for (int k = 0; k < 9; ++k) {
#pragma unroll
            for (int off = S::kWarpLanes / 2; off > 0; off >>= 1)
              v[k] += __shfl_xor_sync(kMask, v[k], off);
          }
          if (lane == 0) {
#pragma unroll
            for (int k = 0; k < 9; ++k) {
              if constexpr (kRows)
                dst[k] = v[k];
              else
                atomicAdd(dst + k, v[k]);
            }
          }
        }
      }
    }
    if constexpr (kRows) {
      // every warp's vectors of this batch are in; one row per position, the
      // warps added in order, then the slots cleared for the next batch
      __syncthreads();
      for (int i = threadIdx.x; i < count * 9; i += S::kThreads) {
        const int j = i / 9, k = i % 9;
        float sum = 0.0f;
#pragma unroll
        for (int w = 0; w < S::kWarps; ++w) {
          sum += s_part[w][j][k];
          s_part[w][j][k] = 0.0f;
        }
        grad_projected[9 * (batch_start + j) + k] = sum;
      }
    }
    if constexpr (kBackwardDoubleBuffer) {
      cp_async_wait_all();
      __syncthreads();
    } else {
      // one buffer: refill it once every warp is done with it
      __syncthreads();
      if (batch_start > lo) {
        const int64_t next_start = batch_start - NB > lo ? batch_start - NB : lo;
        const int64_t after_start = next_start - NB > lo ? next_start - NB : lo;
#pragma unroll
        for (int s = 0; s < kStage; ++s) {
          const int slot = tid + s * S::kThreads;
          if (slot < NB && next_start + slot < batch_start) {
            stage_async(records, next_id[s], s_buf[0], slot);
            if (after_start + slot < next_start)
              next_id[s] = __ldg(gaussian_ids + after_start + slot);
          }
        }
      }
      cp_async_commit();
      cp_async_wait_all();
      __syncthreads();
    }
  }
  };  // walk
  if (part_hi < end) walk(SuffixPass{}, part_hi, end);
  walk(GradientPass{}, part_lo, part_hi);
}

// Pixels per thread of the backward: two, so one warp reduction and one set
// of atomics per Gaussian covers an 8x8 block (the forward keeps one pixel per
// thread; its early exit and 8x4 warp blocks cull best).
#ifndef GS_BWD_PPT
#define GS_BWD_PPT 2
#endif
template <int TS>
struct BwdPpt {
  static constexpr int value = TS * TS / GS_BWD_PPT >= 16 ? GS_BWD_PPT : 1;
};

}  // namespace

#define GS_TILE_DISPATCH(ts, LAUNCH)      \
  switch (ts) {                            \
    case 4: LAUNCH(4); break;              \
    case 8: LAUNCH(8); break;              \
    case 16: LAUNCH(16); break;            \
    case 32: LAUNCH(32); break;            \
    default: return GS_ERR_INVALID_ARGUMENT; \
  }

// Records [n, 4] float4 of the projected Gaussians (the compositors' staged
// form), from the four projected arrays: for callers that have only the
// operator's outputs.
__global__ void __launch_bounds__(256) pack_records_kernel(
    int64_t n, const float* __restrict__ projected_mean,
    const float* __restrict__ inverse_covariance, const float* __restrict__ projected_color,
    const float* __restrict__ projected_opacity, const gs_params p, float4* __restrict__ records) {
  chain_wait();
  const int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (g >= n) return;
  const float4 conic = __ldg(reinterpret_cast<const float4*>(inverse_covariance) + g);
  store_record(records, g,
               make_record(static_cast<int32_t>(g), __ldg(projected_mean + 3 * g),
                           __ldg(projected_mean + 3 * g + 1), conic,
                           __ldg(projected_opacity + g), __ldg(projected_color + 3 * g),
                           __ldg(projected_color + 3 * g + 1), __ldg(projected_color + 3 * g + 2),
                           p));
}

int32_t launch_pack_records(int64_t n, const float* projected_mean,
                            const float* inverse_covariance, const float* projected_color,
                            const float* projected_opacity, const gs_params& p, float* records,
                            cudaStream_t stream) {
  if (n == 0) return GS_OK;
  launch_chained(pack_records_kernel, ceil_div(n, 256), 256, stream,
      n, projected_mean, inverse_covariance, projected_color, projected_opacity, p,
      reinterpret_cast<float4*>(records));
  return check_launch();
}

// Deterministic backward, second step: grad_projected[g] = the sum of g's
// rows in increasing list position (order: positions grouped by Gaussian;
// segments: each Gaussian's [start, end) in order).
__global__ void __launch_bounds__(256) reduce_rows_kernel(
    int64_t n, const uint32_t* __restrict__ order, const int64_t* __restrict__ segments,
    const float* __restrict__ rows, float* __restrict__ grad_projected) {
  chain_wait();
  const int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (g >= n) return;
  float acc[9] = {};
  const int64_t end = segments[2 * g + 1];
  for (int64_t k = segments[2 * g]; k < end; ++k) {
    const float* row = rows + 9 * static_cast<int64_t>(__ldg(order + k));
#pragma unroll
    for (int c = 0; c < 9; ++c) acc[c] += __ldg(row + c);
  }
#pragma unroll
  for (int c = 0; c < 9; ++c) grad_projected[9 * g + c] = acc[c];
}

// ------------------------------------------------------ heavy-first tile order
//
// The compositors take a tile per CTA in CTA order. Tile costs are very
// uneven (config 5's densest tile walks 850k pixel-Gaussian pairs, the mean
// 47k; alone it takes half the backward's time), and in row-major order the
// heavy central tiles start mid-launch on SMs already full of other tiles, so
// they finish last. Visiting tiles by decreasing work starts them first.
// Work classes are a quarter octave wide; order within a class is arbitrary
// (no result depends on which CTA composites a tile).

constexpr int kWorkClasses = 64;

// Lanes of the warp holding the same class as this lane (classes 0..64, 64
// marking no tile): one ballot per bit, cheaper than a match instruction.
__device__ __forceinline__ unsigned same_class_lanes(int c) {
  unsigned peers = 0xffffffffu;
#pragma unroll
  for (int bit = 0; bit < 7; ++bit) {
    const bool set = (c >> bit) & 1;
    const unsigned vote = __ballot_sync(0xffffffffu, set);
    peers &= set ? vote : ~vote;
  }
  return peers;
}

// 0 for no work, else 1 + 4 floor(log2 w) + the two bits of w below its
// leading one, capped at 63.
__device__ __forceinline__ int work_class(uint32_t w) {
  if (w == 0) return 0;
  const int b = 31 - __clz(w);
  const int frac = b >= 2 ? static_cast<int>((w >> (b - 2)) & 3u) : static_cast<int>((w << (2 - b)) & 3u);
  const int c = 1 + 4 * b + frac;
  return c < kWorkClasses - 1 ? c : kWorkClasses - 1;
}

__device__ __forceinline__ uint32_t tile_work(const int64_t* __restrict__ ranges,
                                              const uint32_t* __restrict__ work, int64_t t) {
  if (work) return __ldg(work + t);
  const int64_t len = ranges[2 * t + 1] - ranges[2 * t];
  return len <= 0 ? 0u : (len >= 0xffffffffLL ? 0xffffffffu : static_cast<uint32_t>(len));
}

// Class counts: one thread per tile; the lanes of a warp holding the same
// class are found by ballots and their leader adds them with one atomic.
__global__ void __launch_bounds__(256) order_count_kernel(const int64_t* __restrict__ ranges,
                                                          const uint32_t* __restrict__ work,
                                                          int64_t num_tiles,
                                                          uint32_t* __restrict__ hist) {
  chain_wait();
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int c = t < num_tiles ? work_class(tile_work(ranges, work, t)) : kWorkClasses;
  const unsigned peers = same_class_lanes(c);
  if (c < kWorkClasses && (peers & ((1u << lane) - 1u)) == 0) atomicAdd(hist + c, __popc(peers));
}

// The first place of each class, heaviest class first, from the counts (one
// warp: two classes per lane); *total gets the number of places.
__device__ __forceinline__ void class_starts(const uint32_t* __restrict__ hist, uint32_t* s_start,
                                             uint32_t* total) {
  const int lane = threadIdx.x & 31;
  const uint32_t a = hist[kWorkClasses - 1 - 2 * lane], b = hist[kWorkClasses - 2 - 2 * lane];
  uint32_t incl = a + b;
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const uint32_t excl = incl - a - b;
  s_start[kWorkClasses - 1 - 2 * lane] = excl;
  s_start[kWorkClasses - 2 - 2 * lane] = excl + a;
  if (total) *total = __shfl_sync(0xffffffffu, incl, 31);
}

// Each tile's place in the order: its class's start plus a per-class cursor
// (one atomic per class and warp).
__global__ void __launch_bounds__(256) order_scatter_kernel(
    const int64_t* __restrict__ ranges, const uint32_t* __restrict__ work, int64_t num_tiles,
    const uint32_t* __restrict__ hist, uint32_t* __restrict__ cursor,
    int32_t* __restrict__ order) {
  chain_wait();
  __shared__ uint32_t s_start[kWorkClasses];
  if (threadIdx.x < 32) class_starts(hist, s_start, nullptr);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int c = t < num_tiles ? work_class(tile_work(ranges, work, t)) : kWorkClasses;
  const unsigned peers = same_class_lanes(c);
  const int leader = __ffs(peers) - 1;
  uint32_t base = 0;
  if (c < kWorkClasses && lane == leader) base = atomicAdd(cursor + c, __popc(peers));
  base = __shfl_sync(0xffffffffu, base, leader);
  if (c < kWorkClasses)
    order[s_start[c] + base + __popc(peers & ((1u << lane) - 1u))] = static_cast<int32_t>(t);
}

// The backward's work per tile: its largest contributor count (the backward
// walks each tile's list that far). One warp per tile.
__global__ void __launch_bounds__(256) tile_max_contrib_kernel(
    const int32_t* __restrict__ n_contributors, int width, int tile_size, int tiles_w,
    int64_t num_tiles, uint32_t* __restrict__ work) {
  chain_wait();
  const int64_t t = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= num_tiles) return;
  const int x0 = static_cast<int>(t % tiles_w) * tile_size;
  const int y0 = static_cast<int>(t / tiles_w) * tile_size;
  int m = 0;
#pragma unroll 4
  for (int k = lane; k < tile_size * tile_size; k += 32) {
    const int v = __ldg(n_contributors + static_cast<int64_t>(y0 + k / tile_size) * width + x0 +
                        k % tile_size);
    m = v > m ? v : m;
  }
  m = __reduce_max_sync(0xffffffffu, m);
  if (lane == 0) work[t] = static_cast<uint32_t>(m);
}

// ------------------------------------------------ split backward: the plan
//
// The backward's plan of one view: its work items heavy first -- every tile,
// and the tiles whose walk (list length up to the largest contributor count)
// exceeds split_walk entries cut into parts of at most that many (part k's
// CTA also walks the parts behind it for its suffix, at about a third of the
// per-entry cost, which sets its place in the order). Layout (256-byte
// aligned parts): header (items, extra parts; class counts, class cursors and
// the extra-part counter at words 16, 80 and 144) | items int4 [tiles +
// kExtraParts] | tile parts int2 [tiles] | work uint32 [tiles]. Tiles left
// once kExtraParts parts beyond the tiles' first ones are handed out stay
// whole.

constexpr int kExtraParts = 1024;
constexpr int kMaxSplitParts = 64;
// Default split threshold. Measured on the dense config-5 view (densest
// walk 5,217 entries): 384-768 -> 1.064-1.069 ms per step, 1024 -> 1.049,
// 2048 -> 1.016, 3072 -> 1.028, 4096 -> 1.041, 6144 -> 1.051; more parts
// shorten the longest CTA but repeat more suffix walks on an already busy
// GPU. Views whose walks all stay below it (config 2: 1,116) are unchanged.
constexpr int kDefaultSplitWalk = 2048;

struct BwdPlanLayout {
  uint64_t header, items, tile_parts, work, bytes;
  explicit BwdPlanLayout(int64_t num_tiles) {
    auto align = [](uint64_t x) { return (x + 255) / 256 * 256; };
    const uint64_t t = static_cast<uint64_t>(num_tiles);
    uint64_t at = 0;
    header = at; at = align(at + 1024);
    items = at; at = align(at + 16 * (t + kExtraParts));
    tile_parts = at; at = align(at + 8 * t);
    work = at; at = align(at + 4 * t);
    bytes = at;
  }
};

// A tile's walk: its list up to its largest contributor count.
__device__ __forceinline__ uint32_t tile_walk(const int64_t* __restrict__ ranges,
                                              const uint32_t* __restrict__ max_contrib,
                                              int64_t t) {
  const int64_t len = ranges[2 * t + 1] - ranges[2 * t];
  const int64_t m = static_cast<int64_t>(__ldg(max_contrib + t));
  const int64_t w = len < m ? len : m;
  return w <= 0 ? 0u : static_cast<uint32_t>(w);
}

// Work of part k of a tile cut into `parts` parts of `chunk` entries: its own
// walk plus a third of each entry behind it.
__device__ __forceinline__ uint32_t part_work(uint32_t chunk, int part, int parts) {
  return chunk + static_cast<uint32_t>(parts - 1 - part) * chunk / 3;
}

// The plan's class counts: one thread per tile decides its parts (an extra
// part is one more CTA; kExtraParts of them per view) and counts its items --
// whole tiles by their leader's one atomic per warp and class, the parts of a
// split tile each by its own.
__global__ void __launch_bounds__(256) plan_count_kernel(
    const int64_t* __restrict__ ranges, const uint32_t* __restrict__ max_contrib,
    int64_t num_tiles, int split_walk, uint32_t* __restrict__ hist,
    uint32_t* __restrict__ extra, int2* __restrict__ tile_parts) {
  chain_wait();
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint32_t walk = t < num_tiles ? tile_walk(ranges, max_contrib, t) : 0u;
  int parts = 1;
  if (t < num_tiles && walk > static_cast<uint32_t>(split_walk)) {
    const uint32_t want = (walk + split_walk - 1) / split_walk;
    parts = want < kMaxSplitParts ? static_cast<int>(want) : kMaxSplitParts;
    const uint32_t first = atomicAdd(extra, static_cast<uint32_t>(parts - 1));
    if (first + parts - 1 > kExtraParts) parts = 1;  // out of parts: stays whole
  }
  if (t < num_tiles) tile_parts[t] = make_int2(parts, 0);
  const bool whole = t < num_tiles && parts == 1;
  const int c = whole ? work_class(walk) : kWorkClasses + 1 + lane % 31;
  const unsigned peers = same_class_lanes(c);
  if (whole && (peers & ((1u << lane) - 1u)) == 0) atomicAdd(hist + c, __popc(peers));
  if (t < num_tiles && parts > 1) {
    const uint32_t chunk = (walk + parts - 1) / parts;
    for (int k = 0; k < parts; ++k) atomicAdd(hist + work_class(part_work(chunk, k, parts)), 1u);
  }
}

// The plan's items: each tile's (or part's) place is its class's start plus
// a per-class cursor; the places past the last item are marked empty.
__global__ void __launch_bounds__(256) plan_scatter_kernel(
    const int64_t* __restrict__ ranges, const uint32_t* __restrict__ max_contrib,
    int64_t num_tiles, const uint32_t* __restrict__ hist, uint32_t* __restrict__ cursor,
    const uint32_t* __restrict__ extra, const int2* __restrict__ tile_parts,
    int4* __restrict__ items, uint32_t* __restrict__ header) {
  chain_wait();
  __shared__ uint32_t s_start[kWorkClasses];
  __shared__ uint32_t s_total;
  if (threadIdx.x < 32) class_starts(hist, s_start, &s_total);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const uint32_t walk = t < num_tiles ? tile_walk(ranges, max_contrib, t) : 0u;
  const int parts = t < num_tiles ? tile_parts[t].x : 1;
  const bool whole = t < num_tiles && parts == 1;
  const int c = whole ? work_class(walk) : kWorkClasses + 1 + lane % 31;
  const unsigned peers = same_class_lanes(c);
  const int leader = __ffs(peers) - 1;
  uint32_t base = 0;
  if (whole && lane == leader) base = atomicAdd(cursor + c, __popc(peers));
  base = __shfl_sync(0xffffffffu, base, leader);
  if (whole)
    items[s_start[c] + base + __popc(peers & ((1u << lane) - 1u))] =
        make_int4(static_cast<int>(t), 0, 1, 0);
  if (t < num_tiles && parts > 1) {
    const uint32_t chunk = (walk + parts - 1) / parts;
    for (int k = 0; k < parts; ++k) {
      const int ck = work_class(part_work(chunk, k, parts));
      items[s_start[ck] + atomicAdd(cursor + ck, 1u)] = make_int4(static_cast<int>(t), k, parts, 0);
    }
  }
  const uint32_t total = s_total;
  for (int64_t i = total + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < num_tiles + kExtraParts; i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    items[i] = make_int4(-1, 0, 1, 0);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    header[0] = total;
    header[1] = *extra < kExtraParts ? *extra : kExtraParts;
  }
}

uint64_t composite_bwd_plan_size(const gs_params& p) {
  const int64_t num_tiles =
      static_cast<int64_t>(p.width / p.tile_size) * (p.height / p.tile_size);
  return BwdPlanLayout(num_tiles).bytes;
}

int32_t launch_composite_bwd_plan(const int64_t* ranges, const int32_t* n_contributors,
                                  const gs_params& p, int split_walk, void* plan,
                                  cudaStream_t stream) {
  const int tiles_w = p.width / p.tile_size;
  const int64_t num_tiles = static_cast<int64_t>(tiles_w) * (p.height / p.tile_size);
  const BwdPlanLayout L(num_tiles);
  char* base = static_cast<char*>(plan);
  if (num_tiles == 0) return GS_OK;
  uint32_t* work = reinterpret_cast<uint32_t*>(base + L.work);
  uint32_t* header = reinterpret_cast<uint32_t*>(base + L.header);
  GS_CUDA_TRY(cudaMemsetAsync(header, 0, 1024, stream));
  launch_chained(tile_max_contrib_kernel, ceil_div(num_tiles * 32, 256), 256, stream,
      n_contributors, p.width, p.tile_size, tiles_w, num_tiles, work);
  GS_TRY(check_launch());
  int2* tile_parts = reinterpret_cast<int2*>(base + L.tile_parts);
  const int walk = split_walk > 0 ? split_walk : kDefaultSplitWalk;
  launch_chained(plan_count_kernel, ceil_div(num_tiles, 256), 256, stream,
      ranges, work, num_tiles, walk, header + 16, header + 144, tile_parts);
  GS_TRY(check_launch());
  launch_chained(plan_scatter_kernel, ceil_div(num_tiles, 256), 256, stream,
      ranges, work, num_tiles, header + 16, header + 80, header + 144, tile_parts,
      reinterpret_cast<int4*>(base + L.items), header);
  return check_launch();
}

// tile_work: [num_tiles] per-tile work (the backward's form), then class
// counts and cursors [2 x kWorkClasses].
int32_t launch_tile_order(const int64_t* ranges, const int32_t* n_contributors,
                          const gs_params& p, int32_t* order, uint32_t* tile_work,
                          cudaStream_t stream) {
  const int tiles_w = p.width / p.tile_size;
  const int64_t num_tiles = static_cast<int64_t>(tiles_w) * (p.height / p.tile_size);
  if (num_tiles == 0) return GS_OK;
  uint32_t* hist = tile_work + num_tiles;
  GS_CUDA_TRY(cudaMemsetAsync(hist, 0, 2 * kWorkClasses * sizeof(uint32_t), stream));
  const uint32_t* work = nullptr;
  if (n_contributors != nullptr) {
    launch_chained(tile_max_contrib_kernel, ceil_div(num_tiles * 32, 256), 256, stream,
        n_contributors, p.width, p.tile_size, tiles_w, num_tiles, tile_work);
    GS_TRY(check_launch());
    work = tile_work;
  }
  launch_chained(order_count_kernel, ceil_div(num_tiles, 256), 256, stream, ranges, work,
                 num_tiles, hist);
  GS_TRY(check_launch());
  launch_chained(order_scatter_kernel, ceil_div(num_tiles, 256), 256, stream,
      ranges, work, num_tiles, hist, hist + kWorkClasses, order);
  return check_launch();
}

int32_t launch_composite_fwd(const float* records, const int32_t* gaussian_ids,
                             const int64_t* ranges, const gs_params& p, float* image,
                             float* final_transmittance, int32_t* n_contributors,
                             const int32_t* tile_order, cudaStream_t stream) {
  const int64_t num_tiles =
      static_cast<int64_t>(p.width / p.tile_size) * (p.height / p.tile_size);
  if (num_tiles == 0) return GS_OK;
  const float4* rec = reinterpret_cast<const float4*>(records);
#define GS_LAUNCH(TS)                                                                          \
  if (p.gaussian_mode)                                                                         \
    launch_chained(composite_fwd_kernel<TS, true>, static_cast<unsigned>(num_tiles), TS * TS,   \
                   stream, rec, gaussian_ids, ranges, p, image, final_transmittance,            \
                   n_contributors, tile_order);                                                 \
  else                                                                                          \
    launch_chained(composite_fwd_kernel<TS, false>, static_cast<unsigned>(num_tiles), TS * TS,  \
                   stream, rec, gaussian_ids, ranges, p, image, final_transmittance,            \
                   n_contributors, tile_order)
  GS_TILE_DISPATCH(p.tile_size, GS_LAUNCH)
#undef GS_LAUNCH
  return check_launch();
}

int32_t launch_composite_bwd(int64_t n, const float* records, const int32_t* gaussian_ids,
                             const int64_t* ranges, const float* grad_image,
                             const float* final_transmittance, const int32_t* n_contributors,
                             const gs_params& p, float* grad_projected, void* plan,
                             cudaStream_t stream) {
  GS_CUDA_TRY(cudaMemsetAsync(grad_projected, 0, sizeof(float) * 9 * n, stream));
  const int64_t num_tiles =
      static_cast<int64_t>(p.width / p.tile_size) * (p.height / p.tile_size);
  if (num_tiles == 0 || n == 0) return GS_OK;
  const float4* rec = reinterpret_cast<const float4*>(records);
  const BwdPlanLayout L(num_tiles);
  const int4* items =
      plan ? reinterpret_cast<const int4*>(static_cast<char*>(plan) + L.items) : nullptr;
  const unsigned grid = static_cast<unsigned>(plan ? num_tiles + kExtraParts : num_tiles);
#define GS_LAUNCH_MODE(TS, G)                                                                  \
  launch_chained(composite_bwd_kernel<TS, BwdPpt<TS>::value, G>,                                \
                 grid, TileShape<TS, BwdPpt<TS>::value>::kThreads, stream,                      \
                 rec, gaussian_ids, ranges, grad_image, final_transmittance, n_contributors, p, \
                 grad_projected, nullptr, items)
#define GS_LAUNCH(TS)                 \
  if (p.gaussian_mode)                \
    GS_LAUNCH_MODE(TS, true);         \
  else                                \
    GS_LAUNCH_MODE(TS, false)
  GS_TILE_DISPATCH(p.tile_size, GS_LAUNCH)
#undef GS_LAUNCH
#undef GS_LAUNCH_MODE
  return check_launch();
}

// Deterministic backward workspace: rows [total, 9] float, order [total]
// uint32, segments [n, 2] int64, then the position sort's scratch.
struct DeterministicLayout {
  uint64_t rows, order, segments, sort, bytes;
  DeterministicLayout(int64_t n, int64_t total) {
    auto align = [](uint64_t x) { return (x + 255) / 256 * 256; };
    uint64_t at = 0;
    rows = at; at = align(at + 36 * static_cast<uint64_t>(total));
    order = at; at = align(at + 4 * static_cast<uint64_t>(total));
    segments = at; at = align(at + 16 * static_cast<uint64_t>(n));
    sort = at; at = align(at + radix_sort_workspace_size(total, n));
    bytes = at;
  }
};

uint64_t composite_bwd_deterministic_workspace_size(int64_t n, int64_t total) {
  return DeterministicLayout(n, total).bytes;
}

int32_t launch_composite_bwd_deterministic(int64_t n, int64_t total, const float* records,
                                           const int32_t* gaussian_ids, const int64_t* ranges,
                                           const float* grad_image,
                                           const float* final_transmittance,
                                           const int32_t* n_contributors, const gs_params& p,
                                           void* workspace, float* grad_projected,
                                           const int32_t* tile_order, cudaStream_t stream) {
  const DeterministicLayout L(n, total);
  char* base = static_cast<char*>(workspace);
  float* rows = reinterpret_cast<float*>(base + L.rows);
  uint32_t* order = reinterpret_cast<uint32_t*>(base + L.order);
  int64_t* segments = reinterpret_cast<int64_t*>(base + L.segments);
  GS_CUDA_TRY(cudaMemsetAsync(rows, 0, 36 * static_cast<size_t>(total), stream));
  const int64_t num_tiles =
      static_cast<int64_t>(p.width / p.tile_size) * (p.height / p.tile_size);
  const float4* rec = reinterpret_cast<const float4*>(records);
  if (num_tiles > 0 && total > 0) {
#define GS_LAUNCH(TS)                                                                          \
  if (p.gaussian_mode)                                                                         \
    launch_chained(composite_bwd_kernel<TS, BwdPpt<TS>::value, true, true>,                     \
                   static_cast<unsigned>(num_tiles),                                            \
                   TileShape<TS, BwdPpt<TS>::value>::kThreads, stream, rec, gaussian_ids,       \
                   ranges, grad_image, final_transmittance, n_contributors, p, rows,            \
                   tile_order, nullptr);                                                        \
  else                                                                                         \
    launch_chained(composite_bwd_kernel<TS, BwdPpt<TS>::value, false, true>,                    \
                   static_cast<unsigned>(num_tiles),                                            \
                   TileShape<TS, BwdPpt<TS>::value>::kThreads, stream, rec, gaussian_ids,       \
                   ranges, grad_image, final_transmittance, n_contributors, p, rows,            \
                   tile_order, nullptr)
    GS_TILE_DISPATCH(p.tile_size, GS_LAUNCH)
#undef GS_LAUNCH
    GS_TRY(check_launch());
  }
  GS_TRY(launch_sort_positions(total, n, gaussian_ids, base + L.sort, order, segments, stream));
  if (n == 0) return GS_OK;
  launch_chained(reduce_rows_kernel, ceil_div(n, 256), 256, stream, n, order, segments, rows,
                 grad_projected);
  return check_launch();
}

}  // namespace gs
