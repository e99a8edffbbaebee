// Tile binning: which Gaussians touch which tile, in front-to-back order.
//
// The reference emits one int64 key (tile << 32 | depth bits) per
// (Gaussian, tile) pair in Gaussian order and sorts all of them
// (intersections.py:10-88): a 64-bit radix sort over every intersection.
// The same order -- by tile, then depth bits, then Gaussian index -- comes
// out of two much cheaper stable sorts:
//   1. sort only the Gaussians with count > 0 by their 32-bit depth bits
//      (stable, so equal depths keep index order);
//   2. emit every Gaussian's tiles in that depth order (tile id = key,
//      Gaussian = value) and stably sort by tile id, which needs only
//      ceil(log2(num_tiles)) bits (13 for 1080p at 16x16: two 8-bit passes).
// Within a tile the emission order is the depth order, and the stable tile
// sort keeps it.
//
// Both sorts are LSD radix sorts with 8-bit digits, one kernel per pass in
// the "onesweep" style: each CTA ranks a 4096-key tile in shared memory
// (warp-level ranking: the lanes holding the same digit are found with one
// ballot per digit bit, and lanes are ranked in order, which is stable),
// publishes its per-digit counts, computes its global offsets by decoupled
// look-back over the preceding CTAs (reading several predecessors' status
// words per round trip), and writes the keys out digit-grouped and
// coalesced. CTAs take their tile index from an atomic counter, so a CTA
// only ever waits on CTAs that already started. Every spin is bounded; on
// expiry the CTA records an error word and proceeds, so a fault costs a wrong
// result and an error code, never a hung GPU.
#include "common.cuh"

namespace gs {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kItems = 16;
constexpr int kTile = kThreads * kItems;  // 4096 keys per CTA
constexpr int kRadix = 256;
constexpr uint32_t kFlagAggregate = 1u << 30;
constexpr uint32_t kFlagPrefix = 2u << 30;
constexpr uint32_t kValueMask = (1u << 30) - 1;
constexpr uint64_t kScanFlagAggregate = 1ull << 62;
constexpr uint64_t kScanFlagPrefix = 2ull << 62;
constexpr uint64_t kScanValueMask = (1ull << 62) - 1;
constexpr int kSpinLimit = 1 << 22;  // with 64 ns backoff: ~0.3 s before giving up

// Error word bits (BinHeader::error).
constexpr uint32_t kErrLookbackTimeout = 1u;

__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) {
  return *reinterpret_cast<const volatile uint32_t*>(p);
}
__device__ __forceinline__ uint64_t ld_volatile(const uint64_t* p) {
  return *reinterpret_cast<const volatile uint64_t*>(p);
}
__device__ __forceinline__ void st_volatile(uint32_t* p, uint32_t v) {
  *reinterpret_cast<volatile uint32_t*>(p) = v;
}
__device__ __forceinline__ void st_volatile(uint64_t* p, uint64_t v) {
  *reinterpret_cast<volatile uint64_t*>(p) = v;
}

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Inputs of a sort pass. `valid(i)` filters elements (only the depth sort's
// first pass drops Gaussians with count 0); `key`/`value` read element i.
struct DepthSource {  // key = depth bits of projected_mean[i, 2], value = i
  const float* projected_mean;
  const int32_t* counts;
  static constexpr bool kWeighted = true;  // the upsweep also totals the tile counts
  __device__ __forceinline__ uint32_t weight(int64_t i) const {
    return static_cast<uint32_t>(__ldg(counts + i));
  }
  __device__ __forceinline__ bool valid(int64_t i) const { return __ldg(counts + i) > 0; }
  __device__ __forceinline__ uint32_t key(int64_t i) const {
    return __float_as_uint(__ldg(projected_mean + 3 * i + 2));
  }
  __device__ __forceinline__ uint32_t value(int64_t i) const { return static_cast<uint32_t>(i); }
  // Keys of elements [first, first + R) into keys[]; returns the valid mask.
  template <int R>
  __device__ __forceinline__ uint32_t load_run(int64_t first, int64_t n, uint32_t (&keys)[R]) const {
    uint32_t mask = 0;
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int64_t i = first + j;
      const bool ok = i < n && valid(i);
      keys[j] = ok ? key(i) : 0u;
      mask |= ok ? (1u << j) : 0u;
    }
    return mask;
  }
};

struct ArraySource {
  const uint32_t* keys;
  const uint32_t* values;
  static constexpr bool kWeighted = false;
  __device__ __forceinline__ bool valid(int64_t) const { return true; }
  __device__ __forceinline__ uint32_t key(int64_t i) const { return keys[i]; }
  __device__ __forceinline__ uint32_t value(int64_t i) const { return values[i]; }
  // Keys of elements [first, first + R) (first a multiple of R, R a multiple
  // of 4, the array 16-byte aligned: whole runs load as 16-byte vectors).
  template <int R>
  __device__ __forceinline__ uint32_t load_run(int64_t first, int64_t n, uint32_t (&keys)[R]) const {
    if (first + R <= n) {
#pragma unroll
      for (int j = 0; j < R; j += 4) {
        const uint4 v = *reinterpret_cast<const uint4*>(keys_ptr() + first + j);
        keys[j] = v.x;
        keys[j + 1] = v.y;
        keys[j + 2] = v.z;
        keys[j + 3] = v.w;
      }
      return R == 32 ? 0xffffffffu : (1u << R) - 1u;
    }
    uint32_t mask = 0;
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const bool ok = first + j < n;
      keys[j] = ok ? keys_ptr()[first + j] : 0u;
      mask |= ok ? (1u << j) : 0u;
    }
    return mask;
  }
  __device__ __forceinline__ const uint32_t* keys_ptr() const { return keys; }
};

// Positions 0..n-1 keyed by keys[i]: the first pass of the deterministic
// backward's grouping of list positions by Gaussian.
struct PositionSource {
  const uint32_t* keys;
  static constexpr bool kWeighted = false;
  __device__ __forceinline__ bool valid(int64_t) const { return true; }
  __device__ __forceinline__ uint32_t key(int64_t i) const { return keys[i]; }
  __device__ __forceinline__ uint32_t value(int64_t i) const { return static_cast<uint32_t>(i); }
  template <int R>
  __device__ __forceinline__ uint32_t load_run(int64_t first, int64_t n, uint32_t (&out)[R]) const {
    return ArraySource{keys, nullptr}.load_run<R>(first, n, out);
  }
};

// Element count of a pass: a host value, or a device word written earlier on
// the stream (the number of visible Gaussians), or the smaller of a host
// capacity and a device total (the intersection total, when the buffers were
// sized before the host knew it).
struct Count {
  int64_t host;
  const uint32_t* device;
  const int64_t* device_total = nullptr;
  __device__ __forceinline__ int64_t get() const {
    if (device) return *device;
    if (device_total) {
      const int64_t t = *device_total;
      return t < host ? t : host;
    }
    return host;
  }
};

// Per-digit histograms of every pass at once (the global digit offsets each
// pass needs), plus the number of valid elements. Each thread walks
// kUpsweepRun consecutive elements and adds runs of equal digits with one
// shared-memory atomic: neighbouring keys share their high digits (a
// Gaussian's tiles lie in few tile rows; depths share their exponent), which
// would otherwise put whole warps on one counter.
template <class Source, int kUpsweepRun>
__global__ void __launch_bounds__(kThreads) upsweep_kernel(Source src, Count count, int num_passes,
                                                          int shift0, uint32_t* __restrict__ hist,
                                                          uint32_t* __restrict__ valid_total,
                                                          unsigned long long* __restrict__ weight_total) {
  chain_wait();
  __shared__ uint32_t s_hist[4][kRadix];
  const int64_t n = count.get();
  for (int i = threadIdx.x; i < 4 * kRadix; i += kThreads) (&s_hist[0][0])[i] = 0;
  __syncthreads();
  uint32_t valid_here = 0;
  unsigned long long weight_here = 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads * kUpsweepRun;
  for (int64_t first = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) * kUpsweepRun;
       first < n; first += stride) {
    uint32_t keys[kUpsweepRun];
    uint32_t valid = src.load_run(first, n, keys);  // bit j: element first + j counts
    valid_here += __popc(valid);
    if constexpr (Source::kWeighted) {
#pragma unroll
      for (int j = 0; j < kUpsweepRun; ++j)
        if ((valid >> j) & 1u) weight_here += src.weight(first + j);
    }
    for (int p = 0; p < num_passes; ++p) {
      const int shift = shift0 + 8 * p;
      int current = -1;
      uint32_t run = 0;
#pragma unroll
      for (int j = 0; j < kUpsweepRun; ++j) {
        if (!((valid >> j) & 1u)) continue;
        const int digit = static_cast<int>((keys[j] >> shift) & 0xFFu);
        if (digit != current) {
          if (run) atomicAdd(&s_hist[p][current], run);
          current = digit;
          run = 0;
        }
        ++run;
      }
      if (run) atomicAdd(&s_hist[p][current], run);
    }
  }
  if (valid_total) {
    for (int o = 16; o > 0; o >>= 1) valid_here += __shfl_xor_sync(0xffffffffu, valid_here, o);
    if ((threadIdx.x & 31) == 0 && valid_here) atomicAdd(valid_total, valid_here);
  }
  if (weight_total) {
    for (int o = 16; o > 0; o >>= 1) weight_here += __shfl_xor_sync(0xffffffffu, weight_here, o);
    if ((threadIdx.x & 31) == 0 && weight_here) atomicAdd(weight_total, weight_here);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < num_passes * kRadix; i += kThreads) {
    const uint32_t c = (&s_hist[0][0])[i];
    if (c) atomicAdd(hist + i, c);
  }
}

// Block-wide exclusive scan of one value per thread (kThreads values).
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* s_tmp,
                                                         uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_tmp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < kWarps ? s_tmp[lane] : 0;
    for (int o = 1; o < kWarps; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kWarps) s_tmp[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const uint32_t warp_prefix = warp ? s_tmp[warp - 1] : 0;
  if (total) *total = s_tmp[kWarps - 1];
  __syncthreads();
  return warp_prefix + x - v;
}

// Decoupled look-back for one digit column of the status words: the sum of
// the predecessors' counts from block `b` down to the nearest inclusive
// prefix. The words of kLookback predecessors are loaded together, so a walk
// over many blocks that are still publishing costs one L2 round trip per
// kLookback blocks instead of one per block. Each wait is bounded; on expiry
// the error word is set and the walk stops.
constexpr int kLookback = 4;
__device__ __forceinline__ uint32_t lookback_window(const uint32_t* status, int d, int64_t b,
                                                    uint32_t* error, int64_t stride = kRadix) {
  uint32_t exclusive = 0;
  while (b >= 0) {
    uint32_t words[kLookback];
#pragma unroll
    for (int i = 0; i < kLookback; ++i)
      words[i] = b - i >= 0 ? ld_volatile(status + (b - i) * stride + d) : kFlagPrefix;
#pragma unroll
    for (int i = 0; i < kLookback; ++i) {
      int spins = 0;
      while ((words[i] >> 30) == 0) {
        if (++spins > kSpinLimit) {
          atomicOr(error, kErrLookbackTimeout);
          return exclusive;
        }
        if (spins > 64) __nanosleep(64);
        words[i] = ld_volatile(status + (b - i) * stride + d);
      }
      exclusive += words[i] & kValueMask;
      if ((words[i] >> 30) != 1) return exclusive;  // inclusive prefix (or block < 0)
    }
    b -= kLookback;
  }
  return exclusive;
}

// Lanes of the warp holding the same 9-bit label as this lane (8 digit bits
// plus the invalid marker kRadix): one ballot per bit.
__device__ __forceinline__ unsigned match_digit(int d) {
  unsigned peers = 0xffffffffu;
#pragma unroll
  for (int bit = 0; bit < 9; ++bit) {
    const bool set = (d >> bit) & 1;
    const unsigned vote = __ballot_sync(0xffffffffu, set);
    peers &= set ? vote : ~vote;
  }
  return peers;
}

// One stable LSD pass over 8 bits at `shift`.
template <class Source>
__global__ void __launch_bounds__(kThreads, 4) sort_pass_kernel(
    Source src, Count count, int shift, const uint32_t* __restrict__ pass_hist,
    uint32_t* __restrict__ status, uint32_t* __restrict__ tile_counter,
    uint32_t* __restrict__ keys_out, uint32_t* __restrict__ values_out,
    uint32_t* __restrict__ error) {
  chain_wait();
  __shared__ uint32_t s_warp_hist[kWarps][kRadix];
  __shared__ uint32_t s_local_start[kRadix];
  __shared__ uint32_t s_global_base[kRadix];
  __shared__ uint32_t s_keys[kTile];
  __shared__ uint32_t s_values[kTile];
  __shared__ uint32_t s_tmp[kWarps];
  __shared__ uint32_t s_block, s_total;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) s_block = atomicAdd(tile_counter, 1u);
  for (int i = threadIdx.x; i < kWarps * kRadix; i += kThreads) (&s_warp_hist[0][0])[i] = 0;
  __syncthreads();
  const uint32_t block = s_block;
  const int64_t n = count.get();
  const int64_t tile_start = static_cast<int64_t>(block) * kTile;
  if (tile_start >= n) return;  // uniform: every later tile is empty too

  // Rank: warp w owns keys [w*512, w*512+512) of the tile, 32 per step in
  // order, so (step, lane) order is input order and ranks are stable. Only
  // the keys are held while ranking (the values are read when they are
  // scattered), which keeps the pass at 64 registers and four CTAs per SM.
  uint32_t keys[kItems], ranks[kItems];
  uint32_t valid = 0;  // bit j: element j of this thread exists (and passes the filter)
  const unsigned lt = lanemask_lt();
  const int64_t thread_first = tile_start + warp * (kItems * 32) + lane;
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const int64_t idx = thread_first + j * 32;
    const bool ok = idx < n && src.valid(idx);
    keys[j] = ok ? src.key(idx) : 0u;
    valid |= ok ? (1u << j) : 0u;
  }
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const int d = (valid >> j) & 1u ? static_cast<int>((keys[j] >> shift) & 0xFF) : kRadix;
    const unsigned peers = match_digit(d);
    const int leader = __ffs(peers) - 1;
    uint32_t base = 0;
    if (lane == leader && d < kRadix) {
      base = s_warp_hist[warp][d];
      s_warp_hist[warp][d] = base + __popc(peers);
    }
    base = __shfl_sync(0xffffffffu, base, leader);
    ranks[j] = base + __popc(peers & lt);
    __syncwarp();
  }
  __syncthreads();

  // Per digit (thread d): warp offsets, block count, local start, global base.
  const int d = threadIdx.x;
  uint32_t block_count = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const uint32_t c = s_warp_hist[w][d];
    s_warp_hist[w][d] = block_count;
    block_count += c;
  }
  uint32_t* my_status = status + static_cast<int64_t>(block) * kRadix + d;
  st_volatile(my_status, (block == 0 ? kFlagPrefix : kFlagAggregate) | block_count);
  uint32_t exclusive = 0;
  if (block > 0) {
    exclusive = lookback_window(status, d, static_cast<int64_t>(block) - 1, error);
    st_volatile(my_status, kFlagPrefix | (exclusive + block_count));
  }
  // Global exclusive offset of digit d across the whole pass.
  const uint32_t digit_start = block_exclusive_scan(pass_hist[d], s_tmp, nullptr);
  s_global_base[d] = digit_start + exclusive;
  s_local_start[d] = block_exclusive_scan(block_count, s_tmp, &s_total);
  __syncthreads();

  // Reorder the tile in shared memory by digit, then write runs coalesced.
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    if ((valid >> j) & 1u) {
      const int dj = static_cast<int>((keys[j] >> shift) & 0xFF);
      const uint32_t pos = s_local_start[dj] + s_warp_hist[warp][dj] + ranks[j];
      s_keys[pos] = keys[j];
      s_values[pos] = src.value(thread_first + j * 32);
    }
  }
  __syncthreads();
  const uint32_t total = s_total;
  for (uint32_t k = threadIdx.x; k < total; k += kThreads) {
    const uint32_t key = s_keys[k];
    const int dk = (key >> shift) & 0xFF;
    const uint32_t out = s_global_base[dk] + (k - s_local_start[dk]);
    if (keys_out) keys_out[out] = key;
    values_out[out] = s_values[k];
  }
}

// Exclusive prefix sum of counts[ids[j]] for j < V (decoupled look-back).
// The last CTA writes the grand total.
__global__ void __launch_bounds__(kThreads) count_scan_kernel(
    const uint32_t* __restrict__ ids, const uint32_t* __restrict__ num_valid,
    const int32_t* __restrict__ counts, uint64_t* __restrict__ status,
    uint32_t* __restrict__ tile_counter, uint32_t* __restrict__ offsets,
    int64_t* __restrict__ total_out, uint32_t* __restrict__ error) {
  chain_wait();
  __shared__ uint32_t s_tmp[kWarps];
  __shared__ uint32_t s_block;
  __shared__ uint64_t s_exclusive;
  if (threadIdx.x == 0) s_block = atomicAdd(tile_counter, 1u);
  __syncthreads();
  const uint32_t block = s_block;
  const int64_t n = *num_valid;
  const int64_t tile_start = static_cast<int64_t>(block) * kTile;
  if (tile_start >= n) {
    if (block == 0 && threadIdx.x == 0) *total_out = 0;
    return;
  }
  // Thread t owns kItems consecutive elements.
  uint32_t c[kItems];
  uint32_t local = 0;
  const int64_t base = tile_start + static_cast<int64_t>(threadIdx.x) * kItems;
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const int64_t idx = base + j;
    c[j] = idx < n ? static_cast<uint32_t>(__ldg(counts + ids[idx])) : 0u;
    local += c[j];
  }
  uint32_t block_total;
  const uint32_t thread_prefix = block_exclusive_scan(local, s_tmp, &block_total);
  if (threadIdx.x < 32) {
    // Warp-wide look-back: lane l reads the status of block b - l; the
    // nearest inclusive prefix ends the walk, aggregates before it add up.
    const int lane = threadIdx.x;
    uint64_t* my_status = status + block;
    if (lane == 0)
      st_volatile(my_status, (block == 0 ? kScanFlagPrefix : kScanFlagAggregate) | block_total);
    uint64_t exclusive = 0;
    bool timed_out = false;
    for (int64_t b = static_cast<int64_t>(block) - 1; b >= 0 && !timed_out; b -= 32) {
      const int64_t mine = b - lane;
      uint64_t word = mine >= 0 ? ld_volatile(status + mine) : kScanFlagPrefix;
      int spins = 0;
      while ((word >> 62) == 0) {
        if (++spins > kSpinLimit) {
          atomicOr(error, kErrLookbackTimeout);
          word = kScanFlagPrefix;  // stop here; the result is flagged wrong
          timed_out = true;
          break;
        }
        if (spins > 64) __nanosleep(64);
        word = ld_volatile(status + mine);
      }
      const unsigned prefix_lanes = __ballot_sync(0xffffffffu, (word >> 62) != 1);
      timed_out = __any_sync(0xffffffffu, timed_out);
      // Lanes up to and including the nearest prefix contribute.
      const int stop = prefix_lanes ? __ffs(prefix_lanes) - 1 : 31;
      uint64_t v = lane <= stop ? (word & kScanValueMask) : 0;
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      exclusive += v;
      if (prefix_lanes) break;
    }
    if (lane == 0) {
      if (block > 0) st_volatile(my_status, kScanFlagPrefix | (exclusive + block_total));
      s_exclusive = exclusive;
      if (tile_start + kTile >= n) *total_out = static_cast<int64_t>(exclusive + block_total);
    }
  }
  __syncthreads();
  // Offsets are stored as 32 bits; totals of 2^30 and more are rejected on
  // the host before anything reads them.
  uint32_t run = static_cast<uint32_t>(s_exclusive) + thread_prefix;
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    const int64_t idx = base + j;
    if (idx < n) offsets[idx] = run;
    run += c[j];
  }
}

// Writes every (tile, Gaussian) pair of the depth-ordered Gaussians. A warp
// handles 32 consecutive Gaussians, whose outputs form one contiguous range;
// lanes stride over that range (each output finds its Gaussian by binary
// search over the warp's prefix sums), so writes are coalesced and a Gaussian
// covering many tiles is spread across the warp.
__global__ void __launch_bounds__(kThreads) emit_kernel(
    const uint32_t* __restrict__ sorted_ids, const uint32_t* __restrict__ num_valid,
    const uint32_t* __restrict__ offsets, const int32_t* __restrict__ counts,
    const int4* __restrict__ bounds, int tiles_w, int64_t capacity,
    uint32_t* __restrict__ tile_keys, uint32_t* __restrict__ values) {
  chain_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warp_first = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) - lane;
  const int64_t n = *num_valid;
  if (warp_first >= n) return;  // uniform per warp
  const int64_t j = warp_first + lane;
  const bool ok = j < n;
  const uint32_t g = ok ? sorted_ids[j] : 0u;
  const int4 b = ok ? __ldg(bounds + g) : make_int4(0, 1, 0, 0);
  const uint32_t cnt = ok ? static_cast<uint32_t>(__ldg(counts + g)) : 0u;
  uint32_t incl = cnt;
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const uint32_t excl = incl - cnt;
  const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
  const uint32_t out0 = __shfl_sync(0xffffffffu, ok ? offsets[j] : 0u, 0);
  const int width = b.y - b.x;
  for (uint32_t r = 0; r < total; r += 32) {
    const uint32_t o = r + lane;
    // Largest source lane s with excl[s] <= o (lanes with cnt 0 share excl
    // with the next lane; taking the largest lands on one with cnt > 0).
    int s = 0;
#pragma unroll
    for (int step = 16; step > 0; step >>= 1) {
      const uint32_t e = __shfl_sync(0xffffffffu, excl, s + step);
      if (e <= o) s += step;
    }
    const uint32_t src_excl = __shfl_sync(0xffffffffu, excl, s);
    const uint32_t src_g = __shfl_sync(0xffffffffu, g, s);
    const int src_xmin = __shfl_sync(0xffffffffu, b.x, s);
    const int src_ymin = __shfl_sync(0xffffffffu, b.z, s);
    const int src_width = __shfl_sync(0xffffffffu, width, s);
    if (o < total && static_cast<int64_t>(out0) + o < capacity) {
      const int local = static_cast<int>(o - src_excl);
      const int tile = (src_ymin + local / src_width) * tiles_w + src_xmin + local % src_width;
      tile_keys[out0 + o] = static_cast<uint32_t>(tile);
      values[out0 + o] = src_g;
    }
  }
}

// ranges[t] = [first index with key >= t, first index with key >= t + 1)
// over the sorted tile keys. Each index i (0 <= i <= total) looks at the step
// between key[i-1] and key[i] (key[-1] = -1, key[total] = num_tiles): every
// tile t in (key[i-1], key[i]] starts at i and every tile t in
// [key[i-1], key[i]) ends at i. Each start and end is written exactly once,
// and empty tiles get start == end. A thread takes kRangeItems consecutive
// indices (two 16-byte loads when they are all inside the array).
constexpr int kRangeItems = 8;
__global__ void ranges_kernel(const uint32_t* __restrict__ sorted_keys, Count count,
                              int64_t num_tiles, int64_t* __restrict__ ranges) {
  chain_wait();
  const int64_t total = count.get();
  const int64_t i0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * kRangeItems;
  if (i0 > total) return;
  uint32_t k[kRangeItems];
  if (i0 + kRangeItems <= total) {
    const uint4 a = *reinterpret_cast<const uint4*>(sorted_keys + i0);
    const uint4 b = *reinterpret_cast<const uint4*>(sorted_keys + i0 + 4);
    k[0] = a.x; k[1] = a.y; k[2] = a.z; k[3] = a.w;
    k[4] = b.x; k[5] = b.y; k[6] = b.z; k[7] = b.w;
  } else {
#pragma unroll
    for (int j = 0; j < kRangeItems; ++j) k[j] = i0 + j < total ? sorted_keys[i0 + j] : 0u;
  }
  int64_t prev = i0 > 0 ? static_cast<int64_t>(sorted_keys[i0 - 1]) : -1;
#pragma unroll
  for (int j = 0; j < kRangeItems; ++j) {
    const int64_t i = i0 + j;
    if (i > total) break;
    const int64_t cur = i < total ? static_cast<int64_t>(k[j]) : num_tiles;
    if (cur != prev) {
      for (int64_t t = prev + 1; t <= cur && t < num_tiles; ++t) ranges[2 * t] = i;
      for (int64_t t = prev < 0 ? 0 : prev; t < cur; ++t) ranges[2 * t + 1] = i;
    }
    prev = cur;
  }
}

// ------------------------------------------------------- row/column binning
//
// The list order (tile, depth bits, Gaussian index) is, with tile = row *
// tiles_w + column: by tile row, then tile column, then depth order. Each
// visible Gaussian covers a rectangle of tiles: h row segments of w
// consecutive tiles. So instead of emitting all w*h (tile, Gaussian) pairs and
// radix-sorting them by tile id (two passes over every pair):
//   pass A  scatters the depth-ordered Gaussians into per-row lists of
//           segments (stable: each row's segments stay in depth order);
//   pass B  scatters each row's segments into the row's tile lists (stable:
//           each tile's Gaussians stay in depth order) and writes the ids.
// A config-2 view has 5.15M pairs but 2.2M segments, a config-5 view 56.8M
// pairs but 5M segments.
//
// Each pass is three kernels and no CTA ever waits on another: count (per
// chunk of items, how many land in each bucket -- row or column), scan (per
// bucket, the chunks' exclusive prefix, and the bucket starts), scatter (each
// chunk writes its items from its prefix on). Within a chunk an item's place
// is its stable rank among the chunk's items covering the same bucket: items
// are taken in batches of one per thread, each warp ORs its lanes into a
// bitmask per bucket, and the rank is the popcount of the lanes and warps
// before it -- an interval covers each of its buckets once, so no digit
// ranking is needed. (A decoupled look-back across the thousands of small
// chunks measured 150 us on the config-2 view: every chunk publishes at
// once and the prefix front advances a few chunks per round trip.)

constexpr int kChunkBatches = 4;                         // batches of kThreads items per chunk
constexpr int kChunkItems = kChunkBatches * kThreads;   // 1024
constexpr int kMaxTileRows = 512;       // pass A keeps bitmasks per (warp, row)
constexpr int kMaxTileCols = kThreads;  // pass B keeps bitmasks per (warp, column)
constexpr int kScanThreads = 1024;

// A Gaussian's tile rectangle (xmin, xmax, ymin, ymax) clamped to the grid.
// The projection's rectangles are inside it already, and non-empty wherever
// the count is non-zero; the clamp keeps any other caller's input in bounds.
__device__ __forceinline__ int4 clamp_rect(int4 b, int cols, int rows) {
  const int x0 = min(max(b.x, 0), cols), y0 = min(max(b.z, 0), rows);
  return make_int4(x0, min(max(b.y, x0), cols), y0, min(max(b.w, y0), rows));
}

// Exclusive scan of one value per thread over a CTA of kScanThreads; the
// total goes to *total (every thread).
__device__ __forceinline__ uint32_t wide_exclusive_scan(uint32_t v, uint32_t* s_tmp,
                                                        uint32_t* total) {
  constexpr int kScanWarps = kScanThreads / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t x = v;
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_tmp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = lane < kScanWarps ? s_tmp[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    s_tmp[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const uint32_t prefix = warp ? s_tmp[warp - 1] : 0;
  *total = s_tmp[kScanWarps - 1];
  __syncthreads();
  return prefix + x - v;
}

// The ranks of one batch (one item per thread) among the batch's items that
// cover the same bucket, on top of s_run[bucket], and s_run advanced past the
// batch. Item [lo, hi) covers buckets lo..hi-1; `emit(bucket, position)` is
// called once per covered bucket. s_cover [kWarps][buckets] must be zero on
// entry and is zero again on return; s_base [kWarps][buckets] is scratch.
template <class Emit>
__device__ __forceinline__ void scatter_batch(int lo, int hi, int buckets, uint32_t* s_cover,
                                              uint32_t* s_base, uint32_t* s_run, int stride,
                                              Emit emit) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // Where the warp's intervals overlap heavily (a dense blob), per-lane
  // atomics would serialise on a few words: there one ballot per bucket of
  // the warp's span builds its masks; elsewhere each lane ORs in its own.
  const int span_lo = __reduce_min_sync(0xffffffffu, lo < hi ? lo : 0x7fffffff);
  const int span_hi = __reduce_max_sync(0xffffffffu, lo < hi ? hi : 0);
  const int covered = __reduce_add_sync(0xffffffffu, hi - lo);
  const int span = span_hi - span_lo;
  const bool dense = span > 0 && span <= 64 && covered >= 2 * span;  // warp-uniform
  if (dense) {
    for (int k = span_lo; k < span_hi; ++k) {
      const unsigned mask = __ballot_sync(0xffffffffu, lo <= k && k < hi);
      if (lane == 0) s_cover[warp * stride + k] = mask;
    }
  } else {
    for (int k = lo; k < hi; ++k) atomicOr(&s_cover[warp * stride + k], 1u << lane);
  }
  __syncthreads();
  for (int k = threadIdx.x; k < buckets; k += kThreads) {
    uint32_t run = s_run[k];
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      s_base[w * stride + k] = run;
      run += __popc(s_cover[w * stride + k]);
    }
    s_run[k] = run;
  }
  __syncthreads();
  const unsigned lower = lanemask_lt();
  if (dense) {
    // bucket by bucket: the lanes covering bucket k write consecutive places
    // of k's list together (one coalesced store)
    for (int k = span_lo; k < span_hi; ++k)
      if (lo <= k && k < hi)
        emit(k, s_base[warp * stride + k] + __popc(s_cover[warp * stride + k] & lower));
  } else {
    for (int k = lo; k < hi; ++k)
      emit(k, s_base[warp * stride + k] + __popc(s_cover[warp * stride + k] & lower));
  }
  __syncthreads();
  for (int k = threadIdx.x; k < buckets; k += kThreads) {
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s_cover[w * stride + k] = 0;
  }
  __syncthreads();
}

// Pass A, count: per chunk of kChunkItems depth-ordered Gaussians, the
// segments (Gaussians) and the pairs (Gaussians x width) each tile row gets,
// by difference arrays over rows: seg_counts / pair_counts [rows][chunks].
__global__ void __launch_bounds__(kThreads) row_count_kernel(
    const uint32_t* __restrict__ sorted_ids, const uint32_t* __restrict__ num_valid,
    const int4* __restrict__ bounds, int rows, int cols, int64_t chunks_pitch,
    uint32_t* __restrict__ seg_counts, uint32_t* __restrict__ pair_counts) {
  chain_wait();
  __shared__ int32_t s_seg[kMaxTileRows + 1];
  __shared__ int32_t s_pair[kMaxTileRows + 1];
  __shared__ uint32_t s_tmp[kWarps];
  const int64_t v = *num_valid;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kChunkItems;
  if (first >= v) return;  // uniform
  for (int y = threadIdx.x; y <= rows; y += kThreads) s_seg[y] = s_pair[y] = 0;
  __syncthreads();
#pragma unroll
  for (int bt = 0; bt < kChunkBatches; ++bt) {
    const int64_t j = first + bt * kThreads + threadIdx.x;
    if (j < v) {
      const int4 b = clamp_rect(__ldg(bounds + sorted_ids[j]), cols, rows);
      atomicAdd(&s_seg[b.z], 1);
      atomicAdd(&s_seg[b.w], -1);
      atomicAdd(&s_pair[b.z], b.y - b.x);
      atomicAdd(&s_pair[b.w], b.x - b.y);
    }
  }
  __syncthreads();
  // prefix over rows (rows <= 2 kThreads: two rows per thread)
  const int y0 = 2 * threadIdx.x;
  const int32_t a0 = y0 < rows ? s_seg[y0] : 0, a1 = y0 + 1 < rows ? s_seg[y0 + 1] : 0;
  const int32_t p0 = y0 < rows ? s_pair[y0] : 0, p1 = y0 + 1 < rows ? s_pair[y0 + 1] : 0;
  const int32_t sa = static_cast<int32_t>(
      block_exclusive_scan(static_cast<uint32_t>(a0 + a1), s_tmp, nullptr));
  const int32_t sp = static_cast<int32_t>(
      block_exclusive_scan(static_cast<uint32_t>(p0 + p1), s_tmp, nullptr));
  if (y0 < rows) {
    seg_counts[y0 * chunks_pitch + blockIdx.x] = static_cast<uint32_t>(sa + a0);
    pair_counts[y0 * chunks_pitch + blockIdx.x] = static_cast<uint32_t>(sp + p0);
  }
  if (y0 + 1 < rows) {
    seg_counts[(y0 + 1) * chunks_pitch + blockIdx.x] = static_cast<uint32_t>(sa + a0 + a1);
    pair_counts[(y0 + 1) * chunks_pitch + blockIdx.x] = static_cast<uint32_t>(sp + p0 + p1);
  }
}

// Pass A, scan: CTA y turns row y's per-chunk segment counts into exclusive
// prefixes (in place) and totals the row's segments and pairs.
__global__ void __launch_bounds__(kScanThreads) row_scan_kernel(
    const uint32_t* __restrict__ num_valid, int64_t chunks_pitch,
    uint32_t* __restrict__ seg_counts, const uint32_t* __restrict__ pair_counts,
    uint32_t* __restrict__ row_segs, uint32_t* __restrict__ row_pairs) {
  chain_wait();
  __shared__ uint32_t s_tmp[32];
  const int y = blockIdx.x;
  const int64_t chunks = (static_cast<int64_t>(*num_valid) + kChunkItems - 1) / kChunkItems;
  uint32_t* counts = seg_counts + y * chunks_pitch;
  const uint32_t* pairs = pair_counts + y * chunks_pitch;
  // thread t owns a contiguous run of chunks
  const int64_t per = (chunks + kScanThreads - 1) / kScanThreads;
  const int64_t c0 = threadIdx.x * per;
  const int64_t c1 = c0 + per < chunks ? c0 + per : chunks;
  uint32_t mine = 0, my_pairs = 0;
  for (int64_t c = c0; c < c1; ++c) {
    mine += counts[c];
    my_pairs += pairs[c];
  }
  uint32_t total, total_pairs;
  uint32_t run = wide_exclusive_scan(mine, s_tmp, &total);
  wide_exclusive_scan(my_pairs, s_tmp, &total_pairs);
  for (int64_t c = c0; c < c1; ++c) {
    const uint32_t k = counts[c];
    counts[c] = run;
    run += k;
  }
  if (threadIdx.x == 0) {
    row_segs[y] = total;
    row_pairs[y] = total_pairs;
  }
}

// One CTA: the start of each row's segments (those past `seg_capacity` are
// dropped) and pairs, and pass B's chunks (kChunkItems segments of one row
// each): the first chunk of each row and the row of each chunk.
__global__ void __launch_bounds__(kScanThreads) row_layout_kernel(
    const uint32_t* __restrict__ row_segs, const uint32_t* __restrict__ row_pairs, int rows,
    uint32_t seg_capacity, uint32_t* __restrict__ row_seg_start,
    uint32_t* __restrict__ row_pair_start, uint32_t* __restrict__ row_chunk_start,
    uint32_t* __restrict__ chunk_row) {
  chain_wait();
  __shared__ uint32_t s_tmp[32];
  const int y = threadIdx.x;  // rows <= kScanThreads
  const uint32_t segs = y < rows ? row_segs[y] : 0u;
  uint32_t total, total_pairs;
  const uint32_t start = wide_exclusive_scan(segs, s_tmp, &total);
  const uint32_t pair_start = wide_exclusive_scan(y < rows ? row_pairs[y] : 0u, s_tmp,
                                                  &total_pairs);
  const uint32_t lo = start < seg_capacity ? start : seg_capacity;
  const uint32_t end = start + segs;
  const uint32_t hi = end < seg_capacity ? end : seg_capacity;
  const uint32_t chunks = (hi - lo + kChunkItems - 1) / kChunkItems;
  uint32_t num_chunks;
  const uint32_t first_chunk = wide_exclusive_scan(chunks, s_tmp, &num_chunks);
  if (y < rows) {
    row_seg_start[y] = lo;
    row_pair_start[y] = pair_start;
    row_chunk_start[y] = first_chunk;
    for (uint32_t k = 0; k < chunks; ++k) chunk_row[first_chunk + k] = static_cast<uint32_t>(y);
  }
  if (y == 0) {
    row_seg_start[rows] = total < seg_capacity ? total : seg_capacity;
    row_pair_start[rows] = total_pairs;
    row_chunk_start[rows] = num_chunks;
  }
}

// Pass A, scatter: chunk c of the depth order writes each Gaussian's id into
// its rows' segment lists, from the row start plus the chunk's prefix.
__global__ void __launch_bounds__(kThreads) row_scatter_kernel(
    const uint32_t* __restrict__ sorted_ids, const uint32_t* __restrict__ num_valid,
    const int4* __restrict__ bounds, int rows, int cols, int64_t chunks_pitch,
    const uint32_t* __restrict__ seg_prefix, const uint32_t* __restrict__ row_seg_start,
    uint32_t seg_capacity, uint32_t* __restrict__ segs) {
  chain_wait();
  __shared__ uint32_t s_cover[kWarps * kMaxTileRows];
  __shared__ uint32_t s_base[kWarps * kMaxTileRows];
  __shared__ uint32_t s_run[kMaxTileRows];
  const int64_t v = *num_valid;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kChunkItems;
  if (first >= v) return;  // uniform
  for (int i = threadIdx.x; i < kWarps * rows; i += kThreads) s_cover[(i / rows) * rows + i % rows] = 0;
  for (int y = threadIdx.x; y < rows; y += kThreads)
    s_run[y] = row_seg_start[y] + seg_prefix[y * chunks_pitch + blockIdx.x];
  __syncthreads();
  // All batches' ids, then all their rectangles, before the first barrier:
  // the gathers' latencies overlap instead of one per batch.
  uint32_t g[kChunkBatches];
  int y0[kChunkBatches], y1[kChunkBatches];
#pragma unroll
  for (int bt = 0; bt < kChunkBatches; ++bt) {
    const int64_t j = first + bt * kThreads + threadIdx.x;
    g[bt] = j < v ? sorted_ids[j] : 0xffffffffu;
  }
#pragma unroll
  for (int bt = 0; bt < kChunkBatches; ++bt) {
    y0[bt] = y1[bt] = 0;
    if (g[bt] != 0xffffffffu) {
      const int4 b = clamp_rect(__ldg(bounds + g[bt]), cols, rows);
      y0[bt] = b.z;
      y1[bt] = b.w;
    }
  }
#pragma unroll
  for (int bt = 0; bt < kChunkBatches; ++bt) {
    const uint32_t id = g[bt];
    scatter_batch(y0[bt], y1[bt], rows, s_cover, s_base, s_run, rows, [&](int, uint32_t pos) {
      if (pos < seg_capacity) segs[pos] = id;
    });
  }
}

// Pass B, count: per chunk of one row's segments, the pairs each tile column
// gets (a difference array over columns): col_counts [chunks][cols].
__global__ void __launch_bounds__(kThreads) col_count_kernel(
    const uint32_t* __restrict__ segs, const int4* __restrict__ bounds, int rows, int cols,
    const uint32_t* __restrict__ row_seg_start, const uint32_t* __restrict__ row_chunk_start,
    const uint32_t* __restrict__ chunk_row, uint32_t* __restrict__ col_counts) {
  chain_wait();
  __shared__ int32_t s_diff[kMaxTileCols + 1];
  __shared__ uint32_t s_tmp[kWarps];
  const uint32_t num_chunks = row_chunk_start[rows];
  for (uint32_t c = blockIdx.x; c < num_chunks; c += gridDim.x) {  // uniform
    for (int x = threadIdx.x; x <= cols; x += kThreads) s_diff[x] = 0;
    __syncthreads();
    const uint32_t y = chunk_row[c];
    const uint32_t s0 = row_seg_start[y] + (c - row_chunk_start[y]) * kChunkItems;
    const uint32_t end = row_seg_start[y + 1];
    int2 span[kChunkBatches];
#pragma unroll
    for (int bt = 0; bt < kChunkBatches; ++bt) {
      const uint32_t si = s0 + bt * kThreads + threadIdx.x;
      span[bt] = make_int2(0, 0);
      if (si < end && si < s0 + kChunkItems)
        span[bt] = __ldg(reinterpret_cast<const int2*>(bounds + segs[si]));
    }
#pragma unroll
    for (int bt = 0; bt < kChunkBatches; ++bt) {
      const int x0 = min(max(span[bt].x, 0), cols);  // as clamp_rect
      const int x1 = min(max(span[bt].y, x0), cols);
      if (x0 < x1) {
        atomicAdd(&s_diff[x0], 1);
        atomicAdd(&s_diff[x1], -1);
      }
    }
    __syncthreads();
    const int x = threadIdx.x;  // cols <= kThreads
    const int32_t d = x < cols ? s_diff[x] : 0;
    const int32_t count = static_cast<int32_t>(
        block_exclusive_scan(static_cast<uint32_t>(d), s_tmp, nullptr)) + d;
    if (x < cols) col_counts[static_cast<int64_t>(c) * cols + x] = static_cast<uint32_t>(count);
    __syncthreads();
  }
}

// Pass B, scan: CTA y totals each column of row y over the row's chunks,
// writes the row's tile ranges (start: the row's first pair plus the columns
// before; clamped to the id capacity) and turns the chunks' column counts
// into their first positions (in place). Four threads per column, each over a
// quarter of the row's chunks.
__global__ void __launch_bounds__(kScanThreads) col_scan_kernel(
    int cols, const uint32_t* __restrict__ row_chunk_start,
    const uint32_t* __restrict__ row_pair_start, int64_t id_capacity,
    uint32_t* __restrict__ col_counts, int64_t* __restrict__ ranges) {
  chain_wait();
  constexpr int kParts = kScanThreads / kMaxTileCols;  // 4
  __shared__ uint32_t s_part[kParts][kMaxTileCols];
  __shared__ uint32_t s_tmp[32];
  const int y = blockIdx.x;
  const int x = threadIdx.x % kMaxTileCols, part = threadIdx.x / kMaxTileCols;
  const uint32_t c_begin = row_chunk_start[y], c_end = row_chunk_start[y + 1];
  const uint32_t per = (c_end - c_begin + kParts - 1) / kParts;
  const uint32_t c0 = c_begin + part * per < c_end ? c_begin + part * per : c_end;
  const uint32_t c1 = c0 + per < c_end ? c0 + per : c_end;
  uint32_t mine = 0;
  if (x < cols)
    for (uint32_t c = c0; c < c1; ++c) mine += col_counts[static_cast<int64_t>(c) * cols + x];
  s_part[part][x] = mine;
  __syncthreads();
  // the row's pairs per column (threads of part 0, which come first in thread
  // order, so the CTA-wide scan of their totals is the scan over columns)
  uint32_t total = 0;
  if (part == 0 && x < cols) {
#pragma unroll
    for (int q = 0; q < kParts; ++q) total += s_part[q][x];
  }
  uint32_t all;
  const uint32_t before = wide_exclusive_scan(total, s_tmp, &all);
  if (part == 0) {
    const int64_t start = static_cast<int64_t>(row_pair_start[y]) + before;
    const int64_t end = start + total;
    if (x < cols) {
      const int64_t t = static_cast<int64_t>(y) * cols + x;
      ranges[2 * t] = start < id_capacity ? start : id_capacity;
      ranges[2 * t + 1] = end < id_capacity ? end : id_capacity;
    }
    // each part's first position in the column's tile
    uint32_t run = static_cast<uint32_t>(start);
#pragma unroll
    for (int q = 0; q < kParts; ++q) {
      const uint32_t k = s_part[q][x];
      s_part[q][x] = run;
      run += k;
    }
  }
  __syncthreads();
  if (x < cols) {
    uint32_t run = s_part[part][x];
    for (uint32_t c = c0; c < c1; ++c) {
      uint32_t* p = col_counts + static_cast<int64_t>(c) * cols + x;
      const uint32_t k = *p;
      *p = run;
      run += k;
    }
  }
}

// Pass B, scatter: each chunk of one row's segments writes, for every tile
// column a segment spans, its Gaussian id from the chunk's first position in
// that tile on.
__global__ void __launch_bounds__(kThreads) col_scatter_kernel(
    const uint32_t* __restrict__ segs, const int4* __restrict__ bounds, int rows, int cols,
    const uint32_t* __restrict__ row_seg_start, const uint32_t* __restrict__ row_chunk_start,
    const uint32_t* __restrict__ chunk_row, const uint32_t* __restrict__ col_first,
    int64_t id_capacity, int32_t* __restrict__ ids) {
  chain_wait();
  __shared__ uint32_t s_cover[kWarps * kMaxTileCols];
  __shared__ uint32_t s_base[kWarps * kMaxTileCols];
  __shared__ uint32_t s_run[kMaxTileCols];
  for (int i = threadIdx.x; i < kWarps * kMaxTileCols; i += kThreads) s_cover[i] = 0;
  const uint32_t num_chunks = row_chunk_start[rows];
  for (uint32_t c = blockIdx.x; c < num_chunks; c += gridDim.x) {  // uniform
    for (int x = threadIdx.x; x < cols; x += kThreads)
      s_run[x] = col_first[static_cast<int64_t>(c) * cols + x];
    __syncthreads();
    const uint32_t y = chunk_row[c];
    const uint32_t s0 = row_seg_start[y] + (c - row_chunk_start[y]) * kChunkItems;
    const uint32_t end = row_seg_start[y + 1];
    for (int bt = 0; bt < kChunkBatches; ++bt) {
      const uint32_t si = s0 + bt * kThreads + threadIdx.x;
      uint32_t g = 0;
      int x0 = 0, x1 = 0;
      if (si < end && si < s0 + kChunkItems) {
        g = segs[si];
        const int2 span = __ldg(reinterpret_cast<const int2*>(bounds + g));
        x0 = min(max(span.x, 0), cols);  // as clamp_rect
        x1 = min(max(span.y, x0), cols);
      }
      scatter_batch(x0, x1, cols, s_cover, s_base, s_run, kMaxTileCols, [&](int, uint32_t pos) {
        if (pos < id_capacity) ids[pos] = static_cast<int32_t>(g);
      });
    }
  }
}

// ---------------------------------------------------------------- workspaces

constexpr uint64_t kAlign = 256;
inline uint64_t align_up(uint64_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

// Counters and flags that must start at zero (zeroed with the status words).
struct BinHeader {
  uint32_t hist[4][kRadix];
  uint32_t num_valid;
  uint32_t pass_counters[4];
  uint32_t scan_counter;
  uint32_t error;
  uint32_t pad_;
  int64_t total;
};

struct CountLayout {
  uint64_t header, depth_status, zero_bytes;
  uint64_t keys_a, keys_b, ids_a, ids_b, bytes;
  explicit CountLayout(int64_t n) {
    const uint64_t blocks = (n + kTile - 1) / kTile;
    uint64_t at = 0;
    header = at; at = align_up(at + sizeof(BinHeader));
    depth_status = at; at = align_up(at + blocks * kRadix * 4 * 4);
    zero_bytes = at;
    keys_a = at; at = align_up(at + 4 * static_cast<uint64_t>(n));
    keys_b = at; at = align_up(at + 4 * static_cast<uint64_t>(n));
    ids_a = at; at = align_up(at + 4 * static_cast<uint64_t>(n));
    ids_b = at; at = align_up(at + 4 * static_cast<uint64_t>(n));
    bytes = at;
  }
};

inline int tile_bits(int64_t num_tiles) {
  int bits = 0;
  while ((int64_t{1} << bits) < num_tiles) ++bits;
  return bits;
}

// Scratch of an LSD radix sort of `total` keys below num_keys (the tile sort
// of the fallback path, and the deterministic backward's position sort).
struct RadixLayout {
  uint64_t header, status, zero_bytes, keys_a, keys_b, values_a, values_b, bytes;
  int passes;
  RadixLayout(int64_t total, int64_t num_keys) {
    passes = (tile_bits(num_keys) + 7) / 8;
    const uint64_t blocks = (total + kTile - 1) / kTile;
    uint64_t at = 0;
    header = at; at = align_up(at + sizeof(BinHeader));
    status = at; at = align_up(at + blocks * kRadix * 4 * (passes ? passes : 1));
    zero_bytes = at;
    keys_a = at; at = align_up(at + 4 * static_cast<uint64_t>(total));
    keys_b = at; at = align_up(at + 4 * static_cast<uint64_t>(total));
    values_a = at; at = align_up(at + 4 * static_cast<uint64_t>(total));
    values_b = at; at = align_up(at + 4 * static_cast<uint64_t>(total));
    bytes = at;
  }
};

// Sort-phase scratch for n Gaussians, `total` intersections (the capacity)
// and a tiles_w x tiles_h grid. The row/column path when the grid fits its
// shared-memory tables, else the emit + tile radix sort path (which also
// takes the count scan's offsets here).
struct SortLayout {
  bool rowcol;
  int rows, cols;
  uint64_t header, zero_bytes, bytes;
  // row/column path
  uint64_t chunks_a, max_chunks_b;
  uint64_t seg_counts, pair_counts, row_segs, row_pairs, row_seg_start, row_pair_start,
      row_chunk_start, chunk_row, col_counts, segs;
  // radix path
  uint64_t scan_status, offsets, radix;
  RadixLayout lsd;
  SortLayout(int64_t n, int64_t total, int tiles_w, int tiles_h)
      : rows(tiles_h), cols(tiles_w), lsd(total, static_cast<int64_t>(tiles_w) * tiles_h) {
    rowcol = tiles_h <= kMaxTileRows && tiles_w <= kMaxTileCols;
    const uint64_t un = static_cast<uint64_t>(n), ut = static_cast<uint64_t>(total);
    const uint64_t ur = static_cast<uint64_t>(rows), uc = static_cast<uint64_t>(cols);
    uint64_t at = 0;
    header = at; at = align_up(at + sizeof(BinHeader));
    zero_bytes = at;
    if (rowcol) {
      chunks_a = (un + kChunkItems - 1) / kChunkItems;
      max_chunks_b = (ut + kChunkItems - 1) / kChunkItems + ur;
      seg_counts = at; at = align_up(at + 4 * ur * chunks_a);
      pair_counts = at; at = align_up(at + 4 * ur * chunks_a);
      row_segs = at; at = align_up(at + 4 * ur);
      row_pairs = at; at = align_up(at + 4 * ur);
      row_seg_start = at; at = align_up(at + 4 * (ur + 1));
      row_pair_start = at; at = align_up(at + 4 * (ur + 1));
      row_chunk_start = at; at = align_up(at + 4 * (ur + 1));
      chunk_row = at; at = align_up(at + 4 * max_chunks_b);
      col_counts = at; at = align_up(at + 4 * max_chunks_b * uc);
      segs = at; at = align_up(at + 4 * ut);
    } else {
      chunks_a = max_chunks_b = 0;
      scan_status = at; at = align_up(at + 8 * ((un + kTile - 1) / kTile));
      zero_bytes = at;
      offsets = at; at = align_up(at + 4 * un);
      radix = at; at = align_up(at + lsd.bytes);
    }
    bytes = at;
  }
};

template <class T>
T* at(void* base, uint64_t offset) {
  return reinterpret_cast<T*>(static_cast<char*>(base) + offset);
}
template <class T>
const T* at(const void* base, uint64_t offset) {
  return reinterpret_cast<const T*>(static_cast<const char*>(base) + offset);
}

inline unsigned upsweep_blocks(int64_t n) {
  const int64_t want = (n + kThreads * 8 - 1) / (kThreads * 8);
  return static_cast<unsigned>(want < 4 * kSmCount ? (want > 0 ? want : 1) : 4 * kSmCount);
}

}  // namespace

uint64_t bin_count_workspace_size(int64_t n) { return CountLayout(n).bytes; }
uint64_t bin_sort_workspace_size(int64_t n, int64_t total, const gs_params& p) {
  return SortLayout(n, total, p.width / p.tile_size, p.height / p.tile_size).bytes;
}
uint64_t radix_sort_workspace_size(int64_t total, int64_t num_keys) {
  return RadixLayout(total, num_keys).bytes;
}

// Where the depth-sorted Gaussian ids end up after the 4 passes.
static uint64_t sorted_ids_offset(const CountLayout& L) { return L.ids_a; }

// The count phase without the host wait: the intersection total and the
// error word are copied into the caller's (pinned) host words on `stream`.
int32_t launch_bin_count_async(int64_t n, const float* projected_mean, const int32_t* counts,
                               void* workspace, int64_t* total_host, uint32_t* error_host,
                               cudaStream_t stream);

int32_t launch_bin_count_kernels(int64_t n, const float* projected_mean, const int32_t* counts,
                                 void* workspace, cudaStream_t stream);

int32_t launch_bin_count(int64_t n, const float* projected_mean, const int32_t* counts,
                         void* workspace, int64_t* total_host, uint32_t* error_host,
                         cudaStream_t stream) {
  GS_TRY(launch_bin_count_kernels(n, projected_mean, counts, workspace, stream));
  // error, pad and total are adjacent in the header: one copy brings both back.
  struct {
    uint32_t error, pad;
    int64_t total;
  } tail;
  static_assert(offsetof(BinHeader, total) == offsetof(BinHeader, error) + 8,
                "error and total must be adjacent");
  const BinHeader* h = at<BinHeader>(workspace, CountLayout(n).header);
  GS_CUDA_TRY(cudaMemcpyAsync(&tail, &h->error, sizeof(tail), cudaMemcpyDeviceToHost, stream));
  GS_CUDA_TRY(cudaStreamSynchronize(stream));
  *total_host = tail.total;
  *error_host = tail.error;
  return GS_OK;
}

int32_t launch_bin_count_async(int64_t n, const float* projected_mean, const int32_t* counts,
                               void* workspace, int64_t* total_host, uint32_t* error_host,
                               cudaStream_t stream) {
  GS_TRY(launch_bin_count_kernels(n, projected_mean, counts, workspace, stream));
  const BinHeader* h = at<BinHeader>(workspace, CountLayout(n).header);
  GS_CUDA_TRY(cudaMemcpyAsync(total_host, &h->total, sizeof(int64_t), cudaMemcpyDeviceToHost,
                              stream));
  GS_CUDA_TRY(cudaMemcpyAsync(error_host, &h->error, sizeof(uint32_t), cudaMemcpyDeviceToHost,
                              stream));
  return GS_OK;
}

// Depth order of the visible Gaussians (four stable 8-bit passes over the
// depth bits) and, from the histogram upsweep, their number and the
// intersection total (the sum of their tile counts).
int32_t launch_bin_count_kernels(int64_t n, const float* projected_mean, const int32_t* counts,
                                 void* workspace, cudaStream_t stream) {
  const CountLayout L(n);
  BinHeader* h = at<BinHeader>(workspace, L.header);
  GS_CUDA_TRY(cudaMemsetAsync(workspace, 0, L.zero_bytes, stream));
  if (n > 0) {
    const int64_t blocks = (n + kTile - 1) / kTile;
    static_assert(sizeof(h->total) == sizeof(unsigned long long), "64-bit total");
    launch_chained(upsweep_kernel<DepthSource, 4>, upsweep_blocks(n), kThreads, stream,
        DepthSource{projected_mean, counts}, Count{n, nullptr}, 4, 0, &h->hist[0][0],
        &h->num_valid, reinterpret_cast<unsigned long long*>(&h->total));
    GS_TRY(check_launch());
    uint32_t* depth_status = at<uint32_t>(workspace, L.depth_status);
    uint32_t* kA = at<uint32_t>(workspace, L.keys_a);
    uint32_t* kB = at<uint32_t>(workspace, L.keys_b);
    uint32_t* vA = at<uint32_t>(workspace, L.ids_a);
    uint32_t* vB = at<uint32_t>(workspace, L.ids_b);
    // Pass 0 filters and reads the projection outputs directly; passes 1-3
    // ping-pong A -> B -> A so the ids finish in ids_a.
    launch_chained(sort_pass_kernel<DepthSource>, blocks, kThreads, stream,
        DepthSource{projected_mean, counts}, Count{n, nullptr}, 0, &h->hist[0][0], depth_status,
        &h->pass_counters[0], kB, vB, &h->error);
    GS_TRY(check_launch());
    uint32_t* ins_k[3] = {kB, kA, kB};
    uint32_t* ins_v[3] = {vB, vA, vB};
    uint32_t* outs_k[3] = {kA, kB, nullptr};
    uint32_t* outs_v[3] = {vA, vB, vA};
    for (int p = 1; p < 4; ++p) {
      launch_chained(sort_pass_kernel<ArraySource>, blocks, kThreads, stream,
          ArraySource{ins_k[p - 1], ins_v[p - 1]}, Count{0, &h->num_valid}, 8 * p,
          &h->hist[p][0], depth_status + static_cast<int64_t>(p) * blocks * kRadix,
          &h->pass_counters[p], outs_k[p - 1], outs_v[p - 1], &h->error);
      GS_TRY(check_launch());
    }
  }
  return GS_OK;
}

// The row/column path (see the comment above kChunkBatches).
static int32_t launch_bin_sort_rowcol(int64_t n, int64_t total, const int32_t* bounds,
                                      const SortLayout& L, const void* count_workspace,
                                      void* sort_workspace, int32_t* gaussian_ids,
                                      int64_t* ranges, cudaStream_t stream) {
  const CountLayout C(n);
  const BinHeader* ch = at<BinHeader>(count_workspace, C.header);
  const uint32_t* sorted_ids = at<uint32_t>(count_workspace, sorted_ids_offset(C));
  const int4* b4 = reinterpret_cast<const int4*>(bounds);
  const int rows = L.rows, cols = L.cols;
  const int64_t pitch = static_cast<int64_t>(L.chunks_a);
  const uint32_t capacity = static_cast<uint32_t>(total);  // segments and ids alike
  uint32_t* seg_counts = at<uint32_t>(sort_workspace, L.seg_counts);
  uint32_t* pair_counts = at<uint32_t>(sort_workspace, L.pair_counts);
  uint32_t* row_segs = at<uint32_t>(sort_workspace, L.row_segs);
  uint32_t* row_pairs = at<uint32_t>(sort_workspace, L.row_pairs);
  uint32_t* row_seg_start = at<uint32_t>(sort_workspace, L.row_seg_start);
  uint32_t* row_pair_start = at<uint32_t>(sort_workspace, L.row_pair_start);
  uint32_t* row_chunk_start = at<uint32_t>(sort_workspace, L.row_chunk_start);
  uint32_t* chunk_row = at<uint32_t>(sort_workspace, L.chunk_row);
  uint32_t* col_counts = at<uint32_t>(sort_workspace, L.col_counts);
  uint32_t* segs = at<uint32_t>(sort_workspace, L.segs);
  if (n > 0) {
    launch_chained(row_count_kernel, static_cast<unsigned>(L.chunks_a), kThreads, stream,
        sorted_ids, &ch->num_valid, b4, rows, cols, pitch, seg_counts, pair_counts);
    GS_TRY(check_launch());
  }
  launch_chained(row_scan_kernel, rows, kScanThreads, stream, &ch->num_valid, pitch, seg_counts,
                 pair_counts, row_segs, row_pairs);
  GS_TRY(check_launch());
  launch_chained(row_layout_kernel, 1, kScanThreads, stream, row_segs, row_pairs, rows, capacity,
                 row_seg_start, row_pair_start, row_chunk_start, chunk_row);
  GS_TRY(check_launch());
  if (n > 0) {
    launch_chained(row_scatter_kernel, static_cast<unsigned>(L.chunks_a), kThreads, stream,
        sorted_ids, &ch->num_valid, b4, rows, cols, pitch, seg_counts, row_seg_start, capacity,
        segs);
    GS_TRY(check_launch());
  }
  const uint64_t grid_b = L.max_chunks_b < 8 * kSmCount ? L.max_chunks_b : 8 * kSmCount;
  if (grid_b > 0) {
    launch_chained(col_count_kernel, static_cast<unsigned>(grid_b), kThreads, stream,
        segs, b4, rows, cols, row_seg_start, row_chunk_start, chunk_row, col_counts);
    GS_TRY(check_launch());
  }
  launch_chained(col_scan_kernel, rows, kScanThreads, stream, cols, row_chunk_start,
                 row_pair_start, total, col_counts, ranges);
  GS_TRY(check_launch());
  if (grid_b > 0 && total > 0) {
    launch_chained(col_scatter_kernel, static_cast<unsigned>(grid_b), kThreads, stream,
        segs, b4, rows, cols, row_seg_start, row_chunk_start, chunk_row, col_counts, total,
        gaussian_ids);
    GS_TRY(check_launch());
  }
  return GS_OK;
}

// The fallback path for grids wider than the row/column tables: the count
// scan's offsets, emission in depth order, a stable LSD radix sort of the
// tile ids, then the ranges.
static int32_t launch_bin_sort_radix(int64_t n, int64_t total, const int32_t* bounds,
                                     const int32_t* counts, const gs_params& p,
                                     const SortLayout& L, const void* count_workspace,
                                     void* sort_workspace, int32_t* gaussian_ids,
                                     int64_t* ranges, cudaStream_t stream) {
  const CountLayout C(n);
  const int64_t tiles_w = L.cols;
  const int64_t num_tiles = tiles_w * L.rows;
  const RadixLayout& R = L.lsd;
  const BinHeader* ch = at<BinHeader>(count_workspace, C.header);
  BinHeader* h = at<BinHeader>(sort_workspace, L.header);
  void* radix = at<char>(sort_workspace, L.radix);
  BinHeader* rh = at<BinHeader>(radix, R.header);
  GS_CUDA_TRY(cudaMemsetAsync(radix, 0, R.zero_bytes, stream));
  uint32_t* kA = at<uint32_t>(radix, R.keys_a);
  uint32_t* kB = at<uint32_t>(radix, R.keys_b);
  uint32_t* vA = at<uint32_t>(radix, R.values_a);
  uint32_t* vB = at<uint32_t>(radix, R.values_b);
  uint32_t* out_ids = reinterpret_cast<uint32_t*>(gaussian_ids);
  uint32_t* offsets = at<uint32_t>(sort_workspace, L.offsets);
  const uint32_t* sorted_ids = at<uint32_t>(count_workspace, sorted_ids_offset(C));
  const uint32_t* sorted_keys = kA;
  const Count live{total, nullptr, &ch->total};
  if (n > 0) {
    launch_chained(count_scan_kernel, (n + kTile - 1) / kTile, kThreads, stream,
        sorted_ids, &ch->num_valid, counts, at<uint64_t>(sort_workspace, L.scan_status),
        &h->scan_counter, offsets, &h->total, &h->error);
    GS_TRY(check_launch());
  }
  if (total > 0) {
    const int passes = R.passes;
    launch_chained(emit_kernel, ceil_div(n, kThreads), kThreads, stream,
        sorted_ids, &ch->num_valid, offsets, counts, reinterpret_cast<const int4*>(bounds),
        static_cast<int>(tiles_w), total, kA, passes == 0 ? out_ids : vA);
    GS_TRY(check_launch());
    if (passes > 0) {
      launch_chained(upsweep_kernel<ArraySource, 16>, upsweep_blocks(total), kThreads, stream,
          ArraySource{kA, vA}, live, passes, 0, &rh->hist[0][0], nullptr, nullptr);
      GS_TRY(check_launch());
      const int64_t blocks = (total + kTile - 1) / kTile;
      uint32_t* src_k = kA;
      uint32_t* src_v = vA;
      for (int pass = 0; pass < passes; ++pass) {
        uint32_t* dst_k = (pass % 2 == 0) ? kB : kA;
        uint32_t* dst_v = (pass == passes - 1) ? out_ids : ((pass % 2 == 0) ? vB : vA);
        launch_chained(sort_pass_kernel<ArraySource>, blocks, kThreads, stream,
            ArraySource{src_k, src_v}, live, 8 * pass, &rh->hist[pass][0],
            at<uint32_t>(radix, R.status) + static_cast<int64_t>(pass) * blocks * kRadix,
            &rh->pass_counters[pass], dst_k, dst_v, &h->error);
        GS_TRY(check_launch());
        src_k = dst_k;
        src_v = dst_v;
      }
      sorted_keys = src_k;
    }
  }
  if (num_tiles > 0) {
    launch_chained(ranges_kernel, ceil_div(ceil_div(total + 1, kRangeItems), 256), 256, stream,
        sorted_keys, live, num_tiles, ranges);
    GS_TRY(check_launch());
  }
  return GS_OK;
}

// `total` is the capacity the buffers were sized for: the intersection total
// itself, or more when the caller sized them before reading it. The kernels
// read the true total from the count workspace and clamp to the capacity (an
// overflow leaves a wrong but in-bounds result, for the caller to redo).
int32_t launch_bin_sort(int64_t n, int64_t total, const int32_t* bounds, const int32_t* counts,
                        const gs_params& p, const void* count_workspace, void* sort_workspace,
                        int32_t* gaussian_ids, int64_t* ranges, cudaStream_t stream) {
  const SortLayout L(n, total, p.width / p.tile_size, p.height / p.tile_size);
  GS_CUDA_TRY(cudaMemsetAsync(sort_workspace, 0, L.zero_bytes, stream));
  if (static_cast<int64_t>(L.rows) * L.cols == 0) return GS_OK;
  if (L.rowcol)
    return launch_bin_sort_rowcol(n, total, bounds, L, count_workspace, sort_workspace,
                                  gaussian_ids, ranges, stream);
  return launch_bin_sort_radix(n, total, bounds, counts, p, L, count_workspace, sort_workspace,
                               gaussian_ids, ranges, stream);
}

// Stable sort of the positions 0..total-1 by keys[position] (< num_keys):
// `order` receives the positions grouped by key, increasing within a key, and
// segments [num_keys, 2] each key's [start, end) in `order`. The sort phase's
// machinery on other keys: the deterministic backward groups the per-entry
// gradient rows of each Gaussian this way. `workspace` holds
// radix_sort_workspace_size(total, num_keys) bytes.
int32_t launch_sort_positions(int64_t total, int64_t num_keys, const int32_t* keys,
                              void* workspace, uint32_t* order, int64_t* segments,
                              cudaStream_t stream) {
  const RadixLayout L(total, num_keys);
  BinHeader* h = at<BinHeader>(workspace, L.header);
  GS_CUDA_TRY(cudaMemsetAsync(workspace, 0, L.zero_bytes, stream));
  uint32_t* kA = at<uint32_t>(workspace, L.keys_a);
  uint32_t* kB = at<uint32_t>(workspace, L.keys_b);
  uint32_t* vA = at<uint32_t>(workspace, L.values_a);
  uint32_t* vB = at<uint32_t>(workspace, L.values_b);
  const uint32_t* in_keys = reinterpret_cast<const uint32_t*>(keys);
  const Count all{total, nullptr};
  const uint32_t* sorted_keys = in_keys;
  const int passes = L.passes > 0 ? L.passes : 1;
  if (L.passes == 0 && num_keys > 1) return GS_ERR_INVALID_ARGUMENT;
  if (total > 0) {
    launch_chained(upsweep_kernel<PositionSource, 16>, upsweep_blocks(total), kThreads, stream,
        PositionSource{in_keys}, all, passes, 0, &h->hist[0][0], nullptr, nullptr);
    GS_TRY(check_launch());
    const int64_t blocks = (total + kTile - 1) / kTile;
    uint32_t* status = at<uint32_t>(workspace, L.status);
    for (int pass = 0; pass < passes; ++pass) {
      uint32_t* dst_k = (pass % 2 == 0) ? kB : kA;
      uint32_t* dst_v = (pass == passes - 1) ? order : ((pass % 2 == 0) ? vB : vA);
      uint32_t* pass_status = status + static_cast<int64_t>(pass) * blocks * kRadix;
      if (pass == 0)
        launch_chained(sort_pass_kernel<PositionSource>, blocks, kThreads, stream,
            PositionSource{in_keys}, all, 0, &h->hist[0][0], pass_status, &h->pass_counters[0],
            dst_k, dst_v, &h->error);
      else
        launch_chained(sort_pass_kernel<ArraySource>, blocks, kThreads, stream,
            ArraySource{pass % 2 ? kB : kA, pass % 2 ? vB : vA}, all, 8 * pass,
            &h->hist[pass][0], pass_status, &h->pass_counters[pass], dst_k, dst_v, &h->error);
      GS_TRY(check_launch());
      sorted_keys = dst_k;
    }
  }
  if (num_keys > 0) {
    launch_chained(ranges_kernel, ceil_div(ceil_div(total + 1, kRangeItems), 256), 256, stream,
        sorted_keys, all, num_keys, segments);
    GS_TRY(check_launch());
  }
  return GS_OK;
}

// Error word of the last binning on this workspace pair (sync-free read is
// the caller's job; 0 = no look-back ever timed out).
uint64_t bin_error_word_offset() { return offsetof(BinHeader, error); }

}  // namespace gs
