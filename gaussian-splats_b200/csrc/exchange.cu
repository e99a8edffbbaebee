// Screen-space gradient exchange over peer memory, for view-parallel training
// with one view per rank (no counterpart in the single-device reference).
//
// Every rank owns an exchange arena in memory all ranks can map (symmetric
// memory): a header of step counters, then the rank's screen-space gradient
// [n, 9] (compositing backward writes it there), tile counts [n], its view
// record and the gathered records of every rank. A step is
//   gs_exchange_begin   wait until every peer has finished reading this
//                       rank's arena of the previous step (its `done` flag);
//   ... compositing backward into the arena, counts and record copied in ...
//   gs_exchange_publish bump this rank's epoch, make its writes visible
//                       system-wide, store the epoch into every peer's `ready`
//                       slot, wait for every peer's, and gather the records;
//   gs_exchange_gather  bulk-copy every peer's gradient and counts over
//                       NVLink into this GPU (copy engines, full link rate);
//   gs_exchange_finish  store the epoch into every peer's `done` slot: the
//                       peers may overwrite their arenas from here on;
//   gs_project_bwd_peers  the projection backward summed over all ranks'
//                       views (no collective anywhere in the step).
// Reading the gradients straight from peer memory inside the projection
// backward (gs_project_bwd_peers without gathered buffers) also works, but its
// scattered 36-byte rows over NVLink cost more than the bulk copy.
// Sharded variant (gs_exchange_gather_rows .. gs_exchange_gather_shards): rank
// r owns Gaussians [r*rows, (r+1)*rows). After the publish it copies only its
// shard's rows of every rank's gradient and counts, runs the projection
// backward over all views for its shard alone into the arena's shard region,
// releases `shard_ready` to the peers, waits for theirs and copies every
// rank's finished shard of parameter gradients; then gs_exchange_finish. Per
// rank that moves rows x 40 B from each peer plus the other shards' gradients
// (7/8 of 59 floats per Gaussian at 8 ranks, SH degree 3), and the per-view
// arithmetic of the summed backward is split W ways instead of repeated on
// every rank.
// The epochs live in device memory, so the sequence replays from a CUDA graph.
// Each wait is bounded (about a second): on expiry it records an error bit in
// the header and returns; gs_exchange_status reports it.

#include "common.cuh"

namespace gs {

int32_t exchange_layout(int64_t n, int32_t world, gs_exchange_layout* out);
int32_t launch_exchange_begin(const gs_peer_group& g, cudaStream_t stream);
int32_t launch_exchange_publish(const gs_peer_group& g, int64_t n, cudaStream_t stream);
int32_t launch_exchange_finish(const gs_peer_group& g, cudaStream_t stream);
int32_t exchange_gather(const gs_peer_group& g, int64_t n, float* grad_projected,
                        int32_t* counts, cudaStream_t stream);
int32_t exchange_status(const gs_peer_group& g, cudaStream_t stream);
int32_t exchange_shard_layout(int64_t n, int32_t world, int32_t num_sh, gs_shard_layout* out);
int32_t exchange_gather_rows(const gs_peer_group& g, int64_t n, float* grad_rows,
                             int32_t* count_rows, cudaStream_t stream);
int32_t launch_exchange_publish_shard(const gs_peer_group& g, cudaStream_t stream);
int32_t exchange_gather_shards(const gs_peer_group& g, int64_t n, int32_t num_sh,
                               float* grad_rotation, float* grad_color, float* grad_mean,
                               float* grad_scale, float* grad_opacity, cudaStream_t stream);
int32_t launch_project_bwd_peers(int64_t, int32_t, int32_t, const float*, const float*,
                                 const float*, const float*, const float*, const void*,
                                 const float* const*, const int32_t* const*, float*, float*,
                                 float*, float*, float*, cudaStream_t);
int32_t launch_project_bwd_shard(int64_t n, int32_t num_sh, const gs_peer_group& g,
                                 const float* grad_rows, const int32_t* count_rows,
                                 const float* mean, const float* rotation, const float* scale,
                                 const float* opacity, const float* color, cudaStream_t stream);

namespace {

struct ArenaHeader {
  unsigned long long epoch;  // steps published by this rank (this GPU only)
  unsigned int error;        // wait timeouts seen by this rank
  unsigned int pad;
  unsigned long long ready[GS_MAX_PEERS];  // [p]: last epoch rank p published
  unsigned long long done[GS_MAX_PEERS];   // [p]: last epoch rank p finished reading
  unsigned long long shard_ready[GS_MAX_PEERS];  // [p]: last epoch rank p finished its shard
};
static_assert(sizeof(ArenaHeader) <= 256, "header fits its 256 bytes");

constexpr unsigned kErrReadyTimeout = 1u;
constexpr unsigned kErrDoneTimeout = 2u;
constexpr unsigned kErrShardTimeout = 4u;
constexpr long long kWaitCycles = 2000000000LL;  // ~1 s at the B200's clocks
constexpr int kRecordWords = 29;

__device__ __forceinline__ ArenaHeader* header(void* arena) {
  return static_cast<ArenaHeader*>(arena);
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Spins until *flag >= target (acquire, system scope); false if it gave up.
__device__ bool wait_at_least(const unsigned long long* flag, unsigned long long target) {
  const long long start = clock64();
  while (ld_acquire_sys(flag) < target) {
    if (clock64() - start > kWaitCycles) return false;
    __nanosleep(128);
  }
  return true;
}

// One warp; lane p deals with peer p.
__global__ void exchange_begin_kernel(gs_peer_group g) {
  ArenaHeader* me = header(g.arena[g.rank]);
  const int p = threadIdx.x;
  if (p < g.world && p != g.rank) {
    if (!wait_at_least(&me->done[p], me->epoch)) atomicOr(&me->error, kErrDoneTimeout);
  }
}

__global__ void exchange_publish_kernel(gs_peer_group g, gs_exchange_layout layout) {
  ArenaHeader* me = header(g.arena[g.rank]);
  const int p = threadIdx.x;
  const unsigned long long epoch = me->epoch + 1;
  __syncwarp();
  if (p == 0) me->epoch = epoch;
  // This rank's gradient, counts and record (written by earlier work on this
  // stream) become visible to the peers before its flag does.
  __threadfence_system();
  if (p < g.world && p != g.rank) st_release_sys(&header(g.arena[p])->ready[g.rank], epoch);
  if (p < g.world) {
    if (p != g.rank && !wait_at_least(&me->ready[p], epoch))
      atomicOr(&me->error, kErrReadyTimeout);
    // the lane that acquired peer p's flag copies peer p's record
    const unsigned* src =
        reinterpret_cast<const unsigned*>(static_cast<const char*>(g.arena[p]) + layout.record);
    unsigned* dst = reinterpret_cast<unsigned*>(static_cast<char*>(g.arena[g.rank]) +
                                                layout.gathered) + p * kRecordWords;
    for (int w = 0; w < kRecordWords; ++w) dst[w] = __ldcg(src + w);
  }
}

__global__ void exchange_finish_kernel(gs_peer_group g) {
  ArenaHeader* me = header(g.arena[g.rank]);
  const int p = threadIdx.x;
  if (p < g.world && p != g.rank) st_release_sys(&header(g.arena[p])->done[g.rank], me->epoch);
}

// After this rank's shard of parameter gradients is in its arena (earlier
// work on the stream): release `shard_ready` to every peer and wait for
// theirs. One warp; lane p deals with peer p.
__global__ void exchange_publish_shard_kernel(gs_peer_group g) {
  ArenaHeader* me = header(g.arena[g.rank]);
  const int p = threadIdx.x;
  const unsigned long long epoch = me->epoch;  // bumped by this step's publish
  __threadfence_system();
  if (p < g.world && p != g.rank) {
    st_release_sys(&header(g.arena[p])->shard_ready[g.rank], epoch);
    if (!wait_at_least(&me->shard_ready[p], epoch)) atomicOr(&me->error, kErrShardTimeout);
  }
}

uint64_t align256(uint64_t x) { return (x + 255) & ~uint64_t{255}; }

// Byte ranges one copy launch moves (from peers' arenas or this GPU's own),
// in order. Sources and destinations start on 16-byte boundaries.
constexpr int kMaxSegments = 5 * GS_MAX_PEERS;
struct CopySegment {
  const char* src;
  char* dst;
  uint64_t bytes;
};
struct CopyPlan {
  CopySegment seg[kMaxSegments];
  int count;
};

// Copies `bytes` from src to dst as words of type W (both aligned to W),
// every thread of the grid `kCopyUnroll` words in flight; loads read at L2.
constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 4;
template <class W>
__device__ __forceinline__ void copy_words(const char* src_bytes, char* dst_bytes,
                                           uint64_t bytes, uint64_t tid, uint64_t threads) {
  const uint64_t words = bytes / sizeof(W);
  const W* src = reinterpret_cast<const W*>(src_bytes);
  W* dst = reinterpret_cast<W*>(dst_bytes);
  uint64_t i = tid;
  for (; i + (kCopyUnroll - 1) * threads < words; i += kCopyUnroll * threads) {
    W v[kCopyUnroll];
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) v[u] = __ldcg(src + i + u * threads);
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) dst[i + u * threads] = v[u];
  }
  for (; i < words; i += threads) dst[i] = __ldcg(src + i);
  for (uint64_t b = words * sizeof(W) + tid; b < bytes; b += threads)
    dst_bytes[b] = __ldcg(reinterpret_cast<const signed char*>(src_bytes) + b);
}

// Every CTA of the grid walks every segment: 16-byte words where both ends
// allow, else 4-byte words (every segment holds whole floats or ints). The
// data came from other GPUs this step, so loads read at L2. Peer reads go
// over NVLink from the SMs -- all links of this GPU at once -- instead of one
// copy-engine transfer after another.
__global__ void __launch_bounds__(kCopyThreads) peer_copy_kernel(const __grid_constant__ CopyPlan plan) {
  const uint64_t tid = static_cast<uint64_t>(blockIdx.x) * kCopyThreads + threadIdx.x;
  const uint64_t threads = static_cast<uint64_t>(gridDim.x) * kCopyThreads;
  for (int s = 0; s < plan.count; ++s) {
    const CopySegment seg = plan.seg[s];
    const uintptr_t ends = reinterpret_cast<uintptr_t>(seg.src) | reinterpret_cast<uintptr_t>(seg.dst);
    if (ends % 16 == 0)
      copy_words<uint4>(seg.src, seg.dst, seg.bytes, tid, threads);
    else
      copy_words<uint32_t>(seg.src, seg.dst, seg.bytes, tid, threads);
  }
}

int32_t launch_copy(const CopyPlan& plan, uint64_t bytes, cudaStream_t stream) {
  if (plan.count == 0 || bytes == 0) return GS_OK;
  // enough CTAs to keep every link busy, no more than the work needs
  const uint64_t want = (bytes / 16 + kCopyThreads * kCopyUnroll - 1) / (kCopyThreads * kCopyUnroll);
  const unsigned blocks = static_cast<unsigned>(want < 4 * kSmCount ? (want ? want : 1)
                                                                    : 4 * kSmCount);
  peer_copy_kernel<<<blocks, kCopyThreads, 0, stream>>>(plan);
  return check_launch();
}

// Gaussians per shard: ceil(n / world) rounded up to a multiple of 64, so
// every shard starts at a 16-byte boundary of every per-Gaussian array (the
// copies below move 16-byte words).
int64_t shard_rows(int64_t n, int world) {
  const int64_t rows = (n + world - 1) / world;
  return (rows + 63) / 64 * 64;
}

// Gaussians of rank p's shard: [first, first + count).
void shard_span(int64_t n, int64_t rows, int p, int64_t* first, int64_t* count) {
  const int64_t lo = rows * p < n ? rows * p : n;
  const int64_t hi = rows * (p + 1) < n ? rows * (p + 1) : n;
  *first = lo;
  *count = hi - lo;
}

bool valid_group(const gs_peer_group& g) {
  if (g.world < 1 || g.world > GS_MAX_PEERS || g.rank < 0 || g.rank >= g.world) return false;
  for (int p = 0; p < g.world; ++p)
    if (!g.arena[p] || reinterpret_cast<uintptr_t>(g.arena[p]) % 256) return false;
  return true;
}

}  // namespace

int32_t exchange_layout(int64_t n, int32_t world, gs_exchange_layout* out) {
  if (!out || n < 0 || world < 1 || world > GS_MAX_PEERS) return GS_ERR_INVALID_ARGUMENT;
  uint64_t at = 256;
  out->grad_projected = at;
  at = align256(at + 36 * static_cast<uint64_t>(n));
  out->counts = at;
  at = align256(at + 4 * static_cast<uint64_t>(n));
  out->record = at;
  at = align256(at + 4 * kRecordWords);
  out->gathered = at;
  at = align256(at + 4 * kRecordWords * GS_MAX_PEERS);
  out->bytes = at;
  return GS_OK;
}

int32_t launch_exchange_begin(const gs_peer_group& g, cudaStream_t stream) {
  if (!valid_group(g)) return GS_ERR_INVALID_ARGUMENT;
  exchange_begin_kernel<<<1, 32, 0, stream>>>(g);
  return check_launch();
}

int32_t launch_exchange_publish(const gs_peer_group& g, int64_t n, cudaStream_t stream) {
  if (!valid_group(g)) return GS_ERR_INVALID_ARGUMENT;
  gs_exchange_layout layout;
  GS_TRY(exchange_layout(n, g.world, &layout));
  exchange_publish_kernel<<<1, 32, 0, stream>>>(g, layout);
  return check_launch();
}

int32_t launch_exchange_finish(const gs_peer_group& g, cudaStream_t stream) {
  if (!valid_group(g)) return GS_ERR_INVALID_ARGUMENT;
  exchange_finish_kernel<<<1, 32, 0, stream>>>(g);
  return check_launch();
}

// Copies every peer's gradient and counts into this GPU's [world, n, 9] and
// [world, n] buffers (slot p for rank p; this rank's slot is left alone):
// bulk copies over NVLink instead of the projection backward's scattered peer
// loads. Queued after gs_exchange_publish, whose wait they follow in stream
// order.
int32_t exchange_gather(const gs_peer_group& g, int64_t n, float* grad_projected,
                        int32_t* counts, cudaStream_t stream) {
  if (!valid_group(g) || !grad_projected || !counts) return GS_ERR_INVALID_ARGUMENT;
  gs_exchange_layout layout;
  GS_TRY(exchange_layout(n, g.world, &layout));
  for (int p = 0; p < g.world; ++p) {
    if (p == g.rank) continue;
    const char* base = static_cast<const char*>(g.arena[p]);
    GS_CUDA_TRY(cudaMemcpyAsync(grad_projected + 9 * n * p, base + layout.grad_projected,
                                36 * static_cast<size_t>(n), cudaMemcpyDeviceToDevice, stream));
    GS_CUDA_TRY(cudaMemcpyAsync(counts + n * p, base + layout.counts,
                                4 * static_cast<size_t>(n), cudaMemcpyDeviceToDevice, stream));
  }
  return GS_OK;
}

int32_t exchange_shard_layout(int64_t n, int32_t world, int32_t num_sh, gs_shard_layout* out) {
  if (!out || num_sh < 1 || num_sh > 25) return GS_ERR_INVALID_ARGUMENT;
  gs_exchange_layout base;
  GS_TRY(exchange_layout(n, world, &base));
  const uint64_t rows = static_cast<uint64_t>(shard_rows(n, world));
  uint64_t at = align256(base.bytes);
  out->rotation = at;
  at = align256(at + 16 * rows);
  out->color = at;
  at = align256(at + 12 * static_cast<uint64_t>(num_sh) * rows);
  out->mean = at;
  at = align256(at + 12 * rows);
  out->scale = at;
  at = align256(at + 12 * rows);
  out->opacity = at;
  at = align256(at + 4 * rows);
  out->bytes = at;
  out->rows = static_cast<int64_t>(rows);
  return GS_OK;
}

// Copies this rank's shard rows of every rank's screen-space gradient and
// counts (this rank's own too) into [world, rows, 9] / [world, rows] local
// buffers: one contiguous block of each array per rank.
int32_t exchange_gather_rows(const gs_peer_group& g, int64_t n, float* grad_rows,
                             int32_t* count_rows, cudaStream_t stream) {
  if (!valid_group(g) || !grad_rows || !count_rows) return GS_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(grad_rows) % 4 || reinterpret_cast<uintptr_t>(count_rows) % 4)
    return GS_ERR_MISALIGNED;
  gs_exchange_layout layout;
  GS_TRY(exchange_layout(n, g.world, &layout));
  const int64_t rows = shard_rows(n, g.world);
  int64_t first, count;
  shard_span(n, rows, g.rank, &first, &count);
  if (count <= 0) return GS_OK;
  CopyPlan plan{};
  uint64_t bytes = 0;
  for (int step = 1; step <= g.world; ++step) {
    const int p = (g.rank + step) % g.world;  // peers first (staggered), this rank last
    const char* base = static_cast<const char*>(g.arena[p]);
    const size_t f = static_cast<size_t>(first), c = static_cast<size_t>(count);
    plan.seg[plan.count++] = {base + layout.grad_projected + 36 * f,
                              reinterpret_cast<char*>(grad_rows + 9 * rows * p), 36 * c};
    plan.seg[plan.count++] = {base + layout.counts + 4 * f,
                              reinterpret_cast<char*>(count_rows + rows * p), 4 * c};
    bytes += 40 * c;
  }
  return launch_copy(plan, bytes, stream);
}

// The summed projection backward of this rank's shard, over every rank's
// view, into the shard region of this rank's arena.
int32_t launch_project_bwd_shard(int64_t n, int32_t num_sh, const gs_peer_group& g,
                                 const float* grad_rows, const int32_t* count_rows,
                                 const float* mean, const float* rotation, const float* scale,
                                 const float* opacity, const float* color, cudaStream_t stream) {
  if (!valid_group(g) || !grad_rows || !count_rows) return GS_ERR_INVALID_ARGUMENT;
  gs_exchange_layout layout;
  gs_shard_layout shard;
  GS_TRY(exchange_layout(n, g.world, &layout));
  GS_TRY(exchange_shard_layout(n, g.world, num_sh, &shard));
  int64_t first, count;
  shard_span(n, shard.rows, g.rank, &first, &count);
  if (count <= 0) return GS_OK;
  const float* grads[GS_MAX_PEERS] = {};  // rows of view v: [v * shard.rows, +count)
  const int32_t* counts[GS_MAX_PEERS] = {};
  for (int v = 0; v < g.world; ++v) {
    grads[v] = grad_rows + 9 * shard.rows * v;
    counts[v] = count_rows + shard.rows * v;
  }
  char* me = static_cast<char*>(g.arena[g.rank]);
  const int64_t k3 = 3 * static_cast<int64_t>(num_sh);
  return launch_project_bwd_peers(
      count, num_sh, g.world, mean + 3 * first, rotation + 4 * first, scale + 3 * first,
      opacity + first, color + k3 * first, me + layout.gathered, grads, counts,
      reinterpret_cast<float*>(me + shard.mean), reinterpret_cast<float*>(me + shard.rotation),
      reinterpret_cast<float*>(me + shard.scale), reinterpret_cast<float*>(me + shard.opacity),
      reinterpret_cast<float*>(me + shard.color), stream);
}

int32_t launch_exchange_publish_shard(const gs_peer_group& g, cudaStream_t stream) {
  if (!valid_group(g)) return GS_ERR_INVALID_ARGUMENT;
  exchange_publish_shard_kernel<<<1, 32, 0, stream>>>(g);
  return check_launch();
}

// Copies every rank's finished shard of parameter gradients (this rank's from
// its own arena) into the full gradient arrays.
int32_t exchange_gather_shards(const gs_peer_group& g, int64_t n, int32_t num_sh,
                               float* grad_rotation, float* grad_color, float* grad_mean,
                               float* grad_scale, float* grad_opacity, cudaStream_t stream) {
  if (!valid_group(g) || !grad_rotation || !grad_color || !grad_mean || !grad_scale ||
      !grad_opacity)
    return GS_ERR_INVALID_ARGUMENT;
  for (const float* ptr : {grad_rotation, grad_color, grad_mean, grad_scale, grad_opacity})
    if (reinterpret_cast<uintptr_t>(ptr) % 4) return GS_ERR_MISALIGNED;
  gs_shard_layout shard;
  GS_TRY(exchange_shard_layout(n, g.world, num_sh, &shard));
  const size_t k3 = 3 * static_cast<size_t>(num_sh);
  CopyPlan plan{};
  uint64_t bytes = 0;
  for (int step = 1; step <= g.world; ++step) {
    const int p = (g.rank + step) % g.world;  // peers first (staggered), this rank last
    int64_t first, count;
    shard_span(n, shard.rows, p, &first, &count);
    if (count <= 0) continue;
    const char* base = static_cast<const char*>(g.arena[p]);
    const size_t f = static_cast<size_t>(first), c = static_cast<size_t>(count);
    struct {
      float* dst;
      uint64_t offset;
      size_t width;
    } parts[5] = {{grad_rotation, shard.rotation, 4}, {grad_color, shard.color, k3},
                  {grad_mean, shard.mean, 3}, {grad_scale, shard.scale, 3},
                  {grad_opacity, shard.opacity, 1}};
    for (const auto& part : parts) {
      plan.seg[plan.count++] = {base + part.offset,
                                reinterpret_cast<char*>(part.dst + part.width * f),
                                4 * part.width * c};
      bytes += 4 * part.width * c;
    }
  }
  return launch_copy(plan, bytes, stream);
}

int32_t exchange_status(const gs_peer_group& g, cudaStream_t stream) {
  if (!valid_group(g)) return GS_ERR_INVALID_ARGUMENT;
  unsigned error = 0;
  GS_CUDA_TRY(cudaMemcpyAsync(&error, &static_cast<const ArenaHeader*>(g.arena[g.rank])->error,
                              sizeof(error), cudaMemcpyDeviceToHost, stream));
  GS_CUDA_TRY(cudaStreamSynchronize(stream));
  return error ? GS_ERR_TIMEOUT : GS_OK;
}

}  // namespace gs
