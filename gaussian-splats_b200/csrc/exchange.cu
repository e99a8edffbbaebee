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

namespace {

struct ArenaHeader {
  unsigned long long epoch;  // steps published by this rank (this GPU only)
  unsigned int error;        // wait timeouts seen by this rank
  unsigned int pad;
  unsigned long long ready[GS_MAX_PEERS];  // [p]: last epoch rank p published
  unsigned long long done[GS_MAX_PEERS];   // [p]: last epoch rank p finished reading
};
static_assert(sizeof(ArenaHeader) <= 256, "header fits its 256 bytes");

constexpr unsigned kErrReadyTimeout = 1u;
constexpr unsigned kErrDoneTimeout = 2u;
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

uint64_t align256(uint64_t x) { return (x + 255) & ~uint64_t{255}; }

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

int32_t exchange_status(const gs_peer_group& g, cudaStream_t stream) {
  if (!valid_group(g)) return GS_ERR_INVALID_ARGUMENT;
  unsigned error = 0;
  GS_CUDA_TRY(cudaMemcpyAsync(&error, &static_cast<const ArenaHeader*>(g.arena[g.rank])->error,
                              sizeof(error), cudaMemcpyDeviceToHost, stream));
  GS_CUDA_TRY(cudaStreamSynchronize(stream));
  return error ? GS_ERR_TIMEOUT : GS_OK;
}

}  // namespace gs
