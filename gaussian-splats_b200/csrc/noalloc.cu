// gs_bin_noalloc: tile binning with library-owned scratch, for callers that
// cannot allocate device memory.
//
// The regular binning entry points (gs_bin_count / gs_bin_sort) take their
// scratch from the caller. Some callers have nothing to hand over: a plugin
// or FFI binding driven by a host program that owns every device allocation
// (the library must not call cudaMalloc behind its back, and may not have a
// handle on the host's allocator), or a per-frame render loop that cannot
// afford cudaMalloc's implicit device-wide synchronisation. For them this
// entry point runs the same two binning phases out of a fixed scratch array
// that lives in the library image itself.
//
// The scratch is a file-scope __device__ array of kScratchBytes (64 MiB).
// Every GPU that loads the library holds it until the process exits. Its
// device address is looked up once per device with cudaGetSymbolAddress
// (host code cannot use the array's name as a pointer: on the host that name
// is only a stand-in for the symbol). All calls on a device share the array
// and it keeps whatever the previous call left there; the binning launchers
// clear the counters and status words they need before every use, and calls
// whose work overlaps on the GPU (different streams, or several host
// threads) would race on the array, so the caller must serialise them.
#include <mutex>

#include "common.cuh"

namespace gs {

int32_t launch_bin_count(int64_t, const float*, const int32_t*, void*, int64_t*, uint32_t*,
                         cudaStream_t);
int32_t launch_bin_sort(int64_t, int64_t, const int32_t*, const int32_t*, const gs_params&,
                        const void*, void*, int32_t*, int64_t*, cudaStream_t);
uint64_t bin_count_workspace_size(int64_t);
uint64_t bin_sort_workspace_size(int64_t, int64_t, const gs_params&);
uint64_t bin_error_word_offset();

namespace {

constexpr uint64_t kScratchBytes = uint64_t{64} << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_bin_scratch[kScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_address[kMaxDevices] = {};

// Device address of g_bin_scratch on the current device (looked up once).
int32_t scratch_for_current_device(void** out) {
  int device = 0;
  GS_CUDA_TRY(cudaGetDevice(&device));
  if (device < 0 || device >= kMaxDevices) return GS_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_address[device]) {
    void* address = nullptr;
    GS_CUDA_TRY(cudaGetSymbolAddress(&address, g_bin_scratch));
    g_scratch_address[device] = address;
  }
  *out = g_scratch_address[device];
  return GS_OK;
}

inline uint64_t align256(uint64_t x) { return (x + 255) / 256 * 256; }

}  // namespace
}  // namespace gs

extern "C" int32_t gs_bin_noalloc(int64_t n, const float* projected_mean, const int32_t* counts,
                                  const int32_t* bounds, const gs_params* params,
                                  int32_t* gaussian_ids, int64_t ids_capacity, int64_t* ranges,
                                  int64_t* total_host, gs_stream_t stream) {
  // The same checks as gs_bin_count + gs_bin_sort.
  GS_TRY(gs::check_params(params));
  if (!total_host || n < 0 || n >= gs::kMaxGaussians || ids_capacity < 0)
    return GS_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(bounds) % 16) return GS_ERR_MISALIGNED;
  *total_host = 0;
  const uint64_t count_bytes = gs::align256(gs::bin_count_workspace_size(n));
  if (count_bytes > gs::kScratchBytes) return GS_ERR_CAPACITY;  // too many Gaussians
  void* scratch = nullptr;
  GS_TRY(gs::scratch_for_current_device(&scratch));
  const cudaStream_t s = gs::as_cuda(stream);
  uint32_t error = 0;
  int64_t total = 0;
  GS_TRY(gs::launch_bin_count(n, projected_mean, counts, scratch, &total, &error, s));
  *total_host = total;
  if (error) return GS_ERR_TIMEOUT;
  if (total > ids_capacity || total >= gs::kMaxIntersections ||
      count_bytes + gs::bin_sort_workspace_size(n, total, *params) > gs::kScratchBytes)
    return GS_ERR_CAPACITY;  // *total_host says how many intersections there were
  char* sort_scratch = static_cast<char*>(scratch) + count_bytes;
  GS_TRY(gs::launch_bin_sort(n, total, bounds, counts, *params, scratch, sort_scratch,
                             gaussian_ids, ranges, s));
  // The tile sort's look-back waits report into the sort scratch's error
  // word, which only this library can reach: read it back before returning.
  uint32_t sort_error = 0;
  GS_CUDA_TRY(cudaMemcpyAsync(&sort_error, sort_scratch + gs::bin_error_word_offset(),
                              sizeof(sort_error), cudaMemcpyDeviceToHost, s));
  GS_CUDA_TRY(cudaStreamSynchronize(s));
  return sort_error ? GS_ERR_TIMEOUT : GS_OK;
}
