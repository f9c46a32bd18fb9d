// Forward-only chunkwise GDN2 for callers that cannot allocate device memory.
//
// Some hosts of this operator may not call cudaMalloc at all: serving engines
// that reserve the whole device up front for their state and KV pools and
// forbid allocation afterwards, plugins running inside a framework that owns
// the allocator (and give the plugin no handle to it), and latency-critical
// loops where an allocation's implicit device synchronisation is not
// acceptable.  For them gdn2_chunk_fwd_static_scratch runs the same kernels as
// gdn2_chunk_fwd, but takes its scratch (the WY factors the scan consumes)
// from one file-scope device array of fixed size instead of a caller buffer.
//
// Rules of the array:
//   * it is kStaticScratchBytes (32 MiB) and exists on every GPU that loads
//     this library, for the life of the process;
//   * every call shares it and it keeps whatever the last call wrote.  Nothing
//     in it has to start at zero: the forward writes every scratch element it
//     later reads, and rows past a sequence end are masked on load;
//   * two calls whose kernels overlap on the GPU (different streams, or
//     different host threads on one device) race on it: serialise them;
//   * host code cannot use the array's name as a device address.  The first
//     call on each device (with that device current) asks the runtime for the
//     address with cudaGetSymbolAddress and caches it; make that first call
//     before any stream capture.  The cache is keyed by device ordinal, so it
//     holds for the device's primary context (the one the runtime API uses):
//     a caller that makes another driver context current, or that resets the
//     device (cudaDeviceReset), must restart the process before calling again.
#include <mutex>

#include "chunk_layout.cuh"
#include "common.cuh"

namespace {

constexpr size_t kStaticScratchBytes = size_t(32) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_fwd_scratch[kStaticScratchBytes];

std::mutex g_mu;
void* g_addr[kMaxDevices] = {nullptr};

int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return -static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) return GDN2_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_fwd_scratch);
    if (e != cudaSuccess) return -static_cast<int>(e);
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return GDN2_OK;
}

}  // namespace

extern "C" int gdn2_chunk_fwd_static_scratch(const gdn2_chunk_args* a, gdn2_stream_t stream) {
  if (!a) return GDN2_ERR_NULL_POINTER;
  // the backward reads a context that must outlive this call: not here
  if (a->flags & GDN2_SAVE_FOR_BWD) return GDN2_ERR_FLAGS;
  // skipping the intra kernel would scan whatever factors the previous call
  // (possibly another problem, or another caller) left in the shared array
  if (a->flags & GDN2_SKIP_INTRA) return GDN2_ERR_FLAGS;
  const size_t need = gdn2_chunk_workspace_size(a);
  if (need == 0) return gdn2_chunk_fwd(a, nullptr, 0, stream);  // empty problem, or the argument error
  if (need > kStaticScratchBytes) return GDN2_ERR_SCRATCH_LIMIT;
  void* base = nullptr;
  int st = scratch_address(&base);
  if (st) return st;
  return gdn2_chunk_fwd(a, base, kStaticScratchBytes, stream);
}
