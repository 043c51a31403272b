// fa_sm100_bwd_noalloc: the attention backward for callers that cannot
// allocate device memory.
//
// Some hosts cannot call cudaMalloc (or any allocator) at the point where they
// run the backward: a runtime that hands out only pre-planned buffers, an
// embedding that forbids allocation in its execution phase, or code running
// under a fixed memory budget.  fa_sm100_bwd needs a caller-provided workspace
// (fp32 dQ accumulator plus per-row delta and LSE); this entry point instead
// uses one file-scope device array of FA_SM100_NOALLOC_SCRATCH_BYTES, created
// when the library is loaded on a GPU and kept until the process exits.
//
// The array's name is only a host-side stand-in in host code, so its device
// address is looked up with cudaGetSymbolAddress, once per device, with that
// device current, on the first call made on that device.  Make that first call
// before any stream capture.  The address is kept for the life of the process,
// so a device or primary-context reset (cudaDeviceReset) after that first call
// is not supported: the kept address would belong to the destroyed context.  Every call shares the one array: the kernels
// rewrite and re-zero the part they use on each call, and two calls whose
// kernels overlap on the GPU (different streams, or different host threads)
// race on it and give wrong results.
#include <cuda_runtime.h>

#include <mutex>

#include "fa_kernels.h"

namespace fa_sm100 {
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[FA_SM100_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (nullptr on error).
void* scratch_on_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaSetDevice(dev) != cudaSuccess) return nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return nullptr;
    g_scratch_ptr[dev] = p;
  }
  return g_scratch_ptr[dev];
}

}  // namespace
}  // namespace fa_sm100

extern "C" int fa_sm100_bwd_noalloc(const void* dout, const void* q, const void* k, const void* v,
                                    const void* out, const float* lse, void* dq, void* dk,
                                    void* dv, int batch, int seqlen, int nheads, int head_dim,
                                    float sm_scale, int causal, int* status, void* stream) {
  const size_t need = fa_sm100_bwd_workspace_bytes(batch, seqlen, nheads, head_dim);
  if (need == 0) return FA_ERR_ARG;
  if (need > (size_t)FA_SM100_NOALLOC_SCRATCH_BYTES) return FA_ERR_SCRATCH_LIMIT;
  void* scratch = fa_sm100::scratch_on_current_device();
  if (scratch == nullptr) return FA_ERR_DEVICE;
  return fa_sm100::bwd_impl(-1, dout, q, k, v, out, lse, dq, dk, dv, scratch,
                            (size_t)FA_SM100_NOALLOC_SCRATCH_BYTES, batch, seqlen, seqlen,
                            nheads, nheads, head_dim, FA_DTYPE_F16, sm_scale, causal, status,
                            stream, 0);
}
