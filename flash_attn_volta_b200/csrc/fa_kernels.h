// Internal launch interface between the C ABI layer (fa_api.cu) and the kernel
// translation units.  Not part of the public ABI.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <utility>

#include "../../include/fa_sm100.h"

namespace fa_sm100 {

struct FwdArgs {
  const CUtensorMap* tm_q;  // box rows: 128
  const CUtensorMap* tm_k;  // box rows: 128
  const CUtensorMap* tm_v;  // box rows: 128
  void* o;
  float* lse;
  int B, Sq, H, D;
  int Sk;   // key / value rows (Sq for square attention)
  int Hkv;  // K/V heads (H % Hkv == 0; H for plain multi-head attention)
  int dtype = FA_DTYPE_F16;
  float scale;
  int causal;
  int* status;
  unsigned long long timeout_ns;
  int debug_flags;  // test hooks, see fa_sm100_set_debug_flags
};

struct BwdArgs {
  const CUtensorMap* tm_q;   // box rows: bwd_q_rows(D)
  const CUtensorMap* tm_do;  // box rows: bwd_q_rows(D)
  const CUtensorMap* tm_k;   // box rows: 128
  const CUtensorMap* tm_v;   // box rows: 128
  const void* o;
  const void* dout;
  const float* lse;
  void* dq;
  void* dk;
  void* dv;
  float* dq_acc;   // (B*H, S_pad, D) fp32
  // (B*H, S_pad) rows of 16 fp16 in the MMA's no-swizzle K-major layout: the
  // extra K step of S^T (-LSE/scale) and of dP^T (-delta) as fp16 hi/lo pairs
  uint8_t* q_aug;
  uint8_t* do_aug;
  int B, Sq, H, D, S_pad;  // S_pad: Sq rounded up to kSeqPad
  int Sk;                  // key / value rows
  int Hkv;  // K/V heads (H % Hkv == 0); dk, dv are (B, S, Hkv, D)
  int dtype = FA_DTYPE_F16;
  float scale;
  int causal;
  int* status;
  unsigned long long timeout_ns;
  // dQ mode.  0: fused into the main kernel (partials added into dq_acc with L2
  // reductions, then converted by fa_bwd_post).  1: the main kernel computes
  // dK / dV only and fa_bwd_dq_kernel computes dQ per query tile in a fixed
  // key order (deterministic; needs tm_q128 / tm_do128 and delta).
  int dq_separate = 0;
  const CUtensorMap* tm_q128 = nullptr;   // box rows: 128
  const CUtensorMap* tm_do128 = nullptr;  // box rows: 128
  float* delta = nullptr;  // (B*H, S_pad) fp32 rowsum(O * dO), written by fa_bwd_pre
};

namespace {
// Raise a kernel's dynamic shared-memory limit once per device (the attribute
// is per device and function; setting it on every launch costs a driver call).
// `Tag` separates the callers' kernels; devices beyond 64 are set every time.
// Internal linkage: a function-local static of an inline function with external
// linkage becomes one process-wide symbol, which a second copy of this library
// loaded into the same process would share (and skip its own kernels' limits).
template <int Tag>
bool smem_attr_set(const void* func, int bytes) {
  static std::atomic<unsigned long long> done{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const unsigned long long bit = dev < 64 ? (1ull << dev) : 0ull;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return true;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return false;
  done.fetch_or(bit, std::memory_order_acq_rel);
  return true;
}
// Streaming multiprocessors of the current device (cached per device; 0 on error).
inline int sm_count() {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev < 64) {
    const int c = cache[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (dev < 64) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}
// Grid of a tile-list kernel: one CTA per SM walking the list when there are
// at most persist_max_tiles() tiles per SM (where the set-up and drain of each
// CTA and the balance of the last wave matter most; the persistent grid
// overlaps a tile's epilogue with the next tile's first loads and MMAs),
// otherwise one CTA per tile in list order.  The static split of the
// persistent grid balances tiles of one length well, and causal tiles of very
// different lengths less so, hence a lower limit for long causal sequences.
// Measured on one B200 (D=128, medians of 15 launches, persistent vs one CTA
// per tile):
//   B=8, S=2048, H=16 causal (13.8 tiles per SM): forward 0.229 -> 0.194 ms,
//     backward main kernel 0.528 -> 0.515 ms; non-causal +10 % / +4 %
//   B=1, S=8192, H=16 causal (6.9 per SM): forward 0.323 -> 0.303 ms,
//     backward unchanged
//   B=1, S=8192, H=32 (13.8 per SM): causal forward -4 %, backward -10 %;
//     non-causal +7 % / +3 %
//   B=2, S=8192, H=32 causal (27.7 per SM): forward -5 %
//   B=8, S=8192, H=32 causal (110 per SM): backward -12 %.
inline int persist_max_tiles(bool causal, int seqlen) {
  return (causal && seqlen > 4096) ? 8 : 16;
}
inline int tile_grid(int ntiles, int nsm, int max_per_sm) {
  return ntiles <= max_per_sm * nsm ? (ntiles < nsm ? ntiles : nsm) : ntiles;
}
// Heads per window of a tile list: 16 on the persistent grid (tiles dealt out
// in one round have similar lengths), 8 with one CTA per tile (fewer heads'
// data in L2 at once).
inline int tile_window(int ntiles, int grid) { return grid < ntiles ? 16 : 8; }
}  // namespace

// Launch with programmatic stream serialization: the kernel may start while the
// previous kernel in the stream finishes (it calls griddep_wait() before reading
// that kernel's outputs).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Bytes of one row of the augmented K step (16 fp16).
constexpr int kAugRowBytes = 32;
// Weight of the fourth row term of the augmented K step (a power of two, exact
// in fp16 and bf16): the K / V side holds [1, 1, 1, kAugBig, 0, ...].
constexpr int kAugBig = 2048;

int launch_fwd(const FwdArgs& a, cudaStream_t stream);
// phase -1: all three kernels; 0: delta/LSE prep; 1: main kernel; 2: dQ conversion
int launch_bwd(const BwdArgs& a, cudaStream_t stream, int phase);
// the separate dQ kernel (BwdArgs::dq_separate); fa_bwd_dq.cu
int launch_bwd_dq(const BwdArgs& a, cudaStream_t stream);
int bwd_q_rows(int D);

// Argument checks, tensor maps and launches of the backward on a caller-given
// workspace (phase as in launch_bwd).  Shared by the C ABI entry points.
int bwd_impl(int phase, const void* dout, const void* q, const void* k, const void* v,
             const void* out, const float* lse, void* dq, void* dk, void* dv, void* workspace,
             size_t workspace_bytes, int batch, int seqlen, int seqlen_k, int nheads,
             int nheads_kv, int head_dim, int dtype, float sm_scale, int causal, int* status,
             void* stream, int flags);

// sequence rows are padded to a multiple of this in the backward workspace
constexpr int kSeqPad = 128;

}  // namespace fa_sm100
