// C ABI of libfa_sm100.so (declared in include/fa_sm100.h): argument checks,
// TMA tensor-map construction over the caller's (B, S, H, D) buffers, workspace
// carving and kernel launches.  Holds no per-call state.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "fa_kernels.h"

namespace fa_sm100 {
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

std::atomic<unsigned long long> g_timeout_ns{4000000000ull};
std::atomic<int> g_debug_flags{0};

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// The current device must be compute capability 10.0 (B200 / sm_100a).  Also
// makes the device's primary context current in the calling thread (a thread
// that has only made runtime calls that do not bind a context, such as torch's
// autograd worker, has none, and the driver-level tensor-map encoder then
// fails with CUDA_ERROR_INVALID_CONTEXT).
int check_device() {
  // per host thread: the device whose primary context this thread has bound;
  // per device: 1 = compute capability 10.0, 2 = not (checked once)
  thread_local int bound_dev = -1;
  static std::atomic<int> cc_state[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FA_ERR_DEVICE;
  if (dev != bound_dev) {
    if (cudaSetDevice(dev) != cudaSuccess) return FA_ERR_DEVICE;
    bound_dev = dev;
  }
  int state = dev < 64 ? cc_state[dev].load(std::memory_order_relaxed) : 0;
  if (state == 0) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return FA_ERR_DEVICE;
    state = (major == 10 && minor == 0) ? 1 : 2;
    if (dev < 64) cc_state[dev].store(state, std::memory_order_relaxed);
  }
  return state == 1 ? FA_OK : FA_ERR_DEVICE;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool valid_shape(int B, int S, int H, int D) {
  // grid limits: batch*heads is a grid y extent of the backward's pre/post
  // kernels (<= 65535); the main kernels use a 1-D grid of heads x blocks
  return B > 0 && S > 0 && H > 0 && (D == 16 || D == 32 || D == 64 || D == 128) &&
         (long long)B * H <= 65535LL &&
         (long long)B * H * ((S + 127) / 128) <= 2147483647LL;
}

// Tensor map over a contiguous (B, S, H, D) fp16 tensor; a box is `rows`
// consecutive sequence positions of one (b, h) and one swizzle-width slice of D.
int make_bshd_map(CUtensorMap* m, const void* ptr, int B, int S, int H, int D, int rows,
                  int dtype) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return FA_ERR_DEVICE;
  const int swb = D * 2 >= 128 ? 128 : D * 2;
  const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  const cuuint64_t strides[3] = {(cuuint64_t)H * D * 2, (cuuint64_t)D * 2,
                                 (cuuint64_t)S * H * D * 2};
  const cuuint32_t box[4] = {(cuuint32_t)(swb / 2), (cuuint32_t)rows, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapSwizzle swz = swb == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : swb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                             : CU_TENSOR_MAP_SWIZZLE_32B;
  const CUtensorMapDataType ty =
      dtype == FA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = enc(m, ty, 4, const_cast<void*>(ptr), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS && std::getenv("FA_SM100_DEBUG")) {
    std::fprintf(stderr,
                 "fa_sm100: cuTensorMapEncodeTiled failed (CUresult %d) ptr=%p dims={%d,%d,%d,%d} "
                 "strides={%llu,%llu,%llu} box={%u,%u,1,1}\n",
                 (int)r, ptr, D, S, H, B, (unsigned long long)strides[0],
                 (unsigned long long)strides[1], (unsigned long long)strides[2], box[0], box[1]);
  }
  return r == CUDA_SUCCESS ? FA_OK : FA_ERR_TMA;
}

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct WsLayout {
  size_t dq_acc, q_aug, do_aug, delta, total;
};

// Backward workspace.  Fused dQ: fp32 dQ accumulator, then the extra-K-step
// rows of Q and dO.  Separate dQ kernel (FA_BWD_DETERMINISTIC): the extra-K-step
// rows and delta (fp32 per row); no accumulator.
WsLayout ws_layout(int B, int S, int H, int D, bool sep) {
  const size_t S_pad = round_up((size_t)S, kSeqPad);
  const size_t rows = (size_t)B * H * S_pad;
  WsLayout w;
  w.dq_acc = 0;
  w.q_aug = sep ? 0 : round_up(rows * D * sizeof(float), 256);
  w.do_aug = w.q_aug + round_up(rows * kAugRowBytes, 256);
  w.delta = w.do_aug + round_up(rows * kAugRowBytes, 256);
  w.total = w.delta + (sep ? round_up(rows * sizeof(float), 256) : 0);
  return w;
}

}  // namespace
}  // namespace fa_sm100

using namespace fa_sm100;

extern "C" {

int fa_sm100_abi_version(void) { return FA_SM100_ABI_VERSION; }

const char* fa_sm100_error_string(int code) {
  switch (code) {
    case FA_OK: return "ok";
    case FA_ERR_ARG: return "invalid argument (shape, head_dim, null or misaligned pointer)";
    case FA_ERR_TMA: return "TMA tensor map encoding failed";
    case FA_ERR_LAUNCH: return "kernel launch failed";
    case FA_ERR_DEVICE: return "current device is not sm_100 or the driver entry point is missing";
    case FA_ERR_WORKSPACE: return "workspace missing or too small";
    case FA_ERR_SCRATCH_LIMIT:
      return "shape needs more scratch than the static array of fa_sm100_bwd_noalloc (32 MiB)";
    default: return "unknown error";
  }
}

void fa_sm100_set_wait_timeout_ns(uint64_t ns) { g_timeout_ns.store(ns ? ns : 1ull); }

void fa_sm100_set_debug_flags(int flags) { g_debug_flags.store(flags); }

}  // extern "C"

namespace {
int fwd_impl(const void* q, const void* k, const void* v, void* out, float* lse, int batch,
             int seqlen, int seqlen_k, int nheads, int nheads_kv, int head_dim, int dtype,
             float sm_scale, int causal, int* status, void* stream) {
  if (!valid_shape(batch, seqlen, nheads, head_dim)) return FA_ERR_ARG;
  if (!valid_shape(batch, seqlen_k, nheads, head_dim)) return FA_ERR_ARG;
  if (nheads_kv < 1 || nheads % nheads_kv != 0) return FA_ERR_ARG;
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return FA_ERR_ARG;
  if (!q || !k || !v || !out || !aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return FA_ERR_ARG;
  if (lse && (reinterpret_cast<uintptr_t>(lse) & 3u)) return FA_ERR_ARG;
  int rc = check_device();
  if (rc != FA_OK) return rc;
  CUtensorMap tq, tk, tv;
  if ((rc = make_bshd_map(&tq, q, batch, seqlen, nheads, head_dim, 128, dtype)) != FA_OK)
    return rc;
  if ((rc = make_bshd_map(&tk, k, batch, seqlen_k, nheads_kv, head_dim, 128, dtype)) != FA_OK)
    return rc;
  if ((rc = make_bshd_map(&tv, v, batch, seqlen_k, nheads_kv, head_dim, 128, dtype)) != FA_OK)
    return rc;
  FwdArgs a;
  a.tm_q = &tq;
  a.tm_k = &tk;
  a.tm_v = &tv;
  a.o = out;
  a.lse = lse;
  a.B = batch;
  a.Sq = seqlen;
  a.Sk = seqlen_k;
  a.H = nheads;
  a.Hkv = nheads_kv;
  a.dtype = dtype;
  a.D = head_dim;
  a.scale = sm_scale;
  a.causal = causal ? 1 : 0;
  a.status = status;
  a.timeout_ns = g_timeout_ns.load();
  a.debug_flags = g_debug_flags.load();
  return launch_fwd(a, static_cast<cudaStream_t>(stream));
}
}  // namespace

extern "C" {

int fa_sm100_fwd(const void* q, const void* k, const void* v, void* out, float* lse, int batch,
                 int seqlen, int nheads, int head_dim, float sm_scale, int causal, int* status,
                 void* stream) {
  return fwd_impl(q, k, v, out, lse, batch, seqlen, seqlen, nheads, nheads, head_dim,
                  FA_DTYPE_F16, sm_scale, causal, status, stream);
}

int fa_sm100_fwd_ex(const void* q, const void* k, const void* v, void* out, float* lse,
                    int batch, int seqlen_q, int seqlen_k, int nheads, int nheads_kv,
                    int head_dim, int dtype, float sm_scale, int causal, int* status,
                    void* stream) {
  return fwd_impl(q, k, v, out, lse, batch, seqlen_q, seqlen_k, nheads, nheads_kv, head_dim,
                  dtype, sm_scale, causal, status, stream);
}

size_t fa_sm100_bwd_workspace_bytes(int batch, int seqlen, int nheads, int head_dim) {
  if (!valid_shape(batch, seqlen, nheads, head_dim)) return 0;
  return ws_layout(batch, seqlen, nheads, head_dim, false).total;
}

size_t fa_sm100_bwd_workspace_bytes_flags(int batch, int seqlen, int nheads, int head_dim,
                                          int flags) {
  if (!valid_shape(batch, seqlen, nheads, head_dim) || (flags & ~FA_BWD_DETERMINISTIC)) return 0;
  return ws_layout(batch, seqlen, nheads, head_dim, (flags & FA_BWD_DETERMINISTIC) != 0).total;
}

}  // extern "C"

int fa_sm100::bwd_impl(int phase, const void* dout, const void* q, const void* k,
                              const void* v, const void* out, const float* lse, void* dq, void* dk,
                              void* dv, void* workspace, size_t workspace_bytes, int batch, int seqlen,
                              int seqlen_k, int nheads, int nheads_kv, int head_dim, int dtype,
                              float sm_scale, int causal, int* status, void* stream, int flags) {
  if (!valid_shape(batch, seqlen, nheads, head_dim)) return FA_ERR_ARG;
  if (!valid_shape(batch, seqlen_k, nheads, head_dim)) return FA_ERR_ARG;
  if (nheads_kv < 1 || nheads % nheads_kv != 0) return FA_ERR_ARG;
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return FA_ERR_ARG;
  const void* ptrs[] = {dout, q, k, v, out, dq, dk, dv};
  for (const void* p : ptrs)
    if (!p || !aligned16(p)) return FA_ERR_ARG;
  if (!lse || (reinterpret_cast<uintptr_t>(lse) & 3u)) return FA_ERR_ARG;
  if (flags & ~FA_BWD_DETERMINISTIC) return FA_ERR_ARG;
  const bool sep = (flags & FA_BWD_DETERMINISTIC) != 0;
  const WsLayout w = ws_layout(batch, seqlen, nheads, head_dim, sep);
  if (!workspace || workspace_bytes < w.total || (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return FA_ERR_WORKSPACE;
  int rc = check_device();
  if (rc != FA_OK) return rc;
  const int qrows = bwd_q_rows(head_dim);
  CUtensorMap tq, tdo, tk, tv;
  if ((rc = make_bshd_map(&tq, q, batch, seqlen, nheads, head_dim, qrows, dtype)) != FA_OK)
    return rc;
  if ((rc = make_bshd_map(&tdo, dout, batch, seqlen, nheads, head_dim, qrows, dtype)) != FA_OK)
    return rc;
  if ((rc = make_bshd_map(&tk, k, batch, seqlen_k, nheads_kv, head_dim, 128, dtype)) != FA_OK)
    return rc;
  if ((rc = make_bshd_map(&tv, v, batch, seqlen_k, nheads_kv, head_dim, 128, dtype)) != FA_OK)
    return rc;
  CUtensorMap tq128, tdo128;
  if (sep) {
    if ((rc = make_bshd_map(&tq128, q, batch, seqlen, nheads, head_dim, 128, dtype)) != FA_OK)
      return rc;
    if ((rc = make_bshd_map(&tdo128, dout, batch, seqlen, nheads, head_dim, 128, dtype)) != FA_OK)
      return rc;
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  BwdArgs a;
  a.tm_q = &tq;
  a.tm_do = &tdo;
  a.tm_k = &tk;
  a.tm_v = &tv;
  a.o = out;
  a.dout = dout;
  a.lse = lse;
  a.dq = dq;
  a.dk = dk;
  a.dv = dv;
  a.dq_acc = sep ? nullptr : reinterpret_cast<float*>(ws + w.dq_acc);
  a.dq_separate = sep ? 1 : 0;
  a.tm_q128 = sep ? &tq128 : nullptr;
  a.tm_do128 = sep ? &tdo128 : nullptr;
  a.delta = sep ? reinterpret_cast<float*>(ws + w.delta) : nullptr;
  a.q_aug = ws + w.q_aug;
  a.do_aug = ws + w.do_aug;
  a.B = batch;
  a.Sq = seqlen;
  a.Sk = seqlen_k;
  a.H = nheads;
  a.D = head_dim;
  a.S_pad = (int)round_up((size_t)seqlen, kSeqPad);
  a.Hkv = nheads_kv;
  a.dtype = dtype;
  a.scale = sm_scale;
  a.causal = causal ? 1 : 0;
  a.status = status;
  a.timeout_ns = g_timeout_ns.load();
  return launch_bwd(a, static_cast<cudaStream_t>(stream), phase);
}

extern "C" {

int fa_sm100_bwd(const void* dout, const void* q, const void* k, const void* v, const void* out,
                 const float* lse, void* dq, void* dk, void* dv, void* workspace,
                 size_t workspace_bytes, int batch, int seqlen, int nheads, int head_dim,
                 float sm_scale, int causal, int* status, void* stream) {
  return bwd_impl(-1, dout, q, k, v, out, lse, dq, dk, dv, workspace, workspace_bytes, batch,
                  seqlen, seqlen, nheads, nheads, head_dim, FA_DTYPE_F16, sm_scale, causal, status,
                  stream, 0);
}

int fa_sm100_bwd_ex(const void* dout, const void* q, const void* k, const void* v,
                    const void* out, const float* lse, void* dq, void* dk, void* dv,
                    void* workspace, size_t workspace_bytes, int batch, int seqlen_q,
                    int seqlen_k, int nheads, int nheads_kv, int head_dim, int dtype,
                    float sm_scale, int causal, int* status, void* stream) {
  return bwd_impl(-1, dout, q, k, v, out, lse, dq, dk, dv, workspace, workspace_bytes, batch,
                  seqlen_q, seqlen_k, nheads, nheads_kv, head_dim, dtype, sm_scale, causal, status,
                  stream, 0);
}

int fa_sm100_bwd_flags(const void* dout, const void* q, const void* k, const void* v,
                       const void* out, const float* lse, void* dq, void* dk, void* dv,
                       void* workspace, size_t workspace_bytes, int batch, int seqlen_q,
                       int seqlen_k, int nheads, int nheads_kv, int head_dim, int dtype,
                       float sm_scale, int causal, int flags, int* status, void* stream) {
  return bwd_impl(-1, dout, q, k, v, out, lse, dq, dk, dv, workspace, workspace_bytes, batch,
                  seqlen_q, seqlen_k, nheads, nheads_kv, head_dim, dtype, sm_scale, causal, status,
                  stream, flags);
}

int fa_sm100_bwd_phase(int phase, const void* dout, const void* q, const void* k, const void* v,
                       const void* out, const float* lse, void* dq, void* dk, void* dv,
                       void* workspace, size_t workspace_bytes, int batch, int seqlen, int nheads,
                       int head_dim, float sm_scale, int causal, int* status, void* stream) {
  if (phase < 0 || phase > 2) return FA_ERR_ARG;
  return bwd_impl(phase, dout, q, k, v, out, lse, dq, dk, dv, workspace, workspace_bytes, batch,
                  seqlen, seqlen, nheads, nheads, head_dim, FA_DTYPE_F16, sm_scale, causal, status,
                  stream, 0);
}

}  // extern "C"
