// Merge of a partial attention result into a running one, for ring context
// parallelism (flash_attn_volta_b200/ring.py): each ring step yields, for a
// query chunk, the attention over one key chunk, (O_j, LSE_j); the chunk's
// result over all keys seen so far is
//     LSE = log(exp(LSE_acc) + exp(LSE_j))
//     O   = O_acc * exp(LSE_acc - LSE) + O_j * exp(LSE_j - LSE)
// (the reference has no multi-GPU path).  One pass over the tensors instead of
// a chain of element-wise torch operations.  O_acc is fp32 (B, S, H, D), O_j
// the kernel's fp16 / bf16 output in the same layout, the LSEs (B, H, S) fp32.
// An LSE of +inf (a row that saw no key, the forward's convention) adds
// nothing.  With `first`, O_acc and LSE_acc are simply set from the block.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "fa_kernels.h"
#include "sm100_ptx.cuh"

namespace fa_sm100 {
namespace {

// D/8 threads per (b, s, h) row, 8 consecutive elements each (16-byte loads of O_j)
template <typename T>
__global__ void __launch_bounds__(256) fa_merge_kernel(float* __restrict__ acc_o,
                                                       float* __restrict__ acc_lse,
                                                       const T* __restrict__ o,
                                                       const float* __restrict__ lse, int S, int H,
                                                       int D, long long rows, int first) {
  const int tpr = D / 8;
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long row0 = t / tpr;  // (b * S + s) * H + h
  const int sub = (int)(t % tpr);
  const bool valid = row0 < rows;  // no early return: the row's lanes meet at __syncwarp
  const long long row = valid ? row0 : rows - 1;
  const int h = (int)(row % H);
  const long long bs = row / H;
  const int s = (int)(bs % S);
  const long long b = bs / S;
  const long long li = (b * H + h) * S + s;
  const float INF = __int_as_float(0x7f800000);
  float lb = lse[li];
  if (lb == INF) lb = -INF;  // a fully masked row of the block contributes nothing
  const float la = first ? -INF : acc_lse[li];
  const float m = fmaxf(la, lb);
  float wa = 0.f, wb = 0.f, lnew = -INF;
  if (m != -INF) {
    const float ea = expf(la - m), eb = expf(lb - m);
    const float sum = ea + eb;
    lnew = m + logf(sum);
    wa = ea / sum;
    wb = eb / sum;
  }
  const uint4 ov = *reinterpret_cast<const uint4*>(o + row * D + sub * 8);
  const uint32_t w[4] = {ov.x, ov.y, ov.z, ov.w};
  float4* acc = reinterpret_cast<float4*>(acc_o + row * D + sub * 8);
  float4 a0 = first ? make_float4(0.f, 0.f, 0.f, 0.f) : acc[0];
  float4 a1 = first ? make_float4(0.f, 0.f, 0.f, 0.f) : acc[1];
  const float2 p0 = Elem<T>::unpack2(w[0]), p1 = Elem<T>::unpack2(w[1]);
  const float2 p2 = Elem<T>::unpack2(w[2]), p3 = Elem<T>::unpack2(w[3]);
  a0 = make_float4(a0.x * wa + p0.x * wb, a0.y * wa + p0.y * wb, a0.z * wa + p1.x * wb,
                   a0.w * wa + p1.y * wb);
  a1 = make_float4(a1.x * wa + p2.x * wb, a1.y * wa + p2.y * wb, a1.z * wa + p3.x * wb,
                   a1.w * wa + p3.y * wb);
  if (valid) {
    acc[0] = a0;
    acc[1] = a1;
  }
  // every thread of the row has read LSE_acc (one warp holds the row's threads)
  __syncwarp();
  if (valid && sub == 0) acc_lse[li] = lnew;
}

}  // namespace
}  // namespace fa_sm100

extern "C" int fa_sm100_merge(float* acc_o, float* acc_lse, const void* o, const float* lse,
                              int batch, int seqlen, int nheads, int head_dim, int dtype,
                              int first, void* stream) {
  using namespace fa_sm100;
  if (batch <= 0 || seqlen <= 0 || nheads <= 0) return FA_ERR_ARG;
  if (head_dim != 16 && head_dim != 32 && head_dim != 64 && head_dim != 128) return FA_ERR_ARG;
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return FA_ERR_ARG;
  if (!acc_o || !acc_lse || !o || !lse) return FA_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(acc_o) | reinterpret_cast<uintptr_t>(o)) & 15u) return FA_ERR_ARG;
  const long long rows = (long long)batch * seqlen * nheads;
  const long long threads = rows * (head_dim / 8);
  const unsigned grid = (unsigned)((threads + 255) / 256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == FA_DTYPE_BF16)
    fa_merge_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        acc_o, acc_lse, static_cast<const __nv_bfloat16*>(o), lse, seqlen, nheads, head_dim, rows,
        first);
  else
    fa_merge_kernel<__half><<<grid, 256, 0, st>>>(acc_o, acc_lse, static_cast<const __half*>(o),
                                                  lse, seqlen, nheads, head_dim, rows, first);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}
