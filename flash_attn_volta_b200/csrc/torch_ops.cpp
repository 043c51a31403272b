// PyTorch operators over the C ABI of libfa_sm100.so (include/fa_sm100.h).
//
//   torch.ops.fav.fwd(q, k, v, causal, sm_scale) -> (out, lse)
//   torch.ops.fav.bwd(dout, q, k, v, out, lse, causal, sm_scale, deterministic=False)
//       -> (dq, dk, dv)
//   torch.ops.fav.status(device) -> the device's int32 status word
//   torch.ops.fav.merge_(acc_o, acc_lse, o, lse, first)  (ring: in-place LSE merge)
//
// These are the only callers of the C core on the Python side
// (flash_attn_volta_b200/forward.py, backward.py, autograd.py): the
// reference's flash_attn_forward / flash_attn_backward
// (flash_attn_volta/triton_fa.py:291-397, triton_fa_bwd.py:587-700) become a
// few Python assertions plus one dispatcher call each.  Registered for the
// CUDA key only; shape functions for FakeTensor / meta tensors (torch.compile)
// and the autograd formula are registered from Python (ops.py).
//
// The operators take (B, S, H, D) fp16 / bf16 CUDA tensors (any strides: other
// layouts and misaligned views are copied), k / v with H_kv heads
// (H % H_kv == 0) and S_k rows, lse (B, H, S_q) fp32, and return contiguous
// tensors.  The Python wrappers check the reference's preconditions first;
// errors of the C ABI raise RuntimeError with the library's message.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <mutex>
#include <tuple>

#include "../../include/fa_sm100.h"

namespace {

int dtype_code(const at::Tensor& t) {
  TORCH_CHECK(t.scalar_type() == at::kHalf || t.scalar_type() == at::kBFloat16,
              "flash_attn_volta_b200: fp16 or bf16 tensors only, got ", t.scalar_type());
  return t.scalar_type() == at::kHalf ? FA_DTYPE_F16 : FA_DTYPE_BF16;
}

void check_rc(int rc, const char* what) {
  TORCH_CHECK(rc == FA_OK, what, " failed: ", fa_sm100_error_string(rc), " (code ", rc, ")");
}

// Contiguous (B, S, H, D) with a 16-byte aligned base (what the TMA tensor
// maps need): a view of another layout is copied, and so is a contiguous view
// whose storage offset breaks the alignment.
at::Tensor kernel_input(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.dim() == 4, name, " must be (batch, seqlen, heads, head_dim)");
  at::Tensor c = t.contiguous();
  if (reinterpret_cast<uintptr_t>(c.data_ptr()) % 16 != 0) c = c.clone();
  return c;
}

// The C ABI takes every extent from q and k, so each other tensor must have
// exactly the shape it implies, and every tensor must sit on q's device (a
// mismatch would otherwise become an out-of-bounds or peer read on the GPU).
void check_like(const at::Tensor& t, at::IntArrayRef sizes, const at::Tensor& q, const char* name) {
  TORCH_CHECK(t.sizes() == sizes, name, " has shape ", t.sizes(), ", expected ", sizes);
  TORCH_CHECK(t.device() == q.device(), name, " is on ", t.device(), ", q on ", q.device());
}

void check_qkv(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v) {
  TORCH_CHECK(k.scalar_type() == q.scalar_type() && v.scalar_type() == q.scalar_type(),
              "q, k, v must have the same dtype");
  check_like(k, {q.size(0), k.size(1), k.size(2), q.size(3)}, q, "k");
  check_like(v, k.sizes(), q, "v");
  TORCH_CHECK(k.size(2) > 0 && q.size(2) % k.size(2) == 0,
              "the query heads must be a multiple of the key/value heads");
}

// One int32 status word per device, created on first use (make that first
// call before any CUDA graph capture).
constexpr int kMaxDev = 64;
std::mutex g_status_mu;
at::Tensor g_status[kMaxDev];

at::Tensor status_word(int64_t device) {
  TORCH_CHECK(device >= 0 && device < kMaxDev, "device index out of range");
  std::lock_guard<std::mutex> lock(g_status_mu);
  if (!g_status[device].defined()) {
    c10::cuda::CUDAGuard guard((c10::DeviceIndex)device);
    g_status[device] =
        at::zeros({1}, at::TensorOptions().dtype(at::kInt).device(at::kCUDA, device));
  }
  return g_status[device];
}

std::tuple<at::Tensor, at::Tensor> fwd_cuda(const at::Tensor& q_in, const at::Tensor& k_in,
                                            const at::Tensor& v_in, bool causal, double sm_scale) {
  const at::Tensor q = kernel_input(q_in, "q");
  const at::Tensor k = kernel_input(k_in, "k");
  const at::Tensor v = kernel_input(v_in, "v");
  const int dt = dtype_code(q);
  check_qkv(q, k, v);
  const int64_t B = q.size(0), Sq = q.size(1), H = q.size(2), D = q.size(3);
  const int64_t Sk = k.size(1), Hkv = k.size(2);
  c10::cuda::CUDAGuard guard(q.device());
  at::Tensor out = at::empty(q.sizes(), q.options());
  at::Tensor lse = at::empty({B, H, Sq}, q.options().dtype(at::kFloat));
  if (q.numel() == 0) return {out, lse};
  if (Sk == 0) {
    // no keys: every query row is fully masked (O = 0, LSE = +inf)
    out.zero_();
    lse.fill_(std::numeric_limits<float>::infinity());
    return {out, lse};
  }
  at::Tensor st = status_word(q.get_device());
  const int rc = fa_sm100_fwd_ex(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
                                 lse.data_ptr<float>(), (int)B, (int)Sq, (int)Sk, (int)H,
                                 (int)Hkv, (int)D, dt, (float)sm_scale, causal ? 1 : 0,
                                 st.data_ptr<int>(), at::cuda::getCurrentCUDAStream().stream());
  check_rc(rc, "fa_sm100_fwd_ex");
  return {out, lse};
}

std::tuple<at::Tensor, at::Tensor, at::Tensor> bwd_cuda(
    const at::Tensor& dout_in, const at::Tensor& q_in, const at::Tensor& k_in,
    const at::Tensor& v_in, const at::Tensor& out_in, const at::Tensor& lse_in, bool causal,
    double sm_scale, bool deterministic) {
  const at::Tensor dout = kernel_input(dout_in, "dout");
  const at::Tensor q = kernel_input(q_in, "q");
  const at::Tensor k = kernel_input(k_in, "k");
  const at::Tensor v = kernel_input(v_in, "v");
  const at::Tensor out = kernel_input(out_in, "out");
  const int dt = dtype_code(q);
  check_qkv(q, k, v);
  TORCH_CHECK(dout.scalar_type() == q.scalar_type() && out.scalar_type() == q.scalar_type(),
              "dout and out must have q's dtype");
  TORCH_CHECK(lse_in.scalar_type() == at::kFloat, "lse must be fp32");
  const at::Tensor lse = lse_in.contiguous();
  const int64_t B = q.size(0), Sq = q.size(1), H = q.size(2), D = q.size(3);
  const int64_t Sk = k.size(1), Hkv = k.size(2);
  check_like(dout, q.sizes(), q, "dout");
  check_like(out, q.sizes(), q, "out");
  check_like(lse, {B, H, Sq}, q, "lse");
  c10::cuda::CUDAGuard guard(q.device());
  at::Tensor dq = at::empty(q.sizes(), q.options());
  at::Tensor dk = at::empty(k.sizes(), k.options());
  at::Tensor dv = at::empty(v.sizes(), v.options());
  if (q.numel() == 0 || Sk == 0) {
    dq.zero_();
    dk.zero_();
    dv.zero_();
    return {dq, dk, dv};
  }
  const int flags = deterministic ? FA_BWD_DETERMINISTIC : 0;
  const size_t nbytes = fa_sm100_bwd_workspace_bytes_flags((int)B, (int)Sq, (int)H, (int)D, flags);
  TORCH_CHECK(nbytes > 0, "fa_sm100_bwd_workspace_bytes: unsupported shape");
  at::Tensor ws = at::empty({(int64_t)nbytes}, q.options().dtype(at::kByte));
  at::Tensor st = status_word(q.get_device());
  const int rc = fa_sm100_bwd_flags(
      dout.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
      lse.data_ptr<float>(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), ws.data_ptr(), nbytes,
      (int)B, (int)Sq, (int)Sk, (int)H, (int)Hkv, (int)D, dt, (float)sm_scale, causal ? 1 : 0,
      flags, st.data_ptr<int>(), at::cuda::getCurrentCUDAStream().stream());
  check_rc(rc, "fa_sm100_bwd_flags");
  return {dq, dk, dv};
}

void merge_cuda(at::Tensor& acc_o, at::Tensor& acc_lse, const at::Tensor& o_in,
                const at::Tensor& lse_in, bool first) {
  TORCH_CHECK(acc_o.scalar_type() == at::kFloat && acc_o.is_contiguous(),
              "acc_o must be contiguous fp32");
  TORCH_CHECK(acc_lse.scalar_type() == at::kFloat && acc_lse.is_contiguous(),
              "acc_lse must be contiguous fp32");
  const at::Tensor o = kernel_input(o_in, "o");
  const at::Tensor lse = lse_in.contiguous();
  check_like(acc_o, o.sizes(), o, "acc_o");
  TORCH_CHECK(lse.scalar_type() == at::kFloat, "lse must be fp32");
  check_like(lse, {o.size(0), o.size(2), o.size(1)}, o, "lse");
  check_like(acc_lse, lse.sizes(), o, "acc_lse");
  c10::cuda::CUDAGuard guard(o.device());
  const int rc = fa_sm100_merge(acc_o.data_ptr<float>(), acc_lse.data_ptr<float>(), o.data_ptr(),
                                lse.data_ptr<float>(), (int)o.size(0), (int)o.size(1),
                                (int)o.size(2), (int)o.size(3), dtype_code(o), first ? 1 : 0,
                                at::cuda::getCurrentCUDAStream().stream());
  check_rc(rc, "fa_sm100_merge");
}

}  // namespace

TORCH_LIBRARY(fav, m) {
  m.def("fwd(Tensor q, Tensor k, Tensor v, bool causal, float sm_scale) -> (Tensor, Tensor)");
  m.def(
      "bwd(Tensor dout, Tensor q, Tensor k, Tensor v, Tensor out, Tensor lse, bool causal, "
      "float sm_scale, bool deterministic=False) -> (Tensor, Tensor, Tensor)");
  m.def("status(int device) -> Tensor", &status_word);
  m.def("merge_(Tensor(a!) acc_o, Tensor(b!) acc_lse, Tensor o, Tensor lse, bool first) -> ()");
}

TORCH_LIBRARY_IMPL(fav, CUDA, m) {
  m.impl("fwd", &fwd_cuda);
  m.impl("bwd", &bwd_cuda);
  m.impl("merge_", &merge_cuda);
}
