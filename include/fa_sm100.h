/* C ABI of the B200 (sm_100a) FlashAttention library libfa_sm100.so.
 *
 * Plain pointers and sizes only: every tensor is a caller-owned device buffer,
 * fp16 tensors are contiguous (batch, seqlen, nheads, head_dim) with 16-byte
 * aligned base addresses, LSE is contiguous (batch, nheads, seqlen) fp32.
 * `stream` is a cudaStream_t (NULL = legacy default stream).  `status` is an
 * optional device int the kernels OR error bits into instead of trapping; the
 * host reads it when it wants to.  Bit 0 (1): a bounded on-device wait ran out.
 * Bit 1 (2): a backward row term was beyond the range the kernel represents
 * and was clamped (fp16: |LSE / sm_scale| or |rowsum(O * dO)| above ~1.3e8;
 * bf16: above its largest finite value); the gradients of those rows are wrong.
 * Calls are asynchronous and thread-safe.  All of them except
 * fa_sm100_bwd_noalloc keep no state between calls; that one shares a static
 * device array between calls (see its comment below).
 *
 * Return codes: FA_OK, or one of the FA_ERR_* values below
 * (fa_sm100_error_string() names them).
 */
#ifndef FA_SM100_H
#define FA_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FA_OK 0
#define FA_ERR_ARG 1      /* bad shape, head_dim, null or misaligned pointer */
#define FA_ERR_TMA 2      /* cuTensorMapEncodeTiled refused a tensor map */
#define FA_ERR_LAUNCH 3   /* kernel launch failed */
#define FA_ERR_DEVICE 4   /* current device is not sm_100 / driver entry point missing */
#define FA_ERR_WORKSPACE 5 /* workspace missing or smaller than fa_sm100_bwd_workspace_bytes() */
#define FA_ERR_SCRATCH_LIMIT 6 /* shape needs more than FA_SM100_NOALLOC_SCRATCH_BYTES */

/* Size of the static device scratch array behind fa_sm100_bwd_noalloc. */
#define FA_SM100_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)

#define FA_SM100_ABI_VERSION 3

/* Element types of the _ex entry points (q, k, v, out, dout, dq, dk, dv). */
#define FA_DTYPE_F16 0
#define FA_DTYPE_BF16 1

/* Forward: out = softmax(sm_scale * q k^T [causal mask]) v, and (if lse != NULL)
 * the natural-log log-sum-exp of each query row, +inf for a row with no
 * unmasked key.
 * Replaces flash_attn_volta/triton_fa.py:291-397 (flash_attn_forward with
 * return_softmax_lse, and _run_kernel) — same math, layout and LSE convention. */
int fa_sm100_fwd(const void* q, const void* k, const void* v, void* out, float* lse,
                 int batch, int seqlen, int nheads, int head_dim, float sm_scale, int causal,
                 int* status, void* stream);

/* Bytes of device workspace fa_sm100_bwd needs for this shape (fp32 dQ
 * accumulator and 32 bytes per row each for the -LSE/scale and -delta terms
 * the main kernel adds inside its MMAs, rows padded to 128). */
size_t fa_sm100_bwd_workspace_bytes(int batch, int seqlen, int nheads, int head_dim);

/* Backward: given dout, the forward inputs q, k, v, its output `out` and LSE,
 * writes dq, dk, dv (fp16, same layout as q).  `workspace` is caller-owned
 * device memory of at least fa_sm100_bwd_workspace_bytes() bytes, 256-byte
 * aligned; its contents need not be initialised.
 * Replaces flash_attn_volta/triton_fa_bwd.py:587-700 (flash_attn_backward and
 * _run_bwd_kernels: delta = rowsum(O*dO), then the dQ and dK/dV kernels). */
int fa_sm100_bwd(const void* dout, const void* q, const void* k, const void* v, const void* out,
                 const float* lse, void* dq, void* dk, void* dv, void* workspace,
                 size_t workspace_bytes, int batch, int seqlen, int nheads, int head_dim,
                 float sm_scale, int causal, int* status, void* stream);

/* Extended forward / backward: grouped-query attention, bf16 and Sq != Sk.
 * q, out, dout, dq are (batch, seqlen_q, nheads, head_dim); k, v, dk, dv are
 * (batch, seqlen_k, nheads_kv, head_dim) with nheads % nheads_kv == 0, query
 * head h attending to K/V head h / (nheads / nheads_kv); lse is
 * (batch, nheads, seqlen_q) fp32.  dtype = FA_DTYPE_F16 or FA_DTYPE_BF16 for
 * every (batch, seq, heads, head_dim) tensor.  With seqlen_q != seqlen_k the
 * causal mask is aligned to the bottom-right: query i sees keys
 * j <= i + seqlen_k - seqlen_q (a row that sees no key gets out = 0,
 * lse = +inf).  Otherwise as fa_sm100_fwd / fa_sm100_bwd; the workspace is
 * fa_sm100_bwd_workspace_bytes(batch, seqlen_q, nheads, head_dim); dk, dv hold
 * the sums over each K/V head's query heads.
 * No counterpart in the reference: it is fp16, multi-head and square only
 * (flash_attn_volta/triton_fa.py:313-317) and its HF patches expand K/V with
 * repeat_kv first (flash_attn_volta/patch_hf.py:187-188). */
int fa_sm100_fwd_ex(const void* q, const void* k, const void* v, void* out, float* lse,
                    int batch, int seqlen_q, int seqlen_k, int nheads, int nheads_kv,
                    int head_dim, int dtype, float sm_scale, int causal, int* status,
                    void* stream);
int fa_sm100_bwd_ex(const void* dout, const void* q, const void* k, const void* v,
                    const void* out, const float* lse, void* dq, void* dk, void* dv,
                    void* workspace, size_t workspace_bytes, int batch, int seqlen_q,
                    int seqlen_k, int nheads, int nheads_kv, int head_dim, int dtype,
                    float sm_scale, int causal, int* status, void* stream);

/* Flags of fa_sm100_bwd_flags.
 * FA_BWD_DETERMINISTIC: dQ from its own kernel, one CTA per 128-row query tile
 * summing its key blocks in ascending order inside tensor memory (no atomics),
 * as the reference's dQ kernel does (flash_attn_volta/triton_fa_bwd.py:73-307);
 * the main kernel then computes dK and dV only.  dQ is bit-reproducible from
 * run to run and the workspace holds no fp32 dQ accumulator.  Without the flag
 * dQ partials are added into an fp32 accumulator with L2 reductions whose
 * order varies between runs. */
#define FA_BWD_DETERMINISTIC 1

/* Backward with flags (FA_BWD_*); otherwise as fa_sm100_bwd_ex.  The workspace
 * is fa_sm100_bwd_workspace_bytes_flags() bytes (fa_sm100_bwd_workspace_bytes()
 * is always enough).  Same computation as flash_attn_volta/triton_fa_bwd.py:587-700. */
int fa_sm100_bwd_flags(const void* dout, const void* q, const void* k, const void* v,
                       const void* out, const float* lse, void* dq, void* dk, void* dv,
                       void* workspace, size_t workspace_bytes, int batch, int seqlen_q,
                       int seqlen_k, int nheads, int nheads_kv, int head_dim, int dtype,
                       float sm_scale, int causal, int flags, int* status, void* stream);
size_t fa_sm100_bwd_workspace_bytes_flags(int batch, int seqlen, int nheads, int head_dim,
                                          int flags);

/* The three launches fa_sm100_bwd makes, one at a time, on the same arguments:
 * phase 0 = delta and the -LSE/scale, -delta MMA terms, zeroing of the dQ accumulator,
 * phase 1 = the main backward kernel (dK, dV, dQ partial sums),
 * phase 2 = dQ accumulator -> fp16 dq.  Running 0, 1, 2 in stream order equals
 * one fa_sm100_bwd call.  For callers that schedule or time the phases apart.
 * No counterpart in the reference (its two Triton launches are internal,
 * triton_fa_bwd.py:667-695). */
int fa_sm100_bwd_phase(int phase, const void* dout, const void* q, const void* k, const void* v,
                       const void* out, const float* lse, void* dq, void* dk, void* dv,
                       void* workspace, size_t workspace_bytes, int batch, int seqlen,
                       int nheads, int head_dim, float sm_scale, int causal, int* status,
                       void* stream);

/* Backward that allocates nothing, for callers that cannot allocate device
 * memory when they run it (pre-planned buffer pools, execution phases where
 * allocation is forbidden, fixed memory budgets).  Same arguments and results
 * as fa_sm100_bwd, minus the workspace: the scratch it needs (the same bytes
 * fa_sm100_bwd_workspace_bytes() reports) lives in one static device array of
 * FA_SM100_NOALLOC_SCRATCH_BYTES (32 MiB) per GPU, held from library load
 * until process exit.  Shapes that need more return FA_ERR_SCRATCH_LIMIT
 * (e.g. head_dim 128 fits at most about 58k padded rows batch*nheads*seqlen:
 * 576 bytes per row).
 * The first call on a device looks up the array's device address (with that
 * device current); make it before any stream capture.  The address is cached
 * for the life of the process: a device or primary-context reset
 * (cudaDeviceReset) after that first call is not supported.  All calls share the
 * array, so calls that overlap on the GPU race; inputs and outputs are still
 * caller-owned.  It calls no cudaMalloc / cudaFree.
 * No counterpart in the reference. */
int fa_sm100_bwd_noalloc(const void* dout, const void* q, const void* k, const void* v,
                         const void* out, const float* lse, void* dq, void* dk, void* dv,
                         int batch, int seqlen, int nheads, int head_dim, float sm_scale,
                         int causal, int* status, void* stream);

/* Merge of a partial attention result into a running one (ring context
 * parallelism: the attention of a query chunk over one more key chunk):
 *   lse_acc' = log(exp(lse_acc) + exp(lse)),
 *   acc_o'   = acc_o * exp(lse_acc - lse_acc') + o * exp(lse - lse_acc').
 * acc_o fp32 and o (dtype) are (batch, seqlen, nheads, head_dim), 16-byte
 * aligned; lse_acc, lse are (batch, nheads, seqlen) fp32.  An lse of +inf (a
 * row with no visible key) adds nothing.  first != 0: acc_o = o, lse_acc = lse.
 * No counterpart in the reference (it has no multi-GPU path). */
int fa_sm100_merge(float* acc_o, float* acc_lse, const void* o, const float* lse, int batch,
                   int seqlen, int nheads, int head_dim, int dtype, int first, void* stream);

/* Upper bound, in nanoseconds, of every on-device wait of later launches
 * (default 4e9).  Process-wide. */
void fa_sm100_set_wait_timeout_ns(uint64_t ns);

/* Test hooks, process-wide, 0 in normal use.  Bit 0: the forward kernel skips
 * loading its first V tile, so an on-device wait runs out (after the wait
 * timeout), the kernel ORs 1 into the status word and returns; used to test
 * the timeout path without faulting the GPU.  No counterpart in the reference. */
void fa_sm100_set_debug_flags(int flags);

const char* fa_sm100_error_string(int code);
int fa_sm100_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FA_SM100_H */
