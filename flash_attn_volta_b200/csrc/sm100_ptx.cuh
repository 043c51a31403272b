// Thin inline-PTX wrappers for the sm_100a features the attention kernels use:
// mbarriers with bounded waits, TMA tile loads / bulk copies, tcgen05 tensor
// memory (alloc, ld, st), tcgen05.mma (kind::f16, fp32 accumulate) and the
// shared-memory / instruction descriptors it consumes.
//
// Descriptor encodings follow the PTX ISA "tcgen05 matrix descriptors" and
// "instruction descriptor" tables:
//   smem descriptor : [0,14) start>>4, [16,30) LBO>>4, [32,46) SBO>>4,
//                     [46,48) version=1, [49,52) base offset, [61,64) swizzle
//   instr descriptor: [4,6) D fmt (1=f32), [7,10) A fmt (0=f16), [10,13) B fmt,
//                     15 A MN-major, 16 B MN-major, [17,23) N>>3, [24,29) M>>4
// Canonical layouts (16-bit elements, swizzle width W bytes = 32/64/128, a
// "row" is W bytes, atoms are 8 rows = 8*W bytes and must be 8*W aligned):
//   K-major : rows = M (or N) index, K contiguous inside a row.  SBO = stride
//             between 8-row groups (8*W when dense).  Moving along K inside the
//             atom is a plain byte offset on the start address.
//   MN-major: rows = K index, M/N contiguous inside a row.  SBO = stride between
//             8-row K groups (8*W), LBO = stride between W-wide M/N blocks.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace fa_sm100 {

// ---------------------------------------------------------------- status word
// Error bits a kernel ORs into the caller's status word instead of trapping.
enum : int {
  kStatusOk = 0,
  kStatusTimeout = 1,   // a bounded mbarrier wait ran out
  kStatusRange = 2,     // a backward row term (LSE / scale or delta) beyond the representable range
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait context shared by all warps of a CTA: once any wait runs out,
// `abort` (shared memory) is raised, the status word gets kStatusTimeout and
// every later wait in the CTA returns false at once.
struct WaitCtx {
  volatile int* abort;   // shared-memory flag
  int* status;           // global status word (may be null)
  uint64_t limit_ns;
};

static __device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, const WaitCtx& w) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 63u) {
      if (*w.abort) return false;
      if (globaltimer_ns() - t0 > w.limit_ns) {
        *w.abort = 1;
        if (w.status) atomicOr(w.status, kStatusTimeout);
        __threadfence();
        return false;
      }
    }
  }
}

// Bounded wait used while tearing down after an abort: ignores the abort flag
// (the point is to let this CTA's own in-flight copies / MMAs finish).
static __device__ __noinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity,
                                                    uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 63u && globaltimer_ns() - t0 > limit_ns) return false;
  }
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const WaitCtx& w) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, w);
}

// ---------------------------------------------------------------- dependent launch
// Programmatic dependent launch.  A grid launched with programmatic stream
// serialization may start while the previous grid in the stream runs;
// griddep_wait() returns once that grid has completed and its memory is visible
// (at once for a normal launch).  griddep_launch_dependents() lets the next such
// grid start; every kernel here calls it only after its own griddep_wait(), so
// when a grid starts early, everything before its predecessor has completed.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 4-D tiled load (coordinates innermost first) into shared memory, completing
// `bytes` of transaction count on `bar`.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* m, uint32_t bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// Untiled bulk copy global -> shared (16-byte aligned addresses, size % 16 == 0).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}

// Element-wise fp32 add of `bytes` of shared memory into global memory, done
// in L2 (untiled bulk reduction; 16-byte aligned addresses, size % 16 == 0).
__device__ __forceinline__ void bulk_reduce_add_f32(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile(
      "cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(
          reinterpret_cast<uint64_t>(dst)),
      "r"(src), "r"(bytes)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most N committed bulk groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until every committed bulk group has completed.
__device__ __forceinline__ void bulk_wait_group_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Fire-and-forget fp32 add to global memory (no value returned).
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void st_shared_f32(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy
// (tensor core operand reads, TMA stores).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread completes.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]; A is M lanes x K with two 16-bit elements per
// 32-bit column (element 2c in the low half of column c), K-major.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// lane (taddr.lane + t), columns [taddr.col, taddr.col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}


// ---------------------------------------------------------------- descriptors
// Swizzle-mode field of the smem descriptor for a swizzle width in bytes.
__host__ __device__ constexpr uint32_t swizzle_field(int width_bytes) {
  return width_bytes == 128 ? 2u : width_bytes == 64 ? 4u : width_bytes == 32 ? 6u : 0u;
}

__device__ __forceinline__ uint64_t make_smem_desc(uint32_t saddr, uint32_t lbo_bytes,
                                                   uint32_t sbo_bytes, uint32_t swz_field) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)swz_field << 61;
  return d;
}

// f16 x f16 -> f32 instruction descriptor, M x N tile.
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N, bool a_mn_major,
                                                      bool b_mn_major) {
  return (1u << 4)                                   // D = f32
         | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------- scheduling
// Maps a 1-D block index to (batch*head, tile rank) so that heads go in groups
// of `group` and, inside a group, all heads' rank-0 tiles launch first, then
// rank 1, ...  Blocks launch in index order, so with rank 0 = the longest tile
// this is longest-first within each group, while the blocks resident at once
// touch only one or two groups' K/V (or Q/dO) and share them in L2.
__device__ __forceinline__ void grid_to_tile(int L, int nbh, int ntile, int group, int& bh,
                                             int& rank) {
  const int per_group = group * ntile;
  const int g = L / per_group;
  const int rem = L - g * per_group;
  const int gsize = min(group, nbh - g * group);
  rank = rem / gsize;
  bh = g * group + (rem - rank * gsize);
}
constexpr int kHeadGroup = 8;

// ---------------------------------------------------------------- math
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// ---- packed fp32 pairs (Blackwell f32x2 ALU ops)
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair, on the FMA pipe instead of the MUFU unit.  Cody-Waite style
// range reduction: n = round(x) by adding 1.5*2^23 (the integer lands in the low
// mantissa bits), f = x - n in [-0.5, 0.5]; 2^f by a cubic
// 1 + c1 f + c2 f^2 + c3 f^3 fitted here to 2^f on [-0.5, 0.5] (relative
// least squares with iterative reweighting towards minimax); 2^n applied by
// adding n to the exponent field.  Inputs are clamped to >= -125 (result
// >= ~2^-125.5, i.e. zero after fp16 rounding).  Max relative error 1.0e-4 over
// [-125, 8], checked in float32 arithmetic.
__device__ __forceinline__ uint64_t f2_exp2_poly(uint64_t x2) {
  float x0, x1;
  f2_unpack(x2, x0, x1);
  const uint64_t x = f2_pack(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
  const uint64_t magic = f2_pack(12582912.0f, 12582912.0f);
  const uint64_t nmagic = f2_pack(-12582912.0f, -12582912.0f);
  const uint64_t t = f2_add(x, magic);
  const uint64_t r = f2_add(t, nmagic);
  const uint64_t f = f2_fma(r, f2_pack(-1.f, -1.f), x);
  uint64_t p = f2_fma(f2_pack(0.05500892549753189f, 0.05500892549753189f), f,
                      f2_pack(0.24221095442771912f, 0.24221095442771912f));
  p = f2_fma(p, f, f2_pack(0.6932829022407532f, 0.6932829022407532f));
  p = f2_fma(p, f, f2_pack(1.f, 1.f));
  float t0, t1, p0, p1;
  f2_unpack(t, t0, t1);
  f2_unpack(p, p0, p1);
  const float e0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  const float e1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
  return f2_pack(e0, e1);
}

// Element type of the attention tensors (fp16 or bf16): the MMA operand
// format bits, packing of fp32 pairs (low half = first argument), unpacking,
// and the bit pattern of 1.0.
template <typename T>
struct Elem;
template <>
struct Elem<__half> {
  static constexpr uint32_t kIdescAB = 0;  // A and B format F16 (kind::f16)
  static constexpr uint32_t kOne = 0x3C00u;
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    return r;
  }
  static __device__ __forceinline__ float2 unpack2(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
  }
  static __device__ __forceinline__ uint16_t bits(float x) {
    return __half_as_ushort(__float2half_rn(x));
  }
  static __device__ __forceinline__ float value(uint16_t b) {
    return __half2float(__ushort_as_half(b));
  }
  static constexpr float kMax = 65504.f;
};
template <>
struct Elem<__nv_bfloat16> {
  static constexpr uint32_t kIdescAB = (1u << 7) | (1u << 10);  // A and B format BF16
  static constexpr uint32_t kOne = 0x3F80u;
  static __device__ __forceinline__ uint32_t pack2(float a, float b) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
    return r;
  }
  static __device__ __forceinline__ float2 unpack2(uint32_t w) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
  }
  static __device__ __forceinline__ uint16_t bits(float x) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
  }
  static __device__ __forceinline__ float value(uint16_t b) {
    return __bfloat162float(__ushort_as_bfloat16(b));
  }
  static constexpr float kMax = 3.0e38f;
};

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// Byte offset of the 16-byte chunk `chunk` of row `row` inside a 128B-swizzled
// K-major block whose rows are 128 bytes (Swizzle<3,4,3>: chunk ^= row % 8).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

}  // namespace fa_sm100
