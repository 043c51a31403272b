// FlashAttention backward for sm_100a (B200).
//
// Replaces the reference's backward (flash_attn_volta/triton_fa_bwd.py):
//   delta = rowsum(O * dO)                              (:650, torch op there)
//   P  = exp(S - LSE),  S = scale * Q K^T               (:123-165, :355-411)
//   dV = P^T dO,  dP = dO V^T,  dS = P (dP - delta)      (:169-172, :415-422)
//   dK = scale * dS^T Q,  dQ = scale * dS K             (:176-178, :426-429)
// The reference runs two kernels (dQ parallel over query blocks, dK/dV parallel
// over key blocks) with 7 GEMMs; here one kernel per key block computes all
// five GEMMs and accumulates dQ into an fp32 workspace with L2 reductions.
//
// The row terms LSE and delta ride in the MMAs: Q and dO get one extra K step
// of 16 columns holding -LSE/scale (resp. -delta) as an fp16 hi/lo pair, K and
// V the matching step [1, 1, 0, ...], so the tensor core delivers
// S'^T = S^T - LSE/scale and dP'^T = dP^T - delta and the softmax warps read no
// per-column values from shared memory (a value broadcast to all lanes costs
// four shared-memory wavefronts per 128-bit load, which competes with the
// tensor core's operand reads).  The hi/lo pair keeps the term exact to ~1e-5.
//
// Kernels:
//   fa_bwd_pre   delta = rowsum(O * dO), the extra K-step rows of Q and dO in the
//                MMA's no-swizzle K-major layout, zero the dQ accumulator.
//   fa_bwd_main  a CTA walks a list of 128-row key/value tiles of the (batch,
//                K/V head) pairs (persistent, one CTA per SM, for at most 16
//                tiles per SM, 8 for causal sequences longer than 4096; else
//                one CTA per tile); each tile loops over
//                query tiles of BM rows (64 for D=128, else 128).  On the
//                persistent grid the next tile's K/V load, Q/dO loads and first
//                S^T / dP^T MMAs overlap this tile's last iterations and its
//                dK/dV epilogue.
//     warps 0-7  "softmax": warp w owns key rows 32*(w%4).. (its TMEM lane
//                quarter) and half of the query columns.  Loads S^T and dP^T
//                from tensor memory into registers and releases them at once
//                (so the next tile's S^T / dP^T MMAs run while it computes),
//                P^T = exp2(S'^T * scale * log2e), dS^T = P^T dP'^T;
//                P^T (fp16) goes to tensor memory as the A operand of dV += P^T dO,
//                dS^T to shared memory (for dQ) and, for D=128, to tensor memory
//                too (A operand of dK += dS^T Q); final dK/dV epilogue.
//     warps 8-11 dQ epilogue: read this tile's dQ partial from tensor memory,
//                stage it in shared memory and add it into the fp32 accumulator
//                with one bulk reduction (cp.reduce.async.bulk .add.f32).
//     warp 12    TMA producers: lane 0 K and V of each key tile (once the last
//                MMAs reading the previous tile's have completed); lane 1 Q,
//                dO and their extra K-step rows per query tile (a 3-stage ring
//                that runs across key tiles).
//     warps 13-16 MMA issuers, one per independent chain: S^T = K Q^T,
//                dP^T = V dO^T (issued as soon as the previous tile's values are
//                in registers), dV += P^T dO with dK += dS^T Q, and the dQ
//                partial = dS K (stored transposed for D=128).
//   fa_bwd_post  dQ = fp16(scale * accumulator) in (B, S, H, D).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <type_traits>

#include "fa_kernels.h"
#include "sm100_ptx.cuh"

namespace fa_sm100 {

#ifdef FA_BWD_TRACE
// Debug build only: clock64() stamps of barrier events of CTA (0, 0), read
// back with fa_debug_trace().
__device__ unsigned long long g_trace[64][16];
#define TRACE(slot, it)                                                              \
  do {                                                                               \
    if (blockIdx.x == 0 && (it) < 64) g_trace[it][slot] = clock64(); \
  } while (0)
// per-CTA timeline: SM id, globaltimer at entry, at the first S issue, at exit
__device__ unsigned long long g_bcta[8192][4];
#define CTRACE(slot)                                                                 \
  do {                                                                               \
    if (blockIdx.x < 8192) g_bcta[blockIdx.x][slot] = globaltimer_ns();             \
  } while (0)
#else
#define TRACE(slot, it) \
  do {                  \
  } while (0)
#define CTRACE(slot) \
  do {               \
  } while (0)
#endif

// Q / dO ring depth without the fused dQ path (its staging buffers free the
// shared memory for a fourth stage)
#ifndef FA_BWD_NST_NODQ
#define FA_BWD_NST_NODQ 4
#endif

template <int D, bool DQ = true>
struct BwdCfg {
  static constexpr int BN = 128;                    // key rows per CTA
  static constexpr int BM = (D == 128) ? 64 : 128;  // query rows per iteration
  static constexpr bool DQT = (D == 128);           // dQ accumulated transposed (M = D)
  static constexpr int SWB = (D * 2 >= 128) ? 128 : D * 2;
  static constexpr int AE = SWB / 2;
  static constexpr int NAT = D / AE;
  // Q / dO (+ their extra K-step rows) ring depth.  A stage is held until dV / dK
  // of its query tile (after the softmax) have read it, so the load of tile
  // i + NST waits for them; more stages hide that latency where shared memory
  // allows.
  static constexpr int NST = (DQ || D != 128) ? 3 : FA_BWD_NST_NODQ;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int PT_BYTES = BN * BM * 2;  // [key row][query col], 64-col atoms
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + KV_BYTES;
  static constexpr int OFF_Q = OFF_V + KV_BYTES;
  static constexpr int OFF_DO = OFF_Q + NST * Q_BYTES;
  // extra K step (16 columns, no-swizzle K-major: 8-row core matrices of 16 B,
  // the two 8-column halves 128 B apart, row groups 256 B apart): the [1, 1, 0,
  // ...] rows shared by K and V, and per stage the rows of Q and of dO
  static constexpr int AUG_BYTES = BM * kAugRowBytes;
  static constexpr int OFF_ONE = OFF_DO + NST * Q_BYTES;
  static constexpr int OFF_QA = OFF_ONE + BN * kAugRowBytes;
  static constexpr int OFF_DA = OFF_QA + NST * AUG_BYTES;
  static constexpr int OFF_BAR = OFF_DA + NST * AUG_BYTES;  // barriers, TMEM slot, abort flag
  static constexpr int OFF_P = ((OFF_BAR + 256) + 1023) / 1024 * 1024;
  static constexpr int OFF_DS = OFF_P;  // P^T lives in tensor memory, not here
  static constexpr int DQ_STAGE_BYTES = BM * D * 4;  // one dQ partial, [q][d] fp32
  static constexpr int NDQ = (D <= 32) ? 2 : 1;        // dQ staging buffers
  // dS^T in shared memory: read by the dQ MMA, and by the dK MMA below D=128
  static constexpr bool DS_SMEM = DQ || D != 128;
  static constexpr int OFF_DQS = OFF_DS + (DS_SMEM ? PT_BYTES : 0);
  static constexpr int SMEM = OFF_DQS + (DQ ? NDQ * DQ_STAGE_BYTES : 0) + 1024;  // + slack
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(NST <= 5, "barrier slots of the Q / dO ring");
  static constexpr int THREADS = 544;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t COL_S = 0, COL_DP = BM, COL_DQ = 2 * BM;
  static constexpr uint32_t COL_DV = DQT ? 256 : 384;
  static constexpr uint32_t COL_DK = COL_DV + (DQT ? 128 : 64);
  // P^T (fp16 pairs, BM/2 columns) in tensor memory: A operand of dV += P^T dO.
  static constexpr uint32_t COL_PT = DQT ? 192 : 320;
  // D=128 also keeps dS^T there (A operand of dK += dS^T Q); it goes to shared
  // memory as well, where dQ reads it.
  static constexpr bool DS_TMEM = DQT;
  static constexpr uint32_t COL_DST = 224;
};

enum BwdBar {
  C_KVFULL = 0,
  C_QFULL = 1,   // +NST (<= 5)
  C_QEMPTY = 6,  // +NST
  C_SFULL = 11,
  C_DPFULL = 12,
  C_SFREE = 13,     // 8 arrivals (softmax warps hold S^T / dP^T in registers)
  C_DSREADY = 14,  // 8 arrivals (P^T / dS^T written to shared memory)
  C_PFREE = 15,
  C_DQFULL = 16,
  C_DQFREE = 17,  // 4 arrivals
  C_KVDONE = 18,
  C_DRAIN = 19,   // 4 arrivals: each MMA issuer's last commit
  C_KVEMPTY = 20,  // 3 arrivals: a tile's last S^T, dP^T and dQ MMAs have read K / V
  C_DKVFREE = 21,  // 8 arrivals: the epilogue has read dK / dV
  C_COUNT = 22
};

// -------------------------------------------------------------------------- pre
// Byte offset of element k of `row` in the extra K-step tile of a row block
// (no-swizzle K-major: row group of 8 at 256 B, the two 8-column halves 128 B
// apart, rows 16 B apart inside a core matrix).
__host__ __device__ constexpr uint32_t aug_offset(uint32_t row, uint32_t k) {
  return (row / 8) * 256 + (k / 8) * 128 + (row % 8) * 16 + (k % 8) * 2;
}

// x as four terms of the element type, [t0, t1, t2, a] with
// t0 + t1 + t2 + kAugBig * a == x (the K / V side of the extra K step holds
// [1, 1, 1, kAugBig]), exact to ~2^-22 |x| for fp16 and ~2^-24 |x| for bf16.
// `a` is used only when |x| exceeds the fp16 range of t0 (a delta of a
// loss-scaled dO, very large logits): a = fp16(x / kAugBig) and the three terms
// split the remainder, |x - kAugBig * a| <= 2^15, so fp16 covers |x| up to
// kAugBig * 65504 ~ 1.3e8 exactly.  bf16 has the range for t0 itself and
// keeps a = 0.  A non-finite x (the +inf LSE of a fully masked row) becomes a
// large negative sum that drives every P of the row to zero.  A finite x
// beyond the range is clamped and reported with kStatusRange.  Returned as the
// first 16-byte half of an extra-K-step row, [t0, t1, t2, a, 0, 0, 0, 0].
template <typename T>
__device__ __forceinline__ uint4 split_row(float x, int* status) {
  uint16_t ba = 0;
  if (std::is_same<T, __half>::value) {
    constexpr float kLim = (float)kAugBig * 65504.f;
    if (!(fabsf(x) <= kLim)) {
      if (status && fabsf(x) != __int_as_float(0x7f800000) && x == x) atomicOr(status, kStatusRange);
      x = (x > 0.f) ? kLim : -kLim;
    }
    if (fabsf(x) > 60000.f) {
      ba = Elem<T>::bits(x * (1.0f / (float)kAugBig));
      x -= (float)kAugBig * Elem<T>::value(ba);  // exact: both are multiples of ulp(x)
    }
  } else if (!(fabsf(x) <= Elem<T>::kMax)) {
    if (status && fabsf(x) != __int_as_float(0x7f800000) && x == x) atomicOr(status, kStatusRange);
    x = (x > 0.f) ? Elem<T>::kMax : -Elem<T>::kMax;
  }
  const uint16_t b0 = Elem<T>::bits(x);
  const float r1 = x - Elem<T>::value(b0);
  const uint16_t b1 = Elem<T>::bits(r1);
  const uint16_t b2 = Elem<T>::bits(r1 - Elem<T>::value(b1));
  return make_uint4((uint32_t)b0 | ((uint32_t)b1 << 16), (uint32_t)b2 | ((uint32_t)ba << 16), 0u,
                    0u);
}

// D/8 threads per (bh, row) of the padded row range, 16-byte loads of O and dO:
// delta = rowsum(O * dO); the row's extra K-step entries [t0, t1, t2, a, 0, ...]
// of -LSE/scale (Q side) and -delta (dO side); delta itself in fp32 when
// `delta` is given (the separate dQ kernel reads it); the row of the fp32 dQ
// accumulator zeroed when `dq_acc` is given (the fused dQ path).
template <typename T>
__global__ void __launch_bounds__(256) fa_bwd_pre_kernel(
    const T* __restrict__ o, const T* __restrict__ dout, const float* __restrict__ lse,
    uint8_t* __restrict__ q_aug, uint8_t* __restrict__ do_aug, float* __restrict__ dq_acc,
    float* __restrict__ delta, int S /* query rows */,
    int H, int D, int S_pad, float inv_scale, int* status) {
  griddep_wait();  // O and LSE come from the forward
  griddep_launch_dependents();
  const int tpr = D / 8;  // threads per row: 2, 4, 8 or 16 (a power of two inside a warp)
  const int sub = threadIdx.x % tpr;
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) / tpr;
  const int bh = blockIdx.y;
  const bool in_pad = row < S_pad;  // always true for the exact grid; kept for the shuffle
  const int b = bh / H, h = bh % H;
  const size_t prow = (size_t)bh * S_pad + row;
  float acc = 0.f;
  if (row < S) {
    const size_t off = (((size_t)b * S + row) * H + h) * D + sub * 8;
    const uint4 ov = *reinterpret_cast<const uint4*>(o + off);
    const uint4 dv = *reinterpret_cast<const uint4*>(dout + off);
    const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w};
    const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 a = Elem<T>::unpack2(ow[i]);
      const float2 c = Elem<T>::unpack2(dw[i]);
      acc = fmaf(a.x, c.x, acc);
      acc = fmaf(a.y, c.y, acc);
    }
  }
  for (int m = tpr / 2; m > 0; m >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, m);
  if (!in_pad) return;
  if (sub == 0) {
    const float l = row < S ? lse[(size_t)bh * S + row] : __int_as_float(0x7f800000);
    // row blocks of S_pad rows per (batch, head); S_pad is a multiple of 8
    const size_t base = (size_t)bh * S_pad * kAugRowBytes;
    const uint32_t r = (uint32_t)row;
    *reinterpret_cast<uint4*>(q_aug + base + aug_offset(r, 0)) = split_row<T>(-l * inv_scale, status);
    *reinterpret_cast<uint4*>(q_aug + base + aug_offset(r, 8)) = make_uint4(0u, 0u, 0u, 0u);
    *reinterpret_cast<uint4*>(do_aug + base + aug_offset(r, 0)) = split_row<T>(-acc, status);
    *reinterpret_cast<uint4*>(do_aug + base + aug_offset(r, 8)) = make_uint4(0u, 0u, 0u, 0u);
    if (delta != nullptr) delta[prow] = acc;
  }
  if (dq_acc != nullptr) {
    float4* qa = reinterpret_cast<float4*>(dq_acc + prow * D) + sub * 2;
    qa[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    qa[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// -------------------------------------------------------------------------- post
template <typename T>
__global__ void fa_bwd_post_kernel(const float* __restrict__ dq_acc, T* __restrict__ dq,
                                   int S /* query rows */,
                                   int H, int D, int S_pad, float scale) {
  // one thread per 8 consecutive elements of one (b, s, h) row
  griddep_wait();  // the dQ accumulator comes from the main kernel
  griddep_launch_dependents();
  const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = D / 8;
  const size_t rows = (size_t)gridDim.y * S;
  (void)rows;
  const int bh = blockIdx.y;
  const size_t r = idx / per_row;
  if (r >= (size_t)S) return;
  const int e = (int)(idx % per_row) * 8;
  const int b = bh / H, h = bh % H;
  const float* src = dq_acc + ((size_t)bh * S_pad + r) * D + e;
  const float4 x0 = *reinterpret_cast<const float4*>(src);
  const float4 x1 = *reinterpret_cast<const float4*>(src + 4);
  uint4 w;
  w.x = Elem<T>::pack2(x0.x * scale, x0.y * scale);
  w.y = Elem<T>::pack2(x0.z * scale, x0.w * scale);
  w.z = Elem<T>::pack2(x1.x * scale, x1.y * scale);
  w.w = Elem<T>::pack2(x1.z * scale, x1.w * scale);
  *reinterpret_cast<uint4*>(dq + (((size_t)b * S + r) * H + h) * D + e) = w;
}

// -------------------------------------------------------------------------- main
// DQ: also compute dQ (partial per key tile, added into the fp32 accumulator
// with bulk L2 reductions); without it the kernel computes dK and dV only and
// dQ comes from fa_bwd_dq_kernel.
template <int D, typename T, bool DQ>
__global__ void __launch_bounds__(544, 1)
    fa_bwd_main_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v,
                       const uint8_t* __restrict__ q_aug, const uint8_t* __restrict__ do_aug,
                       float* __restrict__ dq_acc,
                       T* __restrict__ dk, T* __restrict__ dv, int Sq, int Sk, int H, int group,
                       int S_pad, int ntiles, int win,
                       float scale, float scale_log2, int causal, int* status,
                       unsigned long long timeout_ns) {
  using C = BwdCfg<D, DQ>;
  constexpr int HW = C::BM / 2;  // query columns per softmax thread
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + 8 * C_COUNT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_BAR + 8 * C_COUNT + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    CTRACE(1);
#ifdef FA_BWD_TRACE
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    if (blockIdx.x < 8192) g_bcta[blockIdx.x][0] = smid;
#endif
  }
  // The CTA walks a list of 128-row key tiles (one tile when the grid has a
  // CTA per tile).  Tile list: (window of `win` K/V heads, key block, K/V head), key block 0 (the most
  // query tiles under a causal mask) first inside each window; round t gives
  // this CTA tile t * grid + pos, pos = blockIdx.x on even rounds and its
  // mirror on odd ones.  With grouped-query attention (`group` query heads per
  // K/V head) a tile runs through every query head of its group, so dK / dV
  // sum over the group in tensor memory.  Barrier phases count iterations (and
  // tiles) over the whole list.
  const int nkt = (Sk + C::BN - 1) / C::BN;
  const int Hkv = H / group;
  const int rounds = (ntiles + (int)gridDim.x - 1) / (int)gridDim.x;
  const int ntq = (Sq + C::BM - 1) / C::BM;
  // causal mask aligned to the bottom-right: query i sees keys j <= i + Sk - Sq
  const int off = Sk - Sq;
  struct KTile {
    int b, hk, kv0, i0, nq, nit;
  };
  auto tile_at = [&](int t, KTile& tl) -> bool {
    const int pos = (t & 1) ? (int)(gridDim.x - 1 - blockIdx.x) : (int)blockIdx.x;
    const int L = t * (int)gridDim.x + pos;
    if (L >= ntiles) return false;
    int bhk, kt;
    grid_to_tile(L, ntiles / nkt, nkt, win, bhk, kt);
    tl.b = bhk / Hkv;
    tl.hk = bhk % Hkv;
    tl.kv0 = kt * C::BN;
    // first query tile that sees this key tile
    tl.i0 = causal ? max(0, tl.kv0 - off) / C::BM : 0;
    tl.nq = max(0, ntq - tl.i0);  // query tiles per query head
    tl.nit = group * tl.nq;       // iterations: (query head, query tile)
    return true;
  };
  // iteration it of a tile: query head hk * group + it / nq, first row of query
  // tile i0 + it % nq (no division for plain multi-head attention: it sits on
  // the softmax warps' path)
  auto q_head = [&](const KTile& tl, int it) { return group == 1 ? tl.hk : tl.hk * group + it / tl.nq; };
  auto q_row0 = [&](const KTile& tl, int it) {
    return (tl.i0 + (group == 1 ? it : it % tl.nq)) * C::BM;
  };

  WaitCtx wc{abort_flag, status, timeout_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < C_COUNT; ++i) {
      uint32_t cnt = 1;
      if (i == C_SFREE || i == C_DSREADY) cnt = 8;
      if (i == C_SFULL) cnt = 2;  // two issuing threads commit
      if (i == C_PFREE) cnt = DQ ? 2 : 1;
      if (i == C_DQFREE) cnt = 4;
      if (i == C_DRAIN) cnt = DQ ? 4 : 3;
      if (i == C_KVEMPTY) cnt = DQ ? 3 : 2;
      if (i == C_DKVFREE) cnt = 8;
      mbar_init(bar(i), cnt);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 13) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp >= 8 && warp < 12) {
    // the extra K-step rows of K and V: [1, 1, 1, kAugBig, 0, ...] for each of the 128 key rows
    const uint32_t r = threadIdx.x - 256;
    st_shared_v4(sbase + C::OFF_ONE + aug_offset(r, 0), Elem<T>::kOne | (Elem<T>::kOne << 16),
                 Elem<T>::kOne | ((uint32_t)Elem<T>::bits((float)kAugBig) << 16), 0u, 0u);
    st_shared_v4(sbase + C::OFF_ONE + aug_offset(r, 8), 0u, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Set-up overlaps the previous kernel (the prep kernel, whose extra K-step
  // rows and zeroed dQ accumulator this kernel uses); K and V, written before
  // it, are loaded before the wait.
  if (warp != 12) {
    griddep_wait();
    griddep_launch_dependents();
  }

  if (warp == 12) {
    // ------------------------------------------------------------ TMA producers
    // Lane 0: K and V of each tile (the next tile's once the last MMAs reading
    // this tile's have completed); lane 1: the Q / dO ring, which runs on into
    // the next tile's query tiles meanwhile.
    auto load_kv = [&](const KTile& tl) {
      mbar_arrive_expect_tx(bar(C_KVFULL), 2 * C::KV_BYTES);
      for (int a = 0; a < C::NAT; ++a) {
        tma_load_4d(sbase + C::OFF_K + a * C::BN * C::SWB, &tm_k, bar(C_KVFULL), a * C::AE,
                    tl.kv0, tl.hk, tl.b);
        tma_load_4d(sbase + C::OFF_V + a * C::BN * C::SWB, &tm_v, bar(C_KVFULL), a * C::AE,
                    tl.kv0, tl.hk, tl.b);
      }
    };
    // K and V were written before the previous kernel: the first tile's load
    // goes out before the wait for it.
    int t_first = 0;
    KTile first{};
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_do);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      for (; t_first < rounds; ++t_first)
        if (tile_at(t_first, first) && first.nit > 0) break;
      if (t_first < rounds) load_kv(first);
    }
    griddep_wait();
    griddep_launch_dependents();
    if (lane == 0) {
      int nkv = t_first < rounds ? 1 : 0;  // K/V loads issued
      for (int t = t_first + 1; t < rounds; ++t) {
        KTile tl;
        if (!tile_at(t, tl) || tl.nit == 0) continue;
        if (!mbar_wait(bar(C_KVEMPTY), (uint32_t)(nkv - 1) & 1u, wc)) break;
        load_kv(tl);
        ++nkv;
      }
      // After an abort, let the loads this thread issued land before the CTA exits.
      if (*abort_flag && nkv > 0) mbar_wait_drain(bar(C_KVFULL), (uint32_t)(nkv - 1) & 1u, timeout_ns);
    } else if (lane == 1) {
      int q_last[C::NST];  // last iteration loaded into each stage
      for (int t = 0; t < C::NST; ++t) q_last[t] = -1;
      int gs = 0;  // iterations of the earlier tiles
      bool ok = true;
      for (int t = 0; ok && t < rounds; ++t) {
        KTile tl;
        if (!tile_at(t, tl) || tl.nit == 0) continue;
        for (int it = 0; it < tl.nit; ++it) {
          const int gi = gs + it;
          const int st = gi % C::NST;
          const uint32_t ph = (uint32_t)(gi / C::NST) & 1u;
          const int q0 = q_row0(tl, it), h = q_head(tl, it);
          TRACE(0, gi);
          if (gi >= C::NST && !mbar_wait(bar(C_QEMPTY + st), ph ^ 1u, wc)) {
            ok = false;
            break;
          }
          TRACE(1, gi);
          mbar_arrive_expect_tx(bar(C_QFULL + st), 2 * C::Q_BYTES + 2 * C::AUG_BYTES);
          for (int a = 0; a < C::NAT; ++a) {
            tma_load_4d(sbase + C::OFF_Q + st * C::Q_BYTES + a * C::BM * C::SWB, &tm_q,
                        bar(C_QFULL + st), a * C::AE, q0, h, tl.b);
            tma_load_4d(sbase + C::OFF_DO + st * C::Q_BYTES + a * C::BM * C::SWB, &tm_do,
                        bar(C_QFULL + st), a * C::AE, q0, h, tl.b);
          }
          const size_t aug = ((size_t)(tl.b * H + h) * S_pad + q0) * kAugRowBytes;
          bulk_load(sbase + C::OFF_QA + st * C::AUG_BYTES, q_aug + aug, C::AUG_BYTES,
                    bar(C_QFULL + st));
          bulk_load(sbase + C::OFF_DA + st * C::AUG_BYTES, do_aug + aug, C::AUG_BYTES,
                    bar(C_QFULL + st));
          q_last[st] = gi;
        }
        gs += tl.nit;
      }
      if (*abort_flag) {
        for (int t = 0; t < C::NST; ++t)
          if (q_last[t] >= 0)
            mbar_wait_drain(bar(C_QFULL + t), (uint32_t)(q_last[t] / C::NST) & 1u, timeout_ns);
      }
    }
  } else if (warp >= 13) {
    // ------------------------------------------------------------ MMA issuers (warps 13..16)
    // Each independent MMA chain has its own issuing thread: one thread issues
    // about one tcgen05.mma per ~55 clk, while an M128 x N64 x K16 MMA takes 48
    // clk with both operands in shared memory (operand reads at 128 B/clk) and 32
    // with A in tensor memory, so a single issuer would leave the tensor core
    // idle on these small tiles; four concurrent issuers keep work queued.  Roles:
    //   0: S^T = K Q^T        1: dP^T = V dO^T      (tile i, once the softmax
    //                                                warps hold tile i-1's values)
    //   2: dV += P^T dO, dK += dS^T Q (A operands in TMEM)
    //   3: dQ partial = dS K (transposed for D=128)
    // A commit only tracks its own thread's MMAs; barriers that need several
    // chains expect one arrival per chain (SFULL: 0+1, PFREE: 2+3).  Tile i's
    // S^T / dP^T are complete before the softmax warps signal DSREADY(i).
    const int role = warp - 13;
    if (lane == 0 && (DQ || role != 3)) {
      constexpr uint32_t swz = swizzle_field(C::SWB);
      constexpr uint32_t ab = Elem<T>::kIdescAB;
      constexpr uint32_t id_s = make_idesc_f16(C::BN, C::BM, false, false) | ab;  // S^T, dP^T
      constexpr uint32_t id_kv = make_idesc_f16(C::BN, D, false, true) | ab;      // dV, dK
      constexpr uint32_t id_dq = (C::DQT ? make_idesc_f16(D, C::BM, true, true)    // dQ^T
                                         : make_idesc_f16(C::BM, D, true, true)) | ab;  // dQ
      bool ok = true;
      int gs = 0, nt = 0;  // iterations and (non-empty) tiles before this one
      for (int t = 0; ok && t < rounds; ++t) {
        KTile tl;
        if (!tile_at(t, tl) || tl.nit == 0) continue;
        if (role != 2 && !mbar_wait(bar(C_KVFULL), (uint32_t)nt & 1u, wc)) break;
        // the first dV / dK MMAs of a tile overwrite the accumulators: the
        // previous tile's epilogue must have read them
        if (role == 2 && nt > 0 && !mbar_wait(bar(C_DKVFREE), (uint32_t)(nt - 1) & 1u, wc)) break;
        for (int it = 0; it < tl.nit; ++it) {
          const int gi = gs + it;
          const int st = gi % C::NST;
          const uint32_t qb = sbase + C::OFF_Q + st * C::Q_BYTES;
          const uint32_t dob = sbase + C::OFF_DO + st * C::Q_BYTES;
          if (role <= 1) {
            // S^T (role 0) or dP^T (role 1): M = 128 key rows, N = BM, K = D
            if (!mbar_wait(bar(C_QFULL + st), (uint32_t)(gi / C::NST) & 1u, wc)) { ok = false; break; }
            if (role == 0) TRACE(15, gi);
            if (gi > 0 && !mbar_wait(bar(C_SFREE), (uint32_t)(gi - 1) & 1u, wc)) { ok = false; break; }
            if (role == 0) TRACE(2, gi);
            if (role == 0 && gi == 0) CTRACE(2);
            tc_fence_after();
            const uint32_t abase = sbase + (role == 0 ? C::OFF_K : C::OFF_V);
            const uint32_t bbase = role == 0 ? qb : dob;
            const uint32_t dcol = tmem + (role == 0 ? C::COL_S : C::COL_DP);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const int a = (kk * 16) / C::AE;
              const uint32_t koff = (uint32_t)((kk * 16) % C::AE) * 2u;
              const uint64_t ad = make_smem_desc(abase + a * C::BN * C::SWB + koff, 16, 8 * C::SWB, swz);
              const uint64_t bd = make_smem_desc(bbase + a * C::BM * C::SWB + koff, 16, 8 * C::SWB, swz);
              mma_f16_ss(dcol, ad, bd, id_s, kk > 0 ? 1u : 0u);
            }
            // extra K step: + (-LSE/scale) resp. + (-delta) for each query column
            mma_f16_ss(dcol, make_smem_desc(sbase + C::OFF_ONE, 128, 256, 0),
                       make_smem_desc(sbase + (role == 0 ? C::OFF_QA : C::OFF_DA) + st * C::AUG_BYTES,
                                      128, 256, 0),
                       id_s, 1u);
            mma_commit(bar(C_SFULL));
            if (role == 0) TRACE(3, gi);
          } else if (role == 2) {
            if (!mbar_wait(bar(C_DSREADY), (uint32_t)gi & 1u, wc)) { ok = false; break; }
            TRACE(4, gi);
            tc_fence_after();
            // dV += P^T dO ; dK += dS^T Q   (M = 128 key rows, N = D, K = BM)
#pragma unroll
            for (int kk = 0; kk < C::BM / 16; ++kk) {
              const uint64_t bd = make_smem_desc(dob + kk * 16 * C::SWB, C::BM * C::SWB, 8 * C::SWB, swz);
              mma_f16_ts(tmem + C::COL_DV, tmem + C::COL_PT + kk * 8, bd, id_kv, (it > 0 || kk > 0) ? 1u : 0u);
            }
#pragma unroll
            for (int kk = 0; kk < C::BM / 16; ++kk) {
              const uint64_t bd = make_smem_desc(qb + kk * 16 * C::SWB, C::BM * C::SWB, 8 * C::SWB, swz);
              if constexpr (C::DS_TMEM) {
                mma_f16_ts(tmem + C::COL_DK, tmem + C::COL_DST + kk * 8, bd, id_kv,
                           (it > 0 || kk > 0) ? 1u : 0u);
              } else {
                const int a = kk / 4;
                const uint32_t koff = (uint32_t)(kk % 4) * 32u;
                const uint64_t sd =
                    make_smem_desc(sbase + C::OFF_DS + a * C::BN * 128 + koff, 16, 1024, 2);
                mma_f16_ss(tmem + C::COL_DK, sd, bd, id_kv, (it > 0 || kk > 0) ? 1u : 0u);
              }
            }
            mma_commit(bar(C_QEMPTY + st));
            mma_commit(bar(C_PFREE));
            TRACE(6, gi);
          } else if constexpr (DQ) {
            if (!mbar_wait(bar(C_DSREADY), (uint32_t)gi & 1u, wc) ||
                (gi > 0 && !mbar_wait(bar(C_DQFREE), (uint32_t)(gi - 1) & 1u, wc))) {
              ok = false;
              break;
            }
            TRACE(5, gi);
            tc_fence_after();
            // dQ partial over this key tile (K = 128 key rows)
#pragma unroll
            for (int kk = 0; kk < C::BN / 16; ++kk) {
              const uint64_t dsd =
                  make_smem_desc(sbase + C::OFF_DS + kk * 16 * 128, C::BN * 128, 1024, 2);
              const uint64_t kd =
                  make_smem_desc(sbase + C::OFF_K + kk * 16 * C::SWB, C::BN * C::SWB, 8 * C::SWB, swz);
              if constexpr (C::DQT)
                mma_f16_ss(tmem + C::COL_DQ, kd, dsd, id_dq, kk > 0 ? 1u : 0u);  // K^T dS^T
              else
                mma_f16_ss(tmem + C::COL_DQ, dsd, kd, id_dq, kk > 0 ? 1u : 0u);  // dS K
            }
            mma_commit(bar(C_DQFULL));
            mma_commit(bar(C_PFREE));
          }
        }
        if (!ok) break;
        if (role == 2) mma_commit(bar(C_KVDONE));  // dK / dV of this tile complete
        else mma_commit(bar(C_KVEMPTY));           // K / V may be reloaded
        gs += tl.nit;
        ++nt;
      }
      mma_commit(bar(C_DRAIN));  // also on abort: teardown waits for every issued MMA
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ softmax / dS warps 0..7
    const int lq = warp & 3;         // TMEM lane quarter
    const int hf = warp >> 2;        // which half of the query columns
    const int r = lq * 32 + lane;    // key row inside the tile == TMEM lane
    const uint32_t lane_base = (uint32_t)(lq * 32) << 16;
    const int c0 = hf * HW;          // first query column of this thread
    constexpr int EC = (D / 2 >= 16) ? D / 2 : 16;  // dK / dV epilogue columns per warp
    bool ok = true;
    int gs = 0, nt = 0;  // iterations and (non-empty) tiles before this one
    for (int t = 0; ok && t < rounds; ++t) {
      KTile tl;
      if (!tile_at(t, tl)) continue;
      const int kv0 = tl.kv0, nit = tl.nit;
      const int kv_idx = kv0 + r;
      const bool kv_ok = kv_idx < Sk;
      if (nit == 0) {
         // no query row sees this key tile (Sq < Sk): dK = dV = 0
         const size_t row_off = (((size_t)tl.b * Sk + kv_idx) * Hkv + tl.hk) * D + hf * EC;
         if (kv_ok && hf * EC < D)
           for (int c = 0; c < EC; c += 8) {
             *reinterpret_cast<uint4*>(dv + row_off + c) = make_uint4(0u, 0u, 0u, 0u);
             *reinterpret_cast<uint4*>(dk + row_off + c) = make_uint4(0u, 0u, 0u, 0u);
           }
         continue;
      }
      for (int it = 0; it < nit; ++it) {
        const int gi = gs + it;
        const int st = gi % C::NST;
        const int q0 = q_row0(tl, it);
        if (!mbar_wait(bar(C_QFULL + st), (uint32_t)(gi / C::NST) & 1u, wc) ||
            !mbar_wait(bar(C_SFULL), (uint32_t)gi & 1u, wc)) {
          ok = false;
          break;
        }
        if (threadIdx.x == 0) TRACE(7, gi);
        tc_fence_after();
        // 32 query columns at a time (bounds the registers held for BM = 128). S^T and
        // dP^T are released after the last chunk's loads; P^T / dS^T are written only
        // once the previous tile's dV / dK MMAs have read them (PFREE).
        // every (query, key) pair of this tile is unmasked
        const bool full_tile = (kv0 + C::BN <= Sk) && (!causal || q0 + off >= kv0 + C::BN - 1);
        for (int cc = 0; cc < HW / 32; ++cc) {
          const int cb = c0 + cc * 32;  // first query column of this chunk
          uint32_t sr[32], dr[32];
          tmem_ld32(tmem + lane_base + C::COL_S + cb, sr);
          tmem_ld32(tmem + lane_base + C::COL_DP + cb, dr);
          tmem_wait_ld();
          if (threadIdx.x == 0 && cc == 0) TRACE(14, gi);
          if (cc == HW / 32 - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(C_SFREE));
            if (threadIdx.x == 0) TRACE(8, gi);
          }
          // P^T and dS^T for these 32 query columns, packed to fp16 pairs (S'^T and
          // dP'^T already hold -LSE/scale and -delta).  Only tiles that cross the
          // causal diagonal or the end of the sequence need the per-element mask.
          uint32_t pp[16], dd[16];
          if (full_tile) {
            const uint64_t c2 = f2_pack(scale_log2, scale_log2);
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              float x0, x1;
              f2_unpack(f2_mul(f2_pack(__uint_as_float(sr[2 * k]), __uint_as_float(sr[2 * k + 1])), c2),
                        x0, x1);
              const float p0 = ex2(x0), p1 = ex2(x1);
              float d0, d1;
              f2_unpack(f2_mul(f2_pack(p0, p1),
                               f2_pack(__uint_as_float(dr[2 * k]), __uint_as_float(dr[2 * k + 1]))),
                        d0, d1);
              pp[k] = Elem<T>::pack2(p0, p1);
              dd[k] = Elem<T>::pack2(d0, d1);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
              float p4[4], ds4[4];
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const int ql = cb + e + u;
                const bool valid = kv_ok && (!causal || (q0 + ql + off) >= kv_idx);
                const float pe = valid ? ex2(__uint_as_float(sr[e + u]) * scale_log2) : 0.f;
                p4[u] = pe;
                ds4[u] = pe * __uint_as_float(dr[e + u]);
              }
              pp[e / 2] = Elem<T>::pack2(p4[0], p4[1]);
              pp[e / 2 + 1] = Elem<T>::pack2(p4[2], p4[3]);
              dd[e / 2] = Elem<T>::pack2(ds4[0], ds4[1]);
              dd[e / 2 + 1] = Elem<T>::pack2(ds4[2], ds4[3]);
            }
          }
          if (cc == 0) {
            if (threadIdx.x == 0) TRACE(11, gi);
            if (gi > 0 && !mbar_wait(bar(C_PFREE), (uint32_t)(gi - 1) & 1u, wc)) {
              ok = false;
              break;
            }
            if (threadIdx.x == 0) TRACE(9, gi);
          }
          // P^T (and for D=128 dS^T) into tensor memory; dS^T into the [key row][query
          // col] K-major SW128 shared tile (64-column atoms) that the dQ MMA reads.
          tmem_st16(tmem + lane_base + C::COL_PT + cb / 2, pp);
          if constexpr (C::DS_TMEM) tmem_st16(tmem + lane_base + C::COL_DST + cb / 2, dd);
          if constexpr (DQ || !C::DS_TMEM) {
            const int a = cb / 64;
            const int ch0 = (cb % 64) / 8;
            const uint32_t sb = sbase + C::OFF_DS + a * C::BN * 128;
#pragma unroll
            for (int u = 0; u < 4; ++u)
              st_shared_v4(sb + sw128_offset(r, ch0 + u), dd[4 * u], dd[4 * u + 1], dd[4 * u + 2],
                           dd[4 * u + 3]);
          }
        }
        if (!ok) break;
        tmem_wait_st();
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(C_DSREADY));
        if (threadIdx.x == 0) TRACE(10, gi);
      }
      if (!ok) break;
      // ---------------------------------------------------------- dK / dV epilogue
      if (!mbar_wait(bar(C_KVDONE), (uint32_t)nt & 1u, wc)) { ok = false; break; }
      tc_fence_after();
      if (hf * EC < D) {
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
          const uint32_t col = (pass == 0 ? C::COL_DV : C::COL_DK) + hf * EC;
          const float f = pass == 0 ? 1.f : scale;
          T* dst = (pass == 0 ? dv : dk) + (((size_t)tl.b * Sk + kv_idx) * Hkv + tl.hk) * D + hf * EC;
#pragma unroll
          for (int c = 0; c < EC / 16; ++c) {
            uint32_t v[16];
            tmem_ld16(tmem + lane_base + col + c * 16, v);
            tmem_wait_ld();
            uint4 w0, w1;
            w0.x = Elem<T>::pack2(__uint_as_float(v[0]) * f, __uint_as_float(v[1]) * f);
            w0.y = Elem<T>::pack2(__uint_as_float(v[2]) * f, __uint_as_float(v[3]) * f);
            w0.z = Elem<T>::pack2(__uint_as_float(v[4]) * f, __uint_as_float(v[5]) * f);
            w0.w = Elem<T>::pack2(__uint_as_float(v[6]) * f, __uint_as_float(v[7]) * f);
            w1.x = Elem<T>::pack2(__uint_as_float(v[8]) * f, __uint_as_float(v[9]) * f);
            w1.y = Elem<T>::pack2(__uint_as_float(v[10]) * f, __uint_as_float(v[11]) * f);
            w1.z = Elem<T>::pack2(__uint_as_float(v[12]) * f, __uint_as_float(v[13]) * f);
            w1.w = Elem<T>::pack2(__uint_as_float(v[14]) * f, __uint_as_float(v[15]) * f);
            if (kv_ok) {
              reinterpret_cast<uint4*>(dst + c * 16)[0] = w0;
              reinterpret_cast<uint4*>(dst + c * 16)[1] = w1;
            }
          }
        }
      }
      // dK / dV have been read: the next tile's first dV / dK MMAs may overwrite them
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(C_DKVFREE));
      gs += nit;
      ++nt;
    }
  } else if (DQ && warp < 12) {
    // ------------------------------------------------------------ dQ epilogue warps 8..11
    // Each tile's dQ partial goes TMEM -> registers -> shared memory ([q][d] fp32,
    // the accumulator's own layout) -> one bulk fp32 reduction into global memory.
    const int wq = warp - 8;
    const int tid = threadIdx.x - 256;  // 0..127
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    bool ok = true;
    int gs = 0;  // iterations of the earlier tiles
    for (int t = 0; ok && t < rounds; ++t) {
      KTile tl;
      if (!tile_at(t, tl) || tl.nit == 0) continue;
      for (int it = 0; it < tl.nit; ++it) {
        const int gi = gs + it;
        const int q0 = q_row0(tl, it);
        const int bh = tl.b * H + q_head(tl, it);
        const int sbuf = gi % C::NDQ;
        const uint32_t stage = sbase + C::OFF_DQS + sbuf * C::DQ_STAGE_BYTES;
        if (!mbar_wait(bar(C_DQFULL), (uint32_t)gi & 1u, wc)) { ok = false; break; }
        if (tid == 0) TRACE(12, gi);
        tc_fence_after();
        if constexpr (C::DQT) {
          // TMEM lane = d, column = query row
          const int d = wq * 32 + lane;
          uint32_t v0[32], v1[32];
          tmem_ld32(tmem + lane_base + C::COL_DQ, v0);
          tmem_ld32(tmem + lane_base + C::COL_DQ + 32, v1);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(C_DQFREE));
          if (tid == 0) bulk_wait_group_read<C::NDQ - 1>();  // this buffer's last reduction read it
          named_bar_sync(1, 128);
#pragma unroll
          for (int e = 0; e < 32; ++e) st_shared_f32(stage + (uint32_t)(e * D + d) * 4u, __uint_as_float(v0[e]));
#pragma unroll
          for (int e = 0; e < 32; ++e)
            st_shared_f32(stage + (uint32_t)((32 + e) * D + d) * 4u, __uint_as_float(v1[e]));
        } else {
          // TMEM lane = query row, column = d; CW columns at a time (flat register
          // use). The staging buffer must be free before the first chunk's stores;
          // the accumulator is released after the last chunk's loads.
          constexpr int CW = D < 32 ? D : 32;
          constexpr int NP = CW / 4;  // 16-byte pieces per chunk row
          const int qr = wq * 32 + lane;
          if (tid == 0) bulk_wait_group_read<C::NDQ - 1>();  // this buffer's last reduction read it
          named_bar_sync(1, 128);
          const uint32_t rowa = stage + (uint32_t)(qr * D * 4);
#pragma unroll
          for (int c = 0; c < D / CW; ++c) {
            uint32_t v[CW];
            if constexpr (CW == 32)
              tmem_ld32(tmem + lane_base + C::COL_DQ + c * CW, *reinterpret_cast<uint32_t(*)[32]>(v));
            else
              tmem_ld16(tmem + lane_base + C::COL_DQ + c * CW, *reinterpret_cast<uint32_t(*)[16]>(v));
            tmem_wait_ld();
            if (c == D / CW - 1) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(bar(C_DQFREE));
            }
#pragma unroll
            for (int p = 0; p < NP; ++p) {
              const int pc = (p + lane) % NP;  // rotate pieces across lanes: fewer bank conflicts
              uint32_t w0 = v[0], w1 = v[1], w2 = v[2], w3 = v[3];
              // select the rotated piece without dynamic register indexing
#pragma unroll
              for (int t = 0; t < NP; ++t)
                if (t == pc) { w0 = v[4 * t]; w1 = v[4 * t + 1]; w2 = v[4 * t + 2]; w3 = v[4 * t + 3]; }
              st_shared_v4(rowa + (uint32_t)(c * CW + 4 * pc) * 4u, w0, w1, w2, w3);
            }
          }
        }
        fence_proxy_async_smem();
        named_bar_sync(1, 128);
        if (tid == 0) {
          bulk_reduce_add_f32(dq_acc + ((size_t)bh * S_pad + q0) * D, stage, C::DQ_STAGE_BYTES);
          bulk_commit_group();
          TRACE(13, gi);
        }
      }
      gs += tl.nit;
    }
    if (tid == 0) bulk_wait_group_all();
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    if (lane == 0) mbar_wait_drain(bar(C_DRAIN), 0, timeout_ns);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
    if (lane == 0) CTRACE(3);
  }
}

template <int D, typename T, bool DQ>
static int launch_bwd_main(const BwdArgs& a, cudaStream_t stream) {
  using C = BwdCfg<D, DQ>;
  constexpr int tag = 2000 + D + (std::is_same<T, __half>::value ? 0 : 1000) + (DQ ? 0 : 4000);
  if (!smem_attr_set<tag>(reinterpret_cast<const void*>(fa_bwd_main_kernel<D, T, DQ>), C::SMEM))
    return FA_ERR_LAUNCH;
  const int ntiles = a.B * a.Hkv * ((a.Sk + C::BN - 1) / C::BN);
  const int nsm = sm_count();
  if (nsm <= 0) return FA_ERR_DEVICE;
  const int g =
      tile_grid(ntiles, nsm, persist_max_tiles(a.causal != 0, a.Sq > a.Sk ? a.Sq : a.Sk));
  dim3 grid(g);
  const cudaError_t e = launch_pdl(
      fa_bwd_main_kernel<D, T, DQ>, grid, dim3(C::THREADS), C::SMEM, stream, *a.tm_q, *a.tm_do,
      *a.tm_k, *a.tm_v, a.q_aug, a.do_aug, a.dq_acc, static_cast<T*>(a.dk), static_cast<T*>(a.dv),
      a.Sq, a.Sk, a.H, a.H / a.Hkv, a.S_pad, ntiles, tile_window(ntiles, g), a.scale,
      a.scale * 1.4426950408889634f,
      a.causal,
      a.status,
      a.timeout_ns);
  return e == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

int bwd_q_rows(int D) { return D == 128 ? 64 : 128; }

template <typename T>
static int launch_bwd_t(const BwdArgs& a, cudaStream_t stream, int phase) {
  const bool sep = a.dq_separate != 0;
  if (phase < 0 || phase == 0) {
    const int rows_per_block = 256 / (a.D / 8);
    dim3 grid((a.S_pad + rows_per_block - 1) / rows_per_block, a.B * a.H);
    if (launch_pdl(fa_bwd_pre_kernel<T>, grid, dim3(256), 0, stream, static_cast<const T*>(a.o),
                   static_cast<const T*>(a.dout), a.lse, a.q_aug, a.do_aug,
                   sep ? nullptr : a.dq_acc, sep ? a.delta : nullptr, a.Sq, a.H, a.D, a.S_pad,
                   1.0f / a.scale, a.status) != cudaSuccess)
      return FA_ERR_LAUNCH;
  }
  int rc = FA_OK;
  if (phase < 0 || phase == 1) {
    switch (a.D) {
      case 16: rc = sep ? launch_bwd_main<16, T, false>(a, stream) : launch_bwd_main<16, T, true>(a, stream); break;
      case 32: rc = sep ? launch_bwd_main<32, T, false>(a, stream) : launch_bwd_main<32, T, true>(a, stream); break;
      case 64: rc = sep ? launch_bwd_main<64, T, false>(a, stream) : launch_bwd_main<64, T, true>(a, stream); break;
      case 128: rc = sep ? launch_bwd_main<128, T, false>(a, stream) : launch_bwd_main<128, T, true>(a, stream); break;
      default: return FA_ERR_ARG;
    }
  }
  if (rc != FA_OK) return rc;
  if (phase < 0 || phase == 2) {
    if (sep) return launch_bwd_dq(a, stream);
    const int per_row = a.D / 8;
    const size_t n = (size_t)a.Sq * per_row;
    dim3 grid((unsigned)((n + 255) / 256), a.B * a.H);
    if (launch_pdl(fa_bwd_post_kernel<T>, grid, dim3(256), 0, stream, a.dq_acc,
                   static_cast<T*>(a.dq), a.Sq, a.H, a.D, a.S_pad, a.scale) != cudaSuccess)
      return FA_ERR_LAUNCH;
  }
  return FA_OK;
}

int launch_bwd(const BwdArgs& a, cudaStream_t stream, int phase) {
  return a.dtype == FA_DTYPE_BF16 ? launch_bwd_t<__nv_bfloat16>(a, stream, phase)
                                  : launch_bwd_t<__half>(a, stream, phase);
}

}  // namespace fa_sm100

#ifdef FA_BWD_TRACE
extern "C" int fa_debug_trace(void* dst) {
  return (int)cudaMemcpyFromSymbol(dst, fa_sm100::g_trace, sizeof(fa_sm100::g_trace));
}
extern "C" int fa_debug_trace_bwd_cta(void* dst) {
  return (int)cudaMemcpyFromSymbol(dst, fa_sm100::g_bcta, sizeof(fa_sm100::g_bcta));
}
#endif
