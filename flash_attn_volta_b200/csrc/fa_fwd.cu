// FlashAttention forward for sm_100a (B200): O = softmax(scale * Q K^T) V and the
// natural-log log-sum-exp per query row.
//
// Replaces the reference's Triton kernels _fa_fwd_kernel_d64 / _d128
// (flash_attn_volta/triton_fa.py:63-284) and the permute/pad work of its host
// wrapper (triton_fa.py:291-397): Q/K/V are read by TMA straight from the
// (B, S, H, D) fp16 tensors (row stride H*D), every head_dim in {16,32,64,128}
// runs natively (no zero padding), and O is written in (B, S, H, D).
//
// A CTA walks a list of 128-row query tiles of the (batch, head) pairs (round
// r takes tile r * grid + CTA, in reverse CTA order on odd rounds, over a
// longest-first order).  Problems of at most 16 tiles per SM (8 for causal
// sequences longer than 4096) run one persistent CTA per SM, so the set-up is
// paid once per SM and the next tile's Q load and first S = Q K^T overlap this
// tile's last softmax step and its epilogue; larger ones run one CTA per tile.  Tensor memory (512
// columns): S0 [0,128), S1 [128,256) — S = Q K_j^T double-buffered; P0
// [256,320), P1 [320,384) — P (fp16 pairs) double-buffered; O [384, 384+D).
// Because P has its own columns, nothing in the tensor-core stream waits for
// P to be consumed before the next S is computed.  Warp roles:
//   warps 0-15  softmax: warp w owns TMEM lane quarter w % 4 (query rows
//              32*(w%4)..) and key-column quarter w / 4 (32 columns) of each
//              128-column key tile.  Loads its S columns and releases the S
//              buffer at once, trades partial row maxima with the other three
//              warps of its rows (shared memory + a 4-arrival mbarrier),
//              computes P in the exp2 domain (packed f32x2 arithmetic; one pair
//              in four on the FMA pipe), writes P to tensor memory and rescales
//              its share of O when the running max grew by more than 2^8
//              (lazy rescale); epilogue O/l and LSE.
//   warp 16    TMA producers: lane 0 Q of each tile (once the previous tile's
//              last S MMA has read its Q), then K tiles through their ring;
//              lane 1 V tiles through their ring.
//   warp 17    S issuer:  S_b = Q K_j^T (b = j % 2) once the softmax warps
//              have read S_b of tile j-2.
//   warp 18    PV issuer: O += P_b V_j (P_b as the tensor-memory A operand)
//              once the softmax warps have written P_b; a tile's first PV
//              (which overwrites O) waits until the previous tile's epilogue
//              has read O.
// Barrier phases count steps (and tiles) over the CTA's whole tile list.
// One thread issues about one tcgen05.mma per ~55 clk, close to the 64 clk an
// M128 x N128 x K16 MMA takes, so the S and PV chains get a thread each and
// interleave on the tensor core.
//
// Semantics kept from the reference: top-left causal mask (column > row is
// masked, triton_fa.py:124-126), columns >= S masked (:123), LSE = m + ln(l)
// and +inf for a row with l == 0 (:152-159), rows >= S not stored (:149-150).
// Beyond the reference: Sq != Sk (query rows against a key sequence of another
// length) with the causal mask aligned to the bottom-right, query i seeing keys
// j <= i + Sk - Sq (identical to the above when Sq == Sk).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <type_traits>

#include "fa_kernels.h"
#include "sm100_ptx.cuh"

namespace fa_sm100 {

#ifdef FA_FWD_TRACE
#ifndef FA_TRACE_BLOCK
#define FA_TRACE_BLOCK 0
#endif
// Debug build only: clock64() stamps of barrier events of one CTA, read back
// with fa_debug_trace_fwd().
__device__ unsigned long long g_ftrace[64][16];
#define FTRACE(slot, it)                                                                    \
  do {                                                                                      \
    if (blockIdx.x == FA_TRACE_BLOCK && (it) < 64) g_ftrace[it][slot] = clock64();           \
  } while (0)
// per-CTA timeline: SM id, globaltimer at entry, at the first S issue, at exit
__device__ unsigned long long g_fcta[8192][4];
#define CTRACE(slot)                                                                        \
  do {                                                                                      \
    if (blockIdx.x < 8192) g_fcta[blockIdx.x][slot] = globaltimer_ns();                     \
  } while (0)
#else
#define FTRACE(slot, it) \
  do {                   \
  } while (0)
#define CTRACE(slot) \
  do {               \
  } while (0)
#endif

template <int D>
struct FwdCfg {
  static constexpr int BM = 128, BN = 128;  // query rows per CTA, key rows per tile
  static constexpr int SWB = (D * 2 >= 128) ? 128 : D * 2;  // swizzle width (bytes)
  static constexpr int AE = SWB / 2;                        // elements per swizzle row
  static constexpr int NAT = D / AE;                        // swizzle atoms along D
  static constexpr int NSTK = (D == 128) ? 3 : 4;           // K ring depth
  static constexpr int NSTV = (D == 128) ? 2 : 4;           // V ring depth
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + NSTK * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + NSTV * KV_BYTES;
  static constexpr int BAR_BYTES = 512;  // barriers, TMEM slot, abort flag
  static constexpr int OFF_XCH = OFF_BAR + BAR_BYTES;  // row-max / row-sum exchange
  static constexpr int XCH_BYTES = 2 * 4 * 128 * 4;    // [parity][column quarter][row]
  static constexpr int SMEM = OFF_XCH + XCH_BYTES + 1024;  // + alignment slack
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr int THREADS = 608;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t COL_S = 0, COL_P = 256, COL_O = 384;  // S_b: +128 b, P_b: +64 b
};

// barrier slots (8 bytes each) inside the barrier block
enum FwdBar {
  B_QFULL = 0,
  B_KFULL = 1,    // +NSTK (<= 4)
  B_KEMPTY = 5,   // +NSTK
  B_VFULL = 9,    // +NSTV (<= 4)
  B_VEMPTY = 13,  // +NSTV
  B_SFULL = 17,   // +b
  B_SFREE = 19,   // +b, 16 arrivals: softmax warps hold S_b in registers
  B_PFULL = 21,   // +b, 16 arrivals: P_b written (and O rescaled)
  B_PFREE = 23,   // +b: O += P_b V done reading P_b
  B_ODONE = 25,   // every O += P V (waited only where at most one phase is pending)
  B_XCHG = 26,    // +row quarter, 4 arrivals
  B_DRAIN = 30,   // 2 arrivals: each issuer's last commit
  B_QEMPTY = 31,  // a tile's last S MMA has read Q
  B_OFREE = 32,   // 16 arrivals: the epilogue has read O
  B_COUNT = 33
};

template <int D, typename T>
__global__ void __launch_bounds__(608, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, T* __restrict__ out,
                  float* __restrict__ lse, int Sq, int Sk, int H, int group, int ntiles, int win,
                  float scale_log2, int causal,
                  int* status, unsigned long long timeout_ns, int debug_flags) {
  using C = FwdCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + 8 * B_COUNT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_BAR + 8 * B_COUNT + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    CTRACE(1);
#ifdef FA_FWD_TRACE
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    if (blockIdx.x < 8192) g_fcta[blockIdx.x][0] = smid;
#endif
  }
  // Tile list: ntiles tiles in the order (window of `win` heads, query
  // block rank, head), longest blocks first inside each window so that K/V of
  // only a few heads live at once (L2 reuse) while the tiles dealt out in one
  // round have similar lengths.  Round t gives this CTA tile t * grid + pos,
  // pos = blockIdx.x on even rounds and its mirror on odd ones (the CTA with
  // the longest tile of one round gets the shortest of the next).
  const int nblk = (Sq + C::BM - 1) / C::BM;
  const int rounds = (ntiles + (int)gridDim.x - 1) / (int)gridDim.x;
  // causal mask aligned to the bottom-right: query i sees keys j <= i + Sk - Sq
  // (the top-left mask of square attention when Sq == Sk)
  const int off = Sk - Sq;
  const int nkv_all = (Sk + C::BN - 1) / C::BN;
  struct Tile {
    int b, h, hk, bh, q0, nkv;
  };
  auto tile_at = [&](int t, Tile& tl) -> bool {
    const int pos = (t & 1) ? (int)(gridDim.x - 1 - blockIdx.x) : (int)blockIdx.x;
    const int L = t * (int)gridDim.x + pos;
    if (L >= ntiles) return false;
    int bh, rank;
    grid_to_tile(L, ntiles / nblk, nblk, win, bh, rank);
    const int qt = causal ? (nblk - 1 - rank) : rank;
    tl.bh = bh;
    tl.b = bh / H;
    tl.h = bh % H;
    tl.hk = tl.h / group;  // K/V head (grouped-query attention: `group` query heads per K/V head)
    tl.q0 = qt * C::BM;
    tl.nkv = causal ? max(0, min(nkv_all, (tl.q0 + C::BM + off + C::BN - 1) / C::BN)) : nkv_all;
    return true;
  };

  WaitCtx wc{abort_flag, status, timeout_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < B_COUNT; ++i) {
      uint32_t cnt = 1;
      if (i == B_SFREE || i == B_SFREE + 1 || i == B_PFULL || i == B_PFULL + 1 || i == B_OFREE)
        cnt = 16;
      if (i >= B_XCHG && i < B_XCHG + 4) cnt = 4;
      if (i == B_DRAIN) cnt = 2;
      mbar_init(bar(i), cnt);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 17) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Set-up above overlaps the previous kernel's tail; inputs are read below.
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 16) {
    // ------------------------------------------------------------ TMA producers
    // Lane 0: Q, then the K ring; lane 1: the V ring.  K runs ahead on its own
    // thread: were K and V issued by one thread, each K load would queue behind
    // a V slot that frees only when O += P V of two tiles back completes, about
    // one load latency before S needs that K.  (Two lanes of one warp, not two
    // warps: the softmax warps need the registers.)
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      int loaded = 0;  // K loads issued (steps over the whole tile list)
      int nq = 0;      // Q loads issued
      int gs = 0;      // steps of the earlier tiles
      bool ok = true;
      for (int t = 0; ok && t < rounds; ++t) {
        Tile tl;
        if (!tile_at(t, tl) || tl.nkv == 0) continue;
        if (nq > 0 && !mbar_wait(bar(B_QEMPTY), (uint32_t)(nq - 1) & 1u, wc)) break;
        mbar_arrive_expect_tx(bar(B_QFULL), C::Q_BYTES);
        for (int a = 0; a < C::NAT; ++a)
          tma_load_4d(sbase + C::OFF_Q + a * C::BM * C::SWB, &tm_q, bar(B_QFULL), a * C::AE,
                      tl.q0, tl.h, tl.b);
        ++nq;
        for (int j = 0; j < tl.nkv; ++j) {
          const int g = gs + j, sk = g % C::NSTK;
          if (g >= C::NSTK &&
              !mbar_wait(bar(B_KEMPTY + sk), (uint32_t)(g / C::NSTK - 1) & 1u, wc)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar(B_KFULL + sk), C::KV_BYTES);
          for (int a = 0; a < C::NAT; ++a)
            tma_load_4d(sbase + C::OFF_K + sk * C::KV_BYTES + a * C::BN * C::SWB, &tm_k,
                        bar(B_KFULL + sk), a * C::AE, j * C::BN, tl.hk, tl.b);
          loaded = g + 1;
        }
        gs += tl.nkv;
      }
      // After an abort, let the loads this thread issued land before the CTA exits.
      if (*abort_flag) {
        if (nq > 0) mbar_wait_drain(bar(B_QFULL), (uint32_t)(nq - 1) & 1u, timeout_ns);
        for (int g = max(0, loaded - C::NSTK); g < loaded; ++g)
          mbar_wait_drain(bar(B_KFULL + g % C::NSTK), (uint32_t)(g / C::NSTK) & 1u, timeout_ns);
      }
    } else if (lane == 1) {
      tma_prefetch_desc(&tm_v);
      int loaded = 0, gs = 0;
      bool ok = true;
      for (int t = 0; ok && t < rounds; ++t) {
        Tile tl;
        if (!tile_at(t, tl) || tl.nkv == 0) continue;
        for (int j = 0; j < tl.nkv; ++j) {
          const int g = gs + j, sv = g % C::NSTV;
          if (g >= C::NSTV &&
              !mbar_wait(bar(B_VEMPTY + sv), (uint32_t)(g / C::NSTV - 1) & 1u, wc)) {
            ok = false;
            break;
          }
          loaded = g + 1;
          // test hook (fa_sm100_set_debug_flags bit 0): never load the CTA's first
          // V tile, so the PV issuer's wait for it runs out
          if ((debug_flags & 1) && g == 0) continue;
          mbar_arrive_expect_tx(bar(B_VFULL + sv), C::KV_BYTES);
          for (int a = 0; a < C::NAT; ++a)
            tma_load_4d(sbase + C::OFF_V + sv * C::KV_BYTES + a * C::BN * C::SWB, &tm_v,
                        bar(B_VFULL + sv), a * C::AE, j * C::BN, tl.hk, tl.b);
        }
        gs += tl.nkv;
      }
      if (*abort_flag) {
        for (int g = max(0, loaded - C::NSTV); g < loaded; ++g) {
          if ((debug_flags & 1) && g == 0) continue;
          mbar_wait_drain(bar(B_VFULL + g % C::NSTV), (uint32_t)(g / C::NSTV) & 1u, timeout_ns);
        }
      }
    }
  } else if (warp == 17) {
    // ------------------------------------------------------------ S issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_f16(C::BM, C::BN, false, false) | Elem<T>::kIdescAB;
      constexpr uint32_t swz = swizzle_field(C::SWB);
      bool ok = true;
      int gs = 0, nq = 0;
      for (int t = 0; ok && t < rounds; ++t) {
        Tile tl;
        if (!tile_at(t, tl) || tl.nkv == 0) continue;
        if (!mbar_wait(bar(B_QFULL), (uint32_t)nq & 1u, wc)) break;
        for (int j = 0; j < tl.nkv; ++j) {
          const int g = gs + j, sk = g % C::NSTK, sb = g & 1;
          if (!mbar_wait(bar(B_KFULL + sk), (uint32_t)(g / C::NSTK) & 1u, wc) ||
              (g >= 2 && !mbar_wait(bar(B_SFREE + sb), (uint32_t)((g - 2) >> 1) & 1u, wc))) {
            ok = false;
            break;
          }
          FTRACE(0, g);
          if (g == 0) CTRACE(2);
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int a = (kk * 16) / C::AE;
            const uint32_t koff = (uint32_t)((kk * 16) % C::AE) * 2u;
            const uint64_t ad = make_smem_desc(sbase + C::OFF_Q + a * C::BM * C::SWB + koff, 16,
                                               8 * C::SWB, swz);
            const uint64_t bd =
                make_smem_desc(sbase + C::OFF_K + sk * C::KV_BYTES + a * C::BN * C::SWB + koff, 16,
                               8 * C::SWB, swz);
            mma_f16_ss(tmem + C::COL_S + sb * 128, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
          }
          mma_commit(bar(B_SFULL + sb));
          mma_commit(bar(B_KEMPTY + sk));
          FTRACE(1, g);
        }
        if (!ok) break;
        mma_commit(bar(B_QEMPTY));  // Q may be reloaded for the next tile
        ++nq;
        gs += tl.nkv;
      }
      mma_commit(bar(B_DRAIN));  // also on abort: teardown waits for every issued MMA
    }
  } else if (warp == 18) {
    // ------------------------------------------------------------ PV issuer
    if (lane == 0) {
      constexpr uint32_t idesc_pv = make_idesc_f16(C::BM, D, false, true) | Elem<T>::kIdescAB;
      constexpr uint32_t swz = swizzle_field(C::SWB);
      bool ok = true;
      int gs = 0, nt = 0;
      for (int t = 0; ok && t < rounds; ++t) {
        Tile tl;
        if (!tile_at(t, tl) || tl.nkv == 0) continue;
        // the first O += P V of a tile overwrites O: the previous epilogue must have read it
        if (nt > 0 && !mbar_wait(bar(B_OFREE), (uint32_t)(nt - 1) & 1u, wc)) break;
        for (int j = 0; j < tl.nkv; ++j) {
          const int g = gs + j, sv = g % C::NSTV, pb = g & 1;
          if (!mbar_wait(bar(B_PFULL + pb), (uint32_t)(g >> 1) & 1u, wc) ||
              !mbar_wait(bar(B_VFULL + sv), (uint32_t)(g / C::NSTV) & 1u, wc)) {
            ok = false;
            break;
          }
          FTRACE(2, g);
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < C::BN / 16; ++kk) {
            const uint64_t bd = make_smem_desc(sbase + C::OFF_V + sv * C::KV_BYTES + kk * 16 * C::SWB,
                                               C::BN * C::SWB, 8 * C::SWB, swz);
            mma_f16_ts(tmem + C::COL_O, tmem + C::COL_P + pb * 64 + kk * 8, bd, idesc_pv,
                       (j > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(bar(B_ODONE));
          mma_commit(bar(B_VEMPTY + sv));
          mma_commit(bar(B_PFREE + pb));
          FTRACE(3, g);
        }
        ++nt;
        gs += tl.nkv;
      }
      mma_commit(bar(B_DRAIN));
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0..15
    const int lq = warp & 3;  // TMEM lane quarter (query rows 32*lq..)
    const int cq = warp >> 2;  // key-column quarter (32 columns of each key tile)
    const int r = lq * 32 + lane;
    const uint32_t lane_base = (uint32_t)(lq * 32) << 16;
    constexpr int QC = C::BN / 4;                   // key columns per warp
    constexpr int EC = (D / 4 >= 16) ? D / 4 : 16;  // O columns per warp
    const bool o_cols = cq * EC < D;
    float* xch = reinterpret_cast<float*>(smem + C::OFF_XCH);  // [parity][cq][row]
    const uint32_t xbar = bar(B_XCHG + lq);
    const float NEG_INF = -__int_as_float(0x7f800000);
    bool ok = true;
    int gs = 0;  // steps of the earlier tiles
    int xp = 0;  // exchange phases of the earlier tiles (one per step + the row sum)
    for (int t = 0; ok && t < rounds; ++t) {
      Tile tl;
      if (!tile_at(t, tl)) continue;
      const int q0 = tl.q0, nkv = tl.nkv;
      const int q_idx = q0 + r;
      if (nkv == 0) {
        // every key is masked for these rows (only when Sq > Sk): O = 0, LSE = +inf
        if (q_idx < Sq) {
          T* orow = out + (((size_t)tl.b * Sq + q_idx) * H + tl.h) * D + cq * EC;
          if (o_cols)
            for (int c = 0; c < EC; c += 8) *reinterpret_cast<uint4*>(orow + c) = make_uint4(0, 0, 0, 0);
          if (lse != nullptr && cq == 0) lse[(size_t)tl.bh * Sq + q_idx] = __int_as_float(0x7f800000);
        }
        continue;
      }
      float m_run = NEG_INF;  // running max, already multiplied by scale*log2(e)
      float l_run = 0.f;      // this warp's share of the row sum
      // stage(j): S of step j into registers (its buffer released at once), masked,
      // and this quarter's row max posted to the exchange.  The loop stages step
      // j + 1 right after step j's P values are computed, so the load and the four
      // warps' exchange overlap step j's P store instead of stalling all of them
      // together at the top of the next step.
      auto stage = [&](int j, float (&dst)[QC]) -> bool {
        const int g = gs + j, sb = g & 1;
        if (!mbar_wait(bar(B_SFULL + sb), (uint32_t)(g >> 1) & 1u, wc)) return false;
        if (threadIdx.x == 0) FTRACE(8, g);
        tc_fence_after();
        tmem_ld32(tmem + lane_base + C::COL_S + sb * 128 + cq * QC,
                  *reinterpret_cast<uint32_t(*)[32]>(&dst[0]));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B_SFREE + sb));
        const int kv0 = j * C::BN + cq * QC;
        const bool need_mask = (kv0 + QC > Sk) || (causal && kv0 + QC - 1 > q0 + off);
        if (need_mask) {
          const int lim = min(Sk - kv0, causal ? (q_idx + off - kv0 + 1) : QC);
#pragma unroll
          for (int c = 0; c < QC; ++c)
            if (c >= lim) dst[c] = NEG_INF;
        }
        float mx[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) mx[u] = fmaxf(dst[u], dst[4 + u]);
#pragma unroll
        for (int c = 8; c < QC; c += 8)
#pragma unroll
          for (int u = 0; u < 4; ++u) mx[u] = fmax3(mx[u], dst[c + u], dst[c + 4 + u]);
        float* xs = xch + ((xp + j) & 1) * 512;
        xs[cq * 128 + r] = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        __syncwarp();
        if (lane == 0) mbar_arrive(xbar);
        return true;
      };
      float sv[QC];
      if (!stage(0, sv)) { ok = false; break; }
      for (int j = 0; j < nkv; ++j) {
        const int g = gs + j, sb = g & 1;
        // row max over the four column quarters (posted one iteration earlier)
        if (!mbar_wait(xbar, (uint32_t)(xp + j) & 1u, wc)) { ok = false; break; }
        const float* xs = xch + ((xp + j) & 1) * 512;
        const float mt = fmaxf(fmaxf(xs[r], xs[128 + r]), fmaxf(xs[256 + r], xs[384 + r]));
        const float m_new = fmaxf(m_run, mt * scale_log2);
        // Lazy rescale: keep the old reference max unless the row max grew by > 8
        // (a factor 256 in P), or this is the first finite max of the row.
        float m_use = m_run;
        if (m_new > m_run + 8.0f || (m_run == NEG_INF && m_new != NEG_INF)) m_use = m_new;
        const bool rescale = (m_use != m_run);
        const float alpha = rescale ? ex2(m_run - m_use) : 1.0f;
        const float m_safe = (m_use == NEG_INF) ? 0.f : m_use;
        // p = 2^(s*scale*log2e - m) on packed pairs; one pair in four takes the
        // FMA-pipe exp2 so the MUFU unit and the FMA pipe share the load.
        const uint64_t c2 = f2_pack(scale_log2, scale_log2);
        const uint64_t nm2 = f2_pack(-m_safe, -m_safe);
        uint64_t sum2 = f2_pack(0.f, 0.f);
        uint32_t pp[QC / 2];
#pragma unroll
        for (int k = 0; k < QC / 2; ++k) {
          const uint64_t x2 = f2_fma(f2_pack(sv[2 * k], sv[2 * k + 1]), c2, nm2);
          uint64_t p2;
          if ((k & 3) == 3) {
            p2 = f2_exp2_poly(x2);
          } else {
            float x0, x1;
            f2_unpack(x2, x0, x1);
            p2 = f2_pack(ex2(x0), ex2(x1));
          }
          sum2 = f2_add(sum2, p2);
          float p0, p1;
          f2_unpack(p2, p0, p1);
          pp[k] = Elem<T>::pack2(p0, p1);
        }
        float lsum0, lsum1;
        f2_unpack(sum2, lsum0, lsum1);
        l_run = l_run * alpha + (lsum0 + lsum1);
        if (threadIdx.x == 0) FTRACE(9, g);
        // this step's scores are dead: stage the next step into their registers
        if (j + 1 < nkv && !stage(j + 1, sv)) { ok = false; break; }
        // P_b is free once O += P_b V of step g-2 has read it
        if (g >= 2 && !mbar_wait(bar(B_PFREE + sb), (uint32_t)((g - 2) >> 1) & 1u, wc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        tmem_st16(tmem + lane_base + C::COL_P + sb * 64 + cq * (QC / 2), pp);
        // Rescaling O needs O += P V of step g-1 to have completed (rare: lazy
        // rescale; the first step of a tile overwrites O instead)
        if (j > 0 && __any_sync(0xffffffffu, rescale)) {
          if (!mbar_wait(bar(B_ODONE), (uint32_t)(g - 1) & 1u, wc)) { ok = false; break; }
          tc_fence_after();
          if (o_cols) {
#pragma unroll
            for (int c = 0; c < EC / 16; ++c) {
              uint32_t o[16];
              const uint32_t ta = tmem + lane_base + C::COL_O + cq * EC + c * 16;
              tmem_ld16(ta, o);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st16(ta, o);
            }
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B_PFULL + sb));
        if (threadIdx.x == 0) FTRACE(10, g);
        m_run = m_use;
      }
      if (!ok) break;
      // ---------------------------------------------------------- epilogue
      // A row that saw no finite score (every key masked: only when Sq > Sk)
      // keeps l = 0, i.e. O = 0 and LSE = +inf; the FMA-pipe exp2 returns 2^-125,
      // not 0, for masked scores, which only rows with a finite score may absorb.
      if (m_run == NEG_INF) l_run = 0.f;
      // the full row sum: the four column quarters' shares
      {
        float* xs = xch + ((xp + nkv) & 1) * 512;
        xs[cq * 128 + r] = l_run;
        __syncwarp();
        if (lane == 0) mbar_arrive(xbar);
        if (!mbar_wait(xbar, (uint32_t)(xp + nkv) & 1u, wc)) { ok = false; break; }
        l_run = (xs[r] + xs[128 + r]) + (xs[256 + r] + xs[384 + r]);
      }
      // Wait for the tile's last O += P V.  Its P-buffer barrier is unambiguous
      // here (this thread observed that buffer's previous phase), unlike the
      // every-PV ODONE barrier, which may still be two phases behind; a commit
      // covers all of the issuing thread's earlier MMAs.
      const int gl = gs + nkv - 1;
      if (!mbar_wait(bar(B_PFREE + (gl & 1)), (uint32_t)(gl >> 1) & 1u, wc)) { ok = false; break; }
      tc_fence_after();
      const float inv_l = l_run > 0.f ? 1.0f / l_run : 0.f;
      if (o_cols) {
        const bool row_ok = q_idx < Sq;
        T* orow = out + (((size_t)tl.b * Sq + q_idx) * H + tl.h) * D + cq * EC;
#pragma unroll
        for (int c = 0; c < EC / 16; ++c) {
          uint32_t o[16];
          tmem_ld16(tmem + lane_base + C::COL_O + cq * EC + c * 16, o);
          tmem_wait_ld();
          uint4 w0, w1;
          w0.x = Elem<T>::pack2(__uint_as_float(o[0]) * inv_l, __uint_as_float(o[1]) * inv_l);
          w0.y = Elem<T>::pack2(__uint_as_float(o[2]) * inv_l, __uint_as_float(o[3]) * inv_l);
          w0.z = Elem<T>::pack2(__uint_as_float(o[4]) * inv_l, __uint_as_float(o[5]) * inv_l);
          w0.w = Elem<T>::pack2(__uint_as_float(o[6]) * inv_l, __uint_as_float(o[7]) * inv_l);
          w1.x = Elem<T>::pack2(__uint_as_float(o[8]) * inv_l, __uint_as_float(o[9]) * inv_l);
          w1.y = Elem<T>::pack2(__uint_as_float(o[10]) * inv_l, __uint_as_float(o[11]) * inv_l);
          w1.z = Elem<T>::pack2(__uint_as_float(o[12]) * inv_l, __uint_as_float(o[13]) * inv_l);
          w1.w = Elem<T>::pack2(__uint_as_float(o[14]) * inv_l, __uint_as_float(o[15]) * inv_l);
          if (row_ok) {
            reinterpret_cast<uint4*>(orow + c * 16)[0] = w0;
            reinterpret_cast<uint4*>(orow + c * 16)[1] = w1;
          }
        }
      }
      // O has been read: the next tile's first O += P V may overwrite it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_OFREE));
      if (lse != nullptr && q_idx < Sq && cq == 0) {
        const float m_safe = (m_run == NEG_INF) ? 0.f : m_run;
        lse[(size_t)tl.bh * Sq + q_idx] =
            l_run > 0.f ? (m_safe + lg2(l_run)) * 0.69314718055994530942f : __int_as_float(0x7f800000);
      }
      gs += nkv;
      xp += nkv + 1;
    }
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 17) {
    if (lane == 0) mbar_wait_drain(bar(B_DRAIN), 0, timeout_ns);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
    if (lane == 0) CTRACE(3);
  }
}

template <int D, typename T>
static int launch_fwd_d(const FwdArgs& a, cudaStream_t stream) {
  using C = FwdCfg<D>;
  constexpr int tag = D + (std::is_same<T, __half>::value ? 0 : 1000);
  if (!smem_attr_set<tag>(reinterpret_cast<const void*>(fa_fwd_kernel<D, T>), C::SMEM))
    return FA_ERR_LAUNCH;
  const int ntiles = a.B * a.H * ((a.Sq + C::BM - 1) / C::BM);
  const int nsm = sm_count();
  if (nsm <= 0) return FA_ERR_DEVICE;
  const int g =
      tile_grid(ntiles, nsm, persist_max_tiles(a.causal != 0, a.Sq > a.Sk ? a.Sq : a.Sk));
  dim3 grid(g);
  const cudaError_t e = launch_pdl(fa_fwd_kernel<D, T>, grid, dim3(C::THREADS), C::SMEM, stream,
                                   *a.tm_q, *a.tm_k, *a.tm_v, static_cast<T*>(a.o), a.lse,
                                   a.Sq, a.Sk, a.H, a.H / a.Hkv, ntiles, tile_window(ntiles, g),
                                   a.scale * 1.4426950408889634f,
                                   a.causal,
                                   a.status, a.timeout_ns, a.debug_flags);
  return e == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

template <typename T>
static int launch_fwd_t(const FwdArgs& a, cudaStream_t stream) {
  switch (a.D) {
    case 16: return launch_fwd_d<16, T>(a, stream);
    case 32: return launch_fwd_d<32, T>(a, stream);
    case 64: return launch_fwd_d<64, T>(a, stream);
    case 128: return launch_fwd_d<128, T>(a, stream);
    default: return FA_ERR_ARG;
  }
}

int launch_fwd(const FwdArgs& a, cudaStream_t stream) {
  return a.dtype == FA_DTYPE_BF16 ? launch_fwd_t<__nv_bfloat16>(a, stream)
                                  : launch_fwd_t<__half>(a, stream);
}

}  // namespace fa_sm100

#ifdef FA_FWD_TRACE
extern "C" int fa_debug_trace_fwd(void* dst) {
  return (int)cudaMemcpyFromSymbol(dst, fa_sm100::g_ftrace, sizeof(fa_sm100::g_ftrace));
}
extern "C" int fa_debug_trace_fwd_cta(void* dst) {
  return (int)cudaMemcpyFromSymbol(dst, fa_sm100::g_fcta, sizeof(fa_sm100::g_fcta));
}
#endif
