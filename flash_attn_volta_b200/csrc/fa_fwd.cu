// FlashAttention forward for sm_100a (B200): O = softmax(scale * Q K^T) V and the
// natural-log log-sum-exp per query row.
//
// Replaces the reference's Triton kernels _fa_fwd_kernel_d64 / _d128
// (flash_attn_volta/triton_fa.py:63-284) and the permute/pad work of its host
// wrapper (triton_fa.py:291-397): Q/K/V are read by TMA straight from the
// (B, S, H, D) fp16 tensors (row stride H*D), every head_dim in {16,32,64,128}
// runs natively (no zero padding), and O is written in (B, S, H, D).
//
// One CTA = two 128-row query tiles (t = 0, 1) of one (batch, head) that share
// every K/V tile.  Warp roles:
//   warps 0-7 / 8-15  softmax of tile 0 / tile 1: two warps per row quarter,
//              each owning half of the key columns of its rows (its TMEM lanes);
//              reads S_t from tensor memory, online softmax in
//              the exp2 domain, writes P_t (fp16 pairs) back over S_t in
//              tensor memory, rescales O_t there when the running max grows by
//              more than 2^8 (lazy rescale); final O/l and LSE epilogue.
//   warp 16    TMA producer: both Q tiles once, then K/V tiles through a ring.
//   warps 17,18 MMA issuer of tile 0 / tile 1: S_t = Q_t K_j^T, then, once the
//              softmax warps have written P_t, O_t += P_t V_j with P_t as the
//              tensor-memory A operand.  Tile 1 starts half a period after
//              tile 0, so one tile's MMAs run while the other tile's softmax does.
// Tensor memory (512 columns): S0 [0,128), S1 [128,256), O0 [256,256+D),
// O1 [256+D, 256+2D); P_t occupies the first 64 columns of S_t.
//
// Semantics kept from the reference: top-left causal mask (column > row is
// masked, triton_fa.py:124-126), columns >= S masked (:123), LSE = m + ln(l)
// and +inf for a row with l == 0 (:152-159), rows >= S not stored (:149-150).
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "fa_kernels.h"
#include "sm100_ptx.cuh"

namespace fa_sm100 {

#ifdef FA_FWD_TRACE
#ifndef FA_TRACE_BLOCK
#define FA_TRACE_BLOCK 0
#endif
// Debug build only: clock64() stamps of barrier events of CTA (0, 0), read back
// with fa_debug_trace_fwd().
__device__ unsigned long long g_ftrace[64][16];
#define FTRACE(slot, it)                                                              \
  do {                                                                                \
    if (blockIdx.x == FA_TRACE_BLOCK && (it) < 64) g_ftrace[it][slot] = clock64(); \
  } while (0)
#else
#define FTRACE(slot, it) \
  do {                   \
  } while (0)
#endif

template <int D>
struct FwdCfg {
  static constexpr int BM = 128, BN = 128, NT = 2;  // query tile rows, key tile rows, tiles
  static constexpr int SWB = (D * 2 >= 128) ? 128 : D * 2;  // swizzle width (bytes)
  static constexpr int AE = SWB / 2;                        // elements per swizzle row
  static constexpr int NAT = D / AE;                        // swizzle atoms along D
  static constexpr int NST = (D == 128) ? 2 : 3;            // K/V ring depth
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + NT * Q_BYTES;
  static constexpr int OFF_V = OFF_K + NST * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + NST * KV_BYTES;
  static constexpr int BAR_BYTES = 256;
  static constexpr int OFF_XCH = OFF_BAR + BAR_BYTES;  // row-max / row-sum exchange
  static constexpr int SMEM = OFF_XCH + 2 * 2 * 2 * 128 * 4 + 1024;  // + alignment slack
  static_assert(SMEM <= 232448, "shared memory budget");
  static constexpr int THREADS = 608;
  static constexpr uint32_t TMEM_COLS = 512;
  __host__ __device__ static constexpr uint32_t col_s(int t) { return (uint32_t)t * 128u; }
  __host__ __device__ static constexpr uint32_t col_o(int t) { return 256u + (uint32_t)t * D; }
};

// barrier slots (8 bytes each) inside the barrier block
enum FwdBar {
  B_QFULL = 0,
  B_KFULL = 1,    // +NST (<= 3)
  B_KEMPTY = 4,   // +NST, one commit per active tile
  B_VFULL = 7,    // +NST
  B_VEMPTY = 10,  // +NST, one commit per active tile
  B_SFULL = 13,   // +tile
  B_PFULL = 15,   // +tile, 4 arrivals (softmax warps of the tile)
  B_ODONE = 17,   // +tile
  B_DRAIN = 19,   // 2 arrivals: each issuer's last commit
  B_XCHG = 20,    // +4*tile+quarter: 2 arrivals (the two halves of a row quarter)
  B_COUNT = 28
};

template <int D>
__global__ void __launch_bounds__(608, 1)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, __half* __restrict__ out,
                  float* __restrict__ lse, int S, int H, float scale_log2, int causal, int* status,
                  unsigned long long timeout_ns, int debug_flags) {
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
  // 1-D grid over (head group, tile rank, head): longest blocks first inside
  // each group of heads, K/V of only a few heads live at once (L2 reuse)
  const int nblk = (S + C::NT * C::BM - 1) / (C::NT * C::BM);
  int bh, rank;
  grid_to_tile((int)blockIdx.x, (int)(gridDim.x / nblk), nblk, kHeadGroup, bh, rank);
  const int blk = causal ? (nblk - 1 - rank) : rank;
  const int b = bh / H, h = bh % H;
  const int q0 = blk * C::NT * C::BM;
  const int nkv_all = (S + C::BN - 1) / C::BN;
  int nkv_t[C::NT];
#pragma unroll
  for (int t = 0; t < C::NT; ++t) {
    const int qt = q0 + t * C::BM;
    nkv_t[t] = qt >= S ? 0 : (causal ? min(nkv_all, (qt + C::BM + C::BN - 1) / C::BN) : nkv_all);
  }
  const int n_active = (nkv_t[0] > 0) + (nkv_t[1] > 0);
  const int nkv = max(nkv_t[0], nkv_t[1]);

  WaitCtx wc{abort_flag, status, timeout_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < B_COUNT; ++i) {
      uint32_t cnt = 1;
      if ((i >= B_KEMPTY && i < B_KEMPTY + 3) || (i >= B_VEMPTY && i < B_VEMPTY + 3))
        cnt = (uint32_t)n_active;
      if (i == B_PFULL || i == B_PFULL + 1) cnt = 8;
      if (i >= B_XCHG) cnt = 2;
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

  if (warp == 16) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(bar(B_QFULL), C::NT * C::Q_BYTES);
      for (int t = 0; t < C::NT; ++t)
        for (int a = 0; a < C::NAT; ++a)
          tma_load_4d(sbase + C::OFF_Q + t * C::Q_BYTES + a * C::BM * C::SWB, &tm_q, bar(B_QFULL),
                      a * C::AE, q0 + t * C::BM, h, b);
      int k_last[C::NST], v_last[C::NST];  // last tile index loaded into each stage
      for (int s = 0; s < C::NST; ++s) k_last[s] = v_last[s] = -1;
      for (int j = 0; j < nkv; ++j) {
        const int s = j % C::NST;
        const uint32_t ph = (uint32_t)(j / C::NST) & 1u;
        if (j >= C::NST && !mbar_wait(bar(B_KEMPTY + s), ph ^ 1u, wc)) break;
        mbar_arrive_expect_tx(bar(B_KFULL + s), C::KV_BYTES);
        for (int a = 0; a < C::NAT; ++a)
          tma_load_4d(sbase + C::OFF_K + s * C::KV_BYTES + a * C::BN * C::SWB, &tm_k,
                      bar(B_KFULL + s), a * C::AE, j * C::BN, h, b);
        k_last[s] = j;
        if (j >= C::NST && !mbar_wait(bar(B_VEMPTY + s), ph ^ 1u, wc)) break;
        // test hook (fa_sm100_set_debug_flags bit 0): never load the first V tile,
        // so the MMA issuers' wait for it runs out
        if ((debug_flags & 1) && j == 0) continue;
        mbar_arrive_expect_tx(bar(B_VFULL + s), C::KV_BYTES);
        for (int a = 0; a < C::NAT; ++a)
          tma_load_4d(sbase + C::OFF_V + s * C::KV_BYTES + a * C::BN * C::SWB, &tm_v,
                      bar(B_VFULL + s), a * C::AE, j * C::BN, h, b);
        v_last[s] = j;
      }
      // After an abort, let the loads this CTA issued land before it exits.
      if (*abort_flag) {
        mbar_wait_drain(bar(B_QFULL), 0, timeout_ns);
        for (int s = 0; s < C::NST; ++s) {
          if (k_last[s] >= 0)
            mbar_wait_drain(bar(B_KFULL + s), (uint32_t)(k_last[s] / C::NST) & 1u, timeout_ns);
          if (v_last[s] >= 0)
            mbar_wait_drain(bar(B_VFULL + s), (uint32_t)(v_last[s] / C::NST) & 1u, timeout_ns);
        }
      }
    }
  } else if (warp >= 17) {
    // ------------------------------------------------------------ MMA issuers (one per tile)
    const int t = warp - 17;
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_f16(C::BM, C::BN, false, false);
      constexpr uint32_t idesc_pv = make_idesc_f16(C::BM, D, false, true);
      constexpr uint32_t swz = swizzle_field(C::SWB);
      const uint32_t d_s = tmem + C::col_s(t);
      const uint32_t d_o = tmem + C::col_o(t);
      const uint32_t qb = sbase + C::OFF_Q + t * C::Q_BYTES;
      bool ok = nkv_t[t] > 0 && mbar_wait(bar(B_QFULL), 0, wc);
      for (int j = 0; ok && j < nkv_t[t]; ++j) {
        const int s = j % C::NST;
        const uint32_t ph = (uint32_t)(j / C::NST) & 1u;
        // S_t(j) overwrites the TMEM columns that P_t(j-1) occupies; it is issued
        // by this same thread after O_t += P_t(j-1) V, and tcgen05.mma operations
        // of one thread execute in issue order, so no wait is needed here.
        if (!mbar_wait(bar(B_KFULL + s), ph, wc)) break;
        // Tile 1 starts once tile 0's first softmax is done: the two tiles then run
        // half a period apart, so one tile's MMAs overlap the other's softmax.
        if (t == 1 && j == 0 && nkv_t[0] > 0 && !mbar_wait(bar(B_PFULL + 0), 0u, wc)) break;
        FTRACE(0 + 4 * t, j);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int a = (kk * 16) / C::AE;
          const uint32_t koff = (uint32_t)((kk * 16) % C::AE) * 2u;
          const uint64_t ad =
              make_smem_desc(qb + a * C::BM * C::SWB + koff, 16, 8 * C::SWB, swz);
          const uint64_t bd =
              make_smem_desc(sbase + C::OFF_K + s * C::KV_BYTES + a * C::BN * C::SWB + koff, 16,
                             8 * C::SWB, swz);
          mma_f16_ss(d_s, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        mma_commit(bar(B_SFULL + t));
        mma_commit(bar(B_KEMPTY + s));
        FTRACE(1 + 4 * t, j);
        if (!mbar_wait(bar(B_PFULL + t), (uint32_t)j & 1u, wc) ||
            !mbar_wait(bar(B_VFULL + s), ph, wc))
          break;
        FTRACE(2 + 4 * t, j);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < C::BN / 16; ++kk) {
          const uint64_t bd = make_smem_desc(sbase + C::OFF_V + s * C::KV_BYTES + kk * 16 * C::SWB,
                                             C::BN * C::SWB, 8 * C::SWB, swz);
          mma_f16_ts(d_o, d_s + kk * 8, bd, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(bar(B_ODONE + t));
        mma_commit(bar(B_VEMPTY + s));
        FTRACE(3 + 4 * t, j);
      }
      mma_commit(bar(B_DRAIN));  // also on abort: teardown waits for every issued MMA
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0..15
    // Tile t = warp / 8; inside a tile, warp w owns TMEM lane quarter w % 4 (rows
    // 32*(w%4)..) and half hh of each key tile's 128 columns.  The two halves of a
    // row trade partial row maxima through shared memory every step (a 2-arrival
    // mbarrier per row quarter, bounded wait) and add their row sums at the end.
    const int t = warp >> 3;
    const int hh = (warp >> 2) & 1;
    const int lq = warp & 3;
    const int r = lq * 32 + lane;  // query row inside the tile == TMEM lane
    const int q_tile0 = q0 + t * C::BM;
    const int q_idx = q_tile0 + r;
    const uint32_t lane_base = (uint32_t)(lq * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + C::col_s(t);
    const uint32_t o_addr = tmem + lane_base + C::col_o(t);
    constexpr int HC = C::BN / 2;                   // columns per half
    constexpr int EC = (D / 2 >= 16) ? D / 2 : 16;  // O columns per half
    const bool o_cols = hh * EC < D;
    float* xch = reinterpret_cast<float*>(smem + C::OFF_XCH);  // [2][2 tiles][2 halves][128]
    auto xslot = [&](int par, int half) { return xch + ((par * 2 + t) * 2 + half) * 128 + r; };
    const uint32_t xbar = bar(B_XCHG + t * 4 + lq);
    const float NEG_INF = -__int_as_float(0x7f800000);
    float m_run = NEG_INF;  // running max, already multiplied by scale*log2(e)
    float l_run = 0.f;      // this half's share of the row sum
    bool ok = true;
    const int nk = nkv_t[t];
    for (int j = 0; j < nk; ++j) {
      if (!mbar_wait(bar(B_SFULL + t), (uint32_t)j & 1u, wc)) { ok = false; break; }
      // The two tiles' softmaxes take turns (tile 1's step j after tile 0's step
      // j, tile 0's step j after tile 1's step j-1): each runs alone on the exp2
      // unit while the tensor core works on the other tile.
      if (t == 1 && j < nkv_t[0] && !mbar_wait(bar(B_PFULL + 0), (uint32_t)j & 1u, wc)) {
        ok = false;
        break;
      }
      if (t == 0 && j > 0 && j - 1 < nkv_t[1] &&
          !mbar_wait(bar(B_PFULL + 1), (uint32_t)(j - 1) & 1u, wc)) {
        ok = false;
        break;
      }
      if (r == 0 && hh == 0) FTRACE(8 + 4 * t, j);
      tc_fence_after();
      float sv[HC];
      tmem_ld32(s_addr + hh * HC, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
      tmem_ld32(s_addr + hh * HC + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
      tmem_wait_ld();
      const int kv0 = j * C::BN + hh * HC;
      const bool need_mask = (kv0 + HC > S) || (causal && kv0 + HC - 1 > q_tile0);
      if (need_mask) {
        const int lim = min(S - kv0, causal ? (q_idx - kv0 + 1) : HC);
#pragma unroll
        for (int c = 0; c < HC; ++c)
          if (c >= lim) sv[c] = NEG_INF;
      }
      float mt = fmax3(sv[0], sv[1], sv[2]);
#pragma unroll
      for (int c = 3; c < HC - 1; c += 2) mt = fmax3(mt, sv[c], sv[c + 1]);
      mt = fmaxf(mt, sv[HC - 1]);
      // row max over both halves
      *xslot(j & 1, hh) = mt;
      __syncwarp();
      if (lane == 0) mbar_arrive(xbar);
      if (!mbar_wait(xbar, (uint32_t)j & 1u, wc)) { ok = false; break; }
      mt = fmaxf(mt, *xslot(j & 1, hh ^ 1));
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
      uint32_t pp[HC / 2];
#pragma unroll
      for (int k = 0; k < HC / 2; ++k) {
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
        pp[k] = pack_half2(p0, p1);
      }
      float lsum0, lsum1;
      f2_unpack(sum2, lsum0, lsum1);
      l_run = l_run * alpha + (lsum0 + lsum1);
      if (r == 0 && hh == 0) FTRACE(9 + 4 * t, j);
      // P_t (fp16 pairs) over the first 64 columns of S_t: A operand of O_t += P_t V
      tmem_st32(s_addr + hh * (HC / 2), pp);
      // Rescaling O_t needs O_t += P_t V_{j-1} to have completed (rare: lazy rescale)
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
        if (!mbar_wait(bar(B_ODONE + t), (uint32_t)(j - 1) & 1u, wc)) { ok = false; break; }
        tc_fence_after();
        if (o_cols) {
#pragma unroll
          for (int c = 0; c < EC / 16; ++c) {
            uint32_t o[16];
            const uint32_t ta = o_addr + hh * EC + c * 16;
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
      if (lane == 0) mbar_arrive(bar(B_PFULL + t));
      if (r == 0 && hh == 0) FTRACE(10 + 4 * t, j);
      m_run = m_use;
    }
    // ------------------------------------------------------------ epilogue
    if (ok && nk > 0) {
      // the full row sum: this half's plus the other half's
      *xslot(nk & 1, hh) = l_run;
      __syncwarp();
      if (lane == 0) mbar_arrive(xbar);
      ok = mbar_wait(xbar, (uint32_t)nk & 1u, wc);
      if (ok) l_run += *xslot(nk & 1, hh ^ 1);
    }
    if (ok && nk > 0 && mbar_wait(bar(B_ODONE + t), (uint32_t)(nk - 1) & 1u, wc)) {
      tc_fence_after();
      const float inv_l = l_run > 0.f ? 1.0f / l_run : 0.f;
      const bool row_ok = q_idx < S;
      __half* orow = out + (((size_t)b * S + q_idx) * H + h) * D + hh * EC;
      if (o_cols) {
#pragma unroll
        for (int c = 0; c < EC / 16; ++c) {
          uint32_t o[16];
          tmem_ld16(o_addr + hh * EC + c * 16, o);
          tmem_wait_ld();
          uint4 w0, w1;
          w0.x = pack_half2(__uint_as_float(o[0]) * inv_l, __uint_as_float(o[1]) * inv_l);
          w0.y = pack_half2(__uint_as_float(o[2]) * inv_l, __uint_as_float(o[3]) * inv_l);
          w0.z = pack_half2(__uint_as_float(o[4]) * inv_l, __uint_as_float(o[5]) * inv_l);
          w0.w = pack_half2(__uint_as_float(o[6]) * inv_l, __uint_as_float(o[7]) * inv_l);
          w1.x = pack_half2(__uint_as_float(o[8]) * inv_l, __uint_as_float(o[9]) * inv_l);
          w1.y = pack_half2(__uint_as_float(o[10]) * inv_l, __uint_as_float(o[11]) * inv_l);
          w1.z = pack_half2(__uint_as_float(o[12]) * inv_l, __uint_as_float(o[13]) * inv_l);
          w1.w = pack_half2(__uint_as_float(o[14]) * inv_l, __uint_as_float(o[15]) * inv_l);
          if (row_ok) {
            reinterpret_cast<uint4*>(orow + c * 16)[0] = w0;
            reinterpret_cast<uint4*>(orow + c * 16)[1] = w1;
          }
        }
      }
      if (lse != nullptr && row_ok && hh == 0) {
        const float m_safe = (m_run == NEG_INF) ? 0.f : m_run;
        lse[(size_t)bh * S + q_idx] =
            l_run > 0.f ? (m_safe + lg2(l_run)) * 0.69314718055994530942f : __int_as_float(0x7f800000);
      }
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
  }
}

template <int D>
static int launch_fwd_d(const FwdArgs& a, cudaStream_t stream) {
  using C = FwdCfg<D>;
  if (cudaFuncSetAttribute(fa_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           C::SMEM) != cudaSuccess)
    return FA_ERR_LAUNCH;
  dim3 grid(a.B * a.H * ((a.S + C::NT * C::BM - 1) / (C::NT * C::BM)));
  fa_fwd_kernel<D><<<grid, C::THREADS, C::SMEM, stream>>>(
      *a.tm_q, *a.tm_k, *a.tm_v, static_cast<__half*>(a.o), a.lse, a.S, a.H,
      a.scale * 1.4426950408889634f, a.causal, a.status, a.timeout_ns, a.debug_flags);
  return cudaGetLastError() == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

int launch_fwd(const FwdArgs& a, cudaStream_t stream) {
  switch (a.D) {
    case 16: return launch_fwd_d<16>(a, stream);
    case 32: return launch_fwd_d<32>(a, stream);
    case 64: return launch_fwd_d<64>(a, stream);
    case 128: return launch_fwd_d<128>(a, stream);
    default: return FA_ERR_ARG;
  }
}

}  // namespace fa_sm100

#ifdef FA_FWD_TRACE
#ifndef FA_TRACE_BLOCK
#define FA_TRACE_BLOCK 0
#endif
extern "C" int fa_debug_trace_fwd(void* dst) {
  return (int)cudaMemcpyFromSymbol(dst, fa_sm100::g_ftrace, sizeof(fa_sm100::g_ftrace));
}
#endif
