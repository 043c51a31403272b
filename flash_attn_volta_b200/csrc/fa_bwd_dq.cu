// dQ of the attention backward, one CTA per 128-row query tile (sm_100a).
//
// Replaces the reference's dQ kernel _fa_bwd_dq_kernel_d64 / _d128
// (flash_attn_volta/triton_fa_bwd.py:73-307): for a block of query rows it
// walks the key blocks in ascending order, recomputes
//   P  = exp(scale * Q K^T - LSE)                 (triton_fa_bwd.py:123-165)
//   dP = dO V^T,  dS = P (dP - delta)              (:169-172)
// and accumulates dQ += dS K, so dQ = scale * dQ at the end (:176-178).  As in
// the reference there are no atomics: every dQ row is summed by one CTA in a
// fixed order, so dQ is bit-reproducible.  The main backward kernel
// (fa_bwd_main_kernel<D, T, false>) computes dK and dV next to it.
//
// One persistent CTA per SM walks a list of query tiles (longest first under a
// causal mask, snake order over the rounds, like the forward).  Tensor memory
// (512 columns): S [0,128) and dP [128,256) (fp32, one buffer each: the
// dS warps copy all of their columns to registers and release them at once, so the next
// key block's S and dP MMAs run during the math), dS [256,384) as element-type
// pairs in two buffers of 64 columns (the A operand of dQ += dS K), dQ
// [384, 384+D).  Warp roles (G = kDqColGroups):
//   warps 0..4G-1  dS: warp w owns TMEM lane quarter w % 4 (query rows
//              32*(w%4)..) and key-column group w / 4 (128 / G columns).  The
//              row's LSE and delta are per-thread scalars.  Epilogue: dQ *
//              scale -> (B, S, H, D).
//   warp 4G    TMA producers: lane 0 Q and dO of each tile, then the K ring;
//              lane 1 the V ring.
//   warp 4G+1  S = Q K^T and dP = dO V^T (both operands in shared memory).
//   warp 4G+2  dQ += dS K (dS from tensor memory, K from shared memory).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <type_traits>

#include "fa_kernels.h"
#include "sm100_ptx.cuh"

namespace fa_sm100 {

// dS warps: 4 x kDqColGroups (each a TMEM lane quarter x 128 / kDqColGroups key columns)
#ifndef FA_DQ_COL_GROUPS
#define FA_DQ_COL_GROUPS 2
#endif
constexpr int kDqColGroups = FA_DQ_COL_GROUPS;
constexpr int kDqSoftWarps = 4 * kDqColGroups;
#ifndef FA_DQ_NSTK_SMALL
#define FA_DQ_NSTK_SMALL 3
#endif


template <int D>
struct DqCfg {
  static constexpr int BM = 128, BN = 128;                  // query rows, key rows per step
  static constexpr int SWB = (D * 2 >= 128) ? 128 : D * 2;  // swizzle width (bytes)
  static constexpr int AE = SWB / 2;
  static constexpr int NAT = D / AE;
  // K ring depth.  A K stage is read twice, by S of its block and by dQ += dS K,
  // which runs only after that block's dS: with two stages the load of block
  // j + 2 waited for dQ(j) and its latency stalled S(j + 2) (measured at D=128:
  // 3 stages took the deterministic backward 16.0 -> 15.1 ms at B=8, S=8192,
  // H=32 and 138 -> 126 us at B=1, S=4096, H=8).
  static constexpr int NSTK = (D == 128) ? 3 : FA_DQ_NSTK_SMALL;
  static constexpr int NSTV = (D == 128) ? 2 : 3;  // V ring depth
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_DO = OFF_Q + Q_BYTES;
  static constexpr int OFF_K = OFF_DO + Q_BYTES;
  static constexpr int OFF_V = OFF_K + NSTK * KV_BYTES;
  static constexpr int OFF_BAR = OFF_V + NSTV * KV_BYTES;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;  // barriers, TMEM slot, abort flag + slack
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(NSTK <= 5 && NSTV <= 3, "barrier slots of the K / V rings");
  static constexpr int THREADS = (kDqSoftWarps + 3) * 32;  // + TMA, S/dP issuer, dQ issuer
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t COL_S = 0, COL_DP = 128, COL_DS = 256, COL_DQ = 384;
};

enum DqBar {
  Q_FULL = 0,
  Q_EMPTY = 1,   // a tile's last S and dP MMAs have read Q and dO
  K_FULL = 2,    // +NSTK (<= 5)
  K_EMPTY = 7,   // +NSTK: dQ += dS K of that block done
  V_FULL = 12,   // +NSTV (<= 3)
  V_EMPTY = 15,  // +NSTV
  S_FULL = 18,   // S and dP of a key block complete
  S_FREE = 19,   // all dS warps: S and dP copied to registers
  DS_FULL = 20,  // +b, all dS warps: dS_b written
  DS_FREE = 22,  // +b: dQ += dS_b K done reading dS_b
  DQ_DONE = 24,  // a tile's last dQ MMA complete
  DQ_FREE = 25,  // all dS warps: the epilogue has read dQ
  DQ_DRAIN = 26, // 2 arrivals: each issuer's last commit
  DQ_BAR_COUNT = 27
};

template <int D, typename T>
__global__ void __launch_bounds__((kDqSoftWarps + 3) * 32, 1)
    fa_bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_do,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const float* __restrict__ lse,
                     const float* __restrict__ delta, T* __restrict__ dq, int Sq, int Sk, int H,
                     int group, int S_pad, int ntiles, int win, float scale, float scale_log2,
                     int causal, int* status, unsigned long long timeout_ns) {
  using C = DqCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto bar = [&](int i) -> uint32_t { return bar0 + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + 8 * DQ_BAR_COUNT);
  volatile int* abort_flag =
      reinterpret_cast<volatile int*>(smem + C::OFF_BAR + 8 * DQ_BAR_COUNT + 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Tile list as in the forward: (window of `win` heads, query block rank,
  // head), the longest causal block first; round t gives this CTA tile
  // t * grid + pos, pos mirrored on odd rounds.
  const int nblk = (Sq + C::BM - 1) / C::BM;
  const int rounds = (ntiles + (int)gridDim.x - 1) / (int)gridDim.x;
  const int off = Sk - Sq;  // causal mask aligned to the bottom-right
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
    tl.hk = tl.h / group;
    tl.q0 = qt * C::BM;
    tl.nkv = causal ? max(0, min(nkv_all, (tl.q0 + C::BM + off + C::BN - 1) / C::BN)) : nkv_all;
    return true;
  };

  WaitCtx wc{abort_flag, status, timeout_ns};
  if (threadIdx.x == 0) {
    for (int i = 0; i < DQ_BAR_COUNT; ++i) {
      uint32_t cnt = 1;
      if (i == S_FREE || i == DS_FULL || i == DS_FULL + 1 || i == DQ_FREE) cnt = kDqSoftWarps;
      if (i == DQ_DRAIN) cnt = 2;
      mbar_init(bar(i), cnt);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kDqSoftWarps + 1) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // LSE comes from the forward, delta from fa_bwd_pre (both before the main
  // backward kernel, the predecessor of this one)
  griddep_wait();
  griddep_launch_dependents();

  if (warp == kDqSoftWarps) {
    // ------------------------------------------------------------ TMA producers
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_do);
      tma_prefetch_desc(&tm_k);
      int loaded = 0, nq = 0, gs = 0;
      bool ok = true;
      for (int t = 0; ok && t < rounds; ++t) {
        Tile tl;
        if (!tile_at(t, tl) || tl.nkv == 0) continue;
        if (nq > 0 && !mbar_wait(bar(Q_EMPTY), (uint32_t)(nq - 1) & 1u, wc)) break;
        mbar_arrive_expect_tx(bar(Q_FULL), 2 * C::Q_BYTES);
        for (int a = 0; a < C::NAT; ++a) {
          tma_load_4d(sbase + C::OFF_Q + a * C::BM * C::SWB, &tm_q, bar(Q_FULL), a * C::AE, tl.q0,
                      tl.h, tl.b);
          tma_load_4d(sbase + C::OFF_DO + a * C::BM * C::SWB, &tm_do, bar(Q_FULL), a * C::AE,
                      tl.q0, tl.h, tl.b);
        }
        ++nq;
        for (int j = 0; j < tl.nkv; ++j) {
          const int g = gs + j, sk = g % C::NSTK;
          if (g >= C::NSTK &&
              !mbar_wait(bar(K_EMPTY + sk), (uint32_t)(g / C::NSTK - 1) & 1u, wc)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar(K_FULL + sk), C::KV_BYTES);
          for (int a = 0; a < C::NAT; ++a)
            tma_load_4d(sbase + C::OFF_K + sk * C::KV_BYTES + a * C::BN * C::SWB, &tm_k,
                        bar(K_FULL + sk), a * C::AE, j * C::BN, tl.hk, tl.b);
          loaded = g + 1;
        }
        gs += tl.nkv;
      }
      if (*abort_flag) {
        if (nq > 0) mbar_wait_drain(bar(Q_FULL), (uint32_t)(nq - 1) & 1u, timeout_ns);
        for (int g = max(0, loaded - C::NSTK); g < loaded; ++g)
          mbar_wait_drain(bar(K_FULL + g % C::NSTK), (uint32_t)(g / C::NSTK) & 1u, timeout_ns);
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
              !mbar_wait(bar(V_EMPTY + sv), (uint32_t)(g / C::NSTV - 1) & 1u, wc)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar(V_FULL + sv), C::KV_BYTES);
          for (int a = 0; a < C::NAT; ++a)
            tma_load_4d(sbase + C::OFF_V + sv * C::KV_BYTES + a * C::BN * C::SWB, &tm_v,
                        bar(V_FULL + sv), a * C::AE, j * C::BN, tl.hk, tl.b);
          loaded = g + 1;
        }
        gs += tl.nkv;
      }
      if (*abort_flag) {
        for (int g = max(0, loaded - C::NSTV); g < loaded; ++g)
          mbar_wait_drain(bar(V_FULL + g % C::NSTV), (uint32_t)(g / C::NSTV) & 1u, timeout_ns);
      }
    }
  } else if (warp == kDqSoftWarps + 1) {
    // ------------------------------------------------------------ S / dP issuer
    if (lane == 0) {
      constexpr uint32_t swz = swizzle_field(C::SWB);
      constexpr uint32_t id_s = make_idesc_f16(C::BM, C::BN, false, false) | Elem<T>::kIdescAB;
      bool ok = true;
      int gs = 0, nq = 0;
      for (int t = 0; ok && t < rounds; ++t) {
        Tile tl;
        if (!tile_at(t, tl) || tl.nkv == 0) continue;
        if (!mbar_wait(bar(Q_FULL), (uint32_t)nq & 1u, wc)) break;
        for (int j = 0; j < tl.nkv; ++j) {
          const int g = gs + j, sk = g % C::NSTK, sv = g % C::NSTV;
          if (!mbar_wait(bar(K_FULL + sk), (uint32_t)(g / C::NSTK) & 1u, wc) ||
              !mbar_wait(bar(V_FULL + sv), (uint32_t)(g / C::NSTV) & 1u, wc) ||
              (g > 0 && !mbar_wait(bar(S_FREE), (uint32_t)(g - 1) & 1u, wc))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int a = (kk * 16) / C::AE;
            const uint32_t koff = (uint32_t)((kk * 16) % C::AE) * 2u;
            const uint64_t qd = make_smem_desc(sbase + C::OFF_Q + a * C::BM * C::SWB + koff, 16,
                                               8 * C::SWB, swz);
            const uint64_t kd = make_smem_desc(
                sbase + C::OFF_K + sk * C::KV_BYTES + a * C::BN * C::SWB + koff, 16, 8 * C::SWB,
                swz);
            mma_f16_ss(tmem + C::COL_S, qd, kd, id_s, kk > 0 ? 1u : 0u);
          }
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int a = (kk * 16) / C::AE;
            const uint32_t koff = (uint32_t)((kk * 16) % C::AE) * 2u;
            const uint64_t dd = make_smem_desc(sbase + C::OFF_DO + a * C::BM * C::SWB + koff, 16,
                                               8 * C::SWB, swz);
            const uint64_t vd = make_smem_desc(
                sbase + C::OFF_V + sv * C::KV_BYTES + a * C::BN * C::SWB + koff, 16, 8 * C::SWB,
                swz);
            mma_f16_ss(tmem + C::COL_DP, dd, vd, id_s, kk > 0 ? 1u : 0u);
          }
          mma_commit(bar(S_FULL));
          mma_commit(bar(V_EMPTY + sv));
        }
        if (!ok) break;
        mma_commit(bar(Q_EMPTY));  // Q and dO may be reloaded for the next tile
        ++nq;
        gs += tl.nkv;
      }
      mma_commit(bar(DQ_DRAIN));  // also on abort: teardown waits for every issued MMA
    }
  } else if (warp == kDqSoftWarps + 2) {
    // ------------------------------------------------------------ dQ issuer
    if (lane == 0) {
      constexpr uint32_t swz = swizzle_field(C::SWB);
      constexpr uint32_t id_dq = make_idesc_f16(C::BM, D, false, true) | Elem<T>::kIdescAB;
      bool ok = true;
      int gs = 0, nt = 0;
      for (int t = 0; ok && t < rounds; ++t) {
        Tile tl;
        if (!tile_at(t, tl) || tl.nkv == 0) continue;
        // the first dQ MMA of a tile overwrites dQ: the previous epilogue must have read it
        if (nt > 0 && !mbar_wait(bar(DQ_FREE), (uint32_t)(nt - 1) & 1u, wc)) break;
        for (int j = 0; j < tl.nkv; ++j) {
          const int g = gs + j, sk = g % C::NSTK, b = g & 1;
          if (!mbar_wait(bar(DS_FULL + b), (uint32_t)(g >> 1) & 1u, wc)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < C::BN / 16; ++kk) {
            const uint64_t kd =
                make_smem_desc(sbase + C::OFF_K + sk * C::KV_BYTES + kk * 16 * C::SWB,
                               C::BN * C::SWB, 8 * C::SWB, swz);
            mma_f16_ts(tmem + C::COL_DQ, tmem + C::COL_DS + b * 64 + kk * 8, kd, id_dq,
                       (j > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(bar(DS_FREE + b));
          mma_commit(bar(K_EMPTY + sk));
        }
        if (!ok) break;
        mma_commit(bar(DQ_DONE));
        ++nt;
        gs += tl.nkv;
      }
      mma_commit(bar(DQ_DRAIN));
    }
  } else if (warp < kDqSoftWarps) {
    // ------------------------------------------------------------ dS warps
    constexpr int CPW = C::BN / kDqColGroups;  // key columns per warp
    constexpr int NCH = CPW / 32;              // 32-column chunks per warp
    const int lq = warp & 3, hf = warp >> 2;
    const int r = lq * 32 + lane;  // query row inside the tile == TMEM lane
    const uint32_t lane_base = (uint32_t)(lq * 32) << 16;
    const int c0 = hf * CPW;       // first key column of this thread
    constexpr int EC = (D / kDqColGroups >= 16) ? D / kDqColGroups : 16;  // dQ epilogue columns per warp
    const float INF = __int_as_float(0x7f800000);
    bool ok = true;
    int gs = 0, nt = 0;
    for (int t = 0; ok && t < rounds; ++t) {
      Tile tl;
      if (!tile_at(t, tl)) continue;
      const int q_idx = tl.q0 + r;
      const bool row_ok = q_idx < Sq;
      T* drow = dq + (((size_t)tl.b * Sq + q_idx) * H + tl.h) * D + hf * EC;
      if (tl.nkv == 0) {
        // no key is visible to this tile (only when Sq > Sk): dQ = 0
        if (row_ok && hf * EC < D)
          for (int c = 0; c < EC; c += 8) *reinterpret_cast<uint4*>(drow + c) = make_uint4(0, 0, 0, 0);
        continue;
      }
      // per-row scalars: LSE in the exp2 domain, and delta
      const float l2 = row_ok ? lse[(size_t)tl.bh * Sq + q_idx] * 1.4426950408889634f : INF;
      const float dl = row_ok ? delta[(size_t)tl.bh * S_pad + q_idx] : 0.f;
      const uint64_t c2 = f2_pack(scale_log2, scale_log2);
      const uint64_t nl2 = f2_pack(-l2, -l2);
      const uint64_t ndl = f2_pack(-dl, -dl);
      for (int j = 0; j < tl.nkv; ++j) {
        const int g = gs + j, b = g & 1;
        if (!mbar_wait(bar(S_FULL), (uint32_t)g & 1u, wc)) { ok = false; break; }
        tc_fence_after();
        const int kv0 = j * C::BN;
        // every (query, key) pair of this block is unmasked
        const bool full = (kv0 + C::BN <= Sk) && (!causal || kv0 + C::BN - 1 <= tl.q0 + off);
        // all of this thread's columns of S and dP into registers, then release
        // them at once (the next key block's S and dP MMAs run during the math)
        uint32_t sr[NCH][32], dr[NCH][32];
#pragma unroll
        for (int cc = 0; cc < NCH; ++cc) {
          tmem_ld32(tmem + lane_base + C::COL_S + c0 + cc * 32, sr[cc]);
          tmem_ld32(tmem + lane_base + C::COL_DP + c0 + cc * 32, dr[cc]);
        }
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(S_FREE));
#pragma unroll
        for (int cc = 0; cc < NCH; ++cc) {
          const int cb = c0 + cc * 32;  // first key column of this chunk
          uint32_t dd[16];
          if (full) {
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              float x0, x1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(sr[cc][2 * k]),
                                       __uint_as_float(sr[cc][2 * k + 1])),
                               c2, nl2),
                        x0, x1);
              const uint64_t p2 = f2_pack(ex2(x0), ex2(x1));
              float d0, d1;
              f2_unpack(f2_mul(p2, f2_add(f2_pack(__uint_as_float(dr[cc][2 * k]),
                                                  __uint_as_float(dr[cc][2 * k + 1])),
                                          ndl)),
                        d0, d1);
              dd[k] = Elem<T>::pack2(d0, d1);
            }
          } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              float d2[2];
#pragma unroll
              for (int u = 0; u < 2; ++u) {
                const int kv = kv0 + cb + 2 * k + u;
                const bool valid = kv < Sk && (!causal || kv <= q_idx + off);
                const float p =
                    valid ? ex2(fmaf(__uint_as_float(sr[cc][2 * k + u]), scale_log2, -l2)) : 0.f;
                d2[u] = p * (__uint_as_float(dr[cc][2 * k + u]) - dl);
              }
              dd[k] = Elem<T>::pack2(d2[0], d2[1]);
            }
          }
          if (cc == 0 && g >= 2 &&
              !mbar_wait(bar(DS_FREE + b), (uint32_t)((g - 2) >> 1) & 1u, wc)) {
            ok = false;
            break;
          }
          tmem_st16(tmem + lane_base + C::COL_DS + b * 64 + cb / 2, dd);
        }
        if (!ok) break;
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(DS_FULL + b));
      }
      if (!ok) break;
      // ---------------------------------------------------------- epilogue
      if (!mbar_wait(bar(DQ_DONE), (uint32_t)nt & 1u, wc)) { ok = false; break; }
      tc_fence_after();
      if (hf * EC < D) {
#pragma unroll
        for (int c = 0; c < EC / 16; ++c) {
          uint32_t v[16];
          tmem_ld16(tmem + lane_base + C::COL_DQ + hf * EC + c * 16, v);
          tmem_wait_ld();
          uint4 w0, w1;
          w0.x = Elem<T>::pack2(__uint_as_float(v[0]) * scale, __uint_as_float(v[1]) * scale);
          w0.y = Elem<T>::pack2(__uint_as_float(v[2]) * scale, __uint_as_float(v[3]) * scale);
          w0.z = Elem<T>::pack2(__uint_as_float(v[4]) * scale, __uint_as_float(v[5]) * scale);
          w0.w = Elem<T>::pack2(__uint_as_float(v[6]) * scale, __uint_as_float(v[7]) * scale);
          w1.x = Elem<T>::pack2(__uint_as_float(v[8]) * scale, __uint_as_float(v[9]) * scale);
          w1.y = Elem<T>::pack2(__uint_as_float(v[10]) * scale, __uint_as_float(v[11]) * scale);
          w1.z = Elem<T>::pack2(__uint_as_float(v[12]) * scale, __uint_as_float(v[13]) * scale);
          w1.w = Elem<T>::pack2(__uint_as_float(v[14]) * scale, __uint_as_float(v[15]) * scale);
          if (row_ok) {
            reinterpret_cast<uint4*>(drow + c * 16)[0] = w0;
            reinterpret_cast<uint4*>(drow + c * 16)[1] = w1;
          }
        }
      }
      // dQ has been read: the next tile's first dQ MMA may overwrite it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(DQ_FREE));
      gs += tl.nkv;
      ++nt;
    }
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == kDqSoftWarps + 1) {
    if (lane == 0) mbar_wait_drain(bar(DQ_DRAIN), 0, timeout_ns);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int D, typename T>
static int launch_dq_d(const BwdArgs& a, cudaStream_t stream) {
  using C = DqCfg<D>;
  constexpr int tag = 3000 + D + (std::is_same<T, __half>::value ? 0 : 1000);
  if (!smem_attr_set<tag>(reinterpret_cast<const void*>(fa_bwd_dq_kernel<D, T>), C::SMEM))
    return FA_ERR_LAUNCH;
  const int ntiles = a.B * a.H * ((a.Sq + C::BM - 1) / C::BM);
  const int nsm = sm_count();
  if (nsm <= 0) return FA_ERR_DEVICE;
  // always persistent (one CTA per SM walking the tile list): measured at
  // B=1, S=8192, H=16, D=128 the grid of one CTA per tile was 7 % slower (the
  // next tile's Q / dO load and first MMAs overlap this tile's last step here)
  const int g = ntiles < nsm ? ntiles : nsm;
  const cudaError_t e = launch_pdl(
      fa_bwd_dq_kernel<D, T>, dim3(g), dim3(C::THREADS), C::SMEM, stream, *a.tm_q128,
      *a.tm_do128, *a.tm_k, *a.tm_v, a.lse, static_cast<const float*>(a.delta),
      static_cast<T*>(a.dq), a.Sq, a.Sk, a.H, a.H / a.Hkv, a.S_pad, ntiles,
      tile_window(ntiles, g), a.scale, a.scale * 1.4426950408889634f, a.causal, a.status,
      a.timeout_ns);
  return e == cudaSuccess ? FA_OK : FA_ERR_LAUNCH;
}

template <typename T>
static int launch_dq_t(const BwdArgs& a, cudaStream_t stream) {
  switch (a.D) {
    case 16: return launch_dq_d<16, T>(a, stream);
    case 32: return launch_dq_d<32, T>(a, stream);
    case 64: return launch_dq_d<64, T>(a, stream);
    case 128: return launch_dq_d<128, T>(a, stream);
    default: return FA_ERR_ARG;
  }
}

int launch_bwd_dq(const BwdArgs& a, cudaStream_t stream) {
  if (a.tm_q128 == nullptr || a.tm_do128 == nullptr || a.delta == nullptr) return FA_ERR_ARG;
  return a.dtype == FA_DTYPE_BF16 ? launch_dq_t<__nv_bfloat16>(a, stream)
                                  : launch_dq_t<__half>(a, stream);
}

}  // namespace fa_sm100
