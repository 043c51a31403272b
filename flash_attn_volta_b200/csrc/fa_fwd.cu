// FlashAttention forward for sm_100a (B200): O = softmax(scale * Q K^T) V and the
// natural-log log-sum-exp per query row.
//
// Replaces the reference's Triton kernels _fa_fwd_kernel_d64 / _d128
// (flash_attn_volta/triton_fa.py:63-284) and the permute/pad work of its host
// wrapper (triton_fa.py:291-397): Q/K/V are read by TMA straight from the
// (B, S, H, D) fp16 tensors (row stride H*D), every head_dim in {16,32,64,128}
// runs natively (no zero padding), and O is written in (B, S, H, D).
//
// One CTA = one 128-row query tile of one (batch, head).  Warp roles:
//   warps 0-3  softmax: thread r owns query row r; reads S from tensor memory,
//              online softmax in the exp2 domain, writes P (fp16) to shared
//              memory, rescales O in tensor memory when the running max grows
//              by more than 2^8 (lazy rescale), final O/l and LSE epilogue.
//   warp 4     TMA producer: Q once, then K/V tiles through an NST-deep ring.
//   warp 5     MMA issuer (one thread): S_j = Q K_j^T into one of two S
//              buffers in tensor memory, then O += P_{j-1} V_{j-1}; S_{j+1} is
//              issued before waiting for P_j so the tensor core overlaps softmax.
// Tensor memory (512 columns): S0 [0,128), S1 [128,256), O [256, 256+D).
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

template <int D>
struct FwdCfg {
  static constexpr int BM = 128, BN = 128;
  static constexpr int SWB = (D * 2 >= 128) ? 128 : D * 2;  // swizzle width (bytes)
  static constexpr int AE = SWB / 2;                        // elements per swizzle row
  static constexpr int NAT = D / AE;                        // swizzle atoms along D
  static constexpr int NST = (D == 128) ? 2 : 3;            // K/V ring depth
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + NST * KV_BYTES;
  static constexpr int OFF_P = OFF_V + NST * KV_BYTES;
  static constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = OFF_BAR + BAR_BYTES + 1024;   // + alignment slack
  static constexpr int THREADS = 192;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t COL_S0 = 0, COL_S1 = 128, COL_O = 256;
};

// barrier slots (8 bytes each) inside the barrier block
enum FwdBar {
  B_QFULL = 0,
  B_KFULL = 1,    // +NST
  B_KEMPTY = 4,   // +NST
  B_VFULL = 7,    // +NST
  B_VEMPTY = 10,  // +NST
  B_SFULL = 13,   // +2
  B_PFULL = 15,   // +2
  B_PFREE = 17,   // +2
  B_ODONE = 19,
  B_DRAIN = 20,   // the MMA issuer's last commit: all its MMAs are complete
  B_COUNT = 21
};

template <int D>
__global__ void __launch_bounds__(192, 1)
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
  const int ntq = gridDim.x;
  const int qt = causal ? (ntq - 1 - (int)blockIdx.x) : (int)blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int q0 = qt * C::BM;
  const int nkv_all = (S + C::BN - 1) / C::BN;
  const int nkv = causal ? min(nkv_all, (q0 + C::BM + C::BN - 1) / C::BN) : nkv_all;

  WaitCtx wc{abort_flag, status, timeout_ns};

  if (threadIdx.x == 0) {
    for (int i = 0; i < B_COUNT; ++i) {
      uint32_t cnt = 1;
      if (i == B_PFULL || i == B_PFULL + 1) cnt = 4;
      mbar_init(bar(i), cnt);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(bar(B_QFULL), C::Q_BYTES);
      for (int a = 0; a < C::NAT; ++a)
        tma_load_4d(sbase + C::OFF_Q + a * C::BM * C::SWB, &tm_q, bar(B_QFULL), a * C::AE, q0, h, b);
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
        // so the MMA issuer's wait for it runs out
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
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_f16(C::BM, C::BN, false, false);
      constexpr uint32_t idesc_pv = make_idesc_f16(C::BM, D, false, true);
      constexpr uint32_t swz = swizzle_field(C::SWB);
      bool ok = mbar_wait(bar(B_QFULL), 0, wc);
      for (int j = 0; ok && j <= nkv; ++j) {
        if (j < nkv) {
          const int s = j % C::NST;
          const int sb = j & 1;
          if (!mbar_wait(bar(B_KFULL + s), (uint32_t)(j / C::NST) & 1u, wc)) { ok = false; break; }
          if (j >= 2 && !mbar_wait(bar(B_PFULL + sb), (uint32_t)((j - 2) >> 1) & 1u, wc)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_s = tmem + (sb ? C::COL_S1 : C::COL_S0);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const int a = (kk * 16) / C::AE;
            const uint32_t koff = (uint32_t)((kk * 16) % C::AE) * 2u;
            const uint64_t ad = make_smem_desc(sbase + C::OFF_Q + a * C::BM * C::SWB + koff, 16,
                                               8 * C::SWB, swz);
            const uint64_t bd =
                make_smem_desc(sbase + C::OFF_K + s * C::KV_BYTES + a * C::BN * C::SWB + koff, 16,
                               8 * C::SWB, swz);
            mma_f16_ss(d_s, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
          }
          mma_commit(bar(B_SFULL + sb));
          mma_commit(bar(B_KEMPTY + s));
        }
        if (j >= 1) {
          const int jp = j - 1;
          const int sp = jp % C::NST;
          const int pb = jp & 1;
          if (!mbar_wait(bar(B_PFULL + pb), (uint32_t)(jp >> 1) & 1u, wc)) { ok = false; break; }
          if (!mbar_wait(bar(B_VFULL + sp), (uint32_t)(jp / C::NST) & 1u, wc)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < C::BN / 16; ++kk) {
            const int a = kk / 4;
            const uint32_t koff = (uint32_t)(kk % 4) * 32u;
            const uint64_t ad =
                make_smem_desc(sbase + C::OFF_P + pb * C::P_BYTES + a * C::BM * 128 + koff, 16,
                               1024, 2);
            const uint64_t bd =
                make_smem_desc(sbase + C::OFF_V + sp * C::KV_BYTES + kk * 16 * C::SWB,
                               C::BN * C::SWB, 8 * C::SWB, swz);
            mma_f16_ss(tmem + C::COL_O, ad, bd, idesc_pv, (jp > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(bar(B_ODONE));
          mma_commit(bar(B_VEMPTY + sp));
          mma_commit(bar(B_PFREE + pb));
        }
      }
      mma_commit(bar(B_DRAIN));  // also on abort: teardown waits for every issued MMA
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0..3
    const int r = warp * 32 + lane;  // query row inside the tile == TMEM lane
    const int q_idx = q0 + r;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const float NEG_INF = -__int_as_float(0x7f800000);
    float m_run = NEG_INF;  // running max, already multiplied by scale*log2(e)
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(bar(B_SFULL + sb), (uint32_t)(j >> 1) & 1u, wc)) { ok = false; break; }
      tc_fence_after();
      float sv[C::BN];
      {
        uint32_t raw[32];
#pragma unroll
        for (int c = 0; c < C::BN / 32; ++c) {
          tmem_ld32(tmem + lane_base + (sb ? C::COL_S1 : C::COL_S0) + c * 32, raw);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[c * 32 + i] = __uint_as_float(raw[i]);
        }
      }
      const int kv0 = j * C::BN;
      const bool need_mask = (kv0 + C::BN > S) || (causal && kv0 + C::BN - 1 > q0);
      if (need_mask) {
        const int lim = min(S - kv0, causal ? (q_idx - kv0 + 1) : C::BN);
#pragma unroll
        for (int c = 0; c < C::BN; ++c)
          if (c >= lim) sv[c] = NEG_INF;
      }
      float mt = sv[0];
#pragma unroll
      for (int c = 1; c < C::BN; ++c) mt = fmaxf(mt, sv[c]);
      const float m_new = fmaxf(m_run, mt * scale_log2);
      // Lazy rescale: keep the old reference max unless the row max grew by > 8
      // (a factor 256 in P), or this is the first finite max of the row.
      float m_use = m_run;
      if (m_new > m_run + 8.0f || (m_run == NEG_INF && m_new != NEG_INF)) m_use = m_new;
      const bool rescale = (m_use != m_run);
      const float alpha = rescale ? ex2(m_run - m_use) : 1.0f;
      const float m_safe = (m_use == NEG_INF) ? 0.f : m_use;
      float lsum = 0.f;
#pragma unroll
      for (int c = 0; c < C::BN; ++c) {
        sv[c] = ex2(fmaf(sv[c], scale_log2, -m_safe));
        lsum += sv[c];
      }
      l_run = l_run * alpha + lsum;
      if (j >= 2 && !mbar_wait(bar(B_PFREE + sb), (uint32_t)((j - 2) >> 1) & 1u, wc)) {
        ok = false;
        break;
      }
      // P row -> shared memory, K-major 128B-swizzled, two 64-column atoms
      const uint32_t pbase = sbase + C::OFF_P + sb * C::P_BYTES;
#pragma unroll
      for (int a = 0; a < 2; ++a) {
#pragma unroll
        for (int ch = 0; ch < 8; ++ch) {
          const int c = a * 64 + ch * 8;
          st_shared_v4(pbase + a * C::BM * 128 + sw128_offset(r, ch), pack_half2(sv[c], sv[c + 1]),
                       pack_half2(sv[c + 2], sv[c + 3]), pack_half2(sv[c + 4], sv[c + 5]),
                       pack_half2(sv[c + 6], sv[c + 7]));
        }
      }
      fence_proxy_async_smem();
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
        if (!mbar_wait(bar(B_ODONE), (uint32_t)(j - 1) & 1u, wc)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 16; ++c) {
          uint32_t o[16];
          const uint32_t ta = tmem + lane_base + C::COL_O + c * 16;
          tmem_ld16(ta, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st16(ta, o);
        }
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(B_PFULL + sb));
      m_run = m_use;
    }
    // ------------------------------------------------------------ epilogue
    if (ok && nkv > 0 && mbar_wait(bar(B_ODONE), (uint32_t)(nkv - 1) & 1u, wc)) {
      tc_fence_after();
      const float inv_l = l_run > 0.f ? 1.0f / l_run : 0.f;
      const bool row_ok = q_idx < S;
      __half* orow = out + (((size_t)b * S + q_idx) * H + h) * D;
#pragma unroll
      for (int c = 0; c < D / 16; ++c) {
        uint32_t o[16];
        tmem_ld16(tmem + lane_base + C::COL_O + c * 16, o);
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
      if (lse != nullptr && row_ok) {
        const float m_safe = (m_run == NEG_INF) ? 0.f : m_run;
        lse[(size_t)bh * S + q_idx] =
            l_run > 0.f ? (m_safe + lg2(l_run)) * 0.69314718055994530942f : __int_as_float(0x7f800000);
      }
    }
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
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
  dim3 grid((a.S + C::BM - 1) / C::BM, a.B * a.H);
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
