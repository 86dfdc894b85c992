// fa_fwd.cuh -- FlashAttention-2 forward for sm_100a.
//
// Replaces flash::fwd_kernel / flash::launch (reference flash_fwd.cuh:68-355).
// Same math: O = softmax(scale * Q K^T + mask) V with the scale applied to the
// fp32 logit (flash_fwd.cuh:94-103, :220-224), causal and ragged-tail columns
// masked to -inf (:226-243), blocks wholly above the diagonal never visited
// (:127-130), LSE = m + ln(l) in natural log (:321-330), GQA head mapping
// kv_head = q_head / group (:87-92).
//
// Two kernels, chosen by grid size (launch_forward): fwd_kernel_p
// (fa_fwd_persist.cuh), two 128-row query tiles per item and one persistent
// CTA per SM walking the items, when B*Hq*ceil(N/256) fills the GPU;
// fwd_kernel_s (below) with one CTA per 128 rows and 256-key steps when it
// would not. This file holds their shared parameters and MMA issue helpers.
#pragma once
#include "sm100.cuh"

namespace fab {

struct FwdParams {
  uint16_t* o;      // (B, Hq, N, D) fp16 or bf16, strides `so` (D contiguous)
  Strides so;
  float* lse;       // (B*Hq, N), natural log
  int* err;         // device error word
  int n;            // sequence length
  int hq;           // query heads
  int group;        // hq / hkv
  int causal;
  int n_mblocks;    // m-blocks of the launched kernel: ceil(N / 256), or ceil(N / 128)
                    // for the small-grid kernel
  float scale_log2; // softmax scale * log2(e)
  int n_items;      // persistent kernel: B*Hq*n_mblocks (batch, head, m-block) items
  int bh_count;     // B*Hq
};

}  // namespace fab

namespace fab {

// ---------------------------------------------------------------------------
// MMA issue helpers (single thread)
// ---------------------------------------------------------------------------
// S[tmem] = Q_tile (128 x D, K-major) * K_tile^T (128 x D, K-major)
template <int D, bool BF>
__device__ __forceinline__ void issue_qk(uint32_t d_tmem, uint32_t q_s, uint32_t k_s) {
  constexpr uint32_t idesc = idesc_f16(128, 128, false, false, BF);
  const uint64_t dq = sdesc_sw128(q_s, 16, 1024), dk = sdesc_sw128(k_s, 16, 1024);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
    mma_ss(d_tmem, sdesc_add(dq, off), sdesc_add(dk, off), idesc, kk > 0 ? 1u : 0u);
  }
}
// O[tmem] (+)= P (128 x keys [16*KK0, 16*KK1), fp16 pairs in TMEM) * V (those keys x D,
// MN-major)
template <int D, bool BF, int KK0 = 0, int KK1 = 8>
__device__ __forceinline__ void issue_pv(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_s,
                                         bool accumulate) {
  constexpr uint32_t idesc = idesc_f16(128, D, false, true, BF);
  const uint64_t dv = sdesc_sw128(v_s, 16384, 1024);
#pragma unroll
  for (int kk = KK0; kk < KK1; ++kk)
    mma_ts(d_tmem, p_tmem + kk * 8, sdesc_add(dv, kk * 2048), idesc,
           (accumulate || kk > 0) ? 1u : 0u);
}

}  // namespace fab

namespace fab {

// ---------------------------------------------------------------------------
// Small-grid forward: one CTA per 128 query rows (twice the CTAs of the
// two-tile kernel, for grids that would leave SMs idle), keys in steps of 256:
//   warps 0-7   softmax: each warp owns 16 rows; lanes i and i+16 hold keys
//               0..127 and 128..255 of row i's step (TMEM shape 16x32bx2)
//   warp  8     TMEM allocation + MMA issue;  warp 9  TMA loads
// TMEM: S [0,256) fp32 | P [256,384) fp16 pairs of the step's 256 keys | O [384, 384+D).
// P has columns of its own, so S of step j+1 (one N = 256 MMA) is issued as soon
// as the softmax has read S of step j and runs while its exponentials do;
// O += P V (A from TMEM) once P is stored, and P is rewritten only after that
// product has completed. Shared memory: Q, two K steps, one V step.
// ---------------------------------------------------------------------------
template <int D>
struct FwdCfgS {
  static constexpr int BM = 128;                // query rows per CTA
  static constexpr int BN = 256;                // keys per step (one S MMA of N = 256)
  static constexpr int CH = D / 64;             // 64-column chunks per row
  static constexpr int QBYTES = BM * D * 2;
  static constexpr int KVBYTES = BN * D * 2;    // one step of K or V: [chunk][256 rows][128 B]
  static constexpr int CHUNK = BN * 128;        // bytes of one 64-column chunk of a step tile
  static constexpr int KS = 2, VS = 1;          // K steps / V steps resident
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_RING = OFF_Q + QBYTES;
  static constexpr int OFF_BAR = OFF_RING + (KS + VS) * KVBYTES;
  // barriers: q, full[KS+VS], empty[KS+VS], s, sfree, p[2], pv, o
  static constexpr int NBAR = 1 + 2 * (KS + VS) + 6;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16;   // window must start 1024-aligned
  static_assert(SMEM <= 232448, "shared memory over the per-block limit");
  static constexpr int THREADS = 320;
  static constexpr int MMA_WARP = 8, TMA_WARP = 9;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t COL_S = 0, COL_P = 256, COL_O = 384;
};

}  // namespace fab

namespace fab {

// S[tmem] = Q (128 x D, K-major) * K_step^T (256 x D, K-major): N = 256
template <int D, bool BF>
__device__ __forceinline__ void issue_qk256(uint32_t d_tmem, uint32_t q_s, uint32_t k_s) {
  using C = FwdCfgS<D>;
  constexpr uint32_t idesc = idesc_f16(128, 256, false, false, BF);
  const uint64_t dq = sdesc_sw128(q_s, 16, 1024), dk = sdesc_sw128(k_s, 16, 1024);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk)
    mma_ss(d_tmem, sdesc_add(dq, (kk >> 2) * 16384 + (kk & 3) * 32),
           sdesc_add(dk, (kk >> 2) * C::CHUNK + (kk & 3) * 32), idesc, kk > 0 ? 1u : 0u);
}
// O[tmem] (+)= P (128 x keys [16*KK0, 16*KK1) of the step, fp16 pairs in TMEM) * V_step
// (those keys x D, MN-major)
template <int D, bool BF, int KK0, int KK1>
__device__ __forceinline__ void issue_pv256(uint32_t d_tmem, uint32_t p_tmem, uint32_t v_s,
                                         bool accumulate) {
  using C = FwdCfgS<D>;
  constexpr uint32_t idesc = idesc_f16(128, D, false, true, BF);
  const uint64_t dv = sdesc_sw128(v_s, C::CHUNK, 1024);
#pragma unroll
  for (int kk = KK0; kk < KK1; ++kk)
    mma_ts(d_tmem, p_tmem + kk * 8, sdesc_add(dv, kk * 2048), idesc,
           (accumulate || kk > 0) ? 1u : 0u);
}

template <int D, bool BF>
__global__ void __launch_bounds__(320, 1)
    fwd_kernel_s(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
               const FwdParams p) {
  using C = FwdCfgS<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (!smem_aligned_or_report(smem_raw, p.err)) return;
  const uint32_t sbase = smem_u32(smem_raw);
  const uint32_t s_q = sbase + C::OFF_Q, s_ring = sbase + C::OFF_RING;
  const uint32_t b_q = sbase + C::OFF_BAR;
  const uint32_t b_full = b_q + 8, b_empty = b_full + 8 * (C::KS + C::VS);
  // b_p + 8k: keys 128k .. 128k+127 of the step's P are in TMEM
  const uint32_t b_s = b_empty + 8 * (C::KS + C::VS), b_sfree = b_s + 8, b_p = b_sfree + 8,
                 b_pv = b_p + 16, b_o = b_pv + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem_raw + C::OFF_BAR + C::NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid (B*Hq, 128-row m-blocks): every head's longest causal rows first
  const int bh = blockIdx.x;
  const int mb = p.n_mblocks - 1 - static_cast<int>(blockIdx.y);
  const int m0 = mb * C::BM;
  const int b_i = bh / p.hq, hq_i = bh % p.hq, hk_i = hq_i / p.group;
  // keys [0, kend): causal rows see keys up to their own row
  const int kend = p.causal ? min(p.n, m0 + C::BM) : p.n;
  const int nstep = (kend + C::BN - 1) / C::BN;
  const Ctl ctl{abort_flag, p.err};
  auto k_slot = [](int j) { return j % C::KS; };
  auto k_ph = [](int j) { return static_cast<uint32_t>((j / C::KS) & 1); };
  auto v_slot = [](int j) { return C::KS + j % C::VS; };
  auto v_ph = [](int j) { return static_cast<uint32_t>((j / C::VS) & 1); };

  if (threadIdx.x == 0) {
    mbar_init(b_q, 1);
    for (int s = 0; s < C::KS + C::VS; ++s) {
      mbar_init(b_full + 8 * s, 1);
      mbar_init(b_empty + 8 * s, 1);
    }
    mbar_init(b_s, 1);
    mbar_init(b_sfree, 256);
    mbar_init(b_p, 256);
    mbar_init(b_p + 8, 256);
    mbar_init(b_pv, 1);
    mbar_init(b_o, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == C::MMA_WARP) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == C::TMA_WARP) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(b_q, C::QBYTES);
#pragma unroll
      for (int c = 0; c < C::CH; ++c) tma_load_4d(s_q + c * 16384, &tm_q, b_q, c * 64, m0, hq_i, b_i);
      bool ok = true;
      int nk = 0, nv = 0;
      // one step of K (kind 0) or V (kind 1): 256 keys as two 128-row boxes per chunk
      auto issue_step = [&](int kind, int j) -> bool {
        const int slot = kind ? v_slot(j) : k_slot(j);
        const uint32_t ph = kind ? v_ph(j) : k_ph(j);
        if (!mbar_wait(b_empty + 8 * slot, ph ^ 1, ctl, kErrTimeoutLoad)) return false;
        const uint32_t fb = b_full + 8 * slot;
        mbar_arrive_expect_tx(fb, C::KVBYTES);
        const uint32_t dst = s_ring + slot * C::KVBYTES;
#pragma unroll
        for (int c = 0; c < C::CH; ++c)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            tma_load_4d(dst + c * C::CHUNK + h * 16384, kind ? (const void*)&tm_v : (const void*)&tm_k,
                        fb, c * 64, j * C::BN + 128 * h, hk_i, b_i);
        if (kind) ++nv; else ++nk;
        return true;
      };
      constexpr int kAhead = 1;  // L2 prefetch distance, in steps
      auto prefetch = [&](int j) {
        for (int c = 0; c < C::CH; ++c)
          for (int h = 0; h < 2; ++h) {
            tma_prefetch_l2_4d(&tm_k, c * 64, j * C::BN + 128 * h, hk_i, b_i);
            tma_prefetch_l2_4d(&tm_v, c * 64, j * C::BN + 128 * h, hk_i, b_i);
          }
      };
      for (int j = 0; j < kAhead && j < nstep; ++j) prefetch(j);
      // K runs one step ahead of V: K_0, then K_{j+1} before V_j
      for (int j = 0; j < nstep && ok; ++j) {
        if (j + kAhead < nstep) prefetch(j + kAhead);
        if (j == 0) ok = issue_step(0, 0);
        if (ok && j + 1 < nstep) ok = issue_step(0, j + 1);
        if (ok) ok = issue_step(1, j);
      }
      if (!ok) {
        drain_loads(b_q, 1, 1);
        drain_loads(b_full, nk, C::KS);
        drain_loads(b_full + 8 * C::KS, nv, C::VS);
      }
    }
  } else if (warp == C::MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(b_q, 0, ctl, kErrTimeoutMma) &&
                mbar_wait(b_full + 8 * k_slot(0), k_ph(0), ctl, kErrTimeoutMma);
      if (ok) {
        tc_fence_after();
        issue_qk256<D, BF>(tmem + C::COL_S, s_q, s_ring + k_slot(0) * C::KVBYTES);
        mma_commit(b_s);
        mma_commit(b_empty + 8 * k_slot(0));
      }
      for (int j = 0; j < nstep && ok; ++j) {
        // S(j+1) as soon as the softmax has read S(j)
        if (j + 1 < nstep) {
          ok = mbar_wait(b_full + 8 * k_slot(j + 1), k_ph(j + 1), ctl, kErrTimeoutMma) &&
               mbar_wait(b_sfree, j & 1, ctl, kErrTimeoutMma);
          if (!ok) break;
          tc_fence_after();
          issue_qk256<D, BF>(tmem + C::COL_S, s_q, s_ring + k_slot(j + 1) * C::KVBYTES);
          mma_commit(b_s);
          mma_commit(b_empty + 8 * k_slot(j + 1));
        }
        // O += P(j) V_j, in two halves of 128 keys: the first half's products
        // run while the softmax computes the second half's exponentials
        ok = mbar_wait(b_full + 8 * v_slot(j), v_ph(j), ctl, kErrTimeoutMma) &&
             mbar_wait(b_p, j & 1, ctl, kErrTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        issue_pv256<D, BF, 0, 8>(tmem + C::COL_O, tmem + C::COL_P, s_ring + v_slot(j) * C::KVBYTES,
                                 j > 0);
        ok = mbar_wait(b_p + 8, j & 1, ctl, kErrTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        issue_pv256<D, BF, 8, 16>(tmem + C::COL_O, tmem + C::COL_P,
                                  s_ring + v_slot(j) * C::KVBYTES, true);
        mma_commit(b_pv);
        mma_commit(b_empty + 8 * v_slot(j));
        if (j + 1 == nstep) mma_commit(b_o);
      }
      // every MMA issued above completes before TMEM is released
      const uint64_t t0 = globaltimer_ns();
      if (nstep > 0)
        while (!mbar_try_wait(b_pv, (nstep - 1) & 1) && globaltimer_ns() - t0 < FAB_WAIT_LIMIT_NS) {
        }
    }
  } else {
    // ------------------------------------------------------------ softmax
    // warp w owns the 16 rows at lanes 32*(w%4) + 16*(w>>2) of its quadrant;
    // lane i and lane i+16 share row i%16, holding keys 64h..64h+63 and
    // 128+64h..128+64h+63 of each step (h = 0, 1; TMEM shape 16x32bx2), so the
    // row's maximum and sum combine with one shuffle, and P goes back in two
    // halves of 128 keys, each released on its own barrier
    const int h = lane >> 4;
    const int r = 32 * (warp & 3) + 16 * (warp >> 2) + (lane & 15);
    const int row = m0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(32 * (warp & 3) + 16 * (warp >> 2)) << 16;
    const uint32_t t_s = tmem + C::COL_S + lane_off;
    const uint32_t t_p = tmem + C::COL_P + lane_off;
    const uint32_t t_o = tmem + C::COL_O + lane_off;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nstep; ++j) {
      ok = mbar_wait(b_s, j & 1, ctl, kErrTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      // s[c] is key 64h + c (c < 64) or 128 + 64h + (c - 64) of the step
      uint32_t sr[128];
      tmem_ld16x2_x64(t_s, reinterpret_cast<uint32_t(&)[64]>(sr[0]));
      tmem_ld16x2_x64(t_s + 128, reinterpret_cast<uint32_t(&)[64]>(sr[64]));
      tmem_ld_wait(sr);
      tc_fence_before();
      mbar_arrive(b_sfree);   // S(j+1) may overwrite the S columns now
      float* s = reinterpret_cast<float*>(sr);
      const int kb0 = j * C::BN + 64 * h;   // this thread's first key of the step
      const bool need_mask = (j * C::BN + C::BN > kend) || (p.causal && j * C::BN + C::BN - 1 > m0);
      if (need_mask) {
        const int lim = p.causal ? min(kend - 1, row) : (kend - 1);
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (kb0 + c + 64 * (c / 64) > lim) s[c] = -INFINITY;
      }
      float mx8[8];   // as in fwd_kernel_p, over this half's 128 keys
#pragma unroll
      for (int c = 0; c < 8; ++c) mx8[c] = fmaxf(s[c], s[c + 8]);
#pragma unroll
      for (int c = 16; c < 128; c += 16)
#pragma unroll
        for (int k8 = 0; k8 < 8; ++k8) mx8[k8] = max3f(mx8[k8], s[c + k8], s[c + 8 + k8]);
      const float pmx = fmaxf(max3f(mx8[0], mx8[1], mx8[2]),
                              max3f(max3f(mx8[3], mx8[4], mx8[5]), mx8[6], mx8[7]));
      const float mx = fmaxf(pmx, __shfl_xor_sync(0xffffffffu, pmx, 16));
      const float m_new = fmaxf(m_used, mx * p.scale_log2);
      // rescale only when the running max grew by more than 2^8 (P stays below
      // 256; the final 1/l uses the same offset); warp-wide because O is
      // rescaled through TMEM, alpha = 1 for rows that do not need it
      bool rescale = false;
      float alpha = 1.f;
      if (j == 0) {
        m_used = m_new;
      } else {
        const bool need = m_new > m_used + 8.f;
        rescale = __any_sync(0xffffffffu, need);
        if (need) {
          alpha = ex2(m_used - m_new);
          l *= alpha;
          m_used = m_new;
        }
      }
      // P in pair columns (column c holds keys 2c, 2c+1 of the step): this
      // thread's first 32 pairs go to columns 32h .. (keys 0..127 between the
      // two threads of the row), the other 32 to 64 + 32h ..
      const uint64_t sl2 = f32x2(p.scale_log2, p.scale_log2), nm = f32x2(-m_used, -m_used);
      uint64_t lp[2] = {f32x2(0.f, 0.f), f32x2(0.f, 0.f)};
      uint32_t pk[32];
      auto exps32 = [&](int c0) {
#pragma unroll
        for (int q2 = 0; q2 < 32; ++q2) {
          const float2 x = f32x2_split(fma_x2(f32x2(s[c0 + 2 * q2], s[c0 + 2 * q2 + 1]), sl2, nm));
          const float e0 = ex2(x.x), e1 = ex2(x.y);
          lp[q2 & 1] = add_x2(lp[q2 & 1], f32x2(e0, e1));
          pk[q2] = pack2<BF>(e0, e1);
        }
      };
      exps32(0);
      // O += P(j-1) V must be complete before P and O are rewritten
      if (j > 0) {
        ok = mbar_wait(b_pv, (j - 1) & 1, ctl, kErrTimeoutSoftmax);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
      }
      if (rescale) {   // this thread's D/2 columns of the O row
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {
          uint32_t orow[32];
          tmem_ld16x2_x32(t_o + 64 * c, orow);   // columns 64c + 32h ..
          tmem_ld_wait(orow);
#pragma unroll
          for (int i = 0; i < 32; ++i) orow[i] = __float_as_uint(__uint_as_float(orow[i]) * alpha);
          tmem_st16x2_x32(t_o + 64 * c, orow);
        }
      }
      tmem_st16x2_x32(t_p, pk);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(b_p);       // keys 0..127 of P(j) (and O rescaled)
      exps32(64);
      tmem_st16x2_x32(t_p + 64, pk);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(b_p + 8);   // keys 128..255
      const float2 la = f32x2_split(add_x2(lp[0], lp[1]));
      l += la.x + la.y;
    }
    if (ok && nstep > 0) {
      l += __shfl_xor_sync(0xffffffffu, l, 16);   // the row sum is the two halves' sums
      ok = mbar_wait(b_o, 0, ctl, kErrTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        const float inv = 1.f / l;
        // O row rounded to 16 bits, staged as 64-column swizzled boxes over
        // the Q tile (the last S has read it) and written by TMA stores below
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {
          const int col = 64 * c + 32 * h;
          uint32_t orow[32];
          tmem_ld16x2_x32(t_o + 64 * c, orow);
          tmem_ld_wait(orow);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const int piece = 4 * ((col % 64) / 32) + q4;
            st_shared_v4(s_q + (col / 64) * 16384 + r * 128 + ((piece ^ (r & 7)) << 4),
                         pack2<BF>(__uint_as_float(orow[8 * q4 + 0]) * inv, __uint_as_float(orow[8 * q4 + 1]) * inv),
                         pack2<BF>(__uint_as_float(orow[8 * q4 + 2]) * inv, __uint_as_float(orow[8 * q4 + 3]) * inv),
                         pack2<BF>(__uint_as_float(orow[8 * q4 + 4]) * inv, __uint_as_float(orow[8 * q4 + 5]) * inv),
                         pack2<BF>(__uint_as_float(orow[8 * q4 + 6]) * inv, __uint_as_float(orow[8 * q4 + 7]) * inv));
          }
        }
        if (row < p.n && h == 0)
          p.lse[static_cast<size_t>(bh) * p.n + row] = (m_used + __log2f(l)) * 0.69314718055994531f;
      }
    }
    // every softmax thread gets here once, whichever path it took above; a
    // thread that skipped its staging raised the abort flag first
    fence_async_smem();
    named_bar_sync(1, 256);
    if (threadIdx.x == 0 && nstep > 0 && *abort_flag == 0) {
#pragma unroll 1
      for (int c = 0; c < D / 64; ++c) tma_store_4d(&tm_o, s_q + c * 16384, 64 * c, m0, hq_i, b_i);
      bulk_commit_group();
      bulk_wait_read_all();   // boxes read: shared memory may be released
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == C::MMA_WARP) {
    __syncwarp();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace fab

namespace fab {

// Folds one attention result over a further set of keys (16-bit O_p and its
// LSE_p) into a running fp32 (O, LSE), in place:
//   LSE' = logaddexp(LSE, LSE_p),  O' = O e^(LSE - LSE') + O_p e^(LSE_p - LSE').
// The ring's per-step merge, one pass over the rows. One thread per 8 columns;
// the d/8 threads of a row are lanes of one warp (d/8 divides 32), which read
// both LSEs before the row's first lane writes the new one. Rows without keys
// on either side (both LSEs -inf) are left unchanged.
template <bool BF>
__global__ void __launch_bounds__(256) merge_partial_kernel(float* __restrict__ o, Strides so,
                                                            float* __restrict__ lse, Strides sl,
                                                            const uint16_t* __restrict__ op,
                                                            Strides sop,
                                                            const float* __restrict__ lsep,
                                                            Strides slp, int h, int n, int d,
                                                            long long total) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const bool live = i < total;
  const int per_row = d / 8;
  const long long row = live ? i / per_row : 0;
  const int part8 = static_cast<int>(i - row * per_row);
  const int r = static_cast<int>(row % n);
  const long long bh = row / n;
  const int hh = static_cast<int>(bh % h), bb = static_cast<int>(bh / h);
  float la = -INFINITY, lp = -INFINITY;
  if (live) {
    la = lse[sl.at(bb, hh, r)];
    lp = lsep[slp.at(bb, hh, r)];
  }
  __syncwarp();
  const float m = fmaxf(la, lp);
  if (!live || m == -INFINITY) return;
  const float l = m + log1pf(expf(-fabsf(la - lp)));
  const float wa = expf(la - l), wp = expf(lp - l);
  float4* a = reinterpret_cast<float4*>(o + so.at(bb, hh, r)) + 2 * part8;
  const uint4 pk = reinterpret_cast<const uint4*>(op + sop.at(bb, hh, r))[part8];
  const float2 p0 = unpack2<BF>(pk.x), p1 = unpack2<BF>(pk.y), p2 = unpack2<BF>(pk.z),
               p3 = unpack2<BF>(pk.w);
  float4 a0 = a[0], a1 = a[1];
  a0 = make_float4(a0.x * wa + p0.x * wp, a0.y * wa + p0.y * wp, a0.z * wa + p1.x * wp,
                   a0.w * wa + p1.y * wp);
  a1 = make_float4(a1.x * wa + p2.x * wp, a1.y * wa + p2.y * wp, a1.z * wa + p3.x * wp,
                   a1.w * wa + p3.y * wp);
  a[0] = a0;
  a[1] = a1;
  if (part8 == 0) lse[sl.at(bb, hh, r)] = l;
}

}  // namespace fab
