// fa_fwd_persist.cuh -- the two-tile forward (reference flash::fwd_kernel,
// flash_fwd.cuh:68-355; the math as described in fa_fwd.cuh) as a persistent
// kernel: one CTA per SM walks a list of (batch, q-head, 256-row m-block) items.
//
// One item (256 query rows of one (batch, q-head)) in one CTA:
//   warps 0-7   softmax for query tile 0 (rows m0 .. m0+127): each warp owns
//               16 rows; lanes i and i+16 hold columns {0..31, 64..95} and
//               {32..63, 96..127} of row i (TMEM shape 16x32bx2)
//   warps 8-15  softmax for query tile 1 (rows m0+128 .. m0+255), the same way
//   warp  16    TMEM allocation + the single thread that issues tcgen05.mma
//   warp  17    the single thread that issues TMA loads
// Two warps per SMSP share one tile's exponentials; the two halves of a row
// combine their partial maxima (and row sums) with one shuffle, so a tile's
// softmax warps meet only where P_t is handed to the MMA.
// TMEM (512 columns): S0 [0,128)  S1 [128,256)  O0 [256,256+D)  O1 [256+D, 256+2D)
// P_t (fp16 pairs, column 32 + c = keys 2c, 2c+1) is written back over
// columns 32..95 of S_t, inside S columns its warp has already read into
// registers, in two pieces (keys 0..63, then 64..127). O_t += P_t V_j reads P_t
// from TMEM, so P never touches shared memory, and V is the MMA's only shared
// operand. Shared memory: Q0, Q1, a ring of K/V tiles (K_j and V_j
// alternate), and an O staging buffer.
// Per key block j the MMA thread issues, in order,
//   [P0_j] O0 += P0_j V_j (two halves) ; S0_{j+1} ; [P1_j] O1 += P1_j V_j ; S1_{j+1}
// so the tensor core computes one tile's S while the other tile's softmax runs.
// The tensor core executes one thread's MMAs in issue order, so S_t,j+1
// overwrites P_t,j only after O_t += P_t,j V_j has read it; and tcgen05.commit
// tracks every MMA issued before it, so when softmax t sees S_t,j+1 complete,
// PV_t,j is complete too and O_t is free to rescale.
//
// Persistence: a CTA that ran one item paid a fixed cost of ~4.5-7 us (launch,
// barrier and TMEM set-up, Q and first K/V loads, the first S with nothing to
// overlap, the O epilogue), 10-15% of the forward at 7-10 CTAs per SM. Here the
// ring of K/V tiles and every barrier keep running across items, so the next
// item's Q (loaded as soon as the current item's last S has read Q) and first
// K/V blocks arrive while the current item finishes, and its first S runs
// while the softmax warps write the current item's O.
//
// Items are ordered heaviest-first (causal: the last m-blocks first), and CTA
// c takes items c, 2G-1-c, 2G+c, 4G-1-c, ... (G CTAs), which evens out the
// total work per CTA. O leaves through a staging buffer of its own, shared by
// the two tiles' epilogues in turn (tile 0 then tile 1 of each item), so the
// Q buffers can be reloaded without waiting for the O stores.
#pragma once
#include "fa_fwd.cuh"

namespace fab {

template <int D>
struct FwdCfgP {
  static constexpr int BM = 128, BN = 128, CH = D / 64;
  static constexpr int QBYTES = BM * D * 2;
  static constexpr int KVBYTES = BN * D * 2;
  static constexpr int STAGES = (D == 128) ? 4 : 8;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_RING = OFF_Q + 2 * QBYTES;
  static constexpr int OFF_OSTG = OFF_RING + STAGES * KVBYTES;   // one tile's O, 16-bit
  static constexpr int OFF_BAR = OFF_OSTG + QBYTES;
  // q[2], qfree[2], full[STAGES], empty[STAGES], s[2], p[2][2], o[2], stg, fin
  static constexpr int NBAR = 14 + 2 * STAGES;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;   // +1024 for manual alignment
  static_assert(SMEM <= 232448, "shared memory over the per-block limit");
  static constexpr int THREADS = 576;
  static constexpr int MMA_WARP = 16, TMA_WARP = 17;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t COL_S0 = 0, COL_S1 = 128, COL_O0 = 256, COL_O1 = 256 + D;
  static constexpr uint32_t COL_P = 32;
};

// Named barrier over `nthreads` threads that also ORs a predicate: every
// participant gets the same answer (so a group can agree to stop together).
__device__ __forceinline__ bool bar_sync_or(int id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// The g-th item of CTA c out of G: c, 2G-1-c, 2G+c, 4G-1-c, ... The sequence
// never decreases in g, so a CTA stops at its first item past the end.
__device__ __forceinline__ int persist_item(int c, int g, int G) {
  return (g & 1) ? (g + 1) * G - 1 - c : g * G + c;
}

// One item: the heaviest-first m-block index and the (batch, head) slice.
struct FwdItem {
  int bh, m0, b, hq, hk, nt0, nt1, nkv;
  __device__ __forceinline__ FwdItem(int item, const FwdParams& p) {
    const int y = item / p.bh_count;
    bh = item - y * p.bh_count;
    m0 = (p.n_mblocks - 1 - y) * 256;
    b = bh / p.hq;
    hq = bh % p.hq;
    hk = hq / p.group;
    const int nblk = (p.n + 127) / 128;
    nt0 = (m0 >= p.n) ? 0 : (p.causal ? min(nblk, m0 / 128 + 1) : nblk);
    nt1 = (m0 + 128 >= p.n) ? 0 : (p.causal ? min(nblk, (m0 + 128) / 128 + 1) : nblk);
    nkv = max(nt0, nt1);
  }
  __device__ __forceinline__ int nt(int t) const { return t ? nt1 : nt0; }
};

}  // namespace fab

namespace fab {

template <int D, bool BF>
__global__ void __maxnreg__(96)
    fwd_kernel_p(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                 const FwdParams p) {
  using C = FwdCfgP<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));

  const uint32_t s_q0 = sbase + C::OFF_Q, s_q1 = s_q0 + C::QBYTES;
  const uint32_t s_ring = sbase + C::OFF_RING, s_ostg = sbase + C::OFF_OSTG;
  // b_q + 8t: Q_t of the CTA's n-th item loaded (phase n); b_qfree + 8t: its last
  // S has read Q_t (phase n), so Q_t of item n+1 may be loaded
  const uint32_t b_q = sbase + C::OFF_BAR, b_qfree = b_q + 16;
  const uint32_t b_full = b_qfree + 16, b_empty = b_full + 8 * C::STAGES;
  // b_p + 8*(2t + k): P_t's keys 0..63 (k = 0) / 64..127 (k = 1) are in TMEM
  const uint32_t b_s = b_empty + 8 * C::STAGES, b_p = b_s + 16, b_o = b_p + 32;
  // b_stg: the O staging buffer was released by epilogue e (phase e; epilogue
  // 2n + t is tile t of the CTA's n-th item)
  const uint32_t b_stg = b_o + 16, b_fin = b_stg + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + C::OFF_BAR + C::NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta = static_cast<int>(blockIdx.x), G = static_cast<int>(gridDim.x);
  const Ctl ctl{abort_flag, p.err};

  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(b_q + 8 * t, 1);
      mbar_init(b_qfree + 8 * t, 1);
      mbar_init(b_s + 8 * t, 1);
      mbar_init(b_p + 16 * t, 256);
      mbar_init(b_p + 16 * t + 8, 256);
      mbar_init(b_o + 8 * t, 1);
    }
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(b_full + 8 * s, 1);
      mbar_init(b_empty + 8 * s, 1);
    }
    mbar_init(b_stg, 1);
    mbar_init(b_fin, 1);
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
      int it = 0, n = 0;   // ring loads issued; items whose Q tiles were both loaded
      int nq[2] = {0, 0};  // Q_t loads issued
      bool ok = true;
      constexpr int kAhead = 2;  // L2 prefetch distance, in key blocks
      for (int g = 0; ok; ++g) {
        const int item = persist_item(cta, g, G);
        if (item >= p.n_items) break;
        const FwdItem w(item, p);
        // Q_t once the previous item's last S_t has read the buffer
#pragma unroll 1
        for (int t = 0; t < 2 && ok; ++t) {
          if (n > 0) ok = mbar_wait(b_qfree + 8 * t, (n - 1) & 1, ctl, kErrTimeoutLoad);
          if (!ok) break;
          mbar_arrive_expect_tx(b_q + 8 * t, C::QBYTES);
#pragma unroll
          for (int c = 0; c < C::CH; ++c)
            tma_load_4d((t ? s_q1 : s_q0) + c * 16384, &tm_q, b_q + 8 * t, c * 64, w.m0 + 128 * t,
                        w.hq, w.b);
          ++nq[t];
        }
        if (!ok) break;
        ++n;
        for (int j = 0; j < kAhead && j < w.nkv; ++j)
          for (int c = 0; c < C::CH; ++c) {
            tma_prefetch_l2_4d(&tm_k, c * 64, j * 128, w.hk, w.b);
            tma_prefetch_l2_4d(&tm_v, c * 64, j * 128, w.hk, w.b);
          }
        for (int j = 0; j < w.nkv && ok; ++j) {
          if (j + kAhead < w.nkv)
            for (int c = 0; c < C::CH; ++c) {
              tma_prefetch_l2_4d(&tm_k, c * 64, (j + kAhead) * 128, w.hk, w.b);
              tma_prefetch_l2_4d(&tm_v, c * 64, (j + kAhead) * 128, w.hk, w.b);
            }
#pragma unroll 1
          for (int kind = 0; kind < 2 && ok; ++kind, ++it) {
            const int slot = it % C::STAGES;
            const uint32_t ph = (it / C::STAGES) & 1;
            ok = mbar_wait(b_empty + 8 * slot, ph ^ 1, ctl, kErrTimeoutLoad);
            if (!ok) break;
            const uint32_t fb = b_full + 8 * slot;
            mbar_arrive_expect_tx(fb, C::KVBYTES);
            const uint32_t dst = s_ring + slot * C::KVBYTES;
#pragma unroll
            for (int c = 0; c < C::CH; ++c)
              tma_load_4d(dst + c * 16384, kind ? (const void*)&tm_v : (const void*)&tm_k, fb, c * 64,
                          j * 128, w.hk, w.b);
          }
        }
      }
      // Drain: do not leave the CTA while a load it issued may still land.
      if (!ok) {
        drain_loads(b_q, nq[0], 1);
        drain_loads(b_q + 8, nq[1], 1);
        drain_loads(b_full, it, C::STAGES);
      }
    }
  } else if (warp == C::MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    // Per item: S_t,0 for both tiles, then per key block j PV_0(j) in two
    // halves, S_0(j+1), PV_1(j), S_1(j+1). The ring position and the per-tile
    // P / S counts continue from item to item.
    if (lane == 0) {
      int it = 0, n = 0;
      int pc[2] = {0, 0};   // P_t blocks handed over so far (b_p phases)
      bool ok = true;
      for (int g = 0; ok; ++g) {
        const int item = persist_item(cta, g, G);
        if (item >= p.n_items) break;
        const FwdItem w(item, p);
        ok = mbar_wait(b_q, n & 1, ctl, kErrTimeoutMma) && mbar_wait(b_q + 8, n & 1, ctl, kErrTimeoutMma);
        ++n;
        if (!ok) break;
        // prologue: S_t,0 for both tiles (K_0 is ring use `it`)
        ok = mbar_wait(b_full + 8 * (it % C::STAGES), (it / C::STAGES) & 1, ctl, kErrTimeoutMma);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (w.nt(t) > 0) {
            issue_qk<D, BF>(tmem + (t ? C::COL_S1 : C::COL_S0), t ? s_q1 : s_q0,
                            s_ring + (it % C::STAGES) * C::KVBYTES);
            mma_commit(b_s + 8 * t);
          }
          // Q_t is free for the next item once its last S has completed (a
          // tile without rows issued none)
          if (w.nt(t) <= 1) mma_commit(b_qfree + 8 * t);
        }
        mma_commit(b_empty + 8 * (it % C::STAGES));
        ++it;
        for (int j = 0; j < w.nkv && ok; ++j) {
          const int slot_v = it % C::STAGES;
          ok = mbar_wait(b_full + 8 * slot_v, (it / C::STAGES) & 1, ctl, kErrTimeoutMma);
          ++it;
          if (!ok) break;
          tc_fence_after();
          const bool more = (j + 1 < w.nkv);
          const int slot_k = it % C::STAGES;
          const uint32_t ph_k = (it / C::STAGES) & 1;
          if (more) ++it;
          bool have_k = false;
#pragma unroll
          for (int t = 0; t < 2 && ok; ++t) {
            if (j >= w.nt(t)) continue;
            const uint32_t d_o = tmem + (t ? C::COL_O1 : C::COL_O0);
            const uint32_t a_p = tmem + (t ? C::COL_S1 : C::COL_S0) + C::COL_P;
            // P_t in two halves of 64 keys: the first half's products run
            // while the softmax computes the second half's exponentials
            ok = mbar_wait(b_p + 16 * t, pc[t] & 1, ctl, kErrTimeoutMma);
            if (!ok) break;
            tc_fence_after();
            issue_pv<D, BF, 0, 4>(d_o, a_p, s_ring + slot_v * C::KVBYTES, j > 0);
            ok = mbar_wait(b_p + 16 * t + 8, pc[t] & 1, ctl, kErrTimeoutMma);
            if (!ok) break;
            ++pc[t];
            tc_fence_after();
            issue_pv<D, BF, 4, 8>(d_o, a_p, s_ring + slot_v * C::KVBYTES, true);
            if (j + 1 < w.nt(t)) {
              if (!have_k) {
                ok = mbar_wait(b_full + 8 * slot_k, ph_k, ctl, kErrTimeoutMma);
                if (!ok) break;
                tc_fence_after();
                have_k = true;
              }
              issue_qk<D, BF>(tmem + (t ? C::COL_S1 : C::COL_S0), t ? s_q1 : s_q0,
                              s_ring + slot_k * C::KVBYTES);
              mma_commit(b_s + 8 * t);
              if (j + 2 == w.nt(t)) mma_commit(b_qfree + 8 * t);   // the tile's last S
            } else {
              mma_commit(b_o + 8 * t);  // last block of this tile: O_t is final
            }
          }
          if (!ok) break;
          mma_commit(b_empty + 8 * slot_v);
          if (more) {
            if (!have_k) {
              ok = mbar_wait(b_full + 8 * slot_k, ph_k, ctl, kErrTimeoutMma);
              if (!ok) break;
            }
            mma_commit(b_empty + 8 * slot_k);
          }
        }
      }
      // Every MMA issued above must finish before TMEM is released.
      mma_commit(b_fin);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(b_fin, 0) && globaltimer_ns() - t0 < FAB_WAIT_LIMIT_NS) {
      }
    }
  } else {
    // ------------------------------------------------------------ softmax tile t
    // The softmax of one tile, item after item; the S, P and O barrier
    // phases continue across items.
    const int t = warp >> 3;
    const int hf = lane >> 4;
    const int r = 32 * (warp & 3) + 16 * ((warp >> 2) & 1) + (lane & 15);
    const uint32_t lane_off = static_cast<uint32_t>(32 * (warp & 3) + 16 * ((warp >> 2) & 1)) << 16;
    const uint32_t t_s = tmem + (t ? C::COL_S1 : C::COL_S0) + lane_off;
    const uint32_t t_o = tmem + (t ? C::COL_O1 : C::COL_O0) + lane_off;
    int sc = 0, oc = 0, n = 0;   // S_t blocks, O_t results and items seen so far
    bool ok = true;
    for (int g = 0; ok; ++g) {
      const int item = persist_item(cta, g, G);
      if (item >= p.n_items) break;
      const FwdItem w(item, p);
      const int nt = w.nt(t);
      const int row = w.m0 + 128 * t + r;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < nt; ++j, ++sc) {
        ok = mbar_wait(b_s + 8 * t, sc & 1, ctl, kErrTimeoutSoftmax);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        // s[c] is key 32*hf + c (c < 32) or 64 + 32*hf + (c - 32) of the block
        uint32_t sr[64];
        tmem_ld16x2_x32(t_s, reinterpret_cast<uint32_t(&)[32]>(sr[0]));
        tmem_ld16x2_x32(t_s + 64, reinterpret_cast<uint32_t(&)[32]>(sr[32]));
        tmem_ld_wait(sr);
        float* s = reinterpret_cast<float*>(sr);
        const int kb0 = j * 128;
        const int col0 = kb0 + 32 * hf;
        const bool need_mask = (kb0 + 128 > p.n) || (p.causal && kb0 + 127 > w.m0 + 128 * t);
        if (need_mask) {
          const int lim = p.causal ? min(p.n - 1, row) : (p.n - 1);
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (col0 + c + 32 * (c / 32) > lim) s[c] = -INFINITY;
        }
        // this half's max: 8 interleaved chains of three-input maxima, then a
        // tree; the other half's by shuffle
        float mx8[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) mx8[c] = fmaxf(s[c], s[c + 8]);
#pragma unroll
        for (int c = 16; c < 64; c += 16)
#pragma unroll
          for (int k8 = 0; k8 < 8; ++k8) mx8[k8] = max3f(mx8[k8], s[c + k8], s[c + 8 + k8]);
        const float pmx = fmaxf(max3f(mx8[0], mx8[1], mx8[2]),
                                max3f(max3f(mx8[3], mx8[4], mx8[5]), mx8[6], mx8[7]));
        const float mx = fmaxf(pmx, __shfl_xor_sync(0xffffffffu, pmx, 16));
        const float m_new = fmaxf(m_used, mx * p.scale_log2);
        // Rescale only when the running max grew by more than 2^8: P stays
        // below 256, and the final 1/l uses the same offset, so the result is
        // unchanged (only which power of two the partial sums carry). Both
        // halves see the same maxima and so take the same decision.
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
        const uint64_t sl2 = f32x2(p.scale_log2, p.scale_log2), nm = f32x2(-m_used, -m_used);
        uint64_t lp[2] = {f32x2(0.f, 0.f), f32x2(0.f, 0.f)};
        uint32_t pw[16];
#pragma unroll
        for (int hh = 0; hh < 16; ++hh) {
          const float2 x = f32x2_split(fma_x2(f32x2(s[2 * hh], s[2 * hh + 1]), sl2, nm));
          const float e0 = ex2(x.x), e1 = ex2(x.y);
          lp[hh & 1] = add_x2(lp[hh & 1], f32x2(e0, e1));
          pw[hh] = pack2<BF>(e0, e1);
        }
        tmem_st16x2_x16(t_s + C::COL_P, pw);
        if (rescale) {   // O_t *= alpha on this thread's D/2 columns, before P_t is released
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c) {
            uint32_t orow[32];
            const uint32_t a = t_o + 64 * c;
            tmem_ld16x2_x32(a, orow);
            tmem_ld_wait(orow);
#pragma unroll
            for (int i = 0; i < 32; ++i) orow[i] = __float_as_uint(__uint_as_float(orow[i]) * alpha);
            tmem_st16x2_x32(a, orow);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(b_p + 16 * t);   // keys 0..63 of P_t (and O_t rescaled)
#pragma unroll
        for (int hh = 0; hh < 16; ++hh) {
          const float2 x = f32x2_split(fma_x2(f32x2(s[32 + 2 * hh], s[33 + 2 * hh]), sl2, nm));
          const float e0 = ex2(x.x), e1 = ex2(x.y);
          lp[hh & 1] = add_x2(lp[hh & 1], f32x2(e0, e1));
          pw[hh] = pack2<BF>(e0, e1);
        }
        tmem_st16x2_x16(t_s + C::COL_P + 32, pw);
        const float2 la = f32x2_split(add_x2(lp[0], lp[1]));
        l += la.x + la.y;
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(b_p + 16 * t + 8);   // keys 64..127
      }
      // Epilogue 2n + t: once epilogue 2n + t - 1 (the other tile's, or this
      // item's tile 0) has released the staging buffer, O_t's rows rounded to
      // 16 bits go there as 64-column swizzled boxes and leave by TMA stores.
      // A failed wait falls through to the tile's barrier below and stops
      // every warp of the tile together (the abort flag is read after it).
      const int e = 2 * n + t;
      if (ok && nt > 0) {
        l += __shfl_xor_sync(0xffffffffu, l, 16);   // the row sum is the two halves' sums
        ok = mbar_wait(b_o + 8 * t, oc & 1, ctl, kErrTimeoutSoftmax);
        ok = __all_sync(0xffffffffu, ok);
        ++oc;
      }
      if (ok && e > 0) {
        ok = mbar_wait(b_stg, (e - 1) & 1, ctl, kErrTimeoutEpilogue);
        ok = __all_sync(0xffffffffu, ok);
      }
      if (ok && nt > 0) {
        tc_fence_after();
        const float inv = 1.f / l;
        const size_t bhn = static_cast<size_t>(w.bh) * p.n;   // LSE is (B, Hq, N) contiguous
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {
          const int col = 64 * c + 32 * hf;
          uint32_t orow[32];
          tmem_ld16x2_x32(t_o + 64 * c, orow);
          tmem_ld_wait(orow);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const int piece = 4 * ((col % 64) / 32) + q4;
            st_shared_v4(s_ostg + (col / 64) * 16384 + r * 128 + ((piece ^ (r & 7)) << 4),
                         pack2<BF>(__uint_as_float(orow[8 * q4 + 0]) * inv, __uint_as_float(orow[8 * q4 + 1]) * inv),
                         pack2<BF>(__uint_as_float(orow[8 * q4 + 2]) * inv, __uint_as_float(orow[8 * q4 + 3]) * inv),
                         pack2<BF>(__uint_as_float(orow[8 * q4 + 4]) * inv, __uint_as_float(orow[8 * q4 + 5]) * inv),
                         pack2<BF>(__uint_as_float(orow[8 * q4 + 6]) * inv, __uint_as_float(orow[8 * q4 + 7]) * inv));
          }
        }
        if (row < p.n && hf == 0) p.lse[bhn + row] = (m_used + __log2f(l)) * 0.69314718055994531f;
        tc_fence_before();
      }
      fence_async_smem();
      // every thread of the tile learns whether any of them (or another role,
      // through the abort flag) failed, and the tile stops together
      const bool stop = bar_sync_or(1 + t, 256, !ok || *abort_flag != 0);
      if ((threadIdx.x & 255) == 0) {
        if (nt > 0 && !stop) {
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c)
            tma_store_4d(&tm_o, s_ostg + c * 16384, 64 * c, w.m0 + 128 * t, w.hq, w.b);
          bulk_commit_group();
          bulk_wait_read_all();   // boxes read: the staging buffer may be reused
        }
        mbar_arrive(b_stg);
      }
      ++n;
      if (stop) break;
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
