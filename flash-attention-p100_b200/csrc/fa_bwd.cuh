// fa_bwd.cuh -- FlashAttention-2 backward for sm_100a.
//
// Replaces flash_bwd::bwd_preprocess, flash_bwd::bwd_kernel and
// flash_bwd::launch (reference flash_bwd.cuh:63-484). Same math:
//   P  = exp(scale * Q K^T - LSE)          (recomputed from the forward's LSE)
//   Dv = rowsum(dO o O)                    (flash_bwd.cuh:66-78, O is the fp16 output)
//   dS = P o (dO V^T - Dv)
//   dV = P^T dO,  dK = scale * dS^T Q,  dQ = scale * dS K
// Padded rows/columns and causal-masked entries contribute exactly zero
// (flash_bwd.cuh:274-281).
//
// The reference accumulates dQ with fp32 atomicAdd from every key block
// (flash_bwd.cuh:442). Here dQ is computed by its own query-stationary kernel
// that owns each dQ row outright, so there are no global atomics and the
// result is deterministic.
//
// Every MMA here has N = 128: a tcgen05.mma with K = 16 costs about the same
// ~95-110 cycles for N = 64 as for N = 128 (measured on B200), so the query
// step of the dK/dV kernel and the key step of the dQ kernel are 128 wide. dK/dV come from a key-stationary kernel that loops
// over the GQA group and all query blocks, keeping both accumulators in TMEM
// (as the reference keeps them in registers, flash_bwd.cuh:163, :448-463).
//
// Workspace (written by the preprocess, read by the gradient kernels): per
// (batch, q-head) a row of n_pad = roundup(N, 128) floats of -Dv * scale, then
// the same for -LSE * log2(e). Padded rows hold 0 and -inf, so P = 0 there
// without a bounds test, and every 128-row slice starts 512-byte aligned, which
// lets the TMA warp bulk-copy a query block's slice next to its Q tile. Stored
// negated and pre-scaled, P = 2^fma(S, scale*log2e, -LSE*log2e) and
// dS = scale * P o (dP - Dv) = P * fma(dP, scale, -Dv*scale) are one FMA each,
// which also runs on pairs of columns as one packed fp32x2 instruction.
#pragma once
#include "sm100.cuh"

namespace fab {

struct BwdParams {
  const uint16_t* o;   // (B, Hq, N, D) forward output (fp16 or bf16, as all the
  const uint16_t* dO;  // (B, Hq, N, D)          16-bit tensors of one call)
  const float* lse;    // (B*Hq, N) natural log
  float* dvec;         // (B*Hq, n_pad) workspace: -rowsum(dO o O) * scale
  float* lse2;         // (B*Hq, n_pad) workspace: -LSE * log2(e)
  void* dq;            // (B, Hq, N, D) fp32 or fp16
  uint16_t* dk;        // (B, Hkv, N, D)
  uint16_t* dv;        // (B, Hkv, N, D)
  Strides so, sdo;     // element strides of o and dO (D contiguous)
  Strides sdq, sdk, sdv;
  int* err;
  int n, n_pad, hq, group, causal;
  int dq_fp32;
  int head_group;      // fused kernel: (batch, kv-head) slices scheduled together
  int gsplit, gper;    // fused kernel: GQA group split over gsplit CTAs of gper heads
  int n_batch;         // B
  float* dkv_acc;      // gsplit > 1: fp32 dK then dV, (2B, Hkv, N, D), added into
  int dkv_reduce;      // fused kernel: add dK/dV in fp32 into the tm_dka/tm_dva
                       // accumulators (group split, or a caller accumulating)
  float scale;         // 1/sqrt(D)
  float scale_log2;    // scale * log2(e)
};

__host__ __device__ constexpr int pad_rows(int n) { return (n + 127) / 128 * 128; }

// ---------------------------------------------------------------------------
// -Dv * scale = -rowsum(dO o O) * scale and -LSE * log2(e), over padded rows:
// HBM-bound, one 16-byte vector per thread, D/8 threads per row reduced with
// shuffles.
// ---------------------------------------------------------------------------
template <int D, bool BF>
__global__ void __launch_bounds__(256) bwd_preprocess_kernel(const uint16_t* __restrict__ o, Strides so,
                                                              const uint16_t* __restrict__ dO,
                                                              Strides sdo,
                                                              const float* __restrict__ lse,
                                                              float* __restrict__ dvec,
                                                              float* __restrict__ lse2, int n,
                                                              int n_pad, int hq, long long rows_pad,
                                                              float scale,
                                                              float* __restrict__ dq_zero,
                                                              Strides sdq) {
  constexpr int TPR = D / 8;  // threads per row (8 or 16)
  const long long gtid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long prow = gtid / TPR;
  const int part = static_cast<int>(gtid % TPR);
  const long long bh = prow / n_pad;
  const int r = static_cast<int>(prow - bh * n_pad);
  const bool real = prow < rows_pad && r < n;
  const int b = static_cast<int>(bh / hq), h = static_cast<int>(bh % hq);
  float acc = 0.f;
  if (real) {
    if (dq_zero) {  // the fused kernel accumulates dQ into a zeroed fp32 dq
      float4* z = reinterpret_cast<float4*>(dq_zero + sdq.at(b, h, r)) + 2 * part;
      z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
      z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(o + so.at(b, h, r)) + part);
    const uint4 bb = __ldg(reinterpret_cast<const uint4*>(dO + sdo.at(b, h, r)) + part);
    const uint32_t ha[4] = {a.x, a.y, a.z, a.w}, hb[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 fa = unpack2<BF>(ha[i]);
      const float2 fb = unpack2<BF>(hb[i]);
      acc = fmaf(fa.x, fb.x, acc);
      acc = fmaf(fa.y, fb.y, acc);
    }
  }
#pragma unroll
  for (int off = TPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (prow < rows_pad && part == 0) {
    dvec[prow] = real ? -acc * scale : 0.f;
    lse2[prow] = real ? __ldg(lse + bh * n + r) * -1.4426950408889634f : -INFINITY;
  }
}

// Write 32 fp32 values as fp16 / fp32 to global, 16 bytes per store.
// (16-bit: fp16, or bf16 when BF)
template <bool BF>
__device__ __forceinline__ void store_row32_h(uint16_t* dst, const uint32_t (&v)[32], float mul) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 pk;
    pk.x = pack2<BF>(__uint_as_float(v[8 * q + 0]) * mul, __uint_as_float(v[8 * q + 1]) * mul);
    pk.y = pack2<BF>(__uint_as_float(v[8 * q + 2]) * mul, __uint_as_float(v[8 * q + 3]) * mul);
    pk.z = pack2<BF>(__uint_as_float(v[8 * q + 4]) * mul, __uint_as_float(v[8 * q + 5]) * mul);
    pk.w = pack2<BF>(__uint_as_float(v[8 * q + 6]) * mul, __uint_as_float(v[8 * q + 7]) * mul);
    reinterpret_cast<uint4*>(dst)[q] = pk;
  }
}
__device__ __forceinline__ void store_row32_f32(float* dst, const uint32_t (&v)[32], float mul) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float4 f;
    f.x = __uint_as_float(v[4 * q + 0]) * mul;
    f.y = __uint_as_float(v[4 * q + 1]) * mul;
    f.z = __uint_as_float(v[4 * q + 2]) * mul;
    f.w = __uint_as_float(v[4 * q + 3]) * mul;
    reinterpret_cast<float4*>(dst)[q] = f;
  }
}

// Load 32 consecutive TMEM columns of this warp's lanes and wait for them.
__device__ __forceinline__ void tmem_ld32_sync(uint32_t taddr, uint32_t (&r)[32]) {
  tmem_ld32(taddr, r);
  tmem_ld_wait(r);
}

// Thread-row r writes 32 fp16 values (columns 32*half .. +31 of a 64-column
// K-major swizzled tile of 128 rows) as four 16-byte pieces.
template <bool BF>
__device__ __forceinline__ void st_row32_sw128(uint32_t tile, int r, int half, const float (&x)[32]) {
#pragma unroll
  for (int c4 = 0; c4 < 4; ++c4) {
    const int piece = 4 * half + c4;
    st_shared_v4(tile + r * 128 + ((piece ^ (r & 7)) << 4), pack2<BF>(x[8 * c4], x[8 * c4 + 1]),
                 pack2<BF>(x[8 * c4 + 2], x[8 * c4 + 3]), pack2<BF>(x[8 * c4 + 4], x[8 * c4 + 5]),
                 pack2<BF>(x[8 * c4 + 6], x[8 * c4 + 7]));
  }
}

}  // namespace fab



namespace fab {

// Store 64 fp32 values as 32 packed fp16 pairs into TMEM columns [col, col+32)
// of this warp's lanes (the A-operand layout: column c holds elements 2c, 2c+1).
template <bool BF>
__device__ __forceinline__ void tmem_st_pairs(uint32_t taddr, const float (&x)[2][32]) {
  uint32_t v[32];
#pragma unroll
  for (int c = 0; c < 32; ++c) {
    const int h = c >> 4, e = 2 * (c & 15);
    v[c] = pack2<BF>(x[h][e], x[h][e + 1]);
  }
  tmem_st32(taddr, v);
}

// ---------------------------------------------------------------------------
// dK / dV: one CTA per (128 keys, batch, kv-head), looping over the GQA group
// and every query block of 128 at or below the diagonal.
//   warps 0-7  compute: two warpgroups, one thread per key row each; group w
//              owns query columns 64w..64w+63 of every 128-query step
//   warp  8    TMEM allocation + MMA issue
//   warp  9    TMA producer: K, V once; then Q_i (+ its LSE/Dv slices), dO_i
// TMEM: S^T cols 0..127 | dP^T 128..255 | dV 256..256+D | dK 256+D..256+2D
// P^T goes to a shared-memory tile [key][query] (the A operand of dV), so the
// next S^T can overwrite S^T_i as soon as the compute threads have read it
// and the tensor core works on S^T_{i+1} during the P phase. dS^T (fp16
// pairs) is written into dP^T columns its threads have already read (cols
// 160..223; group w writes 160+32w..) and feeds dK as the A operand from TMEM.
// MMA order per step i (brackets = what it waits for):
//   [S^T_i read, Q_{i+1}] S^T_{i+1} ; [P_i] dV_i ; [dS_i] dK_i ;
//   [dO_{i+1}] dP^T_{i+1}
// dP^T_{i+1} overwrites dS_i after dK_i has read it: the tensor core executes
// one CTA's MMAs in issue order. P_{i+1} waits for dV_i (b_dv).
// Every barrier's arrivals are gated on an MMA that needed all arrivals of the
// previous phase, so no phase can receive arrivals from two steps.
// ---------------------------------------------------------------------------
template <int D>
struct DkdvCfg {
  static constexpr int BN = 128;  // keys per CTA
  static constexpr int BM = 128;  // queries per step
  static constexpr int CH = D / 64;
  static constexpr int TILE = 128 * D * 2;    // K, V, Q or dO tile (128 rows)
  static constexpr int STAGES = 4;            // ring of Q / dO tiles
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + TILE;
  static constexpr int OFF_RING = OFF_V + TILE;
  static constexpr int OFF_P = OFF_RING + STAGES * TILE;     // 128 keys x 128 queries fp16
  static constexpr int OFF_LSE = OFF_P + 32768;              // [2][128] LSE*log2e, [2][128] Dv*scale
  static constexpr int OFF_BAR = OFF_LSE + 2048;
  // kv, full[ST], empty[ST], s, dp, sfree, p, ds, dv, fin
  static constexpr int NBAR = 1 + 2 * STAGES + 7;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16;   // window must start 1024-aligned
  static constexpr int THREADS = 320;
  static constexpr int NCOMPUTE = 256;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t COL_S = 0, COL_DP = 128, COL_DV = 256, COL_DK = 256 + D;
  static constexpr uint32_t COL_DS = 160;
};

template <int D, bool BF>
__global__ void __launch_bounds__(320, 1)
    bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                    const BwdParams p) {
  using C = DkdvCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (!smem_aligned_or_report(smem_raw, p.err)) return;
  const uint32_t sbase = smem_u32(smem_raw);
  const uint32_t s_k = sbase + C::OFF_K, s_v = sbase + C::OFF_V, s_ring = sbase + C::OFF_RING;
  const uint32_t s_lse = sbase + C::OFF_LSE, s_p = sbase + C::OFF_P;
  const uint32_t b_kv = sbase + C::OFF_BAR;
  const uint32_t b_full = b_kv + 8, b_empty = b_full + 8 * C::STAGES;
  const uint32_t b_s = b_empty + 8 * C::STAGES, b_dp = b_s + 8, b_sfree = b_dp + 8,
                 b_p = b_sfree + 8, b_ds = b_p + 8, b_dv = b_ds + 8, b_fin = b_dv + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem_raw + C::OFF_BAR + C::NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid (B*Hkv, key blocks): causal key block 0 has the most work and goes first
  const int bkv = blockIdx.x;
  const int kvb = blockIdx.y;
  const int hkv = p.hq / p.group;
  const int b = bkv / hkv, kvh = bkv % hkv;
  const int kv0 = kvb * C::BN;
  const int nqb = (p.n + C::BM - 1) / C::BM;
  const int i_start = p.causal ? kvb : 0;   // BM == BN: the diagonal block
  const int nq_head = nqb - i_start;
  const int total = p.group * nq_head;      // (group head, query block) steps
  const Ctl ctl{abort_flag, p.err};
  auto slot_of = [](int it) { return it % C::STAGES; };
  auto ph_of = [](int it) { return static_cast<uint32_t>((it / C::STAGES) & 1); };

  if (threadIdx.x == 0) {
    mbar_init(b_kv, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(b_full + 8 * s, 1);
      mbar_init(b_empty + 8 * s, 1);
    }
    mbar_init(b_s, 1);
    mbar_init(b_dp, 1);
    mbar_init(b_sfree, C::NCOMPUTE);
    mbar_init(b_p, C::NCOMPUTE);
    mbar_init(b_ds, C::NCOMPUTE);
    mbar_init(b_dv, 1);
    mbar_init(b_fin, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 9) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      mbar_arrive_expect_tx(b_kv, 2 * C::TILE);
#pragma unroll
      for (int c = 0; c < C::CH; ++c) {
        tma_load_4d(s_k + c * 16384, &tm_k, b_kv, c * 64, kv0, kvh, b);
        tma_load_4d(s_v + c * 16384, &tm_v, b_kv, c * 64, kv0, kvh, b);
      }
      int it = 0;
      bool ok = true;
      constexpr int kAhead = 2;  // L2 prefetch distance, in query steps
      auto prefetch_step = [&](int st) {
        const int q0p = (i_start + st % nq_head) * C::BM;
        const int hqp = kvh * p.group + st / nq_head;
        for (int c = 0; c < C::CH; ++c) {
          tma_prefetch_l2_4d(&tm_q, c * 64, q0p, hqp, b);
          tma_prefetch_l2_4d(&tm_do, c * 64, q0p, hqp, b);
        }
      };
      for (int st = 0; st < kAhead && st < total; ++st) prefetch_step(st);
      for (int step = 0; step < total && ok; ++step) {
        const int g = step / nq_head;
        const int q0 = (i_start + step % nq_head) * C::BM;
        const int hq_g = kvh * p.group + g;
        const int bh = b * p.hq + hq_g;
        if (step + kAhead < total) prefetch_step(step + kAhead);
#pragma unroll 1
        for (int kind = 0; kind < 2; ++kind, ++it) {  // Q_i (+LSE, Dv) then dO_i
          const int slot = slot_of(it);
          ok = mbar_wait(b_empty + 8 * slot, ph_of(it) ^ 1, ctl, kErrTimeoutLoad);
          if (!ok) break;
          const uint32_t fb = b_full + 8 * slot;
          const uint32_t dst = s_ring + slot * C::TILE;
          mbar_arrive_expect_tx(fb, kind ? C::TILE : C::TILE + 1024);
#pragma unroll
          for (int c = 0; c < C::CH; ++c)
            tma_load_4d(dst + c * 16384, kind ? (const void*)&tm_do : (const void*)&tm_q, fb,
                        c * 64, q0, hq_g, b);
          if (!kind) {
            // the Q slot of step i is released after dK_i, so slice buffer
            // i & 1 is free again by the time step i + 2 loads into it
            const size_t off = static_cast<size_t>(bh) * p.n_pad + q0;
            const uint32_t ls = s_lse + (step & 1) * 512;
            bulk_load(ls, p.lse2 + off, 512, fb);
            bulk_load(ls + 1024, p.dvec + off, 512, fb);
          }
        }
      }
      if (!ok) {
        drain_loads(b_kv, 1, 1);
        drain_loads(b_full, it, C::STAGES);
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && total > 0) {
      constexpr uint32_t id_t = idesc_f16(128, 128, false, false, BF);  // S^T, dP^T
      constexpr uint32_t id_g = idesc_f16(128, D, false, true, BF);     // dV (SS), dK (TS)
      // X^T = (K or V) (Q or dO)^T: 128 x 128, K = D
      auto issue_t = [&](uint32_t d_tmem, uint32_t a_s, uint32_t b_s_) {
        const uint64_t da = sdesc_sw128(a_s, 16, 1024), db = sdesc_sw128(b_s_, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          mma_ss(d_tmem, sdesc_add(da, off), sdesc_add(db, off), id_t, kk > 0 ? 1u : 0u);
        }
      };
      // acc += (P or dS)^T (TMEM, 128 keys x 128 queries) * (dO or Q) (MN-major smem)
      auto issue_g = [&](uint32_t d_tmem, uint32_t a_tmem, uint32_t y_s, bool acc) {
        const uint64_t dy = sdesc_sw128(y_s, 16384, 1024);
#pragma unroll
        for (int kk = 0; kk < C::BM / 16; ++kk)
          mma_ts(d_tmem, a_tmem + kk * 8, sdesc_add(dy, kk * 2048), id_g, (acc || kk > 0) ? 1u : 0u);
      };
      auto slot_addr = [&](int it) { return s_ring + slot_of(it) * C::TILE; };
      bool ok = mbar_wait(b_kv, 0, ctl, kErrTimeoutMma);
      if (ok) ok = mbar_wait(b_full + 8 * slot_of(0), ph_of(0), ctl, kErrTimeoutMma);
      if (ok) {
        tc_fence_after();
        issue_t(tmem + C::COL_S, s_k, slot_addr(0));
        mma_commit(b_s);
        ok = mbar_wait(b_full + 8 * slot_of(1), ph_of(1), ctl, kErrTimeoutMma);
      }
      if (ok) {
        tc_fence_after();
        issue_t(tmem + C::COL_DP, s_v, slot_addr(1));
        mma_commit(b_dp);
      }
      for (int i = 0; i < total && ok; ++i) {
        const int it_q = 2 * i, it_do = 2 * i + 1;
        const bool more = i + 1 < total;
        if (more) {  // S^T_{i+1} as soon as S^T_i has been read
          ok = mbar_wait(b_sfree, i & 1, ctl, kErrTimeoutMma) &&
               mbar_wait(b_full + 8 * slot_of(it_q + 2), ph_of(it_q + 2), ctl, kErrTimeoutMma);
          if (!ok) break;
          tc_fence_after();
          issue_t(tmem + C::COL_S, s_k, slot_addr(it_q + 2));
          mma_commit(b_s);
        }
        ok = mbar_wait(b_p, i & 1, ctl, kErrTimeoutMma);   // dV_i += P_i^T dO_i
        if (!ok) break;
        tc_fence_after();
        {
          const uint64_t dpt = sdesc_sw128(s_p, 16, 1024);
          const uint64_t ddo = sdesc_sw128(slot_addr(it_do), 16384, 1024);
#pragma unroll
          for (int kk = 0; kk < C::BM / 16; ++kk)
            mma_ss(tmem + C::COL_DV, sdesc_add(dpt, (kk >> 2) * 16384 + (kk & 3) * 32),
                   sdesc_add(ddo, kk * 2048), id_g, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(b_dv);
        mma_commit(b_empty + 8 * slot_of(it_do));
        ok = mbar_wait(b_ds, i & 1, ctl, kErrTimeoutMma);  // dK_i += dS_i^T Q_i
        if (!ok) break;
        tc_fence_after();
        issue_g(tmem + C::COL_DK, tmem + C::COL_DS, slot_addr(it_q), i > 0);
        mma_commit(b_empty + 8 * slot_of(it_q));
        if (more) {
          ok = mbar_wait(b_full + 8 * slot_of(it_do + 2), ph_of(it_do + 2), ctl, kErrTimeoutMma);
          if (!ok) break;
          tc_fence_after();
          issue_t(tmem + C::COL_DP, s_v, slot_addr(it_do + 2));
          mma_commit(b_dp);
        }
      }
      mma_commit(b_fin);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(b_fin, 0) && globaltimer_ns() - t0 < FAB_WAIT_LIMIT_NS) {
      }
    }
  } else {
    // ------------------------------------------------------------ compute (warps 0-7)
    const int w = warp >> 2;            // query half of each step
    const int r = threadIdx.x & 127;    // key row within the block
    const int kvrow = kv0 + r;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int qlim = p.causal ? kvrow : -1;  // a query column is live iff qlim <= q < N
    bool ok = true;
    for (int i = 0; i < total; ++i) {
      const int q0 = (i_start + i % nq_head) * C::BM + 64 * w;
      const int it_q = 2 * i;
      const uint32_t ph = i & 1;
      // one test for the whole CTA: is any (key, query) pair of this half-step masked?
      const bool need_mask = (q0 + 64 > p.n) || (p.causal && q0 < kv0 + 127);
      // LSE/Dv slices come with Q_i: wait for that load so they are visible here
      ok = mbar_wait(b_full + 8 * slot_of(it_q), ph_of(it_q), ctl, kErrTimeoutSoftmax) &&
           mbar_wait(b_s, ph, ctl, kErrTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[2][32];
      tmem_ld32(tmem + C::COL_S + 64 * w + lane_off, sr[0]);
      tmem_ld32(tmem + C::COL_S + 64 * w + 32 + lane_off, sr[1]);
      tmem_ld_wait_only();
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 32; ++c) asm volatile("" : "+r"(sr[h][c]));
      tc_fence_before();
      mbar_arrive(b_sfree);   // S^T_i is in registers: S^T_{i+1} may overwrite it
      // this step's 64 LSE / Dv values for the group, read as 16-byte vectors
      // (a broadcast LDS per value would cost 8 warps x 64 issue slots on the
      // shared-memory pipe per phase)
      const float4* lse4 =
          reinterpret_cast<const float4*>(smem_raw + C::OFF_LSE) + ((i & 1) * 128 + 64 * w) / 4;
      const float4* dvs4 = lse4 + 64;
      float pv[2][32];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const float4 l4 = lse4[8 * h + c4];
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w};
#pragma unroll
          for (int e4 = 0; e4 < 4; ++e4) {
            const int c = 4 * c4 + e4;
            pv[h][c] = ex2(fmaf(__uint_as_float(sr[h][c]), p.scale_log2, lv[e4]));
          }
        }
      // Masking is a separate pass, taken only by the steps that need it (the
      // diagonal block and the ragged tail): a select folded into every
      // element cost more than the exponentials.
      if (need_mask) {
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int q = q0 + 32 * h + c;
            if (q < qlim || q >= p.n) pv[h][c] = 0.f;
          }
      }
      if (i > 0) {  // dV_{i-1} has finished reading P_{i-1} from the tile
        ok = mbar_wait(b_dv, (i - 1) & 1, ctl, kErrTimeoutSoftmax);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
      }
      st_row32_sw128<BF>(s_p + w * 16384, r, 0, pv[0]);
      st_row32_sw128<BF>(s_p + w * 16384, r, 1, pv[1]);
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(b_p);

      ok = mbar_wait(b_dp, ph, ctl, kErrTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      tmem_ld32(tmem + C::COL_DP + 64 * w + lane_off, sr[0]);
      tmem_ld32(tmem + C::COL_DP + 64 * w + 32 + lane_off, sr[1]);
      tmem_ld_wait_only();
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 32; ++c) asm volatile("" : "+r"(sr[h][c]));
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const float4 d4 = dvs4[8 * h + c4];
          const float dv[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
          for (int e4 = 0; e4 < 4; ++e4)
            pv[h][4 * c4 + e4] *= fmaf(__uint_as_float(sr[h][4 * c4 + e4]), p.scale, dv[e4]);
        }
      tmem_st_pairs<BF>(tmem + C::COL_DS + 32 * w + lane_off, pv);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(b_ds);
    }
    if (ok && total > 0) {
      ok = mbar_wait(b_fin, 0, ctl, kErrTimeoutEpilogue);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {
          const int col = w * (D / 2) + 32 * c;
          uint32_t v[32];
          tmem_ld32_sync(tmem + C::COL_DV + col + lane_off, v);
          if (kvrow < p.n) store_row32_h<BF>(p.dv + p.sdv.at(b, kvh, kvrow) + col, v, 1.f);
          tmem_ld32_sync(tmem + C::COL_DK + col + lane_off, v);
          if (kvrow < p.n) store_row32_h<BF>(p.dk + p.sdk.at(b, kvh, kvrow) + col, v, 1.f);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 8) {
    __syncwarp();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace fab

namespace fab {

// ---------------------------------------------------------------------------
// dQ: one CTA per (128 queries, batch*q-head); loops over key blocks of 128.
//   warps 0-7  compute: two warpgroups, one thread per query row each; group w
//              owns key columns 64w..64w+63 of every 128-key step
//   warp  8    TMEM allocation + MMA issue
//   warp  9    TMA producer: Q, dO once; K_j, V_j alternate in a 4-slot ring
//   K_j sits in a 3-slot ring (held from S_j until dQ_j) and V_j in a 2-slot
//   ring (held only for dP_j), so both are loaded well before they are needed
// TMEM: S cols 0..127 | dP 128..255 | dQ 256..256+D | dS[2] (fp16 pairs) at
//       384 and 448, 64 columns each
// MMA order: S_0 dP_0 | per step j: [S_j read] S_{j+1}, [dP_j read] dP_{j+1},
//            [dS_j] dQ += dS_j K_j
// S = Q K^T, dP = dO V^T (A, B K-major in smem); dQ += dS K takes A = dS from
// TMEM (written by the compute threads with tcgen05.st, one query row per
// lane) and B = K MN-major, so dS never touches shared memory.
// dS_{j+1} may overwrite buffer (j+1)&1 once dQ_{j-1} is done, which dP_{j+1}
// being done implies (dP_{j+1} is issued after dQ_{j-1}). dS-ready has one
// barrier per buffer: a warp can be a full step ahead of another there.
// ---------------------------------------------------------------------------
template <int D>
struct DqCfg {
  static constexpr int BM = 128;  // queries per CTA
  static constexpr int BN = 128;  // keys per step
  static constexpr int CH = D / 64;
  static constexpr int TILE = 128 * D * 2;
  static constexpr int KST = 3, VST = 2;   // K ring, V ring
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_DO = OFF_Q + TILE;
  static constexpr int OFF_K = OFF_DO + TILE;
  static constexpr int OFF_V = OFF_K + KST * TILE;
  static constexpr int OFF_BAR = OFF_V + VST * TILE;
  // qdo, kfull[3], kempty[3], vfull[2], vempty[2], s, dp, s_free, dp_free, ds[2], fin
  static constexpr int NBAR = 1 + 2 * KST + 2 * VST + 7;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16;
  static constexpr int THREADS = 320;
  static constexpr int NCOMPUTE = 256;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t COL_S = 0, COL_DP = 128, COL_DQ = 256, COL_DS = 384;
};

template <int D, bool BF>
__global__ void __launch_bounds__(320, 1)
    bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                  const BwdParams p) {
  using C = DqCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (!smem_aligned_or_report(smem_raw, p.err)) return;
  const uint32_t sbase = smem_u32(smem_raw);
  const uint32_t s_q = sbase + C::OFF_Q, s_do = sbase + C::OFF_DO;
  const uint32_t s_kr = sbase + C::OFF_K, s_vr = sbase + C::OFF_V;
  const uint32_t b_qdo = sbase + C::OFF_BAR;
  const uint32_t b_kfull = b_qdo + 8, b_kempty = b_kfull + 8 * C::KST;
  const uint32_t b_vfull = b_kempty + 8 * C::KST, b_vempty = b_vfull + 8 * C::VST;
  const uint32_t b_s = b_vempty + 8 * C::VST, b_dp = b_s + 8, b_sfree = b_dp + 8,
                 b_dpfree = b_sfree + 8, b_ds = b_dpfree + 8, b_fin = b_ds + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem_raw + C::OFF_BAR + C::NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nmb = (p.n + C::BM - 1) / C::BM;
  // grid (B*Hq, query blocks), longest causal rows first
  const int mb = p.causal ? (nmb - 1 - static_cast<int>(blockIdx.y)) : static_cast<int>(blockIdx.y);
  const int m0 = mb * C::BM;
  const int bh = blockIdx.x;
  // tensor-map coordinates: batch, query head, and the kv head it reads
  const int b_i = bh / p.hq, hq_i = bh % p.hq, hk_i = hq_i / p.group;
  const int nblk = (p.n + C::BN - 1) / C::BN;
  const int nkv = p.causal ? min(nblk, mb + 1) : nblk;   // BM == BN
  const Ctl ctl{abort_flag, p.err};
  // block j of K lives in K-ring slot j % 3 (phase (j / 3) & 1), of V in j % 2
  auto kfull = [&](int j) { return b_kfull + 8 * (j % C::KST); };
  auto kempty = [&](int j) { return b_kempty + 8 * (j % C::KST); };
  auto kph = [](int j) { return static_cast<uint32_t>((j / C::KST) & 1); };
  auto vfull = [&](int j) { return b_vfull + 8 * (j % C::VST); };
  auto vempty = [&](int j) { return b_vempty + 8 * (j % C::VST); };
  auto vph = [](int j) { return static_cast<uint32_t>((j / C::VST) & 1); };
  auto k_addr = [&](int j) { return s_kr + (j % C::KST) * C::TILE; };
  auto v_addr = [&](int j) { return s_vr + (j % C::VST) * C::TILE; };

  if (threadIdx.x == 0) {
    mbar_init(b_qdo, 1);
    for (int s = 0; s < C::KST; ++s) {
      mbar_init(b_kfull + 8 * s, 1);
      mbar_init(b_kempty + 8 * s, 1);
    }
    for (int s = 0; s < C::VST; ++s) {
      mbar_init(b_vfull + 8 * s, 1);
      mbar_init(b_vempty + 8 * s, 1);
    }
    mbar_init(b_s, 1);
    mbar_init(b_dp, 1);
    mbar_init(b_sfree, C::NCOMPUTE);
    mbar_init(b_dpfree, C::NCOMPUTE);
    mbar_init(b_ds, C::NCOMPUTE);
    mbar_init(b_ds + 8, C::NCOMPUTE);
    mbar_init(b_fin, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 9) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      mbar_arrive_expect_tx(b_qdo, 2 * C::TILE);
#pragma unroll
      for (int c = 0; c < C::CH; ++c) {
        tma_load_4d(s_q + c * 16384, &tm_q, b_qdo, c * 64, m0, hq_i, b_i);
        tma_load_4d(s_do + c * 16384, &tm_do, b_qdo, c * 64, m0, hq_i, b_i);
      }
      bool ok = true;
      int loaded_k = 0, loaded_v = 0;
      constexpr int kAhead = 3;  // L2 prefetch distance, in key blocks
      for (int j = 0; j < kAhead && j < nkv; ++j)
        for (int c = 0; c < C::CH; ++c) {
          tma_prefetch_l2_4d(&tm_k, c * 64, j * C::BN, hk_i, b_i);
          tma_prefetch_l2_4d(&tm_v, c * 64, j * C::BN, hk_i, b_i);
        }
      for (int j = 0; j < nkv && ok; ++j) {
        if (j + kAhead < nkv)
          for (int c = 0; c < C::CH; ++c) {
            tma_prefetch_l2_4d(&tm_k, c * 64, (j + kAhead) * C::BN, hk_i, b_i);
            tma_prefetch_l2_4d(&tm_v, c * 64, (j + kAhead) * C::BN, hk_i, b_i);
          }
        ok = mbar_wait(kempty(j), kph(j) ^ 1, ctl, kErrTimeoutLoad);
        if (!ok) break;
        mbar_arrive_expect_tx(kfull(j), C::TILE);
#pragma unroll
        for (int c = 0; c < C::CH; ++c)
          tma_load_4d(k_addr(j) + c * 16384, &tm_k, kfull(j), c * 64, j * C::BN, hk_i, b_i);
        ++loaded_k;
        ok = mbar_wait(vempty(j), vph(j) ^ 1, ctl, kErrTimeoutLoad);
        if (!ok) break;
        mbar_arrive_expect_tx(vfull(j), C::TILE);
#pragma unroll
        for (int c = 0; c < C::CH; ++c)
          tma_load_4d(v_addr(j) + c * 16384, &tm_v, vfull(j), c * 64, j * C::BN, hk_i, b_i);
        ++loaded_v;
      }
      if (!ok) {
        drain_loads(b_qdo, 1, 1);
        drain_loads(b_kfull, loaded_k, C::KST);
        drain_loads(b_vfull, loaded_v, C::VST);
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && nkv > 0) {
      constexpr uint32_t id_s = idesc_f16(128, 128, false, false, BF);
      constexpr uint32_t id_q = idesc_f16(128, D, false, true, BF);
      auto issue_t = [&](uint32_t d_tmem, uint32_t a_s, uint32_t b_s_) {
        const uint64_t da = sdesc_sw128(a_s, 16, 1024), db = sdesc_sw128(b_s_, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          mma_ss(d_tmem, sdesc_add(da, off), sdesc_add(db, off), id_s, kk > 0 ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(b_qdo, 0, ctl, kErrTimeoutMma);
      if (ok) ok = mbar_wait(kfull(0), 0, ctl, kErrTimeoutMma);
      if (ok) {
        tc_fence_after();
        issue_t(tmem + C::COL_S, s_q, k_addr(0));
        mma_commit(b_s);
        ok = mbar_wait(vfull(0), 0, ctl, kErrTimeoutMma);
      }
      if (ok) {
        tc_fence_after();
        issue_t(tmem + C::COL_DP, s_do, v_addr(0));
        mma_commit(b_dp);
        mma_commit(vempty(0));  // V_0 no longer needed
      }
      for (int j = 0; j < nkv && ok; ++j) {
        if (j + 1 < nkv) {
          ok = mbar_wait(b_sfree, j & 1, ctl, kErrTimeoutMma) &&
               mbar_wait(kfull(j + 1), kph(j + 1), ctl, kErrTimeoutMma);
          if (!ok) break;
          tc_fence_after();
          issue_t(tmem + C::COL_S, s_q, k_addr(j + 1));
          mma_commit(b_s);
          ok = mbar_wait(b_dpfree, j & 1, ctl, kErrTimeoutMma) &&
               mbar_wait(vfull(j + 1), vph(j + 1), ctl, kErrTimeoutMma);
          if (!ok) break;
          tc_fence_after();
          issue_t(tmem + C::COL_DP, s_do, v_addr(j + 1));
          mma_commit(b_dp);
          mma_commit(vempty(j + 1));  // V_{j+1} no longer needed
        }
        ok = mbar_wait(b_ds + 8 * (j & 1), (j >> 1) & 1, ctl, kErrTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t ds_t = tmem + C::COL_DS + 64 * (j & 1);
        const uint64_t dkb = sdesc_sw128(k_addr(j), 16384, 1024);
#pragma unroll
        for (int kk = 0; kk < C::BN / 16; ++kk)
          mma_ts(tmem + C::COL_DQ, ds_t + kk * 8, sdesc_add(dkb, kk * 2048), id_q,
                 (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(kempty(j));  // K_j no longer needed
      }
      mma_commit(b_fin);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(b_fin, 0) && globaltimer_ns() - t0 < FAB_WAIT_LIMIT_NS) {
      }
    }
  } else {
    // ------------------------------------------------------------ compute (warps 0-7)
    const int w = warp >> 2;
    const int r = threadIdx.x & 127;
    const int row = m0 + r;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    // padded rows (row >= N) read -LSE*log2e = -inf, Dv = 0: their P and dS are 0
    const size_t prow = static_cast<size_t>(bh) * p.n_pad + row;
    const float nlse2 = p.lse2[prow];   // -LSE * log2(e)
    const float ndvs = p.dvec[prow];    // -Dv * scale
    const int klim = p.causal ? min(p.n - 1, row) : (p.n - 1);  // key live iff key <= klim
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const uint32_t ph = j & 1;
      ok = mbar_wait(b_s, ph, ctl, kErrTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[2][32];
      tmem_ld32(tmem + C::COL_S + 64 * w + lane_off, sr[0]);
      tmem_ld32(tmem + C::COL_S + 64 * w + 32 + lane_off, sr[1]);
      tmem_ld_wait_only();
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 32; ++c) asm volatile("" : "+r"(sr[h][c]));
      tc_fence_before();
      mbar_arrive(b_sfree);
      float pv[2][32];
      const int kv0 = j * C::BN + 64 * w;
      const bool need_mask = kv0 + 63 > klim;
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 32; ++c)
          pv[h][c] = ex2(fmaf(__uint_as_float(sr[h][c]), p.scale_log2, nlse2));
      if (need_mask) {  // only the diagonal block and the ragged tail
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (kv0 + 32 * h + c > klim) pv[h][c] = 0.f;
      }
      ok = mbar_wait(b_dp, ph, ctl, kErrTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      tmem_ld32(tmem + C::COL_DP + 64 * w + lane_off, sr[0]);
      tmem_ld32(tmem + C::COL_DP + 64 * w + 32 + lane_off, sr[1]);
      tmem_ld_wait_only();
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 32; ++c) asm volatile("" : "+r"(sr[h][c]));
      tc_fence_before();
      mbar_arrive(b_dpfree);
      // dS = P * (scale * dP - Dv * scale), packed two fp16 per 32-bit TMEM
      // column: this group's 64 keys are columns 32w..32w+31 of buffer j&1
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 32; ++c) pv[h][c] *= fmaf(__uint_as_float(sr[h][c]), p.scale, ndvs);
      tmem_st_pairs<BF>(tmem + C::COL_DS + 64 * (j & 1) + 32 * w + lane_off, pv);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(b_ds + 8 * (j & 1));
    }
    if (ok && nkv > 0) {
      ok = mbar_wait(b_fin, 0, ctl, kErrTimeoutEpilogue);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        const long long rowoff = p.sdq.at(b_i, hq_i, row);
#pragma unroll 1
        for (int c = 0; c < D / 64; ++c) {
          const int col = w * (D / 2) + 32 * c;
          uint32_t v[32];
          tmem_ld32_sync(tmem + C::COL_DQ + col + lane_off, v);
          if (row < p.n) {
            if (p.dq_fp32)
              store_row32_f32(static_cast<float*>(p.dq) + rowoff + col, v, 1.f);
            else
              store_row32_h<BF>(static_cast<uint16_t*>(p.dq) + rowoff + col, v, 1.f);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 8) {
    __syncwarp();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace fab


namespace fab {

// ---------------------------------------------------------------------------
// Fused dK / dV / dQ in one pass: the key-stationary CTA of the dK/dV kernel
// (128 keys, looping over the GQA group and the query blocks) also forms each
// step's dQ contribution dQ_i = dS_i K and adds it into a zeroed fp32 dQ, as
// the reference does with atomicAdd (flash_bwd.cuh:378-444) -- but with no
// recompute of S and dP in a second kernel, and the adds done by the TMA unit:
// a read-out warpgroup stages dQ_i as 32-row x 32-column fp32 boxes (4 KiB,
// swizzled) in shared memory and issues one tiled reduce-add per box into
// global memory, so the adds are coalesced 128-byte rows and run
// asynchronously. The add order varies from run to run, so dQ is not bitwise
// deterministic.
//   warps 0-7   compute: two warpgroups; thread r is key row r for P and dS;
//               group w owns queries 64w.. of each step
//   warps 8-11  dQ read-out: warp 8+q reads TMEM lanes 32q.. (query rows) of
//               dQ_i, frees the columns, then stages and adds its boxes
//   warp  12    TMEM allocation + MMA issue
//   warp  13    TMA producer: K, V once; then Q_i (+ LSE/Dv slices), dO_i
//   warps 14-15 idle (they complete the last warpgroup)
// Registers are launched at 128 a thread and rebalanced per warpgroup
// (setmaxnreg): compute 160, read-out 144, the MMA/TMA warpgroup 48; per lane
// of an SMSP 160 + 160 + 144 + 48 = 512 = the 4 x 128 launched.
// TMEM: S^T 0..127, with P^T (fp16 pairs) written back over cols 32..95 |
//       dP^T 128..255, then (D = 128) dQ_i | dV 256.. | dK 256+D.. |
//       (D = 64) dQ 384..
// Shared: K, V, a 2-slot Q ring and a 1-slot (D = 64: 2-slot) dO ring, the dS
// tile [key][query], two 4 KiB dQ staging boxes per read-out warp, LSE/Dv
// slices for two steps.
// MMA order per step i (brackets = what it waits for):
//   [P_i] dV_i = P^T dO (A in TMEM) ; [Q_{i+1}] S^T_{i+1} ;
//   [dS_i] dQ_i = dS K (A = the dS tile read MN-major, into the dP^T
//   columns), dK_i = dS^T Q (A = the same tile read K-major) ;
//   [dQ_i read, dO_{i+1}] dP^T_{i+1}   (D = 128; with D = 64 dQ has columns
//   of its own and the dQ_i read gates dQ_{i+1} instead)
// and the compute warps run dS_i, then P_{i+1}, so that the P phase of the
// next step overlaps dQ_i and dK_i on the tensor core; the read-out warps take
// dQ_i off the tensor memory while dK_i runs, so dP^T_{i+1} rarely waits.
// Overwrites follow issue order (S^T_{i+1} after dV_i read P_i; dQ_i after
// the compute threads read dP_i; dP^T_{i+1} after the read-out warps read
// dQ_i). The dS
// tile is rewritten for step i+1 only after dP^T_{i+1} completed, which was
// issued after dQ_i and dK_i. The Q slot of step i is released after dK_i,
// so the LSE/Dv slice buffer i & 1, loaded with Q, is reloaded (for step i+2)
// only after every compute thread finished step i; the dO slot of step i is
// released after dV_i, which gives the load of dO_{i+1} the rest of step i.
// ---------------------------------------------------------------------------
template <int D>
struct FusedCfg {
  static constexpr int BN = 128, BM = 128, CH = D / 64;
  static constexpr int TILE = 128 * D * 2;
  // Q and dO tiles live in two rings: QS slots for Q (a Q slot frees when
  // dK_i has read it) and OS for dO (free once dV_i has read it, early in the
  // step, so dO_{i+1} has most of a step to arrive before dP^T_{i+1})
  static constexpr int STAGES = (D == 64) ? 4 : 3;
  static constexpr int QS = 2, OS = STAGES - QS;
  static_assert(QS == 2, "the LSE/Dv slice buffers are double-buffered with the Q ring");
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + TILE;
  static constexpr int OFF_RING = OFF_V + TILE;
  static constexpr int OFF_DS = OFF_RING + STAGES * TILE;    // 128 keys x 128 queries fp16
  static constexpr int OFF_STG = OFF_DS + 32768;             // 4 warps x 2 x (32 rows x 32 fp32)
  static constexpr int OFF_LSE = OFF_STG + 8 * 4096;         // [2][128] LSE*log2e, [2][128] Dv*scale
  static constexpr int OFF_BAR = OFF_LSE + 2048;
  // k, full[ST], empty[ST], s, dp, p, ds, dqfull, dqfree, fin, v
  static constexpr int NBAR = 1 + 2 * STAGES + 8;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16;     // window must start 1024-aligned
  static_assert(SMEM <= 232448, "shared memory over the per-block limit");
  static constexpr int THREADS = 512;
  static constexpr int NCOMPUTE = 256, NREADOUT = 128;
  static constexpr int MMA_WARP = 12, TMA_WARP = 13;
  static constexpr int REGS_COMPUTE = 144, REGS_READOUT = 152, REGS_CONTROL = 72;
  static_assert(2 * REGS_COMPUTE + REGS_READOUT + REGS_CONTROL <= 4 * 128,
                "warpgroup register budgets exceed the 128 per thread launched");
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t COL_S = 0, COL_DP = 128, COL_DV = 256, COL_DK = 256 + D;
  // D = 128 fills TMEM, so dQ_i goes into the dP^T columns and dP^T_{i+1}
  // waits for it to be read out; D = 64 leaves columns 384.. free for a dQ of
  // its own, and only dQ_{i+1} waits for the read-out of dQ_i.
  static constexpr bool DQ_OWN_COLS = (D == 64);
  static constexpr uint32_t COL_P = 32, COL_DQ = DQ_OWN_COLS ? 384 : 128;
};

template <int D, bool BF>
__global__ void __launch_bounds__(512, 1)
    bwd_fused_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                     const __grid_constant__ CUtensorMap tm_dq,
                     const __grid_constant__ CUtensorMap tm_dka,
                     const __grid_constant__ CUtensorMap tm_dva,
                     const __grid_constant__ CUtensorMap tm_dk, const __grid_constant__ CUtensorMap tm_dv,
                     const BwdParams p) {
  using C = FusedCfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (!smem_aligned_or_report(smem_raw, p.err)) return;
  const uint32_t sbase = smem_u32(smem_raw);
  const uint32_t s_k = sbase + C::OFF_K, s_v = sbase + C::OFF_V, s_ring = sbase + C::OFF_RING;
  const uint32_t s_ds = sbase + C::OFF_DS, s_lse = sbase + C::OFF_LSE;
  const uint32_t b_kv = sbase + C::OFF_BAR;
  const uint32_t b_full = b_kv + 8, b_empty = b_full + 8 * C::STAGES;
  const uint32_t b_s = b_empty + 8 * C::STAGES, b_dp = b_s + 8, b_p = b_dp + 8, b_ds = b_p + 8,
                 b_dqfull = b_ds + 8, b_dqfree = b_dqfull + 8, b_fin = b_dqfree + 8,
                 b_v = b_fin + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem_raw + C::OFF_BAR + C::NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1-D grid over (batch, kv-head) slices x key blocks, scheduled in groups of
  // p.head_group slices (the host weighs the groups' L2 footprint against the
  // tail of long CTAs that start late); inside a group the causal key block 0
  // of every slice (the most work) goes first, then block 1, and so on. CTAs
  // that run together work on the group's slices, so the Q/dO tiles they share
  // and the dQ rows they add into are L2 hits rather than DRAM round trips.
  // With p.gsplit > 1 the heads of one GQA group are split over gsplit
  // consecutive CTAs (gper heads each), which add their dK/dV into fp32.
  const int nkb = (p.n + C::BN - 1) / C::BN;
  const int hkv = p.hq / p.group;
  const int split = static_cast<int>(blockIdx.x) % p.gsplit;
  const int unit = static_cast<int>(blockIdx.x) / p.gsplit;
  int bkv, kvb;
  {
    const int per_group = p.head_group * nkb;
    const int g0 = unit / per_group;
    const int r = unit - g0 * per_group;
    const int n_bkv = gridDim.x / (nkb * p.gsplit);     // B * Hkv
    const int hg = min(p.head_group, n_bkv - g0 * p.head_group);
    kvb = r / hg;
    bkv = g0 * p.head_group + r % hg;
  }
  const int gh0 = split * p.gper;                       // this CTA's first head of the group
  const int gcount = min(p.gper, p.group - gh0);
  const int b = bkv / hkv, kvh = bkv % hkv;
  const int kv0 = kvb * C::BN;
  const int nqb = (p.n + C::BM - 1) / C::BM;
  const int i_start = p.causal ? kvb : 0;   // BM == BN: the diagonal block
  const int nq_head = nqb - i_start;
  const int total = gcount * nq_head;       // (group head, query block) steps
  const Ctl ctl{abort_flag, p.err};
  // Q_i in ring slot i % QS, dO_i in slot QS + i % OS; phase = use count & 1
  auto q_slot = [](int i) { return i % C::QS; };
  auto q_ph = [](int i) { return static_cast<uint32_t>((i / C::QS) & 1); };
  auto o_slot = [](int i) { return C::QS + i % C::OS; };
  auto o_ph = [](int i) { return static_cast<uint32_t>((i / C::OS) & 1); };

  if (threadIdx.x == 0) {
    mbar_init(b_kv, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(b_full + 8 * s, 1);
      mbar_init(b_empty + 8 * s, 1);
    }
    mbar_init(b_s, 1);
    mbar_init(b_dp, 1);
    mbar_init(b_p, C::NCOMPUTE);
    mbar_init(b_ds, C::NCOMPUTE);
    mbar_init(b_dqfull, 1);
    mbar_init(b_dqfree, C::NREADOUT);
    mbar_init(b_fin, 1);
    mbar_init(b_v, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == C::MMA_WARP) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= C::MMA_WARP) {
    regs_lower<C::REGS_CONTROL>();
  }
  if (warp == C::TMA_WARP) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      // K first and V after Q_0: S^T_0 needs K and Q_0, dP^T_0 V and dO_0
      mbar_arrive_expect_tx(b_kv, C::TILE);
#pragma unroll
      for (int c = 0; c < C::CH; ++c) tma_load_4d(s_k + c * 16384, &tm_k, b_kv, c * 64, kv0, kvh, b);
      bool v_issued = false;
      int nq = 0, ndo = 0;       // loads issued into the Q and the dO ring
      bool ok = true;
      constexpr int kAhead = 2;  // L2 prefetch distance, in query steps
      auto prefetch_step = [&](int st) {
        const int q0p = (i_start + st % nq_head) * C::BM;
        const int hqp = kvh * p.group + gh0 + st / nq_head;
        for (int c = 0; c < C::CH; ++c) {
          tma_prefetch_l2_4d(&tm_q, c * 64, q0p, hqp, b);
          tma_prefetch_l2_4d(&tm_do, c * 64, q0p, hqp, b);
        }
      };
      for (int st = 0; st < kAhead && st < total; ++st) prefetch_step(st);
      for (int step = 0; step < total && ok; ++step) {
        const int g = gh0 + step / nq_head;
        const int q0 = (i_start + step % nq_head) * C::BM;
        const int hq_g = kvh * p.group + g;
        const int bh = b * p.hq + hq_g;
        if (step + kAhead < total) prefetch_step(step + kAhead);
        // Q_step with its LSE and Dv slices: the slot frees when dK_{step-2}
        // has read it, after every compute thread finished step-2, so the
        // slice buffer step & 1 is free as well
        {
          const int slot = q_slot(step);
          ok = mbar_wait(b_empty + 8 * slot, q_ph(step) ^ 1, ctl, kErrTimeoutLoad);
          if (!ok) break;
          const uint32_t fb = b_full + 8 * slot;
          const uint32_t dst = s_ring + slot * C::TILE;
          mbar_arrive_expect_tx(fb, C::TILE + 1024);
#pragma unroll
          for (int c = 0; c < C::CH; ++c) tma_load_4d(dst + c * 16384, &tm_q, fb, c * 64, q0, hq_g, b);
          const size_t off = static_cast<size_t>(bh) * p.n_pad + q0;
          const uint32_t ls = s_lse + (step & 1) * 512;
          bulk_load(ls, p.lse2 + off, 512, fb);
          bulk_load(ls + 1024, p.dvec + off, 512, fb);
          ++nq;
        }
        if (!v_issued) {
          mbar_arrive_expect_tx(b_v, C::TILE);
#pragma unroll
          for (int c = 0; c < C::CH; ++c) tma_load_4d(s_v + c * 16384, &tm_v, b_v, c * 64, kv0, kvh, b);
          v_issued = true;
        }
        // dO_step: the slot frees when dV_{step-OS} has read it
        {
          const int slot = o_slot(step);
          ok = mbar_wait(b_empty + 8 * slot, o_ph(step) ^ 1, ctl, kErrTimeoutLoad);
          if (!ok) break;
          const uint32_t fb = b_full + 8 * slot;
          const uint32_t dst = s_ring + slot * C::TILE;
          mbar_arrive_expect_tx(fb, C::TILE);
#pragma unroll
          for (int c = 0; c < C::CH; ++c) tma_load_4d(dst + c * 16384, &tm_do, fb, c * 64, q0, hq_g, b);
          ++ndo;
        }
      }
      if (!ok) {
        drain_loads(b_kv, 1, 1);
        if (v_issued) drain_loads(b_v, 1, 1);
        drain_loads(b_full, nq, C::QS);
        drain_loads(b_full + 8 * C::QS, ndo, C::OS);
      }
    }
  } else if (warp == C::MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && total > 0) {
      constexpr uint32_t id_t = idesc_f16(128, 128, false, false, BF);  // S^T, dP^T
      constexpr uint32_t id_g = idesc_f16(128, D, false, true, BF);     // dV (TS), dK (SS)
      constexpr uint32_t id_q = idesc_f16(128, D, true, true, BF);      // dQ: A = dS MN-major
      // X^T = (K or V) (Q or dO)^T: 128 x 128, K = D
      auto issue_t = [&](uint32_t d_tmem, uint32_t a_s, uint32_t b_s_) {
        const uint64_t da = sdesc_sw128(a_s, 16, 1024), db = sdesc_sw128(b_s_, 16, 1024);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          mma_ss(d_tmem, sdesc_add(da, off), sdesc_add(db, off), id_t, kk > 0 ? 1u : 0u);
        }
      };
      auto slot_addr = [&](int slot) { return s_ring + slot * C::TILE; };
      const uint64_t d_dsm = sdesc_sw128(s_ds, 16384, 1024);    // dS tile as MN-major A (dQ)
      const uint64_t d_dsk = sdesc_sw128(s_ds, 16, 1024);       // dS^T, K-major A (dK)
      const uint64_t d_kmn = sdesc_sw128(s_k, 16384, 1024);     // K as MN-major B
      bool ok = mbar_wait(b_kv, 0, ctl, kErrTimeoutMma);
      if (ok) ok = mbar_wait(b_full + 8 * q_slot(0), q_ph(0), ctl, kErrTimeoutMma);
      if (ok) {
        tc_fence_after();
        issue_t(tmem + C::COL_S, s_k, slot_addr(q_slot(0)));
        mma_commit(b_s);
        ok = mbar_wait(b_v, 0, ctl, kErrTimeoutMma) &&
             mbar_wait(b_full + 8 * o_slot(0), o_ph(0), ctl, kErrTimeoutMma);
      }
      if (ok) {
        tc_fence_after();
        issue_t(tmem + C::COL_DP, s_v, slot_addr(o_slot(0)));
        mma_commit(b_dp);
      }
      for (int i = 0; i < total && ok; ++i) {
        const bool more = i + 1 < total;
        // dV_i += P_i^T dO_i
        ok = mbar_wait(b_p, i & 1, ctl, kErrTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        {
          const uint64_t ddo = sdesc_sw128(slot_addr(o_slot(i)), 16384, 1024);
#pragma unroll
          for (int kk = 0; kk < C::BM / 16; ++kk)
            mma_ts(tmem + C::COL_DV, tmem + C::COL_P + kk * 8, sdesc_add(ddo, kk * 2048), id_g,
                   (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(b_empty + 8 * o_slot(i));
        // S^T_{i+1}: its P phase overlaps dK_i and dQ_i
        if (more) {
          ok = mbar_wait(b_full + 8 * q_slot(i + 1), q_ph(i + 1), ctl, kErrTimeoutMma);
          if (!ok) break;
          tc_fence_after();
          issue_t(tmem + C::COL_S, s_k, slot_addr(q_slot(i + 1)));
          mma_commit(b_s);
        }
        // dQ_i = dS_i K, then dK_i += dS_i^T Q_i, both reading dS_i from the
        // shared tile: dQ_i completes first, so its read-out overlaps dK_i and
        // dP^T_{i+1} (which reuses the dQ_i columns when D = 128) need not wait
        ok = mbar_wait(b_ds, i & 1, ctl, kErrTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        if (C::DQ_OWN_COLS && i > 0) {   // dQ_{i-1} has been read out of its columns
          ok = mbar_wait(b_dqfree, (i - 1) & 1, ctl, kErrTimeoutMma);
          if (!ok) break;
          tc_fence_after();
        }
#pragma unroll
        for (int kk = 0; kk < C::BN / 16; ++kk)
          mma_ss(tmem + C::COL_DQ, sdesc_add(d_dsm, kk * 2048), sdesc_add(d_kmn, kk * 2048), id_q,
                 kk > 0 ? 1u : 0u);
        mma_commit(b_dqfull);
        {
          const uint64_t dq_mn = sdesc_sw128(slot_addr(q_slot(i)), 16384, 1024);
#pragma unroll
          for (int kk = 0; kk < C::BM / 16; ++kk)
            mma_ss(tmem + C::COL_DK, sdesc_add(d_dsk, (kk >> 2) * 16384 + (kk & 3) * 32),
                   sdesc_add(dq_mn, kk * 2048), id_g, (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(b_empty + 8 * q_slot(i));
        if (more) {
          ok = (C::DQ_OWN_COLS || mbar_wait(b_dqfree, i & 1, ctl, kErrTimeoutMma)) &&
               mbar_wait(b_full + 8 * o_slot(i + 1), o_ph(i + 1), ctl, kErrTimeoutMma);
          if (!ok) break;
          tc_fence_after();
          issue_t(tmem + C::COL_DP, s_v, slot_addr(o_slot(i + 1)));
          mma_commit(b_dp);
        }
      }
      mma_commit(b_fin);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(b_fin, 0) && globaltimer_ns() - t0 < FAB_WAIT_LIMIT_NS) {
      }
    }
  } else if (warp >= 8 && warp < 12) {
    regs_raise<C::REGS_READOUT>();
    // ------------------------------------------------------------ dQ read-out (warps 8-11)
    // Warp 8+q takes TMEM lanes 32q.. (query rows qb0+32q..) of dQ_i, all D
    // columns, frees the columns for dP^T_{i+1}, then stages its D/32 boxes of
    // 32 x 32 fp32 through two alternating 4 KiB buffers and adds each into dQ
    // with a TMA reduce-add. Before staging a box the warp waits until the TMA
    // unit has read the box staged two earlier in the same buffer, so each
    // warp keeps at most two boxes queued (the L2 accepts the adds slowly, and
    // a warp that waited for each box before staging the next fell behind the
    // tensor core); a warp with no rows below N stages nothing.
    const int q = warp & 3;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t stg = sbase + C::OFF_STG + (warp - 8) * 8192;
    constexpr int NB = D / 32;
    bool ok = true;
    for (int i = 0; i < total && ok; ++i) {
      const int qb0 = (i_start + i % nq_head) * C::BM;
      const int bh = b * p.hq + kvh * p.group + gh0 + i / nq_head;
      ok = mbar_wait(b_dqfull, i & 1, ctl, kErrTimeoutEpilogue);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t v[NB][32];
#pragma unroll
      for (int h = 0; h < NB; ++h) tmem_ld32(tmem + C::COL_DQ + 32 * h + lane_off, v[h]);
      tmem_ld_wait_only();
#pragma unroll
      for (int h = 0; h < NB; ++h)
#pragma unroll
        for (int c = 0; c < 32; ++c) asm volatile("" : "+r"(v[h][c]));
      tc_fence_before();
      mbar_arrive(b_dqfree);     // dP^T_{i+1} may overwrite the dQ_i columns
      const int row0 = qb0 + 32 * q;
      if (row0 >= p.n) continue;   // every row of this box is past N
#pragma unroll
      for (int h = 0; h < NB; ++h) {
        const uint32_t box = stg + (h & 1) * 4096;
        if (lane == 0) bulk_wait_read_all_but_last();   // the buffer's previous box has been read
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 8; ++c)
          st_shared_v4(box + lane * 128 + ((c ^ (lane & 7)) << 4), v[h][4 * c], v[h][4 * c + 1],
                       v[h][4 * c + 2], v[h][4 * c + 3]);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_4d(&tm_dq, box, 32 * h, row0, bh % p.hq, bh / p.hq);
          bulk_commit_group();
        }
      }
    }
    if (lane == 0) bulk_wait_read_all();   // the TMA unit has read every staged dQ box
  } else if (warp < 8) {
    regs_raise<C::REGS_COMPUTE>();
    // ------------------------------------------------------------ compute (warps 0-7)
    const int w = warp >> 2;            // query half of each step
    const int r = threadIdx.x & 127;    // key row within the block
    const int kvrow = kv0 + r;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int qlim = p.causal ? kvrow : -1;  // a query column is live iff qlim <= q < N
    uint32_t sr[2][32];
    float pv[2][32];

    // P_i^T = exp2(S^T * scale*log2e - LSE*log2e), written over S^T in TMEM
    auto phase_p = [&](int i) -> bool {
      const int q0 = (i_start + i % nq_head) * C::BM + 64 * w;
      const bool need_mask = (q0 + 64 > p.n) || (p.causal && q0 < kv0 + 127);
      bool ok = mbar_wait(b_full + 8 * q_slot(i), q_ph(i), ctl, kErrTimeoutSoftmax) &&
                mbar_wait(b_s, i & 1, ctl, kErrTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) return false;
      tc_fence_after();
      tmem_ld32(tmem + C::COL_S + 64 * w + lane_off, sr[0]);
      tmem_ld32(tmem + C::COL_S + 64 * w + 32 + lane_off, sr[1]);
      tmem_ld_wait_only();
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 32; ++c) asm volatile("" : "+r"(sr[h][c]));
      const float4* lse4 =
          reinterpret_cast<const float4*>(smem_raw + C::OFF_LSE) + ((i & 1) * 128 + 64 * w) / 4;
      const uint64_t sl2 = f32x2(p.scale_log2, p.scale_log2);
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const float4 l4 = lse4[8 * h + c4];   // -LSE*log2e of 4 query columns
#pragma unroll
          for (int e2 = 0; e2 < 2; ++e2) {
            const int c = 4 * c4 + 2 * e2;
            const float2 x = f32x2_split(
                fma_x2(f32x2(__uint_as_float(sr[h][c]), __uint_as_float(sr[h][c + 1])), sl2,
                       e2 ? f32x2(l4.z, l4.w) : f32x2(l4.x, l4.y)));
            pv[h][c] = ex2(x.x);
            pv[h][c + 1] = ex2(x.y);
          }
        }
      if (need_mask) {
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const int q = q0 + 32 * h + c;
            if (q < qlim || q >= p.n) pv[h][c] = 0.f;
          }
      }
      tmem_st_pairs<BF>(tmem + C::COL_P + 32 * w + lane_off, pv);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(b_p);
      return true;
    };

    // dS_i^T = P^T o (dP^T * scale - Dv*scale), into TMEM (for dK) and the
    // shared [key][query] tile (for dQ)
    auto phase_ds = [&](int i) -> bool {
      bool ok = mbar_wait(b_dp, i & 1, ctl, kErrTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) return false;
      tc_fence_after();
      tmem_ld32(tmem + C::COL_DP + 64 * w + lane_off, sr[0]);
      tmem_ld32(tmem + C::COL_DP + 64 * w + 32 + lane_off, sr[1]);
      tmem_ld_wait_only();
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 32; ++c) asm volatile("" : "+r"(sr[h][c]));
      const float4* dvs4 =
          reinterpret_cast<const float4*>(smem_raw + C::OFF_LSE) + ((i & 1) * 128 + 64 * w) / 4 + 64;
      const uint64_t sc2 = f32x2(p.scale, p.scale);
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const float4 d4 = dvs4[8 * h + c4];   // -Dv*scale of 4 query columns
#pragma unroll
          for (int e2 = 0; e2 < 2; ++e2) {
            const int c = 4 * c4 + 2 * e2;
            const uint64_t t = fma_x2(f32x2(__uint_as_float(sr[h][c]), __uint_as_float(sr[h][c + 1])),
                                      sc2, e2 ? f32x2(d4.z, d4.w) : f32x2(d4.x, d4.y));
            const float2 ds = f32x2_split(mul_x2(f32x2(pv[h][c], pv[h][c + 1]), t));
            pv[h][c] = ds.x;
            pv[h][c + 1] = ds.y;
          }
        }
      // dS^T rows into the shared [key][query] tile, the A operand of dK
      // (K-major) and of dQ (MN-major)
      st_row32_sw128<BF>(s_ds + w * 16384, r, 0, pv[0]);
      st_row32_sw128<BF>(s_ds + w * 16384, r, 1, pv[1]);
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(b_ds);
      return true;
    };

    bool ok = true;
    if (total > 0) ok = phase_p(0);
    for (int i = 0; i < total && ok; ++i) {
      ok = phase_ds(i);
      if (ok && i + 1 < total) ok = phase_p(i + 1);
    }
    if (ok && total > 0) {
      ok = mbar_wait(b_fin, 0, ctl, kErrTimeoutEpilogue);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        if (!p.dkv_reduce) {
          // dV and dK rounded to 16 bits, staged as 64-column swizzled boxes in
          // the idle Q/dO ring (every load and MMA has completed) and written
          // by TMA stores: whole 128-byte rows instead of one row per thread
#pragma unroll 1
          for (int t = 0; t < 2; ++t)
#pragma unroll 1
            for (int c = 0; c < D / 64; ++c) {
              const int col = w * (D / 2) + 32 * c;
              uint32_t v[32];
              tmem_ld32_sync(tmem + (t ? C::COL_DK : C::COL_DV) + col + lane_off, v);
              float x[32];
#pragma unroll
              for (int e = 0; e < 32; ++e) x[e] = __uint_as_float(v[e]);
              st_row32_sw128<BF>(s_ring + t * C::TILE + (col / 64) * 16384, r, (col % 64) / 32, x);
            }
        } else {
          // dK/dV added in fp32 into the accumulators of tm_dka / tm_dva (a
          // split group's partial sums, or a caller accumulating over calls):
          // 32-row x 32-column boxes staged in the ring and dS tile (idle now:
          // every load and MMA has completed; the read-out warps' staging
          // buffers lie beyond them) and added by TMA reduce-adds
          constexpr int NB = D / 64;               // boxes per tensor per warp
          const uint32_t wbox = s_ring + warp * (2 * NB * 4096);
          const int krow0 = kv0 + 32 * (warp & 3);
#pragma unroll 1
          for (int t = 0; t < 2; ++t) {
#pragma unroll 1
            for (int c = 0; c < NB; ++c) {
              uint32_t v[32];
              tmem_ld32_sync(tmem + (t ? C::COL_DV : C::COL_DK) + w * (D / 2) + 32 * c + lane_off, v);
              const uint32_t box = wbox + (t * NB + c) * 4096;
#pragma unroll
              for (int c4 = 0; c4 < 8; ++c4)
                st_shared_v4(box + lane * 128 + ((c4 ^ (lane & 7)) << 4), v[4 * c4], v[4 * c4 + 1],
                             v[4 * c4 + 2], v[4 * c4 + 3]);
            }
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0 && krow0 < p.n) {
#pragma unroll 1
            for (int t = 0; t < 2; ++t)
#pragma unroll 1
              for (int c = 0; c < NB; ++c)
                tma_reduce_add_4d(t ? (const void*)&tm_dva : (const void*)&tm_dka,
                                  wbox + (t * NB + c) * 4096, w * (D / 2) + 32 * c, krow0, kvh, b);
            bulk_commit_group();
            bulk_wait_read_all();   // boxes read: shared memory may be released
          }
        }
      }
    }
    if (!p.dkv_reduce) {
      // every compute thread gets here once, whichever path it took above; a
      // thread that skipped its staging raised the abort flag first
      fence_async_smem();
      named_bar_sync(1, C::NCOMPUTE);
      if (threadIdx.x == 0 && total > 0 && *abort_flag == 0) {
#pragma unroll 1
        for (int t = 0; t < 2; ++t)
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c)
            tma_store_4d(t ? (const void*)&tm_dk : (const void*)&tm_dv, s_ring + t * C::TILE + c * 16384,
                         64 * c, kv0, kvh, b);
        bulk_commit_group();
        bulk_wait_read_all();   // boxes read: shared memory may be released
      }
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

// The split fused backward's fp32 dK/dV accumulator -- (2B, Hkv, N, D), dK in
// batches 0..B-1 and dV in B..2B-1 -- rounded to the 16-bit dk, dv (fp16, or bf16
// when BF) in their own layouts. HBM-bound: one 32-byte read and one 16-byte
// write per thread.
template <bool BF>
__global__ void __launch_bounds__(256) bwd_dkv_convert_kernel(const float* __restrict__ acc,
                                                               uint16_t* __restrict__ dk, Strides sdk,
                                                               uint16_t* __restrict__ dv, Strides sdv,
                                                               int B, int hkv, int n, int d,
                                                               long long total) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int per_row = d / 8;
  const long long row = i / per_row;
  const int part = static_cast<int>(i - row * per_row);
  const int r = static_cast<int>(row % n);
  const long long bh = row / n;                    // over (2B, Hkv)
  const int h = static_cast<int>(bh % hkv);
  const int bb = static_cast<int>(bh / hkv);
  const float4* src = reinterpret_cast<const float4*>(acc + row * d) + 2 * part;
  const float4 a = src[0], c = src[1];
  uint4 pk;
  pk.x = pack2<BF>(a.x, a.y);
  pk.y = pack2<BF>(a.z, a.w);
  pk.z = pack2<BF>(c.x, c.y);
  pk.w = pack2<BF>(c.z, c.w);
  uint16_t* dst = bb < B ? dk + sdk.at(bb, h, r) : dv + sdv.at(bb - B, h, r);
  reinterpret_cast<uint4*>(dst)[part] = pk;
}

}  // namespace fab
