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
// result is deterministic. dK/dV come from a key-stationary kernel that loops
// over the GQA group and all query blocks, keeping both accumulators in TMEM
// (as the reference keeps them in registers, flash_bwd.cuh:163, :448-463).
#pragma once
#include "sm100.cuh"

namespace fab {

struct BwdParams {
  const __half* o;     // (B*Hq, N, D) forward output
  const __half* dO;    // (B*Hq, N, D)
  const float* lse;    // (B*Hq, N) natural log
  float* dvec;         // (B*Hq, N) workspace: rowsum(dO o O)
  void* dq;            // (B*Hq, N, D) fp32 or fp16
  __half* dk;          // (B*Hkv, N, D)
  __half* dv;          // (B*Hkv, N, D)
  int* err;
  int n, hq, group, causal;
  int dq_fp32;
  float scale;         // 1/sqrt(D)
  float scale_log2;    // scale * log2(e)
};

// ---------------------------------------------------------------------------
// Dv = rowsum(dO o O): HBM-bound, one 16-byte vector per thread, D/8 threads
// per row reduced with shuffles.
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) bwd_preprocess_kernel(const __half* __restrict__ o,
                                                              const __half* __restrict__ dO,
                                                              float* __restrict__ dvec,
                                                              long long rows) {
  constexpr int TPR = D / 8;  // threads per row (8 or 16)
  const long long gtid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long row = gtid / TPR;
  const int part = static_cast<int>(gtid % TPR);
  float acc = 0.f;
  if (row < rows) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(o + row * D) + part);
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(dO + row * D) + part);
    const __half2* ha = reinterpret_cast<const __half2*>(&a);
    const __half2* hb = reinterpret_cast<const __half2*>(&b);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 fa = __half22float2(ha[i]);
      const float2 fb = __half22float2(hb[i]);
      acc = fmaf(fa.x, fb.x, acc);
      acc = fmaf(fa.y, fb.y, acc);
    }
  }
#pragma unroll
  for (int off = TPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (row < rows && part == 0) dvec[row] = acc;
}

// ---------------------------------------------------------------------------
// dK / dV: one CTA per (128 keys, batch, kv-head).
//   warps 0-3  compute: one thread per key row; P^T and dS^T for 64 queries
//   warp  4    TMEM allocation + MMA issue
//   warp  5    TMA producer
// TMEM: S^T[2] cols 0,64 | dP^T[2] cols 128,192 | dV 256..256+D | dK 256+D..
// Per query block i the MMA thread issues
//   [P_i] dV += P_i^T dO_i ; S_{i+1} ; dP_{i+1} ; [dS_i] dK += dS_i^T Q_i
// S^T = K Q^T (A = K, K-major; B = Q, K-major), dP^T = V dO^T (same shapes),
// dV += P^T dO (A = P^T K-major in smem, B = dO MN-major),
// dK += dS^T Q  (A = dS^T K-major in smem, B = Q MN-major).
// dS is stored pre-multiplied by the softmax scale, so dK needs no rescale.
// ---------------------------------------------------------------------------
template <int D>
struct DkdvCfg {
  static constexpr int BN = 128;  // keys per CTA
  static constexpr int BM = 64;   // queries per step
  static constexpr int CH = D / 64;
  static constexpr int KVBYTES = BN * D * 2;   // K or V tile
  static constexpr int QBYTES = BM * D * 2;    // Q or dO tile
  static constexpr int PBYTES = BN * BM * 2;   // P^T or dS^T tile
  static constexpr int STAGES = (D == 128) ? 6 : 8;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + KVBYTES;
  static constexpr int OFF_RING = OFF_V + KVBYTES;
  static constexpr int OFF_P = OFF_RING + STAGES * QBYTES;
  static constexpr int OFF_DS = OFF_P + PBYTES;
  // per compute warp, double-buffered: 64 log2-domain LSE values, 64 Dv values
  static constexpr int OFF_LSE = OFF_DS + PBYTES;
  static constexpr int OFF_DV = OFF_LSE + 4 * 2 * BM * 4;
  static constexpr int OFF_BAR = OFF_DV + 4 * 2 * BM * 4;
  // kv, full[ST], empty[ST], s[2], dp[2], p, ds, dk, fin
  static constexpr int NBAR = 1 + 2 * STAGES + 8;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static constexpr int THREADS = 192;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t COL_S = 0, COL_DP = 128, COL_DV = 256, COL_DK = 256 + D;
};

}  // namespace fab

namespace fab {

// Write one row of 32 fp32 TMEM values as fp16 to global (8 halves per store).
__device__ __forceinline__ void store_row32_f16(__half* dst, const uint32_t (&v)[32], float mul) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 pk;
    pk.x = pack_half2(__uint_as_float(v[8 * q + 0]) * mul, __uint_as_float(v[8 * q + 1]) * mul);
    pk.y = pack_half2(__uint_as_float(v[8 * q + 2]) * mul, __uint_as_float(v[8 * q + 3]) * mul);
    pk.z = pack_half2(__uint_as_float(v[8 * q + 4]) * mul, __uint_as_float(v[8 * q + 5]) * mul);
    pk.w = pack_half2(__uint_as_float(v[8 * q + 6]) * mul, __uint_as_float(v[8 * q + 7]) * mul);
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

template <int D>
__global__ void __launch_bounds__(192, 1)
    bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                    const BwdParams p) {
  using C = DkdvCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  const uint32_t s_k = sbase + C::OFF_K, s_v = sbase + C::OFF_V, s_ring = sbase + C::OFF_RING;
  const uint32_t s_p = sbase + C::OFF_P, s_ds = sbase + C::OFF_DS;
  float* lse_s = reinterpret_cast<float*>(sgen + C::OFF_LSE);
  float* dvec_s = reinterpret_cast<float*>(sgen + C::OFF_DV);
  const uint32_t b_kv = sbase + C::OFF_BAR;
  const uint32_t b_full = b_kv + 8, b_empty = b_full + 8 * C::STAGES;
  const uint32_t b_s = b_empty + 8 * C::STAGES, b_dp = b_s + 16;
  const uint32_t b_p = b_dp + 16, b_ds = b_p + 8, b_dk = b_ds + 8, b_fin = b_dk + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + C::OFF_BAR + C::NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grid (B*Hkv, key blocks): causal key block 0 has the most work and goes first
  const int bkv = blockIdx.x;        // b * hkv + kv head
  const int kvb = blockIdx.y;        // key block
  const int hkv = p.hq / p.group;
  const int b = bkv / hkv, kvh = bkv % hkv;
  const int kv0 = kvb * C::BN;
  const int nqb = (p.n + C::BM - 1) / C::BM;
  const int i_start = p.causal ? (kv0 / C::BM) : 0;
  const int nq_head = nqb - i_start;
  const int total = p.group * nq_head;   // (group head, query block) steps
  const Ctl ctl{abort_flag, p.err};

  if (threadIdx.x == 0) {
    mbar_init(b_kv, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(b_full + 8 * s, 1);
      mbar_init(b_empty + 8 * s, 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(b_s + 8 * t, 1);
      mbar_init(b_dp + 8 * t, 1);
    }
    mbar_init(b_p, 128);
    mbar_init(b_ds, 128);
    mbar_init(b_dk, 1);
    mbar_init(b_fin, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 5) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      mbar_arrive_expect_tx(b_kv, 2 * C::KVBYTES);
#pragma unroll
      for (int c = 0; c < C::CH; ++c) {
        tma_load_3d(s_k + c * 16384, &tm_k, b_kv, c * 64, kv0, bkv);
        tma_load_3d(s_v + c * 16384, &tm_v, b_kv, c * 64, kv0, bkv);
      }
      int it = 0;
      bool ok = true;
      for (int step = 0; step < total && ok; ++step) {
        const int g = step / nq_head;
        const int q0 = (i_start + step % nq_head) * C::BM;
        const int bh = b * p.hq + kvh * p.group + g;
#pragma unroll 1
        for (int kind = 0; kind < 2; ++kind, ++it) {  // Q_i then dO_i
          const int slot = it % C::STAGES;
          ok = mbar_wait(b_empty + 8 * slot, ((it / C::STAGES) & 1) ^ 1, ctl, kErrTimeoutLoad);
          if (!ok) break;
          const uint32_t fb = b_full + 8 * slot;
          mbar_arrive_expect_tx(fb, C::QBYTES);
          const uint32_t dst = s_ring + slot * C::QBYTES;
#pragma unroll
          for (int c = 0; c < C::CH; ++c)
            tma_load_3d(dst + c * (C::BM * 128), kind ? (const void*)&tm_do : (const void*)&tm_q, fb,
                        c * 64, q0, bh);
        }
      }
      if (!ok) {
        drain_loads(b_kv, 1, 1);
        drain_loads(b_full, it, C::STAGES);
      }
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && total > 0) {
      constexpr uint32_t id_s = idesc_f16(128, C::BM, false, false);  // S^T, dP^T
      constexpr uint32_t id_g = idesc_f16(128, D, false, true);       // dV, dK
      auto slot_of = [](int it) { return it % C::STAGES; };
      auto ph_of = [](int it) { return static_cast<uint32_t>((it / C::STAGES) & 1); };
      // S^T_i = K Q_i^T  /  dP^T_i = V dO_i^T
      auto issue_t = [&](uint32_t d_tmem, uint32_t a_s, uint32_t b_s_) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_ss(d_tmem, sdesc_sw128(a_s + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                 sdesc_sw128(b_s_ + (kk >> 2) * (C::BM * 128) + (kk & 3) * 32, 16, 1024), id_s,
                 kk > 0 ? 1u : 0u);
      };
      // acc += X^T_i (128 keys x 64 queries, K-major) * Y_i (64 queries x D, MN-major)
      auto issue_g = [&](uint32_t d_tmem, uint32_t x_s, uint32_t y_s, bool acc) {
#pragma unroll
        for (int kk = 0; kk < C::BM / 16; ++kk)
          mma_ss(d_tmem, sdesc_sw128(x_s + kk * 32, 16, 1024),
                 sdesc_sw128(y_s + kk * 2048, C::BM * 128, 1024), id_g, (acc || kk > 0) ? 1u : 0u);
      };
      bool ok = mbar_wait(b_kv, 0, ctl, kErrTimeoutMma);
      // prologue: S_0, dP_0
      if (ok) ok = mbar_wait(b_full + 8 * slot_of(0), ph_of(0), ctl, kErrTimeoutMma);
      if (ok) {
        tc_fence_after();
        issue_t(tmem + C::COL_S, s_k, s_ring + slot_of(0) * C::QBYTES);
        mma_commit(b_s);
        ok = mbar_wait(b_full + 8 * slot_of(1), ph_of(1), ctl, kErrTimeoutMma);
      }
      if (ok) {
        tc_fence_after();
        issue_t(tmem + C::COL_DP, s_v, s_ring + slot_of(1) * C::QBYTES);
        mma_commit(b_dp);
      }
      for (int i = 0; i < total && ok; ++i) {
        const int it_q = 2 * i, it_do = 2 * i + 1;
        ok = mbar_wait(b_p, i & 1, ctl, kErrTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        issue_g(tmem + C::COL_DV, s_p, s_ring + slot_of(it_do) * C::QBYTES, i > 0);
        mma_commit(b_empty + 8 * slot_of(it_do));
        if (i + 1 < total) {
          const int nb = (i + 1) & 1;
          ok = mbar_wait(b_full + 8 * slot_of(it_q + 2), ph_of(it_q + 2), ctl, kErrTimeoutMma);
          if (!ok) break;
          tc_fence_after();
          issue_t(tmem + C::COL_S + 64 * nb, s_k, s_ring + slot_of(it_q + 2) * C::QBYTES);
          mma_commit(b_s + 8 * nb);
          ok = mbar_wait(b_full + 8 * slot_of(it_do + 2), ph_of(it_do + 2), ctl, kErrTimeoutMma);
          if (!ok) break;
          tc_fence_after();
          issue_t(tmem + C::COL_DP + 64 * nb, s_v, s_ring + slot_of(it_do + 2) * C::QBYTES);
          mma_commit(b_dp + 8 * nb);
        }
        ok = mbar_wait(b_ds, i & 1, ctl, kErrTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        issue_g(tmem + C::COL_DK, s_ds, s_ring + slot_of(it_q) * C::QBYTES, i > 0);
        mma_commit(b_dk);
        mma_commit(b_empty + 8 * slot_of(it_q));
      }
      mma_commit(b_fin);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(b_fin, 0) && globaltimer_ns() - t0 < FAB_WAIT_LIMIT_NS) {
      }
    }
  } else {
    // ------------------------------------------------------------ compute (warps 0-3)
    const int r = threadIdx.x;  // key row within the block
    const int kvrow = kv0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    bool ok = true;
    for (int i = 0; i < total; ++i) {
      const int g = i / nq_head;
      const int q0 = (i_start + i % nq_head) * C::BM;
      const int bh = b * p.hq + kvh * p.group + g;
      const int buf = i & 1;
      // Each warp stages its own copy of this step's 64 LSE / Dv values, so
      // the only synchronisation is within the warp (a failed wait in one
      // warp can never leave another stuck at a barrier).
      float* lse2w = lse_s + (warp * 2 + buf) * C::BM;
      float* dvw = dvec_s + (warp * 2 + buf) * C::BM;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int q = q0 + lane + 32 * h;
        const bool in = q < p.n;
        lse2w[lane + 32 * h] =
            in ? p.lse[static_cast<size_t>(bh) * p.n + q] * 1.4426950408889634f : INFINITY;
        dvw[lane + 32 * h] = in ? p.dvec[static_cast<size_t>(bh) * p.n + q] : 0.f;
      }
      __syncwarp();
      const float* lse2 = lse2w;
      const float* dv_s = dvw;

      ok = mbar_wait(b_s + 8 * buf, (i >> 1) & 1, ctl, kErrTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[2][32];
      tmem_ld32(tmem + C::COL_S + 64 * buf + lane_off, sr[0]);
      tmem_ld32(tmem + C::COL_S + 64 * buf + 32 + lane_off, sr[1]);
      tmem_ld_wait_only();
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int k = 0; k < 32; ++k) asm volatile("" : "+r"(sr[c][k]));
      float pv[64];
      // keys of a causal step at or below the diagonal keep P; the rest is exactly 0
      const int qlim = p.causal ? kvrow : -1;  // valid iff q >= qlim
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float s = __uint_as_float(sr[c >> 5][c & 31]);
        const float e = ex2(fmaf(s, p.scale_log2, -lse2[c]));
        pv[c] = (q0 + c >= qlim) ? e : 0.f;
      }
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
        st_shared_v4(s_p + r * 128 + ((c8 ^ (r & 7)) << 4), pack_half2(pv[8 * c8], pv[8 * c8 + 1]),
                     pack_half2(pv[8 * c8 + 2], pv[8 * c8 + 3]),
                     pack_half2(pv[8 * c8 + 4], pv[8 * c8 + 5]),
                     pack_half2(pv[8 * c8 + 6], pv[8 * c8 + 7]));
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(b_p);

      ok = mbar_wait(b_dp + 8 * buf, (i >> 1) & 1, ctl, kErrTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      tmem_ld32(tmem + C::COL_DP + 64 * buf + lane_off, sr[0]);
      tmem_ld32(tmem + C::COL_DP + 64 * buf + 32 + lane_off, sr[1]);
      tmem_ld_wait_only();
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int k = 0; k < 32; ++k) asm volatile("" : "+r"(sr[c][k]));
#pragma unroll
      for (int c = 0; c < 64; ++c)
        pv[c] = pv[c] * (__uint_as_float(sr[c >> 5][c & 31]) - dv_s[c]) * p.scale;
      if (i > 0) {
        ok = mbar_wait(b_dk, (i - 1) & 1, ctl, kErrTimeoutSoftmax);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
      }
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
        st_shared_v4(s_ds + r * 128 + ((c8 ^ (r & 7)) << 4), pack_half2(pv[8 * c8], pv[8 * c8 + 1]),
                     pack_half2(pv[8 * c8 + 2], pv[8 * c8 + 3]),
                     pack_half2(pv[8 * c8 + 4], pv[8 * c8 + 5]),
                     pack_half2(pv[8 * c8 + 6], pv[8 * c8 + 7]));
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(b_ds);
    }
    if (ok) {
      ok = mbar_wait(b_fin, 0, ctl, kErrTimeoutEpilogue);
      ok = __all_sync(0xffffffffu, ok);
    }
    if (ok) {
      tc_fence_after();
      const size_t rowoff = (static_cast<size_t>(bkv) * p.n + kvrow) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + C::COL_DV + 32 * c + lane_off, v);
        tmem_ld_wait(v);
        if (total == 0) {
#pragma unroll
          for (int k = 0; k < 32; ++k) v[k] = 0u;
        }
        if (kvrow < p.n) store_row32_f16(p.dv + rowoff + 32 * c, v, 1.f);
        tmem_ld32(tmem + C::COL_DK + 32 * c + lane_off, v);
        tmem_ld_wait(v);
        if (total == 0) {
#pragma unroll
          for (int k = 0; k < 32; ++k) v[k] = 0u;
        }
        if (kvrow < p.n) store_row32_f16(p.dk + rowoff + 32 * c, v, 1.f);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 4) {
    __syncwarp();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace fab

namespace fab {

// ---------------------------------------------------------------------------
// dQ: one CTA per (128 queries, batch*q-head); loops over key blocks of 64.
//   warps 0-3  compute: one thread per query row; dS for 64 keys
//   warp  4    TMEM allocation + MMA issue
//   warp  5    TMA producer (K_j, V_j alternate in one ring)
// TMEM: S[2] cols 0,64 | dP[2] cols 128,192 | dQ 256..256+D
// MMA order: S_0 dP_0 S_1 dP_1 [dS_0] dQ+=dS_0 K_0  S_2 dP_2 [dS_1] dQ+=dS_1 K_1 ...
// S = Q K^T (A = Q K-major, B = K K-major), dP = dO V^T (same shapes),
// dQ += dS K (A = dS K-major in smem, B = K MN-major).
// ---------------------------------------------------------------------------
template <int D>
struct DqCfg {
  static constexpr int BM = 128;  // queries per CTA
  static constexpr int BN = 64;   // keys per step
  static constexpr int CH = D / 64;
  static constexpr int QBYTES = BM * D * 2;
  static constexpr int KVBYTES = BN * D * 2;
  static constexpr int DSBYTES = BM * BN * 2;
  static constexpr int STAGES = (D == 128) ? 6 : 8;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_DO = OFF_Q + QBYTES;
  static constexpr int OFF_RING = OFF_DO + QBYTES;
  static constexpr int OFF_DS = OFF_RING + STAGES * KVBYTES;
  static constexpr int OFF_BAR = OFF_DS + 2 * DSBYTES;
  // qdo, full[ST], empty[ST], s[2], dp[2], ds[2], fin
  static constexpr int NBAR = 1 + 2 * STAGES + 7;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;
  static constexpr int THREADS = 192;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t COL_S = 0, COL_DP = 128, COL_DQ = 256;
};

template <int D>
__global__ void __launch_bounds__(192, 1)
    bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                  const BwdParams p) {
  using C = DqCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - smem_u32(smem_raw));
  const uint32_t s_q = sbase + C::OFF_Q, s_do = sbase + C::OFF_DO, s_ring = sbase + C::OFF_RING;
  const uint32_t s_ds = sbase + C::OFF_DS;
  const uint32_t b_qdo = sbase + C::OFF_BAR;
  const uint32_t b_full = b_qdo + 8, b_empty = b_full + 8 * C::STAGES;
  const uint32_t b_s = b_empty + 8 * C::STAGES, b_dp = b_s + 16;
  // dS-ready is one barrier per dS buffer: S/dP of blocks j and j+1 are both in
  // flight, so a warp may finish dS_{j+1} before another warp finishes dS_j;
  // with a single barrier those arrivals would land in the same phase.
  const uint32_t b_ds = b_dp + 16, b_fin = b_ds + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sgen + C::OFF_BAR + C::NBAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nmb = (p.n + C::BM - 1) / C::BM;
  // grid (B*Hq, query blocks), longest causal rows first
  const int mb = p.causal ? (nmb - 1 - static_cast<int>(blockIdx.y)) : static_cast<int>(blockIdx.y);
  const int m0 = mb * C::BM;
  const int bh = blockIdx.x;
  const int bkv = (bh / p.hq) * (p.hq / p.group) + (bh % p.hq) / p.group;
  const int nblk = (p.n + C::BN - 1) / C::BN;
  const int nkv = p.causal ? min(nblk, (m0 + C::BM) / C::BN) : nblk;
  const Ctl ctl{abort_flag, p.err};

  if (threadIdx.x == 0) {
    mbar_init(b_qdo, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(b_full + 8 * s, 1);
      mbar_init(b_empty + 8 * s, 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(b_s + 8 * t, 1);
      mbar_init(b_dp + 8 * t, 1);
    }
    mbar_init(b_ds, 128);
    mbar_init(b_ds + 8, 128);
    mbar_init(b_fin, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 5) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      mbar_arrive_expect_tx(b_qdo, 2 * C::QBYTES);
#pragma unroll
      for (int c = 0; c < C::CH; ++c) {
        tma_load_3d(s_q + c * 16384, &tm_q, b_qdo, c * 64, m0, bh);
        tma_load_3d(s_do + c * 16384, &tm_do, b_qdo, c * 64, m0, bh);
      }
      int it = 0;
      bool ok = true;
      for (int j = 0; j < nkv && ok; ++j) {
#pragma unroll 1
        for (int kind = 0; kind < 2; ++kind, ++it) {  // K_j then V_j
          const int slot = it % C::STAGES;
          ok = mbar_wait(b_empty + 8 * slot, ((it / C::STAGES) & 1) ^ 1, ctl, kErrTimeoutLoad);
          if (!ok) break;
          const uint32_t fb = b_full + 8 * slot;
          mbar_arrive_expect_tx(fb, C::KVBYTES);
          const uint32_t dst = s_ring + slot * C::KVBYTES;
#pragma unroll
          for (int c = 0; c < C::CH; ++c)
            tma_load_3d(dst + c * (C::BN * 128), kind ? (const void*)&tm_v : (const void*)&tm_k, fb,
                        c * 64, j * C::BN, bkv);
        }
      }
      if (!ok) {
        drain_loads(b_qdo, 1, 1);
        drain_loads(b_full, it, C::STAGES);
      }
    }
  } else if (warp == 4) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && nkv > 0) {
      constexpr uint32_t id_s = idesc_f16(128, C::BN, false, false);
      constexpr uint32_t id_q = idesc_f16(128, D, false, true);
      auto slot_of = [](int it) { return it % C::STAGES; };
      auto ph_of = [](int it) { return static_cast<uint32_t>((it / C::STAGES) & 1); };
      auto issue_t = [&](uint32_t d_tmem, uint32_t a_s, uint32_t b_s_) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          mma_ss(d_tmem, sdesc_sw128(a_s + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                 sdesc_sw128(b_s_ + (kk >> 2) * (C::BN * 128) + (kk & 3) * 32, 16, 1024), id_s,
                 kk > 0 ? 1u : 0u);
      };
      bool ok = mbar_wait(b_qdo, 0, ctl, kErrTimeoutMma);
      // S_j and dP_j into TMEM buffer j&1
      auto issue_sdp = [&](int j) -> bool {
        const int nb = j & 1;
        if (!mbar_wait(b_full + 8 * slot_of(2 * j), ph_of(2 * j), ctl, kErrTimeoutMma)) return false;
        tc_fence_after();
        issue_t(tmem + C::COL_S + 64 * nb, s_q, s_ring + slot_of(2 * j) * C::KVBYTES);
        mma_commit(b_s + 8 * nb);
        if (!mbar_wait(b_full + 8 * slot_of(2 * j + 1), ph_of(2 * j + 1), ctl, kErrTimeoutMma))
          return false;
        tc_fence_after();
        issue_t(tmem + C::COL_DP + 64 * nb, s_do, s_ring + slot_of(2 * j + 1) * C::KVBYTES);
        mma_commit(b_dp + 8 * nb);
        mma_commit(b_empty + 8 * slot_of(2 * j + 1));  // V_j no longer needed
        return true;
      };
      if (ok) ok = issue_sdp(0);
      if (ok && nkv > 1) ok = issue_sdp(1);
      for (int j = 0; j < nkv && ok; ++j) {
        ok = mbar_wait(b_ds + 8 * (j & 1), (j >> 1) & 1, ctl, kErrTimeoutMma);
        if (!ok) break;
        tc_fence_after();
        const uint32_t k_s = s_ring + slot_of(2 * j) * C::KVBYTES;
        const uint32_t ds_s = s_ds + (j & 1) * C::DSBYTES;
#pragma unroll
        for (int kk = 0; kk < C::BN / 16; ++kk)
          mma_ss(tmem + C::COL_DQ, sdesc_sw128(ds_s + kk * 32, 16, 1024),
                 sdesc_sw128(k_s + kk * 2048, C::BN * 128, 1024), id_q, (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(b_empty + 8 * slot_of(2 * j));  // K_j no longer needed
        if (j + 2 < nkv) ok = issue_sdp(j + 2);
      }
      mma_commit(b_fin);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(b_fin, 0) && globaltimer_ns() - t0 < FAB_WAIT_LIMIT_NS) {
      }
    }
  } else {
    // ------------------------------------------------------------ compute (warps 0-3)
    const int r = threadIdx.x;
    const int row = m0 + r;
    const bool row_in = row < p.n;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const float lse2 = row_in ? p.lse[static_cast<size_t>(bh) * p.n + row] * 1.4426950408889634f
                              : INFINITY;
    const float dv = row_in ? p.dvec[static_cast<size_t>(bh) * p.n + row] : 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int buf = j & 1;
      ok = mbar_wait(b_s + 8 * buf, (j >> 1) & 1, ctl, kErrTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[2][32];
      tmem_ld32(tmem + C::COL_S + 64 * buf + lane_off, sr[0]);
      tmem_ld32(tmem + C::COL_S + 64 * buf + 32 + lane_off, sr[1]);
      tmem_ld_wait_only();
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int k = 0; k < 32; ++k) asm volatile("" : "+r"(sr[c][k]));
      float pv[64];
      const int kv0 = j * C::BN;
      const bool need_mask = (kv0 + C::BN > p.n) || (p.causal && kv0 + C::BN - 1 > m0);
      const int klim = p.causal ? min(p.n - 1, row) : (p.n - 1);  // valid iff key <= klim
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float e = ex2(fmaf(__uint_as_float(sr[c >> 5][c & 31]), p.scale_log2, -lse2));
        pv[c] = (!need_mask || kv0 + c <= klim) ? e : 0.f;
      }
      ok = mbar_wait(b_dp + 8 * buf, (j >> 1) & 1, ctl, kErrTimeoutSoftmax);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      tmem_ld32(tmem + C::COL_DP + 64 * buf + lane_off, sr[0]);
      tmem_ld32(tmem + C::COL_DP + 64 * buf + 32 + lane_off, sr[1]);
      tmem_ld_wait_only();
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int k = 0; k < 32; ++k) asm volatile("" : "+r"(sr[c][k]));
#pragma unroll
      for (int c = 0; c < 64; ++c)
        pv[c] = pv[c] * (__uint_as_float(sr[c >> 5][c & 31]) - dv) * p.scale;
      const uint32_t ds_s = s_ds + buf * C::DSBYTES;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8)
        st_shared_v4(ds_s + r * 128 + ((c8 ^ (r & 7)) << 4), pack_half2(pv[8 * c8], pv[8 * c8 + 1]),
                     pack_half2(pv[8 * c8 + 2], pv[8 * c8 + 3]),
                     pack_half2(pv[8 * c8 + 4], pv[8 * c8 + 5]),
                     pack_half2(pv[8 * c8 + 6], pv[8 * c8 + 7]));
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(b_ds + 8 * buf);
    }
    if (ok && nkv > 0) {
      ok = mbar_wait(b_fin, 0, ctl, kErrTimeoutEpilogue);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        const size_t rowoff = (static_cast<size_t>(bh) * p.n + row) * D;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem + C::COL_DQ + 32 * c + lane_off, v);
          tmem_ld_wait(v);
          if (row_in) {
            if (p.dq_fp32)
              store_row32_f32(static_cast<float*>(p.dq) + rowoff + 32 * c, v, 1.f);
            else
              store_row32_f16(static_cast<__half*>(p.dq) + rowoff + 32 * c, v, 1.f);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 4) {
    __syncwarp();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace fab
