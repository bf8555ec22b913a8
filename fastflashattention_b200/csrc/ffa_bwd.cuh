// ffa_bwd.cuh — deterministic attention backward for sm_100a.
//
// Two kernels with disjoint output tiles and no atomics, the split of the reference
// backward (fastflash_attention/_kernel.py:379-448 dK/dV, :487-564 dQ, recompute path):
//
//   dkdv kernel (grid over 128-key blocks, loop over 128-query steps)
//     S^T  = K Q^T            P^T  = exp2(scale*log2e*S^T - lse)   (masked)
//     dP^T = V dO^T           dS^T = P^T * (dP^T - delta)
//     dV  += bf16(P^T) dO     dK  += bf16(dS^T) Q        dK *= scale at the end
//   dq kernel (grid over 128-query blocks, loop over 128-key steps)
//     S = Q K^T, dP = dO V^T, dS = P*(dP - delta), dQ += bf16(dS) K, dQ *= scale
//
// The backward preprocess delta = rowsum(O*dO) (ffa_aux.cuh) runs first.
//
// Both kernels share one shape: a CTA owns the 128 TMEM lanes (keys for dkdv, queries
// for dq) and walks the other dimension in 128-wide steps, so every shared-memory
// operand MMA is 128 x 128 x 16 (the narrowest shape whose smem operand traffic the
// tensor core can be fed at full rate).
//   warps 0-7  two compute warpgroups; warpgroup g handles columns [64g, 64g+64) of
//              every step (thread = TMEM lane = one key / query row)
//   warp  8    producer: TMA for the streamed tiles (and lse/delta for dkdv)
//   warp  9    MMA issuer (one thread)
// P and dS are written back over the columns they were computed from, as packed bf16
// (warpgroup g's 64 values land in columns [64g, 64g+32) of the region), and feed the
// gradient MMAs straight from tensor memory.
#pragma once
#include "ffa_common.cuh"

namespace ffa {

namespace bwd {
constexpr int LANES = 128;   // TMEM lanes owned by a CTA
constexpr int STEP = 128;    // width of one step along the streamed dimension
constexpr int STAGES = 2;
constexpr int NTHREADS = 320;
constexpr int PRODUCER_WARP = 8;
constexpr int MMA_WARP = 9;

template <int D>
struct DkdvLayout {
  static constexpr int TILE = 128 * D * 2;  // K, V (resident) and Q, dO (streamed) tiles
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = TILE;
  static constexpr int STAGE_OFF = 2 * TILE;
  // stage: Q tile, dO tile, lse[128], delta[128]
  static constexpr int STAGE_BYTES = ((2 * TILE + 2 * STEP * 4) + 1023) / 1024 * 1024;
  static constexpr int BAR_OFF = STAGE_OFF + STAGES * STAGE_BYTES;
  // kv_full, st_full[2], st_empty[2], s_full, dp_full, p_ready, ds_ready, final, drain
  static constexpr int NBARS = 1 + 2 * STAGES + 6;
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  static constexpr int SMEM_BYTES = MISC_OFF + 16 + 1024;
};

template <int D>
struct DqLayout {
  static constexpr int TILE = 128 * D * 2;  // Q, dO (resident) and K, V (streamed) tiles
  static constexpr int K_STAGES = 3;        // K_j is read by S_j and, a step later, by dQ += dS_j K_j
  static constexpr int V_STAGES = 2;        // V_j is read by dP_j only
  static constexpr int Q_OFF = 0;
  static constexpr int DO_OFF = TILE;
  static constexpr int K_OFF = 2 * TILE;
  static constexpr int V_OFF = K_OFF + K_STAGES * TILE;
  static constexpr int BAR_OFF = V_OFF + V_STAGES * TILE;
  // qd_full, k_full[3], k_empty[3], v_full[2], v_empty[2], s_full[2], dp_full, dp_free,
  // ds_ready, final, drain
  static constexpr int NBARS = 1 + 2 * K_STAGES + 2 * V_STAGES + 2 + 5;
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  static constexpr int SMEM_BYTES = MISC_OFF + 16 + 1024;
};

// TMEM column of the 16-deep K-step `ks` of a packed-bf16 A operand written by the two
// warpgroups (K-steps 0-3 from warpgroup 0 at base, 4-7 from warpgroup 1 at base + 64).
__device__ __forceinline__ uint32_t packed_kstep_col(uint32_t base, int ks) {
  return base + (ks >> 2) * 64 + (ks & 3) * 8;
}

// Store 32 fp32 values (times `mul`) as bf16 to a 64-byte aligned global row segment.
__device__ __forceinline__ void store_row32(__nv_bfloat16* dst, const uint32_t (&r)[32], float mul) {
  uint32_t packed[16];
#pragma unroll
  for (int e = 0; e < 16; ++e)
    packed[e] = pack_bf16x2(__uint_as_float(r[2 * e]) * mul, __uint_as_float(r[2 * e + 1]) * mul);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int e = 0; e < 4; ++e) d4[e] = make_uint4(packed[4 * e], packed[4 * e + 1], packed[4 * e + 2], packed[4 * e + 3]);
}

// Load 64 consecutive fp32 TMEM columns of this thread's lane.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[2][32];
  tmem_ld32(taddr, r[0]);
  tmem_ld32(taddr + 32, r[1]);
  tmem_ld_wait();
#pragma unroll
  for (int e = 0; e < 64; ++e) v[e] = __uint_as_float(r[e >> 5][e & 31]);
}

// Write the accumulator columns [g*D/2, (g+1)*D/2) of this lane to a global bf16 row.
template <int D>
__device__ __forceinline__ void store_acc_half(uint32_t t_acc, int g, __nv_bfloat16* row, bool valid, float mul) {
#pragma unroll 1
  for (int c = g * (D / 64); c < (g + 1) * (D / 64); ++c) {
    uint32_t r[32];
    tmem_ld32(t_acc + 32 * c, r);
    tmem_ld_wait();
    if (valid) store_row32(row + 32 * c, r, mul);
  }
}
}  // namespace bwd

// ====================================================================================
// dK / dV
// ====================================================================================
template <int D, bool CAUSAL>
__global__ void __launch_bounds__(bwd::NTHREADS, 1)
    ffa_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                        const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                        const float* __restrict__ LSE, const float* __restrict__ DELTA,
                        __nv_bfloat16* __restrict__ DK, __nv_bfloat16* __restrict__ DV, int S, long long stride_bh,
                        long long stride_s, float scale_log2, float scale) {
  using L = bwd::DkdvLayout<D>;
  constexpr int SLABS = D / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::BAR_OFF;
  const uint32_t kv_full = bar0;
  auto st_full = [&](int s) { return bar0 + 8 * (1 + s); };
  auto st_empty = [&](int s) { return bar0 + 8 * (1 + bwd::STAGES + s); };
  const uint32_t s_full = bar0 + 8 * (1 + 2 * bwd::STAGES);
  const uint32_t dp_full = s_full + 8;
  const uint32_t p_ready = s_full + 16;
  const uint32_t ds_ready = s_full + 24;
  const uint32_t final_bar = s_full + 32;
  const uint32_t drain_bar = s_full + 40;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);
  auto stage_ptr = [&](int s) { return smem + L::STAGE_OFF + s * L::STAGE_BYTES; };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int kblk = static_cast<int>(blockIdx.x);  // causal: low key blocks carry the most work and run first
  const int bh = blockIdx.y;
  const int n0 = kblk * bwd::LANES;
  const int q_begin = CAUSAL ? n0 : 0;  // first query that can see a key of this block
  const int nq = (S > q_begin) ? (S - q_begin + bwd::STEP - 1) / bwd::STEP : 0;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < bwd::STAGES; ++s) {
      mbar_init(st_full(s), 2);  // TMA expect-tx arrival + lse/delta arrival
      mbar_init(st_empty(s), 1);
    }
    mbar_init(s_full, 1);
    mbar_init(dp_full, 1);
    mbar_init(p_ready, 256);
    mbar_init(ds_ready, 256);
    mbar_init(final_bar, 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == bwd::MMA_WARP) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp == bwd::PRODUCER_WARP && lane == 0) {
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_do);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == bwd::PRODUCER_WARP) {
    // ---------------------------------------------------------------- producer
    const uint64_t keep = policy_evict_last();
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * L::TILE);
      for (int sl = 0; sl < SLABS; ++sl) {
        tma_load_3d(sbase + L::K_OFF + sl * 16384, &tm_k, kv_full, sl * 64, n0, bh, keep);
        tma_load_3d(sbase + L::V_OFF + sl * 16384, &tm_v, kv_full, sl * 64, n0, bh, keep);
      }
    }
    int issued = 0;
    for (int it = 0; it < nq; ++it) {
      const int s = it % bwd::STAGES;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(st_empty(s), ((it / bwd::STAGES) & 1) ^ 1, abort_flag, kErrBwdProducer);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      const int q0 = q_begin + it * bwd::STEP;
      const uint32_t st = smem_u32(stage_ptr(s));
      if (lane == 0) {
        mbar_arrive_expect_tx(st_full(s), 2 * L::TILE);
        for (int sl = 0; sl < SLABS; ++sl) {
          tma_load_3d(st + sl * 16384, &tm_q, st_full(s), sl * 64, q0, bh, keep);
          tma_load_3d(st + L::TILE + sl * 16384, &tm_do, st_full(s), sl * 64, q0, bh, keep);
        }
      }
      float* lse_s = reinterpret_cast<float*>(stage_ptr(s) + 2 * L::TILE);
      float* dl_s = lse_s + bwd::STEP;
#pragma unroll
      for (int r = lane; r < bwd::STEP; r += 32) {
        const int q = q0 + r;
        const long long idx = static_cast<long long>(bh) * S + q;
        // rows past the end get lse = +inf, so their P (and dS) are exactly 0
        lse_s[r] = (q < S) ? LSE[idx] : INFINITY;
        dl_s[r] = (q < S) ? DELTA[idx] : 0.f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(st_full(s));
      ++issued;
    }
    if (lane == 0 && *abort_flag) {
      mbar_wait_drain(kv_full, 0);
      for (int it = max(0, issued - bwd::STAGES); it < issued; ++it)
        mbar_wait_drain(st_full(it % bwd::STAGES), (it / bwd::STAGES) & 1);
    }
  } else if (warp == bwd::MMA_WARP) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_SD = idesc_bf16(128, bwd::STEP, false, false);  // [128 keys x 128 queries]
      constexpr uint32_t IDESC_G = idesc_bf16(128, D, false, true);            // [128 keys x D]
      const uint32_t k_addr = sbase + L::K_OFF, v_addr = sbase + L::V_OFF;
      auto q_addr = [&](int i) { return smem_u32(stage_ptr(i % bwd::STAGES)); };
      auto issue_s = [&](int i) -> bool {  // S^T = K Q_i^T
        if (!mbar_wait(st_full(i % bwd::STAGES), (i / bwd::STAGES) & 1, abort_flag, kErrBwdMma)) return false;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          mma_ss(tmem, kmajor_desc(k_addr, 128, ks), kmajor_desc(q_addr(i), 128, ks), IDESC_SD, ks > 0);
        mma_commit(s_full);
        return true;
      };
      auto issue_dp = [&](int i) {  // dP^T = V dO_i^T
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          mma_ss(tmem + 128, kmajor_desc(v_addr, 128, ks), kmajor_desc(q_addr(i) + L::TILE, 128, ks), IDESC_SD,
                 ks > 0);
        mma_commit(dp_full);
      };
      auto issue_dv = [&](int i) -> bool {  // dV += P^T dO_i
        if (!mbar_wait(p_ready, i & 1, abort_flag, kErrBwdMma)) return false;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < bwd::STEP / 16; ++ks)
          mma_ts(tmem + 256, bwd::packed_kstep_col(tmem, ks), mnmajor_desc(q_addr(i) + L::TILE, 128, ks), IDESC_G,
                 (i > 0 || ks > 0) ? 1u : 0u);
        return true;
      };
      auto issue_dk = [&](int i) -> bool {  // dK += dS^T Q_i
        if (!mbar_wait(ds_ready, i & 1, abort_flag, kErrBwdMma)) return false;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < bwd::STEP / 16; ++ks)
          mma_ts(tmem + 384, bwd::packed_kstep_col(tmem + 128, ks), mnmajor_desc(q_addr(i), 128, ks), IDESC_G,
                 (i > 0 || ks > 0) ? 1u : 0u);
        mma_commit(st_empty(i % bwd::STAGES));
        return true;
      };
      bool ok = mbar_wait(kv_full, 0, abort_flag, kErrBwdMma);
      if (ok && nq > 0) {
        ok = issue_s(0);
        if (ok) issue_dp(0);
      }
      // dV(i), S(i+1), dK(i), dP(i+1): the next step's S and dP run while the
      // warpgroups turn this step's dP into dS and the next step's S into P.
      for (int i = 0; i < nq && ok; ++i) {
        if (!(ok = issue_dv(i))) break;
        if (i + 1 < nq && !(ok = issue_s(i + 1))) break;
        if (!(ok = issue_dk(i))) break;
        if (i + 1 < nq) issue_dp(i + 1);
      }
      if (ok) mma_commit(final_bar);
      mma_commit(drain_bar);
      mbar_wait_drain(drain_bar, 0);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- compute
    const int g = warp >> 2;                  // warpgroup: query columns [64g, 64g+64) of a step
    const int row = (warp & 3) * 32 + lane;   // key row within the block
    const int kg = n0 + row;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + lane_off + 64 * g;
    const uint32_t t_dp = tmem + lane_off + 128 + 64 * g;
    bool ok = true;
    for (int i = 0; i < nq; ++i) {
      const float* lse_s = reinterpret_cast<const float*>(stage_ptr(i % bwd::STAGES) + 2 * L::TILE) + 64 * g;
      const float* dl_s = lse_s + bwd::STEP;
      const int qc = q_begin + i * bwd::STEP + 64 * g;  // first query of this thread's columns
      float p[64];
      if (!(ok = mbar_wait(s_full, i & 1, abort_flag, kErrBwdCompute))) break;
      tc_fence_after();
      bwd::tmem_ld64(t_s, p);
      {
        const bool need_mask = CAUSAL && (qc < kg);  // some query of these columns precedes the key
        uint32_t pk[32];
#pragma unroll
        for (int e = 0; e < 64; e += 4) {
          const float4 l4 = *reinterpret_cast<const float4*>(lse_s + e);
          p[e + 0] = fast_exp2(fmaf(p[e + 0], scale_log2, -l4.x));
          p[e + 1] = fast_exp2(fmaf(p[e + 1], scale_log2, -l4.y));
          p[e + 2] = fast_exp2(fmaf(p[e + 2], scale_log2, -l4.z));
          p[e + 3] = fast_exp2(fmaf(p[e + 3], scale_log2, -l4.w));
          if (need_mask) {
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (qc + e + u < kg) p[e + u] = 0.f;
          }
          pk[e / 2] = pack_bf16x2(p[e], p[e + 1]);
          pk[e / 2 + 1] = pack_bf16x2(p[e + 2], p[e + 3]);
        }
        tmem_st32(t_s, pk);
        tmem_st_wait();
      }
      tc_fence_before();
      mbar_arrive(p_ready);
      if (!(ok = mbar_wait(dp_full, i & 1, abort_flag, kErrBwdCompute))) break;
      tc_fence_after();
      {
        float dp[64];
        bwd::tmem_ld64(t_dp, dp);
        uint32_t dk[32];
#pragma unroll
        for (int e = 0; e < 64; e += 4) {
          const float4 d4 = *reinterpret_cast<const float4*>(dl_s + e);
          dk[e / 2] = pack_bf16x2(p[e] * (dp[e] - d4.x), p[e + 1] * (dp[e + 1] - d4.y));
          dk[e / 2 + 1] = pack_bf16x2(p[e + 2] * (dp[e + 2] - d4.z), p[e + 3] * (dp[e + 3] - d4.w));
        }
        tmem_st32(t_dp, dk);
        tmem_st_wait();
      }
      tc_fence_before();
      mbar_arrive(ds_ready);
    }
    if (ok && nq > 0 && mbar_wait(final_bar, 0, abort_flag, kErrBwdCompute)) {
      tc_fence_after();
      const long long row_off = static_cast<long long>(bh) * stride_bh + static_cast<long long>(kg) * stride_s;
      bwd::store_acc_half<D>(tmem + lane_off + 256, g, DV + row_off, kg < S, 1.f);
      bwd::store_acc_half<D>(tmem + lane_off + 384, g, DK + row_off, kg < S, scale);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == bwd::MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ====================================================================================
// dQ
// ====================================================================================
// TMEM: S double buffer at columns 0 and 384, dP at 128, dQ at 256.
__device__ __forceinline__ uint32_t dq_sbuf(int b) { return b ? 384u : 0u; }

template <int D, bool CAUSAL>
__global__ void __launch_bounds__(bwd::NTHREADS, 1)
    ffa_bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                      const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                      const float* __restrict__ LSE, const float* __restrict__ DELTA, __nv_bfloat16* __restrict__ DQ,
                      int S, long long stride_bh, long long stride_s, float scale_log2, float scale) {
  using L = bwd::DqLayout<D>;
  constexpr int SLABS = D / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::BAR_OFF;
  constexpr int KS = L::K_STAGES, VS = L::V_STAGES;
  const uint32_t qd_full = bar0;
  auto k_full = [&](int s) { return bar0 + 8 * (1 + s); };
  auto k_empty = [&](int s) { return bar0 + 8 * (1 + KS + s); };
  auto v_full = [&](int s) { return bar0 + 8 * (1 + 2 * KS + s); };
  auto v_empty = [&](int s) { return bar0 + 8 * (1 + 2 * KS + VS + s); };
  auto s_full = [&](int b) { return bar0 + 8 * (1 + 2 * KS + 2 * VS + b); };
  const uint32_t dp_full = bar0 + 8 * (3 + 2 * KS + 2 * VS);
  const uint32_t dp_free = dp_full + 8;
  const uint32_t ds_ready = dp_full + 16;
  const uint32_t final_bar = dp_full + 24;
  const uint32_t drain_bar = dp_full + 32;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nblk = gridDim.x;
  const int qblk = CAUSAL ? (nblk - 1 - static_cast<int>(blockIdx.x)) : static_cast<int>(blockIdx.x);
  const int bh = blockIdx.y;
  const int m0 = qblk * bwd::LANES;
  const int nk_all = (S + bwd::STEP - 1) / bwd::STEP;
  const int nk = CAUSAL ? min(nk_all, m0 / bwd::STEP + 1) : nk_all;

  if (threadIdx.x == 0) {
    mbar_init(qd_full, 1);
    for (int s = 0; s < KS; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    mbar_init(s_full(0), 1);
    mbar_init(s_full(1), 1);
    mbar_init(dp_full, 1);
    mbar_init(dp_free, 256);
    mbar_init(ds_ready, 256);
    mbar_init(final_bar, 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == bwd::MMA_WARP) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp == bwd::PRODUCER_WARP && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == bwd::PRODUCER_WARP) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t keep = policy_evict_last();
      mbar_arrive_expect_tx(qd_full, 2 * L::TILE);
      for (int sl = 0; sl < SLABS; ++sl) {
        tma_load_3d(sbase + L::Q_OFF + sl * 16384, &tm_q, qd_full, sl * 64, m0, bh, keep);
        tma_load_3d(sbase + L::DO_OFF + sl * 16384, &tm_do, qd_full, sl * 64, m0, bh, keep);
      }
      int k_issued = 0, v_issued = 0;
      for (int j = 0; j < nk; ++j) {
        const int sk = j % KS, sv = j % VS;
        if (!mbar_wait(k_empty(sk), ((j / KS) & 1) ^ 1, abort_flag, kErrDqProducer)) break;
        mbar_arrive_expect_tx(k_full(sk), L::TILE);
        for (int sl = 0; sl < SLABS; ++sl)
          tma_load_3d(sbase + L::K_OFF + sk * L::TILE + sl * 16384, &tm_k, k_full(sk), sl * 64, j * bwd::STEP, bh,
                      keep);
        ++k_issued;
        if (!mbar_wait(v_empty(sv), ((j / VS) & 1) ^ 1, abort_flag, kErrDqProducer)) break;
        mbar_arrive_expect_tx(v_full(sv), L::TILE);
        for (int sl = 0; sl < SLABS; ++sl)
          tma_load_3d(sbase + L::V_OFF + sv * L::TILE + sl * 16384, &tm_v, v_full(sv), sl * 64, j * bwd::STEP, bh,
                      keep);
        ++v_issued;
      }
      if (*abort_flag) {
        mbar_wait_drain(qd_full, 0);
        for (int it = max(0, k_issued - KS); it < k_issued; ++it) mbar_wait_drain(k_full(it % KS), (it / KS) & 1);
        for (int it = max(0, v_issued - VS); it < v_issued; ++it) mbar_wait_drain(v_full(it % VS), (it / VS) & 1);
      }
    }
  } else if (warp == bwd::MMA_WARP) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_SD = idesc_bf16(128, bwd::STEP, false, false);  // [128 queries x 128 keys]
      constexpr uint32_t IDESC_G = idesc_bf16(128, D, false, true);            // [128 queries x D]
      const uint32_t q_addr = sbase + L::Q_OFF, do_addr = sbase + L::DO_OFF;
      auto k_addr = [&](int j) { return sbase + L::K_OFF + (j % KS) * L::TILE; };
      auto v_addr = [&](int j) { return sbase + L::V_OFF + (j % VS) * L::TILE; };
      auto issue_s = [&](int j) -> bool {  // S_j = Q K_j^T into buffer j&1
        if (!mbar_wait(k_full(j % KS), (j / KS) & 1, abort_flag, kErrDqMma)) return false;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          mma_ss(tmem + dq_sbuf(j & 1), kmajor_desc(q_addr, 128, ks), kmajor_desc(k_addr(j), 128, ks), IDESC_SD,
                 ks > 0);
        mma_commit(s_full(j & 1));
        return true;
      };
      auto issue_dp = [&](int j) -> bool {  // dP_j = dO V_j^T
        if (!mbar_wait(v_full(j % VS), (j / VS) & 1, abort_flag, kErrDqMma)) return false;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          mma_ss(tmem + 128, kmajor_desc(do_addr, 128, ks), kmajor_desc(v_addr(j), 128, ks), IDESC_SD, ks > 0);
        mma_commit(dp_full);
        mma_commit(v_empty(j % VS));
        return true;
      };
      auto issue_g = [&](int j) -> bool {  // dQ += dS_j K_j
        if (!mbar_wait(ds_ready, j & 1, abort_flag, kErrDqMma)) return false;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < bwd::STEP / 16; ++ks)
          mma_ts(tmem + 256, bwd::packed_kstep_col(tmem + dq_sbuf(j & 1), ks), mnmajor_desc(k_addr(j), 128, ks),
                 IDESC_G, (j > 0 || ks > 0) ? 1u : 0u);
        mma_commit(k_empty(j % KS));
        return true;
      };
      bool ok = mbar_wait(qd_full, 0, abort_flag, kErrDqMma);
      if (ok && nk > 0) {
        ok = issue_s(0);
        if (ok) ok = issue_dp(0);
      }
      // S(j+1) and dP(j+1) run while the warpgroups turn step j into dS; dP(j+1) waits
      // only until the warpgroups have copied dP(j) out of tensor memory.
      for (int j = 0; j < nk && ok; ++j) {
        if (j + 1 < nk) {
          if (!(ok = issue_s(j + 1))) break;
          if (!(ok = mbar_wait(dp_free, j & 1, abort_flag, kErrDqMma))) break;
          tc_fence_after();
          if (!(ok = issue_dp(j + 1))) break;
        }
        if (!(ok = issue_g(j))) break;
      }
      if (ok) mma_commit(final_bar);
      mma_commit(drain_bar);
      mbar_wait_drain(drain_bar, 0);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- compute
    const int g = warp >> 2;
    const int row = (warp & 3) * 32 + lane;  // query row within the block
    const int qg = m0 + row;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const long long ridx = static_cast<long long>(bh) * S + qg;
    const float lse = (qg < S) ? LSE[ridx] : INFINITY;
    const float dl = (qg < S) ? DELTA[ridx] : 0.f;
    const int lim = CAUSAL ? min(S - 1, qg) : S - 1;  // last visible key
    bool ok = true;
    for (int j = 0; j < nk; ++j) {
      const int b = j & 1;
      if (!(ok = mbar_wait(s_full(b), (j >> 1) & 1, abort_flag, kErrDqCompute))) break;
      if (!(ok = mbar_wait(dp_full, j & 1, abort_flag, kErrDqCompute))) break;
      tc_fence_after();
      float sv[64], dp[64];
      bwd::tmem_ld64(tmem + lane_off + dq_sbuf(b) + 64 * g, sv);
      bwd::tmem_ld64(tmem + lane_off + 128 + 64 * g, dp);
      tc_fence_before();
      mbar_arrive(dp_free);
      const int kc = j * bwd::STEP + 64 * g;  // first key of this thread's columns
      const bool need_mask = (kc + 64 > S) || (CAUSAL && kc + 63 > qg);
      uint32_t dsp[32];
#pragma unroll
      for (int e = 0; e < 64; e += 2) {
        float p0 = fast_exp2(fmaf(sv[e], scale_log2, -lse));
        float p1 = fast_exp2(fmaf(sv[e + 1], scale_log2, -lse));
        if (need_mask) {
          if (kc + e > lim) p0 = 0.f;
          if (kc + e + 1 > lim) p1 = 0.f;
        }
        dsp[e >> 1] = pack_bf16x2(p0 * (dp[e] - dl), p1 * (dp[e + 1] - dl));
      }
      tmem_st32(tmem + lane_off + dq_sbuf(b) + 64 * g, dsp);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(ds_ready);
    }
    if (ok && nk > 0 && mbar_wait(final_bar, 0, abort_flag, kErrDqCompute)) {
      tc_fence_after();
      const long long row_off = static_cast<long long>(bh) * stride_bh + static_cast<long long>(qg) * stride_s;
      bwd::store_acc_half<D>(tmem + lane_off + 256, g, DQ + row_off, qg < S, scale);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == bwd::MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------------
// host launchers
// ------------------------------------------------------------------------------------
template <int D, bool CAUSAL>
static int launch_dkdv_t(const BwdArgs& a, cudaStream_t stream) {
  using LK = bwd::DkdvLayout<D>;
  CUtensorMap tk, tv, tq, tdo;
  int rc;
  if ((rc = make_tile_map(&tk, a.k, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  if ((rc = make_tile_map(&tv, a.v, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  if ((rc = make_tile_map(&tq, a.q, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  if ((rc = make_tile_map(&tdo, a.dout, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  auto kern = ffa_bwd_dkdv_kernel<D, CAUSAL>;
  static unsigned long long configured = 0;
  if ((rc = set_smem_once(reinterpret_cast<const void*>(kern), LK::SMEM_BYTES, &configured))) return rc;
  const dim3 grid((a.S + bwd::LANES - 1) / bwd::LANES, a.BH);
  kern<<<grid, bwd::NTHREADS, LK::SMEM_BYTES, stream>>>(tk, tv, tq, tdo, a.lse, a.delta,
                                                        static_cast<__nv_bfloat16*>(a.dk),
                                                        static_cast<__nv_bfloat16*>(a.dv), a.S, a.stride_bh,
                                                        a.stride_s, static_cast<float>(a.scale * kLog2e),
                                                        static_cast<float>(a.scale));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FFA_ERR_LAUNCH, cudaGetErrorString(e));
  return FFA_OK;
}

template <int D, bool CAUSAL>
static int launch_dq_t(const BwdArgs& a, cudaStream_t stream) {
  using LQ = bwd::DqLayout<D>;
  CUtensorMap tq, tdo, tk, tv;
  int rc;
  if ((rc = make_tile_map(&tq, a.q, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  if ((rc = make_tile_map(&tdo, a.dout, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  if ((rc = make_tile_map(&tk, a.k, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  if ((rc = make_tile_map(&tv, a.v, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  auto kern = ffa_bwd_dq_kernel<D, CAUSAL>;
  static unsigned long long configured = 0;
  if ((rc = set_smem_once(reinterpret_cast<const void*>(kern), LQ::SMEM_BYTES, &configured))) return rc;
  const dim3 grid((a.S + bwd::LANES - 1) / bwd::LANES, a.BH);
  kern<<<grid, bwd::NTHREADS, LQ::SMEM_BYTES, stream>>>(tq, tdo, tk, tv, a.lse, a.delta,
                                                        static_cast<__nv_bfloat16*>(a.dq), a.S, a.stride_bh,
                                                        a.stride_s, static_cast<float>(a.scale * kLog2e),
                                                        static_cast<float>(a.scale));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FFA_ERR_LAUNCH, cudaGetErrorString(e));
  return FFA_OK;
}

int launch_dkdv(const BwdArgs& a, cudaStream_t stream) {
  if (a.D == 128) return a.causal ? launch_dkdv_t<128, true>(a, stream) : launch_dkdv_t<128, false>(a, stream);
  if (a.D == 64) return a.causal ? launch_dkdv_t<64, true>(a, stream) : launch_dkdv_t<64, false>(a, stream);
  return set_error(FFA_ERR_UNSUPPORTED, "kernel head_dim must be 64 or 128");
}

int launch_dq(const BwdArgs& a, cudaStream_t stream) {
  if (a.D == 128) return a.causal ? launch_dq_t<128, true>(a, stream) : launch_dq_t<128, false>(a, stream);
  if (a.D == 64) return a.causal ? launch_dq_t<64, true>(a, stream) : launch_dq_t<64, false>(a, stream);
  return set_error(FFA_ERR_UNSUPPORTED, "kernel head_dim must be 64 or 128");
}

int launch_bwd(const BwdArgs& a, cudaStream_t stream) {
  int rc;
  if ((rc = launch_preprocess(a.o, a.dout, a.delta, a.BH, a.S, a.D, a.stride_bh, a.stride_s, stream))) return rc;
  if ((rc = launch_dkdv(a, stream))) return rc;
  return launch_dq(a, stream);
}

}  // namespace ffa
