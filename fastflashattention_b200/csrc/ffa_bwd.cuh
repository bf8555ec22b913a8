// ffa_bwd.cuh — deterministic attention backward for sm_100a.
//
// Two kernels with disjoint output tiles and no atomics, the split of the reference
// backward (fastflash_attention/_kernel.py:379-448 dK/dV, :487-564 dQ, recompute path):
//
//   dkdv kernel (grid over 128-key blocks, loop over 64-query blocks)
//     S^T  = K Q^T            P^T  = exp2(scale*log2e*S^T - lse)   (masked)
//     dP^T = V dO^T           dS^T = P^T * (dP^T - delta)
//     dV  += bf16(P^T) dO     dK  += bf16(dS^T) Q        dK *= scale at the end
//   dq kernel (grid over 128-query blocks, loop over 64-key blocks)
//     S = Q K^T, dP = dO V^T, dS = P*(dP - delta), dQ += bf16(dS) K, dQ *= scale
//
// The backward preprocess delta = rowsum(O*dO) (ffa_aux.cuh) runs first.
//
// Both kernels share one shape: a CTA owns 128 TMEM lanes (keys for dkdv, queries
// for dq) and walks the other dimension in 64-wide steps.
//   warps 0-7  two compute warpgroups; warpgroup g handles columns [32g, 32g+32) of
//              every 64-wide step (thread = TMEM lane = one key / query row)
//   warp  8    producer: TMA for the streamed tiles (and lse/delta for dkdv)
//   warp  9    MMA issuer (one thread)
// TMEM: S_b at 64b, dP_b at 128+64b (b = 0,1 double buffer), accumulators at 256/384.
// P and dS are written back over their own S / dP columns as packed bf16 and feed
// the gradient MMAs straight from tensor memory.  The issue order
//   SD(0) SD(1) G(0) SD(2) G(1) ...   (SD = S and dP MMAs, G = gradient MMAs)
// keeps the next step's S/dP on the tensor core while the warpgroups work on this one.
#pragma once
#include "ffa_common.cuh"

namespace ffa {

namespace bwd {
constexpr int LANES = 128;   // TMEM lanes owned by a CTA
constexpr int STEP = 64;     // width of one step along the streamed dimension
constexpr int STAGES = 3;
constexpr int NTHREADS = 320;
constexpr int PRODUCER_WARP = 8;
constexpr int MMA_WARP = 9;

template <int D>
struct DkdvLayout {
  static constexpr int KV_TILE = LANES * D * 2;     // resident K or V tile
  static constexpr int STEP_TILE = STEP * D * 2;    // streamed Q or dO tile
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = KV_TILE;
  static constexpr int STAGE_OFF = 2 * KV_TILE;
  // stage: Q tile, dO tile, lse[64], delta[64]
  static constexpr int STAGE_BYTES = ((2 * STEP_TILE + 2 * STEP * 4) + 1023) / 1024 * 1024;
  static constexpr int BAR_OFF = STAGE_OFF + STAGES * STAGE_BYTES;
  // kv_full, st_full[S], st_empty[S], s_full[2], ready[2], final, drain
  static constexpr int NBARS = 1 + 2 * STAGES + 2 + 2 + 2;
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  static constexpr int SMEM_BYTES = MISC_OFF + 16 + 1024;
};

template <int D>
struct DqLayout {
  static constexpr int QD_TILE = LANES * D * 2;     // resident Q or dO tile
  static constexpr int STEP_TILE = STEP * D * 2;    // streamed K or V tile
  static constexpr int Q_OFF = 0;
  static constexpr int DO_OFF = QD_TILE;
  static constexpr int STAGE_OFF = 2 * QD_TILE;
  static constexpr int STAGE_BYTES = 2 * STEP_TILE;  // K tile, V tile
  static constexpr int BAR_OFF = STAGE_OFF + STAGES * STAGE_BYTES;
  static constexpr int NBARS = 1 + 2 * STAGES + 2 + 2 + 2;
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  static constexpr int SMEM_BYTES = MISC_OFF + 16 + 1024;
};

// TMEM column of the 16-element K-step `ks` of a packed-bf16 operand written by the two
// warpgroups: warpgroup g put columns [32g, 32g+32) of the step at base + 32g (16 cols).
__device__ __forceinline__ uint32_t packed_kstep_col(uint32_t base, int ks) {
  return base + (ks >> 1) * 32 + (ks & 1) * 8;
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
  auto s_full = [&](int b) { return bar0 + 8 * (1 + 2 * bwd::STAGES + b); };
  auto ready = [&](int b) { return bar0 + 8 * (3 + 2 * bwd::STAGES + b); };
  const uint32_t final_bar = bar0 + 8 * (5 + 2 * bwd::STAGES);
  const uint32_t drain_bar = bar0 + 8 * (6 + 2 * bwd::STAGES);
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
    for (int b = 0; b < 2; ++b) {
      mbar_init(s_full(b), 1);
      mbar_init(ready(b), 256);
    }
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
      mbar_arrive_expect_tx(kv_full, 2 * L::KV_TILE);
      for (int sl = 0; sl < SLABS; ++sl) {
        tma_load_3d(sbase + L::K_OFF + sl * (bwd::LANES * 128), &tm_k, kv_full, sl * 64, n0, bh, keep);
        tma_load_3d(sbase + L::V_OFF + sl * (bwd::LANES * 128), &tm_v, kv_full, sl * 64, n0, bh, keep);
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
        mbar_arrive_expect_tx(st_full(s), 2 * L::STEP_TILE);
        for (int sl = 0; sl < SLABS; ++sl) {
          tma_load_3d(st + sl * (bwd::STEP * 128), &tm_q, st_full(s), sl * 64, q0, bh, keep);
          tma_load_3d(st + L::STEP_TILE + sl * (bwd::STEP * 128), &tm_do, st_full(s), sl * 64, q0, bh, keep);
        }
      }
      float* lse_s = reinterpret_cast<float*>(stage_ptr(s) + 2 * L::STEP_TILE);
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
      constexpr uint32_t IDESC_SD = idesc_bf16(128, bwd::STEP, false, false);  // [128 keys x 64 queries]
      constexpr uint32_t IDESC_G = idesc_bf16(128, D, false, true);            // [128 keys x D]
      const uint32_t k_addr = sbase + L::K_OFF, v_addr = sbase + L::V_OFF;
      bool ok = mbar_wait(kv_full, 0, abort_flag, kErrBwdMma);
      auto issue_sd = [&](int i) -> bool {
        const int s = i % bwd::STAGES, b = i & 1;
        if (!mbar_wait(st_full(s), (i / bwd::STAGES) & 1, abort_flag, kErrBwdMma)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(stage_ptr(s)), da = qa + L::STEP_TILE;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          mma_ss(tmem + 64 * b, kmajor_desc(k_addr, bwd::LANES, ks), kmajor_desc(qa, bwd::STEP, ks), IDESC_SD, ks > 0);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          mma_ss(tmem + 128 + 64 * b, kmajor_desc(v_addr, bwd::LANES, ks), kmajor_desc(da, bwd::STEP, ks), IDESC_SD,
                 ks > 0);
        mma_commit(s_full(b));
        return true;
      };
      auto issue_grad = [&](int i) -> bool {
        const int s = i % bwd::STAGES, b = i & 1;
        if (!mbar_wait(ready(b), (i >> 1) & 1, abort_flag, kErrBwdMma)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(stage_ptr(s)), da = qa + L::STEP_TILE;
#pragma unroll
        for (int ks = 0; ks < bwd::STEP / 16; ++ks)  // dV += P^T dO
          mma_ts(tmem + 256, bwd::packed_kstep_col(tmem + 64 * b, ks), mnmajor_desc(da, bwd::STEP, ks), IDESC_G,
                 (i > 0 || ks > 0) ? 1u : 0u);
#pragma unroll
        for (int ks = 0; ks < bwd::STEP / 16; ++ks)  // dK += dS^T Q
          mma_ts(tmem + 384, bwd::packed_kstep_col(tmem + 128 + 64 * b, ks), mnmajor_desc(qa, bwd::STEP, ks),
                 IDESC_G, (i > 0 || ks > 0) ? 1u : 0u);
        mma_commit(st_empty(s));
        return true;
      };
      if (ok && nq > 0) ok = issue_sd(0);
      for (int i = 0; i < nq && ok; ++i) {
        if (i + 1 < nq && !(ok = issue_sd(i + 1))) break;
        ok = issue_grad(i);
      }
      if (ok) mma_commit(final_bar);
      mma_commit(drain_bar);
      mbar_wait_drain(drain_bar, 0);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- compute
    const int g = warp >> 2;                  // warpgroup: columns [32g, 32g+32) of a step
    const int row = (warp & 3) * 32 + lane;   // key row within the block
    const int kg = n0 + row;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    bool ok = true;
    for (int i = 0; i < nq; ++i) {
      const int s = i % bwd::STAGES, b = i & 1;
      if (!(ok = mbar_wait(s_full(b), (i >> 1) & 1, abort_flag, kErrBwdCompute))) break;
      tc_fence_after();
      uint32_t rs[32], rdp[32];
      tmem_ld32(tmem + lane_off + 64 * b + 32 * g, rs);
      tmem_ld32(tmem + lane_off + 128 + 64 * b + 32 * g, rdp);
      tmem_ld_wait();
      const float* lse_s = reinterpret_cast<const float*>(stage_ptr(s) + 2 * L::STEP_TILE) + 32 * g;
      const float* dl_s = lse_s + bwd::STEP;
      const int qc = q_begin + i * bwd::STEP + 32 * g;  // first query of this thread's columns
      const bool need_mask = CAUSAL && (qc < kg);  // some query of these columns precedes the key
      uint32_t pp[16], dsp[16];
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        const float4 l2 = *reinterpret_cast<const float4*>(lse_s + (e & ~3));
        const float4 d2 = *reinterpret_cast<const float4*>(dl_s + (e & ~3));
        const float la = (e & 2) ? l2.z : l2.x, lb = (e & 2) ? l2.w : l2.y;
        const float da = (e & 2) ? d2.z : d2.x, db = (e & 2) ? d2.w : d2.y;
        float p0 = fast_exp2(fmaf(__uint_as_float(rs[e]), scale_log2, -la));
        float p1 = fast_exp2(fmaf(__uint_as_float(rs[e + 1]), scale_log2, -lb));
        if (need_mask) {
          if (qc + e < kg) p0 = 0.f;
          if (qc + e + 1 < kg) p1 = 0.f;
        }
        const float ds0 = p0 * (__uint_as_float(rdp[e]) - da);
        const float ds1 = p1 * (__uint_as_float(rdp[e + 1]) - db);
        pp[e >> 1] = pack_bf16x2(p0, p1);
        dsp[e >> 1] = pack_bf16x2(ds0, ds1);
      }
      {
        uint32_t tmp[32];
#pragma unroll
        for (int e = 0; e < 16; ++e) tmp[e] = pp[e];
#pragma unroll
        for (int e = 16; e < 32; ++e) tmp[e] = 0u;
        // 16 packed columns; the upper 16 columns of this warpgroup's half are not read
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
            "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(tmem + lane_off + 64 * b + 32 * g),
            "r"(tmp[0]), "r"(tmp[1]), "r"(tmp[2]), "r"(tmp[3]), "r"(tmp[4]), "r"(tmp[5]), "r"(tmp[6]), "r"(tmp[7]),
            "r"(tmp[8]), "r"(tmp[9]), "r"(tmp[10]), "r"(tmp[11]), "r"(tmp[12]), "r"(tmp[13]), "r"(tmp[14]),
            "r"(tmp[15])
            : "memory");
        asm volatile(
            "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
            "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(tmem + lane_off + 128 + 64 * b + 32 * g),
            "r"(dsp[0]), "r"(dsp[1]), "r"(dsp[2]), "r"(dsp[3]), "r"(dsp[4]), "r"(dsp[5]), "r"(dsp[6]), "r"(dsp[7]),
            "r"(dsp[8]), "r"(dsp[9]), "r"(dsp[10]), "r"(dsp[11]), "r"(dsp[12]), "r"(dsp[13]), "r"(dsp[14]),
            "r"(dsp[15])
            : "memory");
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(ready(b));
    }
    if (ok && nq > 0 && mbar_wait(final_bar, 0, abort_flag, kErrBwdCompute)) {
      tc_fence_after();
      const long long row_off = static_cast<long long>(bh) * stride_bh + static_cast<long long>(kg) * stride_s;
      // warpgroup g writes columns [g*D/2, (g+1)*D/2) of dV and dK
#pragma unroll 1
      for (int c = g * (D / 64); c < (g + 1) * (D / 64); ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + 256 + 32 * c, r);
        tmem_ld_wait();
        if (kg < S) bwd::store_row32(DV + row_off + 32 * c, r, 1.f);
        tmem_ld32(tmem + lane_off + 384 + 32 * c, r);
        tmem_ld_wait();
        if (kg < S) bwd::store_row32(DK + row_off + 32 * c, r, scale);
      }
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
  const uint32_t qd_full = bar0;
  auto kv_full = [&](int s) { return bar0 + 8 * (1 + s); };
  auto kv_empty = [&](int s) { return bar0 + 8 * (1 + bwd::STAGES + s); };
  auto s_full = [&](int b) { return bar0 + 8 * (1 + 2 * bwd::STAGES + b); };
  auto ready = [&](int b) { return bar0 + 8 * (3 + 2 * bwd::STAGES + b); };
  const uint32_t final_bar = bar0 + 8 * (5 + 2 * bwd::STAGES);
  const uint32_t drain_bar = bar0 + 8 * (6 + 2 * bwd::STAGES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nblk = gridDim.x;
  const int qblk = CAUSAL ? (nblk - 1 - static_cast<int>(blockIdx.x)) : static_cast<int>(blockIdx.x);
  const int bh = blockIdx.y;
  const int m0 = qblk * bwd::LANES;
  const int nk_all = (S + bwd::STEP - 1) / bwd::STEP;
  const int nk = CAUSAL ? min(nk_all, (m0 + bwd::LANES - 1) / bwd::STEP + 1) : nk_all;

  if (threadIdx.x == 0) {
    mbar_init(qd_full, 1);
    for (int s = 0; s < bwd::STAGES; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(s_full(b), 1);
      mbar_init(ready(b), 256);
    }
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
      mbar_arrive_expect_tx(qd_full, 2 * L::QD_TILE);
      for (int sl = 0; sl < SLABS; ++sl) {
        tma_load_3d(sbase + L::Q_OFF + sl * (bwd::LANES * 128), &tm_q, qd_full, sl * 64, m0, bh, keep);
        tma_load_3d(sbase + L::DO_OFF + sl * (bwd::LANES * 128), &tm_do, qd_full, sl * 64, m0, bh, keep);
      }
      int issued = 0;
      for (int j = 0; j < nk; ++j) {
        const int s = j % bwd::STAGES;
        if (!mbar_wait(kv_empty(s), ((j / bwd::STAGES) & 1) ^ 1, abort_flag, kErrDqProducer)) break;
        const uint32_t st = sbase + L::STAGE_OFF + s * L::STAGE_BYTES;
        mbar_arrive_expect_tx(kv_full(s), 2 * L::STEP_TILE);
        for (int sl = 0; sl < SLABS; ++sl) {
          tma_load_3d(st + sl * (bwd::STEP * 128), &tm_k, kv_full(s), sl * 64, j * bwd::STEP, bh, keep);
          tma_load_3d(st + L::STEP_TILE + sl * (bwd::STEP * 128), &tm_v, kv_full(s), sl * 64, j * bwd::STEP, bh,
                      keep);
        }
        ++issued;
      }
      if (*abort_flag) {
        mbar_wait_drain(qd_full, 0);
        for (int it = max(0, issued - bwd::STAGES); it < issued; ++it)
          mbar_wait_drain(kv_full(it % bwd::STAGES), (it / bwd::STAGES) & 1);
      }
    }
  } else if (warp == bwd::MMA_WARP) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_SD = idesc_bf16(128, bwd::STEP, false, false);  // [128 queries x 64 keys]
      constexpr uint32_t IDESC_G = idesc_bf16(128, D, false, true);            // [128 queries x D]
      const uint32_t q_addr = sbase + L::Q_OFF, do_addr = sbase + L::DO_OFF;
      bool ok = mbar_wait(qd_full, 0, abort_flag, kErrDqMma);
      auto issue_sd = [&](int j) -> bool {
        const int s = j % bwd::STAGES, b = j & 1;
        if (!mbar_wait(kv_full(s), (j / bwd::STAGES) & 1, abort_flag, kErrDqMma)) return false;
        tc_fence_after();
        const uint32_t ka = sbase + L::STAGE_OFF + s * L::STAGE_BYTES, va = ka + L::STEP_TILE;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          mma_ss(tmem + 64 * b, kmajor_desc(q_addr, bwd::LANES, ks), kmajor_desc(ka, bwd::STEP, ks), IDESC_SD, ks > 0);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks)
          mma_ss(tmem + 128 + 64 * b, kmajor_desc(do_addr, bwd::LANES, ks), kmajor_desc(va, bwd::STEP, ks), IDESC_SD,
                 ks > 0);
        mma_commit(s_full(b));
        return true;
      };
      auto issue_grad = [&](int j) -> bool {
        const int s = j % bwd::STAGES, b = j & 1;
        if (!mbar_wait(ready(b), (j >> 1) & 1, abort_flag, kErrDqMma)) return false;
        tc_fence_after();
        const uint32_t ka = sbase + L::STAGE_OFF + s * L::STAGE_BYTES;
#pragma unroll
        for (int ks = 0; ks < bwd::STEP / 16; ++ks)  // dQ += dS K
          mma_ts(tmem + 256, bwd::packed_kstep_col(tmem + 128 + 64 * b, ks), mnmajor_desc(ka, bwd::STEP, ks), IDESC_G,
                 (j > 0 || ks > 0) ? 1u : 0u);
        mma_commit(kv_empty(s));
        return true;
      };
      if (ok && nk > 0) ok = issue_sd(0);
      for (int j = 0; j < nk && ok; ++j) {
        if (j + 1 < nk && !(ok = issue_sd(j + 1))) break;
        ok = issue_grad(j);
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
    bool ok = true;
    for (int j = 0; j < nk; ++j) {
      const int b = j & 1;
      if (!(ok = mbar_wait(s_full(b), (j >> 1) & 1, abort_flag, kErrDqCompute))) break;
      tc_fence_after();
      uint32_t rs[32], rdp[32];
      tmem_ld32(tmem + lane_off + 64 * b + 32 * g, rs);
      tmem_ld32(tmem + lane_off + 128 + 64 * b + 32 * g, rdp);
      tmem_ld_wait();
      const int kc = j * bwd::STEP + 32 * g;  // first key of this thread's columns
      const bool need_mask = (kc + 32 > S) || (CAUSAL && kc + 31 > m0);
      const int lim = CAUSAL ? min(S - 1, qg) : S - 1;
      uint32_t dsp[16];
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float p0 = fast_exp2(fmaf(__uint_as_float(rs[e]), scale_log2, -lse));
        float p1 = fast_exp2(fmaf(__uint_as_float(rs[e + 1]), scale_log2, -lse));
        if (need_mask) {
          if (kc + e > lim) p0 = 0.f;
          if (kc + e + 1 > lim) p1 = 0.f;
        }
        dsp[e >> 1] = pack_bf16x2(p0 * (__uint_as_float(rdp[e]) - dl), p1 * (__uint_as_float(rdp[e + 1]) - dl));
      }
      asm volatile(
          "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
          "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(tmem + lane_off + 128 + 64 * b + 32 * g),
          "r"(dsp[0]), "r"(dsp[1]), "r"(dsp[2]), "r"(dsp[3]), "r"(dsp[4]), "r"(dsp[5]), "r"(dsp[6]), "r"(dsp[7]),
          "r"(dsp[8]), "r"(dsp[9]), "r"(dsp[10]), "r"(dsp[11]), "r"(dsp[12]), "r"(dsp[13]), "r"(dsp[14]),
          "r"(dsp[15])
          : "memory");
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(ready(b));
    }
    if (ok && nk > 0 && mbar_wait(final_bar, 0, abort_flag, kErrDqCompute)) {
      tc_fence_after();
      const long long row_off = static_cast<long long>(bh) * stride_bh + static_cast<long long>(qg) * stride_s;
#pragma unroll 1
      for (int c = g * (D / 64); c < (g + 1) * (D / 64); ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_off + 256 + 32 * c, r);
        tmem_ld_wait();
        if (qg < S) bwd::store_row32(DQ + row_off + 32 * c, r, scale);
      }
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
  if ((rc = make_tile_map(&tk, a.k, a.BH, a.S, D, a.stride_bh, a.stride_s, bwd::LANES))) return rc;
  if ((rc = make_tile_map(&tv, a.v, a.BH, a.S, D, a.stride_bh, a.stride_s, bwd::LANES))) return rc;
  if ((rc = make_tile_map(&tq, a.q, a.BH, a.S, D, a.stride_bh, a.stride_s, bwd::STEP))) return rc;
  if ((rc = make_tile_map(&tdo, a.dout, a.BH, a.S, D, a.stride_bh, a.stride_s, bwd::STEP))) return rc;
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
  if ((rc = make_tile_map(&tq, a.q, a.BH, a.S, D, a.stride_bh, a.stride_s, bwd::LANES))) return rc;
  if ((rc = make_tile_map(&tdo, a.dout, a.BH, a.S, D, a.stride_bh, a.stride_s, bwd::LANES))) return rc;
  if ((rc = make_tile_map(&tk, a.k, a.BH, a.S, D, a.stride_bh, a.stride_s, bwd::STEP))) return rc;
  if ((rc = make_tile_map(&tv, a.v, a.BH, a.S, D, a.stride_bh, a.stride_s, bwd::STEP))) return rc;
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
