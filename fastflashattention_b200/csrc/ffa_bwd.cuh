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
//   warp  8    producer: TMA for the streamed tiles (dkdv: Q; warp 10 streams dO with
//              lse/delta beside it)
//   warp  9    MMA issuer (the whole warp runs the loop, an elected lane issues)
// P and dS are written back to tensor memory as packed bf16 and feed the gradient MMAs
// from there.  In the dq kernel dS overwrites the S columns it came from (warpgroup g's
// 64 values land in [64g, 64g+32)).  In the dkdv kernel P and dS both go into the dP
// columns once dP is in registers (warpgroup g: P at [64g, 64g+32), dS at
// [64g+32, 64g+64) of the dP region), which frees the S columns for the next step's
// S = K Q^T while this step's softmax is still running.
#pragma once
#include "ffa_common.cuh"

// Timeline hook for measurement builds (clock64 at fixed points of one CTA); expands to
// nothing in the library.
#ifndef FFA_BWD_TRACE
#define FFA_BWD_TRACE(site, step)
#endif

namespace ffa {

namespace bwd {
constexpr int LANES = 128;   // TMEM lanes owned by a CTA
constexpr int STEP = 128;    // width of one step along the streamed dimension
constexpr int STAGES = 2;
constexpr int NTHREADS = 384;  // 2 compute warpgroups + producer, MMA and 2 idle warps
constexpr int PRODUCER_WARP = 8;
constexpr int MMA_WARP = 9;
constexpr int DO_PRODUCER_WARP = 10;  // dkdv: the dO ring has its own producer
// Register split after launch (384 x 168): compute warpgroups 208, control warpgroup 88.
constexpr int REGS_COMPUTE = 208;
constexpr int REGS_CONTROL = 88;
constexpr int LAUNCH_REGS_NEEDED = (2 * 128 * REGS_COMPUTE + 128 * REGS_CONTROL) / NTHREADS;

template <int D>
struct DkdvLayout {
  static constexpr int TILE = 128 * D * 2;  // K, V (resident) and Q, dO (streamed) tiles
  // Q_i is read by S(i) (issued a step early) and by dK(i) (at the end of step i), dO_i
  // by dP(i) and dV(i) within one step: three Q slots and two dO slots.
  static constexpr int Q_STAGES = 3;
  static constexpr int DO_STAGES = 2;
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = TILE;
  static constexpr int Q_OFF = 2 * TILE;
  static constexpr int DO_OFF = Q_OFF + Q_STAGES * TILE;
  static constexpr int DO_STAGE_BYTES = TILE + 2 * STEP * 4;  // dO tile, lse[128], delta[128]
  static constexpr int BAR_OFF = DO_OFF + DO_STAGES * DO_STAGE_BYTES;
  // kv_full, q_full[3], q_empty[3], do_full[2], do_empty[2], s_full, dp_full, p_ready,
  // ds_ready, final, drain, s_free
  static constexpr int NBARS = 1 + 2 * Q_STAGES + 2 * DO_STAGES + 7;
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  // no alignment slack: the kernel declares its dynamic shared memory 1024-byte aligned
  // (and checks it), which is what lets this layout fit in 227 KB
  static constexpr int SMEM_BYTES = MISC_OFF + 16;
};

template <int D>
struct DqLayout {
  static constexpr int TILE = 128 * D * 2;  // K, V (streamed) tiles; Q and dO live in TMEM
  static constexpr int K_STAGES = 4;        // K_j is read by S_j and, a step later, by dQ += dS_j K_j
  static constexpr int V_STAGES = 3;        // V_j is read by dP_j only
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = K_OFF + K_STAGES * TILE;
  static constexpr int BAR_OFF = V_OFF + V_STAGES * TILE;
  // qd_ready, k_full[4], k_empty[4], v_full[3], v_empty[3], s_full, s_free, dp_full,
  // ds_ready, final, drain
  static constexpr int NBARS = 1 + 2 * K_STAGES + 2 * V_STAGES + 6;
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;
  static constexpr int SMEM_BYTES = MISC_OFF + 16 + 1024;
};

// Whether group g of 4 consecutive exponentials (of the 64 a thread computes per step)
// goes to the FMA pipe instead of MUFU.EX2.  At D=64 the MMAs of a step take half as long
// and 1 group in 4 moves over in both kernels (FFA_BWD_EMU_D64 overrides the count at
// build time, for measurements).  At D=128, 1 group in 4 in the dK/dV kernel measured
// 2.7-3 % faster at B4 H16 causal S=512..8192, while the dQ kernel was 1.5 % slower with
// it and keeps every exponential on MUFU.
#ifndef FFA_BWD_EMU_D64
#define FFA_BWD_EMU_D64 1
#endif
#ifndef FFA_BWD_EMU_DKDV_D128
#define FFA_BWD_EMU_DKDV_D128 1
#endif
#ifndef FFA_BWD_EMU_DQ_D128
#define FFA_BWD_EMU_DQ_D128 0
#endif
template <int D, bool DKDV>
__device__ __forceinline__ constexpr bool emu_group(int g) {
  return (g & 3) < (D == 64 ? FFA_BWD_EMU_D64 : (DKDV ? FFA_BWD_EMU_DKDV_D128 : FFA_BWD_EMU_DQ_D128));
}

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

// Stage the accumulator columns [g*D/2, (g+1)*D/2) of this lane (TMEM row = tile row) as
// bf16 into a 128-row tile in shared memory laid out for a SWIZZLE_128B TMA store.
template <int D>
__device__ __forceinline__ void stage_acc_half(uint32_t t_acc, int g, uint32_t tile, int row, float mul) {
#pragma unroll 1
  for (int c = g * (D / 64); c < (g + 1) * (D / 64); ++c) {
    uint32_t r[32];
    tmem_ld32(t_acc + 32 * c, r);
    tmem_ld_wait();
    stage_row32_sw128(tile, row, 32 * c, r, mul);
  }
}

// Add the accumulator columns [g*D/2, (g+1)*D/2) of this lane, times `mul`, to the fp32
// row `dst` (D floats, 16-byte aligned) when `valid`.  Every lane of the warp must call
// it (tcgen05.ld is warp-wide); lanes past the end pass valid = false.
template <int D>
__device__ __forceinline__ void add_acc_half(uint32_t t_acc, int g, float* dst, bool valid, float mul) {
#pragma unroll 1
  for (int c = g * (D / 64); c < (g + 1) * (D / 64); ++c) {
    uint32_t r[32];
    tmem_ld32(t_acc + 32 * c, r);
    tmem_ld_wait();
    if (valid) {
      float4* d4 = reinterpret_cast<float4*>(dst + 32 * c);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float4 a = d4[e];
        a.x = fmaf(__uint_as_float(r[4 * e + 0]), mul, a.x);
        a.y = fmaf(__uint_as_float(r[4 * e + 1]), mul, a.y);
        a.z = fmaf(__uint_as_float(r[4 * e + 2]), mul, a.z);
        a.w = fmaf(__uint_as_float(r[4 * e + 3]), mul, a.w);
        d4[e] = a;
      }
    }
  }
}

// Every one of the 256 compute threads calls this, staged or not (a thread that left its
// loop early after a timeout passes staged = false): it is a barrier for all of them.  If
// all staged their rows, one thread stores the tiles (64-column boxes) with TMA and waits
// for the stores to finish reading shared memory.  Rows at or past S are clipped by the tensor map.
template <int D, int NT>
__device__ __forceinline__ void store_staged(bool staged, const CUtensorMap* const (&maps)[NT], uint32_t first_tile,
                                             int row0, int bh) {
  fence_proxy_async_smem();
  const bool all = named_barrier_and(1, 256, staged);
  if (all && threadIdx.x == 0) {
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int sl = 0; sl < D / 64; ++sl)
        tma_store_3d(maps[t], first_tile + t * (128 * D * 2) + sl * 16384, sl * 64, row0, bh);
    bulk_commit_group();
    bulk_wait_read();
  }
}
}  // namespace bwd

// ====================================================================================
// dK / dV
// ====================================================================================
// ACC: accumulate mode (ffa_bwd_dkdv_acc), a separate instantiation so the plain kernel
// keeps its register allocation.
template <int D, bool CAUSAL, bool ACC>
__global__ void __launch_bounds__(bwd::NTHREADS, 1)
    ffa_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                        const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                        const __grid_constant__ CUtensorMap tm_dk, const __grid_constant__ CUtensorMap tm_dv,
                        const float* __restrict__ LSE, const float* __restrict__ DELTA,
                        float* __restrict__ DK_ACC, float* __restrict__ DV_ACC, int S, int BH, int group,
                        long long stride_bh, long long stride_s, float scale_log2, float scale) {
  using L = bwd::DkdvLayout<D>;
  constexpr int SLABS = D / 64;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = smem_raw;
  if (smem_u32(smem) & 1023u) {  // the layout has no room to realign: report and leave
    if (threadIdx.x == 0) atomicCAS(&g_status[0], 0u, static_cast<unsigned int>(kErrBwdAlign));
    return;
  }
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::BAR_OFF;
  constexpr int QS = L::Q_STAGES, DS = L::DO_STAGES;
  const uint32_t kv_full = bar0;
  auto q_full = [&](int s) { return bar0 + 8 * (1 + s); };
  auto q_empty = [&](int s) { return bar0 + 8 * (1 + QS + s); };
  auto do_full = [&](int s) { return bar0 + 8 * (1 + 2 * QS + s); };
  auto do_empty = [&](int s) { return bar0 + 8 * (1 + 2 * QS + DS + s); };
  const uint32_t s_full = bar0 + 8 * (1 + 2 * QS + 2 * DS);
  const uint32_t dp_full = s_full + 8;
  const uint32_t p_ready = s_full + 16;
  const uint32_t ds_ready = s_full + 24;
  const uint32_t final_bar = s_full + 32;
  const uint32_t drain_bar = s_full + 40;
  const uint32_t s_free = s_full + 48;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);
  auto q_addr = [&](int i) { return sbase + L::Q_OFF + (i % QS) * L::TILE; };
  auto do_addr = [&](int i) { return sbase + L::DO_OFF + (i % DS) * L::DO_STAGE_BYTES; };
  auto lse_smem = [&](int i) {
    return reinterpret_cast<float*>(smem + L::DO_OFF + (i % DS) * L::DO_STAGE_BYTES + L::TILE);
  };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // causal: low key blocks carry the most work and run first
  const CtaWork work = cta_work((S + bwd::LANES - 1) / bwd::LANES, BH, group);
  const int kblk = work.rank;
  const int bh = work.bh;
  const int n0 = kblk * bwd::LANES;
  const int q_begin = CAUSAL ? n0 : 0;  // first query that can see a key of this block
  const int nq = (S > q_begin) ? (S - q_begin + bwd::STEP - 1) / bwd::STEP : 0;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < QS; ++s) {
      mbar_init(q_full(s), 1);
      mbar_init(q_empty(s), 1);
    }
    for (int s = 0; s < DS; ++s) {
      mbar_init(do_full(s), 2);  // TMA expect-tx arrival + lse/delta arrival
      mbar_init(do_empty(s), 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 256);
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

  if (warp >= 8) {
  setmaxnreg_dec<bwd::REGS_CONTROL>();
  if (warp == bwd::PRODUCER_WARP) {
    // ---------------------------------------------------------------- producer: K, V, Q ring
    if (lane == 0) {
      const uint64_t keep = policy_evict_last();
      mbar_arrive_expect_tx(kv_full, 2 * L::TILE);
      for (int sl = 0; sl < SLABS; ++sl) {
        tma_load_3d(sbase + L::K_OFF + sl * 16384, &tm_k, kv_full, sl * 64, n0, bh, keep);
        tma_load_3d(sbase + L::V_OFF + sl * 16384, &tm_v, kv_full, sl * 64, n0, bh, keep);
      }
      int issued = 0;
      for (int it = 0; it < nq; ++it) {
        const int s = it % QS;
        if (!mbar_wait(q_empty(s), ((it / QS) & 1) ^ 1, abort_flag, kErrBwdProducer)) break;
        mbar_arrive_expect_tx(q_full(s), L::TILE);
        for (int sl = 0; sl < SLABS; ++sl)
          tma_load_3d(q_addr(it) + sl * 16384, &tm_q, q_full(s), sl * 64, q_begin + it * bwd::STEP, bh, keep);
        ++issued;
      }
      if (*abort_flag) {
        mbar_wait_drain(kv_full, 0);
        for (int it = max(0, issued - QS); it < issued; ++it) mbar_wait_drain(q_full(it % QS), (it / QS) & 1);
      }
    }
  } else if (warp == bwd::DO_PRODUCER_WARP) {
    // ---------------------------------------------------------------- producer: dO ring + lse/delta
    const uint64_t keep = policy_evict_last();
    int issued = 0;
    for (int it = 0; it < nq; ++it) {
      const int s = it % DS;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(do_empty(s), ((it / DS) & 1) ^ 1, abort_flag, kErrBwdProducer);
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      const int q0 = q_begin + it * bwd::STEP;
      if (lane == 0) {
        mbar_arrive_expect_tx(do_full(s), L::TILE);
        for (int sl = 0; sl < SLABS; ++sl)
          tma_load_3d(do_addr(it) + sl * 16384, &tm_do, do_full(s), sl * 64, q0, bh, keep);
      }
      float* lse_s = lse_smem(it);
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
      if (lane == 0) mbar_arrive(do_full(s));
      ++issued;
    }
    if (lane == 0 && *abort_flag)
      for (int it = max(0, issued - DS); it < issued; ++it) mbar_wait_drain(do_full(it % DS), (it / DS) & 1);
  } else if (warp == bwd::MMA_WARP) {
    // ---------------------------------------------------------------- MMA issuer
    // The whole warp runs the issue loop and one elected lane issues each group of MMAs
    // and its commits (see the dQ issuer below).
    {
      constexpr uint32_t IDESC_SD = idesc_bf16(128, bwd::STEP, false, false);  // [128 keys x 128 queries]
      constexpr uint32_t IDESC_G = idesc_bf16(128, D, false, true);            // [128 keys x D]
      // Descriptors are built once per tile; a K-step only adds a constant.
      const uint64_t kdesc = kmajor_desc(sbase + L::K_OFF, 128, 0), vdesc = kmajor_desc(sbase + L::V_OFF, 128, 0);
      auto issue_s = [&](int i) -> bool {  // S^T = K Q_i^T
        if (!mbar_wait(q_full(i % QS), (i / QS) & 1, abort_flag, kErrBwdMma)) return false;
        tc_fence_after();
        const uint64_t qd = kmajor_desc(q_addr(i), 128, 0);
        if (elect_one()) {
          mma_ss(tmem, kdesc, qd, IDESC_SD, 0u);
#pragma unroll
          for (int ks = 1; ks < D / 16; ++ks)
            mma_ss_acc(tmem, kdesc + kmajor_step(128, ks), qd + kmajor_step(128, ks), IDESC_SD);
          mma_commit(s_full);
        }
        __syncwarp();
        return true;
      };
      auto issue_dp = [&](int i) -> bool {  // dP^T = V dO_i^T
        if (!mbar_wait(do_full(i % DS), (i / DS) & 1, abort_flag, kErrBwdMma)) return false;
        tc_fence_after();
        const uint64_t dd = kmajor_desc(do_addr(i), 128, 0);
        if (elect_one()) {
          mma_ss(tmem + 128, vdesc, dd, IDESC_SD, 0u);
#pragma unroll
          for (int ks = 1; ks < D / 16; ++ks)
            mma_ss_acc(tmem + 128, vdesc + kmajor_step(128, ks), dd + kmajor_step(128, ks), IDESC_SD);
          mma_commit(dp_full);
        }
        __syncwarp();
        return true;
      };
      auto issue_dv = [&](int i) -> bool {  // dV += P^T dO_i
        if (!mbar_wait(p_ready, i & 1, abort_flag, kErrBwdMma)) return false;
        tc_fence_after();
        const uint64_t dd = mnmajor_desc(do_addr(i), 128, 0);
        if (elect_one()) {
          mma_ts(tmem + 256, tmem + 128, dd, IDESC_G, i > 0 ? 1u : 0u);
#pragma unroll
          for (int ks = 1; ks < bwd::STEP / 16; ++ks)
            mma_ts_acc(tmem + 256, bwd::packed_kstep_col(tmem + 128, ks), dd + mnmajor_step(ks), IDESC_G);
        }
        __syncwarp();
        return true;
      };
      auto issue_dk = [&](int i) -> bool {  // dK += dS^T Q_i
        if (!mbar_wait(ds_ready, i & 1, abort_flag, kErrBwdMma)) return false;
        tc_fence_after();
        const uint64_t qd = mnmajor_desc(q_addr(i), 128, 0);
        if (elect_one()) {
          mma_ts(tmem + 384, tmem + 128 + 32, qd, IDESC_G, i > 0 ? 1u : 0u);
#pragma unroll
          for (int ks = 1; ks < bwd::STEP / 16; ++ks)
            mma_ts_acc(tmem + 384, bwd::packed_kstep_col(tmem + 128 + 32, ks), qd + mnmajor_step(ks), IDESC_G);
          mma_commit(q_empty(i % QS));
          mma_commit(do_empty(i % DS));
        }
        __syncwarp();
        return true;
      };
      bool ok = mbar_wait(kv_full, 0, abort_flag, kErrBwdMma);
      if (ok && nq > 0) {
        ok = issue_s(0);
        if (ok) ok = issue_dp(0);
      }
      // S(i+1) as soon as the warpgroups have copied S(i) into registers, then dV(i),
      // dK(i) and dP(i+1): P(i) and dS(i) live in the dP columns, so the next step's
      // scores are computed during this step's whole softmax.
      for (int i = 0; i < nq && ok; ++i) {
        FFA_BWD_TRACE(0, i);
        if (i + 1 < nq) {
          if (!(ok = mbar_wait(s_free, i & 1, abort_flag, kErrBwdMma))) break;
          tc_fence_after();
          if (!(ok = issue_s(i + 1))) break;
        }
        FFA_BWD_TRACE(1, i);
        if (!(ok = issue_dv(i))) break;
        FFA_BWD_TRACE(2, i);
        if (!(ok = issue_dk(i))) break;
        FFA_BWD_TRACE(3, i);
        if (i + 1 < nq && !(ok = issue_dp(i + 1))) break;
        FFA_BWD_TRACE(4, i);
      }
      // commits track the MMAs of the thread that issues them: the same elected lane
      if (elect_one()) {
        if (ok) mma_commit(final_bar);
        mma_commit(drain_bar);
      }
      __syncwarp();
      mbar_wait_drain(drain_bar, 0);
    }
    __syncwarp();
  }
  } else {
    setmaxnreg_inc<bwd::REGS_COMPUTE>();
    // ---------------------------------------------------------------- compute
    const int g = warp >> 2;                  // warpgroup: query columns [64g, 64g+64) of a step
    const int row = (warp & 3) * 32 + lane;   // key row within the block
    const int kg = n0 + row;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + lane_off + 64 * g;
    const uint32_t t_dp = tmem + lane_off + 128 + 64 * g;
    bool ok = true;
    for (int i = 0; i < nq; ++i) {
      const int qc = q_begin + i * bwd::STEP + 64 * g;  // first query of this thread's columns
      // lse / delta of this step (written next to dO_i by the dO producer)
      if (!(ok = mbar_wait(do_full(i % DS), (i / DS) & 1, abort_flag, kErrBwdCompute))) break;
      const float* lse_s = lse_smem(i) + 64 * g;
      const float* dl_s = lse_s + bwd::STEP;
      float p[64];
      if (!(ok = mbar_wait(s_full, i & 1, abort_flag, kErrBwdCompute))) break;
      if (threadIdx.x == 0) FFA_BWD_TRACE(8, i);
      tc_fence_after();
      bwd::tmem_ld64(t_s, p);
      tc_fence_before();
      mbar_arrive(s_free);  // S may now be overwritten by S(i+1)
      if (threadIdx.x == 0) FFA_BWD_TRACE(12, i);
      uint32_t pk[32];
      {
        const bool need_mask = CAUSAL && (qc < kg);  // some query of these columns precedes the key
#pragma unroll
        for (int e = 0; e < 64; e += 4) {
          const float4 l4 = *reinterpret_cast<const float4*>(lse_s + e);
          const float2 c2 = make_float2(scale_log2, scale_log2);
          const float2 xa = fma2(make_float2(p[e], p[e + 1]), c2, make_float2(-l4.x, -l4.y));
          const float2 xb = fma2(make_float2(p[e + 2], p[e + 3]), c2, make_float2(-l4.z, -l4.w));
          if (bwd::emu_group<D, true>(e >> 2)) {  // this group of 4 on the FMA pipe
            const float2 ea = exp2_fma2(xa), eb = exp2_fma2(xb);
            p[e + 0] = ea.x;
            p[e + 1] = ea.y;
            p[e + 2] = eb.x;
            p[e + 3] = eb.y;
          } else {
            p[e + 0] = fast_exp2(xa.x);
            p[e + 1] = fast_exp2(xa.y);
            p[e + 2] = fast_exp2(xb.x);
            p[e + 3] = fast_exp2(xb.y);
          }
          if (need_mask) {
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (qc + e + u < kg) p[e + u] = 0.f;
          }
          pk[e / 2] = pack_bf16x2(p[e], p[e + 1]);
          pk[e / 2 + 1] = pack_bf16x2(p[e + 2], p[e + 3]);
        }
      }
      if (threadIdx.x == 0) FFA_BWD_TRACE(14, i);
      if (!(ok = mbar_wait(dp_full, i & 1, abort_flag, kErrBwdCompute))) break;
      if (threadIdx.x == 0) FFA_BWD_TRACE(10, i);
      tc_fence_after();
      // dP(i) comes into registers half by half; its columns then take P(i) (first half)
      // and dS(i) (second half), so at most P, packed P and 32 dP values are live at once
      uint32_t dlo[32], dhi[32];
      tmem_ld32(t_dp, dlo);
      tmem_ld_wait();
      tmem_st32(t_dp, pk);
      tmem_ld32(t_dp + 32, dhi);
      tmem_ld_wait();
      tmem_st_wait();
      if (threadIdx.x == 0) FFA_BWD_TRACE(13, i);
      tc_fence_before();
      if (threadIdx.x == 0) FFA_BWD_TRACE(9, i);
      mbar_arrive(p_ready);
      {
        uint32_t dk[32];
#pragma unroll
        for (int e = 0; e < 64; e += 4) {
          const float4 d4 = *reinterpret_cast<const float4*>(dl_s + e);
          const uint32_t* src = (e < 32) ? dlo : dhi;
          const int b = e & 31;
          const float2 da = mul2(make_float2(p[e], p[e + 1]),
                                 sub2(make_float2(__uint_as_float(src[b]), __uint_as_float(src[b + 1])),
                                      make_float2(d4.x, d4.y)));
          const float2 db = mul2(make_float2(p[e + 2], p[e + 3]),
                                 sub2(make_float2(__uint_as_float(src[b + 2]), __uint_as_float(src[b + 3])),
                                      make_float2(d4.z, d4.w)));
          dk[e / 2] = pack_bf16x2(da.x, da.y);
          dk[e / 2 + 1] = pack_bf16x2(db.x, db.y);
        }
        tmem_st32(t_dp + 32, dk);
        tmem_st_wait();
      }
      tc_fence_before();
      if (threadIdx.x == 0) FFA_BWD_TRACE(11, i);
      mbar_arrive(ds_ready);
    }
    const bool staged = ok && nq > 0 && mbar_wait(final_bar, 0, abort_flag, kErrBwdCompute);
    constexpr bool acc_mode = ACC;
    if (staged) {
      tc_fence_after();
      if constexpr (acc_mode) {
        // fp32 accumulate: this CTA is the only writer of its key rows in this launch
        const long long off = (static_cast<long long>(bh) * S + kg) * D;
        bwd::add_acc_half<D>(tmem + lane_off + 256, g, DV_ACC + off, kg < S, 1.f);
        bwd::add_acc_half<D>(tmem + lane_off + 384, g, DK_ACC + off, kg < S, scale);
      } else {
        // every MMA has finished: the Q ring is free and holds the staged dV, dK tiles
        bwd::stage_acc_half<D>(tmem + lane_off + 256, g, sbase + L::Q_OFF, row, 1.f);
        bwd::stage_acc_half<D>(tmem + lane_off + 384, g, sbase + L::Q_OFF + L::TILE, row, scale);
      }
    }
    const CUtensorMap* const maps[2] = {&tm_dv, &tm_dk};
    bwd::store_staged<D, 2>(staged && !acc_mode, maps, sbase + L::Q_OFF, n0, bh);
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
// TMEM (512 columns): S [0,128), dP [128,256), dQ [256,256+D), then Q and dO of the
// block as packed bf16 (D/2 columns each): they are the A operands of S = Q K^T and
// dP = dO V^T, so shared memory holds only the streamed K and V rings (4 + 3 slots).
template <int D>
struct DqTmem {
  static constexpr uint32_t S = 0, DP = 128, DQ = 256, Q = 256 + D, DO = 256 + D + D / 2;
};

// Copy this thread's row of a [S, D] bf16 slice (row stride `stride_s` elements) into
// D/2 packed TMEM columns starting at `taddr` (this warp's lanes); rows past the end
// are zero.  Every lane of the warp calls it (tcgen05.st is warp-wide).
template <int D>
__device__ __forceinline__ void load_row_to_tmem(const __nv_bfloat16* __restrict__ src, bool valid, uint32_t taddr) {
#pragma unroll
  for (int c = 0; c < D / 64; ++c) {
    uint32_t w[32];
    const uint4* s4 = reinterpret_cast<const uint4*>(src + 64 * c);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint4 x = valid ? __ldg(s4 + e) : make_uint4(0u, 0u, 0u, 0u);
      w[4 * e + 0] = x.x;
      w[4 * e + 1] = x.y;
      w[4 * e + 2] = x.z;
      w[4 * e + 3] = x.w;
    }
    tmem_st32(taddr + 32 * c, w);
  }
}

// ACC: accumulate mode (ffa_bwd_dq_acc).
template <int D, bool CAUSAL, bool ACC>
__global__ void __launch_bounds__(bwd::NTHREADS, 1)
    ffa_bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                      const __grid_constant__ CUtensorMap tm_dq, const __nv_bfloat16* __restrict__ Qp,
                      const __nv_bfloat16* __restrict__ DOp, const float* __restrict__ LSE,
                      const float* __restrict__ DELTA, float* __restrict__ DQ_ACC, int S, int BH, int group,
                      long long stride_bh, long long stride_s, float scale_log2, float scale) {
  using L = bwd::DqLayout<D>;
  using T = DqTmem<D>;
  constexpr int SLABS = D / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::BAR_OFF;
  constexpr int KS = L::K_STAGES, VS = L::V_STAGES;
  const uint32_t qd_ready = bar0;
  auto k_full = [&](int s) { return bar0 + 8 * (1 + s); };
  auto k_empty = [&](int s) { return bar0 + 8 * (1 + KS + s); };
  auto v_full = [&](int s) { return bar0 + 8 * (1 + 2 * KS + s); };
  auto v_empty = [&](int s) { return bar0 + 8 * (1 + 2 * KS + VS + s); };
  const uint32_t s_full = bar0 + 8 * (1 + 2 * KS + 2 * VS);
  const uint32_t s_free = s_full + 8;
  const uint32_t dp_full = s_full + 16;
  const uint32_t ds_ready = s_full + 24;
  const uint32_t final_bar = s_full + 32;
  const uint32_t drain_bar = s_full + 40;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nblk = (S + bwd::LANES - 1) / bwd::LANES;
  const CtaWork work = cta_work(nblk, BH, group);
  const int qblk = CAUSAL ? (nblk - 1 - work.rank) : work.rank;
  const int bh = work.bh;
  const int m0 = qblk * bwd::LANES;
  const int nk_all = (S + bwd::STEP - 1) / bwd::STEP;
  const int nk = CAUSAL ? min(nk_all, m0 / bwd::STEP + 1) : nk_all;

  if (threadIdx.x == 0) {
    mbar_init(qd_ready, 256);
    for (int s = 0; s < KS; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 256);
    mbar_init(dp_full, 1);
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
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 8) {
  setmaxnreg_dec<bwd::REGS_CONTROL>();
  if (warp == bwd::PRODUCER_WARP) {
    // ---------------------------------------------------------------- producer: K, V rings
    if (lane == 0) {
      const uint64_t keep = policy_evict_last();
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
        for (int it = max(0, k_issued - KS); it < k_issued; ++it) mbar_wait_drain(k_full(it % KS), (it / KS) & 1);
        for (int it = max(0, v_issued - VS); it < v_issued; ++it) mbar_wait_drain(v_full(it % VS), (it / VS) & 1);
      }
    }
  } else if (warp == bwd::MMA_WARP) {
    // ---------------------------------------------------------------- MMA issuer
    // The whole warp runs the issue loop (its waits, descriptors and loop state are then
    // warp-uniform) and one elected lane issues each group of MMAs and its commits.
    {
      constexpr uint32_t IDESC_SD = idesc_bf16(128, bwd::STEP, false, false);  // [128 queries x 128 keys]
      constexpr uint32_t IDESC_G = idesc_bf16(128, D, false, true);            // [128 queries x D]
      auto k_addr = [&](int j) { return sbase + L::K_OFF + (j % KS) * L::TILE; };
      auto v_addr = [&](int j) { return sbase + L::V_OFF + (j % VS) * L::TILE; };
      auto issue_s = [&](int j) -> bool {  // S_j = Q K_j^T  (Q from TMEM)
        if (!mbar_wait(k_full(j % KS), (j / KS) & 1, abort_flag, kErrDqMma)) return false;
        tc_fence_after();
        const uint64_t kd = kmajor_desc(k_addr(j), 128, 0);
        if (elect_one()) {
          mma_ts(tmem + T::S, tmem + T::Q, kd, IDESC_SD, 0u);
#pragma unroll
          for (int ks = 1; ks < D / 16; ++ks)
            mma_ts_acc(tmem + T::S, tmem + T::Q + 8 * ks, kd + kmajor_step(128, ks), IDESC_SD);
          mma_commit(s_full);
        }
        __syncwarp();
        return true;
      };
      auto issue_dp = [&](int j) -> bool {  // dP_j = dO V_j^T  (dO from TMEM)
        if (!mbar_wait(v_full(j % VS), (j / VS) & 1, abort_flag, kErrDqMma)) return false;
        tc_fence_after();
        const uint64_t vd = kmajor_desc(v_addr(j), 128, 0);
        if (elect_one()) {
          mma_ts(tmem + T::DP, tmem + T::DO, vd, IDESC_SD, 0u);
#pragma unroll
          for (int ks = 1; ks < D / 16; ++ks)
            mma_ts_acc(tmem + T::DP, tmem + T::DO + 8 * ks, vd + kmajor_step(128, ks), IDESC_SD);
          mma_commit(dp_full);
          mma_commit(v_empty(j % VS));
        }
        __syncwarp();
        return true;
      };
      auto issue_g = [&](int j) -> bool {  // dQ += dS_j K_j  (dS_j packed in the dP columns)
        if (!mbar_wait(ds_ready, j & 1, abort_flag, kErrDqMma)) return false;
        tc_fence_after();
        const uint64_t kd = mnmajor_desc(k_addr(j), 128, 0);
        if (elect_one()) {
          mma_ts(tmem + T::DQ, tmem + T::DP, kd, IDESC_G, j > 0 ? 1u : 0u);
#pragma unroll
          for (int ks = 1; ks < bwd::STEP / 16; ++ks)
            mma_ts_acc(tmem + T::DQ, bwd::packed_kstep_col(tmem + T::DP, ks), kd + mnmajor_step(ks), IDESC_G);
          mma_commit(k_empty(j % KS));
        }
        __syncwarp();
        return true;
      };
      // Q and dO reach tensor memory through the compute warps
      bool ok = mbar_wait(qd_ready, 0, abort_flag, kErrDqMma);
      tc_fence_after();
      if (ok && nk > 0) {
        ok = issue_s(0);
        if (ok) ok = issue_dp(0);
      }
      // Per step: S(j+1) once the warpgroups hold S(j) in registers; dQ(j) once dS(j) is
      // in the dP columns; then dP(j+1) over them (in order after dQ(j) has read dS(j)).
      // The warpgroups exponentiate step j+1 while dQ(j) and dP(j+1) run, so the chain
      // dQ(j) -> dP(j+1) -> dS(j+1) -> dQ(j+1) is shorter than a step's three MMAs.
      for (int j = 0; j < nk && ok; ++j) {
        if (j + 1 < nk) {
          if (!(ok = mbar_wait(s_free, j & 1, abort_flag, kErrDqMma))) break;
          tc_fence_after();
          if (!(ok = issue_s(j + 1))) break;
        }
        if (!(ok = issue_g(j))) break;
        if (j + 1 < nk && !(ok = issue_dp(j + 1))) break;
      }
      // commits track the MMAs of the thread that issues them: the same elected lane
      if (elect_one()) {
        if (ok) mma_commit(final_bar);
        mma_commit(drain_bar);
      }
      __syncwarp();
      mbar_wait_drain(drain_bar, 0);
    }
    __syncwarp();
  }
  } else {
    setmaxnreg_inc<bwd::REGS_COMPUTE>();
    // ---------------------------------------------------------------- compute
    const int g = warp >> 2;
    const int row = (warp & 3) * 32 + lane;  // query row within the block
    const int qg = m0 + row;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const long long ridx = static_cast<long long>(bh) * S + qg;
    {
      // warpgroup 0 puts the block's Q rows into tensor memory, warpgroup 1 its dO rows
      const __nv_bfloat16* src = (g ? DOp : Qp) + static_cast<long long>(bh) * stride_bh +
                                 static_cast<long long>(qg < S ? qg : 0) * stride_s;
      load_row_to_tmem<D>(src, qg < S, tmem + lane_off + (g ? T::DO : T::Q));
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(qd_ready);
    }
    const float lse = (qg < S) ? LSE[ridx] : INFINITY;
    const float dl = (qg < S) ? DELTA[ridx] : 0.f;
    const int lim = CAUSAL ? min(S - 1, qg) : S - 1;  // last visible key
    const uint32_t t_s = tmem + lane_off + T::S + 64 * g;
    const uint32_t t_dp = tmem + lane_off + T::DP + 64 * g;
    bool ok = true;
    for (int j = 0; j < nk; ++j) {
      if (!(ok = mbar_wait(s_full, j & 1, abort_flag, kErrDqCompute))) break;
      tc_fence_after();
      float p[64];
      bwd::tmem_ld64(t_s, p);
      tc_fence_before();
      mbar_arrive(s_free);  // S may now be overwritten by S(j+1)
      const int kc = j * bwd::STEP + 64 * g;  // first key of this thread's columns
      const bool need_mask = (kc + 64 > S) || (CAUSAL && kc + 63 > qg);
      const float2 c2 = make_float2(scale_log2, scale_log2), l2 = make_float2(-lse, -lse);
#pragma unroll
      for (int e = 0; e < 64; e += 2) {
        const float2 x = fma2(make_float2(p[e], p[e + 1]), c2, l2);
        float p0, p1;
        if (bwd::emu_group<D, false>(e >> 2)) {  // this pair on the FMA pipe
          const float2 ex = exp2_fma2(x);
          p0 = ex.x;
          p1 = ex.y;
        } else {
          p0 = fast_exp2(x.x);
          p1 = fast_exp2(x.y);
        }
        if (need_mask) {
          if (kc + e > lim) p0 = 0.f;
          if (kc + e + 1 > lim) p1 = 0.f;
        }
        p[e] = p0;
        p[e + 1] = p1;
      }
      if (!(ok = mbar_wait(dp_full, j & 1, abort_flag, kErrDqCompute))) break;
      tc_fence_after();
      uint32_t dlo[32], dhi[32];
      tmem_ld32(t_dp, dlo);
      tmem_ld32(t_dp + 32, dhi);
      tmem_ld_wait();
      uint32_t dsp[32];
      const float2 d2 = make_float2(dl, dl);
#pragma unroll
      for (int e = 0; e < 64; e += 2) {
        const uint32_t* src = (e < 32) ? dlo : dhi;
        const int b = e & 31;
        const float2 ds = mul2(make_float2(p[e], p[e + 1]),
                               sub2(make_float2(__uint_as_float(src[b]), __uint_as_float(src[b + 1])), d2));
        dsp[e >> 1] = pack_bf16x2(ds.x, ds.y);
      }
      // dS(j) over the first half of this warpgroup's dP columns: the A operand of dQ(j)
      tmem_st32(t_dp, dsp);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(ds_ready);
    }
    const bool staged = ok && nk > 0 && mbar_wait(final_bar, 0, abort_flag, kErrDqCompute);
    constexpr bool acc_mode = ACC;
    if (staged) {
      tc_fence_after();
      if constexpr (acc_mode)  // fp32 accumulate: this CTA is the only writer of its query rows
        bwd::add_acc_half<D>(tmem + lane_off + T::DQ, g, DQ_ACC + ridx * D, qg < S, scale);
      else  // every MMA has finished: the K ring is free and holds the staged dQ tile
        bwd::stage_acc_half<D>(tmem + lane_off + T::DQ, g, sbase + L::K_OFF, row, scale);
    }
    const CUtensorMap* const maps[1] = {&tm_dq};
    bwd::store_staged<D, 1>(staged && !acc_mode, maps, sbase + L::K_OFF, m0, bh);
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
template <int D, bool CAUSAL, bool ACC>
static int launch_dkdv_t(const BwdArgs& a, cudaStream_t stream) {
  using LK = bwd::DkdvLayout<D>;
  CUtensorMap tk, tv, tq, tdo;
  int rc;
  if ((rc = make_tile_map(&tk, a.k, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  if ((rc = make_tile_map(&tv, a.v, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  if ((rc = make_tile_map(&tq, a.q, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  if ((rc = make_tile_map(&tdo, a.dout, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  CUtensorMap tdk, tdv;
  // accumulate mode stores nothing through these maps: any valid tensor serves as their base
  if ((rc = make_tile_map(&tdk, a.dk_acc ? a.k : a.dk, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  if ((rc = make_tile_map(&tdv, a.dv_acc ? a.v : a.dv, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  auto kern = ffa_bwd_dkdv_kernel<D, CAUSAL, ACC>;
  static unsigned long long configured = 0;
  if ((rc = set_smem_once(reinterpret_cast<const void*>(kern), LK::SMEM_BYTES, &configured))) return rc;
  if ((rc = check_launch_regs(reinterpret_cast<const void*>(kern), bwd::LAUNCH_REGS_NEEDED))) return rc;
  const dim3 grid(static_cast<unsigned>((a.S + bwd::LANES - 1) / bwd::LANES) * static_cast<unsigned>(a.BH));
  kern<<<grid, bwd::NTHREADS, LK::SMEM_BYTES, stream>>>(tk, tv, tq, tdo, tdk, tdv, a.lse, a.delta, a.dk_acc,
                                                        a.dv_acc, a.S, a.BH,
                                                        work_group(a.BH, a.S, D, CAUSAL), a.stride_bh,
                                                        a.stride_s, static_cast<float>(a.scale * kLog2e),
                                                        static_cast<float>(a.scale));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FFA_ERR_LAUNCH, cudaGetErrorString(e));
  return FFA_OK;
}

template <int D, bool CAUSAL, bool ACC>
static int launch_dq_t(const BwdArgs& a, cudaStream_t stream) {
  using LQ = bwd::DqLayout<D>;
  CUtensorMap tk, tv, tdq;
  int rc;
  if ((rc = make_tile_map(&tk, a.k, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  if ((rc = make_tile_map(&tv, a.v, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  // accumulate mode stores nothing through this map: q serves as its base
  if ((rc = make_tile_map(&tdq, a.dq_acc ? a.q : a.dq, a.BH, a.S, D, a.stride_bh, a.stride_s, 128))) return rc;
  auto kern = ffa_bwd_dq_kernel<D, CAUSAL, ACC>;
  static unsigned long long configured = 0;
  if ((rc = set_smem_once(reinterpret_cast<const void*>(kern), LQ::SMEM_BYTES, &configured))) return rc;
  if ((rc = check_launch_regs(reinterpret_cast<const void*>(kern), bwd::LAUNCH_REGS_NEEDED))) return rc;
  const dim3 grid(static_cast<unsigned>((a.S + bwd::LANES - 1) / bwd::LANES) * static_cast<unsigned>(a.BH));
  kern<<<grid, bwd::NTHREADS, LQ::SMEM_BYTES, stream>>>(
      tk, tv, tdq, static_cast<const __nv_bfloat16*>(a.q), static_cast<const __nv_bfloat16*>(a.dout), a.lse, a.delta,
      a.dq_acc, a.S, a.BH, work_group(a.BH, a.S, D, CAUSAL), a.stride_bh, a.stride_s,
      static_cast<float>(a.scale * kLog2e), static_cast<float>(a.scale));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FFA_ERR_LAUNCH, cudaGetErrorString(e));
  return FFA_OK;
}

template <int D, bool CAUSAL>
static int launch_dkdv_a(const BwdArgs& a, cudaStream_t stream) {
  return a.dk_acc ? launch_dkdv_t<D, CAUSAL, true>(a, stream) : launch_dkdv_t<D, CAUSAL, false>(a, stream);
}

template <int D, bool CAUSAL>
static int launch_dq_a(const BwdArgs& a, cudaStream_t stream) {
  return a.dq_acc ? launch_dq_t<D, CAUSAL, true>(a, stream) : launch_dq_t<D, CAUSAL, false>(a, stream);
}

int launch_dkdv(const BwdArgs& a, cudaStream_t stream) {
  if (a.D == 128) return a.causal ? launch_dkdv_a<128, true>(a, stream) : launch_dkdv_a<128, false>(a, stream);
  if (a.D == 64) return a.causal ? launch_dkdv_a<64, true>(a, stream) : launch_dkdv_a<64, false>(a, stream);
  return set_error(FFA_ERR_UNSUPPORTED, "kernel head_dim must be 64 or 128");
}

int launch_dq(const BwdArgs& a, cudaStream_t stream) {
  if (a.D == 128) return a.causal ? launch_dq_a<128, true>(a, stream) : launch_dq_a<128, false>(a, stream);
  if (a.D == 64) return a.causal ? launch_dq_a<64, true>(a, stream) : launch_dq_a<64, false>(a, stream);
  return set_error(FFA_ERR_UNSUPPORTED, "kernel head_dim must be 64 or 128");
}

// A second stream on which dQ runs beside dK/dV: the two kernels are independent once
// delta exists, and CTAs of one fill the SMs the other leaves idle at its tail.  Fork and
// join are event waits, so the pair also records correctly into a CUDA graph captured on
// the caller's stream.
//
// Each (device, caller stream) pair gets its own side stream and events, created on its
// first backward and kept until exit.  A capture on one caller stream pulls that caller's
// side stream into the capture until the capture ends; keeping side streams apart per
// caller stream means a plain backward issued meanwhile on another stream (another thread)
// never lands in that graph.  Past kMaxSideStreams pairs, dQ runs on the caller's stream
// after dK/dV instead (same results, no overlap).  The caller holds bwd_fork_mutex().
static std::mutex& bwd_fork_mutex() {
  static std::mutex mu;
  return mu;
}

struct SideStream {
  int dev;
  cudaStream_t caller;
  cudaStream_t s;
  cudaEvent_t f, j;
};
constexpr int kMaxSideStreams = 256;

// Side stream and events of (current device, caller); *out = nullptr when the table is
// full.  Returns FFA_OK or an error when creating them failed.
static int side_stream(cudaStream_t caller, SideStream** out) {
  static SideStream table[kMaxSideStreams];
  static int used = 0;
  *out = nullptr;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_error(FFA_ERR_LAUNCH, "cudaGetDevice failed");
  for (int i = 0; i < used; ++i)
    if (table[i].dev == dev && table[i].caller == caller) {
      *out = &table[i];
      return FFA_OK;
    }
  if (used == kMaxSideStreams) return FFA_OK;
  SideStream& sd = table[used];
  sd.dev = dev;
  sd.caller = caller;
  if (cudaStreamCreateWithFlags(&sd.s, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&sd.f, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&sd.j, cudaEventDisableTiming) != cudaSuccess)
    return set_error(FFA_ERR_LAUNCH, "could not create the backward's side stream");
  ++used;
  *out = &sd;
  return FFA_OK;
}

int launch_bwd(const BwdArgs& a, cudaStream_t stream) {
  int rc;
  if ((rc = launch_preprocess(a.o, a.dout, a.delta, a.BH, a.S, a.D, a.stride_bh, a.stride_s, stream))) return rc;
  // record / wait / launch as one unit: another thread's backward on the same caller
  // stream must not re-record the shared events in between
  std::lock_guard<std::mutex> lock(bwd_fork_mutex());
  SideStream* sd = nullptr;
  if ((rc = side_stream(stream, &sd))) return rc;
  if (sd == nullptr) {  // side-stream table full: serial on the caller's stream
    if ((rc = launch_dkdv(a, stream))) return rc;
    return launch_dq(a, stream);
  }
  if (cudaEventRecord(sd->f, stream) != cudaSuccess || cudaStreamWaitEvent(sd->s, sd->f, 0) != cudaSuccess)
    return set_error(FFA_ERR_LAUNCH, "backward fork failed");
  if ((rc = launch_dq(a, sd->s))) return rc;
  if ((rc = launch_dkdv(a, stream))) return rc;
  if (cudaEventRecord(sd->j, sd->s) != cudaSuccess || cudaStreamWaitEvent(stream, sd->j, 0) != cudaSuccess)
    return set_error(FFA_ERR_LAUNCH, "backward join failed");
  return FFA_OK;
}

}  // namespace ffa
