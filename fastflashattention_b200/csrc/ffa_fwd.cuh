// ffa_fwd.cuh — exact bf16 attention forward for sm_100a.
//
// Computes, per (batch*head) slice and per query row i,
//   O_i   = sum_j softmax_j( scale * q_i . k_j  [j <= i if causal] ) v_j
//   LSE_i = m_i + log2(l_i)          (base-2 log-sum-exp of scale*log2(e)*q.k)
// which is the contract of the reference forward `_fastflash_fwd`
// (fastflash_attention/_kernel.py:194-279): exp2 with scale*log2(e) folded into the
// scores, fp32 online softmax, P rounded to bf16 before the P.V product (:245), the
// fully-masked-row guards (:260, :269, :276) and the base-2 LSE (:274-279).
//
// B200 design (one CTA = 256 query rows = two 128-row tiles, one CTA per SM):
//   warps 0-3   softmax warpgroup for tile 0 (thread t owns row t: TMEM lane t)
//   warps 4-7   softmax warpgroup for tile 1
//   warp  8     TMA producer: Q0/Q1 once, then K_j, V_j through a 3-slot smem ring
//   warp  9     MMA issuer (the whole warp runs the loop, an elected lane issues):
//               S_i = Q_i K_j^T  and  O_i += P_i V_j
//   warps 10-11 idle (complete the third warpgroup, which hands its registers to the
//               softmax warpgroups with setmaxnreg: 208 vs 88 registers per thread)
// TMEM (512 columns): S0 [0,128)  S1 [128,256)  O0 [256,384)  O1 [384,512).
// P_i (bf16, two per column) overwrites the first 64 columns of S_i and is the
// A operand of the P.V MMA straight from tensor memory, so P never touches smem.
// While warpgroup 0 exponentiates tile 0, the tensor core works on tile 1 and vice
// versa.  P is handed over in two 64-key halves: the first half's P.V MMAs run while
// the second half is exponentiated (B200, B4 H16 S8192 D128: causal -2 %, non-causal
// -4 %; B8 H16 S4096 D64 -4 %).  The running max is rescaled lazily: O and l are
// rescaled only when a row's max grows by more than 2^8, which keeps every P <= 256
// (exact in fp32 / bf16 range).  CTAs run in longest-job-first order (cta_work).
#pragma once
#include "ffa_common.cuh"


namespace ffa {

namespace fwd {
constexpr int BM = 128;            // rows per Q tile (TMEM lanes)
constexpr int BN = 128;            // keys per K/V tile
constexpr int STAGES = 3;          // K/V smem ring slots
constexpr int NTHREADS = 384;  // 3 warpgroups: softmax tile 0, softmax tile 1, producer + MMA (+2 idle)
constexpr int PRODUCER_WARP = 8;
constexpr int MMA_WARP = 9;
// Register split after launch (384 threads x 168 registers = 64512): the softmax
// warpgroups hold a 128-float score row each and get 208, the producer/MMA warpgroup 88.
constexpr int REGS_SOFTMAX = 208;
constexpr int REGS_CONTROL = 88;
constexpr int LAUNCH_REGS_NEEDED = (2 * 128 * REGS_SOFTMAX + 128 * REGS_CONTROL) / NTHREADS;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units
// Of every 8 column pairs of an unmasked tile, how many are exponentiated on the FMA pipe
// (packed polynomial) instead of MUFU.EX2.  At D=64 the MMAs take half as long, the
// softmax bounds the kernel and 2 of 8 pairs gain 10-13 % (B200, B8 H16 D64).  At D=128,
// 2 of 8 pairs measured 4 % faster than 1 of 8 at B4 H16 causal S=8192 (two interleaved
// A/B rounds), and 3 of 8 about 2 %.  FFA_FWD_EMU_D128 / _D64 override the counts at build
// time (measurement builds).
#ifndef FFA_FWD_EMU_D128
#define FFA_FWD_EMU_D128 2
#endif
#ifndef FFA_FWD_EMU_D64
#define FFA_FWD_EMU_D64 2
#endif
template <int D>
constexpr int emu_pairs() { return D == 64 ? FFA_FWD_EMU_D64 : FFA_FWD_EMU_D128; }
// Whether the two softmax warpgroups take turns on the exponentials.  At D=64 the MMAs
// of a step take half as long, both warpgroups would otherwise exponentiate at the same
// time, and taking turns is 5-6 % faster (B8 H16 S4096 D64); at D=128 it changes
// nothing measurable and stays off.
#ifndef FFA_FWD_SEQ_D128
#define FFA_FWD_SEQ_D128 0
#endif
template <int D>
constexpr bool seq_turns() { return D == 64 || FFA_FWD_SEQ_D128; }

template <int D, bool PERSIST>
struct Layout {
  static constexpr int TILE_BYTES = 128 * D * 2;  // one 128-row bf16 tile
  static constexpr int Q_OFF = 0;                 // Q tiles of a block (two buffers when persistent)
  static constexpr int KV_OFF = (PERSIST ? 4 : 2) * TILE_BYTES;
  static constexpr int BAR_OFF = KV_OFF + STAGES * TILE_BYTES;
  // barriers: q_full[0], kv_full[3], kv_empty[3], s_full[2], p_ready[2], o_final[2], drain,
  // p_half[2], exp_done[2], q_full[1], q_empty[2]
  static constexpr int NBARS = 1 + 2 * STAGES + 2 + 2 + 2 + 1 + 2 + 2 + 3;
  static constexpr int MISC_OFF = BAR_OFF + NBARS * 8;  // tmem base, abort flag
  static constexpr int SMEM_BYTES = MISC_OFF + 16 + 1024;  // + alignment slack
};
}  // namespace fwd

// The softmax hands P over in two halves of 64 keys (barriers p_half, then p_ready), so
// the P.V MMAs of the first half run while the second half is exponentiated.
// SEQ: the two softmax warpgroups take turns on the exponentials (barriers exp_done):
// tile 1 exponentiates step j after tile 0 has, tile 0 step j+1 after tile 1 step j.
// Max of a 128-float row: 16 independent three-input max chains of depth 4, then a
// short tree.  (On B200 the row max takes about 400 cycles either way: the ALU pipe is
// shared with the other tile's exponential loop, not the chain depth, sets its pace.)
__device__ __forceinline__ float row_max128(const float (&s)[fwd::BN]) {
  float a[16];
#pragma unroll
  for (int u = 0; u < 16; ++u) a[u] = fmax3(s[u], s[16 + u], s[32 + u]);
#pragma unroll
  for (int u = 0; u < 16; ++u) a[u] = fmax3(a[u], s[48 + u], s[64 + u]);
#pragma unroll
  for (int u = 0; u < 16; ++u) a[u] = fmax3(a[u], s[80 + u], s[96 + u]);
#pragma unroll
  for (int u = 0; u < 16; ++u) a[u] = fmaxf(a[u], s[112 + u]);
  const float b0 = fmax3(a[0], a[1], a[2]), b1 = fmax3(a[3], a[4], a[5]), b2 = fmax3(a[6], a[7], a[8]);
  const float b3 = fmax3(a[9], a[10], a[11]), b4 = fmax3(a[12], a[13], a[14]);
  return fmax3(fmax3(b0, b1, b2), fmax3(b3, b4, a[15]), b0);
}

// MERGE: the ring's merge mode (ffa_fwd_merge); its epilogue folds the result into an
// fp32 running result instead of storing bf16 O (a separate instantiation, so the plain
// forward keeps its register allocation).
// PERSIST: a CTA works through two blocks of one slice, the i-th and the last-but-i (equal
// total work under a causal mask).  Q is double-buffered: the second block's Q tiles load
// while the first runs, its first S = Q K^T is issued as soon as the first block's last
// P.V is, and the first block's epilogue overlaps the second block's start, so the second
// block pays little of the fixed cost of a CTA (launch, barrier and tensor-memory setup,
// the first loads, the epilogue).
template <int D, bool CAUSAL, bool MERGE, bool PERSIST, int EMU = fwd::emu_pairs<D>(),
          bool SEQ = fwd::seq_turns<D>()>
__global__ void __launch_bounds__(fwd::NTHREADS, 1)
    ffa_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                   float* __restrict__ LSE, int S, int BH, int group,
                   float scale_log2, float* __restrict__ ACC, float* __restrict__ ACC_LSE, int first) {
  static_assert(!(PERSIST && (SEQ || MERGE)), "the persistent forward runs without turn-taking or merge");
  using L = fwd::Layout<D, PERSIST>;
  constexpr int SLABS = D / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + L::BAR_OFF;
  auto kv_full = [&](int s) { return bar0 + 8 * (1 + s); };
  auto kv_empty = [&](int s) { return bar0 + 8 * (1 + fwd::STAGES + s); };
  auto s_full = [&](int i) { return bar0 + 8 * (1 + 2 * fwd::STAGES + i); };
  auto p_ready = [&](int i) { return bar0 + 8 * (3 + 2 * fwd::STAGES + i); };
  auto o_final = [&](int i) { return bar0 + 8 * (5 + 2 * fwd::STAGES + i); };
  const uint32_t drain_bar = bar0 + 8 * (7 + 2 * fwd::STAGES);
  auto p_half = [&](int i) { return bar0 + 8 * (8 + 2 * fwd::STAGES + i); };
  auto exp_done = [&](int i) { return bar0 + 8 * (10 + 2 * fwd::STAGES + i); };
  // Q buffer b (b = block count & 1): q_full[b] when its tiles have landed, q_empty[b]
  // when the block that used it has stored its output from it
  auto q_full = [&](int b) { return b ? bar0 + 8 * (12 + 2 * fwd::STAGES) : bar0; };
  auto q_empty = [&](int b) { return bar0 + 8 * (13 + 2 * fwd::STAGES + b); };
  auto q_buf = [&](int b) { return sbase + L::Q_OFF + b * 2 * L::TILE_BYTES; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::MISC_OFF + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_mblk = (S + 2 * fwd::BM - 1) / (2 * fwd::BM);
  const int n_kv_all = (S + fwd::BN - 1) / fwd::BN;
  // The n-th block of this CTA (rank < 0: none left).  One block per CTA, or (PERSIST) a
  // pair of blocks of one slice whose ranks add up to n_mblk - 1: under a causal mask the
  // pair's key tiles add up to the same count for every pair, so all CTAs carry equal work
  // and the pairs of a group of slices still run together (their K/V stay in L2).
  const int n_pairs = (n_mblk + 1) / 2;
  auto item_of = [&](int n) -> CtaWork {
    if (!PERSIST) return n == 0 ? cta_work(n_mblk, BH, group) : CtaWork{-1, 0};
    const CtaWork w = cta_work(n_pairs, BH, group);
    if (n == 0) return w;
    if (n == 1 && n_mblk - 1 - w.rank != w.rank) return {n_mblk - 1 - w.rank, w.bh};
    return {-1, 0};
  };
  struct Item {
    int bh, m0, nt0, nt1, n_kv;
  };
  auto decode = [&](CtaWork w) -> Item {
    // heaviest causal blocks first
    const int mblk = CAUSAL ? (n_mblk - 1 - w.rank) : w.rank;
    const int m0 = mblk * 2 * fwd::BM;
    // number of key tiles each 128-row query tile visits (0 for a tile past the end)
    auto tiles_for = [&](int mi) {
      if (mi >= S) return 0;
      return CAUSAL ? min(n_kv_all, (mi + fwd::BM - 1) / fwd::BN + 1) : n_kv_all;
    };
    const int t0 = tiles_for(m0), t1 = tiles_for(m0 + fwd::BM);
    return {w.bh, m0, t0, t1, max(t0, t1)};
  };

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(q_full(b), 1);
      mbar_init(q_empty(b), 2);
    }
    for (int s = 0; s < fwd::STAGES; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full(i), 1);
      mbar_init(p_ready(i), 128);
      mbar_init(o_final(i), 1);
      mbar_init(p_half(i), 128);
      mbar_init(exp_done(i), 128);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == fwd::MMA_WARP) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp == fwd::PRODUCER_WARP && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Each warpgroup changes its register budget inside its own branch, so the softmax
  // code is compiled against 208 registers and the control code against 88.
  if (warp >= 8) {
  setmaxnreg_dec<fwd::REGS_CONTROL>();
  if (warp == fwd::PRODUCER_WARP) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t keep = policy_evict_last();
      int issued = 0, q_issued = 0;
      bool ok = true;
      for (int n = 0; ok; ++n) {
        const CtaWork cw = item_of(n);
        if (cw.rank < 0) break;
        const Item w = decode(cw);
        const int b = n & 1;
        // the block two back has stored its output out of this buffer
        if (n >= 2 && !(ok = mbar_wait(q_empty(b), ((n >> 1) - 1) & 1, abort_flag, kErrFwdProducer))) break;
        mbar_arrive_expect_tx(q_full(b), 2 * L::TILE_BYTES);
        for (int i = 0; i < 2; ++i)
          for (int sl = 0; sl < SLABS; ++sl)
            tma_load_3d(q_buf(b) + i * L::TILE_BYTES + sl * 16384, &tm_q, q_full(b), sl * 64, w.m0 + i * fwd::BM,
                        w.bh, keep);
        ++q_issued;
        for (int j = 0; j < w.n_kv && ok; ++j) {
          for (int which = 0; which < 2; ++which) {
            const int it = issued;
            const int s = it % fwd::STAGES;
            if (!mbar_wait(kv_empty(s), ((it / fwd::STAGES) & 1) ^ 1, abort_flag, kErrFwdProducer)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(kv_full(s), L::TILE_BYTES);
            const CUtensorMap* tm = which ? &tm_v : &tm_k;
            for (int sl = 0; sl < SLABS; ++sl)
              tma_load_3d(sbase + L::KV_OFF + s * L::TILE_BYTES + sl * 16384, tm, kv_full(s), sl * 64,
                          j * fwd::BN, w.bh, keep);
            ++issued;
          }
        }
      }
      if (*abort_flag) {
        // let in-flight copies land before the CTA's shared memory goes away
        for (int it = max(0, issued - fwd::STAGES); it < issued; ++it)
          mbar_wait_drain(kv_full(it % fwd::STAGES), (it / fwd::STAGES) & 1);
        for (int n = max(0, q_issued - 2); n < q_issued; ++n) mbar_wait_drain(q_full(n & 1), (n >> 1) & 1);
      }
    }
  } else if (warp == fwd::MMA_WARP) {
    // ------------------------------------------------------------------ MMA issuer
    // The whole warp runs the issue loop (waits, descriptors and loop state are then
    // warp-uniform) and one elected lane issues each group of MMAs and its commits.
    {
      constexpr uint32_t IDESC_QK = idesc_bf16(128, fwd::BN, false, false);
      constexpr uint32_t IDESC_PV = idesc_bf16(128, D, false, true);
      bool ok = true;
      int it = 0;
      int steps[2] = {0, 0};  // P hand-overs of each tile so far (barrier phases)
      // commits track the MMAs of the thread that issues them: the same elected lane
      auto commit = [&](uint32_t bar) {
        if (elect_one()) mma_commit(bar);
        __syncwarp();
      };
      for (int n = 0; ok; ++n) {
        const CtaWork cw = item_of(n);
        if (cw.rank < 0) break;
        const Item w = decode(cw);
        const int b = n & 1;
        if (!(ok = mbar_wait(q_full(b), (n >> 1) & 1, abort_flag, kErrFwdMma))) break;
        // Descriptors are built once per tile / stage; a K-step only adds a constant.
        const uint64_t qdesc0 = kmajor_desc(q_buf(b), 128, 0), qdesc1 = kmajor_desc(q_buf(b) + L::TILE_BYTES, 128, 0);
        auto issue_qk = [&](int i, uint32_t k_addr) {
          const uint64_t qd = i ? qdesc1 : qdesc0;
          const uint64_t kd = kmajor_desc(k_addr, 128, 0);
          const uint32_t d = tmem + i * 128;
          if (elect_one()) {
            mma_ss(d, qd, kd, IDESC_QK, 0u);
#pragma unroll
            for (int ks = 1; ks < D / 16; ++ks)
              mma_ss_acc(d, qd + kmajor_step(128, ks), kd + kmajor_step(128, ks), IDESC_QK);
            mma_commit(s_full(i));
          }
          __syncwarp();
        };
        // K-steps [k0, k1) of O_i += P_i V_j (16 keys = 8 TMEM columns of packed P each)
        auto issue_pv = [&](int i, uint32_t v_addr, int j, int k0, int k1) {
          const uint64_t vd = mnmajor_desc(v_addr, fwd::BN, 0);
          const uint32_t d = tmem + 256 + i * 128, a = tmem + i * 128;
          if (elect_one()) {
            for (int ks = k0; ks < k1; ++ks) {
              if (ks == 0)
                mma_ts(d, a, vd, IDESC_PV, j > 0 ? 1u : 0u);
              else
                mma_ts_acc(d, a + ks * 8, vd + mnmajor_step(ks), IDESC_PV);
            }
          }
          __syncwarp();
        };
        // P_i(j) V_j: in two halves when the softmax hands P over in halves
        auto issue_pv_tile = [&](int i, uint32_t v_addr, int j) -> bool {
          const int ph = (steps[i] + j) & 1;
          if (!mbar_wait(p_half(i), ph, abort_flag, kErrFwdMma)) return false;
          tc_fence_after();
          issue_pv(i, v_addr, j, 0, fwd::BN / 32);
          if (!mbar_wait(p_ready(i), ph, abort_flag, kErrFwdMma)) return false;
          tc_fence_after();
          issue_pv(i, v_addr, j, fwd::BN / 32, fwd::BN / 16);
          return true;
        };
        // prologue: S_i(0)
        if (w.n_kv > 0) {
          const int s = it % fwd::STAGES;
          if (!(ok = mbar_wait(kv_full(s), (it / fwd::STAGES) & 1, abort_flag, kErrFwdMma))) break;
          tc_fence_after();
          const uint32_t k_addr = sbase + L::KV_OFF + s * L::TILE_BYTES;
          if (w.nt0 > 0) issue_qk(0, k_addr);
          if (w.nt1 > 0) issue_qk(1, k_addr);
          commit(kv_empty(s));
          ++it;
        }
        for (int j = 0; j < w.n_kv && ok; ++j) {
          const int sv = it % fwd::STAGES;
          if (!(ok = mbar_wait(kv_full(sv), (it / fwd::STAGES) & 1, abort_flag, kErrFwdMma))) break;
          ++it;
          const uint32_t v_addr = sbase + L::KV_OFF + sv * L::TILE_BYTES;
          const bool next = (j + 1 < w.n_kv);
          int sk = -1;
          uint32_t k_addr = 0;
          // tile 0: O0 += P0 V_j, then S0 = Q0 K_{j+1}^T
          if (j < w.nt0) {
            if (!(ok = issue_pv_tile(0, v_addr, j))) break;
          }
          if (next) {
            sk = it % fwd::STAGES;
            if (!(ok = mbar_wait(kv_full(sk), (it / fwd::STAGES) & 1, abort_flag, kErrFwdMma))) break;
            tc_fence_after();
            k_addr = sbase + L::KV_OFF + sk * L::TILE_BYTES;
            if (j + 1 < w.nt0) issue_qk(0, k_addr);
          }
          // tile 1: O1 += P1 V_j, then S1 = Q1 K_{j+1}^T
          if (j < w.nt1) {
            if (!(ok = issue_pv_tile(1, v_addr, j))) break;
          }
          commit(kv_empty(sv));
          if (next) {
            if (j + 1 < w.nt1) issue_qk(1, k_addr);
            commit(kv_empty(sk));
            ++it;
          }
        }
        if (!ok) break;
        // O_i complete (a tile with no keys gets no commit: its warpgroup does not wait)
        if (w.nt0 > 0) commit(o_final(0));
        if (w.nt1 > 0) commit(o_final(1));
        steps[0] += w.nt0;
        steps[1] += w.nt1;
      }
      // every issued MMA has finished before TMEM is released
      commit(drain_bar);
      mbar_wait_drain(drain_bar, 0);
    }
    __syncwarp();
  }
  } else {
    setmaxnreg_inc<fwd::REGS_SOFTMAX>();
    // ------------------------------------------------------------------ softmax
    const int i = warp >> 2;            // tile
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + lane_off + i * 128;
    const uint32_t t_o = tmem + lane_off + 256 + i * 128;
    bool ok = true;
    int steps = 0, finals = 0;  // this tile's S hand-overs and completed blocks (barrier phases)
    for (int n = 0; ok; ++n) {
      const CtaWork cw = item_of(n);
      if (cw.rank < 0) break;
      const Item w = decode(cw);
      const int bh = w.bh;
      const int mi = w.m0 + i * fwd::BM;
      const int grow = mi + row;
      const int nt = i ? w.nt1 : w.nt0;
      float m_used = -INFINITY;
      float l = 0.f;
      for (int j = 0; j < nt; ++j) {
        if (!(ok = mbar_wait(s_full(i), (steps + j) & 1, abort_flag, kErrFwdSoftmax))) break;
        tc_fence_after();
        float s[fwd::BN];
        {
          uint32_t r[4][32];
#pragma unroll
          for (int c = 0; c < 4; ++c) tmem_ld32(t_s + c * 32, r[c]);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e) s[c * 32 + e] = __uint_as_float(r[c][e]);
        }
        const int n0 = j * fwd::BN;
        const bool need_mask = (n0 + fwd::BN > S) || (CAUSAL && n0 + fwd::BN - 1 > mi);
        // Row max of the scaled scores.  Unmasked tiles reduce the raw scores and scale
        // once (scale*log2e > 0 keeps the order; a negative scale reduces with min);
        // masked tiles (diagonal / ragged tail) scale first and drop masked columns.
        float tmax;
        if (need_mask) {
          const int lim = CAUSAL ? min(S - 1, grow) : (S - 1);
#pragma unroll
          for (int c = 0; c < fwd::BN; ++c) s[c] = (n0 + c > lim) ? -INFINITY : s[c] * scale_log2;
          tmax = row_max128(s);
        } else if (scale_log2 >= 0.f) {
          tmax = row_max128(s) * scale_log2;
        } else {
          float a = s[0];
#pragma unroll
          for (int c = 1; c < fwd::BN; ++c) a = fminf(a, s[c]);
          tmax = a * scale_log2;
        }
        const float m_new = fmaxf(m_used, tmax);
        const bool need = m_new > m_used + fwd::RESCALE_THRESHOLD;
        if (__any_sync(0xffffffffu, need)) {
          const float m_safe = (m_new == -INFINITY) ? 0.f : m_new;
          const float alpha = fast_exp2(m_used - m_safe);
          if (j > 0) {
            // O_i(j-1) is complete: S_i(j) was committed after P_i(j-1) V_{j-1}.
#pragma unroll 1
            for (int c = 0; c < D / 32; ++c) {
              uint32_t r[32];
              tmem_ld32(t_o + c * 32, r);
              tmem_ld_wait();
#pragma unroll
              for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
              tmem_st32(t_o + c * 32, r);
            }
          }
          l *= alpha;
          m_used = m_new;
        }
        const float m_safe = (m_used == -INFINITY) ? 0.f : m_used;
        uint32_t p[2][32];
        float2 sum2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        const float2 c2 = make_float2(scale_log2, scale_log2), nm2 = make_float2(-m_safe, -m_safe);
        // Column pairs [h*32, h*32+32) -> p[h] -> TMEM columns [h*32, h*32+32) of S_i.
        auto half = [&](const int h) {
          if (need_mask) {
#pragma unroll
            for (int u = 0; u < 32; ++u) {
              const int c = h * 32 + u;
              const float p0 = fast_exp2(s[2 * c] - m_safe);
              const float p1 = fast_exp2(s[2 * c + 1] - m_safe);
              sum2[u & 1] = add2(sum2[u & 1], make_float2(p0, p1));
              p[h][u] = pack_bf16x2(p0, p1);
            }
          } else {
            // EMU of every 8 column pairs take the FMA-pipe exp2, the rest MUFU.EX2
#pragma unroll
            for (int u = 0; u < 32; ++u) {
              const int c = h * 32 + u;
              const float2 x = fma2(make_float2(s[2 * c], s[2 * c + 1]), c2, nm2);
              float p0, p1;
              if ((c & 7) < EMU) {
                const float2 e2 = exp2_fma2(x);
                p0 = e2.x;
                p1 = e2.y;
              } else {
                p0 = fast_exp2(x.x);
                p1 = fast_exp2(x.y);
              }
              sum2[u & 1] = add2(sum2[u & 1], make_float2(p0, p1));
              p[h][u] = pack_bf16x2(p0, p1);
            }
          }
          if (SEQ && h == 1) mbar_arrive(exp_done(i));
          tmem_st32(t_s + 32 * h, p[h]);
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(h == 0 ? p_half(i) : p_ready(i));
        };
        if (SEQ) {
          // take turns with the other warpgroup: wait for its exponentials of step j
          // (tile 1) or j-1 (tile 0), when it has such a step (one block per CTA here)
          const int oj = i ? j : j - 1;
          if (oj >= 0 && oj < (i ? w.nt0 : w.nt1) &&
              !(ok = mbar_wait(exp_done(i ^ 1), oj & 1, abort_flag, kErrFwdSoftmax)))
            break;
        }
        half(0);
        half(1);
        const float2 sv = add2(sum2[0], sum2[1]);
        l += sv.x + sv.y;
      }
      steps += nt;
      // Epilogue: O_i / l into its Q tile (free once every MMA of the block has finished),
      // then one TMA store; rows at or past S are clipped by the tensor map.  Every thread
      // of the warpgroup reaches the barrier, finished or not, so none can wait for one
      // that left.
      const bool staged = ok && nt > 0 && mbar_wait(o_final(i), finals & 1, abort_flag, kErrFwdSoftmax);
      if (nt > 0) ++finals;
      const uint32_t o_tile = q_buf(n & 1) + i * L::TILE_BYTES;
      if constexpr (MERGE) {
        // Merge mode: fold this result (O = acc/l, base-2 LSE lp) into the running fp32
        // result of its rows: w_a = 2^(la - m), w_b = 2^(lp - m), m = max(la, lp);
        // acc = (w_a acc + w_b O) / (w_a + w_b), acc_lse = m + log2(w_a + w_b).  This
        // thread's row has no other writer in the launch.
        if (staged) {
          tc_fence_after();
          const bool valid = grow < S;
          const long long idx = static_cast<long long>(bh) * S + grow;
          const float lp = (l == 0.f) ? -INFINITY : m_used + log2f(l);
          const float la = (first || !valid) ? -INFINITY : ACC_LSE[idx];
          const float mm = fmaxf(la, lp);
          const float wa = (mm == -INFINITY) ? 1.f : exp2f(la - mm);
          const float wb = (mm == -INFINITY) ? 0.f : exp2f(lp - mm);
          const float inv = 1.f / (wa + wb);
          const float ca = wa * inv, cb = (l == 0.f) ? 0.f : wb * inv / l;
          float* dst = ACC + idx * D;
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(t_o + c * 32, r);
            tmem_ld_wait();
            if (valid) {
              float4* d4 = reinterpret_cast<float4*>(dst + 32 * c);
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float4 a = first ? make_float4(0.f, 0.f, 0.f, 0.f) : d4[e];
                d4[e] = make_float4(fmaf(a.x, ca, __uint_as_float(r[4 * e + 0]) * cb),
                                    fmaf(a.y, ca, __uint_as_float(r[4 * e + 1]) * cb),
                                    fmaf(a.z, ca, __uint_as_float(r[4 * e + 2]) * cb),
                                    fmaf(a.w, ca, __uint_as_float(r[4 * e + 3]) * cb));
              }
            }
          }
          if (valid) ACC_LSE[idx] = (mm == -INFINITY) ? -INFINITY : mm + log2f(wa + wb);
        }
      } else if (staged) {
        tc_fence_after();
        const float l_safe = (l == 0.f) ? 1.f : l;
        const float inv_l = 1.f / l_safe;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(t_o + c * 32, r);
          tmem_ld_wait();
          stage_row32_sw128(o_tile, row, 32 * c, r, inv_l);
        }
        if (LSE != nullptr && grow < S) {
          const float m_fin = (m_used == -INFINITY) ? 0.f : m_used;
          LSE[static_cast<long long>(bh) * S + grow] = m_fin + __log2f(l_safe);
        }
      }
      fence_proxy_async_smem();
      const bool store = named_barrier_and(1 + i, 128, staged && !MERGE);
      if (row == 0) {
        if (store) {
#pragma unroll
          for (int sl = 0; sl < SLABS; ++sl) tma_store_3d(&tm_o, o_tile + sl * 16384, sl * 64, mi, bh);
          bulk_commit_group();
          bulk_wait_read();
        }
        mbar_arrive(q_empty(n & 1));  // this tile's half of the Q buffer may be reloaded
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == fwd::MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------------
// host launcher
// ------------------------------------------------------------------------------------
template <int D, bool CAUSAL, bool MERGE>
static int launch_fwd_t(const FwdArgs& a, cudaStream_t stream) {
  constexpr bool PERSIST = !MERGE && !fwd::seq_turns<D>();
  using L = fwd::Layout<D, PERSIST>;
  CUtensorMap tq, tk, tv;
  int rc;
  if ((rc = make_tile_map(&tq, a.q, a.BH, a.S, D, a.stride_bh, a.stride_s)) != 0) return rc;
  if ((rc = make_tile_map(&tk, a.k, a.BH, a.S, D, a.stride_bh, a.stride_s)) != 0) return rc;
  if ((rc = make_tile_map(&tv, a.v, a.BH, a.S, D, a.stride_bh, a.stride_s)) != 0) return rc;
  CUtensorMap to;  // merge mode stores nothing through it: q serves as its base
  if ((rc = make_tile_map(&to, a.acc ? a.q : a.o, a.BH, a.S, D, a.stride_bh, a.stride_s)) != 0) return rc;
  auto kern = ffa_fwd_kernel<D, CAUSAL, MERGE, PERSIST>;
  static unsigned long long configured = 0;  // devices with the smem limit raised
  if ((rc = set_smem_once(reinterpret_cast<const void*>(kern), L::SMEM_BYTES, &configured)) != 0) return rc;
  // The setmaxnreg split assumes the kernel is launched with 168 registers per thread;
  // with fewer, setmaxnreg.inc could never be satisfied, so refuse to launch instead.
  static int launch_regs = -1;
  if (launch_regs < 0) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, reinterpret_cast<const void*>(kern)) != cudaSuccess)
      return set_error(FFA_ERR_LAUNCH, "cudaFuncGetAttributes(fwd) failed");
    launch_regs = fa.numRegs;
  }
  if (launch_regs < fwd::LAUNCH_REGS_NEEDED)
    return set_error(FFA_ERR_LAUNCH, "forward kernel compiled with too few registers for its setmaxnreg split");
  const int n_mblk = (a.S + 2 * fwd::BM - 1) / (2 * fwd::BM);
  // PERSIST: one CTA per pair of blocks of a slice
  const int n_rows = PERSIST ? (n_mblk + 1) / 2 : n_mblk;
  const dim3 grid(static_cast<unsigned>(n_rows) * static_cast<unsigned>(a.BH));
  kern<<<grid, fwd::NTHREADS, L::SMEM_BYTES, stream>>>(tq, tk, tv, to, a.lse, a.S, a.BH, work_group(a.BH, a.S, D, CAUSAL),
                                                        static_cast<float>(a.scale * kLog2e), a.acc, a.acc_lse,
                                                        a.first);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FFA_ERR_LAUNCH, cudaGetErrorString(e));
  return FFA_OK;
}

template <int D, bool CAUSAL>
static int launch_fwd_m(const FwdArgs& a, cudaStream_t stream) {
  return a.acc ? launch_fwd_t<D, CAUSAL, true>(a, stream) : launch_fwd_t<D, CAUSAL, false>(a, stream);
}

int launch_fwd(const FwdArgs& a, cudaStream_t stream) {
  if (a.D == 128) return a.causal ? launch_fwd_m<128, true>(a, stream) : launch_fwd_m<128, false>(a, stream);
  if (a.D == 64) return a.causal ? launch_fwd_m<64, true>(a, stream) : launch_fwd_m<64, false>(a, stream);
  return set_error(FFA_ERR_UNSUPPORTED, "kernel head_dim must be 64 or 128");
}

}  // namespace ffa
