// sm100.cuh — hand-written PTX wrappers for the Blackwell (sm_100a) primitives the
// attention kernels are built from: mbarriers with bounded waits, TMA tensor loads,
// tcgen05 tensor-memory allocation / MMA / commit / load / store, and the shared-memory
// matrix and instruction descriptors the tcgen05.mma instruction consumes.
//
// Descriptor bit layouts follow the PTX ISA "Matrix Descriptors" (shared memory
// descriptor, version 1 for tcgen05) and "Instruction descriptor" tables for
// .kind::f16.  Nothing here depends on CUTLASS.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>

namespace ffa {

// ------------------------------------------------------------------------------------
// Device status word: the first failure (a wait that ran out of time) is recorded here
// and read by the host through ffa_last_error().  Codes are defined in ffa.h.
// ------------------------------------------------------------------------------------
// Defined once: the library is built as a single translation unit (ffa_capi.cu).
__device__ unsigned int g_status[4];

// A wait gives up after this many nanoseconds of polling (about one second).  Every
// legitimate wait in these kernels is shorter than a millisecond.
constexpr unsigned long long kWaitLimitNs = 1000ull * 1000ull * 1000ull;

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// True in the lowest active lane of the calling warp (whatever the branch that got here).
__device__ __forceinline__ bool first_active_lane() {
  uint32_t lt;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(lt));
  return (__activemask() & lt) == 0u;
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ------------------------------------------------------------------------------------
// mbarrier
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on the phase with the given parity.  Returns false (and records `site`
// in the status word and raises the CTA-wide abort flag) when the limit is reached or
// when another role of the CTA has already aborted.  Callers then leave their loops and
// fall through to the common teardown, so a lost arrival never hangs the GPU.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          unsigned int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kWaitLimitNs) {
      *abort_flag = 1;
      if (first_active_lane()) {  // one record per waiting warp
        atomicCAS(&g_status[0], 0u, site);
        atomicAdd(&g_status[1], 1u);
      }
      return false;
    }
  }
}

// Bounded wait used during teardown: ignores the abort flag (the point is to let work
// that is already in flight finish before shared or tensor memory is released).
__device__ __forceinline__ void mbar_wait_drain(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitLimitNs) {
      if (first_active_lane()) atomicAdd(&g_status[2], 1u);
      return;
    }
  }
}

// ------------------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), plain loads only; each CTA fetches its own tiles.
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* m, uint32_t bar, int c0,
                                            int c1, int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}

// TMA tile store (shared -> global) in a bulk group.  Box rows and columns outside the
// tensor are not written, so a ragged last tile needs no masking.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* m, uint32_t src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until every committed bulk store of this thread has completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Wait until every committed bulk store of this thread has finished reading its shared
// memory source.  Enough before a CTA exits: the global writes still complete before the
// kernel does (stream order), and the CTA no longer waits for their round trip.
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Barrier among `n` threads (a multiple of 32) on hardware barrier `id` (1..15; 0 is
// __syncthreads) that also returns whether `pred` holds in all of them.
__device__ __forceinline__ bool named_barrier_and(int id, int n, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred p, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(pred ? 1u : 0u), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------------------------
// tcgen05: tensor memory
// ------------------------------------------------------------------------------------
// Allocate `ncols` TMEM columns (power of two >= 32); the base address lands in smem.
// Warp-collective.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]   (A is K-major, bf16 packed two per 32-bit column)
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same, with the accumulate flag fixed to "accumulate" (no runtime predicate setup).
__device__ __forceinline__ void mma_ss_acc(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.eq.u32 p, 1, 1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc)
      : "memory");
}
__device__ __forceinline__ void mma_ts_acc(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.eq.u32 p, 1, 1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc)
      : "memory");
}

// Arrive once on `bar` when every tcgen05 operation issued so far by this thread is done.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// 32 lanes x 32 columns of 32-bit: thread t of the warp receives lane (base_lane + t),
// columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]),
      "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]),
      "r"(r[30]), "r"(r[31])
      : "memory");
}
// 32 lanes x 16 columns of 32-bit.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Warpgroup-wide register reallocation.  The sum over warpgroups after the change must not
// exceed what the CTA was launched with (threads x registers per thread).
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ------------------------------------------------------------------------------------
// Shared-memory matrix descriptors (tcgen05 version 1).
//   bits  0-13 start address >> 4
//   bits 16-29 leading-dimension byte offset >> 4
//   bits 32-45 stride-dimension byte offset >> 4
//   bits 46-47 version (1)
//   bits 49-51 base offset (0: every swizzle atom is 1024-byte aligned)
//   bits 61-63 layout: 2 = 128-byte swizzle
// Tiles are stored exactly as TMA writes them with CU_TENSOR_MAP_SWIZZLE_128B:
// rows of 128 bytes (64 bf16), 8-row groups of 1024 bytes, and the tile split into
// "slabs" of 64 columns, one slab after the other.
// ------------------------------------------------------------------------------------
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// K-major operand (rows = M or N, the contraction dim K contiguous): one MMA consumes
// 16 K-elements = 32 bytes of each row.  K-step `ks` (16 elements each) of a tile with
// `rows` rows starts inside slab ks/4 at byte offset 32*(ks%4).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile_saddr, int rows, int ks) {
  const uint32_t addr = tile_saddr + (ks >> 2) * (rows * 128) + (ks & 3) * 32;
  return sw128_desc(addr, 16, 1024);
}

// MN-major operand (the contraction dim K runs over rows, the N dim is contiguous):
// one MMA consumes 16 rows; N spans slabs at stride rows*128 bytes (LBO).
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile_saddr, int rows, int ks) {
  const uint32_t addr = tile_saddr + ks * 16 * 128;
  return sw128_desc(addr, rows * 128, 1024);
}

// Descriptor increments (in the 16-byte units of the start-address field) that move a
// base descriptor (ks = 0) to K-step ks; adding them never carries out of the 14-bit
// field because shared-memory addresses stay below 2^18.
__host__ __device__ constexpr uint32_t kmajor_step(int rows, int ks) {
  return static_cast<uint32_t>(((ks >> 2) * rows * 128 + (ks & 3) * 32) >> 4);
}
__host__ __device__ constexpr uint32_t mnmajor_step(int ks) { return static_cast<uint32_t>((ks * 16 * 128) >> 4); }

// Instruction descriptor, kind::f16 with bf16 inputs and fp32 accumulation.
//   bits 4-5 D format (1 = f32), 7-9 A format (1 = bf16), 10-12 B format (1 = bf16),
//   bit 15 A major (0 = K), bit 16 B major (0 = K, 1 = MN), 17-22 N>>3, 24-28 M>>4.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// ------------------------------------------------------------------------------------
// Small numeric helpers
// ------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Packed two-wide fp32 arithmetic (sm_100 f32x2): one instruction for two lanes of work.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "sub.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}

// 2^x on the special-function unit (MUFU.EX2).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe, for x >= -126 (smaller x is clamped to -126; callers use it only
// where no score is masked).  Method: Cody–Waite-style range reduction x = n + f with n
// the nearest integer (obtained by adding and subtracting the shifter 1.5*2^23) and
// f in [-1/2, 1/2]; 2^f from a degree-3 polynomial whose coefficients minimise the
// maximum relative error on that interval (Remez exchange, derived by
// tests/test_exp2_poly.py, which re-derives them; max relative error 7.5e-5, 25x below
// bf16's half-ulp; x <= -126 returns about 2^-126, not 0);
// 2^n is applied by adding n to the exponent field.  Offloading part of the softmax
// exponentials here keeps MUFU.EX2 (16/clk/SM) from capping the tensor core.
__device__ __forceinline__ float exp2_fma(float x) {
  constexpr float kShifter = 12582912.0f;  // 1.5 * 2^23
  constexpr float c0 = 0.9999280571937561f, c1 = 0.6932609677314758f, c2 = 0.2426111251115799f,
                  c3 = 0.0551716685295105f;
  x = fmaxf(x, -126.0f);
  const float t = __fadd_rn(x, kShifter);  // low mantissa bits of t hold n = round(x)
  const float n = __fsub_rn(t, kShifter);
  const float f = __fsub_rn(x, n);
  const float p = fmaf(fmaf(fmaf(c3, f, c2), f, c1), f, c0);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// exp2_fma on two values with packed f32x2 arithmetic (the same polynomial and rounding
// as exp2_fma, about half the instructions per value).
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
  constexpr float kShifter = 12582912.0f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const float2 t = add2(x, make_float2(kShifter, kShifter));  // low mantissa bits of t hold round(x)
  const float2 n = sub2(t, make_float2(kShifter, kShifter));
  const float2 f = sub2(x, n);
  float2 p = fma2(make_float2(0.0551716685295105f, 0.0551716685295105f), f,
                  make_float2(0.2426111251115799f, 0.2426111251115799f));
  p = fma2(p, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
  p = fma2(p, f, make_float2(0.9999280571937561f, 0.9999280571937561f));
#if FFA_EXP2_IMAD
  // bits(p) + n * 2^23 as one integer multiply-add (FMA pipe) instead of shift + add (ALU)
  uint32_t rx, ry;
  asm("mad.lo.u32 %0, %1, 8388608, %2;" : "=r"(rx) : "r"(__float_as_uint(t.x)), "r"(__float_as_uint(p.x)));
  asm("mad.lo.u32 %0, %1, 8388608, %2;" : "=r"(ry) : "r"(__float_as_uint(t.y)), "r"(__float_as_uint(p.y)));
  return make_float2(__uint_as_float(rx), __uint_as_float(ry));
#else
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
#endif
}

// Three-input max (sm_100 max.f32 with three sources).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Write 32 fp32 values (times `mul`, as bf16) of row `row`, columns [col0, col0+32), into a
// 128-row bf16 tile staged in shared memory for a SWIZZLE_128B TMA store: 64-column
// slabs of 16 KB, 128 bytes per row, 16-byte chunk k of a row at (k ^ (row & 7)) * 16.
// Rows of a warp hit distinct banks for every chunk.
__device__ __forceinline__ void stage_row32_sw128(uint32_t tile, int row, int col0, const uint32_t (&r)[32],
                                                  float mul) {
  const uint32_t line = tile + (col0 >> 6) * 16384 + row * 128;
  const uint32_t x = static_cast<uint32_t>(row & 7);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint32_t k = static_cast<uint32_t>(((col0 & 63) >> 3) + e);
    uint32_t w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = 8 * e + 2 * u;
      w[u] = pack_bf16x2(__uint_as_float(r[i]) * mul, __uint_as_float(r[i + 1]) * mul);
    }
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(line + ((k ^ x) << 4)), "r"(w[0]), "r"(w[1]),
                 "r"(w[2]), "r"(w[3])
                 : "memory");
  }
}

}  // namespace ffa
