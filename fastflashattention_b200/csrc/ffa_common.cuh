// ffa_common.cuh — shared host/device declarations of the attention library.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <algorithm>
#include <cstdint>
#include <mutex>

#include "../../include/ffa.h"
#include "sm100.cuh"

namespace ffa {

// log2(e), the base change folded into the softmax scale (reference _kernel.py:40)
constexpr double kLog2e = 1.4426950408889634;

// ids of the waits that can time out (recorded in g_status[0])
enum : unsigned int {
  kErrFwdProducer = 0x101,
  kErrFwdMma = 0x102,
  kErrFwdSoftmax = 0x103,
  kErrBwdProducer = 0x201,
  kErrBwdMma = 0x202,
  kErrBwdCompute = 0x203,
  kErrBwdAlign = 0x204,  // dynamic shared memory not 1024-byte aligned
  kErrDqProducer = 0x301,
  kErrDqMma = 0x302,
  kErrDqCompute = 0x303,
};

struct FwdArgs {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  float* lse;
  int BH, S, D;
  long long stride_bh, stride_s;
  double scale;
  int causal;
  // merge mode (ffa_fwd_merge): fold this call's result into a running fp32 result
  // acc [BH, S, D] (row stride D) with base-2 LSE acc_lse [BH, S]; `first` initialises it
  float* acc = nullptr;
  float* acc_lse = nullptr;
  int first = 0;
};

struct BwdArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const void* dout;
  const float* lse;
  float* delta;
  void* dq;
  void* dk;
  void* dv;
  int BH, S, D;
  long long stride_bh, stride_s;
  double scale;
  int causal;
  // accumulate mode (ffa_bwd_dkdv_acc / ffa_bwd_dq_acc): add the gradients in fp32 into
  // [BH, S, D] buffers (row stride D) instead of writing bf16 dq / dk / dv
  float* dq_acc = nullptr;
  float* dk_acc = nullptr;
  float* dv_acc = nullptr;
};

// Work of a CTA in a 1-D grid of nblk x BH CTAs: its block rank (rank 0 = the block
// with the most work) and its (batch, head) slice.  Slices are taken in groups of
// `group`, small enough that the tiles the running CTAs stream (K/V, or Q/dO) stay
// resident in L2; inside a group every slice's rank-0 block launches before any rank-1
// block, so the heaviest blocks of the whole group start first and the grid's tail
// holds the lightest ones (longest job first).  On B200, B4 H16 D128 causal: forward
// -17 % at S=1024, -10 % at S=2048; dK/dV -2 to -4 %.
struct CtaWork {
  int rank;
  int bh;
};
__host__ __device__ __forceinline__ CtaWork cta_work_at(int L, int nblk, int BH, int group) {
  const int per_group = group * nblk;
  const int g = L / per_group;
  const int w = L - g * per_group;
  const int gsize = (group < BH - g * group) ? group : BH - g * group;
  return {w / gsize, g * group + w % gsize};
}
__device__ __forceinline__ CtaWork cta_work(int nblk, int BH, int group) {
  return cta_work_at(static_cast<int>(blockIdx.x), nblk, BH, group);
}

// Slices per work group for kernels that stream two [S, D] bf16 operands per slice.
// Without a causal mask every block of a slice has the same work, there is nothing to
// reorder, and one slice at a time (block-major, the plain grid order) keeps the best
// L2 locality (measured 2-3 % faster on B200 than grouping).
inline int work_group(int BH, int S, int D, bool causal) {
  if (!causal) return 1;
  const long long per_slice = 2LL * S * D * 2;
  const long long budget = 48LL << 20;
  const long long g = budget / (per_slice > 0 ? per_slice : 1);
  return static_cast<int>(g < 1 ? 1 : (g > BH ? BH : g));
}

// host helpers (ffa_capi.cu)
int set_error(int code, const char* msg);
int ensure_context();
// Raise a kernel's dynamic shared-memory limit once per device; `done` is a per-kernel
// bitmask of devices already configured.
int set_smem_once(const void* kernel, int bytes, unsigned long long* done);
// FFA_OK if `kernel` is launched with at least `needed` registers per thread (kernels
// that rebalance registers with setmaxnreg rely on the launch allocation).
int check_launch_regs(const void* kernel, int needed);
// 3-D tensor map over a [BH, S, D] bf16 tensor: box = 64 columns x `box_rows` rows x 1
// slice, 128-byte swizzle (the layout the tcgen05 descriptors in sm100.cuh expect).
int make_tile_map(CUtensorMap* map, const void* base, int BH, int S, int D, long long stride_bh,
                  long long stride_s, int box_rows = 128);

int launch_fwd(const FwdArgs& a, cudaStream_t stream);
int launch_bwd(const BwdArgs& a, cudaStream_t stream);
int launch_dkdv(const BwdArgs& a, cudaStream_t stream);
int launch_dq(const BwdArgs& a, cudaStream_t stream);
int launch_preprocess(const void* o, const void* dout, float* delta, int BH, int S, int D, long long stride_bh,
                      long long stride_s, cudaStream_t stream);
int launch_lse_merge(float* acc, float* acc_lse, const void* part, const float* part_lse, long long rows, int D,
                     int first, cudaStream_t stream);

}  // namespace ffa
