// ffa_aux.cuh — the two memory-bound helper kernels of the attention library:
//   * backward preprocess  delta[bh,i] = sum_d O[bh,i,d] * dO[bh,i,d]   (fp32)
//     (reference `_uni_bwd_preprocess`, fastflash_attention/_kernel.py:323-338)
//   * LSE merge of two partial attention results, used by the context-parallel ring.
// Both stream their inputs once with 16-byte vector loads; they are HBM-bound.
#pragma once
#include "ffa_common.cuh"

namespace ffa {

// One group of D/8 threads per row; each thread owns 8 consecutive columns (16 bytes).
template <int D>
__global__ void __launch_bounds__(256) ffa_preprocess_kernel(const __nv_bfloat16* __restrict__ O,
                                                              const __nv_bfloat16* __restrict__ dO,
                                                              float* __restrict__ delta, int BH, int S,
                                                              long long stride_bh, long long stride_s) {
  constexpr int TPR = D / 8;  // threads per row
  constexpr int ROWS_PER_BLOCK = 256 / TPR;
  const int sub = threadIdx.x % TPR;
  const long long total = static_cast<long long>(BH) * S;
  for (long long r = static_cast<long long>(blockIdx.x) * ROWS_PER_BLOCK + threadIdx.x / TPR; r < total;
       r += static_cast<long long>(gridDim.x) * ROWS_PER_BLOCK) {
    const long long bh = r / S, i = r % S;
    const long long off = bh * stride_bh + i * stride_s + sub * 8;
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(O + off));
    const uint4 b = __ldg(reinterpret_cast<const uint4*>(dO + off));
    const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&b);
    float acc = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 x = __bfloat1622float2(a2[e]);
      const float2 y = __bfloat1622float2(b2[e]);
      acc = fmaf(x.x, y.x, acc);
      acc = fmaf(x.y, y.y, acc);
    }
#pragma unroll
    for (int o = TPR / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (sub == 0) delta[r] = acc;
  }
}

// One warp per row; each lane owns 4 columns (D <= 128).
__global__ void __launch_bounds__(256) ffa_lse_merge_kernel(float* __restrict__ acc, float* __restrict__ acc_lse,
                                                             const __nv_bfloat16* __restrict__ part,
                                                             const float* __restrict__ part_lse, long long rows,
                                                             int D, int first) {
  const int lane = threadIdx.x & 31;
  const long long nwarps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long r = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += nwarps) {
    const float lb = part_lse[r];
    const float la = first ? -INFINITY : acc_lse[r];
    const float m = fmaxf(la, lb);
    // weights of the two partial results; an empty side (lse = -inf) gets weight 0
    const float wa = (m == -INFINITY) ? 1.f : exp2f(la - m);
    const float wb = (m == -INFINITY) ? 0.f : exp2f(lb - m);
    const float inv = 1.f / (wa + wb);
    const int c = lane * 4;
    if (c < D) {
      const uint2 raw = *reinterpret_cast<const uint2*>(part + r * D + c);
      const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
      const float2 p01 = __bfloat1622float2(p2[0]);
      const float2 p23 = __bfloat1622float2(p2[1]);
      float4* dst = reinterpret_cast<float4*>(acc + r * D + c);
      float4 a = first ? make_float4(0.f, 0.f, 0.f, 0.f) : *dst;
      a.x = (wa * a.x + wb * p01.x) * inv;
      a.y = (wa * a.y + wb * p01.y) * inv;
      a.z = (wa * a.z + wb * p23.x) * inv;
      a.w = (wa * a.w + wb * p23.y) * inv;
      *dst = a;
    }
    __syncwarp();  // every lane has read acc_lse[r] before lane 0 replaces it
    if (lane == 0) acc_lse[r] = (m == -INFINITY) ? -INFINITY : m + log2f(wa + wb);
  }
}

}  // namespace ffa
