// ffa_capi.cu — the C ABI of libffa_sm100.so (declared in include/ffa.h).
//
// This is the library's single translation unit: it includes every kernel header, so
// the device status word `ffa::g_status` has exactly one definition.  The entry points
// validate their arguments, build TMA tensor maps and launch on the caller's stream;
// they never allocate device memory.
#include <cstdio>
#include <cstring>
#include <mutex>

#include "ffa_common.cuh"
#include "ffa_fwd.cuh"
#include "ffa_bwd.cuh"
#include "ffa_aux.cuh"

namespace ffa {

namespace {
thread_local int t_last_code = FFA_OK;
thread_local char t_last_msg[256] = "";

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

int set_error(int code, const char* msg) {
  t_last_code = code;
  std::snprintf(t_last_msg, sizeof(t_last_msg), "%s", msg ? msg : "");
  return code;
}

// Make the current device's primary context current on the calling thread.  Callers
// such as torch's autograd worker threads select a device without ever touching the
// runtime, and the driver-level tensor-map encoder needs a current context.
// Done once per thread and device (a thread that switches devices sets the new one).
int ensure_context() {
  static thread_local int t_ctx_dev = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_error(FFA_ERR_LAUNCH, "no usable CUDA device on this thread");
  if (dev != t_ctx_dev) {
    if (cudaSetDevice(dev) != cudaSuccess) return set_error(FFA_ERR_LAUNCH, "no usable CUDA device on this thread");
    t_ctx_dev = dev;
  }
  return FFA_OK;
}

// Encoded tensor maps of recent calls, per thread.  A map depends only on the fields of
// the key (no device memory is read when encoding), so a hit returns exactly what the
// encoder would; callers that reuse their buffers (the torch caching allocator does)
// skip the driver call.
namespace {
struct MapKey {
  const void* base;
  int BH, S, D, box_rows;
  long long stride_bh, stride_s;
  bool operator==(const MapKey& o) const {
    return base == o.base && BH == o.BH && S == o.S && D == o.D && box_rows == o.box_rows &&
           stride_bh == o.stride_bh && stride_s == o.stride_s;
  }
};
struct MapCache {
  static constexpr int N = 16;
  MapKey key[N];
  CUtensorMap map[N];
  bool used[N] = {};
  int next = 0;
};
thread_local MapCache t_maps;
}  // namespace

int make_tile_map(CUtensorMap* map, const void* base, int BH, int S, int D, long long stride_bh,
                  long long stride_s, int box_rows) {
  const MapKey key{base, BH, S, D, box_rows, stride_bh, stride_s};
  for (int i = 0; i < MapCache::N; ++i)
    if (t_maps.used[i] && t_maps.key[i] == key) {
      *map = t_maps.map[i];
      return FFA_OK;
    }
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return set_error(FFA_ERR_LAUNCH, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(BH)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(stride_s) * 2, static_cast<cuuint64_t>(stride_bh) * 2};
  const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_rows), 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[96];
    std::snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
    return set_error(FFA_ERR_INVALID, buf);
  }
  const int slot = t_maps.next;
  t_maps.next = (slot + 1) % MapCache::N;
  t_maps.key[slot] = key;
  t_maps.map[slot] = *map;
  t_maps.used[slot] = true;
  return FFA_OK;
}

int set_smem_once(const void* kernel, int bytes, unsigned long long* done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_error(FFA_ERR_LAUNCH, "cudaGetDevice failed");
  const unsigned long long bit = 1ull << (dev & 63);
  if (__atomic_load_n(done, __ATOMIC_ACQUIRE) & bit) return FFA_OK;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return set_error(FFA_ERR_LAUNCH, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize) failed");
  __atomic_fetch_or(done, bit, __ATOMIC_ACQ_REL);
  return FFA_OK;
}

// ------------------------------------------------------------------------------------
// Fixed scratch of ffa_bwd_noalloc.  The backward needs one fp32 per (slice, row) for
// delta = rowsum(O * dO).  Callers that cannot allocate device memory get it from this
// file-scope array instead; it is part of the library image, so every GPU that loads
// the library holds its 16 MiB until the process exits.  Host code must not use the
// array's name as a device address: the device address is looked up per device with
// cudaGetSymbolAddress (noalloc_delta_ptr below).
// ------------------------------------------------------------------------------------
constexpr long long kNoAllocDeltaRows = 4ll << 20;  // 4,194,304 rows = 16 MiB of fp32
static __device__ __align__(256) float g_noalloc_delta[kNoAllocDeltaRows];

namespace {
std::mutex g_noalloc_mu;
float* g_noalloc_delta_dev[64] = {};  // device address of g_noalloc_delta, per device ordinal
}  // namespace

// Device address of g_noalloc_delta on the current device, looked up on the first call
// for that device (which therefore must not happen inside a stream capture).
static int noalloc_delta_ptr(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_error(FFA_ERR_LAUNCH, "cudaGetDevice failed");
  if (dev < 0 || dev >= 64) return set_error(FFA_ERR_UNSUPPORTED, "device ordinal >= 64");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_delta_dev[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_delta);
    if (e != cudaSuccess || p == nullptr) {
      char buf[160];
      std::snprintf(buf, sizeof(buf), "cudaGetSymbolAddress(no-alloc scratch) failed: %s", cudaGetErrorString(e));
      return set_error(FFA_ERR_LAUNCH, buf);
    }
    g_noalloc_delta_dev[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_delta_dev[dev];
  return FFA_OK;
}

int check_launch_regs(const void* kernel, int needed) {
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, kernel) != cudaSuccess) return set_error(FFA_ERR_LAUNCH, "cudaFuncGetAttributes failed");
  if (fa.numRegs < needed)
    return set_error(FFA_ERR_LAUNCH, "kernel compiled with too few registers for its setmaxnreg split");
  return FFA_OK;
}

// Shape / stride / alignment checks shared by the entry points.
static int check_common(int BH, int S, int D, long long stride_bh, long long stride_s) {
  if (BH < 0 || S < 0) return set_error(FFA_ERR_INVALID, "BH and S must be non-negative");
  if (D != 64 && D != 128) return set_error(FFA_ERR_UNSUPPORTED, "kernel head_dim must be 64 or 128");
  if (stride_s < D || stride_s % 8 != 0) return set_error(FFA_ERR_INVALID, "stride_s must be >= D and a multiple of 8");
  if (BH > 1 && (stride_bh < static_cast<long long>(S) * stride_s || stride_bh % 8 != 0))
    return set_error(FFA_ERR_INVALID, "stride_bh must be >= S*stride_s and a multiple of 8");
  // the kernels run one CTA per 128-row block of every slice in a 1-D grid
  if ((static_cast<long long>(S) + 127) / 128 * BH > 2147483647LL)
    return set_error(FFA_ERR_UNSUPPORTED, "BH * ceil(S/128) exceeds the grid limit of 2^31-1 CTAs");
  return FFA_OK;
}

}  // namespace ffa

using namespace ffa;

extern "C" {

int ffa_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int BH, int S, int D,
            long long stride_bh, long long stride_s, double scale, int causal, void* stream) {
  int rc = check_common(BH, S, D, stride_bh, stride_s);
  if (rc) return rc;
  if (BH == 0 || S == 0) return FFA_OK;
  if (!q || !k || !v || !o) return set_error(FFA_ERR_INVALID, "null tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return set_error(FFA_ERR_INVALID, "tensor pointers must be 16-byte aligned");
  if ((rc = ensure_context()) != FFA_OK) return rc;
  FwdArgs a{q, k, v, o, lse, BH, S, D, stride_bh, stride_s, scale, causal};
  return launch_fwd(a, static_cast<cudaStream_t>(stream));
}

int ffa_fwd_merge(const void* q, const void* k, const void* v, float* acc, float* acc_lse, int BH, int S, int D,
                  long long stride_bh, long long stride_s, double scale, int causal, int first, void* stream) {
  int rc = check_common(BH, S, D, stride_bh, stride_s);
  if (rc) return rc;
  if (BH == 0 || S == 0) return FFA_OK;
  if (!q || !k || !v || !acc || !acc_lse) return set_error(FFA_ERR_INVALID, "null tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(acc))
    return set_error(FFA_ERR_INVALID, "tensor pointers must be 16-byte aligned");
  if ((rc = ensure_context()) != FFA_OK) return rc;
  FwdArgs a{q, k, v, nullptr, nullptr, BH, S, D, stride_bh, stride_s, scale, causal, acc, acc_lse, first ? 1 : 0};
  return launch_fwd(a, static_cast<cudaStream_t>(stream));
}

int ffa_bwd_preprocess(const void* o, const void* dout, float* delta, int BH, int S, int D, long long stride_bh,
                       long long stride_s, void* stream) {
  int rc = check_common(BH, S, D, stride_bh, stride_s);
  if (rc) return rc;
  if (BH == 0 || S == 0) return FFA_OK;
  if (!o || !dout || !delta) return set_error(FFA_ERR_INVALID, "null tensor pointer");
  if (!aligned16(o) || !aligned16(dout)) return set_error(FFA_ERR_INVALID, "tensor pointers must be 16-byte aligned");
  if ((rc = ensure_context()) != FFA_OK) return rc;
  return launch_preprocess(o, dout, delta, BH, S, D, stride_bh, stride_s, static_cast<cudaStream_t>(stream));
}

int ffa_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout, const float* lse,
            float* delta_ws, void* dq, void* dk, void* dv, int BH, int S, int D, long long stride_bh,
            long long stride_s, double scale, int causal, void* stream) {
  int rc = check_common(BH, S, D, stride_bh, stride_s);
  if (rc) return rc;
  if (BH == 0 || S == 0) return FFA_OK;
  if (!q || !k || !v || !o || !dout || !lse || !delta_ws || !dq || !dk || !dv)
    return set_error(FFA_ERR_INVALID, "null tensor pointer");
  for (const void* p : {q, k, v, o, dout, static_cast<const void*>(dq), static_cast<const void*>(dk),
                        static_cast<const void*>(dv)})
    if (!aligned16(p)) return set_error(FFA_ERR_INVALID, "tensor pointers must be 16-byte aligned");
  if ((rc = ensure_context()) != FFA_OK) return rc;
  BwdArgs a{q, k, v, o, dout, lse, delta_ws, dq, dk, dv, BH, S, D, stride_bh, stride_s, scale, causal};
  return launch_bwd(a, static_cast<cudaStream_t>(stream));
}

// Same backward as ffa_bwd, with delta kept in the library's fixed device scratch
// instead of a caller-provided buffer; it allocates nothing.  Calls that overlap on the
// GPU (other streams, other threads) share that scratch and race; serialise them.
int ffa_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const void* dout, const float* lse,
                    void* dq, void* dk, void* dv, int BH, int S, int D, long long stride_bh, long long stride_s,
                    double scale, int causal, void* stream) {
  int rc = check_common(BH, S, D, stride_bh, stride_s);
  if (rc) return rc;
  if (static_cast<long long>(BH) * S > kNoAllocDeltaRows)
    return set_error(FFA_ERR_INVALID, "ffa_bwd_noalloc: BH*S exceeds its fixed scratch of 4194304 rows");
  if (BH == 0 || S == 0) return FFA_OK;
  if (!q || !k || !v || !o || !dout || !lse || !dq || !dk || !dv)
    return set_error(FFA_ERR_INVALID, "null tensor pointer");
  for (const void* p : {q, k, v, o, dout, static_cast<const void*>(dq), static_cast<const void*>(dk),
                        static_cast<const void*>(dv)})
    if (!aligned16(p)) return set_error(FFA_ERR_INVALID, "tensor pointers must be 16-byte aligned");
  if ((rc = ensure_context()) != FFA_OK) return rc;
  float* delta = nullptr;
  if ((rc = noalloc_delta_ptr(&delta)) != FFA_OK) return rc;
  // delta is fully rewritten by the preprocess kernel before it is read: nothing to clear
  BwdArgs a{q, k, v, o, dout, lse, delta, dq, dk, dv, BH, S, D, stride_bh, stride_s, scale, causal};
  return launch_bwd(a, static_cast<cudaStream_t>(stream));
}

// Shared validation of the split backward entry points (lse and delta are inputs).
static int bwd_part(const void* q, const void* k, const void* v, const void* dout, const float* lse,
                    const float* delta, void* dq, void* dk, void* dv, int BH, int S, int D, long long stride_bh,
                    long long stride_s, double scale, int causal, void* stream, bool dkdv) {
  int rc = check_common(BH, S, D, stride_bh, stride_s);
  if (rc) return rc;
  if (BH == 0 || S == 0) return FFA_OK;
  if (!q || !k || !v || !dout || !lse || !delta || (dkdv ? (!dk || !dv) : !dq))
    return set_error(FFA_ERR_INVALID, "null tensor pointer");
  for (const void* p : {q, k, v, dout, static_cast<const void*>(dkdv ? dk : dq), static_cast<const void*>(dkdv ? dv : dq)})
    if (!aligned16(p)) return set_error(FFA_ERR_INVALID, "tensor pointers must be 16-byte aligned");
  if ((rc = ensure_context()) != FFA_OK) return rc;
  BwdArgs a{q, k, v, nullptr, dout, lse, const_cast<float*>(delta), dq, dk, dv, BH, S, D, stride_bh, stride_s, scale,
            causal};
  return dkdv ? launch_dkdv(a, static_cast<cudaStream_t>(stream)) : launch_dq(a, static_cast<cudaStream_t>(stream));
}

int ffa_bwd_dkdv(const void* q, const void* k, const void* v, const void* dout, const float* lse, const float* delta,
                 void* dk, void* dv, int BH, int S, int D, long long stride_bh, long long stride_s, double scale,
                 int causal, void* stream) {
  return bwd_part(q, k, v, dout, lse, delta, nullptr, dk, dv, BH, S, D, stride_bh, stride_s, scale, causal, stream,
                  true);
}

int ffa_bwd_dq(const void* q, const void* k, const void* v, const void* dout, const float* lse, const float* delta,
               void* dq, int BH, int S, int D, long long stride_bh, long long stride_s, double scale, int causal,
               void* stream) {
  return bwd_part(q, k, v, dout, lse, delta, dq, nullptr, nullptr, BH, S, D, stride_bh, stride_s, scale, causal,
                  stream, false);
}

int ffa_bwd_dkdv_acc(const void* q, const void* k, const void* v, const void* dout, const float* lse,
                     const float* delta, float* dk_acc, float* dv_acc, int BH, int S, int D, long long stride_bh,
                     long long stride_s, double scale, int causal, void* stream) {
  if (!dk_acc || !dv_acc) return set_error(FFA_ERR_INVALID, "null tensor pointer");
  if (!aligned16(dk_acc) || !aligned16(dv_acc)) return set_error(FFA_ERR_INVALID, "accumulators must be 16-byte aligned");
  int rc = check_common(BH, S, D, stride_bh, stride_s);
  if (rc) return rc;
  if (BH == 0 || S == 0) return FFA_OK;
  if (!q || !k || !v || !dout || !lse || !delta) return set_error(FFA_ERR_INVALID, "null tensor pointer");
  for (const void* p : {q, k, v, dout})
    if (!aligned16(p)) return set_error(FFA_ERR_INVALID, "tensor pointers must be 16-byte aligned");
  if ((rc = ensure_context()) != FFA_OK) return rc;
  BwdArgs a{q, k, v, nullptr, dout, lse, const_cast<float*>(delta), nullptr, nullptr, nullptr, BH, S, D, stride_bh,
            stride_s, scale, causal, nullptr, dk_acc, dv_acc};
  return launch_dkdv(a, static_cast<cudaStream_t>(stream));
}

int ffa_bwd_dq_acc(const void* q, const void* k, const void* v, const void* dout, const float* lse, const float* delta,
                   float* dq_acc, int BH, int S, int D, long long stride_bh, long long stride_s, double scale,
                   int causal, void* stream) {
  if (!dq_acc) return set_error(FFA_ERR_INVALID, "null tensor pointer");
  if (!aligned16(dq_acc)) return set_error(FFA_ERR_INVALID, "accumulators must be 16-byte aligned");
  int rc = check_common(BH, S, D, stride_bh, stride_s);
  if (rc) return rc;
  if (BH == 0 || S == 0) return FFA_OK;
  if (!q || !k || !v || !dout || !lse || !delta) return set_error(FFA_ERR_INVALID, "null tensor pointer");
  for (const void* p : {q, k, v, dout})
    if (!aligned16(p)) return set_error(FFA_ERR_INVALID, "tensor pointers must be 16-byte aligned");
  if ((rc = ensure_context()) != FFA_OK) return rc;
  BwdArgs a{q, k, v, nullptr, dout, lse, const_cast<float*>(delta), nullptr, nullptr, nullptr, BH, S, D, stride_bh,
            stride_s, scale, causal, dq_acc, nullptr, nullptr};
  return launch_dq(a, static_cast<cudaStream_t>(stream));
}

int ffa_lse_merge(float* acc, float* acc_lse, const void* part, const float* part_lse, long long rows, int D,
                  int first, void* stream) {
  if (rows < 0 || D <= 0 || D > 128 || D % 4 != 0) return set_error(FFA_ERR_INVALID, "bad rows / D for merge");
  if (rows == 0) return FFA_OK;
  if (!acc || !acc_lse || !part || !part_lse) return set_error(FFA_ERR_INVALID, "null tensor pointer");
  if (!aligned16(acc) || (reinterpret_cast<uintptr_t>(part) & 7u))
    return set_error(FFA_ERR_INVALID, "acc must be 16-byte and part 8-byte aligned");
  const int rc = ensure_context();
  if (rc != FFA_OK) return rc;
  return launch_lse_merge(acc, acc_lse, part, part_lse, rows, D, first, static_cast<cudaStream_t>(stream));
}

int ffa_last_error(char* buf, int n) {
  if (buf && n > 0) {
    std::strncpy(buf, t_last_msg, static_cast<size_t>(n - 1));
    buf[n - 1] = '\0';
  }
  return t_last_code;
}

int ffa_device_status(unsigned int* out4) {
  if (!out4) return set_error(FFA_ERR_INVALID, "null output");
  if (cudaDeviceSynchronize() != cudaSuccess) return set_error(FFA_ERR_LAUNCH, "cudaDeviceSynchronize failed");
  unsigned int host[4] = {0, 0, 0, 0};
  if (cudaMemcpyFromSymbol(host, g_status, sizeof(host)) != cudaSuccess)
    return set_error(FFA_ERR_LAUNCH, "reading the device status word failed");
  const unsigned int zero[4] = {0, 0, 0, 0};
  if (cudaMemcpyToSymbol(g_status, zero, sizeof(zero)) != cudaSuccess)
    return set_error(FFA_ERR_LAUNCH, "clearing the device status word failed");
  std::memcpy(out4, host, sizeof(host));
  if (host[0] != 0 || host[1] != 0 || host[2] != 0) {
    char buf[128];
    std::snprintf(buf, sizeof(buf), "device wait timeout: site 0x%x, %u waits, %u drains", host[0], host[1], host[2]);
    return set_error(FFA_ERR_DEVICE, buf);
  }
  return FFA_OK;
}

const char* ffa_version(void) { return "0.2.0+sm100a"; }

}  // extern "C"

namespace ffa {

int launch_preprocess(const void* o, const void* dout, float* delta, int BH, int S, int D, long long stride_bh,
                      long long stride_s, cudaStream_t stream) {
  const long long rows = static_cast<long long>(BH) * S;
  const int rows_per_block = 256 / (D / 8);
  const long long blocks = (rows + rows_per_block - 1) / rows_per_block;
  const int grid = static_cast<int>(blocks < 148 * 16 ? blocks : 148 * 16);
  if (D == 128)
    ffa_preprocess_kernel<128><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(o),
                                                          static_cast<const __nv_bfloat16*>(dout), delta, BH, S,
                                                          stride_bh, stride_s);
  else
    ffa_preprocess_kernel<64><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(o),
                                                         static_cast<const __nv_bfloat16*>(dout), delta, BH, S,
                                                         stride_bh, stride_s);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FFA_ERR_LAUNCH, cudaGetErrorString(e));
  return FFA_OK;
}

int launch_lse_merge(float* acc, float* acc_lse, const void* part, const float* part_lse, long long rows, int D,
                     int first, cudaStream_t stream) {
  const long long blocks = (rows + 7) / 8;
  const int grid = static_cast<int>(blocks < 148 * 16 ? blocks : 148 * 16);
  ffa_lse_merge_kernel<<<grid, 256, 0, stream>>>(acc, acc_lse, static_cast<const __nv_bfloat16*>(part), part_lse,
                                                 rows, D, first);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FFA_ERR_LAUNCH, cudaGetErrorString(e));
  return FFA_OK;
}

}  // namespace ffa
