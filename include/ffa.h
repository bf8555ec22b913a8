/* ffa.h — C ABI of the B200 (sm_100a) exact bf16 attention library `libffa_sm100.so`.
 *
 * Every entry point takes plain device pointers, sizes and strides (in elements) and a
 * CUDA stream passed as `void*` (0 = legacy default stream).  No torch or C++ types cross
 * this boundary.  Tensors are bf16 unless stated; logical layout is [BH, S, D] with the
 * head dimension D contiguous (stride 1), rows `stride_s` elements apart and (batch*head)
 * slices `stride_bh` elements apart.  Each call returns FFA_OK (0) or an FFA_ERR_* code;
 * ffa_last_error() returns the message of the most recent failure on the calling thread.
 *
 * The kernels compute in bf16 with fp32 accumulation and handle D in {64, 128}
 * natively; smaller power-of-two head dims are zero-padded to 64 by the Python layer
 * (exact).  All kernels launch asynchronously on `stream`.
 */
#ifndef FFA_H_
#define FFA_H_

#ifdef __cplusplus
extern "C" {
#endif

#define FFA_OK 0
#define FFA_ERR_INVALID 1      /* bad pointer / size / stride / alignment */
#define FFA_ERR_UNSUPPORTED 2  /* head_dim or shape outside what the kernels handle */
#define FFA_ERR_LAUNCH 3       /* CUDA launch or driver error */
#define FFA_ERR_DEVICE 4       /* a kernel recorded a device-side wait timeout */

/* Forward.  Replaces the reference host launcher `fastflash_attn`
 * (fastflash_attention/_kernel.py:282-318) and its kernel `_fastflash_fwd` (:180-279).
 *   q, k, v  : [BH, S, D] bf16 inputs
 *   o        : [BH, S, D] bf16 output (same strides as q)
 *   lse      : [BH, S] fp32 base-2 log-sum-exp (m + log2 l), or NULL to skip it
 *              (the reference's RETURN_LSE=False path, :303)
 *   scale    : softmax scale; the kernel uses scale*log2(e) as the reference does (:304-305)
 *   causal   : nonzero for top-left-aligned causal masking (key j visible iff j <= i) */
int ffa_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int BH, int S, int D,
            long long stride_bh, long long stride_s, double scale, int causal, void* stream);

/* Forward of one block of a context-parallel ring, merged into a running result (no
 * reference counterpart: the reference has no sequence parallelism; this builds on the
 * base-2 LSE that `_fastflash_fwd` writes, _kernel.py:274-279).  Computes the attention of
 * q over this call's k, v exactly as ffa_fwd does, then folds it, in fp32 and without
 * rounding it to bf16, into
 *   acc     : [BH, S, D] fp32, rows D floats apart, slices S*D apart (16-byte aligned)
 *   acc_lse : [BH, S] fp32 base-2 LSE of acc
 * as acc = (2^acc_lse acc + 2^lse O) / (2^acc_lse + 2^lse), acc_lse = log2 of the
 * denominator.  `first` != 0 initialises acc and acc_lse instead (their contents are not
 * read).  Each row has one writer, so the result does not depend on scheduling. */
int ffa_fwd_merge(const void* q, const void* k, const void* v, float* acc, float* acc_lse, int BH, int S, int D,
                  long long stride_bh, long long stride_s, double scale, int causal, int first, void* stream);

/* Backward preprocess: delta[bh, i] = sum_d O[bh,i,d] * dO[bh,i,d] in fp32.
 * Replaces `_bwd_preprocess` / `_uni_bwd_preprocess` (_kernel.py:323-351). */
int ffa_bwd_preprocess(const void* o, const void* dout, float* delta, int BH, int S, int D,
                       long long stride_bh, long long stride_s, void* stream);

/* Full deterministic backward: preprocess, then dK/dV (key-block grid) and dQ
 * (query-block grid), each output tile written by exactly one CTA, no atomics.
 * Replaces `FastFlashAttn.backward` (_kernel.py:784-906) with its kernels
 * `_uni_bwd_dkdv` (:379-448) and `_uni_bwd_dq` (:487-564).
 * dQ runs on a side stream beside dK/dV; each (device, caller stream) pair gets its own
 * side stream and events on its first call (kept until exit), joined back with events,
 * so the call records correctly into a CUDA graph captured on `stream`.
 *   lse      : [BH, S] fp32 from ffa_fwd
 *   delta_ws : [BH, S] fp32 caller-provided workspace (receives delta)
 *   dq,dk,dv : [BH, S, D] bf16 outputs (same strides as q) */
int ffa_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout, const float* lse,
            float* delta_ws, void* dq, void* dk, void* dv, int BH, int S, int D, long long stride_bh,
            long long stride_s, double scale, int causal, void* stream);

/* ffa_bwd without any device allocation, for callers that cannot call cudaMalloc:
 * a framework whose allocator owns nearly all device memory (XLA/TensorFlow-style
 * preallocation, serving runtimes with a fixed memory pool), or code running where
 * allocating is not allowed.  No counterpart in the reference (its backward always
 * allocates through the torch caching allocator).
 * The caller still passes inputs and outputs; the fp32 delta workspace lives in a
 * fixed 16 MiB array inside the library (held on every GPU that loads the library
 * until the process exits), so BH*S must be <= 4194304 (else FFA_ERR_INVALID).
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress), and the first call on each (device, stream) pair creates
 * the backward's side stream and its two events (as ffa_bwd does); make those first
 * calls outside any stream capture.
 * All calls share the one array: calls that overlap on the GPU race — serialise them. */
int ffa_bwd_noalloc(const void* q, const void* k, const void* v, const void* o, const void* dout, const float* lse,
                    void* dq, void* dk, void* dv, int BH, int S, int D, long long stride_bh, long long stride_s,
                    double scale, int causal, void* stream);

/* The two gradient kernels of ffa_bwd, callable on their own (delta from
 * ffa_bwd_preprocess).  ffa_bwd_dkdv replaces `_bwd_dkdv` (_kernel.py:451-484, kernel
 * :379-448): grid over 128-key blocks, writes dk, dv.  ffa_bwd_dq replaces `_bwd_dq`
 * (_kernel.py:567-602, kernel :487-564, recompute path): grid over 128-query blocks,
 * writes dq.  Each output tile is written by exactly one CTA. */
int ffa_bwd_dkdv(const void* q, const void* k, const void* v, const void* dout, const float* lse, const float* delta,
                 void* dk, void* dv, int BH, int S, int D, long long stride_bh, long long stride_s, double scale,
                 int causal, void* stream);
int ffa_bwd_dq(const void* q, const void* k, const void* v, const void* dout, const float* lse, const float* delta,
               void* dq, int BH, int S, int D, long long stride_bh, long long stride_s, double scale, int causal,
               void* stream);

/* ffa_bwd_dkdv / ffa_bwd_dq that ADD their gradients, in fp32 and unrounded, into caller
 * accumulators instead of writing bf16 (the ring backward sums the blocks of one key or
 * query chunk there; the reference has no counterpart, see ffa_fwd_merge):
 *   dk_acc += scale * dS^T Q,  dv_acc += P^T dO,  dq_acc += scale * dS K
 * Accumulators are [BH, S, D] fp32, rows D floats apart, slices S*D apart, 16-byte
 * aligned.  Every accumulator row has exactly one writer per call, so repeated calls in a
 * fixed order give bitwise-reproducible sums. */
int ffa_bwd_dkdv_acc(const void* q, const void* k, const void* v, const void* dout, const float* lse,
                     const float* delta, float* dk_acc, float* dv_acc, int BH, int S, int D, long long stride_bh,
                     long long stride_s, double scale, int causal, void* stream);
int ffa_bwd_dq_acc(const void* q, const void* k, const void* v, const void* dout, const float* lse, const float* delta,
                   float* dq_acc, int BH, int S, int D, long long stride_bh, long long stride_s, double scale,
                   int causal, void* stream);

/* Merge of partial attention results for the context-parallel ring (no reference
 * counterpart: the reference has no sequence parallelism; it builds on the base-2 LSE
 * that `_fastflash_fwd` writes, _kernel.py:274-279).
 *   acc [rows, D] fp32, acc_lse [rows] fp32 : running result (updated in place)
 *   part [rows, D] bf16, part_lse [rows] fp32 : one partial result
 * acc = (2^acc_lse * acc + 2^part_lse * part) / (2^acc_lse + 2^part_lse), acc_lse = log2 of the
 * denominator.  `first` != 0 initialises acc from part. */
int ffa_lse_merge(float* acc, float* acc_lse, const void* part, const float* part_lse, long long rows, int D,
                  int first, void* stream);

/* Most recent error message of the calling thread ("" if none). Copies at most n-1
 * bytes into buf (NUL-terminated) and returns the last error code. */
int ffa_last_error(char* buf, int n);

/* Reads and clears the device status words of the current device:
 * out[0] = id of the first wait that timed out (0 = none), out[1] = number of timed-out
 * waits, out[2] = number of teardown drains that timed out.  Synchronises the device. */
int ffa_device_status(unsigned int* out4);

/* Library version string, e.g. "0.2.0+sm100a". */
const char* ffa_version(void);

#ifdef __cplusplus
}
#endif
#endif /* FFA_H_ */
