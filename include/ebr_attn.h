/*
 * ebr_attn.h: C ABI of the B200 (sm_100a) second-order attention kernels.
 *
 * Non-causal multi-head softmax attention on [B, H, N, D] tensors, with its backward and the backward of the
 * backward, the three passes behind the reference's fused attention op chain
 *     ebr_fused::attn_fwd -> ebr_fused::attn_bwd -> ebr_fused::attn_bwd_bwd
 * (wwillchen/ebr models/fused_attn/ops.py:65-120). Each entry point replaces one of the reference's Triton launchers in
 * models/fused_attn/triton_kernels.py and keeps its argument meaning:
 *
 *   ebr_attn_fwd      replaces triton_kernels.attn_fwd      (triton_kernels.py:696-728)
 *   ebr_attn_bwd      replaces triton_kernels.attn_bwd      (triton_kernels.py:731-839)
 *   ebr_attn_bwd_bwd  replaces triton_kernels.attn_bwd_bwd  (triton_kernels.py:842-968)
 *
 * Conventions (the reference's, triton_kernels.py:594-609):
 *   - q, k, v, dout and the cotangents gq, gk, gv may have any batch / head / token strides; the head-dim stride is 1.
 *   - o (the stored forward output) and lse are contiguous [B, H, N, D] / [B, H, N]; every output is written
 *     contiguous [B, H, N, D] (lse [B, H, N]).
 *   - lse is float32 (float64 for float64 inputs), the natural-log row logsumexp of scale * Q K^T.
 *   - scale is rounded once to the compute type (float32; float64 for float64 inputs) and used for both the logits
 *     and the gradients (triton_kernels.py:689-693).
 *   - A cotangent with data == NULL is zero (triton_kernels.py:868-873 expands a zero row instead).
 *
 * Ownership: the library never allocates device memory. The caller allocates outputs and the scratch buffer whose
 * size ebr_attn_*_scratch_bytes() reports (the row scalars of the two-pass kernels: B * H * N fp32 values, fp64 for
 * float64, three sets for the double backward), and passes a CUDA stream (cudaStream_t, NULL = legacy default
 * stream). Calls are asynchronous on that stream and reentrant.
 *
 * Errors: every entry point returns EBR_OK or an ebr_status code and never traps. Argument errors are detected on the
 * host before any launch. Device-side waits are bounded; a wait that runs out sets a device error word that
 * ebr_attn_device_status() reads back (a synchronizing call, for tests and debugging).
 */
#ifndef EBR_ATTN_H_
#define EBR_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types, the reference's supported set (triton_kernels.py:558-563). */
typedef enum ebr_dtype {
  EBR_FLOAT32 = 0,
  EBR_FLOAT16 = 1,
  EBR_BFLOAT16 = 2,
  EBR_FLOAT64 = 3,
} ebr_dtype;

typedef enum ebr_status {
  EBR_OK = 0,
  EBR_ERR_NULL = 1,          /* a required pointer is NULL */
  EBR_ERR_SHAPE = 2,         /* negative sizes, D outside [1, 256], B * H >= 2^31 or B * H * N >= 2^40 */
  EBR_ERR_DTYPE = 3,         /* unknown dtype */
  EBR_ERR_STRIDE = 4,        /* head-dim stride is not 1, or a stride is negative */
  EBR_ERR_SCRATCH = 5,       /* scratch missing or smaller than ebr_attn_*_scratch_bytes() */
  EBR_ERR_CUDA = 6,          /* a CUDA runtime call or a kernel launch failed (see ebr_attn_last_error) */
  EBR_ERR_DEVICE = 7,        /* the current device is not sm_100 */
  EBR_ERR_DEVICE_TIMEOUT = 8 /* a bounded device-side wait ran out (reported by ebr_attn_device_status) */
} ebr_status;

/* One strided [B, H, N, D] operand: device pointer to element [0, 0, 0, 0] and its batch / head / token strides in
 * elements. The head-dim stride is 1. */
typedef struct ebr_operand {
  const void* data;
  int64_t stride_b;
  int64_t stride_h;
  int64_t stride_n;
} ebr_operand;

/* Forward: o = softmax(scale q k^T) v and lse = logsumexp(scale q k^T) per row.
 * Replaces triton_kernels.attn_fwd (triton_kernels.py:696-728); oracle reference.attn_fwd (reference.py:32-36). */
int ebr_attn_fwd(int dtype, int64_t B, int64_t H, int64_t N, int64_t D, double scale,
                 const ebr_operand* q, const ebr_operand* k, const ebr_operand* v,
                 void* o, void* lse, void* stream);

/* Backward: (dq, dk, dv) of <dout, o>, with P recomputed from lse and D = rowsum(dout * o) from the stored o.
 * Replaces triton_kernels.attn_bwd (triton_kernels.py:731-839); oracle reference.attn_bwd (reference.py:50-58). */
size_t ebr_attn_bwd_scratch_bytes(int dtype, int64_t B, int64_t H, int64_t N, int64_t D);
int ebr_attn_bwd(int dtype, int64_t B, int64_t H, int64_t N, int64_t D, double scale,
                 const ebr_operand* q, const ebr_operand* k, const ebr_operand* v,
                 const void* o, const void* lse, const ebr_operand* dout,
                 void* dq, void* dk, void* dv, void* scratch, size_t scratch_bytes, void* stream);

/* Backward of the backward: (hq, hk, hv, hdout), the total derivative of <gq, dq> + <gk, dk> + <gv, dv> with
 * respect to (q, k, v, dout). dq (the first backward's output) is accepted for the op contract and not read, as in
 * the reference (reference.py:74). gq / gk / gv with data == NULL are zero.
 * Replaces triton_kernels.attn_bwd_bwd (triton_kernels.py:842-968); oracle reference.attn_bwd_bwd
 * (reference.py:61-91). */
size_t ebr_attn_bwd_bwd_scratch_bytes(int dtype, int64_t B, int64_t H, int64_t N, int64_t D);
int ebr_attn_bwd_bwd(int dtype, int64_t B, int64_t H, int64_t N, int64_t D, double scale,
                     const ebr_operand* q, const ebr_operand* k, const ebr_operand* v,
                     const void* o, const void* lse, const ebr_operand* dout, const void* dq,
                     const ebr_operand* gq, const ebr_operand* gk, const ebr_operand* gv,
                     void* hq, void* hk, void* hv, void* hdout, void* scratch, size_t scratch_bytes, void* stream);

/* Allocation-free variant of ebr_attn_bwd. No counterpart in the reference: it exists for callers that cannot
 * allocate device memory at call time, for example a host program whose GPU memory is handed out up front by another
 * allocator (a serving runtime with a fixed memory plan), or a plugin host that passes a plugin only its input and
 * output buffers and no workspace. Instead of a caller-provided scratch buffer it uses a built-in device buffer of
 * EBR_ATTN_NOALLOC_SCRATCH_BYTES (8 MiB), a static array that every GPU which loads the library holds until the
 * process exits. It calls no allocator of any kind.
 *   - Limit: the row scratch needs B*H*N*4 bytes (B*H*N*8 for float64), so B*H*N <= 2,097,152 rows (1,048,576 for
 *     float64). Larger calls return EBR_ERR_SCRATCH before any launch.
 *   - The first call in a CUDA context (the primary context of a device, or a context the caller created with the
 *     driver API) looks up the buffer's address in that context (cudaGetSymbolAddress) and remembers it for that
 *     context; make that first call before any stream capture. A context destroyed and re-created under the same
 *     handle (cudaDeviceReset) is not detected: after a device reset, reload the library.
 *   - All calls share the one buffer per device and it keeps the last call's contents (every value a call reads is
 *     written earlier in the same call). Calls whose executions overlap on the GPU (for example on two streams) race
 *     on it: serialize them.
 * Arguments and results are those of ebr_attn_bwd without scratch / scratch_bytes. */
#define EBR_ATTN_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)
int ebr_attn_bwd_noalloc(int dtype, int64_t B, int64_t H, int64_t N, int64_t D, double scale,
                         const ebr_operand* q, const ebr_operand* k, const ebr_operand* v,
                         const void* o, const void* lse, const ebr_operand* dout,
                         void* dq, void* dk, void* dv, void* stream);

/* Which kernel family a call with these arguments would use: 1 = tcgen05 tensor-core kernels, 0 = the CUDA-core
 * kernels (float32 / float64, and half types whose shape or strides the tensor-core path does not take). */
int ebr_attn_uses_tensor_cores(int dtype, int64_t D, const ebr_operand* q, const ebr_operand* k,
                               const ebr_operand* v);

/* Synchronizes the current device, returns EBR_OK or EBR_ERR_DEVICE_TIMEOUT if a bounded device wait ran out since
 * the last call, and clears the device error word. */
int ebr_attn_device_status(void);

/* Test support for the error path above, with no counterpart in the reference: launches one thread on `stream` that
 * waits, with a limit of `limit_ns` (1 us to 1 s), on a device barrier that nothing completes. The wait runs out and
 * sets the device error word, so the next ebr_attn_device_status() returns EBR_ERR_DEVICE_TIMEOUT (and clears it);
 * the context stays usable. */
int ebr_attn_test_bounded_wait(int64_t limit_ns, void* stream);

/* Human-readable text of a status code, and of the last CUDA error seen by this thread. */
const char* ebr_attn_status_string(int status);
const char* ebr_attn_last_error(void);

/* Kernel launches made by this process since load (all threads), for launch accounting in benchmarks. */
uint64_t ebr_attn_launch_count(void);

#ifdef __cplusplus
}
#endif

#endif /* EBR_ATTN_H_ */
