/* fa_b200.h -- C ABI of the B200 (sm_100a) FlashAttention-2 library.
 *
 * Plain pointers, sizes and a CUDA stream: no torch or C++ types cross this
 * boundary. Every tensor is dense row-major (contiguous), fp16 unless stated:
 *   q, o, dO, dq   (B, Hq,  N, D)
 *   k, v, dk, dv   (B, Hkv, N, D)
 *   lse            (B, Hq,  N)  fp32, natural log: lse = m + ln(sum exp(s - m))
 * with D in {64, 128}, N >= 1, Hq a multiple of Hkv (Hkv == Hq: MHA, 1: MQA,
 * otherwise GQA), scale fixed at 1/sqrt(D), and causal meaning key j is
 * visible to query i iff j <= i. All device pointers must be 16-byte aligned.
 *
 * Ownership: the caller allocates every buffer (outputs and workspace); the
 * library allocates no device memory. Work is enqueued on `stream` (a
 * cudaStream_t; NULL = legacy default stream) and the calls return before it
 * finishes. Calls are thread-safe.
 *
 * Every entry point returns an int status (FA_B200_OK = 0). Argument errors
 * are reported before anything is launched.
 */
#ifndef FA_B200_H_
#define FA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  FA_B200_OK = 0,
  FA_B200_ERR_NULL_POINTER = 1,    /* a required pointer is NULL */
  FA_B200_ERR_HEAD_DIM = 2,        /* D not in {64, 128} */
  FA_B200_ERR_SHAPE = 3,           /* N < 1, B < 1, Hkv < 1, or Hq % Hkv != 0 */
  FA_B200_ERR_ALIGNMENT = 4,       /* a device pointer is not 16-byte aligned */
  FA_B200_ERR_TENSOR_MAP = 5,      /* cuTensorMapEncodeTiled rejected a tensor */
  FA_B200_ERR_LAUNCH = 6,          /* a kernel launch failed (cudaGetLastError) */
  FA_B200_ERR_WORKSPACE = 7,       /* workspace missing or smaller than required */
  FA_B200_ERR_DEVICE = 8,          /* current device is not compute capability 10.x */
  FA_B200_ERR_TOO_LARGE = 9,       /* a grid dimension would exceed CUDA limits */
  FA_B200_ERR_SCRATCH_LIMIT = 10,  /* B*Hq*roundup(N,128) above fa_b200_backward_noalloc_max_rows() */
  FA_B200_ERR_DTYPE = 11,          /* dtype is not one of FA_B200_DTYPE_* */
  FA_B200_ERR_UNCHECKED_BUILD = 12 /* fa_b200_debug_tma_check on a release build */
};

/* Element type of the 16-bit tensors (q, k, v, o, dO, dk, dv, a 16-bit dq) of
 * the strided entry points; the others take fp16, the reference's only type.
 * Products are exact and accumulate in fp32 either way. */
enum {
  FA_B200_DTYPE_FP16 = 0,
  FA_B200_DTYPE_BF16 = 1
};

/* Forward. Replaces fa_forward (reference fa_p100_ext.cu:53-83) and
 * flash::launch (flash_fwd.cuh:342-355): writes o and lse.
 * `full_precision` is accepted for API compatibility (fa_p100_ext.cu:53) and
 * has no effect: the tensor-core MMAs multiply fp16 exactly and accumulate in
 * fp32, which is the reference's fp32-MAC tier. */
int fa_b200_forward(const void* q, const void* k, const void* v, void* o, float* lse,
                    int B, int Hq, int Hkv, int N, int D, int causal, int full_precision,
                    void* stream);

/* Element strides of a (B, H, N, D) tensor whose D axis is contiguous: the
 * element (b, h, n, d) sits at b*batch + h*head + n*row + d. Every stride must
 * be non-negative and a multiple of 16 bytes (8 fp16 or 4 fp32 elements). */
typedef struct fa_b200_strides {
  int64_t batch, head, row;
} fa_b200_strides;

/* fa_b200_forward in fp16 or bf16 (`dtype`, FA_B200_DTYPE_*) on tensors of any
 * strided (B, H, N, D) layout with D contiguous, e.g. (B, H, N, D) views of (B, N, H, D) storage as attention
 * layers produce them, so the caller needs no contiguous copies; o may be
 * strided too (lse stays (B, Hq, N) contiguous). The reference takes only
 * contiguous tensors and copies (fa_p100_ext.cu:56); no counterpart there. */
int fa_b200_forward_strided(const void* q, fa_b200_strides sq, const void* k, fa_b200_strides sk,
                            const void* v, fa_b200_strides sv, void* o, fa_b200_strides so,
                            float* lse, int B, int Hq, int Hkv, int N, int D, int dtype,
                            int causal, int full_precision, void* stream);

/* Bytes of device workspace fa_b200_backward needs: per query row the row sum
 * Dv = rowsum(dO o O) (the reference's dvec, fa_p100_ext.cu:124) and the
 * log2-scaled LSE (both stored negated and pre-scaled), each head padded to
 * roundup(N, 128) rows: 2 * 4 * B * Hq * roundup(N, 128) bytes. */
size_t fa_b200_backward_workspace_bytes(int B, int Hq, int N);

/* Workspace that also lets the fused backward split a GQA group over several
 * CTAs when B * Hkv * ceil(N/128) is too small to fill the GPU (MQA, short
 * sequences), or when equal-length CTAs would leave a last wave mostly empty
 * (a replay of the CTA dispatch decides): fa_b200_backward_workspace_bytes(B,
 * Hq, N) plus fp32 dK and dV accumulators, 2 * 4 * B * Hkv * N * D bytes. Any
 * backward given at least this much may split; given less it does not. A split
 * backward adds dK/dV partials in fp32 like dQ, so their last bits too depend
 * on the add order. No counterpart in the reference, whose dK/dV are owned by
 * one block each (flash_bwd.cuh:448-463). */
size_t fa_b200_backward_workspace_bytes_gqa(int B, int Hq, int Hkv, int N, int D);

/* The fused backward's schedule for a shape on the current device, as
 * fa_b200_backward (dq_fp32 != 0, not accumulating) given workspace_bytes of
 * workspace would launch it: *gsplit CTAs share each GQA group (1: unsplit;
 * above 1 the backward also zeroes an fp32 dK/dV accumulator and launches a
 * conversion kernel after the fused one) and *head_group (batch, kv-head)
 * slices are scheduled together. Launches nothing. Status codes as
 * fa_b200_backward for the shape and device checks. No counterpart in the
 * reference, whose grid is fixed (flash_bwd.cuh:476-483). */
int fa_b200_backward_plan(int B, int Hq, int Hkv, int N, int D, int causal, size_t workspace_bytes,
                          int* gsplit, int* head_group);

/* Backward. Replaces fa_backward (reference fa_p100_ext.cu:103-142) and
 * flash_bwd::launch (flash_bwd.cuh:466-484). Writes dq, dk and dv (fp16).
 * dq_fp32 != 0 (dq fp32, as the reference returns it): stages ROWSUM | FUSED --
 * one kernel for dK, dV and dQ, dQ added into the zeroed fp32 dq by TMA
 * reduce-adds, so like the reference's atomicAdd (flash_bwd.cuh:442) the last
 * bits of dq depend on the add order. dq_fp32 == 0 (dq fp16): stages ALL --
 * separate dK/dV and dQ kernels, each output row owned by one CTA, bitwise
 * deterministic. */
int fa_b200_backward(const void* q, const void* k, const void* v, const void* dO, const void* o,
                     const float* lse, void* dq, int dq_fp32, void* dk, void* dv, void* workspace,
                     size_t workspace_bytes, int B, int Hq, int Hkv, int N, int D, int causal,
                     void* stream);

/* Folds an attention result over a further set of keys into a running one,
 * in place: with o/lse the fp32 output and natural-log LSE so far and
 * o_part/lse_part (16-bit `dtype` output and its LSE) the same queries'
 * attention over other keys,
 *   lse <- logaddexp(lse, lse_part),
 *   o   <- o e^(lse_old - lse) + o_part e^(lse_part - lse).
 * Rows whose two LSEs are both -inf are left unchanged. The step that combines
 * the pieces of context-parallel (ring) attention; one pass over the rows.
 * o (float, strides in floats) and o_part are (B, H, N, D) with D contiguous
 * (D 64 or 128), 16-byte aligned bases and strides; lse and lse_part are
 * (B, H, N) with any strides. No counterpart in the reference, which has no
 * multi-GPU attention. */
int fa_b200_merge_partial(float* o, fa_b200_strides so, float* lse, fa_b200_strides slse,
                          const void* o_part, fa_b200_strides sop, const float* lse_part,
                          fa_b200_strides slp, int B, int H, int N, int D, int dtype,
                          void* stream);

/* Stages of the backward, for fa_b200_backward_stages. */
enum {
  FA_B200_STAGE_ROWSUM = 1,  /* Dv = rowsum(dO o O) into the workspace; also zeroes an
                              * fp32 dq (the FUSED stage accumulates into it) */
  FA_B200_STAGE_DKDV = 2,    /* dK, dV (reads the workspace) */
  FA_B200_STAGE_DQ = 4,      /* dQ (reads the workspace) */
  FA_B200_STAGE_ALL = 7,      /* ROWSUM | DKDV | DQ: the deterministic set */
  FA_B200_STAGE_FUSED = 8,    /* dK, dV and dQ in one kernel, dQ added by TMA reduce-adds
                               * into a zeroed fp32 dq (the reference's accumulate-into-
                               * fp32 scheme); needs dq_fp32 and a prior ROWSUM stage
                               * (which zeroes dq); excludes DKDV and DQ. Not bitwise
                               * deterministic; the default for dq_fp32 != 0 */
  FA_B200_STAGE_ACCUMULATE = 16 /* with FUSED (and dq_fp32): add this call's gradients to
                               * the contents of dq, dk and dv instead of overwriting
                               * them -- ROWSUM does not zero dq, and dk, dv are fp32
                               * accumulators (float*, strides in floats) that dK and
                               * dV are added into by TMA reduce-adds. For callers that
                               * sum gradients over several calls (context-parallel
                               * rings, chunked sequences). */
};

/* fa_b200_backward restricted to the stages in `stages`. The dK/dV and dQ
 * stages only read the row sums, so once FA_B200_STAGE_ROWSUM has run they may
 * be enqueued on two streams and overlap. fa_b200_backward(...) is
 * fa_b200_backward_stages(..., ROWSUM | FUSED or ALL as described there,
 * stream). No counterpart in the reference, whose backward is one launcher
 * (flash_bwd.cuh:466-484). */
int fa_b200_backward_stages(const void* q, const void* k, const void* v, const void* dO,
                            const void* o, const float* lse, void* dq, int dq_fp32, void* dk,
                            void* dv, void* workspace, size_t workspace_bytes, int B, int Hq,
                            int Hkv, int N, int D, int causal, int stages, void* stream);

/* fa_b200_backward_stages in fp16 or bf16 (`dtype`) on strided tensors (see
 * fa_b200_strides): q, k, v,
 * dO, o read and dq (fp32 or fp16), dk, dv written in their own layouts; lse
 * and the workspace are contiguous. stages == 0 selects the default for the dq
 * dtype. No counterpart in the reference (fa_p100_ext.cu:107-108 copies). */
int fa_b200_backward_strided(const void* q, fa_b200_strides sq, const void* k, fa_b200_strides sk,
                             const void* v, fa_b200_strides sv, const void* dO,
                             fa_b200_strides sdo, const void* o, fa_b200_strides so,
                             const float* lse, void* dq, fa_b200_strides sdq, int dq_fp32,
                             void* dk, fa_b200_strides sdk, void* dv, fa_b200_strides sdv,
                             void* workspace, size_t workspace_bytes, int B, int Hq, int Hkv,
                             int N, int D, int dtype, int causal, int stages, void* stream);

/* Backward that allocates nothing and takes no workspace. No counterpart in
 * the reference. For callers that cannot hand the library device memory of
 * its own: a host whose device memory is owned entirely by another allocator
 * (a framework's caching pool, an engine that only passes its plugins the
 * tensors of the op) or a serving loop that must not call cudaMalloc, whose
 * implicit synchronisation would stall every stream on the device.
 * Same inputs, outputs and results as fa_b200_backward given the per-row
 * workspace only (fa_b200_backward_workspace_bytes): in particular it never
 * splits a GQA/MQA group over several CTAs, which fa_b200_backward does for
 * small grids when given fa_b200_backward_workspace_bytes_gqa bytes -- at an
 * MQA shape such as B=2, Hq=16, Hkv=1, N=1537 the unsplit backward is several
 * times slower. The per-row workspace
 * goes to a 16 MiB array compiled into the library (resident on every GPU that
 * loads it until the process exits), so B*Hq*roundup(N,128) may be at most
 * fa_b200_backward_noalloc_max_rows() = 2,097,152 (FA_B200_ERR_SCRATCH_LIMIT
 * otherwise). The first call on a device looks up that array's device address
 * (and does the library's one-time device set-up); make that first call before
 * any stream capture. Every call on a device shares the one array: calls whose
 * backward passes overlap on the GPU (different streams, or different host
 * threads) race on it and must be serialised by the caller. Nothing in it has
 * to start at zero: each call writes every workspace entry it reads. The
 * looked-up address (like the rest of the library's per-device state) belongs
 * to the device's primary context: after cudaDeviceReset the library must be
 * reloaded before it is used on that device again. */
int fa_b200_backward_noalloc(const void* q, const void* k, const void* v, const void* dO,
                             const void* o, const float* lse, void* dq, int dq_fp32, void* dk,
                             void* dv, int B, int Hq, int Hkv, int N, int D, int causal,
                             void* stream);

/* Largest B*Hq*roundup(N,128) fa_b200_backward_noalloc accepts. */
size_t fa_b200_backward_noalloc_max_rows(void);

/* Codes of the device error word (fa_b200_device_error). A kernel whose
 * bounded internal wait gives up records the first code, stops its CTA without
 * writing the rest of that CTA's outputs, and leaves the CUDA context usable:
 * the outputs of that call are incomplete. */
enum {
  FA_B200_DEVERR_NONE = 0,
  FA_B200_DEVERR_TIMEOUT_LOAD = 1,      /* a TMA producer waited too long for a free slot */
  FA_B200_DEVERR_TIMEOUT_MMA = 2,       /* the MMA issuer waited too long for an operand */
  FA_B200_DEVERR_TIMEOUT_COMPUTE = 3,   /* softmax / gradient warps waited too long for an MMA */
  FA_B200_DEVERR_TIMEOUT_EPILOGUE = 4,  /* an epilogue / read-out waited too long */
  FA_B200_DEVERR_SMEM_ALIGN = 5,        /* dynamic shared memory not 1024-byte aligned */
  FA_B200_DEVERR_SELFTEST = 6           /* fa_b200_selftest_wait's deliberate timeout */
};

/* Reads the device error word the kernels set when a bounded internal wait
 * gives up (FA_B200_DEVERR_*; 0 = none) on `device`, and clears it when
 * `reset` != 0. Synchronises that device. Returns -1 if the read itself fails.
 * Has no counterpart in the reference, whose kernels have no waits; it plays
 * the part of the reference's AT_CUDA_CHECK after each launch
 * (fa_p100_ext.cu:81, :140) for failures that happen inside a kernel. */
int fa_b200_device_error(int device, int reset);

/* Enqueues on `stream` a copy of the current device's error word into
 * *host_word, without synchronising: the caller reads it once the stream has
 * passed that point (an event recorded after this call). host_word should be
 * page-locked host memory (cudaHostAlloc / a pinned tensor); pageable memory
 * makes the copy synchronous. Lets a framework binding check every call for a
 * kernel that gave up a wait at no synchronisation cost. No counterpart in the
 * reference. */
int fa_b200_device_error_async(int* host_word, void* stream);

/* Checked builds only (compiled with -DFAB_CHECK_TMA: FA_B200_DEBUG=1 when
 * building, libfa_b200_debug.so): every TMA copy first checks its innermost
 * coordinate (a non-negative multiple of 16 bytes), that a store or reduce-add
 * starts at no negative coordinate, and its shared-memory alignment; the first
 * violation on a device is recorded and that copy skipped, so the kernel ends
 * through its bounded waits instead of the copy faulting. Writes the record for
 * `device` to *word (0 = none; else op << 60 | smem misaligned << 59 |
 * (inner coordinate & 0xffff) << 32 | (row coordinate & 0xffffffff), op 1 load,
 * 2 L2 prefetch, 3 store, 4 reduce-add, 5 untiled load) and clears it when
 * `reset` != 0; synchronises that device. Returns FA_B200_ERR_UNCHECKED_BUILD
 * from a release build. It stands in for compute-sanitizer, which the GPU pool
 * this was built on does not allow; no counterpart in the reference, whose
 * kernels issue no TMA copies. */
int fa_b200_debug_tma_check(int device, unsigned long long* word, int reset);

/* Failure-detection self-test, no counterpart in the reference: one thread
 * waits on a shared-memory barrier that nothing ever arrives on, with the same
 * bounded wait every kernel uses but a limit of `limit_ns` nanoseconds
 * (clamped to [1 us, 1 s]); when it gives up it records FA_B200_DEVERR_SELFTEST
 * in the device error word (if the word is still clear) and returns. Nothing
 * else is touched, so the context stays usable. */
int fa_b200_selftest_wait(long long limit_ns, void* stream);

/* Human-readable text for a status code. */
const char* fa_b200_status_string(int status);

/* Detail of the most recent failure on the calling host thread (for example
 * the CUresult and arguments of a rejected tensor map); "" if none. No
 * counterpart in the reference, whose errors are TORCH_CHECK messages. */
const char* fa_b200_last_error(void);

/* Layout self-test, no counterpart in the reference: c (128x128 fp32) =
 * A * B^T for one 128x128x128 fp16 tile through the same TMA swizzle, shared-
 * memory descriptors and tcgen05 MMA the attention kernels use. a_mn / b_mn
 * select MN-major operands (a given as [K][M], b as [K][N]); otherwise a is
 * [M][K] and b is [N][K]. a_by_threads = 1 stages A in shared memory with
 * thread stores (the path P and dS take) instead of TMA; 2 stores A into
 * tensor memory with tcgen05.st and issues the A-from-TMEM form of the MMA. */
int fa_b200_selftest_gemm(const void* a, const void* b, float* c, int a_mn, int b_mn,
                          int a_by_threads, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FA_B200_H_ */
