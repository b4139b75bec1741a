/*
 * fp4attn.h -- C ABI of libfp4attn.so, the sm_100a (B200) FP4 fused attention.
 *
 * Drop-in boundary for the reference florianmattana/fp4-fused-attention-sm120.
 * The reference exposes no library: its public surface is the header
 * common.h -- the encoders encode_fp4_e2m1 / compute_scale_ue8m0
 * (common.h:21-48), the kernel template
 *     template<int HEAD_DIM> __global__ void fused_fp4_attention(
 *         const float* Q, const float* K, float* Out, const float* V,
 *         int seq_q, int seq_k, int heads)                      (common.h:68-77)
 * launched as <<<batch*heads, NUM_THREADS>>> (tests/test_attention.cu:160-161),
 * and the constants BLOCK_ELEMENT / BQ (common.h:15, :18).  Each entry point
 * below names the reference interface it replaces.
 *
 * Conventions: all pointers are device pointers unless stated; tensors are
 * contiguous [batch, heads, seq, head_dim] (the reference layout,
 * common.h:99-102); `stream` is a cudaStream_t (0 = legacy default stream).
 * Every call is asynchronous on `stream` and returns an fp4attn_status code;
 * a non-zero code means nothing was launched.  The library keeps no state
 * between calls except, per device, its first-use set-up (the device check
 * and the SM count; kernel attributes per device context), an error word
 * (fp4attn_status_query), the fp4attn_forward_noalloc scratch, and per host
 * thread a cache of recently encoded TMA descriptors.  Calls on different
 * streams may run concurrently; the caller owns all buffers.  The attention
 * kernel of a call is launched as the programmatic dependent of the launch
 * before it in the stream (normally this call's quantiser): it starts while
 * that launch finishes and waits for it before reading the workspace.
 */
#ifndef FP4ATTN_H
#define FP4ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- constants kept from the reference (common.h:12, :15, :18) ---------- */
#define FP4ATTN_BLOCK_ELEMENT 32 /* elements per UE8M0 scale (BLOCK_ELEMENT) */
#define FP4ATTN_BQ 64            /* the reference's fixed Q tile (BQ)         */

/* ---- status codes ------------------------------------------------------- */
typedef enum {
    FP4ATTN_OK = 0,
    FP4ATTN_EINVAL = 1,       /* bad shape, dtype, pointer alignment or size  */
    FP4ATTN_EUNSUPPORTED = 2, /* head_dim not compiled / no sm_100 device     */
    FP4ATTN_ECUDA = 3,        /* a CUDA runtime or driver call failed          */
    FP4ATTN_ETIMEOUT = 4,     /* a kernel's bounded wait expired (reported by  */
                              /* fp4attn_status_query after the stream syncs) */
    FP4ATTN_EWORKSPACE = 5    /* workspace missing or too small               */
} fp4attn_status;

/* ---- element types ------------------------------------------------------ */
typedef enum { FP4ATTN_F32 = 0, FP4ATTN_F16 = 1 } fp4attn_dtype;

/* ---- UE8M0 scale rules -------------------------------------------------- */
typedef enum {
    /* The reference rule, bit-exact with compute_scale_ue8m0 (common.h:39-48)
     * as built on the host with glibc: byte = (uint8)(ceil(log2(max|x|)) + 127),
     * an all-zero block gives 127. */
    FP4ATTN_SCALE_REFERENCE = 0,
    /* OCP-MX style: byte = (uint8)(ceil(log2(max|x| / 6)) + 127).  Not part of
     * the reference; offered because it uses the full E2M1 range. */
    FP4ATTN_SCALE_OCP = 1
} fp4attn_scale_mode;

/* ---- attention masks ------------------------------------------------------ */
typedef enum {
    FP4ATTN_MASK_NONE = 0,   /* every query sees every key (the reference's only mode) */
    /* Causal, bottom-right aligned: query i sees keys j <= i + seq_k - seq_q, so
     * with seq_q == seq_k row i sees keys 0..i.  A query that sees no key
     * (only possible when seq_q > seq_k) gets a zero output row. */
    FP4ATTN_MASK_CAUSAL = 1
} fp4attn_mask;

/* ---- layouts of quantised output ---------------------------------------- */
typedef enum {
    /* codes: rows x head_dim/2 bytes, two E2M1 codes per byte, element 2i in
     * the low nibble; scales: rows x head_dim/32 bytes, row-major. */
    FP4ATTN_LAYOUT_ROWMAJOR = 0
} fp4attn_layout;

/* Quantise `rows` rows of `head_dim` elements (head_dim % 32 == 0) to E2M1
 * codes plus one UE8M0 scale per 32 elements.
 * Replaces: the per-tile quantisation inside the reference kernel
 * (common.h:108-124 for Q, :159-169 for K) built from encode_fp4_e2m1 and
 * compute_scale_ue8m0 (common.h:21-48).  The reference returns each code in an
 * 8-bit container (code << 2, common.h:35); this packs two codes per byte.
 * x: device, dtype elements; codes: rows*head_dim/2 bytes; scales:
 * rows*head_dim/32 bytes. */
int fp4attn_quantize(const void* x, int dtype, int64_t rows, int head_dim, uint8_t* codes,
                     uint8_t* scales, int scale_mode, int layout, void* stream);

/* Bytes of device workspace fp4attn_forward needs for this problem (the
 * quantised Q/K tiles, their scale tiles, an FP16 copy of V when V is FP32,
 * and, for a small problem whose keys are split over several CTAs, the
 * partial results of the key partitions and their arrival counters).  The
 * same for every mask mode.  Returns 0 for an invalid shape. */
size_t fp4attn_workspace_size(int batch, int heads, int seq_q, int seq_k, int head_dim, int in_dtype);

/* Out = softmax(Q K^T * softmax_scale) V per (batch, head) slice, with Q and K
 * quantised to E2M1 + UE8M0 (block 32 along head_dim) and V, P in FP16 on the
 * tensor cores (FP32 accumulation).
 * Replaces: fused_fp4_attention<HEAD_DIM><<<batch*heads, 128>>>(Q, K, Out, V,
 * seq_q, seq_k, heads) (common.h:68-77; tests/test_attention.cu:160-161).
 * Differences, by design: any seq_q >= 1 (the reference computes only the
 * first 64 query rows, common.h:96-102) and any seq_k >= 1 (the reference
 * needs seq_k % 64 == 0, common.h:67); head_dim is a runtime argument among
 * {32, 64, 96, 128, 160, 256}; inputs and output may be FP32 (as in the
 * reference) or FP16.
 * Q: [batch, heads, seq_q, head_dim]; K, V: [batch, heads, seq_k, head_dim];
 * Out: [batch, heads, seq_q, head_dim] of out_dtype; all 16-byte aligned.
 * softmax_scale <= 0 selects 1/sqrt(head_dim) (common.h:130).
 * workspace: device memory of at least fp4attn_workspace_size(...) bytes,
 * 256-byte aligned; it must not be used by another call in flight. */
int fp4attn_forward(const void* Q, const void* K, const void* V, void* Out, int in_dtype, int out_dtype,
                    int batch, int heads, int seq_q, int seq_k, int head_dim, float softmax_scale,
                    int scale_mode, void* workspace, size_t workspace_bytes, void* stream);

/* The two halves of fp4attn_forward, for callers that quantise once and
 * attend many times (e.g. a fixed K/V) or time the attention kernel alone.
 * fp4attn_prepare quantises Q and K into `workspace` (and, for FP32 input,
 * stores an FP16 copy of V there).  Replaces: the quantisation prologue of the
 * reference kernel (common.h:108-124 for Q, :146-169 for K and V). */
int fp4attn_prepare(const void* Q, const void* K, const void* V, int in_dtype, int batch, int heads, int seq_q,
                    int seq_k, int head_dim, int scale_mode, void* workspace, size_t workspace_bytes, void* stream);

/* Runs the attention kernel on a workspace filled by fp4attn_prepare with the
 * same shape and in_dtype.  V is read directly when in_dtype is FP16.  May be
 * called any number of times on one prepared workspace (one call at a time);
 * after a call that reported FP4ATTN_ETIMEOUT, prepare the workspace again.
 * Replaces: the main loop of the reference kernel (common.h:140-327). */
int fp4attn_attend(const void* V, void* Out, int in_dtype, int out_dtype, int batch, int heads, int seq_q, int seq_k,
                   int head_dim, float softmax_scale, const void* workspace, size_t workspace_bytes, void* stream);

/* fp4attn_forward and fp4attn_attend with a mask (fp4attn_mask).  With
 * FP4ATTN_MASK_NONE they are those calls; with FP4ATTN_MASK_CAUSAL each query
 * tile also stops reading keys after the last one it can see, so a causal
 * problem costs about half the unmasked one.  The workspace is the same.
 * No counterpart in the reference, which has no mask (common.h:228-265
 * softmaxes every key of every tile). */
int fp4attn_forward_masked(const void* Q, const void* K, const void* V, void* Out, int in_dtype, int out_dtype,
                           int batch, int heads, int seq_q, int seq_k, int head_dim, float softmax_scale,
                           int scale_mode, int mask_mode, void* workspace, size_t workspace_bytes, void* stream);
int fp4attn_attend_masked(const void* V, void* Out, int in_dtype, int out_dtype, int batch, int heads, int seq_q,
                          int seq_k, int head_dim, float softmax_scale, int mask_mode, const void* workspace,
                          size_t workspace_bytes, void* stream);

/* fp4attn_forward with Q quantised inside the attention kernel instead of in
 * the pre-pass launch, as the reference quantises its Q tile inside its own
 * kernel (common.h:108-124): the pre-pass quantises only K, and the attention
 * kernel reads FP16 Q and encodes it with the same encoder, so the codes,
 * scales and output are those of fp4attn_forward, bit for bit.  Applies to
 * FP16 input with head_dim <= 128, seq_k >= 3008 (48 key tiles of 64) on the
 * large-problem schedule (seq_q > 128 and at least 75 query groups of 256
 * rows); any other problem runs the fp4attn_forward path.  Same arguments and
 * workspace as fp4attn_forward.
 * Replaces: the quantisation prologue of fused_fp4_attention (common.h:108-124). */
int fp4attn_forward_fused_q(const void* Q, const void* K, const void* V, void* Out, int in_dtype, int out_dtype,
                            int batch, int heads, int seq_q, int seq_k, int head_dim, float softmax_scale,
                            int scale_mode, void* workspace, size_t workspace_bytes, void* stream);

/* fp4attn_forward for callers that cannot allocate device memory (code running
 * during CUDA graph capture, runtimes that own all device memory, loops that
 * must not block on an allocation): the same computation, with the workspace
 * taken from a 64 MiB scratch array the library holds on each device from the
 * first call (or from context creation under CUDA_MODULE_LOADING=EAGER) until
 * the process exits.  Problems whose fp4attn_workspace_size exceeds 64 MiB are
 * rejected with FP4ATTN_EWORKSPACE.  The first call on a device looks up the
 * scratch's device address (again after a device reset, which moves it); make
 * it before any stream capture.  All calls on a
 * device share the scratch: calls that may overlap on the GPU must be
 * serialised by the caller.  No counterpart in the reference (its kernel keeps
 * everything in shared memory and needs no workspace). */
int fp4attn_forward_noalloc(const void* Q, const void* K, const void* V, void* Out, int in_dtype, int out_dtype,
                            int batch, int heads, int seq_q, int seq_k, int head_dim, float softmax_scale,
                            int scale_mode, void* stream);

/* fp4attn_forward_masked that also writes, per query row, the natural-log
 * log-sum-exp of the scaled scores, lse[b][h][i] = ln(sum_j exp(scale * S_ij))
 * over the keys the row sees (FP32 [batch, heads, seq_q]; +inf for a row that
 * sees no key) -- the statistic the backward pass rebuilds the probabilities
 * from.  head_dim 32, 64, 96 and 128.  Same workspace as fp4attn_forward.  No
 * counterpart in the reference (forward only; its row max and sum stay in
 * registers, common.h:228-265). */
int fp4attn_forward_lse(const void* Q, const void* K, const void* V, void* Out, float* lse, int in_dtype,
                        int out_dtype, int batch, int heads, int seq_q, int seq_k, int head_dim, float softmax_scale,
                        int scale_mode, int mask_mode, void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes fp4attn_backward needs for this shape and input type (0 if
 * unsupported). */
size_t fp4attn_backward_workspace_size(int batch, int heads, int seq_q, int seq_k, int head_dim, int in_dtype);

/* Gradient of the FP4 fused attention.  Inputs: the forward's Q, K, V and
 * dOut (the gradient of Out), all of in_dtype (FP16 or FP32; FP32 V and dOut
 * are rounded to FP16 for the tensor cores, as the forward rounds V), its
 * output Out (out_dtype FP16 or FP32) and the lse rows of
 * fp4attn_forward_lse (same shape, scale, scale_mode and mask).  Outputs: FP32 dQ, dK, dV in the layout of Q, K, V.  The quantiser
 * is treated as a straight-through estimator: with Qq, Kq the dequantised
 * codes the forward multiplied and P its probabilities,
 *   dV = P^T dOut,  dZ = P o (dOut V^T - rowsum(dOut o Out)),
 *   dQ = scale * dZ Kq,  dK = scale * dZ^T Qq.
 * head_dim 32, 64, 96 and 128.  Every byte of dQ, dK and dV is written.  No
 * counterpart in the reference, which is inference-only. */
int fp4attn_backward(const void* Q, const void* K, const void* V, const void* Out, const void* dOut, const float* lse,
                     float* dQ, float* dK, float* dV, int in_dtype, int out_dtype, int batch, int heads, int seq_q,
                     int seq_k, int head_dim, float softmax_scale, int scale_mode, int mask_mode, void* workspace,
                     size_t workspace_bytes, void* stream);

/* The two halves of fp4attn_backward (as fp4attn_prepare / fp4attn_attend
 * are of fp4attn_forward).  fp4attn_backward_prepare quantises Q and K into
 * the workspace (codes, scale tiles and the dequantised values as BF16), for
 * FP32 input stores FP16 copies of V and dOut there, forms the per-row
 * statistics of dOut, Out and lse, and clears dQ;
 * fp4attn_backward_attend runs the backward kernel on that workspace, adding
 * into dQ and writing dK and dV.  Same shapes, alignment and workspace as
 * fp4attn_backward. */
int fp4attn_backward_prepare(const void* Q, const void* K, const void* V, const void* Out, const void* dOut,
                             const float* lse, float* dQ, int in_dtype, int out_dtype, int batch, int heads, int seq_q,
                             int seq_k, int head_dim, int scale_mode, void* workspace, size_t workspace_bytes,
                             void* stream);
int fp4attn_backward_attend(const void* V, const void* dOut, float* dQ, float* dK, float* dV, int in_dtype, int batch,
                            int heads, int seq_q, int seq_k, int head_dim, float softmax_scale, int mask_mode,
                            const void* workspace, size_t workspace_bytes, void* stream);

/* Self-test of the backward kernel's failure path (the counterpart of
 * fp4attn_selftest_abort): fp4attn_backward_prepare, then the head_dim 64
 * backward kernel in a test instantiation where one gradient thread withholds
 * its first arrival, with every wait bounded by timeout_us.  The wait runs
 * out, every role of every CTA leaves its loop, in-flight copies and MMAs are
 * drained, TMEM is freed; fp4attn_status_query then reports
 * FP4ATTN_ETIMEOUT and the context stays usable.  FP16 inputs, seq_q > 64.
 * dQ, dK and dV hold no result afterwards. */
int fp4attn_selftest_backward_abort(const void* Q, const void* K, const void* V, const void* Out, const void* dOut,
                                    const float* lse, float* dQ, float* dK, float* dV, int batch, int heads, int seq_q,
                                    int seq_k, void* workspace, size_t workspace_bytes, unsigned timeout_us,
                                    void* stream);

/* S = Q K^T (no softmax scale) on the FP4-quantised Q and K of one problem,
 * written as FP32 [batch, heads, seq_q, seq_k].  Because FP4 products with
 * power-of-two scales are exact, S is checkable bit for bit.
 * Replaces: the reference's debug kernel debug_mma (common.h:331-398), which
 * computes one 64x64 tile of Q K^T on FP4 codes. */
int fp4attn_debug_scores(const void* Q, const void* K, float* S, int in_dtype, int batch, int heads,
                         int seq_q, int seq_k, int head_dim, int scale_mode, void* workspace,
                         size_t workspace_bytes, void* stream);

/* Reads and clears the device error word that kernels set when a bounded
 * wait expires.  Synchronises `stream` first.  Returns FP4ATTN_OK or
 * FP4ATTN_ETIMEOUT (or FP4ATTN_ECUDA if the query itself fails).  The word is
 * one per device, shared by every stream: a kernel still running on another
 * stream may set it after this call returns (it is then reported by the next
 * query), and a timeout raised on another stream is reported by whichever
 * query reads the word first.  To attribute a timeout to one stream's work,
 * synchronise the other streams that run this library's kernels (or the
 * device) before querying.  The reference has no device-side error reporting
 * (callers only poll cudaGetLastError, tests/test_attention.cu:103-105). */
int fp4attn_status_query(void* stream);

/* Test hook for the failure path: launches one CTA that waits on an mbarrier
 * nothing will complete, with the given bound, so that the bounded wait runs
 * out and sets the error word.  No fault, trap or hang is involved. */
int fp4attn_selftest_timeout(unsigned timeout_us, void* stream);

/* Test hook for the attention kernel's own failure path: runs the
 * head_dim-64, FP32-output attention kernel (seq_q > 128, a problem without
 * key partitions) over a workspace filled by fp4attn_prepare (FP16 input), in
 * a build in which one softmax thread never makes its first "S copied"
 * arrival.  The kernel's bounded wait for it expires after timeout_us; every
 * role then leaves its loop, drains its in-flight copies and MMAs, frees its
 * tensor memory and returns, and fp4attn_status_query reports
 * FP4ATTN_ETIMEOUT.  No fault, trap or hang is involved; later calls on the
 * same context run normally.  No counterpart in the reference. */
int fp4attn_selftest_abort(const void* V, void* Out, int batch, int heads, int seq_q, int seq_k,
                           const void* workspace, size_t workspace_bytes, unsigned timeout_us, void* stream);

/* Test hook: y[i] = 2^x[i] computed by the FMA-pipe polynomial the softmax
 * uses for part of its exponentials (n even, 16-byte aligned device arrays).
 * No counterpart in the reference, whose softmax calls expf (common.h:236). */
int fp4attn_selftest_exp2(const float* x, float* y, int64_t n, void* stream);

/* Static description of a status code. */
const char* fp4attn_error_string(int status);

/* Detail of the last failure on the calling host thread ("" if none). */
const char* fp4attn_last_error(void);

/* Head dims compiled into this library, written to `dims` (up to `cap`);
 * returns how many there are. */
int fp4attn_supported_head_dims(int* dims, int cap);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* FP4ATTN_H */
