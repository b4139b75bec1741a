/*
 * fp4attn_oracle.h -- CPU restatement of the reference's FP4 attention path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker: tests/, the smoke
 * check in __graft_entry__.py and the cpu_baseline leg of bench.py call it to
 * produce expected values.  The product (libfp4attn.so) never links or calls
 * it, and nothing here is ever timed as the GPU path.
 *
 * Every function restates the algorithm of florianmattana/fp4-fused-attention-sm120
 * (the file:line of the reference code it follows is cited on each one).
 * Parity is pinned against the reference itself: oracle/Makefile compiles the
 * reference's own quantiser (common.h:21-48) and CPU attention
 * (tests/test_attention.cu:9-65) into oracle/_ref/libfp4ref.so, and
 * tests/test_oracle.py checks this restatement against it and against the
 * committed golden vectors in tests/golden/.
 */
#ifndef FP4ATTN_ORACLE_H
#define FP4ATTN_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Scale rules.  0 = the reference rule ceil(log2(max|x|)) + 127
 * (common.h:39-48); 1 = the OCP-MX style rule ceil(log2(max|x| / 6)) + 127
 * (an opt-in variant, not part of the reference). */
#define ORACLE_SCALE_REF 0
#define ORACLE_SCALE_OCP 1

/* encode_fp4_e2m1 (common.h:21-36): returns the 4-bit code (sign in bit 3).
 * The reference returns code<<2 in an 8-bit container; this returns the code. */
uint8_t oracle_encode_e2m1(float v);

/* compute_scale_ue8m0 (common.h:39-48) over one block of 32 floats. */
uint8_t oracle_scale_ue8m0(const float* block32, int scale_mode);

/* E2M1 code (0..15) -> value. */
float oracle_e2m1_value(uint8_t code);

/* Quantise rows x head_dim floats (head_dim % 32 == 0) the way the reference's
 * kernel does for its Q and K tiles (common.h:115-123 and :160-168):
 *   codes  : rows x head_dim bytes, one 4-bit code per byte (unpacked)
 *   scales : rows x head_dim/32 bytes, row-major */
void oracle_quantize(const float* x, int64_t rows, int head_dim,
                     uint8_t* codes, uint8_t* scales, int scale_mode);

/* Dequantise: value(code) * 2^(scale-127); code 0 gives 0 for every scale. */
void oracle_dequantize(const uint8_t* codes, const uint8_t* scales, int64_t rows,
                       int head_dim, float* out);

/* Causal variant of oracle_attention -- not part of the reference, which has
 * no mask: query row i of this call is row first_row + i of a sequence of
 * seq_q_total queries and sees keys j <= first_row + i + seq_k - seq_q_total
 * (bottom-right alignment); a row that sees no key gets a zero output.  The
 * arithmetic of every visible element is that of oracle_attention. */
void oracle_attention_causal(const float* Q, const float* K, const float* V, float* Out,
                             int seq_q, int seq_k, int head_dim, float scale,
                             int first_row, int seq_q_total);

/* oracle_fp4_attention with the causal mask of oracle_attention_causal. */
void oracle_fp4_attention_causal(const float* Q, const float* K, const float* V, float* Out,
                                 int slices, int seq_q, int seq_k, int head_dim,
                                 float scale, int scale_mode, int threads);

/* cpu_attention (tests/test_attention.cu:33-54) for one (batch, head) slice,
 * FP32 throughout: S = Q K^T, S *= scale, row softmax with expf, Out = P V.
 * scale <= 0 selects 1/sqrt(head_dim) as the reference does (:46). */
void oracle_attention(const float* Q, const float* K, const float* V, float* Out,
                      int seq_q, int seq_k, int head_dim, float scale);

/* The full FP4 path for `slices` contiguous [seq, head_dim] slices:
 * quantise Q and K with the reference rule, dequantise, then oracle_attention
 * against FP32 V.  Runs up to `threads` POSIX threads over slices. */
void oracle_fp4_attention(const float* Q, const float* K, const float* V, float* Out,
                          int slices, int seq_q, int seq_k, int head_dim,
                          float scale, int scale_mode, int threads);

/* The same path restricted to selected query rows of selected slices (for
 * parity at sizes where the full oracle would take too long).  rows[i] is the
 * query row index inside slice slice_of[i]; Out holds n x head_dim floats. */
void oracle_fp4_attention_rows(const float* Q, const float* K, const float* V,
                               float* Out, int n, const int* slice_of, const int* rows,
                               int seq_q, int seq_k, int head_dim,
                               float scale, int scale_mode);

/* The same path over every query row of ONE slice, with the rows split over
 * up to `threads` POSIX threads (for whole-slice parity at full sizes, where
 * the per-slice threading of oracle_fp4_attention has one slice to run).
 * Each row is computed exactly as oracle_attention computes it. */
void oracle_fp4_attention_slice(const float* Q, const float* K, const float* V, float* Out,
                                int seq_q, int seq_k, int head_dim, float scale, int scale_mode,
                                int threads);

/* Q K^T for one slice on dequantised FP4 inputs (the S tile of the
 * reference's debug_mma kernel, common.h:331-398, generalised to any
 * seq_q x seq_k with block scales).  No softmax scale applied. */
void oracle_fp4_scores(const float* Q, const float* K, float* S,
                       int seq_q, int seq_k, int head_dim, int scale_mode);

/* Gradient of the FP4 path (not part of the reference, which is forward
 * only), the quantiser taken as a straight-through estimator: for `slices`
 * contiguous slices, dQ = scale dZ Kq, dK = scale dZ^T Qq, dV = P^T dO with
 * dZ = P o (dO V^T - rowsum(P o dO V^T)), Qq / Kq the dequantised codes and
 * P = softmax(scale Qq Kq^T) (causal != 0: the mask of
 * oracle_attention_causal).  Double accumulation; each slice's query rows are
 * split over up to `threads` POSIX threads. */
void oracle_fp4_attention_backward(const float* Q, const float* K, const float* V, const float* dO,
                                   float* dQ, float* dK, float* dV, int slices, int seq_q, int seq_k, int head_dim,
                                   float scale, int scale_mode, int causal, int threads);

/* Per query row the natural-log log-sum-exp of scale * Qq Kq^T over the
 * visible keys (+inf when a row sees none), [slices][seq_q]. */
void oracle_fp4_attention_lse(const float* Q, const float* K, float* lse, int slices, int seq_q, int seq_k,
                              int head_dim, float scale, int scale_mode, int causal);

/* cosine_similarity (tests/test_attention.cu:56-65), accumulated in double. */
double oracle_cosine(const float* a, const float* b, int64_t n);

#ifdef __cplusplus
}
#endif
#endif
