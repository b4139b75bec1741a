/*
 * fp4_fused_attention.h -- C++ drop-in for the reference's launch surface.
 *
 * The reference's callers launch
 *     fused_fp4_attention<HEAD_DIM><<<batch * heads, NUM_THREADS>>>(
 *         Q, K, Out, V, seq_q, seq_k, heads);                (common.h:68-77,
 *                                               tests/test_attention.cu:160-161)
 * on FP32 device buffers in [batch, heads, seq, head_dim] layout.  The
 * templates below keep that argument order and meaning as a host call (a
 * launch needs tensor maps and a workspace, so it cannot be a bare <<<>>>):
 *     fused_fp4_attention_launch<HEAD_DIM>(Q, K, Out, V, seq_q, seq_k, heads,
 *                                          batch, stream);
 * They return an fp4attn_status; the workspace is taken from the stream-ordered
 * allocator and released on the same stream.  Overloads take FP16 inputs and
 * FP32 or FP16 output.  Callers that manage memory themselves use the C ABI in
 * fp4attn.h (fp4attn_workspace_size + fp4attn_forward) directly.
 */
#ifndef FP4_FUSED_ATTENTION_H
#define FP4_FUSED_ATTENTION_H

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "fp4attn.h"

namespace fp4attn_detail {

template <typename T>
constexpr int dtype_code()
{
    return sizeof(T) == 4 ? FP4ATTN_F32 : FP4ATTN_F16;
}

template <int HEAD_DIM, typename InT, typename OutT>
inline int launch(const InT* Q, const InT* K, OutT* Out, const InT* V, int seq_q, int seq_k, int heads, int batch,
                  cudaStream_t stream, bool causal)
{
    const int in = dtype_code<InT>(), out = dtype_code<OutT>();
    const size_t ws_bytes = fp4attn_workspace_size(batch, heads, seq_q, seq_k, HEAD_DIM, in);
    if (ws_bytes == 0) return FP4ATTN_EINVAL;
    void* ws = nullptr;
    if (cudaMallocAsync(&ws, ws_bytes, stream) != cudaSuccess) return FP4ATTN_ECUDA;
    const int rc = fp4attn_forward_masked(Q, K, V, Out, in, out, batch, heads, seq_q, seq_k, HEAD_DIM, 0.0f,
                                          FP4ATTN_SCALE_REFERENCE, causal ? FP4ATTN_MASK_CAUSAL : FP4ATTN_MASK_NONE,
                                          ws, ws_bytes, stream);
    const cudaError_t fe = cudaFreeAsync(ws, stream);
    if (rc != FP4ATTN_OK) return rc;
    return fe == cudaSuccess ? FP4ATTN_OK : FP4ATTN_ECUDA;
}

}  // namespace fp4attn_detail

/* The reference's argument order: Q, K, Out, V, seq_q, seq_k, heads; then the
 * batch the reference infers from its grid, a stream, and (an extension) the
 * bottom-right causal mask. */
template <int HEAD_DIM>
inline int fused_fp4_attention_launch(const float* Q, const float* K, float* Out, const float* V, int seq_q,
                                      int seq_k, int heads, int batch = 1, cudaStream_t stream = 0,
                                      bool causal = false)
{
    return fp4attn_detail::launch<HEAD_DIM>(Q, K, Out, V, seq_q, seq_k, heads, batch, stream, causal);
}

template <int HEAD_DIM>
inline int fused_fp4_attention_launch(const __half* Q, const __half* K, float* Out, const __half* V, int seq_q,
                                      int seq_k, int heads, int batch = 1, cudaStream_t stream = 0,
                                      bool causal = false)
{
    return fp4attn_detail::launch<HEAD_DIM>(Q, K, Out, V, seq_q, seq_k, heads, batch, stream, causal);
}

template <int HEAD_DIM>
inline int fused_fp4_attention_launch(const __half* Q, const __half* K, __half* Out, const __half* V, int seq_q,
                                      int seq_k, int heads, int batch = 1, cudaStream_t stream = 0,
                                      bool causal = false)
{
    return fp4attn_detail::launch<HEAD_DIM>(Q, K, Out, V, seq_q, seq_k, heads, batch, stream, causal);
}

#endif /* FP4_FUSED_ATTENTION_H */
