// backward_api.cuh -- fp4attn_backward and fp4attn_backward_workspace_size:
// the gradient of the FP4 fused attention (attention_bwd.cuh) behind the C
// ABI.  Included once, at the end of fp4attn.cu: the kernels share that
// translation unit's device error word (fp4attn_status_query) and its host
// helpers (fp4attn::host).
//
// fp4attn_backward_prepare launches, in stream order, the quantiser with
// dequantised BF16 copies of Q and K, the per-row Dd / lse2 pass and a clear
// of dQ (the kernel adds every key tile's contribution into it);
// fp4attn_backward_attend launches the backward kernel; fp4attn_backward is
// the two.  The workspace holds the quantised operands and the per-row
// statistics.
#pragma once

#include <cuda_bf16.h>

#include <cstdarg>

#include "attention_bwd.cuh"

namespace fp4attn_bwd {

namespace host = fp4attn::host;

constexpr int kBwdMaxDevices = 64;

bool bwd_aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int failf(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int failf(int code, const char* fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return host::error(code, buf);
}

#define BWD_CUDA(call)                                                                                \
    do {                                                                                              \
        cudaError_t e_ = (call);                                                                      \
        if (e_ != cudaSuccess) return failf(FP4ATTN_ECUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

struct BwdWorkspace {
    size_t q_codes, k_codes, q_sf, k_sf, qq, kq, nlse2, ndd, v16, do16, total;
};

struct BwdShape {
    int64_t slices;
    int sq, sk, d, sq_pad, nq, nk;
};

BwdShape bwd_shape(int batch, int heads, int sq, int sk, int d)
{
    BwdShape s;
    s.slices = static_cast<int64_t>(batch) * heads;
    s.sq = sq;
    s.sk = sk;
    s.d = d;
    s.nq = (sq + 63) / 64;
    s.nk = (sk + 127) / 128;
    s.sq_pad = s.nq * 64;
    return s;
}

// FP32 input adds the FP16 copies of V and dO.
BwdWorkspace plan_bwd_workspace(const BwdShape& s, int in_dtype)
{
    BwdWorkspace w{};
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off = (off + bytes + 255) / 256 * 256;
        return at;
    };
    const size_t n = static_cast<size_t>(s.slices);
    const int dp = (s.d + 63) / 64 * 64;  // code rows padded to the mxf4 K step
    w.q_codes = take(n * s.sq * (dp / 2));
    w.k_codes = take(n * s.sk * (dp / 2));
    w.q_sf = take(n * s.nq * 512);
    w.k_sf = take(n * s.nk * 512);
    w.qq = take(n * s.sq * s.d * 2);
    w.kq = take(n * s.sk * s.d * 2);
    w.nlse2 = take(n * s.sq_pad * 4);
    w.ndd = take(n * s.sq_pad * 4);
    w.v16 = w.do16 = off;
    if (in_dtype == FP4ATTN_F32) {
        w.v16 = take(n * s.sk * s.d * 2);
        w.do16 = take(n * s.sq * s.d * 2);
    }
    w.total = off;
    return w;
}

// Everything before the backward kernel: Q and K codes, scale tiles and BF16
// dequantised copies; -Dd and -lse2 per query row; dQ cleared.
template <int D, typename IT>
int bwd_prepare_t(const BwdShape& s, const void* Q, const void* K, const void* V, const void* Out, int out_dtype,
                  const void* dOut, const float* lse, float* dQ, int ocp, uint8_t* ws, const BwdWorkspace& w,
                  cudaStream_t st)
{
    using C = fp4attn::BwdCfg<D>;
    fp4attn::BwdQuantJob jq{Q, ws + w.q_codes, ws + w.q_sf, reinterpret_cast<__nv_bfloat16*>(ws + w.qq), s.sq, 64, 6,
                            s.nq};
    fp4attn::BwdQuantJob jk{K, ws + w.k_codes, ws + w.k_sf, reinterpret_cast<__nv_bfloat16*>(ws + w.kq), s.sk, 128, 7,
                            s.nk};
    {
        const int64_t per_slice =
            std::max<int64_t>(static_cast<int64_t>(s.nq) * 64, static_cast<int64_t>(s.nk) * 128) * (C::DP / 32);
        const int gx = static_cast<int>(
            std::min<int64_t>((per_slice + 255) / 256, std::max<int64_t>(1, 148 * 32 / s.slices + 1)));
        fp4attn::bwd_quantize_kernel<IT, D>
            <<<dim3(gx, static_cast<unsigned>(s.slices), 2), 256, 0, st>>>(jq, jk, ocp);
        BWD_CUDA(cudaGetLastError());
    }
    if constexpr (sizeof(IT) == 4) {
        const int64_t nv = static_cast<int64_t>(s.slices) * s.sk * D / 4, no = static_cast<int64_t>(s.slices) * s.sq * D / 4;
        const fp4attn::BwdConvJob jv{static_cast<const float4*>(V), reinterpret_cast<uint2*>(ws + w.v16), nv};
        const fp4attn::BwdConvJob jo{static_cast<const float4*>(dOut), reinterpret_cast<uint2*>(ws + w.do16), no};
        const int gx = static_cast<int>(std::min<int64_t>((std::max(nv, no) + 255) / 256, 148 * 16));
        fp4attn::bwd_convert_kernel<<<dim3(gx, 2), 256, 0, st>>>(jv, jo);
        BWD_CUDA(cudaGetLastError());
    }
    float* nlse2 = reinterpret_cast<float*>(ws + w.nlse2);
    float* ndd = reinterpret_cast<float*>(ws + w.ndd);
    const dim3 grid((s.sq_pad + 7) / 8, static_cast<unsigned>(s.slices));
    const IT* go = static_cast<const IT*>(dOut);
    if (out_dtype == FP4ATTN_F32)
        fp4attn::bwd_rows_kernel<D, float, IT>
            <<<grid, 256, 0, st>>>(go, static_cast<const float*>(Out), lse, nlse2, ndd, s.sq, s.sq_pad);
    else
        fp4attn::bwd_rows_kernel<D, __half, IT>
            <<<grid, 256, 0, st>>>(go, static_cast<const __half*>(Out), lse, nlse2, ndd, s.sq, s.sq_pad);
    BWD_CUDA(cudaGetLastError());
    // The kernel adds every key tile's contribution into dQ.
    BWD_CUDA(cudaMemsetAsync(dQ, 0, static_cast<size_t>(s.slices) * s.sq * D * 4, st));
    return FP4ATTN_OK;
}

template <int D>
int bwd_prepare(const BwdShape& s, int in_dtype, const void* Q, const void* K, const void* V, const void* Out,
                int out_dtype, const void* dOut, const float* lse, float* dQ, int ocp, uint8_t* ws,
                const BwdWorkspace& w, cudaStream_t st)
{
    if (in_dtype == FP4ATTN_F32)
        return bwd_prepare_t<D, float>(s, Q, K, V, Out, out_dtype, dOut, lse, dQ, ocp, ws, w, st);
    return bwd_prepare_t<D, __half>(s, Q, K, V, Out, out_dtype, dOut, lse, dQ, ocp, ws, w, st);
}

// The backward kernel on a prepared workspace (FP32 input: V and dO from
// their FP16 copies there).  test_timeout_ns > 0 runs the abort self-test
// instantiation with its waits bounded by that.
template <int D, bool kWithhold = false>
int bwd_attend(const BwdShape& s, int in_dtype, const void* V, const void* dOut, float* dQ, float* dK, float* dV,
               float scale, bool causal, const uint8_t* ws, const BwdWorkspace& w, cudaStream_t st,
               unsigned long long test_timeout_ns = 0)
{
    if (in_dtype == FP4ATTN_F32) {
        V = ws + w.v16;
        dOut = ws + w.do16;
    }
    using C = fp4attn::BwdCfg<D>;
    CUtensorMap tk, tq, tv, tkq, tdo, tqq;
    int rc;
    const uint64_t n = static_cast<uint64_t>(s.slices);
    constexpr int QR = C::QK_ROW, CHE = C::CHE, CB = C::CB;
    if ((rc = host::map3d(&tk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws + w.k_codes, QR, s.sk, n, QR, 128, QR)) ||
        (rc = host::map3d(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws + w.q_codes, QR, s.sq, n, QR, 64, QR)) ||
        (rc = host::map3d(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, V, D, s.sk, n, CHE, 128, CB)) ||
        (rc = host::map3d(&tkq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ws + w.kq, D, s.sk, n, CHE, 128, CB)) ||
        (rc = host::map3d(&tdo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, dOut, D, s.sq, n, CHE, 64, CB)) ||
        (rc = host::map3d(&tqq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ws + w.qq, D, s.sq, n, CHE, 64, CB)))
        return rc;
    fp4attn::BwdArgs a;
    a.seq_q = s.sq;
    a.seq_k = s.sk;
    a.sq_pad = s.sq_pad;
    a.nq_tiles = s.nq;
    a.nk_tiles = s.nk;
    a.slices = static_cast<int>(s.slices);
    const int64_t items = s.slices * s.nk;
    if (items > INT32_MAX) return failf(FP4ATTN_EINVAL, "too many key tiles");
    a.n_items = static_cast<int>(items);
    a.scale = scale;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.q_sf = ws + w.q_sf;
    a.k_sf = ws + w.k_sf;
    a.nlse2 = reinterpret_cast<const float*>(ws + w.nlse2);
    a.ndd = reinterpret_cast<const float*>(ws + w.ndd);
    a.dq = dQ;
    a.dk = dK;
    a.dv = dV;
    a.timeout_ns = kWithhold ? test_timeout_ns : host::timeout_ns();
    a.causal = causal ? 1 : 0;
    a.causal_off = s.sk - s.sq;
    auto kern = fp4attn::fp4_attention_bwd_kernel<D, kWithhold>;
    static std::atomic<unsigned long long> smem_ctx[kBwdMaxDevices]{};
    int dev = 0;
    BWD_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kBwdMaxDevices) return failf(FP4ATTN_EUNSUPPORTED, "device index %d", dev);
    const unsigned long long ctx = fp4attn::current_context_id();
    if (ctx == 0 || smem_ctx[dev].load(std::memory_order_acquire) != ctx) {
        BWD_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES));
        smem_ctx[dev].store(ctx, std::memory_order_release);
    }
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(items, host::sms()));
    kern<<<grid, C::THREADS, C::SMEM_BYTES, st>>>(tk, tq, tv, tkq, tdo, tqq, a);
    BWD_CUDA(cudaGetLastError());
    return FP4ATTN_OK;
}

// Argument and workspace checks shared by the entry points.
int bwd_check(int in_dtype, int batch, int heads, int seq_q, int seq_k, int head_dim, const void* workspace,
              size_t workspace_bytes, BwdShape* s, BwdWorkspace* w)
{
    if (in_dtype != FP4ATTN_F32 && in_dtype != FP4ATTN_F16) return failf(FP4ATTN_EINVAL, "in_dtype %d", in_dtype);
    if (batch < 1 || heads < 1 || seq_q < 1 || seq_k < 1)
        return failf(FP4ATTN_EINVAL, "batch, heads, seq_q and seq_k must be >= 1 (got %d, %d, %d, %d)", batch, heads,
                     seq_q, seq_k);
    if (head_dim != 32 && head_dim != 64 && head_dim != 96 && head_dim != 128)
        return failf(FP4ATTN_EUNSUPPORTED, "the backward pass covers head_dim 32, 64, 96 and 128 (got %d)", head_dim);
    if (static_cast<int64_t>(batch) * heads > 65535) return failf(FP4ATTN_EINVAL, "batch*heads exceeds 65535");
    *s = bwd_shape(batch, heads, seq_q, seq_k, head_dim);
    *w = plan_bwd_workspace(*s, in_dtype);
    if (!workspace || workspace_bytes < w->total)
        return failf(FP4ATTN_EWORKSPACE, "workspace of %zu bytes needed, %zu given", w->total,
                     workspace ? workspace_bytes : 0);
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return failf(FP4ATTN_EINVAL, "workspace must be 256-byte aligned");
    return FP4ATTN_OK;
}

}  // namespace fp4attn_bwd

extern "C" {

size_t fp4attn_backward_workspace_size(int batch, int heads, int seq_q, int seq_k, int head_dim, int in_dtype)
{
    using namespace fp4attn_bwd;
    if (batch < 1 || heads < 1 || seq_q < 1 || seq_k < 1 ||
        (head_dim != 32 && head_dim != 64 && head_dim != 96 && head_dim != 128))
        return 0;
    if (in_dtype != FP4ATTN_F32 && in_dtype != FP4ATTN_F16) return 0;
    return plan_bwd_workspace(bwd_shape(batch, heads, seq_q, seq_k, head_dim), in_dtype).total;
}

int fp4attn_backward_prepare(const void* Q, const void* K, const void* V, const void* Out, const void* dOut,
                             const float* lse, float* dQ, int in_dtype, int out_dtype, int batch, int heads, int seq_q,
                             int seq_k, int head_dim, int scale_mode, void* workspace, size_t workspace_bytes,
                             void* stream)
{
    using namespace fp4attn_bwd;
    fp4attn::set_error_detail("");
    if (!Q || !K || !V || !Out || !dOut || !lse || !dQ) return failf(FP4ATTN_EINVAL, "null pointer");
    if (!bwd_aligned16(Q) || !bwd_aligned16(K) || !bwd_aligned16(V) || !bwd_aligned16(Out) || !bwd_aligned16(dOut) ||
        !bwd_aligned16(dQ) || (reinterpret_cast<uintptr_t>(lse) & 3u))
        return failf(FP4ATTN_EINVAL, "tensor pointers must be 16-byte aligned (lse 4-byte)");
    if (out_dtype != FP4ATTN_F32 && out_dtype != FP4ATTN_F16) return failf(FP4ATTN_EINVAL, "out_dtype %d", out_dtype);
    if (scale_mode != FP4ATTN_SCALE_REFERENCE && scale_mode != FP4ATTN_SCALE_OCP)
        return failf(FP4ATTN_EINVAL, "scale_mode %d", scale_mode);
    BwdShape s;
    BwdWorkspace w;
    int rc = bwd_check(in_dtype, batch, heads, seq_q, seq_k, head_dim, workspace, workspace_bytes, &s, &w);
    if (rc) return rc;
    if ((rc = host::ready())) return rc;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int ocp = scale_mode == FP4ATTN_SCALE_OCP;
    switch (head_dim) {
        case 32: return bwd_prepare<32>(s, in_dtype, Q, K, V, Out, out_dtype, dOut, lse, dQ, ocp, ws, w, st);
        case 64: return bwd_prepare<64>(s, in_dtype, Q, K, V, Out, out_dtype, dOut, lse, dQ, ocp, ws, w, st);
        case 96: return bwd_prepare<96>(s, in_dtype, Q, K, V, Out, out_dtype, dOut, lse, dQ, ocp, ws, w, st);
        default: return bwd_prepare<128>(s, in_dtype, Q, K, V, Out, out_dtype, dOut, lse, dQ, ocp, ws, w, st);
    }
}

int fp4attn_backward_attend(const void* V, const void* dOut, float* dQ, float* dK, float* dV, int in_dtype, int batch,
                            int heads, int seq_q, int seq_k, int head_dim, float softmax_scale, int mask_mode,
                            const void* workspace, size_t workspace_bytes, void* stream)
{
    using namespace fp4attn_bwd;
    fp4attn::set_error_detail("");
    if (!V || !dOut || !dQ || !dK || !dV) return failf(FP4ATTN_EINVAL, "null pointer");
    if (!bwd_aligned16(V) || !bwd_aligned16(dOut) || !bwd_aligned16(dQ) || !bwd_aligned16(dK) || !bwd_aligned16(dV))
        return failf(FP4ATTN_EINVAL, "tensor pointers must be 16-byte aligned");
    if (mask_mode != FP4ATTN_MASK_NONE && mask_mode != FP4ATTN_MASK_CAUSAL)
        return failf(FP4ATTN_EINVAL, "mask_mode %d", mask_mode);
    BwdShape s;
    BwdWorkspace w;
    int rc = bwd_check(in_dtype, batch, heads, seq_q, seq_k, head_dim, workspace, workspace_bytes, &s, &w);
    if (rc) return rc;
    if ((rc = host::ready())) return rc;
    const float scale = softmax_scale > 0.f ? softmax_scale : 1.0f / sqrtf(static_cast<float>(head_dim));
    const bool causal = mask_mode == FP4ATTN_MASK_CAUSAL;
    const uint8_t* ws = static_cast<const uint8_t*>(workspace);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    switch (head_dim) {
        case 32: return bwd_attend<32>(s, in_dtype, V, dOut, dQ, dK, dV, scale, causal, ws, w, st);
        case 64: return bwd_attend<64>(s, in_dtype, V, dOut, dQ, dK, dV, scale, causal, ws, w, st);
        case 96: return bwd_attend<96>(s, in_dtype, V, dOut, dQ, dK, dV, scale, causal, ws, w, st);
        default: return bwd_attend<128>(s, in_dtype, V, dOut, dQ, dK, dV, scale, causal, ws, w, st);
    }
}

int fp4attn_selftest_backward_abort(const void* Q, const void* K, const void* V, const void* Out, const void* dOut,
                                    const float* lse, float* dQ, float* dK, float* dV, int batch, int heads, int seq_q,
                                    int seq_k, void* workspace, size_t workspace_bytes, unsigned timeout_us,
                                    void* stream)
{
    using namespace fp4attn_bwd;
    fp4attn::set_error_detail("");
    if (timeout_us < 1 || timeout_us > 10000000u) return failf(FP4ATTN_EINVAL, "timeout_us in [1, 1e7]");
    if (seq_q <= 64) return failf(FP4ATTN_EINVAL, "the abort self-test needs seq_q > 64 (a second step)");
    int rc = fp4attn_backward_prepare(Q, K, V, Out, dOut, lse, dQ, FP4ATTN_F16, FP4ATTN_F16, batch, heads, seq_q,
                                      seq_k, 64, FP4ATTN_SCALE_REFERENCE, workspace, workspace_bytes, stream);
    if (rc) return rc;
    if (!dK || !dV || !bwd_aligned16(dK) || !bwd_aligned16(dV)) return failf(FP4ATTN_EINVAL, "dK, dV");
    BwdShape s;
    BwdWorkspace w;
    if ((rc = bwd_check(FP4ATTN_F16, batch, heads, seq_q, seq_k, 64, workspace, workspace_bytes, &s, &w))) return rc;
    return bwd_attend<64, true>(s, FP4ATTN_F16, V, dOut, dQ, dK, dV, 0.125f, false,
                                static_cast<const uint8_t*>(workspace), w, static_cast<cudaStream_t>(stream),
                                static_cast<unsigned long long>(timeout_us) * 1000ull);
}

int fp4attn_backward(const void* Q, const void* K, const void* V, const void* Out, const void* dOut, const float* lse,
                     float* dQ, float* dK, float* dV, int in_dtype, int out_dtype, int batch, int heads, int seq_q,
                     int seq_k, int head_dim, float softmax_scale, int scale_mode, int mask_mode, void* workspace,
                     size_t workspace_bytes, void* stream)
{
    using namespace fp4attn_bwd;
    fp4attn::set_error_detail("");
    if (!V || !dK || !dV) return failf(FP4ATTN_EINVAL, "null pointer");
    if (!bwd_aligned16(V) || !bwd_aligned16(dK) || !bwd_aligned16(dV))
        return failf(FP4ATTN_EINVAL, "tensor pointers must be 16-byte aligned");
    if (mask_mode != FP4ATTN_MASK_NONE && mask_mode != FP4ATTN_MASK_CAUSAL)
        return failf(FP4ATTN_EINVAL, "mask_mode %d", mask_mode);
    int rc = fp4attn_backward_prepare(Q, K, V, Out, dOut, lse, dQ, in_dtype, out_dtype, batch, heads, seq_q, seq_k,
                                      head_dim, scale_mode, workspace, workspace_bytes, stream);
    if (rc) return rc;
    return fp4attn_backward_attend(V, dOut, dQ, dK, dV, in_dtype, batch, heads, seq_q, seq_k, head_dim,
                                   softmax_scale, mask_mode, workspace, workspace_bytes, stream);
}

}  // extern "C"
