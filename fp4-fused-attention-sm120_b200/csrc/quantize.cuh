// quantize.cuh -- the E2M1 + UE8M0 quantiser (sm_100a), bit-exact with the
// reference's encode_fp4_e2m1 / compute_scale_ue8m0 (common.h:21-48) and its
// quantisation loop (common.h:115-123, :160-168).
//
// One lane per 32-element block: it reads the block with 16-byte loads, forms
// the scale byte once, and writes 16 bytes of packed codes (element 2i in the
// low nibble) plus the scale byte.  The kernel is HBM-bound: 2 (or 4) bytes in
// and 0.53 bytes out per element.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

#include "log2_compat.h"
#include "ptx_sm100.cuh"

namespace fp4attn {

// See gen_log2_compat.c: largest mantissa remainder, per binade, for which the
// reference's host build (glibc log2f) rounds ceil(log2(y)) down to p.
// The values are part of the module image (no upload), so the table exists
// on a device as soon as the module is loaded there, including after a
// context reset.
__constant__ uint8_t kLog2CeilCompat[FP4ATTN_LOG2_COMPAT_ENTRIES] = FP4ATTN_LOG2_COMPAT_VALUES;

// compute_scale_ue8m0 (common.h:39-48) on the block maximum `amax` (>= +0):
// exponent = ceilf(log2f(y)) as the reference's host build evaluates it,
// byte = (uint8)(exponent + 127).  y = 0 or +inf make the reference's float
// -> int conversion produce INT_MIN, whose low byte after +127 is 0x7F.
__device__ __forceinline__ uint32_t scale_byte(float amax, int ocp_mode)
{
    const float y = ocp_mode ? amax / 6.0f : amax;
    const uint32_t b = __float_as_uint(y);
    const uint32_t e = b >> 23;
    if (b == 0u || e == 0xFFu) return 127u;
    int p;
    uint32_t rem;
    if (e == 0u) {  // subnormal: y = b * 2^-149
        const int msb = 31 - __clz(b);
        p = msb - 149;
        rem = b - (1u << msb);
    } else {
        p = static_cast<int>(e) - 127;
        rem = b & 0x7FFFFFu;
    }
    const int c = (rem == 0u || rem <= kLog2CeilCompat[p + 149]) ? p : p + 1;
    return static_cast<uint32_t>(c + 127) & 0xFFu;
}

// encode_fp4_e2m1 (common.h:21-36) without the <<2 container shift: the
// magnitude index is the number of thresholds (>=, ties up) below |q|, and the
// sign bit is (q < 0).  NaN fails every comparison and encodes as 0.
__device__ __forceinline__ uint32_t encode_e2m1(float q)
{
    const float a = fabsf(q);
    const uint32_t n = (a >= 0.25f) + (a >= 0.75f) + (a >= 1.25f) + (a >= 1.75f) + (a >= 2.5f) + (a >= 3.5f) +
                       (a >= 5.0f);
    return n | (q < 0.f ? 8u : 0u);
}

// Exactly 2^-s for s in [-127, 127] (2^-127 is the subnormal 1 << 22).
__device__ __forceinline__ float exact_pow2_neg(int s)
{
    const int k = -s;
    return k >= -126 ? __uint_as_float(static_cast<uint32_t>(k + 127) << 23) : __uint_as_float(1u << 22);
}

// Each block of 32 elements is handled by 4 consecutive lanes, 8 elements
// (16 B of FP16 or 32 B of FP32) per lane, so a warp's loads are contiguous.
template <typename InT>
__device__ __forceinline__ void load8(const InT* src, float (&v)[8]);

template <>
__device__ __forceinline__ void load8<__half>(const __half* src, float (&v)[8])
{
    uint4 u = __ldg(reinterpret_cast<const uint4*>(src));
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int k = 0; k < 4; k++) {
        float2 f = __half22float2(h[k]);
        v[2 * k] = f.x;
        v[2 * k + 1] = f.y;
    }
}

template <>
__device__ __forceinline__ void load8<float>(const float* src, float (&v)[8])
{
    const float4* p = reinterpret_cast<const float4*>(src);
    float4 a = __ldg(p), b = __ldg(p + 1);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// One lane per 32-element block: the whole block (64 B of FP16 or 128 B of
// FP32) is read with 16-byte loads and reduced to max|x| with 3-input max
// instructions; the reference scale byte is formed and the block is encoded
// (the common.h:118-122 loop: x / exp2f(scale - 127), encoded) into 16 bytes.
//
// Encoding uses the hardware E2M1 conversion, which rounds to nearest with
// ties to even and saturates at 6; the reference rounds ties up (away from
// zero).  The two differ only at exact ties (|q| = 0.25, 1.25, 2.5, 5), at
// -0.0 (the reference gives code 0) and at NaN (code 0).
//  * FP16 input (q then has at most 11 significant bits): q * (1 + 2^-12) + 0
//    moves every exact tie above its threshold and no other value across one
//    (a non-tie is at least 2^-11 relative away from any threshold), and
//    turns -0.0 into +0.0; only a NaN in the block (seen through the block
//    sum) takes the exact encoder.
//  * FP32 input: a block with a possible tie (21 low mantissa bits zero),
//    -0.0 or NaN is redone with the exact encoder.
// The encoding of one block held in registers (InT: the type it was read as,
// which selects the tie handling below); returns the scale byte.
template <typename InT>
__device__ __forceinline__ uint32_t encode32(const float (&v)[32], int ocp_mode, uint4& packed)
{
    float m0 = 0.f, m1 = 0.f, m2 = 0.f, m3 = 0.f;
#pragma unroll
    for (int i = 0; i < 32; i += 8) {
        m0 = ptx::fmax3_abs(m0, v[i], v[i + 1]);
        m1 = ptx::fmax3_abs(m1, v[i + 2], v[i + 3]);
        m2 = ptx::fmax3_abs(m2, v[i + 4], v[i + 5]);
        m3 = ptx::fmax3_abs(m3, v[i + 6], v[i + 7]);
    }
    const float amax = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));  // NaN never wins, as in common.h:44
    const uint32_t sb = scale_byte(amax, ocp_mode);
    const int s = static_cast<int>(sb) - 127;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (s != 128) {  // s == 128: the reference divides by exp2f(128) = inf, every code is 0
        const float inv = exact_pow2_neg(s);
        const float2 inv2 = make_float2(inv, inv);
        if constexpr (sizeof(InT) == 2) {
            const float2 nudge = make_float2(1.0f + 0x1p-12f, 1.0f + 0x1p-12f), zero = make_float2(0.f, 0.f);
            float2 sum = zero;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                float q[8];
#pragma unroll
                for (int i = 0; i < 8; i += 2) {
                    const float2 u = ptx::ffma2(ptx::fmul2(make_float2(v[8 * k + i], v[8 * k + i + 1]), inv2), nudge, zero);
                    q[i] = u.x;
                    q[i + 1] = u.y;
                    sum = ptx::fadd2(sum, make_float2(v[8 * k + i], v[8 * k + i + 1]));
                }
                w[k] = ptx::cvt_e2m1x8(q);
            }
            if (isnan(sum.x + sum.y)) {  // a NaN in the block: exact encoder
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    w[k] = 0u;
#pragma unroll
                    for (int i = 0; i < 8; i++) w[k] |= encode_e2m1(v[8 * k + i] * inv) << (4 * i);
                }
            }
        } else {
            bool exact = false;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                float q[8];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    q[i] = v[8 * k + i] * inv;
                    const uint32_t b = __float_as_uint(q[i]);
                    exact |= ((b << 11) == 0u && b != 0u) || ((b & 0x7FFFFFFFu) > 0x7F800000u);
                }
                w[k] = ptx::cvt_e2m1x8(q);
            }
            if (exact) {
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    w[k] = 0u;
#pragma unroll
                    for (int i = 0; i < 8; i++) w[k] |= encode_e2m1(v[8 * k + i] * inv) << (4 * i);
                }
            }
        }
    }
    packed = make_uint4(w[0], w[1], w[2], w[3]);
    return sb;
}

template <typename InT>
__device__ __forceinline__ uint32_t quantize32(const InT* __restrict__ src, int ocp_mode, uint4& packed)
{
    float v[32];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        float t[8];
        load8<InT>(src + 8 * k, t);
#pragma unroll
        for (int i = 0; i < 8; i++) v[8 * k + i] = t[i];
    }
    return encode32<InT>(v, ocp_mode, packed);
}

// One FP16 block as raw 16-byte words (so a caller can have the next block's
// loads in flight while it encodes this one), and its conversion to floats.
__device__ __forceinline__ void load_raw32(const __half* __restrict__ src, uint4 (&u)[4])
{
#pragma unroll
    for (int k = 0; k < 4; k++) u[k] = __ldg(reinterpret_cast<const uint4*>(src) + k);
}

__device__ __forceinline__ void raw32_to_float(const uint4 (&u)[4], float (&v)[32])
{
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const __half2* h = reinterpret_cast<const __half2*>(&u[k]);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float2 f = __half22float2(h[i]);
            v[8 * k + 2 * i] = f.x;
            v[8 * k + 2 * i + 1] = f.y;
        }
    }
}

// Byte offset of scale (row rr of a tile, scale index b along head_dim) inside
// one tile of the tensor-core scale layout.  For 128-row tiles a 512-byte atom
// holds 128 rows x 4 scales: byte = (rr%32)*16 + (rr/32)*4 + b%4, atoms in
// b/4 order.  For 64-row tiles an atom holds 64 rows x 8 scales:
// byte = (rr%32)*16 + ((b/4)%2)*8 + (rr/32)*4 + b%4, atoms in b/8 order.
// tcgen05.cp.32x128b.warpx4 moves one atom into 4 TMEM columns exactly as the
// block-scaled MMA reads them (row m at column m/32, byte = scale index).
__host__ __device__ __forceinline__ uint32_t sf_tile_offset(int tile_rows, int rr, int b)
{
    if (tile_rows == 128) return static_cast<uint32_t>((b / 4) * 512 + (rr % 32) * 16 + (rr / 32) * 4 + (b % 4));
    return static_cast<uint32_t>((b / 8) * 512 + (rr % 32) * 16 + ((b / 4) % 2) * 8 + (rr / 32) * 4 + (b % 4));
}

struct QuantTileArgs {
    int64_t slices;  // slices quantised: the first `slices` of the launch's (the rest are skipped)
    int seq;         // rows per slice
    int head_dim;    // D (multiple of 32)
    int padded_dim;  // DP, multiple of 64 (the MMA's K step)
    int tile_rows;   // 128 or 64
    int tile_shift;  // log2(tile_rows)
    int ntiles;      // ceil(seq / tile_rows)
    int sf_tile_bytes;
    int ocp_mode;
};

// One tensor to quantise into the layout the attention kernel loads with TMA.
struct QuantJob {
    const void* x;      // [slices][seq][head_dim] of InT
    uint8_t* codes;     // [slices][seq][DP/2]
    uint8_t* sf;        // [slices][ntiles][sf_tile_bytes]
    QuantTileArgs a;
};

// V in FP32, converted to the FP16 copy the attention kernel reads, per slice
// (n4 float4 per slice); and n_zero words of the workspace the attention
// kernel needs at zero (its key-partition arrival counters), cleared by the
// first CTA of the launch.
struct VConvJob {
    const float4* src;
    uint2* dst;
    int64_t n4;
    uint32_t* zero;
    int n_zero;
};

// Quantise Q (blockIdx.z == 0) and K (blockIdx.z == 1) in one launch into the
// layout the attention kernel loads with TMA: codes [slices][seq][DP/2]
// (blocks beyond D are zero) and scale tiles [slices][ntiles][sf_tile_bytes].
// Rows past seq inside the last tile get scale 127 so the (zero-filled)
// padding never multiplies an undefined scale.  A reference scale of 255 only
// occurs with all-zero codes and is stored as 254, which the MMA reads as a
// finite 2^127 (255 would be NaN in E8M0).  Grid: x covers one slice's padded
// rows (kNB blocks of 32 per row, one lane per block), y is the slice, so all
// index arithmetic is 32-bit with a compile-time divisor.
// With FP32 input the same launch also converts V (blockIdx.z == 2).
template <typename InT, int kNB>
__global__ void __launch_bounds__(256) quantize_tiles_kernel(const QuantJob jq, const QuantJob jk, const VConvJob jv)
{
    // The attention kernel (launched as this grid's programmatic dependent)
    // may be scheduled once every CTA of this grid has started, so its launch
    // and prologue overlap this grid's last wave; it waits for this grid's
    // completion (griddepcontrol.wait) before it reads the workspace.
    ptx::grid_launch_dependents();
    if (jv.n_zero > 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
        for (int i = threadIdx.x; i < jv.n_zero; i += blockDim.x) jv.zero[i] = 0u;
    if (blockIdx.z == 2) {
        // FP32 -> FP16 (round to nearest even) for this slice of V.
        const float4* src = jv.src + static_cast<int64_t>(blockIdx.y) * jv.n4;
        uint2* dst = jv.dst + static_cast<int64_t>(blockIdx.y) * jv.n4;
        for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < jv.n4;
             i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
            const float4 f = src[i];
            __half2 a = __floats2half2_rn(f.x, f.y), b = __floats2half2_rn(f.z, f.w);
            dst[i] = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
        }
        return;
    }
    const bool is_k = blockIdx.z != 0;
    const QuantTileArgs a = is_k ? jk.a : jq.a;
    if (blockIdx.y >= a.slices) return;
    const InT* x = static_cast<const InT*>(is_k ? jk.x : jq.x);
    uint8_t* codes = is_k ? jk.codes : jq.codes;
    uint8_t* sf = is_k ? jk.sf : jq.sf;
    const int seq_pad = a.ntiles * a.tile_rows;
    const int total = seq_pad * kNB;  // blocks of 32 in this slice (padded rows included)
    const int64_t slice = blockIdx.y;
    const InT* xs = x + slice * a.seq * a.head_dim;
    uint8_t* cs = codes + slice * a.seq * (kNB * 16);
    uint8_t* fs = sf + slice * a.ntiles * a.sf_tile_bytes;
    for (int blk = blockIdx.x * blockDim.x + threadIdx.x; blk < total; blk += gridDim.x * blockDim.x) {
        const int b = blk % kNB;
        const int r = blk / kNB;
        uint32_t sb = 127u;
        if (r < a.seq) {
            uint4 packed = make_uint4(0u, 0u, 0u, 0u);
            if (b * 32 < a.head_dim) {
                sb = quantize32<InT>(xs + static_cast<int64_t>(r) * a.head_dim + b * 32, a.ocp_mode, packed);
                if (sb == 255u) sb = 254u;
            }
            *reinterpret_cast<uint4*>(cs + static_cast<int64_t>(r) * (kNB * 16) + b * 16) = packed;
        }
        const int tile = r >> a.tile_shift, rr = r & (a.tile_rows - 1);
        fs[static_cast<int64_t>(tile) * a.sf_tile_bytes + sf_tile_offset(a.tile_rows, rr, b)] = static_cast<uint8_t>(sb);
    }
}

// Row-major quantisation for the public fp4attn_quantize: codes rows x D/2,
// scales rows x D/32, raw reference bytes (255 kept).
template <typename InT>
__global__ void __launch_bounds__(256) quantize_rowmajor_kernel(const InT* __restrict__ x, int64_t rows, int head_dim,
                                                                uint8_t* __restrict__ codes, uint8_t* __restrict__ sf,
                                                                int ocp_mode)
{
    const int64_t total = rows * (head_dim / 32);
    for (int64_t blk = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; blk < total;
         blk += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        uint4 packed;
        const uint32_t sb = quantize32<InT>(x + blk * 32, ocp_mode, packed);
        *reinterpret_cast<uint4*>(codes + blk * 16) = packed;
        sf[blk] = static_cast<uint8_t>(sb);
    }
}

}  // namespace fp4attn
