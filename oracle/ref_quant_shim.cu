// ref_quant_shim.cu -- builds the REFERENCE's own quantiser for the host.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile from the reference's
// common.h where it lies (never copied into this repository).  Redefining
// __device__ before the include makes encode_fp4_e2m1 (common.h:21-36) and
// compute_scale_ue8m0 (common.h:39-48) callable from host code; the kernels in
// common.h are only embedded as compute_120a PTX and never launched.
#include <cuda_runtime.h>
#include <cstdint>
#undef __device__
#define __device__ __location__(host) __location__(device)
#include <common.h>

extern "C" uint8_t ref_encode_fp4_e2m1(float v) { return encode_fp4_e2m1(v); }

extern "C" uint8_t ref_compute_scale_ue8m0(const float* block32)
{
    float tmp[BLOCK_ELEMENT];
    for (int i = 0; i < BLOCK_ELEMENT; i++) tmp[i] = block32[i];
    return compute_scale_ue8m0(tmp);
}

// The quantisation loop of the reference kernel (common.h:115-123), run on the
// host over `rows` rows of `head_dim` floats.  codes receives the reference's
// 8-bit containers (code << 2); scales is rows x head_dim/32.
extern "C" void ref_quantize(const float* x, long long rows, int head_dim,
                             uint8_t* codes, uint8_t* scales)
{
    int nb = head_dim / BLOCK_ELEMENT;
    for (long long r = 0; r < rows; r++)
        for (int i = 0; i < nb; i++) {
            const float* blk = x + r * head_dim + i * BLOCK_ELEMENT;
            uint8_t scale = ref_compute_scale_ue8m0(blk);
            scales[r * nb + i] = scale;
            float scale_f = exp2f((float)(scale - 127));
            for (int j = 0; j < BLOCK_ELEMENT; j++)
                codes[r * head_dim + i * BLOCK_ELEMENT + j] = encode_fp4_e2m1(blk[j] / scale_f);
        }
}
