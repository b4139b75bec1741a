// ref_driver.cpp -- host driver around the REFERENCE's own CPU attention.
//
// TEST INFRASTRUCTURE ONLY.  cpu_attention and cosine_similarity come from the
// reference's tests/test_attention.cu:33-65, compiled from its source by
// oracle/Makefile; ref_quantize comes from ref_quant_shim.cu (the reference's
// common.h quantiser).  This file only adds the slice loop, FP4 dequantisation
// and a thread pool so bench.py can time the reference's CPU path on all host
// cores.
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <thread>
#include <vector>

void cpu_attention(const float* Q, const float* K, const float* V, float* Out,
                   int seq_q, int seq_k, int head_dim);
float cosine_similarity(const float* a, const float* b, int n);
extern "C" void ref_quantize(const float* x, long long rows, int head_dim,
                             uint8_t* codes, uint8_t* scales);

extern "C" float ref_cosine_similarity(const float* a, const float* b, int n)
{
    return cosine_similarity(a, b, n);
}

extern "C" void ref_cpu_attention(const float* Q, const float* K, const float* V,
                                  float* Out, int seq_q, int seq_k, int head_dim)
{
    cpu_attention(Q, K, V, Out, seq_q, seq_k, head_dim);
}

static void dequant(const float* x, long long rows, int d, float* out)
{
    std::vector<uint8_t> codes((size_t)rows * d), sc((size_t)rows * (d / 32));
    ref_quantize(x, rows, d, codes.data(), sc.data());
    static const float mag[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
    for (long long r = 0; r < rows; r++)
        for (int j = 0; j < d; j++) {
            uint8_t c = codes[(size_t)r * d + j] >> 2;
            float v = (c & 8) ? -mag[c & 7] : mag[c & 7];
            out[(size_t)r * d + j] = v == 0.f ? 0.f : std::ldexp(v, (int)sc[(size_t)r * (d / 32) + j / 32] - 127);
        }
}

// The reference's FP4 path on the CPU for `slices` contiguous slices:
// quantise Q and K with the reference quantiser, dequantise, then the
// reference's cpu_attention against FP32 V.  One slice per task on `threads`
// std::threads.
extern "C" void ref_fp4_attention(const float* Q, const float* K, const float* V, float* Out,
                                  int slices, int seq_q, int seq_k, int head_dim, int threads)
{
    if (threads < 1) threads = 1;
    if (threads > slices) threads = slices;
    size_t qn = (size_t)seq_q * head_dim, kn = (size_t)seq_k * head_dim;
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; t++)
        pool.emplace_back([=] {
            std::vector<float> qd(qn), kd(kn);
            for (int s = slices * t / threads; s < slices * (t + 1) / threads; s++) {
                dequant(Q + s * qn, seq_q, head_dim, qd.data());
                dequant(K + s * kn, seq_k, head_dim, kd.data());
                cpu_attention(qd.data(), kd.data(), V + s * kn, Out + s * qn, seq_q, seq_k, head_dim);
            }
        });
    for (auto& th : pool) th.join();
}
