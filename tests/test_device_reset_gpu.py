"""A device reset between calls.  cudaDeviceReset destroys the context, and
the library's module with it: on the next call the module is loaded again,
so its __device__ scratch (fp4attn_forward_noalloc) may sit at another
address and every kernel's dynamic shared-memory attribute is unset again.
The library keys those caches on the context, so the calls after a reset
must behave exactly like the calls before it.

A reset would also invalidate the test process's own torch context, so a
small host program (compiled here against include/fp4attn.h and the
library) does the work: forward through the no-allocation entry point and
through fp4attn_forward with a workspace, the log-sum-exp forward and the
backward, then cudaDeviceReset, then all of it again on fresh buffers.  It
exits 0 only if every call succeeded and the two rounds gave the same bytes
(dQ, summed by reductions in any order, to 1e-5 of its largest entry)."""
import pathlib
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = pathlib.Path(__file__).resolve().parents[1]

PROGRAM = r"""
#include "fp4attn.h"
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

static const int B = 1, H = 4, SQ = 200, SK = 333, D = 64;

struct Result { std::vector<float> o_noalloc, o_ws, dq, dk, dv; };

#define CK(x) do { int r_ = (x); if (r_) { fprintf(stderr, "%s -> %d: %s\n", #x, r_, fp4attn_last_error()); return 20; } } while (0)
#define CU(x) do { if ((x) != cudaSuccess) { fprintf(stderr, "%s failed\n", #x); return 21; } } while (0)

static int round_trip(Result& res)
{
    const size_t nq = size_t(B) * H * SQ * D, nk = size_t(B) * H * SK * D;
    std::vector<__half> q(nq), k(nk), v(nk), go(nq);
    unsigned s = 12345u;
    auto rnd = [&]() { s = s * 1664525u + 1013904223u; return ((s >> 8) & 0xFFFF) / 32768.0f - 1.0f; };
    for (auto& x : q) x = __float2half(2.0f * rnd());
    for (auto& x : k) x = __float2half(2.0f * rnd());
    for (auto& x : v) x = __float2half(rnd());
    for (auto& x : go) x = __float2half(rnd());
    __half *dq_in, *dk_in, *dv_in, *dgo, *dout16;
    float *dout, *lse, *gq, *gk, *gv;
    void* ws;
    const size_t ws_fwd = fp4attn_workspace_size(B, H, SQ, SK, D, FP4ATTN_F16);
    const size_t ws_bwd = fp4attn_backward_workspace_size(B, H, SQ, SK, D, FP4ATTN_F16);
    const size_t ws_bytes = ws_fwd > ws_bwd ? ws_fwd : ws_bwd;
    CU(cudaMalloc(&dq_in, nq * 2)); CU(cudaMalloc(&dk_in, nk * 2)); CU(cudaMalloc(&dv_in, nk * 2));
    CU(cudaMalloc(&dgo, nq * 2)); CU(cudaMalloc(&dout16, nq * 2)); CU(cudaMalloc(&dout, nq * 4));
    CU(cudaMalloc(&lse, size_t(B) * H * SQ * 4)); CU(cudaMalloc(&gq, nq * 4)); CU(cudaMalloc(&gk, nk * 4));
    CU(cudaMalloc(&gv, nk * 4)); CU(cudaMalloc(&ws, ws_bytes));
    CU(cudaMemcpy(dq_in, q.data(), nq * 2, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(dk_in, k.data(), nk * 2, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(dv_in, v.data(), nk * 2, cudaMemcpyHostToDevice));
    CU(cudaMemcpy(dgo, go.data(), nq * 2, cudaMemcpyHostToDevice));
    res.o_noalloc.resize(nq); res.o_ws.resize(nq); res.dq.resize(nq); res.dk.resize(nk); res.dv.resize(nk);
    CK(fp4attn_forward_noalloc(dq_in, dk_in, dv_in, dout, FP4ATTN_F16, FP4ATTN_F32, B, H, SQ, SK, D, 0.f,
                               FP4ATTN_SCALE_REFERENCE, nullptr));
    CK(fp4attn_status_query(nullptr));
    CU(cudaMemcpy(res.o_noalloc.data(), dout, nq * 4, cudaMemcpyDeviceToHost));
    CK(fp4attn_forward(dq_in, dk_in, dv_in, dout, FP4ATTN_F16, FP4ATTN_F32, B, H, SQ, SK, D, 0.f,
                       FP4ATTN_SCALE_REFERENCE, ws, ws_bytes, nullptr));
    CK(fp4attn_status_query(nullptr));
    CU(cudaMemcpy(res.o_ws.data(), dout, nq * 4, cudaMemcpyDeviceToHost));
    CK(fp4attn_forward_lse(dq_in, dk_in, dv_in, dout16, lse, FP4ATTN_F16, FP4ATTN_F16, B, H, SQ, SK, D, 0.f,
                           FP4ATTN_SCALE_REFERENCE, FP4ATTN_MASK_NONE, ws, ws_bytes, nullptr));
    CK(fp4attn_backward(dq_in, dk_in, dv_in, dout16, dgo, lse, gq, gk, gv, FP4ATTN_F16, FP4ATTN_F16, B, H, SQ, SK, D,
                        0.f, FP4ATTN_SCALE_REFERENCE, FP4ATTN_MASK_NONE, ws, ws_bytes, nullptr));
    CK(fp4attn_status_query(nullptr));
    CU(cudaMemcpy(res.dq.data(), gq, nq * 4, cudaMemcpyDeviceToHost));
    CU(cudaMemcpy(res.dk.data(), gk, nk * 4, cudaMemcpyDeviceToHost));
    CU(cudaMemcpy(res.dv.data(), gv, nk * 4, cudaMemcpyDeviceToHost));
    cudaFree(dq_in); cudaFree(dk_in); cudaFree(dv_in); cudaFree(dgo); cudaFree(dout16); cudaFree(dout);
    cudaFree(lse); cudaFree(gq); cudaFree(gk); cudaFree(gv); cudaFree(ws);
    return 0;
}

static bool same(const std::vector<float>& a, const std::vector<float>& b)
{
    return a.size() == b.size() && memcmp(a.data(), b.data(), a.size() * 4) == 0;
}

int main()
{
    Result r1, r2;
    if (int rc = round_trip(r1)) return rc;
    if (!same(r1.o_noalloc, r1.o_ws)) { fprintf(stderr, "noalloc != workspace before the reset\n"); return 2; }
    if (cudaDeviceReset() != cudaSuccess) { fprintf(stderr, "cudaDeviceReset failed\n"); return 3; }
    if (int rc = round_trip(r2)) return 100 + rc;
    if (!same(r2.o_noalloc, r2.o_ws)) { fprintf(stderr, "noalloc != workspace after the reset\n"); return 4; }
    if (!same(r1.o_ws, r2.o_ws)) { fprintf(stderr, "forward differs across the reset\n"); return 5; }
    if (!same(r1.dk, r2.dk) || !same(r1.dv, r2.dv)) { fprintf(stderr, "dK / dV differ across the reset\n"); return 6; }
    float mx = 0.f, diff = 0.f;
    for (size_t i = 0; i < r1.dq.size(); i++) {
        mx = fmaxf(mx, fabsf(r1.dq[i]));
        diff = fmaxf(diff, fabsf(r1.dq[i] - r2.dq[i]));
    }
    if (!(mx > 0.f) || diff > 1e-5f * mx) { fprintf(stderr, "dQ differs across the reset (%g of %g)\n", diff, mx); return 7; }
    printf("ok\n");
    return 0;
}
"""


def test_calls_after_a_device_reset_match_the_calls_before(fa, cuda, tmp_path):
    src = tmp_path / "reset.cpp"
    src.write_text(PROGRAM)
    exe = tmp_path / "reset"
    libdir = str(fa.lib_path().parent)
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", str(ROOT / "include"), "-I", "/usr/local/cuda/include",
                    str(src), "-L", libdir, "-lfp4attn", "-L", "/usr/local/cuda/lib64", "-lcudart",
                    f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, (r.returncode, r.stderr)
    assert r.stdout.strip() == "ok"
