"""The reference-order C++ launcher (include/fp4_fused_attention.h) run on the
GPU the way the reference's callers run its kernel (tests/test_attention.cu:
88-105, 150-161): FP32 buffers from cudaMalloc in [batch, heads, seq, head_dim]
layout, arguments (Q, K, Out, V, seq_q, seq_k, heads) then batch, the default
stream.  A small host program is compiled against the header and the library
here, reads its inputs from a file and writes the output back."""
import pathlib
import subprocess

import numpy as np
import pytest

import golden_inputs as gi
import oracle

pytestmark = pytest.mark.gpu

ROOT = pathlib.Path(__file__).resolve().parents[1]
COS_MIN = 0.9999
MAXABS = 2e-2

PROGRAM = r"""
#include "fp4_fused_attention.h"
#include <cstdio>
#include <cstdlib>
#include <vector>

template <int D>
static int run(int B, int H, int sq, int sk, bool causal, const char* in_path, const char* out_path)
{
    const size_t nq = size_t(B) * H * sq * D, nk = size_t(B) * H * sk * D;
    std::vector<float> q(nq), k(nk), v(nk), o(nq);
    FILE* f = fopen(in_path, "rb");
    if (!f || fread(q.data(), 4, nq, f) != nq || fread(k.data(), 4, nk, f) != nk || fread(v.data(), 4, nk, f) != nk)
        return 10;
    fclose(f);
    float *dq, *dk, *dv, *dout;
    if (cudaMalloc(&dq, nq * 4) || cudaMalloc(&dk, nk * 4) || cudaMalloc(&dv, nk * 4) || cudaMalloc(&dout, nq * 4))
        return 11;
    cudaMemcpy(dq, q.data(), nq * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dk, k.data(), nk * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dv, v.data(), nk * 4, cudaMemcpyHostToDevice);
    int rc = fused_fp4_attention_launch<D>(dq, dk, dout, dv, sq, sk, H, B, 0, causal);
    if (rc != FP4ATTN_OK) {
        fprintf(stderr, "launch: %s: %s\n", fp4attn_error_string(rc), fp4attn_last_error());
        return 12;
    }
    if (cudaDeviceSynchronize() != cudaSuccess) return 13;
    if (fp4attn_status_query(0) != FP4ATTN_OK) return 14;
    cudaMemcpy(o.data(), dout, nq * 4, cudaMemcpyDeviceToHost);
    cudaFree(dq); cudaFree(dk); cudaFree(dv); cudaFree(dout);
    FILE* g = fopen(out_path, "wb");
    if (!g || fwrite(o.data(), 4, nq, g) != nq) return 15;
    fclose(g);
    return 0;
}

int main(int argc, char** argv)
{
    if (argc != 9) return 1;
    const int d = atoi(argv[1]), B = atoi(argv[2]), H = atoi(argv[3]), sq = atoi(argv[4]), sk = atoi(argv[5]);
    const bool causal = atoi(argv[6]) != 0;
    switch (d) {
        case 64: return run<64>(B, H, sq, sk, causal, argv[7], argv[8]);
        case 128: return run<128>(B, H, sq, sk, causal, argv[7], argv[8]);
    }
    return 1;
}
"""


@pytest.fixture(scope="module")
def launcher(fa, tmp_path_factory):
    d = tmp_path_factory.mktemp("launcher")
    src = d / "launcher.cpp"
    src.write_text(PROGRAM)
    libdir = str(fa.lib_path().parent)
    exe = d / "launcher"
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", str(ROOT / "include"), "-I", "/usr/local/cuda/include",
                    str(src), "-L", libdir, "-lfp4attn", "-L", "/usr/local/cuda/lib64", "-lcudart",
                    f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    return exe


def _run(launcher, tmp_path, Q, K, V, B, H, causal=False):
    d, sq, sk = Q.shape[-1], Q.shape[-2], K.shape[-2]
    inp, out = tmp_path / "in.bin", tmp_path / "out.bin"
    with open(inp, "wb") as f:
        for a in (Q, K, V):
            f.write(np.ascontiguousarray(a, dtype=np.float32).tobytes())
    r = subprocess.run([str(launcher), str(d), str(B), str(H), str(sq), str(sk), str(int(causal)), str(inp),
                        str(out)], capture_output=True, text=True)
    assert r.returncode == 0, (r.returncode, r.stderr)
    return np.fromfile(out, dtype=np.float32).reshape(B * H, sq, d)


def _close(got, want):
    assert np.isfinite(got).all()
    cos, err = oracle.cosine(got, want), float(np.abs(got - want).max())
    assert cos >= COS_MIN and err <= MAXABS, (cos, err)


def test_reference_fixture_through_the_launcher(cuda, launcher, tmp_path, golden_dir):
    """tests/test_attention.cu's multi-head case (B2 H4, seq_q 64, seq_k 128,
    head_dim 128, srand(42) discrete values) against the golden output of the
    reference's own CPU attention."""
    d, sk, B, H = gi.DISCRETE_CASES["multi_b2_h4_sk128"]
    Q, K, V = gi.discrete_inputs(d, sk, B, H)
    got = _run(launcher, tmp_path, Q, K, V, B, H)
    _close(got, np.load(golden_dir / "discrete_multi_b2_h4_sk128.npz")["out"])
    _close(got, oracle.fp4_attention(Q, K, V))


@pytest.mark.parametrize("d,B,H,sq,sk,causal", [(64, 1, 3, 100, 300, False), (128, 2, 2, 200, 333, True)])
def test_random_inputs_through_the_launcher(cuda, launcher, tmp_path, d, B, H, sq, sk, causal):
    rng = np.random.default_rng(d + sq)
    Q, K, V = (rng.standard_normal((B * H, s, d), dtype=np.float32) for s in (sq, sk, sk))
    got = _run(launcher, tmp_path, Q, K, V, B, H, causal)
    _close(got, oracle.fp4_attention(Q, K, V, causal=causal))
