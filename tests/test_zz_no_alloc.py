"""fp4attn_forward_noalloc: the forward pass for callers that cannot allocate
device memory (work done during CUDA graph capture, runtimes that own all
device memory, loops that must not block on an allocation).  It runs the same
kernels as fp4attn_forward with a caller workspace, so on the same inputs its
output must be the same bytes -- including on later calls that reuse the
scratch an earlier, larger call left behind -- and it must match the oracle at
the attention tests' tolerance.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test."""
import ctypes

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

COS_MIN = 0.9999   # same bars as the other attention tests
MAXABS = 2e-2


def _bind(fa):
    L = fa.lib()
    f = L.fp4attn_forward_noalloc
    vp, i32, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    f.argtypes = [vp, vp, vp, vp] + [i32] * 7 + [f32, i32, vp]
    f.restype = i32
    return f


def _dt(fa, t):
    return fa.F32 if t.dtype == torch.float32 else fa.F16


def _noalloc(fa, Q, K, V, out):
    B, H, Sq, D = Q.shape
    Sk = K.shape[2]
    return _bind(fa)(Q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(), _dt(fa, Q), _dt(fa, out), B, H, Sq,
                     Sk, D, 0.0, fa.SCALE_REFERENCE, torch.cuda.current_stream().cuda_stream)


def _inputs(seed, B, H, Sq, Sk, D, dtype):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, H, s, D, generator=g).half().to(dtype).cuda() for s in (Sq, Sk, Sk)]


def _check_call(fa, seed, shape, in_dtype, out_dtype):
    B, H, Sq, Sk, D = shape
    Q, K, V = _inputs(seed, B, H, Sq, Sk, D, in_dtype)
    out = torch.full((B, H, Sq, D), float("nan"), dtype=out_dtype, device="cuda")
    assert _noalloc(fa, Q, K, V, out) == fa.OK, fa.lib().fp4attn_last_error()
    assert fa.status_query() == fa.OK
    # The workspace entry point on the same inputs: the same kernels, so the
    # same bytes.
    want = fa.fused_fp4_attention(Q, K, V, out_dtype=out_dtype)
    assert fa.status_query() == fa.OK
    assert torch.equal(out, want)
    ref = oracle.fp4_attention(Q[0].float().cpu().numpy(), K[0].float().cpu().numpy(), V[0].float().cpu().numpy())
    if out_dtype == torch.float16:
        ref = ref.astype(np.float16).astype(np.float32)
    got = out[0].float().cpu().numpy()
    assert np.isfinite(got).all()
    assert oracle.cosine(got, ref) >= COS_MIN
    assert float(np.abs(got - ref).max()) <= MAXABS


@pytest.mark.parametrize("in_dtype", [torch.float16, torch.float32])
def test_two_calls_match_the_workspace_entry_point(fa, cuda, in_dtype):
    """A larger call, then a smaller one with the other output type, on the
    scratch the first call left behind.  FP32 input also stages an FP16 copy
    of V in the scratch."""
    _check_call(fa, 100, (1, 8, 300, 1000, 128), in_dtype, torch.float32)
    _check_call(fa, 101, (1, 4, 64, 200, 64), in_dtype, torch.float16)


def test_rejects_problems_larger_than_the_scratch(fa, cuda):
    # 64 slices x 8192 keys x d256 needs ~70 MB of workspace: above the 64 MiB scratch.
    Q = torch.zeros(1, 64, 128, 256, dtype=torch.float16, device="cuda")
    K = torch.zeros(1, 64, 8192, 256, dtype=torch.float16, device="cuda")
    out = torch.empty(1, 64, 128, 256, dtype=torch.float32, device="cuda")
    assert fa.workspace_size(1, 64, 128, 8192, 256) > 64 << 20
    assert _noalloc(fa, Q, K, K, out) == fa.EWORKSPACE
    assert b"bytes of scratch" in fa.lib().fp4attn_last_error()
