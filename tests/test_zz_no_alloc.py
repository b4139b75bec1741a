"""fp4attn_forward_noalloc: the forward pass for callers that cannot allocate
device memory (work done during CUDA graph capture, runtimes that own all
device memory, loops that must not block on an allocation).  It must give
the same result as fp4attn_forward with a caller workspace, including on a
second call that reuses the scratch the first call left behind.

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


def _noalloc(fa, Q, K, V, out):
    B, H, Sq, D = Q.shape
    Sk = K.shape[2]
    rc = _bind(fa)(Q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(), fa.F16,
                   fa.F32 if out.dtype == torch.float32 else fa.F16, B, H, Sq, Sk, D, 0.0, fa.SCALE_REFERENCE,
                   torch.cuda.current_stream().cuda_stream)
    return rc


def _inputs(seed, B, H, Sq, Sk, D):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, H, s, D, generator=g).half().cuda() for s in (Sq, Sk, Sk)]


def test_two_calls_match_the_workspace_entry_point(fa, cuda):
    shapes = [(1, 8, 300, 1000, 128), (2, 4, 64, 200, 64)]
    for call, (B, H, Sq, Sk, D) in enumerate(shapes):
        Q, K, V = _inputs(100 + call, B, H, Sq, Sk, D)
        out = torch.full((B, H, Sq, D), float("nan"), dtype=torch.float32, device="cuda")
        assert _noalloc(fa, Q, K, V, out) == fa.OK, fa.lib().fp4attn_last_error()
        assert fa.status_query() == fa.OK
        want = fa.fused_fp4_attention(Q, K, V, out_dtype=torch.float32)
        assert fa.status_query() == fa.OK
        got, ref = out.cpu().numpy(), want.cpu().numpy()
        assert np.isfinite(got).all()
        assert oracle.cosine(got, ref) >= COS_MIN
        assert float(np.abs(got - ref).max()) <= MAXABS


def test_rejects_problems_larger_than_the_scratch(fa, cuda):
    # 64 slices x 8192 keys x d256 needs ~70 MB of workspace: above the 64 MiB scratch.
    Q = torch.zeros(1, 64, 128, 256, dtype=torch.float16, device="cuda")
    K = torch.zeros(1, 64, 8192, 256, dtype=torch.float16, device="cuda")
    out = torch.empty(1, 64, 128, 256, dtype=torch.float32, device="cuda")
    assert fa.workspace_size(1, 64, 128, 8192, 256) > 64 << 20
    assert _noalloc(fa, Q, K, K, out) == fa.EWORKSPACE
    assert b"bytes of scratch" in fa.lib().fp4attn_last_error()
