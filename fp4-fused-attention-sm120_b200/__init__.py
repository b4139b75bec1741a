"""Host-side Python mirror of the reference's FP4 fused attention interface.

The reference (florianmattana/fp4-fused-attention-sm120) is a CUDA header:
``fused_fp4_attention<HEAD_DIM><<<batch*heads, 128>>>(Q, K, Out, V, seq_q,
seq_k, heads)`` (common.h:68-77) plus the encoders ``encode_fp4_e2m1`` and
``compute_scale_ue8m0`` (common.h:21-48).  This module binds the C ABI of
``libfp4attn.so`` (include/fp4attn.h) with ctypes and exposes the same
operations on torch CUDA tensors.  Torch is used for device memory and streams
only; all arithmetic runs in the library's sm_100a kernels.  There is no CPU
fallback: if the library is missing or the device is not sm_100, calls raise.
"""
from __future__ import annotations

import ctypes
import os
import pathlib

__all__ = [
    "BLOCK_ELEMENT", "BQ", "Fp4AttnError", "lib", "lib_path", "quantize", "workspace_size",
    "fused_fp4_attention", "fused_fp4_attention_into", "debug_scores", "status_query",
    "selftest_timeout", "selftest_abort", "supported_head_dims", "prepare", "attend", "shard_range", "SCALE_REFERENCE", "SCALE_OCP",
    "F32", "F16", "MASK_NONE", "MASK_CAUSAL", "fused_fp4_attention_lse", "backward_workspace_size",
    "fp4_attention_backward", "FP4Attention", "fp4_attention", "selftest_backward_abort",
]

BLOCK_ELEMENT = 32  # common.h:15
BQ = 64             # common.h:18

OK, EINVAL, EUNSUPPORTED, ECUDA, ETIMEOUT, EWORKSPACE = range(6)
F32, F16 = 0, 1
SCALE_REFERENCE, SCALE_OCP = 0, 1
LAYOUT_ROWMAJOR = 0
MASK_NONE = 0    # every query sees every key (the reference's only mode)
MASK_CAUSAL = 1  # query i sees keys j <= i + seq_k - seq_q (bottom-right aligned)

_HERE = pathlib.Path(__file__).resolve().parent
_LIB = None


def lib_path() -> pathlib.Path:
    return pathlib.Path(os.environ.get("FP4ATTN_LIB", _HERE / "libfp4attn.so"))


class Fp4AttnError(RuntimeError):
    def __init__(self, code: int, where: str, detail: str = ""):
        self.code = code
        msg = f"{where}: {_error_string(code)} (code {code})"
        if detail:
            msg += f": {detail}"
        super().__init__(msg)


def lib() -> ctypes.CDLL:
    """Load libfp4attn.so (built by __graft_entry__.build or `make -C csrc`)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    p = lib_path()
    if not p.exists():
        raise ImportError(f"{p} is missing: build it with `make -C {_HERE / 'csrc'}` "
                          "(there is no fallback implementation)")
    L = ctypes.CDLL(str(p))
    vp, i32, i64, sz, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_float
    L.fp4attn_quantize.argtypes = [vp, i32, i64, i32, vp, vp, i32, i32, vp]
    L.fp4attn_quantize.restype = i32
    L.fp4attn_workspace_size.argtypes = [i32] * 6
    L.fp4attn_workspace_size.restype = sz
    L.fp4attn_forward.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, f32, i32, vp, sz, vp]
    L.fp4attn_forward.restype = i32
    L.fp4attn_prepare.argtypes = [vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, vp, sz, vp]
    L.fp4attn_prepare.restype = i32
    L.fp4attn_attend.argtypes = [vp, vp, i32, i32, i32, i32, i32, i32, i32, f32, vp, sz, vp]
    L.fp4attn_attend.restype = i32
    L.fp4attn_forward_fused_q.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, f32, i32, vp, sz, vp]
    L.fp4attn_forward_fused_q.restype = i32
    L.fp4attn_forward_masked.argtypes = [vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, f32, i32, i32, vp, sz, vp]
    L.fp4attn_forward_masked.restype = i32
    L.fp4attn_attend_masked.argtypes = [vp, vp, i32, i32, i32, i32, i32, i32, i32, f32, i32, vp, sz, vp]
    L.fp4attn_attend_masked.restype = i32
    L.fp4attn_debug_scores.argtypes = [vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, vp, sz, vp]
    L.fp4attn_debug_scores.restype = i32
    L.fp4attn_forward_lse.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, i32, f32, i32, i32, vp, sz, vp]
    L.fp4attn_forward_lse.restype = i32
    L.fp4attn_backward_workspace_size.argtypes = [i32] * 6
    L.fp4attn_backward_workspace_size.restype = sz
    L.fp4attn_backward.argtypes = [vp] * 9 + [i32] * 7 + [f32, i32, i32, vp, sz, vp]
    L.fp4attn_backward.restype = i32
    L.fp4attn_backward_prepare.argtypes = [vp] * 7 + [i32] * 8 + [vp, sz, vp]
    L.fp4attn_backward_prepare.restype = i32
    L.fp4attn_backward_attend.argtypes = [vp] * 5 + [i32] * 6 + [f32, i32, vp, sz, vp]
    L.fp4attn_backward_attend.restype = i32
    L.fp4attn_selftest_backward_abort.argtypes = [vp] * 9 + [i32] * 4 + [vp, sz, ctypes.c_uint, vp]
    L.fp4attn_selftest_backward_abort.restype = i32
    L.fp4attn_status_query.argtypes = [vp]
    L.fp4attn_status_query.restype = i32
    L.fp4attn_selftest_timeout.argtypes = [ctypes.c_uint, vp]
    L.fp4attn_selftest_timeout.restype = i32
    L.fp4attn_selftest_abort.argtypes = [vp, vp, i32, i32, i32, i32, vp, sz, ctypes.c_uint, vp]
    L.fp4attn_selftest_abort.restype = i32
    L.fp4attn_selftest_exp2.argtypes = [vp, vp, i64, vp]
    L.fp4attn_selftest_exp2.restype = i32
    L.fp4attn_error_string.argtypes = [i32]
    L.fp4attn_error_string.restype = ctypes.c_char_p
    L.fp4attn_last_error.argtypes = []
    L.fp4attn_last_error.restype = ctypes.c_char_p
    L.fp4attn_supported_head_dims.argtypes = [ctypes.POINTER(i32), i32]
    L.fp4attn_supported_head_dims.restype = i32
    _LIB = L
    return L


def _error_string(code: int) -> str:
    try:
        return lib().fp4attn_error_string(code).decode()
    except ImportError:
        return "error"


def _check(rc: int, where: str) -> None:
    if rc != OK:
        raise Fp4AttnError(rc, where, lib().fp4attn_last_error().decode())


def _torch():
    import torch
    return torch


def _dtype_code(t) -> int:
    torch = _torch()
    if t.dtype == torch.float16:
        return F16
    if t.dtype == torch.float32:
        return F32
    raise TypeError(f"unsupported dtype {t.dtype}; use float16 or float32")


def _stream_ptr(stream) -> int:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def supported_head_dims() -> list[int]:
    L = lib()
    n = L.fp4attn_supported_head_dims(None, 0)
    arr = (ctypes.c_int * n)()
    L.fp4attn_supported_head_dims(arr, n)
    return list(arr)


def workspace_size(batch: int, heads: int, seq_q: int, seq_k: int, head_dim: int, in_dtype: int = F16) -> int:
    return int(lib().fp4attn_workspace_size(batch, heads, seq_q, seq_k, head_dim, in_dtype))


def _scale_mode(mode) -> int:
    if mode in (SCALE_REFERENCE, "reference", "ref"):
        return SCALE_REFERENCE
    if mode in (SCALE_OCP, "ocp"):
        return SCALE_OCP
    raise ValueError(f"unknown scale_mode {mode!r}")


def quantize(x, scale_mode="reference", stream=None):
    """E2M1 codes (two per byte, element 2i in the low nibble) and UE8M0 scales
    (one per 32 elements) of a [..., head_dim] CUDA tensor, bit-exact with the
    reference quantiser (common.h:21-48, :115-123)."""
    torch = _torch()
    if not x.is_cuda or not x.is_contiguous():
        raise ValueError("x must be a contiguous CUDA tensor")
    d = x.shape[-1]
    rows = x.numel() // d if d else 0
    codes = torch.empty(x.shape[:-1] + (d // 2,), dtype=torch.uint8, device=x.device)
    scales = torch.empty(x.shape[:-1] + (d // 32,), dtype=torch.uint8, device=x.device)
    rc = lib().fp4attn_quantize(x.data_ptr(), _dtype_code(x), rows, d, codes.data_ptr(), scales.data_ptr(),
                                _scale_mode(scale_mode), LAYOUT_ROWMAJOR, _stream_ptr(stream))
    _check(rc, "fp4attn_quantize")
    return codes, scales


def _check_qkv(Q, K, V):
    for name, t in (("Q", Q), ("K", K)) + ((("V", V),) if V is not None else ()):
        if not t.is_cuda or not t.is_contiguous() or t.dim() != 4:
            raise ValueError(f"{name} must be a contiguous 4-D CUDA tensor [batch, heads, seq, head_dim]")
    B, H, Sq, D = Q.shape
    if K.shape[:2] != (B, H) or K.shape[3] != D:
        raise ValueError("K must be [batch, heads, seq_k, head_dim] matching Q")
    if V is not None and V.shape != K.shape:
        raise ValueError("V must have K's shape")
    if Q.dtype != K.dtype or (V is not None and V.dtype != Q.dtype):
        raise ValueError("Q, K and V must share a dtype")
    return B, H, Sq, K.shape[2], D


def fused_fp4_attention_into(Q, K, V, out, workspace, softmax_scale=None, scale_mode="reference", stream=None,
                             causal=False, fuse_q=False):
    """Launch into caller-provided `out` and `workspace` (uint8 CUDA tensor of
    at least workspace_size(...) bytes); no allocation, async on `stream`.
    causal=True applies the bottom-right causal mask (fp4attn_forward_masked);
    fuse_q=True quantises Q inside the attention kernel
    (fp4attn_forward_fused_q, same result)."""
    if causal and fuse_q:
        raise ValueError("fuse_q has no causal variant")
    B, H, Sq, Sk, D = _check_qkv(Q, K, V)
    if out.shape != Q.shape or not out.is_contiguous():
        raise ValueError("out must be contiguous with Q's shape")
    args = (Q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(), _dtype_code(Q), _dtype_code(out), B, H, Sq, Sk,
            D, float(softmax_scale or 0.0), _scale_mode(scale_mode))
    tail = (workspace.data_ptr(), workspace.numel(), _stream_ptr(stream))
    if causal:
        _check(lib().fp4attn_forward_masked(*args, MASK_CAUSAL, *tail), "fp4attn_forward_masked")
    elif fuse_q:
        _check(lib().fp4attn_forward_fused_q(*args, *tail), "fp4attn_forward_fused_q")
    else:
        _check(lib().fp4attn_forward(*args, *tail), "fp4attn_forward")
    return out


def prepare(Q, K, V, workspace, scale_mode="reference", stream=None):
    """Quantise Q and K (and stage V) into `workspace` (fp4attn_prepare)."""
    B, H, Sq, Sk, D = _check_qkv(Q, K, V)
    rc = lib().fp4attn_prepare(Q.data_ptr(), K.data_ptr(), V.data_ptr(), _dtype_code(Q), B, H, Sq, Sk, D,
                               _scale_mode(scale_mode), workspace.data_ptr(), workspace.numel(), _stream_ptr(stream))
    _check(rc, "fp4attn_prepare")


def attend(V, out, workspace, in_dtype, batch, heads, seq_q, seq_k, head_dim, softmax_scale=None, stream=None,
           causal=False):
    """The attention kernel on a prepared workspace (fp4attn_attend, or
    fp4attn_attend_masked with the causal mask)."""
    head = (V.data_ptr(), out.data_ptr(), in_dtype, _dtype_code(out), batch, heads, seq_q, seq_k, head_dim,
            float(softmax_scale or 0.0))
    tail = (workspace.data_ptr(), workspace.numel(), _stream_ptr(stream))
    if causal:
        _check(lib().fp4attn_attend_masked(*head, MASK_CAUSAL, *tail), "fp4attn_attend_masked")
    else:
        _check(lib().fp4attn_attend(*head, *tail), "fp4attn_attend")
    return out


def shard_range(n_slices: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous (batch x head) slice range [lo, hi) of `rank` out of
    `world` GPUs.  Slices are independent, and in [batch, heads, seq,
    head_dim] layout a slice range is one contiguous byte range of Q, K, V and
    Out, so a shard needs no data from any other GPU."""
    if world < 1 or not 0 <= rank < world or n_slices < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(n_slices, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def fused_fp4_attention(Q, K, V, out_dtype=None, softmax_scale=None, scale_mode="reference", stream=None,
                        causal=False, fuse_q=False):
    """softmax(Q K^T * scale) V with FP4 (E2M1 + UE8M0/32) Q and K: the
    reference kernel fused_fp4_attention<HEAD_DIM> (common.h:68-328) for
    [batch, heads, seq, head_dim] tensors of any seq_q / seq_k.  causal=True
    adds the bottom-right causal mask (not in the reference)."""
    torch = _torch()
    B, H, Sq, Sk, D = _check_qkv(Q, K, V)
    out = torch.empty((B, H, Sq, D), dtype=out_dtype or Q.dtype, device=Q.device)
    ws = torch.empty(workspace_size(B, H, Sq, Sk, D, _dtype_code(Q)), dtype=torch.uint8, device=Q.device)
    return fused_fp4_attention_into(Q, K, V, out, ws, softmax_scale, scale_mode, stream, causal, fuse_q)


def fused_fp4_attention_lse(Q, K, V, out_dtype=None, softmax_scale=None, scale_mode="reference", stream=None,
                            causal=False):
    """fused_fp4_attention that also returns, per query row, the natural-log
    log-sum-exp of the scaled scores (FP32 [batch, heads, seq_q];
    fp4attn_forward_lse) -- what the backward pass needs.  head_dim 32 to 128."""
    torch = _torch()
    B, H, Sq, Sk, D = _check_qkv(Q, K, V)
    out = torch.empty((B, H, Sq, D), dtype=out_dtype or Q.dtype, device=Q.device)
    lse = torch.empty((B, H, Sq), dtype=torch.float32, device=Q.device)
    ws = torch.empty(workspace_size(B, H, Sq, Sk, D, _dtype_code(Q)), dtype=torch.uint8, device=Q.device)
    rc = lib().fp4attn_forward_lse(Q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(), lse.data_ptr(),
                                   _dtype_code(Q), _dtype_code(out), B, H, Sq, Sk, D, float(softmax_scale or 0.0),
                                   _scale_mode(scale_mode), MASK_CAUSAL if causal else MASK_NONE, ws.data_ptr(),
                                   ws.numel(), _stream_ptr(stream))
    _check(rc, "fp4attn_forward_lse")
    return out, lse


def backward_workspace_size(batch: int, heads: int, seq_q: int, seq_k: int, head_dim: int, in_dtype: int = F16) -> int:
    return int(lib().fp4attn_backward_workspace_size(batch, heads, seq_q, seq_k, head_dim, in_dtype))


def fp4_attention_backward(Q, K, V, out, dout, lse, softmax_scale=None, scale_mode="reference", stream=None,
                           causal=False, workspace=None):
    """Gradients (dQ, dK, dV), FP32, of the FP4 fused attention
    (fp4attn_backward): Q, K, V and dout of one dtype (float16 or float32),
    the forward's `out` (FP16 or FP32) and `lse` from fused_fp4_attention_lse
    with the same scale, scale mode and mask.  The quantiser is a
    straight-through estimator."""
    torch = _torch()
    B, H, Sq, Sk, D = _check_qkv(Q, K, V)
    if dout.dtype != Q.dtype:
        raise TypeError("dout must have Q's dtype")
    if out.shape != Q.shape or dout.shape != Q.shape or not out.is_contiguous() or not dout.is_contiguous():
        raise ValueError("out and dout must be contiguous with Q's shape")
    if lse.shape != (B, H, Sq) or lse.dtype != torch.float32 or not lse.is_contiguous():
        raise ValueError("lse must be a contiguous float32 [batch, heads, seq_q] tensor")
    dq = torch.empty(Q.shape, dtype=torch.float32, device=Q.device)
    dk = torch.empty(K.shape, dtype=torch.float32, device=Q.device)
    dv = torch.empty(V.shape, dtype=torch.float32, device=Q.device)
    if workspace is None:
        workspace = torch.empty(backward_workspace_size(B, H, Sq, Sk, D, _dtype_code(Q)), dtype=torch.uint8,
                                device=Q.device)
    rc = lib().fp4attn_backward(Q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(), dout.data_ptr(),
                                lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), _dtype_code(Q),
                                _dtype_code(out), B, H,
                                Sq, Sk, D, float(softmax_scale or 0.0), _scale_mode(scale_mode),
                                MASK_CAUSAL if causal else MASK_NONE, workspace.data_ptr(), workspace.numel(),
                                _stream_ptr(stream))
    _check(rc, "fp4attn_backward")
    return dq, dk, dv


_FP4_ATTENTION_FN = None


def _autograd_function():
    global _FP4_ATTENTION_FN
    if _FP4_ATTENTION_FN is not None:
        return _FP4_ATTENTION_FN
    torch = _torch()

    class FP4Attention(torch.autograd.Function):
        """Differentiable FP4 fused attention: forward = fused_fp4_attention_lse,
        backward = fp4_attention_backward (straight-through quantiser)."""

        @staticmethod
        def forward(ctx, Q, K, V, softmax_scale, causal):
            out, lse = fused_fp4_attention_lse(Q, K, V, softmax_scale=softmax_scale, causal=causal)
            ctx.save_for_backward(Q, K, V, out, lse)
            ctx.softmax_scale, ctx.causal = softmax_scale, causal
            return out

        @staticmethod
        def backward(ctx, dout):
            Q, K, V, out, lse = ctx.saved_tensors
            dq, dk, dv = fp4_attention_backward(Q, K, V, out, dout.to(Q.dtype).contiguous(), lse,
                                                softmax_scale=ctx.softmax_scale, causal=ctx.causal)
            return dq.to(Q.dtype), dk.to(K.dtype), dv.to(V.dtype), None, None

    _FP4_ATTENTION_FN = FP4Attention
    return FP4Attention


def __getattr__(name):
    if name == "FP4Attention":
        return _autograd_function()
    raise AttributeError(name)


def fp4_attention(Q, K, V, softmax_scale=None, causal=False):
    """softmax(Q K^T * scale) V with FP4 Q, K that autograd can differentiate
    (float16 or float32 [batch, heads, seq, head_dim], head_dim 32 to 128)."""
    return _autograd_function().apply(Q, K, V, softmax_scale, causal)


def debug_scores(Q, K, scale_mode="reference", stream=None):
    """S = Q K^T on the quantised inputs, FP32 [batch, heads, seq_q, seq_k]
    (the reference's debug_mma, common.h:331-398, for whole problems)."""
    torch = _torch()
    B, H, Sq, Sk, D = _check_qkv(Q, K, None)
    S = torch.empty((B, H, Sq, Sk), dtype=torch.float32, device=Q.device)
    ws = torch.empty(workspace_size(B, H, Sq, Sk, D, _dtype_code(Q)), dtype=torch.uint8, device=Q.device)
    rc = lib().fp4attn_debug_scores(Q.data_ptr(), K.data_ptr(), S.data_ptr(), _dtype_code(Q), B, H, Sq, Sk, D,
                                    _scale_mode(scale_mode), ws.data_ptr(), ws.numel(), _stream_ptr(stream))
    _check(rc, "fp4attn_debug_scores")
    return S


def selftest_exp2(x, stream=None):
    """2^x on the device by the softmax's FMA-pipe polynomial (test hook)."""
    torch = _torch()
    if x.dtype != torch.float32 or not x.is_cuda or not x.is_contiguous() or x.numel() % 2:
        raise ValueError("x must be a contiguous float32 CUDA tensor with an even number of elements")
    y = torch.empty_like(x)
    _check(lib().fp4attn_selftest_exp2(x.data_ptr(), y.data_ptr(), x.numel(), _stream_ptr(stream)),
           "fp4attn_selftest_exp2")
    return y


def status_query(stream=None) -> int:
    """Synchronise `stream` and return (and clear) the device error word."""
    return int(lib().fp4attn_status_query(_stream_ptr(stream)))


def selftest_abort(V, out, workspace, batch, heads, seq_q, seq_k, timeout_us: int = 20000, stream=None) -> int:
    """Run the attention kernel's abort self-test (fp4attn_selftest_abort) on a
    workspace prepared for this head_dim-64 FP16 problem; returns
    status_query() (FP4ATTN_ETIMEOUT when the failure path ran)."""
    _check(lib().fp4attn_selftest_abort(V.data_ptr(), out.data_ptr(), batch, heads, seq_q, seq_k,
                                        workspace.data_ptr(), workspace.numel(), timeout_us, _stream_ptr(stream)),
           "fp4attn_selftest_abort")
    return status_query(stream)


def selftest_backward_abort(Q, K, V, out, dout, lse, dq, dk, dv, workspace, timeout_us: int = 20000,
                            stream=None) -> int:
    """Run the backward kernel's abort self-test (fp4attn_selftest_backward_abort)
    on a head_dim-64 FP16 problem; returns status_query() (FP4ATTN_ETIMEOUT
    when the failure path ran)."""
    B, H, Sq, Sk, D = _check_qkv(Q, K, V)
    _check(lib().fp4attn_selftest_backward_abort(Q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(),
                                                 dout.data_ptr(), lse.data_ptr(), dq.data_ptr(), dk.data_ptr(),
                                                 dv.data_ptr(), B, H, Sq, Sk, workspace.data_ptr(), workspace.numel(),
                                                 timeout_us, _stream_ptr(stream)),
           "fp4attn_selftest_backward_abort")
    return status_query(stream)


def selftest_timeout(timeout_us: int = 2000, stream=None) -> int:
    """Run the bounded-wait expiry test kernel; returns status_query()."""
    _check(lib().fp4attn_selftest_timeout(timeout_us, _stream_ptr(stream)), "fp4attn_selftest_timeout")
    return status_query(stream)
