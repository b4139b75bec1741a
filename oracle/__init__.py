"""ctypes bindings of the checker libraries (TEST INFRASTRUCTURE ONLY).

liboracle.so is this repository's C restatement of the reference path
(oracle/fp4attn_oracle.c); _ref/libfp4ref.so is the reference's own quantiser
and CPU attention compiled from its sources by oracle/Makefile.  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg use this module, and
only as the checker / CPU baseline -- never on the product path.
"""
from __future__ import annotations

import ctypes
import pathlib

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libfp4ref.so"

_f32 = np.ctypeslib.ndpointer(np.float32, flags="C")
_u8 = np.ctypeslib.ndpointer(np.uint8, flags="C")
_i32 = np.ctypeslib.ndpointer(np.int32, flags="C")
_o = None
_r = None


def oracle_lib() -> ctypes.CDLL:
    global _o
    if _o is None:
        L = ctypes.CDLL(str(ORACLE_SO))
        c = ctypes
        L.oracle_encode_e2m1.argtypes = [c.c_float]
        L.oracle_encode_e2m1.restype = c.c_uint8
        L.oracle_scale_ue8m0.argtypes = [_f32, c.c_int]
        L.oracle_scale_ue8m0.restype = c.c_uint8
        L.oracle_quantize.argtypes = [_f32, c.c_int64, c.c_int, _u8, _u8, c.c_int]
        L.oracle_dequantize.argtypes = [_u8, _u8, c.c_int64, c.c_int, _f32]
        L.oracle_attention.argtypes = [_f32, _f32, _f32, _f32, c.c_int, c.c_int, c.c_int, c.c_float]
        L.oracle_fp4_attention.argtypes = [_f32, _f32, _f32, _f32] + [c.c_int] * 4 + [c.c_float, c.c_int, c.c_int]
        L.oracle_fp4_attention_rows.argtypes = [_f32, _f32, _f32, _f32, c.c_int, _i32, _i32, c.c_int, c.c_int,
                                                c.c_int, c.c_float, c.c_int]
        L.oracle_attention_causal.argtypes = [_f32, _f32, _f32, _f32, c.c_int, c.c_int, c.c_int, c.c_float,
                                              c.c_int, c.c_int]
        L.oracle_fp4_attention_causal.argtypes = ([_f32, _f32, _f32, _f32] + [c.c_int] * 4 +
                                                  [c.c_float, c.c_int, c.c_int])
        L.oracle_fp4_attention_slice.argtypes = ([_f32, _f32, _f32, _f32] + [c.c_int] * 3 +
                                                 [c.c_float, c.c_int, c.c_int])
        L.oracle_fp4_scores.argtypes = [_f32, _f32, _f32, c.c_int, c.c_int, c.c_int, c.c_int]
        L.oracle_fp4_attention_backward.argtypes = ([_f32] * 7 + [c.c_int] * 4 + [c.c_float] +
                                                    [c.c_int] * 3)
        L.oracle_fp4_attention_lse.argtypes = [_f32, _f32, _f32] + [c.c_int] * 4 + [c.c_float, c.c_int, c.c_int]
        L.oracle_cosine.argtypes = [_f32, _f32, c.c_int64]
        L.oracle_cosine.restype = c.c_double
        _o = L
    return _o


def ref_available() -> bool:
    return REF_SO.exists()


def ref_lib() -> ctypes.CDLL:
    global _r
    if _r is None:
        L = ctypes.CDLL(str(REF_SO))
        c = ctypes
        L.ref_encode_fp4_e2m1.argtypes = [c.c_float]
        L.ref_encode_fp4_e2m1.restype = c.c_uint8
        L.ref_compute_scale_ue8m0.argtypes = [_f32]
        L.ref_compute_scale_ue8m0.restype = c.c_uint8
        L.ref_quantize.argtypes = [_f32, c.c_longlong, c.c_int, _u8, _u8]
        L.ref_cpu_attention.argtypes = [_f32, _f32, _f32, _f32, c.c_int, c.c_int, c.c_int]
        L.ref_fp4_attention.argtypes = [_f32, _f32, _f32, _f32] + [c.c_int] * 5
        L.ref_cosine_similarity.argtypes = [_f32, _f32, c.c_int]
        L.ref_cosine_similarity.restype = c.c_float
        _r = L
    return _r


def _c(a, dt=np.float32):
    return np.ascontiguousarray(a, dtype=dt)


def quantize(x, scale_mode: int = 0):
    """(codes one per byte, scales) of rows x head_dim floats."""
    x = _c(x)
    d = x.shape[-1]
    rows = x.size // d
    codes = np.zeros(x.shape, np.uint8)
    scales = np.zeros(x.shape[:-1] + (d // 32,), np.uint8)
    oracle_lib().oracle_quantize(x, rows, d, codes, scales, scale_mode)
    return codes, scales


def pack_codes(codes):
    """Two codes per byte, element 2i in the low nibble (the product layout)."""
    c = np.asarray(codes, np.uint8)
    return (c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8)


def dequantize(codes, scales):
    codes = _c(codes, np.uint8)
    scales = _c(scales, np.uint8)
    d = codes.shape[-1]
    out = np.zeros(codes.shape, np.float32)
    oracle_lib().oracle_dequantize(codes, scales, codes.size // d, d, out)
    return out


def attention(Q, K, V, scale: float = 0.0):
    """Unquantised FP32 cpu_attention of one slice [seq, head_dim]."""
    Q, K, V = _c(Q), _c(K), _c(V)
    out = np.zeros(Q.shape, np.float32)
    oracle_lib().oracle_attention(Q, K, V, out, Q.shape[0], K.shape[0], Q.shape[1], scale)
    return out


def fp4_attention(Q, K, V, scale: float = 0.0, scale_mode: int = 0, threads: int = 8, causal: bool = False):
    """The FP4 path for [slices, seq, head_dim] (or [B, H, seq, head_dim]) inputs.
    causal=True applies the bottom-right causal mask (our extension; the
    reference has none): query i sees keys j <= i + seq_k - seq_q."""
    Q, K, V = _c(Q), _c(K), _c(V)
    d = Q.shape[-1]
    sq, sk = Q.shape[-2], K.shape[-2]
    slices = Q.size // (sq * d)
    out = np.zeros(Q.shape, np.float32)
    fn = oracle_lib().oracle_fp4_attention_causal if causal else oracle_lib().oracle_fp4_attention
    fn(Q, K, V, out, slices, sq, sk, d, scale, scale_mode, threads)
    return out


def attention_causal(Q, K, V, scale: float = 0.0, first_row: int = 0, seq_q_total=None):
    """Unquantised FP32 causal attention of one slice (query rows first_row...)."""
    Q, K, V = _c(Q), _c(K), _c(V)
    out = np.zeros(Q.shape, np.float32)
    total = Q.shape[0] if seq_q_total is None else seq_q_total
    oracle_lib().oracle_attention_causal(Q, K, V, out, Q.shape[0], K.shape[0], Q.shape[1], scale, first_row, total)
    return out


def fp4_attention_rows(Q, K, V, slice_of, rows, scale: float = 0.0, scale_mode: int = 0):
    """The FP4 path for selected (slice, query row) pairs -> [n, head_dim]."""
    Q, K, V = _c(Q), _c(K), _c(V)
    d = Q.shape[-1]
    sq, sk = Q.shape[-2], K.shape[-2]
    s = _c(slice_of, np.int32)
    r = _c(rows, np.int32)
    out = np.zeros((len(s), d), np.float32)
    oracle_lib().oracle_fp4_attention_rows(Q, K, V, out, len(s), s, r, sq, sk, d, scale, scale_mode)
    return out


def fp4_attention_backward(Q, K, V, dO, scale: float = 0.0, scale_mode: int = 0, causal: bool = False,
                           threads: int = 0):
    """Gradient of the FP4 path (the quantiser as a straight-through
    estimator) for [slices, seq, head_dim] (or [B, H, seq, head_dim]) inputs:
    returns (dQ, dK, dV) as float32 arrays shaped like Q, K, V."""
    import os
    Q, K, V, dO = _c(Q), _c(K), _c(V), _c(dO)
    d = Q.shape[-1]
    sq, sk = Q.shape[-2], K.shape[-2]
    slices = Q.size // (sq * d)
    dQ, dK, dV = np.zeros(Q.shape, np.float32), np.zeros(K.shape, np.float32), np.zeros(V.shape, np.float32)
    oracle_lib().oracle_fp4_attention_backward(Q, K, V, dO, dQ, dK, dV, slices, sq, sk, d, scale, scale_mode,
                                               int(causal), threads or os.cpu_count() or 1)
    return dQ, dK, dV


def fp4_attention_lse(Q, K, scale: float = 0.0, scale_mode: int = 0, causal: bool = False):
    """Per query row ln(sum_j exp(scale * Qq_i . Kq_j)) -> [..., seq_q] float32."""
    Q, K = _c(Q), _c(K)
    d = Q.shape[-1]
    sq, sk = Q.shape[-2], K.shape[-2]
    slices = Q.size // (sq * d)
    out = np.zeros(Q.shape[:-1], np.float32)
    oracle_lib().oracle_fp4_attention_lse(Q, K, out, slices, sq, sk, d, scale, scale_mode, int(causal))
    return out


def fp4_attention_slice(Q, K, V, scale: float = 0.0, scale_mode: int = 0, threads: int = 0):
    """The FP4 path for every query row of one slice [seq, head_dim], the rows
    split over `threads` threads (0: all host cores)."""
    import os
    Q, K, V = _c(Q), _c(K), _c(V)
    out = np.zeros(Q.shape, np.float32)
    oracle_lib().oracle_fp4_attention_slice(Q, K, V, out, Q.shape[0], K.shape[0], Q.shape[1], scale, scale_mode,
                                            threads or os.cpu_count() or 1)
    return out


def redo_warp_steps(Q, K, scale: float = 0.0, scale_mode: int = 0, block_n: int = 64,
                    lazy_log2: float = 15.0) -> tuple[int, int]:
    """Row-max statistics of one slice: how many (32-row warp, 64-key step)
    pairs after the first step of each 256-row work item see some row's
    max of S * scale * log2(e) grow past the running reference max by more
    than 2^lazy_log2 -- the steps the attention kernel redoes max-first
    (its lazy-rescale rule) -- and how many such pairs there are.  S is the
    exact FP4 product (dequantised Q K^T); returns (redone, total)."""
    import math
    qd = dequantize(*quantize(Q, scale_mode)).astype(np.float64)
    kd = dequantize(*quantize(K, scale_mode)).astype(np.float64)
    d = Q.shape[1]
    c = (scale if scale > 0 else 1.0 / math.sqrt(d)) * math.log2(math.e)
    sq, sk = qd.shape[0], kd.shape[0]
    nk = (sk + block_n - 1) // block_n
    redone = total = 0
    for r0 in range(0, sq, 1024):
        S = (qd[r0:r0 + 1024] @ kd.T) * c
        pad = nk * block_n - sk
        if pad:
            S = np.concatenate([S, np.full((S.shape[0], pad), -np.inf)], axis=1)
        mx = S.reshape(S.shape[0], nk, block_n).max(axis=2)   # [rows, steps]
        m = mx[:, 0].copy()
        for j in range(1, nk):
            jump = mx[:, j] > m + lazy_log2
            m = np.where(jump, np.maximum(m, mx[:, j]), m)
            w = jump[: (len(jump) // 32) * 32].reshape(-1, 32).any(axis=1)
            redone += int(w.sum())
            total += len(w)
    return redone, total


def fp4_scores(Q, K, scale_mode: int = 0):
    """Q K^T on dequantised FP4 Q, K of one slice."""
    Q, K = _c(Q), _c(K)
    S = np.zeros((Q.shape[0], K.shape[0]), np.float32)
    oracle_lib().oracle_fp4_scores(Q, K, S, Q.shape[0], K.shape[0], Q.shape[1], scale_mode)
    return S


def cosine(a, b) -> float:
    a, b = _c(a).ravel(), _c(b).ravel()
    return float(oracle_lib().oracle_cosine(a, b, a.size))


def ref_quantize(x):
    """The reference's own quantiser: (codes as code<<2 containers, scales)."""
    x = _c(x)
    d = x.shape[-1]
    codes = np.zeros(x.shape, np.uint8)
    scales = np.zeros(x.shape[:-1] + (d // 32,), np.uint8)
    ref_lib().ref_quantize(x, x.size // d, d, codes, scales)
    return codes, scales


def ref_fp4_attention(Q, K, V, threads: int = 8):
    Q, K, V = _c(Q), _c(K), _c(V)
    d = Q.shape[-1]
    sq, sk = Q.shape[-2], K.shape[-2]
    out = np.zeros(Q.shape, np.float32)
    ref_lib().ref_fp4_attention(Q, K, V, out, Q.size // (sq * d), sq, sk, d, threads)
    return out


def ref_cpu_attention(Q, K, V):
    Q, K, V = _c(Q), _c(K), _c(V)
    out = np.zeros(Q.shape, np.float32)
    ref_lib().ref_cpu_attention(Q, K, V, out, Q.shape[0], K.shape[0], Q.shape[1])
    return out
