"""Inputs of the golden cases, regenerated from seeds (shared by the fixture
generator tests/golden/make_golden.py and the tests that read the fixtures)."""
from __future__ import annotations

import ctypes
import struct

import numpy as np
import torch

# Attention cases with stored reference outputs (slices kept: keep_slices).
ATTN_CASES = {
    # the reference's CPU-checkable shape: B1 H32 sq64 sk128 d128, N(0,1) FP16
    "cpu_check": dict(B=1, H=32, sq=64, sk=128, d=128, std=1.0, of=0.0, om=1.0, seed=101,
                      keep_slices=[0, 7, 31]),
    # short head, long keys, 1% of elements x8
    "short_head_long_key": dict(B=1, H=32, sq=64, sk=1024, d=64, std=1.0, of=0.01, om=8.0, seed=102,
                                keep_slices=[0, 13, 31]),
    # odd head dims and ragged lengths (seq_q not a multiple of 64, seq_k not of 64)
    "ragged_d96": dict(B=1, H=3, sq=77, sk=200, d=96, std=0.5, of=0.0, om=1.0, seed=103, keep_slices=[0, 1, 2]),
    "ragged_d256": dict(B=1, H=2, sq=130, sk=100, d=256, std=0.5, of=0.0, om=1.0, seed=104, keep_slices=[0, 1]),
    "d32": dict(B=2, H=2, sq=64, sk=192, d=32, std=1.0, of=0.0, om=1.0, seed=105, keep_slices=[0, 3]),
    "d160": dict(B=1, H=2, sq=96, sk=320, d=160, std=1.0, of=0.0, om=1.0, seed=106, keep_slices=[0, 1]),
}

# The reference test's own shapes (tests/test_attention.cu:179-184):
# name -> (head_dim, seq_k, batch, heads); seq_q = 64.
DISCRETE_CASES = {
    "single_d128_sk64": (128, 64, 1, 1),
    "single_d128_sk128": (128, 128, 1, 1),
    "single_d64_sk64": (64, 64, 1, 1),
    "single_d64_sk128": (64, 128, 1, 1),
    "multi_b1_h4_sk128": (128, 128, 1, 4),
    "multi_b2_h4_sk128": (128, 128, 2, 4),
}


def attn_inputs(name):
    """[slices, seq, d] FP32 arrays holding FP16-representable values."""
    c = ATTN_CASES[name]
    g = torch.Generator(device="cpu").manual_seed(c["seed"])
    out = []
    for seq in (c["sq"], c["sk"], c["sk"]):
        x = torch.randn((c["B"] * c["H"], seq, c["d"]), generator=g) * c["std"]
        if c["of"]:
            m = torch.rand(x.shape, generator=g) < c["of"]
            x = torch.where(m, x * c["om"], x)
        out.append(x.half().float().numpy())
    return out


def discrete_inputs(d, sk, B, H, sq=64):
    """tests/test_attention.cu:79-86 / :132-139: srand(42), values
    {-1,-0.5,0,0.5,1}[rand() % 5], filled Q then K then V (glibc rand)."""
    libc = ctypes.CDLL("libc.so.6")
    libc.srand(42)
    vals = np.array([-1.0, -0.5, 0.0, 0.5, 1.0], np.float32)
    def fill(n):
        return vals[np.array([libc.rand() % 5 for _ in range(n)])]
    n_q, n_k = B * H * sq * d, B * H * sk * d
    Q = fill(n_q).reshape(B * H, sq, d)
    K = fill(n_k).reshape(B * H, sk, d)
    V = fill(n_k).reshape(B * H, sk, d)
    return Q, K, V


def _f(bits):
    return struct.unpack("<f", struct.pack("<I", bits))[0]


def quant_edge_rows():
    """FP32 rows probing every branch of the reference quantiser: zero blocks,
    signed zero, NaN, +-inf, subnormals, the seven rounding thresholds and
    their neighbours, values just above powers of two (where glibc log2f
    rounds ceil down), huge values, and random magnitudes over the full range."""
    rng = np.random.default_rng(7)
    rows = []
    rows.append(np.zeros(128, np.float32))
    r = np.zeros(128, np.float32)
    r[:8] = [np.nan, np.inf, -np.inf, -0.0, 1e-45, -1e-45, 3.0, -3.0]
    rows.append(r)
    for m in (1.0, 2.0, 4.0, 6.0, 0.5, 8.0):  # block max fixes scale; thresholds scaled into the block
        t = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
        blk = np.concatenate([t, np.nextafter(t, 0).astype(np.float32), np.nextafter(t, 10).astype(np.float32),
                              -t, [0.0, -0.1, 0.1, m, 0.0, 0.0, 0.0, -m]]).astype(np.float32)[:32]
        rows.append(np.tile(blk * (m / 6.0 if m > 4 else 1.0), 4).astype(np.float32))
    for p in (-126, -125, -100, -20, -1, 0, 1, 4, 5, 7, 20, 64, 100, 126, 127):  # 2^p * (1 + k ulp)
        r = np.zeros(128, np.float32)
        for b in range(4):
            k = [1, 2, 11, 22][b] if p not in (4, 5, 7) else [1, 2, 3, 0][b]
            bits = ((p + 127) << 23) + k
            r[b * 32] = _f(bits)
            r[b * 32 + 1:b * 32 + 32] = rng.uniform(-1, 1, 31).astype(np.float32) * _f((p + 127) << 23)
        rows.append(r)
    for m in (0x00040001, 0x00080002, 0x00100005, 0x00200003, 0x0040000b, 0x00000001, 0x007fffff):  # subnormal maxima
        r = np.zeros(128, np.float32)
        r[::32] = _f(m)
        r[5::32] = -_f(m) / 4
        rows.append(r)
    r = np.full(128, 3.0e38, np.float32)
    r[1::2] = -1.0
    rows.append(r)
    for _ in range(24):
        rows.append((rng.standard_normal(128) * np.exp2(rng.integers(-140, 127, 128))).astype(np.float32))
    return np.stack(rows).astype(np.float32)


def quant_fp16_rows():
    """FP16-representable rows: N(0,1), outliers, tiny, huge, subnormal."""
    g = torch.Generator().manual_seed(11)
    parts = [torch.randn(64, 128, generator=g),
             torch.randn(32, 128, generator=g) * 1e-4,
             torch.randn(32, 128, generator=g) * 6e3,
             torch.randn(16, 128, generator=g) * 1e-6]
    x = torch.cat(parts)
    m = torch.rand(x.shape, generator=g) < 0.02
    x = torch.where(m, x * 16, x)
    return x.half().float().numpy()
