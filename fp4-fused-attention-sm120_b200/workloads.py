"""The reference's benchmark/test problem shapes and their synthetic inputs.

The reference benchmarks batch=1, heads=32, seq_q=64 with seq_k in
{128..1024} and head_dim in {64, 128} (tests/benchmark.cu:9-12, :116-124) and
tests fixed shapes (tests/test_attention.cu:177-186).  The workloads below are
the problem set this port is measured on: the reference's CPU-checkable case,
a short-head/long-key case with outliers, the prefill-sized single-GPU case,
the box-scale sharded case, and two odd head dims.  There is no public
dataset; inputs are seeded i.i.d. normals drawn on the device with torch
(Philox), with a Bernoulli outlier mask where the workload asks for one.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Workload:
    name: str
    batch: int
    heads: int
    seq_q: int
    seq_k: int
    head_dim: int
    std: float = 1.0
    outlier_frac: float = 0.0
    outlier_mult: float = 1.0
    out_dtype: str = "float32"

    @property
    def slices(self) -> int:
        return self.batch * self.heads

    def flops(self, slices: int | None = None) -> float:
        """4 * B * H * seq_q * seq_k * head_dim (tests/benchmark.cu:85-86)."""
        s = self.slices if slices is None else slices
        return 4.0 * s * self.seq_q * self.seq_k * self.head_dim

    def describe(self) -> str:
        return (f"B{self.batch} H{self.heads} sq{self.seq_q} sk{self.seq_k} d{self.head_dim}"
                f" std{self.std:g}" + (f" {self.outlier_frac:g}x{self.outlier_mult:g} outliers"
                                       if self.outlier_frac else "") + f" out {self.out_dtype}")


WORKLOADS = {
    "cpu_check": Workload("cpu_check", 1, 32, 64, 128, 128),
    "short_head_long_key": Workload("short_head_long_key", 1, 32, 64, 1024, 64,
                                    outlier_frac=0.01, outlier_mult=8.0),
    "prefill_4k": Workload("prefill_4k", 2, 32, 4096, 4096, 128, out_dtype="float16"),
    "box_sharded_8k": Workload("box_sharded_8k", 16, 32, 8192, 8192, 128,
                               outlier_frac=0.005, outlier_mult=16.0),
    "odd_d96": Workload("odd_d96", 4, 16, 2048, 2048, 96, std=0.5),
    "odd_d256": Workload("odd_d256", 4, 16, 2048, 2048, 256, std=0.5),
}


def make_inputs(w: Workload, seed: int, slices: tuple[int, int] | None = None, device="cuda",
                dtype=None):
    """Q, K, V as [n_slices, seq, head_dim] FP16 tensors for slices
    [lo, hi) of the workload (all slices by default).  Each slice is drawn from
    its own generator (seed, slice index), so any shard is reproducible on its
    own GPU without generating the others."""
    import torch

    lo, hi = slices if slices is not None else (0, w.slices)
    dtype = dtype or torch.float16
    shape_q, shape_k = (hi - lo, w.seq_q, w.head_dim), (hi - lo, w.seq_k, w.head_dim)
    Q = torch.empty(shape_q, dtype=dtype, device=device)
    K = torch.empty(shape_k, dtype=dtype, device=device)
    V = torch.empty(shape_k, dtype=dtype, device=device)
    g = torch.Generator(device=device)
    for i, s in enumerate(range(lo, hi)):
        g.manual_seed(seed * 1_000_003 + s)
        for t in (Q, K, V):
            x = torch.randn(t.shape[1:], generator=g, device=device, dtype=torch.float32) * w.std
            if w.outlier_frac:
                m = torch.rand(t.shape[1:], generator=g, device=device) < w.outlier_frac
                x = torch.where(m, x * w.outlier_mult, x)
            t[i].copy_(x.to(dtype))
    return Q, K, V
