"""Host-side arithmetic of bench.py that decides the reported numbers: the
share of (query, key) pairs a causal run counts, the burst / sustained choice
of the bf16 peak, the mixed FP4/FP16 roofline and the L2-flush rule.  No GPU."""
import numpy as np
import pytest

import bench
import fp4attn_b200.workloads as wl


@pytest.mark.parametrize("sq,sk", [(1, 1), (64, 128), (128, 64), (100, 300), (300, 100), (4096, 4096), (5, 1)])
def test_visible_fraction_counts_the_causal_pairs(sq, sk):
    i = np.arange(sq)[:, None]
    j = np.arange(sk)[None, :]
    want = float((j <= i + sk - sq).sum()) / (sq * sk)  # bottom-right alignment, as the kernels mask
    assert bench.visible_fraction(sq, sk, True) == pytest.approx(want, rel=0, abs=1e-15)
    assert bench.visible_fraction(sq, sk, False) == 1.0


def test_peak_basis_needs_a_long_power_capped_region():
    assert bench.peak_basis(0.008, []) == "burst"
    assert bench.peak_basis(0.5, ["sw_power_cap"]) == "burst"       # too short to settle at the cap
    assert bench.peak_basis(3.0, []) == "burst"                     # long, but never capped
    assert bench.peak_basis(3.0, ["sw_power_cap"]) == "sustained"


def test_mixed_roofline_is_fp4_qk_plus_fp16_pv():
    w = wl.WORKLOADS["prefill_4k"]
    bf16 = 1625.0
    peak = bench.mixed_roofline(w, bf16)
    # Half the FLOPs (QK^T) at 4x the bf16 rate and half (PV) at 1x: 1.6x bf16.
    assert peak == pytest.approx(1.6 * bf16)
    # The time it implies for the 4k prefill: 5.50e11 FLOPs in 211.4 us.
    assert w.flops() / (peak * 1e12) == pytest.approx(211.4e-6, rel=1e-3)


def test_l2_rule_flushes_only_inputs_that_fit_twice_in_l2():
    flush, text = bench.l2_note(64 << 20)
    assert flush and "flush" in text
    flush, text = bench.l2_note(256 << 20)
    assert not flush and "no flush" in text


def _args(workload, causal=False):
    import argparse
    return argparse.Namespace(workload=workload, causal=causal)


@pytest.mark.parametrize("world", [1, 2, 8])
def test_weak_job_gives_each_rank_the_whole_workload(world):
    base = wl.WORKLOADS["prefill_4k"]
    seen = []
    for rank in range(world):
        b, job, strong, lo, hi, config = bench.job_config(_args("prefill_4k"), world, rank)
        assert not strong and b is base
        assert hi - lo == base.slices and job.slices == base.slices * world
        assert config["slices_per_gpu"] == base.slices and config["job_slices"] == base.slices * world
        seen.append((lo, hi))
    assert seen == [(r * base.slices, (r + 1) * base.slices) for r in range(world)]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_box_scale_job_is_split_over_the_ranks(world):
    ranges = [bench.job_config(_args("box_sharded_8k"), world, r)[3:5] for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == 512
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))   # contiguous, no overlap, no gap
    assert {hi - lo for lo, hi in ranges} == {512 // world}
    assert bench.job_config(_args("box_sharded_8k"), world, 0)[2]   # strong scaling


def test_both_arms_print_one_config():
    # The reference arm prints job_config's dictionary as it is; the GPU arm
    # prints the same object, so the keys and values agree by construction.
    *_, config = bench.job_config(_args("prefill_4k"), 1, 0)
    assert set(config) == {"workload", "shape", "slices_per_gpu", "job_slices", "parallelism", "l2"}
    *_, causal = bench.job_config(_args("prefill_4k", causal=True), 1, 0)
    assert causal["mask"].startswith("causal")
