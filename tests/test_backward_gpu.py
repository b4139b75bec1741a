"""GPU backward pass (fp4attn_backward) and the forward's log-sum-exp output
(fp4attn_forward_lse) against the oracle.

The reference is forward only; the oracle's backward
(oracle_fp4_attention_backward) is pinned against float64 torch autograd on
the reference-quantised operands in test_oracle_backward.py.

Tolerance (written here): per gradient tensor, cosine with the oracle
>= 0.9999 (double) and max |gpu - oracle| <= 1e-2 * max |oracle|.  The GPU
rounds P to FP16 and dZ to BF16 for the tensor cores (relative steps of 2^-11
and 2^-8 per element); the oracle keeps everything in double.  The
log-sum-exp is within 2e-3 (absolute) of the oracle's: the forward sums its
FP16-rounded probabilities."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

COS_MIN = 0.9999
REL_MAX = 1e-2
LSE_ABS = 2e-3


def _inputs(seed, B, H, sq, sk, d):
    g = torch.Generator().manual_seed(seed)
    Q, K, V = (torch.randn(B, H, s, d, generator=g).half() for s in (sq, sk, sk))
    dO = torch.randn(B, H, sq, d, generator=g).half()
    return Q, K, V, dO


def _np(t):
    return t.float().cpu().numpy().reshape(-1, t.shape[-2], t.shape[-1])


def _assert_grad(got, want, what):
    got = got.float().cpu().numpy().reshape(want.shape)
    assert np.isfinite(got).all(), what
    if not np.any(want):
        # With one visible key P = 1 and dZ = dP - Dd = 0: dQ = dK = 0 exactly.
        assert float(np.abs(got).max()) <= 1e-6, what
        return
    cos = oracle.cosine(got, want)
    rel = float(np.abs(got - want).max()) / max(float(np.abs(want).max()), 1e-30)
    assert cos >= COS_MIN and rel <= REL_MAX, (what, cos, rel)


def _run(fa, shape, causal, out_dtype=torch.float16, seed=0):
    B, H, sq, sk, d = shape
    Q, K, V, dO = _inputs(seed, B, H, sq, sk, d)
    Qc, Kc, Vc, dOc = (t.cuda() for t in (Q, K, V, dO))
    out, lse = fa.fused_fp4_attention_lse(Qc, Kc, Vc, out_dtype=out_dtype, causal=causal)
    dq, dk, dv = fa.fp4_attention_backward(Qc, Kc, Vc, out, dOc, lse, causal=causal)
    assert fa.status_query() == fa.OK
    return (Q, K, V, dO), out, lse, (dq, dk, dv)


SHAPES = [
    (1, 2, 256, 256, 128),    # whole tiles
    (1, 2, 200, 333, 64),     # ragged seq_q and seq_k
    (2, 1, 64, 640, 128),     # one query tile, several key tiles
    (1, 2, 320, 130, 128),    # seq_k just past one key tile
    (1, 1, 1, 1, 64),         # one query, one key (dQ = dK = 0)
    (1, 1, 1, 3, 64),         # one query, three keys
    (1, 2, 200, 333, 96),     # head_dim 96: 32-column operand chunks, codes padded to 128
    (2, 1, 130, 260, 32),     # head_dim 32: codes padded to 64
]


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("shape", SHAPES)
def test_backward_matches_oracle(fa, cuda, shape, causal):
    (Q, K, V, dO), _, _, (dq, dk, dv) = _run(fa, shape, causal)
    want = oracle.fp4_attention_backward(_np(Q), _np(K), _np(V), _np(dO), causal=causal)
    for got, w, name in zip((dq, dk, dv), want, ("dQ", "dK", "dV")):
        _assert_grad(got, w, name)


def test_backward_with_fp32_forward_output(fa, cuda):
    (Q, K, V, dO), out, _, (dq, dk, dv) = _run(fa, (1, 3, 192, 256, 128), False, out_dtype=torch.float32)
    assert out.dtype == torch.float32
    want = oracle.fp4_attention_backward(_np(Q), _np(K), _np(V), _np(dO))
    for got, w, name in zip((dq, dk, dv), want, ("dQ", "dK", "dV")):
        _assert_grad(got, w, name)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("shape", [(1, 4, 256, 512, 128), (2, 2, 100, 300, 64), (1, 2, 64, 2048, 128),
                                   (1, 1, 300, 100, 64), (1, 2, 300, 500, 96), (1, 2, 200, 200, 32)])
def test_forward_lse(fa, cuda, shape, causal):
    """The log-sum-exp variant writes the same output bytes as the plain
    forward and the oracle's per-row log-sum-exp (+inf where a row sees no
    key).  The (1, 2, 64, 2048) case runs the small-problem schedule with its
    keys split into partitions; (1, 1, 300, 100) causal has rows that see no
    key."""
    B, H, sq, sk, d = shape
    Q, K, V, _ = _inputs(3, B, H, sq, sk, d)
    Qc, Kc, Vc = Q.cuda(), K.cuda(), V.cuda()
    out, lse = fa.fused_fp4_attention_lse(Qc, Kc, Vc, out_dtype=torch.float32, causal=causal)
    ref_out = fa.fused_fp4_attention(Qc, Kc, Vc, out_dtype=torch.float32, causal=causal)
    assert fa.status_query() == fa.OK
    assert torch.equal(out, ref_out)
    want = oracle.fp4_attention_lse(_np(Q), _np(K), causal=causal).reshape(B, H, sq)
    got = lse.cpu().numpy()
    finite = np.isfinite(want)
    assert np.array_equal(np.isfinite(got), finite)
    assert np.all(got[~finite] == np.inf)
    assert float(np.abs(got[finite] - want[finite]).max()) <= LSE_ABS


def test_autograd_function(fa, cuda):
    """fp4_attention under autograd: the gradients are fp4_attention_backward's
    (the same kernels, so the same bytes)."""
    Q, K, V, dO = (t.cuda() for t in _inputs(11, 1, 2, 192, 320, 64))
    q, k, v = (t.clone().requires_grad_(True) for t in (Q, K, V))
    out = fa.fp4_attention(q, k, v)
    out.backward(dO)
    ref_out, lse = fa.fused_fp4_attention_lse(Q, K, V)
    dq, dk, dv = fa.fp4_attention_backward(Q, K, V, ref_out, dO, lse)
    assert torch.equal(out.detach(), ref_out)
    for g, want in ((q.grad, dq), (k.grad, dk), (v.grad, dv)):
        assert g.dtype == torch.float16
        assert torch.equal(g, want.half())


def test_backward_repeats_bit_for_bit(fa, cuda):
    """dK and dV are accumulated by one CTA per key tile in a fixed order, so
    they repeat exactly; dQ sums the key tiles' partial products with
    reduce-add in whatever order they arrive, so it may differ in the last
    bits between runs."""
    shape = (1, 4, 384, 512, 128)
    (_, _, _, _), _, _, a = _run(fa, shape, False, seed=21)
    (_, _, _, _), _, _, b = _run(fa, shape, False, seed=21)
    assert torch.equal(a[1], b[1]) and torch.equal(a[2], b[2])
    assert float((a[0] - b[0]).abs().max()) <= 1e-5 * float(a[0].abs().max())


def test_full_size_prefill_slices(fa, cuda):
    """The 4k x 4k, head_dim 128 prefill shape (B2 H32): slices 0 and 63 of
    every gradient against the oracle run on those two slices."""
    B, H, S, d = 2, 32, 4096, 128
    Q, K, V, dO = _inputs(7, B, H, S, S, d)
    Qc, Kc, Vc, dOc = (t.cuda() for t in (Q, K, V, dO))
    out, lse = fa.fused_fp4_attention_lse(Qc, Kc, Vc)
    dq, dk, dv = fa.fp4_attention_backward(Qc, Kc, Vc, out, dOc, lse)
    assert fa.status_query() == fa.OK
    for s in (0, B * H - 1):
        b, h = divmod(s, H)
        want = oracle.fp4_attention_backward(*(t[b, h].float().numpy()[None] for t in (Q, K, V, dO)))
        for got, w, name in zip((dq[b, h], dk[b, h], dv[b, h]), want, ("dQ", "dK", "dV")):
            _assert_grad(got, w[0], f"{name} slice {s}")


def test_backward_rejects_bad_arguments(fa, cuda):
    Q, K, V, dO = (t.cuda() for t in _inputs(1, 1, 1, 64, 64, 160))
    out, lse = torch.zeros_like(Q), torch.zeros(1, 1, 64, device="cuda")
    with pytest.raises(fa.Fp4AttnError) as e:
        fa.fp4_attention_backward(Q, K, V, out, dO, lse)
    assert e.value.code == fa.EUNSUPPORTED
    Q, K, V, dO = (t.cuda() for t in _inputs(1, 1, 1, 64, 64, 64))
    out = torch.zeros_like(Q)
    ws = torch.empty(fa.backward_workspace_size(1, 1, 64, 64, 64) - 256, dtype=torch.uint8, device="cuda")
    with pytest.raises(fa.Fp4AttnError) as e:
        fa.fp4_attention_backward(Q, K, V, out, dO, lse, workspace=ws)
    assert e.value.code == fa.EWORKSPACE


def test_prepare_then_attend_is_the_backward(fa, cuda):
    """fp4attn_backward_prepare + fp4attn_backward_attend (as bench.py times
    them) give fp4attn_backward's dK and dV bytes; dQ is a sum of reductions
    whose order may vary between runs."""
    B, H, sq, sk, d = 1, 2, 320, 384, 64
    Q, K, V, dO = (t.cuda() for t in _inputs(5, B, H, sq, sk, d))
    out, lse = fa.fused_fp4_attention_lse(Q, K, V)
    dq, dk, dv = fa.fp4_attention_backward(Q, K, V, out, dO, lse)
    ws = torch.empty(fa.backward_workspace_size(B, H, sq, sk, d), dtype=torch.uint8, device="cuda")
    g = [torch.full(t.shape, float("nan"), dtype=torch.float32, device="cuda") for t in (Q, K, V)]
    L = fa.lib()
    st = torch.cuda.current_stream().cuda_stream
    assert L.fp4attn_backward_prepare(Q.data_ptr(), K.data_ptr(), V.data_ptr(), out.data_ptr(), dO.data_ptr(),
                                      lse.data_ptr(), g[0].data_ptr(), fa.F16, fa.F16, B, H, sq, sk, d, 0,
                                      ws.data_ptr(), ws.numel(), st) == fa.OK
    assert L.fp4attn_backward_attend(V.data_ptr(), dO.data_ptr(), g[0].data_ptr(), g[1].data_ptr(), g[2].data_ptr(),
                                     fa.F16, B, H, sq, sk, d, 0.0, 0, ws.data_ptr(), ws.numel(), st) == fa.OK
    assert fa.status_query() == fa.OK
    assert torch.equal(g[1], dk) and torch.equal(g[2], dv)
    assert float((g[0] - dq).abs().max()) <= 1e-5 * float(dq.abs().max())


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("shape", [(1, 2, 200, 333, 64), (1, 2, 256, 384, 128), (1, 2, 100, 200, 96)])
def test_backward_fp32_inputs(fa, cuda, shape, causal):
    """FP32 Q, K, V and dO (the reference's input type): Q and K quantised from
    FP32, V and dO rounded to FP16 for the tensor cores.  The oracle takes the
    same FP32 values (V unrounded)."""
    B, H, sq, sk, d = shape
    g = torch.Generator().manual_seed(13)
    Q, K, V = (torch.randn(B, H, s, d, generator=g) for s in (sq, sk, sk))
    dO = torch.randn(B, H, sq, d, generator=g)
    Qc, Kc, Vc, dOc = (t.cuda() for t in (Q, K, V, dO))
    out, lse = fa.fused_fp4_attention_lse(Qc, Kc, Vc, out_dtype=torch.float32, causal=causal)
    dq, dk, dv = fa.fp4_attention_backward(Qc, Kc, Vc, out, dOc, lse, causal=causal)
    assert fa.status_query() == fa.OK
    want = oracle.fp4_attention_backward(_np(Q), _np(K), _np(V), _np(dO), causal=causal)
    for got, w, name in zip((dq, dk, dv), want, ("dQ", "dK", "dV")):
        _assert_grad(got, w, name)
    # The forward's log-sum-exp from FP32 input.
    wl = oracle.fp4_attention_lse(_np(Q), _np(K), causal=causal).reshape(B, H, sq)
    gl = lse.cpu().numpy()
    fin = np.isfinite(wl)
    assert float(np.abs(gl[fin] - wl[fin]).max()) <= LSE_ABS


def test_backward_kernel_abort_path_drains_and_recovers(fa, cuda):
    """The backward kernel's own failure path: a test instantiation withholds
    one gradient thread's first arrival, the MMA issuer's bounded wait (20 ms)
    runs out, and every role of every CTA leaves, drains its copies and MMAs
    and frees TMEM.  The device reports FP4ATTN_ETIMEOUT; the same context
    then runs the normal backward on the same workspace, matching the
    oracle."""
    B, H, sq, sk, d = 1, 4, 256, 384, 64
    Q, K, V, dO = _inputs(17, B, H, sq, sk, d)
    Qc, Kc, Vc, dOc = (t.cuda() for t in (Q, K, V, dO))
    out, lse = fa.fused_fp4_attention_lse(Qc, Kc, Vc)
    ws = torch.empty(fa.backward_workspace_size(B, H, sq, sk, d), dtype=torch.uint8, device="cuda")
    g = [torch.empty(t.shape, dtype=torch.float32, device="cuda") for t in (Q, K, V)]
    assert fa.selftest_backward_abort(Qc, Kc, Vc, out, dOc, lse, *g, ws, timeout_us=20000) == fa.ETIMEOUT
    assert fa.status_query() == fa.OK  # the word was read and cleared
    dq, dk, dv = fa.fp4_attention_backward(Qc, Kc, Vc, out, dOc, lse, workspace=ws)
    assert fa.status_query() == fa.OK
    want = oracle.fp4_attention_backward(_np(Q), _np(K), _np(V), _np(dO))
    for got, w, name in zip((dq, dk, dv), want, ("dQ", "dK", "dV")):
        _assert_grad(got, w, name)


@pytest.mark.parametrize("scale_mode,softmax_scale", [("ocp", None), ("reference", 0.05), ("ocp", 0.2)])
def test_backward_scale_rule_and_explicit_scale(fa, cuda, scale_mode, softmax_scale):
    """The OCP "/6" scale rule and an explicit softmax scale reach the
    backward's quantiser and kernel the way they reach the forward's."""
    B, H, sq, sk, d = 1, 2, 192, 320, 128
    Q, K, V, dO = _inputs(29, B, H, sq, sk, d)
    Qc, Kc, Vc, dOc = (t.cuda() for t in (Q, K, V, dO))
    out, lse = fa.fused_fp4_attention_lse(Qc, Kc, Vc, softmax_scale=softmax_scale, scale_mode=scale_mode)
    dq, dk, dv = fa.fp4_attention_backward(Qc, Kc, Vc, out, dOc, lse, softmax_scale=softmax_scale,
                                           scale_mode=scale_mode)
    assert fa.status_query() == fa.OK
    mode = 1 if scale_mode == "ocp" else 0
    want = oracle.fp4_attention_backward(_np(Q), _np(K), _np(V), _np(dO), scale=softmax_scale or 0.0,
                                         scale_mode=mode)
    for got, w, name in zip((dq, dk, dv), want, ("dQ", "dK", "dV")):
        _assert_grad(got, w, name)
    wl = oracle.fp4_attention_lse(_np(Q), _np(K), scale=softmax_scale or 0.0, scale_mode=mode).reshape(B, H, sq)
    assert float(np.abs(lse.cpu().numpy() - wl).max()) <= LSE_ABS


@pytest.mark.parametrize("case", range(16))
def test_random_shapes_forward_lse_and_backward(fa, cuda, case):
    """Seeded random problems (head_dim 32-128, ragged seq_q and seq_k from 1
    to 300, both masks, both output types, both scale rules): the log-sum-exp
    forward and the backward against the oracle."""
    rng = np.random.default_rng(1000 + case)
    d = int(rng.choice([32, 64, 96, 128]))
    B, H = int(rng.integers(1, 3)), int(rng.integers(1, 4))
    sq, sk = int(rng.integers(1, 301)), int(rng.integers(1, 301))
    causal = bool(rng.integers(0, 2))
    odt = torch.float16 if rng.integers(0, 2) else torch.float32
    mode = "ocp" if rng.integers(0, 4) == 0 else "reference"
    Q, K, V, dO = _inputs(2000 + case, B, H, sq, sk, d)
    Qc, Kc, Vc, dOc = (t.cuda() for t in (Q, K, V, dO))
    out, lse = fa.fused_fp4_attention_lse(Qc, Kc, Vc, out_dtype=odt, causal=causal, scale_mode=mode)
    dq, dk, dv = fa.fp4_attention_backward(Qc, Kc, Vc, out, dOc, lse, causal=causal, scale_mode=mode)
    assert fa.status_query() == fa.OK
    m = 1 if mode == "ocp" else 0
    wl = oracle.fp4_attention_lse(_np(Q), _np(K), causal=causal, scale_mode=m).reshape(B, H, sq)
    gl = lse.cpu().numpy()
    fin = np.isfinite(wl)
    assert np.array_equal(np.isfinite(gl), fin)
    if fin.any():
        assert float(np.abs(gl[fin] - wl[fin]).max()) <= LSE_ABS
    want = oracle.fp4_attention_backward(_np(Q), _np(K), _np(V), _np(dO), causal=causal, scale_mode=m)
    for got, w, name in zip((dq, dk, dv), want, ("dQ", "dK", "dV")):
        _assert_grad(got, w, f"{name} case {case} d{d} B{B} H{H} sq{sq} sk{sk} causal {causal}")


@pytest.mark.parametrize("std", [16.0, 1e-4])
def test_extreme_input_magnitudes(fa, cuda, std):
    """Inputs scaled far from N(0, 1): sigma 16 (scaled scores in the
    thousands, a nearly one-hot softmax, the lazy rescale firing often) and
    sigma 1e-4 (scales near the bottom of the FP16 range, a nearly uniform
    softmax).  Forward output, log-sum-exp and gradients against the oracle.
    (The log-sum-exp is one FP32 number per row: once the scaled scores reach
    about 2^20 its rounding alone moves the backward's probabilities by
    percents, so far larger scores are not a backward case.)"""
    B, H, sq, sk, d = 1, 2, 192, 320, 64
    g = torch.Generator().manual_seed(31)
    Q, K, V = ((torch.randn(B, H, s, d, generator=g) * std).half() for s in (sq, sk, sk))
    dO = torch.randn(B, H, sq, d, generator=g).half()
    Qc, Kc, Vc, dOc = (t.cuda() for t in (Q, K, V, dO))
    out, lse = fa.fused_fp4_attention_lse(Qc, Kc, Vc, out_dtype=torch.float32)
    dq, dk, dv = fa.fp4_attention_backward(Qc, Kc, Vc, out, dOc, lse)
    assert fa.status_query() == fa.OK
    want_o = oracle.fp4_attention(_np(Q), _np(K), _np(V))
    got_o = out.cpu().numpy().reshape(want_o.shape)
    assert np.isfinite(got_o).all()
    scale_o = max(float(np.abs(want_o).max()), 1e-30)
    assert oracle.cosine(got_o, want_o) >= COS_MIN
    assert float(np.abs(got_o - want_o).max()) <= REL_MAX * scale_o
    wl = oracle.fp4_attention_lse(_np(Q), _np(K)).reshape(B, H, sq)
    assert float(np.abs(lse.cpu().numpy() - wl).max()) <= LSE_ABS * max(1.0, float(np.abs(wl).max()) * 1e-3)
    want = oracle.fp4_attention_backward(_np(Q), _np(K), _np(V), _np(dO))
    for got, w, name in zip((dq, dk, dv), want, ("dQ", "dK", "dV")):
        _assert_grad(got, w, f"{name} std {std}")
