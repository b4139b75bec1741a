"""The backward oracle (oracle_fp4_attention_backward, oracle_fp4_attention_lse)
pinned against an independent implementation: torch autograd in float64 on
the dequantised operands.

The reference is forward only, so there is no reference gradient to compare
with.  What the oracle must get right is (1) the operands -- Qq, Kq are the
reference quantiser's output dequantised, the same numbers the forward's
oracle multiplies (pinned to the reference by test_oracle.py) -- and (2) the
gradient algebra, which autograd computes independently from the forward
expression softmax(scale * Qq Kq^T [+ mask]) V.  The quantiser is a
straight-through estimator: the gradient with respect to Q is the gradient
with respect to Qq."""
import numpy as np
import pytest
import torch

import oracle


def _dequant(x, scale_mode):
    codes, scales = oracle.quantize(x.reshape(-1, x.shape[-1]), scale_mode)
    return oracle.dequantize(codes, scales).reshape(x.shape)


def _autograd(Q, K, V, dO, scale, causal, scale_mode):
    qd = torch.tensor(_dequant(Q, scale_mode), dtype=torch.float64, requires_grad=True)
    kd = torch.tensor(_dequant(K, scale_mode), dtype=torch.float64, requires_grad=True)
    v = torch.tensor(V, dtype=torch.float64, requires_grad=True)
    sq, sk = Q.shape[-2], K.shape[-2]
    z = scale * qd @ kd.transpose(-1, -2)
    if causal:
        i = torch.arange(sq)[:, None]
        j = torch.arange(sk)[None, :]
        z = z.masked_fill(j > i + sk - sq, float("-inf"))
    lse = torch.logsumexp(z, dim=-1)
    p = torch.softmax(z, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)  # rows that see no key
    o = p @ v
    o.backward(torch.tensor(dO, dtype=torch.float64))
    return qd.grad.numpy(), kd.grad.numpy(), v.grad.numpy(), lse.detach().numpy()


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("shape", [(2, 48, 80, 64), (1, 80, 48, 128), (1, 64, 64, 32)])
@pytest.mark.parametrize("scale_mode", [0, 1])
def test_backward_matches_float64_autograd(shape, causal, scale_mode):
    slices, sq, sk, d = shape
    rng = np.random.default_rng(sq * 7 + sk + d + causal)
    Q = rng.standard_normal((slices, sq, d)).astype(np.float16).astype(np.float32)
    K = rng.standard_normal((slices, sk, d)).astype(np.float16).astype(np.float32)
    V = rng.standard_normal((slices, sk, d)).astype(np.float16).astype(np.float32)
    dO = rng.standard_normal((slices, sq, d)).astype(np.float16).astype(np.float32)
    scale = 1.0 / np.sqrt(d)
    dq, dk, dv = oracle.fp4_attention_backward(Q, K, V, dO, scale=scale, scale_mode=scale_mode, causal=causal,
                                               threads=3)
    lse = oracle.fp4_attention_lse(Q, K, scale=scale, scale_mode=scale_mode, causal=causal)
    for s in range(slices):
        gq, gk, gv, glse = _autograd(Q[s], K[s], V[s], dO[s], scale, causal, scale_mode)
        # float32 outputs of double sums: relative 1e-6 of the largest entry.
        for got, want in ((dq[s], gq), (dk[s], gk), (dv[s], gv)):
            assert np.abs(got - want).max() <= 1e-6 * max(1.0, np.abs(want).max())
        finite = np.isfinite(glse)
        assert np.array_equal(np.isfinite(lse[s]), finite)
        assert np.abs(lse[s][finite] - glse[finite]).max() <= 1e-5
        assert np.all(lse[s][~finite] == np.inf)


def test_rows_that_see_no_key_have_zero_gradient():
    # Causal with seq_q > seq_k: the first seq_q - seq_k rows see no key.
    rng = np.random.default_rng(5)
    Q = rng.standard_normal((1, 40, 64)).astype(np.float32)
    K = rng.standard_normal((1, 24, 64)).astype(np.float32)
    V = rng.standard_normal((1, 24, 64)).astype(np.float32)
    dO = rng.standard_normal((1, 40, 64)).astype(np.float32)
    dq, dk, dv = oracle.fp4_attention_backward(Q, K, V, dO, causal=True, threads=2)
    assert np.all(dq[0, :16] == 0)
    assert np.abs(dq[0, 16:]).max() > 0
    lse = oracle.fp4_attention_lse(Q, K, causal=True)
    assert np.all(lse[0, :16] == np.inf) and np.all(np.isfinite(lse[0, 16:]))


def test_dv_is_independent_of_the_threads():
    # The per-thread double accumulators are summed in a fixed order.
    rng = np.random.default_rng(9)
    Q, K, V, dO = (rng.standard_normal((1, 96, 64)).astype(np.float32) for _ in range(4))
    a = oracle.fp4_attention_backward(Q, K, V, dO, threads=1)
    b = oracle.fp4_attention_backward(Q, K, V, dO, threads=5)
    for x, y in zip(a, b):
        assert np.abs(x - y).max() <= 1e-6 * np.abs(x).max()
