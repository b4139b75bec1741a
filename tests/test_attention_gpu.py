"""GPU FP4 attention vs the oracle (the reference's cpu_attention on the
reference-quantised Q and K, tests/test_attention.cu:33-54) and vs golden
vectors made by the reference's own code.

Tolerance (written here, from the spec of the path): cosine >= 0.9999
(computed in double) and max |out - oracle| <= 2e-2.  The GPU rounds P and V
to FP16 for the tensor cores; the oracle keeps them in FP32."""
import numpy as np
import pytest
import torch

import golden_inputs as gi
import oracle

pytestmark = pytest.mark.gpu

COS_MIN = 0.9999
MAXABS = 2e-2


def run_fwd(fa, Q, K, V, in_dtype=torch.float16, out_dtype=torch.float32, mode="reference", scale=None):
    """Q/K/V: [slices, seq, d] numpy float32; runs as [1, slices, seq, d]."""
    t = [torch.from_numpy(np.ascontiguousarray(a)).to(in_dtype).cuda()[None] for a in (Q, K, V)]
    out = fa.fused_fp4_attention(*t, out_dtype=out_dtype, scale_mode=mode, softmax_scale=scale)
    assert fa.status_query() == fa.OK
    return out[0].float().cpu().numpy()


def assert_close(got, want, cos_min=COS_MIN, maxabs=MAXABS):
    assert np.isfinite(got).all()
    cos = oracle.cosine(got, want)
    err = float(np.abs(got - want).max())
    assert cos >= cos_min and err <= maxabs, (cos, err)


@pytest.mark.parametrize("name", list(gi.ATTN_CASES))
def test_golden_cases(fa, cuda, golden_dir, name):
    g = np.load(golden_dir / f"attn_{name}.npz")
    Q, K, V = gi.attn_inputs(name)
    out = run_fwd(fa, Q, K, V)
    assert_close(out[g["slices"]], g["out"])
    assert_close(out, oracle.fp4_attention(Q, K, V))


@pytest.mark.parametrize("name", list(gi.DISCRETE_CASES))
def test_reference_test_fixtures(fa, cuda, golden_dir, name):
    """The reference's test_attention.cu inputs and shapes, compared with its
    unquantised CPU reference as that test does (there at cosine >= 0.99)."""
    d, sk, B, H = gi.DISCRETE_CASES[name]
    Q, K, V = gi.discrete_inputs(d, sk, B, H)
    g = np.load(golden_dir / f"discrete_{name}.npz")["out"]
    out = run_fwd(fa, Q, K, V, in_dtype=torch.float32)
    assert_close(out, g)


@pytest.mark.parametrize("in_dtype,out_dtype", [(torch.float32, torch.float32), (torch.float16, torch.float16),
                                                (torch.float32, torch.float16), (torch.float16, torch.float32)])
def test_dtypes(fa, cuda, in_dtype, out_dtype):
    Q, K, V = gi.attn_inputs("cpu_check")
    out = run_fwd(fa, Q, K, V, in_dtype, out_dtype)
    assert_close(out, oracle.fp4_attention(Q, K, V))


def test_ocp_scale_mode(fa, cuda):
    Q, K, V = gi.attn_inputs("short_head_long_key")
    out = run_fwd(fa, Q, K, V, mode="ocp")
    assert_close(out, oracle.fp4_attention(Q, K, V, scale_mode=1))


def test_explicit_softmax_scale(fa, cuda):
    Q, K, V = gi.attn_inputs("d32")
    out = run_fwd(fa, Q, K, V, scale=0.05)
    assert_close(out, oracle.fp4_attention(Q, K, V, scale=0.05))


@pytest.mark.parametrize("d", [32, 64, 96, 128, 160, 256])
@pytest.mark.parametrize("sq,sk", [(1, 1), (64, 65), (129, 127), (200, 513)])
def test_shapes(fa, cuda, d, sq, sk):
    g = torch.Generator().manual_seed(d * 7 + sq + sk)
    Q, K, V = [(torch.randn(2, s, d, generator=g)).half().float().numpy() for s in (sq, sk, sk)]
    out = run_fwd(fa, Q, K, V)
    assert_close(out, oracle.fp4_attention(Q, K, V))


@pytest.mark.parametrize("d", [32, 64, 96, 128, 160, 256])
def test_scores_bit_exact(fa, cuda, d):
    """S = Q K^T of FP4 codes with power-of-two scales is exact in FP32 here,
    so the tcgen05 block-scaled product must equal the oracle bit for bit
    (the reference's debug_mma, common.h:331-398, for whole problems)."""
    g = torch.Generator().manual_seed(d)
    Q = torch.randn(1, 3, 130, d, generator=g).half()
    K = torch.randn(1, 3, 200, d, generator=g).half()
    S = fa.debug_scores(Q.cuda(), K.cuda())
    assert fa.status_query() == fa.OK
    S = S.cpu().numpy()
    for h in range(3):
        want = oracle.fp4_scores(Q[0, h].float().numpy(), K[0, h].float().numpy())
        assert np.array_equal(S[0, h], want)


def test_zero_inputs_give_mean_of_v(fa, cuda):
    Q = np.zeros((2, 70, 128), np.float32)
    K = np.zeros((2, 300, 128), np.float32)
    V = torch.randn(2, 300, 128, generator=torch.Generator().manual_seed(3)).half().float().numpy()
    out = run_fwd(fa, Q, K, V)
    want = np.broadcast_to(V.mean(axis=1, keepdims=True), out.shape)
    assert_close(out, want)


def test_large_outliers(fa, cuda):
    g = torch.Generator().manual_seed(9)
    Q, K, V = [torch.randn(4, 256, 128, generator=g) for _ in range(3)]
    Q[:, :, ::17] *= 300
    K[:, ::5, 3] *= 200
    Q, K, V = [x.half().float().numpy() for x in (Q, K, V)]
    out = run_fwd(fa, Q, K, V)
    assert_close(out, oracle.fp4_attention(Q, K, V))


@pytest.mark.parametrize("growth", [3, 4, 6])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_row_max_jumps_at_later_key_tiles(fa, cuda, out_dtype, growth):
    """Scores of half of the rows grow from one 64-key tile to the next by
    about 10 (growth 3), 14 (growth 4) or 20 (growth 6) in log2 units.  Below
    the lazy-rescale threshold (2^15) P values up to ~2^14 enter FP16 and the
    P.V MMA with no rescale; above it those rows take the max-first path and
    rescale O at steps after the first.  The other rows keep their reference
    max; the last key tile is ragged."""
    g = torch.Generator().manual_seed(11)
    sq, sk = 300, 64 * 9 + 17
    Q, K, V = (torch.randn(3, sq, 128, generator=g), torch.randn(3, sk, 128, generator=g),
               torch.randn(3, sk, 128, generator=g))
    for k in range(10):
        K[:, 64 * k:64 * (k + 1)] *= 1 + growth * k
    Q[:, 1::2] *= 0.02
    Q, K, V = [x.half().float().numpy() for x in (Q, K, V)]
    out = run_fwd(fa, Q, K, V, out_dtype=out_dtype)
    assert_close(out, oracle.fp4_attention(Q, K, V))


def test_timeout_path_reports_and_recovers(fa, cuda):
    """A bounded wait that nothing completes: the kernel records
    FP4ATTN_ETIMEOUT and returns; the context stays usable."""
    assert fa.selftest_timeout(2000) == fa.ETIMEOUT
    assert fa.status_query() == fa.OK  # the query cleared the word
    Q, K, V = gi.attn_inputs("d32")
    assert_close(run_fwd(fa, Q, K, V), oracle.fp4_attention(Q, K, V))


def test_attention_kernel_abort_path_drains_and_recovers(fa, cuda):
    """The attention kernel's own failure path, made to run without a fault: a
    test build in which one softmax thread withholds its first "S copied"
    arrival, so the S issuer's bounded wait for the next step expires.  Every
    role must leave its loop, drain its in-flight TMA loads and MMAs, free its
    tensor memory and return: the call reports FP4ATTN_ETIMEOUT, and the
    normal kernel then runs on the same context and workspace and matches
    the oracle."""
    B, H, sq, sk, d = 1, 2, 256, 256, 64
    g = torch.Generator().manual_seed(21)
    Q, K, V = (torch.randn(B, H, s, d, generator=g).half().cuda() for s in (sq, sk, sk))
    ws = torch.empty(fa.workspace_size(B, H, sq, sk, d), dtype=torch.uint8, device="cuda")
    out = torch.zeros(B, H, sq, d, dtype=torch.float32, device="cuda")
    fa.prepare(Q, K, V, ws)
    assert fa.status_query() == fa.OK
    assert fa.selftest_abort(V, out, ws, B, H, sq, sk, timeout_us=20000) == fa.ETIMEOUT
    assert b"device wait expired" in fa.lib().fp4attn_last_error()
    assert fa.status_query() == fa.OK  # the query cleared the word
    fa.attend(V, out, ws, fa.F16, B, H, sq, sk, d)
    assert fa.status_query() == fa.OK
    want = oracle.fp4_attention(Q[0].float().cpu().numpy(), K[0].float().cpu().numpy(), V[0].float().cpu().numpy())
    assert_close(out[0].cpu().numpy(), want)


def test_abort_self_test_rejects_other_shapes(fa, cuda):
    ws = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    V = torch.zeros(1, 1, 256, 128, dtype=torch.float16, device="cuda")
    out = torch.zeros(1, 1, 256, 128, dtype=torch.float32, device="cuda")
    rc = fa.lib().fp4attn_selftest_abort(V.data_ptr(), out.data_ptr(), 1, 1, 64, 256, ws.data_ptr(), ws.numel(),
                                         1000, torch.cuda.current_stream().cuda_stream)
    assert rc == fa.EINVAL  # seq_q <= 128 runs the small-problem kernel, not the test build


def test_misaligned_pointer_rejected(fa, cuda):
    x = torch.zeros(1, 1, 65, 128, dtype=torch.float16, device="cuda")
    bad = x.view(-1)[1:1 + 64 * 128].view(1, 1, 64, 128)
    with pytest.raises(fa.Fp4AttnError) as e:
        fa.fused_fp4_attention(bad, bad, bad)
    assert e.value.code == fa.EINVAL


def test_workspace_too_small(fa, cuda):
    Q = torch.zeros(1, 1, 64, 128, dtype=torch.float16, device="cuda")
    out = torch.empty_like(Q)
    ws = torch.empty(16, dtype=torch.uint8, device="cuda")
    with pytest.raises(fa.Fp4AttnError) as e:
        fa.fused_fp4_attention_into(Q, Q, Q, out, ws)
    assert e.value.code == fa.EWORKSPACE


# ------------------------------------------------- full-size workloads
# Each full-size workload is checked three ways: every output lies inside V's
# per-column range (a convex combination of V rows: a size-independent
# property), sampled query rows of sampled slices against the oracle for those
# rows, and whole slices -- every query row -- against the oracle run over the
# host's cores.
def _check_whole_slices(Q, K, V, out, slices, odt):
    for s in slices:
        want = oracle.fp4_attention_slice(Q[s].float().cpu().numpy(), K[s].float().cpu().numpy(),
                                          V[s].float().cpu().numpy())
        if odt == torch.float16:
            want = want.astype(np.float16).astype(np.float32)
        assert_close(out[s].float().cpu().numpy(), want)


def _full_size(fa, name, n_slices_checked=3, rows_per_slice=6, seed=42, whole=(0,)):
    import fp4attn_b200.workloads as wl
    w = wl.WORKLOADS[name]
    Q, K, V = wl.make_inputs(w, seed)
    odt = torch.float16 if w.out_dtype == "float16" else torch.float32
    out = fa.fused_fp4_attention(Q[None], K[None], V[None], out_dtype=odt)[0]
    assert fa.status_query() == fa.OK
    assert torch.isfinite(out).all()
    vmin, vmax = V.float().amin(dim=1, keepdim=True), V.float().amax(dim=1, keepdim=True)
    tol = 1e-2 + 1e-3 * V.float().abs().amax()
    assert (out.float() >= vmin - tol).all() and (out.float() <= vmax + tol).all()
    rng = np.random.default_rng(seed)
    sl = rng.choice(w.slices, size=min(n_slices_checked, w.slices), replace=False)
    s_of, rows = [], []
    for s in sl:
        for r in rng.choice(w.seq_q, size=rows_per_slice, replace=False):
            s_of.append(int(s)); rows.append(int(r))
    s_of, rows = np.array(s_of, np.int32), np.array(rows, np.int32)
    uniq = sorted(set(s_of.tolist()))
    remap = {s: i for i, s in enumerate(uniq)}
    Qc = Q[uniq].float().cpu().numpy(); Kc = K[uniq].float().cpu().numpy(); Vc = V[uniq].float().cpu().numpy()
    want = oracle.fp4_attention_rows(Qc, Kc, Vc, np.array([remap[s] for s in s_of], np.int32), rows)
    got = out.float()[torch.from_numpy(s_of).long(), torch.from_numpy(rows).long()].cpu().numpy()
    if odt == torch.float16:
        want = want.astype(np.float16).astype(np.float32)
    assert_close(got, want)
    _check_whole_slices(Q, K, V, out, list(whole) + [w.slices - 1], odt)


def test_full_prefill_4k(fa, cuda):
    _full_size(fa, "prefill_4k")


def test_full_odd_d96(fa, cuda):
    _full_size(fa, "odd_d96")


def test_full_odd_d256(fa, cuda):
    _full_size(fa, "odd_d256")


def test_full_box_sharded_8k_one_gpu_shard(fa, cuda):
    """The 512-slice box-scale workload as one GPU of eight runs it (64
    slices): two whole 8192-row slices and sampled rows of two more against
    the oracle.  Its outliers (0.5% of elements x16) make a row's max jump
    past the lazy-rescale threshold in many (warp, key step) pairs; the
    row-max statistics of the checked slices must show that the kernel's
    max-first redo path is taken there, so that path is what is checked."""
    import fp4attn_b200.workloads as wl
    w = wl.WORKLOADS["box_sharded_8k"]
    Q, K, V = wl.make_inputs(w, 7, slices=(448, 512))
    out = fa.fused_fp4_attention(Q[None], K[None], V[None], out_dtype=torch.float32)[0]
    assert fa.status_query() == fa.OK
    assert torch.isfinite(out).all()
    whole = [0, 63]
    for s in whole:
        redone, total = oracle.redo_warp_steps(Q[s].float().cpu().numpy(), K[s].float().cpu().numpy())
        assert redone >= 0.02 * total, (redone, total)
    _check_whole_slices(Q, K, V, out, whole, torch.float32)
    idx = [17, 40]
    rows = np.array([5, 8000], np.int32)
    want = oracle.fp4_attention_rows(Q[idx].float().cpu().numpy(), K[idx].float().cpu().numpy(),
                                     V[idx].float().cpu().numpy(), np.array([0, 1], np.int32), rows)
    got = out[torch.tensor(idx), torch.from_numpy(rows).long()].cpu().numpy()
    assert_close(got, want)


def test_fma_pipe_exp2_error_bound(fa, cuda):
    """The polynomial 2^x the softmax computes on the FMA pipe for part of
    the exponentials: relative error <= 7.6e-5 (the degree-3 minimax bound of
    fit_exp2_poly.py) where the result is a normal float, and a finite value
    in [0, 2^-125) for arguments at or below -126, -inf included (zero after
    the FP16 rounding of P)."""
    x = torch.cat([torch.linspace(-130.0, 8.0, 2_000_000),
                   torch.tensor([-126.0, -127.0, -200.0, -1e30, float("-inf"), 0.0])])
    y = fa.selftest_exp2(x.cuda()).cpu().double()
    assert torch.isfinite(y).all()
    want = torch.exp2(x.double())
    body = x > -125.0
    rel = ((y[body] - want[body]).abs() / want[body]).max().item()
    assert rel <= 7.6e-5, rel
    low = x <= -126.0
    assert (y[low] < 2.0 ** -125).all() and (y[low] >= 0).all()


# ---- causal mask (an extension: the reference has no mask) -----------------

@pytest.mark.parametrize("d", [32, 64, 96, 128, 160, 256])
@pytest.mark.parametrize("sq,sk", [(1, 1), (64, 65), (129, 127), (300, 300), (200, 513), (513, 200)])
def test_causal_shapes(fa, cuda, d, sq, sk):
    """Bottom-right causal mask: query i sees keys j <= i + sk - sq; with
    sq > sk the first sq - sk rows see no key and must come out as zeros."""
    g = torch.Generator().manual_seed(d * 1000 + sq + sk)
    Q, K, V = (torch.randn(2, sq, d, generator=g), torch.randn(2, sk, d, generator=g),
               torch.randn(2, sk, d, generator=g))
    Q, K, V = [x.half().float().numpy() for x in (Q, K, V)]
    t = [torch.from_numpy(np.ascontiguousarray(a)).half().cuda()[None] for a in (Q, K, V)]
    out = fa.fused_fp4_attention(*t, out_dtype=torch.float32, causal=True)
    assert fa.status_query() == fa.OK
    got = out[0].cpu().numpy()
    want = oracle.fp4_attention(Q, K, V, causal=True)
    if sq > sk:
        assert np.abs(got[:, :sq - sk]).max() == 0.0
    assert_close(got, want)


def test_causal_many_items_and_split_api(fa, cuda):
    """Several 256-row work items per slice, each stopping at its own last key
    tile; fp4attn_prepare + fp4attn_attend_masked gives the same bytes as
    fp4attn_forward_masked."""
    g = torch.Generator().manual_seed(77)
    sq = sk = 1500
    Q, K, V = (torch.randn(1, 3, sq, 128, generator=g).half().cuda() for _ in range(3))
    out = fa.fused_fp4_attention(Q, K, V, out_dtype=torch.float32, causal=True)
    ws = torch.empty(fa.workspace_size(1, 3, sq, sk, 128), dtype=torch.uint8, device="cuda")
    out2 = torch.empty_like(out)
    fa.prepare(Q, K, V, ws)
    fa.attend(V, out2, ws, fa.F16, 1, 3, sq, sk, 128, causal=True)
    assert fa.status_query() == fa.OK
    assert torch.equal(out, out2)
    want = oracle.fp4_attention(Q[0].float().cpu().numpy(), K[0].float().cpu().numpy(), V[0].float().cpu().numpy(),
                                causal=True)
    assert_close(out[0].cpu().numpy(), want)


def test_causal_full_prefill_sampled_rows(fa, cuda):
    """The bench shape (B2 H32 sq=sk=4096 d128, FP16 out) under the causal
    mask, checked on sampled rows of sampled slices against the oracle."""
    import fp4attn_b200.workloads as wl
    w = wl.WORKLOADS["prefill_4k"]
    Q, K, V = wl.make_inputs(w, 1)
    Q, K, V = Q[None], K[None], V[None]
    out = fa.fused_fp4_attention(Q, K, V, out_dtype=torch.float16, causal=True)
    assert fa.status_query() == fa.OK
    rng = np.random.default_rng(5)
    for s in (0, 37, 63):
        kq = K[0, s].float().cpu().numpy()
        kd = oracle.dequantize(*oracle.quantize(kq))
        vs = V[0, s].float().cpu().numpy()
        for r in sorted(rng.choice(4096, 6, replace=False).tolist()) + [0, 4095]:
            q = Q[0, s, r:r + 1].float().cpu().numpy()
            qd = oracle.dequantize(*oracle.quantize(q))
            want = oracle.attention_causal(qd, kd, vs, first_row=r, seq_q_total=4096)
            got = out[0, s, r:r + 1].float().cpu().numpy()
            assert_close(got, want)


# ---- several work items per persistent CTA ---------------------------------
# Both kernels run one CTA per SM over (slice, query tile[s]) items; with more
# items than SMs each CTA carries its barrier phases, rings and Q buffers from
# one item to the next.  These cases have 300-600 items.

@pytest.mark.parametrize("d", [160, 256])
@pytest.mark.parametrize("causal", [False, True])
def test_one_tile_kernel_many_items(fa, cuda, d, causal):
    g = torch.Generator().manual_seed(d + causal)
    H, sq, sk = 300, 256 if causal else 128, 200
    Q, K, V = (torch.randn(1, H, sq, d, generator=g).half(), torch.randn(1, H, sk, d, generator=g).half(),
               torch.randn(1, H, sk, d, generator=g).half())
    out = fa.fused_fp4_attention(Q.cuda(), K.cuda(), V.cuda(), out_dtype=torch.float32, causal=causal)
    assert fa.status_query() == fa.OK
    want = oracle.fp4_attention(Q[0].float().numpy(), K[0].float().numpy(), V[0].float().numpy(), causal=causal)
    assert_close(out[0].cpu().numpy(), want)


@pytest.mark.parametrize("d", [64, 256])
def test_scores_bit_exact_many_items(fa, cuda, d):
    g = torch.Generator().manual_seed(d + 5)
    Q = torch.randn(1, 200, 130, d, generator=g).half()
    K = torch.randn(1, 200, 70, d, generator=g).half()
    S = fa.debug_scores(Q.cuda(), K.cuda())
    assert fa.status_query() == fa.OK
    S = S.cpu().numpy()
    for h in (0, 77, 199):
        want = oracle.fp4_scores(Q[0, h].float().numpy(), K[0, h].float().numpy())
        assert np.array_equal(S[0, h], want)


# ---- CUDA graphs ----------------------------------------------------------
# The API makes no allocation and no host synchronisation, so a forward pass
# with a caller workspace can be captured once and replayed on new inputs
# copied into the captured buffers.

@pytest.mark.parametrize("d,causal", [(128, False), (128, True), (256, False)])
def test_cuda_graph_replay(fa, cuda, d, causal):
    B, H, sq, sk = 1, 8, 300, 700
    Q, K, V = (torch.empty(B, H, s, d, dtype=torch.float16, device="cuda") for s in (sq, sk, sk))
    out = torch.empty(B, H, sq, d, dtype=torch.float16, device="cuda")
    ws = torch.empty(fa.workspace_size(B, H, sq, sk, d), dtype=torch.uint8, device="cuda")

    def fill(seed):
        g = torch.Generator().manual_seed(seed)
        for t in (Q, K, V):
            t.copy_(torch.randn(t.shape, generator=g).half())

    fill(0)
    fa.fused_fp4_attention_into(Q, K, V, out, ws, causal=causal)  # per-device set-up happens outside capture
    assert fa.status_query() == fa.OK
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fa.fused_fp4_attention_into(Q, K, V, out, ws, causal=causal)
    for seed in (1, 2):
        fill(seed)
        graph.replay()
        assert fa.status_query() == fa.OK
        want = fa.fused_fp4_attention(Q, K, V, out_dtype=torch.float16, causal=causal)
        assert fa.status_query() == fa.OK
        assert torch.equal(out, want)  # the same kernels on the same inputs
        ref = oracle.fp4_attention(Q[0].float().cpu().numpy(), K[0].float().cpu().numpy(),
                                   V[0].float().cpu().numpy(), causal=causal)
        assert_close(out[0].float().cpu().numpy(), ref)
    del graph


# ---- guard bytes --------------------------------------------------------------
# No sanitizer runs here, so writes are checked directly.  The output and the
# workspace sit inside larger buffers filled with a sentinel byte, and after a
# forward pass the bytes on both sides (and the inputs) must be unchanged.
# Ragged seq_q leaves a partial query tile and, for head_dim <= 128, a padding
# tile of the last pair; their rows must not be stored.

@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("sq,causal", [(1, False), (130, False), (300, True)])
def test_no_writes_outside_the_output_and_workspace(fa, cuda, d, out_dtype, sq, causal):
    B, H, sk, guard = 1, 3, 200, 4096
    g = torch.Generator().manual_seed(d + sq)
    Q, K, V = (torch.randn(B, H, s, d, generator=g).half().cuda() for s in (sq, sk, sk))
    inputs_before = [t.clone() for t in (Q, K, V)]
    out_bytes = B * H * sq * d * torch.empty((), dtype=out_dtype).element_size()
    raw_out = torch.full((out_bytes + 2 * guard,), 0xA5, dtype=torch.uint8, device="cuda")
    out = raw_out[guard:guard + out_bytes].view(out_dtype).view(B, H, sq, d)
    ws_bytes = fa.workspace_size(B, H, sq, sk, d)
    raw_ws = torch.full((ws_bytes + 2 * guard,), 0x5A, dtype=torch.uint8, device="cuda")
    ws = raw_ws[guard:guard + ws_bytes]
    fa.fused_fp4_attention_into(Q, K, V, out, ws, causal=causal)
    assert fa.status_query() == fa.OK
    for raw, fill in ((raw_out, 0xA5), (raw_ws, 0x5A)):
        assert bool((raw[:guard] == fill).all()) and bool((raw[-guard:] == fill).all())
    for t, t0 in zip((Q, K, V), inputs_before):
        assert torch.equal(t, t0)
    want = oracle.fp4_attention(Q[0].float().cpu().numpy(), K[0].float().cpu().numpy(), V[0].float().cpu().numpy(),
                                causal=causal)
    got = out[0].float().cpu().numpy()
    if out_dtype == torch.float16:
        want = want.astype(np.float16).astype(np.float32)
    assert_close(got, want)


@pytest.mark.parametrize("sk,d", [(70, 64), (68, 64), (68, 160), (200, 96)])
def test_no_writes_outside_the_scores(fa, cuda, sk, d):
    """fp4attn_debug_scores writes exactly the [slices, seq_q, seq_k] FP32
    scores (ragged in both dimensions) and nothing around them -- by TMA
    stores when seq_k % 4 == 0, by per-thread stores otherwise."""
    import ctypes
    B, H, sq, guard = 1, 2, 130, 4096
    g = torch.Generator().manual_seed(17)
    Q, K = (torch.randn(B, H, s, d, generator=g).half().cuda() for s in (sq, sk))
    n = B * H * sq * sk * 4
    raw = torch.full((n + 2 * guard,), 0xA5, dtype=torch.uint8, device="cuda")
    S = raw[guard:guard + n].view(torch.float32)
    ws = torch.empty(fa.workspace_size(B, H, sq, sk, d), dtype=torch.uint8, device="cuda")
    rc = fa.lib().fp4attn_debug_scores(Q.data_ptr(), K.data_ptr(), S.data_ptr(), fa.F16, B, H, sq, sk, d,
                                       fa.SCALE_REFERENCE, ws.data_ptr(), ws.numel(),
                                       ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == fa.OK and fa.status_query() == fa.OK
    assert bool((raw[:guard] == 0xA5).all()) and bool((raw[-guard:] == 0xA5).all())
    S = S.view(H, sq, sk).cpu().numpy()
    for h in range(H):
        assert np.array_equal(S[h], oracle.fp4_scores(Q[0, h].float().cpu().numpy(), K[0, h].float().cpu().numpy()))


# ---- small problems: one query tile per item, key partitions ---------------
# With seq_q <= 128 a work item is one query tile, and with fewer query groups
# than SMs the keys of each group are split into partitions whose partial
# results the last-finishing CTA merges.  The arrival counters that pick that
# CTA are back at zero after every launch, so repeated launches on one
# prepared workspace give the same bytes.

@pytest.mark.parametrize("d", [32, 64, 96, 128])
@pytest.mark.parametrize("B,H,sq,sk", [(1, 32, 64, 128), (1, 32, 64, 1024), (1, 2, 1, 4000), (1, 3, 128, 77),
                                       (1, 2, 300, 1000), (2, 1, 700, 3000)])
def test_key_partitions(fa, cuda, d, B, H, sq, sk):
    g = torch.Generator().manual_seed(d * 31 + sq + sk)
    Q, K, V = (torch.randn(B, H, s, d, generator=g).half() for s in (sq, sk, sk))
    for odt in (torch.float32, torch.float16):
        out = fa.fused_fp4_attention(Q.cuda(), K.cuda(), V.cuda(), out_dtype=odt)
        assert fa.status_query() == fa.OK
        want = oracle.fp4_attention(Q.reshape(-1, sq, d).float().numpy(), K.reshape(-1, sk, d).float().numpy(),
                                    V.reshape(-1, sk, d).float().numpy())
        if odt == torch.float16:
            want = want.astype(np.float16).astype(np.float32)
        assert_close(out.reshape(-1, sq, d).float().cpu().numpy(), want)


@pytest.mark.parametrize("B,H,sq,sk,d", [(1, 1, 64, 32768, 128), (1, 3, 200, 5000, 96), (1, 2, 128, 700, 32)])
def test_key_partitions_fp32_input_and_long_keys(fa, cuda, B, H, sq, sk, d):
    """FP32 input (V staged as FP16 by the quantiser launch) with key
    partitions, up to the 16-partition cap (32768 keys on one slice)."""
    g = torch.Generator().manual_seed(sk + d)
    Q, K, V = (torch.randn(B, H, s, d, generator=g).half().float() for s in (sq, sk, sk))
    out = fa.fused_fp4_attention(Q.cuda(), K.cuda(), V.cuda(), out_dtype=torch.float32)
    assert fa.status_query() == fa.OK
    want = oracle.fp4_attention(Q.reshape(-1, sq, d).numpy(), K.reshape(-1, sk, d).numpy(),
                                V.reshape(-1, sk, d).numpy())
    assert_close(out.reshape(-1, sq, d).cpu().numpy(), want)


def test_concurrent_calls_on_two_streams(fa, cuda):
    """Two problems (one split into key partitions, one not) on two streams
    with their own workspaces, launched back to back so that they can run
    concurrently: both match the same calls made one at a time."""
    g = torch.Generator().manual_seed(99)
    shapes = [(1, 4, 64, 3000, 64), (1, 16, 1000, 900, 128)]
    ins = [[torch.randn(B, H, s, d, generator=g).half().cuda() for s in (sq, sk, sk)] for B, H, sq, sk, d in shapes]
    outs = [torch.empty(x[0].shape, dtype=torch.float32, device="cuda") for x in ins]
    wss = [torch.empty(fa.workspace_size(B, H, sq, sk, d), dtype=torch.uint8, device="cuda")
           for B, H, sq, sk, d in shapes]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    torch.cuda.synchronize()
    for _ in range(3):
        for x, o, w, st in zip(ins, outs, wss, streams):
            fa.fused_fp4_attention_into(*x, o, w, stream=st)
    torch.cuda.synchronize()
    assert fa.status_query() == fa.OK
    for x, o in zip(ins, outs):
        want = fa.fused_fp4_attention(*x, out_dtype=torch.float32)
        assert fa.status_query() == fa.OK
        assert torch.equal(o, want)


def test_key_partitions_repeat_on_one_workspace(fa, cuda):
    """Launch after launch on one prepared workspace: the same bytes."""
    B, H, sq, sk, d = 1, 4, 64, 2000, 64
    g = torch.Generator().manual_seed(5)
    Q, K, V = (torch.randn(B, H, s, d, generator=g).half().cuda() for s in (sq, sk, sk))
    ws = torch.empty(fa.workspace_size(B, H, sq, sk, d), dtype=torch.uint8, device="cuda")
    fa.prepare(Q, K, V, ws)
    outs = []
    for _ in range(3):
        out = torch.empty(B, H, sq, d, dtype=torch.float32, device="cuda")
        fa.attend(V, out, ws, fa.F16, B, H, sq, sk, d)
        outs.append(out)
    assert fa.status_query() == fa.OK
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    want = oracle.fp4_attention(Q[0].float().cpu().numpy(), K[0].float().cpu().numpy(), V[0].float().cpu().numpy())
    assert_close(outs[0][0].cpu().numpy(), want)


@pytest.mark.parametrize("sq", [1, 64, 128])
def test_single_tile_items_many_slices(fa, cuda, sq):
    """seq_q <= 128 with more slices than SMs: one query tile per item and
    several items per persistent CTA, no key partitions."""
    g = torch.Generator().manual_seed(sq)
    Q, K, V = (torch.randn(1, 400, s, 128, generator=g).half() for s in (sq, 300, 300))
    out = fa.fused_fp4_attention(Q.cuda(), K.cuda(), V.cuda(), out_dtype=torch.float32)
    assert fa.status_query() == fa.OK
    want = oracle.fp4_attention(Q[0].float().numpy(), K[0].float().numpy(), V[0].float().numpy())
    assert_close(out[0].cpu().numpy(), want)


# ---- Q quantised inside the attention kernel (fp4attn_forward_fused_q) -----
# The in-kernel quantiser uses the pre-pass's encoder, so codes, scales and
# output are those of the two-launch path bit for bit; checked with
# torch.equal, and against the oracle.

@pytest.mark.parametrize("d", [32, 64, 96, 128])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_fused_q_matches_the_two_launch_path(fa, cuda, d, out_dtype):
    B, H, sq, sk = 1, 80, 300, 3100  # 160 query groups, 49 key tiles: the in-kernel quantiser; ragged seq_q, seq_k
    g = torch.Generator().manual_seed(d + 3)
    Q, K, V = (torch.randn(B, H, s, d, generator=g).half().cuda() for s in (sq, sk, sk))
    Q[0, 5, 17, 3] = float("nan")  # a block with a NaN takes the exact encoder in both quantisers (code 0)
    Q[0, 6] *= 40.0
    base = fa.fused_fp4_attention(Q, K, V, out_dtype=out_dtype)
    fused = fa.fused_fp4_attention(Q, K, V, out_dtype=out_dtype, fuse_q=True)
    assert fa.status_query() == fa.OK
    assert torch.equal(base, fused)
    want = oracle.fp4_attention(Q[0].float().cpu().numpy(), K[0].float().cpu().numpy(), V[0].float().cpu().numpy())
    if out_dtype == torch.float16:
        want = want.astype(np.float16).astype(np.float32)
    assert_close(fused[0].float().cpu().numpy(), want)


def test_fused_q_ocp_scale_rule_and_fallbacks(fa, cuda):
    g = torch.Generator().manual_seed(8)
    Q, K, V = (torch.randn(1, 80, s, 64, generator=g).half().cuda() for s in (260, 3100, 3100))
    a = fa.fused_fp4_attention(Q, K, V, out_dtype=torch.float32, scale_mode="ocp")
    b = fa.fused_fp4_attention(Q, K, V, out_dtype=torch.float32, scale_mode="ocp", fuse_q=True)
    assert torch.equal(a, b)
    # Outside the in-kernel quantiser's scope (FP32 input; seq_q <= 128; d=256; short keys): the two-launch path.
    for (dt, sq, sk, d) in ((torch.float32, 260, 3100, 64), (torch.float16, 100, 3100, 64),
                            (torch.float16, 260, 3100, 256), (torch.float16, 260, 300, 64)):
        Q2, K2, V2 = (torch.randn(1, 80, s, d, generator=g).to(dt).cuda() for s in (sq, sk, sk))
        a = fa.fused_fp4_attention(Q2, K2, V2, out_dtype=torch.float32)
        b = fa.fused_fp4_attention(Q2, K2, V2, out_dtype=torch.float32, fuse_q=True)
        assert torch.equal(a, b)
    assert fa.status_query() == fa.OK


def test_fused_q_full_prefill_4k(fa, cuda):
    """The bench workload through the fused path: the same bytes as the two-launch path."""
    import fp4attn_b200.workloads as wl
    w = wl.WORKLOADS["prefill_4k"]
    Q, K, V = (t[None] for t in wl.make_inputs(w, 3))
    a = fa.fused_fp4_attention(Q, K, V, out_dtype=torch.float16)
    b = fa.fused_fp4_attention(Q, K, V, out_dtype=torch.float16, fuse_q=True)
    assert fa.status_query() == fa.OK
    assert torch.equal(a, b)
