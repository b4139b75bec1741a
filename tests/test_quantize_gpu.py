"""GPU quantiser vs the oracle and the reference's golden vectors: codes and
scales must be bit-exact (common.h:21-48, :115-123)."""
import numpy as np
import pytest
import torch

import golden_inputs as gi
import oracle

pytestmark = pytest.mark.gpu


def gpu_quant(fa, x_np, dtype=torch.float32, mode="reference"):
    x = torch.from_numpy(np.ascontiguousarray(x_np)).to(dtype).cuda()
    c, s = fa.quantize(x, scale_mode=mode)
    assert fa.status_query() == fa.OK
    return c.cpu().numpy(), s.cpu().numpy()


def test_edge_vectors_fp32_input(fa, cuda, golden_dir):
    g = np.load(golden_dir / "quant_edge.npz")
    c, s = gpu_quant(fa, gi.quant_edge_rows())
    assert np.array_equal(s, g["scales"])
    assert np.array_equal(c, oracle.pack_codes(g["codes"]))


def test_fp16_vectors(fa, cuda, golden_dir):
    g = np.load(golden_dir / "quant_fp16.npz")
    c, s = gpu_quant(fa, gi.quant_fp16_rows(), torch.float16)
    assert np.array_equal(s, g["scales"])
    assert np.array_equal(c, oracle.pack_codes(g["codes"]))


def test_every_fp16_value_as_block_max(fa, cuda):
    """All 31743 positive finite FP16 values, each the maximum of its block."""
    bits = np.arange(1, 0x7C00, dtype=np.uint16)
    xs = bits.view(np.float16).astype(np.float32)
    rng = np.random.default_rng(0)
    blocks = (rng.uniform(-1, 1, (xs.size, 32)) * xs[:, None]).astype(np.float16).astype(np.float32)
    blocks[:, 7] = -xs
    c, s = gpu_quant(fa, blocks, torch.float16)
    oc, os_ = oracle.quantize(blocks)
    assert np.array_equal(s[:, 0], os_[:, 0])
    assert np.array_equal(c, oracle.pack_codes(oc))


def test_fp32_values_just_above_powers_of_two(fa, cuda):
    """Where the reference's host log2f rounds ceil(log2 x) down (x = 2^p + k ulp,
    small k) the GPU must follow it, across every binade and subnormals."""
    vals = []
    for p in range(-126, 128):
        vals += [((p + 127) << 23) + k for k in range(0, 26)] + [((p + 127) << 23) + 0x7FFFFF]
    for msb in range(0, 23):
        vals += [(1 << msb) + k for k in range(0, 13) if (1 << msb) + k < (1 << 23)]
    xs = np.array(vals, np.uint32).view(np.float32)
    blocks = np.zeros((xs.size, 32), np.float32)
    blocks[:, 0] = xs
    blocks[:, 1] = -xs / 3
    blocks[:, 2] = xs / 2
    c, s = gpu_quant(fa, blocks)
    oc, os_ = oracle.quantize(blocks)
    assert np.array_equal(s, os_)
    assert np.array_equal(c, oracle.pack_codes(oc))


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("mode", ["reference", "ocp"])
def test_random_rows_match_oracle(fa, cuda, dtype, mode):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(20000, 256, generator=g) * torch.exp2(torch.randint(-12, 12, (20000, 1), generator=g).float())
    x = x.to(dtype).float().numpy()
    c, s = gpu_quant(fa, x, dtype, mode)
    oc, os_ = oracle.quantize(x, 1 if mode == "ocp" else 0)
    assert np.array_equal(s, os_)
    assert np.array_equal(c, oracle.pack_codes(oc))


@pytest.mark.parametrize("d", [32, 64, 96, 160, 256])
def test_head_dims(fa, cuda, d):
    x = torch.randn(333, d, generator=torch.Generator().manual_seed(d)).half().float().numpy()
    c, s = gpu_quant(fa, x, torch.float16)
    oc, os_ = oracle.quantize(x)
    assert np.array_equal(s, os_) and np.array_equal(c, oracle.pack_codes(oc))


def test_empty_input(fa, cuda):
    x = torch.empty(0, 128, dtype=torch.float16, device="cuda")
    c, s = fa.quantize(x)
    assert c.numel() == 0 and s.numel() == 0 and fa.status_query() == fa.OK


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_devices_in_one_process(fa, cuda):
    """One host process quantising on two devices: each device gets its own
    copy of the scale-rule table, so values where the reference's log2f rounds
    down come out bit-exact on the second device too."""
    vals = []
    for p in range(-126, 128):
        vals += [((p + 127) << 23) + k for k in range(0, 26)]
    xs = np.array(vals, np.uint32).view(np.float32)
    blocks = np.zeros((xs.size, 32), np.float32)
    blocks[:, 0] = xs
    blocks[:, 1] = -xs / 3
    oc, os_ = oracle.quantize(blocks)
    for dev in (0, 1, 0):
        with torch.cuda.device(dev):
            x = torch.from_numpy(blocks).to(f"cuda:{dev}")
            c, s = fa.quantize(x)
            torch.cuda.synchronize(dev)
            assert np.array_equal(s.cpu().numpy(), os_)
            assert np.array_equal(c.cpu().numpy(), oracle.pack_codes(oc))


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_no_writes_outside_codes_and_scales(fa, cuda, dtype):
    """fp4attn_quantize writes rows x D/2 code bytes and rows x D/32 scale
    bytes and nothing around them (guard bytes in place of a sanitizer)."""
    import ctypes
    rows, d, guard = 777, 96, 4096
    x = torch.randn(rows, d, generator=torch.Generator().manual_seed(5)).to(dtype).cuda()
    raw_c = torch.full((rows * d // 2 + 2 * guard,), 0xA5, dtype=torch.uint8, device="cuda")
    raw_s = torch.full((rows * d // 32 + 2 * guard,), 0x5A, dtype=torch.uint8, device="cuda")
    codes, scales = raw_c[guard:guard + rows * d // 2], raw_s[guard:guard + rows * d // 32]
    rc = fa.lib().fp4attn_quantize(x.data_ptr(), fa.F16 if dtype == torch.float16 else fa.F32, rows, d,
                                   codes.data_ptr(), scales.data_ptr(), fa.SCALE_REFERENCE, 0,
                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == fa.OK and fa.status_query() == fa.OK
    for raw, fill in ((raw_c, 0xA5), (raw_s, 0x5A)):
        assert bool((raw[:guard] == fill).all()) and bool((raw[-guard:] == fill).all())
    oc, os_ = oracle.quantize(x.float().cpu().numpy())
    assert np.array_equal(scales.cpu().numpy().reshape(rows, -1), os_)
    assert np.array_equal(codes.cpu().numpy().reshape(rows, -1), oracle.pack_codes(oc))
