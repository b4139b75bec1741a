"""The C ABI boundary without a GPU: the library loads, exports every entry
point include/fp4attn.h declares, and rejects bad arguments before touching
the device (the reference returns no errors at all; common.h:68-77)."""
import ctypes
import pathlib
import re
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "fp4attn.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fp4attn_\w+)\s*\(", text)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for want in ("fp4attn_quantize", "fp4attn_forward", "fp4attn_workspace_size", "fp4attn_debug_scores",
                 "fp4attn_status_query", "fp4attn_error_string", "fp4attn_last_error"):
        assert want in names


def test_library_exports_every_declared_symbol(fa):
    L = fa.lib()
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing


def test_nm_lists_symbols_as_c_linkage(fa):
    out = subprocess.run(["nm", "-D", "--defined-only", str(fa.lib_path())], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r" T (fp4attn_\w+)", out))
    assert set(declared_functions()) <= exported


@pytest.mark.parametrize("compiler,lang", [("gcc", "c"), ("g++", "c++")])
def test_header_compiles_as_c_and_cpp(tmp_path, compiler, lang):
    src = tmp_path / ("t.c" if lang == "c" else "t.cpp")
    src.write_text('#include "fp4attn.h"\nint main(void){ return FP4ATTN_OK + FP4ATTN_BLOCK_ELEMENT - 32; }\n')
    subprocess.run([compiler, "-Wall", "-Werror", "-I", str(ROOT / "include"), str(src), "-o", str(tmp_path / "t")],
                   check=True)


def test_error_strings(fa):
    L = fa.lib()
    for code in range(6):
        assert L.fp4attn_error_string(code)
    assert L.fp4attn_error_string(99) == b"unknown status"


def test_supported_head_dims(fa):
    assert fa.supported_head_dims() == [32, 64, 96, 128, 160, 256]


def test_workspace_size_host_only(fa):
    ws = fa.workspace_size(2, 32, 4096, 4096, 128)
    # Q and K codes (64 B per row) + scale tiles (512 B per 128 Q rows, per
    # 64 K rows)
    assert ws == 2 * 64 * 4096 * 64 + 64 * (32 + 64) * 512
    # head_dim <= 128: Q scale tiles come in pairs (one 128-row tile here,
    # padded to two)
    assert fa.workspace_size(1, 1, 100, 64, 128) == 100 * 64 + 64 * 64 + 2 * 512 + 512
    assert fa.workspace_size(1, 1, 1, 1, 100) == 0
    assert fa.workspace_size(0, 1, 1, 1, 128) == 0
    assert fa.workspace_size(1, 1, 64, 128, 128, fa.F32) > fa.workspace_size(1, 1, 64, 128, 128, fa.F16)


def _fwd(fa, **kw):
    args = dict(Q=16, K=16, V=16, O=16, ind=fa.F16, outd=fa.F32, B=1, H=1, sq=64, sk=128, d=128, scale=0.0,
                mode=0, ws=256, wsb=1 << 30, stream=None)
    args.update(kw)
    return fa.lib().fp4attn_forward(args["Q"], args["K"], args["V"], args["O"], args["ind"], args["outd"],
                                    args["B"], args["H"], args["sq"], args["sk"], args["d"], args["scale"],
                                    args["mode"], args["ws"], args["wsb"], args["stream"])


def test_forward_rejects_bad_arguments_before_the_device(fa):
    assert _fwd(fa, Q=None) == fa.EINVAL
    assert b"null" in fa.lib().fp4attn_last_error()
    assert _fwd(fa, Q=17) == fa.EINVAL          # misaligned
    assert _fwd(fa, ind=7) == fa.EINVAL
    assert _fwd(fa, outd=7) == fa.EINVAL
    assert _fwd(fa, mode=3) == fa.EINVAL
    assert _fwd(fa, sq=0) == fa.EINVAL
    assert _fwd(fa, sk=0) == fa.EINVAL
    assert _fwd(fa, B=-1) == fa.EINVAL
    assert _fwd(fa, d=100) == fa.EUNSUPPORTED
    assert _fwd(fa, d=512) == fa.EUNSUPPORTED
    assert _fwd(fa, B=300, H=300) == fa.EINVAL  # batch*heads > 65535


def test_quantize_rejects_bad_arguments(fa):
    L = fa.lib()
    assert L.fp4attn_quantize(None, fa.F16, 1, 128, 16, 16, 0, 0, None) == fa.EINVAL
    assert L.fp4attn_quantize(16, fa.F16, 1, 100, 16, 16, 0, 0, None) == fa.EINVAL
    assert L.fp4attn_quantize(16, 5, 1, 128, 16, 16, 0, 0, None) == fa.EINVAL
    assert L.fp4attn_quantize(16, fa.F16, 1, 128, 16, 16, 9, 0, None) == fa.EINVAL
    assert L.fp4attn_quantize(16, fa.F16, 1, 128, 16, 16, 0, 4, None) == fa.EINVAL


def test_python_wrapper_errors_carry_detail(fa):
    err = fa.Fp4AttnError(fa.EINVAL, "fp4attn_forward", "null tensor pointer")
    assert "invalid argument" in str(err) and "null tensor pointer" in str(err)


def test_cpp_launcher_header_compiles_and_links(tmp_path, fa):
    """The reference-order C++ launcher (include/fp4_fused_attention.h)
    compiles against the CUDA headers and links against libfp4attn.so."""
    src = tmp_path / "use.cpp"
    src.write_text(
        '#include "fp4_fused_attention.h"\n'
        "int run(const float* q, const float* k, float* o, const float* v) {\n"
        "  return fused_fp4_attention_launch<128>(q, k, o, v, 64, 128, 32);\n}\n"
        "int run16(const __half* q, const __half* k, __half* o, const __half* v) {\n"
        "  return fused_fp4_attention_launch<64>(q, k, o, v, 4096, 4096, 32, 2, nullptr);\n}\n"
        "int main() { return 0; }\n")
    libdir = str(fa.lib_path().parent)
    subprocess.run(["g++", "-std=c++17", "-Wall", "-I", str(ROOT / "include"), "-I", "/usr/local/cuda/include",
                    str(src), "-L", libdir, "-lfp4attn", "-L", "/usr/local/cuda/lib64", "-lcudart",
                    f"-Wl,-rpath,{libdir}", "-o", str(tmp_path / "use")], check=True)


def test_masked_entry_points_reject_bad_mask(fa):
    L = fa.lib()
    assert L.fp4attn_forward_masked(16, 16, 16, 16, fa.F16, fa.F32, 1, 1, 64, 128, 128, 0.0, 0, 7, 256, 1 << 30,
                                    None) == fa.EINVAL
    assert b"mask_mode" in L.fp4attn_last_error()
    assert L.fp4attn_attend_masked(16, 16, fa.F16, fa.F32, 1, 1, 64, 128, 128, 0.0, -1, 256, 1 << 30, None) == fa.EINVAL


def test_backward_workspace_size_host_only(fa):
    # Q codes, K codes (64 B per row), Q scale tiles per 64 rows, K scale tiles
    # per 128 rows, BF16 copies of Q and K, and two FP32 values per padded
    # query row (lse2, Dd).
    B, H, S, d = 2, 32, 4096, 128
    n = B * H
    want = n * S * 64 * 2 + n * (S // 64 + S // 128) * 512 + n * S * d * 2 * 2 + n * S * 4 * 2
    assert fa.backward_workspace_size(B, H, S, S, d) == want
    # FP32 input adds the FP16 copies of V and dO.
    assert fa.backward_workspace_size(B, H, S, S, d, fa.F32) == want + 2 * n * S * d * 2
    assert fa.backward_workspace_size(1, 1, 64, 64, 160) == 0
    assert fa.backward_workspace_size(1, 1, 64, 64, 96) > 0
    assert fa.backward_workspace_size(0, 1, 64, 64, 64) == 0
    assert fa.backward_workspace_size(1, 1, 64, 64, 64, 7) == 0


def _bwd(fa, **kw):
    args = dict(Q=16, K=16, V=16, O=16, dO=16, lse=16, dQ=16, dK=16, dV=16, ind=fa.F16, outd=fa.F16, B=1, H=1,
                sq=64, sk=128, d=128, scale=0.0, mode=0, mask=0, ws=256, wsb=1 << 30, stream=None)
    args.update(kw)
    a = args
    return fa.lib().fp4attn_backward(a["Q"], a["K"], a["V"], a["O"], a["dO"], a["lse"], a["dQ"], a["dK"], a["dV"],
                                     a["ind"], a["outd"], a["B"], a["H"], a["sq"], a["sk"], a["d"], a["scale"],
                                     a["mode"], a["mask"], a["ws"], a["wsb"], a["stream"])


def test_backward_rejects_bad_arguments_before_the_device(fa):
    assert _bwd(fa, dQ=None) == fa.EINVAL
    assert _bwd(fa, lse=18) == fa.EINVAL          # lse must be 4-byte aligned
    assert _bwd(fa, dK=24) == fa.EINVAL           # misaligned
    assert _bwd(fa, outd=5) == fa.EINVAL
    assert _bwd(fa, ind=5) == fa.EINVAL
    assert _bwd(fa, mode=3) == fa.EINVAL
    assert _bwd(fa, mask=2) == fa.EINVAL
    assert _bwd(fa, sq=0) == fa.EINVAL
    assert _bwd(fa, d=160) == fa.EUNSUPPORTED
    assert b"head_dim 32, 64, 96 and 128" in fa.lib().fp4attn_last_error()
    assert _bwd(fa, B=300, H=300) == fa.EINVAL
    assert _bwd(fa, wsb=100) == fa.EWORKSPACE
    assert _bwd(fa, ws=272) == fa.EINVAL          # workspace not 256-byte aligned
    L = fa.lib()
    assert L.fp4attn_backward_attend(16, 16, 16, 16, 16, fa.F16, 1, 1, 64, 128, 64, 0.0, 9, 256, 1 << 30,
                                     None) == fa.EINVAL
    assert L.fp4attn_backward_prepare(16, 16, 16, 16, 16, 16, 16, fa.F16, fa.F16, 1, 1, 64, 128, 256, 0, 256, 1 << 30,
                                      None) == fa.EUNSUPPORTED


def test_forward_lse_rejects_bad_arguments_before_the_device(fa):
    L = fa.lib()
    args = [16, 16, 16, 16, 16, fa.F16, fa.F32, 1, 1, 64, 128, 128, 0.0, 0, 0, 256, 1 << 30, None]
    bad = list(args)
    bad[4] = None  # lse
    assert L.fp4attn_forward_lse(*bad) == fa.EINVAL
    bad = list(args)
    bad[11] = 160  # head_dim outside the backward's dims
    assert L.fp4attn_forward_lse(*bad) == fa.EUNSUPPORTED
    bad = list(args)
    bad[14] = 5    # mask
    assert L.fp4attn_forward_lse(*bad) == fa.EINVAL
