"""CPU-side checks of the drop-in boundary: the library loads without a GPU and exports every symbol the headers
in include/ declare (the C ABI and the reference's C++ operator symbols)."""
import ctypes
import pathlib
import re
import subprocess

import pytest

from __graft_entry__ import PKG_DIR, ROOT, load_package

LIB = PKG_DIR / "libnvfp4_b200.so"


def _declared_c_functions(header: pathlib.Path):
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(nvfp4b_\w+)\s*\(", text)))


def _exported():
    out = subprocess.check_output(["nm", "-D", "--defined-only", str(LIB)], text=True)
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


@pytest.fixture(scope="module")
def built():
    if not LIB.exists():
        pytest.fail("libnvfp4_b200.so not built: run __graft_entry__.build()")
    return LIB


def test_c_abi_symbols_exported(built):
    names = _declared_c_functions(ROOT / "include" / "nvfp4_b200.h")
    assert len(names) >= 8
    exported = _exported()
    missing = [n for n in names if n not in exported]
    assert not missing, missing


def test_reference_cpp_symbols_exported(built):
    demangled = subprocess.check_output(f"nm -D --defined-only {built} | c++filt", shell=True, text=True)
    for sig in ["nvfp4_quantize_activations(float const*, unsigned char*, unsigned char*, int, int, float, CUstream_st*)",
                "nvfp4_scale_buffer_bytes(int, int)",
                "nvfp4_swizzle_scales(unsigned char const*, unsigned char*, int, int)",
                "w4a16_gemm(float*, unsigned char const*, unsigned char const*, float, void const*, int, int, int, CUstream_st*)",
                "fp4_gemv(float*, unsigned char const*, unsigned char const*, float, void const*, int, int, CUstream_st*)",
                "nvfp4_gemm(float*, unsigned char const*, unsigned char const*, float, unsigned char const*, unsigned char const*, float, int, int, int, cublasLtContext*, void*, unsigned long, CUstream_st*)"]:
        assert sig in demangled, sig


def test_library_loads_and_host_only_calls_work(built):
    pkg = load_package()
    L = pkg.lib()
    assert b"sm_100a" in L.nvfp4b_version()
    for outer, k in [(1, 16), (130, 192), (8192, 2816), (1408, 2816), (2816, 704)]:
        assert pkg.nvfp4_scale_buffer_bytes(outer, k) == ((outer + 127) // 128) * ((k // 16 + 3) // 4) * 512


def test_host_swizzle_symbol_matches_oracle(built):
    import numpy as np
    import nvfp4_oracle as orc
    L = ctypes.CDLL(str(built))
    fn = getattr(L, "_Z20nvfp4_swizzle_scalesPKhPhii")
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
    rng = np.random.default_rng(3)
    for outer, k in [(130, 192), (7, 48), (256, 2816)]:
        logical = rng.integers(0, 256, (outer, k // 16), dtype=np.uint8)
        out = np.full(orc.scale_buffer_bytes(outer, k), 0xEE, np.uint8)
        fn(logical.ctypes.data, out.ctypes.data, outer, k)
        assert np.array_equal(out, orc.swizzle_scales(logical, outer, k))


def test_argument_errors_need_no_gpu(built):
    pkg = load_package()
    L = pkg.lib()
    # shape / null checks happen before any CUDA call
    assert L.nvfp4b_quantize_bf16(None, 4, 32, 1.0, None, None, None, None) == -3
    assert L.nvfp4b_quantize_bf16(16, 4, 24, 1.0, None, 16, 16, None) == -1          # K % 16
    assert L.nvfp4b_quantize_bf16(8, 4, 32, 1.0, None, 16, 16, None) == -2           # misaligned x
    assert L.nvfp4b_gemm(16, 16, 1.0, None, 16, 16, 1.0, 4, 4, 48, 16, 0, 4, None) == -1   # K % 32
    assert L.nvfp4b_gemm(16, 16, 1.0, None, 16, 16, 1.0, 4, 4, 64, 16, 9, 4, None) == -7   # out kind
    assert L.nvfp4b_hbm_read_stream(None, 256, 1408, None) == -3
    assert L.nvfp4b_hbm_read_stream(16, 256, 1400, None) == -1                        # row_bytes % 128
    assert L.nvfp4b_hbm_read_stream(8, 256, 1408, None) == -2                         # misaligned


def test_linear_workspace_and_argument_errors_need_no_gpu(built):
    pkg = load_package()
    L = pkg.lib()
    r = lambda b: (b + 255) // 256 * 256
    for M, K in [(1, 2816), (128, 2816), (4096, 2112)]:
        w4a4 = r(M * K // 2) + r(pkg.nvfp4_scale_buffer_bytes(M, K))
        assert L.nvfp4b_linear_workspace_bytes(M, K) == 256 + max(w4a4, r(M * K * 2))
    big = 1 << 40
    assert L.nvfp4b_linear(None, 16, 4, 4, 64, 16, 16, 16, 1.0, 1.0, 0, 16, big, None) == -3      # out NULL
    assert L.nvfp4b_linear(16, 16, 4, 4, 24, 16, 16, 16, 1.0, 1.0, 0, 16, big, None) == -1        # K % 16
    assert L.nvfp4b_linear(16, 16, 4, 4, 64, 16, 16, 16, 1.0, 1.0, 0, 16, 64, None) == -1         # workspace size
    assert L.nvfp4b_linear(16, 16, 4, 4, 64, 16, 16, 16, 1.0, 1.0, 7, 16, big, None) == -7        # mode
    assert L.nvfp4b_linear(16, 16, 4, 4, 64, 16, 16, 16, 0.0, 1.0, 0, 16, big, None) == -1        # w_gscale <= 0
    assert L.nvfp4b_linear(16, 8, 4, 4, 64, 16, 16, 16, 1.0, 1.0, 0, 16, big, None) == -2         # misaligned in
    assert L.nvfp4b_linear(16, 16, 4, 4, 48, 16, 16, 16, 1.0, 1.0, 2, 16, big, None) == -1        # W4A4: K % 32
    assert L.nvfp4b_linear(16, 16, 4, 4, 64, 16, 16, None, 1.0, 1.0, 2, 16, big, None) == -3      # W4A4: no tiles
    assert L.nvfp4b_linear(16, 16, 4, 4, 64, 16, None, 16, 1.0, 1.0, 1, 16, big, None) == -3      # W4A16: no raw
    assert L.nvfp4b_amax_f32(8, 16, 16, None) == -2


def test_ep_p2p_layout_and_argument_errors_need_no_gpu(built):
    pkg = load_package()
    G, C, H = 8, 736, 2816
    nbytes, off = pkg.ep_p2p_buffer_layout(G, C, H)
    rb = pkg.ep_record_bytes(H)
    assert rb == H // 2 + H // 16 + 16
    assert all(o % 256 == 0 for o in off)
    assert off[1] >= G * C * rb and off[2] - off[1] >= G * C * H * 2
    assert off[3] - off[2] >= 4 * G and off[4] - off[3] >= 8 * G and nbytes - off[4] >= 16
    L = pkg._p2p_sigs()
    assert L.nvfp4b_ep_p2p_buffer_bytes(0, C, H, None) == 0
    assert L.nvfp4b_ep_p2p_buffer_bytes(G, C, 100, None) == 0            # H % 256
    peers = pkg.EpPeers()                                                 # all NULL
    assert L.nvfp4b_ep_p2p_combine(4, H, 8, 128, 16, peers, 16, 0, None) == -3
    peers = pkg.EpPeers(0, 0, C, 16, 16, 16, 16, 16, 16, 16, 16, 16)      # G = 0
    assert L.nvfp4b_ep_p2p_combine(4, H, 8, 128, 16, peers, 16, 0, None) == -1
    peers = pkg.EpPeers(2, 2, C, 16, 16, 16, 16, 16, 16, 16, 16, 16)      # rank >= G
    assert L.nvfp4b_ep_p2p_combine(4, H, 8, 128, 16, peers, 16, 0, None) == -1
    peers = pkg.EpPeers(0, 2, C, 16, 16, 16, 16, 16, 16, 16, 16, 16)
    assert L.nvfp4b_ep_p2p_combine(4, H, 8, 128, 16, peers, 16, 4, None) == -7   # unknown flag
    assert L.nvfp4b_ep_p2p_combine_chain(4, H, 8, 128, 16, peers, 16, 0, None, 16, None) == -3
    Lm = pkg._moe_sigs()
    assert Lm.nvfp4b_moe_forward_norm(16, 4, 16, 16, 8, None, None, 1e-6, 1.0, 16, 0, 16, None) == -3
    assert Lm.nvfp4b_moe_forward_norm(16, 4, 16, 16, 8, None, 16, 1e-6, 0.0, 16, 0, 16, None) == -7
