"""CPU tests of the C ABI: the library loads, exports exactly what
include/ferret_moe.h declares, and rejects bad arguments on the host before
touching a device."""
import ctypes
import os
import re

import pytest

from ferret_b200 import _lib, build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "ferret_moe.h")


@pytest.fixture(scope="module")
def L():
    build.build()
    return _lib.lib()


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"FERRET_API\s+[\w\s\*]+?\b(ferret_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "ferret_fp8_grouped_gemm_nt_contiguous" in syms
    assert "ferret_moe_permute" in syms and "ferret_quant_act_fp8_1x128" in syms


def test_library_exports_every_declared_symbol(L):
    for s in declared_symbols():
        assert hasattr(L, s), f"{s} declared in ferret_moe.h but not exported"
    # and the python binding table covers them all
    assert set(declared_symbols()) <= set(_lib.SIGNATURES)


def test_version_and_strerror(L):
    m = re.search(r"#define FERRET_MOE_VERSION (\d+)", open(HEADER).read())
    assert L.ferret_version() == int(m.group(1))
    assert L.ferret_strerror(0) == b"ok"
    assert b"aligned" in L.ferret_strerror(-2)
    assert L.ferret_strerror(-1234) == b"unknown error"


def test_workspace_size(L):
    # segments (2E ints, 256-byte padded); up to 4096 rows also 16 MB of split-K room
    assert L.ferret_fp8_grouped_gemm_workspace_size(8192, 256) == 256 * 2 * 4
    assert L.ferret_fp8_grouped_gemm_workspace_size(1024, 256) == 256 * 2 * 4 + (16 << 20)
    assert L.ferret_fp8_grouped_gemm_workspace_size(1, 0) == 0


P = ctypes.c_void_p(0x1000)   # never dereferenced: validation fails first


@pytest.mark.parametrize("M,N,K,E,flags,code", [
    (16, 256, 100, 2, 0, -1),        # K not a multiple of 128
    (16, 200, 256, 2, 0, -1),        # N not a multiple of 128
    (16, 384, 256, 2, 1, -1),        # SiLU needs N % 256
    (16, 256, 256, 0, 0, -1),        # no experts
    (16, 256, 256, 2000, 0, -1),     # too many experts
    (16, 256, 32768, 2, 0, -1),      # K above the staged-scale limit
    (-1, 256, 256, 2, 0, -1),
    (0, 256, 256, 2, 0, 0),          # empty problem is a no-op
])
def test_gemm_shape_validation(L, M, N, K, E, flags, code):
    rc = L.ferret_fp8_grouped_gemm_nt_contiguous(P, P, P, P, P, P, P, M, N, K, E, flags, None, 0,
                                                 None)
    assert rc == code


def test_gemm_null_and_workspace_validation(L):
    f = L.ferret_fp8_grouped_gemm_nt_contiguous
    assert f(None, P, P, P, P, P, P, 16, 256, 256, 2, 0, None, 0, None) == -3
    assert f(P, P, P, P, P, None, None, 16, 256, 256, 2, 0, None, 0, None) == -3
    unaligned = ctypes.c_void_p(0x1001)
    assert f(unaligned, P, P, P, P, P, P, 16, 256, 256, 2, 0, None, 0, None) == -2


def test_permute_and_quant_validation(L):
    assert L.ferret_moe_permute(P, 4, 2, 0, P, P, P, None, 0, None) == -1
    assert L.ferret_moe_permute(P, 4, 2, 2048, P, P, P, None, 0, None) == -1
    assert L.ferret_moe_permute(P, 4, 2, 8, P, None, P, None, 0, None) == -3
    q = L.ferret_quant_act_fp8_1x128
    assert q(P, 4, None, 1, 4, 100, P, P, None) == -1
    assert q(P, 4, P, 0, 4, 128, P, P, None) == -1
    assert q(P, 2, None, 1, 4, 128, P, P, None) == -1      # R > x_rows without gather
    assert q(P, 4, None, 1, 0, 128, P, P, None) == 0
    assert q(None, 4, None, 1, 4, 128, P, P, None) == -3
    u = L.ferret_quant_act_fp8_1x128_ue8m0          # same validation in the UE8M0 form
    assert u(P, 4, None, 1, 4, 100, P, P, None) == -1
    assert u(P, 4, P, 0, 4, 128, P, P, None) == -1
    assert u(P, 4, None, 1, 0, 128, P, P, None) == 0
    assert u(None, 4, None, 1, 4, 128, P, P, None) == -3


def test_status_requires_pointer(L):
    assert L.ferret_last_device_status(None, None) == -3


def test_ops_import_fails_loudly_without_library(tmp_path, monkeypatch):
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "missing.so"))
    monkeypatch.setattr(_lib, "_LIB", None)
    with pytest.raises(ImportError, match="not found"):
        _lib.lib()


def test_align_block_size_sizes_follow_vllm_formula(L):
    """Buffer sizes of vLLM's moe_align_block_size: numel + E*(bs-1), capped at
    numel*bs when numel < E; blocks = ceil(size / bs)."""
    mp, mb = ctypes.c_int(0), ctypes.c_int(0)
    for T, topk, E, bs in ((64, 8, 384, 16), (1, 8, 384, 16), (4, 3, 4, 4), (7, 2, 5, 1)):
        assert L.ferret_moe_align_block_size_sizes(T, topk, E, bs, ctypes.byref(mp),
                                                   ctypes.byref(mb)) == 0
        numel = T * topk
        want = numel + E * (bs - 1)
        if numel < E:
            want = min(want, numel * bs)
        assert mp.value == want and mb.value == -(-want // bs)
    assert L.ferret_moe_align_block_size_sizes(4, 2, 8, 0, ctypes.byref(mp), ctypes.byref(mb)) == -1
    f = L.ferret_moe_align_block_size
    assert f(P, 4, 2, 8, 16, P, P, P, None, 0, None) == -7          # workspace missing
    assert f(P, 4, 2, 2048, 16, P, P, P, P, 1 << 20, None) == -1     # E beyond the sort's limit


def test_combine_and_ep_validation(L):
    c = L.ferret_moe_combine
    assert c(P, P, None, 0, 4, 2, 100, P, None) == -1                # H % 8
    assert c(P, P, P, 0, 4, 2, 128, P, None) == -1                   # ids without E
    assert c(None, P, None, 0, 4, 2, 128, P, None) == -3
    assert c(ctypes.c_void_p(0x1008), P, None, 0, 4, 2, 128, P, None) == -2
    assert c(P, P, None, 0, 0, 2, 128, P, None) == 0                  # no tokens: no-op
    ctx = ctypes.c_void_p()
    h = (ctypes.c_uint8 * int(L.ferret_ep_handle_bytes()))()
    init = L.ferret_ep_init
    args = lambda **kw: dict(dict(rank=0, world=2, E=256, topk=8, T=64, K=7168, N=4096, flags=0), **kw)
    for bad in (dict(world=9), dict(rank=2), dict(E=255), dict(K=7000), dict(flags=1, N=4224),
                dict(T=0)):
        a = args(**bad)
        assert init(a["rank"], a["world"], a["E"], a["topk"], a["T"], a["K"], a["N"], a["flags"],
                    None, ctypes.cast(h, ctypes.c_void_p), ctypes.byref(ctx)) == -1, bad
    assert init(0, 2, 256, 8, 64, 7168, 4096, 0, None, None, ctypes.byref(ctx)) == -3
    assert L.ferret_ep_connect(None, P) == -3
    assert L.ferret_ep_w13_forward(None, P, P, 1, P, P, P, None) == -3
    assert L.ferret_ep_destroy(None) == -3
    assert L.ferret_ep_output_buffer(None) is None
