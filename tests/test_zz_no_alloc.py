"""GPU test of the allocation-free FP8 grouped GEMM entry point.

ferret_fp8_grouped_gemm_nt_contiguous_noalloc serves callers that cannot
allocate device memory at call time (a server that pre-reserved its HBM, an
FFI plugin host without access to its framework's allocator): it keeps the
expert segments it derives from m_indices in a fixed array inside the
library instead of a caller-provided workspace.  This test calls it through
the C ABI several times in a row, with different expert layouts so that a
stale segment table from an earlier call would show, and compares each result
with the workspace entry point's on the same inputs and with the CPU oracle
(max relative error < 1e-2, no NaN, padding rows untouched).  The cases cover
the swap-AB token tiles (automatic and forced to 64 rows with SiLU), the
prefill kernel (more than 48 rows per expert, which both entry points choose
alike), and E = 1024, the array's limit.  The file sorts last so that a run
stopping at the first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-2
BF16_NAN = 0x7FFF


def _case(seed, seg_counts, N, K, pad):
    rng = np.random.default_rng(seed)
    E = len(seg_counts)
    mi = []
    for e, c in enumerate(seg_counts):
        mi += [e] * c + [-1] * pad
    mi = np.array(mi, np.int32)
    M = len(mi)
    a = O.f32_to_e4m3(rng.standard_normal((M, K)).astype(np.float32) * 100)
    w = O.f32_to_e4m3(rng.standard_normal((E, N, K)).astype(np.float32) * 100)
    a_s = rng.uniform(1e-3, 1e-2, (M, K // 128)).astype(np.float32)
    w_s = rng.uniform(1e-4, 1e-3, (E, N // 128, K // 128)).astype(np.float32)
    t = lambda x: torch.from_numpy(x).cuda()
    return t(a), t(a_s), t(w), t(w_s), t(mi), mi, (a, a_s, w, w_s)


def _out(M, n_out):
    return torch.full((M, n_out), BF16_NAN, dtype=torch.int16).view(torch.bfloat16).cuda()


def test_noalloc_matches_workspace_entry_point_twice(cuda_device):
    from ferret_b200 import _lib
    L = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    tile64 = 64 << 8                                            # FERRET_TILE_SHIFT
    rng = np.random.default_rng(5)
    cases = [
        (_case(21, [9, 0, 33, 2, 17, 1], 512, 512, 3), 512, 512, 0),
        (_case(22, [40, 5, 0], 512, 256, 0), 512, 256, 1),     # fewer experts, SiLU
        (_case(23, [150, 61, 0, 97], 512, 256, 2), 512, 256, 0),   # > 48 rows/expert: prefill kernel
        (_case(24, [150, 61, 0, 97], 512, 256, 2), 512, 256, 1),   # the same with SiLU
        (_case(25, [70, 3, 130], 512, 256, 1), 512, 256, 1 | tile64),  # forced 64-row tile + SiLU
        (_case(26, list(rng.integers(0, 3, 1024)), 128, 128, 0), 128, 128, 0),  # E = 1024
    ]
    for (a, a_s, w, w_s, mi_t, mi, host), N, K, flags in cases:
        M, E = a.shape[0], w.shape[0]
        n_out = N // 2 if flags & 1 else N
        ref = _out(M, n_out)
        ws_bytes = L.ferret_fp8_grouped_gemm_workspace_size(M, E)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        rc = L.ferret_fp8_grouped_gemm_nt_contiguous(p(a), p(a_s), p(w), p(w_s), p(ref), p(mi_t),
                                                    None, M, N, K, E, flags, p(ws), ws_bytes,
                                                    stream)
        assert rc == 0
        got = _out(M, n_out)
        rc = L.ferret_fp8_grouped_gemm_nt_contiguous_noalloc(p(a), p(a_s), p(w), p(w_s), p(got),
                                                            p(mi_t), M, N, K, E, flags, stream)
        assert rc == 0
        torch.cuda.synchronize()
        st = ctypes.c_int32(1)
        assert L.ferret_last_device_status(stream, ctypes.byref(st)) == 0 and st.value == 0
        g = O.bf16_to_f32(got.view(torch.int16).cpu().numpy().view(np.uint16))
        r = O.bf16_to_f32(ref.view(torch.int16).cpu().numpy().view(np.uint16))
        valid = mi >= 0
        err = O.rel_err(g[valid], r[valid])
        assert err["nan"] == 0 and err["max_rel"] < TOL, (E, flags, err)
        oracle = O.fp8_grouped_gemm_fast(*host, mi, silu=bool(flags & 1))
        err = O.rel_err(g[valid], oracle[valid])
        assert err["nan"] == 0 and err["max_rel"] < TOL, (E, flags, "oracle", err)
        assert (got.view(torch.int16).cpu().numpy()[~valid] == BF16_NAN).all()


def test_noalloc_rejects_more_experts_than_its_array(cuda_device):
    from ferret_b200 import _lib
    P = ctypes.c_void_p(0x1000)
    assert _lib.lib().ferret_fp8_grouped_gemm_nt_contiguous_noalloc(
        P, P, P, P, P, P, 16, 256, 256, 1025, 0, None) == -1
