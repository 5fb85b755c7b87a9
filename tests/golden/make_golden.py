"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container that has the reference tree (read-only) and its toolchain:

    python tests/golden/make_golden.py --ref <path of the reference checkout>

It writes, next to this script:

* ``fp8_v007_ref.npz``: inputs and the output of the reference's own FP8 host
  reference ``cpu_ref_bs`` (examples/fp8-group-gemm/v007_dsv3_decode_verified_105.cu:441-467),
  compiled unmodified by ``oracle/Makefile`` (target ``ref``) and run through
  ``oracle/_ref/v007_cpu_ref``.  The inputs use power-of-two scales and
  128-row expert tiles so that the two places where v007 departs from the
  exact-scale, per-row-expert contract (UE8M0 rounding at v007:454-455, the
  tile's first-row expert at v007:449-450) are identities; on such inputs the
  oracle must agree bit for bit.
* ``int4_ref_small.npz``: inputs and output of the reference's INT4 oracle
  ``fp32_oracle_w13_silu`` (correctness/compare_marlin_vs_ref.py:44-100),
  imported from the reference tree and run on the CPU with its module
  constants set to a small shape (H=256, N_R=64, TOP_K=2).
* ``int4_ref_kimi.npz``: the same function at the reference's own shape
  (H=7168, N_R=512, I_R=256, TOP_K=8), T=1 over 8 experts.  The inputs are
  too large to commit; they are regenerated from the stored numpy seed and
  checked against the stored SHA-256 before use.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import oracle as O  # noqa: E402


def fp8_case(seed=7, M=256, N=128, K=256, E=3):
    rng = np.random.default_rng(seed)
    a = rng.integers(0, 256, size=(M, K), dtype=np.uint8)
    a[(a & 0x7F) == 0x7F] = 0x3C       # no NaN codes
    w = rng.integers(0, 256, size=(E, N, K), dtype=np.uint8)
    w[(w & 0x7F) == 0x7F] = 0x3C
    nk = K // 128
    a_scale = np.ldexp(1.0, rng.integers(-9, -3, size=(M, nk))).astype(np.float32)
    w_scale = np.ldexp(1.0, rng.integers(-12, -6, size=(E, N // 128, nk))).astype(np.float32)
    order = rng.permutation(E)
    m_indices = np.repeat(order, 128).astype(np.int32)[:M]
    return a, w, a_scale, w_scale, m_indices


def write_v007_input(path, a, w, a_scale, w_scale, m_indices):
    M, K = a.shape
    E, N, _ = w.shape
    with open(path, "wb") as f:
        np.array([M, N, K, E], np.int32).tofile(f)
        a.tofile(f)
        w.tofile(f)
        a_scale.astype(np.float32).tofile(f)
        w_scale.astype(np.float32).tofile(f)
        m_indices.astype(np.int32).tofile(f)


def make_fp8(ref_root):
    subprocess.check_call(["make", "-s", "-C", os.path.join(REPO, "oracle"), "ref", f"REF={ref_root}"])
    exe = os.path.join(REPO, "oracle", "_ref", "v007_cpu_ref")
    a, w, a_scale, w_scale, m_indices = fp8_case()
    with tempfile.TemporaryDirectory() as td:
        fin, fout = os.path.join(td, "in.bin"), os.path.join(td, "out.bin")
        write_v007_input(fin, a, w, a_scale, w_scale, m_indices)
        subprocess.check_call([exe, fin, fout])
        out = np.fromfile(fout, np.float32).reshape(a.shape[0], w.shape[1])
    np.savez_compressed(os.path.join(HERE, "fp8_v007_ref.npz"), a=a, w=w, a_scale=a_scale,
                        w_scale=w_scale, m_indices=m_indices, out=out)
    print("fp8_v007_ref.npz", out.shape, float(np.abs(out).max()))


def load_ref_int4(ref_root):
    path = os.path.join(ref_root, "correctness", "compare_marlin_vs_ref.py")
    spec = importlib.util.spec_from_file_location("ref_compare_marlin", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.device = "cpu"
    return mod


def int4_inputs(seed, T, E, K, N, topk):
    """numpy-seeded inputs in the reference's distributions
    (correctness/compare_marlin_vs_ref.py:115-130)."""
    rng = np.random.default_rng(seed)
    raw_q = rng.integers(0, 2**31 - 1, size=(E, K // 8, N), dtype=np.int64).astype(np.int32)
    scales = O.f32_to_bf16((rng.standard_normal((E, K // 32, N)) * 0.01).astype(np.float32))
    ids = np.stack([rng.permutation(E)[:topk] for _ in range(T)]).astype(np.int32)
    hidden = O.f32_to_bf16((rng.standard_normal((T, K)) * 0.01).astype(np.float32))
    return hidden, raw_q, scales, ids


def digest(*arrs):
    h = hashlib.sha256()
    for a in arrs:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def run_ref_int4(mod, hidden, raw_q, scales, ids):
    import torch
    out = mod.fp32_oracle_w13_silu(
        torch.from_numpy(hidden.view(np.int16)).view(torch.bfloat16),
        torch.from_numpy(raw_q),
        torch.from_numpy(scales.view(np.int16)).view(torch.bfloat16),
        torch.from_numpy(ids),
    )
    return out.view(torch.int16).numpy().view(np.uint16)


def make_int4(ref_root):
    mod = load_ref_int4(ref_root)
    # small shape: patch the module constants the function reads
    mod.H, mod.N_R, mod.I_R, mod.TOP_K = 256, 64, 32, 2
    hidden, raw_q, scales, ids = int4_inputs(11, T=3, E=4, K=256, N=64, topk=2)
    out = run_ref_int4(mod, hidden, raw_q, scales, ids)
    np.savez_compressed(os.path.join(HERE, "int4_ref_small.npz"), hidden=hidden, raw_q=raw_q,
                        scales=scales, topk_ids=ids, out=out)
    print("int4_ref_small.npz", out.shape)
    # the reference's own shape
    mod.H, mod.N_R, mod.I_R, mod.TOP_K = 7168, 512, 256, 8
    seed = 1234
    hidden, raw_q, scales, ids = int4_inputs(seed, T=1, E=8, K=7168, N=512, topk=8)
    out = run_ref_int4(mod, hidden, raw_q, scales, ids)
    np.savez_compressed(os.path.join(HERE, "int4_ref_kimi.npz"), seed=np.int64(seed),
                        shape=np.array([1, 8, 7168, 512, 8], np.int64),
                        sha256=np.array(digest(hidden, raw_q, scales, ids)), out=out)
    print("int4_ref_kimi.npz", out.shape)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("FERRET_REFERENCE_ROOT", ""))
    ap.add_argument("--only", choices=["fp8", "int4"], default=None)
    args = ap.parse_args()
    if not args.ref or not os.path.isdir(args.ref):
        sys.exit("pass --ref <path to the reference tree>")
    if args.only in (None, "fp8"):
        make_fp8(args.ref)
    if args.only in (None, "int4"):
        make_int4(args.ref)


if __name__ == "__main__":
    main()
