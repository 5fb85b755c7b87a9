"""The product path has no CPU fallback: every public operation rejects host
tensors before any work is done (the CUDA library is the only implementation;
the CPU oracle is test infrastructure and is never reached from ferret_b200)."""
import ast
import os

import pytest
import torch

from ferret_b200 import ops

T, K, N, E, TOPK = 4, 256, 512, 4, 2


def _inputs():
    return dict(
        x=torch.zeros(T, K, dtype=torch.bfloat16),
        ids=torch.zeros(T, TOPK, dtype=torch.int32),
        w=torch.zeros(E, N, K, dtype=torch.float8_e4m3fn),
        ws=torch.ones(E, N // 128, K // 128),
        a=torch.zeros(T * TOPK, K, dtype=torch.float8_e4m3fn),
        asc=torch.ones(T * TOPK, K // 128),
        out=torch.zeros(T * TOPK, N, dtype=torch.bfloat16),
        mi=torch.zeros(T * TOPK, dtype=torch.int32),
        w_raw=torch.zeros(E, K // 8, N, dtype=torch.int32),
        w_s4=torch.ones(E, K // 32, N, dtype=torch.bfloat16),
        w2=torch.zeros(E, K, N // 2, dtype=torch.float8_e4m3fn),
        w2s=torch.ones(E, K // 128, N // 256),
    )


CALLS = {
    "per_token_cast_to_fp8": lambda i: ops.per_token_cast_to_fp8(i["x"]),
    "per_token_cast_to_fp8_ue8m0": lambda i: ops.per_token_cast_to_fp8(i["x"], use_ue8m0=True),
    "m_grouped_fp8_gemm_nt_contiguous": lambda i: ops.m_grouped_fp8_gemm_nt_contiguous(
        (i["a"], i["asc"]), (i["w"], i["ws"]), i["out"], i["mi"]),
    "m_grouped_fp8_gemm_scatter": lambda i: ops.m_grouped_fp8_gemm_scatter(
        (i["a"], i["asc"]), (i["w"], i["ws"]), i["out"], torch.zeros(E + 1, dtype=torch.int32), i["mi"]),
    "moe_permute": lambda i: ops.moe_permute(i["ids"], E),
    "moe_align_block_size": lambda i: ops.moe_align_block_size(i["ids"], 16, E),
    "fp8_moe_w13": lambda i: ops.fp8_moe_w13(i["x"], i["ids"], i["w"], i["ws"]),
    "moe_combine": lambda i: ops.moe_combine(i["out"], torch.ones(T, TOPK), i["ids"]),
    "fp8_moe_ffn": lambda i: ops.fp8_moe_ffn(i["x"], i["ids"], torch.ones(T, TOPK), i["w"], i["ws"],
                                             i["w2"], i["w2s"]),
    "Int4W13Weights": lambda i: ops.Int4W13Weights(i["w_raw"], i["w_s4"]),
}


@pytest.mark.parametrize("name", sorted(CALLS))
def test_public_ops_reject_host_tensors(name):
    with pytest.raises((ValueError, TypeError)):
        CALLS[name](_inputs())


def test_product_package_never_imports_the_oracle():
    """No module of ferret_b200 imports oracle/ (it is the checker, not a path)."""
    pkg = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "ferret_b200")
    for fn in sorted(os.listdir(pkg)):
        if not fn.endswith(".py"):
            continue
        tree = ast.parse(open(os.path.join(pkg, fn)).read())
        for node in ast.walk(tree):
            names = []
            if isinstance(node, ast.Import):
                names = [a.name for a in node.names]
            elif isinstance(node, ast.ImportFrom):
                names = [node.module or ""]
            assert not any(n == "oracle" or n.startswith("oracle.") for n in names), (fn, names)
