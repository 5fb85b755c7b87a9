"""CPU tests of bench.py's contract helpers: algorithmic bytes/FLOPs per the
measurement definition, the roofline choice, and the traffic figures read
from the committed profile summaries."""
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402
from ferret_b200 import data  # noqa: E402


def _counts(cfg):
    ids = data.routing(cfg.T, cfg.E, cfg.topk, cfg.routing, cfg.zipf_s)
    return torch.bincount(ids.reshape(-1).long(), minlength=cfg.E).tolist()


def test_fp8_decode_algorithmic_bytes():
    cfg = data.CONFIGS["dsv3_decode"]
    byts, flops, active = bench.fp8_algorithmic(cfg, _counts(cfg))
    # 252 active experts x (N*K + (N/128)(K/128)*4) + R*K + R*(K/128)*4 + R*N*2
    assert active == 252
    assert byts == 252 * (4096 * 7168 + 32 * 56 * 4) + 1024 * 7168 + 1024 * 56 * 4 + 1024 * 4096 * 2
    assert flops == 2.0 * 1024 * 4096 * 7168


def test_int4_decode_algorithmic_bytes():
    cfg = data.CONFIGS["kimi_int4_decode"]
    byts, flops, active, wbytes = bench.int4_algorithmic(cfg, _counts(cfg))
    assert wbytes == active * 4096 * 7168 // 2
    assert byts == wbytes + active * 4096 * (7168 // 32) * 2 + 64 * 7168 * 2 + 512 * 4096 * 2
    assert flops == 2.0 * 512 * 4096 * 7168


def test_roofline_picks_the_longer_bound():
    pk = {"hbm_gbs": 6456.5, "bf16_tflops": 1635.4, "source": "measured"}
    dec = bench.roofline(7.4e9, 60e9, 1.1, pk, "k")
    assert dec["bound"] == "hbm" and abs(dec["frac"] - 7.4e9 / 1.1e-3 / 6456.5e9) < 1e-3
    big = bench.roofline(1e9, 3.0e12, 1.0, pk, "k")
    assert big["bound"] == "tensor" and big["peak"] == 2 * 1635.4


def test_traffic_figures_come_from_profiles():
    for tag in ("fp8_w13_grouped_dsv3_decode", "fp8_w13_prefill_dsv3_prefill",
                "int4_w13_grouped_kimi_int4_decode", "fp8_w13_prefill_ep_prefill",
                "int4_w13_decode_kimi_int4_decode"):
        t = bench.read_traffic(tag)
        assert t is not None and t > 1e9, tag
    assert bench.read_traffic("no_such_kernel_workload") is None
