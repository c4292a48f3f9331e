"""The benchmark's algorithmic bytes and FLOPs (no GPU): the figures its roofline fractions divide by, against the
closed forms of the configurations (weights of the 8B and 70B shapes in Q4_K / Q8_0, the C3 contexts and their unique
KV bytes, the C4 prefill and tree-verify FLOPs)."""
import os
import sys
from types import SimpleNamespace

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def test_c3_contexts_are_the_seeded_log_normal_draw():
    ctx = bench.contexts()
    assert len(ctx) == 64 and int(np.sum(ctx)) == 168356 and int(np.median(ctx)) in (2146, 2147, 2148)
    assert ctx.min() >= 512 and ctx.max() <= 8192
    assert (ctx[:32] >= 1040).all()          # the 32 sequences that share the 1024-token prefix


def test_weight_bytes_of_the_shapes():
    # every linear layer and the head, read once per step: 7.5047e9 params (8B), 6.9502e10 (70B)
    assert bench.weight_bytes(bench.SPEC8B) == 7_504_658_432 * 144 // 256            # Q4_K: 4.221 GB
    assert bench.weight_bytes(bench.SPEC8B_Q8) * 272 // 144 == 7_504_658_432 * 34 // 32   # Q8_0: 7.974 GB
    assert bench.weight_bytes(bench.SPEC70B) == 69_501_714_432 * 144 // 256          # Q4_K: 39.09 GB


def test_c3_unique_kv_bytes():
    lay = SimpleNamespace(kv_heads=8, head_dim=128, layers=32)
    ctx = bench.contexts()
    got = bench.kv_unique_bytes(ctx, lay)
    # (sum of contexts + the step's own rows - 31 copies of the shared 1024-token prefix) x 64 KiB per row (fp8)
    assert got == (int(np.sum(ctx + 1)) - 31 * 1024) * 2 * 8 * 128 * 32
    assert abs(got / 1e9 - 8.957) < 0.01


def test_c4_flops():
    sp = bench.SPEC8B_Q8
    lin = sp["layers"] * sp["d"] * (sp["d"] * 2 + 2 * sp["d"] // sp["heads"] * sp["kv_heads"] + 3 * sp["ffn"])
    assert lin == 6_979_321_856
    n_seq, ctx = 32, 2048
    prefill = n_seq * (2 * lin * ctx + sp["layers"] * 4 * sp["d"] * ctx * (ctx + 1) / 2 + 2 * sp["d"] * sp["vocab"])
    assert abs(prefill / 1e12 - 950.0) < 1.0
    verify = 2 * lin * n_seq * 16 + 2 * sp["d"] * sp["vocab"] * n_seq * 16 + sp["layers"] * 4 * sp["d"] * ctx * n_seq * 16
    assert abs(verify / 1e12 - 8.23) < 0.02


def test_gemm_roofline_math():
    # five GEMM classes of 1 ms each over 5 steps: 1 ms of GEMMs per step for the 4.221 GB of weights
    sg = SimpleNamespace(class_ms=[1.0 if c in (2, 6, 7, 8, 9) else 0.0 for c in range(16)],
                         class_launches=[5 * (1 if c == 9 else 32) if c in (2, 6, 7, 8, 9) else 0 for c in range(16)])
    r = bench.gemm_roofline(sg, 5, 6454.6, "test")
    assert abs(r["ms_per_step"] - 1.0) < 1e-9 and r["launches_per_step"] == 129
    assert abs(r["frac"] - 4_221_370_368 / 1e-3 / 1e9 / 6454.6) < 1e-3
    # the gate/up launch: 1 ms over 160 launches
    assert abs(r["gateup"]["launch_ms"] - 1.0 / 160) < 1e-4   # reported to 4 decimals
    # chained steps: the gate/up class holds the one launch per layer that also runs down_proj
    sg.class_launches[8], sg.class_ms[8] = 0, 0.0
    sg.class_ms[7] = 2.0
    r = bench.gemm_roofline(sg, 5, 6454.6, "test")
    assert r["launches_per_step"] == 97 and "gateup" not in r and "chained" in r["kernel"]
    mlp = r["gateup_down"]
    assert mlp["algorithmic_bytes_per_launch"] == 2 * 14336 * 4096 * 144 // 256 + 4096 * 14336 * 144 // 256 + \
        64 * 4096 * 2 + 2 * 64 * 14336 * 2 + 64 * 4096 * 4
    assert abs(mlp["launch_ms"] - 2.0 / 160) < 1e-4
