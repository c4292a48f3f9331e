"""The tcgen05 GEMM on CTA pairs against one CTA per MMA.

Steps of more than 64 token rows (128-row token tiles) run a weight with an even number of 128-row bands on clusters
of two CTAs: one M = 256 MMA (tcgen05.mma.cta_group::2) over both CTAs' bands, each CTA holding half of the token tile.
A handle opened with GCK_PAIR=0 runs every GEMM with one CTA per MMA. Each output element sums its K range in the same
order either way, so the two must agree bit for bit, through:

* steps of 100 rows (one 128-row tile, the second CTA's half partly past the last row), 200 rows (two tiles) and
  1764 rows (a 36-sequence prefill), beside steps of 24, 40 and 64 rows that stay on one CTA per MMA;
* a model whose fused q/k/v and LM head have an odd band count (those weights stay on one CTA per MMA) beside even
  ones, so that a step mixes both kernels;
* Q4_K and Q8_0 weights, residual-add, SwiGLU and split-K epilogues (the weights' fixed split counts).

A row's logits must also not depend on its batch: a sequence prefilled and decoded alone (one CTA per MMA) and inside
80-sequence steps (pairs) gives the same bits.
"""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402
from goethe_engine_b200 import build, gck, synth  # noqa: E402

pytestmark = pytest.mark.gpu
PER = 24                        # blocks per sequence's table range
# 8 heads of 64 and one KV head: q/k/v 640 rows (5 bands) and the head 640 rows (5 bands) on one CTA per MMA; o_proj,
# gate/up and down (4, 12 and 4 bands) on pairs
ODD = dict(vocab=640, d=512, layers=2, heads=8, kv_heads=1, ffn=768)
EVEN = dict(vocab=512, d=512, layers=2, heads=4, kv_heads=1, ffn=768)


@pytest.fixture(scope="module", autouse=True)
def built():
    build.build()


def script(be):
    """Prefill steps of 24, 64, 100 and 200 rows (every row's logits), then decode steps of 40 and of 20 rows."""
    on, read = bench.stats_api(be)
    on(False)
    rng = np.random.default_rng(5)
    lens = [24, 64, 100, 200] + [int(x) for x in rng.integers(3, 50, 36)]
    toks = [[int(x) for x in rng.integers(1, 500, n)] for n in lens]
    tabs = [list(range(PER * i, PER * (i + 1))) for i in range(len(lens))]
    out = []
    for i in range(4):
        out.append(be.step([gck.Work(i, toks[i], 0, tabs[i], len(toks[i]))]))
    out.append(be.step([gck.Work(i, toks[i], 0, tabs[i], 1) for i in range(4, len(lens))]))
    for k in range(6):
        live = range(len(lens)) if k % 2 == 0 else range(20)
        res = be.step([gck.Work(i, [toks[i][-1]], len(toks[i]) - 1, tabs[i], 1) for i in live])
        out.append(res)
        for i, r in zip(live, res.reshape(len(live), -1)):
            toks[i].append(int(np.argmax(r)))
    return out, read()


def run(tmp_path, dims, wtype, pairs):
    spec = synth.Spec(**dims, wtype=wtype, seed=23)
    pack, ws = synth.make(str(tmp_path / f"{wtype}_{dims['d']}"), spec, ncol=2048, maxctx=PER * 16)
    if pairs:
        os.environ.pop("GCK_PAIR", None)
    else:
        os.environ["GCK_PAIR"] = "0"
    try:
        with gck.Backend(pack, ws, pool_blocks=PER * 41) as be:
            return script(be)
    finally:
        os.environ.pop("GCK_PAIR", None)


@pytest.mark.parametrize("wtype", ["q4_k", "q8_0"])
@pytest.mark.parametrize("dims", [EVEN, ODD], ids=["even", "odd"])
def test_pairs_equal_single_cta(tmp_path, dims, wtype):
    ref, st_ref = run(tmp_path, dims, wtype, False)
    got, st = run(tmp_path, dims, wtype, True)
    assert st_ref.gemm_pairs == 0
    assert st.gemm_pairs > 0, "the device runs no two-CTA clusters"
    assert len(got) == len(ref)
    for g, r in zip(got, ref):
        assert np.array_equal(g, r)


def test_row_alone_equals_row_in_a_paired_batch(tmp_path):
    """Sequence 7's 12-token prompt prefilled alone (a 16-row tile, one CTA per MMA) and inside an 80-sequence prefill
    (pairs), then its decode alone and inside an 80-row decode step (pairs): the same logits bit for bit."""
    spec = synth.Spec(**EVEN, wtype="q4_k", seed=29)
    pack, ws = synth.make(str(tmp_path), spec, ncol=2048, maxctx=PER * 16)
    rng = np.random.default_rng(8)
    lens = [int(n) for n in rng.integers(5, 24, 80)]
    lens[7] = 12
    toks = [[int(x) for x in rng.integers(1, 500, n)] for n in lens]
    tabs = [list(range(PER * i, PER * (i + 1))) for i in range(80)]
    with gck.Backend(pack, ws, pool_blocks=PER * 81) as be:
        pre_b = be.step([gck.Work(i, toks[i], 0, tabs[i], 1) for i in range(80)])
        batch = be.step([gck.Work(i, [toks[i][-1]], len(toks[i]) - 1, tabs[i], 1) for i in range(80)])
    with gck.Backend(pack, ws, pool_blocks=PER * 81) as be:
        pre_a = be.step([gck.Work(7, toks[7], 0, tabs[7], 1)])
        alone = be.step([gck.Work(7, [toks[7][-1]], len(toks[7]) - 1, tabs[7], 1)])
    assert np.array_equal(np.asarray(pre_b).reshape(80, -1)[7], np.asarray(pre_a).reshape(-1))
    assert np.array_equal(np.asarray(batch).reshape(80, -1)[7], np.asarray(alone).reshape(-1))
