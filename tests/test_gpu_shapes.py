"""Parity at the benchmark's own shapes (3 and 4) with the layer count cut to 2, against the oracle
on the same GGUF (``goethe_engine/ref.py:39-62`` and ``TorchBackend.step``, ``ref.py:94-112``).

* C3: the Llama-3-8B shape (d 4096, 32 query / 8 KV heads of 128, FFN 14336, vocabulary 128256), Q4_K weights (head
  and embedding included), fp8 KV with per-page scales, a batch-invariant bucket. One decode step of 64 sequences:
  eight with contexts from the benchmark's own C3 draw (7969, 838 and 856 tokens of their own; 2234 and four of 1040
  tokens that share the benchmark's 1024-token prefix pages) and 56 more that share the same prefix pages with 16-48
  tokens of their own. The step runs the benchmark's kernels: the tcgen05 GEMM with a 64-row token tile and the split-K
  counts of the 8B weights, attention over fixed 512-entry splits (up to 16 of them) with shared prefix pages read by
  61 sequences, and the 8-part argmax over 128256 head rows. Logits within 3e-2 (fp8 KV); the device argmax equals the
  host argmax of the same logits exactly, and the oracle's wherever its top-2 margin exceeds twice the tolerance.
* C2: the 8B shape with Q8_0 weights and f16 KV, one sequence at context 2048 in a single-stream "tolerance" bucket
  (the decode GEMV and short attention splits); three decode steps within 1e-2.
* C4b: the same Q8_0 weights in a batch-invariant bucket; two sequences at context 2048 each verify a 16-node draft
  tree of depth at most 4 (the benchmark's seeded topology) in one step; all 32 node rows within 1e-2.
"""
import os
import random
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402
from goethe_engine_b200 import build, gck, synth  # noqa: E402
from helpers import TOL_F16, TOL_FP8, assert_logits_close  # noqa: E402
from oracle.load import weights_from_gguf  # noqa: E402
from oracle.model import PagedOracle  # noqa: E402

pytestmark = pytest.mark.gpu
LAYERS = 2
BS = 16


@pytest.fixture(scope="module", autouse=True)
def built():
    build.build()


def spec8b(wtype, ctx):
    return synth.Spec(**dict(bench.SPEC8B, layers=LAYERS, wtype=wtype, ctx=ctx, name=f"t8b-{wtype}-L{LAYERS}"))


# ------------------------------------------------------------------------------------------------------------- C3
@pytest.mark.parametrize("kv", ["fp8", "f16"])
def test_c3_decode_step_matches_oracle(tmp_path, kv):
    """bench.c3_sample: the 64-sequence decode step; the library's logits against the oracle's, and the device argmax
    of the repeated step against the first maximum of the same logits (exact) and the oracle's (margin rule). With
    fp8 KV (the benchmark's) at the fp8 tolerance; with f16 KV over the same weights at 1e-2, which checks every
    kernel of the step at this shape without fp8's rounding noise."""
    spec = spec8b("q4_k", bench.SPEC8B["ctx"])
    pack, ws = synth.make(str(tmp_path), spec, ncol=64, maxctx=spec.ctx, kv=kv,
                          tune=dict(max_cols=2048, kv_scale="page"))
    smp = bench.c3_sample()
    assert len(smp["dec"]) == 64 and max(smp["cs"]) == 7969 and min(smp["cs"]) == 838
    with gck.Backend(pack, ws, pool_blocks=smp["nblk"]) as be:
        got, greedy = bench.c3_sample_run(be, smp)
    assert np.array_equal(greedy, got.argmax(-1))
    ref = bench.c3_sample_oracle(ws[0], smp, kv=kv)
    assert_logits_close(got, ref, TOL_FP8 if kv == "fp8" else TOL_F16)


# -------------------------------------------------------------------------------------------------------- C2, C4b
@pytest.fixture(scope="module")
def q8(tmp_path_factory):
    d = tmp_path_factory.mktemp("q8")
    spec = spec8b("q8_0", 4096)
    ws = synth.make(str(d / "w"), spec, ncol=32, maxctx=4096)[1]
    single = synth.pack_dir(str(d / "single"), spec, [dict(id="b200.FAST.single", ncol=1, batch=False, maxctx=4096,
                                                           determinism="tolerance", tune=dict(max_cols=2048))],
                            weights_file=ws[0])
    batch = synth.pack_dir(str(d / "batch"), spec, [dict(id="b200.BI.main", ncol=32, maxctx=4096,
                                                         tune=dict(max_cols=2048))], weights_file=ws[0])
    return ws, single, batch, weights_from_gguf(ws[0])


def test_c2_gemv_decode_matches_oracle(q8):
    ws, single, _, w = q8
    ctx = 2048
    toks = [int(x) for x in np.random.default_rng(0).integers(1, 128000, ctx + 3)]
    tab = list(range(-(-(ctx + 4) // BS)))
    script = [dict(sid=0, tokens=toks[:ctx - 1], pos=0, blocks=tab, want=0)]
    script += [dict(sid=0, tokens=[toks[ctx - 1 + j]], pos=ctx - 1 + j, blocks=tab, want=1) for j in range(3)]
    with gck.Backend(single, ws, buckets=("b200.FAST.single",), pool_blocks=len(tab) + 4) as be:
        got = [be.step([gck.Work(d["sid"], d["tokens"], d["pos"], d["blocks"], d["want"])]) for d in script]
    o = PagedOracle(w, num_blocks=len(tab) + 4, kv="f16")
    ref = [o.step([d]) for d in script]
    for g, r in zip(got[1:], ref[1:]):
        assert_logits_close(g, r, TOL_F16)


def tree_parents():
    """The benchmark's C4 draft tree: anchor + 15 drafts, each parent uniform over the earlier nodes of depth < 4."""
    r, par, depth = random.Random(1), [-1], [0]
    for i in range(1, 16):
        pj = r.choice([j for j in range(i) if depth[j] < 4])
        par.append(pj)
        depth.append(depth[pj] + 1)
    return par


def test_c4_tree_verify_matches_oracle(q8):
    ws, _, batch, w = q8
    ctx, par = 2048, tree_parents()
    rng = np.random.default_rng(2)
    toks = [[int(x) for x in rng.integers(1, 128000, ctx)] for _ in range(2)]
    draft = [[int(x) for x in rng.integers(1, 128000, 16)] for _ in range(2)]
    per = -(-(ctx + 16) // BS)
    tabs = [list(range(i * per, (i + 1) * per)) for i in range(2)]
    pre = [dict(sid=i, tokens=toks[i], pos=0, blocks=tabs[i], want=0) for i in range(2)]
    ver = [dict(sid=i, tokens=draft[i], pos=ctx, blocks=tabs[i], want=16, parents=par) for i in range(2)]
    with gck.Backend(batch, ws, pool_blocks=2 * per + 4) as be:
        for d in pre:                          # 2048 tokens a step: the bucket's columns
            be.step([gck.Work(d["sid"], d["tokens"], d["pos"], d["blocks"], 0)])
        got = be.step([gck.Work(d["sid"], d["tokens"], d["pos"], d["blocks"], 16, parents=par) for d in ver])
    o = PagedOracle(w, num_blocks=2 * per + 4, kv="f16")
    o.step(pre)
    assert_logits_close(got, o.step(ver), TOL_F16)
