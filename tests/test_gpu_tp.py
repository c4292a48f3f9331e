"""Tensor parallelism (one handle over 2, 4 or 8 GPUs): heads, kv heads and FFN columns split across the ranks,
o_proj / down_proj by their input columns with an all-reduce after each (over peer memory, in rank order; NCCL where
peer access is missing), the head by vocabulary rows.

* the scripted session (prefill chunks, batched decode, tree verify, commit, copy_blocks) at tp = 2, 4, 8 against the
  oracle and against the single-GPU library, to the a16 tolerance;
* greedy tokens of a tp handle equal the single-GPU ones wherever the top-2 margin exceeds the tolerance;
* at tp = 2 a row's logits are bit-identical alone and batched (the all-reduce adds the ranks in a fixed order).
Each test runs only where enough GPUs are visible.
"""
import numpy as np
import pytest

from goethe_engine_b200 import build, gck, synth
from helpers import SCENARIO, TOL_F16, assert_logits_close, oracle_for, replay

pytestmark = pytest.mark.gpu
# dh 64, GQA 4; per rank at tp 8: 4 heads, 1 kv head, o_proj input 256, FFN 512, 125 vocabulary rows
TPSHAPE = dict(vocab=1000, d=2048, layers=2, heads=32, kv_heads=8, ffn=4096)


def gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.fixture(scope="module", autouse=True)
def built():
    build.build()


@pytest.fixture(scope="module")
def tp_model(tmp_path_factory):
    d = tmp_path_factory.mktemp("tp")
    spec = synth.Spec(**TPSHAPE, wtype="q4_k", seed=11)
    ws = synth.make(str(d / "w"), spec, ncol=8, maxctx=512)[1]
    packs = {n: synth.pack_dir(str(d / f"tp{n}"), spec, [dict(id="b200.BI.main", ncol=8, maxctx=512, tp=n)],
                               weights_file=ws[0]) for n in (1, 2, 4, 8)}
    return packs, ws


@pytest.mark.parametrize("n", [2, 4, 8])
def test_tp_session_matches_oracle_and_single_gpu(tp_model, n):
    if gpus() < n:
        pytest.skip(f"{n} GPUs needed, {gpus()} visible")
    packs, ws = tp_model
    with gck.Backend(packs[n], ws, pool_blocks=16, device=0) as be:
        got = replay(be)
    with gck.Backend(packs[1], ws, pool_blocks=16, device=0) as be:
        one = replay(be)
    ref = replay(oracle_for(ws))
    for g, o, r in zip(got, one, ref):
        assert_logits_close(g, r, TOL_F16)
        assert_logits_close(g, o, TOL_F16)


def test_tp2_greedy_and_batch_invariance(tp_model):
    if gpus() < 2:
        pytest.skip("2 GPUs needed")
    packs, ws = tp_model
    rng = np.random.default_rng(2)
    prompts = [[int(x) for x in rng.integers(1, 1000, 21 + 5 * i)] for i in range(3)]
    tabs = [list(range(4 * i, 4 * i + 4)) for i in range(3)]
    with gck.Backend(packs[2], ws, pool_blocks=16, device=0) as tp, \
            gck.Backend(packs[1], ws, pool_blocks=16, device=0) as one:
        for be in (tp, one):
            be.step([gck.Work(i, p[:-1], 0, tabs[i], 0) for i, p in enumerate(prompts)])
        last = [gck.Work(i, [p[-1]], len(p) - 1, tabs[i], 1) for i, p in enumerate(prompts)]
        batched = tp.step(last)
        alone = tp.step([last[1]])
        # the same decode step alone: bit-identical row (the KV row it rewrites holds the same values)
        assert np.array_equal(batched[1:2], alone)
        ref = one.step(last)
        assert_logits_close(batched, ref, TOL_F16)
        g_tp = tp.step([gck.Work(i, [p[-1]], len(p) - 1, tabs[i], 1, greedy=True) for i, p in enumerate(prompts)])
        top2 = np.sort(ref, -1)[:, -2:]
        sure = (top2[:, 1] - top2[:, 0]) / np.abs(ref).max(-1) > 2 * TOL_F16
        assert (np.array([t[0] for t in g_tp])[sure] == ref.argmax(-1)[sure]).all()


def test_tp2_paired_gemms_equal_single_cta(tmp_path):
    """At tp = 2, steps of more than 64 rows run the per-rank GEMMs on CTA pairs (cta_group::2) with the completion
    signal the all-reduce waits for; a handle opened with GCK_PAIR=0 runs them on one CTA per MMA. The logits agree bit
    for bit (the pair's sums equal the single CTA's, and the ranks are added in a fixed order)."""
    if gpus() < 2:
        pytest.skip("2 GPUs needed")
    import os
    spec = synth.Spec(**TPSHAPE, wtype="q4_k", seed=13)
    ws = synth.make(str(tmp_path / "w"), spec, ncol=256, maxctx=512)[1]
    pack = synth.pack_dir(str(tmp_path / "tp2"), spec, [dict(id="b200.BI.main", ncol=256, maxctx=512, tp=2)],
                          weights_file=ws[0])
    rng = np.random.default_rng(5)
    prompts = [[int(x) for x in rng.integers(1, 1000, n)] for n in (100, 90, 60)]
    tabs = [list(range(8 * i, 8 * i + 8)) for i in range(3)]
    outs = []
    for pair in ("1", "0"):
        os.environ["GCK_PAIR"] = pair
        try:
            with gck.Backend(pack, ws, pool_blocks=32, device=0) as be:
                got = [be.step([gck.Work(0, prompts[0], 0, tabs[0], len(prompts[0]))]),
                       be.step([gck.Work(i, p, 0, tabs[i], len(p)) for i, p in enumerate(prompts[1:], 1)])]
                got.append(be.step([gck.Work(i, [p[-1]], len(p), tabs[i], 1) for i, p in enumerate(prompts)]))
        finally:
            os.environ.pop("GCK_PAIR", None)
        outs.append(got)
    for a, b in zip(*outs):
        assert np.array_equal(a, b)
