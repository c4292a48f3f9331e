"""Captured steps against direct launches.

A step whose shape repeats (plan sizes, scratch buffers) is replayed from a CUDA graph captured the second time the
shape is seen; block tables live on the device and each step patches only the entries that differ from the slot's
last table (GCK_GRAPH=0 in the environment turns graphs off for a handle opened under it). The same script through a
handle with graphs and one without must give the same logits and tokens bit for bit, through:

* decode steps whose sequences grow past block boundaries (new table entries) and past 512-entry attention splits;
* a sequence released and its slot taken by another sequence with a different table;
* a table entry replaced in the middle of a sequence after a block copy (copy-on-write, gc.h:214-216);
* greedy steps (device argmax inside the graph) and steps returning host logits.
"""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402
from goethe_engine_b200 import build, gck, synth  # noqa: E402
from helpers import SMALL128, model  # noqa: E402

pytestmark = pytest.mark.gpu
PER = 80                      # blocks per sequence's table range


@pytest.fixture(scope="module", autouse=True)
def built():
    build.build()


def script(be):
    """Runs the script on be; returns every step's output (logits arrays or token lists) and the stats of the decode
    loop."""
    on, read = bench.stats_api(be)
    rng = np.random.default_rng(11)
    lens = [30, 200, 500, 700, 1030, 17]
    toks = [[int(x) for x in rng.integers(1, 500, n)] for n in lens]
    tabs = [list(range(PER * i, PER * (i + 1))) for i in range(len(lens))]
    out = []
    # prefill in two steps (the bucket's 2048 columns)
    out.append(be.step([gck.Work(i, toks[i], 0, tabs[i], 1) for i in range(4)]))
    out.append(be.step([gck.Work(i, toks[i], 0, tabs[i], 1) for i in (4, 5)]))
    live = list(range(len(lens)))
    on(False)
    for k in range(48):
        if k == 16:
            # sequence 5 leaves; sequence 6 takes its slot with another table
            be.release(5)
            live.remove(5)
            toks.append([int(x) for x in rng.integers(1, 500, 40)])
            tabs.append(list(range(PER * 6, PER * 7)))
            out.append(be.step([gck.Work(6, toks[6], 0, tabs[6], 1)]))
            live.append(6)
        if k == 28:
            # copy-on-write: block 3 of sequence 1 copied to a fresh block that replaces it in the table
            fresh = PER * 7 + 5
            be.copy_blocks([(tabs[1][3], fresh)])
            tabs[1][3] = fresh
        greedy = k % 5 != 4
        items = [gck.Work(i, [toks[i][-1]], len(toks[i]) - 1, tabs[i], 1, greedy=greedy) for i in live]
        res = be.step(items)
        out.append(res)
        nxt = [r[0] for r in res] if greedy else [int(np.argmax(r)) for r in res]
        for i, t in zip(live, nxt):
            toks[i].append(int(t))
    return out, read()


def test_captured_steps_equal_direct_launches(tmp_path):
    spec = synth.Spec(**SMALL128, wtype="q4_k", seed=7)
    pack, ws = model(tmp_path, spec, ncol=16, maxctx=2048)
    os.environ["GCK_GRAPH"] = "0"
    try:
        with gck.Backend(pack, ws, pool_blocks=PER * 8) as be:
            ref, st_ref = script(be)
    finally:
        del os.environ["GCK_GRAPH"]
    with gck.Backend(pack, ws, pool_blocks=PER * 8) as be:
        got, st = script(be)
    assert st_ref.graph_steps == 0 and st_ref.graph_captures == 0
    # the decode loop's shapes repeat: most of its steps replay a graph
    assert st.graph_captures >= 1 and st.graph_steps >= 30, (st.graph_steps, st.graph_captures)
    assert st.launches == st_ref.launches
    assert len(got) == len(ref)
    for g, r in zip(got, ref):
        if isinstance(r, np.ndarray):
            assert np.array_equal(g, r)
        else:
            assert g == r


def test_decode_columns_equal_step(tmp_path):
    """Backend.decode (a decode step built from columns) is the same gc_step as Backend.step with one-token items:
    the same tokens and the same logits, bit for bit."""
    spec = synth.Spec(**SMALL128, wtype="q8_0", seed=9)
    pack, ws = model(tmp_path, spec, ncol=16, maxctx=1024)
    rng = np.random.default_rng(4)
    lens = [12, 130, 300, 5, 77, 513]
    toks = [[int(x) for x in rng.integers(1, 500, n)] for n in lens]
    tabs = [np.arange(PER * i, PER * (i + 1), dtype=np.uint32) for i in range(len(lens))]
    outs = {}
    for mode in ("step", "decode"):
        with gck.Backend(pack, ws, pool_blocks=PER * 8) as be:
            seqs = [list(t) for t in toks]
            be.step([gck.Work(i, seqs[i], 0, tabs[i], 0) for i in range(len(lens))])
            got = []
            for k in range(20):
                greedy = k % 4 != 3
                sids = np.arange(len(lens))
                last = [s[-1] for s in seqs]
                pos = [len(s) - 1 for s in seqs]
                if mode == "step":
                    r = be.step([gck.Work(i, [last[i]], pos[i], tabs[i], 1, greedy=greedy) for i in range(len(lens))])
                    nxt = [x[0] for x in r] if greedy else [int(np.argmax(x)) for x in r]
                else:
                    r = be.decode(sids, last, pos, tabs, greedy=greedy)
                    nxt = [int(x) for x in r] if greedy else [int(np.argmax(x)) for x in r]
                got.append(np.array(r).copy())
                for s, t in zip(seqs, nxt):
                    s.append(t)
            outs[mode] = got
    for a, b in zip(outs["step"], outs["decode"]):
        assert np.array_equal(np.asarray(a).reshape(b.shape), b)
