"""gate/up and down_proj as one chained launch against two launches.

Steps of at most 64 token rows (one token tile) on the tcgen05 GEMM run gate/up (SwiGLU epilogue) and down_proj in
one persistent launch: each CTA takes its units from a host schedule, and a down_proj unit waits, per 256-K tile of its
input, until the gate/up bands that write that tile have stored it. A handle opened with GCK_CHAIN=0 launches the two
GEMMs one after the other. Every unit's arithmetic is the same either way (down_proj's split-K is fixed per weight), so
the logits must agree bit for bit, through:

* decode steps of 1, 16, 40 and 64 rows (token tiles of 16, 32 and 64 rows) between prefill steps of more rows
  (those run two launches in both handles);
* Q4_K and Q8_0 weights; a model whose FFN width leaves the last down_proj K tile fed by fewer than four gate/up bands;
* greedy steps (device argmax) and host logits.
The chained handle also launches one kernel fewer per layer at those steps.
"""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402
from goethe_engine_b200 import build, gck, synth  # noqa: E402

pytestmark = pytest.mark.gpu
PER = 24
EVEN = dict(vocab=512, d=512, layers=2, heads=4, kv_heads=1, ffn=768)
# ffn 1088 (Q8_0 only: K a multiple of 32, not of 256): gate/up 17 bands of 64 features, down_proj 5 K tiles, the last
# fed by one band
RAGGED = dict(vocab=512, d=512, layers=2, heads=4, kv_heads=1, ffn=1088)


@pytest.fixture(scope="module", autouse=True)
def built():
    build.build()


def script(be):
    on, read = bench.stats_api(be)
    on(False)
    rng = np.random.default_rng(17)
    n = 64
    lens = [int(x) for x in rng.integers(3, 30, n)]
    toks = [[int(x) for x in rng.integers(1, 500, k)] for k in lens]
    tabs = [list(range(PER * i, PER * (i + 1))) for i in range(n)]
    out = [be.step([gck.Work(i, toks[i], 0, tabs[i], 1) for i in range(n)])]
    for k, width in enumerate((1, 16, 40, 64, 64, 40, 16, 1)):
        greedy = k % 3 == 2
        items = [gck.Work(i, [toks[i][-1]], len(toks[i]) - 1, tabs[i], 1, greedy=greedy) for i in range(width)]
        res = be.step(items)
        out.append(res)
        nxt = [r[0] for r in res] if greedy else [int(np.argmax(r)) for r in np.asarray(res).reshape(width, -1)]
        for i, t in zip(range(width), nxt):
            toks[i].append(int(t))
    return out, read()


def run(tmp_path, dims, wtype, chain):
    spec = synth.Spec(**dims, wtype=wtype, seed=41)
    pack, ws = synth.make(str(tmp_path / f"{wtype}_{dims['ffn']}"), spec, ncol=2048, maxctx=PER * 16)
    os.environ["GCK_CHAIN"] = "1" if chain else "0"
    try:
        with gck.Backend(pack, ws, pool_blocks=PER * 65) as be:
            return script(be)
    finally:
        os.environ.pop("GCK_CHAIN", None)


@pytest.mark.parametrize("wtype", ["q4_k", "q8_0"])
@pytest.mark.parametrize("dims", [EVEN, RAGGED], ids=["even", "ragged"])
def test_chained_equals_two_launches(tmp_path, dims, wtype):
    if wtype == "q4_k" and dims["ffn"] % 256:
        pytest.skip("Q4_K rows are whole 256-weight blocks")
    ref, st_ref = run(tmp_path, dims, wtype, False)
    got, st = run(tmp_path, dims, wtype, True)
    # eight decode steps of one token tile, one launch fewer per layer in each
    assert st_ref.launches - st.launches == 8 * dims["layers"], (st_ref.launches, st.launches)
    assert len(got) == len(ref)
    for g, r in zip(got, ref):
        if isinstance(r, np.ndarray):
            assert np.array_equal(g, r)
        else:
            assert g == r
