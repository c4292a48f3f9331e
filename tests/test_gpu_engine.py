"""Engine-level behaviour through the C ABI, the way goethe_engine's scheduler drives a backend
(reference tests/test_gc_conformance.py:97-131, 165-169):

* every gc_step validation failure is an error code (GC_E_ARG / GC_E_STATE), never a crash, and leaves the handle
  usable (empty steps, tokens outside the vocabulary, bad parents, a sequence twice in one step, positions past the
  context, more tokens than the bucket's columns, more items than its sequences, want > n_tokens);
* forced preemption: sequences released mid-generation and recomputed later from their prompt and the tokens they
  had produced decode to the same greedy tokens as each sequence alone (batch and chunk invariance plus slot and block
  reuse), with a block pool smaller than all requests together.
"""
import numpy as np
import pytest

from goethe_engine_b200 import build, gck, synth
from helpers import SMALL128, model

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def built():
    build.build()


@pytest.fixture(scope="module")
def small(tmp_path_factory):
    spec = synth.Spec(**SMALL128, wtype="q4_k", seed=13)
    return model(tmp_path_factory.mktemp("eng"), spec, ncol=4, maxctx=256, tune=dict(max_cols=128))


def test_step_validation_errors_leave_the_handle_usable(small):
    pack, ws = small
    with gck.Backend(pack, ws, pool_blocks=64) as be:
        V = be.vocab_size
        bad = {
            "empty step": [],
            "token outside the vocabulary": [gck.Work(1, [1, V], 0, [0], 1)],
            "negative token": [gck.Work(1, [-3], 0, [0], 1)],
            "parent not earlier": [gck.Work(1, [1, 2, 3], 0, [0], 3, parents=[-1, 2, 0])],
            "sequence twice": [gck.Work(1, [1], 0, [0], 1), gck.Work(1, [2], 0, [1], 1)],
            "past the context": [gck.Work(1, [1, 2], 255, list(range(17)), 1)],
            "block out of the pool": [gck.Work(1, [1], 0, [64], 1)],
            "table too short": [gck.Work(1, [1] * 20, 0, [0], 1)],
            "more tokens than columns": [gck.Work(1, [1] * 129, 0, list(range(9)), 1)],
            "more items than sequences": [gck.Work(i, [1], 0, [i], 1) for i in range(5)],
        }
        for what, items in bad.items():
            with pytest.raises(gck.GcError) as e:
                be.step(items)
            assert e.value.code == gck.E_ARG, what
        # want > n_tokens is refused before any device work
        with pytest.raises(gck.GcError) as e:
            be.step([gck.Work(1, [1, 2], 0, [0], 3)])
        assert e.value.code == gck.E_ARG
        # full slots: four live sequences, a fifth is GC_E_STATE
        for i in range(4):
            be.step([gck.Work(10 + i, [1, 2], 0, [2 * i], 0)])
        with pytest.raises(gck.GcError) as e:
            be.step([gck.Work(99, [1], 0, [20], 1)])
        assert e.value.code == gck.E_STATE
        be.release(12)
        assert be.step([gck.Work(99, [1], 0, [20], 1)]).shape == (1, V)
        # the last position of the context still runs
        be.release(99)
        assert be.step([gck.Work(99, [3], 255, list(range(30, 46)), 1)]).shape == (1, V)


def generate(be, prompts, max_tokens, batch, preempt_every=0):
    """Greedy decode with at most `batch` running sequences over a shared block pool; every `preempt_every` steps the
    newest running sequence is preempted: released, its blocks freed, and queued again to be recomputed from its prompt
    and the tokens it had produced (what the reference scheduler does on preemption)."""
    bs = be.block_size
    free = list(range(be.num_blocks))
    waiting = list(range(len(prompts)))
    out = {i: [] for i in range(len(prompts))}
    running = {}                     # rid -> (blocks, position of the next token, last token)
    k, sid_of = 0, {}
    next_sid = [100]
    while waiting or running:
        # admit: a whole reservation (prompt + max_tokens) per sequence, as a page-granular KV manager would
        while waiting and len(running) < batch:
            rid = waiting[0]
            need = -(-(len(prompts[rid]) + max_tokens) // bs)
            if need > len(free):
                break
            waiting.pop(0)
            blocks = [free.pop(0) for _ in range(need)]
            toks = prompts[rid] + out[rid]
            sid = next_sid[0]
            next_sid[0] += 1
            sid_of[rid] = sid
            first = be.step([gck.Work(sid, toks, 0, blocks, 1, greedy=True)])[0][0]
            out[rid].append(first)
            running[rid] = (blocks, len(toks), first)
        done = [r for r in running if len(out[r]) >= max_tokens]
        for r in done:
            be.release(sid_of[r])
            free.extend(running.pop(r)[0])
        if not running:
            continue
        rids = sorted(running)
        res = be.step([gck.Work(sid_of[r], [running[r][2]], running[r][1], running[r][0], 1, greedy=True) for r in rids])
        for r, t in zip(rids, res):
            out[r].append(t[0])
            blocks, pos, _ = running[r]
            running[r] = (blocks, pos + 1, t[0])
        k += 1
        if preempt_every and k % preempt_every == 0 and len(running) > 1:
            v = max(running)
            be.release(sid_of[v])
            free.extend(running.pop(v)[0])
            waiting.insert(0, v)
    return [out[i][:max_tokens] for i in range(len(prompts))]


def test_forced_preemption_recomputes_to_the_same_tokens(small):
    pack, ws = small
    rng = np.random.default_rng(8)
    prompts = [[int(x) for x in rng.integers(1, 500, 9 + 7 * i)] for i in range(5)]
    with gck.Backend(pack, ws, pool_blocks=64) as be:
        alone = [generate(be, [p], 14, 1)[0] for p in prompts]
    # a pool that holds the longest request but not all five: the scheduler queues, and preempts every third step
    need = max(-(-(len(p) + 14) // 16) for p in prompts)
    with gck.Backend(pack, ws, pool_blocks=2 * need + 1) as be:
        got = generate(be, prompts, 14, 4, preempt_every=3)
    assert got == alone
