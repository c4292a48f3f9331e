"""Speculative pairs (GC_OPEN_SPEC with policy "ar:K"): a target and a draft model decode one linear stream, and a step
with GC_W_SPEC runs a whole round on the device (gc.h:93,117,136,175-190; backend.py:27,41). A round returns 1 ..
spec_width tokens: the drafts the target accepted, then the target's own next token. So in batch-invariant numerics a
greedy stream decoded in rounds equals the target's plain greedy decode, token for token, whatever the drafter.

* drafter = the target's own weights: every draft is accepted (K + 1 tokens every round), which also checks that a
  verify row equals the drafter's one-row decode of the same token bit for bit (chunk invariance);
* drafter = the same init with Q8_0 instead of Q4_K weights: most drafts agree, some rounds stop early;
* drafter = an unrelated one-layer model: most rounds accept no draft;
* a rewind (a round restarted from an earlier position) and prefill chunks between rounds;
* sequences one after another on the one stream (released in between);
* what a pair refuses: tree items, several anchors, other pages, commit and copy_blocks.
"""
import os

import pytest

from goethe_engine_b200 import build, gck, synth
from helpers import SMALL128

pytestmark = pytest.mark.gpu
K = 3
MAXCTX = 512
PROMPT = [5, 77, 301, 12, 9, 400, 33, 33, 2, 150, 61, 7, 480, 19]


@pytest.fixture(scope="module", autouse=True)
def built():
    build.build()


@pytest.fixture(scope="module")
def pair(tmp_path_factory):
    """Target (Q4_K) and three drafters; a pack whose target bucket pairs with one drafter bucket per drafter file."""
    d = tmp_path_factory.mktemp("spec")
    tgt = synth.Spec(**SMALL128, wtype="q4_k", seed=31)
    files = {"self": synth.make(str(d / "t"), tgt)[1][0],
             "q8": synth.make(str(d / "q8"), synth.Spec(**SMALL128, wtype="q8_0", seed=31))[1][0],
             "other": synth.make(str(d / "o"), synth.Spec(**dict(SMALL128, layers=1), wtype="q8_0", seed=77))[1][0]}
    packs = {}
    for name, f in files.items():
        packs[name] = synth.pack_dir(str(d / f"pack_{name}"), tgt,
                                     [dict(id="b200.BI.t", ncol=1, maxctx=MAXCTX),
                                      dict(id="b200.BI.d", ncol=1, maxctx=MAXCTX, role="drafter")],
                                     weights_file=files["self"], pairs=[("b200.BI.t", "b200.BI.d", K)], drafter_file=f)
    return files, packs


def plain_greedy(pack, weights, prompt, n):
    """The target alone in its own bucket: prefill, then one-token greedy decodes."""
    with gck.Backend(pack, weights, buckets=("b200.BI.t",), pool_blocks=MAXCTX // 16 + 2) as be:
        blocks = list(range(MAXCTX // 16))
        seq = list(prompt) + be.step([gck.Work(0, list(prompt), 0, blocks, 1, greedy=True)])[0]
        while len(seq) < len(prompt) + n:
            seq += be.step([gck.Work(0, [seq[-1]], len(seq) - 1, blocks, 1, greedy=True)])[0]
    return seq[len(prompt):len(prompt) + n]


def rounds(be, prompt, n):
    """The stream decoded in speculative rounds; returns (tokens, tokens per round)."""
    seq = list(prompt) + be.step([gck.Work(0, list(prompt), 0, [0], 1, greedy=True)])[0]
    per = []
    while len(seq) < len(prompt) + n:
        got = be.step([gck.Work(0, [seq[-1]], len(seq) - 1, [0], 1, greedy=True, spec=True)])[0]
        assert 1 <= len(got) <= K + 1
        per.append(len(got))
        seq += got
    return seq[len(prompt):len(prompt) + n], per


def open_pair(pack, files, drafter):
    return gck.Backend(pack, [files["self"]], buckets=("b200.BI.t", "b200.BI.d"), drafter_weights=[files[drafter]])


@pytest.mark.parametrize("drafter", ["self", "q8", "other"])
def test_rounds_equal_plain_greedy(pair, drafter):
    files, packs = pair
    n = 48
    want = plain_greedy(packs[drafter], [files["self"]], PROMPT, n)
    with open_pair(packs[drafter], files, drafter) as be:
        assert be.spec_width == K + 1
        got, per = rounds(be, PROMPT, n)
    assert got == want
    if drafter == "self":
        assert all(c == K + 1 for c in per), per
    print(f"drafter {drafter}: {sum(per) / len(per):.2f} tokens a round over {len(per)} rounds")


def test_rewind_and_prefill_between_rounds(pair):
    """A round restarted from an earlier position (the engine dropping tokens), and a prompt extended by a prefill
    chunk between rounds (the drafter catches up in the next round), both equal the target alone."""
    files, packs = pair
    pack = packs["q8"]
    ext = [44, 45, 46, 47, 48, 49, 50]
    with open_pair(pack, files, "q8") as be:
        first, _ = rounds(be, PROMPT, 20)
        # rewind: resume from the 9th generated token as if the rest had been dropped
        seq = PROMPT + first[:9]
        while len(seq) < len(PROMPT) + 20:
            seq += be.step([gck.Work(0, [seq[-1]], len(seq) - 1, [0], 1, greedy=True, spec=True)])[0]
        again = seq[len(PROMPT):len(PROMPT) + 20]
        # a prefill chunk after the last anchor: the stream continues from PROMPT + first[:12] + ext
        base = PROMPT + first[:12]
        seq = base + ext
        seq += be.step([gck.Work(0, [base[-1]] + ext, len(base) - 1, [0], 1, greedy=True)])[0]
        while len(seq) < len(base) + len(ext) + 16:
            seq += be.step([gck.Work(0, [seq[-1]], len(seq) - 1, [0], 1, greedy=True, spec=True)])[0]
        cont = seq[len(base) + len(ext):len(base) + len(ext) + 16]
    assert again == first
    assert cont == plain_greedy(pack, [files["self"]], base + ext, 16)


def test_sequences_one_after_another(pair):
    """The pair's one stream serves sequence after sequence (the engine's use: max_num_seqs 1, gc_release between
    requests), each equal to the target alone; a new sequence while another still holds the stream is a state error."""
    files, packs = pair
    pack = packs["q8"]
    other = [300, 301, 5, 6, 7, 302, 303]
    with open_pair(pack, files, "q8") as be:
        a, _ = rounds(be, PROMPT, 16)
        be.release(0)
        b = rounds_sid(be, 1, other, 16)
        with pytest.raises(gck.GcError) as e:        # sequence 1 is not released: the stream is busy
            be.step([gck.Work(2, PROMPT, 0, [0], 1, greedy=True)])
        assert e.value.code == gck.E_STATE
        be.release(1)
        c = rounds_sid(be, 2, PROMPT, 16)
    assert a == plain_greedy(pack, [files["self"]], PROMPT, 16)
    assert b == plain_greedy(pack, [files["self"]], other, 16)
    assert c == a


def rounds_sid(be, sid, prompt, n):
    seq = list(prompt) + be.step([gck.Work(sid, list(prompt), 0, [0], 1, greedy=True)])[0]
    while len(seq) < len(prompt) + n:
        seq += be.step([gck.Work(sid, [seq[-1]], len(seq) - 1, [0], 1, greedy=True, spec=True)])[0]
    return seq[len(prompt):len(prompt) + n]


def test_pair_refusals(pair):
    files, packs = pair
    with open_pair(packs["self"], files, "self") as be:
        be.step([gck.Work(0, PROMPT, 0, [0], 1, greedy=True)])
        for bad in (gck.Work(0, [1, 2], len(PROMPT), [0], 1, greedy=True, spec=True),    # one anchor a round
                    gck.Work(0, [1], len(PROMPT), [1], 1, greedy=True, spec=True),       # the one page 0
                    gck.Work(0, [1], len(PROMPT) + 5, [0], 1, greedy=True, spec=True)):  # not contiguous
            with pytest.raises(gck.GcError):
                be.step([bad])
        with pytest.raises(gck.GcError) as e:
            be.commit(0, len(PROMPT), [0])
        assert e.value.code == gck.E_UNSUPPORTED
        with pytest.raises(gck.GcError) as e:
            be.copy_blocks([(0, 1)])
        assert e.value.code == gck.E_UNSUPPORTED
        # the stream still runs after the refusals
        assert 1 <= len(be.step([gck.Work(0, [PROMPT[-1]], len(PROMPT), [0], 1, greedy=True, spec=True)])[0]) <= K + 1


def test_open_refusals(pair):
    files, packs = pair
    for kw in (dict(policy="ar:0"), dict(policy="ar:16"), dict(policy="mtp:K=2")):
        with pytest.raises(gck.GcError):
            gck.Backend(packs["self"], [files["self"]], buckets=("b200.BI.t", "b200.BI.d"),
                        drafter_weights=[files["self"]], **kw)
    with pytest.raises(gck.GcError):      # a pair opens exactly two buckets
        gck.Backend(packs["self"], [files["self"]], buckets=("b200.BI.t",), drafter_weights=[files["self"]])
    assert os.path.exists(files["other"])
