"""The Python binding's step marshalling (no GPU): the gc_work records handed to gc_step carry each Work item's sid,
position, tokens, block table, parents, want and flags (gc.h:133-157), with block tables as lists or uint32 arrays."""
import numpy as np

from goethe_engine_b200 import gck


class FakeLib:
    """Stands in for libgck.so: records what gc_step receives and answers greedy tokens."""

    def __init__(self):
        self.seen = None

    def gc_step(self, h, pin, pout):
        si, so = pin._obj, pout._obj
        self.seen = []
        for i in range(si.n_work):
            r = si.work[i].contents
            self.seen.append(dict(size=r.size, flags=r.flags, sid=r.sid, pos=r.pos, want=r.want,
                                  tokens=[r.tokens[j] for j in range(r.n_tokens)],
                                  blocks=[r.blocks[j] for j in range(r.n_blocks)],
                                  parents=[r.parents[j] for j in range(r.n_tokens)] if r.parents else None))
        if so.tokens:
            for k in range(so.tokens_cap):
                so.tokens[k] = 100 + k
            for i, x in enumerate(self.seen):
                so.counts[i] = x["want"]
        so.n_rows = sum(x["want"] for x in self.seen)
        return 0


def backend(greedy):
    b = gck.Backend.__new__(gck.Backend)
    b.L, b.h, b.device_argmax, b.vocab_size = FakeLib(), None, greedy, 1000
    b._ck = lambda rc: None
    return b


def test_records_match_work_items():
    b = backend(True)
    work = [gck.Work(7, [3, 4, 5], 32, [9, 8, 2], 2, greedy=True),
            gck.Work(2, [11], 17, np.array([4, 6], np.uint32), 1, greedy=True),
            gck.Work(5, [1, 2, 3, 4], 0, np.arange(10, 14, dtype=np.int64), 4, greedy=True, parents=[-1, 0, 0, 1])]
    out = b.step(work)
    assert out == [[100, 101], [102], [103, 104, 105, 106]]
    for w, r in zip(work, b.L.seen):
        assert r["size"] == 56 and r["flags"] == gck.W_GREEDY
        assert (r["sid"], r["pos"], r["want"]) == (w.sid, w.pos, w.want)
        assert r["tokens"] == list(w.tokens) and r["blocks"] == [int(x) for x in w.blocks]
        assert r["parents"] == (list(w.parents) if w.parents is not None else None)


def test_logits_request_without_device_argmax():
    b = backend(False)
    lg = b.step([gck.Work(1, [3], 0, [0], 1)])
    assert lg.shape == (1, 1000) and b.L.seen[0]["flags"] == 0


def test_all_array_tables_and_all_list_tables_give_the_same_records():
    # block tables given as uint32 arrays pass through as one concatenation; Python lists are converted in one pass
    tabs = [[3, 9, 1], [40], list(range(100, 137))]
    b1, b2 = backend(True), backend(True)
    b1.step([gck.Work(i, [i + 1, 7], 16 * i, t, 1, greedy=True) for i, t in enumerate(tabs)])
    b2.step([gck.Work(i, np.array([i + 1, 7], np.int32), 16 * i, np.asarray(t, np.uint32), 1, greedy=True)
             for i, t in enumerate(tabs)])
    assert b1.L.seen == b2.L.seen
    assert [r["blocks"] for r in b1.L.seen] == tabs


def test_values_outside_the_record_types_raise_on_the_host():
    # a negative block id or a token beyond int32 cannot be written into the records: an error, not a wrapped value
    b = backend(True)
    for bad in (gck.Work(1, [3], 0, [0, -1], 1, greedy=True), gck.Work(1, [2 ** 31], 0, [0], 1, greedy=True),
                gck.Work(1, [3], 0, [2 ** 32], 1, greedy=True)):
        try:
            b.step([bad])
        except (OverflowError, ValueError):
            continue
        raise AssertionError(f"accepted {bad}")


def test_decode_columns_build_the_step_records():
    """Backend.decode hands gc_step the same records as step() with one-token items (greedy and logits steps), and
    returns the tokens in item order."""
    rng = np.random.default_rng(3)
    tabs = [np.arange(40 * i, 40 * i + int(rng.integers(3, 40)), dtype=np.uint32) for i in range(5)]
    sids, toks, pos = [9, 2, 7, 4, 11], [5, 6, 7, 8, 9], [3, 50, 17, 600, 1]
    for greedy in (True, False):
        a, b = backend(greedy), backend(greedy)
        a.spec_width = b.spec_width = 0
        out_a = a.step([gck.Work(s, [t], p, tb, 1, greedy=greedy) for s, t, p, tb in zip(sids, toks, pos, tabs)])
        out_b = b.decode(np.array(sids), toks, pos, tabs, greedy=greedy)
        assert a.L.seen == b.L.seen
        if greedy:
            assert [x[0] for x in out_a] == list(out_b) == [100, 101, 102, 103, 104]
        else:
            assert out_a.shape == out_b.shape == (5, 1000)
