"""The drop-in, on the GPU: the reference engine, unchanged, drives libgck.so. A signed .gcpack around the library
(goethe_engine_b200.gcpack, signed with the engine's pack.sign_pack) is opened by the engine's GcBackend
(goethe_engine/gc_c.py), and the engine's Engine, Scheduler, KVManager (radix prefix cache, copy-on-write blocks,
preemption by recompute) and sampler run requests through it. The properties are those the reference's conformance
suite states for any gc-c runtime (tests/test_gc_conformance.py:72-169, 190-211), checked here in this project's
own code:

* greedy generation through the engine against the oracle's logits, token by token (teacher-forced: every token the
  engine produced must be the oracle's argmax wherever the oracle's top-2 margin exceeds twice the a16 tolerance);
* batch and chunk invariance: each prompt alone equals the prompts batched, in small prefill chunks, and in mixed
  budgets, token for token;
* the prefix cache (shared pages and copy-on-write through gc_copy_blocks) gives the tokens of no cache, and a repeated
  prompt hits the cache;
* a pool too small for all requests preempts and recomputes to the same tokens; forced preemption likewise;
* seeded sampling on the logits path is independent of the batch;
* tree verify equals the chain and commit leaves the chain's rows (GcBackend.step / commit);
* errors are codes, an unknown sequence's release is not an error;
* a caller with ABI 1.0 struct sizes (no state_pages, a shorter layout) opens the library and reads its layout.
The engine package comes from baseline/_ref on the GPU box; the tests skip where it is absent."""
import ctypes as C
import os
import random

import numpy as np
import pytest

from engine_ref import Key, engine, signed_pack
from goethe_engine_b200 import build, synth
from helpers import TOL_F16
from oracle.load import weights_from_gguf
from oracle.model import PagedOracle

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(engine() is None, reason="the reference engine is not installed")]
SHAPE = dict(vocab=512, d=512, layers=2, heads=4, kv_heads=1, ffn=768)   # dh 128, GQA 4


@pytest.fixture(scope="module")
def pack(tmp_path_factory):
    build.build()
    d = tmp_path_factory.mktemp("dropin")
    spec = synth.Spec(**SHAPE, wtype="q8_0", seed=17)
    pack_dir, ws = synth.make(str(d / "m"), spec, buckets=[dict(id="b200.BI.8", ncol=8, maxctx=256),
                                                          dict(id="b200.BI.2", ncol=2, maxctx=256)])
    key = Key(str(d))
    return signed_pack(str(d), pack_dir, ws, key), ws, key


@pytest.fixture
def make(pack):
    from goethe_engine.gc_c import GcBackend
    path, ws, key = pack
    made = []

    def factory(**kw):
        be = GcBackend(path, ws, sku="b200", trusted=(key.kid,), **kw)
        made.append(be)
        return be
    yield factory
    for b in made:
        b.close()


def prompts(n=6, seed=3):
    rng = random.Random(seed)
    base = [rng.randrange(1, 500) for _ in range(40)]
    return [base[:rng.choice([1, 5, 9, 17, 33, 40])] + [rng.randrange(1, 500) for _ in range(rng.randint(1, 6))]
            for _ in range(n)]


def gen(be, ps, k=12, params=None, **cfg):
    from goethe_engine import Config, Engine, SamplingParams
    eng = Engine(be, Config(max_model_len=200, **cfg))
    out = eng.generate([(p, params or SamplingParams(max_tokens=k)) for p in ps])
    eng.check()
    return [o[0] for o in out]


def test_layout_through_the_engine(make):
    be = make()
    assert be.L.gc_abi_version() >> 16 == 1
    assert be.paged and be.device_argmax and be.prefix_cache and be.caps["tree"]
    g = be.geometry
    assert (g.block_size, g.layers, g.kv_heads, g.head_dim, g.dtype) == (16, 2, 1, 128, "f16")
    assert be.max_seqs == 8 and be.vocab_size == 512


def test_engine_greedy_matches_the_oracle(make, pack):
    be = make()
    ps = prompts(4)
    got = gen(be, ps, 12, max_num_seqs=4)
    w = weights_from_gguf(pack[1][0])
    for p, out in zip(ps, got):
        assert len(out) == 12
        o = PagedOracle(w, num_blocks=16, kv="f16")
        blocks = list(range(16))
        lg = o.step([dict(sid=0, tokens=p, pos=0, blocks=blocks, want=1)])[-1]
        seq = list(p)
        for t in out:
            srt = np.sort(lg)
            if (srt[-1] - srt[-2]) / np.abs(lg).max() > 2 * TOL_F16:
                assert t == int(lg.argmax()), (p, out)
            seq.append(t)
            lg = o.step([dict(sid=0, tokens=[t], pos=len(seq) - 1, blocks=blocks, want=1)])[-1]


def test_batch_and_chunk_invariance(make):
    be = make()
    ps = prompts()
    alone = [gen(be, [p], 12, max_num_seqs=1, prefix_cache=False)[0] for p in ps]
    for cfg in (dict(max_num_seqs=8), dict(max_num_seqs=8, max_num_batched_tokens=7, prefix_cache=False),
                dict(max_num_seqs=3, max_num_batched_tokens=64)):
        assert gen(be, ps, **cfg) == alone, cfg


def test_prefix_cache_and_copy_blocks(make):
    from goethe_engine import Config, Engine, SamplingParams
    be = make()
    base = prompts(1)[0] * 3
    ps = [base[:30] + [5, 6], base[:30] + [7], base[:30] + [5, 6], base[:19]]
    assert gen(be, ps, max_num_seqs=4) == gen(be, ps, max_num_seqs=4, prefix_cache=False)
    eng = Engine(be, Config(max_model_len=200, max_num_seqs=4))
    cold = eng.generate([(ps[0], SamplingParams(max_tokens=12))])
    warm = eng.generate([(ps[0], SamplingParams(max_tokens=12)), (ps[0] + cold[0][0], SamplingParams(max_tokens=12))])
    assert warm[0] == cold[0]
    assert eng.metrics()["prefix_hit_tokens"] > 0
    eng.check()


def test_small_pool_preempts_and_matches(make):
    from goethe_engine import Config, Engine, SamplingParams
    big = make()
    ps = prompts(6)
    need = [-(-(len(p) + 20) // 16) for p in ps]
    assert sum(need) > max(need) + 1
    small = make(pool_blocks=max(need) + 1)
    cfg = dict(max_model_len=200, prefix_cache=False)
    ref = [o[0] for o in Engine(big, Config(max_num_seqs=1, **cfg)).generate(
        [(p, SamplingParams(max_tokens=20)) for p in ps])]
    eng = Engine(small, Config(max_num_seqs=6, **cfg))
    got = eng.generate([(p, SamplingParams(max_tokens=20)) for p in ps])
    assert [o[0] for o in got] == ref and eng.metrics()["preemptions"] > 0


def test_forced_preemption_recomputes_to_the_same_tokens(make):
    from goethe_engine import Config, Engine, SamplingParams
    be = make()
    ps = prompts(5)
    ref = gen(be, ps, 14, max_num_seqs=1, prefix_cache=False)
    for cache in (False, True):
        eng = Engine(be, Config(max_model_len=200, max_num_seqs=5, prefix_cache=cache))
        for i, p in enumerate(ps):
            eng.add_request(i, p, SamplingParams(max_tokens=14))
        out, k = {}, 0
        while eng.has_work():
            for o in eng.step():
                out.setdefault(o.rid, []).extend(o.token_ids)
            eng.check()
            k += 1
            if k % 3 == 0 and eng.sched.running:
                v = eng.sched.running[-1]
                eng.sched._preempt(v)
                be.release(v.sid)
        assert [out[i] for i in range(len(ps))] == ref and eng.metrics()["preemptions"] > 2


def test_seeded_sampling_on_the_logits_path_is_batch_independent(make):
    from goethe_engine import SamplingParams
    be = make()
    ps = prompts()
    sp = SamplingParams(temperature=0.8, top_k=20, seed=11, max_tokens=10)
    alone = [gen(be, [p], params=sp, max_num_seqs=1, prefix_cache=False)[0] for p in ps]
    assert gen(be, ps, params=sp, max_num_seqs=8) == alone


def test_tree_verify_equals_chain_and_commit(make):
    from goethe_engine.backend import Work
    be = make()
    pre, a, b, c = [3, 9, 4, 1], 7, 11, 13

    def step(sid, pos, toks, par, want, blocks):
        return be.step([Work(sid, toks, pos, blocks, want, False, False, par, False)])
    t1, t2 = list(range(0, 8)), list(range(8, 16))
    step(1, 0, pre, None, 0, t1)
    tree = step(1, 4, [a, b, c], [-1, 0, 0], 3, t1)              # b and c are siblings under a
    step(2, 0, pre, None, 0, t2)
    chain = step(2, 4, [a, c], None, 2, t2)                      # a then c
    assert (tree[2] == chain[1]).all() and (tree[0] == chain[0]).all()
    be.commit(1, 4, [0, 2])                                      # keep a, c as rows 4, 5
    assert (step(1, 6, [a], None, 1, t1) == step(2, 6, [a], None, 1, t2)).all()


def test_errors_are_codes_not_crashes(make):
    from goethe_engine.backend import Work
    be = make()
    with pytest.raises(RuntimeError, match="gc call failed"):
        be.step([Work(1, [1, 2], 0, [10_000], 1)])
    be.release(999)
    assert be.step([Work(1, [1, 2], 0, [0], 1)]).shape == (1, 512)


def test_abi_1_0_struct_sizes_open(pack):
    """A 1.0 caller's OpenParams (no state_pages) and Layout (no state_pages, pad1): gc_open reads only what the caller
    passed and gc_layout_get writes no further than the caller's size."""
    from goethe_engine import gc_c, pack as P
    path, ws, key = pack
    st = P.stage(path, trusted=(key.kid,))
    try:
        m = st.manifest
        b = P.select(m, sku="b200", B=8, ctx=200)
        st.ensure([b])
        L = gc_c.bind(os.path.join(P.materialize(st, b), b["lib"]))

        class Open10(C.Structure):
            _fields_ = gc_c.OpenParams._fields_[:-1]

        class Layout10(C.Structure):
            _fields_ = gc_c.Layout._fields_[:-2]
        wv = gc_c.arr(C.c_char_p, [os.fsencode(w) for w in ws])
        bk = gc_c.arr(C.c_char_p, [b["id"].encode()])
        p = Open10(C.sizeof(Open10), gc_c.OPEN_NO_CHECK, os.fsencode(st.dir), wv, len(ws), -1, bk, 1, 32, None, None)
        h = C.c_void_p()
        rc = L.gc_open(C.cast(C.byref(p), C.POINTER(gc_c.OpenParams)), C.byref(h))
        assert rc == 0, L.gc_last_error(None)
        buf = (C.c_uint8 * (C.sizeof(Layout10) + 16))(*([0xAB] * (C.sizeof(Layout10) + 16)))
        lo = Layout10.from_buffer(buf)
        lo.size = C.sizeof(Layout10)
        assert L.gc_layout_get(h, C.cast(C.byref(lo), C.POINTER(gc_c.Layout))) == 0
        assert lo.size == C.sizeof(Layout10) and lo.num_blocks == 32 and lo.block_size == 16 and lo.vocab == 512
        assert all(x == 0xAB for x in bytes(buf)[C.sizeof(Layout10):])       # nothing written past the caller's size
        L.gc_close(h)
    finally:
        st.close()


def test_engine_speculative_pair_equals_the_target_alone(tmp_path):
    """A speculative pair through the engine (SPEC_CAPS "ar", gc.h:56-59,93,117,136): the pack pairs a Q4_K target
    with a Q8_0 drafter of the same init (policy {kind "ar", K "3"}); GcBackend(..., drafter_weights=...) opens the
    pair, the engine runs its stream in device rounds (backend.spec_width), and greedy generation equals the target
    alone token for token, with drafts accepted."""
    from goethe_engine import Config, Engine, SamplingParams
    from goethe_engine.gc_c import GcBackend
    d = str(tmp_path)
    tgt = synth.make(d + "/t", synth.Spec(**SHAPE, wtype="q4_k", seed=17))[1][0]
    dft = synth.make(d + "/d", synth.Spec(**SHAPE, wtype="q8_0", seed=17))[1][0]
    pack_dir = synth.pack_dir(d + "/p", synth.Spec(**SHAPE, wtype="q4_k", seed=17),
                              [dict(id="b200.BI.t", ncol=8, maxctx=256),
                               dict(id="b200.BI.d", ncol=8, maxctx=256, role="drafter")],
                              weights_file=os.path.basename(tgt), pairs=[("b200.BI.t", "b200.BI.d", 3)],
                              drafter_file=os.path.basename(dft))
    key = Key(d)
    path = signed_pack(d, pack_dir, [tgt], key, drafter_weights=[dft])
    ps = prompts(3, seed=8)
    plain = GcBackend(path, [tgt], sku="b200", trusted=(key.kid,))
    try:
        want = gen(plain, ps, 24)
    finally:
        plain.close()
    pair = GcBackend(path, [tgt], drafter_weights=[dft], sku="b200", trusted=(key.kid,))
    try:
        assert pair.spec_width == 4
        eng = Engine(pair, Config(max_model_len=200))
        got = [o[0] for o in eng.generate([(p, SamplingParams(max_tokens=24)) for p in ps])]
        eng.check()
        m = eng.metrics()
    finally:
        pair.close()
    assert got == want
    assert m["spec_accepted"] > 0, m
