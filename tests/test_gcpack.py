"""The pack form of this library, on the CPU: the engine's own loader (goethe_engine/pack.py stage, schema check,
signature, variant choice by the weights' structure, bucket selection, blob extraction; gc_c.GcBackend and its
bind of the ABI) takes the .gcpack that goethe_engine_b200.gcpack writes around libgck.so. Without a GPU the open
ends at the library's gc_open with its no-device error: everything before the device has been accepted."""
import os

import pytest

from engine_ref import Key, engine, signed_pack
from goethe_engine_b200 import build, synth

pytestmark = pytest.mark.skipif(engine() is None, reason="the reference engine is not installed")


@pytest.fixture(scope="module")
def packed(tmp_path_factory):
    build.build()
    d = tmp_path_factory.mktemp("gcpack")
    spec = synth.Spec(vocab=512, d=256, layers=1, heads=4, kv_heads=2, ffn=512, wtype="q8_0")
    pack_dir, ws = synth.make(str(d / "m"), spec, buckets=[dict(id="b200.BI.8", ncol=8, maxctx=256),
                                                          dict(id="b200.BI.2", ncol=2, maxctx=256)])
    key = Key(str(d))
    return signed_pack(str(d), pack_dir, ws, key), ws, key


def test_engine_stages_and_validates_the_pack(packed):
    from goethe_engine import pack as P
    path, ws, key = packed
    st = P.stage(path, trusted=(key.kid,))
    try:
        m = st.manifest
        assert m["runtime"] == {"kind": "gc-c", "version": 1}
        assert {b["id"] for b in m["buckets"]} == {"b200.BI.8", "b200.BI.2"}
        assert P.pick_variant(m, ws) == "v"
        b = P.select(m, sku="b200", B=4, ctx=200)
        assert b["id"] == "b200.BI.8" and [x["id"] for x in P.ladder(m, b)] == ["b200.BI.2", "b200.BI.8"]
    finally:
        st.close()


def test_engine_refuses_a_pack_signed_by_an_untrusted_key(packed, tmp_path):
    from goethe_engine import pack as P
    path, _, _ = packed
    other = Key(str(tmp_path))
    with pytest.raises(P.PackError):
        P.stage(path, trusted=(other.kid,))


@pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="a device is present: the open would succeed")
def test_gc_backend_reaches_gc_open(packed):
    """GcBackend stages, selects and binds the pack's libgck.so; gc_open then reports the missing device."""
    from goethe_engine import pack as P
    from goethe_engine.gc_c import GcBackend
    path, ws, key = packed
    with pytest.raises(P.PackError, match=r"gc_open -4: no CUDA device"):
        GcBackend(path, ws, sku="b200", trusted=(key.kid,), B=4)


def test_engine_accepts_a_speculative_pair_pack(tmp_path):
    """A pack with a target and a drafter bucket and a spec entry (pack.py:130-141): the engine's loader validates it,
    picks variant v for the target weights and dv for the drafter's, names the pair with its ar policy, and a
    GcBackend with drafter_weights reaches the library's gc_open."""
    from goethe_engine import pack as P
    from goethe_engine.gc_c import GcBackend
    build.build()
    d = str(tmp_path)
    shape = dict(vocab=512, d=256, layers=1, heads=4, kv_heads=2, ffn=512)
    tgt = synth.make(d + "/t", synth.Spec(**shape, wtype="q4_k", seed=5))[1][0]
    dft = synth.make(d + "/d", synth.Spec(**dict(shape, layers=2), wtype="q8_0", seed=6))[1][0]
    pack_dir = synth.pack_dir(d + "/p", synth.Spec(**shape, wtype="q4_k", seed=5),
                              [dict(id="b200.BI.t", ncol=8, maxctx=256),
                               dict(id="b200.BI.d", ncol=8, maxctx=256, role="drafter")],
                              weights_file=os.path.basename(tgt), pairs=[("b200.BI.t", "b200.BI.d", 3)],
                              drafter_file=os.path.basename(dft))
    key = Key(d)
    path = signed_pack(d, pack_dir, [tgt], key, drafter_weights=[dft])
    st = P.stage(path, trusted=(key.kid,))
    try:
        m = st.manifest
        assert P.pick_variant(m, [tgt]) == "v" and P.pick_variant(m, [dft], "drafter") == "dv"
        t, dr, pol = P.spec_pair(P.for_variant(m, "v", "dv"), sku="b200")
        assert (t["id"], dr["id"], pol) == ("b200.BI.t", "b200.BI.d", {"kind": "ar", "K": "3"})
    finally:
        st.close()
    with pytest.raises(P.PackError, match="gc_open -4"):
        GcBackend(path, [tgt], drafter_weights=[dft], sku="b200", trusted=(key.kid,))
