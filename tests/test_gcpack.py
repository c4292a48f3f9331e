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
