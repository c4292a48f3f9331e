"""The C-ABI library on the CPU: it loads, exports every symbol include/gc.h declares, reports ABI 1.2, and turns bad
arguments into error codes (no GPU needed: gc_open checks its arguments, manifest and weights before the device).
Where the reference is mounted, its own binding (goethe_engine/gc_c.py) is checked against this library too."""
import ctypes as C
import os
import re
import sys

import pytest

from goethe_engine_b200 import build, gck, synth

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = "/root/reference"


@pytest.fixture(scope="module")
def lib():
    build.build()
    return gck.load()


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    d = tmp_path_factory.mktemp("tiny")
    spec = synth.Spec(vocab=512, d=256, layers=1, heads=4, kv_heads=2, ffn=512, wtype="q8_0")
    return synth.make(str(d), spec, ncol=4, maxctx=256)


def declared(header):
    txt = open(os.path.join(ROOT, "include", header)).read()
    return re.findall(r"GC_API\s+[\w\s\*]+?\b(gck?_\w+)\s*\(", txt)


def test_exports_every_declared_symbol(lib):
    assert set(declared("gc.h")) == set(gck.SYMBOLS)
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        names = declared(h)
        assert names, h
        for n in names:
            assert hasattr(lib, n), (h, n)


def test_abi_version(lib):
    assert lib.gc_abi_version() == (1 << 16 | 2)


def _open(lib, pack_dir, weights, buckets=("b200.BI.main",), flags=2, size=None):
    ws = gck.arr(C.c_char_p, [os.fsencode(w) if w else None for w in weights])
    bk = gck.arr(C.c_char_p, [b.encode() for b in buckets])
    p = gck.OpenParams(size or C.sizeof(gck.OpenParams), flags, os.fsencode(pack_dir), ws, len(weights), -1, bk,
                       len(buckets), 0, None, None, 0)
    h = C.c_void_p()
    rc = lib.gc_open(C.byref(p), C.byref(h))
    return rc, h, (lib.gc_last_error(None) or b"").decode()


def test_open_errors_are_codes(lib, tiny, tmp_path):
    pack, ws = tiny
    rc, h, msg = _open(lib, str(tmp_path), ws)
    assert rc == gck.E_MANIFEST and "manifest" in msg and not h.value
    rc, h, msg = _open(lib, pack, ws, buckets=("nope",))
    assert rc == gck.E_MANIFEST and "nope" in msg
    rc, h, msg = _open(lib, pack, [str(tmp_path / "missing.gguf")])
    assert rc == gck.E_WEIGHTS
    # a speculative pair: two buckets {target, drafter}; a pair the manifest gives no ar:K policy is not run
    rc, h, msg = _open(lib, pack, ws, flags=3)
    assert rc == gck.E_ARG and "two buckets" in msg
    rc, h, msg = _open(lib, pack, ws, flags=3, buckets=("b200.BI.main", "b200.BI.main"))
    assert rc == gck.E_UNSUPPORTED and "ar:K" in msg
    assert lib.gc_open(None, C.byref(C.c_void_p())) == gck.E_ARG
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"not a gguf")
    rc, h, msg = _open(lib, pack, [str(bad)])
    assert rc == gck.E_WEIGHTS and "GGUF" in msg


def test_open_rejects_bad_tensor_parallel_degree(lib, tiny, tmp_path):
    pack, ws = tiny
    spec = synth.Spec(vocab=512, d=256, layers=1, heads=4, kv_heads=2, ffn=512, wtype="q8_0")
    bad = synth.pack_dir(str(tmp_path / "tp3"), spec, [dict(id="b200.BI.main", ncol=4, maxctx=256, tp=3)])
    rc, h, msg = _open(lib, bad, ws)
    assert rc == gck.E_MANIFEST and "tensor-parallel" in msg and not h.value


def _blob(hbm_gbs, launch_us, sms=148, clock=1965):
    import struct
    return struct.pack("<IIddII", 0x45435250, 1, hbm_gbs, launch_us, sms, clock)


def test_price_is_host_math_over_the_probe_constants(lib):
    """gc_price (abi/gc.h:232-237): the reference step's weight stream at the probed bandwidth plus its launches;
    a faster device prices lower; a blob of the wrong size or kind is an argument error."""
    lib.gc_price.restype = C.c_int
    lib.gc_price.argtypes = [C.c_void_p, C.c_uint64, C.c_char_p, C.POINTER(C.c_double)]
    us = C.c_double()
    b = _blob(6000.0, 2.0)
    assert lib.gc_price(b, len(b), b"b200.BI.main", C.byref(us)) == gck.OK
    assert abs(us.value - (4.221e9 / (6000e9 * 0.85) * 1e6 + 292 * 2.0)) < 1e-6
    fast = C.c_double()
    b2 = _blob(8000.0, 1.5)
    assert lib.gc_price(b2, len(b2), b"b200.BI.main", C.byref(fast)) == gck.OK and fast.value < us.value
    assert lib.gc_price(b, len(b) - 1, b"b200.BI.main", C.byref(us)) == gck.E_ARG
    assert lib.gc_price(b"x" * len(b), len(b), b"b200.BI.main", C.byref(us)) == gck.E_ARG


def test_probe_reports_its_size_first(lib):
    lib.gc_probe.restype = C.c_int
    lib.gc_probe.argtypes = [C.c_int, C.c_void_p, C.c_uint64, C.POINTER(C.c_uint64)]
    n = C.c_uint64()
    assert lib.gc_probe(0, None, 0, C.byref(n)) == gck.E_CAPACITY and n.value == 32
    if not __import__("torch").cuda.is_available():
        buf = C.create_string_buffer(n.value)
        assert lib.gc_probe(0, buf, n.value, C.byref(n)) == gck.E_DEVICE


def test_null_handles(lib):
    assert lib.gc_layout_get(None, None) == gck.E_ARG
    assert lib.gc_step(None, None, None) == gck.E_ARG
    assert lib.gc_release(None, 1) == gck.E_ARG
    lib.gc_close(None)


@pytest.mark.skipif(bool(os.environ.get("CUDA_VISIBLE_DEVICES", "x")) and __import__("torch").cuda.is_available(),
                    reason="a device is present")
def test_open_without_a_device_says_so(lib, tiny):
    pack, ws = tiny
    rc, h, msg = _open(lib, pack, ws)
    assert rc == gck.E_DEVICE and "device" in msg


@pytest.mark.skipif(not os.path.isdir(REF), reason="reference not mounted")
def test_reference_binding_accepts_this_library():
    """The engine's own ctypes binding (gc_c.bind: symbol set and ABI major/minor) loads libgck.so, and its struct
    mirrors have the sizes this library's structs have."""
    sys.path.insert(0, REF)
    try:
        from goethe_engine import gc_c
    finally:
        sys.path.remove(REF)
    build.build()
    L = gc_c.bind(gck.LIB_PATH)
    assert L.gc_abi_version() >> 16 == 1
    assert C.sizeof(gc_c.OpenParams) == C.sizeof(gck.OpenParams)
    assert C.sizeof(gc_c.Work) == C.sizeof(gck.WorkS)
    assert C.sizeof(gc_c.StepIn) == C.sizeof(gck.StepIn)
    assert C.sizeof(gc_c.StepOut) == C.sizeof(gck.StepOut)
    # the engine's Layout stops at pad1 (ABI 1.1); ours has the 1.2 tail
    assert [f[0] for f in gc_c.Layout._fields_] == [f[0] for f in gck.Layout._fields_][:len(gc_c.Layout._fields_)]
