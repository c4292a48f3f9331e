"""libgck.so as a gc-c pack: the ``.gcpack`` container the engine's loader stages, verifies and opens
(``goethe_engine/pack.py`` ``stage`` / ``open_branch``, ``goethe_engine/gc_c.py`` ``GcBackend``).

The engine never loads a library from a path: it reads a signed container, checks the manifest's schema, picks a
variant by the weights' structure and a bucket by device and numerics, extracts the bucket's files by their sha256 and
binds the library from that copy. ``build`` writes such a container around this library and the manifest that
``synth.pack_dir`` (or the caller) wrote for the library's own ``gc_open``:

* container framing (the reader is ``pack.py`` ``read_container_v``): the 8 magic bytes ``GCPACK3\\n``, the header
  length as a little-endian u64, a JSON header ``{"manifest": [offset, length], "blobs": {sha256: [offset, length]}}``
  with offsets counted from the end of the header, then the manifest bytes and each blob;
* the manifest is the pack directory's, completed with what the engine's schema check requires (``pack.py``
  ``validate``): ``compiler``, ``hw`` (one record hash per sku), every bucket's ``files`` (``libgck.so`` by its sha256)
  and ``variants`` (variant ``v``: the weights' structure record, which the caller makes with the engine's
  ``structure.describe``, so the engine's own check is what decides that the weights fit).

Signing stays with the engine's tools: ``pack.sign_pack(path, private_key)`` writes ``PATH.sig`` over the manifest.
"""
import hashlib
import json
import os

MAGIC = b"GCPACK3\n"
LIB_NAME = "libgck.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)


def manifest(pack_dir, lib_sha256, structure, weights=None, commit="0" * 40, drafter_structure=None):
    """The engine-facing manifest (a dict) of a pack directory's manifest.json: every bucket runs the library whose
    sha256 is lib_sha256; variant "v" (the target buckets) has the given structure record and, for a pack with
    drafter buckets (a speculative pair, pack.py:130-141), variant "dv" the drafter weights' structure; weights:
    [{file, bytes, sha256}] records of the model's files, the target's first and the drafter's second (default: the
    directory's list, names only)."""
    with open(os.path.join(pack_dir, "manifest.json")) as f:
        m = json.load(f)
    skus = sorted({b["sku"] for b in m["buckets"]})
    m["compiler"] = dict(commit=commit, dirty=False)
    m["hw"] = {s: hashlib.sha256(f"{s}:sm_100a:148".encode()).hexdigest() for s in skus}
    for b in m["buckets"]:
        b["files"] = {LIB_NAME: lib_sha256}
        b["lib"] = LIB_NAME
        b["variant"] = "v" if b.get("role", "target") == "target" else "dv"
        b.setdefault("variants", [])
        b.setdefault("variant_of", None)
    if weights is not None:
        m["model"]["weights"] = weights
    m["variants"] = {"v": dict(structure=structure, weights=[0])}
    if any(b["variant"] == "dv" for b in m["buckets"]):
        if drafter_structure is None:
            raise ValueError("a pack with drafter buckets needs the drafter weights' structure")
        m["variants"]["dv"] = dict(structure=drafter_structure, weights=[1])
    m.pop("synth", None)
    return m


def write(path, m, blobs):
    """Write the container: manifest m (a dict) and blobs {sha256: bytes}."""
    mb = (json.dumps(m, indent=1, sort_keys=True) + "\n").encode()
    hdr, off, parts = {"manifest": [0, len(mb)], "blobs": {}}, len(mb), [mb]
    for h, data in blobs.items():
        hdr["blobs"][h] = [off, len(data)]
        off += len(data)
        parts.append(data)
    hb = json.dumps(hdr).encode()
    with open(path + ".tmp", "wb") as f:
        f.write(MAGIC + len(hb).to_bytes(8, "little") + hb)
        for p in parts:
            f.write(p)
    os.replace(path + ".tmp", path)
    return path


def build(out, pack_dir, structure, lib=LIB_PATH, weights=None, drafter_structure=None):
    """out: a .gcpack of the library at lib (default: this package's build) under the manifest of pack_dir; returns
    out. Sign it with the engine's pack.sign_pack before GcBackend opens it (or use the engine's development switch
    for unsigned packs)."""
    with open(lib, "rb") as f:
        data = f.read()
    h = hashlib.sha256(data).hexdigest()
    return write(out, manifest(pack_dir, h, structure, weights, drafter_structure=drafter_structure), {h: data})
