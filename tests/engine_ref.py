"""The reference engine as this library's caller, for the drop-in tests: where its package is found, a throwaway
signing key, and a signed .gcpack around libgck.so that the engine's own loader opens.

The engine package comes from ``baseline/_ref`` (the reference installed offline into the repository's working
tree, which travels to the GPU box), else from the reference's mounted source tree (this build container only).
Nothing here is imported by the library."""
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PLACES = (os.path.join(ROOT, "baseline", "_ref"), "/root/reference")


def engine_path():
    """The directory that holds the engine's goethe_engine package, or None."""
    for p in PLACES:
        if os.path.isfile(os.path.join(p, "goethe_engine", "gc_c.py")):
            return p
    return None


def engine():
    """The engine package (goethe_engine) imported from engine_path()."""
    p = engine_path()
    if p is None:
        return None
    if p not in sys.path:
        sys.path.insert(0, p)
    import goethe_engine
    return goethe_engine


class Key:
    """A P-256 key pair made with the openssl command line in dir (test only), and the engine's key id of it."""

    def __init__(self, d):
        from goethe_engine import sign
        self.priv, self.pub = os.path.join(d, "test_key.pem"), os.path.join(d, "test_key_pub.pem")
        subprocess.run(["openssl", "ecparam", "-name", "prime256v1", "-genkey", "-noout", "-out", self.priv],
                       check=True, capture_output=True)
        subprocess.run(["openssl", "ec", "-in", self.priv, "-pubout", "-out", self.pub], check=True, capture_output=True)
        with open(self.pub, "rb") as f:
            self.kid = sign.key_id(f.read())


def signed_pack(d, pack_dir, weights, key, drafter_weights=None):
    """d/model.gcpack: libgck.so under pack_dir's manifest, the variants' structures (the target's and, for a
    speculative pair, the drafter's) from the engine's own structure.describe over the weights, signed with key by the
    engine's pack.sign_pack. Returns the pack path."""
    from goethe_engine import pack as P, structure
    from goethe_engine_b200 import gcpack
    out = os.path.join(d, "model.gcpack")
    st = structure.describe(list(weights), ["general.architecture"])
    dst = structure.describe(list(drafter_weights), ["general.architecture"]) if drafter_weights else None
    ws = [dict(file=os.path.basename(w), bytes=os.path.getsize(w)) for w in list(weights) + list(drafter_weights or [])]
    gcpack.build(out, pack_dir, st, weights=ws, drafter_structure=dst)
    P.sign_pack(out, key.priv)
    return out
