"""Host-side binding of libgck.so through its C ABI (ctypes), mirroring the engine's own backend interface.

The reference engine binds a pack runtime with ``goethe_engine/gc_c.py`` (``bind`` at gc_c.py:58-77, the struct
mirrors at gc_c.py:27-55, ``GcBackend.step/commit/copy_blocks/release`` at gc_c.py:262-316). This module is this
project's own binding of the same ABI so that tests, the benchmark and users without the engine can drive the
library the way the engine does: ``Backend.step(work)`` takes ``Work`` items (``goethe_engine/backend.py:19-29``) and
returns per-item token lists (device argmax, all items greedy) or float32 logits ``[sum(want), vocab]``.

Nothing here computes: every step runs in libgck.so on the GPU. A missing library or a machine without the device
fails loudly (``GcError``); there is no fallback.
"""
import array
import operator
import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

ABI_MAJOR, ABI_MINOR = 1, 2
OK, E_ARG, E_MANIFEST, E_WEIGHTS, E_DEVICE, E_UNSUPPORTED, E_STATE, E_CAPACITY = 0, -1, -2, -3, -4, -5, -6, -7
W_GREEDY, W_SPEC, W_FEATS = 1, 2, 4
S_HOST_LOGITS = 1
L_PAGED, L_DEVICE_ARGMAX, L_SPEC = 1, 2, 4
OPEN_SPEC, OPEN_NO_CHECK = 1, 2
KV_DTYPE = {0: "f16", 1: "fp8"}
P_ = C.POINTER
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libgck.so")
# every symbol include/gc.h declares
SYMBOLS = ("gc_abi_version", "gc_open", "gc_layout_get", "gc_step", "gc_commit", "gc_copy_blocks", "gc_state_save",
           "gc_state_restore", "gc_release", "gc_last_error", "gc_close", "gc_probe", "gc_price")


class GcError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"gc call failed ({code}): {msg}")
        self.code = code


class OpenParams(C.Structure):
    _fields_ = [("size", C.c_uint32), ("flags", C.c_uint32), ("pack_dir", C.c_char_p), ("weights", P_(C.c_char_p)),
                ("n_weights", C.c_uint32), ("device", C.c_int32), ("buckets", P_(C.c_char_p)),
                ("n_buckets", C.c_uint32), ("pool_blocks", C.c_uint32), ("spec_policy", C.c_char_p),
                ("scratch_dir", C.c_char_p), ("state_pages", C.c_uint32)]


class Layout(C.Structure):
    _fields_ = [("size", C.c_uint32)] + [(k, C.c_uint32) for k in (
        "flags", "vocab", "max_cols", "max_seqs", "max_ctx", "block_size", "num_blocks", "layers", "kv_heads",
        "head_dim", "kv_dtype", "spec_width", "feat_width")] + [(k, C.c_uint64) for k in (
        "kv_bytes", "state_bytes", "device_bytes")] + [(k, C.c_uint32) for k in (
        "state_pages", "pad1", "embd_dim", "embd_pool", "enc_frames", "enc_feat")]


class WorkS(C.Structure):
    _fields_ = [("size", C.c_uint32), ("flags", C.c_uint32), ("sid", C.c_uint64), ("pos", C.c_uint32),
                ("n_tokens", C.c_uint32), ("tokens", P_(C.c_int32)), ("parents", P_(C.c_int32)),
                ("blocks", P_(C.c_uint32)), ("n_blocks", C.c_uint32), ("want", C.c_uint32)]


# the same record as a numpy dtype (gc.h gc_work: natural alignment, 56 bytes): a step's records are filled in one array
WORK_DTYPE = np.dtype([("size", "<u4"), ("flags", "<u4"), ("sid", "<u8"), ("pos", "<u4"), ("n_tokens", "<u4"),
                       ("tokens", "<u8"), ("parents", "<u8"), ("blocks", "<u8"), ("n_blocks", "<u4"), ("want", "<u4")])
assert WORK_DTYPE.itemsize == C.sizeof(WorkS) and all(
    WORK_DTYPE.fields[n][1] == getattr(WorkS, n).offset for n, _ in WorkS._fields_)


def _addr(a):
    return a.ctypes.data


_FIELDS = operator.attrgetter("sid", "pos", "want", "greedy", "spec", "feats", "parents", "tokens", "blocks")


def _flat(work, field, code, dtype):
    """Every item's `field` (a sequence of ints) in one contiguous array. array.array converts Python ints at C speed
    (about half the time of numpy.fromiter, a third of a conversion per item); out-of-range values raise."""
    a = array.array(code)
    for w in work:
        a.extend(getattr(w, field))
    return np.frombuffer(a, dtype) if len(a) else np.zeros(0, dtype)


def _u32(x):
    # block tables: a contiguous uint32 array passes through; anything else is converted
    if isinstance(x, np.ndarray) and x.dtype == np.uint32 and x.flags.c_contiguous:
        return x
    return np.ascontiguousarray(x, np.uint32)


class StepIn(C.Structure):
    _fields_ = [("size", C.c_uint32), ("flags", C.c_uint32), ("work", P_(P_(WorkS))), ("n_work", C.c_uint32),
                ("pad", C.c_uint32)]


class StepOut(C.Structure):
    _fields_ = [("size", C.c_uint32), ("n_rows", C.c_uint32), ("tokens", P_(C.c_int32)), ("tokens_cap", C.c_uint32),
                ("pad0", C.c_uint32), ("counts", P_(C.c_uint32)), ("logits", C.c_void_p), ("logits_cap", C.c_uint64),
                ("logits_dev", C.c_uint64), ("feats", C.c_void_p), ("feats_cap", C.c_uint64)]


@dataclass
class Work:
    """One sequence's tokens for a step (goethe_engine/backend.py:19-29)."""
    sid: int
    tokens: list
    pos: int
    blocks: list
    want: int
    greedy: bool = False
    spec: bool = False
    parents: list = None
    feats: bool = False


def load(path=LIB_PATH):
    """ctypes handle of libgck.so with argument and result types set for every gc.h entry point. Raises GcError when
    the file is missing or when gc_abi_version reports a major other than 1 or a minor below the one this binding
    was written for."""
    if not os.path.exists(path):
        raise GcError(E_DEVICE, f"{path} is not built (python -m goethe_engine_b200.build)")
    L = C.CDLL(path)
    sig = dict(gc_abi_version=(C.c_uint32, []), gc_open=(C.c_int, [P_(OpenParams), P_(C.c_void_p)]),
               gc_layout_get=(C.c_int, [C.c_void_p, P_(Layout)]),
               gc_step=(C.c_int, [C.c_void_p, P_(StepIn), P_(StepOut)]),
               gc_commit=(C.c_int, [C.c_void_p, C.c_uint64, C.c_uint32, P_(C.c_uint32), C.c_uint32]),
               gc_copy_blocks=(C.c_int, [C.c_void_p, P_(C.c_uint32), P_(C.c_uint32), C.c_uint32]),
               gc_state_save=(C.c_int, [C.c_void_p, C.c_uint64, C.c_uint32]),
               gc_state_restore=(C.c_int, [C.c_void_p, C.c_uint32, C.c_uint64]),
               gc_release=(C.c_int, [C.c_void_p, C.c_uint64]), gc_last_error=(C.c_char_p, [C.c_void_p]),
               gc_close=(None, [C.c_void_p]))
    for n, (res, args) in sig.items():
        f = getattr(L, n)
        f.restype, f.argtypes = res, args
    v = L.gc_abi_version()
    if v >> 16 != ABI_MAJOR or (v & 0xFFFF) < ABI_MINOR:
        raise GcError(E_ARG, f"{path}: C ABI {v >> 16}.{v & 0xFFFF}, need {ABI_MAJOR}.{ABI_MINOR}+")
    return L


def arr(ctype, xs):
    return (ctype * len(xs))(*xs)


class Backend:
    """One gc_open handle: the engine-facing step / commit / copy_blocks / release of gc_c.GcBackend."""

    def __init__(self, pack_dir, weights, buckets=("b200.BI.main",), pool_blocks=0, device=-1, lib=None,
                 drafter_weights=None, policy=None):
        """drafter_weights: a speculative pair (GC_OPEN_SPEC, gc_c.py:142-191): buckets are {target, drafter} and the
        weight list is the target's files, a NULL, then the drafter's; policy "ar:K" or None for the pack's own."""
        self.L = lib or load()
        self.h = None
        ws = [weights] if isinstance(weights, str) else list(weights)
        spec = drafter_weights is not None
        if spec:
            ws += [None] + ([drafter_weights] if isinstance(drafter_weights, str) else list(drafter_weights))
        keep = [arr(C.c_char_p, [None if w is None else os.fsencode(w) for w in ws]),
                arr(C.c_char_p, [b.encode() for b in buckets])]
        p = OpenParams(C.sizeof(OpenParams), OPEN_NO_CHECK | (OPEN_SPEC if spec else 0), os.fsencode(pack_dir), keep[0],
                       len(ws), device, keep[1], len(buckets), pool_blocks, policy.encode() if policy else None, None, 0)
        h = C.c_void_p()
        rc = self.L.gc_open(C.byref(p), C.byref(h))
        if rc:
            raise GcError(rc, (self.L.gc_last_error(None) or b"").decode())
        self.h = h.value
        lo = Layout(size=C.sizeof(Layout))
        self._ck(self.L.gc_layout_get(self.h, C.byref(lo)))
        self.layout = lo
        self.vocab_size, self.max_seqs, self.max_len = lo.vocab, lo.max_seqs, lo.max_ctx
        self.block_size, self.num_blocks = lo.block_size, lo.num_blocks
        self.kv_dtype = KV_DTYPE.get(lo.kv_dtype, "f16")
        self.device_argmax = bool(lo.flags & L_DEVICE_ARGMAX)
        self.spec_width = lo.spec_width if lo.flags & L_SPEC else 0

    def _ck(self, rc):
        if rc < 0:
            raise GcError(rc, (self.L.gc_last_error(self.h) or b"").decode())

    def step(self, work, logits=None):
        """Tokens per item (every item greedy) or float32 logits [sum(want), vocab] (into `logits` if given)."""
        n = len(work)
        # one pass over the items collects every per-item field; then every item's tokens go into one int32 array, the
        # block tables into one uint32 array, the records into one structured array (a column at a time) and their
        # addresses into another: a handful of numpy calls per step
        sid, pos, want_, gr, sp, ft, par, tk, bl = zip(*map(_FIELDS, work)) if n else ((),) * 9
        greedy = self.device_argmax and all(gr)
        spec_any, tree_any = any(sp), any(p is not None for p in par)
        tables_np = all(type(b) is np.ndarray and b.dtype == np.uint32 for b in bl)
        c = np.empty((n, 6), np.int64)
        c[:, 0], c[:, 1], c[:, 2] = sid, pos, want_
        c[:, 3] = list(map(len, tk))
        c[:, 4] = list(map(len, bl))
        c[:, 5] = np.array(sp, np.int64) * 2 + np.array(ft, np.int64) * 4
        ntok, nblk = c[:, 3], c[:, 4]
        toks = _flat(work, "tokens", "i", np.int32)
        if n and tables_np:
            ball = np.concatenate(bl)
        else:
            ball = _flat(work, "blocks", "I", np.uint32)
        rec = np.zeros(n, WORK_DTYPE)
        keep = [toks, rec, ball]
        rec["size"] = WORK_DTYPE.itemsize
        rec["flags"] = c[:, 5] | (1 if greedy else 0)
        rec["sid"] = c[:, 0]
        rec["pos"] = c[:, 1]
        rec["want"] = c[:, 2]
        rec["n_tokens"] = ntok
        rec["tokens"] = _addr(toks) + 4 * (np.cumsum(ntok) - ntok).astype(np.uint64)
        rec["blocks"] = _addr(ball) + 4 * (np.cumsum(nblk) - nblk).astype(np.uint64)
        rec["n_blocks"] = nblk
        if tree_any:
            for i, w in enumerate(work):
                if w.parents is not None:
                    par = np.ascontiguousarray(w.parents, np.int32)
                    keep.append(par)
                    rec["parents"][i] = _addr(par)
        ptrs = _addr(rec) + WORK_DTYPE.itemsize * np.arange(n, dtype=np.uint64)
        pw = C.cast(C.c_void_p(_addr(ptrs)), P_(P_(WorkS)))
        want = c[:, 2]
        rows = int(want.sum())
        out = StepOut(size=C.sizeof(StepOut))
        counts = np.zeros(n, np.uint32)
        if greedy:
            # a speculative round returns up to spec_width tokens for its one wanted row
            cap = int(np.maximum(want, np.where(c[:, 5] & 2, self.spec_width, 0)).sum()) if spec_any else rows
            tok = np.empty(max(cap, 1), np.int32)
            out.tokens = tok.ctypes.data_as(P_(C.c_int32))
            out.tokens_cap = cap
            out.counts = counts.ctypes.data_as(P_(C.c_uint32))
        else:
            lg = logits if logits is not None else np.empty((rows, self.vocab_size), np.float32)
            out.logits, out.logits_cap = lg.ctypes.data, lg.size
        self._ck(self.L.gc_step(self.h, C.byref(StepIn(C.sizeof(StepIn), 0 if greedy else S_HOST_LOGITS, pw, n, 0)),
                                C.byref(out)))
        del keep, ptrs
        if greedy:
            if not spec_any and rows == n and bool((counts == 1).all()):
                return tok[:n, None].tolist()          # one token per item: the common decode step
            ends = np.cumsum(counts)
            flat = tok.tolist()
            return [flat[e - k:e] for e, k in zip(ends.tolist(), counts.tolist())]
        return lg[:out.n_rows]

    def decode(self, sids, tokens, pos, blocks, greedy=True, logits=None):
        """One decode step of n sequences given as columns: sids [n] ids, tokens [n] (one token each), pos [n] (the
        token's row), blocks: n uint32 block tables. The same gc_step call as step() with n one-token items, want 1,
        built from the columns without a Python object per item. Returns the next token of each sequence (int32 [n],
        every item greedy with the device argmax) or float32 logits [n, vocab]."""
        n = len(sids)
        greedy = greedy and self.device_argmax
        toks = np.ascontiguousarray(tokens, np.int32)
        nblk = np.fromiter(map(len, blocks), np.int64, n)
        ball = np.concatenate([_u32(b) for b in blocks]) if n else np.zeros(0, np.uint32)
        rec = np.zeros(n, WORK_DTYPE)
        rec["size"] = WORK_DTYPE.itemsize
        rec["flags"] = 1 if greedy else 0
        rec["sid"] = sids
        rec["pos"] = pos
        rec["want"] = 1
        rec["n_tokens"] = 1
        rec["tokens"] = _addr(toks) + 4 * np.arange(n, dtype=np.uint64)
        rec["blocks"] = _addr(ball) + 4 * (np.cumsum(nblk) - nblk).astype(np.uint64)
        rec["n_blocks"] = nblk
        ptrs = _addr(rec) + WORK_DTYPE.itemsize * np.arange(n, dtype=np.uint64)
        pw = C.cast(C.c_void_p(_addr(ptrs)), P_(P_(WorkS)))
        out = StepOut(size=C.sizeof(StepOut))
        counts = np.zeros(n, np.uint32)
        if greedy:
            tok = np.empty(max(n, 1), np.int32)
            out.tokens = tok.ctypes.data_as(P_(C.c_int32))
            out.tokens_cap = n
            out.counts = counts.ctypes.data_as(P_(C.c_uint32))
        else:
            lg = logits if logits is not None else np.empty((n, self.vocab_size), np.float32)
            out.logits, out.logits_cap = lg.ctypes.data, lg.size
        self._ck(self.L.gc_step(self.h, C.byref(StepIn(C.sizeof(StepIn), 0 if greedy else S_HOST_LOGITS, pw, n, 0)),
                                C.byref(out)))
        del toks, ball, rec, ptrs
        return tok[:n] if greedy else lg[:out.n_rows]

    def commit(self, sid, base, path):
        self._ck(self.L.gc_commit(self.h, sid, base, arr(C.c_uint32, path), len(path)))

    def copy_blocks(self, pairs):
        self._ck(self.L.gc_copy_blocks(self.h, arr(C.c_uint32, [s for s, _ in pairs]),
                                       arr(C.c_uint32, [d for _, d in pairs]), len(pairs)))

    def release(self, sid):
        self._ck(self.L.gc_release(self.h, sid))

    def close(self):
        if self.h:
            self.L.gc_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    __del__ = close
