"""CPU restatement (numpy, float32) of the reference decoder forward and its paged backend (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this module; it is the checker,
never the thing measured or shipped.

What it follows, line by line:

* ``rms`` — ``goethe_engine/ref.py:14-15``: ``x * rsqrt(mean(x^2) + eps)``. The reference hard-codes eps 1e-6 and
  no gain; here eps and the gain vectors are parameters (the GGUF ``layer_norm_rms_epsilon`` and ``*_norm.weight``),
  and eps 1e-6 with unit gains is exactly ``ref.py``.
* ``RefModel._rope`` / ``inv`` — ``ref.py:31-37``: interleaved pairs ``(x[2i], x[2i+1])`` rotated by ``p * theta^(-2i/dh)``.
* ``RefModel.token`` — ``ref.py:39-62``: per layer ``h = rms(x)``; q, k, v; RoPE at the token's position; the KV
  row write cast to the cache dtype (``ref.py:54``); GQA softmax attention over the visible rows (``ref.py:55-57``);
  ``x += Wo attn``; ``h = rms(x)``; ``x += Wdn (silu(Wg h) * (Wu h))``; logits ``head @ rms(x)``.
* ``TorchBackend`` — ``ref.py:90-126``: slot ``blocks[p // bs] * bs + p % bs``; token j writes slot ``pos + j`` at
  RoPE position ``pos + depth(j)`` and attends to ``slots[:pos]`` then ``slots[pos + path(j)]``; logits of the last
  ``want`` tokens; ``commit`` moves row ``base + path[j]`` to ``base + j`` (all layers, K and V); ``copy_blocks``
  copies whole blocks.
* ``depths`` / ``path`` — ``goethe_engine/spec.py:70-85``.

Tokens of one work item are run layer by layer for all its tokens at once. That is the same computation as the
reference's token-at-a-time loop: a token's attention at layer l reads only rows of the cached prefix and of its
own ancestors, and every such row is written (at layer l) before any attention of that layer runs. A chain item (no
parents) takes its attention in chunks of tokens with a causal mask (each chunk decodes its visible rows once), so
that the oracle can prefill contexts of thousands of rows at the benchmark's model widths; tree items attend token
by token over their paths. Either way every token sees exactly the rows ``TorchBackend.step`` gives it.

fp8 KV: ``kv_scale="unit"`` is the reference's plain e4m3 cast; ``kv_scale="page"`` is the library's per-page
power-of-two scale (``page_scale_exp``): a page's scale is fixed by its first row, later rows are clamped to it.

a8 activations (``act="a8"``; the pack's bucket field ``act``, ``goethe_engine/pack.py:647-663`` ``wanted``): the
reference states a8 as a numerics choice and carries no arithmetic for it (``ref.py`` computes in float32). Here it
is the input of every linear product (q, k, v and gate, up from the RMSNorm output; o from the attention output; down
from the SwiGLU output; the head from the final RMSNorm output) quantized per token row to symmetric int8: scale
``s = amax / 127`` of the row (1 for an all-zero row), codes ``rint(x / s)`` (ties to even), and the product
``(codes @ W.T) * s`` in float32 (``a8_quant``, ``PagedOracle._lin``).
"""
import math

import numpy as np

from . import quants as Q

PAGE_TARGET = 64.0      # the first row's amax is scaled to at most this (448 / 64 = 7x headroom for later rows)
PAGE_EXP_MIN, PAGE_EXP_MAX = -8, 15


def depths(parents, n):
    """Depth of each of n tokens: 0 for parent -1, else depth(parent) + 1; a chain (None) has depth i."""
    if parents is None:
        return list(range(n))
    d = []
    for p in parents:
        d.append(0 if p < 0 else d[p] + 1)
    return d


def path(parents, i):
    """Token indices from the root to i inclusive."""
    if parents is None:
        return list(range(i + 1))
    out = [i]
    while parents[out[-1]] >= 0:
        out.append(parents[out[-1]])
    return out[::-1]


def a8_quant(x):
    """(codes, scales) of the rows of x [n, k] float32: per row s = amax / 127 (1 where the row is all zero) and codes
    rint(x / s) as float32 integers in [-127, 127]."""
    am = np.abs(x).max(-1).astype(np.float32)
    s = np.where(am > 0, am / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    return np.rint(x / s[:, None]).astype(np.float32), s


def rms(x, gain, eps):
    x = np.asarray(x, np.float32)
    r = (1.0 / np.sqrt((x * x).mean(-1, keepdims=True, dtype=np.float32) + np.float32(eps))).astype(np.float32)
    return (x * r * gain).astype(np.float32)


def page_scale_exps(row_amax):
    """page_scale_exp of every element of an array of amax values (float32), without a Python loop."""
    a = np.asarray(row_amax, np.float32)
    ok = (a > 0) & np.isfinite(a)
    m, k = np.frexp(np.where(ok, a, np.float32(1.0)))
    e = 6 - k + (m == 0.5).astype(np.int32)
    return np.where(ok, np.clip(e, PAGE_EXP_MIN, PAGE_EXP_MAX), 0).astype(np.int32)


def page_scale_exp(row_amax):
    """The exponent e of a page's scale 2^e, from the amax of the page's first row (over one layer, head, K or V):
    the largest e with amax * 2^e <= PAGE_TARGET, clamped to [-8, 15]. A stored value is code(x * 2^e)."""
    if not row_amax > 0 or not math.isfinite(row_amax):
        return 0
    m, k = math.frexp(row_amax)            # amax = m * 2^k, m in [0.5, 1): exact, no log rounding
    e = 6 - k + (1 if m == 0.5 else 0)     # PAGE_TARGET = 2^6
    return int(min(max(e, PAGE_EXP_MIN), PAGE_EXP_MAX))


class Weights:
    """Float32 decoder weights in the reference's layout: ``[out, in]`` row-major (``ref.py:25-27``)."""

    def __init__(self, emb, head, layers, out_norm=None, eps=1e-6, theta=1e4, heads=None, kv_heads=None):
        self.emb, self.head, self.layers = emb, head, layers
        self.V, self.d = emb.shape
        self.L = len(layers)
        self.H, self.KVH = heads, kv_heads
        self.dh = self.d // heads
        self.F = layers[0]["g"].shape[0]
        self.eps, self.theta = float(eps), float(theta)
        one = np.ones(self.d, np.float32)
        self.out_norm = one if out_norm is None else out_norm
        for lw in layers:
            lw.setdefault("attn_norm", one)
            lw.setdefault("ffn_norm", one)
        # ref.py:31 computes inv in float32: 10000 ** (-arange(0, dh, 2).float() / dh)
        self.inv = (np.float32(self.theta) ** (-(np.arange(0, self.dh, 2, dtype=np.float32) / np.float32(self.dh)))).astype(np.float32)

    def rope(self, x, p):
        """x [..., dh] rotated at position p (interleaved pairs, ref.py:33-37)."""
        a = (self.inv * np.float32(p)).astype(np.float32)
        c, s = np.cos(a).astype(np.float32), np.sin(a).astype(np.float32)
        x1, x2 = x[..., ::2], x[..., 1::2]
        return np.stack([x1 * c - x2 * s, x1 * s + x2 * c], -1).reshape(x.shape).astype(np.float32)

    def rope_rows(self, x, ps):
        """x [n, heads, dh], row i rotated at position ps[i]: the same float32 operations as rope() row by row."""
        a = (self.inv[None, :] * np.asarray(ps, np.float32)[:, None]).astype(np.float32)
        c, s = np.cos(a).astype(np.float32)[:, None, :], np.sin(a).astype(np.float32)[:, None, :]
        x1, x2 = x[..., ::2], x[..., 1::2]
        return np.stack([x1 * c - x2 * s, x1 * s + x2 * c], -1).reshape(x.shape).astype(np.float32)


class PagedOracle:
    """The reference's TorchBackend semantics over numpy: a KV pool of num_blocks * block_size rows."""

    def __init__(self, w, num_blocks, block_size=16, kv="f16", kv_scale="unit", act="a16"):
        assert act in ("a16", "a8"), act
        self.w, self.bs, self.nb, self.kv, self.kv_scale, self.act = w, block_size, num_blocks, kv, kv_scale, act
        rows = num_blocks * block_size
        shape = (w.L, rows, w.KVH, w.dh)
        if kv == "f16":
            self.kc, self.vc = np.zeros(shape, np.float16), np.zeros(shape, np.float16)
        else:
            self.kc, self.vc = np.zeros(shape, np.uint8), np.zeros(shape, np.uint8)
            # per-page exponents [L, blocks, KVH] for K and V
            self.ke = np.zeros((w.L, num_blocks, w.KVH), np.int32)
            self.ve = np.zeros((w.L, num_blocks, w.KVH), np.int32)
        self.blk, self.nodes = {}, {}

    # -- KV storage --------------------------------------------------------------------------------------------------
    def _write(self, l, slot, k, v, first_row_k=None, first_row_v=None):
        """Row `slot` of layer l gets k, v [KVH, dh] (float32). fp8 page mode: the page exponent is set when the row
        is the page's first (slot % bs == 0), else the page's stored exponent applies."""
        if self.kv == "f16":
            self.kc[l, slot], self.vc[l, slot] = k.astype(np.float16), v.astype(np.float16)
            return
        b = slot // self.bs
        if self.kv_scale == "page":
            if slot % self.bs == 0:
                for h in range(self.w.KVH):
                    self.ke[l, b, h] = page_scale_exp(float(np.abs(k[h]).max()))
                    self.ve[l, b, h] = page_scale_exp(float(np.abs(v[h]).max()))
            sk = np.float32(2.0) ** self.ke[l, b].astype(np.float32)
            sv = np.float32(2.0) ** self.ve[l, b].astype(np.float32)
            self.kc[l, slot] = Q.e4m3_encode(k * sk[:, None])
            self.vc[l, slot] = Q.e4m3_encode(v * sv[:, None])
        else:
            self.kc[l, slot], self.vc[l, slot] = Q.e4m3_encode(k), Q.e4m3_encode(v)

    def _write_rows(self, l, slots, k, v):
        """Rows slots[i] of layer l get k[i], v[i] ([n, KVH, dh] float32): the same result as _write row by row in this
        order. A page's first row among them sets the page's exponents before any row is encoded, and it comes
        before the page's other rows (a page's rows are consecutive positions), so every row sees the exponent the
        sequential order would give it."""
        slots = np.asarray(slots, np.int64)
        if self.kv == "f16":
            self.kc[l, slots], self.vc[l, slots] = k.astype(np.float16), v.astype(np.float16)
            return
        if self.kv_scale != "page":
            self.kc[l, slots], self.vc[l, slots] = Q.e4m3_encode(k), Q.e4m3_encode(v)
            return
        b = slots // self.bs
        first = slots % self.bs == 0
        if first.any():
            self.ke[l, b[first]] = page_scale_exps(np.abs(k[first]).max(-1))
            self.ve[l, b[first]] = page_scale_exps(np.abs(v[first]).max(-1))
        sk = np.float32(2.0) ** self.ke[l, b].astype(np.float32)
        sv = np.float32(2.0) ** self.ve[l, b].astype(np.float32)
        self.kc[l, slots] = Q.e4m3_encode(k * sk[:, :, None])
        self.vc[l, slots] = Q.e4m3_encode(v * sv[:, :, None])

    def _lin(self, x, W):
        """x @ W.T, with x quantized per row first for a8 (a8_quant), the row's scale applied to its products."""
        if self.act == "a16":
            return x @ W.T
        q, sc = a8_quant(x)
        return ((q @ W.T) * sc[:, None]).astype(np.float32)

    CHUNK = 512

    def _attend_chain(self, l, q, sl, pos):
        """Attention of a chain item's n tokens (q [n, H, dh], rotated): token j sees slots sl[:pos + j + 1]
        (ref.py:101-104 with path(None, j) = 0..j), taken CHUNK tokens at a time with a causal mask."""
        w, n = self.w, q.shape[0]
        G = w.H // w.KVH
        att = np.empty((n, w.H * w.dh), np.float32)
        scale = np.float32(math.sqrt(w.dh))
        for j0 in range(0, n, self.CHUNK):
            j1 = min(n, j0 + self.CHUNK)
            c, t = j1 - j0, pos + j1
            K, V = self._read(l, sl[:t])
            lim = np.repeat(pos + np.arange(j0, j1) + 1, G)            # visible rows of each (token, head in group)
            masked = np.arange(t)[None, :] >= lim[:, None]
            qc = q[j0:j1].reshape(c, w.KVH, G, w.dh)
            for h in range(w.KVH):
                sc = (qc[:, h].reshape(c * G, w.dh) @ K[:, h].T) / scale
                sc[masked] = -np.inf
                sc = sc - sc.max(-1, keepdims=True)
                p = np.exp(sc)
                p = p / p.sum(-1, keepdims=True)
                att[j0:j1, h * G * w.dh:(h + 1) * G * w.dh] = (p @ V[:, h]).reshape(c, G * w.dh)
        return att

    def _read(self, l, slots):
        """(K, V) float32 [n, KVH, dh] of the given rows of layer l."""
        if self.kv == "f16":
            return self.kc[l, slots].astype(np.float32), self.vc[l, slots].astype(np.float32)
        K, V = Q.e4m3_decode(self.kc[l, slots]), Q.e4m3_decode(self.vc[l, slots])
        if self.kv_scale == "page":
            b = np.asarray(slots) // self.bs
            K = K * (np.float32(2.0) ** (-self.ke[l, b].astype(np.float32)))[:, :, None]
            V = V * (np.float32(2.0) ** (-self.ve[l, b].astype(np.float32)))[:, :, None]
        return K.astype(np.float32), V.astype(np.float32)

    def slots(self, blocks):
        bs = self.bs
        return (np.asarray(blocks, np.int64)[:, None] * bs + np.arange(bs)).reshape(-1)

    # -- the step ----------------------------------------------------------------------------------------------------
    def step(self, work):
        """work: dicts (sid, tokens, pos, blocks, want, parents=None). Returns float32 logits [sum(want), V] in work
        order (TorchBackend.step, ref.py:94-112).

        The step runs layer by layer over every token of every item at once (one product per weight per layer);
        attention is per item. The reference runs items one after another, token by token: the results are the same
        because a row's arithmetic involves only its own token and the KV rows it sees, and a valid step never lets
        an item see rows another item of the same step writes (each item writes rows of its own pages; shared
        prefix pages were written by earlier steps). Every row of layer l is written before any attention of
        layer l runs, which the token-by-token order also guarantees for the rows a token sees."""
        w = self.w
        its, offs, T = [], [], 0
        for it in work:
            toks, par = list(it["tokens"]), it.get("parents")
            n = len(toks)
            its.append(dict(toks=toks, pos=int(it["pos"]), want=int(it["want"]), par=par, n=n,
                            sl=self.slots(it["blocks"]), dep=depths(par, n)))
            offs.append(T)
            T += n
        if T == 0:
            return np.zeros((0, w.V), np.float32)
        x = w.emb[np.concatenate([np.asarray(i["toks"], np.int64) for i in its])].astype(np.float32)
        ps = np.concatenate([i["pos"] + np.asarray(i["dep"]) for i in its])
        G = w.H // w.KVH
        for l, lw in enumerate(w.layers):
            h = rms(x, lw["attn_norm"], w.eps)
            q = w.rope_rows(self._lin(h, lw["q"]).reshape(T, w.H, w.dh), ps)
            k = w.rope_rows(self._lin(h, lw["k"]).reshape(T, w.KVH, w.dh), ps)
            v = self._lin(h, lw["v"]).reshape(T, w.KVH, w.dh)
            for i, o in zip(its, offs):
                self._write_rows(l, i["sl"][i["pos"]:i["pos"] + i["n"]], k[o:o + i["n"]], v[o:o + i["n"]])
            att = np.empty((T, w.H * w.dh), np.float32)
            for i, o in zip(its, offs):
                n, pos, sl, par = i["n"], i["pos"], i["sl"], i["par"]
                if par is None:
                    att[o:o + n] = self._attend_chain(l, q[o:o + n], sl, pos)
                    continue
                for j in range(n):
                    vis = np.concatenate([sl[:pos], sl[pos + np.asarray(path(par, j))]])
                    K, V = self._read(l, vis)
                    qj = q[o + j].reshape(w.KVH, G, w.dh)
                    sc = np.einsum("kgd,tkd->kgt", qj, K) / np.float32(math.sqrt(w.dh))
                    sc = sc - sc.max(-1, keepdims=True)
                    p = np.exp(sc)
                    p = p / p.sum(-1, keepdims=True)
                    att[o + j] = np.einsum("kgt,tkd->kgd", p, V).reshape(-1)
            x = x + self._lin(att, lw["o"])
            h = rms(x, lw["ffn_norm"], w.eps)
            g = self._lin(h, lw["g"])
            u = self._lin(h, lw["u"])
            x = x + self._lin(((g / (1.0 + np.exp(-g))) * u).astype(np.float32), lw["dn"])
        want = np.concatenate([np.arange(o + i["n"] - i["want"], o + i["n"]) for i, o in zip(its, offs)])
        for it in work:
            self.blk[it["sid"]] = list(it["blocks"])
        if not want.size:
            return np.zeros((0, w.V), np.float32)
        hn = rms(x[want], w.out_norm, w.eps)
        return self._lin(hn, w.head).astype(np.float32)

    def commit(self, sid, base, pth):
        """Row base + pth[j] becomes row base + j, all layers, K and V (ref.py:114-120)."""
        sl = self.slots(self.blk[sid])
        moves = [(int(sl[base + i]), int(sl[base + j])) for j, i in enumerate(pth) if i != j]
        if not moves:
            return
        src = [a for a, _ in moves]
        if self.kv != "f16" and self.kv_scale == "page":
            # every source row is decoded before any destination is written; a moved row is re-encoded in its new
            # page's scale (and, as a page's first row, sets that scale)
            got = [self._read(l, src) for l in range(self.w.L)]
            for r, (_, b) in enumerate(moves):
                for l in range(self.w.L):
                    self._write(l, b, got[l][0][r], got[l][1][r])
        else:
            K, V = self.kc[:, src].copy(), self.vc[:, src].copy()
            for r, (_, b) in enumerate(moves):
                self.kc[:, b], self.vc[:, b] = K[:, r], V[:, r]

    def copy_blocks(self, pairs):
        """Whole blocks src -> dst (ref.py:122-126), page exponents included."""
        bs = self.bs
        for s, d in pairs:
            self.kc[:, d * bs:(d + 1) * bs] = self.kc[:, s * bs:(s + 1) * bs]
            self.vc[:, d * bs:(d + 1) * bs] = self.vc[:, s * bs:(s + 1) * bs]
            if self.kv != "f16":
                self.ke[:, d], self.ve[:, d] = self.ke[:, s], self.ve[:, s]

    def release(self, sid):
        self.blk.pop(sid, None)


def dense_greedy(w, tokens, steps, kv="f16"):
    """Greedy continuation with a private cache (RefModel.dense, ref.py:68-79): the paging-free oracle."""
    n = len(tokens) + steps
    o = PagedOracle(w, num_blocks=-(-n // 16), block_size=16, kv=kv)
    blocks = list(range(o.nb))
    lg = o.step([dict(sid=0, tokens=tokens, pos=0, blocks=blocks, want=1)])
    out = [int(lg[-1].argmax())]
    for p in range(len(tokens), n - 1):
        lg = o.step([dict(sid=0, tokens=[out[-1]], pos=p, blocks=blocks, want=1)])
        out.append(int(lg[-1].argmax()))
    return out
