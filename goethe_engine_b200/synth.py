"""Seeded synthetic decoder checkpoints as llama-architecture GGUF files, and the pack directory the library opens.

There is no network for real checkpoints, so tests and the benchmark build their own:

* ``init="ref"`` draws weights exactly as the reference model does (``goethe_engine/ref.py:22-27``): one
  ``torch.Generator().manual_seed(seed)``, ``randn(*shape) / sqrt(shape[-1])`` in the order emb, head, then per layer
  q, k, v, o, g, u, dn; emb and head times 2; no norm gains (written as ones) and eps 1e-6.
* ``init="baseline"`` draws N(0, 0.02) for every matrix (the benchmark configs), norm gains 1, eps from the spec;
  each tensor has its own counter-based normal stream (``csrc/synth.c``), so an 8B file is made in seconds.

Linear weights are then quantized to the spec's type (Q8_0, Q4_K, F16 or F32) by ``csrc/synth.c`` and streamed to
the GGUF file. ``pack_dir`` writes the ``manifest.json`` that ``gc_open`` reads (bucket ``ncol``, ``maxctx``, ``kv``,
``tune``), in the reference's manifest shape (``goethe_engine/pack.py:82-142``).
"""
import ctypes as C
import json
import math
import os
from dataclasses import asdict, dataclass, field

import numpy as np

from . import gguf as G

TYPES = {"f32": 0, "f16": 1, "q8_0": 8, "q4_k": 12}
_LIB = None


def _lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(os.path.dirname(__file__), "libgcksynth.so")
        if not os.path.exists(path):
            from . import build
            build.build_synth()
        L = C.CDLL(path)
        for n in ("synth_quantize_q8_0", "synth_quantize_q4_k"):
            getattr(L, n).argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_int]
        L.synth_normal.argtypes = [C.c_void_p, C.c_int64, C.c_uint64, C.c_uint64, C.c_int64, C.c_float, C.c_int]
        _LIB = L
    return _LIB


def threads():
    return max(1, min(64, os.cpu_count() or 1))


def quantize(x, ggml_type):
    """Raw GGUF bytes of the float32 matrix x [rows, cols] in the given type."""
    x = np.ascontiguousarray(x, np.float32)
    if ggml_type == 0:
        return x.view(np.uint8).reshape(-1)
    if ggml_type == 1:
        return x.astype(np.float16).view(np.uint8).reshape(-1)
    out = np.empty(G.tensor_bytes(ggml_type, [x.shape[-1], x.size // x.shape[-1]]), np.uint8)
    f = _lib().synth_quantize_q8_0 if ggml_type == 8 else _lib().synth_quantize_q4_k
    rc = f(x.ctypes.data, x.size, out.ctypes.data, threads())
    if rc:
        raise ValueError(f"row length {x.shape[-1]} does not fit ggml type {ggml_type} blocks")
    return out


def normal(shape, seed, stream, std):
    x = np.empty(shape, np.float32)
    _lib().synth_normal(x.ctypes.data, x.size, seed, stream, 0, std, threads())
    return x


@dataclass
class Spec:
    """A llama-style decoder: sizes, numerics and storage types."""
    vocab: int
    d: int
    layers: int
    heads: int
    kv_heads: int
    ffn: int
    eps: float = 1e-5
    theta: float = 1e4
    wtype: str = "q8_0"          # q_proj .. down_proj
    emb_type: str = ""           # token_embd ("" = wtype)
    head_type: str = ""          # output ("" = wtype)
    init: str = "baseline"       # "baseline": N(0, 0.02); "ref": ref.py's init
    std: float = 0.02
    seed: int = 0
    ctx: int = 8192
    name: str = "synthetic-llama"
    extra: dict = field(default_factory=dict)

    @property
    def dh(self):
        return self.d // self.heads

    def tensors(self):
        """[(name, [rows, cols], type name)] in file order (rows = output features)."""
        et, ht, wt = self.emb_type or self.wtype, self.head_type or self.wtype, self.wtype
        out = [("token_embd.weight", [self.vocab, self.d], et)]
        for i in range(self.layers):
            b = f"blk.{i}."
            out += [(b + "attn_norm.weight", [1, self.d], "f32"),
                    (b + "attn_q.weight", [self.heads * self.dh, self.d], wt),
                    (b + "attn_k.weight", [self.kv_heads * self.dh, self.d], wt),
                    (b + "attn_v.weight", [self.kv_heads * self.dh, self.d], wt),
                    (b + "attn_output.weight", [self.d, self.heads * self.dh], wt),
                    (b + "ffn_norm.weight", [1, self.d], "f32"),
                    (b + "ffn_gate.weight", [self.ffn, self.d], wt),
                    (b + "ffn_up.weight", [self.ffn, self.d], wt),
                    (b + "ffn_down.weight", [self.d, self.ffn], wt)]
        out += [("output_norm.weight", [1, self.d], "f32"), ("output.weight", [self.vocab, self.d], ht)]
        return out

    def meta(self):
        return {"general.architecture": "llama", "general.name": self.name, "general.alignment": G.ALIGN,
                "llama.block_count": self.layers, "llama.embedding_length": self.d,
                "llama.feed_forward_length": self.ffn, "llama.attention.head_count": self.heads,
                "llama.attention.head_count_kv": self.kv_heads, "llama.rope.freq_base": float(self.theta),
                "llama.attention.layer_norm_rms_epsilon": float(self.eps), "llama.context_length": self.ctx,
                "llama.vocab_size": self.vocab, "llama.rope.dimension_count": self.dh}

    def params(self):
        return sum(r * c for n, (r, c), t in self.tensors() if t != "f32" or r > 1)


def _ref_init(spec):
    """Float32 matrices in ref.py's draw order (ref.py:22-27) from torch's generator."""
    import torch
    g = torch.Generator().manual_seed(spec.seed)

    def w(*s):
        return (torch.randn(*s, generator=g) / math.sqrt(s[-1])).numpy()
    dh = spec.dh
    mats = {"token_embd.weight": w(spec.vocab, spec.d) * 2, "output.weight": w(spec.vocab, spec.d) * 2}
    for i in range(spec.layers):
        b = f"blk.{i}."
        for k, s in (("attn_q", (spec.heads * dh, spec.d)), ("attn_k", (spec.kv_heads * dh, spec.d)),
                     ("attn_v", (spec.kv_heads * dh, spec.d)), ("attn_output", (spec.d, spec.heads * dh)),
                     ("ffn_gate", (spec.ffn, spec.d)), ("ffn_up", (spec.ffn, spec.d)),
                     ("ffn_down", (spec.d, spec.ffn))):
            mats[b + k + ".weight"] = w(*s)
    return mats


def write_gguf(spec, path):
    """Write the checkpoint of spec to path (streamed tensor by tensor)."""
    tab = spec.tensors()
    ref = _ref_init(spec) if spec.init == "ref" else None
    gt = [(n, [c, r] if r > 1 else [c], TYPES[t]) for n, (r, c), t in tab]
    w = G.Writer(path, spec.meta(), gt)
    for i, (n, (r, c), t) in enumerate(tab):
        if r == 1:                                 # norm gains
            x = np.ones((c,), np.float32)
        elif ref is not None:
            x = ref[n]
        else:
            x = normal((r, c), spec.seed, i, spec.std)
        w.write(n, quantize(x, TYPES[t]))
    w.close()
    return path


def pack_dir(d, spec, buckets, weights_file="model.gguf", pairs=(), drafter_file=None):
    """Write d/manifest.json for the given buckets: [{id, ncol, maxctx, kv, act, tune, tp, determinism, role}] (tune:
    the library's knobs; tp: the tensor-parallel degree, 1 when absent; act: "a16" (default) or "a8" (per-token int8
    activations); determinism: "batch_invariant" (default, contract "BI") or "tolerance" (contract "FAST": the GEMV for
    steps of a few token rows, pack.py:639); role: "target" (default) or "drafter", whose weights are drafter_file).
    pairs: speculative pairs (target id, drafter id, K), written as the manifest's spec list with policy
    {kind: "ar", K} (pack.py:130-141); their targets list "ar" in spec_caps.accept."""
    os.makedirs(d, exist_ok=True)
    bs = []
    targets = {t for t, _, _ in pairs}
    for b in buckets:
        det = b.get("determinism", "batch_invariant")
        role = b.get("role", "target")
        bs.append(dict(id=b["id"], role=role, variant="v" if role == "target" else "dv", sku="b200",
                       contract="BI" if det != "tolerance" else "FAST",
                       ncol=b.get("ncol", 64), batch=b.get("batch", True), maxctx=b.get("maxctx", spec.ctx),
                       weights=0 if role == "target" else 1,
                       files={}, lib="libgck.so", requires=dict(arch="sm_100a", cc="10.0", sms=148, name="NVIDIA B200"),
                       determinism=det, act=b.get("act", "a16"), kv=b.get("kv", "f16"),
                       spec_caps=dict(verify=["linear", "tree"], tree_mask=True, verify_widths=[], taps=[],
                                      recurrent_commit=[], accept=["ar"] if b["id"] in targets else [],
                                      drafter_roles=["ar"] if b["id"] in targets else []),
                       tune=dict(b.get("tune", {}))))
        if b.get("tp", 1) > 1:
            bs[-1]["tp"] = b["tp"]   # tensor-parallel degree: devices device .. device + tp - 1
    files = [dict(file=weights_file)] + ([dict(file=drafter_file)] if drafter_file else [])
    m = dict(schema="gc-pack", abi="3.0.0", arch="sm_100a", cuda="12.9", runtime=dict(kind="gc-c", version=1),
             contracts=sorted({x["contract"] for x in bs}), buckets=bs, model=dict(name=spec.name, weights=files),
             synth=asdict(spec))
    if pairs:
        m["spec"] = [dict(target=t, drafter=dr, policy=dict(kind="ar", K=str(k))) for t, dr, k in pairs]
    with open(os.path.join(d, "manifest.json"), "w") as f:
        json.dump(m, f, indent=1, sort_keys=True)
    return d


def make(d, spec, buckets=None, **bucket_kw):
    """A pack directory and its weights under d; returns (pack_dir, [gguf path])."""
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, "model.gguf")
    if not os.path.exists(path):
        write_gguf(spec, path + ".tmp")
        os.replace(path + ".tmp", path)
    pack_dir(d, spec, buckets or [dict(id="b200.BI.main", **bucket_kw)])
    return d, [path]
