"""Oracle weights from a GGUF checkpoint (test infrastructure only).

The file is parsed by the third-party ``gguf`` package (0.19.0, an independent reader of the format) and every
tensor is dequantized by ``oracle.quants`` into the float32 ``[out, in]`` matrices ``oracle.model.Weights`` takes,
the layout of ``goethe_engine/ref.py:25-27``.
"""
import numpy as np

from . import quants as Q
from .model import Weights


def _reader(path):
    import gguf
    return gguf.GGUFReader(path)


def _meta(r, key, default=None):
    f = r.fields.get(key)
    if f is None:
        return default
    v = f.parts[f.data[0]]
    if f.types and f.types[0] == 8:      # string
        return bytes(v).decode()
    return v.item() if hasattr(v, "item") and v.size == 1 else v


class QuantRows:
    """A quantized [rows, cols] matrix dequantized row by row on indexing (the embedding: a step reads only the rows of
    its tokens, so the whole table is never expanded to float32)."""

    def __init__(self, t):
        ne = [int(x) for x in t.shape]
        self.type, self.shape = int(t.tensor_type), (ne[1], ne[0])
        self.raw = np.asarray(t.data).view(np.uint8).reshape(ne[1], -1)

    def __getitem__(self, idx):
        idx = np.asarray(idx, np.int64).reshape(-1)
        rows = np.ascontiguousarray(self.raw[idx])
        return Q.dequant(self.type, rows.tobytes(), (len(idx), self.shape[1]))


def weights_from_gguf(path, layers=None):
    """oracle Weights of a llama GGUF file; layers: only the first n layers (a bounded CPU sample)."""
    r = _reader(path)
    T = {t.name: t for t in r.tensors}

    def mat(name):
        t = T[name]
        ne = [int(x) for x in t.shape]                 # ggml order: ne[0] = row length
        shape = (ne[1], ne[0]) if len(ne) > 1 else (ne[0],)
        raw = np.asarray(t.data).view(np.uint8).reshape(-1)
        return Q.dequant(int(t.tensor_type), raw.tobytes(), shape)

    L = int(_meta(r, "llama.block_count"))
    n = L if layers is None else min(L, layers)
    lw = []
    for i in range(n):
        b = f"blk.{i}."
        lw.append(dict(q=mat(b + "attn_q.weight"), k=mat(b + "attn_k.weight"), v=mat(b + "attn_v.weight"),
                       o=mat(b + "attn_output.weight"), g=mat(b + "ffn_gate.weight"), u=mat(b + "ffn_up.weight"),
                       dn=mat(b + "ffn_down.weight"), attn_norm=mat(b + "attn_norm.weight"),
                       ffn_norm=mat(b + "ffn_norm.weight")))
    return Weights(QuantRows(T["token_embd.weight"]), mat("output.weight"), lw, out_norm=mat("output_norm.weight"),
                   eps=float(_meta(r, "llama.attention.layer_norm_rms_epsilon", 1e-5)),
                   theta=float(_meta(r, "llama.rope.freq_base", 1e4)),
                   heads=int(_meta(r, "llama.attention.head_count")), kv_heads=int(_meta(r, "llama.attention.head_count_kv")))
