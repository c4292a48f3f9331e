"""GGUF v3 files: a streaming writer and a header reader.

The library finds every tensor by name in the GGUF files ``gc_open`` is given (``abi/gc.h:64-66`` of the reference:
"tensors are found by name"). Weight files are llama-architecture GGUF: ``token_embd.weight``,
``blk.N.{attn_norm,attn_q,attn_k,attn_v,attn_output,ffn_norm,ffn_gate,ffn_up,ffn_down}.weight``,
``output_norm.weight``, ``output.weight``; metadata ``llama.*`` keys. Dimensions are stored ggml-style: ``ne[0]`` is
the row length (the contraction dimension), ``ne[1]`` the number of rows.

Layout of a file: magic ``GGUF``, u32 version 3, u64 tensor count, u64 metadata count, the metadata (key string,
u32 type, value), the tensor infos (name string, u32 n_dims, u64 dims[n_dims], u32 ggml type, u64 offset relative to
the data section), zero padding to ``general.alignment`` (default 32), then the data section. Strings are u64 length
plus bytes. The reference reads the same framing for structure checks (``goethe_engine/structure.py:65-87``).
"""
import struct

import numpy as np

GGUF_MAGIC = b"GGUF"
ALIGN = 32
# metadata value types
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)
_SCALAR = {T_U8: "B", T_I8: "b", T_U16: "H", T_I16: "h", T_U32: "I", T_I32: "i", T_F32: "f", T_BOOL: "?",
           T_U64: "Q", T_I64: "q", T_F64: "d"}
TYPE_BLOCK = {0: (1, 4), 1: (1, 2), 8: (32, 34), 12: (256, 144)}   # ggml type -> (elements, bytes) per block


def tensor_bytes(ggml_type, dims):
    blk, size = TYPE_BLOCK[ggml_type]
    n = int(np.prod(dims))
    assert dims[0] % blk == 0, (ggml_type, dims)
    return n // blk * size


def _str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(v):
    if isinstance(v, bool):
        return struct.pack("<I?", T_BOOL, v)
    if isinstance(v, str):
        return struct.pack("<I", T_STR) + _str(v)
    if isinstance(v, int):
        return struct.pack("<II", T_U32, v) if 0 <= v < 1 << 32 else struct.pack("<Iq", T_I64, v)
    if isinstance(v, float):
        return struct.pack("<If", T_F32, v)
    if isinstance(v, (list, tuple)):
        if v and isinstance(v[0], str):
            return struct.pack("<IIQ", T_ARR, T_STR, len(v)) + b"".join(_str(x) for x in v)
        return struct.pack("<IIQ", T_ARR, T_I32, len(v)) + b"".join(struct.pack("<i", x) for x in v)
    raise TypeError(f"metadata value {v!r}")


class Writer:
    """Write a GGUF file whose tensor table is known up front; tensor bytes are then streamed in table order.

    >>> w = Writer(path, {"general.architecture": "llama"}, [(name, dims, ggml_type), ...])
    >>> for name, ... : w.write(name, raw_bytes)
    >>> w.close()
    """

    def __init__(self, path, meta, tensors, align=ALIGN):
        self.f = open(path, "wb")
        self.tensors, self.align, self.next = list(tensors), align, 0
        hdr = GGUF_MAGIC + struct.pack("<IQQ", 3, len(self.tensors), len(meta))
        for k, v in meta.items():
            hdr += _str(k) + _value(v)
        off, self.sizes = 0, []
        for name, dims, t in self.tensors:
            hdr += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", x) for x in dims)
            hdr += struct.pack("<IQ", t, off)
            n = tensor_bytes(t, dims)
            self.sizes.append(n)
            off += n + (-n % align)
        hdr += b"\0" * (-len(hdr) % align)
        self.f.write(hdr)

    def write(self, name, raw):
        i = self.next
        assert self.tensors[i][0] == name, (name, self.tensors[i][0])
        raw = memoryview(np.ascontiguousarray(raw)).cast("B")
        assert len(raw) == self.sizes[i], (name, len(raw), self.sizes[i])
        self.f.write(raw)
        self.f.write(b"\0" * (-len(raw) % self.align))
        self.next += 1

    def close(self):
        assert self.next == len(self.tensors), "not every tensor was written"
        self.f.close()


class _Rd:
    def __init__(self, f):
        self.f = f

    def get(self, fmt):
        n = struct.calcsize("<" + fmt)
        b = self.f.read(n)
        if len(b) != n:
            raise ValueError("truncated GGUF header")
        return struct.unpack("<" + fmt, b)[0]

    def str(self):
        return self.f.read(self.get("Q")).decode("utf-8", "replace")

    def value(self, t):
        if t in _SCALAR:
            return self.get(_SCALAR[t])
        if t == T_STR:
            return self.str()
        if t == T_ARR:
            et, n = self.get("I"), self.get("Q")
            return [self.value(et) for _ in range(n)]
        raise ValueError(f"GGUF metadata type {t}")


def read_header(path):
    """(metadata dict, {name: (dims, ggml type, absolute file offset)}) of a GGUF file."""
    with open(path, "rb") as f:
        r = _Rd(f)
        if f.read(4) != GGUF_MAGIC:
            raise ValueError(f"{path}: not a GGUF file")
        ver = r.get("I")
        if ver not in (2, 3):
            raise ValueError(f"{path}: GGUF version {ver}")
        nt, nkv = r.get("Q"), r.get("Q")
        meta = {}
        for _ in range(nkv):
            k = r.str()
            meta[k] = r.value(r.get("I"))
        infos = []
        for _ in range(nt):
            name, nd = r.str(), r.get("I")
            dims = [r.get("Q") for _ in range(nd)]
            infos.append((name, dims, r.get("I"), r.get("Q")))
        align = int(meta.get("general.alignment", ALIGN))
        base = f.tell() + (-f.tell() % align)
    return meta, {n: (d, t, base + o) for n, d, t, o in infos}


def read_tensor(path, info):
    """Raw bytes of one tensor given its (dims, type, offset) from read_header."""
    dims, t, off = info
    with open(path, "rb") as f:
        f.seek(off)
        return f.read(tensor_bytes(t, dims))
