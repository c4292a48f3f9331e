"""CPU restatement of the weight and KV storage formats on the decoder path (test infrastructure only).

This module is the parity oracle's view of the bytes the library consumes. It is imported by tests/, by
``__graft_entry__.smoke()`` and by ``bench.py``'s CPU-baseline leg, never by the product path.

Formats:

* GGUF ``Q8_0`` (type id 8, ``structure.py:18`` of the reference names it): 32-element blocks of
  ``fp16 d`` followed by 32 ``int8 q``; the value is ``d * q``. The reference vendors no quant code
  (ggml is an unpinned third-party dependency); the block layout is the published ggml one and is
  pinned against ``gguf`` 0.19.0's ``quants.dequantize`` by ``tests/golden/make_golden.py``.
* GGUF ``Q4_K`` (type id 12): 256-element super-blocks of ``fp16 d``, ``fp16 dmin``, 12 bytes of packed
  6-bit sub-block scales and mins, then 128 bytes of 4-bit quants; value ``d*sc[s]*q - dmin*m[s]`` for the
  32-element sub-block ``s``. Sub-block ``2c`` takes the low nibbles of quant bytes ``32c .. 32c+31``,
  ``2c+1`` the high nibbles of the same bytes.
* ``float8_e4m3fn`` KV rows (``ref.py:11,54`` casts K and V with ``.to(torch.float8_e4m3fn)``): 1 sign,
  4 exponent (bias 7), 3 mantissa bits, no infinities, max 448; round to nearest even.
"""
import numpy as np

QK8_0, Q8_0_BYTES = 32, 34
QK_K, Q4_K_BYTES = 256, 144
GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K = 0, 1, 8, 12
TYPE_BLOCK = {GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_Q8_0: (QK8_0, Q8_0_BYTES), GGML_Q4_K: (QK_K, Q4_K_BYTES)}


def row_bytes(ggml_type, n):
    """Bytes of one row of n elements in a GGUF tensor of the given type."""
    blk, size = TYPE_BLOCK[ggml_type]
    assert n % blk == 0, (ggml_type, n)
    return n // blk * size


def dequant_q8_0(raw, n):
    """float32 [n] from n/32 Q8_0 blocks (raw: uint8 bytes)."""
    b = np.frombuffer(raw, np.uint8)[: n // QK8_0 * Q8_0_BYTES].reshape(-1, Q8_0_BYTES)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:].copy().view(np.int8).astype(np.float32)
    return (d * q).reshape(-1)


def q4_k_scales(sc12):
    """(sc [nb, 8], m [nb, 8]) uint8 6-bit sub-block scales and mins from the 12 packed bytes of each super-block.

    Bytes 0-3 hold scales 0-3 in their low 6 bits, bytes 4-7 mins 0-3; scales/mins 4-7 take their low 4 bits
    from the nibbles of bytes 8-11 and their top 2 bits from the top 2 bits of bytes 0-3 (scales) and 4-7 (mins).
    """
    s = sc12.astype(np.uint8)
    sc = np.empty((s.shape[0], 8), np.uint8)
    m = np.empty((s.shape[0], 8), np.uint8)
    sc[:, :4] = s[:, 0:4] & 63
    m[:, :4] = s[:, 4:8] & 63
    sc[:, 4:] = (s[:, 8:12] & 0xF) | ((s[:, 0:4] >> 6) << 4)
    m[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    return sc, m


def dequant_q4_k(raw, n):
    """float32 [n] from n/256 Q4_K super-blocks (raw: uint8 bytes)."""
    b = np.frombuffer(raw, np.uint8)[: n // QK_K * Q4_K_BYTES].reshape(-1, Q4_K_BYTES)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    dmin = b[:, 2:4].copy().view(np.float16).astype(np.float32)
    sc, m = q4_k_scales(b[:, 4:16])
    qs = b[:, 16:].reshape(-1, 4, 32)
    q = np.empty((b.shape[0], 8, 32), np.float32)
    q[:, 0::2] = qs & 0xF
    q[:, 1::2] = qs >> 4
    q *= (d * sc.astype(np.float32))[:, :, None]          # d * sc[s] * q, then minus dmin * m[s]: float32, in place
    q -= (dmin * m.astype(np.float32))[:, :, None]
    return q.reshape(-1)


def dequant(ggml_type, raw, shape):
    """float32 array of the given shape (rows, cols) from raw GGUF tensor bytes."""
    n = int(np.prod(shape))
    if ggml_type == GGML_F32:
        return np.frombuffer(raw, np.float32, n).reshape(shape).copy()
    if ggml_type == GGML_F16:
        return np.frombuffer(raw, np.float16, n).astype(np.float32).reshape(shape)
    if ggml_type == GGML_Q8_0:
        return dequant_q8_0(raw, n).reshape(shape)
    if ggml_type == GGML_Q4_K:
        return dequant_q4_k(raw, n).reshape(shape)
    raise ValueError(f"ggml type {ggml_type} is not on the decoder path")


# --- float8 e4m3fn ---------------------------------------------------------------------------------------------------

def _e4m3_table():
    codes = np.arange(256, dtype=np.uint32)
    s = (codes >> 7) & 1
    e = (codes >> 3) & 0xF
    m = codes & 7
    v = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1 + m / 8.0) * 2.0 ** (e.astype(np.int32) - 7))
    v = np.where((e == 15) & (m == 7), np.nan, v)
    return np.where(s == 1, -v, v).astype(np.float32)


E4M3_VALUES = _e4m3_table()
E4M3_MAX = 448.0


def e4m3_decode(codes):
    """float32 values of uint8 e4m3fn codes."""
    return E4M3_VALUES[np.asarray(codes, np.uint8)]


def e4m3_encode(x):
    """uint8 e4m3fn codes of float32 x: round to nearest, ties to even (a negative value that rounds to zero keeps its
    sign, -0 = 0x80); |x| > 448 saturates to +-448 (torch gives NaN from 464 up; KV rows never reach it)."""
    x = np.asarray(x, np.float32)
    a = np.minimum(np.abs(x), E4M3_MAX).astype(np.float64)
    # exponent of the binade (subnormals share the binade of 2^-6)
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -6)))
    e = np.clip(e, -6, 8)
    step = 2.0 ** (e - 3)
    q = a / step
    r = np.floor(q)
    frac = q - r
    r = r + ((frac > 0.5) | ((frac == 0.5) & (r % 2 == 1)))
    v = np.minimum(r * step, E4M3_MAX)
    # re-derive the code from the rounded value
    out = np.zeros(x.shape, np.uint8)
    nz = v > 0
    ev = np.floor(np.log2(np.where(nz, v, 1.0)))
    sub = nz & (ev < -6)
    norm = nz & ~sub
    mant_n = np.round((v / 2.0 ** ev - 1.0) * 8).astype(np.int64)
    code_n = ((ev + 7).astype(np.int64) << 3) | mant_n
    code_s = np.round(v / 2.0 ** -9).astype(np.int64)
    out = np.where(norm, code_n, np.where(sub, code_s, 0)).astype(np.uint8)
    out = out | np.where(np.signbit(x), 0x80, 0).astype(np.uint8)
    return out


def f16_round(x):
    """x rounded to float16 and back (round to nearest even), as ``.to(torch.float16)`` does."""
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)
