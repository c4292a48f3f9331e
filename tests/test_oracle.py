"""The oracle pinned against the reference's own outputs (committed golden fixtures; CPU only).

* ``quants`` against ``gguf`` 0.19.0 dequantization and torch's e4m3 cast;
* ``model.PagedOracle`` against ``goethe_engine/ref.py`` (``RefModel`` + ``TorchBackend``) over the scripted session
  of ``tests/golden/make_golden.py``: prefill chunks, batched decode, tree verify, commit, copy_blocks; f16 and fp8 KV.
"""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
from make_golden import SCENARIO  # noqa: E402

from oracle import quants as Q  # noqa: E402
from oracle.model import PagedOracle, Weights, depths, path  # noqa: E402

GOLD = os.path.join(HERE, "golden")


def replay(w, kv, kv_scale="unit"):
    o = PagedOracle(w, num_blocks=16, block_size=16, kv=kv, kv_scale=kv_scale)
    out = []
    for op, a in SCENARIO:
        if op == "step":
            out.append(o.step(a))
        elif op == "commit":
            o.commit(*a)
        elif op == "copy":
            o.copy_blocks(a)
    return out


def test_q8_0_and_q4_k_match_gguf_dequantize():
    g = np.load(os.path.join(GOLD, "quant_golden.npz"))
    got8 = Q.dequant_q8_0(g["q8_0"].tobytes(), g["q8_0"].shape[0] * 32)
    got4 = Q.dequant_q4_k(g["q4_k"].tobytes(), g["q4_k"].shape[0] * 256)
    assert np.array_equal(got8, g["q8_0_f32"])
    assert np.array_equal(got4, g["q4_k_f32"])


def test_e4m3_encode_decode_match_torch_cast():
    g = np.load(os.path.join(GOLD, "e4m3_golden.npz"))
    assert np.array_equal(Q.e4m3_encode(g["x"]), g["codes"])
    dec = Q.e4m3_decode(g["codes"])
    assert np.array_equal(Q.e4m3_encode(dec), g["codes"])


def test_depths_and_path_follow_spec():
    par = [-1, 0, 0, 1, 2]
    assert depths(par, 5) == [0, 1, 1, 2, 2] and depths(None, 3) == [0, 1, 2]
    assert path(par, 4) == [0, 2, 4] and path(None, 2) == [0, 1, 2]


def tiny_weights():
    g = np.load(os.path.join(GOLD, "ref_tiny.npz"))
    L = 2
    layers = [{k: g[f"l{i}.{k}"] for k in ("q", "k", "v", "o", "g", "u", "dn")} for i in range(L)]
    return Weights(g["emb"], g["head"], layers, eps=1e-6, heads=4, kv_heads=2), g


@pytest.mark.parametrize("kv", ["f16", "fp8"])
def test_oracle_matches_ref_tiny(kv):
    w, g = tiny_weights()
    for i, lg in enumerate(replay(w, kv)):
        ref = g[f"{kv}.step{i}"]
        assert lg.shape == ref.shape
        if not ref.size:
            continue
        np.testing.assert_allclose(lg, ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())
        assert (lg.argmax(1) == ref.argmax(1)).all()


def test_tree_rows_equal_chain_rows_in_the_oracle():
    w, _ = tiny_weights()
    out = replay(w, "f16")
    tree, chain = out[8], out[10]            # sid 4: [7, 11, 13] parents [-1,0,0]; sid 5: chain [7, 13]
    np.testing.assert_allclose(tree[0], chain[0], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(tree[2], chain[1], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("kv", ["f16", "fp8"])
def test_oracle_matches_ref_config1_shape(kv):
    from goethe_engine_b200.synth import Spec, _ref_init
    spec = Spec(vocab=32000, d=512, layers=4, heads=8, kv_heads=2, ffn=1408, init="ref", seed=0, eps=1e-6)
    m = _ref_init(spec)
    layers = [dict(q=m[f"blk.{i}.attn_q.weight"], k=m[f"blk.{i}.attn_k.weight"], v=m[f"blk.{i}.attn_v.weight"],
                   o=m[f"blk.{i}.attn_output.weight"], g=m[f"blk.{i}.ffn_gate.weight"], u=m[f"blk.{i}.ffn_up.weight"],
                   dn=m[f"blk.{i}.ffn_down.weight"]) for i in range(4)]
    w = Weights(m["token_embd.weight"], m["output.weight"], layers, eps=1e-6, heads=8, kv_heads=2)
    g = np.load(os.path.join(GOLD, "ref_c1.npz"))
    cols = g["cols"]
    for i, lg in enumerate(replay(w, kv)):
        ref = g[f"{kv}.step{i}.cols"]
        if not ref.size:
            continue
        np.testing.assert_allclose(lg[:, cols], ref, rtol=1e-3, atol=1e-3 * np.abs(ref).max())
        np.testing.assert_allclose(np.linalg.norm(lg, axis=1), g[f"{kv}.step{i}.norm"], rtol=1e-4)
        assert (lg.argmax(1) == g[f"{kv}.step{i}.argmax"]).all()


@pytest.mark.parametrize("kv,kv_scale", [("f16", "unit"), ("fp8", "page")])
def test_chunked_chain_attention_equals_token_by_token(kv, kv_scale, monkeypatch):
    """A chain item's attention runs in chunks with a causal mask; the same tokens as a tree whose parents form a chain
    take the token-by-token path over their paths. Both see the same rows, so the logits agree to float32 rounding,
    across several chunks (CHUNK 8 here) and a cached prefix."""
    rng = np.random.default_rng(0)
    d, L, H, KVH, F, V = 64, 2, 4, 2, 96, 50
    mk = lambda *s: (rng.standard_normal(s) / np.sqrt(s[-1])).astype(np.float32)
    w = Weights(mk(V, d) * 2, mk(V, d) * 2, [dict(q=mk(d, d), k=mk(KVH * 16, d), v=mk(KVH * 16, d), o=mk(d, d),
                                                  g=mk(F, d), u=mk(F, d), dn=mk(d, F)) for _ in range(L)],
                eps=1e-6, heads=H, kv_heads=KVH)
    monkeypatch.setattr(PagedOracle, "CHUNK", 8)
    toks = [int(x) for x in rng.integers(0, V, 45)]
    out = {}
    for mode in ("chain", "tree"):
        o = PagedOracle(w, num_blocks=8, block_size=16, kv=kv, kv_scale=kv_scale)
        o.step([dict(sid=1, tokens=toks[:19], pos=0, blocks=list(range(8)), want=0)])
        par = None if mode == "chain" else [-1] + list(range(25))
        out[mode] = o.step([dict(sid=1, tokens=toks[19:], pos=19, blocks=list(range(8)), want=26, parents=par)])
    np.testing.assert_allclose(out["chain"], out["tree"], rtol=0, atol=1e-4 * np.abs(out["tree"]).max())
