"""Generate the golden fixtures that pin the oracle (run in a container where the reference is mounted).

    python tests/golden/make_golden.py [/path/to/reference]

Writes into this directory:

* ``quant_golden.npz`` — random Q8_0 and Q4_K block bytes and their dequantized values from the third-party
  ``gguf`` 0.19.0 package (``gguf.quants.dequantize``); the reference itself has no quant code.
* ``e4m3_golden.npz`` — float32 values and their ``torch.float8_e4m3fn`` codes (the cast of ``ref.py:54``).
* ``ref_tiny.npz`` / ``ref_c1.npz`` — logits from the reference's own ``RefModel`` + ``TorchBackend``
  (``goethe_engine/ref.py``) over a scripted session of prefill chunks, batched decode, tree verify, commit and
  copy_blocks (the script is ``SCENARIO`` below; tests/test_oracle.py replays it through the oracle). ``ref_tiny``
  uses ``RefModel()``'s defaults; ``ref_c1`` the config-1 shape (vocab 32000, d 512, 4 layers, 8/2 heads, ffn 1408)
  with ref.py's init, storing only a fixed column sample of each logits row, its argmax and its norm.

Nothing at run time reads the reference: the fixtures are committed.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# A session over block_size-16 pages: (op, args). Blocks are explicit so prefix sharing and CoW are exercised.
SCENARIO = [
    ("step", [dict(sid=1, tokens=list(range(3, 23)), pos=0, blocks=[0, 1], want=1)]),
    ("step", [dict(sid=2, tokens=[5, 9, 1, 7, 3, 2, 8], pos=0, blocks=[2], want=0)]),
    ("step", [dict(sid=2, tokens=[11, 4, 6, 10, 12, 13], pos=7, blocks=[2], want=2)]),
    ("step", [dict(sid=1, tokens=[30], pos=20, blocks=[0, 1], want=1),
              dict(sid=2, tokens=[31], pos=13, blocks=[2], want=1)]),
    ("step", [dict(sid=1, tokens=[40, 41, 42, 43, 44], pos=21, blocks=[0, 1], want=5, parents=[-1, 0, 0, 1, 2])]),
    ("commit", (1, 21, [0, 2, 4])),
    ("step", [dict(sid=1, tokens=[45], pos=24, blocks=[0, 1], want=1)]),
    ("copy", [(0, 5), (1, 6)]),
    ("step", [dict(sid=3, tokens=[46, 47], pos=25, blocks=[5, 6], want=2),
              dict(sid=2, tokens=[48], pos=14, blocks=[2], want=1)]),
    # a chain and a tree that must agree on the shared path (gc.h:139-146)
    ("step", [dict(sid=4, tokens=[3, 9, 4, 1], pos=0, blocks=[7], want=0)]),
    ("step", [dict(sid=4, tokens=[7, 11, 13], pos=4, blocks=[7], want=3, parents=[-1, 0, 0])]),
    ("step", [dict(sid=5, tokens=[3, 9, 4, 1], pos=0, blocks=[8], want=0)]),
    ("step", [dict(sid=5, tokens=[7, 13], pos=4, blocks=[8], want=2)]),
]


def run_ref(model, kv, num_blocks=16):
    from goethe_engine.backend import Work
    from goethe_engine.ref import TorchBackend
    be = TorchBackend(model, num_blocks=num_blocks, block_size=16, kv=kv)
    out = []
    for op, a in SCENARIO:
        if op == "step":
            ws = [Work(w["sid"], w["tokens"], w["pos"], w["blocks"], w["want"], parents=w.get("parents")) for w in a]
            out.append(be.step(ws).numpy().astype(np.float32))
        elif op == "commit":
            be.commit(*a)
        elif op == "copy":
            be.copy_blocks(a)
    return out


def main(ref_root="/root/reference"):
    sys.path.insert(0, ref_root)
    import gguf
    import torch
    from goethe_engine.ref import RefModel

    rng = np.random.default_rng(0)
    # Q8_0: random int8 with positive and negative fp16 scales
    nb = 64
    q8 = np.zeros((nb, 34), np.uint8)
    q8[:, :2] = (rng.uniform(-0.01, 0.01, nb).astype(np.float16)).view(np.uint8).reshape(nb, 2)
    q8[:, 2:] = rng.integers(0, 256, (nb, 32), dtype=np.uint8)
    # Q4_K: random packed scales / quants, d and dmin of either sign
    q4 = rng.integers(0, 256, (nb, 144), dtype=np.uint8)
    q4[:, 0:2] = rng.uniform(-0.01, 0.01, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    q4[:, 2:4] = rng.uniform(-0.01, 0.01, nb).astype(np.float16).view(np.uint8).reshape(nb, 2)
    np.savez_compressed(os.path.join(HERE, "quant_golden.npz"),
                        q8_0=q8, q8_0_f32=gguf.quants.dequantize(q8, gguf.GGMLQuantizationType.Q8_0).reshape(-1),
                        q4_k=q4, q4_k_f32=gguf.quants.dequantize(q4, gguf.GGMLQuantizationType.Q4_K).reshape(-1))

    x = (rng.standard_normal(20000) * np.exp(rng.uniform(-10, 5, 20000))).astype(np.float32)
    x = x[np.abs(x) <= 448]
    np.savez_compressed(os.path.join(HERE, "e4m3_golden.npz"), x=x,
                        codes=torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy())

    m = RefModel()
    tiny = dict(emb=m.emb.numpy(), head=m.head.numpy())
    for i, lw in enumerate(m.layers):
        for k, v in lw.items():
            tiny[f"l{i}.{k}"] = v.numpy()
    for kv in ("f16", "fp8"):
        for i, lg in enumerate(run_ref(m, kv)):
            tiny[f"{kv}.step{i}"] = lg
    np.savez_compressed(os.path.join(HERE, "ref_tiny.npz"), **tiny)

    m = RefModel(vocab=32000, d=512, layers=4, heads=8, kv_heads=2, ffn=1408, seed=0)
    cols = np.sort(np.random.default_rng(1).choice(32000, 256, replace=False))
    c1 = dict(cols=cols)
    for kv in ("f16", "fp8"):
        for i, lg in enumerate(run_ref(m, kv)):
            c1[f"{kv}.step{i}.cols"] = lg[:, cols]
            c1[f"{kv}.step{i}.argmax"] = lg.argmax(1)
            c1[f"{kv}.step{i}.norm"] = np.linalg.norm(lg, axis=1).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "ref_c1.npz"), **c1)


if __name__ == "__main__":
    main(*sys.argv[1:])
