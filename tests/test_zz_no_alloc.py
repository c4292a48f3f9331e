"""gck_commit_static: the tree-verify commit for callers that may not allocate device memory while they run (a server
that reserves the GPU's memory at start-up, or one bound to a fixed memory budget). It does what gc_commit does with
its scratch in a fixed 16 MiB array inside the library, so it must leave exactly the KV rows gc_commit leaves.

Two sequences get the same prompt and the same draft trees; after each verify, one commits with gc_commit, the other
with gck_commit_static, and both then decode the same token. The two commits run the same kernels over the same rows,
so the logits must be identical, bit for bit (f16 and fp8 KV). Two verify/commit rounds run in a row, so the second
call finds the array holding the first call's contents. The device's free memory is read around the first static
commit: it must not change (the array was committed when gc_open looked its address up). A path that moves more rows
than the array holds is refused with GC_E_ARG before any device work. This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

from goethe_engine_b200 import build, gck, synth
from helpers import SMALL128, model

pytestmark = pytest.mark.gpu


def static_commit(be):
    fn = be.L.gck_commit_static
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p, C.c_uint64, C.c_uint32, C.POINTER(C.c_uint32), C.c_uint32]

    def call(sid, base, path):
        arr = (C.c_uint32 * len(path))(*path)
        return fn(be.h, sid, base, arr, len(path))
    return call


@pytest.mark.parametrize("kv", ["f16", "fp8"])
def test_static_commit_matches_gc_commit_twice(tmp_path, kv):
    import torch
    build.build()
    spec = synth.Spec(**SMALL128, wtype="q4_k", seed=21)
    pack, ws = model(tmp_path, spec, ncol=8, maxctx=512, kv=kv)
    with gck.Backend(pack, ws, pool_blocks=32) as be:
        commit = static_commit(be)
        prompt = [int(x) for x in np.random.default_rng(4).integers(1, 500, 13)]
        ta, tb = list(range(0, 8)), list(range(8, 16))
        be.step([gck.Work(1, prompt, 0, ta, 0), gck.Work(2, prompt, 0, tb, 0)])
        pos = len(prompt)
        rounds = [([40, 41, 42, 43, 44, 45], [-1, 0, 0, 1, 2, 4], [0, 2, 4, 5]),
                  ([50, 51, 52, 53, 54], [-1, 0, 1, 1, 3], [0, 1, 3, 4])]
        for r, (toks, parents, path) in enumerate(rounds):
            va = be.step([gck.Work(1, toks, pos, ta, len(toks), parents=parents)])
            vb = be.step([gck.Work(2, toks, pos, tb, len(toks), parents=parents)])
            assert np.array_equal(va, vb)
            be.commit(1, pos, path)
            torch.cuda.synchronize()
            free0 = torch.cuda.mem_get_info(0)[0]
            rc = commit(2, pos, path)
            assert rc == 0, (be.L.gc_last_error(be.h) or b"").decode()
            if r == 0:
                # the first static commit on this device allocated nothing
                assert torch.cuda.mem_get_info(0)[0] == free0
            pos += len(path)
            nxt = toks[path[-1]]
            a = be.step([gck.Work(1, [nxt], pos, ta, 1)])
            b = be.step([gck.Work(2, [nxt], pos, tb, 1)])
            assert np.array_equal(b, a)
            pos += 1
        # an unknown sequence is an error code, as with gc_commit
        assert commit(99, 0, [0, 1]) == gck.E_STATE
        # this model stages 2 layers x K, V x 1 kv head x 128 dims x 4 bytes = 2 KiB per moved row, plus 8 bytes of
        # move list (the list rounded up to 256 bytes): (16 MiB - 256) / 2056 = 8160 moves fit. A sequence whose table
        # repeats one free block 520 times covers 8320 rows; moving rows 1..8200 down by one needs 8200 moves.
        limit = ((16 << 20) - 256) // (2 * 2 * 1 * 128 * 4 + 8)
        assert limit == 8160
        be.step([gck.Work(3, [1], 0, [31] * 520, 0)])
        assert commit(3, 0, [j + 1 for j in range(8200)]) == gck.E_ARG
        msg = (be.L.gc_last_error(be.h) or b"").decode()
        assert f"at most {limit} moved rows" in msg, msg
        # the refusal left the handle usable
        assert np.array_equal(be.step([gck.Work(1, [nxt], pos, ta, 1)]).shape, (1, be.vocab_size))
