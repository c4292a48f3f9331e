"""gck_commit_static: the tree-verify commit for callers that may not allocate device memory while they run (a server
that reserves the GPU's memory at start-up, or one bound to a fixed memory budget). It does what gc_commit does with
its scratch in a fixed 16 MiB array inside the library, so it must leave exactly the KV rows gc_commit leaves.

Two sequences get the same prompt and the same draft trees; after each verify, one commits with gc_commit, the other
with gck_commit_static, and both then decode the same token: their logits must agree (within the tolerance the parity
tests use; the kernels are the same, so they are in fact identical). Two verify/commit rounds run in a row, so the
second call finds the array holding the first call's contents. This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

from goethe_engine_b200 import build, gck, synth
from helpers import SMALL128, TOL_F16, TOL_FP8, assert_logits_close, model

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kv", ["f16", "fp8"])
def test_static_commit_matches_gc_commit_twice(tmp_path, kv):
    build.build()
    spec = synth.Spec(**SMALL128, wtype="q4_k", seed=21)
    pack, ws = model(tmp_path, spec, ncol=8, maxctx=512, kv=kv)
    with gck.Backend(pack, ws, pool_blocks=32) as be:
        fn = be.L.gck_commit_static
        fn.restype = C.c_int
        fn.argtypes = [C.c_void_p, C.c_uint64, C.c_uint32, C.POINTER(C.c_uint32), C.c_uint32]
        tol = TOL_F16 if kv == "f16" else TOL_FP8
        prompt = [int(x) for x in np.random.default_rng(4).integers(1, 500, 13)]
        ta, tb = list(range(0, 8)), list(range(8, 16))
        be.step([gck.Work(1, prompt, 0, ta, 0), gck.Work(2, prompt, 0, tb, 0)])
        pos = len(prompt)
        rounds = [([40, 41, 42, 43, 44, 45], [-1, 0, 0, 1, 2, 4], [0, 2, 4, 5]),
                  ([50, 51, 52, 53, 54], [-1, 0, 1, 1, 3], [0, 1, 3, 4])]
        for toks, parents, path in rounds:
            va = be.step([gck.Work(1, toks, pos, ta, len(toks), parents=parents)])
            vb = be.step([gck.Work(2, toks, pos, tb, len(toks), parents=parents)])
            assert np.array_equal(va, vb)
            be.commit(1, pos, path)
            arr = (C.c_uint32 * len(path))(*path)
            rc = fn(be.h, 2, pos, arr, len(path))
            assert rc == 0, (be.L.gc_last_error(be.h) or b"").decode()
            pos += len(path)
            nxt = toks[path[-1]]
            a = be.step([gck.Work(1, [nxt], pos, ta, 1)])
            b = be.step([gck.Work(2, [nxt], pos, tb, 1)])
            assert_logits_close(b, a, tol)
            pos += 1
        # an unknown sequence is an error code, as with gc_commit
        one = (C.c_uint32 * 2)(0, 1)
        assert fn(be.h, 99, 0, one, 2) == gck.E_STATE
