"""hxb_matmul_noalloc: the matmul for callers that cannot allocate device memory when they run it
(an engine that reserved all of HBM for its own pool, code running during CUDA-graph capture, an
application that budgets device memory once at start). Its Q8/Q4 activation scratch is a static
device array, so the test checks it against the allocating entry point hxb_matmul, bit for bit
(the tolerance of every matmul parity test here), on two calls in a row — the second call finds
the first call's leftovers in the shared array — and against the oracle (the CPU restatement of the
reference's matmul). This file is collected last on purpose: it loads no state from the other tests
and passes alone in a fresh process as well as after them."""
import ctypes as C

import numpy as np
import pytest

import hearth_b200 as hb
from hearth_b200 import native
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _weights(rng, dt, rows, cols):
    W = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
    if O.ref_lib() is not None:
        return O.ref_quantize(dt, W)
    rb = O.row_bytes(dt, cols)
    q = rng.integers(0, 256, (rows, rb), dtype=np.uint8)
    bs = 34 if dt == O.Q4 else 66
    for b in range(cols // 64):
        q[:, b * bs:b * bs + 2] = np.frombuffer(np.full(rows, 0.003, np.float16).tobytes(), np.uint8).reshape(rows, 2)
    return q


def test_noalloc_matmul_equals_hxb_matmul_on_two_calls(gpu):
    import torch
    L = hb.lib()
    rng = np.random.default_rng(20)
    cases = [(O.Q4, 96, 2048, 3), (O.Q8, 40, 768, 5), (O.Q4, 17, 7168, 1)]
    for call in range(2):
        for dt, rows, cols, T in cases:
            W = _weights(rng, dt, rows, cols)
            X = rng.standard_normal((T, cols)).astype(np.float32)
            want = native.matmul(dt, W, rows, cols, X)                 # allocating entry point
            assert np.array_equal(want.view(np.uint32), O.matmul(dt, W, rows, cols, X).view(np.uint32))
            Wd = torch.from_numpy(np.ascontiguousarray(W)).cuda()
            Xd = torch.from_numpy(X).cuda()
            Yd = torch.full((T, rows), float("nan"), dtype=torch.float32, device="cuda")
            rc = L.hxb_matmul_noalloc(dt, C.c_void_p(Wd.data_ptr()), rows, cols, C.c_void_p(Xd.data_ptr()), T,
                                      C.c_void_p(Yd.data_ptr()), None)
            assert rc == 0, hb.last_error()
            torch.cuda.synchronize()
            got = Yd.cpu().numpy()
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (call, dt, rows, cols, T)


def test_noalloc_rejects_more_than_the_scratch(gpu):
    import torch
    L = hb.lib()
    cols, T = 7168, 600           # 600 * 112 * 72 bytes > 4 MiB
    W = torch.zeros((4, cols // 64 * 34), dtype=torch.uint8, device="cuda")
    X = torch.zeros((T, cols), dtype=torch.float32, device="cuda")
    Y = torch.zeros((T, 4), dtype=torch.float32, device="cuda")
    rc = L.hxb_matmul_noalloc(O.Q4, C.c_void_p(W.data_ptr()), 4, cols, C.c_void_p(X.data_ptr()), T,
                              C.c_void_p(Y.data_ptr()), None)
    assert rc == -3
    assert "static scratch" in hb.last_error()
