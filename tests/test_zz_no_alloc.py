"""The allocation-free entry point (jdg_logits_argmax_noalloc), checked against the existing
packed/f32 product entry point (jdg_qmatvec).

Callers that cannot call cudaMalloc -- every device buffer they hold comes from another
allocator -- use this call for the vocabulary projection and greedy pick.  The test hands it
buffers from PyTorch's allocator, calls it twice in a row with different sizes (the shared
scratch must be left ready for the next call), and compares the logits with jdg_qmatvec on
the same inputs and the index with the first maximum of those logits.  This file sorts last
so that a run stopping at its first failure has already run every other test.  The argument
checks (sizes past the scratch, misaligned views) are tested on the CPU through
jdg_logits_argmax_noalloc_check, the same function the entry point runs first, so no test
ever hands the launch path a pointer it must reject (tests/test_abi.py).
"""
import ctypes as C

import numpy as np
import pytest

from _util import LOGIT_TOL

pytestmark = pytest.mark.gpu


def _fn(jd):
    f = jd.lib().jdg_logits_argmax_noalloc
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
    f.restype = C.c_int
    return f


def test_noalloc_matches_existing_entry_point(jd):
    import torch
    f = _fn(jd)
    ctx = jd.Context(0)
    try:
        for trial, (rows, cols) in enumerate([(8256, 768), (32000, 2048)]):
            rng = np.random.default_rng(100 + trial)
            W = (rng.standard_normal((rows, cols)) * 0.02).astype(np.float32)
            x = rng.standard_normal(cols).astype(np.float32)
            ref = jd.qmatvec(ctx, W.view(np.uint8).reshape(rows, -1), jd.JD_F32, x, rows, cols)
            Wd = torch.from_numpy(W).cuda()
            xd = torch.from_numpy(x).cuda()
            lg = torch.full((rows,), float("nan"), device="cuda")
            am = torch.full((1,), -1, dtype=torch.int32, device="cuda")
            rc = f(Wd.data_ptr(), xd.data_ptr(), rows, cols, lg.data_ptr(), am.data_ptr(),
                   torch.cuda.current_stream().cuda_stream)
            assert rc == jd.JD_OK, jd.lib().jdg_last_error(None)
            torch.cuda.synchronize()
            got = lg.cpu().numpy()
            err = float(np.max(np.abs(got - ref)) / np.max(np.abs(ref)))
            assert err <= LOGIT_TOL * 1e-2, err
            assert int(am.item()) == int(np.argmax(got))
    finally:
        ctx.close()
