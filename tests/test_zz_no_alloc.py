"""g4a_attend_static, the entry point for callers that cannot allocate device
memory when they attend (for example a server whose device memory is already
handed to its own pools). It keeps its scratch in a file-scope device array,
so it must give what the oracle (the reference's attend) and g4a_attend give,
call after call, while sharing that array. Collected last so that a failure
here stops a -x run only after every other test has run.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-4  # the decode tolerance used by the other attention tests


def test_static_scratch_attend_matches_attend(oracle):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import g4attn
    fn = g4attn.lib.g4a_attend_static
    vp = ctypes.c_void_p
    fn.argtypes = [vp, vp, vp, vp, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_float, vp]
    fn.restype = ctypes.c_int
    ctx = g4attn.Context(0)
    stream = torch.cuda.Stream()
    ctx.set_stream(stream.cuda_stream)
    r = np.random.default_rng(2468)
    # Consecutive calls on one stream share the array; the third repeats the
    # first shape after a different one has overwritten the scratch. Lengths
    # past 2016 rows use all 64 row ranges (more than 32 rows each), 5000 and
    # 4097 with a last 64-row block that is cut short.
    for hd, length in ((512, 628), (256, 1000), (512, 628), (256, 7), (512, 5000), (256, 4097), (512, 5000)):
        q_h = r.standard_normal(8 * hd).astype(np.float32) / np.float32(np.sqrt(hd))
        k_h = r.standard_normal((length, hd)).astype(np.float32)
        v_h = r.standard_normal((length, hd)).astype(np.float32)
        q, k, v = (torch.from_numpy(a).cuda() for a in (q_h, k_h, v_h))
        want = torch.empty(8 * hd, device="cuda")
        got = torch.full((8 * hd,), float("nan"), device="cuda")
        torch.cuda.synchronize()
        ctx.attend(q, k, v, 8, 1, 1.0, want)
        rc = fn(stream.cuda_stream, q.data_ptr(), k.data_ptr(), v.data_ptr(), length, 8, 1, hd, 1.0, got.data_ptr())
        assert rc == g4attn.OK
        stream.synchronize()
        ctx.sync()
        got_h = got.cpu().numpy()
        ref = oracle.attend(q_h, k_h, v_h, 8, 1, 1.0)
        assert float(np.max(np.abs(got_h - ref))) <= TOL, (hd, length, "vs oracle")
        assert float((got - want).abs().max()) <= TOL, (hd, length, "vs g4a_attend")
    x = torch.zeros(8 * 1024, device="cuda")
    rc = fn(stream.cuda_stream, x.data_ptr(), x.data_ptr(), x.data_ptr(), 4, 8, 1, 1024, 1.0, x.data_ptr())
    assert rc == g4attn.COMPUTE  # beyond the static scratch's 512 columns per head
    ctx.close()
