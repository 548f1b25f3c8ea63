"""rtk_rotatek_decode_static: the allocation-free decode entry point.

Callers such as a serving runtime that owns all of HBM, or a foreign-language
binding that only forwards tensor pointers, cannot give this library a
workspace.  This entry point keeps its scratch in one fixed device array
instead.  The test calls it through the C ABI twice in a row and compares each
result with the workspace entry point's (the tolerance of the decode tests),
then checks that over-sized shapes are refused.  This file is collected last,
and passes alone in a fresh process as well as after the other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

from rotatek_b200 import _lib, synthetic as syn
from rotatek_b200.kernels import rotatek_decode

pytestmark = pytest.mark.gpu


def _static_decode(d, out):
    lib = _lib.load()
    D = _lib.describe
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return lib.rtk_rotatek_decode_static(
        D(d.q_full), D(d.R_partial), D(d.delta_mu), D(d.k_full), D(d.v_full), D(d.mask_full),
        D(d.k_sparse), D(d.v_sparse), d.num_kv_groups, D(out), stream)


@pytest.mark.parametrize("dtype,B,Hq,Hkv,Sv,Sf", [
    (torch.bfloat16, 32, 28, 4, 15360, 640),   # benchmark config 2 (tensor-core kernel)
    (torch.float32, 2, 8, 2, 576, 96),         # config-1 shape (generic kernel)
])
def test_static_entry_matches_workspace_entry(dtype, B, Hq, Hkv, Sv, Sf):
    d = syn.make_decode(B, Hq, Hkv, Sv, Sf, keep=32, seed=77, device="cuda", dtype=dtype)
    want, _, _ = rotatek_decode(**d.as_kwargs())
    atol, rtol = {torch.float32: (1e-5, 1e-5), torch.bfloat16: (2e-3, 2.0 ** -8)}[dtype]
    for _ in range(2):                              # two calls in a row share the scratch
        out = torch.full((B, 1, Hq, 128), float("nan"), dtype=dtype, device="cuda")
        assert _static_decode(d, out) == _lib.RTK_OK, _lib.load().rtk_last_error()
        got = out.float().cpu().numpy()
        ref = want.float().cpu().numpy()
        assert np.all(np.abs(got - ref) <= atol + rtol * np.abs(ref))
        assert _lib.read_static_status() == 0       # no bounded wait gave up
    torch.cuda.synchronize()


def test_static_entry_rejects_oversized_shapes_and_bad_input():
    lib = _lib.load()
    # 4096 units x 148 CTAs of partials is far beyond the 16 MiB static scratch
    d = syn.make_decode(512, 64, 8, 64, 32, keep=32, seed=5, device="cuda", dtype=torch.bfloat16)
    out = torch.empty((512, 1, 64, 128), dtype=torch.bfloat16, device="cuda")
    assert _static_decode(d, out) == _lib.RTK_ERR_WORKSPACE
    assert "static scratch holds" in lib.rtk_last_error().decode()
    bad = syn.make_decode(1, 8, 2, 64, 8, keep=32, seed=6, device="cuda", dtype=torch.bfloat16)
    bad.num_kv_groups = 2                          # H_q / groups != H_kv
    assert _static_decode(bad, torch.empty((1, 1, 8, 128), dtype=torch.bfloat16,
                                           device="cuda")) == _lib.RTK_ERR_INVALID
    assert "R_partial H_kv=2 but H_q=8" in lib.rtk_last_error().decode()
