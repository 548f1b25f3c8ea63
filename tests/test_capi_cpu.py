"""The C-ABI library without a GPU: it loads, exports every function the
header declares, and rejects bad arguments with the reference's messages
before touching the device."""
import ctypes
import os
import re

import pytest
import torch

from rotatek_b200 import _lib
from rotatek_b200.kernels import full_channel_decode, rotatek_decode

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "rotatek_b200.h")


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_lib.LIB_PATH):
        from rotatek_b200.csrc import build
        build.build()
    return _lib.load()


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rtk_[a-z0-9_]+)\s*\(", text)))


def test_header_symbols_exported(lib):
    names = header_functions()
    assert "rtk_rotatek_decode" in names and "rtk_full_channel_decode" in names
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_abi_version(lib):
    assert lib.rtk_abi_version() == 1


def _fake(shape, dtype=1, data=0x1000):
    d = _lib.RtkTensor()
    d.data = data
    d.dtype = dtype
    d.ndim = len(shape)
    stride = 1
    for i in reversed(range(len(shape))):
        d.shape[i] = shape[i]
        d.stride[i] = stride
        stride *= shape[i]
    return ctypes.byref(d)


def test_c_validation_messages(lib):
    q, R, dm = _fake((2, 8, 128)), _fake((2, 2, 128, 32)), _fake((2, 2, 128))
    kf, vf, mask = _fake((2, 2, 10, 128)), _fake((2, 2, 10, 128)), _fake((2, 10), dtype=3)
    ks, vs, out = _fake((2, 2, 50, 32)), _fake((2, 2, 50, 128)), _fake((2, 1, 8, 128))

    def call(**kw):
        a = dict(q=q, R=R, dm=dm, kf=kf, vf=vf, mask=mask, ks=ks, vs=vs, g=4, out=out)
        a.update(kw)
        code = lib.rtk_rotatek_decode(a["q"], a["R"], a["dm"], a["kf"], a["vf"], a["mask"],
                                      a["ks"], a["vs"], a["g"], a["out"], None, 0, None)
        return code, lib.rtk_last_error().decode()

    assert call(q=_fake((8, 128))) == (1, "q_full must be [B, H_q, D]")
    assert call(R=_fake((2, 128, 32))) == (1, "R_partial must be [B, H_kv, D, D_keep]")
    assert call(mask=_fake((2, 10), dtype=1)) == (1, "mask_full must be uint8")
    assert call(g=2) == (1, "R_partial H_kv=2 but H_q=8, num_kv_groups=2")
    assert call(vs=_fake((2, 2, 49, 128)))[1] == "v_sparse must be [B, H_kv, S_sparse, D]"
    assert call(out=_fake((2, 8, 64)))[1] == "out must be [B, H_q, D] or [B, 1, H_q, D]"
    code, msg = call()                      # valid shapes, but no workspace
    assert code == _lib.RTK_ERR_WORKSPACE or code == _lib.RTK_ERR_CUDA, (code, msg)
    code = lib.rtk_full_channel_decode(_fake((2, 8, 128)), _fake((2, 2, 10, 64)),
                                       _fake((2, 2, 10, 128)), 4, out, None, 0, None)
    assert (code, lib.rtk_last_error().decode()) == (1, "k/v head_dim must match q's")


def test_spark_validation_messages(lib):
    q, kf, vf = _fake((2, 8, 128)), _fake((2, 2, 10, 128)), _fake((2, 2, 10, 128))
    kk, idx, mean = _fake((2, 2, 50, 32)), _fake((2, 2, 50, 32), dtype=3), _fake((2, 2, 50, 1))
    vs, out = _fake((2, 2, 50, 128)), _fake((2, 1, 8, 128))

    def call(**kw):
        a = dict(q=q, kf=kf, vf=vf, mask=None, kk=kk, idx=idx, mean=mean, vs=vs, g=4, out=out)
        a.update(kw)
        code = lib.rtk_spark_decode(a["q"], a["kf"], a["vf"], a["mask"], a["kk"], a["idx"], a["mean"],
                                    a["vs"], a["g"], a["out"], None, 0, None)
        return code, lib.rtk_last_error().decode()

    assert call(q=_fake((8, 128))) == (1, "q_full must be [B, H_q, D]")
    assert call(g=3) == (1, "H_q=8 is not H_kv=2 * num_kv_groups=3")
    assert call(idx=_fake((2, 2, 50, 32)))[1] == "keep_idx must be a uint8 [B, H_kv, S_sparse, D_keep]"
    assert call(mean=_fake((2, 2, 50)))[1] == "pruned_mean must be [B, H_kv, S_sparse, 1]"
    assert call(vs=_fake((2, 2, 49, 128)))[1] == "v_sparse must be [B, H_kv, S_sparse, D]"
    assert call(mean=_fake((2, 2, 50, 1), dtype=2))[1].startswith("all tensors but mask_full and keep_idx")
    code, _ = call()                        # valid shapes, but no workspace
    assert code in (_lib.RTK_ERR_WORKSPACE, _lib.RTK_ERR_CUDA)
    code = lib.rtk_spark_pack(_fake((2, 2, 50, 64), dtype=3), _fake((2, 2, 50, 32), dtype=3), None, None)
    assert (code, lib.rtk_last_error().decode()) == (2, "keep_mask needs D = 128 with a unit channel stride")
    code = lib.rtk_spark_pack(_fake((2, 2, 50, 128), dtype=3), _fake((2, 2, 49, 32), dtype=3), None, None)
    assert (code, lib.rtk_last_error().decode()) == (1, "keep_idx_out must be a uint8 [B, H_kv, S, D_keep]")


def test_key_projection_validation(lib):
    """rtk_key_projection rejects bad shapes before any device work."""
    bf = 1   # RTK_BF16
    x, w, bias = _fake((2, 300, 256), bf), _fake((256, 256), bf), _fake((256,), bf)
    cs = _fake((2, 300, 128), bf)
    keys, cov, ksum = _fake((2, 2, 300, 128), bf), _fake((2, 2, 128, 128), 0), _fake((2, 2, 128), 0)

    def call(**kw):
        a = dict(x=x, w=w, bias=bias, cos=cs, sin=cs, vs=20, vl=230, keys=keys, cov=cov, ksum=ksum)
        a.update(kw)
        code = lib.rtk_key_projection(a["x"], a["w"], a["bias"], a["cos"], a["sin"], a["vs"], a["vl"],
                                      a["keys"], a["cov"], a["ksum"], ctypes.c_void_p(0x1000), 256, None)
        return code, lib.rtk_last_error().decode()

    assert call(x=_fake((300, 256), bf)) == (1, "hidden_states must be [B, S, hidden]")
    assert call(x=_fake((2, 300, 256), 0))[0] == _lib.RTK_ERR_UNSUPPORTED
    assert call(w=_fake((200, 256), bf)) == (1, "w_k must be [H_kv * 128, hidden] in the hidden states' dtype")
    assert call(bias=_fake((128,), bf))[1].startswith("bias must be a contiguous [H_kv * 128] vector")
    assert call(cos=_fake((2, 299, 128), bf))[1].startswith("cos / sin must be [B or 1, S, 128]")
    assert call(vl=290) == (1, "the visual span [20, 310) is not inside [0, 300)")
    assert call(keys=_fake((2, 2, 300, 64), bf))[1].startswith("keys_out must be [B, H_kv, S, 128]")
    assert call(cov=_fake((2, 2, 128, 128), bf))[1] == "cov_out must be a contiguous float32 [B, H_kv, 128, 128]"
    assert call(x=_fake((2, 300, 100), bf), w=_fake((256, 100), bf))[0] == _lib.RTK_ERR_UNSUPPORTED


def test_python_errors_match_reference_and_no_cpu_fallback():
    q = torch.zeros(2, 8, 128)
    R = torch.zeros(2, 2, 128, 32)
    kf = torch.zeros(2, 2, 10, 128)
    mask = torch.ones(2, 10, dtype=torch.uint8)
    ks, vs = torch.zeros(2, 2, 50, 32), torch.zeros(2, 2, 50, 128)
    kw = dict(q_full=q, R_partial=R, delta_mu=None, k_full=kf, v_full=kf, mask_full=mask,
              k_sparse=ks, v_sparse=vs, num_kv_groups=4)
    with pytest.raises(ValueError, match=r"q_full must be \[B, H_q, D\]"):
        rotatek_decode(**{**kw, "q_full": q[0]})
    with pytest.raises(ValueError, match="mask_full must be uint8"):
        rotatek_decode(**{**kw, "mask_full": mask.float()})
    with pytest.raises(ValueError, match="R_partial H_kv=2 but H_q=8, num_kv_groups=2"):
        rotatek_decode(**{**kw, "num_kv_groups": 2})
    with pytest.raises(ValueError, match=r"H_q=8 is not H_kv=2 \* num_kv_groups=3"):
        rotatek_decode(**{**kw, "num_kv_groups": 3})
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        rotatek_decode(**kw)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        full_channel_decode(q, kf, kf, 4)


def test_decode_sm_reserve_validation(lib):
    """rtk_decode_set_sm_reserve takes 0..64 SMs; anything else is refused
    before it changes the setting."""
    assert lib.rtk_decode_set_sm_reserve(-1) == _lib.RTK_ERR_INVALID
    assert "sms must be in [0, 64]" in lib.rtk_last_error().decode()
    assert lib.rtk_decode_set_sm_reserve(65) == _lib.RTK_ERR_INVALID
    assert lib.rtk_decode_set_sm_reserve(0) == _lib.RTK_OK
    with pytest.raises(ValueError, match="sms must be"):
        _lib.set_decode_sm_reserve(100)
