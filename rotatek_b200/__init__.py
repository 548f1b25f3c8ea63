"""rotatek_b200 -- the RotateK hot path on B200 (sm_100a).

Same Python surface as the reference package ``rotatek``:

    rotation.power_iteration_gpu   top-k eigenbasis of the Key covariance
    rotation.build_rotation        fused prefill builder (covariance -> eigh -> rotate)
    kernels.rotatek_decode         decode over rotated-truncated visual Keys
    kernels.full_channel_decode    full-width split-K decode

backed by the hand-written CUDA kernels of ``librotatek_b200.so`` (C ABI:
include/rotatek_b200.h).  There is no Triton and no CPU fallback.
"""
from rotatek_b200.kernels import ROTATEK_KERNEL, full_channel_decode, rotatek_decode

__all__ = ["ROTATEK_KERNEL", "full_channel_decode", "rotatek_decode"]
