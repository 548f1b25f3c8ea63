"""CPU oracle for the RotateK hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs may import this package; the product (``rotatek_b200``) never does, and
has no CPU fallback.

Contents
  decode.py     numpy float64 restatement of the decode attention of
                rotatek/kernels/fused_decode.py and full_channel_flash_decoding.py
  rotation.py   numpy restatement of ChannelPruner.update_rotatek
                (integrations/lmms_eval/models/model_utils/kv_pruning_utils.py:92-160)
                with the exact-eigh solver, including the bf16 roundings the
                reference performs on bf16 inputs
  bf16.py       round-to-nearest-even float32 -> bfloat16 emulation in numpy
  eager_torch.py the reference's eager PyTorch path restated in torch (CPU),
                timed as the CPU baseline

Pinning: the reference ships no golden vectors or tests.  The oracle is pinned
against outputs of the reference's own code run in the build container
(tests/golden/make_golden.py runs the `paper` Triton kernels under
TRITON_INTERPRET=1 and `update_rotatek` with ROTATEK_SOLVER=eigh), committed as
fixtures under tests/golden/.
"""
