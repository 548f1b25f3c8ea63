"""The reference's own pruner module driven through this library's binding.

A maintainer switches a reference checkout over by assigning
``ChannelPruner.update_rotatek = rotatek_b200.pruner.update_rotatek`` in
integrations/lmms_eval/models/model_utils/kv_pruning_utils.py (the binding
shown in INTEGRATION.md).  These tests load that unmodified module by path --
from baseline/_ref (an unmodified copy of the reference checkout kept beside
this repository, outside git) or from the checkout named by $ROTATEK_REFERENCE
-- apply the assignment, and check the contract the adapters rely on
(kv_pruning_utils.py:92-160): the 5-tuple return and the
``current_rotatek_R_partial`` / ``current_rotatek_delta_mu`` attributes.
"""
import importlib.util
import inspect
import os

import numpy as np
import pytest
import torch

from oracle import rotation as orot
from rotatek_b200 import pruner as b200_pruner

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
_REL = os.path.join("integrations", "lmms_eval", "models", "model_utils", "kv_pruning_utils.py")


def _module_path():
    for root in (os.environ.get("ROTATEK_REFERENCE"), os.path.join(REPO, "baseline", "_ref")):
        if root and os.path.isfile(os.path.join(root, _REL)):
            return os.path.join(root, _REL)
    return None


def load_reference_pruner():
    path = _module_path()
    if path is None:
        pytest.skip("no reference checkout: baseline/_ref or $ROTATEK_REFERENCE must hold "
                    "integrations/lmms_eval/models/model_utils/kv_pruning_utils.py")
    spec = importlib.util.spec_from_file_location("ref_kv_pruning_utils", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def patched_pruner_class():
    mod = load_reference_pruner()
    cls = mod.ChannelPruner
    original = cls.update_rotatek
    cls.update_rotatek = b200_pruner.update_rotatek
    return mod, cls, original


def test_binding_replaces_the_method_with_the_same_signature():
    mod, cls, original = patched_pruner_class()
    assert list(inspect.signature(original).parameters) == \
        list(inspect.signature(b200_pruner.update_rotatek).parameters)
    pr = cls(ratio=0.75, prompt_seqlen=32, query_seqlen=64)
    assert pr.update_rotatek.__func__ is b200_pruner.update_rotatek
    # the other methods of the reference's pruner are untouched
    assert cls.update_think is mod.ChannelPruner.update_think


@pytest.mark.parametrize("p,t,s", [(32, 64, 672), (0, 64, 200), (32, 0, 200), (500, 500, 300), (0, 0, 10)])
def test_span_split_matches_the_reference(p, t, s):
    """kv_pruning_utils.py:26-35 against pruner.split_spans on the same views."""
    mod = load_reference_pruner()
    pr = mod.ChannelPruner(ratio=0.75, prompt_seqlen=p, query_seqlen=t)
    keys = torch.arange(2 * 2 * s * 4, dtype=torch.float32).view(2, 2, s, 4)
    for a, b in zip(mod._split_spans(pr, keys), b200_pruner.split_spans(pr, keys)):
        assert a.shape == b.shape and torch.equal(a, b)


@pytest.mark.gpu
def test_reference_pruner_runs_the_b200_build(golden):
    """The patched reference pruner on the cfg1_fp32 fixture's inputs: the
    5-tuple and side attributes as the adapters read them, and the rotation
    matching update_rotatek's own (eigh) output."""
    _, cls, _ = patched_pruner_class()
    g = golden("cfg1_fp32")
    dev = "cuda"
    p, v, t = int(g["prompt_len"]), int(g["vision_len"]), int(g["text_len"])
    keys = torch.as_tensor(g["keys"]).to(dev)
    values = torch.as_tensor(g["values"]).to(dev)
    w = g["queries_window"].shape[2]
    queries = torch.zeros(keys.shape[0], g["queries_window"].shape[1], keys.shape[2], 128, device=dev)
    queries[:, :, -w:] = torch.as_tensor(g["queries_window"]).to(dev)
    pr = cls(ratio=float(g["ratio"]), prompt_seqlen=p, query_seqlen=t)
    kept, kv_prompt, kv_text, keep_mask, vals = pr.update_rotatek(keys, queries, values, None,
                                                                  int(g["num_kv_groups"]))
    keep = orot.keep_count(128, g["ratio"])
    assert kept.shape == (keys.shape[0], keys.shape[1], v, keep)
    assert torch.equal(kv_prompt, keys[:, :, :p]) and torch.equal(kv_text, keys[:, :, -t:])
    assert vals is values
    np.testing.assert_array_equal(keep_mask.cpu().numpy(), g["keep_mask"])
    R = pr.current_rotatek_R_partial.double().cpu().numpy()
    dm = pr.current_rotatek_delta_mu.double().cpu().numpy()
    assert orot.projector_distance(R, g["R_partial"]).max() < 1e-4
    np.testing.assert_allclose(dm, g["delta_mu"], atol=2e-4)
    # kept = K_vis . R with this R
    want = np.einsum("bhsd,bhdk->bhsk", g["keys"][:, :, p:p + v].astype(np.float64), R)
    np.testing.assert_allclose(kept.double().cpu().numpy(), want, rtol=0, atol=1e-4 * np.abs(want).max())
