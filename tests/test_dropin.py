"""The drop-in: ``use_native`` on the reference package's own classes.

The reference package is found at ``baseline/_ref`` (an installed copy of
NeuraTensor 4.0.4 that travels with the repository) or under the directory
named by ``$NEURATENSOR_REFERENCE``; without either the tests skip and say so.

CPU: the patch installs and removes cleanly (every class restored exactly,
all-or-nothing when a class is missing).  GPU: the reference's own
``InferenceEngine.run`` and ``NeuraTensorModel.generate`` run on the B200
kernels through the patch and match the pico fp32 golden produced by the
reference itself (logits rtol 1e-4, per-layer spike rates).
"""
import importlib
import os
import sys
import types

import numpy as np
import pytest
import torch

from conftest import ROOT, load_golden


def _reference():
    cands = [os.path.join(ROOT, "baseline", "_ref"), os.environ.get("NEURATENSOR_REFERENCE", "")]
    for c in cands:
        if c and os.path.isdir(os.path.join(c, "neuratensor")):
            if c not in sys.path:
                sys.path.insert(0, c)
            os.environ.setdefault("NEURATENSOR_TELEMETRY", "0")
            return importlib.import_module("neuratensor")
    pytest.skip("reference package not importable (no baseline/_ref and no $NEURATENSOR_REFERENCE)")


_CLASSES = [("fused", "FusedSpikeBlock"), ("model", "NeuraTensorModel"), ("model", "SlidingWindowAttention"),
            ("snn", "LIFLayer"), ("snn", "AdaptiveLIFLayer"), ("ssm", "SelectiveSSMLayer")]


def _snapshot(nt):
    out = {}
    for mod, name in _CLASSES:
        cls = getattr(importlib.import_module(f"neuratensor.core.{mod}"), name)
        out[cls] = dict(vars(cls))
    return out


def test_patch_round_trip_restores_every_class():
    nt = _reference()
    from neuratensor_b200.backends import native as bn
    before = _snapshot(nt)
    bn.use_native(True, nt)
    try:
        from neuratensor.core import fused, model
        assert model.SlidingWindowAttention.forward is not before[model.SlidingWindowAttention]["forward"]
        assert fused.FusedSpikeBlock._state_cls is fused.BlockState
        assert hasattr(model.NeuraTensorModel, "forward_device")
        bn.use_native(True, nt)                 # idempotent: originals are kept from the first patch
    finally:
        bn.use_native(False)
    after = _snapshot(nt)
    for cls, d in before.items():
        assert d.keys() == after[cls].keys(), (cls.__name__, set(d) ^ set(after[cls]))
        for k, v in d.items():
            assert after[cls][k] is v, (cls.__name__, k)
    assert not bn.is_patched()


def test_patch_is_all_or_nothing():
    nt = _reference()
    from neuratensor_b200.backends import native as bn
    before = _snapshot(nt)
    # a stand-in package whose core lacks SlidingWindowAttention
    fake = types.ModuleType("fake_nt")
    core = types.ModuleType("fake_nt.core")
    sys.modules["fake_nt"], sys.modules["fake_nt.core"] = fake, core
    for mod in ("fused", "snn", "ssm", "model"):
        real = importlib.import_module(f"neuratensor.core.{mod}")
        m = types.ModuleType(f"fake_nt.core.{mod}")
        m.__dict__.update({k: v for k, v in vars(real).items() if k != "SlidingWindowAttention"})
        sys.modules[f"fake_nt.core.{mod}"] = m
    try:
        with pytest.raises(AttributeError, match="SlidingWindowAttention"):
            bn.patch_reference(fake)
        assert not bn.is_patched()
        after = _snapshot(nt)
        for cls, d in before.items():
            assert d.keys() == after[cls].keys()
    finally:
        for k in [k for k in sys.modules if k == "fake_nt" or k.startswith("fake_nt.")]:
            del sys.modules[k]


@pytest.mark.gpu
def test_reference_engine_runs_on_the_kernels():
    """The reference's own engine and model classes, patched, against the reference's golden run."""
    nt = _reference()
    from neuratensor_b200 import native
    from neuratensor_b200.backends import native as bn
    from neuratensor.core.fused import BlockState
    from neuratensor.core.model import NeuraTensorModel
    from neuratensor.config.presets import get_preset
    from neuratensor.inference.engine import InferenceEngine

    g = load_golden("pico_fp32.npz")
    torch.manual_seed(0)
    model = NeuraTensorModel(get_preset("pico"))          # seed 0 -> the golden's weights
    ids = torch.from_numpy(g["ids"]).long()
    bn.use_native(True, nt)
    try:
        eng = InferenceEngine(model, device="cuda", dtype=torch.float32)
        before = native.launch_count()
        res = eng.run(ids, reset_state=True)
        assert native.launch_count() > before, "no native kernel launched"
        logits = res.logits[0].float().cpu().numpy()
        np.testing.assert_allclose(logits[g["logits_row_idx"]], g["logits_rows"], rtol=1e-4, atol=1e-5)
        np.testing.assert_array_equal(logits.argmax(-1), g["logit_argmax"])
        np.testing.assert_allclose(res.metrics["per_layer_spike_rate"], g["per_layer_rate"], rtol=0, atol=2e-4)
        assert all(isinstance(s, BlockState) for s in res.states)
        # streaming continuation and generation through the reference's engine
        out = eng.generate(ids[:, :8], max_new_tokens=4, top_k=1)
        assert out.shape == (1, 12)
    finally:
        bn.use_native(False)
