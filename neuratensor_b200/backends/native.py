"""The native-kernel switch and the drop-in patch for an installed NeuraTensor.

``patch_reference(neuratensor)`` installs the B200 forwards on the
reference package's own classes (``LIFLayer``, ``SelectiveSSMLayer``,
``FusedSpikeBlock``, ``NeuraTensorModel``), so an existing NeuraTensor user
keeps constructing models, presets and engines exactly as before while the
hot path runs on libneuratensor_native.so.  Parameter names are identical
in both packages, which is what makes the methods interchangeable.  With the
switch on there is no fallback: a CPU tensor or a missing library raises.
"""
from __future__ import annotations

import os
from typing import Dict, Optional

_PATCHED: Dict[tuple, object] = {}


def native_available() -> bool:
    """True when the shared library is present and loads."""
    from .. import native
    try:
        native.load()
        return True
    except Exception:
        return False


def _methods():
    from ..core import fused, model, snn, ssm
    return {
        "LIFLayer": {"forward": snn.LIFLayer.forward},
        "AdaptiveLIFLayer": {"forward": snn.AdaptiveLIFLayer.forward},
        "SelectiveSSMLayer": {"forward": ssm.SelectiveSSMLayer.forward,
                              "packed_proj_weight": ssm.SelectiveSSMLayer.packed_proj_weight},
        "FusedSpikeBlock": {"forward": fused.FusedSpikeBlock.forward,
                            "forward_native": fused.FusedSpikeBlock.forward_native,
                            "_native_weights": fused.FusedSpikeBlock._native_weights,
                            "_sparse_out_proj": fused.FusedSpikeBlock._sparse_out_proj},
        "SlidingWindowAttention": {"forward": model.SlidingWindowAttention.forward,
                                   "forward_native": model.SlidingWindowAttention.forward_native,
                                   "forward_torch": model.SlidingWindowAttention.forward_torch},
        "NeuraTensorModel": {"forward": model.NeuraTensorModel.forward,
                             "forward_device": model.NeuraTensorModel.forward_device,
                             "_workspace": model.NeuraTensorModel._workspace,
                             "metrics_from_counts": model.NeuraTensorModel.metrics_from_counts},
    }


def patch_reference(nt_module=None) -> None:
    """Route an imported ``neuratensor`` package's hot path through the B200 kernels."""
    if nt_module is None:
        import neuratensor as nt_module  # noqa: F401
    from neuratensor.core import fused as rf, model as rm, snn as rs, ssm as rss
    owners = {"LIFLayer": rs, "AdaptiveLIFLayer": rs, "SelectiveSSMLayer": rss, "FusedSpikeBlock": rf,
              "NeuraTensorModel": rm}
    for cls_name, meths in _methods().items():
        cls = getattr(owners[cls_name], cls_name)
        for name, fn in meths.items():
            key = (cls, name)
            if key not in _PATCHED:
                _PATCHED[key] = cls.__dict__.get(name, None)
            setattr(cls, name, fn)


def unpatch_reference() -> None:
    """Restore the reference's own methods."""
    for (cls, name), orig in list(_PATCHED.items()):
        if orig is None:
            delattr(cls, name)
        else:
            setattr(cls, name, orig)
    _PATCHED.clear()


def use_native(enable: bool = True, nt_module=None) -> None:
    """Switch an installed NeuraTensor between its PyTorch path and the B200 kernels.

    ``NEURATENSOR_NATIVE=1`` in the environment has the same effect at import
    of this package when ``neuratensor`` is importable.
    """
    if enable:
        patch_reference(nt_module)
    else:
        unpatch_reference()


if os.environ.get("NEURATENSOR_NATIVE") == "1":  # pragma: no cover - opt-in hook
    try:
        use_native(True)
    except ImportError:
        pass
