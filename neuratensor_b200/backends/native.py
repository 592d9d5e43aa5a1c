"""The native-kernel switch and the drop-in patch for an installed NeuraTensor.

``patch_reference(neuratensor)`` installs the B200 forwards on the
reference package's own classes (``LIFLayer``, ``AdaptiveLIFLayer``,
``SelectiveSSMLayer``, ``FusedSpikeBlock``, ``SlidingWindowAttention``,
``NeuraTensorModel``), so an existing NeuraTensor user keeps constructing
models, presets and engines exactly as before while the hot path runs on
libneuratensor_native.so.  Parameter and submodule names are identical in
both packages, which is what makes the methods interchangeable.

Each class gets (a) the methods listed in ``_OVERRIDES``, replacing the
reference's own, and (b) every helper the B200 class defines that the
reference class lacks (workspace caches, packed weights, captured graphs).
The patch is all-or-nothing: every target class is looked up and every
assignment planned before the first one is made, so a reference package
that lacks one of the classes is left untouched.  ``unpatch_reference``
restores each class exactly (methods put back, added helpers removed).
With the switch on there is no fallback: a CPU tensor or a missing library
raises.
"""
from __future__ import annotations

import importlib
import os
from typing import Dict, List, Tuple

_MISSING = object()
# (class, attribute) -> the reference's own value (or _MISSING when the
# attribute was added by the patch)
_PATCHED: Dict[Tuple[type, str], object] = {}

# class name -> (module under neuratensor.core, methods replaced even though the reference defines them)
_OVERRIDES = {
    "LIFLayer": ("snn", ("forward",)),
    "AdaptiveLIFLayer": ("snn", ("forward",)),
    "SelectiveSSMLayer": ("ssm", ("forward",)),
    "FusedSpikeBlock": ("fused", ("forward", "_sparse_out_proj")),
    "SlidingWindowAttention": ("model", ("forward",)),
    "NeuraTensorModel": ("model", ("forward", "generate")),
}

# attributes never copied from the B200 classes (object plumbing and
# constructors: the reference's own stay in charge of building modules)
_SKIP = {"__init__", "__module__", "__qualname__", "__doc__", "__dict__", "__weakref__", "__annotations__",
         "__firstlineno__", "__static_attributes__", "_init_weights", "extra_repr", "info",
         "count_parameters", "count_trainable_parameters", "from_preset", "_state_cls"}


def native_available() -> bool:
    """True when the shared library is present and loads."""
    from .. import native
    try:
        native.load()
        return True
    except Exception:
        return False


def _b200_class(module: str, name: str) -> type:
    return getattr(importlib.import_module(f"neuratensor_b200.core.{module}"), name)


def _plan(nt_module) -> List[Tuple[type, str, object]]:
    """Every (reference class, attribute, new value) the patch assigns; raises before any change."""
    plan = []
    for cls_name, (mod, overrides) in _OVERRIDES.items():
        ref_mod = importlib.import_module(f"{nt_module.__name__}.core.{mod}")
        ref_cls = getattr(ref_mod, cls_name, None)
        if not isinstance(ref_cls, type):
            raise AttributeError(f"{ref_mod.__name__} has no class {cls_name}; nothing was patched")
        src = _b200_class(mod, cls_name)
        for name in overrides:
            if name not in src.__dict__:
                raise AttributeError(f"neuratensor_b200 {cls_name} lacks {name}")
            plan.append((ref_cls, name, src.__dict__[name]))
        for name, val in src.__dict__.items():
            if name in _SKIP or name in overrides or hasattr(ref_cls, name):
                continue
            plan.append((ref_cls, name, val))
        if cls_name == "FusedSpikeBlock":
            # returned states are the reference's own BlockState dataclass
            state_cls = getattr(ref_mod, "BlockState", None)
            if not isinstance(state_cls, type):
                raise AttributeError(f"{ref_mod.__name__} has no BlockState; nothing was patched")
            plan.append((ref_cls, "_state_cls", state_cls))
    return plan


def patch_reference(nt_module=None) -> None:
    """Route an imported ``neuratensor`` package's hot path through the B200 kernels."""
    if nt_module is None:
        import neuratensor as nt_module  # noqa: F811
    plan = _plan(nt_module)
    for cls, name, val in plan:
        key = (cls, name)
        if key not in _PATCHED:
            _PATCHED[key] = cls.__dict__.get(name, _MISSING)
        setattr(cls, name, val)


def unpatch_reference() -> None:
    """Restore the reference's own methods and remove the helpers the patch added."""
    for (cls, name), orig in list(_PATCHED.items()):
        if orig is _MISSING:
            if name in cls.__dict__:
                delattr(cls, name)
        else:
            setattr(cls, name, orig)
    _PATCHED.clear()


def is_patched() -> bool:
    return bool(_PATCHED)


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
