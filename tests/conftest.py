import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
os.environ.setdefault("NEURATENSOR_TELEMETRY", "0")

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


def load_golden(name):
    return dict(np.load(os.path.join(GOLDEN, name), allow_pickle=False))


def gget(d, key):
    """Golden value as float32 (bf16 fixtures are stored as raw uint16 under key + '_bf16')."""
    from oracle.neuratensor_oracle import bf16_from_bits
    if key + "_bf16" in d:
        return bf16_from_bits(d[key + "_bf16"])
    return d[key]


def unbits(bits, shape):
    shape = tuple(int(s) for s in shape)
    return np.unpackbits(bits, axis=-1)[..., : shape[-1]].reshape(shape).astype(np.float32)


def golden_params(d, prefix="w_"):
    """Fixture weights back to state_dict names (keys were stored with '.' -> '_')."""
    names = {
        "norm_weight": "norm.weight", "in_proj_weight": "in_proj.weight", "snn_beta_logit": "snn.beta_logit",
        "snn_threshold": "snn.threshold", "ssm_log_A": "ssm.log_A", "ssm_D": "ssm.D",
        "ssm_B_proj_weight": "ssm.B_proj.weight", "ssm_C_proj_weight": "ssm.C_proj.weight",
        "ssm_dt_proj_weight": "ssm.dt_proj.weight", "ssm_dt_proj_bias": "ssm.dt_proj.bias",
        "out_proj_weight": "out_proj.weight", "out_scale": "out_scale",
        "log_A": "log_A", "D": "D", "B_proj_weight": "B_proj.weight", "C_proj_weight": "C_proj.weight",
        "dt_proj_weight": "dt_proj.weight", "dt_proj_bias": "dt_proj.bias",
        "qkv_weight": "qkv.weight", "o_proj_weight": "o_proj.weight",
    }
    out = {}
    for k in d:
        if not k.startswith(prefix):
            continue
        base = k[len(prefix):]
        if base.endswith("_bf16"):
            base = base[:-5]
        if base in names:
            out[names[base]] = gget(d, prefix + base)
    return out
