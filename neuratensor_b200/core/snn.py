"""LIF spiking layers with the B200 kernels behind their forward.

Interface mirror of NeuraTensor's ``neuratensor/core/snn.py``: the same
classes, constructor arguments, parameter / buffer names and initial values,
so state_dicts load unchanged.  ``forward`` runs ``nt_lif_scan`` (the
sequential LIF recurrence of ``_lif_sequential_scan``, snn.py:167-182; the
T=1 step of snn.py:64-75 is the same recurrence with one step).  The
chunked-scan switch (``use_chunked``, snn.py:231,296-302) is accepted for
compatibility; the kernel always evaluates the exact sequential recurrence,
which is what the reference computes by default.

Inference only: the surrogate gradient (snn.py:27-59) is a training feature
and is not provided, so these modules refuse to run with grad enabled.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
from torch import Tensor

from .. import native


def _no_grad_check(module: nn.Module, *ts: Optional[Tensor]) -> None:
    """Outputs never carry autograd history; refuse inputs that ask for gradients."""
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in ts):
        raise RuntimeError(f"{type(module).__name__}: the B200 kernels implement the inference path only "
                           "(no backward); detach the inputs or run under torch.no_grad()")


class LIFLayer(nn.Module):
    """Leaky integrate-and-fire layer (snn.py:187-322).

    V(t) = beta*V(t-1) + I(t);  S(t) = V(t) >= theta;  V(t) -= theta*S(t).
    beta = sigmoid(beta_logit) per neuron; theta fixed per neuron.
    """

    def __init__(self, size: int, beta_init: float = 0.9, threshold: float = 1.0, learn_beta: bool = True,
                 surrogate_slope: float = 10.0, dropout: float = 0.0, use_chunked: bool = False,
                 chunk_size: int = 64, multi_threshold: bool = False) -> None:
        super().__init__()
        self.size = size
        self.surrogate_slope = surrogate_slope
        self.use_chunked = use_chunked
        self.chunk_size = chunk_size
        logit = math.log(beta_init / (1.0 - beta_init))
        init = torch.full((size,), logit)
        if learn_beta:
            self.beta_logit = nn.Parameter(init)
        else:
            self.register_buffer("beta_logit", init)
        if multi_threshold:
            # thirds of the population at theta, 1.5*theta and 2*theta (snn.py:249-254)
            scale = torch.ones(size)
            k = size // 3
            scale[k:2 * k] = 1.5
            scale[2 * k:] = 2.0
            self.register_buffer("threshold", threshold * scale)
        else:
            self.register_buffer("threshold", torch.full((size,), threshold))
        self.drop = nn.Dropout(dropout) if dropout > 0.0 else None

    @property
    def beta(self) -> Tensor:
        return torch.sigmoid(self.beta_logit)

    def forward(self, x: Tensor, membrane: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
        """x [B, T, size] -> (spikes [B, T, size] as 0/1 in x.dtype, membrane [B, size])."""
        if x.shape[-1] != self.size:
            raise AssertionError(f"Expected size={self.size}, got {x.shape[-1]}")
        _no_grad_check(self, x, membrane)
        with torch.no_grad():
            return native.lif_scan(x, self.beta.to(x.dtype), self.threshold.to(x.dtype), membrane)

    def extra_repr(self) -> str:
        return f"size={self.size}, scan=native"


class AdaptiveLIFLayer(nn.Module):
    """LIF with per-neuron thresholds theta = softplus(threshold_raw) (snn.py:327-422)."""

    def __init__(self, size: int, beta_init: float = 0.9, threshold_init: float = 1.0, learn_beta: bool = True,
                 surrogate_slope: float = 10.0, dropout: float = 0.0, use_chunked: bool = False,
                 chunk_size: int = 64) -> None:
        super().__init__()
        self.size = size
        self.surrogate_slope = surrogate_slope
        self.use_chunked = use_chunked
        self.chunk_size = chunk_size
        logit = math.log(beta_init / (1.0 - beta_init))
        init = torch.full((size,), logit)
        if learn_beta:
            self.beta_logit = nn.Parameter(init)
        else:
            self.register_buffer("beta_logit", init)
        self.threshold_raw = nn.Parameter(torch.full((size,), math.log(math.exp(threshold_init) - 1.0)))
        self.drop = nn.Dropout(dropout) if dropout > 0.0 else None

    @property
    def beta(self) -> Tensor:
        return torch.sigmoid(self.beta_logit)

    @property
    def threshold(self) -> Tensor:
        return nn.functional.softplus(self.threshold_raw)

    def forward(self, x: Tensor, membrane: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
        if x.shape[-1] != self.size:
            raise AssertionError(f"Expected size={self.size}, got {x.shape[-1]}")
        _no_grad_check(self, x, membrane)
        with torch.no_grad():
            return native.lif_scan(x, self.beta.to(x.dtype), self.threshold.to(x.dtype), membrane)
