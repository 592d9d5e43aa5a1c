"""Selective SSM layer with the B200 kernels behind its forward.

Interface mirror of NeuraTensor's ``neuratensor/core/ssm.py``
(``SelectiveSSMLayer``, ssm.py:46-353): same constructor, parameters
(``log_A``, ``D``, ``B_proj``, ``C_proj``, ``dt_proj``) and initialisation
order, so seeded models and state_dicts match the reference.  ``forward``
runs ``nt_ssm_forward``: one tensor-core GEMM for the dt/B/C projections
(softplus fused in its epilogue), then the selective-scan kernel (ZOH
discretisation fused, state carried in registers).
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
from torch import Tensor

from .. import native
from .snn import _no_grad_check


def _hippo_init_log_A(d_model: int, d_state: int) -> Tensor:
    """log|A| with A[:, n] = -(n+1) (ssm.py:34-43)."""
    n = torch.arange(1, d_state + 1, dtype=torch.float32)
    return n.log().expand(d_model, d_state).clone()


class SelectiveSSMLayer(nn.Module):
    """Diagonal selective SSM: h = A_bar*h + B_bar*u, y = C.h + D*u (ssm.py:46-353)."""

    def __init__(self, d_model: int, d_state: int = 16, dt_min: float = 0.001, dt_max: float = 0.1,
                 bidirectional: bool = False) -> None:
        super().__init__()
        self.d_model = d_model
        self.d_state = d_state
        self.bidirectional = bidirectional
        self.log_A = nn.Parameter(_hippo_init_log_A(d_model, d_state))
        self.D = nn.Parameter(torch.ones(d_model))
        self.B_proj = nn.Linear(d_model, d_state, bias=False)
        self.C_proj = nn.Linear(d_model, d_state, bias=False)
        self.dt_proj = nn.Linear(d_model, d_model, bias=True)
        with torch.no_grad():
            # dt log-uniform in [dt_min, dt_max]; bias = log(clamp(dt - 1, 1e-8)) (ssm.py:87-95)
            u = torch.rand(d_model)
            dt = torch.exp(u * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min))
            self.dt_proj.bias.copy_((dt - 1.0).clamp(min=1e-8).log())
        if bidirectional:
            self.B_proj_rev = nn.Linear(d_model, d_state, bias=False)
            self.C_proj_rev = nn.Linear(d_model, d_state, bias=False)
        self._packed = None

    def packed_proj_weight(self, dtype: torch.dtype) -> Tensor:
        """[W_dt; W_B; W_C] as one [d + 2N, d] weight, cached until a parameter changes."""
        ps = (self.dt_proj.weight, self.B_proj.weight, self.C_proj.weight)
        key = (dtype, ps[0].device) + tuple((p.data_ptr(), p._version) for p in ps)
        cached = getattr(self, "_packed", None)
        if cached is None or cached[0] != key:
            with torch.no_grad():
                w = torch.cat([p.detach().to(dtype) for p in ps], 0).contiguous()
            self._packed = (key, w)
        return self._packed[1]

    def forward(self, x: Tensor, state: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
        """x [B, T, d_model] -> (y [B, T, d_model], state [B, d_model, d_state])."""
        if self.bidirectional:
            raise NotImplementedError("bidirectional scan is not part of the B200 inference path")
        _no_grad_check(self, x, state)
        dt = x.dtype
        with torch.no_grad():
            return native.ssm_forward(x, self.packed_proj_weight(dt), self.dt_proj.bias.detach().to(dt).contiguous(),
                                      self.log_A.detach().to(dt).contiguous(), self.D.detach().to(dt).contiguous(),
                                      state, state_dtype=(state.dtype if state is not None else dt))

    def extra_repr(self) -> str:
        return f"d_model={self.d_model}, d_state={self.d_state}, selective=True, bidirectional={self.bidirectional}"


SSMLayer = SelectiveSSMLayer
