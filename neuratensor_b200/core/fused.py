"""FusedSpikeBlock with the whole block on B200 kernels.

Interface mirror of NeuraTensor's ``neuratensor/core/fused.py``:
``BlockState`` (fused.py:38-42) and ``FusedSpikeBlock`` (fused.py:45-165)
keep their constructor, submodules, parameter names and initialisation
order.  ``forward`` makes one C-ABI call, ``nt_block_forward``, that runs

    RMSNorm -> in_proj (tcgen05 GEMM) -> LIF -> row compaction
    -> dt/B/C projections (tcgen05 GEMM, softplus epilogue)
    -> selective scan with y*silu(gate) fused (rows compacted when sparse)
    -> out_proj on the active rows (tcgen05 GEMM) with *out_scale + residual

and decides the sparse/dense out_proj branch (fused.py:149-165) on the
device.  The spike count lands in a device counter, so a model forward
reads all its metrics with a single device-to-host copy.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np
import torch
import torch.nn as nn
from torch import Tensor

from .. import native
from .snn import LIFLayer, _no_grad_check
from .ssm import SelectiveSSMLayer


@dataclass
class BlockState:
    """Streaming state carried between forward calls (fused.py:38-42)."""
    membrane: Optional[Tensor] = None
    ssm_state: Optional[Tensor] = None


def rate_like_reference(count: int, numel: int, dtype: torch.dtype) -> float:
    """``spikes.mean().item()`` for 0/1 spikes: float32 mean, rounded to the spike dtype."""
    r = np.float32(count) / np.float32(max(numel, 1))
    if dtype == torch.bfloat16:
        return float(torch.tensor(float(r)).to(torch.bfloat16).item())
    if dtype == torch.float16:
        return float(torch.tensor(float(r)).to(torch.float16).item())
    return float(r)


class FusedSpikeBlock(nn.Module):
    """RMSNorm -> in_proj -> LIF -> selective SSM -> gate -> sparse out_proj -> residual."""

    # class of the returned streaming state (the drop-in patch points it at
    # the reference package's own BlockState)
    _state_cls = BlockState

    def __init__(self, d_model: int, d_state: int = 16, expand: int = 2, beta_init: float = 0.9,
                 learn_beta: bool = True, dropout: float = 0.0) -> None:
        super().__init__()
        self.d_model = d_model
        self.d_inner = d_model * expand
        self.norm = nn.RMSNorm(d_model)
        self.in_proj = nn.Linear(d_model, self.d_inner * 2, bias=False)
        self.snn = LIFLayer(size=self.d_inner, beta_init=beta_init, learn_beta=learn_beta, dropout=dropout)
        self.ssm = SelectiveSSMLayer(d_model=self.d_inner, d_state=d_state)
        self.out_proj = nn.Linear(self.d_inner, d_model, bias=False)
        self.out_scale = nn.Parameter(torch.ones(1) * 0.1)
        self._sparse_inference = True
        self._cache = None

    # ------------------------------------------------------------------ #
    def _native_weights(self, dtype: torch.dtype, device: torch.device):
        """Contiguous weights in the activation dtype, rebuilt when a parameter changes."""
        params = (self.norm.weight, self.in_proj.weight, self.snn.beta_logit, self.snn.threshold,
                  self.ssm.log_A, self.ssm.D, self.ssm.dt_proj.weight, self.ssm.B_proj.weight,
                  self.ssm.C_proj.weight, self.ssm.dt_proj.bias, self.out_proj.weight, self.out_scale)
        key = (dtype, device) + tuple((p.data_ptr(), p._version, p.device) for p in params)
        cache = getattr(self, "_cache", None)
        if cache is None or cache[0] != key:
            with torch.no_grad():
                cv = lambda p: p.detach().to(device=device, dtype=dtype).contiguous()
                beta = torch.sigmoid(self.snn.beta_logit.detach().to(device)).to(dtype).contiguous()
                w = dict(norm_w=cv(self.norm.weight), W_in=cv(self.in_proj.weight), beta=beta,
                         threshold=cv(self.snn.threshold), log_A=cv(self.ssm.log_A), D=cv(self.ssm.D),
                         W_proj=self.ssm.packed_proj_weight(dtype).to(device), b_dt=cv(self.ssm.dt_proj.bias),
                         W_out=cv(self.out_proj.weight), out_scale=cv(self.out_scale))
                mean_beta = float(torch.sigmoid(self.snn.beta_logit.detach()).mean().item())
            self._cache = (key, w, mean_beta)
        return self._cache[1], self._cache[2]

    def forward_native(self, x: Tensor, state: Optional[BlockState], spike_count: Tensor,
                       workspace: Optional[Tensor] = None) -> Tuple[Tensor, BlockState]:
        """One ``nt_block_forward`` call; adds the block's spike count to ``spike_count`` (device int64)."""
        if self.snn.drop is not None and self.training:
            raise NotImplementedError("spike dropout is a training feature; use eval() for the B200 path")
        _no_grad_check(self, x)
        w, _ = self._native_weights(x.dtype, x.device)
        mem = state.membrane if state is not None else None
        st = state.ssm_state if state is not None else None
        sparse = (not self.training) and self._sparse_inference
        out, mem_out, st_out = native.block_forward(
            x, w["norm_w"], w["W_in"], w["beta"], w["threshold"], w["log_A"], w["D"], w["W_proj"], w["b_dt"],
            w["W_out"], w["out_scale"], mem, st, spike_count, sparse=sparse, state_dtype=x.dtype,
            workspace=workspace)
        return out, self._state_cls(membrane=mem_out, ssm_state=st_out)

    def forward(self, x: Tensor, state: Optional[BlockState] = None) -> Tuple[Tensor, BlockState, dict]:
        """x [B, T, d_model] -> (out, BlockState, {"spike_rate", "mean_beta"}) (fused.py:101-147)."""
        native._require_cuda(x)
        count = torch.zeros((), dtype=torch.int64, device=x.device)
        with torch.no_grad():
            out, new_state = self.forward_native(x, state, count)
        _, mean_beta = self._native_weights(x.dtype, x.device)
        B, T, _ = x.shape
        metrics = {"spike_rate": rate_like_reference(int(count.item()), B * T * self.d_inner, x.dtype),
                   "mean_beta": mean_beta}
        return out, new_state, metrics

    def _sparse_out_proj(self, x: Tensor, spikes: Tensor) -> Tensor:
        """Output projection that skips rows without spikes (fused.py:149-165)."""
        with torch.no_grad():
            out, _ = native.sparse_out_proj(x, spikes, self.out_proj.weight.detach().to(x.dtype))
        return out

    def extra_repr(self) -> str:
        return f"d_model={self.d_model}, d_inner={self.d_inner}, d_state={self.ssm.d_state}"


FusedSNNSSMBlock = FusedSpikeBlock
