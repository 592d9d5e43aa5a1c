"""One decode step of the whole model as a CUDA graph.

Autoregressive generation (model.py:301-370) runs the model on one new token
per step with the block states carried over.  At one token per step the work
per kernel is tiny and the step is bound by launch latency and host
overhead: ~10 launches per block plus attention and the lm_head.  This module
captures that step once per batch size into a CUDA graph and replays it:

* static inputs: the token ids [B, 1] and, per block, the membrane [B, d_inner]
  and SSM state [B, d_inner, d_state] in the model dtype;
* the captured region runs ``NeuraTensorModel.forward_device`` on them and
  copies the new states back into the static state buffers, so replay k+1
  continues from replay k;
* static outputs: the last position's logits [B, vocab] and the per-layer
  spike counts.

Sampling (temperature, top-k/top-p, repetition penalty) stays eager on the
returned logits, exactly as in the uncaptured loop.
"""
from __future__ import annotations

from typing import List, Optional

import torch
from torch import Tensor

from ..core.fused import BlockState


class DecodeGraph:
    """A captured single-token step for one batch size, device and dtype."""

    def __init__(self, model, batch: int, device: torch.device, dtype: torch.dtype) -> None:
        cfg = model.config
        di = cfg.d_model * cfg.expand
        self.model = model
        self.batch = batch
        self.tok = torch.zeros((batch, 1), dtype=torch.int64, device=device)
        self.mem = [torch.zeros((batch, di), dtype=dtype, device=device) for _ in model.blocks]
        self.st = [torch.zeros((batch, di, cfg.d_state), dtype=dtype, device=device) for _ in model.blocks]
        from .. import native
        nbytes = native.block_workspace_bytes(dtype, batch, 1, cfg.d_model, di, cfg.d_state)
        self.ws = torch.empty(nbytes, dtype=torch.uint8, device=device)   # owned: the graph keeps its address
        self.logits: Optional[Tensor] = None
        self.counts: Optional[Tensor] = None
        self.graph = torch.cuda.CUDAGraph()
        self._capture()

    def _states(self) -> List[BlockState]:
        return [BlockState(membrane=m, ssm_state=s) for m, s in zip(self.mem, self.st)]

    def _step(self):
        logits, new_states, counts = self.model.forward_device(self.tok, self._states(), workspace=self.ws)
        for i, ns in enumerate(new_states):
            self.mem[i].copy_(ns.membrane)
            self.st[i].copy_(ns.ssm_state)
        return logits[:, -1, :], counts

    def _capture(self) -> None:
        side = torch.cuda.Stream(device=self.tok.device)
        side.wait_stream(torch.cuda.current_stream(self.tok.device))
        with torch.cuda.stream(side), torch.no_grad():
            # warm-up outside the capture: builds weight caches, the workspace, the
            # RoPE tables and each kernel's one-time attributes
            for _ in range(2):
                self._step()
        torch.cuda.current_stream(self.tok.device).wait_stream(side)
        with torch.no_grad(), torch.cuda.graph(self.graph):
            self.logits, self.counts = self._step()

    def load_states(self, states: List[Optional[BlockState]]) -> None:
        for i, s in enumerate(states):
            if s is None:
                self.mem[i].zero_()
                self.st[i].zero_()
            else:
                self.mem[i].copy_(s.membrane)
                self.st[i].copy_(s.ssm_state)

    def step(self, tok: Tensor) -> Tensor:
        """Advance every sequence by the token ids `tok` [B, 1]; returns the logits [B, vocab]."""
        self.tok.copy_(tok)
        self.graph.replay()
        return self.logits

    def states(self) -> List[BlockState]:
        """Copies of the carried states (the static buffers change on the next step)."""
        return [BlockState(membrane=m.clone(), ssm_state=s.clone()) for m, s in zip(self.mem, self.st)]
