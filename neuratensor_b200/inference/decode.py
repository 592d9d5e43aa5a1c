"""The whole model forward as a replayable CUDA graph, for a fixed batch and length.

A forward of the native path is ~10 launches per block plus attention and the
lm_head.  When the per-launch work is small (decoding one token, or a small
per-GPU batch) the host's launch work is exposed; a captured graph replays
all of it with one call.  ``StepGraph`` captures ``forward_device`` once for
a (batch, length) shape:

* static inputs: the token ids [B, T] and, per block, the membrane
  [B, d_inner] and SSM state [B, d_inner, d_state] in the model dtype (zero
  buffers stand for "no state", which the kernels treat as zeros);
* the captured region runs the forward on them and copies the new states back
  into the static state buffers, so replay k+1 continues from replay k;
* static outputs: the logits [B, T, vocab] and the per-layer spike counts.

The graph holds raw device addresses: it owns its workspace, and the model
rebuilds it when a parameter changes or a RoPE table is rebuilt
(``NeuraTensorModel.step_graph``).  Sampling stays eager on the logits.
"""
from __future__ import annotations

from typing import List, Optional

import torch
from torch import Tensor

from ..core.fused import BlockState


class StepGraph:
    """A captured forward for one (batch, length), device and dtype."""

    def __init__(self, model, batch: int, seq: int, device: torch.device, dtype: torch.dtype) -> None:
        from .. import native
        cfg = model.config
        di = cfg.d_model * cfg.expand
        self.model = model
        self.tok = torch.zeros((batch, seq), dtype=torch.int64, device=device)
        # every block's membrane and SSM state as views of one flat buffer (one memset,
        # one copy for all of them)
        n_mem, n_st = batch * di, batch * di * cfg.d_state
        self.flat = torch.zeros(len(model.blocks) * (n_mem + n_st), dtype=dtype, device=device)
        self._split = lambda buf: (
            [buf[i * (n_mem + n_st):i * (n_mem + n_st) + n_mem].view(batch, di) for i in range(len(model.blocks))],
            [buf[i * (n_mem + n_st) + n_mem:(i + 1) * (n_mem + n_st)].view(batch, di, cfg.d_state)
             for i in range(len(model.blocks))])
        self.mem, self.st = self._split(self.flat)
        nbytes = native.block_workspace_bytes(dtype, batch, seq, cfg.d_model, di, cfg.d_state)
        self.ws = torch.empty(nbytes, dtype=torch.uint8, device=device)   # owned: the graph keeps its address
        self.logits: Optional[Tensor] = None
        self.counts: Optional[Tensor] = None
        self.graph = torch.cuda.CUDAGraph()
        self._capture()

    def _states(self) -> List[BlockState]:
        return [BlockState(membrane=m, ssm_state=s) for m, s in zip(self.mem, self.st)]

    def _forward(self):
        logits, new_states, counts = self.model.forward_device(self.tok, self._states(), workspace=self.ws)
        for i, ns in enumerate(new_states):
            self.mem[i].copy_(ns.membrane)
            self.st[i].copy_(ns.ssm_state)
        return logits, counts

    def _capture(self) -> None:
        dev = self.tok.device
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.no_grad():
            # warm-up outside the capture: weight caches, RoPE tables and each
            # kernel's one-time attributes are set up here
            for _ in range(2):
                self._forward()
        torch.cuda.current_stream(dev).wait_stream(side)
        with torch.no_grad(), torch.cuda.graph(self.graph):
            self.logits, self.counts = self._forward()

    def load_states(self, states: Optional[List[Optional[BlockState]]]) -> None:
        """Start the next replay from `states` (None, or None entries: zero state)."""
        if states is None or all(s is None for s in states):
            self.flat.zero_()
            return
        for i in range(len(self.mem)):
            s = states[i]
            if s is None:
                self.mem[i].zero_()
                self.st[i].zero_()
            else:
                self.mem[i].copy_(s.membrane)
                self.st[i].copy_(s.ssm_state)

    def replay(self, tok: Tensor) -> Tensor:
        """Run the captured forward on token ids `tok` [B, T]; returns the static logits."""
        self.tok.copy_(tok, non_blocking=True)
        self.graph.replay()
        return self.logits

    def step(self, tok: Tensor) -> Tensor:
        """Decode step (T = 1): the logits [B, vocab] of the new token."""
        return self.replay(tok)[:, -1, :]

    def states(self) -> List[BlockState]:
        """Copies of the carried states (the static buffers change on the next replay)."""
        mem, st = self._split(self.flat.clone())
        state_cls = self.model.blocks[0]._state_cls
        return [state_cls(membrane=m, ssm_state=s) for m, s in zip(mem, st)]
