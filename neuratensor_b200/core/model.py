"""NeuraTensorModel on the B200 block kernels.

Interface mirror of NeuraTensor's ``neuratensor/core/model.py``:
``ModelConfig`` (model.py:32-85), ``RotaryEmbedding`` / ``apply_rotary`` /
``SlidingWindowAttention`` (model.py:88-181) and ``NeuraTensorModel``
(model.py:184-396) keep their names, fields, submodule layout and
initialisation order (embedding, blocks with attention interleaved, final
norm, tied lm_head, then ``_init_weights``), so a seed gives the reference's
weights and checkpoints load either way.

The spike blocks, the embedding gather, the sliding-window attention layers
(RMSNorm, projections and the windowed attention core) and the final RMSNorm +
tied lm_head (bf16 logits on the tcgen05 GEMM) run on the native kernels.
The forward collects every block's spike count in one device buffer and
reads it once, instead of the reference's three host syncs per block.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch import Tensor

from .fused import BlockState, FusedSpikeBlock, rate_like_reference


@dataclass
class ModelConfig:
    """Full model configuration (model.py:32-85)."""
    vocab_size: int = 32_000
    d_model: int = 512
    n_layers: int = 8
    d_state: int = 16
    expand: int = 2
    beta_init: float = 0.9
    learn_beta: bool = True
    dropout: float = 0.0
    tie_weights: bool = True
    max_seq_len: int = 2048
    attn_every: int = 0
    attn_heads: int = 4
    attn_window: int = 256
    model_name: str = "custom"

    @property
    def n_attn_layers(self) -> int:
        return 0 if self.attn_every <= 0 else self.n_layers // self.attn_every

    def n_params_estimate(self) -> int:
        di = self.d_model * self.expand
        block = (2 * self.d_model + 4 * self.d_model * di + di + 2 * di * self.d_state + di * di + di
                 + di * self.d_state + di + 1)
        attn = (2 * self.d_model + 4 * self.d_model * self.d_model) if self.attn_every > 0 else 0
        head = 0 if self.tie_weights else self.vocab_size * self.d_model
        return self.vocab_size * self.d_model + self.n_layers * block + self.n_attn_layers * attn + head


class RotaryEmbedding(nn.Module):
    """Rotary position embedding tables (model.py:88-116)."""

    def __init__(self, dim: int, max_seq_len: int = 8192, base: float = 10000.0) -> None:
        super().__init__()
        inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
        self.register_buffer("inv_freq", inv_freq, persistent=False)
        self._max_cached = 0
        self.register_buffer("cos_cached", torch.empty(0), persistent=False)
        self.register_buffer("sin_cached", torch.empty(0), persistent=False)

    def _build_cache(self, seq_len: int, device, dtype) -> None:
        if seq_len <= self._max_cached and self.cos_cached.dtype == dtype and self.cos_cached.device == device:
            return
        self._max_cached = seq_len
        pos = torch.arange(seq_len, device=device, dtype=torch.float32)
        ang = torch.outer(pos, self.inv_freq.to(device))
        ang = torch.cat([ang, ang], dim=-1)
        self.cos_cached = ang.cos().to(dtype)
        self.sin_cached = ang.sin().to(dtype)

    def forward(self, x: Tensor, offset: int = 0) -> Tuple[Tensor, Tensor]:
        T = x.shape[-2]
        self._build_cache(offset + T, x.device, x.dtype)
        return self.cos_cached[offset:offset + T], self.sin_cached[offset:offset + T]


def _rotate_half(x: Tensor) -> Tensor:
    a, b = x.chunk(2, dim=-1)
    return torch.cat([-b, a], dim=-1)


def apply_rotary(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """RoPE on x [B, H, T, hd]."""
    return x * cos + _rotate_half(x) * sin


class SlidingWindowAttention(nn.Module):
    """Causal multi-head attention limited to the last ``window`` keys (model.py:129-181).

    For T <= window plain causal attention; for T > window query i sees keys
    j with i - window <= j <= i.  Stateless across calls, like the reference
    (a T=1 decode step attends to itself only).
    """

    def __init__(self, d_model: int, n_heads: int = 4, window: int = 256, max_seq_len: int = 8192) -> None:
        super().__init__()
        self.d_model = d_model
        self.n_heads = n_heads
        self.head_dim = d_model // n_heads
        self.window = window
        self.norm = nn.RMSNorm(d_model)
        self.qkv = nn.Linear(d_model, d_model * 3, bias=False)
        self.o_proj = nn.Linear(d_model, d_model, bias=False)
        self.rope = RotaryEmbedding(self.head_dim, max_seq_len=max_seq_len)
        self._mask = None

    def _window_mask(self, T: int, device) -> Tensor:
        m = getattr(self, "_mask", None)
        if m is None or m.shape[-1] != T or m.device != device:
            i = torch.arange(T, device=device)
            rel = i[:, None] - i[None, :]
            m = self._mask = ((rel >= 0) & (rel <= self.window))[None, None]
        return m

    def forward(self, x: Tensor) -> Tensor:
        if x.is_cuda and x.dtype == torch.bfloat16 and self.head_dim in (64, 128):
            return self.forward_native(x)
        return self.forward_torch(x)

    def forward_native(self, x: Tensor, workspace: Optional[Tensor] = None) -> Tensor:
        """The whole layer in one native call (nt_attention_forward): RMSNorm, the
        qkv projection and o_proj + residual on the tcgen05 GEMM, RoPE and the
        windowed causal softmax attention in one kernel."""
        from .. import native
        cos, sin = self.rope(x)                     # rows [0, T) in x's dtype
        return native.attention_forward(x, self.norm.weight, self.qkv.weight, self.o_proj.weight, self.n_heads,
                                        self.window, cos, sin, workspace=workspace)

    def forward_torch(self, x: Tensor) -> Tensor:
        """The reference's op sequence (fp32, CPU tensors, head dims other than 64 and 128)."""
        B, T, _ = x.shape
        h = self.norm(x)
        q, k, v = self.qkv(h).view(B, T, 3, self.n_heads, self.head_dim).permute(2, 0, 3, 1, 4).unbind(0)
        cos, sin = self.rope(q)
        q = apply_rotary(q, cos, sin)
        k = apply_rotary(k, cos, sin)
        if T <= self.window:
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        else:
            o = F.scaled_dot_product_attention(q, k, v, attn_mask=self._window_mask(T, x.device))
        return self.o_proj(o.transpose(1, 2).reshape(B, T, self.d_model)) + x


class NeuraTensorModel(nn.Module):
    """Embedding -> FusedSpikeBlocks (+ attention every ``attn_every``) -> RMSNorm -> tied lm_head."""

    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.config = config
        self.embedding = nn.Embedding(config.vocab_size, config.d_model)
        self.blocks = nn.ModuleList()
        self.attn_layers = nn.ModuleDict()
        for i in range(config.n_layers):
            self.blocks.append(FusedSpikeBlock(d_model=config.d_model, d_state=config.d_state,
                                               expand=config.expand, beta_init=config.beta_init,
                                               learn_beta=config.learn_beta, dropout=config.dropout))
            if config.attn_every > 0 and (i + 1) % config.attn_every == 0:
                self.attn_layers[str(i)] = SlidingWindowAttention(d_model=config.d_model, n_heads=config.attn_heads,
                                                                  window=config.attn_window,
                                                                  max_seq_len=config.max_seq_len)
        self.norm = nn.RMSNorm(config.d_model)
        self.lm_head = nn.Linear(config.d_model, config.vocab_size, bias=False)
        if config.tie_weights:
            self.lm_head.weight = self.embedding.weight
        self._init_weights()
        self._ws = None

    def _init_weights(self) -> None:
        nn.init.normal_(self.embedding.weight, std=0.02)
        for blk in self.blocks:
            nn.init.xavier_uniform_(blk.in_proj.weight)
            nn.init.xavier_uniform_(blk.out_proj.weight)
        for attn in self.attn_layers.values():
            nn.init.xavier_uniform_(attn.qkv.weight)
            nn.init.xavier_uniform_(attn.o_proj.weight)

    @classmethod
    def from_preset(cls, name: str) -> "NeuraTensorModel":
        from ..config.presets import get_preset
        return cls(get_preset(name))

    def _workspace(self, x: Tensor) -> Tensor:
        """One block workspace reused by every block of a forward."""
        from .. import native
        c = self.config
        B, T, _ = x.shape
        n = native.block_workspace_bytes(x.dtype, B, T, c.d_model, c.d_model * c.expand, c.d_state)
        ws = getattr(self, "_ws", None)
        if ws is None or ws.numel() < n or ws.device != x.device:
            self._ws = torch.empty(n, dtype=torch.uint8, device=x.device)
        return self._ws

    # The kernels index activations with 32-bit element offsets in places; a
    # forward whose widest activation (the in_proj output [rows, 2*d_inner] or
    # attention's qkv [rows, 3*d_model]) would pass 2^30 elements runs the
    # batch in groups of sequences instead (sequences are independent, so
    # the result is the same).
    MAX_ACTIVATION_ELEMS = 1 << 30

    def group_size(self, seq: int) -> int:
        """Sequences of length `seq` that one pass of the blocks takes at most."""
        c = self.config
        width = max(2 * c.d_model * c.expand, 3 * c.d_model)
        return max(1, self.MAX_ACTIVATION_ELEMS // (max(seq, 1) * width))

    def forward_device(self, input_ids: Tensor, states: Optional[List[Optional[BlockState]]] = None,
                       workspace: Optional[Tensor] = None, last_only: bool = False):
        """Forward without any host sync: returns (logits, states, per-layer spike counts on device).

        ``last_only``: logits of the last position only ([B, 1, vocab]), as a
        generation prefill needs them."""
        if states is None:
            states = [None] * len(self.blocks)
        if input_ids.shape[1] > self.config.max_seq_len:
            import warnings
            warnings.warn(f"Input sequence length {input_ids.shape[1]} exceeds max_seq_len "
                          f"{self.config.max_seq_len}; truncating.", UserWarning, stacklevel=3)
            input_ids = input_ids[:, : self.config.max_seq_len]
        B, T = input_ids.shape
        g = self.group_size(T)
        if B <= g:
            return self._forward_rows(input_ids, states, workspace, last_only)
        parts = []
        for a in range(0, B, g):
            sub = [None if s is None else BlockState(membrane=s.membrane[a:a + g], ssm_state=s.ssm_state[a:a + g])
                   for s in states]
            parts.append(self._forward_rows(input_ids[a:a + g], sub, workspace, last_only))
        logits = torch.cat([p[0] for p in parts])
        state_cls = self.blocks[0]._state_cls
        new_states = [state_cls(membrane=torch.cat([p[1][i].membrane for p in parts]),
                                ssm_state=torch.cat([p[1][i].ssm_state for p in parts]))
                      for i in range(len(self.blocks))]
        counts = torch.stack([p[2] for p in parts]).sum(0)
        return logits, new_states, counts

    def _forward_rows(self, input_ids: Tensor, states: List[Optional[BlockState]], workspace: Optional[Tensor],
                      last_only: bool):
        from .. import native
        x = native.embedding(input_ids, self.embedding.weight)
        counts = torch.zeros(len(self.blocks), dtype=torch.int64, device=x.device)
        ws = workspace if workspace is not None else self._workspace(x)
        new_states: List[BlockState] = []
        with torch.no_grad():
            for i, (blk, st) in enumerate(zip(self.blocks, states)):
                x, ns = blk.forward_native(x, st, counts[i], workspace=ws)
                new_states.append(ns)
                key = str(i)
                if key in self.attn_layers:
                    x = self.attn_layers[key](x)
            if last_only:
                x = x[:, -1:]
            # final RMSNorm + tied lm_head on the tcgen05 GEMM; the block
            # workspace is free again here and holds the normalised rows
            logits = native.lm_head(x, self.norm.weight, self.lm_head.weight, workspace=ws)
        return logits, new_states, counts

    def metrics_from_counts(self, counts: List[int], numel: int, dtype: torch.dtype) -> Dict:
        rates = [rate_like_reference(c, numel, dtype) for c in counts]
        mean = sum(rates) / len(rates)
        return {"spike_rate": mean, "per_layer_spike_rate": rates, "estimated_sparsity_pct": (1.0 - mean) * 100}

    def forward(self, input_ids: Tensor, states: Optional[List[Optional[BlockState]]] = None
                ) -> Tuple[Tensor, List[BlockState], Dict]:
        """input_ids [B, T] -> (logits [B, T, vocab], states, metrics) (model.py:240-293)."""
        logits, new_states, counts = self.forward_device(input_ids, states)
        B, T = logits.shape[:2]
        di = self.config.d_model * self.config.expand
        metrics = self.metrics_from_counts(counts.tolist(), B * T * di, logits.dtype)
        return logits, new_states, metrics

    def count_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters())

    def count_trainable_parameters(self) -> int:
        return sum(p.numel() for p in self.parameters() if p.requires_grad)

    @torch.no_grad()
    def step_graph(self, batch: int, seq: int, device, dtype):
        """The captured forward for this (batch, length) (``inference/decode.py``).
        A graph holds raw addresses, so it is rebuilt when a parameter changes
        (version or storage) or an attention layer's RoPE tables were rebuilt;
        the four most recently used shapes are kept."""
        from ..inference.decode import StepGraph
        sig = (tuple((p.data_ptr(), p._version) for p in self.parameters()),
               tuple((a.rope.cos_cached.data_ptr(), a.rope.sin_cached.data_ptr()) for a in self.attn_layers.values()))
        key = (batch, seq, str(device), dtype)
        cache = self.__dict__.setdefault("_step_graphs", {})
        hit = cache.pop(key, None)
        if hit is None or hit[0] != sig:
            hit = None
            while len(cache) >= 4:
                cache.pop(next(iter(cache)))
            hit = (sig, StepGraph(self, batch, seq, torch.device(device), dtype))
        cache[key] = hit                          # most recently used last
        return hit[1]

    def decode_graph(self, batch: int, device, dtype):
        """The captured single-token step for this batch size."""
        return self.step_graph(batch, 1, device, dtype)

    def generate(self, input_ids: Tensor, max_new_tokens: int = 50, temperature: float = 1.0, top_k: int = 50,
                 top_p: float = 1.0, repetition_penalty: float = 1.0, stop_tokens: Optional[List[int]] = None,
                 states: Optional[List[Optional[BlockState]]] = None,
                 use_graph: bool = True) -> Tuple[Tensor, List[BlockState]]:
        """Autoregressive sampling with carried block state (model.py:301-370).

        On CUDA the per-token steps replay one captured graph of the whole model
        (``inference/decode.py``); ``use_graph=False`` runs them one launch at a
        time.  Both run the same kernels on the same inputs."""
        self.eval()
        out = input_ids
        stop = set(stop_tokens or [])
        logits, states, _ = self.forward_device(out, states, last_only=True)
        nxt_logits = logits[:, -1, :]
        graph = None
        if use_graph and out.is_cuda and max_new_tokens > 1:
            graph = self.decode_graph(out.shape[0], out.device, logits.dtype)
            graph.load_states(states)
        # top_k = 1 without nucleus filtering leaves the tied row maxima with
        # equal probability: one kernel picks among them with a uniform drawn
        # here for every step at once (the other filters run as written)
        greedy = out.is_cuda and top_k == 1 and top_p >= 1.0
        if greedy:
            from .. import native
            u_all = torch.rand((max_new_tokens, out.shape[0]), device=out.device)
        for step in range(max_new_tokens):
            if repetition_penalty != 1.0:
                for b in range(out.shape[0]):
                    for tok in out[b].tolist():
                        v = nxt_logits[b, tok]
                        nxt_logits[b, tok] = v / repetition_penalty if v > 0 else v * repetition_penalty
            if temperature != 1.0:
                nxt_logits = nxt_logits / temperature
            if greedy:
                tok = native.greedy_tokens(nxt_logits, u_all[step])
            elif top_k > 0:
                kth = torch.topk(nxt_logits, min(top_k, nxt_logits.size(-1))).values[:, [-1]]
                nxt_logits[nxt_logits < kth] = float("-inf")
            if top_p < 1.0:
                srt, idx = torch.sort(nxt_logits, descending=True, dim=-1)
                p = torch.softmax(srt, dim=-1)
                drop = p.cumsum(-1) - p > top_p
                srt = srt.masked_fill(drop, float("-inf"))
                nxt_logits = torch.zeros_like(nxt_logits).scatter_(-1, idx, srt)
            if not greedy:
                tok = torch.multinomial(torch.softmax(nxt_logits, dim=-1), num_samples=1)
            out = torch.cat([out, tok], dim=1)
            if stop and tok.item() in stop:
                break
            if graph is not None:
                nxt_logits = graph.step(tok).clone()
            else:
                logits, states, _ = self.forward_device(tok, states)
                nxt_logits = logits[:, -1, :]
        if graph is not None:
            states = graph.states()
        return out, states

    def info(self) -> str:
        c = self.config
        rows = [("Parameters", f"{self.count_parameters():,}"), ("Layers", c.n_layers), ("d_model", c.d_model),
                ("d_state", c.d_state), ("expand", c.expand), ("vocab", f"{c.vocab_size:,}"),
                ("max_seq_len", c.max_seq_len)]
        if c.attn_every > 0:
            rows += [("attn_every", c.attn_every), ("attn_heads", c.attn_heads), ("attn_window", c.attn_window),
                     ("attn_layers", c.n_attn_layers)]
        bar = "=" * 60
        body = "\n".join(f"  {k + ':':<14} {v:>14}" for k, v in rows)
        return f"{bar}\n  NeuraTensor v4 (B200 kernels) -- {c.model_name.upper()}\n{bar}\n{body}\n{bar}"


NeuraTensor = NeuraTensorModel
