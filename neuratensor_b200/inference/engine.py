"""InferenceEngine on the B200 model.

Interface mirror of NeuraTensor's ``neuratensor/inference/engine.py``
(``InferenceResult``, ``InferenceEngine``: run / generate / benchmark /
reset_state / save / from_preset / from_checkpoint, engine.py:33-281).
Device placement and dtype follow the reference (bf16 on CUDA with
compute capability >= 8).  The timed region of ``run`` covers the model
forward plus the single metrics read-back, as the reference's does.

Not carried over: telemetry (network side channel, no compute role) and
``torch.compile`` (the block path is hand-written kernels).
"""
from __future__ import annotations

import os
import statistics
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, List, Optional

import torch
from torch import Tensor

from ..config.presets import get_preset
from ..core.fused import BlockState
from ..core.model import ModelConfig, NeuraTensorModel
from . import ranks


@dataclass
class InferenceResult:
    logits: Tensor
    states: List[Optional[BlockState]]
    latency_ms: float
    metrics: Dict
    device: str


def _best_device() -> str:
    if torch.cuda.is_available():
        return "cuda"
    raise RuntimeError("neuratensor_b200 needs a CUDA (sm_100) device")


def _best_dtype(device: str) -> torch.dtype:
    if device.startswith("cuda"):
        major = torch.cuda.get_device_properties(torch.device(device)).major
        return torch.bfloat16 if major >= 8 else torch.float16
    return torch.float32


class InferenceEngine:
    """Device placement, precision, streaming state and benchmarking around the model."""

    def __init__(self, model: NeuraTensorModel, device: Optional[str] = None, dtype: Optional[torch.dtype] = None,
                 compile_model: bool = False, distributed: Optional[bool] = None) -> None:
        self.device = device or _best_device()
        if not self.device.startswith("cuda"):
            raise RuntimeError("neuratensor_b200 runs on CUDA (sm_100) only; got device=" + self.device)
        self.dtype = dtype or _best_dtype(self.device)
        self._states: List[Optional[BlockState]] = [None] * len(model.blocks)
        # run() replays one captured CUDA graph per input shape (see inference/decode.py);
        # False launches the kernels one by one (same kernels, same results)
        self.use_graphs = True
        # Under torchrun (one process per GPU, each running its own rows of the
        # batch) run() returns the metrics of the whole global batch, as one
        # process over all rows would (model.py:286-291): the per-layer spike
        # counts and element counts are summed over the ranks.  Default: on
        # when a process group with more than one rank is initialised.
        if distributed is None:
            import torch.distributed as dist
            distributed = dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1
        self.distributed = bool(distributed)
        model = model.to(self.device).to(self.dtype)
        model.eval()
        self.model = model

    # ------------------------------------------------------------------ #
    @classmethod
    def from_preset(cls, name: str, device: Optional[str] = None, dtype: Optional[torch.dtype] = None,
                    compile_model: bool = False) -> "InferenceEngine":
        return cls(NeuraTensorModel(get_preset(name)), device=device, dtype=dtype)

    @classmethod
    def from_checkpoint(cls, path: str, device: Optional[str] = None,
                        dtype: Optional[torch.dtype] = None) -> "InferenceEngine":
        """Load ``{"config", "model", "version"}`` as written by ``save`` (engine.py:90-103,267-272)."""
        import torch.serialization as ser
        ser.add_safe_globals([ModelConfig])
        try:
            from neuratensor.core.model import ModelConfig as RefConfig  # checkpoints written by the reference
            ser.add_safe_globals([RefConfig])
        except Exception:
            pass
        ckpt = torch.load(path, map_location="cpu", weights_only=True)
        cfg = ckpt["config"]
        if not isinstance(cfg, ModelConfig):
            cfg = ModelConfig(**{k: getattr(cfg, k) for k in ModelConfig.__dataclass_fields__})
        model = NeuraTensorModel(cfg)
        model.load_state_dict(ckpt["model"])
        return cls(model, device=device, dtype=dtype)

    @classmethod
    def from_pretrained(cls, name: str, cache_dir: Optional[str] = None, device: Optional[str] = None,
                        dtype: Optional[torch.dtype] = None) -> "InferenceEngine":
        """Load a hub checkpoint from the local cache (engine.py:105-139 layout); no download."""
        cache = Path(cache_dir or os.path.expanduser("~/.neuratensor/models"))
        path = cache / (name.replace("/", "--") + ".pt")
        if not path.exists():
            raise RuntimeError(f"checkpoint for '{name}' not found at {path}")
        return cls.from_checkpoint(str(path), device=device, dtype=dtype)

    # ------------------------------------------------------------------ #
    @torch.no_grad()
    def run(self, input_ids: Tensor, reset_state: bool = False) -> InferenceResult:
        """One forward with the carried state (engine.py:145-178)."""
        if reset_state:
            self.reset_state()
        ids = input_ids.to(self.device, non_blocking=True)
        torch.cuda.synchronize(self.device)
        t0 = time.perf_counter()
        with torch.autocast(device_type="cuda", dtype=self.dtype, enabled=self.dtype != torch.float32):
            if self.use_graphs and ids.is_cuda:
                logits, new_states, counts = self._run_graph(ids)
            else:
                logits, new_states, counts = self.model.forward_device(ids, self._states)
        B, T = logits.shape[:2]
        numel = B * T * self.model.config.d_model * self.model.config.expand
        if self.distributed:
            counts, numel = ranks.global_counts(counts, numel)
        metrics = self.model.metrics_from_counts(counts.tolist(), numel, logits.dtype)
        torch.cuda.synchronize(self.device)
        latency_ms = (time.perf_counter() - t0) * 1000.0
        self._states = new_states
        return InferenceResult(logits=logits, states=new_states, latency_ms=latency_ms, metrics=metrics,
                               device=self.device)

    def _run_graph(self, ids: Tensor):
        """The forward as one replay of the captured graph for this shape; the
        logits and states returned are copies (the graph reuses its buffers)."""
        B, T = ids.shape
        g = self.model.step_graph(B, T, ids.device, self.dtype)
        g.load_states(self._states)
        logits = g.replay(ids).clone()
        return logits, g.states(), g.counts.clone()

    @torch.no_grad()
    def generate(self, input_ids: Tensor, max_new_tokens: int = 64, temperature: float = 1.0, top_k: int = 50,
                 top_p: float = 1.0, repetition_penalty: float = 1.0, stop_tokens: Optional[List[int]] = None,
                 reset_state: bool = True) -> Tensor:
        """Returns [B, T + generated] token ids (engine.py:180-208)."""
        if reset_state:
            self.reset_state()
        ids = input_ids.to(self.device)
        with torch.autocast(device_type="cuda", dtype=self.dtype, enabled=self.dtype != torch.float32):
            out, states = self.model.generate(ids, max_new_tokens=max_new_tokens, temperature=temperature,
                                              top_k=top_k, top_p=top_p, repetition_penalty=repetition_penalty,
                                              stop_tokens=stop_tokens, states=self._states)
        self._states = states
        return out

    @torch.no_grad()
    def benchmark(self, batch_size: int = 1, seq_length: int = 64, n_iter: int = 50, n_warmup: int = 10) -> Dict:
        """Latency statistics of ``run`` on random ids (engine.py:214-254)."""
        ids = torch.randint(0, self.model.config.vocab_size, (batch_size, seq_length), device=self.device)
        for _ in range(n_warmup):
            self.run(ids, reset_state=True)
        lat, rates = [], []
        for _ in range(n_iter):
            r = self.run(ids, reset_state=True)
            lat.append(r.latency_ms)
            rates.append(r.metrics["spike_rate"])
        mean_ms = statistics.mean(lat)
        return {
            "mean_ms": mean_ms,
            "std_ms": statistics.stdev(lat) if n_iter > 1 else 0.0,
            "min_ms": min(lat),
            "p99_ms": sorted(lat)[int(n_iter * 0.99)],
            "throughput_seq_per_s": batch_size * 1000.0 / mean_ms,
            "spike_rate": statistics.mean(rates),
            "sparsity_pct": (1.0 - statistics.mean(rates)) * 100,
            "batch_size": batch_size,
            "seq_length": seq_length,
            "device": self.device,
            "dtype": str(self.dtype),
            "n_params": self.model.count_parameters(),
            "preset": self.model.config.model_name,
        }

    def reset_state(self) -> None:
        self._states = [None] * len(self.model.blocks)

    def save(self, path: str) -> None:
        torch.save({"config": self.model.config, "model": self.model.state_dict(), "version": "4.0.0"}, path)

    def print_info(self) -> None:
        print(self.model.info())
        print(f"  Device:  {self.device}")
        print(f"  Dtype:   {self.dtype}")
        print("  Compiled:False")
        print()
