"""Backend detection (the reference's ``neuratensor/backends/detect.py:34-70``) plus the native-kernel status."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch


@dataclass
class BackendInfo:
    name: str
    device: str
    dtype: torch.dtype
    gpu_name: Optional[str] = None
    compute_capability: Optional[str] = None
    memory_gb: Optional[float] = None
    bf16: bool = False
    compile_ready: bool = False
    native_kernels: bool = False
    notes: list = field(default_factory=list)

    def print(self) -> None:
        """One line per known fact about the device and the native library."""
        rows = [("backend", self.name), ("device", f"{self.device} ({self.dtype})")]
        if self.gpu_name:
            rows += [("gpu", f"{self.gpu_name}, compute capability {self.compute_capability}"),
                     ("memory", f"{self.memory_gb:.1f} GiB"), ("bfloat16", "yes" if self.bf16 else "no")]
        rows.append(("B200 kernels", "loaded" if self.native_kernels else "not available"))
        width = max(len(k) for k, _ in rows)
        print("\n".join(f"{k.rjust(width)} : {v}" for k, v in rows))
        for n in self.notes:
            print(f"{'note'.rjust(width)} : {n}")


def detect_backend() -> BackendInfo:
    from .native import native_available
    if torch.cuda.is_available():
        p = torch.cuda.get_device_properties(0)
        ok = p.major == 10 and p.minor == 0
        notes = [] if ok else [f"sm_{p.major}{p.minor} is not sm_100: the B200 kernels cannot run here"]
        return BackendInfo(name="b200" if ok else "cuda", device="cuda",
                           dtype=torch.bfloat16 if p.major >= 8 else torch.float16, gpu_name=p.name,
                           compute_capability=f"{p.major}.{p.minor}", memory_gb=p.total_memory / 1024 ** 3,
                           bf16=p.major >= 8, compile_ready=hasattr(torch, "compile"),
                           native_kernels=ok and native_available(), notes=notes)
    return BackendInfo(name="cpu", device="cpu", dtype=torch.float32, compile_ready=hasattr(torch, "compile"),
                       notes=["No GPU detected: the B200 kernels need an sm_100 device"])
