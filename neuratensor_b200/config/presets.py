"""Model presets (the reference's ``neuratensor/config/presets.py:17-101``, same values)."""
from __future__ import annotations

from ..core.model import ModelConfig

PRESETS: dict = {
    "pico": ModelConfig(model_name="pico", vocab_size=32_000, d_model=96, n_layers=4, d_state=8, expand=2,
                        beta_init=0.9, learn_beta=True, dropout=0.0, max_seq_len=512, attn_every=0),
    "nano": ModelConfig(model_name="nano", vocab_size=32_000, d_model=288, n_layers=6, d_state=16, expand=2,
                        beta_init=0.9, learn_beta=True, dropout=0.0, max_seq_len=1024, attn_every=6,
                        attn_heads=6, attn_window=256),
    "small": ModelConfig(model_name="small", vocab_size=32_000, d_model=640, n_layers=12, d_state=32, expand=2,
                         beta_init=0.9, learn_beta=True, dropout=0.0, max_seq_len=2048, attn_every=6,
                         attn_heads=10, attn_window=256),
    "medium": ModelConfig(model_name="medium", vocab_size=32_000, d_model=1152, n_layers=20, d_state=64, expand=2,
                          beta_init=0.9, learn_beta=True, dropout=0.0, max_seq_len=4096, attn_every=5,
                          attn_heads=16, attn_window=512),
    "large": ModelConfig(model_name="large", vocab_size=32_000, d_model=2048, n_layers=28, d_state=128, expand=2,
                         beta_init=0.9, learn_beta=True, dropout=0.0, max_seq_len=8192, attn_every=7,
                         attn_heads=16, attn_window=512),
}
PRESETS["64m"] = PRESETS["small"]
PRESETS["256m"] = PRESETS["medium"]
PRESETS["1b"] = PRESETS["large"]


def get_preset(name: str) -> ModelConfig:
    """Return a ModelConfig by preset name (case-insensitive)."""
    key = name.lower().strip()
    if key not in PRESETS:
        avail = ", ".join(sorted(k for k in PRESETS if not k[-1].isdigit()))
        raise ValueError(f"Unknown preset '{name}'. Available: {avail}")
    return PRESETS[key]


def list_presets() -> None:
    print(f"\n{'Preset':<10} {'d_model':>8} {'layers':>7} {'d_state':>8} {'attn':>5} {'max_seq':>8}  Est. params")
    print("-" * 72)
    for name in ("pico", "nano", "small", "medium", "large"):
        c = PRESETS[name]
        print(f"{name:<10} {c.d_model:>8} {c.n_layers:>7} {c.d_state:>8} {c.n_attn_layers:>5} "
              f"{c.max_seq_len:>8}  {c.n_params_estimate():>12,}")
    print()
