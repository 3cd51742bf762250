"""TIDEConfig: the reference's configuration dataclass (python/TIDE/config.py:
9-33), same fields, defaults and YAML layout, plus one field of its own:
live_compaction (default off, the reference's post-hoc forward) runs the
layers after each checkpoint on the still-active tokens only
(tide_b200/live.py), with exited tokens' K/V handled as kv_cache_strategy
says ("zero_pad", the reference's default and the one implemented).  The hot
path reads exit_threshold, min_layers, live_compaction and profile."""
from __future__ import annotations

from dataclasses import asdict, dataclass
from pathlib import Path

import yaml


@dataclass
class TIDEConfig:
    checkpoint_interval: int = 4
    exit_threshold: float = 0.85
    min_layers: int = 8
    compaction_threshold: float = 0.25
    exit_strategy: str = "identity"
    calibration_samples: int = 2000
    calibration_dataset: str = "wikitext"
    router_bottleneck_dim: int = 128
    convergence_threshold: float = 0.98
    kv_cache_strategy: str = "zero_pad"
    profile: bool = False
    live_compaction: bool = False

    def save(self, path: str | Path) -> None:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        with open(path, "w") as f:
            yaml.safe_dump(asdict(self), f, default_flow_style=False)

    @classmethod
    def load(cls, path: str | Path) -> "TIDEConfig":
        with open(path) as f:
            data = yaml.safe_load(f) or {}
        return cls(**data)
