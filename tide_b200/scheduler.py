"""ExitStats: per-layer exit accounting, the metrics surface of the
reference (python/TIDE/scheduler.py:12-36), same fields and summary text."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict


@dataclass
class ExitStats:
    total_tokens: int = 0
    exits_per_layer: Dict[int, int] = field(default_factory=dict)
    remaining_tokens: int = 0

    @property
    def total_exited(self) -> int:
        return sum(self.exits_per_layer.values())

    @property
    def exit_rate(self) -> float:
        return self.total_exited / self.total_tokens if self.total_tokens else 0.0

    def summary(self) -> str:
        lines = [f"Total tokens: {self.total_tokens}, Exited: {self.total_exited} "
                 f"({self.exit_rate:.1%})"]
        for layer in sorted(self.exits_per_layer):
            c = self.exits_per_layer[layer]
            pct = c / self.total_tokens * 100 if self.total_tokens else 0
            lines.append(f"  Layer {layer}: {c} exits ({pct:.1f}%)")
        lines.append(f"  Ran all layers: {self.remaining_tokens}")
        return "\n".join(lines)
