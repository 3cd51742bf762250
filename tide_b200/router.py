"""Router module and the router.pt file format.

TokenRouter matches the reference's module (python/TIDE/router.py:11-19):
down = Linear(H, B, bias=False), up = Linear(B, 1), SiLU, sigmoid, output
squeezed to [N].  The file written by RouterCheckpoint.save is the
reference's layout (router.py:28-38):
    {"hidden_dim": int, "bottleneck_dim": int,
     "router_layers": {layer_idx: {"down.weight": [B, H], "up.weight": [1, B]}}}
Optional keys understood on top of it, in a layer's state dict:
  "up.bias" ([1]): a scalar added before the sigmoid;
  "exit_proj.weight" ([H, H]) and "exit_proj.bias" ([H]): the learned exit
    projection of the reference's declared "Mode B" (csrc/kernels/
    exit_projection.cu:5-8, TIDEConfig.exit_strategy = "learned"): an exiting
    token's output row is exit_proj(final_norm(h)) instead of final_norm(h).
Files without them (every file the reference writes) load unchanged and mean
a zero bias and no projection.  Layer keys may be ints or strings, as in
router.py:47.
"""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Dict

import torch
import torch.nn as nn


class TokenRouter(nn.Module):
    def __init__(self, hidden_dim: int, bottleneck_dim: int = 128, up_bias: bool = False,
                 exit_proj: bool = False, exit_proj_bias: bool = False):
        super().__init__()
        self.down = nn.Linear(hidden_dim, bottleneck_dim, bias=False)
        self.up = nn.Linear(bottleneck_dim, 1, bias=up_bias)
        self.act = nn.SiLU()
        self.exit_proj = nn.Linear(hidden_dim, hidden_dim, bias=exit_proj_bias) if exit_proj else None

    def forward(self, hidden_state: torch.Tensor) -> torch.Tensor:
        return torch.sigmoid(self.up(self.act(self.down(hidden_state)))).squeeze(-1)

    @property
    def up_bias_value(self) -> float:
        return float(self.up.bias.detach().reshape(-1)[0]) if self.up.bias is not None else 0.0


@dataclass
class RouterCheckpoint:
    routers: Dict[int, TokenRouter]
    hidden_dim: int
    bottleneck_dim: int

    def save(self, path: str | Path) -> None:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        state = {"hidden_dim": self.hidden_dim, "bottleneck_dim": self.bottleneck_dim,
                 "router_layers": {int(k): r.state_dict() for k, r in self.routers.items()}}
        torch.save(state, path)

    @classmethod
    def load(cls, path: str | Path, device: str = "cpu") -> "RouterCheckpoint":
        state = torch.load(path, map_location=device, weights_only=True)
        h, b = int(state["hidden_dim"]), int(state["bottleneck_dim"])
        routers: Dict[int, TokenRouter] = {}
        for key, sd in state["router_layers"].items():
            r = TokenRouter(h, b, up_bias="up.bias" in sd, exit_proj="exit_proj.weight" in sd,
                            exit_proj_bias="exit_proj.bias" in sd)
            r.load_state_dict(sd)
            routers[int(key)] = r.to(device)
        return cls(routers=routers, hidden_dim=h, bottleneck_dim=b)
