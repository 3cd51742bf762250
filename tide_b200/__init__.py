"""tide_b200 -- B200-native (sm_100a) early-exit hot path of TIDE.

Drop-in for the reference package's public API (`import tide_b200 as TIDE`):
TIDE (the runtime), TIDEConfig, calibrate, register_adapter, UniversalAdapter,
plus the `torch.ops.tide.*` operators registered by the native extension.
`calibrate` (offline router training, python/TIDE/calibrate.py) is importable
for scripts written against the reference but raises NotImplementedError:
router.pt files it writes load here unchanged.
"""
from __future__ import annotations

__version__ = "0.1.0"

__all__ = ["TIDE", "TIDEConfig", "calibrate", "register_adapter", "UniversalAdapter",
           "__version__"]


def __getattr__(name):
    if name == "TIDE":
        from tide_b200.runtime import TIDERuntime
        return TIDERuntime
    if name == "calibrate":
        from tide_b200.runtime import TIDERuntime
        return TIDERuntime.calibrate
    if name == "TIDEConfig":
        from tide_b200.config import TIDEConfig
        return TIDEConfig
    if name in ("register_adapter", "UniversalAdapter"):
        from tide_b200 import adapters
        return getattr(adapters, name)
    raise AttributeError(name)
