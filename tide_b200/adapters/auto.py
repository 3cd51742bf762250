"""Adapter resolution: an exact class-name registry first, then
UniversalAdapter probing (python/TIDE/adapters/auto.py:14-43)."""
from __future__ import annotations

import logging

import torch.nn as nn

from tide_b200.adapters.base import BaseAdapter
from tide_b200.adapters.families import LlamaAdapter, MistralAdapter, QwenAdapter
from tide_b200.adapters.universal import UniversalAdapter

logger = logging.getLogger("TIDE")

ADAPTER_REGISTRY: dict[str, type[BaseAdapter]] = {
    "LlamaForCausalLM": LlamaAdapter,
    "MistralForCausalLM": MistralAdapter,
    "Qwen2ForCausalLM": QwenAdapter,
}


def register_adapter(class_name: str, adapter_cls: type[BaseAdapter]) -> None:
    ADAPTER_REGISTRY[class_name] = adapter_cls


def get_adapter(model: nn.Module) -> BaseAdapter:
    name = type(model).__name__
    if name in ADAPTER_REGISTRY:
        return ADAPTER_REGISTRY[name]()
    logger.info(f"No registered adapter for '{name}', trying UniversalAdapter")
    return UniversalAdapter.probe(model)
