from tide_b200.adapters.auto import ADAPTER_REGISTRY, get_adapter, register_adapter
from tide_b200.adapters.base import BaseAdapter
from tide_b200.adapters.families import LlamaAdapter, MistralAdapter, QwenAdapter
from tide_b200.adapters.universal import UniversalAdapter

__all__ = ["ADAPTER_REGISTRY", "BaseAdapter", "LlamaAdapter", "MistralAdapter", "QwenAdapter",
           "UniversalAdapter", "get_adapter", "register_adapter"]
