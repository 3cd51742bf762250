"""Adapter interface: how the runtime finds a model's decoder layers, final
norm, LM head and embedding.  Same abstract methods as the reference's
BaseAdapter (python/TIDE/adapters/base.py:10-51)."""
from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Optional

import torch
import torch.nn as nn


def hidden_of(layer_output) -> torch.Tensor:
    """The hidden states a decoder layer returned.  Older transformers
    releases return a tuple whose first element is the hidden states (what
    the reference's adapters index with `layer_output[0]`); current ones
    return the tensor itself, where `[0]` would select the first sequence."""
    if isinstance(layer_output, (tuple, list)):
        return layer_output[0]
    return layer_output


class BaseAdapter(ABC):
    @abstractmethod
    def get_layers(self, model: nn.Module) -> list[nn.Module]: ...

    @abstractmethod
    def get_hidden_state(self, layer_output) -> torch.Tensor: ...

    @abstractmethod
    def get_final_norm(self, model: nn.Module) -> nn.Module: ...

    @abstractmethod
    def get_lm_head(self, model: nn.Module) -> nn.Module: ...

    @abstractmethod
    def get_router_input_dim(self, model: nn.Module) -> int: ...

    @abstractmethod
    def get_embedding(self, model: nn.Module) -> nn.Module: ...

    def get_router_extra_features(self, layer_output) -> Optional[torch.Tensor]:
        return None

    def get_position_embeddings(self, model: nn.Module, position_ids: torch.Tensor,
                                hidden: torch.Tensor) -> Optional[tuple]:
        return None


class DecoderOnlyAdapter(BaseAdapter):
    """HF decoder-only layout: model.model.{layers,norm,embed_tokens},
    model.lm_head, model.config.hidden_size, model.model.rotary_emb."""

    def get_layers(self, model):
        return list(model.model.layers)

    def get_hidden_state(self, layer_output):
        return hidden_of(layer_output)

    def get_final_norm(self, model):
        return model.model.norm

    def get_lm_head(self, model):
        return model.lm_head

    def get_router_input_dim(self, model):
        return model.config.hidden_size

    def get_embedding(self, model):
        return model.model.embed_tokens

    def get_position_embeddings(self, model, position_ids, hidden):
        rotary = getattr(model.model, "rotary_emb", None)
        return None if rotary is None else rotary(hidden, position_ids)
