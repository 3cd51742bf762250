"""UniversalAdapter: finds the components of an arbitrary HF causal LM.

Behaviour follows the reference's UniversalAdapter
(python/TIDE/adapters/universal.py:14-247): try known attribute paths per
architecture family, then fall back to structural heuristics (the largest
ModuleList for layers, a norm module next to the layers, a Linear / Embedding
sized like the vocabulary), cache the result per model instance, and raise a
RuntimeError naming every missing component.
"""
from __future__ import annotations

import logging
from typing import Optional

import torch.nn as nn

from tide_b200.adapters.base import BaseAdapter, hidden_of

logger = logging.getLogger("TIDE")

# Attribute paths per component, most common architectures first.
LAYER_PATHS = ("model.layers", "transformer.h", "transformer.layers", "gpt_neox.layers",
               "model.decoder.layers")
NORM_PATHS = ("model.norm", "transformer.ln_f", "transformer.final_layernorm",
              "model.decoder.final_layer_norm", "model.final_layernorm")
LM_HEAD_PATHS = ("lm_head", "output")
EMBEDDING_PATHS = ("model.embed_tokens", "transformer.wte", "transformer.word_embeddings",
                   "gpt_neox.embed_in", "model.decoder.embed_tokens")


def resolve(obj, dotted: str):
    """getattr along a dotted path; None as soon as a step is missing."""
    for part in dotted.split(".") if dotted else ():
        obj = getattr(obj, part, None)
        if obj is None:
            return None
    return obj


def is_norm(module: nn.Module) -> bool:
    if isinstance(module, nn.LayerNorm) or (hasattr(nn, "RMSNorm") and isinstance(module, nn.RMSNorm)):
        return True
    name = type(module).__name__.lower()
    return "rmsnorm" in name or "layernorm" in name


class UniversalAdapter(BaseAdapter):
    def __init__(self):
        self._model_id: Optional[int] = None
        self._layers = self._norm = self._lm_head = self._embedding = None
        self._hidden: Optional[int] = None

    # -- probing --------------------------------------------------------
    def _find_layers(self, model, notes):
        for path in LAYER_PATHS:
            obj = resolve(model, path)
            if isinstance(obj, nn.ModuleList) and len(obj) > 0:
                notes.append(f"layers at '{path}' ({len(obj)})")
                return list(obj)
        best_name, best = None, None
        for name, mod in model.named_modules():
            if isinstance(mod, nn.ModuleList) and (best is None or len(mod) > len(best)):
                best_name, best = name, mod
        if best is not None and len(best) >= 2:
            notes.append(f"layers: largest ModuleList '{best_name}' ({len(best)})")
            return list(best)
        return None

    def _first_path(self, model, paths):
        for path in paths:
            obj = resolve(model, path)
            if obj is not None:
                return obj
        return None

    def _sibling_norm(self, model, notes):
        if not self._layers:
            return None
        first = self._layers[0]
        for name, mod in model.named_modules():
            if isinstance(mod, nn.ModuleList) and len(mod) > 0 and mod[0] is first:
                parent = resolve(model, name.rsplit(".", 1)[0]) if "." in name else model
                if parent is None:
                    continue
                for child_name, child in parent.named_children():
                    if is_norm(child):
                        notes.append(f"final_norm: sibling '{child_name}' of '{name}'")
                        return child
        return None

    def _by_vocab(self, model, kind):
        vocab = getattr(getattr(model, "config", None), "vocab_size", None)
        if vocab is None:
            return None
        for _, mod in model.named_modules():
            if kind is nn.Linear and isinstance(mod, nn.Linear) and mod.out_features == vocab:
                return mod
            if kind is nn.Embedding and isinstance(mod, nn.Embedding) and mod.num_embeddings == vocab:
                return mod
        return None

    def _probe(self, model: nn.Module) -> None:
        notes: list[str] = []
        self._layers = self._find_layers(model, notes)
        self._norm = self._first_path(model, NORM_PATHS) or self._sibling_norm(model, notes)
        if self._norm is None:
            notes.append("final_norm: no known path and no norm next to the layers")
        self._lm_head = self._first_path(model, LM_HEAD_PATHS) or self._by_vocab(model, nn.Linear)
        if self._lm_head is None:
            notes.append("lm_head: no known path and no Linear sized like the vocabulary")
        self._embedding = (self._first_path(model, EMBEDDING_PATHS)
                           or self._by_vocab(model, nn.Embedding))
        if self._embedding is None:
            notes.append("embedding: no known path and no Embedding sized like the vocabulary")
        self._hidden = getattr(getattr(model, "config", None), "hidden_size", None)
        if self._hidden is None:
            notes.append("hidden_dim: model.config.hidden_size not found")
        missing = [k for k, v in (("layers", self._layers), ("final_norm", self._norm),
                                  ("lm_head", self._lm_head), ("hidden_dim", self._hidden))
                   if v is None]
        if missing:
            raise RuntimeError(
                f"UniversalAdapter failed to probe model {type(model).__name__}. "
                f"Missing components: {missing}. Diagnostics:\n"
                + "\n".join(f"  - {n}" for n in notes))
        logger.info(f"UniversalAdapter probed {type(model).__name__}: {len(self._layers)} layers, "
                    f"hidden_dim={self._hidden}")

    def _ensure(self, model):
        if self._model_id != id(model):
            self._probe(model)
            self._model_id = id(model)

    # -- BaseAdapter ------------------------------------------------------
    def get_layers(self, model):
        self._ensure(model)
        return self._layers

    def get_hidden_state(self, layer_output):
        return hidden_of(layer_output)

    def get_final_norm(self, model):
        self._ensure(model)
        return self._norm

    def get_lm_head(self, model):
        self._ensure(model)
        return self._lm_head

    def get_router_input_dim(self, model):
        self._ensure(model)
        return self._hidden

    def get_embedding(self, model):
        self._ensure(model)
        return self._embedding

    def get_position_embeddings(self, model, position_ids, hidden):
        for attr in ("model", "transformer", "gpt_neox"):
            rotary = getattr(getattr(model, attr, None), "rotary_emb", None)
            if rotary is not None:
                return rotary(hidden, position_ids)
        return None

    @classmethod
    def probe(cls, model: nn.Module) -> "UniversalAdapter":
        a = cls()
        a._probe(model)
        a._model_id = id(model)
        return a
