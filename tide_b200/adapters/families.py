"""Adapters for the registered HF families (LLaMA 2/3, Mistral, Qwen2), the
three entries of the reference's registry (python/TIDE/adapters/auto.py:14-18,
llama.py, mistral.py, qwen.py); they share the decoder-only layout."""
from __future__ import annotations

from tide_b200.adapters.base import DecoderOnlyAdapter


class LlamaAdapter(DecoderOnlyAdapter):
    """LlamaForCausalLM (LLaMA 2/3, CodeLlama, ...)."""


class MistralAdapter(DecoderOnlyAdapter):
    """MistralForCausalLM."""


class QwenAdapter(DecoderOnlyAdapter):
    """Qwen2ForCausalLM."""
