"""The live executor's layer math on the CPU (tide_b200/live.py): a layer run
on the active rows only must give, for those rows, what the model's own HF
layer gives on the whole batch when the exited tokens' keys and values are
zeros (the reference's "zero_pad" K/V policy, python/TIDE/runtime.py:194-221).
With every token active it must give the HF layer's output itself."""
import pytest
import torch

from tide_b200.live import family_of


class ZeroPadKV:
    """A stand-in for the HF cache: returns this step's keys and values with
    the rows of exited tokens set to zero (keep [B, S] bool)."""

    def __init__(self, keep):
        self.keep = keep

    def update(self, k, v, layer_idx, cache_kwargs=None):
        m = self.keep[:, None, :, None].to(k.dtype)
        return k * m, v * m

    def get_seq_length(self, layer_idx=0):
        return 0


def tiny_llama(qk_norm=False):
    from transformers import LlamaConfig, LlamaForCausalLM, Qwen3Config, Qwen3ForCausalLM

    torch.manual_seed(0)
    if qk_norm:
        cfg = Qwen3Config(vocab_size=97, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                          num_attention_heads=4, num_key_value_heads=2, head_dim=16)
        m = Qwen3ForCausalLM(cfg)
    else:
        cfg = LlamaConfig(vocab_size=97, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                          num_attention_heads=4, num_key_value_heads=2, rope_theta=500000.0)
        m = LlamaForCausalLM(cfg)
    return m.eval()


def tiny_gpt2():
    from transformers import GPT2Config, GPT2LMHeadModel

    torch.manual_seed(0)
    return GPT2LMHeadModel(GPT2Config(vocab_size=97, n_embd=64, n_layer=2, n_head=4,
                                      n_positions=64)).eval()


def hf_layer(model, fam, i, h_full, keep, B, S):
    """The model's own layer i on the whole [B, S] batch, K/V of tokens with
    keep False zeroed."""
    cache = ZeroPadKV(keep)
    x = h_full.view(B, S, -1)
    if hasattr(model, "model"):
        pos_ids = torch.arange(S, device=x.device)[None]
        pe = model.model.rotary_emb(x, pos_ids)
        out = model.model.layers[i](x, attention_mask=None, position_ids=pos_ids,
                                    past_key_values=cache, use_cache=False, position_embeddings=pe)
    else:
        out = model.transformer.h[i](x, past_key_values=cache, use_cache=False)
    out = out[0] if isinstance(out, tuple) else out
    return out.reshape(B * S, -1)


@pytest.mark.parametrize("kind", ["llama", "qwen3", "gpt2"])
def test_live_layer_matches_model_layer(kind):
    model = tiny_gpt2() if kind == "gpt2" else tiny_llama(qk_norm=kind == "qwen3")
    fam = family_of(model)
    B, S = 3, 11
    ids = torch.randint(0, 97, (B, S), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        h = fam.embed_tokens(ids)
        seq = torch.arange(S).repeat(B)
        # every token active
        ours = fam.layer(0, h, None, seq, B, S)
        ref = hf_layer(model, fam, 0, h, torch.ones(B, S, dtype=torch.bool), B, S)
        torch.testing.assert_close(ours, ref, atol=1e-5, rtol=1e-5)
        # a subset active: the rows of the active tokens, exited K/V zero
        keep = torch.rand(B, S, generator=torch.Generator().manual_seed(2)) < 0.6
        pos = keep.reshape(-1).nonzero()[:, 0]
        ours = fam.layer(1, h[pos], pos, pos % S, B, S)
        ref = hf_layer(model, fam, 1, h, keep, B, S)[pos]
        torch.testing.assert_close(ours, ref, atol=1e-5, rtol=1e-5)


def test_live_embedding_matches_model():
    for model in (tiny_llama(), tiny_gpt2()):
        fam = family_of(model)
        ids = torch.randint(0, 97, (2, 9), generator=torch.Generator().manual_seed(3))
        with torch.no_grad():
            hs = model(ids, output_hidden_states=True).hidden_states
            torch.testing.assert_close(fam.embed_tokens(ids), hs[0].reshape(18, -1))


class CaptureKV:
    """A stand-in for the HF cache that keeps the keys and values it is given."""

    def __init__(self):
        self.k = self.v = None

    def update(self, k, v, layer_idx, cache_kwargs=None):
        self.k, self.v = k, v
        return k, v

    def get_seq_length(self, layer_idx=0):
        return 0


@pytest.mark.parametrize("kind", ["llama", "qwen3"])
def test_prefill_layer_stores_the_models_keys_and_values(kind):
    """The live decoder's prefill layer gives the model layer's output and
    stores, per sequence slot and position, the keys and values the model's
    attention uses (after rotary embedding and, for Qwen3, the k-norm)."""
    model = tiny_llama(qk_norm=kind == "qwen3")
    fam = family_of(model)
    B, S = 3, 7
    ids = torch.randint(0, 97, (B, S), generator=torch.Generator().manual_seed(4))
    nkv, d = fam.kv_heads(), fam.head_dim()
    kc = torch.zeros(B + 2, nkv, 12, d)
    vc = torch.zeros_like(kc)
    with torch.no_grad():
        h = fam.embed_tokens(ids)
        ours = fam.prefill_layer(0, h, B, S, kc, vc)
        cap = CaptureKV()
        x = h.view(B, S, -1)
        pos_ids = torch.arange(S)[None]
        pe = model.model.rotary_emb(x, pos_ids)
        ref = model.model.layers[0](x, attention_mask=None, position_ids=pos_ids,
                                    past_key_values=cap, use_cache=False, position_embeddings=pe)
        ref = ref[0] if isinstance(ref, tuple) else ref
    torch.testing.assert_close(ours, ref.reshape(B * S, -1), atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(kc[:B, :, :S], cap.k, atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(vc[:B, :, :S], cap.v, atol=1e-6, rtol=1e-6)
    assert torch.all(kc[B:] == 0) and torch.all(kc[:, :, S:] == 0)
