"""Host-side API on the CPU: the package's exported names (python/TIDE/
__init__.py:1-7), TIDEConfig's YAML layout (python/TIDE/config.py:9-33),
ExitStats (python/TIDE/scheduler.py:12-36), the TokenRouter module on a
router.pt the reference wrote (python/TIDE/router.py:11-52), and adapter
resolution (python/TIDE/adapters/auto.py:14-43).  No device code runs."""
import numpy as np
import pytest
import torch
import yaml

from tests.conftest import GOLDEN

REFERENCE_EXPORTS = ["TIDE", "TIDEConfig", "calibrate", "register_adapter", "UniversalAdapter"]
REFERENCE_CONFIG_FIELDS = {
    "checkpoint_interval": 4, "exit_threshold": 0.85, "min_layers": 8,
    "compaction_threshold": 0.25, "exit_strategy": "identity", "calibration_samples": 2000,
    "calibration_dataset": "wikitext", "router_bottleneck_dim": 128,
    "convergence_threshold": 0.98, "kv_cache_strategy": "zero_pad", "profile": False,
}


def test_package_exports_the_reference_names():
    import tide_b200
    from tide_b200.runtime import TIDERuntime

    for name in REFERENCE_EXPORTS:
        assert name in tide_b200.__all__
        assert getattr(tide_b200, name) is not None
    assert tide_b200.TIDE is TIDERuntime
    with pytest.raises(NotImplementedError):
        tide_b200.calibrate(None, None)
    with pytest.raises(AttributeError):
        tide_b200.not_an_export


def test_config_defaults_and_yaml_round_trip(tmp_path):
    from tide_b200 import TIDEConfig

    c = TIDEConfig()
    for k, v in REFERENCE_CONFIG_FIELDS.items():
        assert getattr(c, k) == v, k
    assert c.live_compaction is False
    c2 = TIDEConfig(exit_threshold=0.7, min_layers=4, exit_strategy="learned", live_compaction=True)
    c2.save(tmp_path / "sub" / "tide.yaml")
    assert TIDEConfig.load(tmp_path / "sub" / "tide.yaml") == c2


def test_config_written_with_the_reference_fields_loads(tmp_path):
    """A file holding only the reference's eleven fields (what its save()
    writes) loads, with this package's own field at its default."""
    from tide_b200 import TIDEConfig

    fields = dict(REFERENCE_CONFIG_FIELDS, exit_threshold=0.9, checkpoint_interval=2)
    (tmp_path / "ref.yaml").write_text(yaml.dump(fields, default_flow_style=False))
    c = TIDEConfig.load(tmp_path / "ref.yaml")
    assert c.exit_threshold == 0.9 and c.checkpoint_interval == 2 and c.live_compaction is False
    (tmp_path / "empty.yaml").write_text("")
    assert TIDEConfig.load(tmp_path / "empty.yaml") == TIDEConfig()


def test_exit_stats_accounting():
    from tide_b200.scheduler import ExitStats

    s = ExitStats(total_tokens=200, exits_per_layer={11: 30, 7: 20}, remaining_tokens=150)
    assert s.total_exited == 50 and s.exit_rate == 0.25
    lines = s.summary().splitlines()
    assert lines[0] == "Total tokens: 200, Exited: 50 (25.0%)"
    assert lines[1:] == ["  Layer 7: 20 exits (10.0%)", "  Layer 11: 30 exits (15.0%)",
                         "  Ran all layers: 150"]
    assert ExitStats().exit_rate == 0.0


def test_token_router_module_on_a_reference_router_file(tmp_path):
    """The module forward of routers loaded from the reference-written
    router.pt gives the scores the reference's own TokenRouter gave on the
    same rows; saving and loading again keeps the layout and the scores."""
    from tide_b200.router import RouterCheckpoint

    ck = RouterCheckpoint.load(GOLDEN / "router_ref.pt")
    ref = np.load(GOLDEN / "router_ref_scores.npz")
    assert (ck.hidden_dim, ck.bottleneck_dim, sorted(ck.routers)) == (64, 32, [3, 7])
    x = torch.from_numpy(ref["x"])
    with torch.no_grad():
        for layer, key in ((3, "s3"), (7, "s7")):
            r = ck.routers[layer]
            assert r.up.bias is None and r.exit_proj is None and r.up_bias_value == 0.0
            np.testing.assert_allclose(r(x).numpy(), ref[key], atol=1e-6, rtol=0)
    ck.save(tmp_path / "again.pt")
    state = torch.load(tmp_path / "again.pt", weights_only=True)
    assert set(state) == {"hidden_dim", "bottleneck_dim", "router_layers"}
    assert sorted(state["router_layers"]) == [3, 7]
    assert set(state["router_layers"][3]) == {"down.weight", "up.weight"}
    ck2 = RouterCheckpoint.load(tmp_path / "again.pt")
    with torch.no_grad():
        np.testing.assert_array_equal(ck2.routers[7](x).numpy(), ck.routers[7](x).numpy())


def _tiny(kind):
    from transformers import (GPT2Config, GPT2LMHeadModel, LlamaConfig, LlamaForCausalLM,
                              Qwen3Config, Qwen3ForCausalLM)

    torch.manual_seed(0)
    if kind == "llama":
        return LlamaForCausalLM(LlamaConfig(vocab_size=97, hidden_size=64, intermediate_size=128,
                                            num_hidden_layers=3, num_attention_heads=4,
                                            num_key_value_heads=2))
    if kind == "qwen3":
        return Qwen3ForCausalLM(Qwen3Config(vocab_size=97, hidden_size=64, intermediate_size=128,
                                            num_hidden_layers=3, num_attention_heads=4,
                                            num_key_value_heads=2, head_dim=16))
    return GPT2LMHeadModel(GPT2Config(vocab_size=97, n_embd=64, n_layer=3, n_head=4,
                                      n_positions=64))


@pytest.mark.parametrize("kind", ["llama", "qwen3", "gpt2"])
def test_adapter_resolution(kind):
    """Registered class names get their adapter; anything else is probed by
    UniversalAdapter, which must find the layer stack, the final norm, the
    lm_head and the embedding of each family."""
    from tide_b200.adapters.auto import get_adapter

    m = _tiny(kind).eval()
    a = get_adapter(m)
    layers = a.get_layers(m)
    assert len(layers) == 3
    assert a.get_router_input_dim(m) == 64
    head = a.get_lm_head(m)
    assert head.weight.shape == (97, 64)
    emb = a.get_embedding(m)
    assert emb.weight.shape[0] == 97
    norm = a.get_final_norm(m)
    seen = []
    hook = layers[-1].register_forward_hook(
        lambda mod, args, out: seen.append(a.get_hidden_state(out)))
    try:
        with torch.no_grad():
            ids = torch.randint(0, 97, (2, 5))
            out = m(ids, output_hidden_states=True)
            # the model's last hidden state is its final norm applied to the
            # last layer's output, and its logits are the lm_head of that
            last = out.hidden_states[-1]
            assert seen[0].shape == last.shape
            assert torch.allclose(norm(seen[0]), last, atol=1e-5)
            assert torch.allclose(head(last), out.logits, atol=1e-5)
            # older transformers releases return (hidden, ...) tuples
            assert a.get_hidden_state((last, None)) is last
    finally:
        hook.remove()


def test_register_adapter_takes_precedence():
    from tide_b200 import register_adapter
    from tide_b200.adapters.auto import ADAPTER_REGISTRY, get_adapter
    from tide_b200.adapters.base import DecoderOnlyAdapter

    class MarkedAdapter(DecoderOnlyAdapter):
        pass

    m = _tiny("qwen3")
    name = type(m).__name__
    before = ADAPTER_REGISTRY.get(name)
    try:
        register_adapter(name, MarkedAdapter)
        assert isinstance(get_adapter(m), MarkedAdapter)
    finally:
        if before is None:
            ADAPTER_REGISTRY.pop(name, None)
        else:
            ADAPTER_REGISTRY[name] = before
