"""Host logic of the HF decode integration on CPU: patching and unpatching of the attention modules,
per-layer budgets, and the errors raised before any kernel is launched."""
import pytest
import torch


def _model(layers=3):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    torch.manual_seed(0)
    cfg = Qwen3Config(vocab_size=64, hidden_size=64, intermediate_size=128, num_hidden_layers=layers,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128)
    return Qwen3ForCausalLM(cfg).eval()


def test_patch_budgets_and_unpatch():
    from fathom_b200.hf import OffloadedDecoder
    model = _model()
    orig = [layer.self_attn.forward for layer in model.model.layers]
    dec = OffloadedDecoder(model, budget={0: 40, 1: 48, 2: 80}, index="hbm", rows="hbm")
    assert dec.budgets == [40.0, 48.0, 80.0] and dec.G == 2 and dec.D == 128
    assert all(layer.self_attn.forward != f for layer, f in zip(model.model.layers, orig))
    with pytest.raises(RuntimeError, match="offload"):
        dec.decode(torch.zeros(1, 1, dtype=torch.long))
    with pytest.raises(RuntimeError, match="prefill"):
        with torch.no_grad():
            model(torch.zeros(1, 4, dtype=torch.long), use_cache=False)
    dec.unpatch()
    assert all(layer.self_attn.forward == f for layer, f in zip(model.model.layers, orig))
    with torch.no_grad():
        model(torch.zeros(1, 4, dtype=torch.long), use_cache=False)      # dense again
    assert OffloadedDecoder(model, budget=[32, 48, 64]).budgets == [32.0, 48.0, 64.0]
    dec2 = OffloadedDecoder(model, budget=48)
    assert dec2.budgets == [48.0] * 3
    dec2.unpatch()


def test_bad_arguments():
    from fathom_b200.hf import OffloadedDecoder
    model = _model(layers=2)
    with pytest.raises(ValueError, match="budgets"):
        OffloadedDecoder(model, budget=[48])
    with pytest.raises(ValueError, match="host"):
        OffloadedDecoder(model, index="disk")
