"""The HF seam's host side, on CPU: its fp32 RoPE tables equal what the model's own rotary
embedding computes for those positions, a patched model on the CPU (where the fused op cannot
run) takes the original forward and gives the unpatched logits bit for bit, and patching is
reversible and refuses to stack."""
import pytest
import torch

from decode_llm_kernel_b200 import hf_seam


def _mistral():
    from transformers import MistralConfig, MistralForCausalLM
    cfg = MistralConfig(vocab_size=64, hidden_size=32, intermediate_size=64,
                        num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                        head_dim=8, max_position_embeddings=128, sliding_window=None,
                        rope_theta=500000.0, attn_implementation="sdpa")
    cfg.layer_types = ["full_attention"] * 2
    torch.manual_seed(0)
    return MistralForCausalLM(cfg).eval()


def _phi3():
    from transformers import Phi3Config, Phi3ForCausalLM
    cfg = Phi3Config(vocab_size=64, hidden_size=48, intermediate_size=64, num_hidden_layers=2,
                     num_attention_heads=6, num_key_value_heads=2, max_position_embeddings=128,
                     rope_theta=10000.0, attn_implementation="sdpa", pad_token_id=0)
    torch.manual_seed(1)
    return Phi3ForCausalLM(cfg).eval()


@pytest.mark.parametrize("make", [_mistral, _phi3], ids=["mistral", "phi3"])
def test_tables_equal_the_models_rotary_embedding(make):
    model = make()
    rot = model.model.rotary_emb
    cos, sin = hf_seam.rope_tables_from_inv_freq(rot.inv_freq, 100,
                                                 float(rot.attention_scaling))
    c, s = rot(torch.zeros(1, 1, 8), torch.arange(100)[None])
    assert torch.equal(c[0], cos) and torch.equal(s[0], sin)


def _decode(model):
    from transformers.cache_utils import StaticCache
    cache = StaticCache(config=model.config, max_cache_len=16)
    ids = torch.randint(0, 64, (2, 6), generator=torch.Generator().manual_seed(3))
    with torch.inference_mode():
        model(input_ids=ids, past_key_values=cache, cache_position=torch.arange(6),
              use_cache=True)
        out = [model(input_ids=torch.full((2, 1), 5 + i), past_key_values=cache,
                     cache_position=torch.tensor([6 + i]), use_cache=True).logits
               for i in range(3)]
    return torch.cat(out)


@pytest.mark.parametrize("make", [_mistral, _phi3], ids=["mistral", "phi3"])
def test_on_the_cpu_the_patched_model_takes_the_original_path(make):
    model = make()
    want = _decode(model)
    patch = hf_seam.patch_decoder(model)
    with pytest.raises(RuntimeError, match="already patched"):
        hf_seam.patch_decoder(model)
    got = _decode(model)
    patch.restore()
    assert torch.equal(got, want)
    assert all("forward" not in layer.self_attn.__dict__ for layer in model.model.layers)


def test_models_without_the_layout_are_refused():
    with pytest.raises(ValueError, match="model.layers"):
        hf_seam.patch_decoder(torch.nn.Linear(2, 2))
