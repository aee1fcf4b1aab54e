"""The HF seam on real decoders: tiny random-weight Mistral (the shape of the reference's own
fake, tests/test_amdahl_probe.py:32-47: 2 layers, 4 query / 2 KV heads, head_dim 8) and Phi-3
(fused qkv_proj) models run a prefill and several decode steps against a StaticCache, once
unpatched and once with every attention layer's decode step going through the fused op.

Checked: the logits of every decode step agree (fp32 to 1e-5; bf16 within the rounding of its
cos/sin, which HF applies in the model dtype); the cache slots each step appends agree (K to
an fp32 ulp, V of the first step's first layer bit for bit: same projection of the same
input), the prefill part of the caches is untouched by the patch, and the layers' position
counters advance alike. No pretrained weights are involved.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

CTX, STEPS, BATCH, HEADROOM = 8, 4, 3, 8


@pytest.fixture(scope="module", autouse=True)
def _require_cuda():
    if not torch.cuda.is_available():
        pytest.fail("the gpu tests need a CUDA device")
    from decode_llm_kernel_b200 import cuda
    cuda.require()


def mistral(dtype):
    from transformers import MistralConfig, MistralForCausalLM
    cfg = MistralConfig(vocab_size=64, hidden_size=32, intermediate_size=64,
                        num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                        head_dim=8, max_position_embeddings=128, sliding_window=None,
                        rope_theta=10000.0, attn_implementation="sdpa")
    cfg.layer_types = ["full_attention"] * cfg.num_hidden_layers
    torch.manual_seed(0)
    return MistralForCausalLM(cfg).to("cuda", dtype).eval()


def phi3(dtype):
    from transformers import Phi3Config, Phi3ForCausalLM
    cfg = Phi3Config(vocab_size=64, hidden_size=48, intermediate_size=64, num_hidden_layers=2,
                     num_attention_heads=6, num_key_value_heads=2, max_position_embeddings=128,
                     rope_theta=10000.0, attn_implementation="sdpa", pad_token_id=0)
    torch.manual_seed(1)
    return Phi3ForCausalLM(cfg).to("cuda", dtype).eval()


def decode(model):
    """Prefill CTX tokens per sequence, then STEPS single-token steps; logits and cache."""
    from transformers.cache_utils import StaticCache
    cache = StaticCache(config=model.config, max_cache_len=CTX + HEADROOM)
    g = torch.Generator().manual_seed(1234)
    ids = torch.randint(0, model.config.vocab_size, (BATCH, CTX), generator=g).cuda()
    steps = torch.randint(0, model.config.vocab_size, (STEPS, BATCH, 1), generator=g).cuda()
    logits = []
    with torch.inference_mode():
        model(input_ids=ids, past_key_values=cache, cache_position=torch.arange(CTX).cuda(),
              use_cache=True)
        for i in range(STEPS):
            out = model(input_ids=steps[i], past_key_values=cache,
                        cache_position=torch.tensor([CTX + i]).cuda(), use_cache=True)
            logits.append(out.logits[:, -1].float())
    torch.cuda.synchronize()
    return torch.stack(logits), cache


@pytest.mark.parametrize("make", [mistral, phi3], ids=["mistral", "phi3"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["fp32", "bf16"])
def test_patched_decode_matches_the_unpatched_model(make, dtype):
    from decode_llm_kernel_b200 import cuda, hf_seam
    model = make(dtype)
    want, cache_want = decode(model)
    calls = {"n": 0}
    real = hf_seam.ops.fused_rope_kv_append_ex

    def counting(*a, **k):
        calls["n"] += 1
        return real(*a, **k)
    hf_seam.ops.fused_rope_kv_append_ex = counting
    patch = hf_seam.patch_decoder(model)
    try:
        got, cache_got = decode(model)
    finally:
        patch.restore()
        hf_seam.ops.fused_rope_kv_append_ex = real
    cuda.check_status()
    layers = model.config.num_hidden_layers
    assert calls["n"] == STEPS * layers          # every decode step of every layer went through
    atol = 1e-5 if dtype == torch.float32 else 3e-2
    assert torch.allclose(got, want, atol=atol, rtol=1e-4 if dtype == torch.float32 else 3e-2), \
        float((got - want).abs().max())
    for lw, lg in zip(cache_want.layers, cache_got.layers):
        assert int(lw.cumulative_length) == int(lg.cumulative_length) == CTX + STEPS
        # the prefill part is written by HF's own path in both runs
        assert torch.equal(lw.keys[:, :, :CTX], lg.keys[:, :, :CTX])
        assert torch.equal(lw.values[:, :, :CTX], lg.values[:, :, :CTX])
        new = slice(CTX, CTX + STEPS)
        tol = 1e-5 if dtype == torch.float32 else 3e-2
        assert torch.allclose(lg.keys[:, :, new].float(), lw.keys[:, :, new].float(), atol=tol)
        assert torch.allclose(lg.values[:, :, new].float(), lw.values[:, :, new].float(), atol=tol)
        assert bool((lg.keys[:, :, CTX + STEPS:] == 0).all())     # nothing past the last step
    first = cache_want.layers[0], cache_got.layers[0]
    assert torch.equal(first[0].values[:, :, CTX], first[1].values[:, :, CTX])


def test_the_patch_refuses_twice_and_restores():
    from decode_llm_kernel_b200 import hf_seam
    model = mistral(torch.float32)
    before = [layer.self_attn.forward for layer in model.model.layers]
    patch = hf_seam.patch_decoder(model)
    with pytest.raises(RuntimeError, match="already patched"):
        hf_seam.patch_decoder(model)
    patch.restore()
    after = [layer.self_attn.forward for layer in model.model.layers]
    assert all(a == b for a, b in zip(before, after))
    assert all("forward" not in layer.self_attn.__dict__ for layer in model.model.layers)
