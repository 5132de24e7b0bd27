"""SquishCache: an HF transformers model decoding with this package's quantized KV codecs."""
import pytest
import torch


@pytest.mark.parametrize("kv_dtype,tol", [("int8", 0.02), ("int4", 0.25), ("k8v4", 0.25)])
def test_squish_cache_tracks_the_full_precision_cache(kv_dtype, tol):
    from transformers import DynamicCache, LlamaConfig, LlamaForCausalLM

    from squish_b200.integrations.hf import SquishCache

    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=128, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=32, max_position_embeddings=256)
    model = LlamaForCausalLM(cfg).eval()
    ids = torch.randint(0, 128, (1, 24))
    steps = torch.randint(0, 128, (1, 12))

    def run(cache):
        out = []
        with torch.no_grad():
            r = model(ids, past_key_values=cache, use_cache=True)
            out.append(r.logits[:, -1])
            for i in range(steps.shape[1]):
                r = model(steps[:, i:i + 1], past_key_values=cache, use_cache=True)
                out.append(r.logits[:, -1])
        return torch.cat(out)

    ref = run(DynamicCache())
    sq_cache = SquishCache(cfg, kv_dtype=kv_dtype, group=32, residual_length=4)
    got = run(sq_cache)
    assert sq_cache.get_seq_length() == 24 + 12
    assert torch.equal(got[0], ref[0])  # the prompt step attends to unquantized states
    err = ((got - ref).norm() / ref.norm()).item()
    assert 0 < err < tol, err  # > 0: older tokens really went through the codec
    with pytest.raises(ValueError):
        SquishCache(cfg, kv_dtype="int3")
