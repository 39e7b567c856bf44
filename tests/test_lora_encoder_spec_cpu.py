"""LoRA adapters, the embedding encoder and tied embeddings on CPU: construction, forward, merge,
adapter files, trainable-parameter set, pooling and save/load. Behaviour the reference's module
suite specifies (tests/module/test_lora.py, test_encoder.py, test_tie_weight.py there), written
against this framework's public API."""

import logging
import os

import pytest
import torch

from astrai_b200.config import AutoRegressiveLMConfig, EncoderConfig
from astrai_b200.models import AutoModel, AutoRegressiveLM, EmbeddingEncoder, LoRAConfig, LoRALinear
from astrai_b200.models import inject_lora, load_lora, merge_lora, save_lora
from astrai_b200.models.components.basic import Linear
from astrai_b200.models.components.lora import TARGET_MODULES_ATTN, TARGET_MODULES_FFN, lora_count


def lm_config(**kw):
    base = dict(vocab_size=64, hidden_size=32, num_hidden_layers=2, rms_norm_eps=1e-5, intermediate_size=64,
                max_position_embeddings=32, rope_theta=1e4, num_attention_heads=4, num_key_value_heads=2)
    base.update(kw)
    return AutoRegressiveLMConfig(**base)


def lm(**kw):
    torch.manual_seed(0)
    return AutoRegressiveLM(lm_config(**kw)).eval()


def ids(B=2, S=8, V=64, seed=1):
    return torch.randint(0, V, (B, S), generator=torch.Generator().manual_seed(seed))


def randomise_b(model):
    with torch.no_grad():
        for m in model.modules():
            if isinstance(m, LoRALinear) and not m.merged:
                m.lora_B.normal_(0, 0.5)


# ---------------------------------------------------------------------------------------- LoRALinear
def test_loralinear_shapes_and_init():
    base = Linear(16, 24)
    m = LoRALinear(base, r=4, alpha=8)
    assert m.lora_A.shape == (4, 16) and m.lora_B.shape == (24, 4)
    assert torch.count_nonzero(m.lora_B) == 0 and m.scaling == 2.0
    assert m.weight is base.weight and not m.weight.requires_grad


def test_loralinear_starts_as_the_base_projection():
    base = Linear(16, 24)
    x = torch.randn(3, 16)
    ref = base(x)
    assert torch.allclose(LoRALinear(base, r=4)(x), ref)


def test_loralinear_adds_the_scaled_low_rank_update():
    base = Linear(16, 24)
    m = LoRALinear(base, r=4, alpha=12)
    with torch.no_grad():
        m.lora_B.normal_()
    x = torch.randn(5, 16)
    expect = x @ base.weight.T + (x @ m.lora_A.T) @ m.lora_B.T * 3.0
    assert torch.allclose(m(x), expect, atol=1e-5)


def test_loralinear_merge_keeps_the_output_and_drops_the_adapter():
    m = LoRALinear(Linear(16, 24), r=4)
    with torch.no_grad():
        m.lora_B.normal_()
    x = torch.randn(5, 16)
    before = m(x)
    m.merge()
    assert m.merged and not hasattr(m, "lora_A")
    assert torch.allclose(m(x), before, atol=1e-4)


def test_loralinear_merge_twice_changes_nothing():
    m = LoRALinear(Linear(16, 24), r=4)
    with torch.no_grad():
        m.lora_B.normal_()
    m.merge()
    w = m.weight.clone()
    m.merge()
    assert torch.equal(m.weight, w)


def test_loralinear_residual_argument():
    m = LoRALinear(Linear(16, 24), r=2)
    x, res = torch.randn(3, 16), torch.randn(3, 24)
    assert torch.allclose(m(x, residual=res), m(x) + res, atol=1e-6)


# ---------------------------------------------------------------------------------------- inject / merge
def test_inject_default_targets_the_attention_projections():
    model = lm()
    inject_lora(model)
    names = {n.rpartition(".")[2] for n, m in model.named_modules() if isinstance(m, LoRALinear)}
    assert names == TARGET_MODULES_ATTN


def test_inject_ffn_targets():
    model = lm()
    inject_lora(model, target_modules=TARGET_MODULES_FFN)
    names = {n.rpartition(".")[2] for n, m in model.named_modules() if isinstance(m, LoRALinear)}
    assert names == TARGET_MODULES_FFN


def test_inject_returns_the_adapter_config():
    cfg = inject_lora(lm(), r=8, alpha=16, target_modules={"v_proj", "q_proj"})
    assert cfg == LoRAConfig(r=8, alpha=16, target_modules=("q_proj", "v_proj"))


def test_inject_with_no_matching_name_warns(caplog):
    with caplog.at_level(logging.WARNING):
        inject_lora(lm(), target_modules={"not_a_layer"})
    assert "not_a_layer" in caplog.text and lora_count(lm()) == 0


def test_inject_keeps_the_model_output():
    model, x = lm(), ids()
    ref = model(x)["logits"]
    inject_lora(model, target_modules=TARGET_MODULES_ATTN | TARGET_MODULES_FFN)
    assert torch.allclose(model(x)["logits"], ref, atol=1e-5)


def test_inject_twice_does_not_wrap_adapters():
    model = lm()
    inject_lora(model, target_modules={"q_proj"})
    n = lora_count(model)
    inject_lora(model, target_modules={"q_proj"})
    assert lora_count(model) == n == model.config.num_hidden_layers


def test_inject_adds_only_adapter_parameters():
    model = lm()
    before = {n for n, _ in model.named_parameters()}
    inject_lora(model, target_modules={"q_proj"})
    added = {n for n, _ in model.named_parameters()} - before
    assert added and all(n.endswith((".lora_A", ".lora_B")) for n in added)


def test_inject_on_an_mla_model():
    model = lm(attn_type="mla", kv_lora_rank=16, qk_nope_head_dim=4, qk_rope_head_dim=4, num_key_value_heads=4)
    inject_lora(model, target_modules={"q_proj", "o_proj"})
    assert lora_count(model) == 2 * model.config.num_hidden_layers
    assert torch.isfinite(model(ids())["logits"]).all()


def test_inject_on_a_moe_model():
    model = lm(ffn_type="moe", n_routed_experts=4, n_shared_experts=1, n_activated_experts=2,
               moe_intermediate_size=32)
    inject_lora(model, target_modules=TARGET_MODULES_ATTN)
    assert lora_count(model) == 4 * model.config.num_hidden_layers
    assert torch.isfinite(model(ids())["logits"]).all()


def test_adapter_state_dict_keys_follow_the_module_path():
    model = lm()
    inject_lora(model, target_modules={"v_proj"})
    keys = [k for k in model.state_dict() if "lora" in k]
    assert "layers.0.attention.v_proj.lora_A" in keys or any(k.endswith("v_proj.lora_A") for k in keys)
    assert all(k.endswith((".lora_A", ".lora_B")) for k in keys)


def test_only_adapters_train_after_freezing_the_rest():
    model = lm()
    inject_lora(model)
    for n, p in model.named_parameters():
        p.requires_grad_("lora_" in n)
    loss = model(ids())["logits"].float().pow(2).mean()
    loss.backward()
    grads = {n for n, p in model.named_parameters() if p.grad is not None}
    assert grads and all("lora_" in n for n in grads)


def test_base_weights_keep_their_state_dict_names():
    model = lm()
    names = set(model.state_dict())
    inject_lora(model, target_modules=TARGET_MODULES_ATTN | TARGET_MODULES_FFN)
    assert names <= set(model.state_dict())


def test_merge_keeps_the_model_output():
    model, x = lm(), ids()
    inject_lora(model, target_modules={"q_proj", "up"})
    randomise_b(model)
    before = model(x)["logits"]
    merge_lora(model)
    assert lora_count(model) == 0
    assert torch.allclose(model(x)["logits"], before, atol=1e-4)


def test_merge_without_adapters_warns(caplog):
    with caplog.at_level(logging.WARNING):
        merge_lora(lm())
    assert "adapter" in caplog.text


# ---------------------------------------------------------------------------------------- adapter files
def test_save_load_round_trip_gives_the_same_output(tmp_path):
    model, x = lm(), ids()
    cfg = inject_lora(model, r=4, alpha=8, target_modules={"q_proj", "down"})
    randomise_b(model)
    want = model(x)["logits"]
    save_lora(model, str(tmp_path), cfg)
    assert sorted(os.listdir(tmp_path)) == ["adapter_config.json", "adapter_model.safetensors"]
    fresh = lm()
    assert load_lora(fresh, str(tmp_path)) == cfg
    assert torch.allclose(fresh(x)["logits"], want, atol=1e-5)


def test_saving_after_merge_raises(tmp_path):
    model = lm()
    cfg = inject_lora(model)
    merge_lora(model)
    with pytest.raises(RuntimeError):
        save_lora(model, str(tmp_path), cfg)


def test_load_into_an_already_injected_model(tmp_path):
    src = lm()
    cfg = inject_lora(src, r=4, target_modules={"k_proj"})
    randomise_b(src)
    save_lora(src, str(tmp_path), cfg)
    dst = lm()
    inject_lora(dst, r=4, target_modules={"k_proj"})
    load_lora(dst, str(tmp_path))
    a = dict(src.named_parameters())
    for n, p in dst.named_parameters():
        if "lora_" in n:
            assert torch.equal(p, a[n])


def test_loading_an_adapter_of_another_rank_raises(tmp_path):
    src = lm()
    save_lora(src, str(tmp_path), inject_lora(src, r=4))
    dst = lm()
    inject_lora(dst, r=8)
    with pytest.raises(RuntimeError):
        load_lora(dst, str(tmp_path))


def test_adapter_targets_that_match_nothing_raise(tmp_path):
    src = lm()
    save_lora(src, str(tmp_path), inject_lora(src, r=2, target_modules={"q_proj"}))
    import json

    p = tmp_path / "adapter_config.json"
    cfg = json.loads(p.read_text())
    cfg["target_modules"] = ["nothing_here"]
    p.write_text(json.dumps(cfg))
    with pytest.raises(RuntimeError):
        load_lora(lm(), str(tmp_path))


# ---------------------------------------------------------------------------------------- encoder
def enc_config(**kw):
    base = dict(vocab_size=64, hidden_size=32, num_hidden_layers=2, rms_norm_eps=1e-5, intermediate_size=64,
                max_position_embeddings=32, rope_theta=1e4, num_attention_heads=4, num_key_value_heads=2)
    base.update(kw)
    return EncoderConfig(**base)


@pytest.mark.parametrize("pooling", ["cls", "last", "mean"])
def test_encoder_pools_one_vector_per_sequence(pooling):
    enc = EmbeddingEncoder(enc_config(pooling_type=pooling)).eval()
    out = enc(ids(B=3, S=10))
    assert out.shape == (3, 32) and torch.isfinite(out).all()


def test_encoder_ignores_padding():
    enc = EmbeddingEncoder(enc_config(pooling_type="mean")).eval()
    x = ids(B=1, S=6)
    mask = torch.ones(1, 6, dtype=torch.bool)
    padded = torch.cat([x, torch.zeros(1, 3, dtype=torch.long)], 1)
    pmask = torch.cat([mask, torch.zeros(1, 3, dtype=torch.bool)], 1)
    assert torch.allclose(enc(x, mask), enc(padded, pmask), atol=1e-5)


def test_encoder_last_pooling_picks_the_last_valid_token():
    enc = EmbeddingEncoder(enc_config(pooling_type="last")).eval()
    x = ids(B=1, S=5)
    padded = torch.cat([x, torch.zeros(1, 2, dtype=torch.long)], 1)
    pmask = torch.tensor([[1, 1, 1, 1, 1, 0, 0]], dtype=torch.bool)
    assert torch.allclose(enc(x, torch.ones(1, 5, dtype=torch.bool)), enc(padded, pmask), atol=1e-5)


def test_encoder_normalised_embeddings_have_unit_norm():
    enc = EmbeddingEncoder(enc_config(normalize_embeddings=True)).eval()
    assert torch.allclose(enc(ids(B=4)).norm(dim=-1), torch.ones(4), atol=1e-5)


def test_encoder_is_registered_as_embedding():
    assert AutoModel.get_component_class("embedding") is EmbeddingEncoder


def test_encoder_loads_an_lm_checkpoint_without_its_head():
    src = lm()
    enc = EmbeddingEncoder(enc_config())
    enc.load_state_dict(src.state_dict())
    assert torch.equal(enc.embed_tokens.weight, src.embed_tokens.weight)


def test_encoder_save_and_from_pretrained(tmp_path):
    enc = EmbeddingEncoder(enc_config(pooling_type="cls")).eval()
    enc.save_pretrained(str(tmp_path))
    back = AutoModel.from_pretrained(str(tmp_path)).eval()
    x = ids()
    assert isinstance(back, EmbeddingEncoder) and torch.allclose(back(x), enc(x), atol=1e-6)


def test_encoder_rejects_unknown_pooling():
    with pytest.raises(ValueError):
        EmbeddingEncoder(enc_config(pooling_type="max"))


# ---------------------------------------------------------------------------------------- tied embeddings
def test_tied_model_shares_one_tensor():
    model = lm(tie_word_embeddings=True)
    assert model.lm_head.weight is model.embed_tokens.weight
    assert "lm_head.weight" not in model.state_dict()


def test_tied_model_save_load_keeps_the_tie(tmp_path):
    model = lm(tie_word_embeddings=True)
    model.save_pretrained(str(tmp_path))
    back = AutoModel.from_pretrained(str(tmp_path)).eval()
    assert back.lm_head.weight is back.embed_tokens.weight
    x = ids()
    assert torch.allclose(back(x)["logits"], model(x)["logits"], atol=1e-6)


def test_from_pretrained_places_and_casts(tmp_path):
    lm().save_pretrained(str(tmp_path))
    back = AutoModel.from_pretrained(str(tmp_path), device="cpu", dtype=torch.bfloat16)
    assert all(p.dtype == torch.bfloat16 for p in back.parameters())
    assert back.rotary_embedding.freqs_cis.dtype == torch.float32
    assert torch.isfinite(back.rotary_embedding.freqs_cis).all()


def test_from_pretrained_with_random_init_still_loads_weights(tmp_path):
    src = lm()
    src.save_pretrained(str(tmp_path))
    back = AutoModel.from_pretrained(str(tmp_path), disable_random_init=False)
    assert all(torch.equal(a, b) for a, b in zip(back.state_dict().values(), src.state_dict().values()))


def test_from_pretrained_without_config_raises(tmp_path):
    with pytest.raises(FileNotFoundError):
        AutoModel.from_pretrained(str(tmp_path))
