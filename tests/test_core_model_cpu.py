"""CPU tests: registries, configs, model variants, checkpoint layout, LoRA, encoder."""

import json
import os

import pytest
import torch

from tests.conftest import TINY_CFG


def test_registry_filters_kwargs_and_validates():
    from astrai_b200.factory import Registry

    class Base:
        pass

    class Fac(Registry[Base]):
        pass

    @Fac.register("a")
    class A(Base):
        def __init__(self, x, y=2):
            self.x, self.y = x, y

    obj = Fac.create("a", x=1, y=3, unrelated=5)
    assert (obj.x, obj.y) == (1, 3)
    assert Fac.list_registered() == ["a"] and Fac.is_registered("a")
    with pytest.raises(ValueError):
        Fac.register("a")(A)
    with pytest.raises(TypeError):
        Fac.register("b")(int)
    with pytest.raises(ValueError):
        Fac.create("missing")


def test_config_roundtrip(tmpdir_path):
    from astrai_b200.config import AutoRegressiveLMConfig, ConfigFactory, EncoderConfig

    cfg = AutoRegressiveLMConfig(**TINY_CFG, rope_scaling={"type": "ntk", "factor": 2.0})
    p = os.path.join(tmpdir_path, "c.json")
    cfg.to_file(p)
    back = AutoRegressiveLMConfig.from_file(p)
    assert back == cfg
    raw = json.load(open(p))
    raw["hidden_size"] = 64.0  # coerced back to int
    assert isinstance(ConfigFactory.load(raw).hidden_size, int)
    assert isinstance(ConfigFactory.load({"model_type": "embedding", "hidden_size": 8}), EncoderConfig)


CONFIGS = {
    "gqa_mlp": {},
    "mla_mlp": dict(attn_type="mla", kv_lora_rank=16, qk_nope_head_dim=8, qk_rope_head_dim=8, num_key_value_heads=4),
    "gqa_moe": dict(ffn_type="moe", n_routed_experts=4, n_shared_experts=1, n_activated_experts=2),
    "gqa_moe_first_dense_aux": dict(ffn_type="moe", n_routed_experts=4, n_shared_experts=2, n_activated_experts=2,
                                    first_k_dense=1, moe_aux_loss_coef=0.01),
    "gqa_qk_norm_gated": dict(use_qk_norm=True, use_gated_attention=True),
    "gqa_tied_ntk": dict(tie_word_embeddings=True, rope_scaling={"type": "ntk", "factor": 2.0}),
}


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_forward_backward_and_reload(name, tmpdir_path):
    from astrai_b200.config import AutoRegressiveLMConfig
    from astrai_b200.models import AutoModel, AutoRegressiveLM

    torch.manual_seed(0)
    cfg = AutoRegressiveLMConfig(**{**TINY_CFG, **CONFIGS[name]})
    m = AutoRegressiveLM(cfg)
    ids = torch.randint(0, 512, (2, 17))
    out = m(ids)
    assert out["logits"].shape == (2, 17, 512)
    loss = out["logits"].float().logsumexp(-1).mean() + out.get("aux_loss", 0.0)
    loss.backward()
    assert all(p.grad is not None for n, p in m.named_parameters() if "routed_experts" not in n)
    m.save_pretrained(tmpdir_path)
    if cfg.tie_word_embeddings:
        from safetensors.torch import load_file

        assert "lm_head.weight" not in load_file(os.path.join(tmpdir_path, "model.safetensors"))
    m2 = AutoModel.from_pretrained(tmpdir_path)
    m.eval()
    m2.eval()
    torch.testing.assert_close(m(ids)["logits"], m2(ids)["logits"])
    if cfg.tie_word_embeddings:
        assert m2.lm_head.weight is m2.embed_tokens.weight


def test_state_dict_keys_match_reference_layout():
    from astrai_b200.config import AutoRegressiveLMConfig
    from astrai_b200.models import AutoRegressiveLM

    keys = set(AutoRegressiveLM(AutoRegressiveLMConfig(**TINY_CFG)).state_dict())
    for k in ("embed_tokens.weight", "norm.weight", "lm_head.weight", "layers.0.input_norm.weight",
              "layers.0.post_attention_norm.weight", "layers.1.attention.q_proj.weight",
              "layers.1.attention.k_proj.weight", "layers.1.attention.v_proj.weight",
              "layers.1.attention.o_proj.weight", "layers.0.mlp.up.weight", "layers.0.mlp.gate.weight",
              "layers.0.mlp.down.weight"):
        assert k in keys
    assert not any("freqs_cis" in k for k in keys)


def test_masks_fast_path_equals_dense_mask():
    """Segment ids (fast path) == dense doc-boundary mask (reference API)."""
    from astrai_b200.config import AutoRegressiveLMConfig
    from astrai_b200.models import AutoRegressiveLM
    from astrai_b200.trainer.strategy import doc_ids_from_positions, make_doc_boundary_mask

    torch.manual_seed(0)
    m = AutoRegressiveLM(AutoRegressiveLMConfig(**TINY_CFG)).eval()
    pos = torch.tensor([[0, 1, 2, 0, 1, 2, 3, 0], [0, 1, 2, 3, 4, 5, 6, 7]])
    ids = torch.randint(0, 512, (2, 8))
    a = m(ids, position_ids=pos, seg_ids=doc_ids_from_positions(pos))["logits"]
    b = m(ids, input_mask=make_doc_boundary_mask(pos), position_ids=pos)["logits"]
    torch.testing.assert_close(a, b, atol=1e-4, rtol=1e-4)


def test_lora_inject_merge_save_load(tmpdir_path):
    from astrai_b200.config import AutoRegressiveLMConfig
    from astrai_b200.models import AutoRegressiveLM, LoRALinear, inject_lora, load_lora, merge_lora, save_lora

    torch.manual_seed(0)
    m = AutoRegressiveLM(AutoRegressiveLMConfig(**TINY_CFG))
    cfg = inject_lora(m, r=4, alpha=8, target_modules={"q_proj", "v_proj", "up"})
    n = sum(isinstance(x, LoRALinear) for x in m.modules())
    assert n == 2 * 3
    assert not m.layers[0].attention.q_proj.weight.requires_grad
    ids = torch.randint(0, 512, (1, 9))
    with torch.no_grad():
        for mod in m.modules():
            if isinstance(mod, LoRALinear):
                mod.lora_B.normal_()
    ref = m(ids)["logits"]
    save_lora(m, tmpdir_path, cfg)
    assert json.load(open(os.path.join(tmpdir_path, "adapter_config.json")))["r"] == 4
    m2 = AutoRegressiveLM(AutoRegressiveLMConfig(**TINY_CFG))
    m2.load_state_dict({k: v for k, v in m.state_dict().items() if "lora" not in k}, strict=False)
    load_lora(m2, tmpdir_path)
    torch.testing.assert_close(m2(ids)["logits"], ref)
    merge_lora(m2)
    assert sum(isinstance(x, LoRALinear) for x in m2.modules()) == n
    torch.testing.assert_close(m2(ids)["logits"], ref, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("pool", ["mean", "cls", "last"])
def test_encoder_pooling(pool, tmpdir_path):
    from astrai_b200.config import EncoderConfig
    from astrai_b200.models import AutoModel, EmbeddingEncoder

    cfg = EncoderConfig(**{k: v for k, v in TINY_CFG.items()}, model_type="embedding", pooling_type=pool,
                        normalize_embeddings=True)
    enc = EmbeddingEncoder(cfg).eval()
    ids = torch.randint(0, 512, (2, 6))
    mask = torch.tensor([[1, 1, 1, 1, 0, 0], [1, 1, 1, 1, 1, 1]])
    e = enc(ids, input_mask=mask)
    assert e.shape == (2, 64)
    torch.testing.assert_close(e.norm(dim=-1), torch.ones(2))
    enc.save_pretrained(tmpdir_path)
    torch.testing.assert_close(AutoModel.from_pretrained(tmpdir_path).eval()(ids, input_mask=mask), e)


def test_tokenizer_and_chat_template(test_tokenizer, tmpdir_path):
    tok = test_tokenizer
    ids = tok.encode("hello world")
    assert tok.decode(ids) == "hello world"
    assert tok.encode(["hello", "world"]) == [tok.encode("hello"), tok.encode("world")]
    assert tok.eos_token == "<|im_end|>" and isinstance(tok.eos_token_id, int)
    assert set(tok.stop_ids) >= {tok.eos_token_id}
    text = tok.apply_chat_template([{"role": "user", "content": "hi"}], tokenize=False)
    assert text.endswith("<|im_start|>assistant\n")
    batch = tok.apply_chat_template([[{"role": "user", "content": "a"}], [{"role": "user", "content": "b"}]])
    assert len(batch) == 2 and all(isinstance(b, list) for b in batch)
    import pickle

    pickle.loads(pickle.dumps(tok))
    tok.save_pretrained(tmpdir_path)
    from astrai_b200.tokenize import AutoTokenizer

    assert AutoTokenizer.from_pretrained(tmpdir_path).encode("hello") == tok.encode("hello")
