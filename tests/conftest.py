import json
import os
import shutil
import sys
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

CHATML = ("{% for m in messages %}<|im_start|>{{ m['role'] }}\n{{ m['content'] }}<|im_end|>\n{% endfor %}"
          "{% if add_generation_prompt %}<|im_start|>assistant\n{% endif %}")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built sm_100a extension")
    config.addinivalue_line("markers", "slow: long-running test")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def make_tokenizer_files(path: str) -> None:
    """A small byte-level BPE tokenizer (HF tokenizers format) + chatml config."""
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers

    tok = Tokenizer(models.BPE(unk_token=None))
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    tok.decoder = decoders.ByteLevel()
    specials = ["<|endoftext|>", "<|im_start|>", "<|im_end|>", "<|pad|>"]
    trainer = trainers.BpeTrainer(vocab_size=400, special_tokens=specials,
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), show_progress=False)
    corpus = ["hello world, this is a tiny corpus for a test tokenizer.",
              "The quick brown fox jumps over the lazy dog 0123456789.",
              "user assistant system tool function arguments name json"] * 20
    tok.train_from_iterator(corpus, trainer)
    os.makedirs(path, exist_ok=True)
    tok.save(os.path.join(path, "tokenizer.json"))
    with open(os.path.join(path, "tokenizer_config.json"), "w") as fh:
        json.dump({"special_tokens": {"eos_token": "<|im_end|>", "pad_token": "<|pad|>",
                                      "bos_token": "<|endoftext|>"}, "chat_template": CHATML}, fh)


TINY_CFG = dict(vocab_size=512, hidden_size=64, num_attention_heads=4, num_key_value_heads=2,
                intermediate_size=128, max_position_embeddings=256, num_hidden_layers=2, rms_norm_eps=1e-5)


@pytest.fixture(scope="session")
def tokenizer_dir():
    d = tempfile.mkdtemp(prefix="astrai_tok_")
    make_tokenizer_files(d)
    yield d
    shutil.rmtree(d, ignore_errors=True)


@pytest.fixture(scope="session")
def test_tokenizer(tokenizer_dir):
    from astrai_b200.tokenize import AutoTokenizer

    return AutoTokenizer.from_pretrained(tokenizer_dir)


@pytest.fixture
def model_dir(tokenizer_dir):
    """Model directory with config.json, random weights and the tokenizer."""
    import torch

    from astrai_b200.config import AutoRegressiveLMConfig
    from astrai_b200.models import AutoRegressiveLM

    d = tempfile.mkdtemp(prefix="astrai_model_")
    torch.manual_seed(0)
    AutoRegressiveLM(AutoRegressiveLMConfig(**TINY_CFG)).save_pretrained(d)
    for f in ("tokenizer.json", "tokenizer_config.json"):
        shutil.copy(os.path.join(tokenizer_dir, f), d)
    yield d
    shutil.rmtree(d, ignore_errors=True)


@pytest.fixture
def tmpdir_path():
    d = tempfile.mkdtemp(prefix="astrai_test_")
    yield d
    shutil.rmtree(d, ignore_errors=True)
