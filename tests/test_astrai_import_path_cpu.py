"""The reference's import paths resolve to this framework's modules (README quick-start code runs unchanged)."""

import subprocess
import sys

import pytest


def test_top_level_names_are_the_frameworks():
    import astrai
    import astrai_b200

    for name in astrai_b200.__all__:
        assert getattr(astrai, name) is getattr(astrai_b200, name), name


@pytest.mark.parametrize("ref_path,b200_path", [
    ("astrai.model", "astrai_b200.models"),
    ("astrai.model.components.linear", "astrai_b200.models.components.basic"),
    ("astrai.model.components.rope", "astrai_b200.models.components.basic"),
    ("astrai.model.components.lora", "astrai_b200.models.components.lora"),
    ("astrai.config.train_config", "astrai_b200.config.train_config"),
    ("astrai.inference.core.cache", "astrai_b200.inference.core.cache"),
    ("astrai.inference.api.server", "astrai_b200.inference.api.server"),
    ("astrai.parallel.executor", "astrai_b200.parallel.executor"),
    ("astrai.trainer.strategy", "astrai_b200.trainer.strategy"),
    ("astrai.tokenize.chat_template", "astrai_b200.tokenize.tokenizer"),
    ("astrai.preprocessing.packing", "astrai_b200.preprocessing.pipeline"),
    ("astrai.extension.ops", "astrai_b200.extension"),
])
def test_submodules_alias_the_same_module_object(ref_path, b200_path):
    import importlib

    assert importlib.import_module(ref_path) is importlib.import_module(b200_path)


def test_reference_style_quick_start_imports():
    from astrai.config import AutoRegressiveLMConfig, TrainConfig  # noqa: F401
    from astrai.inference import GenerationRequest, InferenceEngine  # noqa: F401
    from astrai.model import AutoModel, AutoRegressiveLM
    from astrai.parallel import spawn_parallel_fn  # noqa: F401
    from astrai.trainer import SchedulerFactory, StrategyFactory, Trainer  # noqa: F401

    cfg = AutoRegressiveLMConfig(vocab_size=64, hidden_size=32, num_hidden_layers=1, rms_norm_eps=1e-5,
                                 intermediate_size=64, max_position_embeddings=16, rope_theta=1e4,
                                 num_attention_heads=2, num_key_value_heads=1)
    m = AutoRegressiveLM(cfg)
    assert isinstance(m, AutoModel)
    assert "seq" in StrategyFactory.list_registered() and "cosine" in SchedulerFactory.list_registered()


def test_registries_are_shared():
    from astrai.model import AutoModel as A
    from astrai_b200.models import AutoModel as B

    @A.register("alias_probe_model")
    class Probe(A):
        pass

    assert B.get_component_class("alias_probe_model") is Probe


def test_module_cli_runs_under_the_reference_name():
    out = subprocess.run([sys.executable, "-m", "astrai.cli.preprocess", "--help"], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0 and "--tokenizer_path" in out.stdout


def test_unknown_submodule_is_an_import_error():
    with pytest.raises(ImportError):
        __import__("astrai.model.no_such_module")
