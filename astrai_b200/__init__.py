"""astrai_b200: a Blackwell-native (sm_100a) Transformer training and inference framework.

Public API mirrors the reference package's top level (astrai/__init__.py):
models and configs, tokenizer, datasets, trainer, parallel executors,
inference engine and server, preprocessing, serialization.
"""

__version__ = "0.1.0"

from astrai_b200.config import (AutoRegressiveLMConfig, BaseModelConfig, ConfigFactory, EncoderConfig,
                                PipelineConfig, TrainConfig)
from astrai_b200.dataset import BaseDataset, DatasetFactory, RDSampler, Store, StoreFactory
from astrai_b200.factory import BaseFactory, Registry
from astrai_b200.inference import (GenerationRequest, InferenceEngine, ProtocolHandler, SamplingPipeline, get_app,
                                   run_server, sample)
from astrai_b200.models import AutoModel, AutoRegressiveLM, EmbeddingEncoder, LoRAConfig, inject_lora
from astrai_b200.parallel import ExecutorFactory, get_rank, get_world_size, only_on_rank, spawn_parallel_fn
from astrai_b200.preprocessing import Pipeline, filter_by_length
from astrai_b200.serialization import Checkpoint
from astrai_b200.tokenize import AutoTokenizer, ChatTemplate
from astrai_b200.trainer import (BaseScheduler, BaseStrategy, CallbackFactory, SchedulerFactory, StrategyFactory,
                                 TrainCallback, Trainer)

__all__ = [
    "AutoRegressiveLM", "AutoRegressiveLMConfig", "AutoModel", "AutoTokenizer", "BaseDataset", "BaseFactory",
    "BaseModelConfig", "BaseScheduler", "BaseStrategy", "CallbackFactory", "ChatTemplate", "Checkpoint",
    "ConfigFactory", "DatasetFactory", "EmbeddingEncoder", "EncoderConfig", "ExecutorFactory", "GenerationRequest",
    "InferenceEngine", "LoRAConfig", "Pipeline", "PipelineConfig", "ProtocolHandler", "RDSampler", "Registry",
    "SamplingPipeline", "SchedulerFactory", "Store", "StoreFactory", "StrategyFactory", "TrainCallback",
    "TrainConfig", "Trainer", "filter_by_length", "get_app", "get_rank", "get_world_size", "inject_lora",
    "only_on_rank", "run_server", "sample", "spawn_parallel_fn",
]
