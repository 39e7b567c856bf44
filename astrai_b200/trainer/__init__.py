from astrai_b200.trainer.rollout import BaseRewardModel, RawRollout, RolloutGenerator, RolloutResult, RolloutRunner
from astrai_b200.trainer.schedule import BaseScheduler, SchedulerFactory
from astrai_b200.trainer.strategy import BaseStrategy, StrategyFactory
from astrai_b200.trainer.train_callback import CallbackFactory, TrainCallback
from astrai_b200.trainer.train_context import TrainContext, TrainContextBuilder
from astrai_b200.trainer.trainer import Trainer

__all__ = [
    "Trainer", "TrainContext", "TrainContextBuilder", "StrategyFactory", "BaseStrategy", "SchedulerFactory",
    "BaseScheduler", "CallbackFactory", "TrainCallback", "BaseRewardModel", "RawRollout", "RolloutGenerator",
    "RolloutResult", "RolloutRunner",
]
