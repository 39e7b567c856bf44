from astrai_b200.parallel.executor import (
    AccumOptimizer,
    AccumScheduler,
    BaseExecutor,
    DDPExecutor,
    ExecutorFactory,
    FSDP2Executor,
    GradientState,
    NoneExecutor,
)
from astrai_b200.parallel.module import ColumnParallelLinear, ParallelModel, RowParallelLinear
from astrai_b200.parallel.setup import (
    find_free_port,
    get_current_device,
    get_rank,
    get_world_size,
    only_on_rank,
    setup_parallel,
    spawn_parallel_fn,
)

FSDPExecutor = FSDP2Executor

__all__ = [
    "ColumnParallelLinear", "ParallelModel", "RowParallelLinear", "AccumOptimizer", "AccumScheduler", "BaseExecutor", "DDPExecutor", "ExecutorFactory", "FSDPExecutor",
    "FSDP2Executor", "GradientState", "NoneExecutor", "find_free_port", "get_current_device", "get_rank",
    "get_world_size", "only_on_rank", "setup_parallel", "spawn_parallel_fn",
]
