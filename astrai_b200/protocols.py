"""Structural types for the optimizer / LR-scheduler objects the trainer drives.

Parity: astrai/protocols.py:6-21 (step / zero_grad / state_dict round trip).
"""

from typing import Any, Dict, Protocol, runtime_checkable


@runtime_checkable
class OptimizerProtocol(Protocol):
    def step(self, closure=None) -> Any: ...

    def zero_grad(self) -> None: ...

    def state_dict(self) -> Dict[str, Any]: ...

    def load_state_dict(self, state_dict: Dict[str, Any]) -> None: ...


@runtime_checkable
class SchedulerProtocol(Protocol):
    def step(self) -> None: ...

    def state_dict(self) -> Dict[str, Any]: ...

    def load_state_dict(self, state_dict: Dict[str, Any]) -> None: ...
