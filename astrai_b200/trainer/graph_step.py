"""One training micro-step (strategy forward + loss + backward) replayed from a CUDA graph.

The reference runs every micro-batch eagerly (astrai/trainer/trainer.py:74-96): a 1.1B dense
micro-step is about 640 kernel launches, and Python dispatch plus autograd bookkeeping cost a few
microseconds per launch, which leaves the GPU idle between short kernels (RMSNorm, RoPE, SwiGLU)
for roughly 4 % of the step. Here the micro-step is captured once and replayed: the host does one
input copy and one graph launch per micro-batch.

What the capture relies on (checked before every replay, re-captured if violated):

* the batch has the shapes it had at capture; its tensors are copied into static device buffers
  (from pinned host memory when the DataLoader pins, so the copy is asynchronous);
* every parameter gradient exists and stays at the same address: the optimizer's ``zero_grad``
  must zero in place (``set_to_none=False``), and the captured backward accumulates into the
  gradients as eager autograd does when they exist;
* nothing in the forward or backward synchronises with the host (the dense, SFT and MoE paths do
  not: the MoE expert layout is computed on the device and the rank exchanges wait on device
  counters); a module whose ``cuda_graph_safe`` is False keeps the micro-step eager.

The first ``eager_calls`` micro-steps run eagerly, so that everything built lazily on first use
(optimizer state, gradient buckets, packed weights, GEMM fix-up buffers, RoPE tables) exists
before the capture. The capture happens on a dedicated stream, after one eager micro-step on that
stream (the real work of that call), in thread-local capture mode so that the DataLoader's pinning
thread may keep allocating.

Kernel launches inside a replay are not seen by the extension's host launch counter; every replay
adds the number counted during capture (``add_launches``), so ``launch_count()`` stays the number
of kernels this library ran.
"""

from __future__ import annotations

import logging
from typing import Callable, Dict, List, Optional

import torch
import torch.nn as nn

logger = logging.getLogger(__name__)


class GraphedMicroStep:
    """``step(batch) -> loss``: runs ``loss_fn(batch)`` and ``(loss * scale).backward()``."""

    def __init__(self, loss_fn: Callable[[Dict[str, torch.Tensor]], torch.Tensor], model: nn.Module,
                 device: torch.device, scale: float = 1.0, eager_calls: int = 2):
        self.loss_fn = loss_fn
        self.model = model
        self.device = torch.device(device)
        self.scale = float(scale)
        self.eager_calls = eager_calls
        self.calls = 0
        self.replays = 0
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.disabled_reason: Optional[str] = None
        self._stream: Optional[torch.cuda.Stream] = None
        self._static: Dict[str, torch.Tensor] = {}
        self._loss: Optional[torch.Tensor] = None
        self._grad_ptrs: List[int] = []
        self._launches = 0
        unsafe = [type(m).__name__ for m in model.modules() if getattr(m, "cuda_graph_safe", True) is False]
        if unsafe:
            self.disabled_reason = f"{unsafe[0]} synchronises with the host"
        elif self.device.type != "cuda":
            self.disabled_reason = "not a CUDA device"

    # ------------------------------------------------------------------ helpers
    def _params(self) -> List[torch.nn.Parameter]:
        return [p for p in self.model.parameters() if p.requires_grad]

    def _grads_ready(self) -> bool:
        return all(p.grad is not None for p in self._params())

    def _current_grad_ptrs(self) -> List[int]:
        return [p.grad.data_ptr() if p.grad is not None else 0 for p in self._params()]

    def _shapes_match(self, batch: Dict[str, torch.Tensor]) -> bool:
        if set(batch) != set(self._static):
            return False
        for k, v in batch.items():
            s = self._static[k]
            if not isinstance(v, torch.Tensor) or v.shape != s.shape or v.dtype != s.dtype:
                return False
        return True

    def _copy_in(self, batch: Dict[str, torch.Tensor]) -> None:
        for k, v in batch.items():
            self._static[k].copy_(v, non_blocking=True)

    def _eager(self, batch) -> torch.Tensor:
        loss = self.loss_fn(batch)
        (loss * self.scale).backward()
        return loss.detach()

    @staticmethod
    def _graphable(batch) -> bool:
        return isinstance(batch, dict) and all(isinstance(v, torch.Tensor) for v in batch.values())

    # ------------------------------------------------------------------ capture
    def _capture(self, batch: Dict[str, torch.Tensor]) -> torch.Tensor:
        from astrai_b200.ops._ext import native

        self._static = {k: torch.empty(v.shape, dtype=v.dtype, device=self.device) for k, v in batch.items()}
        self._copy_in(batch)
        if self._stream is None:
            self._stream = torch.cuda.Stream(device=self.device)
        cur = torch.cuda.current_stream(self.device)
        self._stream.wait_stream(cur)
        with torch.cuda.stream(self._stream):
            # this call's real micro-step, on the capture stream (lazy per-stream state is made here)
            loss = self._eager(self._static)
        self._stream.synchronize()
        g = torch.cuda.CUDAGraph()
        n0 = native().launch_count()
        # the backward runs on the stream its forward ran on: the capture stream
        with torch.cuda.graph(g, stream=self._stream, capture_error_mode="thread_local"):
            out = self.loss_fn(self._static)
            (out * self.scale).backward()
            self._loss = out.detach()
        self._launches = native().launch_count() - n0
        cur.wait_stream(self._stream)
        self.graph = g
        self._grad_ptrs = self._current_grad_ptrs()
        logger.info("captured the training micro-step: %d kernels of this library per replay", self._launches)
        return loss

    # ------------------------------------------------------------------ call
    def __call__(self, batch) -> torch.Tensor:
        self.calls += 1
        if self.disabled_reason is not None or self.calls <= self.eager_calls or not self._graphable(batch):
            return self._eager(batch)
        if not self._grads_ready():
            # gradients freed (zero_grad with set_to_none) or not made yet: nothing to accumulate into
            self.graph = None
            return self._eager(batch)
        if self.graph is not None and (not self._shapes_match(batch) or self._current_grad_ptrs() != self._grad_ptrs):
            self.graph = None  # new shapes or moved gradients: capture again
        if self.graph is None:
            try:
                return self._capture(batch)
            except Exception as e:  # capture not possible for this model: stay eager
                self.disabled_reason = f"{type(e).__name__}: {e}"
                self.graph = None
                logger.warning("CUDA-graph micro-step disabled, running eagerly (%s)", self.disabled_reason)
                torch.cuda.synchronize(self.device)
                return self._eager(batch)
        from astrai_b200.ops._ext import native

        self._copy_in(batch)
        self.graph.replay()
        native().add_launches(self._launches)
        self.replays += 1
        return self._loss
