"""VRAM-pressure policy for the KV-cache data plane.

Same public surface and policy as the reference scheduler
(src/memopt/scheduler.py:63-461):

* ``SchedulerConfig`` validates ``poll_interval_sec`` (> 0),
  ``vram_high_threshold`` in (0, 1], ``vram_low_threshold`` in
  [0, high), ``drop_retain_ratio`` in [0, 1) and carries ``num_sink_tokens``.
* ``MemoryScheduler`` owns ``retain_ratio`` / ``use_int4`` under a lock.
  ``adjust_policy()`` samples utilisation; at or above the high threshold it
  switches to (``drop_retain_ratio``, INT4), at or below the low threshold
  back to (1.0, fp16), and in between it keeps the current state.
* ``start()``/``stop()`` run a daemon polling thread; ``attach_hook`` runs
  ``adjust_policy`` as a forward pre-hook.

Addition: the utilisation sampler can be injected (``sampler=``), which is
how the policy is exercised without a GPU.
"""
from __future__ import annotations

import logging
import threading
from dataclasses import dataclass, field
from typing import Any, Callable, Optional

import torch
import torch.nn as nn

__all__ = ["MemoryScheduler", "SchedulerConfig"]

logger = logging.getLogger(__name__)

_FULL_RETAIN = 1.0


@dataclass
class SchedulerConfig:
    """Configuration of :class:`MemoryScheduler` (reference scheduler.py:63-106)."""

    poll_interval_sec: float = field(default=0.1)
    vram_high_threshold: float = field(default=0.85)
    vram_low_threshold: float = field(default=0.50)
    drop_retain_ratio: float = field(default=0.75)
    num_sink_tokens: int = field(default=4)

    def __post_init__(self) -> None:
        if not 0.0 < self.vram_high_threshold <= 1.0:
            raise ValueError(
                f"vram_high_threshold must be in (0.0, 1.0], got {self.vram_high_threshold}"
            )
        if not 0.0 <= self.vram_low_threshold < self.vram_high_threshold:
            raise ValueError(
                "vram_low_threshold must be in [0.0, vram_high_threshold), "
                f"got low={self.vram_low_threshold}, high={self.vram_high_threshold}"
            )
        if not 0.0 <= self.drop_retain_ratio < 1.0:
            raise ValueError(f"drop_retain_ratio must be in [0.0, 1.0), got {self.drop_retain_ratio}")
        if self.poll_interval_sec <= 0.0:
            raise ValueError(f"poll_interval_sec must be positive, got {self.poll_interval_sec}")


def _torch_vram_utilization() -> Optional[float]:
    """Allocated / total bytes of CUDA device 0, or None when unavailable."""
    try:
        total = torch.cuda.get_device_properties(0).total_memory
        if total == 0:
            return None
        return torch.cuda.memory_allocated() / total
    except Exception:  # noqa: BLE001 - sampling must never raise
        return None


class MemoryScheduler:
    """Thread-safe owner of the ``retain_ratio`` / ``use_int4`` policy."""

    def __init__(
        self,
        config: Optional[SchedulerConfig] = None,
        sampler: Optional[Callable[[], Optional[float]]] = None,
    ) -> None:
        self._config = config or SchedulerConfig()
        self._retain_ratio = _FULL_RETAIN
        self._use_int4 = False
        self._lock = threading.Lock()
        self._stop_event = threading.Event()
        self._thread = self._new_thread()
        self._hook_handle: Optional[Any] = None
        self._sampler = sampler
        # With an injected sampler the policy runs without CUDA.
        self._cuda_available = sampler is not None or torch.cuda.is_available()
        if not self._cuda_available:
            logger.warning(
                "MemoryScheduler: CUDA is not available.  "
                "VRAM polling is disabled; policy variables will remain at defaults."
            )

    @property
    def config(self) -> SchedulerConfig:
        return self._config

    @property
    def retain_ratio(self) -> float:
        with self._lock:
            return self._retain_ratio

    @property
    def use_int4(self) -> bool:
        with self._lock:
            return self._use_int4

    def snapshot(self) -> tuple[float, bool]:
        """Both policy values read under one lock acquisition."""
        with self._lock:
            return self._retain_ratio, self._use_int4

    def _new_thread(self) -> threading.Thread:
        return threading.Thread(target=self._poll_loop, name="memopt-scheduler", daemon=True)

    def start(self) -> None:
        """Start the polling thread (no-op when it already runs)."""
        if self._thread.is_alive():
            return
        if self._stop_event.is_set() or self._thread.ident is not None:
            self._stop_event.clear()
            self._thread = self._new_thread()
        self._thread.start()

    def stop(self) -> None:
        """Signal the polling thread and wait for it (bounded)."""
        self._stop_event.set()
        if self._thread.is_alive():
            self._thread.join(timeout=self._config.poll_interval_sec * 10)
            if self._thread.is_alive():
                logger.warning("MemoryScheduler.stop(): thread did not terminate within timeout.")

    def attach_hook(self, model: nn.Module) -> None:
        if not isinstance(model, nn.Module):
            raise TypeError(f"attach_hook expects a torch.nn.Module, got {type(model).__name__}")
        if self._hook_handle is not None:
            self._hook_handle.remove()

        def _pre_hook(module: nn.Module, args: tuple) -> None:  # noqa: ARG001
            self.adjust_policy()

        self._hook_handle = model.register_forward_pre_hook(_pre_hook)

    def detach_hook(self) -> None:
        if self._hook_handle is not None:
            self._hook_handle.remove()
            self._hook_handle = None

    def _sample(self) -> Optional[float]:
        if self._sampler is not None:
            try:
                return self._sampler()
            except Exception:  # noqa: BLE001
                return None
        return _torch_vram_utilization()

    def adjust_policy(self) -> None:
        """Sample utilisation once and apply the hysteresis rule."""
        if not self._cuda_available:
            return
        util = self._sample()
        if util is None:
            return
        cfg = self._config
        with self._lock:
            before = (self._retain_ratio, self._use_int4)
            if util >= cfg.vram_high_threshold:
                self._retain_ratio, self._use_int4 = cfg.drop_retain_ratio, True
            elif util <= cfg.vram_low_threshold:
                self._retain_ratio, self._use_int4 = _FULL_RETAIN, False
            after = (self._retain_ratio, self._use_int4)
        if after != before:
            logger.info(
                "MemoryScheduler policy change: vram=%.1f%% retain_ratio %.2f->%.2f use_int4 %s->%s",
                util * 100, before[0], after[0], before[1], after[1],
            )

    def _poll_loop(self) -> None:
        while not self._stop_event.is_set():
            try:
                self.adjust_policy()
            except Exception:  # noqa: BLE001 - the poller must survive
                logger.exception("MemoryScheduler: unhandled exception in poll loop; continuing.")
            self._stop_event.wait(timeout=self._config.poll_interval_sec)

    def __repr__(self) -> str:
        util = self._sample() if self._cuda_available else None
        vram = f"{util * 100:.1f}%" if util is not None else "N/A (no CUDA)"
        rr, q = self.snapshot()
        return (
            f"MemoryScheduler(vram={vram}, retain_ratio={rr:.2f}, use_int4={q}, "
            f"thread={'running' if self._thread.is_alive() else 'stopped'}, "
            f"hook={'attached' if self._hook_handle is not None else 'none'}, "
            f"poll_interval={self._config.poll_interval_sec:.3f}s)"
        )
