"""`EventOverlap`: CUDA-event wrapper for compute/communication overlap.

API parity with the reference's `deep_ep/utils/event.py:1-81` (`current_stream_wait`, context manager,
`extra_tensors` that keep tensors alive without `record_stream` under CUDA graphs).
"""
from typing import Any, Optional, Tuple

import torch


class EventOverlap:
    """A CUDA event of an asynchronous call plus the tensors it keeps alive until the caller
    waits on it (`current_stream_wait`), usable as a context manager (the reference's `EventOverlap`)."""

    def __init__(self, event=None, extra_tensors: Optional[Tuple[torch.Tensor, ...]] = None) -> None:
        self.event = event
        self.extra_tensors = extra_tensors
        self._release_handle_by_call = False

    def current_stream_wait(self, release_handle: bool = False) -> None:
        assert self.event is not None
        self.event.current_stream_wait()
        if release_handle:
            self.event = None

    def __call__(self, release_handle: bool = False) -> 'EventOverlap':
        self._release_handle_by_call = release_handle
        return self

    def __enter__(self) -> Any:
        return self

    def __exit__(self, exc_type: Any, exc_val: Any, exc_tb: Any) -> None:
        if self.event is not None:
            self.current_stream_wait(release_handle=self._release_handle_by_call)
        self._release_handle_by_call = False

