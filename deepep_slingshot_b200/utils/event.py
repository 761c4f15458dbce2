"""`EventOverlap`: the handle an asynchronous call returns, for compute / communication overlap.

Interface parity with the reference's `EventOverlap` ([DE]deep_ep/utils/event.py:1-81), which
callers depend on: `current_stream_wait(release_handle)`, use as a context manager (directly, or
called with `release_handle`), and `extra_tensors` that a caller keeps alive until it has waited,
in place of `record_stream` under CUDA graphs.

Here the native event (`_C.EventHandle`, recorded on the comm stream) does the stream ordering; this
class only decides when the caller's current stream joins it. Leaving a `with` block joins the
event; `with ev(release_handle=True):` also drops the event afterwards, so the native event and
whatever it pins can be freed before the Python object goes away.
"""
from typing import Any, Optional, Tuple

import torch


class _JoinOnExit:
    """Context object of one `with`: on exit the owner's event (if any) joins the current stream."""

    __slots__ = ('owner', 'release')

    def __init__(self, owner: 'EventOverlap', release: bool) -> None:
        self.owner, self.release = owner, release

    def __enter__(self) -> 'EventOverlap':
        return self.owner

    def __exit__(self, *exc_info: Any) -> None:
        if self.owner.event is not None:
            self.owner.current_stream_wait(release_handle=self.release)


class EventOverlap:
    """A CUDA event of an asynchronous call plus tensors that must outlive it."""

    def __init__(self, event=None, extra_tensors: Optional[Tuple[torch.Tensor, ...]] = None) -> None:
        self.event = event
        self.extra_tensors = extra_tensors

    def current_stream_wait(self, release_handle: bool = False) -> None:
        """Make the current CUDA stream wait for the event; with `release_handle`, drop the event."""
        if self.event is None:
            raise RuntimeError('this EventOverlap holds no event (the call was synchronous or it was released)')
        self.event.current_stream_wait()
        if release_handle:
            self.event = None

    def __call__(self, release_handle: bool = False) -> _JoinOnExit:
        return _JoinOnExit(self, release_handle)

    def __enter__(self) -> 'EventOverlap':
        return self

    def __exit__(self, *exc_info: Any) -> None:
        if self.event is not None:
            self.current_stream_wait()
