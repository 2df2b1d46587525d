"""One-copy upload of a step's host inputs.

A step's inputs that live on the host (query/key/value rows and the
attention metadata, when the caller builds them there) are packed into one
pinned buffer, 16-byte aligned per tensor, and reach the device with a single
``cudaMemcpyAsync``; the device tensors are views into one device buffer.
The reference moves each metadata tensor with its own ``torch.tensor(...,
device=...)`` (src/micro_vllm/worker/model_runner.py:751-900), one copy per
tensor.

``UploadPipeline`` keeps two such buffers and a copy stream, so that the
upload of the next step's inputs and the read-back of the previous step's
result overlap the current step's kernels.
"""

from __future__ import annotations

import torch

_ALIGN = 16


class PinnedStaging:
    """Fixed layout for a set of named tensors (shapes and dtypes of the
    first ``pack``); ``pack`` copies host tensors into the pinned buffer and
    ``upload`` issues the one copy and returns device views by name."""

    __slots__ = ("device", "_layout", "_host", "_dev", "_uploaded", "_views")

    def __init__(self, device: torch.device | str) -> None:
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("PinnedStaging uploads to a CUDA device")
        self._layout: dict[str, tuple[int, torch.dtype, tuple[int, ...]]] | None = None
        self._host: torch.Tensor | None = None
        self._dev: torch.Tensor | None = None
        self._uploaded: torch.cuda.Event | None = None
        self._views: dict[str, torch.Tensor] | None = None

    @property
    def nbytes(self) -> int:
        return 0 if self._host is None else self._host.numel()

    def pack(self, tensors: dict[str, torch.Tensor]) -> None:
        if self._layout is None:
            layout, off = {}, 0
            for name, t in tensors.items():
                layout[name] = (off, t.dtype, tuple(t.shape))
                off += -(-t.numel() * t.element_size() // _ALIGN) * _ALIGN
            self._layout = layout
            self._host = torch.empty(off, dtype=torch.uint8).pin_memory()
            self._dev = torch.empty(off, dtype=torch.uint8, device=self.device)
        if self._uploaded is not None:
            self._uploaded.synchronize()  # the last upload has left the pinned buffer
        for name, t in tensors.items():
            off, dtype, shape = self._layout[name]
            if t.dtype != dtype or tuple(t.shape) != shape:
                raise ValueError(f"{name}: {t.dtype} {tuple(t.shape)} does not match the staged layout")
            n = t.numel() * t.element_size()
            self._host[off:off + n].view(dtype).view(shape).copy_(t)

    def upload(self) -> dict[str, torch.Tensor]:
        """One host-to-device copy on the current stream; the returned device
        views are the same tensors every call (the layout is fixed), so they
        may be held."""

        assert self._layout is not None and self._host is not None and self._dev is not None
        stream = torch.cuda.current_stream(self.device)
        self._dev.copy_(self._host, non_blocking=True)
        self._uploaded = torch.cuda.Event()
        self._uploaded.record(stream)
        if self._views is None:
            views = {}
            for name, (off, dtype, shape) in self._layout.items():
                n = 1
                for d in shape:
                    n *= d
                nbytes = n * torch.empty((), dtype=dtype).element_size()
                views[name] = self._dev[off:off + nbytes].view(dtype).view(shape)
            self._views = views
        return dict(self._views)


class UploadPipeline:
    """Double-buffered uploads and read-backs on their own streams.

    ``slot(i)`` is step i's ``PinnedStaging`` (two, used in turn: pack each
    once, or again before its step).  ``upload(i)`` copies slot i % 2 to the
    device on the upload stream, once the kernels that last read that slot's
    device buffer (step i - 2) have finished, and makes the current stream
    wait for that copy alone; it returns the device views.  Step i's kernels
    are the work the caller queues on the current stream between
    ``upload(i)`` and ``upload(i + 1)``: ``upload(i + 1)`` marks their end as
    the release of slot i % 2, whether or not the step read anything back.
    ``download(i, result, host)`` reads the step's result back on the
    read-back stream once the current stream has produced it.  ``drain()``
    makes the current stream wait for every copy issued so far.  Step i's
    kernels then overlap step i + 1's upload and step i - 1's read-back.
    """

    __slots__ = ("device", "_slots", "_h2d", "_d2h", "_released")

    def __init__(self, device: torch.device | str) -> None:
        self.device = torch.device(device)
        self._slots = (PinnedStaging(self.device), PinnedStaging(self.device))
        self._h2d = torch.cuda.Stream(self.device)
        self._d2h = torch.cuda.Stream(self.device)
        self._released: list[torch.cuda.Event | None] = [None, None]

    def slot(self, i: int) -> PinnedStaging:
        return self._slots[i % 2]

    def upload(self, i: int) -> dict[str, torch.Tensor]:
        compute = torch.cuda.current_stream(self.device)
        # Everything queued so far (step i - 1's kernels, the last readers of
        # the other slot's device buffer) releases that slot for step i + 1.
        queued = torch.cuda.Event()
        queued.record(compute)
        released = self._released[i % 2]
        self._released[(i + 1) % 2] = queued
        if released is not None:
            self._h2d.wait_event(released)
        else:  # first use: after everything the caller queued so far
            self._h2d.wait_stream(compute)
        with torch.cuda.stream(self._h2d):
            views = self._slots[i % 2].upload()
            copied = torch.cuda.Event()
            copied.record(self._h2d)
        compute.wait_event(copied)
        return views

    def download(self, i: int, result: torch.Tensor, host: torch.Tensor) -> None:
        compute = torch.cuda.current_stream(self.device)
        done = torch.cuda.Event()
        done.record(compute)  # the step's result is complete
        self._d2h.wait_event(done)
        with torch.cuda.stream(self._d2h):
            host.copy_(result, non_blocking=True)
        result.record_stream(self._d2h)

    def drain(self) -> None:
        compute = torch.cuda.current_stream(self.device)
        compute.wait_stream(self._h2d)
        compute.wait_stream(self._d2h)
