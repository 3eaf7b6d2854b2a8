"""Engine context, step context and tensor views over CUDA.

Mirrors the reference's encode-only engine surface
(vllm_apple/engine/context.py, step.py:58-618, tensor.py:106-219) with CUDA
semantics:

* ``EngineContext`` owns a device and a CUDA stream; buffers are torch
  tensors on that device (``create_buffer``).
* ``EngineStepContext`` keeps the ENCODE -> SUBMIT -> READBACK phases.  Ops
  "encode" by enqueuing kernels on the context's stream; ``submit`` records an
  event and ``wait_until_completed`` waits on it (the step's single host sync,
  like ``waitUntilCompleted``).  ``memory_barrier`` is a no-op: kernels on one
  stream are ordered.  Device-side data errors raised by the kernels surface
  at ``wait_until_completed`` as a ``RuntimeError``, like a failed command
  buffer.
* ``EngineTensor`` is a (buffer, byte offset, shape, dtype) view, so ops can
  address e.g. the K part of a planar QKV buffer without a copy.
"""
from __future__ import annotations

import enum
import threading
from typing import Any, Optional

import torch

from .. import _lib
from .. import ops as _ops


class EnginePhase(enum.Enum):
    IDLE = "idle"
    ENCODE = "encode"
    SUBMIT = "submit"
    READBACK = "readback"


class EngineContext:
    """Per-device engine state (the counterpart of MetalEngineContext)."""

    _instances: dict[int, "EngineContext"] = {}
    _lock = threading.Lock()

    def __init__(self, device: int | str | torch.device | None = None,
                 stream: Optional[torch.cuda.Stream] = None):
        if not torch.cuda.is_available():
            raise RuntimeError("EngineContext needs a CUDA device (sm_100a); there is no fallback")
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else \
            torch.device(device if not isinstance(device, int) else f"cuda:{device}")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.stream = stream if stream is not None else torch.cuda.current_stream(dev)
        _lib.load()  # fail loudly now if the library is missing

    @classmethod
    def get_instance(cls, device: int | None = None) -> "EngineContext":
        idx = torch.cuda.current_device() if device is None else device
        with cls._lock:
            if idx not in cls._instances:
                cls._instances[idx] = cls(idx)
            return cls._instances[idx]

    def create_buffer(self, size: int) -> torch.Tensor:
        """An uninitialised device buffer of ``size`` bytes."""
        return torch.empty(size, dtype=torch.uint8, device=self.device)

    def create_buffer_from_bytes(self, data: bytes) -> torch.Tensor:
        host = torch.frombuffer(bytearray(data), dtype=torch.uint8)
        return host.to(self.device)

    def new_step(self, step_id: int = 0, step_kind: str = "decode", num_tokens: int = 0,
                 num_seqs: int = 0) -> "EngineStepContext":
        return EngineStepContext(self, step_id, step_kind, num_tokens, num_seqs)


class EngineTensor:
    """A typed view into an engine buffer at a byte offset."""

    def __init__(self, buffer: torch.Tensor, shape, dtype: torch.dtype = torch.float16,
                 offset: int = 0, strides=None):
        self._buffer = buffer
        self._shape = tuple(int(s) for s in shape)
        self._dtype = dtype
        self._offset = int(offset)
        if strides is None:
            st, acc = [], 1
            for s in reversed(self._shape):
                st.append(acc)
                acc *= s
            strides = tuple(reversed(st))
        self._strides = tuple(strides)
        if self._offset < 0:
            raise ValueError("negative offset")
        end = self._offset + self.nbytes
        if end > buffer_nbytes(buffer):
            raise ValueError(f"view [{self._offset}, {end}) exceeds buffer of "
                             f"{buffer_nbytes(buffer)} bytes")

    buffer = property(lambda self: self._buffer)
    shape = property(lambda self: self._shape)
    strides = property(lambda self: self._strides)
    dtype = property(lambda self: self._dtype)
    offset = property(lambda self: self._offset)

    @property
    def numel(self) -> int:
        n = 1
        for s in self._shape:
            n *= s
        return n

    @property
    def itemsize(self) -> int:
        return torch.empty((), dtype=self._dtype).element_size()

    @property
    def nbytes(self) -> int:
        return self.numel * self.itemsize

    def data_ptr(self) -> int:
        return self._buffer.data_ptr() + self._offset

    def as_torch(self) -> torch.Tensor:
        """A torch view of the same memory (no copy)."""
        flat = self._buffer.view(torch.uint8).reshape(-1)
        raw = flat[self._offset:self._offset + self.nbytes]
        return raw.view(self._dtype).view(self._shape)


def buffer_nbytes(buf: Any) -> int:
    if isinstance(buf, EngineTensor):
        return buf.nbytes
    return buf.numel() * buf.element_size()


def resolve(buf: Any, offset: int = 0) -> tuple[int, int]:
    """(device pointer, remaining bytes) of an engine buffer or view plus a byte offset."""
    if isinstance(buf, EngineTensor):
        base, size = buf.buffer.data_ptr() + buf.offset, buf.nbytes
    elif isinstance(buf, torch.Tensor):
        if not buf.is_cuda:
            raise RuntimeError("engine buffers live on the CUDA device (no CPU fallback)")
        base, size = buf.data_ptr(), buf.numel() * buf.element_size()
    else:
        raise TypeError(f"unsupported buffer type {type(buf)!r}")
    if offset < 0 or offset > size:
        raise ValueError(f"offset {offset} outside buffer of {size} bytes")
    return base + offset, size - offset


def buffer_dtype(buf: Any) -> torch.dtype:
    return buf.dtype if isinstance(buf, (EngineTensor, torch.Tensor)) else torch.uint8


class EngineStepContext:
    """One scheduler step: ops enqueue on the context stream; one wait at the end."""

    def __init__(self, engine_context: EngineContext, step_id: int = 0,
                 step_kind: str = "decode", num_tokens: int = 0, num_seqs: int = 0):
        self._context = engine_context
        self.step_id = step_id
        self.step_kind = step_kind
        self.num_tokens = num_tokens
        self.num_seqs = num_seqs
        self._phase = EnginePhase.IDLE
        self._done: Optional[torch.cuda.Event] = None
        self._is_submitted = False
        self._is_completed = False
        self._num_dispatches = 0
        self._num_barriers = 0
        self._scratch: list[torch.Tensor] = []

    # -- phases -------------------------------------------------------------
    def __enter__(self) -> "EngineStepContext":
        self._phase = EnginePhase.ENCODE
        return self

    def __exit__(self, exc_type, exc, tb):
        self._scratch.clear()
        self._phase = EnginePhase.IDLE
        return False

    @property
    def is_encoding(self) -> bool:
        return self._phase == EnginePhase.ENCODE

    @property
    def is_submitted(self) -> bool:
        return self._is_submitted

    @property
    def is_completed(self) -> bool:
        return self._is_completed

    @property
    def context(self) -> EngineContext:
        return self._context

    @property
    def stream(self) -> torch.cuda.Stream:
        return self._context.stream

    @property
    def stream_handle(self) -> int:
        return self._context.stream.cuda_stream

    def require_encoding(self, what: str) -> None:
        if not self.is_encoding:
            raise RuntimeError(f"{what} called outside ENCODE phase")

    def note_dispatch(self, n: int = 1) -> None:
        self._num_dispatches += n

    def memory_barrier(self) -> None:
        """Ordering point between dependent ops; stream order already provides it."""
        if self._phase != EnginePhase.ENCODE:
            raise RuntimeError("memory_barrier only allowed during ENCODE phase")
        self._num_barriers += 1

    def end_encoding(self) -> None:
        if self._phase != EnginePhase.ENCODE:
            raise RuntimeError("end_encoding only allowed during ENCODE phase")

    def submit(self) -> None:
        if self._phase != EnginePhase.ENCODE:
            raise RuntimeError("submit only allowed from ENCODE phase")
        self._phase = EnginePhase.SUBMIT
        self._done = torch.cuda.Event()
        self._done.record(self._context.stream)
        self._is_submitted = True

    def wait_until_completed(self, check_errors: bool = True) -> None:
        if not self._is_submitted:
            raise RuntimeError("Must call submit() before wait_until_completed()")
        if self._is_completed:
            return
        self._phase = EnginePhase.READBACK
        self._done.synchronize()
        self._is_completed = True
        if check_errors:
            bits = int(_ops.err_flag(self._context.device.index).item())
            if bits:
                _ops.err_flag(self._context.device.index).zero_()
                raise RuntimeError("GPU step reported: " + "; ".join(_lib.describe_flags(bits)))

    def readback_complete(self) -> None:
        if self._phase != EnginePhase.READBACK:
            raise RuntimeError("readback_complete only allowed in READBACK phase")

    def allocate_scratch(self, size: int, name: str = "scratch") -> torch.Tensor:
        buf = self._context.create_buffer(size)
        self._scratch.append(buf)
        return buf

    def get_profiling_stats(self) -> dict:
        return {"dispatches": self._num_dispatches, "barriers": self._num_barriers}


class CapturedStep:
    """A step's encoded ops recorded once into a CUDA graph and replayed.

    ``encode(step_ctx)`` must encode the ops of one step against FIXED buffers
    (the graph replays the same pointers); to run the next step, copy its
    inputs into those buffers and call :meth:`replay`.  The first call runs
    ``encode`` eagerly ``warmup`` times (kernel attributes, workspaces and the
    error word are set up outside the capture), then captures it.  This removes
    the per-layer host encode cost the reference pays on every step
    (vllm_apple/engine/runner.py:829-1176 re-encodes each step).
    """

    def __init__(self, context: EngineContext, encode, warmup: int = 1):
        self._context = context
        self._encode = encode
        self._graph: Optional[torch.cuda.CUDAGraph] = None
        self._warmup = warmup

    def _run_eager(self):
        with EngineStepContext(self._context) as sc:
            self._encode(sc)

    def capture(self) -> None:
        stream = torch.cuda.Stream(self._context.device)
        stream.wait_stream(self._context.stream)
        saved = self._context.stream
        try:
            self._context.stream = stream
            with torch.cuda.stream(stream):
                for _ in range(self._warmup):
                    self._run_eager()
                stream.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    self._run_eager()
            self._graph = g
        finally:
            self._context.stream = saved
        self._context.stream.wait_stream(stream)

    def replay(self) -> None:
        if self._graph is None:
            self.capture()
        self._graph.replay()
