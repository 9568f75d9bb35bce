"""Per-task timing regions, record-compatible with fluidgpu_torch.worker_trace
(fluidgpu_runtime/fluidgpu_torch/worker_trace.py:14-123): a recorder, when
installed, collects {kind, name, mode, peer, bytes, start_us/elapsed_us}
per compute task and comm op; CUDA regions are timed with events and
resolved lazily, so tracing adds no synchronisation inside the step.
"""
from __future__ import annotations

import contextlib
import json
import time
from pathlib import Path
from typing import Any

import torch

_recorder: "TraceRecorder | None" = None


class TraceRecorder:
    def __init__(self, path: str | Path | None = None, use_cuda_events: bool = True) -> None:
        self.path = Path(path) if path else None
        self.use_cuda_events = use_cuda_events
        self._pending: list[tuple[dict[str, Any], Any, Any]] = []
        self.records: list[dict[str, Any]] = []

    @contextlib.contextmanager
    def region(self, **meta: Any):
        dev = meta.get("device")
        cuda = self.use_cuda_events and dev is not None and torch.device(dev).type == "cuda"
        meta = {k: (str(v) if k == "device" else v) for k, v in meta.items()}
        if cuda:
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            try:
                yield
            finally:
                e.record()
                self._pending.append((meta, s, e))
        else:
            t0 = time.perf_counter()
            try:
                yield
            finally:
                meta["elapsed_us"] = (time.perf_counter() - t0) * 1e6
                self.records.append(meta)

    def flush(self) -> list[dict[str, Any]]:
        if self._pending:
            torch.cuda.synchronize()
            for meta, s, e in self._pending:
                meta["elapsed_us"] = s.elapsed_time(e) * 1e3
                self.records.append(meta)
            self._pending.clear()
        if self.path is not None:
            with self.path.open("a") as f:
                for r in self.records:
                    f.write(json.dumps(r) + "\n")
            out = list(self.records)
            self.records.clear()
            return out
        return list(self.records)


def install_trace_recorder(recorder: TraceRecorder | None) -> None:
    global _recorder
    _recorder = recorder


@contextlib.contextmanager
def trace_region(**meta: Any):
    rec = _recorder
    if rec is None:
        yield
        return
    with rec.region(**meta):
        yield
