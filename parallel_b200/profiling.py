"""Step-level collective accounting, scheduled torch.profiler traces and a
``profile`` timer.

The public functions and the ``[COLLECTIVE]`` / ``[PROFILE]`` log lines are
those of the reference (parallel/parallel/profiling.py:37-541), so its log
parsers keep working; the implementation is this repository's own:

* every ``collective_profile(...)`` scope becomes one row of the current step
  (phase, op, mode, detail, payload, host time, an optional CUDA-event pair),
  and opens a ``record_function`` / NVTX range
  ``collective.<phase>.<op>.<mode>.<detail>`` so traces show it by name;
* ``finish_collective_profile_step()`` resolves the event pairs once (one
  device synchronisation per step), gathers every rank's rows and prints one
  line per (phase, op, mode) with per-rank totals, percentiles and the
  slowest call.  Rows of the fused GEMM + collective kernels may carry FLOPs
  and NVLink bytes, which add achieved TF/s and the fraction of the op's
  roofline to the line;
* ``profile(name)`` is a context manager / decorator that logs wall time,
  optionally a CUDA-event interval and a torch.profiler operator table.
"""
from __future__ import annotations

import logging
import math
import os
from collections import defaultdict
from contextlib import ContextDecorator, contextmanager
from pathlib import Path
from time import perf_counter
from typing import Any

from .logging import get_logger

_LOG = get_logger(__name__)
_CURRENT_PHASE = ["other"]

# row fields, in the order the rows travel between ranks
_FIELDS = ("rank", "phase", "operation", "mode", "detail", "payload_bytes", "cpu_ms", "cuda_ms", "flops",
           "link_bytes")


def _roofline_peaks() -> tuple[float, float]:
    """(bf16 GEMM FLOP/s, NVLink bytes/s) behind the roofline fractions."""
    return (float(os.environ.get("PB_ROOFLINE_TFLOPS", "1700")) * 1e12,
            float(os.environ.get("PB_ROOFLINE_LINK_GBPS", "770")) * 1e9)


def _size_text(n: int) -> str:
    gib = n / float(1 << 30)
    return f"{gib:.2f}GiB" if gib >= 1.0 else f"{n / float(1 << 20):.1f}MiB"


def _quantile(sorted_vals: list[float], q: float) -> float:
    """Upper nearest-rank quantile of an ascending list (0 for none)."""
    return sorted_vals[math.ceil((len(sorted_vals) - 1) * q)] if sorted_vals else 0.0


def _summarize(rows: list[dict]) -> list[str]:
    """One [COLLECTIVE] line per (phase, op, mode) over every rank's rows."""
    by_key: dict[tuple, list[dict]] = defaultdict(list)
    for r in rows:
        by_key[(r["phase"], r["operation"], r["mode"])].append(r)
    out = []
    for (phase, op, mode) in sorted(by_key):
        group = by_key[(phase, op, mode)]
        use_cuda = any(r["cuda_ms"] is not None for r in group)
        clock = "cuda" if use_cuda else "cpu"

        def t(r):
            return (r["cuda_ms"] if use_cuda else r["cpu_ms"]) or 0.0

        ranks: dict[int, list[dict]] = defaultdict(list)
        for r in group:
            ranks[r["rank"]].append(r)
        counts = sorted(len(v) for v in ranks.values())
        calls = str(counts[0]) if counts[0] == counts[-1] else f"{counts[0]}-{counts[-1]}"
        payload = max(sum(r["payload_bytes"] for r in v) for v in ranks.values())
        total = max(sum(t(r) for r in v) for v in ranks.values())
        durations = sorted(t(r) for r in group)
        worst = max(group, key=t)
        line = (f"[COLLECTIVE] phase={phase} op={op} mode={mode} calls/rank={calls} "
                f"payload/max-rank={_size_text(payload)} {clock} total/max-rank={total:.3f}ms "
                f"p50={_quantile(durations, 0.50):.3f}ms p95={_quantile(durations, 0.95):.3f}ms "
                f"max={t(worst):.3f}ms slowest=rank{worst['rank']}:{worst['detail']} "
                f"({_size_text(worst['payload_bytes'])})")
        flops = sum(r["flops"] for r in group)
        if flops and total > 0:
            n_ranks = len(ranks)
            peak, link = _roofline_peaks()
            roof_ms = 1e3 * max(flops / peak, sum(r["link_bytes"] for r in group) / link) / n_ranks
            line += (f" tflops/rank={flops / n_ranks / (total * 1e-3) / 1e12:.1f}"
                     f" roofline={roof_ms:.3f}ms frac={roof_ms / total:.2f}")
        out.append(line)
    return out


class _StepRecorder:
    """Rows of the current step; the CUDA intervals stay as event pairs until
    the step is summarised."""

    def __init__(self) -> None:
        self.enabled = False
        self.recording = False
        self.device = None
        self.records: list[dict] = []

    def configure(self, *, enabled: bool, device: Any = None) -> None:
        self.enabled, self.device = enabled, device
        self.recording = False
        self.records = []

    def start_step(self) -> None:
        self.records = []
        self.recording = self.enabled

    def add(self, row: dict) -> None:
        if self.recording:
            self.records.append(row)

    def finish_step(self) -> list[str]:
        if not self.enabled:
            return []
        self.recording = False
        rows, self.records = self.records, []
        pairs = [(r, r.pop("_pair", None)) for r in rows]
        if any(pair is not None for _, pair in pairs):
            import torch

            torch.cuda.synchronize(self.device)
            for r, pair in pairs:
                if pair is not None:
                    r["cuda_ms"] = pair[0].elapsed_time(pair[1])
        import torch.distributed as dist

        me = dist.get_rank() if dist.is_initialized() else 0
        mine = [tuple(me if f == "rank" else r.get(f) for f in _FIELDS) for r in rows]
        if dist.is_initialized():
            gathered: list[Any] = [None] * dist.get_world_size()
            dist.all_gather_object(gathered, mine)
            mine = [row for part in gathered for row in part]
        return _summarize([dict(zip(_FIELDS, row)) for row in mine])


_COLLECTIVE_PROFILER = _StepRecorder()


class _Span:
    """One collective call: host time, and with a CUDA device an event pair on
    the current stream (the end event of an asynchronous collective is
    recorded later by ``complete()``, on the stream that waits for it)."""

    def __init__(self, row: dict, device: Any, deferred: bool):
        self.row, self.device, self.deferred = row, device, deferred
        self._t0 = None
        self._pair = None
        self._range = None
        self._nvtx = False
        self._closed = False

    def __enter__(self):
        if not _COLLECTIVE_PROFILER.recording:
            return self
        import torch

        self.row["phase"] = _CURRENT_PHASE[-1]
        name = ".".join(x for x in ("collective", self.row["phase"], self.row["operation"], self.row["mode"],
                                     self.row["detail"]) if x)
        self._range = torch.profiler.record_function(name)
        self._range.__enter__()
        dev = torch.device(self.device) if self.device is not None else None
        if dev is not None and dev.type == "cuda" and torch.cuda.is_available():
            torch.cuda.nvtx.range_push(name)
            self._nvtx = True
            self._pair = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            self._pair[0].record(torch.cuda.current_stream(dev))
        self._t0 = perf_counter()
        return self

    def __exit__(self, *exc):
        if self._t0 is None:
            return False
        import torch

        if self._pair is not None and not self.deferred:
            self._pair[1].record(torch.cuda.current_stream(self.device))
        self.row["cpu_ms"] = 1e3 * (perf_counter() - self._t0)
        if self._nvtx:
            torch.cuda.nvtx.range_pop()
        self._range.__exit__(*exc)
        if not self.deferred:
            self._commit()
        return False

    def _commit(self) -> None:
        if self._pair is not None:
            self.row["_pair"] = self._pair
        self._closed = True
        _COLLECTIVE_PROFILER.add(self.row)

    def complete(self) -> None:
        """End a deferred span once the asynchronous collective was waited for."""
        if not self.deferred or self._closed:
            raise RuntimeError(f"collective span {self.row['operation']!r} is not waiting for completion")
        if self._t0 is None:  # opened while not recording: nothing to close
            return
        if self._pair is not None:
            import torch

            self._pair[1].record(torch.cuda.current_stream(self.device))
        self._commit()


def configure_collective_profiling(*, enabled: bool, device: Any = None) -> None:
    _COLLECTIVE_PROFILER.configure(enabled=enabled, device=device)


def start_collective_profile_step() -> None:
    _COLLECTIVE_PROFILER.start_step()


def finish_collective_profile_step() -> list[str]:
    return _COLLECTIVE_PROFILER.finish_step()


@contextmanager
def collective_phase(phase: str):
    """Attribute the collectives issued inside to ``phase`` (nested phases
    restore the outer one)."""
    _CURRENT_PHASE.append(phase)
    try:
        yield
    finally:
        _CURRENT_PHASE.pop()


def collective_profile(operation: str, *, value: Any = None, payload_bytes: int | None = None, mode: str = "",
                       detail: str = "", device: Any = None, defer_cuda_end: bool = False,
                       flops: float = 0.0, link_bytes: int = 0) -> _Span:
    """Scope of one collective.  ``value`` gives the payload size and device
    when they are not passed.  ``flops`` / ``link_bytes`` (fused GEMM +
    collective kernels) add achieved TF/s and the roofline fraction (the slower
    of the FLOPs at the bf16 GEMM peak and the bytes this rank receives over
    NVLink at the peer-copy bandwidth; ``PB_ROOFLINE_TFLOPS`` /
    ``PB_ROOFLINE_LINK_GBPS``, defaults the measured 1700 TF/s and 770 GB/s of
    this B200 pool) to the step line."""
    if payload_bytes is None:
        payload_bytes = value.numel() * value.element_size() if value is not None else 0
    if device is None and value is not None:
        device = value.device
    row = {"phase": "other", "operation": operation, "mode": mode, "detail": detail,
           "payload_bytes": int(payload_bytes), "cpu_ms": 0.0, "cuda_ms": None, "flops": float(flops),
           "link_bytes": int(link_bytes)}
    return _Span(row, device, defer_cuda_end)


def scheduled_torch_profiler(*, enabled: bool, trace_dir: str | Path, rank: int, warmup_steps: int = 1,
                             active_steps: int = 1):
    """torch.profiler with a warm-up / active schedule writing one gzip
    TensorBoard trace per rank into ``trace_dir`` (None when disabled)."""
    if not enabled:
        return None
    if warmup_steps < 0 or active_steps < 1:
        raise ValueError(f"profiler schedule needs warmup_steps >= 0 and active_steps >= 1 "
                         f"(got {warmup_steps}, {active_steps})")
    import torch

    out = Path(trace_dir)
    out.mkdir(parents=True, exist_ok=True)
    activities = [torch.profiler.ProfilerActivity.CPU]
    if torch.cuda.is_available():
        activities.append(torch.profiler.ProfilerActivity.CUDA)
    return torch.profiler.profile(
        activities=activities,
        schedule=torch.profiler.schedule(wait=0, warmup=warmup_steps, active=active_steps, repeat=1),
        on_trace_ready=torch.profiler.tensorboard_trace_handler(str(out), worker_name=f"rank{rank}",
                                                                use_gzip=True))


class _BlockTimer(ContextDecorator):
    """Logs ``[PROFILE] <name>: <ms> ms`` for the block (also when it raises),
    then the optional torch.profiler table and CUDA-event interval."""

    def __init__(self, name: str, logger, level: int, enabled: bool, synchronize: bool, device: Any,
                 use_torch_profiler: bool, use_cuda_events: bool):
        if not name:
            raise ValueError("profile() needs a non-empty name")
        self.name, self.logger, self.level, self.enabled = name, logger, level, enabled
        self.synchronize, self.device = synchronize, device
        self.use_torch_profiler, self.use_cuda_events = use_torch_profiler, use_cuda_events
        self._state = None  # per entry: (t0, profiler, record_function, events, sort key)

    def _recreate_cm(self):
        # a decorated function gets a fresh timer per call
        return _BlockTimer(self.name, self.logger, self.level, self.enabled, self.synchronize, self.device,
                           self.use_torch_profiler, self.use_cuda_events)

    def _cuda_device(self):
        """The CUDA device to time on (None = current); False for a non-CUDA device."""
        if self.device is None:
            return None
        import torch

        d = torch.device(self.device)
        return d if d.type == "cuda" else False

    def _maybe_sync(self) -> None:
        import torch

        dev = self._cuda_device()
        if self.synchronize and dev is not False and torch.cuda.is_available():
            torch.cuda.synchronize(dev)

    def __enter__(self):
        if not self.enabled:
            return self
        import torch

        self._maybe_sync()
        dev = self._cuda_device()
        prof = rf = events = None
        sort = "self_cpu_time_total"
        if self.use_cuda_events and (dev is False or not torch.cuda.is_available()):
            raise ValueError(f"profile({self.name!r}): CUDA-event timing needs an available CUDA device")
        if self.use_torch_profiler:
            kinds = [torch.profiler.ProfilerActivity.CPU]
            if dev is not False and torch.cuda.is_available():
                kinds.append(torch.profiler.ProfilerActivity.CUDA)
                sort = "self_cuda_time_total"
            prof = torch.profiler.profile(activities=kinds)
            prof.__enter__()
            rf = torch.profiler.record_function(self.name)
            rf.__enter__()
        if self.use_cuda_events:
            events = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            events[0].record(torch.cuda.current_stream(dev))
        self._state = (perf_counter(), prof, rf, events, sort)
        return self

    def __exit__(self, *exc):
        if not self.enabled:
            return False
        if self._state is None:
            raise RuntimeError(f"profile({self.name!r}) exited without being entered")
        t0, prof, rf, events, sort = self._state
        self._state = None
        if events is not None:
            import torch

            events[1].record(torch.cuda.current_stream(self._cuda_device()))
        self._maybe_sync()
        ms = 1e3 * (perf_counter() - t0)
        table = None
        if rf is not None:
            rf.__exit__(*exc)
        if prof is not None:
            prof.__exit__(*exc)
            table = prof.key_averages().table(sort_by=sort, row_limit=10)
        self.logger.log(self.level, "[PROFILE] %s: %.3f ms", self.name, ms)
        if table is not None:
            self.logger.log(self.level, "[PROFILE] %s torch profiler:\n%s", self.name, table)
        if events is not None:
            events[1].synchronize()
            self.logger.log(self.level, "[PROFILE] %s CUDA event: %.3f ms", self.name,
                            events[0].elapsed_time(events[1]))
        return False


def profile(name: str, *, logger: logging.Logger | logging.LoggerAdapter | None = None, level: int = logging.INFO,
            enabled: bool = True, synchronize: bool = False, device: Any = None, use_torch_profiler: bool = False,
            use_cuda_events: bool = False) -> _BlockTimer:
    """Time a block or a decorated function and log the duration.
    ``enabled=False``: no-op; ``synchronize``: device syncs around the block;
    ``use_cuda_events``: also an event interval on the current stream;
    ``use_torch_profiler``: also a ten-row operator table."""
    return _BlockTimer(name, logger if logger is not None else _LOG, level, enabled, synchronize, device,
                       use_torch_profiler, use_cuda_events)
