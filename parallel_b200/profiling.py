"""Collective profiling, scheduled torch.profiler traces and a ``profile`` timer.

Public surface and the ``[COLLECTIVE]`` / ``[PROFILE]`` line formats match
the reference (parallel/parallel/profiling.py:37-541) so existing log
parsers keep working:

* ``collective_profile(op, value=..., mode=..., detail=..., defer_cuda_end=...)``
  wraps one collective; under ``collective_phase("forward"|...)`` it records
  CPU time, a CUDA-event interval on the current stream, payload bytes, and
  opens a ``record_function`` + NVTX range ``collective.<phase>.<op>.<mode>.<detail>``;
* ``finish_collective_profile_step()`` gathers all ranks' records and returns
  one aggregated line per (phase, op, mode);
* ``profile(name, ...)`` times a block / decorated function.

Additions for the fused kernels: ``flops=`` on a record (achieved TFLOP/s is
appended to the line when present).
"""
from __future__ import annotations

import logging
import math
import os
from collections import defaultdict
from contextlib import ContextDecorator, contextmanager
from dataclasses import dataclass
from pathlib import Path
from time import perf_counter
from typing import Any

from .logging import get_logger

_LOG = get_logger(__name__)
_PHASE = "other"


@dataclass
class CollectiveRecord:
    operation: str
    phase: str
    mode: str
    detail: str
    payload_bytes: int
    cpu_ms: float
    flops: float = 0.0
    ev_start: Any = None
    ev_end: Any = None
    cuda_ms: float | None = None
    link_bytes: int = 0


def _roofline_peaks() -> tuple[float, float]:
    """(bf16 GEMM FLOP/s, NVLink peer bytes/s) used for roofline fractions."""
    tf = float(os.environ.get("PB_ROOFLINE_TFLOPS", "1700"))
    gbps = float(os.environ.get("PB_ROOFLINE_LINK_GBPS", "770"))
    return tf * 1e12, gbps * 1e9


def _nbytes(t: Any) -> int:
    return t.numel() * t.element_size()


def _fmt_bytes(n: int) -> str:
    return f"{n / 1024 ** 3:.2f}GiB" if n >= 1024 ** 3 else f"{n / 1024 ** 2:.1f}MiB"


def _pct(values: list[float], q: float) -> float:
    if not values:
        return 0.0
    s = sorted(values)
    return s[math.ceil((len(s) - 1) * q)]


class CollectiveProfiler:
    """Per-step store of collective records with deferred CUDA resolution."""

    def __init__(self) -> None:
        self.enabled = False
        self.recording = False
        self.device = None
        self.records: list[CollectiveRecord] = []

    def configure(self, *, enabled: bool, device: Any = None) -> None:
        self.enabled, self.device, self.recording = enabled, device, False
        self.records.clear()

    def start_step(self) -> None:
        self.records.clear()
        self.recording = self.enabled

    def add(self, rec: CollectiveRecord) -> None:
        if self.recording:
            self.records.append(rec)

    def _resolve(self) -> None:
        pending = [r for r in self.records if r.ev_end is not None]
        if not pending:
            return
        import torch

        torch.cuda.synchronize(self.device)
        for r in pending:
            r.cuda_ms = r.ev_start.elapsed_time(r.ev_end)

    def finish_step(self) -> list[str]:
        if not self.enabled:
            return []
        self.recording = False
        self._resolve()
        import torch.distributed as dist

        rank = dist.get_rank() if dist.is_initialized() else 0
        mine = [dict(rank=rank, operation=r.operation, phase=r.phase, mode=r.mode, detail=r.detail,
                     payload_bytes=r.payload_bytes, cpu_ms=r.cpu_ms, cuda_ms=r.cuda_ms, flops=r.flops,
                     link_bytes=r.link_bytes)
                for r in self.records]
        if dist.is_initialized():
            everyone: list[Any] = [None] * dist.get_world_size()
            dist.all_gather_object(everyone, mine)
            rows = [r for part in everyone for r in part]
        else:
            rows = mine
        groups: dict[tuple, list[dict]] = defaultdict(list)
        for r in rows:
            groups[(r["phase"], r["operation"], r["mode"])].append(r)
        lines = []
        for (phase, op, mode), recs in sorted(groups.items()):
            per_rank: dict[int, list[dict]] = defaultdict(list)
            for r in recs:
                per_rank[r["rank"]].append(r)
            calls = [len(v) for v in per_rank.values()]
            payload = max(sum(r["payload_bytes"] for r in v) for v in per_rank.values())
            key = "cuda_ms" if any(r["cuda_ms"] is not None for r in recs) else "cpu_ms"
            times = [r[key] or 0.0 for r in recs]
            total = max(sum(r[key] or 0.0 for r in v) for v in per_rank.values())
            slow = max(recs, key=lambda r: r[key] or 0.0)
            call_txt = str(calls[0]) if min(calls) == max(calls) else f"{min(calls)}-{max(calls)}"
            line = (f"[COLLECTIVE] phase={phase} op={op} mode={mode} calls/rank={call_txt} "
                    f"payload/max-rank={_fmt_bytes(payload)} {key[:-3]} total/max-rank={total:.3f}ms "
                    f"p50={_pct(times, 0.50):.3f}ms p95={_pct(times, 0.95):.3f}ms max={slow[key] or 0.0:.3f}ms "
                    f"slowest=rank{slow['rank']}:{slow['detail']} ({_fmt_bytes(slow['payload_bytes'])})")
            fl = sum(r["flops"] for r in recs)
            if fl and total > 0:
                line += f" tflops/rank={fl / len(per_rank) / (total * 1e-3) / 1e12:.1f}"
                peak_flops, link_bw = _roofline_peaks()
                lb = sum(r.get("link_bytes", 0) for r in recs)
                roof_ms = max(fl / peak_flops, lb / link_bw) / len(per_rank) * 1e3
                line += f" roofline={roof_ms:.3f}ms frac={roof_ms / total:.2f}"
            lines.append(line)
        self.records.clear()
        return lines


_COLLECTIVE_PROFILER = CollectiveProfiler()


class _CollectiveScope:
    def __init__(self, operation, *, mode, detail, payload_bytes, device, defer_cuda_end, flops=0.0):
        self.operation, self.mode, self.detail = operation, mode, detail
        self.payload_bytes, self.device, self.defer_cuda_end = payload_bytes, device, defer_cuda_end
        self.flops = flops
        self.phase = "other"
        self._t0 = None
        self._ev0 = self._ev1 = None
        self._rf = None
        self._nvtx = False
        self._rec = None

    def __enter__(self):
        if not _COLLECTIVE_PROFILER.recording:
            return self
        import torch

        self.phase = _PHASE
        label = ".".join(p for p in ("collective", self.phase, self.operation, self.mode, self.detail) if p)
        self._rf = torch.profiler.record_function(label)
        self._rf.__enter__()
        dev = torch.device(self.device) if self.device is not None else None
        if dev is not None and dev.type == "cuda" and torch.cuda.is_available():
            torch.cuda.nvtx.range_push(label)
            self._nvtx = True
            self._ev0 = torch.cuda.Event(enable_timing=True)
            self._ev1 = torch.cuda.Event(enable_timing=True)
            self._ev0.record(torch.cuda.current_stream(dev))
        self._t0 = perf_counter()
        return self

    def __exit__(self, *exc):
        if self._t0 is None:
            return False
        import torch

        if self._ev1 is not None and not self.defer_cuda_end:
            self._ev1.record(torch.cuda.current_stream(self.device))
        cpu_ms = (perf_counter() - self._t0) * 1e3
        if self._nvtx:
            torch.cuda.nvtx.range_pop()
        if self._rf is not None:
            self._rf.__exit__(*exc)
        self._rec = CollectiveRecord(self.operation, self.phase, self.mode, self.detail, self.payload_bytes,
                                     cpu_ms, self.flops, self._ev0, self._ev1,
                                     link_bytes=getattr(self, "link_bytes", 0))
        if not self.defer_cuda_end:
            _COLLECTIVE_PROFILER.add(self._rec)
        return False

    def complete(self) -> None:
        """Close the CUDA interval of a collective that was launched async."""
        if not self.defer_cuda_end:
            raise RuntimeError("Only deferred collective profiles can be completed")
        if self._t0 is None:
            return
        if self._rec is None:
            raise RuntimeError("Deferred collective profile has not been entered")
        if self._ev1 is not None:
            import torch

            self._ev1.record(torch.cuda.current_stream(self.device))
        _COLLECTIVE_PROFILER.add(self._rec)
        self.defer_cuda_end = False


def configure_collective_profiling(*, enabled: bool, device: Any = None) -> None:
    _COLLECTIVE_PROFILER.configure(enabled=enabled, device=device)


def start_collective_profile_step() -> None:
    _COLLECTIVE_PROFILER.start_step()


def finish_collective_profile_step() -> list[str]:
    return _COLLECTIVE_PROFILER.finish_step()


@contextmanager
def collective_phase(phase: str):
    global _PHASE
    prev, _PHASE = _PHASE, phase
    try:
        yield
    finally:
        _PHASE = prev


def collective_profile(operation: str, *, value: Any = None, payload_bytes: int | None = None, mode: str = "",
                       detail: str = "", device: Any = None, defer_cuda_end: bool = False,
                       flops: float = 0.0, link_bytes: int = 0) -> _CollectiveScope:
    """``flops`` / ``link_bytes`` (fused GEMM + collective ops): the step line then
    adds the achieved TF/s and the fraction of the op's roofline, the slower of
    the FLOPs at the bf16 GEMM peak and the bytes this rank receives over NVLink
    at the peer-copy bandwidth (``PB_ROOFLINE_TFLOPS`` / ``PB_ROOFLINE_LINK_GBPS``,
    defaults: the measured 1700 TF/s and 770 GB/s of this B200 pool)."""
    if payload_bytes is None:
        payload_bytes = _nbytes(value) if value is not None else 0
    if device is None and value is not None:
        device = value.device
    scope = _CollectiveScope(operation, mode=mode, detail=detail, payload_bytes=payload_bytes, device=device,
                             defer_cuda_end=defer_cuda_end, flops=flops)
    scope.link_bytes = link_bytes
    return scope


def scheduled_torch_profiler(*, enabled: bool, trace_dir: str | Path, rank: int, warmup_steps: int = 1,
                             active_steps: int = 1):
    """Scheduled CPU(+CUDA) profiler writing one gzip TensorBoard trace per rank."""
    if not enabled:
        return None
    if warmup_steps < 0:
        raise ValueError("torch profiler warmup steps cannot be negative")
    if active_steps < 1:
        raise ValueError("torch profiler active steps must be positive")
    import torch

    trace_dir = Path(trace_dir)
    trace_dir.mkdir(parents=True, exist_ok=True)
    acts = [torch.profiler.ProfilerActivity.CPU]
    if torch.cuda.is_available():
        acts.append(torch.profiler.ProfilerActivity.CUDA)
    return torch.profiler.profile(
        activities=acts,
        schedule=torch.profiler.schedule(wait=0, warmup=warmup_steps, active=active_steps, repeat=1),
        on_trace_ready=torch.profiler.tensorboard_trace_handler(str(trace_dir), worker_name=f"rank{rank}",
                                                                use_gzip=True),
        record_shapes=False, profile_memory=False, with_stack=False, with_flops=False, with_modules=False,
    )


class _Timer(ContextDecorator):
    def __init__(self, name, *, logger, level, enabled, synchronize, device, use_torch_profiler,
                 use_cuda_events):
        if not name:
            raise ValueError("profile name cannot be empty")
        self.name, self.logger, self.level, self.enabled = name, logger, level, enabled
        self.synchronize, self.device = synchronize, device
        self.use_torch_profiler, self.use_cuda_events = use_torch_profiler, use_cuda_events
        self._t0 = None
        self._ev0 = self._ev1 = None
        self._prof = None
        self._rf = None
        self._sort = "self_cpu_time_total"

    def _recreate_cm(self):
        return type(self)(self.name, logger=self.logger, level=self.level, enabled=self.enabled,
                          synchronize=self.synchronize, device=self.device,
                          use_torch_profiler=self.use_torch_profiler, use_cuda_events=self.use_cuda_events)

    def _cuda_dev(self, torch):
        dev = torch.device(self.device) if self.device is not None else None
        return None if (dev is not None and dev.type != "cuda") else dev

    def _sync(self):
        if not self.synchronize:
            return
        import torch

        dev = self._cuda_dev(torch)
        if self.device is not None and dev is None:
            return
        if torch.cuda.is_available():
            torch.cuda.synchronize(dev)

    def __enter__(self):
        if not self.enabled:
            return self
        self._sync()
        if self.use_torch_profiler or self.use_cuda_events:
            import torch

            if self.use_cuda_events:
                if self.device is not None and self._cuda_dev(torch) is None:
                    raise ValueError("use_cuda_events requires a CUDA device")
                if not torch.cuda.is_available():
                    raise RuntimeError("use_cuda_events requires CUDA to be available")
            if self.use_torch_profiler:
                acts = [torch.profiler.ProfilerActivity.CPU]
                dev = self._cuda_dev(torch)
                if torch.cuda.is_available() and (self.device is None or dev is not None):
                    acts.append(torch.profiler.ProfilerActivity.CUDA)
                    self._sort = "self_cuda_time_total"
                self._prof = torch.profiler.profile(activities=acts)
                self._prof.__enter__()
                self._rf = torch.profiler.record_function(self.name)
                self._rf.__enter__()
            if self.use_cuda_events:
                stream = torch.cuda.current_stream(self._cuda_dev(torch))
                self._ev0 = torch.cuda.Event(enable_timing=True)
                self._ev1 = torch.cuda.Event(enable_timing=True)
                self._ev0.record(stream)
        self._t0 = perf_counter()
        return self

    def __exit__(self, *exc):
        if not self.enabled:
            return False
        if self._ev1 is not None:
            import torch

            self._ev1.record(torch.cuda.current_stream(self._cuda_dev(torch)))
        self._sync()
        if self._t0 is None:
            raise RuntimeError("profile context exited before it was entered")
        ms = (perf_counter() - self._t0) * 1e3
        table = None
        if self._rf is not None:
            self._rf.__exit__(*exc)
        if self._prof is not None:
            self._prof.__exit__(*exc)
            table = self._prof.key_averages().table(sort_by=self._sort, row_limit=10)
        cuda_ms = None
        if self._ev0 is not None and self._ev1 is not None:
            self._ev1.synchronize()
            cuda_ms = self._ev0.elapsed_time(self._ev1)
        self.logger.log(self.level, "[PROFILE] %s: %.3f ms", self.name, ms)
        if table is not None:
            self.logger.log(self.level, "[PROFILE] %s torch profiler:\n%s", self.name, table)
        if cuda_ms is not None:
            self.logger.log(self.level, "[PROFILE] %s CUDA event: %.3f ms", self.name, cuda_ms)
        return False


def profile(name: str, *, logger: logging.Logger | logging.LoggerAdapter | None = None, level: int = logging.INFO,
            enabled: bool = True, synchronize: bool = False, device: Any = None, use_torch_profiler: bool = False,
            use_cuda_events: bool = False) -> _Timer:
    """Time a block or decorated function and log its duration (``enabled=False``
    makes it a no-op; ``synchronize=True`` brackets it with device syncs;
    ``use_cuda_events`` adds a CUDA-event interval; ``use_torch_profiler``
    logs a ten-row operator table)."""
    return _Timer(name, logger=logger if logger is not None else _LOG, level=level, enabled=enabled,
                  synchronize=synchronize, device=device, use_torch_profiler=use_torch_profiler,
                  use_cuda_events=use_cuda_events)
