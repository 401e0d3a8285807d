"""profile() timer and the collective profiler's aggregation lines."""
import logging
from unittest import mock

import pytest
import torch

from parallel_b200 import profiling as P


def test_profile_logs_duration():
    log = mock.Mock()
    with mock.patch.object(P, "perf_counter", side_effect=[1.0, 1.25]):
        with P.profile("block", logger=log):
            pass
    log.log.assert_called_once_with(logging.INFO, "[PROFILE] %s: %.3f ms", "block", 250.0)


def test_profile_decorator_and_disabled():
    log = mock.Mock()

    @P.profile("fn", logger=log)
    def f(x):
        return x + 1

    assert f(1) == 2 and f(2) == 3
    assert log.log.call_count == 2
    log2 = mock.Mock()
    with P.profile("off", logger=log2, enabled=False):
        pass
    log2.log.assert_not_called()
    with pytest.raises(ValueError):
        P.profile("")


def test_collective_aggregation_line():
    P.configure_collective_profiling(enabled=True, device=None)
    P.start_collective_profile_step()
    times = iter([0.0, 0.002, 0.0, 0.004, 0.0, 0.001])
    with mock.patch.object(P, "perf_counter", side_effect=lambda: next(times)):
        with P.collective_phase("backward"):
            for i in range(2):
                with P.collective_profile("fsdp_reduce_scatter", value=torch.zeros(1024 * 256), mode="overlapped",
                                          detail=f"unit{i}"):
                    pass
        with P.collective_phase("forward"):
            with P.collective_profile("fsdp_all_gather", payload_bytes=2 * 1024 ** 3, mode="prefetch", detail="u"):
                pass
    lines = P.finish_collective_profile_step()
    assert len(lines) == 2
    bw = [l for l in lines if "phase=backward" in l][0]
    assert "op=fsdp_reduce_scatter mode=overlapped calls/rank=2" in bw
    assert "payload/max-rank=2.0MiB" in bw and "cpu total/max-rank=6.000ms" in bw
    assert "slowest=rank0:unit1 (1.0MiB)" in bw
    fw = [l for l in lines if "phase=forward" in l][0]
    assert "payload/max-rank=2.00GiB" in fw
    P.configure_collective_profiling(enabled=False)


def test_fused_op_line_reports_tflops_and_roofline_fraction(monkeypatch):
    monkeypatch.setenv("PB_ROOFLINE_TFLOPS", "1000")
    monkeypatch.setenv("PB_ROOFLINE_LINK_GBPS", "500")
    P.configure_collective_profiling(enabled=True, device=None)
    P.start_collective_profile_step()
    times = iter([0.0, 0.004])
    with mock.patch.object(P, "perf_counter", side_effect=lambda: next(times)):
        with P.collective_phase("forward"):
            # 2 TFLOP and 1 GB over the link in 4 ms: roofline = max(2 ms, 2 ms) = 2 ms
            with P.collective_profile("sp_all_gather_gemm", payload_bytes=1 << 20, mode="fused", flops=2e12,
                                      link_bytes=1_000_000_000):
                pass
    (line,) = P.finish_collective_profile_step()
    assert "op=sp_all_gather_gemm mode=fused" in line
    assert "tflops/rank=500.0" in line and "roofline=2.000ms frac=0.50" in line, line
    P.configure_collective_profiling(enabled=False)


def test_deferred_completion_records_only_after_complete():
    P.configure_collective_profiling(enabled=True)
    P.start_collective_profile_step()
    scope = P.collective_profile("fsdp_reduce_scatter", payload_bytes=4, mode="overlapped", defer_cuda_end=True)
    with scope:
        pass
    assert P._COLLECTIVE_PROFILER.records == []
    scope.complete()
    assert len(P._COLLECTIVE_PROFILER.records) == 1
    with pytest.raises(RuntimeError):
        scope.complete()
    P.configure_collective_profiling(enabled=False)


def test_scheduled_profiler_validation(tmp_path):
    assert P.scheduled_torch_profiler(enabled=False, trace_dir=tmp_path, rank=0) is None
    with pytest.raises(ValueError):
        P.scheduled_torch_profiler(enabled=True, trace_dir=tmp_path, rank=0, warmup_steps=-1)
    with pytest.raises(ValueError):
        P.scheduled_torch_profiler(enabled=True, trace_dir=tmp_path, rank=0, active_steps=0)
    prof = P.scheduled_torch_profiler(enabled=True, trace_dir=tmp_path / "t", rank=3)
    assert prof is not None and (tmp_path / "t").is_dir()
