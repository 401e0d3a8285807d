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


def test_profile_logs_when_the_block_raises():
    log = mock.Mock()
    with mock.patch.object(P, "perf_counter", side_effect=[2.0, 2.5]):
        with pytest.raises(KeyError):
            with P.profile("failing", logger=log):
                raise KeyError("x")
    log.log.assert_called_once_with(logging.INFO, "[PROFILE] %s: %.3f ms", "failing", 500.0)


def test_profile_cuda_events_interval_is_logged():
    """use_cuda_events records an event pair on the current stream and logs
    their elapsed time (CUDA mocked: the test needs no device)."""
    log = mock.Mock()
    ev0, ev1 = mock.Mock(), mock.Mock()
    ev0.elapsed_time.return_value = 7.5
    stream = object()
    with mock.patch.object(torch.cuda, "is_available", return_value=True), \
            mock.patch.object(torch.cuda, "Event", side_effect=[ev0, ev1]), \
            mock.patch.object(torch.cuda, "current_stream", return_value=stream), \
            mock.patch.object(P, "perf_counter", side_effect=[0.0, 0.01]):
        with P.profile("kernel", logger=log, use_cuda_events=True):
            pass
    ev0.record.assert_called_once_with(stream)
    ev1.record.assert_called_once_with(stream)
    ev1.synchronize.assert_called_once()
    ev0.elapsed_time.assert_called_once_with(ev1)
    assert log.log.call_args_list[-1] == mock.call(logging.INFO, "[PROFILE] %s CUDA event: %.3f ms", "kernel", 7.5)
    with pytest.raises(ValueError):
        with P.profile("cpu", logger=log, device="cpu", use_cuda_events=True):
            pass


def test_profile_torch_profiler_table_on_cpu():
    log = mock.Mock()
    with mock.patch.object(torch.cuda, "is_available", return_value=False):
        with P.profile("matmul", logger=log, use_torch_profiler=True):
            torch.ones(64, 64) @ torch.ones(64, 64)
    msgs = [c.args for c in log.log.call_args_list]
    assert msgs[0][1] == "[PROFILE] %s: %.3f ms"
    assert msgs[1][1] == "[PROFILE] %s torch profiler:\n%s" and "aten::" in msgs[1][3]


def test_scheduled_profiler_warms_up_then_writes_one_trace_per_rank(tmp_path):
    with mock.patch.object(torch.cuda, "is_available", return_value=False):
        prof = P.scheduled_torch_profiler(enabled=True, trace_dir=tmp_path, rank=5, warmup_steps=1, active_steps=1)
    prof.__enter__()
    for _ in range(3):
        torch.ones(32, 32) @ torch.ones(32, 32)
        prof.step()
    prof.__exit__(None, None, None)
    traces = list(tmp_path.glob("rank5*.pt.trace.json.gz"))
    assert len(traces) == 1, list(tmp_path.iterdir())
