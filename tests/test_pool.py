"""EvaluationPool on CPU: spawned workers with fake evaluators (no GPU).
Failures are made on the host (a worker that exits, one that is killed, one
that raises)."""

from __future__ import annotations

import os
import signal
import threading
import time

import pytest

from kernel_mcts_b200.domain import KernelProgram, ProposalStatus
from kernel_mcts_b200.pool import EvaluationPool, WorkerSpec
from kernel_mcts_b200.workloads import gemm_workload

WORKLOAD = gemm_workload("pool_test", 64, 64, 64)


def spec(tmp_path, delay=0.0):
    return WorkerSpec("pool_fakes:make", {"marker_dir": str(tmp_path), "delay": delay})


def test_jobs_spread_over_workers_and_come_back_in_order(tmp_path):
    with EvaluationPool([0, 1], spec(tmp_path, delay=0.05)) as pool:
        programs = [KernelProgram(f"candidate-{i}") for i in range(12)]
        results = pool.evaluate_many(programs, WORKLOAD)
    assert [r.program.source for r in results] == [p.source for p in programs]
    assert all(r.status == ProposalStatus.VALID for r in results)
    assert {r.metadata["visible_devices"] for r in results} == {"0", "1"}  # each worker pinned to its GPU
    assert len({r.metadata["pid"] for r in results}) == 2


def test_a_worker_that_exits_mid_job_is_restarted_and_its_job_requeued(tmp_path):
    with EvaluationPool([0, 1], spec(tmp_path)) as pool:
        results = pool.evaluate_many([KernelProgram("ok-1"), KernelProgram("CRASH_ONCE:a"), KernelProgram("ok-2")],
                                     WORKLOAD)
        assert pool.restarts == 1
    assert [r.status for r in results] == [ProposalStatus.VALID] * 3


def test_a_job_that_kills_every_worker_is_reported_not_retried_forever(tmp_path):
    with EvaluationPool([0], spec(tmp_path), max_attempts=2) as pool:
        results = pool.evaluate_many([KernelProgram("CRASH_ALWAYS"), KernelProgram("ok")], WORKLOAD)
        assert pool.restarts == 2
    assert results[0].status == ProposalStatus.INFRASTRUCTURE_FAILURE
    assert "died 2 time(s)" in results[0].metadata["reason"]
    assert results[1].status == ProposalStatus.VALID


def test_an_exception_in_the_evaluator_is_an_infrastructure_failure(tmp_path):
    with EvaluationPool([0], spec(tmp_path)) as pool:
        (result,) = pool.evaluate_many([KernelProgram("RAISE")], WORKLOAD)
        assert pool.restarts == 0
    assert result.status == ProposalStatus.INFRASTRUCTURE_FAILURE
    assert "backend exploded" in result.metadata["reason"]


def test_a_worker_killed_from_outside_is_replaced(tmp_path):
    with EvaluationPool([0, 1], spec(tmp_path)) as pool:
        victim = pool.worker_pids()[0]
        killer = threading.Timer(1.0, lambda: os.kill(victim, signal.SIGKILL))
        killer.start()
        results = pool.evaluate_many([KernelProgram(f"sleep=0.4;#{i}") for i in range(8)], WORKLOAD)
        killer.join()
        assert pool.restarts >= 1
    assert all(r.status == ProposalStatus.VALID for r in results)


def test_stuck_worker_times_out(tmp_path):
    with EvaluationPool([0], spec(tmp_path), job_timeout_seconds=1.0, max_attempts=1) as pool:
        (result,) = pool.evaluate_many([KernelProgram("sleep=30;")], WORKLOAD)
    assert result.status == ProposalStatus.INFRASTRUCTURE_FAILURE


def test_single_evaluate_keeps_the_evaluator_call_shape(tmp_path):
    with EvaluationPool([3], spec(tmp_path)) as pool:
        result = pool.evaluate(KernelProgram("x"), WORKLOAD)
    assert result.status == ProposalStatus.VALID and result.metadata["visible_devices"] == "3"


def test_prepare_reaches_every_worker(tmp_path):
    with EvaluationPool([0, 1, 2], spec(tmp_path)) as pool:
        pool.prepare(WORKLOAD)  # fake evaluators have no prepare hook: a no-op ack per worker
        assert pool.evaluate(KernelProgram("x"), WORKLOAD).status == ProposalStatus.VALID


def test_host_compile_pool_builds_ahead_of_the_gpu_workers(tmp_path):
    """Candidate sources are built on host threads while the (fake) GPU
    worker evaluates: no candidate reaches a worker before its build is done,
    and builds overlap evaluations (serialised, build + evaluation would take
    4 x (0.3 + 0.2) s)."""
    from test_backend import FakeRunner

    from kernel_mcts_b200.pool import HostCompilePool

    class SlowNvcc(FakeRunner):
        def __init__(self):
            super().__init__()
            self.finished: dict[str, float] = {}

        def __call__(self, command, *, timeout, env):
            out = super().__call__(command, timeout=timeout, env=env)
            if command[0].endswith("nvcc") and "-c" in command:
                source = next((c for c in command if c.endswith(".cu") and "candidate." in c), None)
                if source is not None:
                    time.sleep(0.3)
                    text = open(source).read()
                    self.finished[text.split("sleep=")[1].split(";")[0] + text.split("#")[-1].strip()] = time.time()
            return out

    runner = SlowNvcc()
    programs = [KernelProgram(f"// sleep=0.2;\nextern \"C\" __global__ void bf16_gemm_root() {{}}\n#{i}",
                              "cuda_cpp") for i in range(4)]
    with EvaluationPool([0], spec(tmp_path)) as pool, HostCompilePool(tmp_path, jobs=4, runner=runner) as builds:
        start = time.time()
        results = pool.evaluate_many(programs, WORKLOAD, compile_ahead=builds)
        wall = time.time() - start
    assert [r.status for r in results] == [ProposalStatus.VALID] * 4
    assert len(runner.finished) == 4
    for i, r in enumerate(results):
        assert r.metadata["started"] >= runner.finished[f"0.2{i}"] - 0.05  # built before it ran
    assert wall < 1.7, wall
