"""The benchmark's request sharding (bench.py step_requests): every step's requests are shared out
once each over the ranks, `per` each, with balanced token counts (the weak-scaling runs on 2-8 GPUs
time the slowest rank); one rank takes the step's requests in order."""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_request_tokens_match_the_requests(bench):
    for i in (0, 1, 17, 4095):
        sids, qs, _ = bench.request(i)
        assert bench.request_tokens(i) == len(sids) + sum(len(q) for q, _ in qs)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_steps_are_partitions(bench, world):
    per = 8
    for step in range(4):
        parts = [bench.step_requests(step, r, world, per) for r in range(world)]
        flat = sorted(i for p in parts for i in p)
        order = bench.sweep_order()
        assert flat == sorted(order[(step * world * per + j) % bench.N_REQUESTS] for j in range(world * per))
        assert all(len(p) == per for p in parts)


def test_one_rank_takes_the_step_in_order(bench):
    assert bench.step_requests(3, 0, 1, 8) == bench.sweep_order()[24:32]


def test_sweep_order_is_a_representative_permutation(bench):
    """Every request once; the 160 requests of the default timed steps have the sweep's mean state
    length within 1%."""
    order = bench.sweep_order()
    assert sorted(order) == list(range(bench.N_REQUESTS))
    mean_all, _, _ = bench.sweep_stats()
    state = lambda i: len(bench.request(i)[0])  # noqa: E731
    sample = [state(i) for i in order[24:184]]
    assert abs(sum(sample) / len(sample) - mean_all) < 0.01 * mean_all


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ranks_are_balanced(bench, world):
    per = 8
    for step in range(4):
        loads = [sum(bench.request_tokens(i) for i in bench.step_requests(step, r, world, per)) for r in range(world)]
        assert max(loads) - min(loads) <= 0.1 * (sum(loads) / world), loads
