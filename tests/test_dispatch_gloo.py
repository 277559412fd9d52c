"""The multi-GPU bench's request dispatch on two CPU ranks over gloo: each rank takes its share of
every step (bench.py step_requests), answers its requests (state once with a snapshot, a question
continued from it, the pointer head: the oracle on the small model stands in for a GPU engine), and
the answers are gathered. Their union must be exactly the single-rank run's answers for the same
steps, and bench.py's max/sum over ranks must reduce across the group. Requests carry no state from
one to another (`src/engine.rs:529-662`), so replicas need no collective on the data path.
"""
import datetime
import importlib.util
import os
import pickle
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STEPS, PER = 2, 4


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _answer(bench, eng, head, i):
    """Request i of the sweep, cut so the CPU answers it in a moment: the first 12 state tokens and
    the first 8 tokens of its first question (rows 3, 5 and 7), ids folded into the small model's
    8192-row vocabulary."""
    from oracle import oracle
    sids, qs, _ = bench.request(i)
    q = qs[0][0][:8]
    _, snap, _ = eng.forward(sids[:12] % 8192, [], keep=True)
    hidden, _, _ = eng.forward(q % 8192, [3, 5, 7], cache=snap)
    return oracle.head_probs(hidden, head, 1.0)


def _rank_main(rank, world, port, model_dir, out):
    import torch.distributed as dist

    from oracle import oracle
    from strands_decider import model
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        bench = _bench()
        oracle.set_threads(1)
        eng = oracle.Engine(model_dir)
        head = model.read_safetensors(os.path.join(model_dir, "head.safetensors"))
        mine = {}
        for s in range(STEPS):
            for i in bench.step_requests(s, rank, world, PER):
                mine[i] = _answer(bench, eng, head, i)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        mx = bench.max_over_ranks(world, float(rank + 1))
        total = bench.sum_over_ranks(world, float(len(mine)))
        if rank == 0:
            with open(out, "wb") as f:
                pickle.dump((gathered, mx, total), f)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(600)
def test_two_gloo_ranks_answer_the_single_rank_run(small_model, tmp_path):
    import torch.multiprocessing as mp

    from oracle import oracle
    from strands_decider import model
    out = str(tmp_path / "gathered.pkl")
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), small_model, out), nprocs=world, join=True,
                       start_method="spawn")
    with open(out, "rb") as f:
        gathered, mx, total = pickle.load(f)
    # every request of every step answered once, by one rank, PER each
    assert all(len(g) == STEPS * PER for g in gathered)
    union = {}
    for g in gathered:
        assert not set(g) & set(union)
        union.update(g)
    assert mx == world and total == world * STEPS * PER
    # one rank taking each step's world x PER requests answers exactly the same requests the same way
    bench = _bench()
    oracle.set_threads(1)
    eng = oracle.Engine(small_model)
    head = model.read_safetensors(os.path.join(small_model, "head.safetensors"))
    single = [i for s in range(STEPS) for i in bench.step_requests(s, 0, 1, world * PER)]
    assert sorted(single) == sorted(union)
    for i in single:
        assert np.array_equal(_answer(bench, eng, head, i), union[i])
