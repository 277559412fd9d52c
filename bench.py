#!/usr/bin/env python
"""Benchmark of the sequence-mixing forward: answered questions/s on the throughput sweep.

Workload (the reference's headline metric is answered questions/s and prefill tok/s; the sweep is the
configuration it is quoted on): independent requests of the full random-init 24-layer model, each a
state of 64-4096 random non-special token ids (clipped so state + longest question fits the
4096-token context) and 3 questions (noul: 2 options, choice: 3, score: 3) of 42-84 tokens. A request
runs as the reference's `Decider::run` does (src/lib.rs:185-198): the state once with a snapshot,
then each question continued from the snapshot, hidden rows at the option tokens and the last token,
then the pointer head. A step is a batch of --requests-per-step requests per GPU (weak scaling:
each rank takes its own requests, no collective on the data path): the states of all of them and
their questions in one packed tree pass, each question continuing its own request's state within the
pass (sd_forward_tree: every layer writes the states' recurrent state, conv history and K/V before
the questions read them), then the pointer head of every question on the GPU (f64), as a server
answers concurrent requests. `--two-pass` runs the states as one packed pass kept as snapshots
(sd_forward_batch), then the questions as one batched fork (sd_forward_fork_multi) instead.

`value`: device-resident inputs (token ids and rows staged in HBM before the timed region),
passes queued with sd_forward_tree_dev / sd_head_probs_dev (or the two passes), probabilities left
in HBM; CUDA events on the engine's stream.
`e2e`: the same requests through the C ABI with host buffers (sd_forward_tree_probs, or
sd_forward_batch then sd_forward_fork_multi_probs: ids host->device, each question's probabilities
device->host, synchronous per call).
`roofline`: the dominant kernel (the dequantizing GEMM), from per-launch CUDA events on the engine's
stream over a profiled pass of the same steps.
"""
from __future__ import annotations

import argparse
import functools
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "strands-decider-rs_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

VOCAB = 248320
SPECIAL = (6000, 6001, 6002)  # the synthetic tokenizer's added tokens
N_REQUESTS = 8192
CONTEXT = 4096
QLEN = (42, 84)  # question token counts of the reference's fixtures (tests/golden/prompt_cases.json)
KINDS = (("noul", 2), ("choice", 3), ("score", 3))


def request(i: int, seed: int = 0):
    """Request i of the seeded sweep: (state ids, [(question ids, rows)] x 3, clipped?)."""
    rng = np.random.default_rng([seed, i])
    qlens = rng.integers(QLEN[0], QLEN[1] + 1, 3)
    s = int(rng.integers(64, 4097))
    clipped = s + int(qlens.max()) > CONTEXT
    s = min(s, CONTEXT - int(qlens.max()))

    def ids(n):
        x = rng.integers(0, VOCAB - len(SPECIAL), n)
        return (x + (x >= SPECIAL[0]) * len(SPECIAL)).astype(np.uint32)
    qs = []
    for (_, nopt), ql in zip(KINDS, qlens):
        ql = int(ql)
        rows = sorted(rng.choice(np.arange(ql // 2, ql - 1), nopt, replace=False).tolist()) + [ql - 1]
        qs.append((ids(ql), np.array(rows, np.int32)))
    return ids(s), qs, clipped


def sweep_stats(seed: int = 0, n: int = N_REQUESTS):
    """Mean state length, tokens per question and clip count over the whole sweep (lengths only)."""
    tot_state = tot_tokens = clips = 0
    for i in range(n):
        rng = np.random.default_rng([seed, i])
        qlens = rng.integers(QLEN[0], QLEN[1] + 1, 3)
        s = int(rng.integers(64, 4097))
        clips += s + int(qlens.max()) > CONTEXT
        s = min(s, CONTEXT - int(qlens.max()))
        tot_state += s
        tot_tokens += s + int(qlens.sum())
    return tot_state / n, tot_tokens / (3 * n), clips


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        # nvidia-smi takes a moment to start: wait (at most 10 s) for its first sample, which is taken
        # before the timed region and dropped
        self.skip = 0
        t0 = time.time()
        while self.p is not None and self.p.poll() is None and time.time() - t0 < 10:
            if self._rows():
                self.skip = len(self._rows())
                break
            time.sleep(0.05)

    def _rows(self):
        self.f.flush()
        return [ln.split(",") for ln in open(self.f.name).read().strip().splitlines() if ln.count(",") >= 8]

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        rows = self._rows()
        rows = rows[self.skip:] or rows[-1:]  # the samples of the timed region (the last one if it was shorter)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        mx = max(float(r[2]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[j] for r in rows for j in range(4) if "Active" in r[5 + j] and "Not" not in r[5 + j]})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": reasons, "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows)}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return m["hbm_gbs"], m["bf16_tflops"], m["bf16_tflops_sustained"], "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, 1400.0, "fallback"


class PassRoofline:
    """The aggregate roofline of the sweep: for each packed pass, the slower of its bytes at the
    measured HBM bandwidth and its FLOPs at the measured sustained tensor peak, summed over the
    passes. A pass streams every layer weight once (int4 g32: 0.5625 B per weight), moves each
    GEMM's f16 activations in and out, reads and writes the gated-delta states of its sequences
    (written only when kept) and their K/V rows; FLOPs are the GEMMs (2 N K per token), causal
    attention (4 hd hq per query-key pair, over the prefix too) and the chunked gated-delta rule
    (8 C dk + 6 dk^2 + 2 C^2 / 3 per token and head, C = 64)."""

    def __init__(self, path: str):
        from strands_decider import model
        m = model.read_manifest(path)
        c = m["config"]
        self.n_lin = sum(t == "linear_attention" for t in c["layer_types"])
        self.n_full = sum(t == "full_attention" for t in c["layer_types"])
        mats = [(t["N"], t["K"]) for n, t in m["tensors"].items() if n.endswith(".q") and n != "embed.q"]
        self.weight_bytes = sum(nn * k for nn, k in mats) * 0.5625
        self.flop_tok = 2.0 * sum(nn * k for nn, k in mats)
        self.act_tok = 2.0 * sum(nn + k for nn, k in mats)
        self.h, self.dk, self.dv = c["linear_num_key_heads"], c["linear_key_head_dim"], c["linear_value_head_dim"]
        self.hq, self.hk, self.hd = c["num_attention_heads"], c["num_key_value_heads"], c["head_dim"]
        C = 64
        self.gdn_flop_tok = (8 * C * self.dk + 6 * self.dk * self.dk + 2 * C * C / 3) * self.h * self.n_lin
        self.gdn_bytes_tok = (3 * self.h * self.dk * 2 + 8 * self.h + 4 * self.h * self.dv) * self.n_lin
        self.state_bytes = self.h * self.dk * self.dv * 4 * self.n_lin
        self.kv_tok = 2 * self.hk * self.hd * 2 * self.n_full
        self.bound_s = 0.0

    def add(self, seqs, keep: bool, hbm_gbs: float, tflops: float):
        """One pass over sequences (prefix length, new tokens)."""
        tok = sum(l for _, l in seqs)
        pairs = sum(l * p + l * (l + 1) / 2 for p, l in seqs)
        flops = self.flop_tok * tok + 4.0 * self.hd * self.hq * pairs * self.n_full + self.gdn_flop_tok * tok
        nbytes = (self.weight_bytes + (self.act_tok + self.gdn_bytes_tok + self.kv_tok) * tok
                  + self.state_bytes * len(seqs) * (2 if keep else 1) + self.kv_tok * sum(p for p, _ in seqs))
        self.bound_s += max(nbytes / (hbm_gbs * 1e9), flops / (tflops * 1e12))


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(minutes=10), device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def _reduce(world, x: float, op: str) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    # NCCL reduces device tensors; the CPU (gloo) process groups of the tests reduce host ones
    t = torch.tensor([x], dtype=torch.float64, device="cuda" if dist.get_backend() == "nccl" else "cpu")
    dist.all_reduce(t, op=getattr(dist.ReduceOp, op))
    return float(t.item())


def max_over_ranks(world, x: float) -> float:
    return _reduce(world, x, "MAX")


def sum_over_ranks(world, x: float) -> float:
    return _reduce(world, x, "SUM")


def model_path(world, rank):
    from strands_decider import model
    path = os.path.join(ROOT, "_models", "full_s0")
    if rank == 0:
        model.ensure_model(path, seed=0)
    barrier(world)
    return path


def request_tokens(i: int, seed: int = 0) -> int:
    """Tokens of request i of the sweep (its state and its questions), from the lengths alone."""
    rng = np.random.default_rng([seed, i])
    qlens = rng.integers(QLEN[0], QLEN[1] + 1, 3)
    s = min(int(rng.integers(64, 4097)), CONTEXT - int(qlens.max()))
    return s + int(qlens.sum())


@functools.lru_cache(maxsize=4)
def sweep_order(seed: int = 0):
    """The order in which the bench takes the sweep's requests: sorted by state length, then visited in
    bit-reversed rank order (a van der Corput sequence over the length quantiles), so that any run of
    consecutive requests, the timed steps among them, spreads evenly over the sweep's length
    distribution (160 requests: mean state within 0.5% of the sweep's 2080 tokens)."""
    lens = [request_tokens(i, seed) for i in range(N_REQUESTS)]
    srt = sorted(range(N_REQUESTS), key=lambda i: (lens[i], i))
    bits = (N_REQUESTS - 1).bit_length()
    return [srt[int(format(k, f"0{bits}b")[::-1], 2)] for k in range(N_REQUESTS)]


def step_requests(step: int, rank: int, world: int, per: int, seed: int = 0):
    """This rank's requests of step `step`: the step takes the next world x per requests of the sweep
    (in sweep_order) and shares them out as a server balances concurrent requests over its GPUs,
    longest first to the rank with the fewest tokens so far (each rank gets `per`), so that no rank
    waits on another holding all the long states."""
    base = step * world * per
    order = sweep_order(seed)
    ids = [order[(base + j) % N_REQUESTS] for j in range(world * per)]
    if world == 1:
        return ids
    load = [0] * world
    mine = [[] for _ in range(world)]
    for i in sorted(ids, key=lambda i: -request_tokens(i, seed)):
        r = min((r for r in range(world) if len(mine[r]) < per), key=lambda r: load[r])
        mine[r].append(i)
        load[r] += request_tokens(i, seed)
    return sorted(mine[rank])


def cpu_baseline(path: str, seed: int = 0, state_len: int = 96, questions: int = 3, eng=None):
    """The oracle (the CPU restatement of the reference's shader math) on a bounded sample: request 0's
    first `questions` questions after a state cut to `state_len` tokens, on every host core (torchrun
    sets OMP_NUM_THREADS=1, so the count is set explicitly); throughput scaled to the sweep's mean
    tokens per question (cost is linear in tokens to within the attention share, about 2%)."""
    from oracle import oracle
    oracle.set_threads(os.cpu_count() or 1)
    if eng is None:
        eng = oracle.Engine(path)
    sids, qs, _ = request(0, seed)
    sids, qs = sids[:state_len], qs[:questions]
    t0 = time.perf_counter()
    _, snap, _ = eng.forward(sids, [], keep=True)
    for qids, rows in qs:
        eng.forward(qids, rows, cache=snap)
    dt = time.perf_counter() - t0
    tokens = len(sids) + sum(len(q) for q, _ in qs)
    return dt, tokens


def run_reference(args, world, rank):
    """`--impl reference`: the reference's own CPU path for the sweep. The reference (Rust + WGSL on
    wgpu) has no CPU implementation of its own and cannot run here (no Rust toolchain, no graphics
    stack), so this times the oracle port of its shader math on the host's cores, per step one
    bounded sample request, scaled to the sweep's mean tokens per question."""
    if rank != 0:
        return
    path = model_path(1, 0)
    _, mean_tokens_q, _ = sweep_stats(args.seed)
    cores = os.cpu_count()
    from oracle import oracle
    eng = oracle.Engine(path)
    times = []
    tokens = 0
    for s in range(args.warmup + args.steps):
        dt, tok = cpu_baseline(path, args.seed + s, state_len=32, questions=1, eng=eng)
        if s >= args.warmup:
            times.append(dt)
            tokens += tok
    total = sum(times)
    tok_s = tokens / total
    qps = tok_s / mean_tokens_q
    sample = (f"per step: one sweep request with its state cut to 32 tokens + its first question (oracle port, {cores} threads), "
              f"{tok_s:.1f} tok/s scaled to the sweep's {mean_tokens_q:.0f} tokens per question")
    line = {"impl": "reference", "metric": "answered questions/s", "value": qps, "unit": "questions/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "sweep (bounded CPU sample)", "model": "random-init 2B hybrid, 24 layers"},
            "cpu_baseline": {"value": qps, "unit": "questions/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": qps, "unit": "questions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "prefill_tok_s": tok_s}
    print(json.dumps(line), flush=True)


def run_ours(args, world, rank, local):
    import torch
    from strands_decider.engine import Engine, Head

    path = model_path(world, rank)
    torch.cuda.set_device(local)
    t_load = time.perf_counter()
    eng = Engine.load(path, local)
    t_load = time.perf_counter() - t_load
    head = Head.load(os.path.join(path, "head.safetensors"))
    stream = torch.cuda.ExternalStream(eng.stream)
    per = args.requests_per_step
    steps_all = args.warmup + args.steps
    # stage every request of every step in HBM before timing
    reqs = {}
    staged = {}
    for s in range(steps_all + 1):
        for i in step_requests(s, rank, world, per, args.seed):
            if i in reqs:
                continue
            sids, qs, _ = request(i, args.seed)
            reqs[i] = (sids, qs)
            # the state's ids and the questions' ids (back to back) in HBM; lengths and rows on the host
            staged[i] = (torch.from_numpy(sids.view(np.int32)).cuda(),
                         torch.from_numpy(np.concatenate([q for q, _ in qs]).view(np.int32)).cuda(),
                         [len(q) for q, _ in qs], [list(r) for _, r in qs])
    # the states and the questions of a step's requests back to back in HBM, for the passes across requests
    # (the tree pass: all states, then all questions)
    step_s, step_q, step_t = {}, {}, {}
    for s in range(steps_all + 1):
        ii = step_requests(s, rank, world, per, args.seed)
        step_s[s] = torch.cat([staged[i][0] for i in ii])
        step_q[s] = torch.cat([staged[i][1] for i in ii])
        step_t[s] = torch.cat([step_s[s], step_q[s]])
    hidden_dev = torch.empty((per * 12, 2048), dtype=torch.float32, device="cuda")
    probs_dev = torch.empty(per * 12, dtype=torch.float64, device="cuda")
    # working memory for the largest pass of any step, up front (as a server sizes it at start-up)
    eng.reserve(max(t.numel() for t in step_t.values()), per * 4, per * 12)
    torch.cuda.synchronize()

    # a request as the Decider runs it (`Decider::run`, src/lib.rs:156-208): the state once, kept as
    # a snapshot, then its questions continued from the snapshot. The states of all the step's
    # requests run as one packed pass (sd_forward_batch, a snapshot each), then their questions as
    # one batched fork (each continuing its own request's snapshot)
    hbm_gbs, _, tf_sustained, _ = peaks()
    roof = PassRoofline(path)

    def one_step_dev(s):
        ii = step_requests(s, rank, world, per, args.seed)
        slens = [staged[i][0].numel() for i in ii]
        if not args.two_pass:  # the states and their questions in one tree pass, then the head
            lens, rows, parents = list(slens), [[] for _ in ii], [-1] * len(ii)
            for j, i in enumerate(ii):
                _, _, ql, qr = staged[i]
                lens += ql
                rows += qr
                parents += [j] * len(ql)
            eng.forward_tree_dev(None, parents, step_t[s].data_ptr(), lens, rows, hidden_dev.data_ptr())
            qrows = rows[len(ii):]
            eng.head_probs_dev(head, hidden_dev.data_ptr(), [len(r) for r in qrows], 1.0, probs_dev.data_ptr())
            return len(qrows), sum(lens)
        snaps = eng.forward_batch_dev(None, step_s[s].data_ptr(), slens, [[]] * len(ii), None, keep=True)
        caches, lens, rows = [], [], []
        n_tok = sum(slens)
        for i, snap in zip(ii, snaps):
            _, qd, ql, qr = staged[i]
            caches += [snap] * len(ql)
            lens += ql
            rows += qr
            n_tok += qd.numel()
        eng.forward_fork_dev(caches, step_q[s].data_ptr(), lens, rows, hidden_dev.data_ptr())
        eng.head_probs_dev(head, hidden_dev.data_ptr(), [len(r) for r in rows], 1.0, probs_dev.data_ptr())
        for snap in snaps:
            snap.close()
        return len(lens), n_tok

    h2d = d2h = 0

    def one_step_host(s):
        nonlocal h2d, d2h
        ii = step_requests(s, rank, world, per, args.seed)
        states = [reqs[i][0] for i in ii]
        if not args.two_pass:
            qids, qrows, parents = [], [], [-1] * len(ii)
            for j, i in enumerate(ii):
                qs = reqs[i][1]
                qids += [q for q, _ in qs]
                qrows += [r for _, r in qs]
                parents += [j] * len(qs)
            outs = eng.forward_tree_probs(None, parents, states + qids, [[] for _ in ii] + qrows, head, 1.0)
            h2d += sum(x.nbytes for x in states)
            for q, r, probs in zip(qids, qrows, outs):
                h2d += q.nbytes + r.nbytes
                d2h += probs.nbytes
            return len(outs)
        _, snaps = eng.forward_batch(None, states, [[]] * len(ii), keep=True)
        h2d += sum(x.nbytes for x in states)
        caches, qids, qrows = [], [], []
        for i, snap in zip(ii, snaps):
            qs = reqs[i][1]
            caches += [snap] * len(qs)
            qids += [q for q, _ in qs]
            qrows += [r for _, r in qs]
        outs = eng.forward_fork_probs(caches, qids, qrows, head, 1.0)
        for q, r, probs in zip(qids, qrows, outs):
            h2d += q.nbytes + r.nbytes
            d2h += probs.nbytes
        for snap in snaps:
            snap.close()
        return len(outs)

    def timed(fn, first, count):
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(world)
        torch.cuda.synchronize()
        eng.synchronize()
        ev0.record(stream)
        res = [fn(first + s) for s in range(count)]
        ev1.record(stream)
        eng.synchronize()
        torch.cuda.synchronize()
        barrier(world)
        return ev0.elapsed_time(ev1), res

    # warm-up (both paths)
    for s in range(args.warmup):
        one_step_dev(s)
    eng.synchronize()
    for s in range(min(args.warmup, 1)):
        one_step_host(s)

    clocks = Clocks(local)
    l0 = eng.launches()
    ms_dev, res = timed(one_step_dev, args.warmup, args.steps)
    launches = eng.launches() - l0
    clk = clocks.stop()
    q_dev = sum(r[0] for r in res)
    tok_dev = sum(r[1] for r in res)
    h2d = d2h = 0
    ms_host, res_h = timed(one_step_host, args.warmup, args.steps)
    q_host = sum(res_h)
    h2d_step, d2h_step = h2d / args.steps, d2h / args.steps

    # profiled pass over the same steps (per-launch events), for the roofline
    eng.profile(True)
    for s in range(args.steps):
        one_step_dev(args.warmup + s)
    prof = eng.profile_get()
    eng.profile(False)

    for s in range(args.steps):  # the timed steps' passes, counted outside the timed region
        ii = step_requests(args.warmup + s, rank, world, per, args.seed)
        roots = [(0, staged[i][0].numel()) for i in ii]
        qs_ = [(staged[i][0].numel(), n) for i in ii for n in staged[i][2]]
        if args.two_pass:
            roof.add(roots, True, hbm_gbs, tf_sustained)
            roof.add(qs_, False, hbm_gbs, tf_sustained)
        else:
            roof.add(roots + qs_, True, hbm_gbs, tf_sustained)
    bound_all = sum_over_ranks(world, roof.bound_s)
    t_dev = max_over_ranks(world, ms_dev) / 1e3
    t_host = max_over_ranks(world, ms_host) / 1e3
    q_all = sum_over_ranks(world, q_dev)
    tok_all = sum_over_ranks(world, tok_dev)
    qh_all = sum_over_ranks(world, q_host)
    if rank != 0:
        return
    hbm, tf_burst, tf_sus, src = peaks()
    g = prof["gemm"]
    gemm_tflops = g["work"] / (g["ms"] / 1e3) / 1e12 if g["ms"] > 0 else 0.0
    a = prof["attention"]
    d = prof["gdn"]
    mean_state, mean_tok_q, clips = sweep_stats(args.seed)
    timed_ids = [i for st_ in range(args.warmup, args.warmup + args.steps) for i in step_requests(st_, rank, world, per, args.seed)]
    sample_mean_state = sum(staged[i][0].numel() for i in timed_ids) / max(1, len(timed_ids))
    line = {
        "metric": "answered questions/s", "value": q_all / t_dev, "unit": "questions/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t_dev / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": "sweep: requests of a 64-4096-token state (clipped to fit 4096 with the longest question) "
                               "+ 3 questions of 42-84 tokens (noul/choice/score), random non-special ids",
                   "model": "random-init 2B hybrid (24 layers: 18 gated-delta + 6 attention, int4 g32 weights, int3 embedding)",
                   "requests_per_step_per_gpu": per, "requests_timed": int(q_all // 3), "sweep_mean_state_tokens": round(mean_state, 1),
                   "sample_mean_state_tokens": round(sample_mean_state, 1),
                   "sample": "the requests in sweep_order (length quantiles in bit-reversed order), so the timed ones spread over the sweep's length distribution",
                   "sweep_clipped_requests": clips, "l2": "inputs larger than L2 (0.8 GB of weights streamed per forward)",
                   "parallelism": f"replicas x{world} (requests sharded, no collective)"},
        "prefill_tok_s": tok_all / t_dev,
        "engine_load_s": round(t_load, 3),
        "aggregate_roofline": {"bound_ms_per_step": 1e3 * bound_all / world / args.steps, "frac": bound_all / world / t_dev,
                               "basis": "per packed pass max(bytes / measured HBM, FLOPs / measured sustained bf16), summed over the timed passes"},
        "e2e": {"value": qh_all / t_host, "unit": "questions/s", "h2d_bytes_per_step": int(h2d_step),
                "d2h_bytes_per_step": int(d2h_step), "path": ("sd_forward_batch (the step's states, one snapshot each) + sd_forward_fork_multi_probs (the step's questions, each from its request's snapshot, and the pointer head on the GPU; host ids in, host probabilities out)" if args.two_pass else "sd_forward_tree_probs (the step's states and their questions in one packed pass, each question continuing its request's state, and the pointer head on the GPU; host ids in, host probabilities out)")},
        "gpu_launches": int(launches),
        "roofline": {"kernel": "gemm_q4_tc (dequantizing tcgen05 GEMM)", "bound": "tensor", "achieved": gemm_tflops,
                     "peak": tf_sus, "unit": "TFLOP/s", "frac": gemm_tflops / tf_sus,
                     # dram read+write of one gate_up launch at m=2048 from an ncu capture of
                     # `bench.py --workload gemm --m 2048 --n 12288` (algorithmic: 22.6 MB read)
                     "traffic": 22.586e6, "traffic_launch": "gate_up m=2048 n=12288 k=2048",
                     "peak_source": f"{src} bf16 sustained (kernel timed inside a long step)",
                     "share_of_device_time": g["ms"] / max(1e-9, sum(v["ms"] for v in prof.values()))},
        "kernels": {k: {"ms": round(v["ms"], 3), "launches": v["launches"],
                        "achieved": (v["work"] / (v["ms"] / 1e3) / (1e12 if k in ("gemm", "attention") else 1e9)) if v["ms"] > 0 else 0,
                        "unit": "TFLOP/s" if k in ("gemm", "attention") else "GB/s"} for k, v in prof.items()},
        "clocks": clk,
    }
    if world == 1 and not args.no_configs:
        # the other configurations of the reference's benchmark, beside the sweep (one GPU)
        cf = {}
        cf["1_ask_all"] = config1_ask_all(path, steps=20, warmup=3)
        cf["2_attention"] = kernel_attention(10, 3, args.seed)
        cf["3_gdn"] = kernel_gdn(10, 3, args.seed)
        cf["4_fork"] = config4_fork(eng, head, steps=20, warmup=3)
        cf["5_sweep"] = {"questions_per_s": q_all / t_dev, "e2e_questions_per_s": qh_all / t_host,
                         "sample": f"{int(q_all // 3)} requests in sweep_order (mean state "
                                   f"{sample_mean_state:.0f} tokens; the sweep's {mean_state:.0f})"}
        line["configs"] = cf
    if world == 1 and not args.no_cpu_baseline:
        path = model_path(1, 0)
        dt, tok = cpu_baseline(path, args.seed)
        tok_s = tok / dt
        line["cpu_baseline"] = {"value": tok_s / mean_tok_q, "unit": "questions/s", "cores": os.cpu_count(), "kind": "port",
                                "sample": f"oracle port on request 0 with its state cut to 96 tokens + its 3 questions "
                                          f"({tok} tokens, {dt:.1f} s, {tok_s:.1f} tok/s) scaled to the sweep's "
                                          f"{mean_tok_q:.0f} tokens per question"}
    print(json.dumps(line), flush=True)


def _timed_launches(fn, steps, warmup, flush=None, stream=None):
    """Median device time (ms) of `steps` launches of fn after `warmup`, each timed alone with CUDA
    events on the launching stream, with L2 flushed (a 256 MB write) before each. A 100k-cycle spin
    kernel (torch.cuda._sleep, ~50 us) goes between the flush and the first event, so that the host's
    work of the call (ctypes, tensor maps, launch) is done while the device is busy and the events
    bracket device time only."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(steps):
        if flush is not None:
            flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(100_000)
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    return statistics.median(ts)


def kernel_attention(steps, warmup, seed=0):
    """Config 2: B=4, S=2048, causal GQA 8/2 heads x 256, gated, one sd_attention_batch launch.
    FLOPs = 4 HD HQ B S(S+1)/2 = 6.875e10 (tensor-bound)."""
    import torch
    from strands_decider.engine import attention_batch
    g = torch.Generator(device="cuda").manual_seed(seed)
    B, S, hq, hk, hd = 4, 2048, 8, 2, 256
    q = torch.randn(B, hq, S, hd, generator=g, device="cuda").half()
    k = torch.randn(B, hk, S, hd, generator=g, device="cuda").half()
    v = torch.randn(B, hk, S, hd, generator=g, device="cuda").half()
    gate = torch.randn(B, S, hq * 2 * hd, generator=g, device="cuda").half()
    o = torch.empty(B, S, hq * hd, device="cuda").half()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def fn():
        attention_batch(q.data_ptr(), k.data_ptr(), v.data_ptr(), gate.data_ptr(), hq * 2 * hd, hd, 2 * hd, o.data_ptr(), B, S,
                        0, S, hq, hk, hd)
    ms = _timed_launches(fn, steps, warmup, flush)
    work = 4.0 * hd * hq * B * S * (S + 1) / 2
    _, tf_burst, _, src = peaks()
    return {"us": ms * 1e3, "flops": work, "achieved": work / ms / 1e9, "unit": "TFLOP/s", "peak": tf_burst,
            "frac": work / ms / 1e9 / tf_burst, "peak_source": f"{src} bf16 burst",
            "workload": "config 2: B=4 S=2048 HQ=8 HK=2 HD=256 causal, gated (sd_attention_batch, one launch)",
            "l2": "flushed before each timed launch"}


def kernel_gdn(steps, warmup, seed=0, algo=0):
    """Config 3: B=16, L=1024, 16 heads of 128 x 128, f16 q/k/v, beta = sigmoid(N(0,1)), g =
    -softplus(N(0,1)), the chunked scan with the final states written. Algorithmic bytes: q, k, v f16 +
    beta, g f32 + o f32 + final state f32 = 354.4 MB (HBM-bound)."""
    import torch
    from strands_decider.engine import gdn
    g = torch.Generator(device="cuda").manual_seed(seed)
    B, L, H = 16, 1024, 16
    x = torch.randn(B, L, 3, H * 128, generator=g, device="cuda").half()
    beta = torch.sigmoid(torch.randn(B, L, H, generator=g, device="cuda"))
    gl = -torch.nn.functional.softplus(torch.randn(B, L, H, generator=g, device="cuda"))
    st = torch.zeros(B, H, 128, 128, device="cuda")
    o = torch.empty(B, L, H * 128, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    qp = x.data_ptr()

    def fn():
        gdn(qp, qp + H * 128 * 2, 3 * H * 128, qp + 2 * H * 128 * 2, 3 * H * 128, beta.data_ptr(), gl.data_ptr(),
            st.data_ptr(), 0, o.data_ptr(), L, H, batch=B, seq_qk=L * 3 * H * 128, seq_v=L * 3 * H * 128, in_f16=True, algo=algo)
    ms = _timed_launches(fn, steps, warmup, flush)
    byts = B * L * H * (3 * 128 * 2 + 8 + 128 * 4) + B * H * 128 * 128 * 4
    hbm, _, _, src = peaks()
    return {"us": ms * 1e3, "bytes": byts, "achieved": byts / ms / 1e6, "unit": "GB/s", "peak": hbm,
            "frac": byts / ms / 1e6 / hbm, "peak_source": f"{src} HBM copy",
            "workload": "config 3: B=16 L=1024 H=16 DK=DV=128, f16 q/k/v, fused tcgen05 chunked scan" if algo == 0 else
                        f"config 3 through sd_gdn algo {algo}", "l2": "flushed before each timed launch"}


def kernel_gemm(m, n, k, steps, warmup, seed=0, algo=0):
    import torch
    from strands_decider import model as M
    from strands_decider.engine import QWeight
    g = torch.Generator(device="cuda").manual_seed(seed)
    rng = np.random.default_rng(seed)
    silu = n == 12288
    packed, scales = M._quant_tensor(rng, n, k, 4, 1.0 / np.sqrt(k))
    qd = torch.from_numpy(packed).cuda()
    sd = torch.from_numpy(scales.view(np.uint16)).cuda()
    w = QWeight(qd.data_ptr(), sd.data_ptr(), n, k, interleave=silu)
    a = torch.randn(m, k, generator=g, device="cuda").half()
    y = torch.empty(m, n, device="cuda").half()
    ws = torch.empty(16 << 20, dtype=torch.float32, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def fn():
        w.matmul_ex(a.data_ptr(), m, y.data_ptr(), n // 2 if silu else n, silu=silu, ws_dev=ws.data_ptr(),
                    ws_bytes=ws.numel() * 4, algo=algo)
    ms = _timed_launches(fn, steps, warmup, flush)
    fl = 2.0 * m * n * k
    _, tf_burst, _, src = peaks()
    return {"us": ms * 1e3, "achieved": fl / ms / 1e9, "unit": "TFLOP/s", "peak": tf_burst, "frac": fl / ms / 1e9 / tf_burst,
            "peak_source": f"{src} bf16 burst", "bound": "tensor" if m > 71 else "hbm", "weight_gbs": n * k * 0.5625 / ms / 1e6,
            "workload": f"gemm m={m} n={n} k={k}" + (" (SwiGLU epilogue)" if silu else "") +
                        {0: "", 1: ", tcgen05 tiles", 2: ", small-M mma.sync kernel"}[algo],
            "l2": "flushed before each timed launch"}


WORDS = ("payout", "failing", "account", "billing", "urgent", "refund", "customer", "support", "invoice", "delay",
         "error", "card", "bank", "transfer", "status", "pending", "help", "days", "please", "order", "ticket",
         "escalate", "charge", "merchant", "dashboard", "settings", "email", "phone", "reply", "waiting")


def config1_request(path, n_tokens=128, seed=1):
    """Config 1's System One request: a state of random words rendering to n_tokens tokens (or just
    over) and three questions (noul; choice over 3; score over 3)."""
    from strands_decider import prompt
    from strands_decider.tokenizer import Tokenizer
    with open(os.path.join(path, "tokenizer.json"), encoding="utf-8") as f:
        tok = Tokenizer.from_json(f.read())
    rng = np.random.default_rng(seed)
    words = []
    while len(tok.encode(prompt.render_state(" ".join(words))).ids) < n_tokens:
        words.append(WORDS[int(rng.integers(len(WORDS)))])
    state = " ".join(words)
    return {"state": state, "questions": {
        "urgent": {"type": "noul", "instructions": "Does this convey urgency?"},
        "team": {"type": "choice", "instructions": "Which team should handle this?",
                 "criteria": {"billing": "payments and invoices", "technical": "errors and outages", "sales": "plans and pricing"}},
        "mood": {"type": "score", "instructions": "How frustrated is the writer?", "criteria": ["calm", "frustrated", "very angry"]}}}, \
        len(tok.encode(prompt.render_state(state)).ids)


def config1_ask_all(path, steps, warmup):
    """Config 1: one `ask_all` (sd_decider_ask_all: System One JSON in, the response JSON out, batch 1)
    on a 128-token state with 3 questions: wall-clock latency per call (tokenizer, prompt, the state's
    forward, the batched fork of the questions, the head, the answers)."""
    from strands_decider.engine import NativeDecider
    req, ntok = config1_request(path)
    dec = NativeDecider.load(path)
    for _ in range(warmup):
        dec.ask_all(req)
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        dec.ask_all(req)
        ts.append(time.perf_counter() - t0)
    dec.close()
    lat = statistics.median(ts)
    return {"latency_ms": lat * 1e3, "questions_per_s": 3 / lat, "state_tokens": ntok, "calls": steps,
            "path": "sd_decider_ask_all: JSON request in, JSON response out (host tokenizer and prompt in C++)"}


def config4_fork(eng, head, steps, warmup, seed=4):
    """Config 4: a 512-token state encoded once (kept as a snapshot), then 64 questions of 24-48 random
    non-special tokens continued from it in one batched fork (sd_forward_fork_multi_probs: host ids in,
    each question's probabilities out; the pointer head on the GPU over 2 option rows + the answer
    row). Questions/s from the wall time of the fork calls (host copies included)."""
    rng = np.random.default_rng(seed)

    def ids(n):
        x = rng.integers(0, VOCAB - len(SPECIAL), n)
        return (x + (x >= SPECIAL[0]) * len(SPECIAL)).astype(np.uint32)
    snap = eng.forward(ids(512), [], keep=True).snapshot
    qs = [ids(int(n)) for n in rng.integers(24, 49, 64)]
    rows = [np.array([len(q) // 3, 2 * len(q) // 3, len(q) - 1], np.int32) for q in qs]
    for _ in range(warmup):
        eng.forward_fork_probs([snap] * 64, qs, rows, head, 1.0)
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        eng.forward_fork_probs([snap] * 64, qs, rows, head, 1.0)
        ts.append(time.perf_counter() - t0)
    snap.close()
    t = statistics.median(ts)
    return {"ms_per_fork": t * 1e3, "questions_per_s": 64 / t, "question_tokens": int(sum(len(q) for q in qs)),
            "path": "sd_forward_fork_multi_probs over one 512-token snapshot (64 questions, one packed pass + head)"}


def run_kernel_workload(args):
    """Isolated kernel workloads (not the headline; used for kernel rooflines and ncu captures):
    attention = config 2, gdn = config 3, gemm = one dequantizing matmul shape. Inputs are seeded
    synthetic tensors with the configs' shapes."""
    import torch
    torch.cuda.set_device(0)
    if args.workload == "attention":
        r = kernel_attention(args.steps, args.warmup, args.seed)
        metric = "attention TFLOP/s (config 2)"
    elif args.workload == "gdn":
        r = kernel_gdn(args.steps, args.warmup, args.seed, args.gdn_algo)
        metric = "gated delta rule GB/s (config 3)"
    else:
        r = kernel_gemm(args.m, args.n, args.k, args.steps, args.warmup, args.seed, args.gemm_algo)
        metric = "dequantizing GEMM TFLOP/s"
    line = {"metric": metric, "value": r["achieved"], "unit": r["unit"], "us_per_launch": r["us"],
            "roofline": {k: r[k] for k in ("achieved", "peak", "unit", "frac", "peak_source")}, "config": r,
            "steps": args.steps, "warmup": args.warmup, "n_gpus": 1, "data": "synthetic", "dtype": "f16"}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--requests-per-step", type=int, default=8)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", choices=["sweep", "attention", "gdn", "gemm"], default="sweep",
                    help="sweep: the headline; the others: isolated kernels (config 2, config 3, one GEMM shape)")
    ap.add_argument("--m", type=int, default=2048)
    ap.add_argument("--n", type=int, default=12288)
    ap.add_argument("--k", type=int, default=2048)
    ap.add_argument("--two-pass", action="store_true",
                    help="sweep: the states as one pass kept as snapshots, then the questions as one fork (not one tree pass)")
    ap.add_argument("--gemm-algo", type=int, default=0, choices=[0, 1, 2],
                    help="sd_matmul_ex algo for --workload gemm (0: the planner, 1: tcgen05 tiles, 2: small-M kernel)")
    ap.add_argument("--gdn-algo", type=int, default=0, help="sd_gdn algo for --workload gdn (0: the fused tcgen05 scan)")
    ap.add_argument("--no-configs", action="store_true", help="skip configs 1-4 beside the sweep (N=1 only)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.workload != "sweep":
        run_kernel_workload(args)
        return
    if args.impl == "reference":
        # CPU only and rank 0 only: no process group (the other ranks leave at once, and nothing
        # waits on them)
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
        return
    world, rank, local = dist_setup(args)
    try:
        run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
