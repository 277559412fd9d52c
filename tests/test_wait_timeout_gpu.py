"""The failure path of the warp-specialised kernels, which no valid input reaches: every wait on a
barrier is bounded, and a wait that runs out records an error code for the host and makes the rest of
its CTA leave instead of waiting on (the reference returns device errors as `Err`,
`src/engine.rs:648-651`). `sd_engine_selftest_wait` runs one such wait on purpose (on a barrier that
nothing completes, so no GPU fault is involved): the call must fail with SD_ERR_KERNEL and the timeout's
message, well before the 2 s limit of the second warp (it must leave on the abort flag), and the engine
must answer correctly afterwards."""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_a_wait_that_runs_out_fails_the_call_and_the_engine_recovers(small_model):
    from strands_decider.engine import Engine, Error
    eng = Engine.load(small_model)
    ids = np.random.default_rng(3).integers(0, 8000, 40)
    before = eng.forward(ids, [39]).hidden
    t0 = time.perf_counter()
    with pytest.raises(Error) as ei:
        eng.selftest_wait(2000)  # 2 ms
    elapsed = time.perf_counter() - t0
    assert ei.value.code == -5 and "bounded wait ran out" in str(ei.value)
    assert elapsed < 1.0, elapsed  # the warp with the 2 s limit left on the abort flag
    with pytest.raises(Error):
        eng.selftest_wait(0)  # a limit out of range is refused before anything runs
    after = eng.forward(ids, [39]).hidden
    assert np.array_equal(before, after)
    eng.close()
