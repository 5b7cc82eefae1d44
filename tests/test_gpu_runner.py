"""The runner through its C ABI (BatchRunner, include/azgo/inference_hub.hpp:41-53),
following the reference's runner tests (tests/test_cuda.cpp:1022-1091,
1220-1237): with 1 and 2 slots, every batch size gives the bits of the
positions evaluated one at a time; a pass is reported only after its outputs
reached the host (checked with the copy-out delay hook); done is called
exactly once per begin, also for a batch out of range; destroying a runner
drains the passes in flight."""
import threading
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def make(engine, oracle, precision, max_batch=32, slots=2, own=False):
    cfg = oracle.NetConfig(9, 1, 2, 16, 16, own)
    params, buffers = oracle.make_network(cfg, 701, oracle.KIND_TEST)
    desc = engine.NetDesc.of(cfg)
    return cfg, desc, params, buffers


class Waiter:
    def __init__(self):
        self.cv = threading.Condition()
        self.done = []

    def __call__(self, slot, err):
        with self.cv:
            self.done.append((slot, err))
            self.cv.notify_all()

    def wait(self, n, timeout=30.0):
        end = time.time() + timeout
        with self.cv:
            while len(self.done) < n:
                left = end - time.time()
                assert left > 0, "done was not called"
                self.cv.wait(left)
            return list(self.done)


@pytest.mark.parametrize("precision", ["bf16", "tf32x3"])
@pytest.mark.parametrize("slots", [1, 2])
def test_runner_equals_one_at_a_time(engine, oracle, precision, slots):
    cfg, desc, params, buffers = make(engine, oracle, precision)
    prec = engine.PRECISIONS[precision]
    x = oracle.random_planes(cfg, 702, 32)
    with engine.CudaInference(desc, params, buffers, 1, 0, prec) as alone:
        ref = [alone.infer(x[i:i + 1]) for i in range(32)]
    runner = engine.make_cuda_runner(desc, params, buffers, 32, slots, 0, prec)
    assert runner.slots() == slots and runner.max_batch() == 32
    for B in (1, 2, 7, 31, 32):
        w = Waiter()
        for s in range(slots):
            runner.input(s)[:B] = x[:B]
            runner.begin(s, B, w)
        got = w.wait(slots)
        assert sorted(s for s, _ in got) == list(range(slots)) and all(e == "" for _, e in got)
        for s in range(slots):
            for i in range(B):
                assert np.array_equal(runner.logits(s, B)[i], ref[i][0][0])
                assert np.array_equal(runner.values(s, B)[i], ref[i][1][0])
    runner.close()


def test_pass_reported_after_copy_out(engine, oracle):
    cfg, desc, params, buffers = make(engine, oracle, "bf16")
    x = oracle.random_planes(cfg, 703, 8)
    runner = engine.make_cuda_runner(desc, params, buffers, 8, 1, 0, engine.BF16)
    runner.input(0)[:8] = x
    w = Waiter()
    runner.begin(0, 8, w)
    w.wait(1)
    first = runner.logits(0, 8).copy()
    runner.logits(0, 8)[:] = np.nan        # scribble over the host staging
    engine.cuda_probe.set_copy_out_delay(20000)
    try:
        before = engine.cuda_probe.passes_completed()
        w2 = Waiter()
        runner.begin(0, 8, w2)
        w2.wait(1)
        assert engine.cuda_probe.passes_completed() == before + 1
        assert np.array_equal(runner.logits(0, 8), first)   # the copy landed before done
    finally:
        engine.cuda_probe.set_copy_out_delay(0)
    runner.close()


def test_batch_out_of_range_reports_through_done(engine, oracle):
    cfg, desc, params, buffers = make(engine, oracle, "bf16")
    runner = engine.make_cuda_runner(desc, params, buffers, 8, 2, 0, engine.BF16)
    w = Waiter()
    runner.begin(1, 9, w)
    (slot, err), = w.wait(1)
    assert slot == 1 and "batch out of range" in err
    with pytest.raises(IndexError):
        runner.begin(2, 1, w)
    runner.close()


def test_destroy_drains_in_flight(engine, oracle):
    cfg, desc, params, buffers = make(engine, oracle, "bf16")
    runner = engine.make_cuda_runner(desc, params, buffers, 32, 2, 0, engine.BF16)
    w = Waiter()
    engine.cuda_probe.set_copy_out_delay(50000)
    try:
        runner.begin(0, 32, w)
        runner.begin(1, 32, w)
        runner.close()            # returns only after both passes reported
        assert len(w.done) == 2 and all(e == "" for _, e in w.done)
    finally:
        engine.cuda_probe.set_copy_out_delay(0)


def test_slots_validated(engine, oracle):
    cfg, desc, params, buffers = make(engine, oracle, "bf16")
    for slots in (0, 3):
        with pytest.raises(ValueError, match="slots must be in"):
            engine.make_cuda_runner(desc, params, buffers, 8, slots, 0, engine.BF16)


def test_memory_check(engine, oracle):
    desc = engine.NetDesc(19, 1, 20, 256, 256, 0)
    engine.check_cuda_inference_memory(desc, 1024, 1, 2, 0, engine.BF16)
    with pytest.raises(engine.CudaError, match="lower inference_batch"):
        engine.check_cuda_inference_memory(desc, 1024, 400, 2, 0, engine.BF16)
    engine.cuda_probe.set_memory_limit(1 << 20)
    try:
        with pytest.raises(engine.CudaError, match="inference needs"):
            engine.check_cuda_inference_memory(desc, 8, 1, 1, 0, engine.BF16)
    finally:
        engine.cuda_probe.set_memory_limit(0)
