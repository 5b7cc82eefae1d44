"""The persistent tower (alphazero-go_b200/csrc/conv_tc.cu, kPersist): every
tower conv of a network in one launch (bf16 and tf32; tf32x3 at 128 channels
or fewer, in its accumulation segments), CTAs taking (layer, tile group)
items from a counter, each item's halo loads waiting (bounded) for the
previous layer's groups whose rows they read.

Each item runs the per-layer kernel's MMAs and epilogue on the same rows,
so its outputs must equal the per-layer path's bit for bit (logits, values,
ownership): batches of one board, ragged batches whose last tile is
partial, batches of several tile groups per SM, odd and even tower depths
(the trunk ends in a different buffer), 19x19 down to 11x11, 32 to 256
channels. A board alone and the same board inside a batch give the same
bits. Two passes in flight on the runner's two slots (two persistent
launches on two streams, sharing the SMs) complete and agree.
"""
import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(engine, c, params, buffers, x, precision, persistent):
    engine.cuda_probe.set_tower_persistent(1 if persistent else 0)
    try:
        with engine.CudaInference(engine.NetDesc.of(c), params, buffers, x.shape[0], 0, precision) as net:
            return net.infer(x)
    finally:
        engine.cuda_probe.set_tower_persistent(-1)


@pytest.mark.parametrize("precision", ["bf16", "tf32", "tf32x3"])
@pytest.mark.parametrize("shape,B", [((19, 2, 64, 1, False), 64), ((19, 3, 128, 1, False), 7), ((13, 2, 32, 8, True), 5),
                                     ((11, 1, 64, 1, False), 1), ((19, 2, 128, 1, True), 200),
                                     ((19, 1, 256, 1, False), 33), ((15, 4, 64, 2, False), 300)])
def test_persistent_tower_equals_per_layer(engine, oracle, precision, shape, B):
    O = oracle
    n, blocks, filters, history, own = shape
    c = O.NetConfig(n, history, blocks, filters, 64, own)
    params, buffers = O.make_network(c, 81, O.KIND_TEST)
    x = O.random_planes(c, 82, B)
    prec = engine.PRECISIONS[precision]
    persistent = _run(engine, c, params, buffers, x, prec, True)
    layered = _run(engine, c, params, buffers, x, prec, False)
    for k in range(3):
        if persistent[k] is not None:
            assert np.array_equal(persistent[k], layered[k]), (precision, shape, B, k)


def test_persistent_tower_batch_independent(engine, oracle):
    """A board's outputs are the same bits alone and at any slot of a batch."""
    O = oracle
    c = O.NetConfig(19, 1, 2, 128, 64, False)
    params, buffers = O.make_network(c, 83, O.KIND_TEST)
    pool = O.random_planes(c, 84, 96)
    engine.cuda_probe.set_tower_persistent(1)
    try:
        with engine.CudaInference(engine.NetDesc.of(c), params, buffers, 96, 0, engine.BF16) as net:
            whole = net.infer(pool)
            for s in (0, 1, 40, 95):
                alone = net.infer(pool[s:s + 1])
                for k in range(2):
                    assert np.array_equal(whole[k][s], alone[k][0]), (s, k)
    finally:
        engine.cuda_probe.set_tower_persistent(-1)


def test_persistent_towers_on_two_streams(engine, oracle):
    """The runner's two slots put two persistent launches in flight at once;
    both complete (items are taken only by running CTAs, so neither waits on
    a CTA the other keeps from starting) and match the synchronous pass."""
    O = oracle
    c = O.NetConfig(19, 1, 3, 128, 64, False)
    params, buffers = O.make_network(c, 85, O.KIND_TEST)
    B = 256
    x = [O.random_planes(c, 86 + i, B) for i in range(2)]
    desc = engine.NetDesc.of(c)
    engine.cuda_probe.set_tower_persistent(1)
    try:
        with engine.CudaInference(desc, params, buffers, B, 0, engine.BF16) as net:
            want = [net.infer(xi) for xi in x]
        runner = engine.make_cuda_runner(desc, params, buffers, B, 2, 0, engine.BF16)
        try:
            for rounds in range(4):
                done, cv = [], threading.Condition()

                def cb(slot, err):
                    with cv:
                        done.append((slot, err))
                        cv.notify()

                for sl in range(2):
                    runner.input(sl)[:] = x[sl]
                for sl in range(2):
                    runner.begin(sl, B, cb)
                with cv:
                    assert cv.wait_for(lambda: len(done) == 2, timeout=30), done
                assert all(err == "" for _, err in done), done
                for sl in range(2):
                    assert np.array_equal(runner.logits(sl, B), want[sl][0]), (rounds, sl)
                    assert np.array_equal(runner.values(sl, B), want[sl][1]), (rounds, sl)
        finally:
            runner.close()
    finally:
        engine.cuda_probe.set_tower_persistent(-1)


def test_persistent_tower_wait_runs_out_and_recovers(engine, oracle):
    """Failure detection without a GPU fault: with the counters' target one
    step beyond what the epilogue warps add, the first wait for a previous
    layer ends after its bound, the pass reports it, and the next pass on the
    same handle gives the per-layer path's bits."""
    O = oracle
    c = O.NetConfig(19, 1, 2, 64, 64, False)
    params, buffers = O.make_network(c, 87, O.KIND_TEST)
    x = O.random_planes(c, 88, 16)
    layered = _run(engine, c, params, buffers, x, engine.BF16, False)
    engine.cuda_probe.set_tower_persistent(1)
    try:
        with engine.CudaInference(engine.NetDesc.of(c), params, buffers, 16, 0, engine.BF16) as net:
            engine.cuda_probe.starve_tower(True)
            try:
                with pytest.raises(RuntimeError, match="the persistent tower waited too long for the previous layer"):
                    net.infer(x)
            finally:
                engine.cuda_probe.starve_tower(False)
            again = net.infer(x)
            for k in range(2):
                assert np.array_equal(again[k], layered[k]), k
    finally:
        engine.cuda_probe.set_tower_persistent(-1)
