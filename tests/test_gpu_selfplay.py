"""Self-play on the engine through the reference's own search and hub.

Mirrors the reference's tests/test_cuda.cpp:1270-1348 (the determinism
contract of a cuda engine's slice): the same games, byte for byte, for 1, 3
and 8 workers, batches capped at 8 or 256, and the hub's chaos mode on or
off. Records are compared through the driver's FNV-1a hash of every game in
index order.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_LIB = os.path.join(ROOT, "alphazero-go_b200", "host", "_ref", "libazselfplay.so")


@pytest.fixture(scope="module")
def sp(engine):
    if not os.path.exists(PKG_LIB):
        pytest.skip("alphazero-go_b200/host/_ref/libazselfplay.so is not built (needs the reference tree)")
    import selfplay

    return selfplay


@pytest.mark.parametrize("shape", [(5, 1, 8, 16), (9, 2, 16, 32)])
@pytest.mark.parametrize("precision", ["tf32x3", "bf16"])
def test_slice_independent_of_workers_and_batching(engine, sp, shape, precision):
    d = engine.NetDesc(shape[0], 1, shape[1], shape[2], shape[3], 0)
    p, b = engine.synth_network(d, 801, 1)
    reference = None
    for workers in (1, 3, 8):
        for batch in (8, 256):
            for chaos in (0, 21):
                engine.cuda_probe.set_hub_chaos_seed(chaos)
                try:
                    r = sp.play(d, p, b, backend="cuda", workers=workers, inference_batch=batch,
                                precision=engine.PRECISIONS[precision], simulations=32, mcts_batch=8,
                                temperature_moves=6, seed=802, generation=3, first=10, count=6)
                finally:
                    engine.cuda_probe.set_hub_chaos_seed(0)
                assert r["evaluations"] > 0
                if reference is None:
                    reference = r["record_hash"]
                assert r["record_hash"] == reference, (workers, batch, chaos)


WAVE = [(0, 1, 6, 901), (0, ("bot", 8), 4, 902), (0, 2, 4, 903)]


def test_arena_wave_independent_of_workers_and_batching(engine, sp):
    """tests/test_cuda.cpp:1301-1348: an arena wave on the cuda engine (one hub per network, three
    networks sharing the GPU) plays the same games for any workers, batch cap and chaos mode, and a
    wave played in two slices plays what the whole wave plays."""
    d = engine.NetDesc(5, 1, 1, 8, 16, 0)
    nets = [engine.synth_network(d, s, 1) for s in (811, 812, 813)]
    kw = dict(simulations=16, mcts_batch=4, temperature_moves=2, backend="cuda", precision=engine.TF32X3)
    reference = None
    for workers in (1, 3, 0):
        for batch in (8, 256):
            for chaos in (0, 23):
                engine.cuda_probe.set_hub_chaos_seed(chaos)
                try:
                    r = sp.arena(d, nets, WAVE, first=0, count=14, workers=workers, inference_batch=batch, **kw)
                finally:
                    engine.cuda_probe.set_hub_chaos_seed(0)
                assert r["evaluations"] > 0
                if reference is None:
                    reference = r["games"]
                assert r["games"] == reference, (workers, batch, chaos)
    a = sp.arena(d, nets, WAVE, first=0, count=5, **kw)
    b = sp.arena(d, nets, WAVE, first=5, count=9, **kw)
    assert a["games"] + b["games"] == reference


@pytest.mark.parametrize("precision", ["tf32x3", "bf16"])
def test_engine_hub_plays_the_reference_hubs_games(engine, sp, precision):
    """The engine's own hub (azb_hub: workers copy their own rows, passes
    capped at whole tiles, a lane per GPU) plays byte for byte the games the
    reference's InferenceHub plays over the same engine, with planes or with
    stone records carried to the GPU, for any worker count and batch cap;
    on every GPU present as lanes, the same again."""
    d = engine.NetDesc(9, 1, 2, 32, 32, 0)
    p, b = engine.synth_network(d, 805, 1)
    kw = dict(precision=engine.PRECISIONS[precision], simulations=32, mcts_batch=8, temperature_moves=6, seed=806,
              generation=2, first=4, count=8)
    want = sp.play(d, p, b, backend="cuda", workers=4, inference_batch=64, **kw)["record_hash"]
    devices = list(range(min(engine.device_count(), 2)))
    for records in (False, True):
        for workers, batch in ((1, 8), (8, 64), (8, 100)):
            for devs in ({0}, set(devices)):
                r = sp.play_hub(d, p, b, devices=sorted(devs), records=records, workers=workers,
                                inference_batch=batch, **kw)
                assert r["record_hash"] == want, (records, workers, batch, devs)
                assert r["evaluations"] > 0 and r["passes"] > 0
                # 9x9 frames run in the small-board tower's groups of one board: any cap is whole tiles
                assert r["pass_cap"] == batch


def test_engine_hub_pass_cap_whole_tiles(engine):
    """19x19 frames are 400 rows: a pass is whole 128-row tiles when its
    boards are a multiple of 8, so a cap of 100 becomes 96."""
    d = engine.NetDesc(19, 1, 1, 32, 32, 0)
    p, b = engine.synth_network(d, 807, 1)
    with engine.Hub(d, p, b, devices=[0], max_batch=100, precision=engine.BF16) as hub:
        assert hub.pass_cap() == 96
        x = engine.synth_positions(d, 807, 8)
        with engine.CudaInference(d, p, b, 8, 0, engine.BF16) as net:
            want = net.infer(x)
        got = hub.evaluate(0, x)
        assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1])
