"""The hub's host logic (azb_hub) without a GPU, over its CPU stand-in for
the passes (azb_hub_create_fake): every position's outputs are a hash of
its own planes, so a row delivered to the wrong request, a pass over the
tile cap or a lost request shows up as a mismatch.

Follows the reference's hub tests in intent (tests/test_inference_hub.cpp:
results independent of how requests are batched, a failure that sticks,
shutdown with requests waiting): many worker threads on several lanes,
random request sizes, planes and stone-record inputs."""
import threading

import numpy as np
import pytest

import azb200 as E


def fnv_value(row: np.ndarray) -> float:
    h = 1469598103934665603
    for c in np.ascontiguousarray(row, np.float32).tobytes():
        h = ((h ^ c) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return float(np.float32(float(h >> 40) / 16777216.0))


def stone_planes(rng, B, n, H):
    """0/1 planes of random positions, as encodePlanes writes them."""
    A, P = n * n, 2 * H + 2
    x = np.zeros((B, P, A), np.float32)
    for b in range(B):
        black = rng.integers(0, 2)
        for k in range(H):
            stones = rng.choice(3, size=A, p=[0.6, 0.2, 0.2])
            x[b, 2 * k][stones == 1] = 1.0
            x[b, 2 * k + 1][stones == 2] = 1.0
        x[b, 2 * H + (0 if black else 1)] = 1.0
    return x


def check(x, logits, values):
    for b in range(x.shape[0]):
        v = fnv_value(x[b])
        assert values[b] == v, (b, values[b], v)
        assert np.array_equal(logits[b], np.float32(v) + np.arange(logits.shape[1], dtype=np.float32))


def hammer(hub, lanes, workers, requests, n, H, seed, max_request=8):
    errors = []

    def work(w):
        rng = np.random.default_rng(seed + w)
        try:
            for _ in range(requests):
                x = stone_planes(rng, int(rng.integers(1, max_request + 1)), n, H)
                lg, v = hub.evaluate(w % lanes, x)
                check(x, lg, v)
        except Exception as e:   # noqa: BLE001
            errors.append(e)

    threads = [threading.Thread(target=work, args=(w,)) for w in range(workers)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    if errors:
        raise errors[0]


@pytest.mark.parametrize("mode", [E.HUB_PLANES, E.HUB_RECORDS], ids=["planes", "records"])
def test_every_request_gets_its_own_rows(mode):
    d = E.NetDesc(5, 2, 1, 8, 8, 0)
    with E.Hub(d, max_batch=40, slots=2, input_mode=mode, fake={"lanes": 2, "quantum": 8, "delay_us": 300}) as hub:
        assert hub.lanes() == 2 and hub.pass_cap() == 40
        hammer(hub, 2, 12, 15, 5, 2, 100)
        for lane in range(2):
            st = hub.stats(lane)
            assert st["passes"] > 0 and st["positions"] >= st["passes"]
            assert st["positions"] <= st["passes"] * hub.pass_cap()


def test_pass_cap_is_whole_tiles():
    d = E.NetDesc(5, 1, 1, 8, 8, 0)
    with E.Hub(d, max_batch=100, fake={"quantum": 32}) as hub:
        assert hub.pass_cap() == 96
        with pytest.raises(E.CudaError, match="a request of 97 positions"):
            hub.evaluate(0, np.zeros((97, 4, 25), np.float32))
    with E.Hub(d, max_batch=20, fake={"quantum": 32}) as hub:   # below one tile: the limit itself
        assert hub.pass_cap() == 20


def test_full_passes_under_load():
    """Requests of 8 positions (MCTS's leaf batch) from more workers than a
    pass holds: passes go out full while the pass in flight computes."""
    d = E.NetDesc(5, 1, 1, 8, 8, 0)
    xs = [stone_planes(np.random.default_rng(50 + w), 8, 5, 1) for w in range(32)]
    outs = [[] for _ in range(32)]
    with E.Hub(d, max_batch=32, slots=2, fake={"quantum": 8, "delay_us": 5000}) as hub:
        def work(w):
            for _ in range(6):
                outs[w].append(hub.evaluate(0, xs[w]))

        threads = [threading.Thread(target=work, args=(w,)) for w in range(32)]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        st = hub.stats(0)
    assert st["positions"] == 32 * 6 * 8
    assert st["full_passes"] >= st["passes"] // 2, st
    for w in range(32):
        for lg, v in outs[w]:
            check(xs[w], lg, v)


def test_records_match_planes():
    """A records hub gives the planes hub's outputs, from planes or records."""
    d = E.NetDesc(7, 2, 1, 8, 8, 0)
    rng = np.random.default_rng(3)
    x = stone_planes(rng, 9, 7, 2)
    with E.Hub(d, max_batch=16, fake={}) as plain, E.Hub(d, max_batch=16, input_mode=E.HUB_RECORDS, fake={}) as rec:
        a = plain.evaluate(0, x)
        b = rec.evaluate(0, x)
        # the same positions as records: stones k plies ago (1 Black, 2 White), side to move, all present
        A = 49
        to_move = np.where(x[:, 4, 0] == 1.0, 1, 2).astype(np.uint8)
        stones = np.zeros((9, 2, A), np.uint8)
        for i in range(9):
            own, opp = (1, 2) if to_move[i] == 1 else (2, 1)
            for k in range(2):
                stones[i, k][x[i, 2 * k] == 1.0] = own
                stones[i, k][x[i, 2 * k + 1] == 1.0] = opp
        c = rec.evaluate_records(0, E.stones_records(stones, to_move))
    for u, v in zip(a, b):
        assert np.array_equal(u, v)
    for u, v in zip(a, c):
        assert np.array_equal(u, v)
    check(x, *a)


def test_records_mode_refuses_non_stone_planes_and_goes_on():
    d = E.NetDesc(5, 1, 1, 8, 8, 0)
    with E.Hub(d, max_batch=8, input_mode=E.HUB_RECORDS, fake={}) as hub:
        x = stone_planes(np.random.default_rng(1), 2, 5, 1)
        bad = x.copy()
        bad[1, 0, 3] = 0.5
        with pytest.raises(E.CudaError, match="not stone planes"):
            hub.evaluate(0, bad)
        check(x, *hub.evaluate(0, x))   # not a hub failure


def test_planes_hub_refuses_records():
    d = E.NetDesc(5, 1, 1, 8, 8, 0)
    with E.Hub(d, max_batch=8, fake={}) as hub:
        with pytest.raises(E.CudaError, match="takes planes"):
            hub.evaluate_records(0, np.zeros((1, E.stones_record_bytes(1, 5)), np.uint8))


def test_failure_sticks():
    d = E.NetDesc(5, 1, 1, 8, 8, 0)
    with E.Hub(d, max_batch=8, slots=1, fake={"fail_after": 2}) as hub:
        x = stone_planes(np.random.default_rng(2), 1, 5, 1)
        check(x, *hub.evaluate(0, x))
        check(x, *hub.evaluate(0, x))
        with pytest.raises(E.CudaError, match="GPU inference failed: fake: injected failure"):
            hub.evaluate(0, x)
        with pytest.raises(E.CudaError, match="GPU inference failed: fake: injected failure"):
            hub.evaluate(0, x)


def test_destroy_waits_for_requests_in_flight():
    d = E.NetDesc(5, 1, 1, 8, 8, 0)
    hub = E.Hub(d, max_batch=8, slots=1, fake={"delay_us": 200000})
    x = stone_planes(np.random.default_rng(4), 2, 5, 1)
    out, errs = [], []

    def work():
        try:
            out.append(hub.evaluate(0, x))
        except Exception as e:   # noqa: BLE001
            errs.append(str(e))

    threads = [threading.Thread(target=work) for _ in range(3)]
    for t in threads:
        t.start()
    import time

    time.sleep(0.05)   # the first pass is in flight, the others wait for a pass
    hub.close()        # returns once every thread has left evaluate
    for t in threads:
        t.join(timeout=10)
        assert not t.is_alive()
    assert len(out) + len(errs) == 3
    assert len(out) >= 1
    for lg, v in out:
        check(x, lg, v)
    assert all("shut down" in e or "after shutdown" in e for e in errs), errs
