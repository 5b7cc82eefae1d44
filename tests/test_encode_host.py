"""Position records and the reference's encoder, on the CPU.

The engine's device encoder (azb_infer_run_stones) writes what the
reference's encodePlanes (src/encode.cpp:15-43) writes from the same
stones, side to move, history length and symmetry. Here the record layout
and a numpy restatement of encodePlanes are checked against the reference
itself (oracle/_ref/libazref.so); the GPU test compares the device encoder
with both.
"""
import numpy as np
import pytest


def transform_point(sym, p, n):
    """src/symmetry.cpp:6-19."""
    row, col = divmod(p, n)
    if sym & 4:
        col = n - 1 - col
    for _ in range(sym & 3):
        row, col = col, n - 1 - row
    return row * n + col


def encode_planes(stones, to_move, available, sym, n, H):
    """A restatement of encodePlanes for one record."""
    A = n * n
    out = np.zeros((2 * H + 2, A), np.float32)
    own, opp = to_move, 3 - to_move
    dest = [transform_point(sym, p, n) for p in range(A)]
    for k in range(min(H, available)):
        for p in range(A):
            if stones[k][p] == own:
                out[2 * k][dest[p]] = 1.0
            elif stones[k][p] == opp:
                out[2 * k + 1][dest[p]] = 1.0
    out[2 * H + (0 if to_move == 1 else 1)] = 1.0
    return out


def random_records(E, n, H, B, seed):
    rng = np.random.default_rng(seed)
    stones = rng.choice(np.array([0, 1, 2], np.uint8), size=(B, H, n * n), p=[0.5, 0.25, 0.25])
    to_move = rng.integers(1, 3, B)
    available = rng.integers(0, H + 1, B)
    sym = rng.integers(0, 8, B)
    return stones, to_move, available, sym, E.stones_records(stones, to_move, available, sym)


@pytest.mark.parametrize("n,H", [(5, 1), (9, 8), (19, 2)])
def test_restated_encoder_matches_the_reference(oracle, n, H):
    import azb200 as E

    if not oracle.ref_available():
        pytest.skip("oracle/_ref/libazref.so is not built")
    stones, to_move, available, sym, rec = random_records(E, n, H, 12, 5 + n + H)
    assert rec.shape[1] == E.stones_record_bytes(H, n) and rec.shape[1] % 4 == 0
    cfg = oracle.NetConfig(n, H, 1, 8, 8, False)
    ref = oracle.ref_encode_records(cfg, rec)
    for b in range(rec.shape[0]):
        mine = encode_planes(stones[b], int(to_move[b]), int(available[b]), int(sym[b]), n, H)
        assert np.array_equal(mine, ref[b]), b
