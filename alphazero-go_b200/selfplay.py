"""Self-play with the reference's own search on a chosen engine.

ctypes over host/_ref/libazselfplay.so (host/Makefile): the reference's
playSelfPlayGame (src/selfplay.cpp:50) and WorkerEvaluators/InferenceHub
(src/inference_hub.cpp), compiled from its sources with this package's
drop-in bridge as its "cuda" engine. A slice of games is played the way the
reference's playSelfPlayQueue plays one (src/selfplay_slice.cpp:93-149); the
statistics are SliceStats', and playouts/s = positions x simulations /
seconds, as the reference reports it. `arena` plays an arena wave (several
matches, one hub per network) through the reference's playArenaGames.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "host", "_ref", "libazselfplay.so")

_libs: dict[str, C.CDLL] = {}


def _lib(path: str) -> C.CDLL:
    if path not in _libs:
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is not built: make -C {os.path.join(HERE, 'host')} (needs the reference tree)")
        L = C.CDLL(path)
        F = C.POINTER(C.c_float)
        L.azsp_play.argtypes = ([C.c_int] * 5 + [F, C.c_size_t, F, C.c_size_t, C.c_char_p] + [C.c_int] * 6 +
                                [C.c_float, C.c_int, C.c_float, C.c_int, C.c_uint64, C.c_int, C.c_int, C.c_int,
                                 C.POINTER(C.c_double), C.POINTER(C.c_longlong), C.POINTER(C.c_longlong),
                                 C.POINTER(C.c_uint64), C.c_char_p, C.c_size_t])
        L.azsp_play.restype = C.c_int
        PF, PS = C.POINTER(F), C.POINTER(C.c_size_t)
        PI, PU = C.POINTER(C.c_int), C.POINTER(C.c_uint64)
        L.azsp_arena.argtypes = ([C.c_int] * 6 + [PF, PS, PF, PS, C.c_int, PI, PI, PI, PI, PU] + [C.c_int] * 5 +
                                 [C.c_char_p] + [C.c_int] * 4 + [C.POINTER(C.c_double), C.POINTER(C.c_longlong),
                                                                 PU, PU, C.c_char_p, C.c_size_t])
        L.azsp_arena.restype = C.c_int
        if hasattr(L, "azsp_play_hub"):
            PL, PD = C.POINTER(C.c_longlong), C.POINTER(C.c_double)
            L.azsp_play_hub.argtypes = ([C.c_int] * 5 + [F, C.c_size_t, F, C.c_size_t, PI] + [C.c_int] * 7 +
                                        [C.c_float, C.c_int, C.c_float, C.c_int, C.c_uint64, C.c_int, C.c_int,
                                         C.c_int, PD, PL, PL, PU, PL, PL, PI, C.c_char_p, C.c_size_t])
            L.azsp_play_hub.restype = C.c_int
        _libs[path] = L
    return _libs[path]


def play(desc, params: np.ndarray, buffers: np.ndarray, *, backend: str = "cuda", workers: int = 512,
         inference_batch: int = 256, device: int = 0, precision: int = 2, simulations: int = 200,
         mcts_batch: int = 8, c_puct: float = 1.5, temperature_moves: int = 7, komi: float = 7.5,
         max_moves: int = 0, seed: int = 1, generation: int = 0, first: int = 0, count: int = 512,
         lib_path: str | None = None) -> dict:
    """Plays games [first, first + count) and returns the slice's statistics.

    desc: an object with board, history, blocks, filters, value_hidden (the
    network's shape); params/buffers: its two ParamLayout arenas (float32).
    """
    L = _lib(lib_path or LIB_PATH)
    p = np.ascontiguousarray(params, np.float32)
    b = np.ascontiguousarray(buffers, np.float32)
    F = C.POINTER(C.c_float)
    secs, pos, evals, h = C.c_double(), C.c_longlong(), C.c_longlong(), C.c_uint64()
    err = C.create_string_buffer(1024)
    rc = L.azsp_play(desc.board, desc.history, desc.blocks, desc.filters, desc.value_hidden,
                     p.ctypes.data_as(F), p.size, b.ctypes.data_as(F), b.size, backend.encode(), workers,
                     inference_batch, device, precision, simulations, mcts_batch, c_puct, temperature_moves, komi,
                     max_moves, seed, generation, first, count, C.byref(secs), C.byref(pos), C.byref(evals),
                     C.byref(h), err, 1024)
    if rc != 0:
        raise RuntimeError(err.value.decode())
    s = secs.value
    return {"seconds": s, "positions": pos.value, "evaluations": evals.value, "record_hash": h.value,
            "playouts_per_s": pos.value * simulations / s if s > 0 else 0.0,
            "evaluations_per_s": evals.value / s if s > 0 else 0.0}


def play_hub(desc, params: np.ndarray, buffers: np.ndarray, *, devices=(0,), records: bool = False,
             workers: int = 512, inference_batch: int = 256, precision: int = 2, simulations: int = 200,
             mcts_batch: int = 8, c_puct: float = 1.5, temperature_moves: int = 7, komi: float = 7.5,
             max_moves: int = 0, seed: int = 1, generation: int = 0, first: int = 0, count: int = 512,
             lib_path: str | None = None) -> dict:
    """play() on the engine's own hub (azb_hub): a lane per device in
    `devices`, worker w on lane w % len(devices); records=True carries stone
    records to the GPU. Adds the hub's passes, its full passes and its cap."""
    L = _lib(lib_path or LIB_PATH)
    p = np.ascontiguousarray(params, np.float32)
    b = np.ascontiguousarray(buffers, np.float32)
    F = C.POINTER(C.c_float)
    devs = (C.c_int * len(devices))(*devices)
    secs, pos, evals, h = C.c_double(), C.c_longlong(), C.c_longlong(), C.c_uint64()
    passes, full, cap = C.c_longlong(), C.c_longlong(), C.c_int()
    err = C.create_string_buffer(1024)
    rc = L.azsp_play_hub(desc.board, desc.history, desc.blocks, desc.filters, desc.value_hidden,
                         p.ctypes.data_as(F), p.size, b.ctypes.data_as(F), b.size, devs, len(devices), int(records),
                         workers, inference_batch, precision, simulations, mcts_batch, c_puct, temperature_moves,
                         komi, max_moves, seed, generation, first, count, C.byref(secs), C.byref(pos),
                         C.byref(evals), C.byref(h), C.byref(passes), C.byref(full), C.byref(cap), err, 1024)
    if rc != 0:
        raise RuntimeError(err.value.decode())
    s = secs.value
    return {"seconds": s, "positions": pos.value, "evaluations": evals.value, "record_hash": h.value,
            "playouts_per_s": pos.value * simulations / s if s > 0 else 0.0,
            "evaluations_per_s": evals.value / s if s > 0 else 0.0,
            "passes": passes.value, "full_passes": full.value, "pass_cap": cap.value}


def arena(desc, nets: list, matches: list, *, first: int = 0, count: int | None = None, simulations: int = 100,
          mcts_batch: int = 8, temperature_moves: int = 4, backend: str = "cuda", workers: int = 0,
          inference_batch: int = 256, device: int = 0, precision: int = 2, lib_path: str | None = None) -> dict:
    """An arena wave through the reference's playArenaGames (src/arena.cpp).

    nets: [(params, buffers), ...]; matches: [(a, b, games, seed), ...] with
    a, b network indices, or b = ("bot", simulations) for a uniform bot.
    Games [first, first + count) of the wave (match-major) are played."""
    L = _lib(lib_path or LIB_PATH)
    F = C.POINTER(C.c_float)
    arrs = [(np.ascontiguousarray(p, np.float32), np.ascontiguousarray(b, np.float32)) for p, b in nets]
    n = len(arrs)
    P = (F * n)(*[a[0].ctypes.data_as(F) for a in arrs])
    B = (F * n)(*[a[1].ctypes.data_as(F) for a in arrs])
    NP = (C.c_size_t * n)(*[a[0].size for a in arrs])
    NB = (C.c_size_t * n)(*[a[1].size for a in arrs])
    m = len(matches)
    a_net = (C.c_int * m)(*[x[0] for x in matches])
    b_net = (C.c_int * m)(*[x[1] if isinstance(x[1], int) else -1 for x in matches])
    bots = (C.c_int * m)(*[0 if isinstance(x[1], int) else x[1][1] for x in matches])
    games = (C.c_int * m)(*[x[2] for x in matches])
    seeds = (C.c_uint64 * m)(*[x[3] for x in matches])
    if count is None:
        count = sum(x[2] for x in matches) - first
    score, evals, h = C.c_double(), C.c_longlong(), C.c_uint64()
    per_game = (C.c_uint64 * max(1, count))()
    err = C.create_string_buffer(1024)
    rc = L.azsp_arena(desc.board, desc.history, desc.blocks, desc.filters, desc.value_hidden, n, P, NP, B, NB, m,
                      a_net, b_net, bots, games, seeds, first, count, simulations, mcts_batch, temperature_moves,
                      backend.encode(), workers, inference_batch, device, precision, C.byref(score), C.byref(evals),
                      C.byref(h), per_game, err, 1024)
    if rc != 0:
        raise RuntimeError(err.value.decode())
    return {"score_a": score.value, "evaluations": evals.value, "record_hash": h.value,
            "games": list(per_game)[:count]}
