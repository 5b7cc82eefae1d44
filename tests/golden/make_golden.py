"""Generates the golden fixtures in this directory from the REFERENCE's own
code (robominds/alphazero-go compiled from its sources into
oracle/_ref/libazref.so by `make -C oracle ref`).

The reference ships no golden-vector files (its tests generate networks and
inputs from its seeded generator and compare on the fly), so these fixtures
record what its own code produces for fixed seeds:

  rng.json         raw outputs of its Rng (next/uniform/below/normal) and
                   deriveSeed for a few seeds (src/rng.cpp);
  nets.json        per network case: the ParamLayout (names, sizes, offsets),
                   sha256 of the two weight arenas after Network(cfg, seed)
                   and the batch-norm randomiser, sha256 of the inputs;
  <case>.npz       its Network::infer outputs with the naive backend (bit
                   exact: a fixed float summation order) and with OpenBLAS.

Regenerate with:  python tests/golden/make_golden.py   (needs the reference tree)
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))

import oracle as O  # noqa: E402

# (name, NetConfig, seed, kind, input kind, input seed, batch)
CASES = [
    ("c1_5x5_b4_f32", O.NetConfig(5, 1, 4, 32, 64, False), 40, O.KIND_BENCH, "positions", 7, 8),
    ("c1_5x5_b4_f32_test", O.NetConfig(5, 1, 4, 32, 64, False), 41, O.KIND_TEST, "planes", 8, 5),
    ("h8_9x9_b2_f16_own", O.NetConfig(9, 8, 2, 16, 16, True), 40, O.KIND_TEST, "planes", 9, 4),
    ("c2_9x9_b6_f64", O.NetConfig(9, 1, 6, 64, 128, False), 1, O.KIND_BENCH, "positions", 1, 3),
    ("b0_19x19_f16", O.NetConfig(19, 1, 0, 16, 32, False), 3, O.KIND_TEST, "positions", 3, 2),
    ("init_9x9_b1_f8", O.NetConfig(9, 1, 1, 8, 8, False), 5, None, "positions", 5, 3),
]

RNG_SEEDS = [0, 1, 12345, 2**64 - 1]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def inputs(cfg, kind, seed, B):
    if kind == "positions":
        return O.ref_positions(cfg, seed, B)
    out = np.zeros((B, cfg.planes, cfg.area), np.float32)
    O.ref().azref_inputs_planes(seed, out.size, out.ctypes.data_as(O._F))
    return out


def main():
    if not O.ref_available():
        raise SystemExit("make -C oracle ref first (needs the reference tree)")
    rng = {"seeds": {}}
    for s in RNG_SEEDS:
        rng["seeds"][str(s)] = {
            "next": O.ref_rng_sample(s, 0, 8).astype(np.int64).tolist(),
            "uniform": O.ref_rng_sample(s, 1, 8).tolist(),
            "below7": O.ref_rng_sample(s, 2, 8, 7).astype(int).tolist(),
            "normal": O.ref_rng_sample(s, 3, 8).tolist(),
        }
    rng["derive"] = [[a, b, c, d, str(int(O.ref().azref_derive_seed(a, b, c, d)))]
                     for a, b, c, d in [(0, 0, 0, 0), (1, 2, 3, 4), (4, 3, 2, 1), (40, 1, 0, 0), (1, 2, 7, 0)]]
    with open(os.path.join(HERE, "rng.json"), "w") as f:
        json.dump(rng, f, indent=1)

    nets = {}
    for name, cfg, seed, kind, ikind, iseed, B in CASES:
        net = O.RefNetwork(cfg, seed, kind)
        params, buffers = net.arenas()
        x = inputs(cfg, ikind, iseed, B)
        ln, vn, on = net.infer(x, "naive")
        lb, vb, ob = net.infer(x, "blas")
        nets[name] = {
            "config": {"board": cfg.board, "history": cfg.history, "blocks": cfg.blocks, "filters": cfg.filters,
                       "value_hidden": cfg.value_hidden, "ownership": cfg.ownership},
            "seed": seed, "kind": kind, "inputs": {"kind": ikind, "seed": iseed, "batch": B},
            "layout": {"params": net.layout(0), "buffers": net.layout(1)},
            "sha256": {"params": sha(params), "buffers": sha(buffers), "inputs": sha(x)},
            "blas": O.blas_description(),
        }
        arrays = {"logits_naive": ln, "values_naive": vn, "logits_blas": lb, "values_blas": vb}
        if cfg.ownership:
            arrays.update(ownership_naive=on, ownership_blas=ob)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
    with open(os.path.join(HERE, "nets.json"), "w") as f:
        json.dump(nets, f, indent=1)
    print(f"wrote rng.json, nets.json and {len(CASES)} case files")


if __name__ == "__main__":
    main()
