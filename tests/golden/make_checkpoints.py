"""Writes the checkpoint fixtures in this directory with the REFERENCE's own
saveNetwork (robominds/alphazero-go src/checkpoint.cpp, compiled from its
sources into oracle/_ref/libazref.so by `make -C oracle ref`):

  ckpt_9x9_b2_f16.azn          version 1 (no ownership head): Network(cfg, 5)
                               plus the test batch-norm randomiser;
  ckpt_9x9_h8_b1_f8_own.azn    version 2 (ownership head), history 8.

checkpoints.json records, per file, the shape and the sha256 of the two
ParamLayout arenas the reference's loadNetwork rebuilds from it.

Regenerate with:  python tests/golden/make_checkpoints.py   (needs the reference tree)
"""
import hashlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))

import oracle as O  # noqa: E402

CASES = [
    ("ckpt_9x9_b2_f16.azn", O.NetConfig(9, 1, 2, 16, 16, False), 5),
    ("ckpt_9x9_h8_b1_f8_own.azn", O.NetConfig(9, 8, 1, 8, 8, True), 6),
]


def main():
    out = {}
    for name, cfg, seed in CASES:
        path = os.path.join(HERE, name)
        O.RefNetwork(cfg, seed, O.KIND_TEST).save_checkpoint(path)
        shape, params, buffers = O.ref_load_checkpoint(path)
        out[name] = {"shape": list(shape), "seed": seed, "kind": "test",
                     "params_sha256": hashlib.sha256(params.tobytes()).hexdigest(),
                     "buffers_sha256": hashlib.sha256(buffers.tobytes()).hexdigest(),
                     "params_floats": int(params.size), "buffers_floats": int(buffers.size)}
    with open(os.path.join(HERE, "checkpoints.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)
        f.write("\n")


if __name__ == "__main__":
    main()
