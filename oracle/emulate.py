"""Numeric emulation of the engine's precision modes on the CPU (test
infrastructure only).

The forward of the reference network (Network::forward in inference mode,
src/network.cpp:228-309) in float64, with the engine's roundings applied where
the engine applies them:
  * "tf32": every conv operand rounded to tf32 (weights nearest, activations
    truncated, as a tf32 MMA reads fp32 bits), fp32 activations;
  * "bf16": conv weights and activations rounded to bf16 (nearest even),
    activations stored bf16;
  * "f64": no rounding at all (the reference for the others).
It predicts the parity the GPU can reach in each mode; the GPU's own numbers
are measured by tests/test_gpu_network.py. Usage:

    python oracle/emulate.py C2 C3 C4
"""
from __future__ import annotations

import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import oracle as O  # noqa: E402


def round_bits(x, bits: int, mode: str = "rn") -> np.ndarray:
    """Keep `bits` mantissa bits of float32 x: nearest-even ("rn") or truncation."""
    x = np.asarray(x, np.float32).copy()
    u = x.view(np.uint32)
    drop = 23 - bits
    if mode == "rn":
        u[:] = (u + ((u >> drop) & 1) + np.uint32((1 << (drop - 1)) - 1)) & ~np.uint32((1 << drop) - 1)
    else:
        u[:] = u & ~np.uint32((1 << drop) - 1)
    return x


def conv3(x: np.ndarray, w: np.ndarray, n: int) -> np.ndarray:
    """'Same' 3x3 conv: x [B][A][C], w [cout][C*9] (reference order c*9 + tap)."""
    B, A, C = x.shape
    xp = np.zeros((B, n + 2, n + 2, C))
    xp[:, 1:-1, 1:-1, :] = x.reshape(B, n, n, C)
    cols = np.stack([xp[:, dy:dy + n, dx:dx + n, :] for dy in range(3) for dx in range(3)], axis=-1)
    return (cols.reshape(B * A, C * 9) @ w.T).reshape(B, A, -1)


def forward(cfg: O.NetConfig, params, buffers, inp: np.ndarray, mode: str):
    """(logits, values) with the roundings of `mode`."""
    offs = {n: (s, o) for n, s, o in O.layout(cfg, 0)}
    boffs = {n: (s, o) for n, s, o in O.layout(cfg, 1)}

    def T(name):
        s, o = offs[name] if name in offs else boffs[name]
        arr = params if name in offs else buffers
        return arr[o:o + s].astype(np.float64)

    n, A, F = cfg.board, cfg.area, cfg.filters

    def opw(w):
        if mode == "tf32":
            return round_bits(w, 10).astype(np.float64)
        if mode == "bf16":
            return round_bits(w, 7).astype(np.float64)
        return w

    def opa(a):
        if mode == "tf32":
            return round_bits(a, 10, "trunc").astype(np.float64)
        return a

    def store(a):
        if mode == "bf16":
            return round_bits(a, 7).astype(np.float64)
        return a if mode == "f64" else np.asarray(a, np.float32).astype(np.float64)

    def bn(x, pre):
        sc = T(pre + ".gamma") / np.sqrt(T(pre + ".runVar") + np.float64(np.float32(1e-5)))
        return (x - T(pre + ".runMean")) * sc + T(pre + ".beta")

    x = inp.transpose(0, 2, 1).astype(np.float64)
    h = store(np.maximum(bn(conv3(opa(x), opw(T("stem.conv.w")).reshape(F, -1), n), "stem.bn"), 0))
    for i in range(cfg.blocks):
        m = store(np.maximum(bn(conv3(opa(h), opw(T(f"block{i}.conv1.w")).reshape(F, -1), n), f"block{i}.bn1"), 0))
        o = bn(conv3(opa(m), opw(T(f"block{i}.conv2.w")).reshape(F, -1), n), f"block{i}.bn2")
        h = store(np.maximum(o + h, 0))
    pol = np.maximum(bn(h @ T("policy.conv.w").reshape(2, F).T, "policy.bn"), 0)
    flat = pol.transpose(0, 2, 1).reshape(len(h), 2 * A)
    logits = flat @ T("policy.fc.w").reshape(A + 1, 2 * A).T + T("policy.fc.b")
    val = np.maximum(bn(h @ T("value.conv.w").reshape(1, F).T, "value.bn"), 0)[:, :, 0]
    hid = np.maximum(val @ T("value.fc1.w").reshape(cfg.value_hidden, A).T + T("value.fc1.b"), 0)
    v = np.tanh(hid @ T("value.fc2.w").reshape(1, -1).T + T("value.fc2.b"))[:, 0]
    return logits, v


def calibrated_network(cfg: O.NetConfig, seed: int, calib_seed: int = 99, calib_positions: int = 16):
    """A seeded network whose batch norms normalise what reaches them.

    Network(cfg, seed) with BASELINE.json's batch-norm distributions
    (make_network, KIND_BENCH), then, layer by layer in forward order, each
    batch norm's running mean and variance replaced by the float64 mean and
    variance (+1e-3) of its input over `calib_positions` positions
    (positions(cfg, calib_seed, ...)), as a trained network's running
    statistics describe its own activations. gamma and beta keep their
    random values. With 20 residual blocks the uncalibrated network's logits
    span +-1e4 and its values saturate at +-1; calibrated, logits stay within
    a few units, values spread over (-1, 1) and the best moves are nearly
    tied, so precision gates on it can fail. Returns (params, buffers)."""
    params, buffers = O.make_network(cfg, seed, O.KIND_BENCH)
    offs = {n: (s, o) for n, s, o in O.layout(cfg, 0)}
    boffs = {n: (s, o) for n, s, o in O.layout(cfg, 1)}

    def T(name):
        s, o = offs[name] if name in offs else boffs[name]
        return (params if name in offs else buffers)[o:o + s].astype(np.float64)

    def fit(pre, z):
        flat = z.reshape(-1, z.shape[-1])
        for stat, v in (("runMean", flat.mean(0)), ("runVar", flat.var(0) + 1e-3)):
            s, o = boffs[f"{pre}.{stat}"]
            buffers[o:o + s] = v.astype(np.float32)
        sc = T(pre + ".gamma") / np.sqrt(T(pre + ".runVar") + np.float64(np.float32(1e-5)))
        return (z - T(pre + ".runMean")) * sc + T(pre + ".beta")

    n, F = cfg.board, cfg.filters
    x = positions_f64(cfg, calib_seed, calib_positions)
    h = np.maximum(fit("stem.bn", conv3(x, T("stem.conv.w").reshape(F, -1), n)), 0)
    for i in range(cfg.blocks):
        m = np.maximum(fit(f"block{i}.bn1", conv3(h, T(f"block{i}.conv1.w").reshape(F, -1), n)), 0)
        h = np.maximum(fit(f"block{i}.bn2", conv3(m, T(f"block{i}.conv2.w").reshape(F, -1), n)) + h, 0)
    fit("policy.bn", h @ T("policy.conv.w").reshape(2, F).T)
    fit("value.bn", h @ T("value.conv.w").reshape(1, F).T)
    if cfg.ownership:
        fit("ownership.bn", h @ T("ownership.conv.w").reshape(1, F).T)
    return params, buffers


def positions_f64(cfg: O.NetConfig, seed: int, B: int) -> np.ndarray:
    """positions(cfg, seed, B) as float64 [B][A][planes] (channels last)."""
    return O.positions(cfg, seed, B).transpose(0, 2, 1).astype(np.float64)


def gates(logits, values, ref_logits, ref_values) -> dict:
    pr, pm = O.softmax(ref_logits), O.softmax(logits)
    return {
        "maxErr_logits": O.max_err(logits, ref_logits),
        "max_dv": float(np.max(np.abs(values - ref_values))),
        "max_dp": float(np.max(np.abs(pr - pm))),
        "top1": float(np.mean(np.argmax(ref_logits, 1) == np.argmax(logits, 1))),
    }


CONFIGS = {
    "C1": (O.NetConfig(5, 1, 4, 32, 64), 64),
    "C2": (O.NetConfig(9, 1, 6, 64, 128), 256),
    "C3": (O.NetConfig(19, 1, 10, 128, 256), 16),
    "C4": (O.NetConfig(19, 1, 20, 256, 256), 4),
}


if __name__ == "__main__":
    for name in sys.argv[1:] or ["C1", "C2"]:
        cfg, B = CONFIGS[name]
        p, b = O.make_network(cfg, 1, O.KIND_BENCH)
        x = O.positions(cfg, 1, B)
        ref = forward(cfg, p, b, x, "f64")
        for mode in ("tf32", "bf16"):
            g = gates(*forward(cfg, p, b, x, mode), *ref)
            print(name, mode, " ".join(f"{k} {v:.3g}" for k, v in g.items()))
