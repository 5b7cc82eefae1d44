"""GPU checks of the engine's context and its tensor-core path.

Modelled on the reference's tests/test_cuda.cpp context and kernel tests
(:227-262 availability, description and architecture; :264-290 gemm against
an exact reference): the tcgen05 MMA on row-shifted views of a staged halo
tile must give exactly the sums numpy computes, for every view a 3x3 conv
uses, since the inputs are small integers whose products and sums are exact.
"""
import re

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_available_and_description(engine):
    ok, why = engine.cuda_available(0)
    assert ok, why
    d = engine.cuda_description(0, engine.BF16)
    assert re.match(r"^.+ sm_100, driver API \d+\.\d+, runtime \d+\.\d+, kernels [0-9a-f]{8}, bf16$", d), d
    assert d == engine.cuda_description(0, engine.BF16)


def test_architecture_matches(engine):
    assert engine.cuda_probe.binary_version() == engine.cuda_probe.device_architecture() == 100


def test_fill(engine):
    for n in (0, 1, 1000, 1 << 20):
        tail = 37
        data = np.full(n + tail, -3.0, np.float32)
        engine.cuda_probe.fill(data, n, 2.5, tail)
        assert np.all(data[:n] == 2.5) and np.all(data[n:] == -3.0)


def test_bounded_wait_reports_instead_of_hanging(engine):
    """A wait nothing satisfies ends after its limit with an error status, and
    the context stays usable."""
    assert engine.cuda_probe.bounded_wait(20_000_000) == 5   # kErrProbeTimeout
    data = np.zeros(16, np.float32)
    engine.cuda_probe.fill(data, 16, 1.0)
    assert np.all(data == 1.0)


def _small_ints(rng, shape):
    return (rng.integers(-8, 9, size=shape) / 8.0).astype(np.float32)


@pytest.mark.parametrize("precision", ["bf16", "tf32"])
@pytest.mark.parametrize("n_out", [32, 64, 128, 256])
def test_umma_shifted_views_exact(engine, precision, n_out):
    prec = engine.PRECISIONS[precision]
    kc = 64 if precision == "bf16" else 32
    rng = np.random.default_rng(n_out)
    board = 19
    halo = 128 + 2 * (board + 2)
    k_chunks = 2
    a = _small_ints(rng, (halo, kc * k_chunks))
    w = _small_ints(rng, (n_out, 9 * kc * k_chunks))
    wt = np.concatenate([w[:, c * 9 * kc:(c * 9 + 1) * kc] for c in range(k_chunks)], axis=1)
    # every tap offset of a 3x3 conv on this board, plus an unaligned sweep
    shifts = sorted({board + 2 + dy * (board + 1) + dx for dy in (-1, 0, 1) for dx in (-1, 0, 1)} | {0, 1, 3, 7, 8})
    for s in shifts:
        d = engine.cuda_probe.umma(prec, n_out, halo, s, k_chunks, a, w)
        ref = a[s:s + 128].astype(np.float64) @ wt.T.astype(np.float64)
        np.testing.assert_array_equal(d, ref.astype(np.float32), err_msg=f"shift {s}")
