"""The fused small-board tower (alphazero-go_b200/csrc/tower_fused.cu): the
whole residual tower of boards up to 10x10 with 32 or 64 channels in one
launch, activations resident in shared memory.

It runs the per-layer kernels' arithmetic in the same order, so its outputs
must equal theirs bit for bit (logits, values, ownership) in every
precision, for batches that fill whole CTA groups and ones that leave the
last group partial, and for batches larger than one group per SM (each CTA
then takes several groups). Parity with the reference forward follows (the
per-layer path's gates); it is also checked directly here.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(engine, c, params, buffers, x, precision, fused):
    engine.cuda_probe.set_tower_fused(-1 if fused else 0)
    try:
        with engine.CudaInference(engine.NetDesc.of(c), params, buffers, x.shape[0], 0, precision) as net:
            return net.infer(x)
    finally:
        engine.cuda_probe.set_tower_fused(-1)


@pytest.mark.parametrize("precision", ["bf16", "tf32x3", "tf32"])
@pytest.mark.parametrize("shape,B", [((5, 4, 32, 1, False), 7), ((9, 6, 64, 1, False), 64), ((9, 2, 16, 8, True), 5),
                                     ((7, 3, 64, 2, True), 33), ((9, 1, 64, 1, False), 400), ((5, 2, 48, 1, False), 1),
                                     ((10, 2, 64, 1, True), 13)])
def test_fused_tower_equals_per_layer(engine, oracle, precision, shape, B):
    O = oracle
    n, blocks, filters, history, own = shape
    c = O.NetConfig(n, history, blocks, filters, 64, own)
    params, buffers = O.make_network(c, 71, O.KIND_TEST)
    x = O.random_planes(c, 72, B)
    prec = engine.PRECISIONS[precision]
    fused = _run(engine, c, params, buffers, x, prec, True)
    layered = _run(engine, c, params, buffers, x, prec, False)
    for k in range(3):
        if fused[k] is not None:
            assert np.array_equal(fused[k], layered[k]), (precision, shape, B, k)
    if precision == "tf32x3":
        lr, vr, orf = O.forward(c, params, buffers, x, threads=8)
        assert O.max_err(fused[0], lr) <= 1e-4
        assert np.max(np.abs(fused[1] - vr)) <= 1e-4
        if own:
            assert np.max(np.abs(fused[2] - orf)) <= 1e-4


def test_fused_tower_batch_independent(engine, oracle):
    """A board's outputs are the same bits alone and at any slot of a batch
    (its CTA group's other boards do not reach it)."""
    O = oracle
    c = O.NetConfig(5, 1, 3, 32, 32, True)
    params, buffers = O.make_network(c, 73, O.KIND_TEST)
    pool = O.random_planes(c, 74, 50)
    with engine.CudaInference(engine.NetDesc.of(c), params, buffers, 50, 0, engine.TF32X3) as net:
        whole = net.infer(pool)
        for s in (0, 1, 2, 3, 49):
            alone = net.infer(pool[s:s + 1])
            for k in range(3):
                assert np.array_equal(whole[k][s], alone[k][0]), (s, k)


@pytest.mark.parametrize("shape,B", [((9, 6, 64, 1, False), 1), ((9, 6, 64, 1, False), 2), ((9, 6, 64, 1, False), 3),
                                     ((9, 2, 64, 1, False), 301), ((7, 3, 64, 2, True), 5), ((5, 2, 64, 1, False), 20),
                                     ((10, 2, 64, 8, True), 9)])
def test_fused_pairs_equal_one_group(engine, oracle, shape, B):
    """The split mode at 64 channels runs two groups of boards per CTA: the
    same bits as one group per CTA, for odd and even group counts, several
    pairs per CTA, the stem in the launch or not (history 8)."""
    O = oracle
    n, blocks, filters, history, own = shape
    c = O.NetConfig(n, history, blocks, filters, 64, own)
    params, buffers = O.make_network(c, 75, O.KIND_TEST)
    x = O.random_planes(c, 76, B)
    outs = []
    for mode in (1, 2):
        engine.cuda_probe.set_tower_fused(mode)
        try:
            with engine.CudaInference(engine.NetDesc.of(c), params, buffers, B, 0, engine.TF32X3) as net:
                outs.append(net.infer(x, probs=True))
        finally:
            engine.cuda_probe.set_tower_fused(-1)
    for k in range(len(outs[0])):
        if outs[0][k] is not None:
            assert np.array_equal(outs[0][k], outs[1][k]), (shape, B, k)
