"""kore_b200.qweights (GGUF Q4_K / Q6_K block layouts of the projection
weights), CPU only: sizes, validation and the synthetic generator."""
import numpy as np
import pytest

from kore_b200.qweights import BLOCK_BYTES, Q4_K, Q6_K, QMat, random_qmat
from oracle import oracle as O


def test_block_sizes_are_ggufs():
    assert BLOCK_BYTES == {Q4_K: 144, Q6_K: 210}


@pytest.mark.parametrize("qtype", [Q4_K, Q6_K])
def test_random_qmat_shape_determinism_and_finite_scales(qtype):
    a = random_qmat(qtype, 8, 512, np.random.default_rng(3))
    b = random_qmat(qtype, 8, 512, np.random.default_rng(3))
    assert a.nbytes == 8 * 2 * BLOCK_BYTES[qtype] == a.data.size
    assert np.array_equal(a.data, b.data)
    blocks = a.data.reshape(-1, BLOCK_BYTES[qtype])
    offs = (0, 2) if qtype == Q4_K else (208,)
    for o in offs:
        f = blocks[:, o:o + 2].copy().view(np.float16).astype(np.float32)
        assert np.isfinite(f).all() and (f >= 0).all()
    assert a.row(7).size == 2 * BLOCK_BYTES[qtype]


@pytest.mark.parametrize("qtype", [Q4_K, Q6_K])
def test_random_weights_give_products_of_the_requested_scale(qtype):
    rng = np.random.default_rng(4)
    m = random_qmat(qtype, 256, 3584, rng, sigma=0.02)
    x = rng.standard_normal(3584).astype(np.float32)
    y = O.qmatvec(m, x)
    # a row of N(0, sigma^2) weights against N(0, 1) inputs: std ~ sigma * sqrt(cols)
    assert 0.5 < float(np.std(y)) / (0.02 * np.sqrt(3584)) < 2.0


def test_qmat_validation():
    with pytest.raises(ValueError):
        QMat(13, 1, 256, np.zeros(144, np.uint8))          # not Q4_K / Q6_K
    with pytest.raises(ValueError):
        QMat(Q4_K, 1, 300, np.zeros(144, np.uint8))        # cols not a multiple of 256
    with pytest.raises(ValueError):
        QMat(Q6_K, 2, 256, np.zeros(210, np.uint8))        # one row's bytes for two rows
