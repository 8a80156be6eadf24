"""The oracle's single-layer entry point (the CPU side of the one-layer
benchmark configuration) is the body of its whole-forward layer loop: fed the
enc.{i-1} tap (the embed tap for layer 0) it reproduces the enc.{i} tap bit
for bit, on a ragged request with padding rows."""
import numpy as np
import pytest

from laya_rust_b200 import modelgen


@pytest.fixture(scope="module")
def oracle():
    from oracle.oracle import OracleModel
    m = OracleModel(modelgen.cached_model(seed=0))
    yield m
    m.close()


def test_encoder_layer_reproduces_the_forward_taps(oracle):
    n, l, k = 2, 24, 2
    rng = np.random.default_rng(0)
    ids = rng.integers(0, 50280, (n, l))
    att = np.ones((n, l), np.int64)
    att[1, 20:] = 0
    ids[1, 20:] = 0
    mpos = np.array([[3, 5], [4, 6]])
    mmask = np.ones((n, k), np.int64)
    taps = {}
    oracle.forward(n, l, k, ids, att, mpos, mmask, np.array([0, 2]), taps=taps)
    for layer in (0, 1, 3, 27):
        y = oracle.encoder_layer(n, l, att, layer, taps[f"enc.{layer - 1}" if layer else "embed"])
        assert np.array_equal(y.ravel(), taps[f"enc.{layer}"]), layer


def test_encoder_layer_rejects_a_layer_out_of_range(oracle):
    for layer in (-1, 28):
        with pytest.raises(RuntimeError):
            oracle.encoder_layer(1, 4, np.ones(4, np.int64), layer, np.zeros((4, 1024), np.float32))
