"""Pins the C oracle to the reference's own op known-answer tests.

Each test restates one test of laya-rust ``tests/ops.rs`` (line numbers in the
docstrings) with the same inputs, expected values and tolerance rule
``|got - want| <= tol * (1 + |want|)`` (tests/ops.rs:7-9).
"""
import math

import numpy as np
import pytest

from oracle import oracle as O

NEG_BIG = np.float32(-3.4e38)


def assert_close(got, want, tol, what):
    got = np.asarray(got, dtype=np.float32).ravel()
    want = np.asarray(want, dtype=np.float32).ravel()
    assert got.size == want.size, f"{what}: length"
    for i, (g, w) in enumerate(zip(got, want)):
        assert abs(float(g) - float(w)) <= tol * (1.0 + abs(float(w))), f"{what}[{i}]: got {g} want {w}"


def test_layernorm_z_scores_rows():
    """tests/ops.rs:42-49"""
    y = O.layernorm(np.array([[1.0, -1.0], [0.5, -0.5]]), np.array([1.0, 1.0]), None, 1e-5)
    assert y.shape == (2, 2)
    assert_close(y, [1.0, -1.0, 1.0, -1.0], 1e-4, "layernorm")


def test_layernorm_applies_weight_and_bias():
    """tests/ops.rs:51-58"""
    y = O.layernorm(np.array([[2.0, 2.0]]), np.array([3.0, 5.0]), np.array([1.0, -1.0]), 1e-5)
    assert_close(y, [1.0, -1.0], 1e-4, "layernorm+bias")


def test_matmul_and_matmul_t_agree_on_the_same_matrix():
    """tests/ops.rs:60-78"""
    x = np.array([[1.0, 2.0], [3.0, 4.0]])
    wdata = np.array([1.0, 0.0, 1.0, 2.0, 0.0, 1.0, 3.0, 4.0])
    a = O.matmul(x, wdata.reshape(2, 4))
    assert a.shape == (2, 4)
    assert_close(a.ravel()[0:2], [1.0, 2.0], 1e-5, "matmul identity")
    assert_close(a.ravel()[4:6], [3.0, 4.0], 1e-5, "matmul identity")
    wt = np.zeros(8)
    for i in range(2):
        for o in range(4):
            wt[o * 2 + i] = wdata[i * 4 + o]
    b = O.matmul_t(x, wt.reshape(4, 2))
    assert_close(a, b, 1e-5, "mm vs mm_t")


def test_gelu_matches_reference_points():
    """tests/ops.rs:80-90"""
    y = O.gelu(np.array([[-1.0, 0.0, 1.0, 2.0]]))
    assert_close(y, [-0.158655, 0.0, 0.841345, 1.954500], 1e-4, "gelu")


def test_relu_clamps_negatives():
    """tests/ops.rs:92-97"""
    y = O.relu(np.array([[-2.0, -0.0, 0.5, 3.0]]))
    assert_close(y, [0.0, 0.0, 0.5, 3.0], 1e-6, "relu")


def test_gelu_mul_gates_the_first_half_with_the_second():
    """tests/ops.rs:99-106"""
    y = O.gelu_mul(np.array([[1.0, 0.0, 2.0, -3.0]]), 2)
    assert y.shape == (1, 2)
    g = O.gelu(np.array([[1.0, 0.0]])).ravel()
    assert_close(y, [g[0] * 2.0, g[1] * -3.0], 1e-5, "gelu_mul")


def test_split_qkv_without_rope_scales_qk_not_v():
    """tests/ops.rs:108-120"""
    qkv = np.array([[1.0, 2.0, 3.0, 4.0, 5.0, 6.0]])
    q, k, v = O.split_qkv_rope(qkv, None, 1.0, 1, 2, 1)
    assert q.shape == (1, 1, 1, 2)
    assert_close(q, [1.0, 2.0], 1e-6, "q")
    assert_close(k, [3.0, 4.0], 1e-6, "k")
    assert_close(v, [5.0, 6.0], 1e-6, "v")
    q2, k2, _ = O.split_qkv_rope(qkv, None, 0.5, 1, 2, 1)
    assert_close(q2, [0.5, 1.0], 1e-6, "scaled q")
    assert_close(k2, [1.5, 2.0], 1e-6, "scaled k")


def test_split_qkv_rope_uses_the_rotate_half_pairing():
    """tests/ops.rs:122-134"""
    qkv = np.arange(1.0, 13.0).reshape(1, 12)
    cos = np.array([[0.0, 1.0]])
    sin = np.array([[1.0, 0.0]])
    q, k, v = O.split_qkv_rope(qkv, (cos, sin), 1.0, 1, 4, 1)
    assert_close(q, [-3.0, 2.0, 1.0, 4.0], 1e-6, "rope q")
    assert_close(k, [-7.0, 6.0, 5.0, 8.0], 1e-6, "rope k")
    assert_close(v, [9.0, 10.0, 11.0, 12.0], 1e-6, "rope v")


def test_attention_is_softmax_qk_over_v():
    """tests/ops.rs:136-147"""
    eye = np.array([1.0, 0.0, 0.0, 1.0]).reshape(1, 1, 2, 2)
    out = O.attention(eye, eye, eye, np.zeros((1, 2, 2)), 1, 2)
    assert out.shape == (2, 2), "heads_to_seq layout"
    e = math.e
    p = e / (e + 1.0)
    assert_close(out, [p, 1.0 - p, 1.0 - p, p], 1e-5, "attention")


def test_attention_mask_drops_keys():
    """tests/ops.rs:149-158"""
    eye = np.array([1.0, 0.0, 0.0, 1.0]).reshape(1, 1, 2, 2)
    mask = np.array([0.0, NEG_BIG, 0.0, 0.0], dtype=np.float32).reshape(1, 2, 2)
    out = O.attention(eye, eye, eye, mask, 1, 2)
    e = math.e
    p = e / (e + 1.0)
    assert_close(out, [1.0, 0.0, 1.0 - p, p], 1e-5, "masked attention")


@pytest.mark.parametrize("r,kk,n", [(1, 1, 1), (3, 5, 7), (4, 64, 8), (9, 33, 517), (40, 1024, 3072),
                                    (66, 2624, 1024)])
def test_tiled_matmul_is_bitwise_the_reference_traversal(r, kk, n):
    """The register-tiled gemm_nt of LAYA_ORACLE_FAST performs the same
    multiplies and adds in the same order per element as cpu/mod.rs:80-101."""
    rng = np.random.default_rng(r * 7 + n)
    x = rng.standard_normal((r, kk)).astype(np.float32)
    w = rng.standard_normal((kk, n)).astype(np.float32)
    assert O.matmul_order(x, w, tiled=False).tobytes() == O.matmul_order(x, w, tiled=True).tobytes()


def test_threaded_attention_is_bitwise_the_single_threaded_one(monkeypatch):
    """LAYA_ORACLE_FAST splits the attention's (sequence, head) pairs over
    threads; every output element runs the same code, so nothing changes."""
    rng = np.random.default_rng(5)
    n, nh, length, hd = 3, 4, 37, 8
    q, k, v = (rng.standard_normal((n, nh, length, hd)).astype(np.float32) for _ in range(3))
    att = np.ones((n, length), np.int64)
    att[1, 30:] = 0
    mask = O.window_mask(att, n, length, 5)
    outs = []
    for flag in ("0", "1"):
        monkeypatch.setenv("LAYA_ORACLE_FAST", flag)
        outs.append(O.attention(q, k, v, mask, nh, length))
    assert outs[0].tobytes() == outs[1].tobytes()


def test_window_mask_marks_padding_and_distant_keys():
    """tests/ops.rs:160-180 (exact -3.4e38)"""
    m = O.window_mask([1, 1, 0, 1], 1, 4, None)
    assert m.shape == (1, 4, 4)
    d = m.ravel()
    for s in range(4):
        assert d[s * 4 + 2] == NEG_BIG
        for t in (0, 3):
            assert d[s * 4 + t] == 0.0
    d = O.window_mask([1, 1, 1, 1], 1, 4, 1).ravel()
    for s in range(4):
        for t in range(4):
            want = NEG_BIG if abs(s - t) > 1 else 0.0
            assert d[s * 4 + t] == want


def test_embedding_copies_rows():
    """tests/ops.rs:182-188"""
    out = O.embedding(np.arange(1.0, 7.0).reshape(3, 2), [2, 0])
    assert out.shape == (2, 2)
    assert_close(out, [5.0, 6.0, 1.0, 2.0], 1e-6, "embedding")


def test_add_bias_wraps_over_the_last_axis():
    """tests/ops.rs:190-201"""
    y = O.add_bias(np.arange(1.0, 7.0).reshape(3, 2), np.array([10.0, 20.0]))
    assert_close(y, [11.0, 22.0, 13.0, 24.0, 15.0, 26.0], 1e-6, "add_bias")


def test_add_type_uses_the_sequence_index():
    """tests/ops.rs:203-214"""
    y = O.add_type(np.zeros((4, 2)), np.array([[1.0, 1.0], [100.0, 100.0]]), [1, 0], 2)
    assert_close(y, [100.0, 100.0, 100.0, 100.0, 1.0, 1.0, 1.0, 1.0], 1e-6, "add_type")


def test_gather_markers_picks_the_right_rows():
    """tests/ops.rs:216-234"""
    data = []
    for b in range(2):
        for s in range(3):
            data += [b * 100 + s, b * 100 + s + 0.5]
    y = O.gather_markers(np.array(data).reshape(6, 2), [2, 0, 1, 1], 2)
    assert y.shape == (4, 2)
    assert_close(y, [2.0, 2.5, 0.0, 0.5, 101.0, 101.5, 101.0, 101.5], 1e-6, "gather_markers")


def test_act_input_concatenates_first_token_with_features():
    """tests/ops.rs:236-243"""
    y = O.act_input(np.arange(1.0, 9.0).reshape(4, 2), np.array([[0.25], [0.75]]), 2)
    assert y.shape == (2, 3)
    assert_close(y, [1.0, 2.0, 0.25, 5.0, 6.0, 0.75], 1e-6, "act_input")


def close(got, want, tol):
    return abs(got - want) <= tol * (1.0 + abs(want))


def test_post_masks_scores_and_derives_features():
    """tests/ops.rs:245-258"""
    logits, feats = O.post(np.array([1.0, 2.0, 3.0]), [1, 0, 1], 3)
    assert logits.shape == (3,)
    assert feats.shape == (1, 4)
    assert_close(logits, [1.0, -10000.0, 3.0], 1e-6, "masked logits")
    f = feats.ravel()
    assert close(f[0], 0.8808, 1e-3)
    assert close(f[1], 0.8808 - 0.1192, 1e-3)
    assert 0.0 < f[2] < 1.0
    assert close(f[3], 2.0 / 255.0, 1e-4)


def test_post_survives_a_single_visible_marker():
    """tests/ops.rs:260-267"""
    logits, feats = O.post(np.array([5.0, 1.0]), [1, 0], 2)
    f = feats.ravel()
    assert np.isfinite(f[0]) and np.isfinite(f[2])
    assert_close(logits[1:2], [-10000.0], 1e-6, "sentinel")


@pytest.mark.parametrize("v", [0.0, 1.0, -1.0, 0.5, 0.25, 1024.0, -0.0, 65504.0, 5.9604645e-8,
                               9.5367432e-7, -2.0, 0.33325195])
def test_f16_round_trip_is_exact_for_representable_values(v):
    """tests/gguf.rs:122-145 (oracle f2h/h2f, weights.rs:8-64)"""
    v = float(np.float32(v))
    assert O.h2f(O.f2h(v)) == v


def test_f16_known_answers():
    """tests/gguf.rs:141-144"""
    assert O.f2h(1e-5) == 0x00A8
    assert O.h2f(0x00A8) == float(np.float32(168.0 * 2.0 ** -24))
    assert O.f2h(float("inf")) & 0x7FFF == 0x7C00
    assert O.h2f(O.f2h(1234.5)) == 1234.0


def test_f16_rounds_within_half_an_ulp():
    """tests/gguf.rs:147-170"""
    for v in [1e-5, 0.35355338, 3.14159, -2.71828, 1234.5, 0.1005828, 1.636903]:
        v = float(np.float32(v))
        back = O.h2f(O.f2h(v))
        tol = max(abs(v) * 2.0 ** -11, 2.0 ** -25)
        assert abs(back - v) <= tol


def test_numpy_f16_conversion_matches_reference_f2h():
    """The generator rounds weights with numpy; it must equal weights.rs f2h."""
    rng = np.random.default_rng(7)
    vals = np.concatenate([rng.standard_normal(20000).astype(np.float32) * 0.02,
                           rng.standard_normal(2000).astype(np.float32) * 1e-6,
                           rng.standard_normal(2000).astype(np.float32) * 3e4,
                           np.array([2.0 ** -25, -2.0 ** -25, 3 * 2.0 ** -26, 65520.0, 65519.0],
                                    dtype=np.float32)])
    ref = np.array([O.f2h(float(v)) for v in vals], dtype=np.uint16)
    got = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(ref, got)


def test_rope_freq_matches_generator():
    """convert.rs:16-21 in the oracle equals the generator's table bit for bit."""
    from laya_rust_b200 import modelgen
    for theta in (160000.0, 10000.0):
        assert np.array_equal(O.rope_freq(theta).view(np.uint32),
                              modelgen.rope_table(theta).view(np.uint32))
