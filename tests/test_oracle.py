"""The CPU checker itself: pinned against the reference's own code and the
committed golden fixtures (no GPU)."""
import numpy as np
import pytest

from conftest import GOLDEN_DIR, load_oracle, load_pkg

import sys
sys.path.insert(0, str(GOLDEN_DIR))
from cases import CASES, case_inputs, sha256_of  # noqa: E402

oracle = load_oracle()


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("name", sorted(CASES))
def test_golden_fixture(name, orc):
    """Oracle reproduces every committed fixture bit for bit."""
    pkg = load_pkg()
    layer, x = case_inputs(pkg, name)
    g = np.load(GOLDEN_DIR / f"{name}.npz")
    assert str(g["sha256"]) == sha256_of(layer, x), "input generator changed"
    c = CASES[name]
    if "phi_y" in g:
        y, idx, w, logits = orc.moe_forward(x, layer, 2, oracle.POLICY_PHI)
        assert np.array_equal(bits(logits), bits(g["phi_logits"]))
        assert np.array_equal(idx, g["phi_idx"])
        assert np.array_equal(w, g["phi_w"])
        assert np.array_equal(bits(y), bits(g["phi_y"]))
    y, idx, w, logits = orc.moe_forward(x, layer, c["k"], oracle.POLICY_SOFTMAX)
    assert np.array_equal(idx, g["soft_idx"])
    assert np.array_equal(bits(w), bits(g["soft_w"]))
    assert np.array_equal(bits(y), bits(g["soft_y"]))


need_ref8 = pytest.mark.skipif(not oracle.Reference.available(8),
                               reason="reference not compiled here (no reference tree)")


@need_ref8
def test_matmul_matches_reference(orc):
    """k-ascending FMA chain == tensor_ops::matmul_transposed (src/tensor.cu:136-148)."""
    ref = oracle.Reference(8)
    g = np.random.default_rng(5)
    for (m, k, n) in [(1, 7, 3), (17, 512, 8), (33, 1000, 13)]:
        a = g.standard_normal((m, k), dtype=np.float32)
        b = g.standard_normal((n, k), dtype=np.float32)
        c_ref = ref.matmul_transposed(a, b)
        c = orc.router_logits(a, b)
        assert np.array_equal(bits(c), bits(c_ref))


@need_ref8
@pytest.mark.parametrize("T", [1, 5, 64])
def test_phi_layer_matches_reference(T, tmp_path, orc):
    """Full PhiMoE::forward (src/layer.cu:80-103) vs the restatement."""
    pkg = load_pkg()
    layer = pkg.synthetic_layer(11, 128, 200, 8)
    x = pkg.synthetic_tokens(11, T, 128)
    pkg.write_model_bin(tmp_path / "m.bin", [layer])
    ref = oracle.Reference(8).load(str(tmp_path / "m.bin"))
    r_logits, r_idx, r_w = ref.route(x)
    r_y = ref.forward(x)
    ref.close()
    y, idx, w, logits = orc.moe_forward(x, layer, 2, oracle.POLICY_PHI)
    assert np.array_equal(bits(logits), bits(r_logits))
    assert np.array_equal(idx, r_idx)
    assert np.array_equal(bits(y), bits(r_y))


@need_ref8
def test_phi_route_ties_and_quantum_edges():
    """Hand-built logits at the reference router's edges: exact ties, the tie
    margin, quantum boundaries, negative scores, all-equal rows."""
    ref = oracle.Reference(8)
    rows = np.array([
        [0.1, 0.1, 0.1, 0.1, 0.1, 0.1, 0.1, 0.1],          # all tied -> 0, 1
        [0.0, 0.019, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0],         # inside tie-eps
        [0.0, 0.021, 0.0, 0.0, 0.0, 0.0, 0.0, 0.05],        # beats the margin
        [-1.0, -0.5, -0.25, -2.0, -0.2496, -3, -4, -5],     # negatives, quantum rounding
        [0.0005, 0.0004999, 0.0, 0.0015, 0.0025, 0, 0, 0],  # half-quantum boundaries
        [np.nan, 1.0, 2.0, 0, 0, 0, 0, 0],
    ], np.float32)
    # Route through the reference on logits = x . gate^T with gate = identity rows.
    import tempfile, os
    pkg = load_pkg()
    layer = pkg.synthetic_layer(1, 8, 8, 8)
    layer.wg = np.eye(8, dtype=np.float32)
    with tempfile.TemporaryDirectory() as td:
        p = os.path.join(td, "m.bin")
        pkg.write_model_bin(p, [layer])
        r = oracle.Reference(8).load(p)
        r_logits, r_idx, r_w = r.route(rows)
        r.close()
    # The identity gate passes finite rows through unchanged (a NaN input
    # makes the whole logit row NaN, as in the reference's matmul).
    assert np.array_equal(bits(r_logits[:5]), bits(rows[:5]))
    assert np.isnan(r_logits[5]).all()
    idx, w = oracle.Oracle().route(r_logits, 2, oracle.POLICY_PHI)
    assert np.array_equal(idx, r_idx)
    assert np.array_equal(w, r_w)
    assert list(idx[0]) == [0, 1]
    # NaN inside a row: compares false, so an earlier best is never replaced.
    idx, _ = oracle.Oracle().route(np.array([[np.nan, 1, 2, 0, 0, 0, 0, 0]], np.float32), 2,
                                   oracle.POLICY_PHI)
    assert list(idx[0]) == [0, 2]


def test_softmax_route_semantics(orc):
    rows = np.array([
        [1.0, 3.0, 3.0, 2.0],          # exact tie -> lower index first
        [np.nan, 0.0, -1.0, 0.0],      # NaN ranks last; tie 1 vs 3 -> 1
        [-np.inf, -np.inf, 5.0, -np.inf],
    ], np.float32)
    idx, w = orc.route(rows, 2, oracle.POLICY_SOFTMAX)
    assert list(idx[0]) == [1, 2] and w[0][0] == w[0][1] == np.float32(0.5)
    assert list(idx[1]) == [1, 3]
    assert idx[2][0] == 2 and w[2][0] == 1.0 and w[2][1] == 0.0
    # Weights are the renormalised softmax of the chosen logits.
    g = np.random.default_rng(0).standard_normal((50, 16)).astype(np.float32)
    idx, w = orc.route(g, 4, oracle.POLICY_SOFTMAX)
    top = np.argsort(-g, axis=1, kind="stable")[:, :4]
    assert np.array_equal(idx, top)
    e = np.exp(np.take_along_axis(g, top, 1).astype(np.float64) - g.max(1, keepdims=True))
    assert np.allclose(w, e / e.sum(1, keepdims=True), rtol=1e-6)


def test_sampled_rows_match_full(orc):
    pkg = load_pkg()
    layer = pkg.synthetic_layer(4, 64, 96, 8)
    x = pkg.synthetic_tokens(4, 30, 64)
    y_full, *_ = orc.moe_forward(x, layer, 2, oracle.POLICY_SOFTMAX)
    sample = [0, 7, 29]
    y_s, *_ = orc.moe_forward(x, layer, 2, oracle.POLICY_SOFTMAX, sample=sample)
    assert np.array_equal(bits(y_s[sample]), bits(y_full[sample]))


def test_empty_input(orc):
    pkg = load_pkg()
    layer = pkg.synthetic_layer(4, 64, 96, 8)
    x = np.zeros((0, 64), np.float32)
    y, idx, w, logits = orc.moe_forward(x, layer, 2, oracle.POLICY_PHI)
    assert y.shape == (0, 64)


@need_ref8
def test_layer_norm_matches_reference(orc):
    """tensor_ops::layer_norm (src/tensor.cu:174-189), bit for bit."""
    ref = oracle.Reference(8)
    g = np.random.default_rng(9)
    for (T, d) in [(1, 64), (7, 512), (33, 4096)]:
        x = (g.standard_normal((T, d)) * 3 + 0.5).astype(np.float32)
        w = g.standard_normal(d).astype(np.float32)
        b = g.standard_normal(d).astype(np.float32)
        assert np.array_equal(bits(orc.layer_norm(x, w, b, 1e-5)), bits(ref.layer_norm(x, w, b, 1e-5)))


@pytest.mark.parametrize("name", [n for n in sorted(CASES)
                                  if "block_phi_y" in np.load(GOLDEN_DIR / f"{n}.npz")])
def test_block_fixture(name, orc):
    """The decoder layer's MoE half (src/layer.cu:157-161) from the reference,
    committed as a fixture: the restatement reproduces the normalised rows,
    the expert indices and y bit for bit."""
    pkg = load_pkg()
    layer, x = case_inputs(pkg, name)
    g = np.load(GOLDEN_DIR / f"{name}.npz")
    y, idx, post = orc.block_forward(x, layer, 2, oracle.POLICY_PHI, g["block_norm_w"],
                                     g["block_norm_b"], 1e-5)
    assert np.array_equal(bits(post), bits(g["block_post"]))
    assert np.array_equal(idx, g["block_phi_idx"])
    assert np.array_equal(bits(y), bits(g["block_phi_y"]))
