"""The decoder layer's MoE half on the GPU: y = attn + MoE(layer_norm(attn))
(PhiDecoderLayer::forward, src/layer.cu:157-161).

* moe_layer_norm_device is bit-exact with tensor_ops::layer_norm
  (src/tensor.cu:174-189): against the restatement, which is pinned to the
  reference's compiled function, and against the reference's own output in
  the golden fixtures.
* The fused block (norm applied inside the router and the dispatch permute,
  residual added after the combine) routes exactly like the reference on the
  normalised rows -- every (token, expert) pair, read back through the
  dispatch layout -- and its output is within the precision's rel-L2 bound.
* Fusing changes nothing: the block equals layer_norm_device -> forward_device
  -> + attn, bit for bit.
"""
import sys

import numpy as np
import pytest

from conftest import GOLDEN_DIR, load_oracle, load_pkg, ref_elementwise_failures, rel_l2

sys.path.insert(0, str(GOLDEN_DIR))
from cases import CASES, case_inputs  # noqa: E402

pytestmark = pytest.mark.gpu
oracle = load_oracle()
TOL = {0: 1e-3, 1: 2e-2, 2: 1e-3}   # precision -> rel-L2 bound
EPS = 1e-5                 # NORM_EPS, include/config.h:19


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def ln_on_gpu(pkg, x, w, b, eps=EPS, inplace=False):
    import torch
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    wd = torch.from_numpy(w).cuda()
    bd = torch.from_numpy(b).cuda()
    yd = xd if inplace else torch.full_like(xd, float("nan"))
    pkg.layer_norm_device(xd.data_ptr(), wd.data_ptr(), bd.data_ptr(), eps, x.shape[0],
                          x.shape[1], yd.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return yd.cpu().numpy()


def assert_same_routing(m, idx_ref, E):
    """Every expert's packed rows hold exactly the tokens that chose it."""
    counts = m.expert_counts()
    assert np.array_equal(counts, np.bincount(idx_ref.ravel(), minlength=E))
    tok, _, eoff = m.dispatch_layout(rows_cap=int(counts.sum()) + 128 * (E + 1))
    for e in range(E):
        valid = tok[eoff[e]:eoff[e] + counts[e]]
        assert np.array_equal(valid, np.nonzero((idx_ref == e).any(1))[0]), f"expert {e}"


@pytest.mark.parametrize("T,d,scale,offset", [
    (1, 128, 1.0, 0.0), (7, 384, 3.0, 0.5), (33, 512, 1.0, 0.0), (300, 4096, 2.0, -1.0),
    (5, 4096, 100.0, 1000.0),      # large common offset: the variance cancels heavily
])
def test_layer_norm_device_bit_exact(T, d, scale, offset, orc):
    g = np.random.default_rng(T * 7 + d)
    x = (g.standard_normal((T, d)) * scale + offset).astype(np.float32)
    w = g.standard_normal(d).astype(np.float32)
    b = g.standard_normal(d).astype(np.float32)
    pkg = load_pkg()
    y = ln_on_gpu(pkg, x, w, b)
    assert np.array_equal(bits(y), bits(orc.layer_norm(x, w, b, EPS)))
    assert np.array_equal(bits(ln_on_gpu(pkg, x, w, b, inplace=True)), bits(y))


def test_layer_norm_device_edge_rows(orc):
    """A constant row (variance 0: inv = 1/sqrt(eps)), a row of zeros, and a
    row holding a NaN, which makes its whole output NaN on both sides."""
    d = 256
    g = np.random.default_rng(5)
    x = g.standard_normal((4, d)).astype(np.float32)
    x[0] = 3.25
    x[1] = 0.0
    x[2, 17] = np.nan
    w = g.standard_normal(d).astype(np.float32)
    b = g.standard_normal(d).astype(np.float32)
    y = ln_on_gpu(load_pkg(), x, w, b)
    ref = orc.layer_norm(x, w, b, EPS)
    assert np.isnan(y[2]).all() and np.isnan(ref[2]).all()
    keep = [0, 1, 3]
    assert np.array_equal(bits(y[keep]), bits(ref[keep]))


def test_layer_norm_device_rejects_bad_shapes():
    pkg = load_pkg()
    with pytest.raises(pkg.MoeError):
        pkg.layer_norm_device(16, 16, 16, EPS, 4, 100, 16)   # cols not a multiple of 128


BLOCK_CASES = [n for n in sorted(CASES) if "block_phi_y" in np.load(GOLDEN_DIR / f"{n}.npz")]


@pytest.mark.parametrize("name", BLOCK_CASES)
def test_layer_norm_device_matches_reference_fixture(name):
    pkg = load_pkg()
    _, x = case_inputs(pkg, name)
    g = np.load(GOLDEN_DIR / f"{name}.npz")
    y = ln_on_gpu(pkg, x, g["block_norm_w"], g["block_norm_b"])
    assert np.array_equal(bits(y), bits(g["block_post"]))


GEMMS = pytest.mark.parametrize("gemm", [2, 1], ids=["ctapair", "single"])


@GEMMS
@pytest.mark.parametrize("precision", [0, 1, 2], ids=["fp32", "bf16", "bf16x3"])
@pytest.mark.parametrize("name", BLOCK_CASES)
def test_block_forward_matches_reference_fixture(name, precision, gemm):
    """PHI router (the reference's own): routing bit-exact, y within bound."""
    pkg = load_pkg()
    layer, x = case_inputs(pkg, name)
    g = np.load(GOLDEN_DIR / f"{name}.npz")
    layer.norm_weight, layer.norm_bias = g["block_norm_w"], g["block_norm_b"]
    with pkg.MoeLayer(layer, top_k=2, policy=0, precision=precision, gemm_variant=gemm) as m:
        y = m.block_forward_host(x)
        assert_same_routing(m, g["block_phi_idx"], layer.E)
        y2 = m.block_forward_host(x)
    assert rel_l2(y, g["block_phi_y"]) <= TOL[precision]
    if precision != 1:
        assert ref_elementwise_failures(y, g["block_phi_y"]) == 0
    assert np.array_equal(bits(y), bits(y2)), "top-2 block forward is not deterministic"


@pytest.mark.parametrize("precision", [0, 1, 2], ids=["fp32", "bf16", "bf16x3"])
@pytest.mark.parametrize("T", [1, 5, 16, 33, 300])
def test_block_forward_decode_and_prefill_match_oracle(T, precision, orc):
    """Both paths: small T runs the decode kernels (norm applied in the row
    packing; T <= 14 in FP32, T = 1 in BF16), larger T the grouped GEMMs."""
    pkg = load_pkg()
    layer = pkg.synthetic_layer(41, 512, 448, 8)
    layer.norm_weight, layer.norm_bias = pkg.synthetic_post_norm(41, 512)
    attn = (pkg.synthetic_tokens(41, T, 512) * 2.0 + 0.25).astype(np.float32)
    y_ref, idx_ref, _ = orc.block_forward(attn, layer, 2, oracle.POLICY_SOFTMAX,
                                          layer.norm_weight, layer.norm_bias, EPS)
    with pkg.MoeLayer(layer, top_k=2, policy=1, precision=precision) as m:
        y = m.block_forward_host(attn)
        assert_same_routing(m, idx_ref, 8)
    assert rel_l2(y, y_ref) <= TOL[precision]


@pytest.mark.parametrize("precision", [0, 1, 2], ids=["fp32", "bf16", "bf16x3"])
@pytest.mark.parametrize("T", [1, 3, 4, 33, 300])
def test_rms_block_forward_matches_oracle(T, precision, orc):
    """y = x + MoE(rms_norm(x)) (moe_set_post_rms_norm, the decoder's MoE
    block): up to 4 tokens the small-batch router computes the RMS
    statistics itself, larger batches take them from rms_stats_kernel.
    Against the oracle MoE on the float64 RMS-normalised rows (as fp32)."""
    pkg = load_pkg()
    d = 512
    layer = pkg.synthetic_layer(43, d, 448, 8)
    w = (1.0 + 0.1 * np.random.default_rng(43).standard_normal(d)).astype(np.float32)
    x = (pkg.synthetic_tokens(43, T, d) * 1.5 + 0.1).astype(np.float32)
    x64 = x.astype(np.float64)
    inv = 1.0 / np.sqrt((x64 * x64).mean(axis=1, keepdims=True) + EPS)
    xn = (x64 * inv * w.astype(np.float64)).astype(np.float32)
    y_moe, _, _, _ = orc.moe_forward(xn, layer, 2, oracle.POLICY_SOFTMAX)
    y_ref = y_moe.astype(np.float64) + x64
    with pkg.MoeLayer(layer, top_k=2, policy=1, precision=precision,
                      decode_max_tokens=64) as m:
        m.set_post_rms_norm(w, EPS)
        y = m.block_forward_host(x)
        y2 = m.block_forward_host(x)
    assert rel_l2(y, y_ref) <= TOL[precision], rel_l2(y, y_ref)
    assert np.array_equal(bits(y), bits(y2))


@pytest.mark.parametrize("precision", [0, 1, 2], ids=["fp32", "bf16", "bf16x3"])
@pytest.mark.parametrize("T", [3, 200])
def test_fused_block_equals_unfused_composition(T, precision):
    """layer_norm_device -> forward_device -> + attn (torch) gives the same
    bits as the fused block: the router and permute see identical values."""
    import torch
    pkg = load_pkg()
    d = 256
    layer = pkg.synthetic_layer(42, d, 320, 8)
    nw, nb = pkg.synthetic_post_norm(42, d)
    attn = pkg.synthetic_tokens(42, T, d)
    s = torch.cuda.current_stream().cuda_stream
    with pkg.MoeLayer(layer, top_k=2, policy=1, precision=precision) as m:
        m.set_post_norm(nw, nb)
        ad = torch.from_numpy(attn).cuda()
        yf = torch.empty_like(ad)
        m.block_forward_device(ad.data_ptr(), yf.data_ptr(), T, s)
        post = torch.empty_like(ad)
        wd, bd = torch.from_numpy(nw).cuda(), torch.from_numpy(nb).cuda()
        pkg.layer_norm_device(ad.data_ptr(), wd.data_ptr(), bd.data_ptr(), EPS, T, d,
                              post.data_ptr(), s)
        ff = torch.empty_like(ad)
        m.forward_device(post.data_ptr(), ff.data_ptr(), T, s)
        torch.cuda.synchronize()
        yu = (ff + ad).cpu().numpy()
    assert np.array_equal(bits(yf.cpu().numpy()), bits(yu))


@pytest.mark.parametrize("precision", [0, 1, 2], ids=["fp32", "bf16", "bf16x3"])
def test_block_pipelined_host_matches_device(precision):
    import torch
    pkg = load_pkg()
    layer = pkg.synthetic_layer(43, 256, 384, 8)
    layer.norm_weight, layer.norm_bias = pkg.synthetic_post_norm(43, 256)
    attn = pkg.synthetic_tokens(43, 6144, 256)
    with pkg.MoeLayer(layer, top_k=2, policy=1, precision=precision) as m:
        y_host = m.block_forward_host(attn)
        ad = torch.from_numpy(attn).cuda()
        yd = torch.empty_like(ad)
        m.block_forward_device(ad.data_ptr(), yd.data_ptr(), attn.shape[0], 0)
        torch.cuda.synchronize()
    assert np.array_equal(bits(y_host), bits(yd.cpu().numpy()))


def test_model_bin_attaches_post_norm(tmp_path):
    pkg = load_pkg()
    layer, x = case_inputs(pkg, "phi16")
    plain = tmp_path / "plain.bin"
    pkg.write_model_bin(plain, [layer])
    layer.norm_weight, layer.norm_bias = pkg.synthetic_post_norm(7, layer.d)
    normed = tmp_path / "normed.bin"
    pkg.write_model_bin(normed, [layer])
    with pkg.MoeLayer(layer, top_k=2, policy=0) as a, \
            pkg.MoeLayer(model_bin=str(normed), top_k=2, policy=0) as b, \
            pkg.MoeLayer(model_bin=str(plain), top_k=2, policy=0) as c:
        assert np.array_equal(bits(a.block_forward_host(x)), bits(b.block_forward_host(x)))
        with pytest.raises(pkg.MoeError):
            c.block_forward_host(x)
