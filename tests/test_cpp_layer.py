"""The C++ drop-in layer (include/tensor.h, model_loader.h, layer.h) used the
way the reference's code uses its own classes."""
import subprocess
import sys

import numpy as np
import pytest

from conftest import GOLDEN_DIR, PKG_DIR, ROOT, load_oracle, load_pkg, rel_l2

sys.path.insert(0, str(GOLDEN_DIR))
from cases import case_inputs  # noqa: E402


@pytest.fixture(scope="module")
def test_bin(tmp_path_factory):
    out = tmp_path_factory.mktemp("cpp") / "test_phimoe"
    lib = PKG_DIR / "libmoe_layer.so"
    if not lib.exists():
        pytest.fail("libmoe_layer.so not built")
    subprocess.run(["/usr/bin/g++", "-std=c++17", "-O1", "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "cpp" / "test_phimoe.cpp"), "-o", str(out),
                    f"-L{PKG_DIR}", "-lmoe_layer", "-lmoe_b200", f"-Wl,-rpath,{PKG_DIR}"],
                   check=True)
    return out


def test_errors_and_tensor_semantics(test_bin, tmp_path):
    r = subprocess.run([str(test_bin), "errors", str(tmp_path)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.gpu
def test_phimoe_forward_matches_reference(test_bin, tmp_path):
    pkg = load_pkg()
    oracle = load_oracle()
    layer, x = case_inputs(pkg, "c1")
    g = np.load(GOLDEN_DIR / "c1.npz")
    model = tmp_path / "m.bin"
    pkg.write_model_bin(model, [layer])
    xp = tmp_path / "x.bin"
    x.tofile(xp)
    T, d = x.shape
    r = subprocess.run([str(test_bin), "forward", str(model), str(xp), str(T), str(d),
                        str(tmp_path / "out")], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    y = np.fromfile(tmp_path / "out.moe.bin", np.float32).reshape(T, d)
    assert rel_l2(y, g["phi_y"]) <= 1e-3          # PhiMoE(loader, 0): the reference's router
    idx = np.fromfile(tmp_path / "out.route_idx.bin", np.int32).reshape(T, 2)
    w = np.fromfile(tmp_path / "out.route_w.bin", np.float32).reshape(T, 2)
    assert np.array_equal(idx, g["phi_idx"]) and np.array_equal(w, g["phi_w"])
    ym = np.fromfile(tmp_path / "out.mlp.bin", np.float32).reshape(T, d)
    ym_ref = oracle.Oracle().expert_ffn(x, layer.w1[0], layer.w3[0], layer.w2[0])
    assert rel_l2(ym, ym_ref) <= 1e-3             # PhiMLP::forward (src/layer.cu:32-45)


def _block_model(pkg, tmp_path, name="c1"):
    layer, x = case_inputs(pkg, name)
    g = np.load(GOLDEN_DIR / f"{name}.npz")
    layer.norm_weight, layer.norm_bias = g["block_norm_w"], g["block_norm_b"]
    model = tmp_path / "mb.bin"
    pkg.write_model_bin(model, [layer])
    xp = tmp_path / "x.bin"
    x.tofile(xp)
    return model, xp, x.shape, g


def test_host_layer_norm_matches_reference_fixture(test_bin, tmp_path):
    """tensor_ops::layer_norm of the drop-in (host) gives the reference's bits."""
    model, xp, (T, d), g = _block_model(load_pkg(), tmp_path)
    r = subprocess.run([str(test_bin), "layernorm", str(model), str(xp), str(T), str(d),
                        str(tmp_path / "out")], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    y = np.fromfile(tmp_path / "out.ln.bin", np.float32).reshape(T, d)
    assert np.array_equal(y.view(np.uint32), g["block_post"].view(np.uint32))


@pytest.mark.gpu
def test_phimoe_block_matches_reference(test_bin, tmp_path):
    """PhiMoEBlock(loader, 0): layer_norm -> PhiMoE -> + attn of the reference."""
    model, xp, (T, d), g = _block_model(load_pkg(), tmp_path)
    r = subprocess.run([str(test_bin), "block", str(model), str(xp), str(T), str(d),
                        str(tmp_path / "out")], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    y = np.fromfile(tmp_path / "out.block.bin", np.float32).reshape(T, d)
    assert rel_l2(y, g["block_phi_y"]) <= 1e-3
