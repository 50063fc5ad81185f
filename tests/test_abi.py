"""The C-ABI library: built for sm_100a, loads, and exports exactly what
include/moe_b200.h declares (no compute without a GPU)."""
import re
import subprocess

import pytest

from conftest import PKG_DIR, ROOT, load_pkg

HEADER = ROOT / "include" / "moe_b200.h"


def declared_functions():
    src = HEADER.read_text()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\**\s*(moe_[a-z0-9_]+)\s*\(",
                       src, flags=re.M)
    return sorted(set(names))


def test_header_lists_match_binding():
    pkg = load_pkg()
    assert declared_functions() == sorted(pkg.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    pkg = load_pkg()
    lib = pkg.LIB_PATH
    if not lib.exists():
        pytest.fail(f"{lib} not built")
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (moe_[a-z0-9_]+)\b", out))
    missing = set(declared_functions()) - exported
    assert not missing, missing
    L = pkg.load_library()
    assert L.moe_abi_version() == 1


def test_library_carries_sm100a_code():
    lib = load_pkg().LIB_PATH
    out = subprocess.run(["/usr/local/cuda/bin/cuobjdump", "--list-elf", str(lib)],
                         capture_output=True, text=True).stdout
    assert "sm_100a" in out


def test_config_defaults_are_reference_constants():
    """moe_config_init mirrors include/config.h:8-23 of the reference."""
    pkg = load_pkg()
    c = pkg.default_config()
    assert (c.d_model, c.d_ff, c.num_experts, c.top_k) == (4096, 448, 16, 2)
    assert c.router_policy == pkg.ROUTER_PHI_QUANTISED
    assert abs(c.router_quantum - 1e-3) < 1e-9 and abs(c.router_tie_eps - 2e-2) < 1e-9
    assert c.decode_max_tokens == pkg.DECODE_AUTO == -1   # resolved per precision by a handle


def test_invalid_config_is_rejected_before_any_device_work():
    pkg = load_pkg()
    layer = pkg.synthetic_layer(0, 96, 64, 4)   # d_model 96 is not a multiple of 64
    with pytest.raises(pkg.MoeError) as ei:
        pkg.MoeLayer(layer, top_k=2)
    assert ei.value.code == -2
    with pytest.raises(pkg.MoeError) as ei:
        pkg.MoeLayer(pkg.synthetic_layer(0, 64, 64, 4), top_k=3,
                     policy=pkg.ROUTER_PHI_QUANTISED)
    assert ei.value.code == -1


def test_model_bin_errors_are_io(tmp_path):
    pkg = load_pkg()
    with pytest.raises(pkg.MoeError) as ei:
        pkg.MoeLayer(model_bin=str(tmp_path / "missing.bin"))
    assert ei.value.code == -5
    p = tmp_path / "trunc.bin"
    pkg.write_model_bin(p, [pkg.synthetic_layer(0, 64, 64, 4)])
    data = p.read_bytes()
    p.write_bytes(data[:200])
    with pytest.raises(pkg.MoeError) as ei:
        pkg.MoeLayer(model_bin=str(p))
    assert ei.value.code == -5
