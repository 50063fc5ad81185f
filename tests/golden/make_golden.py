"""Regenerate the golden fixtures in this directory.

    python tests/golden/make_golden.py

Needs the reference's own PhiMoE compiled from its sources
(oracle/_ref/libref_e<E>.so, built by `make -C oracle` where the reference
tree is present).  For each case:
  * PHI_QUANTISED policy (k = 2, E in {8, 16}): logits, expert indices and y
    come from the reference's PhiMoE::route / forward (src/layer.cu:47-103).
    The CPU restatement (oracle/moe_oracle.c) is asserted bit-identical to
    them before anything is written.
  * SOFTMAX_TOPK policy: the reference has no such router (softmax_last_dim
    is declared at include/tensor.h:67 but never defined), so idx / weights /
    y come from the restatement, whose router logits and expert arithmetic
    are the ones just pinned against the reference.
"""
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE))
from conftest import load_oracle, load_pkg  # noqa: E402
from cases import CASES, case_inputs, sha256_of  # noqa: E402


def main():
    pkg = load_pkg()
    oracle = load_oracle()
    orc = oracle.Oracle()
    for name, c in CASES.items():
        layer, x = case_inputs(pkg, name)
        out = {"sha256": np.array(sha256_of(layer, x))}
        if c["k"] == 2 and c["E"] in (8, 16) and not c["bias"]:
            ref = oracle.Reference(c["E"])
            model = Path("/tmp") / f"golden_{name}.bin"
            pkg.write_model_bin(model, [layer])
            ref.load(str(model), 0)
            r_logits, r_idx, r_w = ref.route(x)
            r_y = ref.forward(x)
            ref.close()
            model.unlink()
            y, idx, w, logits = orc.moe_forward(x, layer, 2, oracle.POLICY_PHI)
            assert np.array_equal(logits.view(np.uint32), r_logits.view(np.uint32)), name
            assert np.array_equal(idx, r_idx), name
            assert np.array_equal(w, r_w), name
            assert np.array_equal(y.view(np.uint32), r_y.view(np.uint32)), name
            out.update(phi_logits=r_logits, phi_idx=r_idx, phi_w=r_w, phi_y=r_y)
            print(f"{name}: oracle == reference PhiMoE, bit for bit")
        y, idx, w, logits = orc.moe_forward(x, layer, c["k"], oracle.POLICY_SOFTMAX)
        out.update(soft_logits=logits, soft_idx=idx, soft_w=w, soft_y=y)
        np.savez_compressed(HERE / f"{name}.npz", **out)
        print(f"{name}: wrote {name}.npz")


if __name__ == "__main__":
    main()
