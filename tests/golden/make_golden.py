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
  * block_*: the decoder layer's MoE half (PhiDecoderLayer::forward,
    src/layer.cu:157-161) on the same x taken as the attention output, with
    a seeded post-attention LayerNorm: post = tensor_ops::layer_norm(x) and,
    for PHI, y = PhiMoE::forward(post) + x, all from the reference; the
    restatement's layer_norm and forward are asserted identical first.
"""
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
sys.path.insert(0, str(HERE))
from conftest import load_oracle, load_pkg  # noqa: E402
from cases import CASES, case_inputs, sha256_of  # noqa: E402

NORM_EPS = 1e-5   # include/config.h:19


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
            # The decoder layer's MoE half with the reference's own ops.
            nw, nb = pkg.synthetic_post_norm(c["seed"], c["d"])
            post = ref.layer_norm(x, nw, nb, NORM_EPS)
            assert np.array_equal(post.view(np.uint32),
                                  orc.layer_norm(x, nw, nb, NORM_EPS).view(np.uint32)), name
            ref = oracle.Reference(c["E"])
            pkg.write_model_bin(model, [layer])
            ref.load(str(model), 0)
            b_logits, b_idx, _ = ref.route(post)
            b_y = ref.forward(post) + x          # tensor_ops::add_inplace(ff, attn)
            ref.close()
            model.unlink()
            oy, oidx, _, _ = orc.moe_forward(post, layer, 2, oracle.POLICY_PHI)
            assert np.array_equal(oidx, b_idx), name
            assert np.array_equal((oy + x).view(np.uint32), b_y.view(np.uint32)), name
            out.update(block_norm_w=nw, block_norm_b=nb, block_post=post, block_phi_idx=b_idx,
                       block_phi_logits=b_logits, block_phi_y=b_y)
            print(f"{name}: block (layer_norm -> PhiMoE -> +attn) pinned to the reference")
        y, idx, w, logits = orc.moe_forward(x, layer, c["k"], oracle.POLICY_SOFTMAX)
        out.update(soft_logits=logits, soft_idx=idx, soft_w=w, soft_y=y)
        np.savez_compressed(HERE / f"{name}.npz", **out)
        print(f"{name}: wrote {name}.npz")


if __name__ == "__main__":
    main()
