"""Golden cases: the seeded inputs behind each committed fixture.

Each case names its shapes, seed and routing policy.  Inputs are regenerated
from the seed by the package's synthetic generators (numpy PCG64), and their
SHA-256 is stored in the fixture so a generator change is caught before any
comparison is made.
"""
CASES = {
    # T=64, d=512, E=8, top-2, ff=1024, W~N(0,0.02), x~N(0,1), seed 0.
    "c1": dict(seed=0, T=64, d=512, ff=1024, E=8, k=2, bias=False),
    # Phi-tiny-MoE-like routing (16 experts, d_ff 448 is not a multiple of the
    # 128-row block), ragged token count.
    "phi16": dict(seed=7, T=40, d=256, ff=448, E=16, k=2, bias=False),
    # BASELINE config 5 in miniature: 64 experts, top-8, Zipf router bias,
    # router weights scaled so logits are ~N(0,1).
    "c5mini": dict(seed=3, T=48, d=256, ff=192, E=64, k=8, bias=True),
}


def case_inputs(pkg, name):
    import numpy as np
    c = CASES[name]
    bias = pkg.zipf_router_bias(c["E"]) if c["bias"] else None
    router_std = (1.0 / np.sqrt(c["d"])) if c["bias"] else None
    layer = pkg.synthetic_layer(c["seed"], c["d"], c["ff"], c["E"], router_std=router_std,
                                router_bias=bias)
    x = pkg.synthetic_tokens(c["seed"], c["T"], c["d"])
    return layer, x


def sha256_of(layer, x):
    import hashlib
    h = hashlib.sha256()
    for a in (x, layer.wg, *layer.w1, *layer.w3, *layer.w2):
        h.update(a.tobytes())
    if layer.router_bias is not None:
        h.update(layer.router_bias.tobytes())
    return h.hexdigest()
