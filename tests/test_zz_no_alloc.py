"""moe_dispatch_noalloc, the dispatch entry point that allocates nothing
(needs a B200).

Some callers cannot call cudaMalloc: code running inside a stream capture
that must not touch the allocator, serving frameworks whose own pool owns all
device memory, latency-critical paths that cannot take an allocation's
implicit synchronisation.  For them moe_dispatch_noalloc keeps its only
scratch in a fixed 1 MiB device array inside the library.  Given the same
routing decisions, it must produce exactly the packed layout that the forward
path builds in its own workspace -- checked here on two calls in a row, since
every call reuses (and must not depend on) the array's previous contents.

This file is collected last so that a run stopping at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""
import ctypes
import sys

import numpy as np
import pytest

from conftest import GOLDEN_DIR, load_pkg

sys.path.insert(0, str(GOLDEN_DIR))
from cases import CASES, case_inputs  # noqa: E402

pytestmark = pytest.mark.gpu


def _call(lib, idx, w, T, E, k, tok, wt, cap, eoff, cnt, stream):
    vp = ctypes.c_void_p
    return lib.moe_dispatch_noalloc(vp(idx), vp(w), T, E, k, vp(tok), vp(wt), cap, vp(eoff),
                                    vp(cnt), vp(stream))


@pytest.mark.parametrize("name", ["c1", "c5mini"])
def test_noalloc_dispatch_matches_forward_layout(name):
    import torch
    pkg = load_pkg()
    lib = pkg.load_library()
    layer, x = case_inputs(pkg, name)
    T, E, k = x.shape[0], layer.E, CASES[name]["k"]
    cap = (T * k // 128 + E + 1) * 128
    with pkg.MoeLayer(layer, top_k=k, policy=pkg.ROUTER_SOFTMAX_TOPK) as m:
        m.forward_host(x)
        tok_ref, w_ref, eoff_ref = m.dispatch_layout(rows_cap=cap)
        counts_ref = m.expert_counts()
        xd = torch.from_numpy(x).cuda()
        idx = torch.empty((T, k), dtype=torch.int32, device="cuda")
        w = torch.empty((T, k), dtype=torch.float32, device="cuda")
        m.route_device(xd.data_ptr(), T, 0, idx.data_ptr(), w.data_ptr(),
                       torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    rows = int(eoff_ref[-1])
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        # Sentinels catch any output element the entry point fails to write.
        tok = torch.full((cap,), 0x7FFF0000, dtype=torch.int32, device="cuda")
        wt = torch.full((cap,), float("nan"), dtype=torch.float32, device="cuda")
        eoff = torch.full((E + 1,), -7, dtype=torch.int32, device="cuda")
        cnt = torch.full((E,), -7, dtype=torch.int32, device="cuda")
        rc = _call(lib, idx.data_ptr(), w.data_ptr(), T, E, k, tok.data_ptr(), wt.data_ptr(),
                   cap, eoff.data_ptr(), cnt.data_ptr(), stream)
        assert rc == 0, lib.moe_last_error().decode()
        torch.cuda.synchronize()
        assert np.array_equal(cnt.cpu().numpy(), counts_ref)
        assert np.array_equal(eoff.cpu().numpy(), eoff_ref)
        assert np.array_equal(tok.cpu().numpy()[:rows], tok_ref)
        got_w = wt.cpu().numpy()[:rows]
        assert np.array_equal(got_w.view(np.uint32), np.ascontiguousarray(w_ref).view(np.uint32))


def test_noalloc_rejects_sizes_beyond_its_scratch():
    pkg = load_pkg()
    lib = pkg.load_library()
    # ceil(T / 32) * E = 32768 * 16 = 524288 > 262144 scratch entries.
    T, E, k = 1 << 20, 16, 2
    cap = (T * k // 128 + E + 1) * 128
    rc = _call(lib, 16, 16, T, E, k, 16, 16, cap, 16, 16, 0)
    assert rc == -1
    assert "static scratch" in lib.moe_last_error().decode()
    # rows_cap below the bound is rejected too.
    rc = _call(lib, 16, 16, 64, 8, 2, 16, 16, 128, 16, 16, 0)
    assert rc == -1
