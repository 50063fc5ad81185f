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


def _expected_layout(idx, w, E):
    """The packed layout on the host: per expert, its (token, slot) entries
    in ascending order, blocks padded to 128 rows (token -1, weight 0)."""
    T, k = idx.shape
    flat, fw = idx.reshape(-1), w.reshape(-1)
    valid = (flat >= 0) & (flat < E)
    counts = np.bincount(flat[valid], minlength=E).astype(np.int32)
    eoff = np.concatenate([[0], np.cumsum((counts + 127) // 128 * 128)]).astype(np.int32)
    order = np.argsort(np.where(valid, flat, E), kind="stable")[: int(valid.sum())]
    tok = np.full(int(eoff[-1]), -1, np.int32)
    wt = np.zeros(int(eoff[-1]), np.float32)
    start = 0
    for e in range(E):
        ent = order[start:start + counts[e]]
        tok[eoff[e]:eoff[e] + counts[e]] = ent // k
        wt[eoff[e]:eoff[e] + counts[e]] = fw[ent]
        start += counts[e]
    return tok, wt, eoff, counts


def _run_noalloc(lib, idx_h, w_h, E):
    import torch
    T, k = idx_h.shape
    cap = (T * k // 128 + E + 1) * 128
    idx = torch.from_numpy(np.ascontiguousarray(idx_h)).cuda()
    w = torch.from_numpy(np.ascontiguousarray(w_h)).cuda()
    tok = torch.full((cap,), 0x7FFF0000, dtype=torch.int32, device="cuda")
    wt = torch.full((cap,), float("nan"), dtype=torch.float32, device="cuda")
    eoff = torch.full((E + 1,), -7, dtype=torch.int32, device="cuda")
    cnt = torch.full((E,), -7, dtype=torch.int32, device="cuda")
    rc = _call(lib, idx.data_ptr(), w.data_ptr(), T, E, k, tok.data_ptr(), wt.data_ptr(), cap,
               eoff.data_ptr(), cnt.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.moe_last_error().decode()
    torch.cuda.synchronize()
    return tok.cpu().numpy(), wt.cpu().numpy(), eoff.cpu().numpy(), cnt.cpu().numpy()


def test_noalloc_duplicates_out_of_range_and_empty():
    """Inputs the router never produces: an expert listed twice by one token
    gets two rows (slot order), indices -1 and E are skipped, and T = 0
    writes zero counts and offsets -- each on two calls in a row."""
    pkg = load_pkg()
    lib = pkg.load_library()
    rng = np.random.default_rng(11)
    T, E, k = 77, 8, 3
    idx = rng.integers(0, E, size=(T, k)).astype(np.int32)
    idx[5] = [2, 2, 2]
    idx[9, 1] = -1
    idx[40, 2] = E
    w = rng.random((T, k)).astype(np.float32)
    tok_e, wt_e, eoff_e, cnt_e = _expected_layout(idx, w, E)
    for _ in range(2):
        tok, wt, eoff, cnt = _run_noalloc(lib, idx, w, E)
        assert np.array_equal(cnt, cnt_e) and np.array_equal(eoff, eoff_e)
        n = int(eoff_e[-1])
        assert np.array_equal(tok[:n], tok_e)
        assert np.array_equal(wt[:n].view(np.uint32), wt_e.view(np.uint32))
    for _ in range(2):
        _, _, eoff, cnt = _run_noalloc(lib, np.zeros((0, 2), np.int32), np.zeros((0, 2), np.float32), E)
        assert (cnt == 0).all() and (eoff == 0).all()


def test_noalloc_at_the_scratch_limit():
    """ceil(T / 32) * num_experts exactly at the 262144-entry limit is
    accepted and placed correctly."""
    pkg = load_pkg()
    lib = pkg.load_library()
    E, k = 8, 1
    T = 32 * (262144 // E)
    rng = np.random.default_rng(12)
    idx = rng.integers(0, E, size=(T, k)).astype(np.int32)
    w = rng.random((T, k)).astype(np.float32)
    tok_e, wt_e, eoff_e, cnt_e = _expected_layout(idx, w, E)
    tok, wt, eoff, cnt = _run_noalloc(lib, idx, w, E)
    assert np.array_equal(cnt, cnt_e) and np.array_equal(eoff, eoff_e)
    n = int(eoff_e[-1])
    assert np.array_equal(tok[:n], tok_e)
    assert np.array_equal(wt[:n].view(np.uint32), wt_e.view(np.uint32))
