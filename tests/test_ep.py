"""Expert parallelism.

CPU (gloo, world size 2): the expert-parallel data flow of moe_ep_forward_device,
run with the library's own exchange plan (moe_ep_plan) and the CPU oracle as
the experts: local routing, counts exchange, compact expert-sorted packing,
payload all-to-all, the experts on each rank's slice, the return all-to-all
and the weighted combine.  The result must equal the single-process oracle.

CPU (gloo): the deduplicated fused transport's layout restated the same way
(one row per token and destination rank, selections as metadata, the
expert-rank sum, one returned row), which must also equal the oracle and
place every selection in exactly one GEMM row.

GPU (2, 4 and 8 B200s, each skipped with fewer): moe_ep_forward_device
itself against the oracle, per rank, with both transports: the fused one
(rows and metadata stored into the other GPUs' buffers over NVLink, flags in
peer memory) and NCCL send/recv; two steps must agree bit for bit.
"""
import os
import socket
import sys

import numpy as np
import pytest

from conftest import GOLDEN_DIR, ROOT, load_oracle, load_pkg, rel_l2

sys.path.insert(0, str(GOLDEN_DIR))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


# Layer of the test: 8 experts over 2 ranks, top-2 softmax, router bias for skew.
D, FF, E, K, T_LOCAL = 64, 96, 8, 2, 37


def _layer(pkg):
    bias = np.linspace(0.0, -1.5, E).astype(np.float32)
    return pkg.synthetic_layer(41, D, FF, E, router_bias=bias)


def _tokens(pkg, rank):
    return pkg.synthetic_tokens(100 + rank, T_LOCAL + 5 * rank, D)   # ragged across ranks


def _gloo_rank(rank, world, port, q):
    try:
        import torch
        import torch.distributed as dist
        sys.path.insert(0, str(ROOT / "tests"))
        from conftest import load_oracle as lo, load_pkg as lp
        pkg, oracle = lp(), lo()
        orc = oracle.Oracle()
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        layer = _layer(pkg)
        x = _tokens(pkg, rank)
        T = x.shape[0]
        # 1-2: route and pack compactly, sorted by dispatch position then
        # token.  Round-robin placement: rank r holds experts r, r + G, ...;
        # expert e's dispatch position is (e % G) * El + e // G.
        El = E // world
        pos = lambda e: (e % world) * El + e // world  # noqa: E731
        logits = orc.router_logits(x, layer.wg, layer.router_bias)
        idx, w = orc.route(logits, K, oracle.POLICY_SOFTMAX)
        counts = np.bincount([pos(int(e)) for e in idx.ravel()], minlength=E).astype(np.int32)
        order = sorted(((pos(int(idx[t, s])), t, s) for t in range(T) for s in range(K)))
        send_rows = np.stack([x[t] for (_, t, _) in order])
        send_tok = np.array([t for (_, t, _) in order])
        send_w = np.array([w[t, s] for (_, t, s) in order], np.float32)
        # 3: counts exchange: rank j gets my counts for its experts.
        cin = torch.empty(world * El, dtype=torch.int32)
        dist.all_to_all_single(cin, torch.from_numpy(counts))
        counts_in = cin.numpy().reshape(world, El)
        s_rows, s_off, r_rows, r_off = pkg.ep_plan(counts, counts_in, world, El)
        # 4: payload exchange.
        recv = torch.empty(int(r_off[-1]), D)
        dist.all_to_all_single(recv, torch.from_numpy(send_rows), [int(v) for v in r_rows],
                               [int(v) for v in s_rows])
        recv = recv.numpy()
        # 5-6: my experts on the rows that arrived ([source][local expert][token]).
        out = np.zeros_like(recv)
        for src in range(world):
            base = int(r_off[src])
            for el in range(El):
                n = int(counts_in[src, el])
                if n:
                    e = el * world + rank
                    out[base:base + n] = orc.expert_ffn(recv[base:base + n], layer.w1[e],
                                                        layer.w3[e], layer.w2[e])
                base += n
        # 7: return exchange.
        back = torch.empty(int(s_off[-1]), D)
        dist.all_to_all_single(back, torch.from_numpy(out), [int(v) for v in s_rows],
                               [int(v) for v in r_rows])
        # 8: combine.
        y = np.zeros((T, D), np.float64)
        np.add.at(y, send_tok, send_w[:, None].astype(np.float64) * back.numpy())
        y_ref, *_ = orc.moe_forward(x, layer, K, oracle.POLICY_SOFTMAX)
        q.put((rank, rel_l2(y, y_ref), int(counts.sum()), int(r_off[-1])))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), -1, -1))


K_DD = 4   # top-4 of 8 experts on 2 ranks: most tokens have several experts on one rank


def _gloo_dedup_rank(rank, world, port, q):
    """The deduplicated fused transport's layout, restated on gloo: one row
    per (token, destination rank) carrying its selections on that rank as
    (local expert, position inside the expert's block from this source,
    weight); the receiver places each selection at eoff[e] + base[source][e]
    + position, sums the row's weighted expert outputs, and returns one row;
    the source adds its ranks' rows in ascending rank order."""
    try:
        import torch
        import torch.distributed as dist
        sys.path.insert(0, str(ROOT / "tests"))
        from conftest import load_oracle as lo, load_pkg as lp
        pkg, oracle = lp(), lo()
        orc = oracle.Oracle()
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        layer = _layer(pkg)
        x = _tokens(pkg, rank)
        T = x.shape[0]
        El = E // world
        kmax = min(K_DD, El)
        pos_of = lambda e: (e % world) * El + e // world  # noqa: E731
        logits = orc.router_logits(x, layer.wg, layer.router_bias)
        idx, w = orc.route(logits, K_DD, oracle.POLICY_SOFTMAX)
        P = np.vectorize(pos_of)(idx)                      # dispatch positions [T][K]
        # Source side: positions inside each expert's block (ascending token),
        # per-expert counts, rows per destination and their metadata.
        seen = np.zeros(E, np.int64)
        pin = np.zeros_like(P)
        for t in range(T):
            for s_ in range(K_DD):
                pin[t, s_] = seen[P[t, s_]]
                seen[P[t, s_]] += 1
        counts = seen.astype(np.int32)
        rows, metas, slot = [[] for _ in range(world)], [[] for _ in range(world)], {}
        for t in range(T):
            for g in range(world):
                sel = [(int(P[t, s_]) - g * El, int(pin[t, s_]), float(w[t, s_]))
                       for s_ in range(K_DD) if P[t, s_] // El == g]
                if not sel:
                    continue
                assert len(sel) <= kmax
                slot[(t, g)] = len(rows[g])
                rows[g].append(x[t])
                metas[g].append(sel + [(-1, 0, 0.0)] * (kmax - len(sel)))
        n_send = [len(r) for r in rows]
        # Exchange counts, row counts, rows and metadata.
        cin = torch.empty(world * El, dtype=torch.int32)
        dist.all_to_all_single(cin, torch.from_numpy(counts))
        counts_in = cin.numpy().reshape(world, El)
        nin = torch.empty(world, dtype=torch.int64)
        dist.all_to_all_single(nin, torch.tensor(n_send, dtype=torch.int64))
        n_recv = [int(v) for v in nin]
        send = np.concatenate([np.asarray(r, np.float32).reshape(-1, D) for r in rows])
        recv = torch.empty(sum(n_recv), D)
        dist.all_to_all_single(recv, torch.from_numpy(send), n_recv, n_send)
        mi = np.concatenate([np.asarray([[(e, p_) for e, p_, _ in m] for m in metas[g]],
                                        np.int64).reshape(-1, kmax * 2) for g in range(world)])
        mw = np.concatenate([np.asarray([[w_ for _, _, w_ in m] for m in metas[g]],
                                        np.float32).reshape(-1, kmax) for g in range(world)])
        rmi = torch.empty(sum(n_recv), kmax * 2, dtype=torch.int64)
        rmw = torch.empty(sum(n_recv), kmax)
        dist.all_to_all_single(rmi, torch.from_numpy(mi), n_recv, n_send)
        dist.all_to_all_single(rmw, torch.from_numpy(mw), n_recv, n_send)
        recv, rmi, rmw = recv.numpy(), rmi.numpy().reshape(-1, kmax, 2), rmw.numpy()
        # Receiver side: arrival scan and arrangement.
        total = counts_in.sum(axis=0)
        eoff = np.concatenate([[0], np.cumsum(total)])
        base = np.cumsum(counts_in, axis=0) - counts_in          # [source][local expert]
        A = np.full((int(eoff[-1]), D), np.nan, np.float32)
        owner = np.full(int(eoff[-1]), -1, np.int64)
        wt = np.zeros(int(eoff[-1]), np.float64)
        src_of = np.repeat(np.arange(world), n_recv)
        for i in range(len(recv)):
            sidx = int(src_of[i])
            for j in range(kmax):
                e, p_ = int(rmi[i, j, 0]), int(rmi[i, j, 1])
                if e < 0:
                    break
                prow = int(eoff[e] + base[sidx, e] + p_)
                assert owner[prow] == -1, "two selections placed in one row"
                owner[prow], wt[prow] = i, float(rmw[i, j])
                A[prow] = recv[i]
        assert (owner >= 0).all(), "a row of an expert block left unplaced"
        y_recv = np.zeros((len(recv), D), np.float64)
        for e in range(El):
            lo_, hi_ = int(eoff[e]), int(eoff[e + 1])
            if hi_ > lo_:
                ge = e * world + rank
                out = orc.expert_ffn(A[lo_:hi_], layer.w1[ge], layer.w3[ge], layer.w2[ge])
                np.add.at(y_recv, owner[lo_:hi_], wt[lo_:hi_, None] * out.astype(np.float64))
        # Return one row per received row; combine in ascending rank order.
        back = torch.empty(sum(n_send), D, dtype=torch.float64)
        dist.all_to_all_single(back, torch.from_numpy(y_recv), n_send, n_recv)
        back = back.numpy()
        seg = np.concatenate([[0], np.cumsum(n_send)])
        y = np.zeros((T, D), np.float64)
        for t in range(T):
            for g in range(world):
                if (t, g) in slot:
                    y[t] += back[seg[g] + slot[(t, g)]]
        y_ref, *_ = orc.moe_forward(x, layer, K_DD, oracle.POLICY_SOFTMAX)
        q.put((rank, rel_l2(y, y_ref), T * K_DD, sum(n_send)))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), -1, -1))


def test_ep_dedup_layout_on_gloo_matches_oracle():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_dedup_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    res.sort()
    for rank, err, selections, rows_sent in res:
        assert isinstance(err, float), err
        assert err <= 1e-6, (rank, err)
        # Deduplication: at most one row per (token, rank), fewer rows than selections.
        assert rows_sent < selections


def test_ep_dataflow_on_gloo_matches_oracle():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    res.sort()
    for rank, err, sent, got in res:
        assert isinstance(err, float), err
        assert err <= 1e-6, (rank, err)
        assert sent == (T_LOCAL + 5 * rank) * K
    # every routed row was received exactly once by some rank
    assert sum(r[3] for r in res) == sum(r[2] for r in res)


def test_ep_plan_offsets_and_rejection():
    pkg = load_pkg()
    counts = np.array([3, 0, 2, 5], np.int32)          # 2 ranks x 2 local experts
    counts_in = np.array([[1, 2], [4, 0]], np.int32)
    s_rows, s_off, r_rows, r_off = pkg.ep_plan(counts, counts_in, 2, 2)
    assert list(s_rows) == [3, 7] and list(s_off) == [0, 3, 10]
    assert list(r_rows) == [3, 4] and list(r_off) == [0, 3, 7]
    with pytest.raises(pkg.MoeError):
        pkg.ep_plan(np.array([1, -1], np.int32), np.array([[0], [0]], np.int32), 2, 1)


def _gpu_rank(rank, world, idbytes, q, precision, transport, k=K):
    try:
        import torch
        sys.path.insert(0, str(ROOT / "tests"))
        from conftest import load_oracle as lo, load_pkg as lp
        pkg, oracle = lp(), lo()
        torch.cuda.set_device(rank)
        layer = _layer(pkg)
        x = _tokens(pkg, rank)
        m = pkg.MoeLayer.expert_parallel(rank, world, idbytes, d=D, ff=FF, E=E, wg=layer.wg,
                                         w1=layer.w1, w3=layer.w3, w2=layer.w2,
                                         bias=layer.router_bias, top_k=k, policy=1,
                                         precision=precision, device=rank,
                                         ep_transport=transport,
                                         max_tokens=T_LOCAL + 5 * (world - 1))
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty_like(xd)
        ys = []
        for _ in range(2):
            m.ep_forward_device(xd.data_ptr(), yd.data_ptr(), x.shape[0],
                                torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            ys.append(yd.cpu().numpy().copy())
        y_ref, *_ = oracle.Oracle().moe_forward(x, layer, k, oracle.POLICY_SOFTMAX)
        m.close()
        same = bool(np.array_equal(ys[0].view(np.uint32), ys[1].view(np.uint32)))
        q.put((rank, rel_l2(ys[0], y_ref), rel_l2(ys[1], y_ref), same))
    except Exception as e:
        q.put((rank, repr(e), None, None))


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("k", [2, 4])
@pytest.mark.parametrize("transport", [0, 1], ids=["p2p", "nccl"])
@pytest.mark.parametrize("precision", [0, 1, 2], ids=["fp32", "bf16", "bf16x3"])
def test_ep_forward_on_gpus(precision, transport, k, world):
    """Each rank's y against the oracle, twice (the epochs advance), and the
    two steps bit-identical: the expert-rank sums and the combine run in a
    fixed order whatever the arrival order.  Top-4 of 8 experts puts up to 4
    of a token's experts on one rank at 2 GPUs."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    pkg = load_pkg()
    idbytes = pkg.ep_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gpu_rank, args=(r, world, idbytes, q, precision, transport, k))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    tol = 2e-2 if precision == 1 else 1e-3
    for rank, e1, e2, same in res:
        assert isinstance(e1, float), e1
        assert e1 <= tol and e2 <= tol, (rank, e1, e2)
        assert same, f"rank {rank}: two identical steps differ"



def _timeout_rank(rank, world, idbytes, q, bar):
    """Rank 1 misses step 2 (it sleeps between steps, nothing in flight);
    rank 0's bounded peer wait runs out, its group is marked failed, and both
    ranks report MOE_ERR_TIMEOUT instead of hanging."""
    try:
        import time
        import torch
        sys.path.insert(0, str(ROOT / "tests"))
        from conftest import load_pkg as lp
        pkg = lp()
        torch.cuda.set_device(rank)
        layer = _layer(pkg)
        x = _tokens(pkg, rank)
        m = pkg.MoeLayer.expert_parallel(rank, world, idbytes, d=D, ff=FF, E=E, wg=layer.wg,
                                         w1=layer.w1, w3=layer.w3, w2=layer.w2,
                                         bias=layer.router_bias, top_k=K, policy=1,
                                         precision=1, device=rank, max_tokens=64,
                                         ep_transport=0, ep_wait_ms=300)
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty_like(xd)
        s = torch.cuda.current_stream().cuda_stream
        out = []
        m.ep_forward_device(xd.data_ptr(), yd.data_ptr(), x.shape[0], s)     # step 1, both ranks
        m.ep_check()
        out.append("step1 ok")
        t0 = time.monotonic()
        if rank == 1:
            time.sleep(1.5)                                                  # misses step 2
        for step in (2, 3, 4):
            try:
                m.ep_forward_device(xd.data_ptr(), yd.data_ptr(), x.shape[0], s)
                m.ep_check()
                out.append(f"step{step} ok")
            except pkg.MoeError as e:
                out.append(f"step{step} err {e.code}")
        torch.cuda.synchronize()
        dt = time.monotonic() - t0
        # No rank frees its buffers while another may still store into them.
        bar.wait(timeout=60)
        m.close()
        q.put((rank, out, dt))
    except Exception as e:  # noqa: BLE001 -- reported to the parent
        q.put((rank, repr(e), None))


@pytest.mark.gpu
def test_ep_peer_timeout_fails_the_group_without_hanging():
    """Failure detection without a GPU fault: the missed step is made on the
    host (a rank that sleeps between steps); every wait is bounded (300 ms
    here), so both ranks end with MOE_ERR_TIMEOUT and the handle stays
    failed.  Child processes with NVLS off; the fused transport uses plain
    peer stores."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    pkg = load_pkg()
    idbytes = pkg.ep_unique_id()
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    bar = ctx.Barrier(2)
    procs = [ctx.Process(target=_timeout_rank, args=(r, 2, idbytes, q, bar)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for rank, out, dt in res:
        assert isinstance(out, list), out
        assert out[0] == "step1 ok"
        assert any(o.endswith("err -6") for o in out[1:]), (rank, out)
        # once failed, the handle stays failed
        first = next(i for i, o in enumerate(out) if o.endswith("err -6"))
        assert all(o.endswith("err -6") for o in out[first:]), (rank, out)
        assert dt < 30.0, (rank, dt)
