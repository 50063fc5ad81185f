"""Expert parallelism.

CPU (gloo, world size 2): the expert-parallel data flow of moe_ep_forward_device,
run with the library's own exchange plan (moe_ep_plan) and the CPU oracle as
the experts: local routing, counts exchange, compact expert-sorted packing,
payload all-to-all, the experts on each rank's slice, the return all-to-all
and the weighted combine.  The result must equal the single-process oracle.

GPU (2 B200s, skipped with fewer): moe_ep_forward_device itself against the
oracle, per rank, with both transports: the fused one (dispatch permute and
down-GEMM epilogue storing rows into the other GPU's buffers over NVLink,
flags in peer memory) and NCCL send/recv.
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


def _gpu_rank(rank, world, idbytes, q, precision, transport):
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
                                         bias=layer.router_bias, top_k=K, policy=1,
                                         precision=precision, device=rank,
                                         ep_transport=transport, max_tokens=64)
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty_like(xd)
        ys = []
        for _ in range(2):
            m.ep_forward_device(xd.data_ptr(), yd.data_ptr(), x.shape[0],
                                torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            ys.append(yd.cpu().numpy().copy())
        y_ref, *_ = oracle.Oracle().moe_forward(x, layer, K, oracle.POLICY_SOFTMAX)
        m.close()
        q.put((rank, rel_l2(ys[0], y_ref), rel_l2(ys[1], y_ref)))
    except Exception as e:
        q.put((rank, repr(e), None))


@pytest.mark.gpu
@pytest.mark.parametrize("transport", [0, 1], ids=["p2p", "nccl"])
@pytest.mark.parametrize("precision", [0, 1], ids=["fp32", "bf16"])
def test_ep_forward_on_two_gpus(precision, transport):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    pkg = load_pkg()
    idbytes = pkg.ep_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gpu_rank, args=(r, 2, idbytes, q, precision, transport))
             for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    tol = 1e-3 if precision == 0 else 2e-2
    for rank, e1, e2 in res:
        assert isinstance(e1, float), e1
        assert e1 <= tol and e2 <= tol, (rank, e1, e2)
