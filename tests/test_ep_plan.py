"""CPU, multi-process (gloo): the expert-parallel exchange plan.

Each rank routes random (token, slot) pairs, builds its send counts from the
stable permutation, exchanges counts with its peers, and asks the library's
MoeEpPlan (pure host code, through the C ABI) for the offsets and the
expert-major segment table.  The test then replays the GPU data path in numpy,
with gloo standing in for NCCL: dispatch, expert-major reorder, a stand-in
"expert" (row * (global expert id + 1)), the scatter back to source-major order,
the return exchange and the indexed combine.  Each rank's y must equal the
direct single-process computation.  No GPU is involved.
"""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, n, port, E, K, T, H, q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "tests"))
    from _moe_loader import load
    from oracle import oracle as O

    moe = load()
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=n)
    try:
        El = E // n
        rng = np.random.default_rng(100 + rank)
        # ragged load: rank-dependent skew so some (source, expert) blocks are empty
        probs = rng.dirichlet(np.full(E, 0.3))
        ids = np.stack([rng.choice(E, size=K, replace=False, p=probs) for _ in range(T)]).astype(np.int32)
        w = rng.random((T, K))
        x = rng.standard_normal((T, H))
        perm, offs = O.permute(ids, E)
        dest = np.empty_like(perm)
        dest[perm] = np.arange(perm.size)
        xp = x[perm // K]
        send = (offs[1:] - offs[:-1]).reshape(n, El).astype(np.int32)
        all_send = [None] * n
        dist.all_gather_object(all_send, send)
        recv = np.stack([all_send[s][rank] for s in range(n)]).astype(np.int32)
        so, ro, eo_off, seg = moe.ep_plan(send, recv)
        assert np.array_equal(so, offs[::El][: n + 1]) if E % n == 0 else True
        # dispatch
        all_xp = [None] * n
        all_so = [None] * n
        dist.all_gather_object(all_xp, xp)
        dist.all_gather_object(all_so, so)
        rbuf = np.zeros((ro[n], H))
        for s in range(n):
            rbuf[ro[s]:ro[s + 1]] = all_xp[s][all_so[s][rank]:all_so[s][rank + 1]]
        # expert-major reorder, stand-in expert, scatter back to source-major
        row_src = np.empty(ro[n], np.int64)
        for e in range(El):
            for s in range(n):
                d, src, ln = seg[e * n + s]
                row_src[d:d + ln] = np.arange(src, src + ln)
        xr = rbuf[row_src]
        out = np.empty_like(xr)
        for e in range(El):
            out[eo_off[e]:eo_off[e + 1]] = xr[eo_off[e]:eo_off[e + 1]] * (rank * El + e + 1)
        eo = np.empty_like(rbuf)
        eo[row_src] = out
        # return
        all_eo = [None] * n
        all_ro = [None] * n
        dist.all_gather_object(all_eo, eo)
        dist.all_gather_object(all_ro, ro)
        ret = np.zeros_like(xp)
        for p in range(n):
            ret[so[p]:so[p + 1]] = all_eo[p][all_ro[p][rank]:all_ro[p][rank + 1]]
        y = np.zeros((T, H))
        for k in range(K):
            y += w[:, k:k + 1] * ret[dest.reshape(T, K)[:, k]]
        ref = np.zeros((T, H))
        for k in range(K):
            ref += w[:, k:k + 1] * x * (ids[:, k:k + 1] + 1)
        q.put((rank, float(np.abs(y - ref).max()), int(ro[n])))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n,E,K", [(2, 8, 2), (4, 16, 3)])
def test_ep_plan_roundtrip_gloo(n, E, K):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, n, port, E, K, 37 + 11 * r, 16, q)) for r in range(n)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(n)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, rows in res:
        assert err < 1e-12, (rank, err)


def test_ep_plan_rejects_bad_counts(moe):
    with pytest.raises(moe.MoeError):
        moe.ep_plan(np.array([[1, -1]]), np.array([[0, 0]]))
    so, ro, eo, seg = moe.ep_plan(np.zeros((3, 2)), np.zeros((3, 2)))
    assert so[-1] == 0 and ro[-1] == 0 and eo[-1] == 0
