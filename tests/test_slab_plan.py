"""Slab-decomposition plans and halo exchange on CPU: two gloo ranks reproduce a global
message-passing computation and its reverse pass (no GPU)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from tt_atom.slab import DistExchange, LockstepGroup, Plan


def _graph(N=60, deg=7, seed=0):
    """Random receiver-major graph: every receiver has `deg` random sources."""
    g = torch.Generator().manual_seed(seed)
    tgt = torch.arange(N).repeat_interleave(deg)
    src = torch.randint(0, N, (N * deg,), generator=g)
    w = torch.randn(N * deg, generator=g, dtype=torch.float64)
    recv_ptr = torch.arange(0, N * deg + 1, deg)
    x0 = torch.randn(N, 3, generator=g, dtype=torch.float64)
    return src, tgt, torch.zeros_like(src), recv_ptr, w, x0


def _global(src, tgt, w, x0, L=2):
    x = x0.clone().requires_grad_(True)
    h = x
    for _ in range(L):
        h = h + torch.zeros_like(h).index_add(0, tgt, w[:, None] * torch.tanh(h[src]))
    E = (h * h).sum()
    (g,) = torch.autograd.grad(E, x)
    return E.detach(), g


def _local_run(plan, w_all, x0, exch_fwd, exch_rev, L=2):
    e0, e1 = plan.edge_range
    w = w_all[e0:e1]
    n = plan.global_ids.numel()
    x = torch.zeros(n, 3, dtype=torch.float64)
    x[:plan.n_own] = x0[plan.global_ids[:plan.n_own]]
    xs = []
    exch_fwd(x)
    for _ in range(L):
        xs.append(x.clone())
        y = x.clone()
        y[:plan.n_own] += torch.zeros(n, 3, dtype=torch.float64).index_add(
            0, plan.tgt, w[:, None] * torch.tanh(x[plan.src]))[:plan.n_own]
        x = y
        exch_fwd(x)
    E = (x[:plan.n_own] ** 2).sum()
    g = torch.zeros(n, 3, dtype=torch.float64)
    g[:plan.n_own] = 2 * x[:plan.n_own]
    for xl in reversed(xs):
        gn = g.clone()
        t = 1 - torch.tanh(xl[plan.src]) ** 2
        gn.index_add_(0, plan.src, w[:, None] * t * g[plan.tgt])
        g = gn
        exch_rev(g)
    return E, g[:plan.n_own]


def test_lockstep_plans_reproduce_global():
    src, tgt, img, rp, w, x0 = _graph()
    E_ref, g_ref = _global(src, tgt, w, x0)
    ranges = [(0, 17), (17, 40), (40, 60)]
    plans = [Plan(src, tgt, img, rp, ranges, r) for r in range(3)]
    grp = LockstepGroup(plans)
    # lock-step emulation of the three ranks
    n = [p.global_ids.numel() for p in plans]
    xs = [torch.zeros(k, 3, dtype=torch.float64) for k in n]
    for p, x in zip(plans, xs):
        x[:p.n_own] = x0[p.global_ids[:p.n_own]]
    grp.forward(xs)
    hist = []
    for _ in range(2):
        hist.append([x.clone() for x in xs])
        new = []
        for p, x in zip(plans, xs):
            e0, e1 = p.edge_range
            y = x.clone()
            y[:p.n_own] += torch.zeros_like(x).index_add(
                0, p.tgt, w[e0:e1, None] * torch.tanh(x[p.src]))[:p.n_own]
            new.append(y)
        xs = new
        grp.forward(xs)
    E = sum(float((x[:p.n_own] ** 2).sum()) for p, x in zip(plans, xs))
    gs = []
    for p, x in zip(plans, xs):
        g = torch.zeros_like(x)
        g[:p.n_own] = 2 * x[:p.n_own]
        gs.append(g)
    for xl in reversed(hist):
        new = []
        for p, x, g in zip(plans, xl, gs):
            e0, e1 = p.edge_range
            gn = g.clone()
            gn.index_add_(0, p.src, w[e0:e1, None] * (1 - torch.tanh(x[p.src]) ** 2) * g[p.tgt])
            new.append(gn)
        gs = new
        grp.reverse(gs)
    assert abs(E - float(E_ref)) < 1e-9 * abs(float(E_ref))
    got = torch.zeros_like(g_ref)
    for p, g in zip(plans, gs):
        got[p.global_ids[:p.n_own]] = g[:p.n_own]
    assert torch.allclose(got, g_ref, rtol=1e-10, atol=1e-10)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        src, tgt, img, rp, w, x0 = _graph()
        ranges = [(0, 28), (28, 60)]
        plan = Plan(src, tgt, img, rp, ranges, rank)
        ex = DistExchange(plan)
        E, g = _local_run(plan, w, x0, ex.forward, ex.reverse)
        Et = torch.tensor([float(E)], dtype=torch.float64)
        dist.all_reduce(Et)
        q.put((rank, float(Et), plan.global_ids[:plan.n_own], g))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.timeout(120)
def test_two_gloo_ranks_reproduce_global():
    src, tgt, img, rp, w, x0 = _graph()
    E_ref, g_ref = _global(src, tgt, w, x0)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=100) for _ in range(2)]
    for p in procs:
        p.join(timeout=30)
    got = torch.zeros_like(g_ref)
    for rank, E, ids, g in res:
        assert abs(E - float(E_ref)) < 1e-9 * abs(float(E_ref))
        got[ids] = g
    assert torch.allclose(got, g_ref, rtol=1e-10, atol=1e-10)
