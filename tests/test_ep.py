"""Expert parallelism: routing plan, the dispatch/compute/combine decomposition
on CPU ranks (gloo, oracle arithmetic), and the NCCL path through the C-ABI
on two GPUs.

The decomposition claim checked here: a layer computed as
  dispatch (each (token, slot) pair to its expert's rank)
  -> per-pair FFN with one slot and unit router weight
  -> pairs back home -> slot-order combine
gives the bits of the one-process layer (the oracle's moe_layer over all
experts), for both placements and any world size.
"""
import os
import socket

import numpy as np
import pytest


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _owner(placement, E, G, e):
    if placement == 0:
        return e % G, e // G
    block = (E + G - 1) // G
    return e // block, e - (e // block) * block


@pytest.mark.parametrize("placement", [0, 1])
@pytest.mark.parametrize("E,G", [(128, 2), (128, 8), (10, 3), (256, 8), (7, 7)])
def test_ep_owner_and_plan(gxlib, placement, E, G):
    from galactus_b200.moe import ep_owner, ep_plan
    rng = np.random.default_rng(E * 31 + G)
    for e in range(E):
        assert ep_owner(placement, E, G, e) == _owner(placement, E, G, e)
    T, k = 5, min(8, E)
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    counts, pairs = ep_plan(placement, E, G, ids)
    want = [[i for i in range(T * k) if _owner(placement, E, G, int(ids.flat[i]))[0] == r] for r in range(G)]
    assert counts.tolist() == [len(w) for w in want]
    assert pairs.tolist() == [i for w in want for i in w]


def test_ep_plan_rejects_out_of_domain(gxlib):
    from galactus_b200.moe import ep_plan
    with pytest.raises(gxlib.GxError) as err:
        ep_plan(0, 16, 2, np.array([[1, 16]], np.int32))
    from galactus_b200 import _lib
    assert err.value.code == _lib.GX_ERR_DOMAIN


# ------------------------------------------------- CPU ranks, oracle compute

def _rank_inputs(m, rank, T, seed):
    rng = np.random.default_rng(seed + 1000 * rank)
    k = m.used
    ids = np.stack([rng.choice(m.experts, k, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.random((T, k)).astype(np.float32)
    x = rng.standard_normal((T, m.hidden)).astype(np.float32)
    return x, ids, w


def _gloo_rank(rank, world, port, name, placement, T, result_q):
    import torch
    import torch.distributed as dist

    import galactus_b200 as gx
    from galactus_b200.models import ModelShape
    from galactus_b200.moe import ep_plan
    from oracle import oracle as orc

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        base = gx.MODELS[name]
        m = ModelShape(**{**base.__dict__, "experts": 12, "layers": 1})
        k, H, L = m.used, m.hidden, 0
        x, ids, w = _rank_inputs(m, rank, T, seed=77)
        counts, pairs = ep_plan(placement, m.experts, world, ids)
        # 1. counts and global expert ids to every peer (point to point)
        send_off = np.concatenate([[0], np.cumsum(counts)[:-1]])
        # (gloo has no send to self: a rank's own pairs are copied locally)
        cnt_in = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        reqs = []
        for r in range(world):
            if r == rank:
                cnt_in[r][0] = int(counts[r])
                continue
            reqs.append(dist.isend(torch.tensor([int(counts[r])], dtype=torch.int64), r))
            reqs.append(dist.irecv(cnt_in[r], r))
        for q in reqs:
            q.wait()
        rc = [int(c.item()) for c in cnt_in]
        reqs, ids_in, x_in = [], [], []
        for r in range(world):
            sel = pairs[send_off[r]:send_off[r] + counts[r]]
            ids_out = torch.from_numpy(ids.reshape(-1)[sel].astype(np.int64))
            x_out = torch.from_numpy(np.ascontiguousarray(x[sel // k]))
            if r == rank:
                ids_in.append(ids_out.clone())
                x_in.append(x_out.clone())
                continue
            if counts[r]:
                reqs.append(dist.isend(ids_out, r))
                reqs.append(dist.isend(x_out, r))
            ids_in.append(torch.zeros(rc[r], dtype=torch.int64))
            x_in.append(torch.zeros((rc[r], H), dtype=torch.float32))
            if rc[r]:
                reqs.append(dist.irecv(ids_in[r], r))
                reqs.append(dist.irecv(x_in[r], r))
        for q in reqs:
            q.wait()
        # 2. local compute: one slot per pair, unit weight, on this rank's experts
        ge = np.concatenate([t.numpy() for t in ids_in]).astype(np.int32)
        xr = np.concatenate([t.numpy() for t in x_in]) if len(ge) else np.zeros((0, H), np.float32)
        owned = [e for e in range(m.experts) if (e % world if placement == 0 else e // ((m.experts + world - 1) // world)) == rank]
        local = {e: i for i, e in enumerate(owned)}
        recs_local = np.stack([orc.synth_record(m, m.seed, L, e) for e in owned]) if owned else None
        if len(ge):
            lid = np.array([[local[int(e)]] for e in ge], np.int32)
            y = orc.moe_layer(m, recs_local, xr, lid, np.ones((len(ge), 1), np.float32))
        else:
            y = np.zeros((0, H), np.float32)
        # 3. pair outputs back home, in the order they were sent
        recv_off = np.concatenate([[0], np.cumsum(rc)[:-1]])
        reqs, back = [], []
        for r in range(world):
            y_out = torch.from_numpy(np.ascontiguousarray(y[recv_off[r]:recv_off[r] + rc[r]]))
            if r == rank:
                back.append(y_out.clone())
                continue
            if rc[r]:
                reqs.append(dist.isend(y_out, r))
            back.append(torch.zeros((int(counts[r]), H), dtype=torch.float32))
            if counts[r]:
                reqs.append(dist.irecv(back[r], r))
        for q in reqs:
            q.wait()
        full = np.zeros((T * k, H), np.float32)
        full[pairs] = np.concatenate([b.numpy() for b in back])
        out = orc.combine(full.reshape(T, k, H), w)
        # the one-process layer over all experts
        recs_all = np.stack([orc.synth_record(m, m.seed, L, e) for e in range(m.experts)])
        want = orc.moe_layer(m, recs_all, x, ids, w)
        result_q.put((rank, bool(np.array_equal(out.view(np.uint32), want.view(np.uint32))), int(sum(rc))))
    except Exception as exc:   # report instead of leaving the parent waiting
        result_q.put((rank, False, repr(exc)))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name,placement,world", [("olmoe", 0, 2), ("qwen3-30b", 1, 2), ("gpt-oss-120b", 0, 3)])
def test_ep_decomposition_gloo(gxlib, orc, name, placement, world):
    """World-size-2/3 CPU ranks (gloo): dispatch by gx_ep_plan, per-pair oracle
    FFN on the owning rank, combine at home == the one-process oracle layer."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, world, port, name, placement, 3, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(ok for _, ok, _ in res), res
    assert sum(n for _, _, n in res) == world * 3 * gxlib.MODELS[name].used


# ---------------------------------------------------- GPUs, NCCL, the C-ABI

def _nccl_rank(rank, world, port, name, placement, T, result_q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import galactus_b200 as gx
    from galactus_b200.models import ModelShape
    from galactus_b200.moe import ExpertParallel
    from oracle import oracle as orc

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    ok = False
    try:
        gx.check(gx.lib().gx_device_init(rank))
        base = gx.MODELS[name]
        m = ModelShape(**{**base.__dict__, "experts": 12, "layers": 2})
        owned = [e for e in range(m.experts) if (e % world if placement == 0 else e // ((m.experts + world - 1) // world)) == rank]
        # the local arena: this rank's experts only, every one resident
        lm = ModelShape(**{**m.__dict__, "experts": len(owned), "used": min(m.used, len(owned))})
        # the local arena: this rank's experts, a cache of 4 slots per layer
        # (the owners run the received pairs in waves when they do not fit)
        arena = gx.Arena(lm, capacity_bytes=4 * m.record * m.layers, policy=gx.POLICY_AUTO,
                         max_tokens=world * (T + 2 * world) * m.used, device=rank)
        for L in range(m.layers):
            for li, e in enumerate(owned):
                arena.load_record(L, li, orc.synth_record(m, m.seed, L, e))
        pg = dist.distributed_c10d._get_default_group()
        comm = pg._get_backend(dev)._comm_ptr()
        ep = ExpertParallel(arena, comm, rank, world, m.experts, placement)
        recs = [np.stack([orc.synth_record(m, m.seed, L, e) for e in range(m.experts)]) for L in range(m.layers)]
        stream = torch.cuda.current_stream()
        good = True
        for step in range(3):
            for L in range(m.layers):
                x, ids, w = _rank_inputs(m, rank, T, seed=100 * step + L)
                xd = torch.from_numpy(x).to(dev)
                wd = torch.from_numpy(w).to(dev)
                out = torch.full((T, m.hidden), float("nan"), device=dev)
                ep.layer_forward(L, xd, ids, wd, out, stream)
                got = out.cpu().numpy()
                want = orc.moe_layer(m, recs[L], x, ids, w)
                good = good and bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))
        # both layers in one step, each rank with its own token count
        Tr = T + 1 + 2 * rank
        xs, ids_s, ws = zip(*[_rank_inputs(m, rank, Tr, seed=900 + L) for L in range(m.layers)])
        xd = [torch.from_numpy(v).to(dev) for v in xs]
        wd = [torch.from_numpy(v).to(dev) for v in ws]
        outs = [torch.full((Tr, m.hidden), float("nan"), device=dev) for _ in range(m.layers)]
        ep.stack_forward(0, xd, np.stack(ids_s), wd, outs, stream)
        for L in range(m.layers):
            want = orc.moe_layer(m, recs[L], xs[L], ids_s[L], ws[L])
            good = good and bool(np.array_equal(outs[L].cpu().numpy().view(np.uint32), want.view(np.uint32)))
        # a call that rank 1 rejects (an expert id out of range) fails on every
        # rank with the same status, and the next step runs normally
        bad = np.stack(ids_s).copy()
        if rank == 1:
            bad[0, 0, 0] = m.experts + 5
        rc, _ = ep.stack_forward(0, xd, bad, wd, outs, stream, check=False)
        good = good and rc == gx.GX_ERR_DOMAIN
        ep.stack_forward(0, xd, np.stack(ids_s), wd, outs, stream)
        want = orc.moe_layer(m, recs[1], xs[1], ids_s[1], ws[1])
        good = good and bool(np.array_equal(outs[1].cpu().numpy().view(np.uint32), want.view(np.uint32)))
        from galactus_b200.moe import device_error
        good = good and device_error() == 0
        ep.close()
        arena.close()
        ok = good
    finally:
        result_q.put((rank, ok))
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("name,placement", [("qwen3-30b", 0), ("qwen3-235b", 1)])
def test_ep_nccl_two_gpus(gxlib, name, placement):
    """gx_ep_layer_forward and gx_ep_stack_forward over two GPUs (NCCL
    send/recv on torch's communicator): every rank's outputs are the
    one-process oracle layer's bits, for two layers, three steps, pairs local
    and remote, owners running waves through a 4-slot cache, ranks with
    different token counts; a call one rank rejects fails on both ranks with
    the same status and the next step runs."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 2
    procs = [ctx.Process(target=_nccl_rank, args=(r, world, port, name, placement, 2, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    assert all(ok for _, ok in res), res


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["qwen3-235b", "deepseek-v3"])
def test_ep_one_rank_stack_step(gxlib, orc, dev, name):
    """The expert-parallel step on one GPU (no communicator: the exchanges are
    local copies): gx_ep_stack_forward over three layers through a small slot
    cache (waves) equals the oracle layers bit for bit, and a rejected call
    returns its status and leaves the next step intact."""
    import torch
    from galactus_b200.models import ModelShape
    from galactus_b200.moe import ExpertParallel, device_error
    base = gxlib.MODELS[name]
    m = ModelShape(**{**base.__dict__, "experts": 16, "layers": 3})
    T, k = 4, m.used
    arena = gxlib.Arena(m, capacity_bytes=(k + 2) * m.record * m.layers, policy=gxlib.POLICY_AUTO,
                        max_tokens=T * k)
    try:
        recs = [np.stack([orc.synth_record(m, m.seed, L, e) for e in range(m.experts)]) for L in range(m.layers)]
        for L in range(m.layers):
            for e in range(m.experts):
                arena.load_record(L, e, recs[L][e])
        ep = ExpertParallel(arena, 0, 0, 1, m.experts, 0)
        stream = torch.cuda.current_stream()
        rng = np.random.default_rng(11)
        for step in range(3):
            ids = np.stack([np.stack([rng.choice(m.experts, k, replace=False) for _ in range(T)])
                            for _ in range(m.layers)]).astype(np.int32)
            w = rng.random((m.layers, T, k)).astype(np.float32)
            x = rng.standard_normal((m.layers, T, m.hidden)).astype(np.float32)
            xd, wd = torch.from_numpy(x).to(dev), torch.from_numpy(w).to(dev)
            out = torch.full((m.layers, T, m.hidden), float("nan"), device=dev)
            ep.stack_forward(0, [xd[L] for L in range(m.layers)], ids, [wd[L] for L in range(m.layers)],
                             [out[L] for L in range(m.layers)], stream)
            got = out.cpu().numpy()
            for L in range(m.layers):
                want = orc.moe_layer(m, recs[L], x[L], ids[L], w[L])
                np.testing.assert_array_equal(got[L].view(np.uint32), want.view(np.uint32), err_msg=f"step {step} L {L}")
            if step == 1:
                bad = ids.copy()
                bad[2, 1, 0] = -3
                rc, _ = ep.stack_forward(0, [xd[L] for L in range(m.layers)], bad, [wd[L] for L in range(m.layers)],
                                         [out[L] for L in range(m.layers)], stream, check=False)
                assert rc == gxlib.GX_ERR_DOMAIN
        assert arena.stats()["misses"] > 0
        assert device_error() == 0
        ep.close()
    finally:
        arena.close()
