"""Expert parallelism: the dispatch plan (host form of the device kernels of
qmoe_forward_ep), a two-rank exchange of that plan over gloo on the CPU, and
on two GPUs the collective forward itself against the C restatement.

Rank g of W owns experts [g E/W, (g+1) E/W); each rank routes its own
tokens, sends each token once to every rank that owns one of its experts,
and gets one combined partial row per (token, rank) back: the
expert-parallel layout of the workload's prefill and batched-decode
configurations."""
import ctypes as C
import os
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _plan(idx, E, W, cap):
    import qmoe
    idx = np.ascontiguousarray(idx, np.int32)
    n, k = idx.shape
    counts = np.zeros(W, np.int32)
    pos = np.zeros(W * n, np.int32)
    rc = qmoe.lib().qmoe_ep_plan_host(idx.ctypes.data, n, k, E, W, cap, counts.ctypes.data,
                                      pos.ctypes.data)
    assert rc == 0
    return counts, pos.reshape(W, n)


def test_plan_sends_each_token_once_per_owner_rank(built):
    rng = np.random.default_rng(7)
    E, W, n, k, cap = 64, 4, 50, 6, 56
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(n)]).astype(np.int32)
    counts, pos = _plan(idx, E, W, cap)
    owner = idx // (E // W)
    goes = np.stack([(owner == g).any(1) for g in range(W)])      # [W, n]
    assert counts.tolist() == goes.sum(1).tolist()
    assert np.array_equal(pos >= 0, goes)
    for g in range(W):                                             # row t of block g
        t = np.nonzero(goes[g])[0]
        assert pos[g][t].tolist() == (g * cap + t).tolist()


def test_plan_rejects_bad_arguments(built):
    import qmoe
    idx = np.zeros((2, 2), np.int32)
    counts = np.zeros(4, np.int32)
    f = qmoe.lib().qmoe_ep_plan_host
    assert f(idx.ctypes.data, 2, 2, 10, 4, 2, counts.ctypes.data, None) == -1   # E % W
    assert f(idx.ctypes.data, 2, 2, 16, 4, 1, counts.ctypes.data, None) == -1   # cap < n
    bad = np.array([[0, 99]], np.int32)
    assert f(bad.ctypes.data, 1, 2, 16, 4, 1, counts.ctypes.data, None) == -1   # expert id


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _gloo_rank(rank, world, port, result):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "qwen3.8-flash-next_b200"))
    import torch
    import torch.distributed as dist

    import oracle
    import qmoe
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        d, E, k, I = 256, 16, 4, 128
        cfg = qmoe.make_config(d, E, k, I, max_tokens=32)
        s = qmoe.SynthLayer(cfg, 20261201)
        x = qmoe.synth_tokens(20261201, 40 + rank, 12 + 5 * rank, d)   # ranks differ in n
        idx, w, _ = oracle.restatement().route(s, x)
        cap = 32                                                     # rows per rank pair
        counts, pos = _plan(idx, E, world, cap)
        # the fixed-size exchange: cap rows to every rank, each sent row
        # with the token's slots (other ranks' experts as -1), unused rows
        # all -1
        n, k = idx.shape
        send_e = np.full((world * cap, k), -1, np.int32)
        for g in range(world):
            for t in range(n):
                if pos[g, t] >= 0:
                    own = idx[t] // (E // world) == g
                    send_e[pos[g, t]] = np.where(own, idx[t], -1)
        recv_e = torch.zeros((world * cap, k), dtype=torch.int32)
        dist.all_to_all_single(recv_e, torch.from_numpy(send_e))
        # every row received is for one of this rank's experts, and the rows
        # received are exactly every rank's assignments to those experts
        all_idx = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(all_idx, torch.tensor([idx.size]))
        mx = max(int(t) for t in all_idx)   # gloo gathers equal sizes: pad with -1
        padded = np.full(mx, -1, np.int32)
        padded[:idx.size] = idx.ravel()
        gathered = [torch.zeros(mx, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(padded))
        every = np.concatenate([g.numpy() for g in gathered])
        every = every[every >= 0]
        lo, hi = rank * E // world, (rank + 1) * E // world
        got = recv_e.numpy().ravel()
        got = got[got >= 0]
        ok = bool(np.all((got >= lo) & (got < hi)))
        ok = ok and np.bincount(got, minlength=E)[lo:hi].tolist() == \
            np.bincount(every, minlength=E)[lo:hi].tolist()
        result[rank] = ok
    finally:
        dist.destroy_process_group()


def test_two_rank_dispatch_over_gloo(built):
    """World size 2 on the CPU (gloo): each rank routes its own tokens with
    the C restatement, plans its dispatch with the library's host plan, and
    after the fixed-size exchange every expert id received is one of the
    rank's own and the ids received are exactly every rank's assignments to
    those experts."""
    import torch.multiprocessing as mp
    world = 2
    # the manager's server process is spawned, not forked from this
    # (multi-threaded) test process
    with mp.get_context("spawn").Manager() as m:
        result = m.dict()
        mp.spawn(_gloo_rank, args=(world, _free_port(), result), nprocs=world, join=True)
        assert dict(result) == {0: True, 1: True}


def _ep_rank(rank, world, uid_q, out_q, T_per, exchange="p2p"):
    import sys
    if exchange == "nccl":
        os.environ["QMOE_EP_P2P"] = "0"
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "qwen3.8-flash-next_b200"))
    import torch

    import qmoe
    torch.cuda.set_device(rank)
    d, E, k, I = 2048, 512, 10, 512
    cfg = qmoe.make_config(d, E, k, I, max_tokens=T_per, device=rank, ep_rank=rank,
                           ep_world=world)
    s = qmoe.SynthLayer(cfg, 20261201, zipf_s=1.1)
    ctx = qmoe.Context(cfg)
    ctx.upload(0, s)
    if rank == 0:
        uid = qmoe.ep_unique_id()
        for _ in range(world - 1):
            uid_q.put(uid)
    else:
        uid = uid_q.get(timeout=120)
    ctx.ep_connect(uid)
    x = qmoe.synth_tokens(20261201, 60 + rank, T_per, d)
    xd = torch.from_numpy(x).cuda().to(torch.bfloat16)
    out = torch.empty((T_per, d), dtype=torch.float32, device="cuda")
    for _ in range(2):   # twice: the second call reuses every buffer
        ctx.forward_ep(0, xd.data_ptr(), qmoe.QMOE_BF16, T_per, out.data_ptr(), None)
        ctx.sync()
    idx, _, _ = ctx.routing(T_per)
    import ctypes
    p2p = qmoe.lib().qmoe__ep_p2p
    p2p.restype, p2p.argtypes = ctypes.c_int, [ctypes.c_void_p]
    out_q.put((rank, out.cpu().numpy(), idx, int(p2p(ctx.h))))
    ctx.close()


@pytest.mark.gpu
@pytest.mark.parametrize("exchange", ["p2p", "nccl"])
def test_expert_parallel_forward_two_gpus(built, exchange):
    """Two GPUs, one process each, the exchanges through peer memory (the
    default where the GPUs have peer access) or NCCL (QMOE_EP_P2P=0): every
    token's routing equals the restatement's and a spread sample of outputs
    is within the parity tolerance (the same bars as the one-GPU path)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    import oracle
    import qmoe
    world, T_per = 2, 256
    ctx = mp.get_context("spawn")
    uid_q, out_q = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_ep_rank, args=(r, world, uid_q, out_q, T_per, exchange))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    modes = set()
    try:
        for _ in range(world):
            r, out, idx, p2p = out_q.get(timeout=600)
            results[r] = (out, idx)
            modes.add(p2p)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    if exchange == "nccl":
        assert modes == {0}
    elif torch.cuda.can_device_access_peer(0, 1):
        assert modes == {1}
    cfg = qmoe.make_config(2048, 512, 10, 512, max_tokens=T_per)
    s = qmoe.SynthLayer(cfg, 20261201, zipf_s=1.1)
    for r in range(world):
        out, idx = results[r]
        x = qmoe.synth_tokens(20261201, 60 + r, T_per, 2048)
        sample = np.linspace(0, T_per - 1, 12).astype(int)
        ro, ri, _ = oracle.restatement().forward(s, x[sample])
        assert np.array_equal(idx[sample], ri)
        mab = float(np.abs(out[sample] - ro).max())
        rr = float(np.linalg.norm(out[sample] - ro) / np.linalg.norm(ro))
        assert mab <= 2e-2 and rr <= 1e-3, (r, mab, rr)


def _ep_stack_rank(rank, world, uid_q, out_q, T_per, n_layers):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "qwen3.8-flash-next_b200"))
    import torch

    import qmoe
    torch.cuda.set_device(rank)
    d, E, k, I = 2048, 512, 10, 512
    cfg = qmoe.make_config(d, E, k, I, layers=n_layers, max_tokens=T_per, device=rank,
                           ep_rank=rank, ep_world=world)
    ctx = qmoe.Context(cfg)
    for l in range(n_layers):
        ctx.upload(l, qmoe.SynthLayer(cfg, 20261202, l))
    if rank == 0:
        uid = qmoe.ep_unique_id()
        for _ in range(world - 1):
            uid_q.put(uid)
    else:
        uid = uid_q.get(timeout=120)
    ctx.ep_connect(uid)
    h = torch.from_numpy(qmoe.synth_tokens(20261202, 70 + rank, T_per, d)).cuda()
    # captured as one graph, as the benchmark runs it
    st = torch.cuda.Stream()
    ctx.capture_begin(st.cuda_stream)
    ctx.forward_stack(0, n_layers, h.data_ptr(), T_per, 1e-6, st.cuda_stream)
    g = ctx.capture_end(st.cuda_stream)
    g.launch(st.cuda_stream)
    st.synchronize()
    ctx.sync()
    g.close()
    out_q.put((rank, h.cpu().numpy()))
    ctx.close()


@pytest.mark.gpu
def test_expert_parallel_stack_two_gpus(built):
    """Two GPUs: a two-layer MoE-only stack (RMSNorm + MoE + residual), every
    layer expert-parallel and the whole stack one captured graph per rank,
    against the restatement composed layer by layer."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    import qmoe
    from test_stack import compose
    world, T_per, n_layers = 2, 32, 2
    ctx = mp.get_context("spawn")
    uid_q, out_q = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_ep_stack_rank, args=(r, world, uid_q, out_q, T_per, n_layers))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r, h = out_q.get(timeout=600)
            results[r] = h
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    cfg = qmoe.make_config(2048, 512, 10, 512, layers=n_layers, max_tokens=T_per)
    layers = [qmoe.SynthLayer(cfg, 20261202, l) for l in range(n_layers)]
    for r in range(world):
        h0 = qmoe.synth_tokens(20261202, 70 + r, T_per, 2048)
        ref, _ = compose(layers, h0)
        delta, rdelta = results[r] - h0, ref - h0   # relative RMS: see test_stack._check
        rr = float(np.linalg.norm(delta - rdelta) / np.linalg.norm(rdelta))
        assert rr <= 1e-3, (r, rr)


def _ep_stream_rank(rank, world, uid_q, out_q, n_layers, pool_slots):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "qwen3.8-flash-next_b200"))
    import torch

    import qmoe
    torch.cuda.set_device(rank)
    d, E, k, I = 2048, 512, 10, 512
    T_per = 8
    slot = qmoe.lib().qmoe_slot_bytes(qmoe.make_config(d, E, k, I))
    outs = []
    for pool in (0, pool_slots):   # resident, then streaming from the pinned host store
        cfg = qmoe.make_config(d, E, k, I, layers=n_layers, max_tokens=T_per, device=rank,
                               ep_rank=rank, ep_world=world, prefetch=2,
                               pool_bytes=pool * slot)
        ctx = qmoe.Context(cfg)
        for l in range(n_layers):
            ctx.synth_layer_dev(l, 20261203, 1.1)
        if rank == 0:
            uid = qmoe.ep_unique_id()
            for _ in range(world - 1):
                uid_q.put(uid)
        else:
            uid = uid_q.get(timeout=120)
        ctx.ep_connect(uid)
        st = torch.cuda.Stream()
        res = []
        # every rank with tokens, then the batch-1 decode form (rank 0 only)
        for n in (T_per, 1 if rank == 0 else 0):
            h = torch.from_numpy(qmoe.synth_tokens(20261203, 80 + rank, T_per, d)).cuda()
            torch.cuda.synchronize()
            ctx.forward_stack(0, n_layers, h.data_ptr(), n, 1e-6, st.cuda_stream)
            st.synchronize()
            res.append(h[:n].cpu().numpy())
        ctx.sync()
        s = ctx.stats()
        outs.append((res, int(s["expert_loads"]), int(s["routed_lookups"])))
        ctx.close()
    out_q.put((rank, outs))


@pytest.mark.gpu
def test_expert_parallel_streaming_stack_two_gpus(built):
    """Two GPUs, expert-parallel, each rank streaming its own experts from a
    pinned host store into a small pool: the stack's outputs equal the
    resident expert-parallel stack's bit for bit, for a call with tokens on
    both ranks and for the batch-1 decode form (the token on rank 0, rank 1
    serving its experts with no tokens of its own)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    world, n_layers = 2, 3
    ctx = mp.get_context("spawn")
    uid_q, out_q = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_ep_stream_rank, args=(r, world, uid_q, out_q, n_layers, 128))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r, o = out_q.get(timeout=600)
            results[r] = o
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    for r in range(world):
        (res_a, loads_a, _), (res_b, loads_b, lookups_b) = results[r]
        assert loads_a == 0 and loads_b > 0 and lookups_b > 0, (r, loads_a, loads_b, lookups_b)
        for a, b in zip(res_a, res_b):
            assert a.shape == b.shape and np.array_equal(a, b), r
