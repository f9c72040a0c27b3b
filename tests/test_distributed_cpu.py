"""Multi-GPU host logic on CPU ranks (gloo, world size 2): sequence sharding
(no collective on the data path) and KV-head sharding with
an all-gather of per-head outputs (config 5). Each rank computes its shard with
the CPU oracle; the reassembled result must equal the unsharded one bit for bit.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup(rank, port):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "lucciola-rs_b200"), str(root / "tests")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)


def _sequence_shard_worker(rank, port, q):
    _setup(rank, port)
    try:
        import lucciola as L
        import oracle.oracle as O
        from workloads import make_case
        rng = np.random.default_rng(7)
        ctx = rng.integers(1, 600, 12).astype(np.int32)
        case = make_case(12, 14, 2, 64, ctx, seed=7)
        owner = np.array(L.shard_sequences(ctx.tolist(), WORLD))
        mine = np.nonzero(owner == rank)[0]
        out = O.paged_decode(case.q[mine], case.k_pool, case.v_pool, case.layer, 14, 2, 64,
                             case.tables[mine], ctx[mine], case.num_layers)
        parts = [None] * WORLD
        dist.all_gather_object(parts, (mine.tolist(), out))
        if rank == 0:
            full = np.zeros((12, 14 * 64), np.uint16)
            for idx, o in parts:
                full[idx] = o
            ref = O.paged_decode(case.q, case.k_pool, case.v_pool, case.layer, 14, 2, 64,
                                 case.tables, ctx, case.num_layers)
            loads = [int(ctx[owner == r].sum()) for r in range(WORLD)]
            q.put(("seq", bool(np.array_equal(full, ref)), loads))
    finally:
        dist.destroy_process_group()


def _head_shard_worker(rank, port, q):
    _setup(rank, port)
    try:
        import lucciola as L
        import oracle.oracle as O
        from workloads import make_case
        hq, hkv, hd, B = 16, 4, 64, 5
        ctx = np.array([33, 1, 200, 64, 129], np.int32)
        case = make_case(B, hq, hkv, hd, ctx, seed=3)
        first, nloc = L.shard_kv_heads(hq, hkv, WORLD, rank)
        grp = hq // hkv
        # this rank's pools hold only its kv heads; identical block tables everywhere
        kp = np.ascontiguousarray(case.k_pool[:, :, first:first + nloc])
        vp = np.ascontiguousarray(case.v_pool[:, :, first:first + nloc])
        qh = case.q.reshape(B, hq, hd)[:, first * grp:(first + nloc) * grp].reshape(B, -1)
        out = O.paged_decode(np.ascontiguousarray(qh), kp, vp, case.layer, nloc * grp, nloc, hd,
                             case.tables, ctx, case.num_layers)
        # bf16 pairs travel as int32 (gloo has no 16-bit integer type)
        mine = torch.from_numpy(np.ascontiguousarray(out).view(np.int32).copy())
        gathered = [torch.empty_like(mine) for _ in range(WORLD)]
        dist.all_gather(gathered, mine)
        if rank == 0:
            full = L.assemble_head_shards(torch.cat(gathered, 0), WORLD).contiguous().numpy()
            full = full.view(np.uint16)
            ref = O.paged_decode(case.q, case.k_pool, case.v_pool, case.layer, hq, hkv, hd,
                                 case.tables, ctx, case.num_layers)
            q.put(("head", bool(np.array_equal(full, ref)), None))
    finally:
        dist.destroy_process_group()


def _head_shard_tables_worker(rank, port, q):
    """KV-head sharding keeps one pool per rank with identical block tables: every
    rank issues the same allocator calls (no table traffic), and a fingerprint
    all-reduce confirms the agreement; a rank that diverges is caught."""
    _setup(rank, port)
    try:
        import lucciola as L
        first, nloc = L.shard_kv_heads(64, 8, WORLD, rank)
        blocks = L.pool_blocks_for_budget(80, nloc, 128, 170 << 30, 183359 << 20, 0.9)
        a = L.BlockAlloc(2000, 16, 512)
        rng = np.random.default_rng(5)  # the scheduler's decisions, the same on every rank
        live = []
        for _ in range(300):
            if len(live) < 16 and rng.random() < 0.3:
                live.append(a.add())
            elif live and rng.random() < 0.1:
                s = live.pop(int(rng.integers(0, len(live))))
                a.release(s)
            elif live:
                s = live[int(rng.integers(0, len(live)))]
                try:
                    a.reserve(s, len(a.pages(s)) * 16 + int(rng.integers(1, 64)))
                except L.LucciolaError:
                    pass

        def agree():
            f = torch.tensor([a.fingerprint() & 0x7FFFFFFFFFFFFFFF], dtype=torch.int64)
            lo, hi = f.clone(), f.clone()
            dist.all_reduce(lo, op=dist.ReduceOp.MIN)
            dist.all_reduce(hi, op=dist.ReduceOp.MAX)
            return bool(lo.item() == hi.item())

        tables = [None] * WORLD
        dist.all_gather_object(tables, {s: a.pages(s) for s in live})
        same_before = agree()
        if rank == 1 and live:
            s = live[0]
            a.reserve(s, len(a.pages(s)) * 16 + 1)  # one page more on one rank only
        same_after = agree()
        sizes = [None] * WORLD
        dist.all_gather_object(sizes, (first, nloc, blocks))
        if rank == 0:
            ok = (same_before and not same_after and tables[0] == tables[1]
                  and len({x[2] for x in sizes}) == 1 and sizes[0][2] > 0)
            q.put(("tables", ok, None))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("worker", [_sequence_shard_worker, _head_shard_worker,
                                    _head_shard_tables_worker])
def test_sharded_decode_equals_unsharded(worker):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    kind, equal, loads = q.get()
    assert equal, f"{kind}-sharded result differs from the unsharded oracle"
    if loads is not None:  # longest-first packing keeps the two ranks within one sequence
        assert abs(loads[0] - loads[1]) <= 600
