"""KV-head-sharded decode with the peer exchange (lc_rope_append_decode_peer +
lc_peer_wait) against the same shards decoded by lc_rope_append_decode into one
buffer: every rank's region must hold all heads' rows, bit for bit, and the
pools the same appended rows.

On one GPU two ranks are emulated by one process (lc_peer_group_local over two
regions of this device): each launch's signal is complete before the wait
that reads it is queued, so nothing waits on a kernel running beside it. With
N >= 2 GPUs, N processes (one per GPU) exchange IPC handles and run the real
NVLink path; 2, 4 and 8 ranks are covered where that many GPUs are present.
"""
import ctypes as C
import os
import socket

import numpy as np
import pytest

import lucciola as L
from workloads import from_device, make_case, randn_bf16, to_device

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

HQ, HKV, HD = 32, 8, 128  # 8 kv heads: 1, 2, 4 or 8 per rank
CTX = np.array([0, 15, 300, 2000, 4095, 17, 1023], np.int32)


def _inputs(world, seed=11):
    """Full case plus each rank's slices (pools of its kv heads, qkv rows of
    its q/k/v heads, biases)."""
    rng = np.random.default_rng(seed)
    B = len(CTX)
    case = make_case(B, HQ, HKV, HD, CTX + 1, seed=seed)
    qkv = randn_bf16(rng, (B, (HQ + 2 * HKV) * HD))
    qb, kb, vb = (randn_bf16(rng, (n * HD,)) for n in (HQ, HKV, HKV))
    cos, sin = L.rope_table_host(int(CTX.max()) + 8, HD, 1e6)
    g = HQ // HKV
    shards = []
    for r in range(world):
        f, n = L.shard_kv_heads(HQ, HKV, world, r)
        q_cols = slice(f * g * HD, (f + n) * g * HD)
        k_cols = slice((HQ + f) * HD, (HQ + f + n) * HD)
        v_cols = slice((HQ + HKV + f) * HD, (HQ + HKV + f + n) * HD)
        shards.append({
            "first": f, "n": n, "q_cols": q_cols,
            "qkv": np.ascontiguousarray(np.concatenate(
                [qkv[:, q_cols], qkv[:, k_cols], qkv[:, v_cols]], axis=1)),
            "k_pool": np.ascontiguousarray(case.k_pool[:, :, f:f + n]),
            "v_pool": np.ascontiguousarray(case.v_pool[:, :, f:f + n]),
            "bias": (qb[q_cols], kb[f * HD:(f + n) * HD], vb[f * HD:(f + n) * HD]),
        })
    return case, (cos, sin), shards


class _Rank:
    """Device copies of one rank's shard."""

    def __init__(self, case, rope, sh):
        self.sh = sh
        self.n = sh["n"]
        self.qkv = to_device(sh["qkv"])
        self.k, self.v = to_device(sh["k_pool"]), to_device(sh["v_pool"])
        self.bias = [to_device(b) for b in sh["bias"]]
        self.rope = [to_device(x) for x in rope]
        self.pos, self.tables = to_device(CTX), to_device(case.tables)
        self.ws = L.alloc_decode_workspace(len(CTX), self.n * HQ // HKV, self.n, HD)
        self.status = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.case = case

    def decode(self, out_full, layer, group=None):
        out = out_full[:, self.sh["q_cols"]]
        L.rope_append_decode(out, self.qkv, self.pos, *self.bias, *self.rope, self.k, self.v,
                             self.case.num_blocks, self.case.num_layers, layer,
                             self.n * HQ // HKV, self.n, HD, self.tables,
                             int(CTX.max()) + 1, workspace=self.ws, dev_status=self.status,
                             peer_group=group)


def _region_bytes(slots):
    return L.PEER_SIGNAL_BYTES + slots * len(CTX) * HQ * HD * 2


def _slot(region, s):
    off = L.PEER_SIGNAL_BYTES + s * len(CTX) * HQ * HD * 2
    return region.view(off, (len(CTX), HQ * HD), torch.bfloat16)


@pytest.mark.parametrize("pdl", [0, 2])
def test_peer_decode_two_ranks_on_one_gpu(pdl):
    world = 2
    case, rope, shards = _inputs(world)
    old = L.set_dependent_launch(pdl)
    try:
        ref_ranks = [_Rank(case, rope, sh) for sh in shards]
        peer_ranks = [_Rank(case, rope, sh) for sh in shards]
        regions = [L.PeerRegion(_region_bytes(2)) for _ in range(world)]
        groups = [L.PeerGroup.local(r, world, regions) for r in range(world)]
        try:
            for it, layer in enumerate((1, 0, 1)):
                ref = torch.full((len(CTX), HQ * HD), float("nan"), dtype=torch.bfloat16,
                                 device="cuda")
                for rk in ref_ranks:
                    rk.decode(ref, layer)
                for rk, g in zip(peer_ranks, groups):
                    rk.decode(_slot(regions[g.rank], it % 2), layer, group=g)
                for rk, g in zip(peer_ranks, groups):
                    g.wait(dev_status=rk.status)
                torch.cuda.synchronize()
                for reg in regions:
                    assert torch.equal(_slot(reg, it % 2).view(torch.int16),
                                       ref.view(torch.int16)), f"iteration {it}"
                for a, b in zip(ref_ranks, peer_ranks):
                    assert torch.equal(a.k.view(torch.int16), b.k.view(torch.int16))
                    assert torch.equal(a.v.view(torch.int16), b.v.view(torch.int16))
                    assert int(a.status.item()) == 0 and int(b.status.item()) == 0
                for r, reg in enumerate(regions):
                    w = from_device(reg.signal_words())
                    assert w[1 - r] == it + 1 and w[r] == 0      # the peer's launch count
                    assert w[16] == 0 and w[17] == it + 1 and w[18] == it + 1
        finally:
            for g in groups:
                g.close()
            torch.cuda.synchronize()
            for reg in regions:
                reg.close()
    finally:
        L.set_dependent_launch(old)


def test_peer_decode_batch_of_zero_still_signals():
    case, rope, shards = _inputs(1)
    rk = _Rank(case, rope, shards[0])
    region = L.PeerRegion(_region_bytes(1))
    group = L.PeerGroup.local(0, 1, [region])
    try:
        out = _slot(region, 0)
        p = lambda t: t.data_ptr()  # noqa: E731  (an empty torch slice has a null pointer)
        rc = L.lib.lc_rope_append_decode_peer(
            p(out), out.stride(0), p(rk.qkv), rk.qkv.stride(0), p(rk.pos), *map(p, rk.bias),
            *map(p, rk.rope), rk.rope[0].shape[0], p(rk.k), p(rk.v), case.num_blocks,
            case.num_layers, 1, HQ, HKV, HD, p(rk.tables), rk.tables.stride(0), 0, 0, 0,
            1.0 / HD ** 0.5, p(rk.ws), rk.ws.numel() * rk.ws.element_size(), p(rk.status),
            group.handle, torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        group.wait(dev_status=rk.status)
        torch.cuda.synchronize()
        w = from_device(region.signal_words())
        assert w[16] == 0 and w[17] == 1 and w[18] == 1 and int(rk.status.item()) == 0
    finally:
        group.close()
        torch.cuda.synchronize()
        region.close()


def test_peer_group_rejects_a_region_smaller_than_the_group_size():
    """A region (this rank's or a peer's) with less room than region_bytes
    would let the decode store past a peer's allocation: refused up front."""
    region = L.PeerRegion(1 << 20)
    try:
        arr = (C.c_void_p * 1)(region.ptr)
        g = C.c_void_p()
        rc = L.lib.lc_peer_group_local(0, 1, arr, 64 << 20, C.byref(g))
        assert rc == 1 and not g.value  # LC_ERR_INVALID_ARGUMENT, no group
        # a region starting 4 KiB before the end of its allocation
        arr2 = (C.c_void_p * 1)(region.ptr + (1 << 20) - 4096)
        assert L.lib.lc_peer_group_local(0, 1, arr2, 8192, C.byref(g)) == 1
        assert L.lib.lc_peer_group_local(0, 1, arr2, 4096, C.byref(g)) == 0
        L.lib.lc_peer_group_destroy(g)
        rc = L.lib.lc_peer_group_open(0, 1, region.ptr, 64 << 20, region.handle, C.byref(g))
        assert rc == 1
    finally:
        region.close()


def test_peer_wait_gives_up_and_the_context_stays_usable():
    """Rank 0 of a two-rank group waits for a peer that never launches: the
    wait stops after its 2 s limit with LC_DEV_TIMEOUT in the status word,
    its wait count still advances (so later waits stay paired with later
    launches), and the GPU keeps working."""
    world = 2
    case, rope, shards = _inputs(world)
    rk = _Rank(case, rope, shards[0])
    regions = [L.PeerRegion(_region_bytes(1)) for _ in range(world)]
    group = L.PeerGroup.local(0, world, regions)
    try:
        out = torch.full((len(CTX), HQ * HD), float("nan"), dtype=torch.bfloat16, device="cuda")
        rk.decode(_slot(regions[0], 0), 1, group=group)  # rank 1 never runs
        group.wait(dev_status=rk.status)
        torch.cuda.synchronize()
        assert int(rk.status.item()) & L.LC_DEV_TIMEOUT
        w = from_device(regions[0].signal_words())
        assert w[1] == 0 and w[18] == 1  # nothing from rank 1; the wait counted itself
        assert from_device(regions[1].signal_words())[0] == 1  # rank 0 did signal rank 1
        # the context still runs kernels: the same shard without the exchange
        ok = _Rank(case, rope, shards[0])
        ok.decode(out, 1)
        torch.cuda.synchronize()
        assert int(ok.status.item()) == 0
        mine = from_device(out[:, shards[0]["q_cols"]].contiguous())
        assert np.array_equal(mine, from_device(_slot(regions[0], 0)[:, shards[0]["q_cols"]]
                                                .contiguous()))
    finally:
        group.close()
        torch.cuda.synchronize()
        for reg in regions:
            reg.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gpu_worker(rank, world, port, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root), str(root / "lucciola-rs_b200"), str(root / "tests")]
    import datetime

    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    ok, msg = False, ""
    try:
        import lucciola as L
        case, rope, shards = _inputs(world)
        ref_rank, peer_rank = _Rank(case, rope, shards[rank]), _Rank(case, rope, shards[rank])
        region = L.PeerRegion(_region_bytes(2))
        handles = [None] * world
        dist.all_gather_object(handles, region.handle)
        group = L.PeerGroup.open(rank, world, region, handles)
        L.set_dependent_launch(2)
        try:
            for it, layer in enumerate((1, 0, 1, 0)):
                ref = torch.zeros((len(CTX), HQ * HD), dtype=torch.bfloat16, device="cuda")
                ref_rank.decode(ref, layer)
                torch.cuda.synchronize()
                dist.barrier()  # both ranks launch their peer decode together
                peer_rank.decode(_slot(region, it % 2), layer, group=group)
                group.wait(dev_status=peer_rank.status)
                torch.cuda.synchronize()
                # all ranks' reference shards, assembled on the host
                mine = from_device(ref[:, shards[rank]["q_cols"]])
                parts = [None] * world
                dist.all_gather_object(parts, mine)
                full = np.concatenate(parts, axis=1)
                got = from_device(_slot(region, it % 2))
                if not np.array_equal(got, full):
                    msg = f"iteration {it}: {int((got != full).sum())} elements differ"
                elif int(peer_rank.status.item()) != 0:
                    msg = f"iteration {it}: status {int(peer_rank.status.item())}"
                verdicts = [None] * world
                dist.all_gather_object(verdicts, msg)  # every rank stops at the same point
                if any(verdicts):
                    msg = msg or "a peer failed"
                    break
            else:
                ok = True
        finally:
            torch.cuda.synchronize()
            dist.barrier()
            group.close()
            dist.barrier()
            region.close()
    finally:
        dist.destroy_process_group()
    q.put((rank, ok, msg))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_decode_processes_over_nvlink(world):
    """One process per GPU: every rank's region ends up with all ranks' rows,
    bit for bit, over four layers in a row."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_gpu_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    results = sorted(q.get() for _ in range(world))
    assert all(ok for _, ok, _ in results), results
