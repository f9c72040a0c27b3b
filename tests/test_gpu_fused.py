"""lc_rope_append_decode (one launch) against lc_rope_append + lc_paged_decode
(two launches) and against the CPU oracle: identical pool writes and attention
outputs; the fused form leaves the qkv rows unmodified."""
import numpy as np
import pytest

import lucciola as L
import oracle.oracle as O
from conftest import ATTN_ATOL
from workloads import from_device, make_case, randn_bf16, to_device

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def run_both(hq, hkv, hd, ctx, seed, partition_tokens=0):
    rng = np.random.default_rng(seed)
    ctx = np.asarray(ctx, np.int32)
    B = len(ctx)
    case = make_case(B, hq, hkv, hd, ctx + 1, seed=seed)  # room for the new token
    row = (hq + 2 * hkv) * hd + 16
    qkv = randn_bf16(rng, (B, row))
    qb, kb, vb = (randn_bf16(rng, (n * hd,)) for n in (hq, hkv, hkv))
    cos, sin = O.rope_table(int(ctx.max()) + 8, hd, 1e6)
    dev = [to_device(x) for x in (qb, kb, vb, cos, sin, ctx, case.tables)]
    ws = L.alloc_decode_workspace(B, hq, hkv, hd)

    # two launches
    qkv_a, ka, va = to_device(qkv), to_device(case.k_pool), to_device(case.v_pool)
    out_a = torch.empty(B, hq * hd, dtype=torch.bfloat16, device="cuda")
    L.rope_append(qkv_a, dev[5], dev[0], dev[1], dev[2], dev[3], dev[4], ka, va, case.num_blocks,
                  case.num_layers, case.layer, hq, hkv, hd, dev[6])
    L.paged_decode(out_a, qkv_a, ka, va, case.num_blocks, case.num_layers, case.layer, hq, hkv, hd,
                   dev[6], dev[5], int(ctx.max()) + 1, len_offset=1,
                   partition_tokens=partition_tokens, workspace=ws)
    # one launch
    qkv_b, kb_, vb_ = to_device(qkv), to_device(case.k_pool), to_device(case.v_pool)
    out_b = torch.empty(B, hq * hd, dtype=torch.bfloat16, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.rope_append_decode(out_b, qkv_b, dev[5], dev[0], dev[1], dev[2], dev[3], dev[4], kb_, vb_,
                         case.num_blocks, case.num_layers, case.layer, hq, hkv, hd, dev[6],
                         int(ctx.max()) + 1, partition_tokens=partition_tokens, workspace=ws,
                         dev_status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    return case, qkv, (qb, kb, vb, cos, sin), (qkv_a, ka, va, out_a), (qkv_b, kb_, vb_, out_b)


@pytest.mark.parametrize("hq,hkv,hd", [(14, 2, 64), (28, 4, 128), (12, 2, 128), (64, 8, 128),
                                       (32, 2, 64), (8, 8, 64)])
def test_fused_equals_two_launches_and_oracle(hq, hkv, hd):
    ctx = [0, 15, 16, 31, 300, 511, 1023, 2000]
    case, qkv, bias, a, b = run_both(hq, hkv, hd, ctx, seed=hq + hd)
    for x, y in zip(a[1:], b[1:]):  # pools and outputs
        assert torch.equal(x.view(torch.int16), y.view(torch.int16))
    assert np.array_equal(from_device(b[0]), qkv)  # qkv only read
    # oracle: rope -> append -> attention over positions 0..ctx inclusive
    qb, kb, vb, cos, sin = bias
    q2 = qkv.copy()
    O.rope_append(q2, np.asarray(ctx, np.int32), qb, kb, vb, cos, sin, case.k_pool, case.v_pool,
                  case.num_layers, case.layer, hq, hkv, hd, case.tables)
    assert np.array_equal(from_device(a[0]), q2)
    ref = O.paged_decode(q2, case.k_pool, case.v_pool, case.layer, hq, hkv, hd, case.tables,
                         np.asarray(ctx, np.int32), case.num_layers, len_offset=1, threads=8)
    got = O.bf16_to_f32(from_device(b[3]))
    assert float(np.abs(got - O.bf16_to_f32(ref)).max()) <= ATTN_ATOL


@pytest.mark.parametrize("ptok", [16, 64])
def test_fused_new_token_page_owned_by_a_later_cta(ptok):
    """Small partitions: the page holding the new token belongs to a CTA that
    does not own the segment's first page; every CTA rotates q itself."""
    case, qkv, bias, a, b = run_both(28, 4, 128, [4095, 1040, 17], seed=ptok, partition_tokens=ptok)
    for x, y in zip(a[1:], b[1:]):
        assert torch.equal(x.view(torch.int16), y.view(torch.int16))


@pytest.mark.parametrize("mode", [1, 2])
def test_dependent_launch_modes_give_identical_results(mode):
    """Back-to-back fused decode launches of several layers, eager and captured
    in a CUDA graph, with programmatic dependent launch on: same outputs and
    pools as plain launches."""
    hq, hkv, hd, layers = 14, 2, 64, 3
    rng = np.random.default_rng(mode)
    ctx = rng.integers(1, 3000, 24).astype(np.int32)
    case = make_case(24, hq, hkv, hd, ctx + 1, num_layers=layers, layer=0, seed=mode)
    row = (hq + 2 * hkv) * hd
    qkv = to_device(randn_bf16(rng, (layers, 24, row)))
    qb, kb, vb = (to_device(randn_bf16(rng, (n * hd,))) for n in (hq, hkv, hkv))
    cos, sin = (to_device(x) for x in O.rope_table(4096, hd, 1e6))
    pos, tables = to_device(ctx), to_device(case.tables)
    ws = L.alloc_decode_workspace(24, hq, hkv, hd)

    def run(m, graph):
        kp, vp = to_device(case.k_pool), to_device(case.v_pool)
        out = torch.zeros(layers, 24, hq * hd, dtype=torch.bfloat16, device="cuda")
        old = L.set_dependent_launch(m)
        try:
            def step():
                for l in range(layers):
                    L.rope_append_decode(out[l], qkv[l], pos, qb, kb, vb, cos, sin, kp, vp,
                                         case.num_blocks, layers, l, hq, hkv, hd, tables,
                                         int(ctx.max()) + 1, workspace=ws)
            if graph:
                step()  # warm-up outside capture
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                s = torch.cuda.Stream()
                with torch.cuda.graph(g, stream=s):
                    step()
                g.replay()
                g.replay()
            else:
                step()
            torch.cuda.synchronize()
        finally:
            L.set_dependent_launch(old)
        return out, kp, vp

    base = run(0, False)
    for graph in (False, True):
        got = run(mode, graph)
        for x, y in zip(base, got):
            assert torch.equal(x.view(torch.int16), y.view(torch.int16))


def _gated_case(seed):
    hq, hkv, hd, B = 14, 2, 64, 12
    rng = np.random.default_rng(seed)
    ctx = rng.integers(1, 2000, B).astype(np.int32)
    case = make_case(B, hq, hkv, hd, ctx + 1, seed=seed)
    row = (hq + 2 * hkv) * hd
    d = dict(qkv=to_device(randn_bf16(rng, (B, row))), pos=to_device(ctx),
             tables=to_device(case.tables), ws=L.alloc_decode_workspace(B, hq, hkv, hd))
    d["qb"], d["kb"], d["vb"] = (to_device(randn_bf16(rng, (n * hd,))) for n in (hq, hkv, hkv))
    d["cos"], d["sin"] = (to_device(x) for x in O.rope_table(4096, hd, 1e6))
    return case, d, (hq, hkv, hd, B, int(ctx.max()) + 1)


def _decode(case, d, shape, out, gate=None, status=None):
    hq, hkv, hd, B, max_ctx = shape
    kp, vp = to_device(case.k_pool), to_device(case.v_pool)
    L.rope_append_decode(out, d["qkv"], d["pos"], d["qb"], d["kb"], d["vb"], d["cos"], d["sin"],
                         kp, vp, case.num_blocks, case.num_layers, case.layer, hq, hkv, hd,
                         d["tables"], max_ctx, workspace=d["ws"], dev_status=status, gate=gate)
    return kp, vp


def test_gated_decode_to_host_memory_equals_plain():
    """lc_rope_append_decode_gated: an open gate and outputs written into mapped
    pinned host memory give the plain launch's outputs and pools bit for bit."""
    import ctypes
    from cuda.bindings import runtime as cudart
    case, d, shape = _gated_case(1)
    hq, hkv, hd, B, _ = shape
    out_a = torch.empty(B, hq * hd, dtype=torch.bfloat16, device="cuda")
    ka, va = _decode(case, d, shape, out_a)
    nbytes = B * hq * hd * 2
    err, hptr = cudart.cudaHostAlloc(nbytes, cudart.cudaHostAllocMapped)
    assert int(err) == 0
    try:
        out_h = torch.frombuffer((ctypes.c_uint8 * nbytes).from_address(int(hptr)),
                                 dtype=torch.bfloat16).view(B, hq * hd)
        gate = torch.ones(1, dtype=torch.int32, device="cuda")
        st = torch.zeros(1, dtype=torch.int32, device="cuda")
        kb_, vb_ = _decode(case, d, shape, out_h, gate=gate, status=st)
        torch.cuda.synchronize()
        assert int(st.item()) == 0
        assert torch.equal(out_a.cpu().view(torch.int16), out_h.view(torch.int16))
        assert torch.equal(ka.view(torch.int16), kb_.view(torch.int16))
        assert torch.equal(va.view(torch.int16), vb_.view(torch.int16))
    finally:
        torch.cuda.synchronize()
        cudart.cudaFreeHost(hptr)


def test_gate_opened_late_by_a_copy():
    """The launch waits on the device for a gate that a copy on another stream
    opens later (issued by the host after a pause); same result as plain."""
    import time
    case, d, shape = _gated_case(2)
    hq, hkv, hd, B, _ = shape
    out_a = torch.empty(B, hq * hd, dtype=torch.bfloat16, device="cuda")
    _decode(case, d, shape, out_a)
    torch.cuda.synchronize()
    gate = torch.zeros(1, dtype=torch.int32, device="cuda")
    one = torch.ones(1, dtype=torch.int32).pin_memory()
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    out_b = torch.empty(B, hq * hd, dtype=torch.bfloat16, device="cuda")
    _decode(case, d, shape, out_b, gate=gate, status=st)
    time.sleep(0.05)  # the launch is waiting on the device by now
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        gate.copy_(one, non_blocking=True)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert torch.equal(out_a.view(torch.int16), out_b.view(torch.int16))


def test_gate_never_opened_times_out_with_status():
    """A gate nothing opens: the bounded wait gives up (2 s), the launch
    returns with LC_DEV_TIMEOUT in the status word, and the context stays
    usable: after the workspace is zeroed again (the aborted launch may leave
    arrival counters set) the next launches are exact."""
    case, d, shape = _gated_case(3)
    hq, hkv, hd, B, _ = shape
    gate = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty(B, hq * hd, dtype=torch.bfloat16, device="cuda")
    _decode(case, d, shape, out, gate=gate, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) & L.LC_DEV_TIMEOUT
    d["ws"].zero_()
    out_a = torch.empty(B, hq * hd, dtype=torch.bfloat16, device="cuda")
    out_c = torch.empty(B, hq * hd, dtype=torch.bfloat16, device="cuda")
    _decode(case, d, shape, out_a)
    _decode(case, d, shape, out_c, gate=torch.ones(1, dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    assert torch.equal(out_a.view(torch.int16), out_c.view(torch.int16))
