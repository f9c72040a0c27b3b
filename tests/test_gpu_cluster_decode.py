"""Single-sequence decode (lc_rope_append_decode and lc_paged_decode with batch 1), which
splits each segment's pages over a thread-block cluster and merges the pieces
in rank 0's shared memory: pool writes bit-identical to lc_rope_append, the
qkv rows untouched, outputs against the CPU oracle and against the batched
two-launch path (lc_rope_append + lc_paged_decode). Covers clusters of 2 to
16 CTAs, GQA groups above 8 (two segments per kv head), and a context-length
hint far above the real length, which leaves the higher ranks of each
cluster without pages."""
import numpy as np
import pytest

import lucciola as L
import oracle.oracle as O
from conftest import ATTN_ATOL
from workloads import from_device, make_case, randn_bf16, to_device

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def run_single(hq, hkv, hd, ctx, hint, seed):
    rng = np.random.default_rng(seed)
    ctx_a = np.asarray([ctx], np.int32)
    case = make_case(1, hq, hkv, hd, ctx_a + 1, seed=seed)  # room for the new token
    qkv = randn_bf16(rng, (1, (hq + 2 * hkv) * hd))
    qb, kb, vb = (randn_bf16(rng, (n * hd,)) for n in (hq, hkv, hkv))
    cos, sin = O.rope_table(max(ctx, hint) + 8, hd, 1e6)
    dev = [to_device(x) for x in (qb, kb, vb, cos, sin, ctx_a, case.tables)]
    ws = L.alloc_decode_workspace(1, hq, hkv, hd)
    # batched path: two launches
    qkv_a, ka, va = to_device(qkv), to_device(case.k_pool), to_device(case.v_pool)
    out_a = torch.empty(1, hq * hd, dtype=torch.bfloat16, device="cuda")
    L.rope_append(qkv_a, dev[5], dev[0], dev[1], dev[2], dev[3], dev[4], ka, va, case.num_blocks,
                  case.num_layers, case.layer, hq, hkv, hd, dev[6])
    L.paged_decode(out_a, qkv_a, ka, va, case.num_blocks, case.num_layers, case.layer, hq, hkv, hd,
                   dev[6], dev[5], ctx + 1, len_offset=1, partition_tokens=0, workspace=ws)
    # single-sequence path, repeated: every launch starts its barriers afresh
    qkv_b = to_device(qkv)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    outs = []
    for _ in range(3):
        kb_, vb_ = to_device(case.k_pool), to_device(case.v_pool)
        out_b = torch.full((1, hq * hd), float("nan"), dtype=torch.bfloat16, device="cuda")
        L.rope_append_decode(out_b, qkv_b, dev[5], dev[0], dev[1], dev[2], dev[3], dev[4], kb_,
                             vb_, case.num_blocks, case.num_layers, case.layer, hq, hkv, hd,
                             dev[6], hint + 1, partition_tokens=0, workspace=ws, dev_status=st)
        outs.append(out_b)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert not ws.any()  # the workspace is left as found
    return case, qkv, (qb, kb, vb, cos, sin), (ka, va, out_a), (qkv_b, kb_, vb_, outs)


@pytest.mark.parametrize("hq,hkv,hd", [(14, 2, 64), (28, 4, 128), (32, 2, 64), (64, 8, 128)])
@pytest.mark.parametrize("ctx,hint", [(40, 40), (127, 127), (1023, 1023), (4096, 4096),
                                      (20000, 20000), (40, 1023), (300, 4000)])
def test_single_sequence_cluster_decode(hq, hkv, hd, ctx, hint):
    case, qkv, bias, a, b = run_single(hq, hkv, hd, ctx, hint, seed=ctx + hq)
    ka, va, out_a = a
    qkv_b, kb_, vb_, outs = b
    assert torch.equal(ka.view(torch.int16), kb_.view(torch.int16))
    assert torch.equal(va.view(torch.int16), vb_.view(torch.int16))
    assert np.array_equal(from_device(qkv_b), qkv)  # qkv only read
    for o in outs[1:]:  # the same bits every launch
        assert torch.equal(o.view(torch.int16), outs[0].view(torch.int16))
    qb, kb, vb, cos, sin = bias
    q2 = qkv.copy()
    ctx_a = np.asarray([ctx], np.int32)
    O.rope_append(q2, ctx_a, qb, kb, vb, cos, sin, case.k_pool, case.v_pool, case.num_layers,
                  case.layer, hq, hkv, hd, case.tables)
    ref = O.bf16_to_f32(O.paged_decode(q2, case.k_pool, case.v_pool, case.layer, hq, hkv, hd,
                                       case.tables, ctx_a, case.num_layers, len_offset=1,
                                       threads=8))
    got = O.bf16_to_f32(from_device(outs[0]))
    assert np.isfinite(got).all()
    assert float(np.abs(got - ref).max()) <= ATTN_ATOL
    two = O.bf16_to_f32(from_device(out_a))
    assert float(np.abs(got - two).max()) <= ATTN_ATOL


@pytest.mark.parametrize("hq,hkv,hd", [(14, 2, 64), (28, 4, 128), (32, 2, 64)])
@pytest.mark.parametrize("ctx,hint,len_offset", [(1024, 1024, 0), (1025, 1025, 1), (300, 4096, 0),
                                                 (9000, 9000, 1)])
def test_single_sequence_cluster_plain_decode(hq, hkv, hd, ctx, hint, len_offset):
    """lc_paged_decode with batch 1 (what lc_flash_decoding, the reference-shaped
    entry, always runs) takes the same cluster path: outputs against the CPU
    oracle, the same bits on every launch, the workspace left as found."""
    case = make_case(1, hq, hkv, hd, [ctx], seed=ctx + hd)
    q, k, v = to_device(case.q), to_device(case.k_pool), to_device(case.v_pool)
    tables = to_device(case.tables)
    lens = to_device(np.asarray([ctx - len_offset], np.int32))
    ws = L.alloc_decode_workspace(1, hq, hkv, hd)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    outs = []
    for _ in range(3):
        out = torch.full((1, hq * hd), float("nan"), dtype=torch.bfloat16, device="cuda")
        L.paged_decode(out, q, k, v, case.num_blocks, case.num_layers, case.layer, hq, hkv, hd,
                       tables, lens, hint, len_offset=len_offset, workspace=ws, dev_status=st)
        outs.append(out)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert not ws.any()
    for o in outs[1:]:
        assert torch.equal(o.view(torch.int16), outs[0].view(torch.int16))
    ref = O.bf16_to_f32(O.paged_decode(case.q, case.k_pool, case.v_pool, case.layer, hq, hkv, hd,
                                       case.tables, np.asarray([ctx - len_offset], np.int32),
                                       case.num_layers, len_offset=len_offset, threads=8))
    got = O.bf16_to_f32(from_device(outs[0]))
    assert np.isfinite(got).all()
    assert float(np.abs(got - ref).max()) <= ATTN_ATOL
