"""lc_paged_decode_static: the decode entry point that allocates nothing.

It exists for callers that cannot allocate device memory while they decode
(serving loops that must not hit cudaMalloc/cudaFree, which may synchronise the
device, or hosts whose device memory is all reserved for their own pools): its
split-K scratch is a fixed array the library keeps on each GPU. These tests call
it through the C ABI, twice in a row on the same inputs, and check each result
against lc_paged_decode with a caller-allocated workspace, within the attention
tolerance of the other tests. The file is named so that pytest collects it last.
"""
import numpy as np
import pytest

import lucciola as L
import oracle.oracle as O
from conftest import ATTN_ATOL
from workloads import from_device, make_case, to_device

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _max_err(a, b):
    return float(np.abs(O.bf16_to_f32(from_device(a)) - O.bf16_to_f32(from_device(b))).max())


@pytest.mark.parametrize("hq,hkv,hd,batch,lo,hi", [
    (14, 2, 64, 64, 256, 4096),   # Qwen2.5-0.5B shape, ragged batch
    (28, 4, 128, 8, 1000, 8192),  # Qwen2.5-7B shape
    (14, 2, 64, 1, 1024, 1024),   # one sequence split over many CTAs
])
def test_static_scratch_matches_workspace_entry_twice(hq, hkv, hd, batch, lo, hi):
    rng = np.random.default_rng(batch * 31 + hd)
    ctx = rng.integers(lo, hi + 1, batch).astype(np.int32)
    case = make_case(batch, hq, hkv, hd, ctx, seed=batch + hd)
    k, v = to_device(case.k_pool), to_device(case.v_pool)
    q, tables, lens = to_device(case.q), to_device(case.tables), to_device(case.ctx)

    ref = torch.empty(batch, hq * hd, dtype=torch.bfloat16, device="cuda")
    ws = L.alloc_decode_workspace(batch, hq, hkv, hd)
    L.paged_decode(ref, q, k, v, case.num_blocks, case.num_layers, case.layer, hq, hkv, hd,
                   tables, lens, int(ctx.max()), workspace=ws)

    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    outs = []
    for _ in range(2):  # two calls in a row share (and reuse) the fixed scratch
        out = torch.full((batch, hq * hd), float("nan"), dtype=torch.bfloat16, device="cuda")
        L.paged_decode_static(out, q, k, v, case.num_blocks, case.num_layers, case.layer, hq,
                              hkv, hd, tables, lens, int(ctx.max()), dev_status=status)
        outs.append(out)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    for out in outs:
        assert _max_err(out, ref) <= ATTN_ATOL


def test_static_scratch_rejects_batches_beyond_its_size():
    hq, hkv, hd, batch = 64, 8, 128, 4096
    need = L.paged_decode_workspace_size(batch, hq, hkv, hd)
    assert need > L.lib.lc_paged_decode_workspace_size(1, hq, hkv, hd)
    assert need > (8 << 20)  # LC_PAGED_DECODE_STATIC_SCRATCH_BYTES
    case = make_case(1, hq, hkv, hd, [16], seed=0)
    k, v, q = to_device(case.k_pool), to_device(case.v_pool), to_device(case.q)
    tables = torch.zeros(batch, 1, dtype=torch.int32, device="cuda")
    lens = torch.ones(batch, dtype=torch.int32, device="cuda")
    out = torch.zeros(batch, hq * hd, dtype=torch.bfloat16, device="cuda")
    qq = q.expand(batch, -1).contiguous()
    with pytest.raises(L.LucciolaError) as e:
        L.paged_decode_static(out, qq, k, v, case.num_blocks, case.num_layers, case.layer, hq,
                              hkv, hd, tables, lens, 16)
    assert e.value.status == 4  # LC_ERR_WORKSPACE_TOO_SMALL
    torch.cuda.synchronize()
    assert not out.any()  # nothing was launched
