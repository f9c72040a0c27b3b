"""Causal prefill on the tensor cores (lc_paged_prefill) against the reference
algorithm: the oracle runs the reference's per-token loop (rope -> append ->
flash-decoding over 0..pos, src/models.rs:486-550) and the reference kernels
themselves run it on the GPU. Attention outputs within ATTN_ATOL."""
import ctypes as C

import numpy as np
import pytest

import lucciola as L
import oracle.oracle as O
from conftest import ATTN_ATOL
from workloads import from_device, make_case, randn_bf16, to_device

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def run_prefill(hq, hkv, hd, T, start, seed, q_stride_pad=0):
    start = np.asarray(start, np.int32)
    B = len(start)
    case = make_case(B, hq, hkv, hd, start + T, seed=seed)
    rng = np.random.default_rng(seed + 1)
    q = randn_bf16(rng, (B * T, hq * hd + q_stride_pad))
    dq = to_device(q)
    out = torch.full((B * T, hq * hd), float("nan"), dtype=torch.bfloat16, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.paged_prefill(out, dq, to_device(case.k_pool), to_device(case.v_pool), case.num_blocks,
                    case.num_layers, case.layer, hq, hkv, hd, to_device(case.tables),
                    to_device(start), T, int(start.max()), dev_status=st)
    torch.cuda.synchronize()
    ref = O.paged_prefill(np.ascontiguousarray(q[:, :hq * hd]), case.k_pool, case.v_pool,
                          case.layer, hq, hkv, hd, case.tables, start, T, case.num_layers,
                          threads=8)
    return from_device(out), ref, int(st.item())


def max_err(a, b):
    return float(np.abs(O.bf16_to_f32(a) - O.bf16_to_f32(b)).max())


@pytest.mark.parametrize("hq,hkv,hd,T,start", [
    (12, 2, 128, 300, [0, 37]),      # Qwen2.5-1.5B shape, prior context on one sequence
    (14, 2, 64, 257, [0, 100]),      # head_dim 64, partial last tile
    (28, 4, 128, 129, [500]),        # long prior context, GQA 7
    (64, 8, 128, 200, [0]),          # GQA 8
    (12, 2, 128, 256, [0, 0, 16]),   # whole tiles
    (12, 2, 128, 1, [0, 5]),         # one-token prompts
    (8, 8, 64, 70, [3]),             # MHA
])
def test_prefill_matches_per_token_reference(hq, hkv, hd, T, start):
    out, ref, st = run_prefill(hq, hkv, hd, T, start, seed=hq + T + hd)
    assert st == 0
    assert np.isfinite(O.bf16_to_f32(out)).all()
    assert max_err(out, ref) <= ATTN_ATOL


def test_prefill_score_growth_rescales():
    """Keys whose scores outgrow the running reference max by far more than the
    rescale bound (K of tokens >= 300 scaled by 100): the kernel must notice it
    from the row sums, rescale O and l, and still match the oracle."""
    hq, hkv, hd, T = 12, 2, 128, 520
    start = np.array([0], np.int32)
    case = make_case(1, hq, hkv, hd, start + T, seed=21)
    kf = O.bf16_to_f32(case.k_pool)
    for tok in range(300, T):
        blk = case.tables[0, tok // 16]
        kf[blk, case.layer, :, tok % 16, :] *= 100.0
    case.k_pool = O.f32_to_bf16(kf)
    rng = np.random.default_rng(22)
    q = randn_bf16(rng, (T, hq * hd))
    out = torch.full((T, hq * hd), float("nan"), dtype=torch.bfloat16, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.paged_prefill(out, to_device(q), to_device(case.k_pool), to_device(case.v_pool),
                    case.num_blocks, case.num_layers, case.layer, hq, hkv, hd,
                    to_device(case.tables), to_device(start), T, 0, dev_status=st)
    torch.cuda.synchronize()
    ref = O.paged_prefill(q, case.k_pool, case.v_pool, case.layer, hq, hkv, hd, case.tables,
                          start, T, case.num_layers, threads=8)
    got = from_device(out)
    assert int(st.item()) == 0
    assert np.isfinite(O.bf16_to_f32(got)).all()
    assert max_err(got, ref) <= ATTN_ATOL


def test_prefill_strided_q_rows():
    out, ref, st = run_prefill(12, 2, 128, 140, [0, 9], seed=3, q_stride_pad=4 * 128)
    assert st == 0 and max_err(out, ref) <= ATTN_ATOL


def test_prefill_after_rope_append_matches_reference_kernels():
    """The whole prompt path: lc_rope_append (T rows per sequence) then
    lc_paged_prefill, against the reference's own kernels run token by token."""
    R = O.ref_lib()
    hq, hkv, hd, T = 12, 2, 128, 150
    start = np.array([0, 20], np.int32)
    B = len(start)
    case = make_case(B, hq, hkv, hd, start + T, seed=11)
    rng = np.random.default_rng(12)
    row = (hq + 2 * hkv) * hd
    qkv = randn_bf16(rng, (B * T, row))
    qb, kb, vb = (randn_bf16(rng, (n * hd,)) for n in (hq, hkv, hkv))
    cos, sin = O.rope_table(1024, hd, 1e6)
    pos = (start[:, None] + np.arange(T, dtype=np.int32)[None, :]).ravel().astype(np.int32)
    d = [to_device(x) for x in (qb, kb, vb, cos, sin, pos, case.tables, start)]

    # ours
    dqkv, dk, dv = to_device(qkv), to_device(case.k_pool), to_device(case.v_pool)
    L.rope_append(dqkv, d[5], d[0], d[1], d[2], d[3], d[4], dk, dv, case.num_blocks,
                  case.num_layers, case.layer, hq, hkv, hd, d[6], tokens_per_seq=T)
    out = torch.empty(B * T, hq * hd, dtype=torch.bfloat16, device="cuda")
    L.paged_prefill(out, dqkv, dk, dv, case.num_blocks, case.num_layers, case.layer, hq, hkv, hd,
                    d[6], d[7], T, int(start.max()))
    # the reference kernels, one token at a time
    rqkv, rk, rv = to_device(qkv), to_device(case.k_pool), to_device(case.v_pool)
    rout = torch.empty(B * T, hq * hd, dtype=torch.bfloat16, device="cuda")
    host_pos = (C.c_int * (B * T))(*pos.tolist())
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert R.ref_prefill(P(rout), hq * hd, P(rqkv), row, B, T, P(d[5]), host_pos, P(d[0]),
                         P(d[1]), P(d[2]), P(d[3]), P(d[4]), P(rk), P(rv), case.num_layers,
                         case.layer, hq, hkv, hd, P(d[6]), case.tables.shape[1], 32768, s) == 0
    torch.cuda.synchronize()
    assert torch.equal(dk.view(torch.int16), rk.view(torch.int16))  # bit-exact cache writes
    assert torch.equal(dv.view(torch.int16), rv.view(torch.int16))
    assert max_err(from_device(out), from_device(rout)) <= ATTN_ATOL


def test_prefill_reports_bad_block():
    hq, hkv, hd, T = 12, 2, 128, 64
    case = make_case(1, hq, hkv, hd, [T], seed=5)
    case.tables[0, 1] = case.num_blocks + 3
    rng = np.random.default_rng(6)
    q = to_device(randn_bf16(rng, (T, hq * hd)))
    out = torch.empty(T, hq * hd, dtype=torch.bfloat16, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.paged_prefill(out, q, to_device(case.k_pool), to_device(case.v_pool), case.num_blocks,
                    case.num_layers, case.layer, hq, hkv, hd, to_device(case.tables),
                    to_device(np.array([0], np.int32)), T, 0, dev_status=st)
    torch.cuda.synchronize()
    assert int(st.item()) & L.LC_DEV_BAD_BLOCK
