"""Projections either side of attention on the tensor cores (lc_proj_gemm,
lc_qkv_proj_rope_append). The reference runs them with cublasGemmEx, fp32
compute and a bf16 result (src/models.rs:252-292): the GEMM is checked against
a float64 product within the bf16 rounding of the result plus fp32
accumulation-order slack. The fused QKV projection must equal lc_proj_gemm
followed by lc_rope_append bit for bit (rows, pools and status words)."""
import numpy as np
import pytest

import lucciola as L
import oracle.oracle as O
from workloads import from_device, make_case, randn_bf16, to_device

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _gemm_ref(x, w, residual=None):
    ref = x.double() @ w.double().T
    if residual is not None:
        ref = ref + residual.double()
    return ref


def _check_gemm(out, ref, K):
    err = (out.double() - ref).abs()
    # half a bf16 step of the result, plus fp32 accumulation-order slack
    bound = ref.abs() * 2.0 ** -8 + 2.0 ** -20 * K * 8
    assert bool((err <= bound).all()), float((err - bound).max())


@pytest.mark.parametrize("M,N,K", [
    (300, 1152, 896),    # Qwen2.5-0.5B qkv_proj, a 300-token prompt
    (128, 256, 64),      # one tile, one K block
    (1, 896, 896),       # a single row (decode shape of o_proj)
    (517, 2048, 1536),   # Qwen2.5-1.5B qkv_proj, ragged M
    (70, 96, 200),       # N and K tails (partial tile, K not a multiple of 64)
    # decode steps (M = batch <= 128: the weight-streaming kernel, K split
    # over a cluster): Qwen2.5-0.5B at batch 64, Qwen2.5-7B at batch 32
    (64, 1152, 896),     # 0.5B qkv_proj
    (64, 896, 896),      # 0.5B o_proj
    (32, 4608, 3584),    # 7B qkv_proj
    (32, 3584, 3584),    # 7B o_proj
    (128, 2048, 1536),   # 1.5B qkv_proj, the largest decode batch
    (17, 4608, 3584),    # a batch that is not a multiple of 16
])
def test_proj_gemm_matches_float64(M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device="cuda") * K ** -0.5).to(torch.bfloat16)
    out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
    L.proj_gemm(out, x, w)
    torch.cuda.synchronize()
    _check_gemm(out, _gemm_ref(x, w), K)


@pytest.mark.parametrize("M,N,K", [(200, 896, 896), (64, 896, 896), (32, 3584, 3584)])
def test_proj_gemm_residual_in_place(M, N, K):
    """o_proj with beta 1: hidden = bf16(attn . w_o^T + hidden), in place."""
    g = torch.Generator(device="cuda").manual_seed(3 + M)
    x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g, device="cuda") * K ** -0.5).to(torch.bfloat16)
    hidden = torch.randn(M, N, generator=g, device="cuda").to(torch.bfloat16)
    ref = _gemm_ref(x, w, hidden)
    L.proj_gemm(hidden, x, w, residual=hidden)
    torch.cuda.synchronize()
    _check_gemm(hidden, ref, K)


def test_proj_gemm_strided_rows():
    M, N, K = 150, 512, 384
    g = torch.Generator(device="cuda").manual_seed(4)
    xs = torch.randn(M, K + 64, generator=g, device="cuda").to(torch.bfloat16)
    ws = (torch.randn(N, K + 32, generator=g, device="cuda") * K ** -0.5).to(torch.bfloat16)
    outs = torch.zeros(M, N + 128, dtype=torch.bfloat16, device="cuda")
    x, w, out = xs[:, :K], ws[:, :K], outs[:, :N]
    L.proj_gemm(out, x, w)
    torch.cuda.synchronize()
    _check_gemm(out, _gemm_ref(x, w), K)
    assert not outs[:, N:].any()  # nothing written past the row


def test_proj_gemm_rejects_bad_shapes():
    x = torch.zeros(4, 64, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(40, 64, dtype=torch.bfloat16, device="cuda")  # N not a multiple of 32
    out = torch.zeros(4, 40, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(L.LucciolaError) as e:
        L.proj_gemm(out, x, w)
    assert e.value.status == 3  # LC_ERR_UNSUPPORTED_SHAPE


def _qkv_case(hq, hkv, hd, hidden, T, start, seed, bad_block=False, past_rope=False):
    start = np.asarray(start, np.int32)
    B = len(start)
    case = make_case(B, hq, hkv, hd, start + T, seed=seed)
    rng = np.random.default_rng(seed + 1)
    N = (hq + 2 * hkv) * hd
    x = randn_bf16(rng, (B * T, hidden))
    w = O.f32_to_bf16((rng.standard_normal((N, hidden)) * hidden ** -0.5).astype(np.float32))
    qb, kb, vb = (randn_bf16(rng, (n * hd,)) for n in (hq, hkv, hkv))
    rope_rows = 4096
    cos, sin = O.rope_table(rope_rows, hd, 1e6)
    pos = (start[:, None] + np.arange(T, dtype=np.int32)[None, :]).ravel().astype(np.int32)
    tables = case.tables.copy()
    if bad_block:
        tables[0, 1] = case.num_blocks + 7  # tokens 16..31 of sequence 0
    if past_rope:
        pos[3] = rope_rows + 5
    return case, x, w, (qb, kb, vb), (cos, sin), pos, tables


@pytest.mark.parametrize("hq,hkv,hd,hidden,T,start,flags", [
    (14, 2, 64, 896, 150, [0, 37], {}),                        # Qwen2.5-0.5B
    (12, 2, 128, 1536, 129, [0], {}),                          # Qwen2.5-1.5B
    (28, 4, 128, 3584, 70, [100, 0, 5], {}),                   # Qwen2.5-7B
    (14, 2, 64, 896, 40, [0, 0], {"bad_block": True}),         # a table entry outside the pool
    (14, 2, 64, 896, 20, [0], {"past_rope": True}),            # a position past the RoPE table
    # decode steps: one new token per sequence (the weight-streaming kernel)
    (14, 2, 64, 896, 1, list(range(7, 4000, 63))[:64], {}),    # 0.5B, batch 64
    (28, 4, 128, 3584, 1, list(range(11, 4000, 125))[:32], {}),  # 7B, batch 32
    (12, 2, 128, 1536, 1, list(range(0, 3900, 31))[:125], {}),  # 1.5B, batch 125
])
def test_qkv_proj_rope_append_equals_gemm_then_rope_append(hq, hkv, hd, hidden, T, start, flags):
    case, x, w, bias, rope, pos, tables = _qkv_case(hq, hkv, hd, hidden, T, start,
                                                    seed=hq + T, **flags)
    B = len(start)
    N = (hq + 2 * hkv) * hd
    dx, dw = to_device(x), to_device(w)
    db = [to_device(b) for b in bias]
    dcos, dsin = (to_device(r) for r in rope)
    dpos, dtab = to_device(pos), to_device(tables)
    runs = []
    for fused in (False, True):
        k, v = to_device(case.k_pool), to_device(case.v_pool)
        qkv = torch.full((B * T, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        st = torch.zeros(1, dtype=torch.int32, device="cuda")
        if fused:
            L.qkv_proj_rope_append(qkv, dx, dw, dpos, *db, dcos, dsin, k, v, case.num_blocks,
                                   case.num_layers, case.layer, hq, hkv, hd, dtab,
                                   tokens_per_seq=T, dev_status=st)
        else:
            L.proj_gemm(qkv, dx, dw)
            L.rope_append(qkv, dpos, *db, dcos, dsin, k, v, case.num_blocks, case.num_layers,
                          case.layer, hq, hkv, hd, dtab, tokens_per_seq=T, dev_status=st)
        torch.cuda.synchronize()
        runs.append((from_device(qkv), from_device(k), from_device(v), int(st.item())))
    (q0, k0, v0, s0), (q1, k1, v1, s1) = runs
    assert np.array_equal(q0, q1)
    assert np.array_equal(k0, k1)
    assert np.array_equal(v0, v1)
    assert s0 == s1
    if flags.get("bad_block"):
        assert s1 & L.LC_DEV_BAD_BLOCK
    elif flags.get("past_rope"):
        assert s1 & L.LC_DEV_BAD_POS
    else:
        assert s1 == 0
        # the appended rows changed the pools
        assert not np.array_equal(k1, case.k_pool)


def test_qkv_proj_then_prefill_matches_oracle():
    """Prompt path with the fused projection: lc_qkv_proj_rope_append, then
    lc_paged_prefill, against the oracle run on the same projected rows."""
    from conftest import ATTN_ATOL
    hq, hkv, hd, hidden, T = 14, 2, 64, 896, 200
    case, x, w, bias, rope, pos, tables = _qkv_case(hq, hkv, hd, hidden, T, [0], seed=9)
    N = (hq + 2 * hkv) * hd
    k, v = to_device(case.k_pool), to_device(case.v_pool)
    qkv = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
    dpos, dtab = to_device(pos), to_device(tables)
    db = [to_device(b) for b in bias]
    L.qkv_proj_rope_append(qkv, to_device(x), to_device(w), dpos, *db, *(to_device(r) for r in rope),
                           k, v, case.num_blocks, case.num_layers, case.layer, hq, hkv, hd, dtab,
                           tokens_per_seq=T)
    raw = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
    L.proj_gemm(raw, to_device(x), to_device(w))
    out = torch.empty(T, hq * hd, dtype=torch.bfloat16, device="cuda")
    L.paged_prefill(out, qkv, k, v, case.num_blocks, case.num_layers, case.layer, hq, hkv, hd,
                    dtab, to_device(np.zeros(1, np.int32)), T, 0)
    torch.cuda.synchronize()
    # oracle: the same projected rows through the CPU restatement
    rows = from_device(raw)
    kp, vp = case.k_pool.copy(), case.v_pool.copy()
    O.rope_append(rows, pos, *bias, *rope, kp, vp, case.num_layers, case.layer, hq, hkv, hd,
                  tables, tokens_per_seq=T)
    assert np.array_equal(from_device(k), kp) and np.array_equal(from_device(v), vp)
    assert np.array_equal(from_device(qkv), rows)
    ref = O.paged_prefill(np.ascontiguousarray(rows[:, :hq * hd]), kp, vp, case.layer, hq, hkv,
                          hd, tables, np.zeros(1, np.int32), T, case.num_layers, threads=8)
    got = from_device(out)
    assert float(np.abs(O.bf16_to_f32(got) - O.bf16_to_f32(ref)).max()) <= ATTN_ATOL
