"""The reference's own CUDA kernels (compiled unchanged into oracle/_ref) run on
the GPU: they pin the CPU oracle (bit-exact RoPE/append, attention within a
bf16 ulp) and are compared directly with the new kernels."""
import ctypes as C

import numpy as np
import pytest

import lucciola as L
import oracle.oracle as O
from conftest import ATTN_ATOL
from workloads import from_device, make_case, randn_bf16, to_device

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def p(t):
    return C.c_void_p(t.data_ptr())


def stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("hd,hq,hkv", [(64, 14, 2), (128, 28, 4), (128, 12, 2)])
def test_reference_rope_pins_contraction_mode(hd, hq, hkv):
    R = O.ref_lib()
    rng = np.random.default_rng(hd + hq)
    cos, sin = O.rope_table(32768, hd, 1e6)
    dcos, dsin = to_device(cos), to_device(sin)
    qb, kb = randn_bf16(rng, (hq * hd,)), randn_bf16(rng, (hkv * hd,))
    dqb, dkb = to_device(qb), to_device(kb)
    matches = {(s, a): True for s in range(3) for a in range(3)}
    for pos in list(range(0, 32768, 997)) + [32767]:
        q = randn_bf16(rng, (hq * hd,))
        k = randn_bf16(rng, (hkv * hd,))
        dq, dk = to_device(q), to_device(k)
        dpos = to_device(np.array([pos], np.int32))
        assert R.ref_rope(p(dq), p(dqb), p(dk), p(dkb), p(dcos), p(dsin), p(dpos), hd, hq, hkv,
                          stream()) == 0
        torch.cuda.synchronize()
        gq, gk = from_device(dq), from_device(dk)
        for mode in matches:
            q2, k2 = q.copy(), k.copy()
            O.rope(q2, qb, k2, kb, cos, sin, pos, hd, hq, hkv, *mode)
            if not (np.array_equal(q2, gq) and np.array_equal(k2, gk)):
                matches[mode] = False
    good = [m for m, ok in matches.items() if ok]
    print("reference rope contraction modes matching bit-exactly:", good)
    assert (1, 1) in good, f"kernel/oracle contraction mode (1,1) not bit-exact; matching: {good}"


def test_reference_update_kv_cache_matches_oracle():
    R = O.ref_lib()
    hq, hkv, hd = 14, 2, 64
    rng = np.random.default_rng(1)
    case = make_case(1, hq, hkv, hd, [300], seed=1, table_stride=64)
    dk, dv, dt = to_device(case.k_pool), to_device(case.v_pool), to_device(case.tables)
    vb = randn_bf16(rng, (hkv * hd,))
    dvb = to_device(vb)
    for pos in (0, 15, 16, 17, 299):
        k, v = randn_bf16(rng, (hkv * hd,)), randn_bf16(rng, (hkv * hd,))
        dpos = to_device(np.array([pos], np.int32))
        dkk, dvv = to_device(k), to_device(v)  # keep alive until the launch is queued
        assert R.ref_update_kv_cache(p(dk), p(dv), p(dkk), p(dvv), p(dvb),
                                     p(dt), case.layer, p(dpos), case.num_layers, hkv, 32768, hd,
                                     16, stream()) == 0
        torch.cuda.synchronize()
        O.update_kv_cache(case.k_pool, case.v_pool, k, v, vb, case.tables[0], case.layer, pos,
                          case.num_layers, hkv, hd)
    assert np.array_equal(from_device(dk), case.k_pool)
    assert np.array_equal(from_device(dv), case.v_pool)


@pytest.mark.parametrize("hq,hkv,hd,pos", [(14, 2, 64, 1023), (28, 4, 128, 200), (12, 2, 128, 0),
                                           (64, 8, 128, 2047)])
def test_reference_attention_pins_oracle_and_matches_ours(hq, hkv, hd, pos):
    R = O.ref_lib()
    case = make_case(1, hq, hkv, hd, [pos + 1], seed=pos + hq, table_stride=256)
    d_k, d_v, d_t, d_q = (to_device(case.k_pool), to_device(case.v_pool), to_device(case.tables),
                          to_device(case.q))
    out_ref = torch.empty(hq * hd, dtype=torch.bfloat16, device="cuda")
    dpos = to_device(np.array([pos], np.int32))
    assert R.ref_flash_decoding(p(out_ref), p(d_q), p(d_k), p(d_v), p(d_t), case.layer, hq, hkv,
                                hd, 4096, p(dpos), pos, 16, case.num_layers, stream()) == 0
    out = torch.empty(hq * hd, dtype=torch.bfloat16, device="cuda")
    ws = torch.zeros(L.flash_decoding_workspace_size(hq, hd, 4096), dtype=torch.uint8,
                     device="cuda")
    L.flash_decoding(out, d_q, d_k, d_v, d_t, case.layer, hq, hkv, hd, 4096, dpos,
                     1.0 / np.sqrt(hd), 16, case.num_layers, pos, case.num_blocks, ws)
    torch.cuda.synchronize()
    ref_gpu = O.bf16_to_f32(from_device(out_ref))
    ours = O.bf16_to_f32(from_device(out))
    orc = O.bf16_to_f32(O.flash_decoding(case.q[0], case.k_pool, case.v_pool, case.tables[0],
                                         case.layer, hq, hkv, hd, pos, case.num_layers))
    # The oracle restates the reference's summation order; only expf ulps differ.
    assert np.abs(orc - ref_gpu).max() <= 4e-3
    assert np.abs(ours - ref_gpu).max() <= ATTN_ATOL


def test_batched_ours_vs_reference_kernels():
    R = O.ref_lib()
    hq, hkv, hd = 14, 2, 64
    rng = np.random.default_rng(5)
    ctx = rng.integers(256, 4097, 8).astype(np.int32)
    case = make_case(8, hq, hkv, hd, ctx, seed=5)
    d_k, d_v, d_t, d_q = (to_device(case.k_pool), to_device(case.v_pool), to_device(case.tables),
                          to_device(case.q))
    pos = (ctx - 1).astype(np.int32)
    d_pos = to_device(pos)
    out_ref = torch.empty(8, hq * hd, dtype=torch.bfloat16, device="cuda")
    host_pos = (C.c_int * 8)(*pos.tolist())
    assert R.ref_paged_decode(p(out_ref), hq * hd, p(d_q), hq * hd, p(d_k), p(d_v),
                              case.num_layers, case.layer, hq, hkv, hd, p(d_t),
                              case.tables.shape[1], p(d_pos), host_pos, 8, 32768, stream()) == 0
    out = torch.empty(8, hq * hd, dtype=torch.bfloat16, device="cuda")
    ws = L.alloc_decode_workspace(8, hq, hkv, hd)
    L.paged_decode(out, d_q, d_k, d_v, case.num_blocks, case.num_layers, case.layer, hq, hkv, hd,
                   d_t, d_pos, int(ctx.max()), len_offset=1, partition_tokens=512, workspace=ws)
    torch.cuda.synchronize()
    err = np.abs(O.bf16_to_f32(from_device(out)) - O.bf16_to_f32(from_device(out_ref))).max()
    assert err <= ATTN_ATOL


def test_rope_append_ours_vs_reference_kernels():
    R = O.ref_lib()
    hq, hkv, hd, B = 28, 4, 128, 6
    rng = np.random.default_rng(9)
    ctx = rng.integers(100, 900, B).astype(np.int32)
    case = make_case(B, hq, hkv, hd, ctx + 1, seed=9)
    row = (hq + 2 * hkv) * hd
    qkv = randn_bf16(rng, (B, row))
    qb, kb, vb = (randn_bf16(rng, (n * hd,)) for n in (hq, hkv, hkv))
    cos, sin = O.rope_table(1024, hd, 1e6)
    args = [to_device(x) for x in (qb, kb, vb, cos, sin, ctx)]
    dqkv_a, dqkv_b = to_device(qkv), to_device(qkv)
    ka, va = to_device(case.k_pool), to_device(case.v_pool)
    kb_, vb_ = to_device(case.k_pool), to_device(case.v_pool)
    dt = to_device(case.tables)
    assert R.ref_rope_append(p(dqkv_a), row, B, 1, p(args[5]), p(args[0]), p(args[1]), p(args[2]),
                             p(args[3]), p(args[4]), p(ka), p(va), case.num_layers, case.layer,
                             hq, hkv, hd, p(dt), case.tables.shape[1], 32768, stream()) == 0
    L.rope_append(dqkv_b, args[5], args[0], args[1], args[2], args[3], args[4], kb_, vb_,
                  case.num_blocks, case.num_layers, case.layer, hq, hkv, hd, dt)
    torch.cuda.synchronize()
    assert torch.equal(dqkv_a.view(torch.int16), dqkv_b.view(torch.int16))
    assert torch.equal(ka.view(torch.int16), kb_.view(torch.int16))
    assert torch.equal(va.view(torch.int16), vb_.view(torch.int16))
