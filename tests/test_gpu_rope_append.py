"""Fused bias + RoPE + KV append on the GPU (lc_rope_append, lc_rope,
lc_update_kv_cache) against the CPU oracle: bit-exact q/k rotation and KV-cache
writes. Also the owning KVCache mirror driven like src/models.rs:486-549."""
import numpy as np
import pytest

import lucciola as L
import oracle.oracle as O
from conftest import ATTN_ATOL
from workloads import from_device, make_case, randn_bf16, to_device

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def biases(rng, hq, hkv, hd):
    return randn_bf16(rng, (hq * hd,)), randn_bf16(rng, (hkv * hd,)), randn_bf16(rng, (hkv * hd,))


# pad 8 keeps rows 16-byte aligned (the 16-byte vector kernel); pad 4 does not
# (the element-wise kernel). Both must write the same bits.
@pytest.mark.parametrize("hq,hkv,hd,T,pad", [(14, 2, 64, 1, 8), (28, 4, 128, 1, 8),
                                             (12, 2, 128, 37, 8), (64, 8, 128, 1, 8),
                                             (16, 2, 64, 20, 8), (12, 2, 128, 37, 4),
                                             (14, 2, 64, 9, 4)])
def test_rope_append_bit_exact(hq, hkv, hd, T, pad):
    rng = np.random.default_rng(hq + T)
    B = 5
    start = rng.integers(0, 3000, B).astype(np.int32)
    case = make_case(B, hq, hkv, hd, start + T, seed=hq + T + 1)
    row = (hq + 2 * hkv) * hd + pad  # padded row stride
    qkv = randn_bf16(rng, (B * T, row))
    qb, kb, vb = biases(rng, hq, hkv, hd)
    cos, sin = O.rope_table(4096, hd, 1e6)
    pos = (start[:, None] + np.arange(T, dtype=np.int32)[None, :]).ravel().astype(np.int32)

    d_qkv = to_device(qkv)
    dk, dv = to_device(case.k_pool), to_device(case.v_pool)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.rope_append(d_qkv, to_device(pos), to_device(qb), to_device(kb), to_device(vb),
                  to_device(cos), to_device(sin), dk, dv, case.num_blocks, case.num_layers,
                  case.layer, hq, hkv, hd, to_device(case.tables), tokens_per_seq=T, dev_status=st)
    torch.cuda.synchronize()

    O.rope_append(qkv, pos, qb, kb, vb, cos, sin, case.k_pool, case.v_pool, case.num_layers,
                  case.layer, hq, hkv, hd, case.tables, tokens_per_seq=T)
    assert int(st.item()) == 0
    assert np.array_equal(from_device(d_qkv), qkv)
    assert np.array_equal(from_device(dk), case.k_pool)
    assert np.array_equal(from_device(dv), case.v_pool)


def test_rope_append_reports_bad_positions_and_blocks():
    hq, hkv, hd = 14, 2, 64
    rng = np.random.default_rng(0)
    case = make_case(3, hq, hkv, hd, [16, 16, 16], seed=0)
    qkv = randn_bf16(rng, (3, (hq + 2 * hkv) * hd))
    qb, kb, vb = biases(rng, hq, hkv, hd)
    cos, sin = O.rope_table(64, hd, 1e6)
    case.tables[2, 0] = case.num_blocks  # outside the pool
    pos = np.array([5, 16 * 7, 3], np.int32)  # row 1 beyond its table row
    dk, dv = to_device(case.k_pool), to_device(case.v_pool)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.rope_append(to_device(qkv), to_device(pos), to_device(qb), to_device(kb), to_device(vb),
                  to_device(cos), to_device(sin), dk, dv, case.num_blocks, case.num_layers,
                  case.layer, hq, hkv, hd, to_device(case.tables), dev_status=st)
    torch.cuda.synchronize()
    s = int(st.item())
    assert s & L.LC_DEV_BAD_BLOCK and s & L.LC_DEV_BAD_POS
    # Only row 0 was appended.
    kp = from_device(dk)
    blk = case.tables[0, 0]
    changed = np.argwhere((kp != case.k_pool).any(axis=(1, 2, 3, 4)))[:, 0]
    assert set(changed.tolist()) <= {blk}


@pytest.mark.parametrize("hq,hkv,hd", [(14, 2, 64), (28, 4, 128)])
def test_reference_shaped_rope_and_update(hq, hkv, hd):
    rng = np.random.default_rng(hd)
    cos, sin = O.rope_table(32768, hd, 1e6)
    dcos, dsin = to_device(cos), to_device(sin)
    qb, kb, vb = biases(rng, hq, hkv, hd)
    case = make_case(1, hq, hkv, hd, [32768], seed=1, table_stride=2048)
    dk, dv, dt = to_device(case.k_pool), to_device(case.v_pool), to_device(case.tables)
    for pos in (0, 1, 15, 16, 1023, 4097, 32767):
        q = randn_bf16(rng, (hq * hd,))
        k = randn_bf16(rng, (hkv * hd,))
        v = randn_bf16(rng, (hkv * hd,))
        dq, dkk, dvv = to_device(q), to_device(k), to_device(v)
        pos_t = to_device(np.array([pos], np.int32))
        L.rope(dq, to_device(qb), dkk, to_device(kb), dcos, dsin, pos_t, hd, hq, hkv)
        L.update_kv_cache(dk, dv, dkk, dvv, to_device(vb), dt, case.layer, pos_t, case.num_layers,
                          hkv, 32768, hd)
        torch.cuda.synchronize()
        O.rope(q, qb, k, kb, cos, sin, pos, hd, hq, hkv)
        O.update_kv_cache(case.k_pool, case.v_pool, k, v, vb, case.tables[0], case.layer, pos,
                          case.num_layers, hkv, hd)
        assert np.array_equal(from_device(dq), q)
        assert np.array_equal(from_device(dkk), k)
    assert np.array_equal(from_device(dk), case.k_pool)
    assert np.array_equal(from_device(dv), case.v_pool)


def test_kv_cache_mirror_token_loop():
    """KVCache + rope + apply_flash_decoding, per token, as forward_layer does."""
    Lyr, hq, hkv, hd, max_pos = 2, 14, 2, 64, 512
    rng = np.random.default_rng(3)
    kv = L.KVCache(Lyr, hq, hkv, hd, max_pos, 0.9)
    assert kv.num_physical_blocks == max_pos // 16
    assert kv.max_seq_len == max_pos
    nb = kv.num_physical_blocks
    cos, sin = O.rope_table(max_pos, hd, 1e6)
    dcos, dsin = to_device(cos), to_device(sin)
    qb, kb, vb = biases(rng, hq, hkv, hd)
    dqb, dkb, dvb = to_device(qb), to_device(kb), to_device(vb)
    k_pool = np.zeros((nb, Lyr, hkv, 16, hd), np.uint16)
    v_pool = np.zeros_like(k_pool)
    table = np.arange(max_pos // 16, dtype=np.int32)  # LIFO free list pops 0, 1, 2, ...
    pos_t = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty(hq * hd, dtype=torch.bfloat16, device="cuda")
    for pos in range(0, 70):
        for layer in range(Lyr):
            qkv = randn_bf16(rng, ((hq + 2 * hkv) * hd,))
            dqkv = to_device(qkv)
            pos_t.fill_(pos)
            qs, ks = dqkv[:hq * hd], dqkv[hq * hd:(hq + hkv) * hd]
            vs = dqkv[(hq + hkv) * hd:]
            L.rope(qs, dqb, ks, dkb, dcos, dsin, pos_t, hd, hq, hkv)
            kv.update(layer, pos, pos_t, ks, vs, dvb)
            kv.apply_flash_decoding(out, qs, layer, pos, pos_t)
            torch.cuda.synchronize()
            q, k, v = qkv[:hq * hd].copy(), qkv[hq * hd:(hq + hkv) * hd].copy(), qkv[(hq + hkv) * hd:].copy()
            O.rope(q, qb, k, kb, cos, sin, pos, hd, hq, hkv)
            O.update_kv_cache(k_pool, v_pool, k, v, vb, table, layer, pos, Lyr, hkv, hd)
            ref = O.flash_decoding(q, k_pool, v_pool, table, layer, hq, hkv, hd, pos, Lyr)
            got = from_device(out)
            assert float(np.abs(O.bf16_to_f32(got) - O.bf16_to_f32(ref)).max()) <= ATTN_ATOL
    assert kv.num_allocated_blocks == (69 // 16) + 1
    kv.close()
