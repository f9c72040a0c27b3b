"""Parity at the full BASELINE sizes (configs 3, 4 and 5), through the C ABI.

Each case runs the product path on the config's exact shape and compares it
with the reference's own kernels (oracle/_ref: rope.cu, kv_cache.cu and
attention.cu compiled unchanged, launched per sequence and, for the prefill,
per token as src/models.rs:486-550 does) on the same seeded inputs:

* pool writes (K after bias + RoPE, V + bias) and rotated q/k rows bit-exact;
* attention outputs within ATTN_ATOL (max-abs, bf16 in, fp32 accumulate).

A sampled subset of rows or sequences is also checked against the CPU oracle
(oracle/lc_oracle.c), which restates the same algorithm, so that a fault
shared by both GPU paths would still show.

Inputs are synthetic: bf16 ~N(0,1) Q/K/V rows and stale pool contents, biases
at 0.01 scale (the bench's), RoPE theta 1e6, seeded torch generators on the
device (the config-5 pool alone is ~9 GB).
"""
import ctypes as C

import numpy as np
import pytest

import lucciola as L
import oracle.oracle as O
from conftest import ATTN_ATOL
from workloads import from_device, to_device

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _P(t):
    return C.c_void_p(t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def max_err(a_bits, b_bits):
    return float(np.abs(O.bf16_to_f32(a_bits) - O.bf16_to_f32(b_bits)).max())


def bits(t):
    return t.view(torch.int16)


def rand_bf16(gen, shape, scale=1.0):
    """bf16 ~N(0, scale^2) on the device, in slices of 2^28 elements."""
    t = torch.empty(shape, dtype=torch.bfloat16, device="cuda")
    flat = t.view(-1)
    for i in range(0, flat.numel(), 1 << 28):
        chunk = flat[i:i + (1 << 28)]
        r = torch.randn(chunk.numel(), generator=gen, device="cuda", dtype=torch.float32)
        chunk.copy_((r * scale).to(torch.bfloat16))
    return t


def shuffled_tables(gen, pages):
    """One row of distinct random pool blocks per sequence (-1 padded)."""
    pages = np.asarray(pages, np.int64)
    nb = int(pages.sum()) + 1
    perm = torch.randperm(nb, generator=gen, device="cuda").to(torch.int32).cpu().numpy()
    tables = np.full((len(pages), int(pages.max())), -1, np.int32)
    off = 0
    for b, n in enumerate(pages):
        tables[b, :n] = perm[off:off + n]
        off += n
    return tables, nb


def split_bias(bias, hq, hkv, hd):
    return (bias[:hq * hd].contiguous(), bias[hq * hd:(hq + hkv) * hd].contiguous(),
            bias[(hq + hkv) * hd:].contiguous())


def compact_pool(k_pool, v_pool, tables, seqs, pages):
    """Host copies of only the pages of sequences `seqs` (first `pages[i]`
    entries of their table rows), renumbered 0..n-1, with matching tables."""
    rows = [tables[b, :pages[i]] for i, b in enumerate(seqs)]
    idx = torch.from_numpy(np.concatenate(rows).astype(np.int64)).to(k_pool.device)
    k = from_device(k_pool.index_select(0, idx).contiguous())
    v = from_device(v_pool.index_select(0, idx).contiguous())
    t = np.full((len(seqs), max(pages)), -1, np.int32)
    off = 0
    for i, n in enumerate(pages):
        t[i, :n] = np.arange(off, off + n, dtype=np.int32)
        off += n
    return k, v, t


# --------------------------------------------------------------- config 4 --

def test_c4_prefill_full_shape_matches_reference_kernels():
    """Config 4 at its exact shape: 4 sequences x 4096 tokens, Hq 12 / Hkv 2,
    hd 128. Ours: lc_rope_append over the prompt rows, then lc_paged_prefill
    (tcgen05; 16 query blocks of 256 per head, heaviest first). Reference: its
    kernels token by token (rope -> append -> flash-decoding over 0..=t)."""
    R = O.ref_lib()
    hq, hkv, hd, B, T = 12, 2, 128, 4, 4096
    gen = torch.Generator(device="cuda")
    gen.manual_seed(4404)
    tables_np, nb = shuffled_tables(gen, [T // 16] * B)
    shape = (nb, 1, hkv, 16, hd)
    k0, v0 = rand_bf16(gen, shape), rand_bf16(gen, shape)  # stale contents, overwritten
    row = (hq + 2 * hkv) * hd
    qkv0 = rand_bf16(gen, (B * T, row))
    qb, kb, vb = split_bias(rand_bf16(gen, (row,), 0.01), hq, hkv, hd)
    cos_np, sin_np = O.rope_table(T, hd, 1e6)
    cos, sin = to_device(cos_np), to_device(sin_np)
    tables = to_device(tables_np)
    pos_np = np.tile(np.arange(T, dtype=np.int32), B)
    pos = to_device(pos_np)
    start = torch.zeros(B, dtype=torch.int32, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")

    qkv, k, v = qkv0.clone(), k0.clone(), v0.clone()
    L.rope_append(qkv, pos, qb, kb, vb, cos, sin, k, v, nb, 1, 0, hq, hkv, hd, tables,
                  tokens_per_seq=T, dev_status=st)
    out = torch.full((B * T, hq * hd), float("nan"), dtype=torch.bfloat16, device="cuda")
    L.paged_prefill(out, qkv, k, v, nb, 1, 0, hq, hkv, hd, tables, start, T, 0, dev_status=st)

    rqkv, rk, rv = qkv0.clone(), k0.clone(), v0.clone()
    rout = torch.empty((B * T, hq * hd), dtype=torch.bfloat16, device="cuda")
    host_pos = (C.c_int * (B * T))(*pos_np.tolist())
    assert R.ref_prefill(_P(rout), hq * hd, _P(rqkv), row, B, T, _P(pos), host_pos, _P(qb),
                         _P(kb), _P(vb), _P(cos), _P(sin), _P(rk), _P(rv), 1, 0, hq, hkv, hd,
                         _P(tables), tables_np.shape[1], 32768, _stream()) == 0
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert torch.equal(bits(qkv), bits(rqkv))  # rotated q / k rows
    assert torch.equal(bits(k), bits(rk))      # every K write of the prompt
    assert torch.equal(bits(v), bits(rv))
    o = from_device(out)
    assert np.isfinite(O.bf16_to_f32(o)).all()
    assert max_err(o, from_device(rout)) <= ATTN_ATOL

    # CPU oracle: the same rows rotated and appended on the host (bit-exact),
    # then attention for sampled rows (decode of row t over 0..t) across tile,
    # page and query-block boundaries of every sequence.
    h_qkv = from_device(qkv0)
    h_k, h_v = from_device(k0), from_device(v0)
    O.rope_append(h_qkv, pos_np, from_device(qb), from_device(kb), from_device(vb), cos_np,
                  sin_np, h_k, h_v, 1, 0, hq, hkv, hd, tables_np, tokens_per_seq=T)
    assert np.array_equal(h_qkv, from_device(qkv))
    assert np.array_equal(h_k, from_device(k))
    assert np.array_equal(h_v, from_device(v))
    ts = [0, 1, 15, 16, 127, 128, 255, 256, 257, 511, 1000, 2047, 2048, 3071, 3840, 4095]
    rows = np.array([b * T + t for b in range(B) for t in ts])
    ref = O.paged_decode(np.ascontiguousarray(h_qkv[rows]), h_k, h_v, 0, hq, hkv, hd,
                         np.repeat(tables_np, len(ts), axis=0),
                         np.array([t + 1 for _ in range(B) for t in ts], np.int32), 1,
                         threads=8)
    assert max_err(o[rows], ref) <= ATTN_ATOL


# --------------------------------------------------------------- config 3 --

def test_c3_decode_full_shape_matches_reference_kernels():
    """Config 3 at its exact shape: 32 sequences with 8192 cached tokens,
    Hq 28 / Hkv 4, hd 128; the new token (position 8192) is biased, rotated
    and appended by the fused launch (lc_rope_append_decode) before attention
    over all 8193 tokens. Reference: rope -> update_kv_cache -> flash-decoding
    per sequence."""
    R = O.ref_lib()
    hq, hkv, hd, B, ctx = 28, 4, 128, 32, 8192
    gen = torch.Generator(device="cuda")
    gen.manual_seed(3303)
    tables_np, nb = shuffled_tables(gen, [(ctx + 1 + 15) // 16] * B)
    shape = (nb, 1, hkv, 16, hd)
    k0, v0 = rand_bf16(gen, shape), rand_bf16(gen, shape)
    row = (hq + 2 * hkv) * hd
    qkv0 = rand_bf16(gen, (B, row))
    qb, kb, vb = split_bias(rand_bf16(gen, (row,), 0.01), hq, hkv, hd)
    cos_np, sin_np = O.rope_table(ctx + 16, hd, 1e6)
    cos, sin = to_device(cos_np), to_device(sin_np)
    tables = to_device(tables_np)
    pos_np = np.full(B, ctx, np.int32)
    pos = to_device(pos_np)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")

    k, v = k0.clone(), v0.clone()
    out = torch.empty((B, hq * hd), dtype=torch.bfloat16, device="cuda")
    L.rope_append_decode(out, qkv0, pos, qb, kb, vb, cos, sin, k, v, nb, 1, 0, hq, hkv, hd,
                         tables, ctx + 1, partition_tokens=512,
                         workspace=L.alloc_decode_workspace(B, hq, hkv, hd), dev_status=st)

    rqkv, rk, rv = qkv0.clone(), k0.clone(), v0.clone()
    rout = torch.empty((B, hq * hd), dtype=torch.bfloat16, device="cuda")
    s = _stream()
    assert R.ref_rope_append(_P(rqkv), row, B, 1, _P(pos), _P(qb), _P(kb), _P(vb), _P(cos),
                             _P(sin), _P(rk), _P(rv), 1, 0, hq, hkv, hd, _P(tables),
                             tables_np.shape[1], 32768, s) == 0
    host_pos = (C.c_int * B)(*pos_np.tolist())
    assert R.ref_paged_decode(_P(rout), hq * hd, _P(rqkv), row, _P(rk), _P(rv), 1, 0, hq, hkv,
                              hd, _P(tables), tables_np.shape[1], _P(pos), host_pos, B, 32768,
                              s) == 0
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert torch.equal(bits(k), bits(rk)) and torch.equal(bits(v), bits(rv))
    o = from_device(out)
    assert max_err(o, from_device(rout)) <= ATTN_ATOL

    # CPU oracle on every sequence (the pool fits host memory: ~0.5 GB).
    h_qkv = from_device(qkv0)
    h_k, h_v = from_device(k0), from_device(v0)
    O.rope_append(h_qkv, pos_np, from_device(qb), from_device(kb), from_device(vb), cos_np,
                  sin_np, h_k, h_v, 1, 0, hq, hkv, hd, tables_np)
    assert np.array_equal(h_k, from_device(k)) and np.array_equal(h_v, from_device(v))
    ref = O.paged_decode(h_qkv, h_k, h_v, 0, hq, hkv, hd, tables_np, pos_np, 1, len_offset=1,
                         threads=8)
    assert max_err(o, ref) <= ATTN_ATOL


# --------------------------------------------------------------- config 5 --

def test_c5_decode_full_shape_matches_reference_kernels():
    """Config 5 at its exact shape on one GPU (all 8 kv heads): 128 sequences,
    contexts U[1024, 32768], Hq 64 / Hkv 8, hd 128, ~9 GB of pages. Ours: the
    fused launch. Reference: its kernels per sequence. The new tokens' pages
    are saved before the first run and put back before the second, so that
    both runs start from the same pool and their appended rows can be compared
    bit for bit."""
    R = O.ref_lib()
    hq, hkv, hd, B = 64, 8, 128, 128
    rng = np.random.default_rng(5150)
    ctx = rng.integers(1024, 32768 + 1, B).astype(np.int32)
    pages = (ctx + 1 + 15) // 16
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5505)
    tables_np, nb = shuffled_tables(gen, pages)
    shape = (nb, 1, hkv, 16, hd)
    k, v = rand_bf16(gen, shape), rand_bf16(gen, shape)
    row = (hq + 2 * hkv) * hd
    qkv0 = rand_bf16(gen, (B, row))
    qb, kb, vb = split_bias(rand_bf16(gen, (row,), 0.01), hq, hkv, hd)
    cos_np, sin_np = O.rope_table(32768 + 16, hd, 1e6)
    cos, sin = to_device(cos_np), to_device(sin_np)
    tables = to_device(tables_np)
    pos = to_device(ctx)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    new_pages = torch.from_numpy(tables_np[np.arange(B), ctx // 16].astype(np.int64)).cuda()
    k_saved, v_saved = k.index_select(0, new_pages), v.index_select(0, new_pages)

    out = torch.empty((B, hq * hd), dtype=torch.bfloat16, device="cuda")
    L.rope_append_decode(out, qkv0, pos, qb, kb, vb, cos, sin, k, v, nb, 1, 0, hq, hkv, hd,
                         tables, int(ctx.max()) + 1,
                         workspace=L.alloc_decode_workspace(B, hq, hkv, hd), dev_status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    ours_k, ours_v = k.index_select(0, new_pages), v.index_select(0, new_pages)

    k.index_copy_(0, new_pages, k_saved)
    v.index_copy_(0, new_pages, v_saved)
    rqkv = qkv0.clone()
    rout = torch.empty((B, hq * hd), dtype=torch.bfloat16, device="cuda")
    s = _stream()
    assert R.ref_rope_append(_P(rqkv), row, B, 1, _P(pos), _P(qb), _P(kb), _P(vb), _P(cos),
                             _P(sin), _P(k), _P(v), 1, 0, hq, hkv, hd, _P(tables),
                             tables_np.shape[1], 32768, s) == 0
    host_pos = (C.c_int * B)(*ctx.tolist())
    assert R.ref_paged_decode(_P(rout), hq * hd, _P(rqkv), row, _P(k), _P(v), 1, 0, hq, hkv,
                              hd, _P(tables), tables_np.shape[1], _P(pos), host_pos, B, 32768,
                              s) == 0
    torch.cuda.synchronize()
    assert torch.equal(bits(ours_k), bits(k.index_select(0, new_pages)))
    assert torch.equal(bits(ours_v), bits(v.index_select(0, new_pages)))
    o = from_device(out)
    assert max_err(o, from_device(rout)) <= ATTN_ATOL

    # CPU oracle on four sequences (the longest, the shortest, two others),
    # from a compact host copy of their pages as they were before the step.
    k.index_copy_(0, new_pages, k_saved)
    v.index_copy_(0, new_pages, v_saved)
    seqs = sorted({int(ctx.argmax()), int(ctx.argmin()), 7, 100})
    hk, hv, ht = compact_pool(k, v, tables_np, seqs, [int(pages[b]) for b in seqs])
    h_qkv = from_device(qkv0)[seqs]
    O.rope_append(h_qkv, ctx[seqs], from_device(qb), from_device(kb), from_device(vb), cos_np,
                  sin_np, hk, hv, 1, 0, hq, hkv, hd, ht)
    ref = O.paged_decode(h_qkv, hk, hv, 0, hq, hkv, hd, ht, ctx[seqs], 1, len_offset=1,
                         threads=8)
    assert max_err(o[seqs], ref) <= ATTN_ATOL
    # the oracle's appended rows equal ours
    for i, b in enumerate(seqs):
        page = ht[i, ctx[b] // 16]
        r = ctx[b] % 16
        assert np.array_equal(hk[page, 0, :, r], from_device(ours_k[b])[0, :, r])
        assert np.array_equal(hv[page, 0, :, r], from_device(ours_v[b])[0, :, r])
