"""The CPU oracle itself: bf16 rounding, the reference algorithm against an
independent float64 statement of attention, the split-K / online-softmax
algebra the CUDA kernel relies on, prefill-as-sequential-decode, and the
page gather. No GPU needed."""
import numpy as np
import pytest

import oracle.oracle as O
from conftest import ATTN_ATOL
from workloads import make_case, randn_bf16


def test_bf16_round_to_nearest_even():
    import torch
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 10 ** rng.uniform(-3, 3, 100000).astype(np.float32),
                        np.array([0.0, -0.0, 1.0, 1.00390625, 1.005859375, 3.4e38, -3.4e38,
                                  1e-40, np.inf, -np.inf], np.float32)])
    ours = O.f32_to_bf16(x)
    ref = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, ref)
    lib = O.lib()
    for v in x[:2000]:
        assert lib.lco_f32_to_bf16(float(v)) == O.f32_to_bf16(np.array([v]))[0]
    # ties go to even
    assert O.f32_to_bf16(np.array([1.00390625], np.float32))[0] == 0x3F80
    assert O.f32_to_bf16(np.array([1.01171875], np.float32))[0] == 0x3F82


def dense_kv(case, b, n):
    """Gather of sequence b's first n tokens: [n, Hkv, hd] float64."""
    k, v = O.gather_kv(case.k_pool, case.v_pool, case.layer, case.hkv, case.hd, case.tables[b:b + 1],
                       np.array([n], np.int32), n, case.num_layers)
    return O.bf16_to_f32(k[0]).astype(np.float64), O.bf16_to_f32(v[0]).astype(np.float64)


def attention_f64(q, k, v, hq, hkv, hd, scale):
    """q [Hq*hd] f64, k/v [n, Hkv, hd] -> [Hq, hd]."""
    q = q.reshape(hq, hd)
    grp = hq // hkv
    out = np.zeros((hq, hd))
    for h in range(hq):
        s = k[:, h // grp, :] @ q[h] * scale
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ v[:, h // grp, :]
    return out


@pytest.mark.parametrize("hq,hkv,hd,n", [(14, 2, 64, 1), (14, 2, 64, 37), (28, 4, 128, 300),
                                         (12, 2, 128, 16), (8, 8, 64, 33), (16, 1, 128, 129)])
def test_oracle_attention_matches_float64(hq, hkv, hd, n):
    case = make_case(1, hq, hkv, hd, [n], seed=n)
    out = O.paged_decode(case.q, case.k_pool, case.v_pool, case.layer, hq, hkv, hd, case.tables,
                         case.ctx, case.num_layers)
    k, v = dense_kv(case, 0, n)
    ref = attention_f64(O.bf16_to_f32(case.q[0]).astype(np.float64), k, v, hq, hkv, hd,
                        1.0 / np.sqrt(hd))
    got = O.bf16_to_f32(out[0]).reshape(hq, hd)
    assert np.abs(got - ref).max() < 1e-2  # bf16 output rounding dominates
    assert np.abs(got - ref).max() <= np.abs(ref).max() * 2 ** -7 + 1e-6


def test_batched_oracle_is_per_sequence_reference():
    case = make_case(5, 14, 2, 64, [1, 17, 16, 200, 63], seed=3)
    out = O.paged_decode(case.q, case.k_pool, case.v_pool, case.layer, 14, 2, 64, case.tables,
                         case.ctx, case.num_layers, threads=3)
    for b in range(5):
        one = O.flash_decoding(case.q[b], case.k_pool, case.v_pool, case.tables[b], case.layer, 14,
                               2, 64, int(case.ctx[b]) - 1, case.num_layers)
        assert np.array_equal(out[b], one)
    # len_offset=1: lengths given as positions
    out2 = O.paged_decode(case.q, case.k_pool, case.v_pool, case.layer, 14, 2, 64, case.tables,
                          case.ctx - 1, case.num_layers, len_offset=1)
    assert np.array_equal(out, out2)


def split_k_reference(s, v, part):
    """Split-K in the kernel's form: per partition o_p = softmax-weighted mean and
    lse_p = log2 sum 2^(s*log2e); merged with weights 2^(lse_p - max lse)."""
    s2 = s * np.log2(np.e)
    outs, lses = [], []
    for t0 in range(0, len(s), part):
        x = s2[t0:t0 + part]
        m = x.max()
        p = np.exp2(x - m)
        outs.append(p @ v[t0:t0 + part] / p.sum())
        lses.append(m + np.log2(p.sum()))
    lses = np.array(lses)
    w = np.exp2(lses - lses.max())
    return (w[:, None] * np.array(outs)).sum(0) / w.sum()


def online_reference(s, v, page):
    """Online softmax over pages in the kernel's form (running max, rescale)."""
    s2 = s * np.log2(np.e)
    m, l, o = -np.inf, 0.0, np.zeros(v.shape[1])
    for t0 in range(0, len(s), page):
        x = s2[t0:t0 + page]
        mn = max(m, x.max())
        a = np.exp2(m - mn)
        p = np.exp2(x - mn)
        l = l * a + p.sum()
        o = o * a + p @ v[t0:t0 + page]
        m = mn
    return o / l


@pytest.mark.parametrize("n,part", [(1, 16), (100, 16), (4096, 512), (777, 64), (513, 512)])
def test_split_k_and_online_softmax_equal_two_pass(n, part):
    rng = np.random.default_rng(n)
    s = rng.standard_normal(n) * 3
    v = rng.standard_normal((n, 64))
    p = np.exp(s - s.max())
    two_pass = p @ v / p.sum()
    np.testing.assert_allclose(split_k_reference(s, v, part), two_pass, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(online_reference(s, v, 16), two_pass, rtol=1e-12, atol=1e-12)


def test_prefill_oracle_is_causal_attention():
    hq, hkv, hd, T = 12, 2, 128, 40
    start = np.array([0, 23], np.int32)
    case = make_case(2, hq, hkv, hd, start + T, seed=7)
    q = randn_bf16(np.random.default_rng(1), (2 * T, hq * hd))
    out = O.paged_prefill(q, case.k_pool, case.v_pool, case.layer, hq, hkv, hd, case.tables,
                          start, T, case.num_layers, threads=2)
    for b in range(2):
        k, v = dense_kv(case, b, int(start[b]) + T)
        for t in (0, 1, T // 2, T - 1):
            n = int(start[b]) + t + 1
            ref = attention_f64(O.bf16_to_f32(q[b * T + t]).astype(np.float64), k[:n], v[:n], hq,
                                hkv, hd, 1 / np.sqrt(hd))
            got = O.bf16_to_f32(out[b * T + t]).reshape(hq, hd)
            assert np.abs(got - ref).max() < ATTN_ATOL / 2


def test_gather_oracle_is_table_lookup():
    case = make_case(3, 14, 2, 64, [5, 16, 40], seed=11)
    k, v = O.gather_kv(case.k_pool, case.v_pool, case.layer, 2, 64, case.tables, case.ctx, 48,
                       case.num_layers)
    for b in range(3):
        for t in range(int(case.ctx[b])):
            blk = case.tables[b, t // 16]
            assert np.array_equal(k[b, t], case.k_pool[blk, case.layer, :, t % 16, :])
            assert np.array_equal(v[b, t], case.v_pool[blk, case.layer, :, t % 16, :])
        assert not k[b, int(case.ctx[b]):].any()


def test_oracle_rejects_out_of_range_block():
    case = make_case(1, 14, 2, 64, [40], seed=2)
    case.tables[0, 1] = case.num_blocks
    with pytest.raises(ValueError):
        O.paged_decode(case.q, case.k_pool, case.v_pool, case.layer, 14, 2, 64, case.tables,
                       case.ctx, case.num_layers)


def test_rope_append_oracle_semantics():
    """rope -> append: q/k rotated (norm-preserving up to bf16), pools get k and v+bias."""
    hq, hkv, hd = 14, 2, 64
    rng = np.random.default_rng(5)
    case = make_case(2, hq, hkv, hd, [30, 70], seed=5, extra_pages=1)
    row = (hq + 2 * hkv) * hd
    qkv = randn_bf16(rng, (2, row))
    qb, kb, vb = (randn_bf16(rng, (n * hd,)) for n in (hq, hkv, hkv))
    cos, sin = O.rope_table(128, hd, 1e6)
    pos = case.ctx.copy()  # append at position ctx (the page after is reserved)
    before = qkv.copy()
    kp, vp = case.k_pool.copy(), case.v_pool.copy()
    O.rope_append(qkv, pos, qb, kb, vb, cos, sin, kp, vp, case.num_layers, case.layer, hq, hkv,
                  hd, case.tables)
    for b in range(2):
        x = O.bf16_to_f32(before[b]) + np.concatenate([O.bf16_to_f32(qb), O.bf16_to_f32(kb),
                                                       O.bf16_to_f32(vb)])
        y = O.bf16_to_f32(qkv[b])
        nq = (hq + hkv) * hd
        xr = x[:nq].reshape(-1, 2, hd // 2)
        yr = y[:nq].reshape(-1, 2, hd // 2)
        np.testing.assert_allclose(np.hypot(yr[:, 0], yr[:, 1]), np.hypot(xr[:, 0], xr[:, 1]),
                                   rtol=2e-2, atol=2e-2)
        assert np.array_equal(qkv[b, nq:], before[b, nq:])  # v is not modified
        p = int(pos[b])
        blk = case.tables[b, p // 16]
        assert np.array_equal(kp[blk, case.layer, :, p % 16, :].ravel(), qkv[b, hq * hd:nq])
        assert np.array_equal(vp[blk, case.layer, :, p % 16, :].ravel(),
                              O.f32_to_bf16(O.bf16_to_f32(before[b, nq:]) + O.bf16_to_f32(vb)))


# ----------------------------------------------------------------- sampling --

def _bf(values):
    return O.f32_to_bf16(np.asarray(values, np.float32))


def test_oracle_argmax_tie_order():
    """argmax_kernel keeps, among equal maxima, the lowest thread i % 1024 and
    then that thread's first index (src/kernels/sampling.cu)."""
    x = np.full(5000, O.f32_to_bf16(np.float32(0.0)), np.uint16)
    x[[10, 1029, 4000]] = O.f32_to_bf16(np.float32(3.0))   # threads 10, 5, 928
    assert int(O.argmax(x)[0]) == 1029
    x[[1029]] = O.f32_to_bf16(np.float32(1.0))
    x[[2058, 10]] = O.f32_to_bf16(np.float32(3.0))           # thread 10 twice: first index
    assert int(O.argmax(x)[0]) == 10
    assert int(O.argmax(_bf([-2e30] * 64))[0]) == -1         # nothing above -1e30


def test_oracle_top_k_filter_partitions_and_ties():
    """Each of 32 partitions yields its own top k/32 (not the global top-k);
    equal values go in the bit-reversed warp / lane order of thread i % 256."""
    vocab = 32 * 600
    x = np.zeros(vocab, np.float32)
    x[:600] = np.arange(600, dtype=np.float32) / 100.0   # partition 0 holds the 600 largest
    keys, vals = O.top_k_filter(O.f32_to_bf16(x), 128)   # 4 per partition
    assert keys[0] == 599 and vals[0] == 6.0               # partition 0: its own top 4
    # 5.97 and 5.98 round to the same bf16 as 5.96: indices 596-598 tie on
    # threads 84-86 (warp 2, lanes 20-22; bit-reversed lane order 20, 22, 21)
    assert list(keys[1:4]) == [596, 598, 597]
    # partition 1 is all zeros: thread 0 (warp 0, lane 0) comes first with all
    # of its elements (offsets 0, 256, 512), then lane 16 (bit-reversed 1)
    assert list(keys[4:8]) == [600, 856, 1112, 616] and (vals[4:8] == 0).all()


def test_oracle_top_p_sample_small_cases():
    keys = np.arange(32, dtype=np.int32)
    vals = np.full(32, -1e30, np.float32)
    vals[0], vals[1] = 0.0, float(np.log(3.0))    # probabilities 1/4, 3/4 after sorting: 3/4 first
    k, m = O.top_p_sample(keys, vals, 0.5, 0.5)   # cutoff at 3/4: always key 1
    assert k == 1
    k, m = O.top_p_sample(keys, vals, 0.9, 0.9)   # cutoff 1.0, target 0.9 > 0.75: key 0
    assert k == 0
