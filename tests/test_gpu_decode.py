"""Paged decode attention on the GPU (lc_paged_decode / lc_flash_decoding /
lc_gather_kv through the C ABI) against the CPU oracle of the reference
algorithm: max-abs error <= ATTN_ATOL for outputs, bit-exact for gathers."""
import numpy as np
import pytest

import lucciola as L
import oracle.oracle as O
from conftest import ATTN_ATOL
from workloads import from_device, make_case, to_device

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev_case(case):
    return dict(k=to_device(case.k_pool), v=to_device(case.v_pool), q=to_device(case.q),
                tables=to_device(case.tables))


def gpu_decode(case, d=None, partition_tokens=0, len_offset=0, q=None, out=None, ws=None,
               lens=None):
    d = d or dev_case(case)
    q = d["q"] if q is None else q
    if out is None:
        out = torch.empty(case.batch, case.hq * case.hd, dtype=torch.bfloat16, device="cuda")
    if lens is None:
        lens = to_device((case.ctx - len_offset).astype(np.int32))
    if ws is None:
        ws = L.alloc_decode_workspace(case.batch, case.hq, case.hkv, case.hd)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.paged_decode(out, q, d["k"], d["v"], case.num_blocks, case.num_layers, case.layer, case.hq,
                   case.hkv, case.hd, d["tables"], lens, max(case.max_ctx, 1),
                   len_offset=len_offset, partition_tokens=partition_tokens, workspace=ws,
                   dev_status=status)
    torch.cuda.synchronize()
    return out, int(status.item())


def oracle_decode(case, q=None):
    return O.paged_decode(case.q if q is None else q, case.k_pool, case.v_pool, case.layer,
                          case.hq, case.hkv, case.hd, case.tables, case.ctx, case.num_layers,
                          threads=8)


def max_err(a_bits, b_bits):
    return float(np.abs(O.bf16_to_f32(a_bits) - O.bf16_to_f32(b_bits)).max())


SHAPES = [(14, 2, 64), (28, 4, 128), (12, 2, 128), (64, 8, 128), (16, 2, 64), (40, 8, 128),
          (32, 2, 64), (8, 8, 64), (24, 2, 128)]


@pytest.mark.parametrize("hq,hkv,hd", SHAPES)
def test_decode_ragged_matches_oracle(hq, hkv, hd):
    ctx = [1, 15, 16, 17, 33, 64, 65, 100, 511, 512, 513, 1000]
    case = make_case(len(ctx), hq, hkv, hd, ctx, seed=hq * 7 + hkv + hd)
    out, st = gpu_decode(case)
    ref = oracle_decode(case)
    assert st == 0
    assert max_err(from_device(out), ref) <= ATTN_ATOL


@pytest.mark.parametrize("ptok", [16, 64, 128, 512, 4096])
def test_decode_partition_sizes(ptok):
    ctx = [1, 16, 17, 700, 2049, 4096]
    case = make_case(len(ctx), 14, 2, 64, ctx, seed=ptok)
    out, st = gpu_decode(case, partition_tokens=ptok)
    assert st == 0
    assert max_err(from_device(out), oracle_decode(case)) <= ATTN_ATOL


def test_decode_long_context_many_partitions():
    case = make_case(2, 28, 4, 128, [8192, 5000], seed=5)
    out, st = gpu_decode(case, partition_tokens=64)  # 128 partitions per sequence
    assert st == 0
    assert max_err(from_device(out), oracle_decode(case)) <= ATTN_ATOL


def test_decode_context_hint_below_real_lengths():
    # max_context_len hint far below the real lengths trims the grid; the split
    # over the CTAs that remain still covers every page.
    case = make_case(2, 14, 2, 64, [3000, 1200], seed=9)
    d = dev_case(case)
    out = torch.empty(2, 14 * 64, dtype=torch.bfloat16, device="cuda")
    ws = L.alloc_decode_workspace(2, 14, 2, 64)
    L.paged_decode(out, d["q"], d["k"], d["v"], case.num_blocks, case.num_layers, case.layer, 14,
                   2, 64, d["tables"], to_device(case.ctx), 128, partition_tokens=64, workspace=ws)
    torch.cuda.synchronize()
    assert max_err(from_device(out), oracle_decode(case)) <= ATTN_ATOL


def test_decode_strided_q_and_out_rows():
    """q read straight from qkv_states rows; out written into a wider buffer."""
    hq, hkv, hd = 28, 4, 128
    case = make_case(5, hq, hkv, hd, [40, 300, 1, 77, 1024], seed=21)
    d = dev_case(case)
    row = (hq + 2 * hkv) * hd
    qkv = torch.randn(case.batch, row, device="cuda").to(torch.bfloat16)
    qkv[:, :hq * hd] = d["q"]
    wide = torch.zeros(case.batch, hq * hd + 256, dtype=torch.bfloat16, device="cuda")
    out, st = gpu_decode(case, d=d, q=qkv, out=wide)
    assert st == 0
    assert max_err(from_device(wide[:, :hq * hd].contiguous()), oracle_decode(case)) <= ATTN_ATOL
    assert not wide[:, hq * hd:].any()


def test_decode_out_rows_without_16_byte_alignment():
    """out rows 2 bytes past a 16-byte boundary with an odd stride: the
    kernels fall back to element stores there."""
    hq, hkv, hd = 14, 2, 64
    case = make_case(6, hq, hkv, hd, [1, 40, 700, 1500, 3000, 17], seed=31)
    d = dev_case(case)
    wide = torch.zeros(case.batch, hq * hd + 3, dtype=torch.bfloat16, device="cuda")
    out = wide[:, 1:1 + hq * hd]
    _, st = gpu_decode(case, d=d, out=out)
    assert st == 0
    assert max_err(from_device(out.contiguous()), oracle_decode(case)) <= ATTN_ATOL
    assert not wide[:, 0].any() and not wide[:, 1 + hq * hd:].any()


def test_decode_positions_mode_and_workspace_reuse():
    """len_offset=1 (positions, like the reference's pos_ptr) and two calls in a
    row on one workspace give the same result (arrival counters reset)."""
    case = make_case(6, 14, 2, 64, [5, 600, 1024, 1025, 2000, 16], seed=4)
    d = dev_case(case)
    ws = L.alloc_decode_workspace(6, 14, 2, 64)
    a, _ = gpu_decode(case, d=d, partition_tokens=64, len_offset=1, ws=ws)
    a = from_device(a)
    b, _ = gpu_decode(case, d=d, partition_tokens=64, len_offset=1, ws=ws)
    assert np.array_equal(a, from_device(b))
    assert max_err(a, oracle_decode(case)) <= ATTN_ATOL
    # arrival counters and every tagged partial word back at zero
    assert not ws.any()


def test_decode_empty_context_gives_zeros():
    case = make_case(3, 14, 2, 64, [0, 20, 0], seed=1)
    case.tables[0, :] = -1
    out, st = gpu_decode(case)
    o = from_device(out)
    assert st == 0
    assert not o[0].any() and not o[2].any()
    ref = oracle_decode(case)
    assert max_err(o[1], ref[1]) <= ATTN_ATOL


def test_decode_bad_block_is_reported_not_dereferenced():
    case = make_case(2, 14, 2, 64, [40, 40], seed=8)
    case.tables[1, 1] = case.num_blocks + 5
    out, st = gpu_decode(case)
    assert st & L.LC_DEV_BAD_BLOCK
    assert L.lib.lc_status_from_device_word(st) == 7
    o = O.bf16_to_f32(from_device(out))
    assert np.isfinite(o).all()
    # sequence 0 is unaffected
    good = make_case(2, 14, 2, 64, [40, 40], seed=8)
    assert max_err(from_device(out)[0], oracle_decode(good)[0]) <= ATTN_ATOL


def test_decode_context_beyond_table_is_clamped_and_reported():
    case = make_case(1, 14, 2, 64, [64], seed=3)
    d = dev_case(case)
    lens = to_device(np.array([64 + 50], np.int32))  # table has 4 pages
    out, st = gpu_decode(case, d=d, lens=lens)
    assert st & L.LC_DEV_BAD_POS
    assert max_err(from_device(out), oracle_decode(case)) <= ATTN_ATOL


@pytest.mark.parametrize("hq,hkv,hd,batch,lo,hi", [
    (14, 2, 64, 64, 256, 4096),     # BASELINE config 2 shape
    (28, 4, 128, 8, 8192, 8192),    # config 3 shape, fewer sequences
    (14, 2, 64, 3000, 1, 40),       # many short sequences: multi-entry scan slices
    (64, 8, 128, 16, 1024, 9000),   # config 5 shape, fewer/shorter sequences
])
def test_decode_persistent_split_shapes(hq, hkv, hd, batch, lo, hi):
    rng = np.random.default_rng(batch + hd)
    ctx = rng.integers(lo, hi + 1, batch).astype(np.int32)
    ctx[rng.integers(0, batch, max(1, batch // 10))] = 0  # some empty sequences
    case = make_case(batch, hq, hkv, hd, ctx, seed=batch)
    out, st = gpu_decode(case)
    assert st == 0
    o = from_device(out)
    assert max_err(o, oracle_decode(case)) <= ATTN_ATOL
    assert not o[ctx == 0].any()


def test_decode_one_sequence_split_over_many_ctas():
    """C1 shape: one sequence, each segment spread over dozens of CTAs."""
    case = make_case(1, 14, 2, 64, [1024], seed=12)
    for ptok in (0, 16, 32):
        out, st = gpu_decode(case, partition_tokens=ptok)
        assert st == 0
        assert max_err(from_device(out), oracle_decode(case)) <= ATTN_ATOL


@pytest.mark.parametrize("hd", [64, 128])
def test_gather_is_bit_exact(hd):
    case = make_case(4, 8, 2, hd, [1, 16, 47, 300], seed=hd)
    d = dev_case(case)
    M = 320
    ko = torch.zeros(4, M, 2, hd, dtype=torch.bfloat16, device="cuda")
    vo = torch.zeros_like(ko)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.gather_kv(ko, vo, d["k"], d["v"], case.num_blocks, case.num_layers, case.layer, 2, hd,
                d["tables"], to_device(case.ctx), M, dev_status=st)
    torch.cuda.synchronize()
    rk, rv = O.gather_kv(case.k_pool, case.v_pool, case.layer, 2, hd, case.tables, case.ctx, M,
                         case.num_layers)
    assert int(st.item()) == 0
    assert np.array_equal(from_device(ko), rk)
    assert np.array_equal(from_device(vo), rv)


def test_flash_decoding_reference_shape():
    """lc_flash_decoding: the drop-in for flash_decoding_kernel_{64,128}."""
    for hq, hkv, hd, pos in [(14, 2, 64, 1023), (28, 4, 128, 0), (12, 2, 128, 517)]:
        case = make_case(1, hq, hkv, hd, [pos + 1], seed=pos, table_stride=2048)
        d = dev_case(case)
        max_seq = 32768
        ws = torch.zeros(L.flash_decoding_workspace_size(hq, hd, max_seq), dtype=torch.uint8,
                         device="cuda")
        out = torch.empty(hq * hd, dtype=torch.bfloat16, device="cuda")
        pos_t = to_device(np.array([pos], np.int32))
        L.flash_decoding(out, d["q"], d["k"], d["v"], d["tables"], case.layer, hq, hkv, hd,
                         max_seq, pos_t, 1.0 / np.sqrt(hd), 16, case.num_layers, pos,
                         case.num_blocks, ws)
        torch.cuda.synchronize()
        ref = O.flash_decoding(case.q[0], case.k_pool, case.v_pool, case.tables[0], case.layer,
                               hq, hkv, hd, pos, case.num_layers)
        assert max_err(from_device(out), ref) <= ATTN_ATOL


def test_decode_all_sequences_empty():
    case = make_case(5, 14, 2, 64, [0, 0, 0, 0, 0], seed=2)
    d = dev_case(case)
    out = torch.full((5, 14 * 64), 7.0, dtype=torch.bfloat16, device="cuda")
    gpu_decode(case, d=d, out=out)
    assert not out.any()
