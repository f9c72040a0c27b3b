"""C-ABI library: loads, exports every declared symbol, validates arguments on
the host, and its host-side logic (RoPE table, sharding, workspace sizing)
behaves as specified. No GPU needed."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

import lucciola as L
import oracle.oracle as O

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions():
    names = []
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"^[A-Za-z_][\w \*]*?\b(lc_\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_headers_declare_the_path():
    names = declared_functions()
    for must in ("lc_rope", "lc_update_kv_cache", "lc_flash_decoding", "lc_rope_append",
                 "lc_paged_decode", "lc_paged_prefill", "lc_gather_kv", "lc_kv_cache_new"):
        assert must in names


@pytest.mark.parametrize("name", declared_functions())
def test_library_exports_declared_symbol(name):
    assert hasattr(L.lib, name), f"{name} declared in include/ but not exported"
    assert name in L.SIGNATURES, f"{name} has no ctypes signature in lucciola.py"


def test_status_strings():
    for code in range(0, 12):
        assert L.lib.lc_status_string(code)
    assert L.lib.lc_status_from_device_word(0) == 0
    assert L.lib.lc_status_from_device_word(L.LC_DEV_BAD_BLOCK) == 7
    assert L.lib.lc_status_from_device_word(L.LC_DEV_BAD_POS) == 7
    assert L.lib.lc_status_from_device_word(L.LC_DEV_TIMEOUT | 1) == 8
    assert "sm_100a" in L.version()


FAKE = 0x10000  # aligned non-null pointer value; never dereferenced by host validation


def decode_call(**kw):
    a = dict(out=FAKE, out_stride=14 * 64, q=FAKE, q_stride=14 * 64, k_pool=FAKE, v_pool=FAKE,
             num_blocks=64, num_layers=2, layer=1, hq=14, hkv=2, hd=64, tables=FAKE,
             table_stride=64, lens=FAKE, len_offset=0, batch=1, max_ctx=1024, ptok=0,
             scale=0.125, ws=None, ws_bytes=0, status=None, stream=None)
    a.update(kw)
    return L.lib.lc_paged_decode(a["out"], a["out_stride"], a["q"], a["q_stride"], a["k_pool"],
                                 a["v_pool"], a["num_blocks"], a["num_layers"], a["layer"],
                                 a["hq"], a["hkv"], a["hd"], a["tables"], a["table_stride"],
                                 a["lens"], a["len_offset"], a["batch"], a["max_ctx"], a["ptok"],
                                 a["scale"], a["ws"], a["ws_bytes"], a["status"], a["stream"])


def test_decode_rejects_bad_arguments_before_launch():
    assert decode_call(hd=96) == 2            # kernels.rs:40-45 supports 64/128 only
    assert decode_call(hd=80) == 2
    assert decode_call(hq=14, hkv=3) == 3     # GQA needs Hq % Hkv == 0
    assert decode_call(out=None) == 1
    assert decode_call(layer=2) == 1
    assert decode_call(num_blocks=0) == 1
    assert decode_call(k_pool=FAKE + 8) == 5  # TMA needs 16-byte aligned pools
    assert decode_call(q_stride=14 * 64 + 3) == 5
    assert decode_call(len_offset=2) == 1
    assert decode_call(batch=0) == 0          # nothing to do


def test_update_kv_cache_rejects_block_size():
    rc = L.lib.lc_update_kv_cache(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 0, FAKE, 2, 2, 1024, 64, 32,
                                  None)
    assert rc == 3


def test_rope_append_rejects_bad_arguments():
    def call(**kw):
        a = dict(hd=64, hq=14, hkv=2, row_stride=18 * 64, rope_rows=32768)
        a.update(kw)
        return L.lib.lc_rope_append(FAKE, a["row_stride"], 1, 1, FAKE, FAKE, FAKE, FAKE, FAKE,
                                    FAKE, a["rope_rows"], FAKE, FAKE, 64, 2, 0, a["hq"], a["hkv"],
                                    a["hd"], FAKE, 64, None, None)
    assert call(hd=72) == 2
    assert call(hkv=4) == 3
    assert call(row_stride=17 * 64) == 1
    assert call(rope_rows=0) == 1


def test_prefill_rejects_bad_arguments():
    rc = L.lib.lc_paged_prefill(FAKE, 12 * 128, FAKE, 12 * 128, FAKE, FAKE, 64, 2, 0, 12, 2, 96,
                                FAKE, 64, FAKE, 1, 128, 0, 0.1, None, None)
    assert rc in (2, 11)


def test_proj_gemm_rejects_bad_arguments():
    def call(**kw):
        a = dict(out=FAKE, out_stride=1152, x=FAKE, x_stride=896, w=FAKE, w_stride=896, M=300,
                 N=1152, K=896, res=None, res_stride=0)
        a.update(kw)
        return L.lib.lc_proj_gemm(a["out"], a["out_stride"], a["x"], a["x_stride"], a["w"],
                                  a["w_stride"], a["M"], a["N"], a["K"], a["res"],
                                  a["res_stride"], None)
    assert call(out=None) == 1
    assert call(N=40, out_stride=40) == 3        # N a multiple of the 32-column store box
    assert call(K=900, x_stride=904, w_stride=904) == 3  # K a multiple of 8
    assert call(M=-1) == 3
    assert call(x_stride=800) == 1               # row shorter than K
    assert call(out_stride=1000) == 1
    assert call(x=FAKE + 8) == 5                 # TMA sources 16-byte aligned
    assert call(w_stride=900) == 5
    assert call(res=FAKE + 2, res_stride=1152) == 5
    assert call(res=FAKE, res_stride=1000) == 1
    assert call(M=0) == 0                        # nothing to do
    assert call(M=0, res=FAKE, res_stride=1152) == 0


def test_qkv_proj_rope_append_rejects_bad_arguments():
    def call(**kw):
        a = dict(qkv=FAKE, hd=64, hq=14, hkv=2, hidden=896, seqs=2, tps=8, layer=0, layers=2,
                 q_bias=FAKE, rope_rows=4096)
        a.update(kw)
        n = (a["hq"] + 2 * a["hkv"]) * a["hd"]
        return L.lib.lc_qkv_proj_rope_append(
            a["qkv"], n, FAKE, a["hidden"], FAKE, a["hidden"], a["hidden"], a["seqs"], a["tps"],
            FAKE, a["q_bias"], FAKE, FAKE, FAKE, FAKE, a["rope_rows"], FAKE, FAKE, 64,
            a["layers"], a["layer"], a["hq"], a["hkv"], a["hd"], FAKE, 64, None, None)
    assert call(hd=96) == 2
    assert call(hkv=3) == 3
    assert call(layer=2) == 1
    assert call(tps=0) == 1
    assert call(rope_rows=0) == 1
    assert call(q_bias=None) == 1
    assert call(q_bias=FAKE + 4) == 5
    assert call(qkv=None) == 1
    assert call(hidden=900) == 3
    assert call(seqs=0) == 0


def test_token_selection_rejects_bad_arguments():
    V = 151936
    assert L.lib.lc_argmax(None, V, V, 1, FAKE, None) == 1
    assert L.lib.lc_argmax(FAKE, V - 1, V, 1, FAKE, None) == 1  # row shorter than vocab
    assert L.lib.lc_argmax(FAKE, V, V, -1, FAKE, None) == 1
    assert L.lib.lc_argmax(FAKE, V, V, 0, FAKE, None) == 0

    # candidate counts: 32 * (top_k / 32), a power of two in 32 .. 1024
    assert L.lib.lc_sample_workspace_size(4, 64) == 4 * 64 * 8
    assert L.lib.lc_sample_workspace_size(4, 70) == 4 * 64 * 8
    assert L.lib.lc_sample_workspace_size(2, 1024) == 2 * 1024 * 8
    for bad in (0, 31, 96, 100, 2048):
        assert L.lib.lc_sample_workspace_size(4, bad) == 0
    assert L.lib.lc_sample_workspace_size(0, 64) == 0

    def sample(vocab=V, batch=2, top_k=64, ws=FAKE, ws_bytes=2 * 64 * 8, top_p=FAKE):
        return L.lib.lc_sample_top_p(FAKE, vocab, vocab, batch, top_k, top_p, FAKE, FAKE, ws,
                                     ws_bytes, None)
    assert sample(top_p=None) == 1
    assert sample(top_k=96) == 3                 # no reference kernel for 96 candidates
    assert sample(vocab=31) == 3
    assert sample(ws_bytes=2 * 64 * 8 - 1) == 4
    assert sample(ws=None) == 4
    assert sample(batch=0, ws=None, ws_bytes=0) == 0


def test_gated_decode_needs_a_gate():
    rc = L.lib.lc_rope_append_decode_gated(
        FAKE, 14 * 64, FAKE, 18 * 64, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 4096, FAKE, FAKE, 64, 2,
        0, 14, 2, 64, FAKE, 64, 1, 1024, 0, 0.125, None, 0, None, None, None)
    assert rc == 1


def test_peer_exchange_rejects_bad_arguments():
    region = C.c_void_p()
    handle = (C.c_uint8 * L.PEER_HANDLE_BYTES)()
    assert L.lib.lc_peer_region_alloc(L.PEER_SIGNAL_BYTES, C.byref(region), handle) == 1
    g = C.c_void_p()
    regs = (C.c_void_p * 2)(FAKE, FAKE + 4096)
    assert L.lib.lc_peer_group_local(2, 2, regs, 4096, C.byref(g)) == 1   # rank outside
    assert L.lib.lc_peer_group_local(0, 9, regs, 4096, C.byref(g)) == 1   # > 8 ranks
    assert L.lib.lc_peer_group_local(0, 2, regs, 256, C.byref(g)) == 1    # signal words only
    assert L.lib.lc_peer_group_open(0, 2, None, 4096, bytes(128), C.byref(g)) == 1
    assert L.lib.lc_peer_wait(None, None, None) == 1
    # a group over addresses this process holds: host bookkeeping only
    assert L.lib.lc_peer_group_local(0, 2, regs, 4096, C.byref(g)) == 0

    def call(out, batch, group=g):
        return L.lib.lc_rope_append_decode_peer(
            out, 14 * 64, FAKE, 18 * 64, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 4096, FAKE, FAKE,
            64, 2, 0, 14, 2, 64, FAKE, 64, batch, 1024, 0, 0.125, FAKE, 1 << 30, None, group,
            None)
    assert call(FAKE, 2) == 1             # rows over the signal words
    assert call(FAKE + 256, 3) == 1       # row 2 ends past the region's 4096 bytes
    assert call(FAKE + 256, 2, None) == 1  # no group
    L.lib.lc_peer_group_destroy(g)


def test_workspace_sizes():
    # host-only sizing assumes a 148-SM B200: 3 CTAs/SM at hd 64, 2 at hd 128;
    # int32 counters, then tagged 64-bit partial words (log2-sum-exp, outputs)
    segs = 64 * 2                      # batch x (kv heads x 8-head slices)
    slots = segs + 148 * 3
    want = ((segs * 4 + 255) // 256 * 256 + (slots * 8 * 8 + 255) // 256 * 256
            + slots * 8 * 64 * 8)
    assert L.paged_decode_workspace_size(64, 14, 2, 64) == want
    assert L.paged_decode_workspace_size(1, 64, 4, 128) > 0   # group 16: two slices per kv head
    assert L.paged_decode_workspace_size(4, 14, 3, 64) == 0   # invalid shape
    assert L.paged_decode_workspace_size(4, 14, 2, 96) == 0
    assert L.flash_decoding_workspace_size(14, 64, 32768) >= L.paged_decode_workspace_size(1, 14, 2, 64)


@pytest.mark.parametrize("hd,base,scale", [(64, 1e6, 0.0), (128, 1e6, 0.0), (128, 1e4, 4.0),
                                            (64, 10000.0, 0.0)])
def test_rope_table_host_matches_oracle_bit_exact(hd, base, scale):
    c, s = L.rope_table_host(2048, hd, base, scale)
    oc, os_ = O.rope_table(2048, hd, base, scale)
    assert np.array_equal(c.view(np.uint32), oc.view(np.uint32))
    assert np.array_equal(s.view(np.uint32), os_.view(np.uint32))


def py_lpt(lens, ranks):
    order = sorted(range(len(lens)), key=lambda b: (-lens[b], b))
    load = [0] * ranks
    out = [0] * len(lens)
    for b in order:
        r = min(range(ranks), key=lambda i: (load[i], i))
        out[b] = r
        load[r] += max(lens[b], 0)
    return out


@pytest.mark.parametrize("ranks", [1, 2, 4, 8])
def test_shard_sequences_lpt(ranks):
    rng = np.random.default_rng(ranks)
    lens = rng.integers(256, 4097, 64).tolist()
    got = L.shard_sequences(lens, ranks)
    assert got == py_lpt(lens, ranks)
    loads = [sum(l for l, r in zip(lens, got) if r == k) for k in range(ranks)]
    assert max(loads) - min(loads) <= max(lens)          # LPT bound
    assert sorted(set(got)) == list(range(ranks))


def test_shard_kv_heads():
    assert [L.shard_kv_heads(64, 8, 8, r) for r in range(8)] == [(r, 1) for r in range(8)]
    assert [L.shard_kv_heads(64, 8, 4, r) for r in range(4)] == [(2 * r, 2) for r in range(4)]
    with pytest.raises(L.LucciolaError):
        L.shard_kv_heads(64, 8, 3, 0)
