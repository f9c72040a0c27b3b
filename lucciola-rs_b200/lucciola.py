"""Python binding of liblucciola_b200.so (the C ABI in include/lucciola_attn.h).

A thin ctypes layer: every wrapper forwards device pointers of torch tensors and
the current CUDA stream to the C entry point of the same name and raises
LucciolaError on a non-zero status. There is no fallback: if the library is
missing, importing this module fails.
"""
from __future__ import annotations

import ctypes as C
import math
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "liblucciola_b200.so"

if not LIB_PATH.exists():
    raise ImportError(
        f"{LIB_PATH} is missing; build it with `python lucciola-rs_b200/build.py`")

lib = C.CDLL(str(LIB_PATH))

_vp, _i32, _i64, _f32, _sz = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t
_pi32 = C.POINTER(C.c_int)

# name -> (restype, argtypes), in the order of include/lucciola_attn.h
SIGNATURES = {
    "lc_status_string": (C.c_char_p, [_i32]),
    "lc_status_from_device_word": (_i32, [_i32]),
    "lc_version": (C.c_char_p, []),
    "lc_set_dependent_launch": (_i32, [_i32]),
    "lc_rope": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    "lc_update_kv_cache": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _vp, _i32, _i32, _i32,
                                  _i32, _i32, _vp]),
    "lc_flash_decoding_workspace_size": (_sz, [_i32, _i32, _i32]),
    "lc_flash_decoding": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp,
                                 _f32, _i32, _i32, _i32, _i64, _vp, _sz, _vp]),
    "lc_rope_append": (_i32, [_vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _vp,
                              _vp, _i64, _i32, _i32, _i32, _i32, _i32, _vp, _i32, _vp, _vp]),
    "lc_paged_decode_workspace_size": (_sz, [_i32, _i32, _i32, _i32]),
    "lc_paged_decode_workspace_init": (_i32, [_vp, _sz, _vp]),
    "lc_paged_decode": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _i32, _i32, _i32, _i32,
                               _i32, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _f32, _vp, _sz,
                               _vp, _vp]),
    "lc_rope_append_decode": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _i32,
                                     _vp, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _vp, _i32,
                                     _i32, _i32, _i32, _f32, _vp, _sz, _vp, _vp]),
    "lc_rope_append_decode_gated": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp,
                                           _i32, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _i32,
                                           _vp, _i32, _i32, _i32, _i32, _f32, _vp, _sz, _vp, _vp,
                                           _vp]),
    "lc_paged_decode_static": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _i32, _i32, _i32,
                                      _i32, _i32, _vp, _i32, _vp, _i32, _i32, _i32, _i32, _f32,
                                      _vp, _vp]),
    "lc_proj_decode_plan": (_i32, [_i32, _i32, _pi32, _pi32, _pi32, _pi32]),
    "lc_paged_prefill": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _i32, _i32, _i32, _i32,
                                _i32, _vp, _i32, _vp, _i32, _i32, _i32, _f32, _vp, _vp]),
    "lc_gather_kv": (_i32, [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _vp, _i32, _vp,
                            _i32, _i32, _i32, _vp, _vp]),
    "lc_rope_table_host": (None, [_i32, _i32, _f32, _f32, _vp, _vp]),
    "lc_rope_cache_new": (_i32, [_i32, _i32, _f32, _f32, _vp, C.POINTER(_vp)]),
    "lc_rope_cache_cos": (_vp, [_vp]),
    "lc_rope_cache_sin": (_vp, [_vp]),
    "lc_rope_cache_free": (None, [_vp]),
    "lc_kv_cache_new": (_i32, [_i32, _i32, _i32, _i32, _i32, _f32, _vp, C.POINTER(_vp)]),
    "lc_kv_cache_prepare_for_step": (_i32, [_vp, _vp, _i32]),
    "lc_kv_cache_update": (_i32, [_vp, _vp, _i32, _i32, _vp, _vp, _vp, _vp]),
    "lc_kv_cache_k_pool": (_vp, [_vp]),
    "lc_kv_cache_v_pool": (_vp, [_vp]),
    "lc_kv_cache_block_table": (_vp, [_vp]),
    "lc_kv_cache_num_physical_blocks": (_i64, [_vp]),
    "lc_kv_cache_max_seq_len": (_i32, [_vp]),
    "lc_kv_cache_num_allocated_blocks": (_i32, [_vp]),
    "lc_kv_cache_free": (None, [_vp]),
    "lc_apply_flash_decoding": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _vp, _i32]),
    "lc_proj_gemm": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _vp, _i64, _vp]),
    "lc_qkv_proj_rope_append": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _vp,
                                       _vp, _vp, _vp, _vp, _vp, _i32, _vp, _vp, _i64, _i32, _i32,
                                       _i32, _i32, _i32, _vp, _i32, _vp, _vp]),
    "lc_argmax": (_i32, [_vp, _i64, _i32, _i32, _vp, _vp]),
    "lc_sample_workspace_size": (_sz, [_i32, _i32]),
    "lc_sample_top_p": (_i32, [_vp, _i64, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _sz, _vp]),
    "lc_block_alloc_new": (_i32, [_i64, _i32, _i32, C.POINTER(_vp)]),
    "lc_block_alloc_add_seq": (_i32, [_vp, _pi32]),
    "lc_block_alloc_release_seq": (_i32, [_vp, _i32]),
    "lc_block_alloc_reserve": (_i32, [_vp, _i32, _i32]),
    "lc_block_alloc_row": (_i32, [_vp, _i32, _pi32, _i32]),
    "lc_block_alloc_num_free": (_i64, [_vp]),
    "lc_block_alloc_fingerprint": (C.c_uint64, [_vp]),
    "lc_block_alloc_free": (None, [_vp]),
    "lc_kv_pool_blocks_for_budget": (_i64, [_i32, _i32, _i32, C.c_uint64, C.c_uint64, _f32]),
    "lc_kv_pool_capacity": (_i32, [_i32, _i32, _i32, _f32, C.POINTER(_i64)]),
    "lc_kv_pool_new": (_i32, [_i32, _i32, _i32, _i32, _i32, _i32, _i64, _vp, C.POINTER(_vp)]),
    "lc_kv_pool_add_sequence": (_i32, [_vp, _pi32]),
    "lc_kv_pool_release_sequence": (_i32, [_vp, _i32]),
    "lc_kv_pool_prepare_step": (_i32, [_vp, _vp, _i32, _pi32, _pi32]),
    "lc_kv_pool_decode_layer": (_i32, [_vp, _vp, _i32, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp,
                                       _vp, _i32, _vp]),
    "lc_kv_pool_prepare_prefill": (_i32, [_vp, _vp, _i32, _i32, _i32]),
    "lc_kv_pool_prefill_layer": (_i32, [_vp, _vp, _i32, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp,
                                        _vp, _i32, _vp]),
    "lc_kv_pool_k_pool": (_vp, [_vp]),
    "lc_kv_pool_v_pool": (_vp, [_vp]),
    "lc_kv_pool_step_tables": (_vp, [_vp]),
    "lc_kv_pool_step_positions": (_vp, [_vp]),
    "lc_kv_pool_table_stride": (_i32, [_vp]),
    "lc_kv_pool_num_blocks": (_i64, [_vp]),
    "lc_kv_pool_num_free_blocks": (_i64, [_vp]),
    "lc_kv_pool_sequence_pages": (_i32, [_vp, _i32, _pi32, _i32]),
    "lc_kv_pool_fingerprint": (C.c_uint64, [_vp]),
    "lc_kv_pool_recover": (_i32, [_vp, _vp]),
    "lc_kv_pool_free": (None, [_vp]),
    "lc_shard_sequences": (_i32, [_pi32, _i32, _i32, _pi32]),
    "lc_shard_kv_heads": (_i32, [_i32, _i32, _i32, _i32, _pi32, _pi32]),
    "lc_peer_region_alloc": (_i32, [_sz, C.POINTER(_vp), _vp]),
    "lc_peer_region_free": (_i32, [_vp]),
    "lc_peer_group_open": (_i32, [_i32, _i32, _vp, _sz, _vp, C.POINTER(_vp)]),
    "lc_peer_group_local": (_i32, [_i32, _i32, C.POINTER(_vp), _sz, C.POINTER(_vp)]),
    "lc_peer_group_destroy": (None, [_vp]),
    "lc_rope_append_decode_peer": (_i32, [_vp, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp,
                                          _i32, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _i32,
                                          _vp, _i32, _i32, _i32, _i32, _f32, _vp, _sz, _vp, _vp,
                                          _vp]),
    "lc_peer_wait": (_i32, [_vp, _vp, _vp]),
}

for _name, (_res, _args) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args

LC_OK = 0
LC_DEV_BAD_BLOCK, LC_DEV_BAD_POS, LC_DEV_TIMEOUT = 1, 2, 4


class LucciolaError(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        super().__init__(f"{where}: {lib.lc_status_string(status).decode()} (status {status})")


def check(status: int, where: str) -> None:
    if status != LC_OK:
        raise LucciolaError(status, where)


def set_dependent_launch(mode: int) -> int:
    """Programmatic dependent launch mode for decode launches (0, 1 or 2); returns the old one."""
    old = lib.lc_set_dependent_launch(mode)
    if old < 0:
        raise ValueError(f"invalid dependent-launch mode {mode}")
    return old


def version() -> str:
    return lib.lc_version().decode()


def _p(t):
    """Device pointer of a tensor (or None)."""
    return None if t is None else t.data_ptr()


def _stream(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


# ----------------------------------------------------------- reference shape --

def rope(q, q_bias, k, k_bias, cos, sin, pos_ptr, head_dim, num_q_heads, num_k_heads,
         stream=None):
    check(lib.lc_rope(_p(q), _p(q_bias), _p(k), _p(k_bias), _p(cos), _p(sin), _p(pos_ptr),
                      head_dim, num_q_heads, num_k_heads, _stream(stream)), "lc_rope")


def update_kv_cache(k_pool, v_pool, new_k, new_v, v_bias, block_table, layer_id, pos_ptr,
                    num_layers, num_kv_heads, max_seq_len, head_dim, block_size=16, stream=None):
    check(lib.lc_update_kv_cache(_p(k_pool), _p(v_pool), _p(new_k), _p(new_v), _p(v_bias),
                                 _p(block_table), layer_id, _p(pos_ptr), num_layers,
                                 num_kv_heads, max_seq_len, head_dim, block_size,
                                 _stream(stream)), "lc_update_kv_cache")


def flash_decoding_workspace_size(num_q_heads, head_dim, max_seq_len) -> int:
    return lib.lc_flash_decoding_workspace_size(num_q_heads, head_dim, max_seq_len)


def flash_decoding(out, q, k_pool, v_pool, block_table, layer_idx, num_q_heads, num_kv_heads,
                   head_dim, max_seq_len, pos_ptr, sm_scale, block_size, num_layers, host_pos,
                   num_physical_blocks, workspace, stream=None):
    check(lib.lc_flash_decoding(_p(out), _p(q), _p(k_pool), _p(v_pool), _p(block_table),
                                layer_idx, num_q_heads, num_kv_heads, head_dim, max_seq_len,
                                _p(pos_ptr), sm_scale, block_size, num_layers, host_pos,
                                num_physical_blocks, _p(workspace),
                                0 if workspace is None else workspace.numel() * workspace.element_size(),
                                _stream(stream)), "lc_flash_decoding")


# ------------------------------------------------------------------ batched --

def rope_append(qkv, positions, q_bias, k_bias, v_bias, cos, sin, k_pool, v_pool, num_blocks,
                num_layers, layer, num_q_heads, num_kv_heads, head_dim, block_tables,
                tokens_per_seq=1, dev_status=None, stream=None):
    rows = qkv.shape[0]
    assert rows % tokens_per_seq == 0
    check(lib.lc_rope_append(_p(qkv), qkv.stride(0), rows // tokens_per_seq, tokens_per_seq,
                             _p(positions), _p(q_bias), _p(k_bias), _p(v_bias), _p(cos), _p(sin),
                             cos.shape[0], _p(k_pool), _p(v_pool), num_blocks, num_layers, layer,
                             num_q_heads, num_kv_heads, head_dim, _p(block_tables),
                             block_tables.stride(0), _p(dev_status), _stream(stream)),
          "lc_rope_append")


def paged_decode_workspace_size(batch, num_q_heads, num_kv_heads, head_dim) -> int:
    return lib.lc_paged_decode_workspace_size(batch, num_q_heads, num_kv_heads, head_dim)


def alloc_decode_workspace(batch, num_q_heads, num_kv_heads, head_dim, device="cuda",
                           stream=None):
    """Allocates (torch) and zero-initialises a workspace for lc_paged_decode."""
    import torch
    nbytes = paged_decode_workspace_size(batch, num_q_heads, num_kv_heads, head_dim)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
    check(lib.lc_paged_decode_workspace_init(_p(ws), nbytes, _stream(stream)),
          "lc_paged_decode_workspace_init")
    return ws


def paged_decode(out, q, k_pool, v_pool, num_blocks, num_layers, layer, num_q_heads,
                 num_kv_heads, head_dim, block_tables, context_lens, max_context_len=0,
                 sm_scale=None, len_offset=0, partition_tokens=0, workspace=None,
                 dev_status=None, stream=None):
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(head_dim)
    batch = context_lens.shape[0]
    check(lib.lc_paged_decode(_p(out), out.stride(0), _p(q), q.stride(0), _p(k_pool), _p(v_pool),
                              num_blocks, num_layers, layer, num_q_heads, num_kv_heads, head_dim,
                              _p(block_tables), block_tables.stride(0), _p(context_lens),
                              len_offset, batch, max_context_len, partition_tokens, sm_scale,
                              _p(workspace),
                              0 if workspace is None else workspace.numel() * workspace.element_size(),
                              _p(dev_status), _stream(stream)), "lc_paged_decode")


def rope_append_decode(out, qkv, positions, q_bias, k_bias, v_bias, cos, sin, k_pool, v_pool,
                       num_blocks, num_layers, layer, num_q_heads, num_kv_heads, head_dim,
                       block_tables, max_context_len=0, sm_scale=None, partition_tokens=0,
                       workspace=None, dev_status=None, stream=None, gate=None,
                       peer_group=None):
    """One launch: bias + RoPE + append of each sequence's new token, then decode.
    With `gate` (int32 device tensor) the qkv rows are read once it is non-zero.
    With `peer_group` (PeerGroup) the output rows also land in every peer's
    region (out must be a view of this rank's region); pair it with
    peer_group.wait()."""
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(head_dim)
    batch = positions.shape[0]
    args = [_p(out), out.stride(0), _p(qkv), qkv.stride(0), _p(positions), _p(q_bias), _p(k_bias),
            _p(v_bias), _p(cos), _p(sin), cos.shape[0], _p(k_pool), _p(v_pool), num_blocks,
            num_layers, layer, num_q_heads, num_kv_heads, head_dim, _p(block_tables),
            block_tables.stride(0), batch, max_context_len, partition_tokens, sm_scale,
            _p(workspace),
            0 if workspace is None else workspace.numel() * workspace.element_size(),
            _p(dev_status)]
    if peer_group is not None:
        if gate is not None:
            raise ValueError("a peer decode takes no gate")
        check(lib.lc_rope_append_decode_peer(*args, peer_group.handle, _stream(stream)),
              "lc_rope_append_decode_peer")
    elif gate is None:
        check(lib.lc_rope_append_decode(*args, _stream(stream)), "lc_rope_append_decode")
    else:
        check(lib.lc_rope_append_decode_gated(*args, _p(gate), _stream(stream)),
              "lc_rope_append_decode_gated")


def paged_decode_static(out, q, k_pool, v_pool, num_blocks, num_layers, layer, num_q_heads,
                        num_kv_heads, head_dim, block_tables, context_lens, max_context_len=0,
                        sm_scale=None, len_offset=0, partition_tokens=0, dev_status=None,
                        stream=None):
    """lc_paged_decode without a workspace: the library's fixed device scratch."""
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(head_dim)
    batch = context_lens.shape[0]
    check(lib.lc_paged_decode_static(_p(out), out.stride(0), _p(q), q.stride(0), _p(k_pool),
                                     _p(v_pool), num_blocks, num_layers, layer, num_q_heads,
                                     num_kv_heads, head_dim, _p(block_tables),
                                     block_tables.stride(0), _p(context_lens), len_offset, batch,
                                     max_context_len, partition_tokens, sm_scale, _p(dev_status),
                                     _stream(stream)), "lc_paged_decode_static")


def paged_prefill(out, q, k_pool, v_pool, num_blocks, num_layers, layer, num_q_heads,
                  num_kv_heads, head_dim, block_tables, start_pos, tokens_per_seq, max_start_pos,
                  sm_scale=None, dev_status=None, stream=None):
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(head_dim)
    num_seqs = start_pos.shape[0]
    check(lib.lc_paged_prefill(_p(out), out.stride(0), _p(q), q.stride(0), _p(k_pool),
                               _p(v_pool), num_blocks, num_layers, layer, num_q_heads,
                               num_kv_heads, head_dim, _p(block_tables), block_tables.stride(0),
                               _p(start_pos), num_seqs, tokens_per_seq, max_start_pos, sm_scale,
                               _p(dev_status), _stream(stream)), "lc_paged_prefill")


def gather_kv(k_out, v_out, k_pool, v_pool, num_blocks, num_layers, layer, num_kv_heads,
              head_dim, block_tables, context_lens, max_context_len, len_offset=0,
              dev_status=None, stream=None):
    check(lib.lc_gather_kv(_p(k_out), _p(v_out), _p(k_pool), _p(v_pool), num_blocks, num_layers,
                           layer, num_kv_heads, head_dim, _p(block_tables),
                           block_tables.stride(0), _p(context_lens), len_offset,
                           context_lens.shape[0], max_context_len, _p(dev_status),
                           _stream(stream)), "lc_gather_kv")


# ------------------------------------------------------------ host mirrors --

def rope_table_host(max_pos, head_dim, base, scale_factor=0.0):
    """RopeCache's f32 cos/sin tables computed on the host (numpy arrays)."""
    import numpy as np
    half = head_dim // 2
    cos = np.empty((max_pos, half), dtype=np.float32)
    sin = np.empty((max_pos, half), dtype=np.float32)
    lib.lc_rope_table_host(max_pos, head_dim, base, scale_factor,
                           cos.ctypes.data_as(C.c_void_p), sin.ctypes.data_as(C.c_void_p))
    return cos, sin


def shard_sequences(context_lens, num_ranks):
    """Rank of each sequence under longest-first bin packing (list of ints)."""
    n = len(context_lens)
    lens = (C.c_int * n)(*[int(x) for x in context_lens])
    out = (C.c_int * n)()
    check(lib.lc_shard_sequences(lens, n, num_ranks, out), "lc_shard_sequences")
    return list(out)


def shard_kv_heads(num_q_heads, num_kv_heads, num_ranks, rank):
    first, count = C.c_int(), C.c_int()
    check(lib.lc_shard_kv_heads(num_q_heads, num_kv_heads, num_ranks, rank, C.byref(first),
                                C.byref(count)), "lc_shard_kv_heads")
    return first.value, count.value


PEER_MAX_RANKS = 8
PEER_SIGNAL_BYTES = 256
PEER_HANDLE_BYTES = 64


class _DeviceSpan:
    """__cuda_array_interface__ over library-owned device memory (keeps its
    owner alive while a torch view exists)."""

    def __init__(self, owner, ptr, shape, typestr):
        self.owner = owner
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


class PeerRegion:
    """One rank's exchange region (lc_peer_region_alloc): LC_PEER_SIGNAL_BYTES
    of signal words, then output buffers at offsets shared by every rank."""

    def __init__(self, nbytes):
        ptr = C.c_void_p()
        h = (C.c_uint8 * PEER_HANDLE_BYTES)()
        check(lib.lc_peer_region_alloc(nbytes, C.byref(ptr), h), "lc_peer_region_alloc")
        self.ptr = ptr.value
        self.nbytes = nbytes
        self.handle = bytes(h)

    def view(self, offset, shape, dtype):
        """A torch tensor over [offset, offset + size) of the region (bf16,
        int32 or uint8)."""
        import torch
        codes = {torch.bfloat16: ("<i2", 2), torch.int32: ("<i4", 4), torch.uint8: ("|u1", 1)}
        typestr, size = codes[dtype]
        n = math.prod(shape) * size
        if offset < 0 or offset % size or offset + n > self.nbytes:
            raise ValueError("view outside the region")
        t = torch.as_tensor(_DeviceSpan(self, self.ptr + offset, shape, typestr), device="cuda")
        return t.view(torch.bfloat16) if dtype == torch.bfloat16 else t

    def signal_words(self):
        import torch
        return self.view(0, (PEER_SIGNAL_BYTES // 4,), torch.int32)

    def close(self):
        if self.ptr:
            check(lib.lc_peer_region_free(self.ptr), "lc_peer_region_free")
            self.ptr = None


class PeerGroup:
    """lc_peer_group: the group's regions as this process addresses them."""

    def __init__(self, handle, rank, world):
        self.handle, self.rank, self.world = handle, rank, world

    @classmethod
    def open(cls, rank, world, region, handles):
        """`handles`: the ranks' PeerRegion.handle values, in rank order."""
        buf = b"".join(handles)
        if len(handles) != world or len(buf) != world * PEER_HANDLE_BYTES:
            raise ValueError("one handle per rank")
        g = C.c_void_p()
        check(lib.lc_peer_group_open(rank, world, region.ptr, region.nbytes, buf, C.byref(g)),
              "lc_peer_group_open")
        return cls(g, rank, world)

    @classmethod
    def local(cls, rank, world, regions):
        """Regions that this process already addresses (one process, several ranks)."""
        arr = (C.c_void_p * world)(*[r.ptr for r in regions])
        g = C.c_void_p()
        check(lib.lc_peer_group_local(rank, world, arr, regions[0].nbytes, C.byref(g)),
              "lc_peer_group_local")
        return cls(g, rank, world)

    def wait(self, dev_status=None, stream=None):
        check(lib.lc_peer_wait(self.handle, _p(dev_status), _stream(stream)), "lc_peer_wait")

    def close(self):
        if self.handle:
            lib.lc_peer_group_destroy(self.handle)
            self.handle = None


def assemble_head_shards(gathered, num_ranks):
    """[R*B, Hq/R*hd] rows from an all-gather of per-rank head slices (rank-major)
    -> [B, Hq*hd]: rank r's slice holds q heads [r*Hq/R, (r+1)*Hq/R)."""
    rows, width = gathered.shape
    batch = rows // num_ranks
    return gathered.reshape(num_ranks, batch, width).transpose(0, 1).reshape(batch, num_ranks * width)


class KVCache:
    """Owning mirror of the reference's KVCache (src/layers/kv_cache.rs)."""

    def __init__(self, num_hidden_layers, num_attention_heads, num_key_value_heads, head_dim,
                 max_position_embeddings, memory_fraction, stream=None):
        h = C.c_void_p()
        check(lib.lc_kv_cache_new(num_hidden_layers, num_attention_heads, num_key_value_heads,
                                  head_dim, max_position_embeddings, memory_fraction,
                                  _stream(stream), C.byref(h)), "lc_kv_cache_new")
        self._h = h
        self.num_layers, self.num_q_heads = num_hidden_layers, num_attention_heads
        self.num_kv_heads, self.head_dim = num_key_value_heads, head_dim

    def prepare_for_step(self, pos, stream=None):
        check(lib.lc_kv_cache_prepare_for_step(self._h, _stream(stream), pos),
              "lc_kv_cache_prepare_for_step")

    def update(self, layer_idx, pos, pos_ptr, k, v, v_bias, stream=None):
        check(lib.lc_kv_cache_update(self._h, _stream(stream), layer_idx, pos, _p(pos_ptr),
                                     _p(k), _p(v), _p(v_bias)), "lc_kv_cache_update")

    def apply_flash_decoding(self, out, q, layer_idx, pos, pos_ptr, stream=None):
        check(lib.lc_apply_flash_decoding(self._h, _stream(stream), _p(out), _p(q), layer_idx,
                                          pos, _p(pos_ptr), self.num_q_heads),
              "lc_apply_flash_decoding")

    @property
    def k_pool(self):
        return lib.lc_kv_cache_k_pool(self._h)

    @property
    def v_pool(self):
        return lib.lc_kv_cache_v_pool(self._h)

    @property
    def block_table(self):
        return lib.lc_kv_cache_block_table(self._h)

    @property
    def num_physical_blocks(self):
        return lib.lc_kv_cache_num_physical_blocks(self._h)

    @property
    def max_seq_len(self):
        return lib.lc_kv_cache_max_seq_len(self._h)

    @property
    def num_allocated_blocks(self):
        return lib.lc_kv_cache_num_allocated_blocks(self._h)

    def close(self):
        if self._h:
            lib.lc_kv_cache_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# --------------------------------------------------- batched token-step driver --

def _ints(vals):
    vals = [int(v) for v in vals]
    return (C.c_int * max(1, len(vals)))(*vals)


class BlockAlloc:
    """Page bookkeeping of a multi-sequence pool (host only): sequence slots,
    their page lists, one LIFO free list."""

    def __init__(self, num_blocks, max_seqs, max_blocks_per_seq):
        h = C.c_void_p()
        check(lib.lc_block_alloc_new(num_blocks, max_seqs, max_blocks_per_seq, C.byref(h)),
              "lc_block_alloc_new")
        self._h = h
        self.max_blocks_per_seq = max_blocks_per_seq

    def add(self):
        slot = C.c_int()
        check(lib.lc_block_alloc_add_seq(self._h, C.byref(slot)), "lc_block_alloc_add_seq")
        return slot.value

    def release(self, slot):
        check(lib.lc_block_alloc_release_seq(self._h, slot), "lc_block_alloc_release_seq")

    def reserve(self, slot, tokens):
        check(lib.lc_block_alloc_reserve(self._h, slot, tokens), "lc_block_alloc_reserve")

    def pages(self, slot):
        buf = (C.c_int * self.max_blocks_per_seq)()
        n = lib.lc_block_alloc_row(self._h, slot, buf, self.max_blocks_per_seq)
        if n < 0:
            raise LucciolaError(1, "lc_block_alloc_row")
        return list(buf[:n])

    @property
    def num_free(self):
        return lib.lc_block_alloc_num_free(self._h)

    def fingerprint(self):
        return lib.lc_block_alloc_fingerprint(self._h)

    def close(self):
        if self._h:
            lib.lc_block_alloc_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def proj_decode_plan(n, k):
    """(split, ctas, clusters_that_fit, ctas_per_sm) of the decode-step
    projection kernel."""
    a, b, c, d = C.c_int(), C.c_int(), C.c_int(), C.c_int()
    check(lib.lc_proj_decode_plan(n, k, C.byref(a), C.byref(b), C.byref(c), C.byref(d)),
          "lc_proj_decode_plan")
    return a.value, b.value, c.value, d.value


def proj_gemm(out, x, w, residual=None, stream=None):
    """out = x . w^T (+ residual): bf16 [M, K] x [N, K] -> [M, N], fp32 accumulation."""
    M, K = x.shape
    N = w.shape[0]
    check(lib.lc_proj_gemm(_p(out), out.stride(0), _p(x), x.stride(0), _p(w), w.stride(0), M, N,
                           K, _p(residual), residual.stride(0) if residual is not None else 0,
                           _stream(stream)), "lc_proj_gemm")


def qkv_proj_rope_append(qkv, x, w_qkv, positions, q_bias, k_bias, v_bias, cos, sin, k_pool,
                         v_pool, num_blocks, num_layers, layer, num_q_heads, num_kv_heads,
                         head_dim, block_tables, tokens_per_seq=1, dev_status=None, stream=None):
    """qkv = x . w_qkv^T with lc_rope_append fused into the epilogue."""
    rows, hidden = x.shape
    assert rows % tokens_per_seq == 0
    check(lib.lc_qkv_proj_rope_append(
        _p(qkv), qkv.stride(0), _p(x), x.stride(0), _p(w_qkv), w_qkv.stride(0), hidden,
        rows // tokens_per_seq, tokens_per_seq, _p(positions), _p(q_bias), _p(k_bias),
        _p(v_bias), _p(cos), _p(sin), cos.shape[0], _p(k_pool), _p(v_pool), num_blocks,
        num_layers, layer, num_q_heads, num_kv_heads, head_dim, _p(block_tables),
        block_tables.stride(0), _p(dev_status), _stream(stream)), "lc_qkv_proj_rope_append")


def argmax(out_idx, logits, stream=None):
    """out_idx[b] = index of the largest logit of row b (int32 tensor, bits of uint32)."""
    batch, vocab = logits.shape
    check(lib.lc_argmax(_p(logits), logits.stride(0), vocab, batch, _p(out_idx), _stream(stream)),
          "lc_argmax")


def alloc_sample_workspace(batch, top_k, device="cuda"):
    import torch
    n = lib.lc_sample_workspace_size(batch, top_k)
    if n == 0:
        raise LucciolaError(3, "lc_sample_workspace_size")
    return torch.zeros(n, dtype=torch.uint8, device=device)


def sample_top_p(out_idx, logits, top_k, top_p, rand_vals, workspace, stream=None):
    """Top-k / top-p draw per row; top_p and rand_vals are float32 device tensors [batch]."""
    batch, vocab = logits.shape
    check(lib.lc_sample_top_p(_p(logits), logits.stride(0), vocab, batch, top_k, _p(top_p),
                              _p(rand_vals), _p(out_idx), _p(workspace), workspace.numel(),
                              _stream(stream)), "lc_sample_top_p")


def pool_blocks_for_budget(num_layers, num_kv_heads, head_dim, free_bytes, total_bytes,
                           memory_fraction):
    """Pages a pool gets from a memory budget (src/layers/kv_cache.rs:37-59 rule)."""
    return lib.lc_kv_pool_blocks_for_budget(num_layers, num_kv_heads, head_dim, free_bytes,
                                            total_bytes, memory_fraction)


def pool_capacity(num_layers, num_kv_heads, head_dim, memory_fraction):
    """pool_blocks_for_budget with the current device's free/total memory."""
    n = C.c_int64()
    check(lib.lc_kv_pool_capacity(num_layers, num_kv_heads, head_dim, memory_fraction,
                                  C.byref(n)), "lc_kv_pool_capacity")
    return n.value


class KVPool:
    """Batched token-step driver: one paged K/V pool shared by many sequences
    (lc_kv_pool). prepare_step() then decode_layer() per layer runs one decode
    token of a batch; prepare_prefill() then prefill_layer() per layer runs a
    prompt of one sequence."""

    def __init__(self, num_layers, num_q_heads, num_kv_heads, head_dim, max_seqs, max_seq_len,
                 num_blocks, stream=None):
        h = C.c_void_p()
        check(lib.lc_kv_pool_new(num_layers, num_q_heads, num_kv_heads, head_dim, max_seqs,
                                 max_seq_len, num_blocks, _stream(stream), C.byref(h)),
              "lc_kv_pool_new")
        self._h = h
        self.num_layers, self.num_q_heads, self.num_kv_heads = num_layers, num_q_heads, num_kv_heads
        self.head_dim, self.max_seqs, self.num_blocks = head_dim, max_seqs, num_blocks
        self.table_stride = lib.lc_kv_pool_table_stride(h)

    def add_sequence(self):
        slot = C.c_int()
        check(lib.lc_kv_pool_add_sequence(self._h, C.byref(slot)), "lc_kv_pool_add_sequence")
        return slot.value

    def release_sequence(self, slot):
        check(lib.lc_kv_pool_release_sequence(self._h, slot), "lc_kv_pool_release_sequence")

    def prepare_step(self, slots, positions, stream=None):
        check(lib.lc_kv_pool_prepare_step(self._h, _stream(stream), len(slots), _ints(slots),
                                          _ints(positions)), "lc_kv_pool_prepare_step")

    def decode_layer(self, layer, out, qkv, q_bias, k_bias, v_bias, cos, sin, dev_status=None,
                     stream=None):
        check(lib.lc_kv_pool_decode_layer(self._h, _stream(stream), layer, _p(out), out.stride(0),
                                          _p(qkv), qkv.stride(0), _p(q_bias), _p(k_bias),
                                          _p(v_bias), _p(cos), _p(sin), cos.shape[0],
                                          _p(dev_status)), "lc_kv_pool_decode_layer")

    def prepare_prefill(self, slot, start_pos, tokens, stream=None):
        check(lib.lc_kv_pool_prepare_prefill(self._h, _stream(stream), slot, start_pos, tokens),
              "lc_kv_pool_prepare_prefill")

    def prefill_layer(self, layer, out, qkv, q_bias, k_bias, v_bias, cos, sin, dev_status=None,
                      stream=None):
        check(lib.lc_kv_pool_prefill_layer(self._h, _stream(stream), layer, _p(out), out.stride(0),
                                           _p(qkv), qkv.stride(0), _p(q_bias), _p(k_bias),
                                           _p(v_bias), _p(cos), _p(sin), cos.shape[0],
                                           _p(dev_status)), "lc_kv_pool_prefill_layer")

    def pages(self, slot):
        buf = (C.c_int * self.table_stride)()
        n = lib.lc_kv_pool_sequence_pages(self._h, slot, buf, self.table_stride)
        if n < 0:
            raise LucciolaError(1, "lc_kv_pool_sequence_pages")
        return list(buf[:n])

    def pools(self):
        """(k_pool, v_pool) as torch bf16 views [num_blocks][L][Hkv][16][hd] (no copy)."""
        import torch
        shape = (self.num_blocks, self.num_layers, self.num_kv_heads, 16, self.head_dim)
        n = 1
        for d in shape:
            n *= d
        out = []
        for ptr in (lib.lc_kv_pool_k_pool(self._h), lib.lc_kv_pool_v_pool(self._h)):
            cls = type("_Cai", (), {"__cuda_array_interface__": {
                "shape": (n,), "typestr": "<i2", "data": (ptr, False), "version": 3}})
            out.append(torch.as_tensor(cls(), device="cuda").view(torch.bfloat16).view(shape))
        return tuple(out)

    @property
    def num_free_blocks(self):
        return lib.lc_kv_pool_num_free_blocks(self._h)

    def fingerprint(self):
        return lib.lc_kv_pool_fingerprint(self._h)

    def recover(self, stream=None):
        """Zero the split-K workspace after a step that reported LC_DEV_TIMEOUT."""
        check(lib.lc_kv_pool_recover(self._h, _stream(stream)), "lc_kv_pool_recover")

    def close(self):
        if self._h:
            lib.lc_kv_pool_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
