"""ctypes/numpy front end of the CPU oracle (liblc_oracle.so) and of the
reference's own CUDA kernels (oracle/_ref/libref_kernels.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline / reference legs of bench.py as the checker; the product library
never uses it. bf16 arrays are numpy uint16 bit patterns.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "_build" / "liblc_oracle.so"
REF_LIB = HERE / "_ref" / "libref_kernels.so"
# Checkout of the reference (lucciola-rs): $REF_ROOT, else a directory named
# `reference` beside this repository. Only the build of oracle/_ref reads it.
REF_ROOT = Path(os.environ.get("REF_ROOT", HERE.parent.parent / "reference"))

_vp, _i32, _i64, _f32 = C.c_void_p, C.c_int, C.c_int64, C.c_float

_lib = None
_ref = None


def build(ref: bool = False) -> None:
    """Builds the oracle (and, when asked and the reference sources exist, the
    reference kernels) with oracle/Makefile."""
    targets = ["oracle"]
    if ref and (REF_ROOT / "src" / "kernels").is_dir():
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", str(HERE), f"REF_ROOT={REF_ROOT}", *targets], check=True)


def lib():
    global _lib
    if _lib is None:
        if not ORACLE_LIB.exists():
            build()
        L = C.CDLL(str(ORACLE_LIB))
        L.lco_f32_to_bf16.restype = C.c_uint16
        L.lco_f32_to_bf16.argtypes = [_f32]
        L.lco_bf16_to_f32.restype = _f32
        L.lco_bf16_to_f32.argtypes = [C.c_uint16]
        L.lco_rope_table.argtypes = [_i32, _i32, _f32, _f32, _vp, _vp]
        L.lco_rope.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32]
        L.lco_update_kv_cache.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32,
                                          _i32, _i32]
        L.lco_flash_decoding.argtypes = [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32,
                                         _f32, _i32, _i32, _i64]
        L.lco_flash_decoding.restype = _i32
        L.lco_paged_decode.argtypes = [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _i32, _i32, _i32,
                                       _i32, _i32, _vp, _i32, _vp, _i32, _i32, _f32, _i32]
        L.lco_paged_decode.restype = _i32
        L.lco_rope_append.argtypes = [_vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                      _vp, _i32, _i32, _i32, _i32, _i32, _vp, _i32, _i32, _i32]
        L.lco_rope_append.restype = _i32
        L.lco_paged_prefill.argtypes = [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _i32, _i32, _i32,
                                        _i32, _i32, _vp, _i32, _vp, _i32, _i32, _f32, _i32]
        L.lco_paged_prefill.restype = _i32
        L.lco_argmax.argtypes = [_vp, _i32]
        L.lco_argmax.restype = _i32
        L.lco_top_k_filter.argtypes = [_vp, _i32, _i32, _vp, _vp]
        L.lco_top_p_sample.argtypes = [_vp, _vp, _i32, _f32, _f32, C.POINTER(C.c_double)]
        L.lco_top_p_sample.restype = _i32
        L.lco_gather_kv.argtypes = [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _vp, _i32,
                                    _vp, _i32, _i32, _i32]
        L.lco_gather_kv.restype = _i32
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(C.c_void_p)


# ------------------------------------------------------------------ bf16 ----

def f32_to_bf16(x) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bits (vectorised, same rule as the C oracle)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FFF
    return r


def bf16_to_f32(h) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# -------------------------------------------------------------- functions ---

def rope_table(max_pos: int, head_dim: int, base: float, scale_factor: float = 0.0):
    half = head_dim // 2
    cos = np.empty((max_pos, half), np.float32)
    sin = np.empty((max_pos, half), np.float32)
    lib().lco_rope_table(max_pos, head_dim, base, scale_factor, _ptr(cos), _ptr(sin))
    return cos, sin


def rope(q, q_bias, k, k_bias, cos, sin, pos, head_dim, num_q_heads, num_k_heads,
         sub_mode=1, add_mode=1):
    """In place on q and k (uint16 arrays)."""
    lib().lco_rope(_ptr(q), _ptr(q_bias), _ptr(k), _ptr(k_bias), _ptr(cos), _ptr(sin), pos,
                   head_dim, num_q_heads, num_k_heads, sub_mode, add_mode)


def update_kv_cache(k_pool, v_pool, new_k, new_v, v_bias, block_table, layer, pos, num_layers,
                    num_kv_heads, head_dim):
    lib().lco_update_kv_cache(_ptr(k_pool), _ptr(v_pool), _ptr(new_k), _ptr(new_v),
                              _ptr(v_bias), _ptr(block_table), layer, pos, num_layers,
                              num_kv_heads, head_dim, 16)


def flash_decoding(q, k_pool, v_pool, block_table, layer, num_q_heads, num_kv_heads, head_dim,
                   pos, num_layers, sm_scale=None):
    if sm_scale is None:
        sm_scale = np.float32(1.0) / np.sqrt(np.float32(head_dim))
    out = np.zeros(num_q_heads * head_dim, np.uint16)
    rc = lib().lco_flash_decoding(_ptr(out), _ptr(q), _ptr(k_pool), _ptr(v_pool),
                                  _ptr(block_table), layer, num_q_heads, num_kv_heads, head_dim,
                                  pos, float(sm_scale), 16, num_layers, k_pool.shape[0])
    if rc:
        raise ValueError("block table entry outside the pool")
    return out


def paged_decode(q, k_pool, v_pool, layer, num_q_heads, num_kv_heads, head_dim, block_tables,
                 context_lens, num_layers, sm_scale=None, len_offset=0, threads=1):
    """q: [B, >= Hq*hd] uint16 rows; returns out [B, Hq*hd] uint16."""
    if sm_scale is None:
        sm_scale = 1.0 / np.sqrt(np.float32(head_dim))
    q = np.ascontiguousarray(q)
    tables = np.ascontiguousarray(block_tables, dtype=np.int32)
    lens = np.ascontiguousarray(context_lens, dtype=np.int32)
    B = lens.shape[0]
    out = np.zeros((B, num_q_heads * head_dim), np.uint16)
    rc = lib().lco_paged_decode(_ptr(out), out.shape[1], _ptr(q), q.shape[1], _ptr(k_pool),
                                _ptr(v_pool), k_pool.shape[0], num_layers, layer, num_q_heads,
                                num_kv_heads, head_dim, _ptr(tables), tables.shape[1], _ptr(lens),
                                len_offset, B, float(sm_scale), threads)
    if rc:
        raise ValueError("block table entry outside the pool")
    return out


def rope_append(qkv, positions, q_bias, k_bias, v_bias, cos, sin, k_pool, v_pool, num_layers,
                layer, num_q_heads, num_kv_heads, head_dim, block_tables, tokens_per_seq=1,
                sub_mode=1, add_mode=1):
    """In place on qkv [rows, row_stride] and the pools."""
    positions = np.ascontiguousarray(positions, dtype=np.int32)
    tables = np.ascontiguousarray(block_tables, dtype=np.int32)
    rows = qkv.shape[0]
    lib().lco_rope_append(_ptr(qkv), qkv.shape[1], rows // tokens_per_seq, tokens_per_seq,
                          _ptr(positions), _ptr(q_bias), _ptr(k_bias), _ptr(v_bias), _ptr(cos),
                          _ptr(sin), _ptr(k_pool), _ptr(v_pool), num_layers, layer, num_q_heads,
                          num_kv_heads, head_dim, _ptr(tables), tables.shape[1], sub_mode,
                          add_mode)


def paged_prefill(q, k_pool, v_pool, layer, num_q_heads, num_kv_heads, head_dim, block_tables,
                  start_pos, tokens_per_seq, num_layers, sm_scale=None, threads=1):
    """q: [num_seqs*T, >= Hq*hd] uint16 rows (already rotated); pool already holds the K/V."""
    if sm_scale is None:
        sm_scale = 1.0 / np.sqrt(np.float32(head_dim))
    q = np.ascontiguousarray(q)
    tables = np.ascontiguousarray(block_tables, dtype=np.int32)
    start = np.ascontiguousarray(start_pos, dtype=np.int32)
    rows = q.shape[0]
    out = np.zeros((rows, num_q_heads * head_dim), np.uint16)
    rc = lib().lco_paged_prefill(_ptr(out), out.shape[1], _ptr(q), q.shape[1], _ptr(k_pool),
                                 _ptr(v_pool), k_pool.shape[0], num_layers, layer, num_q_heads,
                                 num_kv_heads, head_dim, _ptr(tables), tables.shape[1],
                                 _ptr(start), start.shape[0], tokens_per_seq, float(sm_scale),
                                 threads)
    if rc:
        raise ValueError("block table entry outside the pool")
    return out


def gather_kv(k_pool, v_pool, layer, num_kv_heads, head_dim, block_tables, context_lens,
              max_context_len, num_layers, len_offset=0):
    tables = np.ascontiguousarray(block_tables, dtype=np.int32)
    lens = np.ascontiguousarray(context_lens, dtype=np.int32)
    B = lens.shape[0]
    k = np.zeros((B, max_context_len, num_kv_heads, head_dim), np.uint16)
    v = np.zeros_like(k)
    rc = lib().lco_gather_kv(_ptr(k), _ptr(v), _ptr(k_pool), _ptr(v_pool), k_pool.shape[0],
                             num_layers, layer, num_kv_heads, head_dim, _ptr(tables),
                             tables.shape[1], _ptr(lens), len_offset, B, max_context_len)
    if rc:
        raise ValueError("block table entry outside the pool")
    return k, v


# --------------------------------------------- reference kernels (GPU) ------

def ref_lib():
    """The reference's own kernels (oracle/_ref/libref_kernels.so), GPU only."""
    global _ref
    if _ref is None:
        if not REF_LIB.exists():
            raise FileNotFoundError(f"{REF_LIB} not built (make -C oracle ref)")
        R = C.CDLL(str(REF_LIB))
        R.ref_rope.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]
        R.ref_update_kv_cache.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _vp, _i32, _i32,
                                          _i32, _i32, _i32, _vp]
        R.ref_flash_decoding.argtypes = [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32,
                                         _vp, _i32, _i32, _i32, _vp]
        R.ref_paged_decode.argtypes = [_vp, _i64, _vp, _i64, _vp, _vp, _i32, _i32, _i32, _i32,
                                       _i32, _vp, _i32, _vp, _vp, _i32, _i32, _vp]
        R.ref_rope_append.argtypes = [_vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                      _vp, _i32, _i32, _i32, _i32, _i32, _vp, _i32, _i32, _vp]
        R.ref_rope_table.argtypes = [_i32, _i32, _f32, _f32, _vp, _vp]
        R.ref_rope_table.restype = None
        R.ref_argmax.argtypes = [_vp, _i32, _vp, _vp]
        R.ref_sample_top_p.argtypes = [_vp, _i32, _i32, _f32, _f32, _vp, _vp, _vp]
        R.ref_prefill.argtypes = [_vp, _i64, _vp, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp,
                                  _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp, _i32,
                                  _i32, _vp]
        for f in ("ref_rope", "ref_update_kv_cache", "ref_flash_decoding", "ref_paged_decode",
                  "ref_rope_append", "ref_prefill"):
            getattr(R, f).restype = _i32
        _ref = R
    return _ref


def ref_rope_table(max_pos: int, head_dim: int, base: float, scale_factor: float = 0.0):
    """RopeCache::new's tables (src/layers/rope.rs:20-31) computed by the
    reference-kernel library's host code: the reference arm of bench.py uses
    them so that it loads nothing but oracle/_ref."""
    half = head_dim // 2
    cos = np.empty((max_pos, half), np.float32)
    sin = np.empty((max_pos, half), np.float32)
    ref_lib().ref_rope_table(max_pos, head_dim, base, scale_factor, _ptr(cos), _ptr(sin))
    return cos, sin


# ----------------------------------------------------------------- sampling --

def argmax(logits):
    """argmax_kernel (src/kernels/sampling.cu): per row, with its tie order."""
    logits = np.ascontiguousarray(logits, dtype=np.uint16)
    rows = logits.reshape(-1, logits.shape[-1])
    return np.array([lib().lco_argmax(_ptr(np.ascontiguousarray(r)), r.shape[0]) for r in rows],
                    np.int64)


def top_k_filter(logits, top_k):
    """top_k_filter (src/kernels/sampling_optimized.cu): 32 partitions x top_k/32
    candidates of one row, partition-major: (keys int32, values float32)."""
    row = np.ascontiguousarray(logits, dtype=np.uint16)
    kpb = top_k // 32
    keys = np.zeros(32 * kpb, np.int32)
    vals = np.zeros(32 * kpb, np.float32)
    lib().lco_top_k_filter(_ptr(row), row.shape[0], kpb, _ptr(keys), _ptr(vals))
    return keys, vals


def top_p_sample(keys, values, top_p, rand_val):
    """fused_top_p_sample_impl: (chosen key or -1, margin to the nearest boundary)."""
    keys = np.ascontiguousarray(keys, dtype=np.int32)
    values = np.ascontiguousarray(values, dtype=np.float32)
    m = C.c_double()
    k = lib().lco_top_p_sample(_ptr(keys), _ptr(values), keys.shape[0], float(top_p),
                               float(rand_val), C.byref(m))
    return k, m.value
