"""Generates the golden fixtures that pin the CPU oracle to the reference.

Runs the reference's own CUDA kernels (src/kernels/{rope,kv_cache,attention}.cu,
compiled unchanged into oracle/_ref/libref_kernels.so) on seeded inputs on a
GPU and stores inputs and outputs as small .npz files next to this script.
tests/test_golden.py then checks the CPU oracle against them on any machine.

    python tests/golden/make_golden.py [--out DIR]   # needs a GPU and oracle/_ref
"""
from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "tests")]

import torch  # noqa: E402

import oracle.oracle as O  # noqa: E402
from workloads import from_device, make_case, randn_bf16, to_device  # noqa: E402


def p(t):
    return C.c_void_p(t.data_ptr())


def s():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def rope_fixture(R, hd, hq, hkv, seed):
    rng = np.random.default_rng(seed)
    max_pos = 32768
    cos, sin = O.rope_table(max_pos, hd, 1e6)
    dcos, dsin = to_device(cos), to_device(sin)
    positions = np.array([0, 1, 2, 15, 16, 255, 1023, 4095, 8191, 16384, 32767], np.int32)
    n = len(positions)
    q = randn_bf16(rng, (n, hq * hd))
    k = randn_bf16(rng, (n, hkv * hd))
    qb, kb = randn_bf16(rng, (hq * hd,)), randn_bf16(rng, (hkv * hd,))
    dqb, dkb = to_device(qb), to_device(kb)
    q_out, k_out = q.copy(), k.copy()
    for i, pos in enumerate(positions):
        dq, dk = to_device(q[i]), to_device(k[i])
        dpos = to_device(np.array([pos], np.int32))
        assert R.ref_rope(p(dq), p(dqb), p(dk), p(dkb), p(dcos), p(dsin), p(dpos), hd, hq, hkv,
                          s()) == 0
        torch.cuda.synchronize()
        q_out[i], k_out[i] = from_device(dq), from_device(dk)
    # cos/sin rows are stored for the used positions only (the tables are
    # recomputed and compared on the CPU side).
    return dict(hd=hd, hq=hq, hkv=hkv, positions=positions, q=q, k=k, q_bias=qb, k_bias=kb,
                cos_rows=cos[positions], sin_rows=sin[positions], q_out=q_out, k_out=k_out)


def update_fixture(R, seed):
    rng = np.random.default_rng(seed)
    hq, hkv, hd = 14, 2, 64
    case = make_case(1, hq, hkv, hd, [70], seed=seed, table_stride=8)
    kp0, vp0 = case.k_pool.copy(), case.v_pool.copy()
    dk, dv, dt = to_device(case.k_pool), to_device(case.v_pool), to_device(case.tables)
    vb = randn_bf16(rng, (hkv * hd,))
    positions = np.array([0, 15, 16, 17, 69], np.int32)
    ks = randn_bf16(rng, (len(positions), hkv * hd))
    vs = randn_bf16(rng, (len(positions), hkv * hd))
    for i, pos in enumerate(positions):
        dpos = to_device(np.array([pos], np.int32))
        dki, dvi, dvb = to_device(ks[i]), to_device(vs[i]), to_device(vb)  # alive at launch
        assert R.ref_update_kv_cache(p(dk), p(dv), p(dki), p(dvi),
                                     p(dvb), p(dt), case.layer, p(dpos),
                                     case.num_layers, hkv, 32768, hd, 16, s()) == 0
    torch.cuda.synchronize()
    return dict(hkv=hkv, hd=hd, num_layers=case.num_layers, layer=case.layer, table=case.tables[0],
                k_pool=kp0, v_pool=vp0, v_bias=vb, positions=positions, k=ks, v=vs,
                k_pool_out=from_device(dk), v_pool_out=from_device(dv))


def attention_fixture(R, hq, hkv, hd, pos, seed):
    case = make_case(1, hq, hkv, hd, [pos + 1], seed=seed)
    dq, dk, dv, dt = (to_device(case.q), to_device(case.k_pool), to_device(case.v_pool),
                      to_device(case.tables))
    out = torch.empty(hq * hd, dtype=torch.bfloat16, device="cuda")
    dpos = to_device(np.array([pos], np.int32))
    assert R.ref_flash_decoding(p(out), p(dq), p(dk), p(dv), p(dt), case.layer, hq, hkv, hd,
                                32768, p(dpos), pos, 16, case.num_layers, s()) == 0
    torch.cuda.synchronize()
    return dict(hq=hq, hkv=hkv, hd=hd, pos=pos, num_layers=case.num_layers, layer=case.layer,
                table=case.tables[0], q=case.q[0], k_pool=case.k_pool, v_pool=case.v_pool,
                out=from_device(out))


def main() -> int:
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(HERE), help="directory for the .npz files")
    out_dir = Path(ap.parse_args().out)
    out_dir.mkdir(parents=True, exist_ok=True)
    R = O.ref_lib()
    fx = {
        "rope_hd64": rope_fixture(R, 64, 14, 2, 1),
        "rope_hd128": rope_fixture(R, 128, 28, 4, 2),
        "update_kv_cache": update_fixture(R, 3),
        "attention_hd64": attention_fixture(R, 14, 2, 64, 150, 4),
        "attention_hd128": attention_fixture(R, 12, 2, 128, 77, 5),
        "attention_hd128_gqa8": attention_fixture(R, 16, 2, 128, 40, 6),
    }
    for name, d in fx.items():
        path = out_dir / f"{name}.npz"
        np.savez_compressed(path, **{k: np.asarray(v) for k, v in d.items()})
        print(f"wrote {path} ({path.stat().st_size} bytes)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
