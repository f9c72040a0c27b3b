"""Generates the golden fixtures that pin the CPU oracle to the reference.

Runs the reference's own CUDA kernels (src/kernels/{rope,kv_cache,attention,
sampling,sampling_optimized}.cu, compiled unchanged into oracle/_ref/libref_kernels.so)
on seeded inputs on a
GPU and stores inputs and outputs as small .npz files next to this script.
tests/test_golden.py then checks the CPU oracle against them on any machine.

    python tests/golden/make_golden.py [--out DIR] [--only NAME ...]   # needs a GPU and oracle/_ref
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


def sampling_fixture(R, vocab, rows, seed):
    """argmax_kernel, top_k_filter (top_k 64 and 256) and fused_top_p_sample on
    quantised logits (many ties), with a few (top_p, rand) draws per row."""
    rng = np.random.default_rng(seed)
    x = np.round(rng.standard_normal((rows, vocab)).astype(np.float32) * 6.0) / 2.0
    logits = O.f32_to_bf16(x)
    d = to_device(logits)
    draws = np.array([(0.3, 0.25), (0.9, 0.5), (0.9, 0.97), (1.0, 0.61)], np.float32)
    out = dict(vocab=vocab, logits=logits, draws=draws)
    am = []
    for r in range(rows):
        o = torch.zeros(1, dtype=torch.int32, device="cuda")
        assert R.ref_argmax(p(d[r]), vocab, p(o), s()) == 0
        torch.cuda.synchronize()
        am.append(int(from_device(o).view(np.uint32)[0]))
    out["argmax"] = np.array(am, np.int64)
    for top_k in (64, 256):
        keys, vals, picks = [], [], []
        for r in range(rows):
            row_picks = []
            for top_p, rand in draws:
                cand = torch.zeros(2 * top_k, dtype=torch.int32, device="cuda")
                o = torch.full((1,), -1, dtype=torch.int32, device="cuda")
                assert R.ref_sample_top_p(p(d[r]), vocab, top_k, float(top_p), float(rand),
                                          p(cand), p(o), s()) == 0
                torch.cuda.synchronize()
                row_picks.append(int(from_device(o)[0]))
            c = from_device(cand).reshape(top_k, 2)
            keys.append(c[:, 0].copy())
            vals.append(c[:, 1].view(np.float32).copy())
            picks.append(row_picks)
        out[f"keys_{top_k}"] = np.stack(keys)
        out[f"values_{top_k}"] = np.stack(vals)
        out[f"picks_{top_k}"] = np.array(picks, np.int64)
    return out


def main() -> int:
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=str(HERE), help="directory for the .npz files")
    ap.add_argument("--only", nargs="*", default=None, help="fixture names to (re)generate")
    args = ap.parse_args()
    out_dir = Path(args.out)
    out_dir.mkdir(parents=True, exist_ok=True)
    R = O.ref_lib()
    makers = {
        "rope_hd64": lambda: rope_fixture(R, 64, 14, 2, 1),
        "rope_hd128": lambda: rope_fixture(R, 128, 28, 4, 2),
        "update_kv_cache": lambda: update_fixture(R, 3),
        "attention_hd64": lambda: attention_fixture(R, 14, 2, 64, 150, 4),
        "attention_hd128": lambda: attention_fixture(R, 12, 2, 128, 77, 5),
        "attention_hd128_gqa8": lambda: attention_fixture(R, 16, 2, 128, 40, 6),
        "sampling": lambda: sampling_fixture(R, 8192 + 37, 4, 7),
    }
    names = args.only if args.only else list(makers)
    fx = {name: makers[name]() for name in names}
    for name, d in fx.items():
        path = out_dir / f"{name}.npz"
        np.savez_compressed(path, **{k: np.asarray(v) for k, v in d.items()})
        print(f"wrote {path} ({path.stat().st_size} bytes)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
