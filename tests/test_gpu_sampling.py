"""Token selection (lc_argmax, lc_sample_top_p) against the CPU oracle and the
reference's own kernels (argmax_kernel, top_k_filter + fused_top_p_sample_<n>,
compiled unchanged into oracle/_ref and launched as src/kernels.rs:322-490
launches them). The greedy index and the top-k candidate set are exact, ties
included; the sampled index equals both wherever the draw is not within fp32
rounding of a cumulative-probability boundary (the oracle reports the margin)."""
import ctypes as C

import numpy as np
import pytest

import lucciola as L
import oracle.oracle as O
from workloads import from_device, to_device

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

VOCAB = 151936  # Qwen2 vocabulary
MARGIN = 1e-5   # draws this close to a boundary may go either way in fp32


def _logits(rng, rows, vocab=VOCAB, quantum=None, scale=3.0):
    x = rng.standard_normal((rows, vocab)).astype(np.float32) * scale
    if quantum:  # few distinct values: many ties
        x = np.round(x / quantum) * quantum
    return O.f32_to_bf16(x)


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def test_argmax_matches_oracle_and_reference_with_ties():
    rng = np.random.default_rng(1)
    x = _logits(rng, 6)
    # equal maxima placed so that lower index and lower i % 1024 disagree
    big = O.f32_to_bf16(np.float32(40.0))
    x[1, [10, 1024 + 5, 5000]] = big         # thread 5 (index 1029) beats thread 10
    x[2, [2048 + 7, 7, 99999]] = big         # same thread 7: the lower index
    x[3, [VOCAB - 1, VOCAB - 2]] = big       # vocabulary tail
    x[4, :] = O.f32_to_bf16(np.float32(-2e30))  # nothing above -1e30
    d = to_device(x)
    out = torch.zeros(6, dtype=torch.int32, device="cuda")
    L.argmax(out, d)
    torch.cuda.synchronize()
    ours = from_device(out).view(np.uint32).astype(np.int64)
    orc = O.argmax(x) & 0xFFFFFFFF
    R = O.ref_lib()
    ref = []
    for r in range(6):
        o = torch.zeros(1, dtype=torch.int32, device="cuda")
        assert R.ref_argmax(_ptr(d[r]), VOCAB, _ptr(o), _stream()) == 0
        torch.cuda.synchronize()
        ref.append(int(from_device(o).view(np.uint32)[0]))
    assert list(ours) == list(orc) == ref
    assert ours[1] == 1024 + 5 and ours[2] == 7 and ours[4] == 0xFFFFFFFF
    # rows of odd length (unaligned rows: element by element), with ties
    y = _logits(rng, 3, vocab=300001, quantum=0.5)
    out3 = torch.zeros(3, dtype=torch.int32, device="cuda")
    L.argmax(out3, to_device(y))
    torch.cuda.synchronize()
    assert list(from_device(out3).view(np.uint32).astype(np.int64)) == list(O.argmax(y))


@pytest.mark.parametrize("top_k,quantum,vocab", [
    (64, None, VOCAB), (256, 0.25, VOCAB), (1024, None, VOCAB), (32, 0.5, VOCAB),
    (64, 0.5, 300001),  # odd row length: unaligned rows and partitions
])
def test_top_k_candidates_match_oracle_and_reference(top_k, quantum, vocab):
    rng = np.random.default_rng(top_k)
    rows = 3
    x = _logits(rng, rows, vocab=vocab, quantum=quantum)
    d = to_device(x)
    n = 32 * (top_k // 32)
    ws = L.alloc_sample_workspace(rows, top_k)
    out = torch.zeros(rows, dtype=torch.int32, device="cuda")
    tp = torch.full((rows,), 0.9, dtype=torch.float32, device="cuda")
    rv = torch.full((rows,), 0.5, dtype=torch.float32, device="cuda")
    L.sample_top_p(out, d, top_k, tp, rv, ws)
    torch.cuda.synchronize()
    raw = ws.cpu().numpy()
    keys = raw[:rows * n * 4].view(np.int32).reshape(rows, n)
    vals = raw[rows * n * 4:rows * n * 8].view(np.float32).reshape(rows, n)
    R = O.ref_lib()
    for r in range(rows):
        ok, ov = O.top_k_filter(x[r], top_k)
        assert np.array_equal(keys[r], ok) and np.array_equal(vals[r], ov)
        cand = torch.zeros(n * 2, dtype=torch.int32, device="cuda")  # {int key, float value}
        o = torch.zeros(1, dtype=torch.int32, device="cuda")
        assert R.ref_sample_top_p(_ptr(d[r]), vocab, top_k, 0.9, 0.5, _ptr(cand), _ptr(o),
                                  _stream()) == 0
        torch.cuda.synchronize()
        rc = from_device(cand).reshape(n, 2)
        assert np.array_equal(rc[:, 0], ok)
        assert np.array_equal(rc[:, 1].view(np.float32), ov)


@pytest.mark.parametrize("top_k", [32, 64, 256, 1024])
def test_sampled_index_matches_oracle_and_reference(top_k):
    rng = np.random.default_rng(100 + top_k)
    rows = 8
    x = _logits(rng, rows, scale=2.0)
    d = to_device(x)
    ws = L.alloc_sample_workspace(rows, top_k)
    R = O.ref_lib()
    cand = torch.zeros(2048, dtype=torch.int32, device="cuda")
    checked = 0
    for top_p in (0.3, 0.9, 1.0):
        rv = rng.random(rows).astype(np.float32)
        out = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
        L.sample_top_p(out, d, top_k, to_device(np.full(rows, top_p, np.float32)),
                       to_device(rv), ws)
        torch.cuda.synchronize()
        ours = from_device(out)
        for r in range(rows):
            ok, ov = O.top_k_filter(x[r], top_k)
            want, margin = O.top_p_sample(ok, ov, top_p, rv[r])
            o = torch.full((1,), -7, dtype=torch.int32, device="cuda")
            assert R.ref_sample_top_p(_ptr(d[r]), VOCAB, top_k, float(top_p), float(rv[r]),
                                      _ptr(cand), _ptr(o), _stream()) == 0
            torch.cuda.synchronize()
            ref = int(from_device(o)[0])
            if margin < MARGIN:
                continue
            assert int(ours[r]) == want == ref, (r, top_p, rv[r], int(ours[r]), want, ref)
            checked += 1
    assert checked >= rows * 3 - 2  # boundary draws are rare


def test_sampling_rejects_unsupported_candidate_counts():
    x = torch.zeros(2, 4096, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(2, dtype=torch.int32, device="cuda")
    tp = torch.ones(2, dtype=torch.float32, device="cuda")
    ws = L.alloc_sample_workspace(2, 64)
    with pytest.raises(L.LucciolaError) as e:
        L.sample_top_p(out, x, 100, tp, tp, ws)  # 96 candidates: no reference kernel
    assert e.value.status == 3
    with pytest.raises(L.LucciolaError) as e:
        L.sample_top_p(out, x, 128, tp, tp, ws)  # workspace sized for 64
    assert e.value.status == 4
