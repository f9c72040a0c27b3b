"""The batched token-step driver (lc_kv_pool) on the GPU: prompts prefilled one
sequence at a time, then batched decode steps with sequences leaving and
joining, all checked against the CPU oracle (bit-exact cache writes, attention
within ATTN_ATOL); and the per-layer launches captured once in a CUDA graph and
replayed every step, against the same steps run eagerly."""
import numpy as np
import pytest

import lucciola as L
import oracle.oracle as O
from conftest import ATTN_ATOL
from workloads import from_device, to_device

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

HQ, HKV, HD, LAYERS, MAX_LEN, NB = 14, 2, 64, 2, 1024, 200
ROW = (HQ + 2 * HKV) * HD


def max_err(a, b):
    return float(np.abs(O.bf16_to_f32(a) - O.bf16_to_f32(b)).max())


def scaled(rng, shape, scale):
    return O.f32_to_bf16((rng.standard_normal(shape) * scale).astype(np.float32))


def rows(rng, shape):
    """qkv rows at half scale and biases (below) at quarter scale: attention
    outputs then stay below 2 in magnitude, where the bf16 output step is
    1/128 and a rounding on each side fits inside ATTN_ATOL. With unit-scale
    biases the outputs reach 4-8, whose step (1/32) alone exceeds it."""
    return scaled(rng, shape, 0.5)


def check_attention(out, ref):
    assert np.abs(O.bf16_to_f32(ref)).max() < 2.0  # the premise of ATTN_ATOL here
    assert max_err(from_device(out), ref) <= ATTN_ATOL


class Mirror:
    """Host copy of a pool's contents, advanced by the oracle."""

    def __init__(self, pool, seed):
        self.pool = pool
        shape = (NB, LAYERS, HKV, 16, HD)
        self.k = np.zeros(shape, np.uint16)
        self.v = np.zeros(shape, np.uint16)
        self.rng = np.random.default_rng(seed)
        self.bias = [tuple(scaled(self.rng, (n * HD,), 0.25) for n in (HQ, HKV, HKV))
                     for _ in range(LAYERS)]
        self.dbias = [tuple(to_device(b) for b in layer) for layer in self.bias]
        self.cos, self.sin = O.rope_table(MAX_LEN, HD, 1e6)
        self.dcos, self.dsin = to_device(self.cos), to_device(self.sin)

    def tables(self, slots):
        t = np.zeros((len(slots), self.pool.table_stride), np.int32)
        for i, s in enumerate(slots):
            pg = self.pool.pages(s)
            t[i, :len(pg)] = pg
        return t

    def prefill(self, slot, tokens, start=0):
        self.pool.prepare_prefill(slot, start, tokens)
        tab = self.tables([slot])
        pos = np.arange(start, start + tokens, dtype=np.int32)
        for layer in range(LAYERS):
            qkv = rows(self.rng, (tokens, ROW))
            dqkv = to_device(qkv)
            out = torch.empty(tokens, HQ * HD, dtype=torch.bfloat16, device="cuda")
            self.pool.prefill_layer(layer, out, dqkv, *self.dbias[layer], self.dcos, self.dsin)
            qb, kb, vb = self.bias[layer]
            O.rope_append(qkv, pos, qb, kb, vb, self.cos, self.sin, self.k, self.v, LAYERS,
                          layer, HQ, HKV, HD, tab, tokens_per_seq=tokens)
            ref = O.paged_prefill(np.ascontiguousarray(qkv[:, :HQ * HD]), self.k, self.v, layer,
                                  HQ, HKV, HD, tab, np.full(1, start, np.int32), tokens, LAYERS,
                                  threads=8)
            torch.cuda.synchronize()
            check_attention(out, ref)

    def decode_inputs(self, batch):
        return [rows(self.rng, (batch, ROW)) for _ in range(LAYERS)]

    def decode_reference(self, slots, positions, qkvs):
        tab = self.tables(slots)
        pos = np.asarray(positions, np.int32)
        refs = []
        for layer in range(LAYERS):
            qkv = qkvs[layer].copy()
            qb, kb, vb = self.bias[layer]
            O.rope_append(qkv, pos, qb, kb, vb, self.cos, self.sin, self.k, self.v, LAYERS,
                          layer, HQ, HKV, HD, tab)
            refs.append(O.paged_decode(qkv, self.k, self.v, layer, HQ, HKV, HD, tab, pos, LAYERS,
                                       len_offset=1))
        return refs

    def check_pools(self):
        torch.cuda.synchronize()
        kp, vp = self.pool.pools()
        assert np.array_equal(from_device(kp), self.k)
        assert np.array_equal(from_device(vp), self.v)


def test_pool_prefill_and_batched_decode_match_oracle():
    pool = L.KVPool(LAYERS, HQ, HKV, HD, 4, MAX_LEN, NB)
    m = Mirror(pool, seed=1)
    lens = {}
    for tokens in (37, 100, 5):
        s = pool.add_sequence()
        m.prefill(s, tokens)
        lens[s] = tokens
    assert pool.pages(0) == [0, 1, 2]  # a fresh pool hands out pages in order

    def step(order):
        positions = [lens[s] for s in order]
        pool.prepare_step(order, positions)
        qkvs = m.decode_inputs(len(order))
        outs = []
        for layer in range(LAYERS):
            out = torch.empty(len(order), HQ * HD, dtype=torch.bfloat16, device="cuda")
            pool.decode_layer(layer, out, to_device(qkvs[layer]), *m.dbias[layer], m.dcos, m.dsin)
            outs.append(out)
        refs = m.decode_reference(order, positions, qkvs)
        torch.cuda.synchronize()
        for out, ref in zip(outs, refs):
            check_attention(out, ref)
        for s in order:
            lens[s] += 1

    for _ in range(3):
        step([2, 0, 1])  # batch order differs from slot order
    freed = pool.pages(1)
    pool.release_sequence(1)
    lens.pop(1)
    s3 = pool.add_sequence()
    assert s3 == 1
    m.prefill(s3, 20)
    lens[s3] = 20
    assert pool.pages(s3) == freed[:2]  # released pages come back in order
    for _ in range(3):
        step([2, 0, s3])
    step([0])  # a smaller batch on the same pool
    m.check_pools()
    pool.close()


def test_pool_decode_graph_replay_matches_eager():
    pools = [L.KVPool(LAYERS, HQ, HKV, HD, 4, MAX_LEN, NB) for _ in range(2)]
    mirrors = [Mirror(p, seed=5) for p in pools]  # same seed: same prompts and inputs
    order, lens = [], []
    for tokens in (300, 17, 64):
        for m in mirrors:
            s = m.pool.add_sequence()
            m.prefill(s, tokens)
        order.append(s)
        lens.append(tokens)
    B = len(order)
    eager, graphed = pools
    # static buffers of the captured step
    qkv_in = [torch.empty(B, ROW, dtype=torch.bfloat16, device="cuda") for _ in range(LAYERS)]
    out_g = [torch.empty(B, HQ * HD, dtype=torch.bfloat16, device="cuda") for _ in range(LAYERS)]
    graph = None
    for _ in range(4):
        qkvs = mirrors[0].decode_inputs(B)
        mirrors[1].decode_inputs(B)  # keep the two generators in step
        eager.prepare_step(order, lens)
        out_e = []
        for layer in range(LAYERS):
            out = torch.empty(B, HQ * HD, dtype=torch.bfloat16, device="cuda")
            eager.decode_layer(layer, out, to_device(qkvs[layer]), *mirrors[0].dbias[layer],
                               mirrors[0].dcos, mirrors[0].dsin)
            out_e.append(out)
        graphed.prepare_step(order, lens)
        for layer in range(LAYERS):
            qkv_in[layer].copy_(to_device(qkvs[layer]))
        if graph is None:
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for layer in range(LAYERS):
                    graphed.decode_layer(layer, out_g[layer], qkv_in[layer],
                                         *mirrors[1].dbias[layer], mirrors[1].dcos,
                                         mirrors[1].dsin)
        graph.replay()
        torch.cuda.synchronize()
        for a, b in zip(out_e, out_g):
            assert torch.equal(a.view(torch.int16), b.view(torch.int16))
        lens = [n + 1 for n in lens]
    ke, ve = eager.pools()
    kg, vg = graphed.pools()
    assert torch.equal(ke.view(torch.int16), kg.view(torch.int16))
    assert torch.equal(ve.view(torch.int16), vg.view(torch.int16))
    del graph
    for p in pools:
        p.close()


def test_pool_chunked_prefill_then_decode():
    """A prompt in three chunks (prepare_prefill with a start position): each
    chunk attends over the pages the earlier chunks filled; then decode steps."""
    pool = L.KVPool(LAYERS, HQ, HKV, HD, 2, MAX_LEN, NB)
    m = Mirror(pool, seed=9)
    s = pool.add_sequence()
    start = 0
    for tokens in (100, 37, 130):  # chunk boundaries inside pages
        m.prefill(s, tokens, start=start)
        start += tokens
    assert len(pool.pages(s)) == (start + 15) // 16
    for _ in range(2):
        pool.prepare_step([s], [start])
        qkvs = m.decode_inputs(1)
        outs = []
        for layer in range(LAYERS):
            out = torch.empty(1, HQ * HD, dtype=torch.bfloat16, device="cuda")
            pool.decode_layer(layer, out, to_device(qkvs[layer]), *m.dbias[layer], m.dcos, m.dsin)
            outs.append(out)
        refs = m.decode_reference([s], [start], qkvs)
        torch.cuda.synchronize()
        for out, ref in zip(outs, refs):
            check_attention(out, ref)
        start += 1
    m.check_pools()
    pool.close()
