"""GPU parity of split-K decode attention over the fp16 KV cache.

Oracle: the engine's decode attention restated in oracle/fyodor_oracle.c
(llm_cpu.c:510-535) on the same fp16 values widened to F32, so the only
difference is summation order; bound |a - e| <= 1e-3 * (1 + |e|)."""
import ctypes as C

import numpy as np
import pytest

import fyodor_b200 as F
import oracle as O

pytestmark = pytest.mark.gpu


def run_attention(lengths, heads, kv_heads, hd, capacity, splits, seed):
    import torch
    rng = np.random.default_rng(seed)
    nseq = len(lengths)
    q = rng.standard_normal((nseq, heads, hd)).astype(np.float32)
    k = rng.standard_normal((nseq, kv_heads, capacity, hd)).astype(np.float16)
    v = rng.standard_normal((nseq, kv_heads, capacity, hd)).astype(np.float16)
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    dl = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    out = torch.empty((nseq, heads, hd), dtype=torch.float32, device="cuda")
    ws_bytes = F.lib.fyb_attention_workspace(nseq, heads, kv_heads, hd, splits)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    scale = 1.0 / np.sqrt(hd)
    P = lambda t: C.c_void_p(t.data_ptr())
    for _ in range(2):  # second call checks the scratch counters were reset
        r = F.lib.fyb_attention_decode(P(dq), P(dk), P(dv), kv_heads * capacity * hd, P(dl), nseq, heads, kv_heads,
                                       hd, capacity, C.c_float(scale), P(out), splits, P(ws), ws_bytes, None)
        assert r == 0
        torch.cuda.synchronize()
    got = out.cpu().numpy()
    for s in range(nseq):
        L = lengths[s]
        keys = np.transpose(k[s, :, :L, :], (1, 0, 2)).astype(np.float32)
        vals = np.transpose(v[s, :, :L, :], (1, 0, 2)).astype(np.float32)
        e = O.attention(q[s].reshape(-1), keys, vals, heads, kv_heads, hd, L, np.float32(scale)).reshape(heads, hd)
        err = np.abs(got[s] - e) / (1 + np.abs(e))
        assert err.max() <= 1e-3, (s, L, float(err.max()))


@pytest.mark.parametrize("hd,heads,kv_heads", [(128, 32, 8), (64, 16, 2), (128, 8, 8)])
def test_ragged_edges(hd, heads, kv_heads):
    lengths = [1, 2, 31, 32, 33, 255, 257, 1000]
    run_attention(lengths, heads, kv_heads, hd, 1024, 8, seed=hd + heads)


def test_ragged_batch_c4_subset():
    """C4 shape (32 q / 8 kv heads, hd 128) with lengths drawn from [128, 32768]."""
    rng = np.random.default_rng(77)
    lengths = [int(x) for x in rng.integers(128, 32769, size=6)] + [32768]
    run_attention(lengths, 32, 8, 128, 32768, 4, seed=5)


@pytest.mark.parametrize("splits", [1, 3, 37])
def test_split_counts(splits):
    run_attention([700, 5, 129], 32, 8, 128, 1024, splits, seed=splits)


def run_verify(lengths, queries, heads, kv_heads, hd, capacity, splits, seed):
    """fyb_attention_verify: query j of sequence s attends positions
    0 .. lengths[s] - queries + j (causal within the draft); each row is
    checked against the oracle's decode attention at that length."""
    import torch
    rng = np.random.default_rng(seed)
    nseq = len(lengths)
    q = rng.standard_normal((nseq, queries, heads, hd)).astype(np.float32)
    k = rng.standard_normal((nseq, kv_heads, capacity, hd)).astype(np.float16)
    v = rng.standard_normal((nseq, kv_heads, capacity, hd)).astype(np.float16)
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    dl = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    out = torch.empty((nseq, queries, heads, hd), dtype=torch.float32, device="cuda")
    ws_bytes = F.lib.fyb_attention_workspace(nseq * queries, heads, kv_heads, hd, splits)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    scale = 1.0 / np.sqrt(hd)
    P = lambda t: C.c_void_p(t.data_ptr())
    for _ in range(2):
        r = F.lib.fyb_attention_verify(P(dq), P(dk), P(dv), kv_heads * capacity * hd, P(dl), nseq, queries, heads,
                                       kv_heads, hd, capacity, C.c_float(scale), P(out), splits, P(ws), ws_bytes,
                                       None)
        assert r == 0
        torch.cuda.synchronize()
    got = out.cpu().numpy()
    for s in range(nseq):
        for j in range(queries):
            L = lengths[s] - queries + 1 + j
            keys = np.transpose(k[s, :, :L, :], (1, 0, 2)).astype(np.float32)
            vals = np.transpose(v[s, :, :L, :], (1, 0, 2)).astype(np.float32)
            e = O.attention(q[s, j].reshape(-1), keys, vals, heads, kv_heads, hd, L,
                            np.float32(scale)).reshape(heads, hd)
            err = np.abs(got[s, j] - e) / (1 + np.abs(e))
            assert err.max() <= 1e-3, (s, j, L, float(err.max()))


@pytest.mark.parametrize("hd,heads,kv_heads", [(128, 32, 8), (64, 16, 2)])
def test_verify_draft_of_8(hd, heads, kv_heads):
    """The C4 speculative-verify variant: 8 draft tokens per sequence."""
    run_verify([8, 9, 40, 300, 1000], 8, heads, kv_heads, hd, 1024, 8, seed=hd)


@pytest.mark.parametrize("queries,heads,kv_heads,hd", [(5, 32, 8, 128), (16, 32, 8, 128), (3, 8, 8, 64),
                                                      (17, 32, 8, 128)])
def test_verify_row_counts(queries, heads, kv_heads, hd):
    """Query rows (queries x group) that are not a multiple of the 16-row
    MMA tile (5 x 4 = 20, 3 x 1), the largest the shared-tile kernel takes
    (16 x 4 = 64), and one above it (17 x 4) that runs a CTA per row."""
    run_verify([queries, queries + 1, 100, 1023], queries, heads, kv_heads, hd, 1024, 5, seed=queries + hd)


@pytest.mark.parametrize("splits", [1, 3, 16])
def test_verify_c4_subset(splits):
    """C4's speculative-verify variant (32/8 heads, hd 128, 8 draft rows)
    with lengths up to 32768 and several partition counts."""
    rng = np.random.default_rng(91)
    lengths = [int(x) for x in rng.integers(128, 32769, size=3)] + [32768]
    run_verify(lengths, 8, 32, 8, 128, 32768, splits, seed=splits)


def test_verify_one_query_is_decode():
    """queries == 1 is plain decode attention."""
    run_verify([1, 77, 512], 1, 32, 8, 128, 512, 4, seed=3)


def test_verify_rejects_bad_shapes():
    import torch
    t = torch.zeros(16, device="cuda")
    P = C.c_void_p(t.data_ptr())
    # zero queries, more queries than the cache holds, too many query rows
    for nseq, queries, capacity in [(1, 0, 64), (1, 65, 64), (9000, 8, 64)]:
        assert F.lib.fyb_attention_verify(P, P, P, 0, P, nseq, queries, 32, 8, 128, capacity, C.c_float(0.1), P, 8,
                                          P, 1 << 30, None) == -1
