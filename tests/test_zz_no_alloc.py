"""fyb_attention_decode_static (scratch in a fixed device array, no
allocation) against fyb_attention_decode with a caller workspace.

Both run the same kernel, so each of two calls in a row must agree with the
workspace entry point within the attention tests' bound
|a - e| <= 1e-3 * (1 + |e|). Shapes change between calls so the counters land
at different offsets of the array. The file name keeps it last in collection:
it must pass after the other GPU tests as well as alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest

import fyodor_b200 as F

pytestmark = pytest.mark.gpu

STATIC_MAX = 4 << 20  # FYB_ATTENTION_STATIC_SCRATCH_BYTES


def _inputs(lengths, heads, kv_heads, hd, capacity, seed):
    import torch
    rng = np.random.default_rng(seed)
    nseq = len(lengths)
    q = torch.from_numpy(rng.standard_normal((nseq, heads, hd)).astype(np.float32)).cuda()
    k = torch.from_numpy(rng.standard_normal((nseq, kv_heads, capacity, hd)).astype(np.float16)).cuda()
    v = torch.from_numpy(rng.standard_normal((nseq, kv_heads, capacity, hd)).astype(np.float16)).cuda()
    dl = torch.tensor(lengths, dtype=torch.int32, device="cuda")
    return q, k, v, dl


def _P(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


@pytest.mark.parametrize("shape", [
    ([1, 33, 257, 1000], 32, 8, 128, 1024, 8),
    ([5, 700], 16, 2, 64, 768, 3),
    ([4096, 17, 2048], 32, 8, 128, 4096, 16),
])
def test_static_matches_workspace(shape):
    import torch
    lengths, heads, kv_heads, hd, capacity, splits = shape
    nseq = len(lengths)
    need = F.lib.fyb_attention_workspace(nseq, heads, kv_heads, hd, splits)
    assert 0 < need <= STATIC_MAX
    q, k, v, dl = _inputs(lengths, heads, kv_heads, hd, capacity, seed=hd + splits)
    scale = C.c_float(1.0 / np.sqrt(hd))
    stride = kv_heads * capacity * hd
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    ref = torch.empty((nseq, heads, hd), dtype=torch.float32, device="cuda")
    assert F.lib.fyb_attention_decode(_P(q), _P(k), _P(v), stride, _P(dl), nseq, heads, kv_heads, hd, capacity,
                                      scale, _P(ref), splits, _P(ws), need, None) == 0
    torch.cuda.synchronize()
    e = ref.cpu().numpy()
    outs = [torch.full((nseq, heads, hd), float("nan"), dtype=torch.float32, device="cuda") for _ in range(2)]
    free_after_first = None
    for call, out in enumerate(outs):
        r = F.lib.fyb_attention_decode_static(_P(q), _P(k), _P(v), stride, _P(dl), nseq, heads, kv_heads, hd,
                                              capacity, scale, _P(out), splits, None)
        assert r == 0, (call, r)
        torch.cuda.synchronize()
        # the entry point allocates nothing: free device memory does not move
        # between the first call (which looks up the array) and the next
        free = torch.cuda.mem_get_info()[0]
        if free_after_first is None:
            free_after_first = free
        else:
            assert free == free_after_first, (free, free_after_first)
        got = out.cpu().numpy()
        assert np.isfinite(got).all(), call
        err = np.abs(got - e) / (1 + np.abs(e))
        assert err.max() <= 1e-3, (call, float(err.max()))


def test_static_rejects_oversize():
    """A problem needing more scratch than the array holds returns -3 and
    launches nothing (the output keeps its sentinel)."""
    import torch
    heads, kv_heads, hd, capacity, splits = 32, 8, 128, 64, 64
    nseq = 16
    assert F.lib.fyb_attention_workspace(nseq, heads, kv_heads, hd, splits) > STATIC_MAX
    q, k, v, dl = _inputs([capacity] * nseq, heads, kv_heads, hd, capacity, seed=3)
    out = torch.full((nseq, heads, hd), 7.0, dtype=torch.float32, device="cuda")
    r = F.lib.fyb_attention_decode_static(_P(q), _P(k), _P(v), kv_heads * capacity * hd, _P(dl), nseq, heads,
                                          kv_heads, hd, capacity, C.c_float(0.088), _P(out), splits, None)
    assert r == -3
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())


def test_static_rejects_bad_arguments():
    """Unsupported head dimension or group size, or a null pointer, returns -1
    before anything is queued (the output keeps its sentinel)."""
    import torch
    q, k, v, dl = _inputs([40, 50], 32, 8, 128, 64, seed=9)
    out = torch.full((2, 32, 128), 5.0, dtype=torch.float32, device="cuda")
    sc = C.c_float(0.088)
    call = lambda **kw: F.lib.fyb_attention_decode_static(
        kw.get("q", _P(q)), _P(k), _P(v), 8 * 64 * 128, _P(dl), 2, kw.get("heads", 32), kw.get("kv", 8),
        kw.get("hd", 128), 64, sc, _P(out), 4, None)
    assert call(hd=96) == -1      # head dimension other than 64 or 128
    assert call(heads=24) == -1   # 3 query heads per KV head
    assert call(q=None) == -1     # null query
    torch.cuda.synchronize()
    assert bool((out == 5.0).all())
