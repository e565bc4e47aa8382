"""GPU parity of batched decode (fyb_batch_*): B sequences of one plan's
model, each with its own KV cache and its own (ragged) position, against one
fp16-KV oracle session per sequence. Sizes cover every GEMM form of a step:
two sequences (tensor-core GEMV), five (mma.sync small-batch GEMM) and twelve
(tcgen05 GEMM). Logits within 1e-3 of the logit scale, argmax equal, and
greedy tokens decoded on the device identical to the oracle's."""
import numpy as np
import pytest

import fyodor_b200 as F
import oracle as O

pytestmark = pytest.mark.gpu

CFG = dict(layers=2, embedding=512, heads=8, kv_heads=2, feed_forward=1024, vocabulary=1024, context=48,
           matrix_type=F.Q4_K, seed=21, norm_mode=2)


def logit_error(a, b):
    return float(np.max(np.abs(a - b)) / (1 + np.max(np.abs(b))))


@pytest.mark.parametrize("nseq", [2, 5, 12])
def test_batch_matches_oracle(provider, nseq):
    m = F.SynthModel(**CFG)
    plan = provider.plan(m, CFG["context"])
    assert plan is not None
    batch = F.Batch(plan, nseq)
    refs = [O.Session(m.ptr, CFG["context"], m.vocabulary, kv_f16=True) for _ in range(nseq)]
    rng = np.random.default_rng(nseq)
    stop = 6 + 3 * np.arange(nseq) % 17  # sequence b stays at position stop[b] once it gets there (ragged)
    pos = np.zeros(nseq, np.uint32)
    for s in range(24):
        pos = np.minimum(s, stop).astype(np.uint32)
        toks = rng.integers(0, m.vocabulary, nseq).astype(np.uint32)
        lg, am = batch.step(toks, pos)
        for b in range(nseq):
            e = refs[b].forward(int(toks[b]), int(pos[b]))
            assert logit_error(lg[b], e) <= 1e-3, (s, b, logit_error(lg[b], e))
            assert am[b] == np.argmax(lg[b]) == np.argmax(e), (s, b)
    # greedy continuation on the device from each sequence's next position
    start = (pos + 1).astype(np.uint32)
    first = am.copy()
    got = batch.decode_greedy(first, start, 8)
    for b in range(nseq):
        t = int(first[b])
        for i in range(8):
            t = int(np.argmax(refs[b].forward(t, int(start[b]) + i)))
            assert got[i, b] == t, (b, i)
    batch.close()
    plan.close()
    m.close()
