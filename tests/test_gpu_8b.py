"""Full-depth parity of the 8B configuration the bench times.

The 32-layer 8B-class model of the decode benchmark (d 4096, 32/8 heads of
128, FFN 14336, vocabulary 128256, Q4_K projections, Q6_K embedding and
output head, fp16 KV cache; the bench's seed and norm distribution) runs a
64-token prompt through plan_prefill, then 64 greedy steps through the
device greedy loop (fyb_plan_decode_greedy, the path behind the bench's
`value`). The oracle is the restated engine with an fp16 KV cache
(oracle/fyodor_oracle.c, pinned bit-identical to the engine's scalar path),
with its products spread over the host's cores. Logits at the last prompt
token must agree within 1e-3 of the logit scale with the same argmax, and
all 64 greedy tokens must be identical."""
import os

import numpy as np
import pytest

import fyodor_b200 as F
import oracle as O
from tests.patterns import bench_tokens
from tests.test_gpu_plan import logit_error

pytestmark = pytest.mark.gpu

CFG8B = dict(layers=32, embedding=4096, heads=32, kv_heads=8, feed_forward=14336, vocabulary=128256, context=1024,
             matrix_type=F.Q4_K, embed_type=F.Q6_K, output_type=F.Q6_K, rope_base=500000.0, epsilon=1e-5,
             seed=1234, norm_mode=1)
PROMPT, STEPS = 64, 64


@pytest.fixture(scope="module")
def model_8b():
    m = F.SynthModel(**CFG8B)
    yield m
    m.close()


def test_8b_prompt_then_64_greedy_steps(provider, model_8b):
    m = model_8b
    prompt = bench_tokens(PROMPT, m.vocabulary)
    plan = provider.plan(m, PROMPT + STEPS + 1)
    assert plan is not None
    assert plan.prefill(prompt, 0) == 0
    got = plan.logits.copy()
    first = int(np.argmax(got))
    tokens = plan.decode_greedy(first, PROMPT, STEPS)
    assert tokens is not None
    plan.close()

    O.set_threads(os.cpu_count() or 1)
    try:
        ref = O.Session(m.ptr, PROMPT + STEPS + 1, m.vocabulary, kv_f16=True)
        for i, t in enumerate(prompt[:-1]):
            ref.forward(int(t), i, logits=False)
        e = ref.forward(int(prompt[-1]), PROMPT - 1)
        assert logit_error(got, e) <= 1e-3, logit_error(got, e)
        assert O.argmax(e) == first
        t, expected = first, []
        for i in range(STEPS):
            t = O.argmax(ref.forward(t, PROMPT + i))
            expected.append(t)
        ref.close()
    finally:
        O.set_threads(1)
    assert list(tokens) == expected
