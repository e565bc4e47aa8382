"""GPU parity of the dataflow form of the persistent decode kernel
(NYA_CUDA_DATAFLOW=1): GEMV phases start per 256-column input block as its
producers finish, RMSNorm scales are applied at the tile outputs and shared
tiles are summed by whichever warp completes them. The results must meet the
same bounds as the default form: logits within 1e-3 of the logit scale of
the fp16-KV oracle with the same argmax, greedy tokens equal to the oracle's
over 64 steps, and the KV cache within one fp16 rounding step of the default
form's. The geometries cover one, two, four and eight query heads per KV head
(with one, an attention-output block spans two KV heads) and head
dimensions 64 and 128."""
import os

import numpy as np
import pytest

import fyodor_b200 as F
import oracle as O
from tests.patterns import Q4_K, Q6_K, Q8_0, SMALL_MODELS, bench_tokens
from tests.test_gpu_plan import logit_error

pytestmark = pytest.mark.gpu

MODELS = SMALL_MODELS + [
    ("q4k_g1", dict(layers=2, embedding=512, heads=4, kv_heads=4, feed_forward=1024, vocabulary=1024, context=80,
                    matrix_type=Q4_K, embed_type=Q6_K, output_type=Q6_K, seed=21, norm_mode=2, centered=1),
     [int(t) for t in bench_tokens(9, 1024, 5)]),
    ("q4k_g8", dict(layers=3, embedding=512, heads=8, kv_heads=1, feed_forward=1536, vocabulary=2048, context=80,
                    matrix_type=Q4_K, embed_type=Q8_0, output_type=Q6_K, seed=22, norm_mode=1),
     [int(t) for t in bench_tokens(9, 2048, 7)]),
]


def _plan(provider, model, capacity, dataflow):
    if dataflow:
        os.environ["NYA_CUDA_DATAFLOW"] = "1"
    try:
        plan = provider.plan(model, capacity)
    finally:
        os.environ.pop("NYA_CUDA_DATAFLOW", None)
    assert plan is not None
    assert plan.decode_form() == (2 if dataflow else 1)
    return plan


@pytest.mark.parametrize("name,cfg,tokens", MODELS)
def test_dataflow_logits_and_kv(provider, name, cfg, tokens):
    m = F.SynthModel(**cfg)
    df = _plan(provider, m, len(tokens), True)
    base = _plan(provider, m, len(tokens), False)
    ref16 = O.Session(m.ptr, len(tokens), m.vocabulary, kv_f16=True)
    for i, t in enumerate(tokens):
        assert df.token(t, i) == 0 and base.token(t, i) == 0
        e16 = ref16.forward(t, i)
        assert logit_error(df.logits, e16) <= 1e-3, (i, logit_error(df.logits, e16))
        assert np.argmax(df.logits) == np.argmax(e16)
        assert logit_error(df.logits, base.logits) <= 2e-4, (i, logit_error(df.logits, base.logits))
    for layer in range(cfg["layers"]):
        a, b = df.read_kv(layer, 0, len(tokens)), base.read_kv(layer, 0, len(tokens))
        assert logit_error(a[0], b[0]) <= 1e-3 and logit_error(a[1], b[1]) <= 1e-3, layer
    m.close()


@pytest.mark.parametrize("name,cfg,tokens", MODELS)
def test_dataflow_greedy_64_steps(provider, name, cfg, tokens):
    cfg = dict(cfg, context=80)
    m = F.SynthModel(**cfg)
    plan = _plan(provider, m, 80, True)
    ref16 = O.Session(m.ptr, 80, m.vocabulary, kv_f16=True)
    got = plan.decode_greedy(tokens[0], 0, 64)
    assert got is not None
    t, expected = tokens[0], []
    for i in range(64):
        t = O.argmax(ref16.forward(t, i))
        expected.append(t)
    assert list(got) == expected
    m.close()


def test_dataflow_8b_layer_shapes(provider):
    """Two layers at the 8B geometry after a prefill (the attention spans
    several partitions)."""
    m = F.SynthModel(layers=2, embedding=4096, heads=32, kv_heads=8, feed_forward=14336, vocabulary=128256,
                     context=48, seed=99, norm_mode=2, centered=1)
    plan = _plan(provider, m, 48, True)
    ref16 = O.Session(m.ptr, 48, m.vocabulary, kv_f16=True)
    toks = [int(t) for t in bench_tokens(40, m.vocabulary)]
    assert plan.prefill(np.array(toks[:36], np.uint32), 0) == 0
    for i, t in enumerate(toks[:36]):
        ref16.forward(t, i)
    for i in range(36, 40):
        assert plan.token(toks[i], i) == 0
        e = ref16.forward(toks[i], i)
        assert logit_error(plan.logits, e) <= 1e-3, (i, logit_error(plan.logits, e))
        assert np.argmax(plan.logits) == np.argmax(e)
    m.close()
