"""Pins the C restatement (oracle/fyodor_oracle.c) to the reference engine.

Golden fixtures in tests/golden/ were produced by the compiled Fyodor engine
(tests/golden/make_golden.py); the known-answer K-quant blocks and the
binary16 boundary cases come from the reference's own tests
(test_architectures.c:232-307, test_kv_precision.c, test_quant_kernels.c).
"""
import os

import numpy as np
import pytest

import fyodor_b200 as F
import oracle as O
from tests.conftest import ROOT
from tests.patterns import k_quant_blocks, quant_kernel_inputs, quant_kernel_weights, SMALL_MODELS

GOLD = os.path.join(ROOT, "tests", "golden")


def load(name):
    return np.load(os.path.join(GOLD, name))


@pytest.mark.parametrize("kind,type_id", [(0, F.Q4_K), (1, F.Q6_K)])
def test_k_quant_known_answers(kind, type_id):
    data, expected = k_quant_blocks(kind)
    g = load("kquant_known.npz")
    assert (g["data_%d" % type_id] == data).all()
    got = O.dequantize(data, type_id, 1024)
    assert (got == expected).all()                      # exact, independently constructed
    assert (got == g["ref_values_%d" % type_id]).all()  # equals the engine
    x = np.array([((i % 23) - 11) / 16.0 for i in range(512)], np.float32)
    y = O.matvec(data, type_id, x, 512, 2)
    dot = expected.reshape(2, 512).astype(np.float64) @ x.astype(np.float64)
    assert (y.astype(np.float64) == dot).all()          # exact for these power-of-two fixtures
    assert (y == g["ref_matvec_%d" % type_id]).all()


@pytest.mark.parametrize("type_id", [F.F32, F.F16, F.BF16, F.Q4_0, F.Q8_0, F.Q4_K, F.Q6_K])
def test_quant_kernel_patterns_match_engine(type_id):
    g = load("quant_kernels.npz")
    data = quant_kernel_weights(type_id, 65, 1024)
    assert (data == g["data_%d" % type_id]).all()
    assert (O.dequantize(data, type_id, 65 * 1024) == g["values_%d" % type_id]).all()
    for p in range(3):
        y = O.matvec(data, type_id, quant_kernel_inputs(1024, p), 1024, 65)
        assert (y == g["y_%d_%d" % (type_id, p)]).all()


def test_half_conversion_exhaustive():
    bits = np.arange(65536, dtype=np.uint32)
    finite = ((bits >> 10) & 31) != 31
    ours = np.array([O.half_to_float(int(b)) for b in bits[finite]], np.float32)
    numpy = bits[finite].astype(np.uint16).view(np.float16).astype(np.float32)
    assert (ours.view(np.uint32) == numpy.view(np.uint32)).all()


def test_round_f16_boundaries():
    """test_kv_precision.c: every encoding is a fixed point; midpoints go to even."""
    rng = np.random.default_rng(5)
    hs = np.concatenate([np.arange(0, 0x7bff, 97), rng.integers(0, 0x7bff, 2000)]).astype(np.uint16)
    for h in hs:
        a = np.float32(np.uint16(h).view(np.float16))
        b = np.float32(np.uint16(h + 1).view(np.float16))
        mid = np.float32((a + b) * np.float32(0.5))
        expected = b if (h & 1) else a
        assert O.round_f16(float(a)) == a
        assert O.round_f16(float(mid)) == expected
        assert O.round_f16(float(np.nextafter(mid, np.float32(0)))) == a
        assert O.round_f16(float(np.nextafter(mid, np.float32(np.inf)))) == b
    assert np.isinf(O.round_f16(65520.0)) and O.round_f16(float(np.nextafter(np.float32(65520), 0))) == 65504.0
    assert np.isnan(O.round_f16(float("nan")))


@pytest.mark.parametrize("name,cfg,tokens", SMALL_MODELS)
def test_session_logits_match_engine(name, cfg, tokens):
    g = load("small_models.npz")
    m = F.SynthModel(**cfg)
    s = O.Session(m.ptr, len(tokens), m.vocabulary, kv_f16=False)
    for i, t in enumerate(tokens):
        logits = s.forward(t, i)
        assert (logits == g[name + "_logits"][i]).all(), i  # bit-identical to the engine
    k, v = s.read_kv(cfg["layers"] - 1, 0, len(tokens), m.kv_dim)
    assert (k == g[name + "_k_last"]).all() and (v == g[name + "_v_last"]).all()


def test_engine_cross_check_when_built():
    """Where the reference engine was compiled here, compare live as well."""
    if not O.reference_available():
        pytest.skip("reference engine not built in this checkout")
    rng = np.random.default_rng(1)
    for type_id in (F.Q4_K, F.Q6_K, F.Q8_0):
        m = F.SynthModel(layers=1, embedding=512, heads=4, kv_heads=2, feed_forward=512, vocabulary=64, context=4,
                         matrix_type=type_id, embed_type=F.Q6_K, output_type=F.Q6_K, seed=int(rng.integers(1 << 30)))
        data = m.tensor_bytes(4)
        x = rng.standard_normal(512).astype(np.float32)
        assert (O.matvec(data, type_id, x, 512, 512) == O.ref_matvec(data, type_id, x, 512, 512)).all()


@pytest.mark.parametrize("type_id", [F.Q4_K, F.Q6_K, F.Q8_0, F.F16])
@pytest.mark.parametrize("threads", [1, 3, 8])
def test_threaded_matvec_bit_identical(type_id, threads):
    """The threaded oracle product (rows spread over threads, K-quant rows four
    at a time) equals the scalar restatement bit for bit: every row keeps the
    engine's summation order (llm_quant.c:145-312)."""
    g = load("quant_kernels.npz")
    data = quant_kernel_weights(type_id, 65, 1024)
    O.set_threads(threads)
    try:
        for p in range(3):
            x = quant_kernel_inputs(1024, p)
            assert (O.matvec_threaded(data, type_id, x, 1024, 65) == g["y_%d_%d" % (type_id, p)]).all()
        rng = np.random.default_rng(threads)
        m = F.SynthModel(layers=1, embedding=512, heads=4, kv_heads=2, feed_forward=1024, vocabulary=64, context=4,
                         matrix_type=type_id if type_id in (F.Q4_K, F.Q6_K) else F.Q4_K, seed=threads)
        w = m.tensor_bytes(10)  # blk.0.ffn_down.weight: 512 rows x 1024 columns
        x = rng.standard_normal(1024).astype(np.float32)
        tid = type_id if type_id in (F.Q4_K, F.Q6_K) else F.Q4_K
        assert (O.matvec_threaded(w, tid, x, 1024, 512) == O.matvec(w, tid, x, 1024, 512)).all()
    finally:
        O.set_threads(1)


def test_threaded_session_bit_identical():
    """A session whose products run on several threads gives the same logits
    as the single-threaded session (and so as the engine)."""
    name, cfg, tokens = SMALL_MODELS[0]
    g = load("small_models.npz")
    m = F.SynthModel(**cfg)
    O.set_threads(5)
    try:
        s = O.Session(m.ptr, len(tokens), m.vocabulary, kv_f16=False)
        for i, t in enumerate(tokens):
            assert (s.forward(t, i) == g[name + "_logits"][i]).all(), i
    finally:
        O.set_threads(1)
