"""GPU parity of the resident plan (full decode) through the provider vtable.

Two oracles per model: the restated engine with an fp16 KV cache (same
cache semantics as the provider) and the compiled engine's F32 KV logits
stored in tests/golden/small_models.npz. Logits must agree within 1e-3 of
the logit scale with the fp16-KV oracle and within 2e-3 with the F32-KV
engine, and all three argmaxes must agree; greedy tokens must match the
fp16-KV oracle."""
import os
import subprocess
import sys

import numpy as np
import pytest

import fyodor_b200 as F
import oracle as O
from tests.conftest import ROOT
from tests.patterns import SMALL_MODELS, bench_tokens

pytestmark = pytest.mark.gpu
GOLD = np.load(os.path.join(ROOT, "tests", "golden", "small_models.npz"))


def scaled_error(a, b):
    """Per-element |a - b| / (1 + |b|) (test_inference.c:219), for O(1) values."""
    return float(np.max(np.abs(a - b) / (1 + np.abs(b))))


def logit_error(a, b):
    """Error relative to the logit scale, max|a - b| / (1 + max|b|). With an
    fp16 KV cache a near-zero logit of a high-gain random model moves by
    ~1e-4 of the scale when one cached value rounds to the other neighbour,
    which the per-element form would report as ~1e-1."""
    return float(np.max(np.abs(a - b)) / (1 + np.max(np.abs(b))))


@pytest.mark.parametrize("name,cfg,tokens", SMALL_MODELS)
def test_plan_logits(provider, name, cfg, tokens):
    m = F.SynthModel(**cfg)
    plan = provider.plan(m, len(tokens))
    assert plan is not None
    ref16 = O.Session(m.ptr, len(tokens), m.vocabulary, kv_f16=True)
    for i, t in enumerate(tokens):
        assert plan.token(t, i) == 0
        got = plan.logits.copy()
        e16 = ref16.forward(t, i)
        assert logit_error(got, e16) <= 1e-3, (i, logit_error(got, e16))
        # the engine keeps an F32 cache: its logits differ from any fp16-KV run
        # by up to ~7e-4 of the scale on these models (oracle vs oracle), so
        # the bound against it carries that margin
        assert logit_error(got, GOLD[name + "_logits"][i]) <= 2e-3, (i, logit_error(got, GOLD[name + "_logits"][i]))
        assert np.argmax(got) == np.argmax(e16) == np.argmax(GOLD[name + "_logits"][i])
    kv = plan.read_kv(cfg["layers"] - 1, 0, len(tokens))
    k16, v16 = ref16.read_kv(cfg["layers"] - 1, 0, len(tokens), m.kv_dim)
    # last layer of a high-gain model: compare on the tensor's scale, as the logits
    assert logit_error(kv[0], k16) <= 2e-3 and logit_error(kv[1], v16) <= 2e-3, \
        (logit_error(kv[0], k16), logit_error(kv[1], v16))
    st = plan.stats()
    assert st["graph_captures"] == 1 and st["graph_replays"] == len(tokens)
    assert st["kv_bytes"] == cfg["layers"] * m.kv_dim * len(tokens) * 2 * 2


@pytest.mark.parametrize("name,cfg,tokens", SMALL_MODELS)
def test_greedy_64_steps(provider, name, cfg, tokens):
    cfg = dict(cfg, context=80)
    m = F.SynthModel(**cfg)
    plan = provider.plan(m, 80)
    ref16 = O.Session(m.ptr, 80, m.vocabulary, kv_f16=True)
    first = tokens[0]
    got = plan.decode_greedy(first, 0, 64)
    assert got is not None
    t, expected = first, []
    for i in range(64):
        t = O.argmax(ref16.forward(t, i))
        expected.append(t)
    assert list(got) == expected


def test_prefill_then_decode_matches_tokens(provider):
    """plan_prefill (one chunk of 8 prompt tokens through the batched step)
    against plan_token steps and the fp16-KV oracle: the two GPU paths sum in
    different orders, so they meet on the oracle's bound, not bitwise."""
    name, cfg, tokens = SMALL_MODELS[0]
    m = F.SynthModel(**cfg)
    a = provider.plan(m, 32)
    b = provider.plan(m, 32)
    ref16 = O.Session(m.ptr, 32, m.vocabulary, kv_f16=True)
    assert a.prefill(np.array(tokens[:8], np.uint32), 0) == 0
    la = a.logits.copy()
    assert a.stats()["prefill_batch"] == 16  # the chunked path ran
    for i, t in enumerate(tokens[:8]):
        assert b.token(t, i, logits=(i == 7)) == 0
        e = ref16.forward(t, i)
    assert logit_error(la, e) <= 1e-3 and logit_error(b.logits, e) <= 1e-3
    assert np.argmax(la) == np.argmax(b.logits) == np.argmax(e)
    assert a.token(tokens[8], 8) == 0 and b.token(tokens[8], 8) == 0
    e = ref16.forward(tokens[8], 8)
    assert logit_error(a.logits, e) <= 1e-3 and logit_error(b.logits, e) <= 1e-3


@pytest.mark.parametrize("name,cfg,tokens", SMALL_MODELS)
def test_chunked_prefill(provider, name, cfg, tokens):
    """Prompts of 37 tokens (chunks of 16, 16 and 5) at positions 0 and then
    3 (a second prefill after the first three tokens rewrites the rest):
    logits of the last token and every cached K/V row against the fp16-KV
    oracle."""
    m = F.SynthModel(**cfg)
    prompt = bench_tokens(37, m.vocabulary, 5)
    plan = provider.plan(m, 48)
    ref16 = O.Session(m.ptr, 48, m.vocabulary, kv_f16=True)
    assert plan.prefill(prompt, 0) == 0
    for i, t in enumerate(prompt):
        e = ref16.forward(int(t), i, logits=i == len(prompt) - 1)
    assert logit_error(plan.logits, e) <= 1e-3, logit_error(plan.logits, e)
    assert np.argmax(plan.logits) == np.argmax(e)
    kv = plan.read_kv(cfg["layers"] - 1, 0, len(prompt))
    k16, v16 = ref16.read_kv(cfg["layers"] - 1, 0, len(prompt), m.kv_dim)
    assert logit_error(kv[0], k16) <= 2e-3 and logit_error(kv[1], v16) <= 2e-3
    second = bench_tokens(30, m.vocabulary, 11)
    assert plan.prefill(second, 3) == 0
    for i, t in enumerate(second):
        e = ref16.forward(int(t), 3 + i, logits=i == len(second) - 1)
    assert logit_error(plan.logits, e) <= 1e-3, logit_error(plan.logits, e)
    assert np.argmax(plan.logits) == np.argmax(e)
    t = int(np.argmax(e))
    assert plan.token(t, 33) == 0
    assert logit_error(plan.logits, ref16.forward(t, 33)) <= 1e-3


def test_plan_argument_validation(provider):
    name, cfg, tokens = SMALL_MODELS[0]
    m = F.SynthModel(**cfg)
    p = provider.plan(m, 16)
    assert p.token(m.vocabulary, 0) == -1        # token outside the vocabulary
    assert p.token(1, 3) == -1                   # skips positions 0..2
    assert p.token(1, 16) == -1                  # beyond capacity
    assert p.api.plan_token(p.ptr, 1, 0, 1, None) == -1  # logits without output
    assert p.token(1, 0) == 0                    # still usable afterwards
    assert provider.plan(m, m.config.context + 1) is None  # capacity above the model context
    assert p.read_kv(0, 0, 2) is None            # only the valid prefix is readable


def test_8b_layer_shapes(provider):
    """Two layers at the 8B geometry (d 4096, 32/8 heads, FFN 14336, V 128256)."""
    m = F.SynthModel(layers=2, embedding=4096, heads=32, kv_heads=8, feed_forward=14336, vocabulary=128256,
                     context=16, seed=99, norm_mode=2, centered=1)
    plan = provider.plan(m, 8)
    ref16 = O.Session(m.ptr, 8, m.vocabulary, kv_f16=True)
    for i, t in enumerate(bench_tokens(3, m.vocabulary)):
        assert plan.token(int(t), i) == 0
        e = ref16.forward(int(t), i)
        assert logit_error(plan.logits, e) <= 1e-3, (i, logit_error(plan.logits, e))
        assert np.argmax(plan.logits) == np.argmax(e)


@pytest.mark.parametrize("name,cfg,tokens", SMALL_MODELS)
def test_persistent_matches_per_kernel(provider, name, cfg, tokens):
    """The persistent decode kernel (default) and the one-kernel-per-operation
    step (NYA_CUDA_PERSISTENT=0) compute the same logits; they differ only in
    summation order (sums of squares per tile, split-K partitions)."""
    m = F.SynthModel(**cfg)
    plan = provider.plan(m, len(tokens))
    assert plan.launches_per_token() == 2  # request + one decode kernel
    os.environ["NYA_CUDA_PERSISTENT"] = "0"
    try:
        multi = provider.plan(m, len(tokens))
    finally:
        del os.environ["NYA_CUDA_PERSISTENT"]
    assert multi.launches_per_token() == 3 + 5 * cfg["layers"]
    for i, t in enumerate(tokens):
        assert plan.token(t, i) == 0 and multi.token(t, i) == 0
        assert logit_error(plan.logits, multi.logits) <= 2e-4, (i, logit_error(plan.logits, multi.logits))
        assert np.argmax(plan.logits) == np.argmax(multi.logits)
    for layer in range(cfg["layers"]):
        a, b = plan.read_kv(layer, 0, len(tokens)), multi.read_kv(layer, 0, len(tokens))
        # fp16 cache: one rounding step at the largest magnitude is ~1e-3 of the scale
        assert logit_error(a[0], b[0]) <= 1e-3 and logit_error(a[1], b[1]) <= 1e-3


def _env_run(code, **env):
    e = dict(os.environ, **{k: str(v) for k, v in env.items()})
    return subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=e, capture_output=True, text=True, timeout=300)


def test_fail_after_injection():
    """NYA_CUDA_FAIL_AFTER=N fails the step at position N (resident.inc:192-198)."""
    code = ("import fyodor_b200 as F\n"
            "m=F.SynthModel(layers=1,embedding=512,heads=4,kv_heads=2,feed_forward=512,vocabulary=256,context=8)\n"
            "p=F.Provider().plan(m,8)\n"
            "print([p.token(3,i) for i in range(4)])\n")
    r = _env_run(code, NYA_CUDA_FAIL_AFTER=2)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "[0, 0, -1, -1]"


def test_allocation_failure_injection():
    """NYA_CUDA_FAIL_ALLOCATION_AFTER=N declines the plan and rolls back."""
    code = ("import fyodor_b200 as F\n"
            "m=F.SynthModel(layers=1,embedding=512,heads=4,kv_heads=2,feed_forward=512,vocabulary=256,context=8)\n"
            "pr=F.Provider(); print(pr.plan(m,8) is None, pr.active())\n")
    r = _env_run(code, NYA_CUDA_FAIL_ALLOCATION_AFTER=3)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "True True"


def test_graphs_disabled_matches():
    code = ("import fyodor_b200 as F, numpy as np\n"
            "m=F.SynthModel(layers=2,embedding=512,heads=4,kv_heads=2,feed_forward=512,vocabulary=256,context=8,seed=4)\n"
            "p=F.Provider().plan(m,8)\n"
            "out=[]\n"
            "for i in range(4):\n"
            "    p.token(5+i,i); out.append(p.logits.copy())\n"
            "np.save('/tmp/fyb_graphs.npy' if __import__('os').environ.get('NYA_CUDA_GRAPHS','1')!='0' else '/tmp/fyb_eager.npy', np.stack(out))\n")
    assert _env_run(code).returncode == 0
    assert _env_run(code, NYA_CUDA_GRAPHS=0).returncode == 0
    a, b = np.load("/tmp/fyb_graphs.npy"), np.load("/tmp/fyb_eager.npy")
    assert (a == b).all()


@pytest.mark.parametrize("ring", ["4608", "0", "13440"])
def test_ring_sizes_match(ring):
    """NYA_CUDA_RING_BYTES changes only how many weight units each warp keeps
    in flight: a request below two Q6_K units is raised to two, 0 takes what
    shared memory leaves. Logits must equal the default ring's bitwise."""
    code = ("import fyodor_b200 as F, numpy as np, sys\n"
            "m=F.SynthModel(layers=2,embedding=512,heads=4,kv_heads=2,feed_forward=1024,vocabulary=1024,context=8,"
            "matrix_type=F.Q4_K,embed_type=F.Q6_K,output_type=F.Q6_K,seed=6,norm_mode=2)\n"
            "p=F.Provider().plan(m,8)\n"
            "assert p.decode_form()==1\n"
            "out=[]\n"
            "for i in range(4):\n"
            "    assert p.token(9+i,i)==0; out.append(p.logits.copy())\n"
            "np.save(sys.argv[1] if len(sys.argv)>1 else '/tmp/x.npy', np.stack(out))\n")
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        a, b = os.path.join(d, "a.npy"), os.path.join(d, "b.npy")
        run = lambda path, **env: subprocess.run([sys.executable, "-c", code, path], cwd=ROOT, capture_output=True,
                                                 text=True, timeout=300, env=dict(os.environ, **env))
        r1 = run(a)
        assert r1.returncode == 0, r1.stderr
        r2 = run(b, NYA_CUDA_RING_BYTES=ring)
        assert r2.returncode == 0, r2.stderr
        assert (np.load(a) == np.load(b)).all()


@pytest.mark.parametrize("name,cfg,tokens", SMALL_MODELS)
def test_verify_draft(provider, name, cfg, tokens):
    """fyb_plan_verify: a prompt, then an 8-token draft checked in one pass
    (every row's logits against the fp16-KV oracle at its position), then a
    second draft from inside the first (the rejected tail is rewritten),
    then a plain decode step after it."""
    m = F.SynthModel(**cfg)
    plan = provider.plan(m, 48)
    ref16 = O.Session(m.ptr, 48, m.vocabulary, kv_f16=True)
    prompt = bench_tokens(11, m.vocabulary, 2)
    assert plan.prefill(prompt, 0) == 0
    for i, t in enumerate(prompt):
        ref16.forward(int(t), i, logits=False)
    for start, draft in ((11, bench_tokens(8, m.vocabulary, 7)), (14, bench_tokens(16, m.vocabulary, 9))):
        got = plan.verify(draft, start)
        assert got is not None and got.shape == (len(draft), m.vocabulary)
        for i, t in enumerate(draft):
            e = ref16.forward(int(t), start + i)
            assert logit_error(got[i], e) <= 1e-3, (start, i, logit_error(got[i], e))
            assert np.argmax(got[i]) == np.argmax(e)
    t = int(np.argmax(e))
    assert plan.token(t, 30) == 0
    assert logit_error(plan.logits, ref16.forward(t, 30)) <= 1e-3
    assert plan.verify(bench_tokens(17, m.vocabulary), 0) is None  # more than one chunk


def test_profile_switch():
    """NYA_CUDA_PROFILE=1 (the reference's switch, resident.inc:176-183):
    steps run the per-operation kernels without graphs, still match the
    oracle, and plan_free prints the per-class and per-projection times."""
    code = ("import numpy as np, fyodor_b200 as F, oracle as O\n"
            "from tests.patterns import SMALL_MODELS\n"
            "name, cfg, tokens = SMALL_MODELS[0]\n"
            "m=F.SynthModel(**cfg)\n"
            "pr=F.Provider()\n"
            "p=pr.plan(m,32)\n"
            "ref=O.Session(m.ptr,32,m.vocabulary,kv_f16=True)\n"
            "assert p.prefill(np.array(tokens[:5],np.uint32),0)==0\n"
            "for i,t in enumerate(tokens[:5]): e=ref.forward(t,i,logits=i==4)\n"
            "err=[float(np.max(np.abs(p.logits-e))/(1+np.max(np.abs(e))))]\n"
            "for i,t in enumerate(tokens[5:9]):\n"
            "    assert p.token(t,5+i)==0\n"
            "    e=ref.forward(t,5+i); err.append(float(np.max(np.abs(p.logits-e))/(1+np.max(np.abs(e)))))\n"
            "st=p.stats()\n"
            "print('ERR',max(err),'CAPTURES',st['graph_captures'])\n"
            "p.close()\n")
    r = _env_run(code, NYA_CUDA_PROFILE=1)
    assert r.returncode == 0, r.stderr
    line = [x for x in r.stdout.splitlines() if x.startswith("ERR")][0].split()
    assert float(line[1]) <= 1e-3 and line[3] == "0"  # oracle parity; no graph was captured
    prof = [x for x in r.stderr.splitlines() if x.startswith("fyodor_b200 profile:")]
    assert prof and "steps=4" in prof[0], r.stderr
    vals = dict(kv.split("=") for kv in prof[0].split("milliseconds:")[1].split("(")[0].split())
    assert float(vals["matrix"]) > 0 and float(vals["attention"]) > 0 and float(vals["prefill_chunks"]) > 0
    shapes = [x for x in r.stderr.splitlines() if x.startswith("fyodor_b200 matrix profile:")]
    assert len(shapes) == 5 and all("calls=" in x for x in shapes), r.stderr
