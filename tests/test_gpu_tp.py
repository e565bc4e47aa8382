"""Tensor parallelism over two GPUs: two processes, each holding one shard of
every layer (half of the heads and FFN rows, half of the vocabulary), run
the same decode steps; the persistent kernel exchanges the partial
attention-output and down rows over NVLink. Both ranks must return the same
logits (bitwise: every rank adds the partials in rank order), within 1e-3 of
the logit scale of the fp16-KV oracle with the same argmax, and the same
greedy tokens as the oracle over 64 steps.

The ranks meet through a gloo process group on 127.0.0.1 (handle exchange and
barriers only); NVLink SHARP stays off (NCCL_NVLS_ENABLE=0) although no NCCL
collective runs. Every device wait in the kernel is bounded."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WORLD = 2
PREFILL = 3  # tokens taken by plan_prefill before single steps


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, cfg, tokens, greedy_steps, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NYA_CUDA_DEVICE=str(rank),
                      NYA_CUDA_TP_SIZE=str(world), NYA_CUDA_TP_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    import datetime

    import torch.distributed as dist

    import fyodor_b200 as F
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        m = F.SynthModel(**cfg)
        provider = F.Provider()
        capacity = len(tokens) + greedy_steps + 1
        plan = provider.plan(m, capacity)
        assert plan is not None, "the shard plan was declined"
        assert plan.tp_info() == (rank, world)
        assert plan.token(tokens[0], 0) == -1  # not connected yet
        assert plan.tp_connect(F.tp_exchange(plan.tp_handle())) == 0
        # a prefill (steps without logits, then one with) and single steps after it
        logits = []
        assert plan.prefill(tokens[:PREFILL], 0) == 0
        logits.append(plan.logits.copy())
        for i in range(PREFILL, len(tokens)):
            assert plan.token(tokens[i], i) == 0
            logits.append(plan.logits.copy())
        first = int(np.argmax(logits[-1]))
        greedy = plan.decode_greedy(first, len(tokens), greedy_steps)
        assert greedy is not None
        np.savez(os.path.join(out_dir, "rank%d.npz" % rank), logits=np.stack(logits), greedy=np.array(greedy))
        dist.barrier()
        plan.close()
        provider.close()
        m.close()
    finally:
        dist.destroy_process_group()


def _run(cfg, tokens, greedy_steps, tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs %d GPUs" % WORLD)
    mp.spawn(_rank_main, args=(WORLD, _free_port(), cfg, tokens, greedy_steps, str(tmp_path)), nprocs=WORLD,
             join=True)
    return [np.load(os.path.join(str(tmp_path), "rank%d.npz" % r)) for r in range(WORLD)]


def _check(cfg, tokens, greedy_steps, tmp_path):
    import fyodor_b200 as F
    import oracle as O
    from tests.test_gpu_plan import logit_error
    res = _run(cfg, tokens, greedy_steps, tmp_path)
    for r in range(1, WORLD):
        assert (res[r]["logits"] == res[0]["logits"]).all()
        assert (res[r]["greedy"] == res[0]["greedy"]).all()
    m = F.SynthModel(**cfg)
    ref = O.Session(m.ptr, len(tokens) + greedy_steps + 1, m.vocabulary, kv_f16=True)
    for i, t in enumerate(tokens):
        e = ref.forward(t, i)
        if i < PREFILL - 1:
            continue  # prefill steps without logits
        got = res[0]["logits"][i - (PREFILL - 1)]
        assert logit_error(got, e) <= 1e-3, (i, logit_error(got, e))
        assert np.argmax(got) == np.argmax(e)
    t = int(np.argmax(res[0]["logits"][-1]))
    expected = []
    for i in range(greedy_steps):
        t = O.argmax(ref.forward(t, len(tokens) + i))
        expected.append(t)
    assert list(res[0]["greedy"]) == expected
    m.close()


def test_tp2_small_model(tmp_path):
    from tests.patterns import SMALL_MODELS
    name, cfg, tokens = SMALL_MODELS[0]
    _check(dict(cfg, context=96), tokens, 64, tmp_path)


def test_tp2_8b_layer_shapes(tmp_path):
    """Two layers at the 8B geometry, sharded in two (16/4 heads, 7168 FFN rows,
    64128 vocabulary rows per rank)."""
    from tests.patterns import bench_tokens
    cfg = dict(layers=2, embedding=4096, heads=32, kv_heads=8, feed_forward=14336, vocabulary=128256, context=32,
               seed=99, norm_mode=2, centered=1)
    _check(cfg, [int(t) for t in bench_tokens(5, 128256)], 8, tmp_path)
