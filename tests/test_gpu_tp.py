"""Tensor parallelism over 2, 4 and 8 GPUs: one process per GPU, each holding
one shard of every layer (1/N of the heads and FFN rows, 1/N of the
vocabulary), run the same decode steps; the persistent kernel exchanges the partial
attention-output and down rows over NVLink. All ranks must return the same
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

WORLDS = [2, 4, 8]
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
        assert F.tp_connect_all(plan)
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


def _run(world, cfg, tokens, greedy_steps, tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    mp.spawn(_rank_main, args=(world, _free_port(), cfg, tokens, greedy_steps, str(tmp_path)), nprocs=world,
             join=True)
    return [np.load(os.path.join(str(tmp_path), "rank%d.npz" % r)) for r in range(world)]


def _check(world, cfg, tokens, greedy_steps, tmp_path):
    import fyodor_b200 as F
    import oracle as O
    from tests.test_gpu_plan import logit_error
    res = _run(world, cfg, tokens, greedy_steps, tmp_path)
    for r in range(1, world):
        assert (res[r]["logits"] == res[0]["logits"]).all()
        assert (res[r]["greedy"] == res[0]["greedy"]).all()
    m = F.SynthModel(**cfg)
    O.set_threads(os.cpu_count() or 1)
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
    O.set_threads(1)
    assert list(res[0]["greedy"]) == expected
    m.close()


# a small model every world size shards: 16/8 heads of 128, FFN 2048, vocabulary 1024
SMALL_TP = dict(layers=2, embedding=2048, heads=16, kv_heads=8, feed_forward=2048, vocabulary=1024, context=96,
                seed=21, norm_mode=2, centered=1)


@pytest.mark.parametrize("world", WORLDS)
def test_tp_small_model(world, tmp_path):
    from tests.patterns import bench_tokens
    _check(world, SMALL_TP, [int(t) for t in bench_tokens(12, 1024)], 64, tmp_path)


@pytest.mark.parametrize("world", WORLDS)
def test_tp_8b_layer_shapes(world, tmp_path):
    """Two layers at the 8B geometry, sharded N ways (32/N query and 8/N KV
    heads, 14336/N FFN rows and 128256/N vocabulary rows per rank)."""
    from tests.patterns import bench_tokens
    cfg = dict(layers=2, embedding=4096, heads=32, kv_heads=8, feed_forward=14336, vocabulary=128256, context=32,
               seed=99, norm_mode=2, centered=1)
    _check(world, cfg, [int(t) for t in bench_tokens(5, 128256)], 8, tmp_path)


@pytest.mark.parametrize("world", [2, 8])
def test_tp_70b_layer_shapes(world, tmp_path):
    """Two layers at the 70B geometry (d 8192, 64/8 heads of 128, FFN 28672,
    vocabulary 128256; Q4_K projections and output head, Q6_K embedding)."""
    from tests.patterns import bench_tokens
    import fyodor_b200 as F
    cfg = dict(layers=2, embedding=8192, heads=64, kv_heads=8, feed_forward=28672, vocabulary=128256, context=32,
               matrix_type=F.Q4_K, embed_type=F.Q6_K, output_type=F.Q4_K, seed=70, norm_mode=2, centered=1)
    _check(world, cfg, [int(t) for t in bench_tokens(5, 128256)], 8, tmp_path)
