"""A bounded wait that runs out, on one GPU, with no fault.

Two tensor-parallel shard plans (ranks 0 and 1 of 2) live in this process on
one GPU and are connected through fyb_plan_tp_connect_local. Only rank 0
runs a decode step: its first exchange waits for rank 1's partial
attention-output rows, which nothing writes. Every device wait in the decode
kernel is bounded, so the kernel records ERR_TIMEOUT, raises its abort word,
lets its bulk copies land and returns; plan_token returns -1, the plan stays
failed, and the CUDA context stays usable (a plan without tensor parallelism
then decodes on the same provider). Rank 1's kernel never runs, so no two
kernels on this GPU wait on each other."""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG = dict(layers=2, embedding=2048, heads=16, kv_heads=8, feed_forward=2048, vocabulary=1024, context=32,
           seed=21, norm_mode=2, centered=1)


def test_missing_rank_times_out(monkeypatch):
    import fyodor_b200 as F
    m = F.SynthModel(**CFG)
    provider = F.Provider()
    assert provider.active()
    monkeypatch.setenv("NYA_CUDA_TP_SIZE", "2")
    plans = []
    for r in range(2):
        monkeypatch.setenv("NYA_CUDA_TP_RANK", str(r))
        plans.append(provider.plan(m, 16))
    monkeypatch.delenv("NYA_CUDA_TP_SIZE")
    monkeypatch.delenv("NYA_CUDA_TP_RANK")
    assert all(p is not None for p in plans), "the shard plans were declined"
    rank0 = plans[0]
    assert rank0.tp_info() == (0, 2)
    assert rank0.decode_form() == 1, "the test needs the persistent decode kernel"
    assert rank0.tp_connect_local([plans[1], plans[0]]) == -1  # wrong rank order
    assert rank0.tp_connect_local(plans) == 0
    assert rank0.error() == 0

    t0 = time.time()
    assert rank0.token(7, 0) == -1
    elapsed = time.time() - t0
    assert rank0.error() == 1, "expected ERR_TIMEOUT from the bounded wait"
    assert elapsed < 120
    assert rank0.token(7, 0) == -1  # a failed plan declines without launching

    for p in plans:
        p.close()
    # the context is still usable
    plain = provider.plan(m, 16)
    assert plain is not None
    assert plain.token(7, 0) == 0
    assert plain.error() == 0
    assert np.isfinite(plain.logits).all()
    plain.close()
    provider.close()
    m.close()
