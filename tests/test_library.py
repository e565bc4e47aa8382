"""The C-ABI library loads, exports every declared symbol and carries the
engine's vtable identity (CUDA/cuda.c:457-462) - no GPU needed."""
import ctypes as C
import os
import re
import subprocess

import fyodor_b200 as F
from tests.conftest import ROOT


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "fyodor_b200.h")).read()
    return sorted(set(re.findall(r"\b((?:nya_cuda_backend|fyb_[a-z_0-9]+))\s*\(", text)))


def test_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", F.LIB_PATH], check=True, capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (\S+)", out))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing
    assert set(F.EXPORTS) <= exported


def test_vtable_identity():
    api = F.api()
    assert api.name == b"cuda"
    assert api.type == 1  # NYA_BACKEND_CUDA
    assert api.capabilities == (1 | 2 | 4 | 8)
    for field in ("create", "destroy", "active", "matvec", "plan_create", "plan_free", "plan_token",
                  "plan_prefill", "plan_stats", "matmul", "plan_read_kv"):
        assert C.cast(getattr(api, field), C.c_void_p).value
    assert not api.attention_f32 and not api.context_stats  # NULL, as in the reference


def test_synth_model_layout():
    m = F.SynthModel(layers=2, embedding=512, heads=4, kv_heads=2, feed_forward=768, vocabulary=300, context=16)
    t = m.tensor(3 + 1)  # blk.0.attn_q.weight
    assert t.name == b"blk.0.attn_q.weight" and t.type == F.Q4_K
    assert (t.dimensions[0], t.dimensions[1]) == (512, 512)
    assert t.data_size == 512 * 2 * 144
    emb = m.tensor(0)
    assert emb.name == b"token_embd.weight" and emb.dimensions[1] == 300
    m2 = F.SynthModel(layers=2, embedding=512, heads=4, kv_heads=2, feed_forward=768, vocabulary=300, context=16)
    assert (m.tensor_bytes(4) == m2.tensor_bytes(4)).all()  # seeded and deterministic


def test_provider_declines_without_device():
    if F.lib.fyb_device_count() > 0:
        return
    assert not F.api().create()


def _shared_model_worker(path, out):
    import numpy as np

    import fyodor_b200 as F
    m = F.SynthModel(layers=2, embedding=512, heads=4, kv_heads=2, feed_forward=1024, vocabulary=1024, context=64,
                     seed=9, path=path)
    np.save(out, np.concatenate([m.tensor_bytes(i) for i in (0, 4, 10)]))
    m.close()


def test_shared_file_model(tmp_path):
    """A model created with `path` lives in one shared file: the first
    process fills it, the others wait for it and map it; every process sees
    the bytes the private-memory generator makes."""
    import multiprocessing as mp

    import numpy as np
    path = str(tmp_path / "model.bin")
    ctx = mp.get_context("spawn")
    outs = [str(tmp_path / ("w%d.npy" % i)) for i in range(3)]
    procs = [ctx.Process(target=_shared_model_worker, args=(path, o)) for o in outs]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ref = F.SynthModel(layers=2, embedding=512, heads=4, kv_heads=2, feed_forward=1024, vocabulary=1024, context=64,
                       seed=9)
    expect = np.concatenate([ref.tensor_bytes(i) for i in (0, 4, 10)])
    for o in outs:
        assert (np.load(o) == expect).all()
    # a file made for another configuration is not used
    other = F.SynthModel(layers=2, embedding=512, heads=4, kv_heads=2, feed_forward=1024, vocabulary=1024,
                         context=64, seed=10, path=None)
    assert not (other.tensor_bytes(4) == ref.tensor_bytes(4)).all()


def test_batch_and_verify_reject_bad_arguments():
    """The batched-decode and draft-verification entry points validate their
    arguments before touching a device: a missing plan or batch is refused."""
    import numpy as np
    tok = np.zeros(16, np.uint32)
    out = np.zeros(16, np.float32)
    p = C.c_void_p(tok.ctypes.data)
    assert not F.lib.fyb_batch_create(None, 4)
    assert F.lib.fyb_batch_step(None, p, p, None, None) == -1
    assert F.lib.fyb_batch_decode_greedy(None, p, p, 4, p) == -1
    assert F.lib.fyb_batch_time_greedy(None, p, p, 4) < 0
    assert F.lib.fyb_batch_launches_per_step(None) == 0
    F.lib.fyb_batch_free(None)  # a no-op
    assert F.lib.fyb_plan_verify(None, p, 8, 0, C.c_void_p(out.ctypes.data)) == -1
