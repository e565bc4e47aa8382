"""Generate the golden fixtures in tests/golden/ from the compiled Fyodor engine.

Run where oracle/_ref/libnya_ref.so exists (it is built from the reference
sources by oracle/Makefile):

    make -C oracle && python tests/golden/make_golden.py

Every fixture is produced by the reference engine itself, never by this
repository's code: nya_llm_tensor_value, the scalar nya_llm_matvec and a
scalar nya_llm_session (compute = NULL). Inputs are the reference tests' own
deterministic patterns (test_quant_kernels.c:141-176, test_architectures.c:
232-285) and small seeded synthetic models built by fyb_synth_create.
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle as O  # noqa: E402
import fyodor_b200 as F  # noqa: E402
from tests.patterns import k_quant_blocks, quant_kernel_weights, quant_kernel_inputs, SMALL_MODELS  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def kquant_known():
    """check_k_quants: Q4_K/Q6_K built from logical fields, 4 blocks each."""
    out = {}
    for kind, type_id in ((0, F.Q4_K), (1, F.Q6_K)):
        data, expected = k_quant_blocks(kind)
        out["data_%d" % type_id] = data
        out["expected_%d" % type_id] = expected
        out["ref_values_%d" % type_id] = O.ref_tensor_values(data, type_id, 1024)
        x = np.array([((i % 23) - 11) / 16.0 for i in range(512)], np.float32)
        out["ref_matvec_%d" % type_id] = O.ref_matvec(data, type_id, x, 512, 2)
    np.savez_compressed(os.path.join(OUT, "kquant_known.npz"), **out)


def quant_kernels():
    """test_quant_kernels: 65 rows x 1024 columns of every storage type."""
    out = {}
    for type_id in (F.F32, F.F16, F.BF16, F.Q4_0, F.Q8_0, F.Q4_K, F.Q6_K):
        data = quant_kernel_weights(type_id, 65, 1024)
        out["data_%d" % type_id] = data
        out["values_%d" % type_id] = O.ref_tensor_values(data, type_id, 65 * 1024)
        for p in range(3):
            x = quant_kernel_inputs(1024, p)
            out["y_%d_%d" % (type_id, p)] = O.ref_matvec(data, type_id, x, 1024, 65)
    np.savez_compressed(os.path.join(OUT, "quant_kernels.npz"), **out)


def small_models():
    """Logits of the engine's scalar session on seeded synthetic models."""
    out = {}
    for name, cfg, tokens in SMALL_MODELS:
        m = F.SynthModel(**cfg)
        s = O.RefSession(m.ptr, len(tokens), m.vocabulary)
        logits = []
        for t in tokens:
            s.run([t])
            logits.append(s.logits())
        k, v = s.read_kv(cfg["layers"] - 1, 0, len(tokens), m.kv_dim)
        s.close()
        out[name + "_tokens"] = np.array(tokens, np.uint32)
        out[name + "_logits"] = np.stack(logits)
        out[name + "_k_last"] = k
        out[name + "_v_last"] = v
        m.close()
    np.savez_compressed(os.path.join(OUT, "small_models.npz"), **out)


if __name__ == "__main__":
    if not O.reference_available():
        sys.exit("oracle/_ref/libnya_ref.so missing: run `make -C oracle` first")
    kquant_known()
    quant_kernels()
    small_models()
    print("golden fixtures written to", OUT)
