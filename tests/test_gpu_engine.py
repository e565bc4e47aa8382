"""The provider as a drop-in: the Fyodor engine (compiled from its sources by
oracle/Makefile with NYA_ENABLE_CUDA) loads libfyodor_b200.so through its own
compute.c and runs its own test programs and a resident session on it."""
import os
import subprocess

import numpy as np
import pytest

import fyodor_b200 as F
import oracle as O
from tests.conftest import ROOT

pytestmark = pytest.mark.gpu
REF = os.path.join(ROOT, "oracle", "_ref")


def run_ref_test(name, *args):
    exe = os.path.join(REF, name)
    if not os.path.exists(exe):
        pytest.fail("%s was not built (make -C oracle)" % exe)
    env = dict(os.environ, NYA_COMPUTE="cuda")
    return subprocess.run([exe, *args], env=env, capture_output=True, text=True, timeout=600)


def test_reference_quant_kernels_on_provider():
    r = run_ref_test("test_quant_kernels")
    assert r.returncode == 0, r.stderr


def test_reference_quant_kernels_long_columns():
    env_r = subprocess.run([os.path.join(REF, "test_quant_kernels")], capture_output=True, text=True, timeout=600,
                           env=dict(os.environ, NYA_COMPUTE="cuda", NYA_TEST_NATIVE_LONG="1"))
    assert env_r.returncode == 0, env_r.stderr


def test_reference_compute_on_provider():
    r = run_ref_test("test_compute", "--cuda")
    assert r.returncode == 0, r.stderr + r.stdout


def test_engine_resident_session_on_provider():
    """nya_llm_session with compute = the provider runs 'resident' and matches
    the fp16-KV oracle within 1e-3 of the logit scale."""
    import ctypes as C
    lib = C.CDLL(os.path.join(REF, "libnya_ref_cuda.so"))
    lib.nya_compute_create_for.restype = C.c_void_p
    lib.nya_compute_create_for.argtypes = [C.c_char_p]
    lib.nya_compute_name.restype = C.c_char_p
    lib.nya_compute_name.argtypes = [C.c_void_p]
    lib.nya_llm_session_create.restype = C.c_void_p
    lib.nya_llm_session_create.argtypes = [C.c_void_p, C.c_size_t, C.c_char_p, C.c_size_t]
    lib.nya_llm_session_run.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
    lib.nya_llm_session_logits.restype = C.POINTER(C.c_float)
    lib.nya_llm_session_logits.argtypes = [C.c_void_p]
    lib.nya_llm_session_execution.restype = C.c_char_p
    lib.nya_llm_session_execution.argtypes = [C.c_void_p]
    lib.nya_llm_session_free.argtypes = [C.c_void_p]
    lib.nya_compute_free.argtypes = [C.c_void_p]
    m = F.SynthModel(layers=2, embedding=512, heads=4, kv_heads=2, feed_forward=768, vocabulary=512, context=32,
                     matrix_type=F.Q6_K, seed=21)
    comp = lib.nya_compute_create_for(b"cuda")
    assert comp and lib.nya_compute_name(comp) == b"cuda"
    C.c_void_p.from_address(m.ptr).value = comp
    err = C.create_string_buffer(256)
    s = lib.nya_llm_session_create(C.c_void_p(m.ptr), 16, err, 256)
    assert s, err.value
    assert lib.nya_llm_session_execution(s) == b"resident"
    ref16 = O.Session(m.ptr, 16, m.vocabulary, kv_f16=True)
    toks = np.array([3, 100, 7, 400, 9], np.uint32)
    for i, t in enumerate(toks):
        one = np.array([t], np.uint32)
        assert lib.nya_llm_session_run(s, C.c_void_p(one.ctypes.data), 1, 1) == 0
        got = np.ctypeslib.as_array(lib.nya_llm_session_logits(s), shape=(m.vocabulary,)).copy()
        e = ref16.forward(int(t), i)
        assert float(np.max(np.abs(got - e)) / (1 + np.max(np.abs(e)))) <= 1e-3
        assert np.argmax(got) == np.argmax(e)
    assert lib.nya_llm_session_execution(s) == b"resident"
    lib.nya_llm_session_free(s)
    lib.nya_compute_free(comp)
    C.c_void_p.from_address(m.ptr).value = None
