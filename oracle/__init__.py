"""Parity oracles for the B200 provider - TEST INFRASTRUCTURE ONLY.

Two checkers, both CPU:
  * ``liboracle.so``: this repository's C restatement of the engine's decode
    path (oracle/fyodor_oracle.c), with an optional fp16 KV cache.
  * ``_ref/libnya_ref.so``: the Fyodor engine itself, compiled from the
    reference sources by oracle/Makefile (present where it was built).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this
package. The provider never calls into it.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libnya_ref.so")
_P = C.c_void_p


def _arr(a):
    return C.c_void_p(a.ctypes.data)


def _load_oracle():
    if not os.path.exists(ORACLE_LIB):
        raise ImportError("oracle/liboracle.so is not built; run `make -C oracle oracle`")
    o = C.CDLL(ORACLE_LIB)
    o.orc_half_to_float.restype = C.c_float
    o.orc_half_to_float.argtypes = [C.c_uint16]
    o.orc_float_to_half_bits.restype = C.c_uint16
    o.orc_float_to_half_bits.argtypes = [C.c_float]
    o.orc_round_f16.restype = C.c_float
    o.orc_round_f16.argtypes = [C.c_float]
    o.orc_dequantize.argtypes = [_P, C.c_uint32, C.c_size_t, _P]
    o.orc_matvec.argtypes = [_P, _P, C.c_uint32, _P, C.c_size_t, C.c_size_t]
    o.orc_matvec_threaded.argtypes = [_P, _P, C.c_uint32, _P, C.c_size_t, C.c_size_t]
    o.orc_set_threads.argtypes = [C.c_int]
    o.orc_attention.restype = C.c_int
    o.orc_attention.argtypes = [_P, _P, _P, _P, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t,
                                C.c_float, _P]
    o.orc_session_create.restype = _P
    o.orc_session_create.argtypes = [_P, C.c_size_t, C.c_int]
    o.orc_session_free.argtypes = [_P]
    o.orc_session_forward.restype = C.c_int
    o.orc_session_forward.argtypes = [_P, C.c_uint32, C.c_size_t, C.c_int]
    o.orc_session_logits.restype = C.POINTER(C.c_float)
    o.orc_session_logits.argtypes = [_P]
    o.orc_session_read_kv.argtypes = [_P, C.c_size_t, C.c_size_t, C.c_size_t, _P, _P]
    o.orc_argmax.restype = C.c_int
    o.orc_argmax.argtypes = [_P, C.c_size_t, C.POINTER(C.c_uint32)]
    return o


lib = _load_oracle()


def half_to_float(bits):
    return lib.orc_half_to_float(bits)


def round_f16(x):
    return lib.orc_round_f16(x)


def dequantize(data, type_id, count):
    out = np.empty(count, np.float32)
    data = np.ascontiguousarray(data)
    lib.orc_dequantize(_arr(data), type_id, count, _arr(out))
    return out


def matvec(data, type_id, x, cols, rows):
    """The engine's scalar nya_llm_matvec, same summation order."""
    out = np.empty(rows, np.float32)
    data = np.ascontiguousarray(data)
    x = np.ascontiguousarray(x, np.float32)
    lib.orc_matvec(_arr(out), _arr(data), type_id, _arr(x), cols, rows)
    return out


def set_threads(n):
    """Threads of the oracle's matrix products (sessions and matvec_threaded).
    Each row keeps the engine's summation order, so results do not change."""
    lib.orc_set_threads(int(n))


def matvec_threaded(data, type_id, x, cols, rows):
    """matvec with rows spread over the threads set by set_threads()."""
    out = np.empty(rows, np.float32)
    data = np.ascontiguousarray(data)
    x = np.ascontiguousarray(x, np.float32)
    lib.orc_matvec_threaded(_arr(out), _arr(data), type_id, _arr(x), cols, rows)
    return out


def attention(q, keys, values, heads, kv_heads, hd, length, scale):
    """One token of decode attention over an F32 [length][kv_heads][hd] cache."""
    out = np.empty(heads * hd, np.float32)
    scratch = np.empty(max(length, 1), np.float32)
    q = np.ascontiguousarray(q, np.float32)
    keys = np.ascontiguousarray(keys, np.float32)
    values = np.ascontiguousarray(values, np.float32)
    r = lib.orc_attention(_arr(q), _arr(keys), _arr(values), _arr(out), heads, kv_heads, hd, 0, length - 1,
                          scale, _arr(scratch))
    if r:
        raise ValueError("oracle attention rejected the input")
    return out


def argmax(logits):
    t = C.c_uint32()
    logits = np.ascontiguousarray(logits, np.float32)
    if lib.orc_argmax(_arr(logits), logits.size, C.byref(t)):
        raise ValueError("non-finite logits")
    return t.value


class Session:
    """Restated engine session over a model pointer (nya_llm_context*)."""

    def __init__(self, model_ptr, capacity, vocabulary, kv_f16=False):
        self.ptr = lib.orc_session_create(C.c_void_p(model_ptr), capacity, 1 if kv_f16 else 0)
        if not self.ptr:
            raise ValueError("oracle session rejected the model")
        self.vocabulary = vocabulary

    def forward(self, token, position, logits=True):
        r = lib.orc_session_forward(self.ptr, token, position, 1 if logits else 0)
        if r:
            raise ValueError("oracle forward failed at position %d" % position)
        if logits:
            return np.ctypeslib.as_array(lib.orc_session_logits(self.ptr), shape=(self.vocabulary,)).copy()
        return None

    def read_kv(self, layer, position, count, width):
        k = np.empty((count, width), np.float32)
        v = np.empty((count, width), np.float32)
        lib.orc_session_read_kv(self.ptr, layer, position, count, _arr(k), _arr(v))
        return k, v

    def close(self):
        if self.ptr:
            lib.orc_session_free(self.ptr)
            self.ptr = None

    def __del__(self):
        self.close()


# ---------------------------------------------------------------- reference engine
def reference_available():
    return os.path.exists(REF_LIB)


_ref = None


def ref():
    """The compiled Fyodor engine (CPU providers only)."""
    global _ref
    if _ref is None:
        if not reference_available():
            raise ImportError("oracle/_ref/libnya_ref.so is not built (make -C oracle reference)")
        r = C.CDLL(REF_LIB)
        r.nya_llm_tensor_value.restype = C.c_float
        r.nya_llm_tensor_value.argtypes = [_P, C.c_size_t]
        r.nya_llm_round_f16.restype = C.c_float
        r.nya_llm_round_f16.argtypes = [C.c_float]
        r.nya_llm_matvec.argtypes = [_P, _P, _P, _P, C.c_size_t, C.c_size_t]
        r.nya_llm_session_create.restype = _P
        r.nya_llm_session_create.argtypes = [_P, C.c_size_t, C.c_char_p, C.c_size_t]
        r.nya_llm_session_free.argtypes = [_P]
        r.nya_llm_session_reset.argtypes = [_P]
        r.nya_llm_session_run.restype = C.c_int
        r.nya_llm_session_run.argtypes = [_P, _P, C.c_size_t, C.c_int]
        r.nya_llm_session_logits.restype = C.POINTER(C.c_float)
        r.nya_llm_session_logits.argtypes = [_P]
        r.nya_llm_session_execution.restype = C.c_char_p
        r.nya_llm_session_execution.argtypes = [_P]
        r.nya_llm_session_read_kv.restype = C.c_int
        r.nya_llm_session_read_kv.argtypes = [_P, C.c_size_t, C.c_size_t, C.c_size_t, _P, _P, C.c_size_t]
        r.nya_compute_create_for.restype = _P
        r.nya_compute_create_for.argtypes = [C.c_char_p]
        r.nya_compute_free.argtypes = [_P]
        r.nya_compute_matvec_typed.restype = C.c_int
        r.nya_compute_matvec_typed.argtypes = [_P, _P, C.c_size_t, C.c_size_t, C.c_uint, _P, _P]
        r.nya_compute_matmul_typed.restype = C.c_int
        r.nya_compute_matmul_typed.argtypes = [_P, _P, C.c_size_t, C.c_size_t, C.c_uint, _P, _P, C.c_size_t]
        _ref = r
    return _ref


class TensorView(C.Structure):
    """nya_llm_tensor layout (backend/core/llm_internal.h:22-31) for loose buffers."""
    _fields_ = [("name", C.c_char * 128), ("type", C.c_uint32), ("dimension_count", C.c_uint32),
                ("dimensions", C.c_uint64 * 4), ("relative_offset", C.c_uint64), ("data", C.c_void_p),
                ("data_size", C.c_size_t), ("bound", C.c_int)]


def ref_tensor_values(data, type_id, count):
    """nya_llm_tensor_value over a byte buffer, from the compiled engine."""
    data = np.ascontiguousarray(data)
    t = TensorView()
    t.type = type_id
    t.data = data.ctypes.data
    t.data_size = data.size
    r = ref()
    return np.array([r.nya_llm_tensor_value(C.byref(t), i) for i in range(count)], np.float32)


def ref_matvec(data, type_id, x, cols, rows):
    """nya_llm_matvec(NULL, ...) - the engine's scalar CPU kernel."""
    data = np.ascontiguousarray(data)
    x = np.ascontiguousarray(x, np.float32)
    t = TensorView()
    t.type = type_id
    t.data = data.ctypes.data
    t.data_size = data.size
    out = np.empty(rows, np.float32)
    ref().nya_llm_matvec(None, _arr(out), C.byref(t), _arr(x), cols, rows)
    return out


class RefSession:
    """nya_llm_session of the compiled engine on a model pointer.

    provider=None keeps the scalar reference path (compute = NULL); "cpu"
    attaches the engine's optimized CPU provider (its SIMD kernels and worker
    pool), as fyodor-bench -b cpu does.
    """

    def __init__(self, model_ptr, capacity, vocabulary, provider=None):
        r = ref()
        self.model_ptr = model_ptr
        self.compute = None
        if provider:
            self.compute = r.nya_compute_create_for(provider.encode())
            if not self.compute:
                raise RuntimeError("engine provider %s unavailable" % provider)
        C.c_void_p.from_address(model_ptr).value = self.compute  # nya_llm_context.compute (offset 0)
        err = C.create_string_buffer(512)
        self.ptr = r.nya_llm_session_create(C.c_void_p(model_ptr), capacity, err, 512)
        if not self.ptr:
            raise RuntimeError("engine session failed: %s" % err.value.decode(errors="replace"))
        self.vocabulary = vocabulary

    def run(self, tokens, each=True):
        tokens = np.ascontiguousarray(tokens, np.uint32)
        if ref().nya_llm_session_run(self.ptr, _arr(tokens), tokens.size, 1 if each else 0):
            raise RuntimeError("engine session run failed")

    def logits(self):
        p = ref().nya_llm_session_logits(self.ptr)
        return np.ctypeslib.as_array(p, shape=(self.vocabulary,)).copy()

    def execution(self):
        return ref().nya_llm_session_execution(self.ptr).decode()

    def reset(self):
        ref().nya_llm_session_reset(self.ptr)

    def read_kv(self, layer, position, count, width):
        k = np.empty((count, width), np.float32)
        v = np.empty((count, width), np.float32)
        if ref().nya_llm_session_read_kv(self.ptr, layer, position, count, _arr(k), _arr(v), count * width):
            raise RuntimeError("engine read_kv failed")
        return k, v

    def close(self):
        r = ref()
        if self.ptr:
            r.nya_llm_session_free(self.ptr)
            self.ptr = None
        if self.compute:
            r.nya_compute_free(self.compute)
            self.compute = None
            C.c_void_p.from_address(self.model_ptr).value = None

    def __del__(self):
        self.close()


class RefCompute:
    """The engine's "cpu" compute provider (backend/core/compute.c:85-99 over
    cpu_backend.c's worker pool): matvec / matmul of GGUF weights from host
    memory, for the CPU side of the matvec benchmark configurations."""

    def __init__(self, provider="cpu"):
        self.ptr = ref().nya_compute_create_for(provider.encode())
        if not self.ptr:
            raise RuntimeError("engine provider %s unavailable" % provider)

    def matmul(self, data, rows, cols, type_id, xs, batch):
        """y[batch][rows] = W x for each of the batch rows of xs; None on -1."""
        xs = np.ascontiguousarray(xs, np.float32)
        y = np.empty((batch, rows), np.float32)
        if batch == 1:
            r = ref().nya_compute_matvec_typed(self.ptr, _arr(data), rows, cols, type_id, _arr(xs), _arr(y))
        else:
            r = ref().nya_compute_matmul_typed(self.ptr, _arr(data), rows, cols, type_id, _arr(xs), _arr(y), batch)
        return y if r == 0 else None

    def time(self, data, rows, cols, type_id, xs, batch, seconds=0.5, max_calls=50):
        """Microseconds per call: one warm-up call, then calls until `seconds`
        have passed (at least two)."""
        import time
        assert self.matmul(data, rows, cols, type_id, xs, batch) is not None
        n, t0 = 0, time.perf_counter()
        while n < 2 or (n < max_calls and time.perf_counter() - t0 < seconds):
            self.matmul(data, rows, cols, type_id, xs, batch)
            n += 1
        return (time.perf_counter() - t0) / n * 1e6

    def close(self):
        if self.ptr:
            ref().nya_compute_free(self.ptr)
            self.ptr = None

    def __del__(self):
        self.close()
