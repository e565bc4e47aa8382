"""fyodor_b200 - Python mirror of the Fyodor provider interface for B200.

The product is the C-ABI library ``libfyodor_b200.so`` next to this file
(built by ``fyodor_b200.build``). This module binds it with ctypes and
exposes the same operations the engine reaches through its compute layer
(backend/include/compute.h): typed matvec/matmul on a provider context,
resident plans (create, token, prefill, stats, KV snapshot), plus the
device-level extensions declared in include/fyodor_b200.h.

There is no CPU fallback: if the library is missing, importing the module
raises; if the provider declines (no B200), ``Provider()`` raises.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("FYB_LIBRARY") or os.path.join(HERE, "libfyodor_b200.so")  # override: another build

# GGML storage ids (backend/core/llm_internal.h:11-19)
F32, F16, Q4_0, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 2, 8, 12, 14, 30
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}


def row_bytes(type_id, cols):
    vals, nbytes = BLOCK[type_id]
    return cols // vals * nbytes


class ComputeStats(C.Structure):
    """nya_compute_stats (backend/include/compute.h:13-22)."""
    _fields_ = [("weights_bytes", C.c_size_t), ("kv_bytes", C.c_size_t), ("scratch_bytes", C.c_size_t),
                ("prefill_batch", C.c_size_t), ("external_matmul_bytes", C.c_size_t),
                ("kernel_launches", C.c_ulonglong), ("uploads", C.c_ulonglong), ("downloads", C.c_ulonglong),
                ("synchronizations", C.c_ulonglong), ("external_matmul_calls", C.c_ulonglong),
                ("graph_captures", C.c_ulonglong), ("graph_replays", C.c_ulonglong),
                ("external_matmul_kind", C.c_uint), ("cutlass_matmul_calls", C.c_ulonglong),
                ("tiled_attention_calls", C.c_ulonglong)]

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


_P = C.c_void_p
_CREATE = C.CFUNCTYPE(_P)
_DESTROY = C.CFUNCTYPE(None, _P)
_ACTIVE = C.CFUNCTYPE(C.c_int, _P)
_MATVEC = C.CFUNCTYPE(C.c_int, _P, _P, C.c_size_t, C.c_size_t, C.c_uint, _P, _P)
_PLAN_CREATE = C.CFUNCTYPE(_P, _P, _P, C.c_size_t)
_PLAN_FREE = C.CFUNCTYPE(None, _P)
_PLAN_TOKEN = C.CFUNCTYPE(C.c_int, _P, C.c_uint32, C.c_size_t, C.c_int, _P)
_PLAN_PREFILL = C.CFUNCTYPE(C.c_int, _P, _P, C.c_size_t, C.c_size_t, _P)
_PLAN_STATS = C.CFUNCTYPE(None, _P, C.POINTER(ComputeStats))
_MATMUL = C.CFUNCTYPE(C.c_int, _P, _P, C.c_size_t, C.c_size_t, C.c_uint, _P, _P, C.c_size_t)
_ATTN = C.CFUNCTYPE(C.c_int, _P, _P)
_READ_KV = C.CFUNCTYPE(C.c_int, _P, C.c_size_t, C.c_size_t, C.c_size_t, _P, _P, C.c_size_t)


class BackendInterface(C.Structure):
    """nya_backend_interface (backend/include/compute_backend.h:12-29)."""
    _fields_ = [("type", C.c_int), ("name", C.c_char_p), ("capabilities", C.c_uint),
                ("create", _CREATE), ("destroy", _DESTROY), ("active", _ACTIVE), ("matvec", _MATVEC),
                ("plan_create", _PLAN_CREATE), ("plan_free", _PLAN_FREE), ("plan_token", _PLAN_TOKEN),
                ("plan_prefill", _PLAN_PREFILL), ("plan_stats", _PLAN_STATS), ("matmul", _MATMUL),
                ("attention_f32", _P), ("plan_read_kv", _READ_KV), ("context_stats", _P)]


class Tensor(C.Structure):
    """nya_llm_tensor (backend/core/llm_internal.h:22-31)."""
    _fields_ = [("name", C.c_char * 128), ("type", C.c_uint32), ("dimension_count", C.c_uint32),
                ("dimensions", C.c_uint64 * 4), ("relative_offset", C.c_uint64), ("data", C.POINTER(C.c_ubyte)),
                ("data_size", C.c_size_t), ("bound", C.c_int)]


class SynthConfig(C.Structure):
    """fyb_synth_config (include/fyodor_b200.h)."""
    _fields_ = [("layers", C.c_uint32), ("embedding", C.c_uint32), ("heads", C.c_uint32),
                ("kv_heads", C.c_uint32), ("feed_forward", C.c_uint32), ("vocabulary", C.c_uint32),
                ("context", C.c_uint32), ("matrix_type", C.c_uint32), ("embed_type", C.c_uint32),
                ("output_type", C.c_uint32), ("rope_base", C.c_float), ("epsilon", C.c_float),
                ("seed", C.c_uint64), ("norm_mode", C.c_int), ("threads", C.c_int), ("centered", C.c_int),
                ("path", C.c_char_p)]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError("libfyodor_b200.so is not built; run `python -m fyodor_b200.build`")
    lib = C.CDLL(LIB_PATH)
    lib.nya_cuda_backend.restype = C.POINTER(BackendInterface)
    lib.fyb_version.restype = C.c_char_p
    lib.fyb_device_count.restype = C.c_int
    lib.fyb_dequantize.argtypes = [_P, C.c_size_t, C.c_uint, _P, _P]
    lib.fyb_quant_matmul_workspace.restype = C.c_size_t
    lib.fyb_quant_matmul_workspace.argtypes = [C.c_size_t, C.c_size_t, C.c_uint, C.c_size_t]
    lib.fyb_quant_matmul.argtypes = [_P, C.c_size_t, C.c_size_t, C.c_uint, _P, _P, C.c_size_t, _P, C.c_size_t, _P]
    lib.fyb_quant_repack.argtypes = [_P, C.c_size_t, C.c_size_t, C.c_uint, _P, C.c_size_t, _P]
    lib.fyb_quant_matmul_prepared.argtypes = [C.c_size_t, C.c_size_t, C.c_uint, _P, _P, C.c_size_t, _P,
                                              C.c_size_t, _P]
    lib.fyb_attention_workspace.restype = C.c_size_t
    lib.fyb_attention_workspace.argtypes = [C.c_uint] * 5
    lib.fyb_attention_decode.argtypes = [_P, _P, _P, C.c_size_t, _P, C.c_uint, C.c_uint, C.c_uint, C.c_uint,
                                         C.c_uint, C.c_float, _P, C.c_uint, _P, C.c_size_t, _P]
    lib.fyb_attention_verify.argtypes = [_P, _P, _P, C.c_size_t, _P, C.c_uint, C.c_uint, C.c_uint, C.c_uint,
                                         C.c_uint, C.c_uint, C.c_float, _P, C.c_uint, _P, C.c_size_t, _P]
    lib.fyb_attention_decode_static.argtypes = [_P, _P, _P, C.c_size_t, _P, C.c_uint, C.c_uint, C.c_uint, C.c_uint,
                                                C.c_uint, C.c_float, _P, C.c_uint, _P]
    lib.fyb_plan_tp_info.argtypes = [_P, _P, _P]
    lib.fyb_plan_tp_handle.argtypes = [_P, _P, C.c_size_t]
    lib.fyb_plan_tp_connect.argtypes = [_P, _P, C.c_size_t]
    lib.fyb_plan_tp_disconnect.argtypes = [_P]
    lib.fyb_plan_tp_connect_local.argtypes = [_P, C.POINTER(C.c_void_p), C.c_size_t]
    lib.fyb_plan_error.argtypes = [_P]
    lib.fyb_plan_trace.restype = C.c_long
    lib.fyb_plan_trace.argtypes = [_P, C.c_uint32, C.c_size_t, _P, C.c_size_t, _P, _P, C.c_size_t]
    lib.fyb_plan_decode_greedy.argtypes = [_P, C.c_uint32, C.c_size_t, C.c_size_t, _P]
    lib.fyb_plan_verify.argtypes = [_P, _P, C.c_size_t, C.c_size_t, _P]
    lib.fyb_plan_time_greedy.restype = C.c_double
    lib.fyb_plan_time_greedy.argtypes = [_P, C.c_uint32, C.c_size_t, C.c_size_t]
    lib.fyb_plan_launches_per_token.restype = C.c_ulonglong
    lib.fyb_plan_launches_per_token.argtypes = [_P]
    lib.fyb_plan_decode_form.restype = C.c_int
    lib.fyb_plan_decode_form.argtypes = [_P]
    lib.fyb_plan_profile.argtypes = [_P, C.c_uint32, C.c_size_t, C.c_size_t, _P]
    lib.fyb_plan_time_projection.restype = C.c_double
    lib.fyb_plan_time_projection.argtypes = [_P, C.c_uint, C.c_uint, C.c_uint, C.POINTER(C.c_size_t)]
    lib.fyb_batch_create.restype = _P
    lib.fyb_batch_create.argtypes = [_P, C.c_uint]
    lib.fyb_batch_free.argtypes = [_P]
    lib.fyb_batch_step.argtypes = [_P, _P, _P, _P, _P]
    lib.fyb_batch_decode_greedy.argtypes = [_P, _P, _P, C.c_size_t, _P]
    lib.fyb_batch_time_greedy.restype = C.c_double
    lib.fyb_batch_time_greedy.argtypes = [_P, _P, _P, C.c_size_t]
    lib.fyb_batch_launches_per_step.restype = C.c_ulonglong
    lib.fyb_batch_launches_per_step.argtypes = [_P]
    lib.fyb_synth_create.restype = _P
    lib.fyb_synth_create.argtypes = [C.POINTER(SynthConfig)]
    lib.fyb_synth_free.argtypes = [_P]
    lib.fyb_synth_fill.argtypes = [_P, C.c_size_t, C.c_size_t, C.c_uint32, C.c_uint64, C.c_uint64]
    return lib


lib = _load()

# exported names declared in include/fyodor_b200.h
EXPORTS = ["nya_cuda_backend", "fyb_version", "fyb_device_count", "fyb_dequantize", "fyb_quant_matmul_workspace",
           "fyb_quant_matmul", "fyb_quant_repack", "fyb_quant_matmul_prepared", "fyb_attention_workspace",
           "fyb_attention_decode", "fyb_attention_verify",
           "fyb_attention_decode_static", "fyb_plan_decode_greedy", "fyb_plan_verify",
           "fyb_plan_time_greedy", "fyb_plan_launches_per_token", "fyb_plan_decode_form", "fyb_plan_profile", "fyb_plan_trace",
           "fyb_plan_tp_info", "fyb_plan_tp_handle", "fyb_plan_tp_connect", "fyb_plan_tp_disconnect",
           "fyb_plan_tp_connect_local", "fyb_plan_error", "fyb_plan_time_projection",
           "fyb_batch_create", "fyb_batch_free", "fyb_batch_step", "fyb_batch_decode_greedy", "fyb_batch_time_greedy",
           "fyb_batch_launches_per_step",
           "fyb_synth_create",
           "fyb_synth_free", "fyb_synth_fill"]


def _ptr(a):
    return C.c_void_p(a.ctypes.data) if a is not None else None


def api():
    return lib.nya_cuda_backend().contents


# ---------------------------------------------------------------- models
class SynthModel:
    """A seeded random model in the engine's binding layout (fyb_synth_create)."""

    def __init__(self, layers=2, embedding=512, heads=4, kv_heads=2, feed_forward=1024, vocabulary=1024,
                 context=512, matrix_type=Q4_K, embed_type=Q6_K, output_type=Q6_K, rope_base=500000.0,
                 epsilon=1e-5, seed=1234, norm_mode=2, threads=0, centered=0, path=None):
        cfg = SynthConfig(layers, embedding, heads, kv_heads, feed_forward, vocabulary, context, matrix_type,
                          embed_type, output_type, rope_base, epsilon, seed, norm_mode, threads, centered,
                          path.encode() if path else None)
        self.config = cfg
        self.ptr = lib.fyb_synth_create(C.byref(cfg))
        if not self.ptr:
            raise ValueError("invalid synthetic model configuration")
        self.vocabulary = vocabulary
        self.embedding = embedding
        self.layers = layers
        self.kv_dim = embedding // heads * kv_heads
        self.head_dim = embedding // heads
        self.heads, self.kv_heads = heads, kv_heads

    def tensor(self, index):
        """The index-th nya_llm_tensor (0 token_embd, 1 output_norm, 2 output, then 9 per layer)."""
        # nya_llm_context.tensors is at the offset recorded in the ABI golden file (80)
        tensors = C.cast(C.c_void_p.from_address(self.ptr + 80).value, C.POINTER(Tensor))
        return tensors[index]

    def tensor_bytes(self, index):
        t = self.tensor(index)
        return np.ctypeslib.as_array(t.data, shape=(t.data_size,))

    def close(self):
        if self.ptr:
            lib.fyb_synth_free(self.ptr)
            self.ptr = None

    def __del__(self):
        self.close()


# ---------------------------------------------------------------- provider
IPC_HANDLE_BYTES = 64  # FYB_IPC_HANDLE_BYTES


def tp_exchange(handle, group=None):
    """Gather every rank's exchange-region handle in rank order through a
    torch.distributed group (any backend): the host side of connecting a
    tensor-parallel plan."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, bytes(handle), group=group)
    if any(h is None or len(h) != IPC_HANDLE_BYTES for h in out):
        raise ValueError("a rank has no exchange-region handle")
    return out


def tp_connect_all(plan, group=None):
    """Connect one rank's shard plan with every other rank's, or none of them.

    Every rank calls this with its plan (None when its plan_create declined).
    Returns True when all ranks opened all exchange regions. When any rank
    has no plan or no handle, no rank connects; when any rank fails to open
    the regions, the ranks that succeeded disconnect again. In both cases
    every rank returns False and its plan declines its steps (-1) without
    launching anything that would wait for the failed rank."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    handle = plan.tp_handle() if plan is not None else None
    handles = [None] * world
    dist.all_gather_object(handles, bytes(handle) if handle is not None else None, group=group)
    if any(h is None or len(h) != IPC_HANDLE_BYTES for h in handles):
        return False
    ok = plan.tp_connect(handles) == 0
    oks = [None] * world
    dist.all_gather_object(oks, ok, group=group)
    if not all(oks):
        if ok:
            plan.tp_disconnect()
        return False
    return True


class Provider:
    """A provider context: what nya_compute_create_for("cuda") owns.

    Plans must be freed before their context (backend/include/compute.h:6-8);
    close() frees any plan still alive first."""

    def __init__(self):
        import weakref
        self.api = api()
        self.state = self.api.create()
        if not self.state:
            raise RuntimeError("the B200 provider declined (no sm_100 device visible)")
        self._plans = weakref.WeakSet()

    def active(self):
        return bool(self.api.active(self.state))

    def matvec(self, weights, rows, cols, type_id, x):
        y = np.empty(rows, np.float32)
        r = self.api.matvec(self.state, _ptr(weights), rows, cols, type_id, _ptr(x), _ptr(y))
        return y if r == 0 else None

    def matmul(self, weights, rows, cols, type_id, x, batch):
        y = np.empty((batch, rows), np.float32)
        r = self.api.matmul(self.state, _ptr(weights), rows, cols, type_id, _ptr(x), _ptr(y), batch)
        return y if r == 0 else None

    def plan(self, model, capacity):
        p = self.api.plan_create(self.state, C.c_void_p(model.ptr), capacity)
        if not p:
            return None
        plan = Plan(self, p, model)
        self._plans.add(plan)
        return plan

    def close(self):
        if self.state:
            for plan in list(self._plans):
                plan.close()
            self.api.destroy(self.state)
            self.state = None

    def __del__(self):
        self.close()


class Batch:
    """B sequences (1..16) of one plan's model decoded together (fyb_batch_*):
    each sequence has its own KV cache and position; every projection reads
    each weight once per step for all of them. The plan must outlive it."""

    def __init__(self, plan, batch):
        self.plan, self.B = plan, batch
        self.V = plan.model.vocabulary
        self.ptr = lib.fyb_batch_create(C.c_void_p(plan.ptr), batch)
        if not self.ptr:
            raise ValueError("batch of %d declined" % batch)

    def _req(self, tokens, positions):
        t = np.ascontiguousarray(tokens, np.uint32)
        p = np.ascontiguousarray(positions, np.uint32)
        assert t.shape == (self.B,) and p.shape == (self.B,)
        return t, p

    def step(self, tokens, positions, logits=True):
        """One step: (logits [B][V] or None, argmax [B])."""
        t, p = self._req(tokens, positions)
        lg = np.empty((self.B, self.V), np.float32) if logits else None
        am = np.empty(self.B, np.uint32)
        r = lib.fyb_batch_step(C.c_void_p(self.ptr), _ptr(t), _ptr(p), _ptr(lg), _ptr(am))
        if r:
            raise RuntimeError("fyb_batch_step failed (%d)" % r)
        return lg, am

    def decode_greedy(self, tokens, positions, steps):
        """Greedy tokens [steps][B] decoded on the device."""
        t, p = self._req(tokens, positions)
        out = np.empty((steps, self.B), np.uint32)
        r = lib.fyb_batch_decode_greedy(C.c_void_p(self.ptr), _ptr(t), _ptr(p), steps, _ptr(out))
        if r:
            raise RuntimeError("fyb_batch_decode_greedy failed (%d)" % r)
        return out

    def time_greedy(self, tokens, positions, steps):
        """Milliseconds per greedy step (device events)."""
        t, p = self._req(tokens, positions)
        return lib.fyb_batch_time_greedy(C.c_void_p(self.ptr), _ptr(t), _ptr(p), steps)

    def launches_per_step(self):
        return lib.fyb_batch_launches_per_step(C.c_void_p(self.ptr))

    def close(self):
        if self.ptr:
            lib.fyb_batch_free(C.c_void_p(self.ptr))
            self.ptr = None

    def __del__(self):
        self.close()


class Plan:
    """A resident plan (nya_compute_plan)."""

    def __init__(self, provider, ptr, model):
        self.provider, self.ptr, self.model = provider, ptr, model
        self.api = provider.api
        self.logits = np.empty(model.vocabulary, np.float32)

    def token(self, token, position, logits=True):
        out = self.logits if logits else None
        r = self.api.plan_token(self.ptr, token, position, 1 if logits else 0, _ptr(out))
        return r

    def prefill(self, tokens, position):
        tokens = np.ascontiguousarray(tokens, np.uint32)
        return self.api.plan_prefill(self.ptr, _ptr(tokens), len(tokens), position, _ptr(self.logits))

    def stats(self):
        s = ComputeStats()
        self.api.plan_stats(self.ptr, C.byref(s))
        return s.as_dict()

    def read_kv(self, layer, position, count):
        width = self.model.kv_dim
        k = np.empty((count, width), np.float32)
        v = np.empty((count, width), np.float32)
        r = self.api.plan_read_kv(self.ptr, layer, position, count, _ptr(k), _ptr(v), count * width)
        return (k, v) if r == 0 else None

    def verify(self, tokens, position):
        """Logits [k][V] of k draft tokens at positions position.. (one pass)."""
        t = np.ascontiguousarray(tokens, np.uint32)
        out = np.empty((len(t), self.model.vocabulary), np.float32)
        r = lib.fyb_plan_verify(C.c_void_p(self.ptr), _ptr(t), len(t), position, _ptr(out))
        return out if r == 0 else None

    def decode_greedy(self, token, position, steps):
        out = np.empty(steps, np.uint32)
        r = lib.fyb_plan_decode_greedy(C.c_void_p(self.ptr), token, position, steps, _ptr(out))
        return out if r == 0 else None

    def time_greedy(self, token, position, steps):
        return lib.fyb_plan_time_greedy(C.c_void_p(self.ptr), token, position, steps)

    def launches_per_token(self):
        return lib.fyb_plan_launches_per_token(C.c_void_p(self.ptr))

    def decode_form(self):
        """0 per-operation kernels, 1 the persistent decode kernel."""
        return lib.fyb_plan_decode_form(C.c_void_p(self.ptr))

    def tp_info(self):
        """(rank, size) of the plan's tensor-parallel shard."""
        r, n = C.c_uint(0), C.c_uint(0)
        lib.fyb_plan_tp_info(C.c_void_p(self.ptr), C.byref(r), C.byref(n))
        return r.value, n.value

    def tp_handle(self):
        """This rank's exchange-region handle (bytes), or None."""
        buf = C.create_string_buffer(IPC_HANDLE_BYTES)
        if lib.fyb_plan_tp_handle(C.c_void_p(self.ptr), buf, IPC_HANDLE_BYTES) != 0:
            return None
        return buf.raw

    def tp_connect(self, handles):
        """Open the other ranks' regions; handles: one bytes object per rank, in rank order."""
        blob = b"".join(handles)
        return lib.fyb_plan_tp_connect(C.c_void_p(self.ptr), C.c_char_p(blob), len(handles))

    def tp_disconnect(self):
        """Decline every later step without launching (another rank failed)."""
        return lib.fyb_plan_tp_disconnect(C.c_void_p(self.ptr))

    def tp_connect_local(self, plans):
        """Connect this plan to the other shard plans of this process
        (plans: every rank's Plan, in rank order)."""
        arr = (C.c_void_p * len(plans))(*[q.ptr for q in plans])
        return lib.fyb_plan_tp_connect_local(C.c_void_p(self.ptr), arr, len(plans))

    def error(self):
        """The device error word: 0 none, 1 a bounded wait ran out, 2 non-finite
        logits, 4 an index out of range."""
        return lib.fyb_plan_error(C.c_void_p(self.ptr))

    def trace(self, token, position, detail=False):
        """Per-CTA trace points of one persistent decode step: array
        [points][grid] of globaltimer nanoseconds (start, then per layer the
        ends of QKV, attention, O, gate/up and down, the end of the logits,
        exit), or None. With detail=True, a pair (that array, per-warp
        records of layer layers // 2 [grid][16][32], decode_kernel.cuh)."""
        grid = C.c_uint(0)
        L = self.model.config.layers
        points = 1 + 5 * L + 2
        n = points * 1024
        out = np.zeros(n, np.uint64)
        wn = 1024 * 16 * 32
        wout = np.zeros(wn, np.uint64) if detail else None
        r = lib.fyb_plan_trace(C.c_void_p(self.ptr), token, position, _ptr(out), n, C.byref(grid),
                               _ptr(wout) if detail else None, wn if detail else 0)
        if r < 0:
            return None
        cta = out[: r * grid.value].reshape(r, grid.value)
        if not detail:
            return cta
        return cta, wout[: grid.value * 16 * 32].reshape(grid.value, 16, 32)

    def profile(self, token, position, steps):
        """Per-class milliseconds of one decode step: matrix, attention, other."""
        out = np.zeros(3, np.float64)
        r = lib.fyb_plan_profile(C.c_void_p(self.ptr), token, position, steps, _ptr(out))
        return out if r == 0 else None

    def time_projection(self, layer, which, reps):
        """(ms per launch, algorithmic bytes) of one fused projection kernel."""
        nbytes = C.c_size_t()
        ms = lib.fyb_plan_time_projection(C.c_void_p(self.ptr), layer, which, reps, C.byref(nbytes))
        return ms, nbytes.value

    def close(self):
        if self.ptr:
            self.api.plan_free(self.ptr)
            self.ptr = None

    def __del__(self):
        self.close()
