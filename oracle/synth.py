"""Seeded synthetic models for the CPU arms - TEST INFRASTRUCTURE ONLY.

The same generator as the provider's fyb_synth_create (the source is
fyodor_b200/csrc/synth.cpp), built on its own into oracle/libsynth.so by
oracle/Makefile, so the bench's reference arm and CPU baseline produce the
bench model's exact bytes without loading the provider library. Model
contents are a pure function of the configuration and seed.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
SYNTH_LIB = os.path.join(HERE, "libsynth.so")
F32, F16, Q4_0, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 2, 8, 12, 14, 30


class SynthConfig(C.Structure):
    """fyb_synth_config (include/fyodor_b200.h)."""
    _fields_ = [("layers", C.c_uint32), ("embedding", C.c_uint32), ("heads", C.c_uint32),
                ("kv_heads", C.c_uint32), ("feed_forward", C.c_uint32), ("vocabulary", C.c_uint32),
                ("context", C.c_uint32), ("matrix_type", C.c_uint32), ("embed_type", C.c_uint32),
                ("output_type", C.c_uint32), ("rope_base", C.c_float), ("epsilon", C.c_float),
                ("seed", C.c_uint64), ("norm_mode", C.c_int), ("threads", C.c_int), ("centered", C.c_int),
                ("path", C.c_char_p)]


_lib = None


def library():
    global _lib
    if _lib is None:
        if not os.path.exists(SYNTH_LIB):
            raise ImportError("oracle/libsynth.so is not built; run `make -C oracle oracle`")
        _lib = C.CDLL(SYNTH_LIB)
        _lib.fyb_synth_create.restype = C.c_void_p
        _lib.fyb_synth_create.argtypes = [C.POINTER(SynthConfig)]
        _lib.fyb_synth_free.argtypes = [C.c_void_p]
    return _lib


class SynthModel:
    """nya_llm_context of a seeded random model; the same keyword arguments
    as fyodor_b200.SynthModel."""

    def __init__(self, layers=2, embedding=512, heads=4, kv_heads=2, feed_forward=1024, vocabulary=1024,
                 context=512, matrix_type=Q4_K, embed_type=Q6_K, output_type=Q6_K, rope_base=500000.0,
                 epsilon=1e-5, seed=1234, norm_mode=2, threads=0, centered=0, path=None):
        lib = library()
        self.config = SynthConfig(layers, embedding, heads, kv_heads, feed_forward, vocabulary, context,
                                  matrix_type, embed_type, output_type, rope_base, epsilon, seed, norm_mode,
                                  threads, centered, path.encode() if path else None)
        self.ptr = lib.fyb_synth_create(C.byref(self.config))
        if not self.ptr:
            raise ValueError("invalid synthetic model configuration")
        self.vocabulary = vocabulary

    def close(self):
        if self.ptr:
            library().fyb_synth_free(self.ptr)
            self.ptr = None

    def __del__(self):
        self.close()
