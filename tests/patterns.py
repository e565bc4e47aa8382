"""Deterministic input patterns restated from the reference's own tests.

k_quant_blocks        test_architectures.c:232-285 (check_k_quants)
quant_kernel_weights  test_quant_kernels.c:141-172
quant_kernel_inputs   test_quant_kernels.c:175
bench_tokens          bench_main.c:109
"""
import numpy as np

F32, F16, Q4_0, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 2, 8, 12, 14, 30
STRIDE = {F32: lambda c: c * 4, F16: lambda c: c * 2, BF16: lambda c: c * 2, Q4_0: lambda c: c // 32 * 18,
          Q8_0: lambda c: c // 32 * 34, Q4_K: lambda c: c // 256 * 144, Q6_K: lambda c: c // 256 * 210}


def k_quant_blocks(kind):
    """Four Q4_K (kind 0) or Q6_K (kind 1) blocks built from logical fields, with
    their exact values (powers of two keep every product exact)."""
    stride = 144 if kind == 0 else 210
    data = np.zeros(4 * stride, np.uint8)
    expected = np.zeros(1024, np.float32)
    for b in range(4):
        p = b * stride
        if kind == 0:
            data[p + 1] = 0x38
            data[p + 3] = 0x34  # d = 1/2, dmin = 1/4
            scales = [(g * 11 + b * 7) % 64 for g in range(8)]
            minima = [(g * 17 + b * 13) % 64 for g in range(8)]
            for g in range(4):
                data[p + 4 + g] = scales[g] | ((scales[g + 4] >> 4) << 6)
                data[p + 8 + g] = minima[g] | ((minima[g + 4] >> 4) << 6)
                data[p + 12 + g] = (scales[g + 4] & 15) | ((minima[g + 4] & 15) << 4)
            for pair in range(4):
                for j in range(32):
                    lo = (j * 3 + pair + b) % 16
                    hi = (j * 7 + pair * 3 + b) % 16
                    data[p + 16 + pair * 32 + j] = lo | (hi << 4)
                    expected[b * 256 + pair * 64 + j] = 0.5 * (scales[pair * 2] * lo) - 0.25 * minima[pair * 2]
                    expected[b * 256 + pair * 64 + 32 + j] = 0.5 * (scales[pair * 2 + 1] * hi) - 0.25 * minima[pair * 2 + 1]
        else:
            data[p + 209] = 0x30  # d = 1/8
            scales = [(g * 37 + b * 53) % 256 - 128 for g in range(16)]
            for g in range(16):
                data[p + 192 + g] = scales[g] & 255
            for half in range(2):
                for j in range(32):
                    q = [(j * 13 + k * 19 + half * 31 + b * 7) % 64 for k in range(4)]
                    for k in range(4):
                        n = half * 128 + k * 32 + j
                        expected[b * 256 + n] = 0.125 * scales[n // 16] * (q[k] - 32)
                    data[p + half * 64 + j] = (q[0] & 15) | ((q[2] & 15) << 4)
                    data[p + half * 64 + 32 + j] = (q[1] & 15) | ((q[3] & 15) << 4)
                    data[p + 128 + half * 32 + j] = (q[0] >> 4) | ((q[1] >> 4) << 2) | ((q[2] >> 4) << 4) | ((q[3] >> 4) << 6)
    return data, expected


def quant_kernel_weights(type_id, rows, columns):
    stride = STRIDE[type_id](columns)
    n = stride * rows
    i = np.arange(n, dtype=np.int64)
    data = ((i * 73 + i // 17 + 31) & 255).astype(np.uint8)
    if type_id in (F32, F16, BF16):
        k = np.arange(rows * columns, dtype=np.int64)
        value = ((k % 127) - 63).astype(np.float32) / 64
        if type_id == F32:
            data = value.view(np.uint8).copy()
        elif type_id == BF16:
            data = (value.view(np.uint32) >> 16).astype(np.uint16).view(np.uint8).copy()
        else:
            v = (0x3000 + (k % 1024) + np.where(k % 2 == 1, 0x8000, 0)).astype(np.uint16)
            data = v.view(np.uint8).copy()
    else:
        block = {Q4_0: 18, Q8_0: 34, Q4_K: 144, Q6_K: 210}[type_id]
        scale = 208 if type_id == Q6_K else 0
        for s in range(0, n, block):
            data[s + scale] = 0
            data[s + scale + 1] = 0x28
            if type_id == Q4_K:
                data[s + 2] = 0
                data[s + 3] = 0x24
    return data


def quant_kernel_inputs(columns, p):
    i = np.arange(columns)
    return (((i + p * 3) % 97) - 48).astype(np.float32) / 49


def bench_tokens(count, vocabulary, start=0):
    i = np.arange(start, start + count, dtype=np.int64)
    return ((i * 15485863 + 17) % vocabulary).astype(np.uint32)


# Small seeded models: (name, fyodor_b200.SynthModel kwargs, token ids).
SMALL_MODELS = [
    ("q4k_h128", dict(layers=2, embedding=512, heads=4, kv_heads=2, feed_forward=1024, vocabulary=1024, context=64,
                      matrix_type=Q4_K, embed_type=Q6_K, output_type=Q6_K, seed=11, norm_mode=2, centered=1),
     [int(t) for t in bench_tokens(12, 1024)]),
    ("q6k_h64", dict(layers=2, embedding=512, heads=8, kv_heads=4, feed_forward=768, vocabulary=768, context=64,
                     matrix_type=Q6_K, embed_type=Q8_0, output_type=Q4_K, seed=12, norm_mode=1),
     [int(t) for t in bench_tokens(10, 768, 3)]),
]
