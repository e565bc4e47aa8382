"""GPU parity of the quantized matvec / small-batch matmul through the C ABI.

Oracle: the engine's scalar kernel (oracle.matvec, pinned bit-exact to the
compiled engine) plus the double-precision forward-error bound of
test_quant_kernels.c:13-25 (|a - s| <= 1e-6 * (1 + sum |w x|)). Full-size
projection shapes use the north-star bound |a - e| <= 1e-3 * (1 + |e|).
"""
import ctypes as C

import numpy as np
import pytest

import fyodor_b200 as F
import oracle as O
from tests.patterns import k_quant_blocks, quant_kernel_inputs, quant_kernel_weights

pytestmark = pytest.mark.gpu
TYPES = [F.F32, F.F16, F.BF16, F.Q4_0, F.Q8_0, F.Q4_K, F.Q6_K]


def double_bound_ok(values, x, actual):
    prod = values.astype(np.float64) * x.astype(np.float64)
    s = prod.sum(axis=-1)
    mag = np.abs(prod).sum(axis=-1)
    return np.all(np.isfinite(actual)) and np.all(np.abs(actual.astype(np.float64) - s) <= 1e-6 * (1 + mag))


@pytest.mark.parametrize("type_id", TYPES)
def test_matvec_quant_kernel_patterns(provider, type_id):
    rows, cols = 65, 1024
    data = quant_kernel_weights(type_id, rows, cols)
    values = O.dequantize(data, type_id, rows * cols).reshape(rows, cols)
    for p in range(3):
        x = quant_kernel_inputs(cols, p)
        y = provider.matvec(data, rows, cols, type_id, x)
        assert y is not None
        assert double_bound_ok(values, x, y)
        e = O.matvec(data, type_id, x, cols, rows)
        assert np.all(np.abs(y[:17] - e[:17]) <= 1.5e-4 * (1 + np.abs(e[:17])))


@pytest.mark.parametrize("type_id", TYPES)
@pytest.mark.parametrize("batch", [2, 3, 17, 65])
def test_matmul_batches(provider, type_id, batch):
    rows, cols = 65, 1024
    data = quant_kernel_weights(type_id, rows, cols)
    values = O.dequantize(data, type_id, rows * cols).reshape(rows, cols)
    xs = (((np.arange(batch * cols) % 61) - 30) / 31).astype(np.float32).reshape(batch, cols)
    y = provider.matmul(data, rows, cols, type_id, xs, batch)
    assert y is not None
    for b in range(batch):
        assert double_bound_ok(values, xs[b], y[b]), b


@pytest.mark.parametrize("kind,type_id", [(0, F.Q4_K), (1, F.Q6_K)])
def test_k_quant_matvec_exact(provider, kind, type_id):
    """check_k_quants: the CUDA matvec must equal the double dot exactly."""
    data, expected = k_quant_blocks(kind)
    x = np.array([((i % 23) - 11) / 16.0 for i in range(512)], np.float32)
    y = provider.matvec(data, 2, 512, type_id, x)
    dot = expected.reshape(2, 512).astype(np.float64) @ x.astype(np.float64)
    assert (y.astype(np.float64) == dot).all()


def test_boundary_rejections(provider):
    """test_compute.c:99-106: invalid sizes decline with -1 before any write."""
    api, st = provider.api, provider.state
    w = np.ones(4, np.float32)
    x = np.ones(4, np.float32)
    y = np.full(4, 7.0, np.float32)
    P = lambda a: C.c_void_p(a.ctypes.data)
    assert api.matvec(st, P(w), (1 << 64) - 1, 2, 0, P(x), P(y)) == -1
    assert api.matvec(st, P(w), 0, 2, 0, P(x), P(y)) == -1
    assert api.matvec(st, None, 1, 1, 0, P(x), P(y)) == -1
    assert api.matvec(st, P(w), 1, 255, F.Q4_K, P(x), P(y)) == -1  # columns not a block multiple
    assert api.matvec(st, P(w), 1, 4, 99, P(x), P(y)) == -1        # unknown storage type
    assert api.matmul(st, P(w), 1, 4, 0, P(x), P(y), 513) == -1     # batch above 512
    assert (y == 7.0).all()
    assert provider.active()


def test_cached_weight_reuse_and_resizing(provider):
    """test_compute.c:57-85: alternate buffers and shapes through the cache."""
    small = (np.arange(6) / 10.0).astype(np.float32)
    large = (((np.arange(325) % 17) - 8) / 19.0).astype(np.float32)
    for p in range(6):
        rows, cols, w = (2, 3, small) if p % 2 == 0 else (5, 65, large)
        x = ((np.arange(cols) + p) / 71.0).astype(np.float32)
        y = provider.matvec(w, rows, cols, F.F32, x)
        e = w.reshape(rows, cols).astype(np.float64) @ x.astype(np.float64)
        assert np.all(np.abs(y - e) <= 1e-4 * (1 + np.abs(e)))


SWEEP = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]


def double_reference(data, type_id, xs, cols, rows, chunk=8192):
    """sum_k w*x and sum_k |w*x| in double over the exactly dequantized
    weights (the forward-error oracle of test_quant_kernels.c:13-25)."""
    rb = F.row_bytes(type_id, cols)
    s = np.empty((xs.shape[0], rows))
    mag = np.empty((xs.shape[0], rows))
    x64 = xs.astype(np.float64)
    for r0 in range(0, rows, chunk):
        n = min(chunk, rows - r0)
        w = O.dequantize(data[r0 * rb:(r0 + n) * rb], type_id, n * cols).reshape(n, cols).astype(np.float64)
        s[:, r0:r0 + n] = x64 @ w.T
        mag[:, r0:r0 + n] = np.abs(x64) @ np.abs(w).T
    return s, mag


@pytest.mark.parametrize("type_id", [F.Q4_K, F.Q6_K])
@pytest.mark.parametrize("rows,cols", SWEEP)
def test_projection_sweep(provider, type_id, rows, cols):
    """C2 shapes with the benchmark's value distributions; batches 1, 2, 4, 8 and 16.
    Bounds: the reference's forward-error bound against the double dot,
    |a - s| <= 1e-6 (1 + sum|w x|), and the north-star 1e-3 relative."""
    nbytes = rows * F.row_bytes(type_id, cols)
    data = np.empty(nbytes, np.uint8)
    F.lib.fyb_synth_fill(C.c_void_p(data.ctypes.data), rows, cols, type_id, 2024, rows * 7 + cols)
    rng = np.random.default_rng(rows + cols)
    xs = rng.standard_normal((16, cols)).astype(np.float32)
    s, mag = double_reference(data, type_id, xs, cols, rows)
    for batch in (1, 2, 4, 8, 16):
        y = provider.matmul(data, rows, cols, type_id, xs[:batch], batch)
        assert y is not None
        for b in range(batch):
            err = np.abs(y[b].astype(np.float64) - s[b])
            assert np.all(err <= 1e-6 * (1 + mag[b])), (batch, b, float((err / (1 + mag[b])).max()))
            assert np.all(err <= 1e-3 * (1 + np.abs(s[b]))), (batch, b)


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (1000, 14336), (37, 32768)])
def test_q8_0_matvec(provider, rows, cols):
    """C1 (Q8_0 4096x4096, the benchmark's value distribution: int8 uniform in
    [-127, 127], d = |N(0,1)| * 0.01) and row widths that split a row over 2
    and 4 warps; batches 1, 5 and 8 through the engine's matvec / matmul.
    Bounds as in test_projection_sweep, and the engine's own scalar Q8_0
    matvec (oracle.matvec, llm_quant.c:145-312) within 1e-4 relative."""
    nbytes = rows * F.row_bytes(F.Q8_0, cols)
    data = np.empty(nbytes, np.uint8)
    F.lib.fyb_synth_fill(C.c_void_p(data.ctypes.data), rows, cols, F.Q8_0, 2024, rows * 7 + cols)
    rng = np.random.default_rng(rows * 3 + cols)
    xs = rng.standard_normal((8, cols)).astype(np.float32)
    s, mag = double_reference(data, F.Q8_0, xs, cols, rows)
    e0 = O.matvec(data, F.Q8_0, xs[0], cols, rows)
    y = provider.matvec(data, rows, cols, F.Q8_0, xs[0])
    assert y is not None
    assert np.all(np.abs(y.astype(np.float64) - s[0]) <= 1e-6 * (1 + mag[0]))
    assert np.all(np.abs(y - e0) <= 1e-4 * (1 + np.abs(e0)))
    for batch in (5, 8):
        y = provider.matmul(data, rows, cols, F.Q8_0, xs[:batch], batch)
        assert y is not None
        for b in range(batch):
            err = np.abs(y[b].astype(np.float64) - s[b])
            assert np.all(err <= 1e-6 * (1 + mag[b])), (batch, b)


def test_dequantize_bit_exact_all_types():
    import torch
    for type_id in [F.F32, F.F16, F.BF16, F.Q4_0, F.Q8_0, F.Q4_K, F.Q6_K]:
        rows, cols = 33, 1024
        data = quant_kernel_weights(type_id, rows, cols)
        expected = O.dequantize(data, type_id, rows * cols)
        d = torch.from_numpy(data).cuda()
        out = torch.empty(rows * cols, dtype=torch.float32, device="cuda")
        assert F.lib.fyb_dequantize(C.c_void_p(d.data_ptr()), rows * cols, type_id, C.c_void_p(out.data_ptr()), None) == 0
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert (got.view(np.uint32) == expected.view(np.uint32)).all(), type_id


def test_f32_257x1025_like_engine_test(provider):
    """test_compute.c check_matvec(257, 1025): every row of three passes."""
    rows, cols = 257, 1025
    i = np.arange(rows * cols)
    w = (((i % 23) - 11) / 17.0).astype(np.float32)
    for p in range(3):
        x = ((((np.arange(cols) % 13) - 6 + p)) / 7.0).astype(np.float32)
        y = provider.matvec(w, rows, cols, F.F32, x)
        e = w.reshape(rows, cols).astype(np.float64) @ x.astype(np.float64)
        bad = np.nonzero(np.abs(y - e) > 1e-4 * (1 + np.abs(e)))[0]
        assert bad.size == 0, (p, bad[:8].tolist(), y[bad[:4]].tolist(), e[bad[:4]].tolist())


@pytest.mark.parametrize("type_id", [F.Q4_K, F.Q6_K])
def test_prepared_matches_one_call(type_id):
    """fyb_quant_repack + fyb_quant_matmul_prepared (repack once, multiply
    many times) give fyb_quant_matmul's results bitwise, for odd and even
    batches; the workspace's counters stay zero between calls."""
    import torch
    rows, cols = 1040, 4096
    nbytes = rows * F.row_bytes(type_id, cols)
    data = np.empty(nbytes, np.uint8)
    F.lib.fyb_synth_fill(C.c_void_p(data.ctypes.data), rows, cols, type_id, 7, 3)
    dw = torch.from_numpy(data).cuda()
    wsb = F.lib.fyb_quant_matmul_workspace(rows, cols, type_id, 5)
    ws1 = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
    ws2 = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr())
    assert F.lib.fyb_quant_repack(P(dw), rows, cols, type_id, P(ws2), wsb, None) == 0
    x = torch.randn((5, cols), device="cuda")
    for batch in (1, 2, 3, 5):
        y1 = torch.empty((batch, rows), device="cuda")
        y2 = torch.empty((batch, rows), device="cuda")
        assert F.lib.fyb_quant_matmul(P(dw), rows, cols, type_id, P(x), P(y1), batch, P(ws1), wsb, None) == 0
        for _ in range(2):
            assert F.lib.fyb_quant_matmul_prepared(rows, cols, type_id, P(x), P(y2), batch, P(ws2), wsb, None) == 0
        torch.cuda.synchronize()
        assert torch.equal(y1, y2), batch
    assert F.lib.fyb_quant_matmul_prepared(rows, cols, F.Q8_0, P(x), P(y2), 1, P(ws2), wsb, None) == -1


@pytest.mark.parametrize("type_id", [F.Q4_K, F.Q6_K])
@pytest.mark.parametrize("rows,cols", [(4096, 4096), (1024, 14336), (3000, 4096)])
def test_prepared_small_batch_gemm(type_id, rows, cols):
    """Batches of 3..17 through fyb_quant_matmul_prepared (the weight-reusing
    small-batch GEMM for groups of 3..16 vectors: the integer mma.sync kernel
    for 3, the tcgen05 kernel with 16, 32 and 64 B columns for 4, 5..8 and
    9..16; the GEMV for a remainder of one or two) against the double
    reference, with the forward-error bound of the GEMV tests. K = 14336 needs several K-slices at 16 vectors (their
    partial rows are added in slice order); 3000 rows end in a partial tile."""
    import torch
    P = lambda t: C.c_void_p(t.data_ptr())
    nbytes = rows * F.row_bytes(type_id, cols)
    data = np.empty(nbytes, np.uint8)
    F.lib.fyb_synth_fill(C.c_void_p(data.ctypes.data), rows, cols, type_id, 77, rows * 3 + cols)
    rng = np.random.default_rng(rows * 31 + cols)
    xs = rng.standard_normal((17, cols)).astype(np.float32)
    s, mag = double_reference(data, type_id, xs, cols, rows)
    wsb = F.lib.fyb_quant_matmul_workspace(rows, cols, type_id, 17)
    ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
    dw = torch.from_numpy(data).cuda()
    assert F.lib.fyb_quant_repack(P(dw), rows, cols, type_id, P(ws), wsb, None) == 0
    x = torch.from_numpy(xs).cuda()
    for batch in (3, 4, 5, 8, 12, 16, 17):
        y = torch.full((batch, rows), float("nan"), device="cuda")
        for rep in range(2):  # twice: the scratch counters must be back at zero
            assert F.lib.fyb_quant_matmul_prepared(rows, cols, type_id, P(x), P(y), batch, P(ws), wsb, None) == 0
            torch.cuda.synchronize()
            got = y.cpu().numpy().astype(np.float64)
            for b in range(batch):
                err = np.abs(got[b] - s[b])
                assert np.all(err <= 1e-6 * (1 + mag[b])), (batch, rep, b, float((err / (1 + mag[b])).max()))
