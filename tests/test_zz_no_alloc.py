"""mlxd_cuda_linear_noalloc against mlxd_cuda_linear (S == 1), through the C ABI.

The allocation-free decode GEMV keeps its split partial sums in one static
device array shared by every call, so these tests call it twice in a row on
the same stream (and across matrices of different shapes) before reading
anything back: the second call must not see the first call's counters. The
file is named to be collected last and initialises the device itself, so it
passes alone in a fresh process and after the rest of the suite.
"""
import numpy as np
import pytest

from mlxd_b200 import cuda
from tests.helpers import bf16_to_f32, rand_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _init():
    cuda.init(0)
    yield


def _triplet(rows, cols, group, seed, f32_scales=False):
    w = np.zeros((rows, cols // 8), np.uint32)
    s = np.zeros((rows, cols // group), np.uint16)
    b = np.zeros((rows, cols // group), np.uint16)
    cuda.lib().mlxd_host_synth_quantized(cuda.ptr(w), cuda.ptr(s), cuda.ptr(b), rows, cols,
                                         group, seed, 0.02)
    if f32_scales:
        return w, bf16_to_f32(s).copy(), bf16_to_f32(b).copy()
    return w, s, b


def _close(g, o):
    # the decode GEMV tolerance of the parity tests: within 2 bf16 ulps
    g, o = bf16_to_f32(g), bf16_to_f32(o)
    tol = 2 * 2.0 ** -8 * np.maximum(np.abs(o), 1e-3 * np.abs(o).max())
    return bool(np.all(np.abs(g - o) <= tol)), float(np.abs(g - o).max())


# fast block-of-8 kernel, many-slot split rows (down-projection shape),
# generic G=32 kernel with f32 scales, a 1-slot-per-unit small matrix
SHAPES = [(4096, 4096, 64, False), (4096, 12288, 64, False), (96, 64, 32, True),
          (256, 512, 64, False)]


@pytest.mark.parametrize("rows,cols,group,f32", SHAPES)
def test_noalloc_matches_linear_twice(rows, cols, group, f32):
    L = cuda.lib()
    rng = np.random.default_rng(rows * 3 + cols)
    lin = cuda.Linear(*_triplet(rows, cols, group, rows + cols, f32), group)
    xs = [cuda.DeviceBuffer.from_array(rand_bf16(cols, rng)) for _ in range(2)]
    ref = [cuda.DeviceBuffer(rows * 2) for _ in range(2)]
    out = [cuda.DeviceBuffer(rows * 2) for _ in range(2)]
    for i in range(2):
        cuda.check(L.mlxd_cuda_linear(lin.h, xs[i].ptr, 1, ref[i].ptr, None), "linear")
    # two no-alloc calls in a row on one stream, no host sync between them
    for i in range(2):
        cuda.check(L.mlxd_cuda_linear_noalloc(lin.h, xs[i].ptr, out[i].ptr, None), "linear_noalloc")
    cuda.synchronize()
    for i in range(2):
        ok, err = _close(out[i].to_array(np.uint16, rows), ref[i].to_array(np.uint16, rows))
        assert ok, (i, err)


def test_noalloc_alternating_shapes():
    """Calls on matrices with different workspace layouts share the array."""
    L = cuda.lib()
    rng = np.random.default_rng(7)
    shapes = [(4096, 12288, 64), (1024, 4096, 64), (4096, 12288, 64)]
    lins = {}
    results = []
    for rows, cols, group in shapes:
        if (rows, cols) not in lins:
            lins[(rows, cols)] = cuda.Linear(*_triplet(rows, cols, group, rows ^ cols), group)
        lin = lins[(rows, cols)]
        x = cuda.DeviceBuffer.from_array(rand_bf16(cols, rng))
        y = cuda.DeviceBuffer(rows * 2)
        cuda.check(L.mlxd_cuda_linear_noalloc(lin.h, x.ptr, y.ptr, None), "linear_noalloc")
        results.append((lin, x, y, rows))
    cuda.synchronize()
    for lin, x, y, rows in results:
        r = cuda.DeviceBuffer(rows * 2)
        cuda.check(L.mlxd_cuda_linear(lin.h, x.ptr, 1, r.ptr, None), "linear")
        cuda.synchronize()
        ok, err = _close(y.to_array(np.uint16, rows), r.to_array(np.uint16, rows))
        assert ok, err


def test_noalloc_rejects_matrix_beyond_scratch():
    """262160 rows need 16385 row-block counters; the array holds 16384."""
    L = cuda.lib()
    rows, cols, group = 262160, 64, 64
    lin = cuda.Linear(*_triplet(rows, cols, group, 11), group)
    x = cuda.DeviceBuffer.from_array(rand_bf16(cols, np.random.default_rng(1)))
    y = cuda.DeviceBuffer(rows * 2)
    y.zero()
    rc = L.mlxd_cuda_linear_noalloc(lin.h, x.ptr, y.ptr, None)
    assert rc == -1
    assert b"static scratch" in L.mlxd_cuda_last_error()
    cuda.synchronize()
    assert not y.to_array(np.uint16, rows).any()
    # the allocating entry point still serves it
    cuda.check(L.mlxd_cuda_linear(lin.h, x.ptr, 1, y.ptr, None), "linear")
    cuda.synchronize()
    assert y.to_array(np.uint16, rows).any()
