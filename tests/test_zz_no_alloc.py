"""mlxd_cuda_linear_noalloc through the C ABI, against mlxd_cuda_linear
(S == 1) and against the oracle.

Some callers cannot allocate device memory at the moment they need a
projection: code running inside a caching allocator's callback (allocating
there re-enters the allocator) and serving loops that hand all of HBM to a
fixed plan up front. For them the one-token projection keeps its workspace
(the input staged in per-group fixed point, for the formats the generic
kernel serves) in one static device array shared by every call. These tests
call it twice in a row on the same stream, and across matrices of different
shapes, before reading anything back: a call must not depend on what the
previous one left in the array. The file is named to be collected last and
initialises the device itself, so it passes alone in a fresh process and
after the rest of the suite.
"""
import numpy as np
import pytest

from mlxd_b200 import cuda
from oracle import pyoracle as po
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


# generic kernel (the static workspace in use): group 32 with f32 scales, a
# width that is not a multiple of 512, a wide input; integer-MMA kernel (no
# workspace needed): a fast-format matrix
SHAPES = [(96, 64, 32, True), (256, 320, 64, False), (1024, 20032, 64, False),
          (4096, 4096, 64, False)]


@pytest.mark.parametrize("rows,cols,group,f32", SHAPES)
def test_noalloc_matches_linear_and_oracle_twice(rows, cols, group, f32):
    L = cuda.lib()
    rng = np.random.default_rng(rows * 3 + cols)
    w, s, b = _triplet(rows, cols, group, rows + cols, f32)
    lin = cuda.Linear(w, s, b, group)
    xh = [rand_bf16(cols, rng) for _ in range(2)]
    xs = [cuda.DeviceBuffer.from_array(x) for x in xh]
    ref = [cuda.DeviceBuffer(rows * 2) for _ in range(2)]
    out = [cuda.DeviceBuffer(rows * 2) for _ in range(2)]
    for i in range(2):
        cuda.check(L.mlxd_cuda_linear(lin.h, xs[i].ptr, 1, ref[i].ptr, None), "linear")
    # two no-alloc calls in a row on one stream, no host sync between them
    for i in range(2):
        cuda.check(L.mlxd_cuda_linear_noalloc(lin.h, xs[i].ptr, out[i].ptr, None), "linear_noalloc")
    cuda.synchronize()
    for i in range(2):
        got = out[i].to_array(np.uint16, rows)
        # the same arithmetic as the allocating entry point and the oracle:
        # identical bits
        assert np.array_equal(got, ref[i].to_array(np.uint16, rows)), i
        assert np.array_equal(got, po.qlinear(xh[i], w, s, b, group, exact=True)[0]), i


def test_noalloc_alternating_shapes():
    """Calls on matrices of different widths share the array."""
    L = cuda.lib()
    rng = np.random.default_rng(7)
    shapes = [(512, 20032, 64), (128, 320, 64), (512, 20032, 64)]
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
        assert np.array_equal(y.to_array(np.uint16, rows), r.to_array(np.uint16, rows))


def test_noalloc_rejects_input_beyond_scratch():
    """An input of 262208 columns needs more fixed-point workspace than the
    array's limit of 262144 columns: rejected, output untouched."""
    L = cuda.lib()
    rows, cols, group = 16, 262208, 64
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
