"""sq_argmax_noalloc (no counterpart in the reference): the argmax with its partial
states in the library's static device memory. Checked against sq_argmax, the
allocating entry point it mirrors, on two calls in a row; its size limit and its
promise of no pool allocation are checked directly. The file name sorts last so
the test also runs after every other test of the suite has used the library."""
import ctypes

import numpy as np
import pytest

from conftest import has_gpu

torch = pytest.importorskip("torch")

MAX_N = 1 << 24


def test_limit_and_empty_rejected_on_host():
    """Oversize and empty inputs fail on the host, before any CUDA call."""
    from sqb200 import lib
    L = lib.load()
    st = L.sq_argmax_noalloc(None, ctypes.c_void_p(256), MAX_N + 1, ctypes.c_void_p(256))
    assert lib.STATUS[st] == "InvalidArgument"
    assert "exceeds the fixed scratch limit of 16777216" in L.sq_last_error().decode()
    assert lib.STATUS[L.sq_argmax_noalloc(None, ctypes.c_void_p(256), 0, ctypes.c_void_p(256))] == "EmptyInput"
    assert lib.STATUS[L.sq_argmax_noalloc(None, None, 4, ctypes.c_void_p(256))] == "InvalidArgument"
    assert lib.ARGMAX_NOALLOC_MAX_N == MAX_N


def _inputs(case):
    rng = np.random.default_rng({"vocab": 1, "ties": 2, "nan": 3, "max": 4, "one": 5}[case])
    if case == "vocab":  # Llama-3.2 vocabulary
        return rng.standard_normal(128256).astype(np.float32), rng.standard_normal(4099).astype(np.float32)
    if case == "ties":  # greedy.rs:6-15 through max_by: equal maxima resolve to the later index
        a = np.zeros(70000, np.float32)
        a[[5, 4096, 69999]] = 3.0
        b = np.full(4096 * 3, -1.0, np.float32)
        b[[0, 8191]] = 2.0
        return a, b
    if case == "nan":
        a = rng.standard_normal(50000).astype(np.float32)
        a[[100, 30000]] = np.nan
        b = rng.standard_normal(9000).astype(np.float32)
        b[8999] = np.nan
        return a, b
    if case == "max":  # the largest n the fixed scratch holds, then a one-chunk input
        a = rng.standard_normal(MAX_N).astype(np.float32)
        a[MAX_N - 7] = 50.0
        return a, rng.standard_normal(4096).astype(np.float32)
    return np.float32([-1.5]), np.float32([0.25, 0.5])


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["vocab", "ties", "nan", "max", "one"])
def test_two_calls_in_a_row_match_sq_argmax(gpu_lib, case):
    from sqb200 import lib
    a, b = (torch.from_numpy(x).cuda() for x in _inputs(case))
    out = torch.full((2,), -1, dtype=torch.int64, device="cuda")
    # two calls back to back on one stream, no host sync between them
    lib.argmax_noalloc(a, out[0:1])
    lib.argmax_noalloc(b, out[1:2])
    want = torch.cat([lib.argmax(a), lib.argmax(b)])
    torch.cuda.synchronize()
    assert out.tolist() == want.tolist()


@pytest.mark.gpu
def test_no_pool_allocation():
    """The stream-ordered pool's high-water mark does not move across two calls,
    while one sq_argmax call moves it (so the measurement sees allocations)."""
    if not has_gpu():
        pytest.skip("no CUDA device")
    drv = pytest.importorskip("cuda.bindings.driver")
    from sqb200 import lib
    lib.load()
    x = torch.randn(300000, device="cuda")
    out = torch.empty(2, dtype=torch.int64, device="cuda")
    lib.argmax_noalloc(x, out[0:1])  # first call on the device: address lookup
    torch.cuda.synchronize()
    err, pool = drv.cuDeviceGetDefaultMemPool(torch.cuda.current_device())
    assert err == drv.CUresult.CUDA_SUCCESS
    high = drv.CUmemPool_attribute.CU_MEMPOOL_ATTR_USED_MEM_HIGH

    def watermark():
        e, v = drv.cuMemPoolGetAttribute(pool, high)
        assert e == drv.CUresult.CUDA_SUCCESS
        return int(v)

    (e,) = drv.cuMemPoolSetAttribute(pool, high, drv.cuuint64_t(0))
    assert e == drv.CUresult.CUDA_SUCCESS
    base = watermark()
    lib.argmax_noalloc(x, out[0:1])
    lib.argmax_noalloc(x[:5000], out[1:2])
    torch.cuda.synchronize()
    assert watermark() == base
    assert out.tolist() == [int(torch.argmax(x)), int(torch.argmax(x[:5000]))]
    lib.argmax(x)
    torch.cuda.synchronize()
    assert watermark() > base


@pytest.mark.gpu
def test_oversize_rejected_with_device_buffers(gpu_lib):
    from sqb200 import lib
    x = torch.zeros(MAX_N + 1, device="cuda")
    out = torch.full((1,), -1, dtype=torch.int64, device="cuda")
    with pytest.raises(lib.KernelError) as e:
        lib.argmax_noalloc(x, out)
    assert e.value.kind == "InvalidArgument" and "use sq_argmax" in str(e.value)
    assert int(out.item()) == -1
    assert int(lib.argmax(x).item()) == MAX_N  # all zeros: the later element wins
