"""vk_gemm_q8_0_noalloc: the Q8_0 GEMM for callers that cannot allocate
device memory (hosts whose device memory is budgeted up front, plugins inside
an engine that owns every allocation).  It unpacks into a fixed array inside
the library instead of a cudaMalloc'd workspace; its results must equal the
allocating entry point's bit for bit (the Q8_0 path is bit-exact), on two
calls in a row that reuse the array.

Collected last on purpose (file name), so a failure here comes after every
other test has run."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _blocks(x):
    from oracle import oracle

    q = oracle.quantize_rows_q8_0(x)
    return torch.from_numpy(q.view(np.uint8).ravel().copy()).cuda()


def test_noalloc_matches_allocating_entry_point_twice():
    import vestra_kernels as vk

    lib = vk.lib()
    ctx = vk.Context(0)
    shapes = [(865, 768, 768), (300, 256, 3072)]  # the second call reuses the array with other sizes
    for i, (m, n, k) in enumerate(shapes):
        r = np.random.default_rng(100 + i)
        a = _blocks(r.standard_normal((m, k)).astype(np.float32))
        b = _blocks((r.standard_normal((n, k)) * 0.02).astype(np.float32))
        ref = torch.empty(m * n, device="cuda")
        got = torch.full((m * n,), float("nan"), device="cuda")
        assert lib.vk_gemm_q8_0(ctx.handle, m, n, k, ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()),
                                ctypes.c_void_p(ref.data_ptr())) == vk.VK_OK
        ctx.synchronize()
        st = lib.vk_gemm_q8_0_noalloc(None, m, n, k, ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()),
                                      ctypes.c_void_p(got.data_ptr()))
        assert st == vk.VK_OK, vk.last_error()
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int32), ref.view(torch.int32))
    ctx.close()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    import vestra_kernels as vk

    lib = vk.lib()
    dummy = ctypes.c_void_p(16)  # never dereferenced: the size check comes first
    st = lib.vk_gemm_q8_0_noalloc(None, 4096, 3072, 3072, dummy, dummy, dummy)
    assert st == vk.VK_UNSUPPORTED_SHAPE
    assert "scratch" in vk.last_error()
    # a row count whose byte count would wrap 64 bits is rejected, not run
    st = lib.vk_gemm_q8_0_noalloc(None, 1 << 60, 128, 128, dummy, dummy, dummy)
    assert st == vk.VK_UNSUPPORTED_SHAPE
    assert "scratch" in vk.last_error()
