"""CPU-side checks of the C ABI: the library builds for sm_100a, loads, and
exports every entry point include/vestra_b200.h declares; calls without a GPU
fail with a status, never a crash."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "vestra_b200.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(vk_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    import vestra_kernels

    lib = vestra_kernels.lib()
    names = declared()
    assert len(names) >= 30
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(vestra_kernels.SIGNATURES), set(names) ^ set(vestra_kernels.SIGNATURES)


def test_init_without_gpu_returns_status():
    import torch
    import vestra_kernels

    if torch.cuda.is_available():
        return
    lib = vestra_kernels.lib()
    h = ctypes.c_void_p()
    st = lib.vk_init(0, ctypes.byref(h))
    assert st == vestra_kernels.VK_ERR_NO_DEVICE
    assert "device" in vestra_kernels.last_error()
    assert lib.vk_synchronize(None) == vestra_kernels.VK_ERR_INVALID_ARGUMENT
    assert lib.vk_version().decode().startswith("vestra-b200")


def test_null_arguments_are_rejected():
    import vestra_kernels

    lib = vestra_kernels.lib()
    assert lib.vk_init(0, None) == vestra_kernels.VK_ERR_INVALID_ARGUMENT
    assert lib.vk_layernorm(None, None, 1, 1, None, None, 1e-6) == vestra_kernels.VK_ERR_INVALID_ARGUMENT
    assert lib.vk_encoder_prepare(None, None, None, None) == vestra_kernels.VK_ERR_INVALID_ARGUMENT
