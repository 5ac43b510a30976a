"""Exact-size pinned host memory and its device view (lazykv/pinned.py:31-92).

`pinned_empty` page-locks an ordinary allocation in place with cudaHostRegister, so the host store
is pinned at its real size (torch's caching host allocator rounds up to a power of two).
`device_view` wraps the device address of such memory as a CUDA tensor: kernels that read it read
host RAM over the link (zero-copy), which is how the exact pass reads a host-resident cold tier.
"""

from __future__ import annotations

import ctypes
import weakref

import torch


def _unregister(ptr: int) -> None:
    try:
        torch.cuda.cudart().cudaHostUnregister(ptr)
    except Exception:  # noqa: BLE001 -- at interpreter exit the context may be gone
        pass


def pinned_empty(shape: tuple[int, ...], dtype: torch.dtype) -> torch.Tensor:
    """An uninitialised CPU tensor, page-locked at exactly its size, unpinned when collected."""
    t = torch.empty(shape, dtype=dtype)
    nbytes = t.numel() * t.element_size()
    if nbytes == 0:
        return t
    rc = torch.cuda.cudart().cudaHostRegister(t.data_ptr(), nbytes, 0)
    if rc != torch.cuda.cudart().cudaError.success:
        raise RuntimeError(f"cudaHostRegister of {nbytes} bytes failed: {rc}")
    weakref.finalize(t, _unregister, t.data_ptr())
    return t


class _DeviceArray:
    def __init__(self, ptr: int, nbytes: int) -> None:
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3, "strides": None}


def _device_pointer(host_ptr: int) -> int:
    lib = torch.cuda.cudart()
    fn = getattr(lib, "cudaHostGetDevicePointer", None)
    if fn is not None:
        rc, dptr = fn(host_ptr, 0)
        if rc != lib.cudaError.success:
            raise RuntimeError(f"cudaHostGetDevicePointer failed: {rc}")
        return int(dptr)
    # torch's cudart binding lacks the call: ask the runtime library directly.
    import glob
    import os

    names = sorted(glob.glob(os.path.join(os.path.dirname(torch.__file__), "lib", "libcudart.so*"))) + sorted(glob.glob("/usr/local/cuda/lib64/libcudart.so*"))
    if not names:
        raise RuntimeError("CUDA runtime library not found")
    cudart = ctypes.CDLL(names[0])
    out = ctypes.c_void_p()
    rc = cudart.cudaHostGetDevicePointer(ctypes.byref(out), ctypes.c_void_p(host_ptr), 0)
    if rc != 0 or out.value is None:
        raise RuntimeError(f"cudaHostGetDevicePointer failed: {rc}")
    return int(out.value)


def device_view(t: torch.Tensor) -> torch.Tensor:
    """A CUDA tensor aliasing the pinned CPU tensor `t` (zero-copy reads over the link).

    The caller keeps `t` alive for as long as the view.
    """
    if not t.is_pinned() or not t.is_contiguous():
        raise ValueError("device_view needs a contiguous pinned tensor")
    torch.cuda.init()
    nbytes = t.numel() * t.element_size()
    raw = torch.as_tensor(_DeviceArray(_device_pointer(t.data_ptr()), nbytes), device="cuda")
    return raw.view(t.dtype).view(t.shape)
