"""Device buffers for the GPU tests, through the library's own C ABI (no other GPU runtime)."""

from __future__ import annotations

import ctypes

import numpy as np


class DeviceArray:
    """A device allocation holding one NumPy array's bytes."""

    def __init__(self, runtime, host: np.ndarray | None = None, *, shape=None, dtype=None, fill: int | None = None):
        self.rt = runtime
        if host is not None:
            host = np.ascontiguousarray(host)
            shape, dtype = host.shape, host.dtype
        self.shape, self.dtype = tuple(shape), np.dtype(dtype)
        self.nbytes = int(np.prod(self.shape, dtype=np.int64)) * self.dtype.itemsize
        ptr = ctypes.c_void_p()
        runtime.check(runtime.library().nc_device_alloc(max(self.nbytes, 1), ctypes.byref(ptr)))
        self.ptr = ptr
        if host is not None:
            self.upload(host)
        elif fill is not None:
            self.upload(np.full(self.shape, fill, self.dtype))

    def upload(self, host: np.ndarray) -> None:
        host = np.ascontiguousarray(host, self.dtype)
        if self.nbytes:
            self.rt.check(self.rt.library().nc_copy_to_device(self.ptr, host.ctypes.data, self.nbytes))

    def numpy(self) -> np.ndarray:
        out = np.empty(self.shape, self.dtype)
        if self.nbytes:
            self.rt.check(self.rt.library().nc_copy_to_host(out.ctypes.data, self.ptr, self.nbytes))
        return out

    def free(self) -> None:
        if self.ptr:
            self.rt.library().nc_device_free(self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def packed_int8(runtime, values: np.ndarray) -> DeviceArray:
    """int8 weights as the kernels read them (+128), packed by the library."""
    values = np.ascontiguousarray(values, np.int8)
    buf = DeviceArray(runtime, shape=values.shape, dtype=np.uint8)
    runtime.check(runtime.library().nc_pack_int8_weights(buf.ptr, values.ctypes.data, values.nbytes))
    return buf


def call(runtime, name: str, pointers, sizes) -> None:
    """Call a fused-group entry point: p[] device pointers (DeviceArray or None), s[] int64 sizes."""
    p = (ctypes.c_void_p * len(pointers))(*[(x.ptr.value if isinstance(x, DeviceArray) else x) for x in pointers])
    s = (ctypes.c_int64 * len(sizes))(*sizes)
    runtime.check(getattr(runtime.library(), name)(p, s, None))
    runtime.check(runtime.library().nc_device_synchronize())


def f32_bits(x: float) -> int:
    return int(np.array([x], np.float32).view(np.uint32)[0])
