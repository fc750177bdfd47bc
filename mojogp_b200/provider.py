"""Provider handles and device buffers over the C ABI (NumPy host, no torch).

`init_provider` / `destroy_provider` keep the reference's kernel-module
protocol (mojogp/codegen_engine/emit/fn_ptr_module.py:998-1196): they take
X, engine params and noise and return a dict describing the live provider.
Instead of raw function-pointer integers the dict carries a Provider object
whose methods are the same operations (forward_matvec, cross_matvec,
gradient_matvec, extract_diagonal, update_params, update_noise, ...).
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np

from . import _lib
from .kernel import KernelNode


def _ptr(a: np.ndarray) -> C.c_void_p:
    return C.c_void_p(a.ctypes.data)


class DeviceBuffer:
    """A float32 (or float64) device allocation owned by Python."""

    def __init__(self, shape, device: int = 0, dtype=np.float32):
        self.shape = tuple(int(s) for s in (shape if isinstance(shape, (tuple, list)) else (shape,)))
        self.dtype = np.dtype(dtype)
        self.device = int(device)
        self.nbytes = int(np.prod(self.shape, dtype=np.int64)) * self.dtype.itemsize
        p = C.c_void_p()
        _lib.call("gpb_device_alloc", self.device, max(self.nbytes, 1), C.byref(p))
        self.ptr = p.value

    @classmethod
    def from_host(cls, a: np.ndarray, device: int = 0) -> "DeviceBuffer":
        a = np.ascontiguousarray(a)
        buf = cls(a.shape, device, a.dtype)
        buf.upload(a)
        return buf

    def upload(self, a: np.ndarray) -> None:
        a = np.ascontiguousarray(a, dtype=self.dtype)
        if a.nbytes != self.nbytes:
            raise ValueError(f"size mismatch: {a.nbytes} vs {self.nbytes} bytes")
        _lib.call("gpb_memcpy_h2d", self.device, C.c_void_p(self.ptr), _ptr(a), self.nbytes)

    def download(self, out: np.ndarray | None = None) -> np.ndarray:
        if out is None:
            out = np.empty(self.shape, dtype=self.dtype)
        elif out.nbytes != self.nbytes or not out.flags.c_contiguous or out.dtype != self.dtype:
            raise ValueError("out must be a C-contiguous array of the buffer's size and dtype")
        _lib.call("gpb_memcpy_d2h", self.device, _ptr(out), C.c_void_p(self.ptr), self.nbytes)
        return out

    def zero(self) -> None:
        _lib.call("gpb_memset_d", self.device, C.c_void_p(self.ptr), 0, self.nbytes)

    @property
    def cptr(self) -> C.c_void_p:
        return C.c_void_p(self.ptr)

    def free(self) -> None:
        if getattr(self, "ptr", None):
            try:
                _lib.lib().gpb_device_free(self.device, C.c_void_p(self.ptr))
            finally:
                self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Provider:
    """A live gpb_provider: device X, kernel program, params and noise."""

    def __init__(self, X: np.ndarray, kernel: KernelNode, params: np.ndarray, noise: float,
                 device: int = 0, noise_vector: Optional[np.ndarray] = None):
        X = np.ascontiguousarray(X, dtype=np.float32)
        if X.ndim == 1:
            X = X[:, None]
        if X.ndim != 2:
            raise ValueError("X must be 2-D [n, d]")
        self.n, self.d = X.shape
        self.kernel = kernel
        self.spec = kernel.to_spec(self.d)
        self.num_params = int(self.spec[1])
        params = np.ascontiguousarray(params, dtype=np.float32).ravel()
        if params.shape[0] != self.num_params:
            raise ValueError(f"params has {params.shape[0]} entries, kernel expects {self.num_params}")
        nv = None
        if noise_vector is not None:
            nv = np.ascontiguousarray(noise_vector, dtype=np.float32).ravel()
            if nv.shape[0] != self.n:
                raise ValueError("noise_vector must have n entries")
        self.device = int(device)
        h = C.c_void_p()
        _lib.call("gpb_provider_create", _ptr(X), self.n, self.d, _ptr(self.spec), len(self.spec),
                  _ptr(params), self.num_params, float(noise),
                  _ptr(nv) if nv is not None else None, self.device, C.byref(h))
        self.handle = h.value
        self._params = params.copy()
        self._noise = float(noise)

    # ------------------------------------------------------------ lifecycle
    def destroy(self) -> None:
        if getattr(self, "handle", None):
            _lib.lib().gpb_provider_destroy(C.c_void_p(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass

    @property
    def h(self) -> C.c_void_p:
        if not self.handle:
            raise RuntimeError("provider was destroyed")
        return C.c_void_p(self.handle)

    def synchronize(self) -> None:
        _lib.call("gpb_provider_synchronize", self.h)

    # ------------------------------------------------------------ state
    def update_params(self, params: np.ndarray) -> None:
        params = np.ascontiguousarray(params, dtype=np.float32).ravel()
        _lib.call("gpb_update_params", self.h, _ptr(params), len(params))
        self._params = params.copy()

    def update_noise(self, noise: float) -> None:
        _lib.call("gpb_update_noise", self.h, float(noise))
        self._noise = float(noise)

    def get_noise(self) -> float:
        v = C.c_float()
        _lib.call("gpb_get_noise", self.h, C.byref(v))
        return float(v.value)

    def get_noise_mode(self) -> int:
        v = C.c_int32()
        _lib.call("gpb_get_noise_mode", self.h, C.byref(v))
        return int(v.value)

    def get_diagonal_value(self) -> float:
        v = C.c_float()
        _lib.call("gpb_get_diagonal_value", self.h, C.byref(v))
        return float(v.value)

    @property
    def params(self) -> np.ndarray:
        return self._params.copy()

    # ------------------------------------------------------------ operations
    def forward_matvec(self, out: DeviceBuffer, v: DeviceBuffer, ncols: int) -> None:
        _lib.call("gpb_forward_matvec", self.h, out.cptr, v.cptr, int(ncols))

    LAYOUTS = {0: "scalar", 1: "ffma2", 2: "tensor-core", 3: "gram-tensor-core-tf32", 4: "gram-narrow",
               5: "gram-tensor-core"}

    def matvec_layout(self, ncols: int = 16) -> str:
        """Name of the tile kernel the forward matvec uses for `ncols` columns."""
        v = C.c_int32()
        _lib.call("gpb_matvec_layout", self.h, int(ncols), C.byref(v))
        return self.LAYOUTS[v.value]

    def forward_matvec_rows(self, out: DeviceBuffer, v: DeviceBuffer, ncols: int, r0: int,
                            r1: int) -> None:
        _lib.call("gpb_forward_matvec_rows", self.h, out.cptr, v.cptr, int(ncols), int(r0), int(r1))

    def cross_matvec(self, out: DeviceBuffer, xtest: DeviceBuffer, v: DeviceBuffer, n_test: int,
                     ncols: int) -> None:
        _lib.call("gpb_cross_matvec", self.h, out.cptr, xtest.cptr, v.cptr, int(n_test), int(ncols))

    def extract_diagonal(self, out: DeviceBuffer) -> None:
        _lib.call("gpb_extract_diagonal", self.h, out.cptr)

    def extract_diagonal_test(self, out: DeviceBuffer, xtest: DeviceBuffer, n_test: int) -> None:
        _lib.call("gpb_extract_diagonal_test", self.h, out.cptr, xtest.cptr, int(n_test))

    def kernel_column(self, out: DeviceBuffer, pivot: int) -> None:
        _lib.call("gpb_kernel_column", self.h, out.cptr, int(pivot))

    def gradient_matvec(self, out: DeviceBuffer, v: DeviceBuffer, ncols: int,
                        param_index: int) -> None:
        _lib.call("gpb_gradient_matvec", self.h, out.cptr, v.cptr, int(ncols), int(param_index))

    def fused_gradient_matvec(self, out: DeviceBuffer, v: DeviceBuffer, ncols: int) -> None:
        _lib.call("gpb_fused_gradient_matvec", self.h, out.cptr, v.cptr, int(ncols))

    def gradient_bilinear(self, a: DeviceBuffer, b: DeviceBuffer, ncols: int):
        data = np.zeros(self.num_params, dtype=np.float64)
        trace = np.zeros(self.num_params, dtype=np.float64)
        _lib.call("gpb_gradient_bilinear", self.h, a.cptr, b.cptr, int(ncols), _ptr(data), _ptr(trace))
        return data, trace

    # ------------------------------------------------------------ host helpers
    def matvec_host(self, V: np.ndarray) -> np.ndarray:
        """out = (K + noise I) V for a host array V [n] or [n, t] (column layout)."""
        V = np.asarray(V, dtype=np.float32)
        squeeze = V.ndim == 1
        Vc = np.ascontiguousarray((V[:, None] if squeeze else V).T)  # [t][n]
        out = np.empty_like(Vc)
        _lib.call("gpb_forward_matvec_host", self.h, _ptr(out), _ptr(Vc), Vc.shape[0])
        res = out.T
        return res[:, 0].copy() if squeeze else np.ascontiguousarray(res)

    def cross_matvec_host(self, Xtest: np.ndarray, V: np.ndarray) -> np.ndarray:
        Xtest = np.ascontiguousarray(Xtest, dtype=np.float32)
        if Xtest.ndim == 1:
            Xtest = Xtest[:, None]
        V = np.asarray(V, dtype=np.float32)
        squeeze = V.ndim == 1
        Vc = np.ascontiguousarray((V[:, None] if squeeze else V).T)
        xt = DeviceBuffer.from_host(Xtest, self.device)
        vd = DeviceBuffer.from_host(Vc, self.device)
        od = DeviceBuffer((Vc.shape[0], Xtest.shape[0]), self.device)
        self.cross_matvec(od, xt, vd, Xtest.shape[0], Vc.shape[0])
        self.synchronize()
        res = od.download().T
        return res[:, 0].copy() if squeeze else np.ascontiguousarray(res)


def init_provider(X: np.ndarray, params: np.ndarray, noise: float, kernel: KernelNode,
                  device: int = 0, obs_noise: Optional[np.ndarray] = None) -> dict:
    """Create a provider and return its info dict (fn_ptr_module.py:998-1169)."""
    prov = Provider(X, kernel, params, noise, device=device, noise_vector=obs_noise)
    return {
        "provider": prov,
        "provider_ptr": prov.handle,
        "n": prov.n,
        "dim": prov.d,
        "num_gradient_params": prov.num_params,
        "supports_fused_gradient": True,
        "supports_fused_ls_os": False,
        "supports_fused_3param": False,
        "is_ard": kernel.has_ard(),
        "materialization_mode": 0,
        "noise_mode": prov.get_noise_mode(),
    }


def destroy_provider(info: dict) -> None:
    """Release a provider created by init_provider (fn_ptr_module.py:1183-1196)."""
    prov = info.get("provider")
    if prov is not None:
        prov.destroy()


class pinned:
    """Page-lock the given C-contiguous host arrays for the duration of a
    ``with`` block (gpb_host_register / gpb_host_unregister), so copies to and
    from them are DMA transfers from pinned memory."""

    def __init__(self, *arrays: np.ndarray):
        for a in arrays:
            if not a.flags.c_contiguous:
                raise ValueError("pinned arrays must be C-contiguous")
        self.arrays = [a for a in arrays if a.nbytes > 0]
        self._done: list[np.ndarray] = []

    def __enter__(self):
        for a in self.arrays:
            _lib.call("gpb_host_register", _ptr(a), a.nbytes)
            self._done.append(a)
        return self

    def __exit__(self, *exc):
        while self._done:
            _lib.call("gpb_host_unregister", _ptr(self._done.pop()))
        return False
