"""Host-side mirror of the reference's ``Backend`` trait over the C ABI.

Reference contract: crates/dragonwing-core/src/backend.rs:127-199
(``name``, ``alloc``, ``upload``, ``download``, ``synchronize``) and
``BackendBuffer::len_bytes`` (backend.rs:21-33).  Errors are raised as
``BackendError`` carrying the backend's reason string, like the reference's
``Error::Backend(String)``; lengths are never truncated.
"""
from __future__ import annotations

import ctypes
import enum

import numpy as np

from . import _lib as L


class BackendError(RuntimeError):
    """A failed backend call: ``status`` is the dw_status code."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{L.STATUS_NAMES.get(status, status)}: {message}")
        self.status = status
        self.message = message


class BufferKind(enum.Enum):
    """backend.rs BufferKind: every allocation is a linear storage buffer."""

    Storage = 0


class CudaBuffer:
    """Device byte buffer (``impl BackendBuffer``)."""

    __slots__ = ("_backend", "handle", "_len", "__weakref__")

    def __init__(self, backend: "CudaBackend", handle: ctypes.c_void_p, length: int):
        self._backend = backend
        self.handle = handle
        self._len = length

    def len_bytes(self) -> int:
        return self._len

    @property
    def device_ptr(self) -> int:
        return int(L.load().dw_buf_device_ptr(self.handle) or 0)

    def free(self) -> None:
        if self.handle:
            self._backend._check(L.load().dw_free(self._backend.handle, self.handle))
            self.handle = None

    def __del__(self):
        try:
            if self.handle and self._backend.handle:
                L.load().dw_free(self._backend.handle, self.handle)
                self.handle = None
        except Exception:
            pass


def _host_view(data) -> tuple[ctypes.c_void_p, int, object]:
    if isinstance(data, np.ndarray):
        arr = np.ascontiguousarray(data)
        return ctypes.c_void_p(arr.ctypes.data), arr.nbytes, arr
    if isinstance(data, (bytes, bytearray, memoryview)):
        arr = np.frombuffer(data, dtype=np.uint8)
        return ctypes.c_void_p(arr.ctypes.data), arr.nbytes, arr
    raise TypeError(f"unsupported host buffer type {type(data)!r}")


class CudaEvent:
    """A stream-ordering point between backends (streams) of one GPU."""

    def __init__(self, backend: "CudaBackend"):
        self._lib = L.load()
        out = ctypes.c_void_p()
        backend._check(self._lib.dw_event_create(backend.handle, ctypes.byref(out)))
        self.handle = out

    def close(self) -> None:
        if self.handle:
            self._lib.dw_event_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CudaBackend:
    """One B200 GPU and one CUDA stream (``impl Backend for CudaBackend``)."""

    def __init__(self, device: int = 0, wait_cap_ms: int = 0, trace: bool = False, conv_path: int = L.PATH_AUTO,
                 dw_variant: int = 0):
        self._lib = L.load()
        cfg = L.DwConfig()
        cfg.wait_cap_ms = wait_cap_ms
        cfg.trace = 1 if trace else 0
        cfg.conv_path = conv_path
        cfg.dw_variant = dw_variant
        out = ctypes.c_void_p()
        st = self._lib.dw_create(device, ctypes.byref(cfg), ctypes.byref(out))
        if st != L.DW_OK:
            raise BackendError(st, f"dw_create(device={device}) failed")
        self.handle = out
        self.device = device

    # -- Backend trait ------------------------------------------------------
    def name(self) -> str:
        return self._lib.dw_name().decode()

    def alloc(self, len_bytes: int, kind: BufferKind = BufferKind.Storage) -> CudaBuffer:
        out = ctypes.c_void_p()
        self._check(self._lib.dw_alloc(self.handle, len_bytes, ctypes.byref(out)))
        return CudaBuffer(self, out, len_bytes)

    def upload(self, dst: CudaBuffer, src) -> None:
        ptr, n, _keep = _host_view(src)
        self._check(self._lib.dw_upload(self.handle, dst.handle, ptr, n))

    def download(self, src: CudaBuffer, dst) -> None:
        if isinstance(dst, np.ndarray) and not dst.flags.c_contiguous:
            raise ValueError("download destination must be C-contiguous")
        ptr, n, _keep = _host_view(dst)
        self._check(self._lib.dw_download(self.handle, src.handle, ptr, n))

    def synchronize(self, timeout_ms: int = 0) -> None:
        self._check(self._lib.dw_synchronize(self.handle, timeout_ms))

    # -- extras ---------------------------------------------------------------
    def wrap(self, device_ptr: int, len_bytes: int) -> CudaBuffer:
        """Wraps caller-owned device memory (e.g. a torch tensor's storage)."""
        out = ctypes.c_void_p()
        self._check(self._lib.dw_buf_wrap(self.handle, ctypes.c_void_p(device_ptr), len_bytes, ctypes.byref(out)))
        return CudaBuffer(self, out, len_bytes)

    def upload_array(self, arr: np.ndarray) -> CudaBuffer:
        arr = np.ascontiguousarray(arr)
        buf = self.alloc(max(arr.nbytes, 1))
        if arr.nbytes:
            self.upload(buf, arr)
        return buf

    def download_array(self, buf: CudaBuffer, dtype, shape=None) -> np.ndarray:
        out = np.empty(buf.len_bytes() // np.dtype(dtype).itemsize, dtype=dtype)
        self.download(buf, out)
        return out if shape is None else out.reshape(shape)

    def host_alloc(self, nbytes: int) -> tuple[int, np.ndarray]:
        """Page-locked host memory: returns (pointer, uint8 numpy view)."""
        out = ctypes.c_void_p()
        self._check(self._lib.dw_host_alloc(self.handle, nbytes, ctypes.byref(out)))
        arr = np.ctypeslib.as_array(ctypes.cast(out, ctypes.POINTER(ctypes.c_uint8)), shape=(nbytes,))
        return int(out.value), arr

    def host_free(self, ptr: int) -> None:
        self._check(self._lib.dw_host_free(self.handle, ctypes.c_void_p(ptr)))

    def upload_async(self, dst: CudaBuffer, host_ptr: int, nbytes: int, dst_offset: int = 0) -> None:
        self._check(self._lib.dw_upload_async(self.handle, dst.handle, dst_offset, ctypes.c_void_p(host_ptr), nbytes))

    def download_async(self, src: CudaBuffer, host_ptr: int, nbytes: int, src_offset: int = 0) -> None:
        self._check(self._lib.dw_download_async(self.handle, src.handle, src_offset, ctypes.c_void_p(host_ptr), nbytes))

    def copy_async(self, dst: CudaBuffer, src: CudaBuffer, nbytes: int, dst_offset: int = 0,
                   src_offset: int = 0) -> None:
        self._check(self._lib.dw_copy_async(self.handle, dst.handle, dst_offset, src.handle, src_offset, nbytes))

    def event(self) -> "CudaEvent":
        return CudaEvent(self)

    def record(self, ev: "CudaEvent") -> None:
        """Records `ev` at the current end of this backend's stream."""
        self._check(self._lib.dw_event_record(self.handle, ev.handle))

    def wait(self, ev: "CudaEvent") -> None:
        """Work enqueued on this backend after the call waits for `ev`."""
        self._check(self._lib.dw_stream_wait_event(self.handle, ev.handle))

    def stream(self) -> int:
        return int(self._lib.dw_stream(self.handle) or 0)

    def sm_count(self) -> int:
        return int(self._lib.dw_sm_count(self.handle))

    def launch_count(self) -> int:
        return int(self._lib.dw_launch_count(self.handle))

    def scratch_bytes(self) -> int:
        """Device scratch the backend holds (grown by ops that need temporaries)."""
        return int(self._lib.dw_scratch_bytes(self.handle))

    def last_error(self) -> str:
        return self._lib.dw_last_error(self.handle).decode(errors="replace")

    def close(self) -> None:
        if self.handle:
            self._lib.dw_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, status: int) -> None:
        if status != L.DW_OK:
            raise BackendError(status, self.last_error() if self.handle else "")


def device_count() -> int:
    """Number of CUDA devices visible (0 when the driver is absent)."""
    try:
        import torch
        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:  # pragma: no cover - torch always present in this image
        return 0
