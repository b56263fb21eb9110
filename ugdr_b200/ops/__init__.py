"""Device kernels callable from Python on tensors of the current CUDA device.

* copy_core(dst, src)      the executor's warp copy core over one range (one warp; for tests)
* grid_copy_ms(dst, src)   mean ms of a whole-grid copy with the executor's copy core
* bulk_copy_ms(dst, src)   the same copy staged through shared memory by the TMA bulk engine
* moe_route(ids, nexp)     deterministic counting sort of (token, k) rows by expert
* register(pd, tensor)     a verbs MR over a tensor's bytes (local write + remote read / write)
* kernel_attributes()      registers, spills, static shared memory and blocks per SM of every
                           kernel of the library on the current device

The collectives themselves live in ugdr_b200.parallel (they need a peer group).
"""
from __future__ import annotations

import ctypes as C

import torch

from .. import _native as N
from ..parallel.collectives import moe_route  # noqa: F401  (re-exported)


class KernelAttr(C.Structure):
    _fields_ = [("name", C.c_char * 48), ("threads_per_block", C.c_int), ("registers_per_thread", C.c_int),
                ("local_bytes_per_thread", C.c_int), ("static_smem_bytes", C.c_int),
                ("max_threads_per_block", C.c_int), ("blocks_per_sm", C.c_int)]


def _lib():
    L = N.lib()
    if not getattr(L, "_ops_sigs", False):
        L.ugdr_x_copy_core_test.restype = C.c_int
        L.ugdr_x_copy_core_test.argtypes = [C.c_void_p, C.c_void_p, C.c_uint64, C.c_void_p]
        L.ugdr_x_grid_copy_bench.restype = C.c_int
        L.ugdr_x_grid_copy_bench.argtypes = [C.c_void_p, C.c_void_p, C.c_uint64, C.c_int, C.c_int, C.c_void_p,
                                             C.POINTER(C.c_float)]
        for fn in ("ugdr_x_kernel_attributes", "ugdr_x_collective_kernel_attributes"):
            getattr(L, fn).restype = C.c_int
            getattr(L, fn).argtypes = [C.c_int, C.POINTER(KernelAttr)]
        L.ugdr_x_bulk_copy_bench.restype = C.c_int
        L.ugdr_x_bulk_copy_bench.argtypes = [C.c_void_p, C.c_void_p, C.c_uint64, C.c_int, C.c_int, C.c_void_p,
                                             C.POINTER(C.c_float), C.POINTER(C.c_uint)]
        L._ops_sigs = True
    return L


def _stream(stream: torch.cuda.Stream | None) -> C.c_void_p:
    return C.c_void_p((stream or torch.cuda.current_stream()).cuda_stream)


def copy_core(dst: torch.Tensor, src: torch.Tensor, nbytes: int | None = None,
              stream: torch.cuda.Stream | None = None) -> None:
    """Copy `nbytes` (default: all of src) from src's storage to dst's with one warp of the
    executor's copy core, on `stream`."""
    n = src.numel() * src.element_size() if nbytes is None else nbytes
    if n > dst.numel() * dst.element_size() or n > src.numel() * src.element_size():
        raise ValueError("copy larger than a tensor")
    rc = _lib().ugdr_x_copy_core_test(C.c_void_p(dst.data_ptr()), C.c_void_p(src.data_ptr()), n, _stream(stream))
    if rc != 0:
        raise RuntimeError(f"ugdr_x_copy_core_test failed: cudaError {rc}")


def grid_copy_ms(dst: torch.Tensor, src: torch.Tensor, ctas: int = 0, iters: int = 10,
                 stream: torch.cuda.Stream | None = None) -> float:
    """Mean milliseconds of a whole-grid copy of src into dst (CUDA events on `stream`)."""
    n = src.numel() * src.element_size()
    if n > dst.numel() * dst.element_size():
        raise ValueError("destination smaller than source")
    ms = C.c_float()
    rc = _lib().ugdr_x_grid_copy_bench(C.c_void_p(dst.data_ptr()), C.c_void_p(src.data_ptr()), n, ctas, iters,
                                      _stream(stream), C.byref(ms))
    if rc != 0:
        raise RuntimeError(f"ugdr_x_grid_copy_bench failed: cudaError {rc}")
    return float(ms.value)


def bulk_copy_ms(dst: torch.Tensor, src: torch.Tensor, ctas: int = 0, iters: int = 10,
                 stream: torch.cuda.Stream | None = None) -> float:
    """Mean milliseconds of a whole-grid copy of src into dst through the TMA bulk-copy engine
    (global -> shared -> global); both tensors and the size must be 16-byte aligned."""
    n = src.numel() * src.element_size()
    if n > dst.numel() * dst.element_size():
        raise ValueError("destination smaller than source")
    ms, st = C.c_float(), C.c_uint()
    rc = _lib().ugdr_x_bulk_copy_bench(C.c_void_p(dst.data_ptr()), C.c_void_p(src.data_ptr()), n, ctas, iters,
                                      _stream(stream), C.byref(ms), C.byref(st))
    if rc != 0:
        raise RuntimeError(f"ugdr_x_bulk_copy_bench failed: cudaError {rc}")
    if st.value != 0:
        raise RuntimeError("bulk copy: a bounded wait ran out")
    return float(ms.value)


def register(pd, tensor: torch.Tensor, access: int | None = None):
    """A memory region over `tensor`'s bytes (contiguous CUDA or ugdr host memory)."""
    if not tensor.is_contiguous():
        raise ValueError("register() needs a contiguous tensor")
    acc = access if access is not None else (N.ACCESS_LOCAL_WRITE | N.ACCESS_REMOTE_WRITE | N.ACCESS_REMOTE_READ)
    return pd.reg_mr(tensor.data_ptr(), tensor.numel() * tensor.element_size(), acc)


def kernel_attributes() -> list[dict]:
    """One dict per kernel of libugdr.so (executor translation unit first, then the collective
    kernels): compiled resources and resident blocks per SM at the launch block size."""
    L = _lib()
    out = []
    for fn in (L.ugdr_x_kernel_attributes, L.ugdr_x_collective_kernel_attributes):
        i = 0
        while True:
            a = KernelAttr()
            rc = fn(i, C.byref(a))
            if rc == -1:
                break
            if rc != 0:
                raise RuntimeError(f"kernel attributes failed: cudaError {rc}")
            out.append({f: (getattr(a, f).decode() if f == "name" else getattr(a, f)) for f, _ in KernelAttr._fields_})
            i += 1
    return out
