"""ctypes binding of the C ABI (include/fp8linear_b200.h).

This is the binding a non-torch host would write against ``libfp8linear_b200.so``;
here it takes torch CUDA tensors only as carriers of device pointers and streams.
Every call checks the returned status and raises ``RuntimeError`` with the
library's message on failure.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libfp8linear_b200.so"

OK = 0
DTYPE = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}
DTYPE_NONE = -1

# name -> (restype, argtypes); mirrors the declarations in include/fp8linear_b200.h
_P, _I, _I64, _SZ, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_float
SIGNATURES = {
    "fp8lin_abi_version": (_I, []),
    "fp8lin_build_info": (ctypes.c_char_p, []),
    "fp8lin_last_error": (ctypes.c_char_p, []),
    "fp8lin_quantize_fp8": (_I, [_P, _I, _I64, _I64, _P, _P, _P]),
    "fp8lin_quantize_weight": (_I, [_P, _I, _I64, _I64, _P, _P, _P]),
    "fp8lin_mx_scale_bytes": (_SZ, [_I64, _I64]),
    "fp8lin_quantize_mxfp8": (_I, [_P, _I, _I64, _I64, _P, _P, _P]),
    "fp8lin_mxfp8_gemm": (_I, [_P, _P, _P, _P, _P, _I, _P, _I, _I64, _I64, _I64, _P]),
    "fp8lin_mxfp8_linear_workspace_size": (_SZ, [_I64, _I64]),
    "fp8lin_mxfp8_linear": (_I, [_P, _I, _P, _P, _P, _I, _P, _I, _I64, _I64, _I64, _P, _SZ, _P]),
    "fp8lin_layernorm_modulate_quantize_fp8": (_I, [_P, _I, _I64, _I64, _I64, _P, _P, _F, _P, _P, _P]),
    "fp8lin_fp8_linear_modulated": (_I, [_P, _I, _I64, _I64, _I64, _P, _P, _F, _P, _P, _P, _I, _P,
                                        _I, _I64, _P, _SZ, _P]),
    "fp8lin_fp8_linear_host_workspace_size": (_SZ, [_I64, _I64, _I64]),
    "fp8lin_fp8_linear_host": (_I, [_P, _I, _P, _P, _P, _I, _P, _I, _I64, _I64, _I64, _P, _SZ, _P]),
    "fp8lin_nv_scale_bytes": (_SZ, [_I64, _I64]),
    "fp8lin_quantize_nvfp4": (_I, [_P, _I, _I64, _I64, _P, _P, _P]),
    "fp8lin_nvfp4_gemm": (_I, [_P, _P, _P, _P, _P, _I, _P, _I, _I64, _I64, _I64, _P]),
    "fp8lin_nvfp4_linear_workspace_size": (_SZ, [_I64, _I64]),
    "fp8lin_nvfp4_linear": (_I, [_P, _I, _P, _P, _P, _I, _P, _I, _I64, _I64, _I64, _P, _SZ, _P]),
    "fp8lin_fp8_gemm": (_I, [_P, _P, _P, _P, _P, _I, _P, _I, _I64, _I64, _I64, _P]),
    "fp8lin_linear_workspace_size": (_SZ, [_I64, _I64]),
    "fp8lin_fp8_linear": (_I, [_P, _I, _P, _P, _P, _I, _P, _I, _I64, _I64, _I64, _P, _SZ, _P]),
    "fp8lin_device_status": (_I, [ctypes.POINTER(ctypes.c_uint), _I]),
    "fp8lin_fp8_linear_noalloc": (_I, [_P, _I, _P, _P, _P, _I, _P, _I, _I64, _I64, _I64, _P]),
    "fp8lin_selftest_watchdog": (_I, [ctypes.c_uint, ctypes.POINTER(ctypes.c_uint), _P]),
    "fp8lin_fp8_linear_allgather": (_I, [_P, _I, _P, _P, _P, _I, ctypes.POINTER(ctypes.c_void_p),
                                         _I, _I, _I64, _I64, _I64, _I64, _P, _SZ, _P]),
    "fp8lin_peer_buffer_alloc": (_I, [_SZ, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]),
    "fp8lin_peer_buffer_open": (_I, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
    "fp8lin_peer_buffer_close": (_I, [_P]),
    "fp8lin_peer_buffer_free": (_I, [_P]),
}

# FP8LIN_PEER_HANDLE_BYTES in the header
PEER_HANDLE_BYTES = 64

# fp8lin_fp8_linear_noalloc's fixed scratch (FP8LIN_NOALLOC_SCRATCH_BYTES in the header)
NOALLOC_SCRATCH_BYTES = 64 * 1024 * 1024


class CApi:
    def __init__(self, path: str | Path = LIB_PATH):
        self.path = Path(path)
        if not self.path.exists():
            raise ImportError(f"{self.path} not built; run `python fp8linear_b200/_build.py`")
        self.lib = ctypes.CDLL(str(self.path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(self.lib, name)
            fn.restype = res
            fn.argtypes = args

    # -- helpers
    def _check(self, rc: int, op: str) -> None:
        if rc != OK:
            raise RuntimeError(f"{op} failed (status {rc}): {self.last_error()}")

    def last_error(self) -> str:
        return self.lib.fp8lin_last_error().decode()

    @staticmethod
    def _stream(t: torch.Tensor | None = None) -> int:
        dev = t.device if t is not None else torch.device("cuda")
        return torch.cuda.current_stream(dev).cuda_stream

    @staticmethod
    def _bias_ptr(bias):
        return None if bias is None else bias.data_ptr()

    @staticmethod
    def _bias_dtype(bias):
        return DTYPE_NONE if bias is None else DTYPE[bias.dtype]

    # -- entry points
    def quantize_fp8(self, x: torch.Tensor, xq: torch.Tensor | None = None,
                     scale: torch.Tensor | None = None):
        M, K = x.shape
        xq = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=x.device) if xq is None else xq
        scale = torch.empty((M,), dtype=torch.float32, device=x.device) if scale is None else scale
        rc = self.lib.fp8lin_quantize_fp8(x.data_ptr(), DTYPE[x.dtype], M, K, xq.data_ptr(),
                                          scale.data_ptr(), self._stream(x))
        self._check(rc, "fp8lin_quantize_fp8")
        return xq, scale

    def mx_scale_bytes(self, rows: int, K: int) -> int:
        return int(self.lib.fp8lin_mx_scale_bytes(rows, K))

    def quantize_mxfp8(self, x: torch.Tensor, xq: torch.Tensor | None = None,
                       scales: torch.Tensor | None = None):
        M, K = x.shape
        xq = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=x.device) if xq is None else xq
        if scales is None:
            scales = torch.empty((self.mx_scale_bytes(M, K),), dtype=torch.uint8, device=x.device)
        rc = self.lib.fp8lin_quantize_mxfp8(x.data_ptr(), DTYPE[x.dtype], M, K, xq.data_ptr(),
                                            scales.data_ptr(), self._stream(x))
        self._check(rc, "fp8lin_quantize_mxfp8")
        return xq, scales

    def mxfp8_gemm(self, xq, x_scales, wq, w_scales, bias=None, out_dtype=torch.bfloat16,
                   out=None):
        M, K = xq.shape
        N = wq.shape[0]
        out = torch.empty((M, N), dtype=out_dtype, device=xq.device) if out is None else out
        rc = self.lib.fp8lin_mxfp8_gemm(xq.data_ptr(), x_scales.data_ptr(), wq.data_ptr(),
                                        w_scales.data_ptr(), self._bias_ptr(bias),
                                        self._bias_dtype(bias), out.data_ptr(), DTYPE[out.dtype],
                                        M, N, K, self._stream(xq))
        self._check(rc, "fp8lin_mxfp8_gemm")
        return out

    def mxfp8_linear(self, x, wq, w_scales, bias=None, out=None, workspace=None):
        M, K = x.shape
        N = wq.shape[0]
        out = torch.empty((M, N), dtype=x.dtype, device=x.device) if out is None else out
        need = int(self.lib.fp8lin_mxfp8_linear_workspace_size(M, K))
        if workspace is None:
            workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
        rc = self.lib.fp8lin_mxfp8_linear(x.data_ptr(), DTYPE[x.dtype], wq.data_ptr(),
                                          w_scales.data_ptr(), self._bias_ptr(bias),
                                          self._bias_dtype(bias), out.data_ptr(),
                                          DTYPE[out.dtype], M, N, K, workspace.data_ptr(),
                                          workspace.numel(), self._stream(x))
        self._check(rc, "fp8lin_mxfp8_linear")
        return out

    def nv_scale_bytes(self, rows: int, K: int) -> int:
        return int(self.lib.fp8lin_nv_scale_bytes(rows, K))

    def quantize_nvfp4(self, x: torch.Tensor, xq: torch.Tensor | None = None,
                       scales: torch.Tensor | None = None):
        M, K = x.shape
        xq = torch.empty((M, K // 2), dtype=torch.uint8, device=x.device) if xq is None else xq
        if scales is None:
            scales = torch.empty((self.nv_scale_bytes(M, K),), dtype=torch.uint8, device=x.device)
        rc = self.lib.fp8lin_quantize_nvfp4(x.data_ptr(), DTYPE[x.dtype], M, K, xq.data_ptr(),
                                            scales.data_ptr(), self._stream(x))
        self._check(rc, "fp8lin_quantize_nvfp4")
        return xq, scales

    def nvfp4_gemm(self, xq, x_scales, wq, w_scales, bias=None, out_dtype=torch.bfloat16,
                   out=None):
        M, K = xq.shape[0], xq.shape[1] * 2
        N = wq.shape[0]
        out = torch.empty((M, N), dtype=out_dtype, device=xq.device) if out is None else out
        rc = self.lib.fp8lin_nvfp4_gemm(xq.data_ptr(), x_scales.data_ptr(), wq.data_ptr(),
                                        w_scales.data_ptr(), self._bias_ptr(bias),
                                        self._bias_dtype(bias), out.data_ptr(), DTYPE[out.dtype],
                                        M, N, K, self._stream(xq))
        self._check(rc, "fp8lin_nvfp4_gemm")
        return out

    def nvfp4_linear(self, x, wq, w_scales, bias=None, out=None, workspace=None):
        M, K = x.shape
        N = wq.shape[0]
        out = torch.empty((M, N), dtype=x.dtype, device=x.device) if out is None else out
        need = int(self.lib.fp8lin_nvfp4_linear_workspace_size(M, K))
        if workspace is None:
            workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
        rc = self.lib.fp8lin_nvfp4_linear(x.data_ptr(), DTYPE[x.dtype], wq.data_ptr(),
                                          w_scales.data_ptr(), self._bias_ptr(bias),
                                          self._bias_dtype(bias), out.data_ptr(),
                                          DTYPE[out.dtype], M, N, K, workspace.data_ptr(),
                                          workspace.numel(), self._stream(x))
        self._check(rc, "fp8lin_nvfp4_linear")
        return out

    def layernorm_modulate_quantize_fp8(self, x, shift, scale, eps=1e-6, xq=None, x_scale=None):
        K = x.shape[-1]
        M = x.numel() // K
        xq = torch.empty((M, K), dtype=torch.float8_e4m3fn, device=x.device) if xq is None else xq
        x_scale = torch.empty((M,), dtype=torch.float32, device=x.device) if x_scale is None else x_scale
        rc = self.lib.fp8lin_layernorm_modulate_quantize_fp8(
            x.data_ptr(), DTYPE[x.dtype], M, K, shift.shape[0], shift.data_ptr(),
            scale.data_ptr(), float(eps), xq.data_ptr(), x_scale.data_ptr(), self._stream(x))
        self._check(rc, "fp8lin_layernorm_modulate_quantize_fp8")
        return xq, x_scale

    def fp8_linear_modulated(self, x, shift, scale, wq, w_scale, bias=None, eps=1e-6, out=None,
                             workspace=None):
        K = x.shape[-1]
        M = x.numel() // K
        N = wq.shape[0]
        out = torch.empty((M, N), dtype=x.dtype, device=x.device) if out is None else out
        need = int(self.lib.fp8lin_linear_workspace_size(M, K))
        if workspace is None:
            workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
        rc = self.lib.fp8lin_fp8_linear_modulated(
            x.data_ptr(), DTYPE[x.dtype], M, K, shift.shape[0], shift.data_ptr(),
            scale.data_ptr(), float(eps), wq.data_ptr(), w_scale.data_ptr(), self._bias_ptr(bias),
            self._bias_dtype(bias), out.data_ptr(), DTYPE[out.dtype], N, workspace.data_ptr(),
            workspace.numel(), self._stream(x))
        self._check(rc, "fp8lin_fp8_linear_modulated")
        return out

    def fp8_linear_host(self, x_host, wq, w_scale, bias=None, out_host=None, out_dtype=None,
                        workspace=None):
        """x_host / out_host in (pinned) host memory; weights on the device. Queued on the
        current stream of wq's device; synchronize it before reading out_host."""
        M, K = x_host.shape
        N = wq.shape[0]
        out_dtype = x_host.dtype if out_dtype is None else out_dtype
        if out_host is None:
            out_host = torch.empty((M, N), dtype=out_dtype, pin_memory=True)
        need = int(self.lib.fp8lin_fp8_linear_host_workspace_size(M, N, K))
        if workspace is None:
            workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=wq.device)
        rc = self.lib.fp8lin_fp8_linear_host(x_host.data_ptr(), DTYPE[x_host.dtype], wq.data_ptr(),
                                             w_scale.data_ptr(), self._bias_ptr(bias),
                                             self._bias_dtype(bias), out_host.data_ptr(),
                                             DTYPE[out_host.dtype], M, N, K, workspace.data_ptr(),
                                             workspace.numel(), self._stream(wq))
        self._check(rc, "fp8lin_fp8_linear_host")
        return out_host

    def quantize_weight(self, w: torch.Tensor):
        N, K = w.shape
        wq = torch.empty((N, K), dtype=torch.float8_e4m3fn, device=w.device)
        scale = torch.empty((N,), dtype=torch.float32, device=w.device)
        rc = self.lib.fp8lin_quantize_weight(w.data_ptr(), DTYPE[w.dtype], N, K, wq.data_ptr(),
                                             scale.data_ptr(), self._stream(w))
        self._check(rc, "fp8lin_quantize_weight")
        return wq, scale

    def fp8_gemm(self, xq, x_scale, wq, w_scale, bias=None, out_dtype=torch.bfloat16, out=None):
        M, K = xq.shape
        N = wq.shape[0]
        out = torch.empty((M, N), dtype=out_dtype, device=xq.device) if out is None else out
        rc = self.lib.fp8lin_fp8_gemm(
            xq.data_ptr(), x_scale.data_ptr(), wq.data_ptr(), w_scale.data_ptr(),
            None if bias is None else bias.data_ptr(),
            DTYPE_NONE if bias is None else DTYPE[bias.dtype],
            out.data_ptr(), DTYPE[out.dtype], M, N, K, self._stream(xq))
        self._check(rc, "fp8lin_fp8_gemm")
        return out

    def workspace_size(self, M: int, K: int) -> int:
        return int(self.lib.fp8lin_linear_workspace_size(M, K))

    def fp8_linear(self, x, wq, w_scale, bias=None, out=None, workspace=None):
        M, K = x.shape
        N = wq.shape[0]
        out = torch.empty((M, N), dtype=x.dtype, device=x.device) if out is None else out
        need = self.workspace_size(M, K)
        if workspace is None:
            workspace = torch.empty((max(need, 1),), dtype=torch.uint8, device=x.device)
        rc = self.lib.fp8lin_fp8_linear(
            x.data_ptr(), DTYPE[x.dtype], wq.data_ptr(), w_scale.data_ptr(),
            None if bias is None else bias.data_ptr(),
            DTYPE_NONE if bias is None else DTYPE[bias.dtype],
            out.data_ptr(), DTYPE[out.dtype], M, N, K, workspace.data_ptr(),
            workspace.numel(), self._stream(x))
        self._check(rc, "fp8lin_fp8_linear")
        return out

    def fp8_linear_noalloc(self, x, wq, w_scale, bias=None, out=None):
        """fp8_linear without a workspace: the library's fixed device scratch is used
        (for callers that cannot allocate device memory)."""
        M, K = x.shape
        N = wq.shape[0]
        out = torch.empty((M, N), dtype=x.dtype, device=x.device) if out is None else out
        rc = self.lib.fp8lin_fp8_linear_noalloc(
            x.data_ptr(), DTYPE[x.dtype], wq.data_ptr(), w_scale.data_ptr(),
            None if bias is None else bias.data_ptr(),
            DTYPE_NONE if bias is None else DTYPE[bias.dtype],
            out.data_ptr(), DTYPE[out.dtype], M, N, K, self._stream(x))
        self._check(rc, "fp8lin_fp8_linear_noalloc")
        return out

    def fp8_linear_allgather(self, x, wq, w_scale, bias, out_ptrs, ldo, out_dtype=None,
                             workspace=None):
        """Column-parallel linear writing this rank's [M, N] block (N = wq rows) into
        every buffer in ``out_ptrs`` (device addresses of this rank's first column in each
        GPU's [M, ldo] output; the first is this GPU's)."""
        M, K = x.shape
        N = wq.shape[0]
        out_dtype = x.dtype if out_dtype is None else out_dtype
        need = self.workspace_size(M, K)
        if workspace is None:
            workspace = torch.empty((max(need, 1),), dtype=torch.uint8, device=x.device)
        arr = (ctypes.c_void_p * len(out_ptrs))(*[int(p) for p in out_ptrs])
        rc = self.lib.fp8lin_fp8_linear_allgather(
            x.data_ptr(), DTYPE[x.dtype], wq.data_ptr(), w_scale.data_ptr(),
            None if bias is None else bias.data_ptr(),
            DTYPE_NONE if bias is None else DTYPE[bias.dtype],
            arr, len(out_ptrs), DTYPE[out_dtype], M, N, K, ldo, workspace.data_ptr(),
            workspace.numel(), self._stream(x))
        self._check(rc, "fp8lin_fp8_linear_allgather")

    # -- peer buffers (one process per GPU; CUDA IPC mappings, no multicast object)
    def peer_alloc(self, nbytes: int) -> tuple[int, bytes]:
        """Allocate ``nbytes`` on the current device; returns (device address, handle)."""
        ptr = ctypes.c_void_p()
        h = ctypes.create_string_buffer(PEER_HANDLE_BYTES)
        self._check(self.lib.fp8lin_peer_buffer_alloc(nbytes, ctypes.byref(ptr), h),
                    "fp8lin_peer_buffer_alloc")
        return int(ptr.value), h.raw

    def peer_open(self, handle: bytes) -> int:
        """Map another process's buffer; returns its address in this process."""
        if len(handle) != PEER_HANDLE_BYTES:
            raise ValueError(f"peer handle must be {PEER_HANDLE_BYTES} bytes")
        ptr = ctypes.c_void_p()
        self._check(self.lib.fp8lin_peer_buffer_open(handle, ctypes.byref(ptr)),
                    "fp8lin_peer_buffer_open")
        return int(ptr.value)

    def peer_close(self, ptr: int) -> None:
        self._check(self.lib.fp8lin_peer_buffer_close(ptr), "fp8lin_peer_buffer_close")

    def peer_free(self, ptr: int) -> None:
        self._check(self.lib.fp8lin_peer_buffer_free(ptr), "fp8lin_peer_buffer_free")

    @staticmethod
    def peer_tensor(ptr: int, nbytes: int, device: torch.device) -> torch.Tensor:
        """A uint8 tensor over ``nbytes`` at device address ``ptr`` (not owned: the
        memory lives until peer_free / peer_close)."""

        class _Mem:
            __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                        "data": (ptr, False), "version": 3, "strides": None}

        with torch.cuda.device(device):
            return torch.as_tensor(_Mem(), device=device)

    def selftest_watchdog(self, limit_us: int = 50_000) -> int:
        """Run the bounded-wait self-test; returns the recorded status (32 = the wait ran
        out and the kernel returned cleanly)."""
        v = ctypes.c_uint(0)
        self._check(self.lib.fp8lin_selftest_watchdog(limit_us, ctypes.byref(v), self._stream()),
                    "fp8lin_selftest_watchdog")
        return int(v.value)

    def device_status(self, clear: bool = False) -> int:
        v = ctypes.c_uint(0)
        self._check(self.lib.fp8lin_device_status(ctypes.byref(v), int(clear)),
                    "fp8lin_device_status")
        return int(v.value)
