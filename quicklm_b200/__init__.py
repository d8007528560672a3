"""quicklm_b200 — B200 (sm_100a) int8 quantized-matmul path for QuickLM.

Python binding over the C ABI in ``include/qlm_b200.h`` (library
``quicklm_b200/lib/libqlm_b200.so``, built by ``quicklm_b200.build``). The
names mirror QuickLM's operator interface for this path:

* ``Int8Weight.quantize(...)`` — ``SafetensorsLoader::get_tensor_keep_int8``
  (src/io/safetensors.cpp:517-585) done on the device: the result is an int8
  weight resident in HBM instead of ``Tensor::int8_data``/``int8_scales``
  (src/tensor/tensor.hpp:30-43).
* ``matmul(A, B, C)`` — ``math::matmul(A, B, C, transpose_B=true)``
  (src/ops/math_ops.hpp:92, src/ops/math_ops.cpp:820-900) for an int8 B:
  C[m, n] = A[m, :] . B[n, :], C overwritten. Bit-identical to the reference
  by default.

There is no CPU fallback: if the CUDA library is missing or fails to load,
``load()`` raises.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

__all__ = ["QlmError", "Int8Weight", "matmul", "matmul_grouped", "argmax", "load", "LIB_PATH", "EXACT", "TENSOR", "HOST_IO", "SYNC",
           "BLOCK", "Comm", "exchange_handles", "shard_rows", "matmul_allgather", "save", "store_info", "rms_norm", "add_rms_norm",
           "silu_mul", "rope_neox", "rope_neox_tables", "silu", "conv1d_update_tapmajor", "l2norm_heads",
           "gdn_gates", "gdn_recurrence", "rms_norm_gain", "gqa_attend", "Model"]

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libqlm_b200.so")
BLOCK = 32
EXACT, TENSOR, HOST_IO, SYNC = 0x0, 0x1, 0x2, 0x4
SRC_F32, SRC_BF16 = 0, 1

# Every symbol the header declares; tests check the library exports all of them.
ABI_SYMBOLS = (
    "qlm_abi_version", "qlm_last_error", "qlm_weight_quantize_upload", "qlm_weight_import_int8",
    "qlm_weight_export_int8", "qlm_weight_shape", "qlm_weight_bytes", "qlm_weight_free", "qlm_linear_int8",
    "qlm_device_status", "qlm_stream_sync", "qlm_linear_int8_tc_noalloc", "qlm_comm_handle_bytes",
    "qlm_comm_create", "qlm_comm_connect", "qlm_comm_free", "qlm_linear_int8_allgather", "qlm_argmax_f32",
    "qlm_linear_int8_grouped", "qlm_weight_quantize_upload_q4", "qlm_weight_export_int4", "qlm_weight_bits",
    "qlm_weight_import_int4", "qlm_store_save", "qlm_store_load", "qlm_store_info", "qlm_rms_norm",
    "qlm_add_rms_norm", "qlm_add_then_rms_norm", "qlm_silu_mul", "qlm_rope_neox", "qlm_rope_neox_tables", "qlm_silu",
    "qlm_conv1d_update_tapmajor", "qlm_l2norm_heads", "qlm_gdn_gates", "qlm_gdn_recurrence", "qlm_rms_norm_gain",
    "qlm_gqa_attend", "qlm_comm_set_timeout_us", "qlm_comm_status", "qlm_model_load", "qlm_model_reset",
    "qlm_model_decode", "qlm_model_info", "qlm_model_free", "qlm_model_load_batch", "qlm_model_decode_batch", "qlm_model_stream",
    "qlm_prof_enable", "qlm_prof_matmul_ms", "qlm_prof_reset", "qlm_prof_report",
)

_STATUS = {0: "OK", 1: "INVALID_ARG", 2: "CUDA", 3: "OUT_OF_MEMORY", 4: "UNSUPPORTED", 5: "TIMEOUT", 6: "NCCL",
           7: "INTERNAL"}


class QlmError(RuntimeError):
    """A failing qlm_* call; ``status`` is the qlm_status code."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"{_STATUS.get(status, status)}: {msg}")
        self.status = status


_lib = None


def load(path: str = LIB_PATH):
    """Load the CUDA library (once). Raises if it is missing — no fallback."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise QlmError(4, f"{path} is missing; build it with `python -m quicklm_b200.build`")
    lib = ctypes.CDLL(path)
    P, I, L = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    lib.qlm_abi_version.restype = I
    lib.qlm_last_error.restype = ctypes.c_char_p
    lib.qlm_weight_quantize_upload.argtypes = [P, I, L, I, I, I, I, I, P, ctypes.POINTER(P)]
    lib.qlm_weight_import_int8.argtypes = [P, P, I, I, I, I, I, P, ctypes.POINTER(P)]
    lib.qlm_weight_export_int8.argtypes = [P, P, P]
    lib.qlm_weight_quantize_upload_q4.argtypes = [P, I, L, I, I, I, I, I, P, ctypes.POINTER(P)]
    lib.qlm_weight_export_int4.argtypes = [P, P, P]
    lib.qlm_weight_bits.argtypes = [P]
    lib.qlm_weight_import_int4.argtypes = [P, P, I, I, I, I, I, P, ctypes.POINTER(P)]
    lib.qlm_store_save.argtypes = [ctypes.c_char_p, I, P, P]
    lib.qlm_store_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p, I, I, I, P, ctypes.POINTER(P)]
    lib.qlm_store_info.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(I), ctypes.POINTER(L),
                                   ctypes.POINTER(L)]
    F = ctypes.c_float
    lib.qlm_rms_norm.argtypes = [P, P, P, I, I, F, P]
    lib.qlm_add_rms_norm.argtypes = [P, P, P, P, I, I, F, P]
    lib.qlm_add_then_rms_norm.argtypes = [P, P, P, P, I, I, F, P]
    lib.qlm_silu_mul.argtypes = [P, P, L, P]
    lib.qlm_rope_neox.argtypes = [P, I, I, I, I, P, P, P]
    lib.qlm_rope_neox_tables.argtypes = [I, I, F, I, P, P]
    lib.qlm_silu.argtypes = [P, L, P]
    lib.qlm_conv1d_update_tapmajor.argtypes = [P, P, I, P, P, I, I, P]
    lib.qlm_l2norm_heads.argtypes = [P, I, I, F, P]
    lib.qlm_gdn_gates.argtypes = [P, P, P, P, P, P, I, P]
    lib.qlm_gdn_recurrence.argtypes = [P, P, P, P, P, P, P, I, I, P]
    lib.qlm_rms_norm_gain.argtypes = [P, P, P, I, I, F, P]
    lib.qlm_gqa_attend.argtypes = [P, I, P, P, P, I, I, I, I, P, P]
    lib.qlm_weight_shape.argtypes = [P] + [ctypes.POINTER(I)] * 5
    lib.qlm_weight_bytes.argtypes = [P]
    lib.qlm_weight_bytes.restype = L
    lib.qlm_weight_free.argtypes = [P]
    lib.qlm_weight_free.restype = None
    lib.qlm_linear_int8.argtypes = [P, I, I, L, P, P, L, I, P]
    lib.qlm_stream_sync.argtypes = [P]
    lib.qlm_device_status.argtypes = [I, I]
    lib.qlm_linear_int8_tc_noalloc.argtypes = [P, I, I, L, P, P, L, I, P]
    lib.qlm_comm_handle_bytes.restype = I
    lib.qlm_comm_create.argtypes = [I, I, I, L, ctypes.POINTER(P), P]
    lib.qlm_comm_connect.argtypes = [P, P]
    lib.qlm_comm_free.argtypes = [P]
    lib.qlm_comm_free.restype = None
    lib.qlm_comm_set_timeout_us.argtypes = [P, L]
    lib.qlm_model_load.argtypes = [ctypes.c_char_p, I, I, ctypes.POINTER(P)]
    lib.qlm_model_reset.argtypes = [P]
    lib.qlm_model_decode.argtypes = [P, I, I, ctypes.POINTER(I), P]
    lib.qlm_model_info.argtypes = [P] + [ctypes.POINTER(I)] * 5
    lib.qlm_model_load_batch.argtypes = [ctypes.c_char_p, I, I, I, ctypes.POINTER(P)]
    lib.qlm_model_decode_batch.argtypes = [P, P, I, P, P]
    lib.qlm_model_stream.argtypes = [P]
    lib.qlm_model_stream.restype = P
    lib.qlm_model_free.argtypes = [P]
    lib.qlm_model_free.restype = None
    lib.qlm_comm_status.argtypes = [P]
    lib.qlm_linear_int8_allgather.argtypes = [P, I, I, L, P, P, P, L, I, P]
    lib.qlm_argmax_f32.argtypes = [P, I, L, P, P, P, I, P]
    lib.qlm_linear_int8_grouped.argtypes = [P, I, I, L, P, I, P, P, I, P]
    lib.qlm_prof_enable.argtypes = [I]
    lib.qlm_prof_matmul_ms.argtypes = [ctypes.POINTER(ctypes.c_double), ctypes.POINTER(L)]
    lib.qlm_prof_report.argtypes = [ctypes.c_char_p, L, ctypes.POINTER(L)]
    if lib.qlm_abi_version() != 1:
        raise QlmError(7, "ABI version mismatch")
    _lib = lib
    return lib


def _check(rc: int) -> None:
    if rc != 0:
        raise QlmError(rc, load().qlm_last_error().decode())


def _is_torch(t) -> bool:
    return type(t).__module__.startswith("torch")


def _stream_ptr(stream) -> int | None:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)  # torch.cuda.Stream


class Int8Weight:
    """A device-resident quantized weight (rows [row_begin, row_end) of
    [n_total, k]) with per-32-block fp32 scales, owned by a ``qlm_w8`` handle.
    ``bits`` is 8 (the reference's int8 tensors) or 4 (its Q4_0 int4 tensors)."""

    def __init__(self, handle: int):
        self._h = ctypes.c_void_p(handle)
        lib = load()
        vals = [ctypes.c_int() for _ in range(5)]
        _check(lib.qlm_weight_shape(self._h, *[ctypes.byref(v) for v in vals]))
        self.rows, self.k, self.row_begin, self.row_end, self.n_total = (v.value for v in vals)
        self.bits = int(lib.qlm_weight_bits(self._h))
        self.device = None

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._h:
            raise QlmError(1, "weight already freed")
        return self._h

    @property
    def shape(self):
        return (self.rows, self.k)

    @property
    def nbytes(self) -> int:
        """Device bytes one M=1 product reads (packed codes + scales)."""
        return int(load().qlm_weight_bytes(self.handle))

    @classmethod
    def quantize(cls, w, device: int = 0, row_begin: int = 0, row_end: int | None = None, stream=None,
                 bits: int = 8):
        """Quantize an [n, k] float32 (or bf16-bits uint16 / torch bf16)
        matrix on the device. ``w`` is a numpy array (host, e.g. an mmap) or a
        torch tensor (host or CUDA). ``bits=8`` follows get_tensor_keep_int8,
        ``bits=4`` get_tensor_keep_int4 (src/io/safetensors.cpp:517, 587)."""
        lib = load()
        if bits not in (4, 8):
            raise QlmError(1, f"bits must be 4 or 8, not {bits}")
        upload = lib.qlm_weight_quantize_upload if bits == 8 else lib.qlm_weight_quantize_upload_q4
        if _is_torch(w):
            import torch
            if w.dim() != 2 or w.stride(1) != 1:
                raise QlmError(1, "weight must be a 2-D tensor with unit column stride")
            dt = {torch.float32: SRC_F32, torch.bfloat16: SRC_BF16}.get(w.dtype)
            if dt is None:
                raise QlmError(1, f"unsupported weight dtype {w.dtype}")
            ptr, stride = w.data_ptr(), w.stride(0)
            n, k = w.shape
            keep = w
        else:
            arr = np.asarray(w)
            if arr.ndim != 2:
                raise QlmError(1, "weight must be 2-D")
            if arr.dtype == np.float32:
                dt = SRC_F32
            elif arr.dtype == np.uint16:
                dt = SRC_BF16
            else:
                raise QlmError(1, f"unsupported weight dtype {arr.dtype}")
            if arr.strides[1] != arr.itemsize:
                arr = np.ascontiguousarray(arr)
            ptr, stride = arr.ctypes.data, arr.strides[0] // arr.itemsize
            n, k = arr.shape
            keep = arr
        if row_end is None:
            row_end = n
        h = ctypes.c_void_p()
        _check(upload(ptr, dt, stride, n, k, row_begin, row_end, device, _stream_ptr(stream), ctypes.byref(h)))
        del keep
        out = cls(h.value)
        out.device = device
        return out

    @classmethod
    def from_int8(cls, q: np.ndarray, scales: np.ndarray, device: int = 0, row_begin: int = 0,
                  row_end: int | None = None, stream=None):
        """Upload a weight already in the reference Tensor's int8 layout."""
        q = np.ascontiguousarray(q, np.int8)
        scales = np.ascontiguousarray(scales, np.float32)
        n, k = q.shape
        if scales.shape != (n, (k + BLOCK - 1) // BLOCK):
            raise QlmError(1, f"scales shape {scales.shape} != {(n, (k + BLOCK - 1) // BLOCK)}")
        if row_end is None:
            row_end = n
        h = ctypes.c_void_p()
        _check(load().qlm_weight_import_int8(q.ctypes.data, scales.ctypes.data, n, k, row_begin, row_end, device,
                                             _stream_ptr(stream), ctypes.byref(h)))
        out = cls(h.value)
        out.device = device
        return out

    @classmethod
    def from_int4(cls, packed: np.ndarray, scales: np.ndarray, k: int, device: int = 0, row_begin: int = 0,
                  row_end: int | None = None, stream=None):
        """Upload a weight already in the reference Tensor's int4 layout
        (packed [n, (k+1)/2] uint8, value + 8, low nibble = even column)."""
        packed = np.ascontiguousarray(packed, np.uint8)
        scales = np.ascontiguousarray(scales, np.float32)
        n = packed.shape[0]
        if packed.shape != (n, (k + 1) // 2) or scales.shape != (n, (k + BLOCK - 1) // BLOCK):
            raise QlmError(1, f"shapes {packed.shape}, {scales.shape} do not match k={k}")
        if row_end is None:
            row_end = n
        h = ctypes.c_void_p()
        _check(load().qlm_weight_import_int4(packed.ctypes.data, scales.ctypes.data, n, k, row_begin, row_end, device,
                                             _stream_ptr(stream), ctypes.byref(h)))
        out = cls(h.value)
        out.device = device
        return out

    @classmethod
    def from_file(cls, path: str, name: str, device: int = 0, row_begin: int = 0, row_end: int = -1, stream=None):
        """Load a pre-quantized weight written by :func:`save` (no quantization)."""
        h = ctypes.c_void_p()
        _check(load().qlm_store_load(os.fsencode(path), name.encode(), row_begin, row_end, device,
                                     _stream_ptr(stream), ctypes.byref(h)))
        out = cls(h.value)
        out.device = device
        return out

    def to_int8(self):
        """(q int8 [rows, k], scales float32 [rows, ceil(k/32)]) in the reference layout."""
        q = np.empty((self.rows, self.k), np.int8)
        s = np.empty((self.rows, (self.k + BLOCK - 1) // BLOCK), np.float32)
        _check(load().qlm_weight_export_int8(self.handle, q.ctypes.data, s.ctypes.data))
        return q, s

    def to_int4(self):
        """(packed uint8 [rows, (k+1)/2], scales float32 [rows, ceil(k/32)]) in
        the reference Tensor's int4 layout (low nibble = even column, value + 8)."""
        q = np.empty((self.rows, (self.k + 1) // 2), np.uint8)
        s = np.empty((self.rows, (self.k + BLOCK - 1) // BLOCK), np.float32)
        _check(load().qlm_weight_export_int4(self.handle, q.ctypes.data, s.ctypes.data))
        return q, s

    def free(self) -> None:
        if self._h:
            load().qlm_weight_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def save(path: str, weights: dict) -> None:
    """Write {name: Int8Weight} as a pre-quantized safetensors file."""
    names = list(weights)
    c_names = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
    c_ws = (ctypes.c_void_p * len(names))(*[weights[n].handle.value for n in names])
    _check(load().qlm_store_save(os.fsencode(path), len(names), c_names, c_ws))


def store_info(path: str, name: str):
    """(bits, rows, k) of a pre-quantized weight in a file (no GPU needed)."""
    b, r, k = ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64()
    _check(load().qlm_store_info(os.fsencode(path), name.encode(), ctypes.byref(b), ctypes.byref(r), ctypes.byref(k)))
    return b.value, r.value, k.value


def _host_addr(a) -> int:
    """Address of a numpy array's first element. A writable C-contiguous array
    exports it through the buffer protocol in ~0.5 us; `.ctypes.data` builds
    an object (1.3-2.2 us), which is the fallback for any other array."""
    try:
        return ctypes.addressof(ctypes.c_char.from_buffer(a))
    except (TypeError, ValueError, BufferError):
        return a.ctypes.data


def matmul(A, B: Int8Weight, C=None, transpose_B: bool = True, flags: int = EXACT, stream=None):
    """C = A . B^T for an int8 or int4 B (``math::matmul`` with transpose_B=true).

    * numpy A/C: host buffers; the call copies in, runs, copies out and
      returns with C complete (the reference's synchronous contract).
    * torch CUDA A/C: device buffers on B's device; asynchronous on
      ``stream`` (default: torch's current stream) unless ``flags`` has SYNC.
    A is [M, K] or [K]; C (allocated when None) is [M, N] with any row stride.
    """
    if not transpose_B:
        raise QlmError(1, "quantized weights are only supported with transpose_B=true, as in the reference")
    lib = load()
    if _is_torch(A):
        import torch
        if not A.is_cuda:
            A = A.numpy()
        else:
            a2 = A if A.dim() == 2 else A.view(1, -1)
            if a2.dtype != torch.float32 or a2.stride(1) != 1:
                raise QlmError(1, "A must be float32 with unit column stride")
            M, K = a2.shape
            if C is None:
                C = torch.empty((M, B.rows), dtype=torch.float32, device=A.device)
            c2 = C if C.dim() == 2 else C.view(1, -1)
            if c2.dtype != torch.float32 or c2.stride(1) != 1 or tuple(c2.shape) != (M, B.rows):
                raise QlmError(1, "C must be float32 [M, N] with unit column stride")
            st = _stream_ptr(stream) if stream is not None else torch.cuda.current_stream(A.device).cuda_stream
            _check(lib.qlm_linear_int8(a2.data_ptr(), M, K, a2.stride(0), B.handle, c2.data_ptr(), c2.stride(0),
                                       flags & ~HOST_IO, st))
            return C
    a = np.asarray(A, dtype=np.float32)
    a2 = a if a.ndim == 2 else a.reshape(1, -1)
    if a2.strides[1] != 4:
        a2 = np.ascontiguousarray(a2)
    M, K = a2.shape
    if C is None:
        C = np.empty((M, B.rows), np.float32)
    c2 = C if C.ndim == 2 else C.reshape(1, -1)
    if c2.dtype != np.float32 or c2.strides[1] != 4 or c2.shape != (M, B.rows):
        raise QlmError(1, "C must be float32 [M, N] with unit column stride")
    _check(lib.qlm_linear_int8(_host_addr(a2), M, K, a2.strides[0] // 4, B.handle, _host_addr(c2),
                               c2.strides[0] // 4, flags | HOST_IO, _stream_ptr(stream)))
    return C


def prof_enable(on: bool | None = None) -> bool:
    """Switch per-matmul device timing on or off (None: only ask); returns the
    state before the call. The counterpart of QuickLM's QUICKLM_PROF switch
    (src/ops/math_ops.cpp:821-823), which also turns it on here."""
    return bool(load().qlm_prof_enable(-1 if on is None else int(bool(on))))


def prof_matmul_ms() -> tuple[float, int]:
    """(cumulative device ms, timed calls) of the linear entry points since the
    last reset — math::get_matmul_ms (src/ops/math_ops.hpp:85-87)."""
    ms, n = ctypes.c_double(), ctypes.c_int64()
    _check(load().qlm_prof_matmul_ms(ctypes.byref(ms), ctypes.byref(n)))
    return ms.value, n.value


def prof_reset() -> None:
    """Zero the totals — math::reset_matmul_ms (src/ops/math_ops.hpp:87)."""
    _check(load().qlm_prof_reset())


def prof_report() -> list[dict]:
    """Per-(entry point, M, N, K) totals, largest total first."""
    lib = load()
    need = ctypes.c_int64()
    _check(lib.qlm_prof_report(None, 0, ctypes.byref(need)))
    buf = ctypes.create_string_buffer(int(need.value) + 256)
    _check(lib.qlm_prof_report(buf, len(buf), ctypes.byref(need)))
    rows = []
    for line in buf.value.decode().splitlines():
        kind, m, n, k, calls, ms = line.split("\t")
        rows.append({"entry": kind, "M": int(m), "N": int(n), "K": int(k), "calls": int(calls), "ms": float(ms)})
    return rows


def shard_rows(n: int, nranks: int, rank: int):
    """Output rows [begin, end) that `rank` owns when n rows are split over
    nranks GPUs as evenly as possible (the first n % nranks ranks get one more)."""
    if not (0 <= rank < nranks):
        raise QlmError(1, f"rank {rank} not in [0, {nranks})")
    q, r = divmod(n, nranks)
    begin = rank * q + min(rank, r)
    return begin, begin + q + (1 if rank < r else 0)


def exchange_handles(local: bytes, nranks: int, exchange) -> bytes:
    """All ranks' exchange handles, in rank order, as one buffer for
    qlm_comm_connect. ``exchange(local)`` must return every rank's handle in
    rank order (e.g. ``all_gather_object`` over torch.distributed); each must
    be as long as this rank's."""
    handles = exchange(bytes(local))
    if handles is None or len(handles) != nranks or any(not isinstance(h, (bytes, bytearray)) or
                                                        len(h) != len(local) for h in handles):
        raise QlmError(1, "handle exchange returned the wrong number or size of handles")
    return b"".join(bytes(h) for h in handles)


class Comm:
    """One rank's NVLink exchange buffer for row-sharded outputs.

    ``exchange`` maps this rank's handle (bytes) to the list of every rank's
    handle in rank order — e.g. ``lambda h: all_gather_object(h)`` over
    torch.distributed; the data path itself never touches it."""

    def __init__(self, device: int, rank: int, nranks: int, max_out: int, exchange):
        lib = load()
        nb = lib.qlm_comm_handle_bytes()
        buf = ctypes.create_string_buffer(nb)
        h = ctypes.c_void_p()
        _check(lib.qlm_comm_create(device, rank, nranks, max_out, ctypes.byref(h), buf))
        self._h = h
        self.device, self.rank, self.nranks, self.max_out = device, rank, nranks, max_out
        try:
            allb = exchange_handles(buf.raw, nranks, exchange)
        except QlmError:
            self.free()
            raise
        _check(lib.qlm_comm_connect(self._h, ctypes.create_string_buffer(allb, len(allb))))

    def set_timeout(self, seconds: float) -> None:
        """Bound of every wait for a peer in later calls (default 2 s)."""
        _check(load().qlm_comm_set_timeout_us(self.handle, max(1, int(seconds * 1e6))))

    def status(self) -> None:
        """Raise QlmError (TIMEOUT) if a wait of this rank gave up; the
        communicator must then be freed and recreated on every rank."""
        _check(load().qlm_comm_status(self.handle))

    @property
    def handle(self):
        if not self._h:
            raise QlmError(1, "communicator already freed")
        return self._h

    def free(self) -> None:
        if self._h:
            load().qlm_comm_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def matmul_allgather(x, w: Int8Weight, comm: Comm, y=None, flags: int = 0, stream=None):
    """y[0:n_total] = x . W^T for a row-sharded W (this rank holds ``w``), the
    shards gathered over NVLink by the GEMV kernel. x: CUDA float32 [K] or
    [1, K]; y (allocated when None): CUDA float32 [1, n_total]."""
    import torch
    lib = load()
    a2 = x if x.dim() == 2 else x.view(1, -1)
    if a2.shape[0] != 1 or a2.dtype != torch.float32 or not a2.is_cuda:
        raise QlmError(1, "x must be a CUDA float32 row")
    if y is None:
        y = torch.empty((1, w.n_total), dtype=torch.float32, device=x.device)
    st = _stream_ptr(stream) if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
    _check(lib.qlm_linear_int8_allgather(a2.data_ptr(), 1, a2.shape[1], a2.stride(0), w.handle, comm.handle,
                                         y.data_ptr(), y.shape[-1], flags, st))
    return y


def argmax(logits, comm: "Comm" = None, col0: int = 0, stream=None):
    """Greedy token choice on the device, as QuickLM's
    DecoderModel::sample(logits, 0, 0) (model/model.cpp:259-272): 0 if logit 0
    is NaN, else the lowest index of the largest non-NaN logit. logits: CUDA
    float32 [n] or [1, n] — with ``comm`` (row-sharded lm_head) this rank's
    shard, whose first logit is global index ``col0``; every rank calls it and
    all get the choice over all shards. Returns (index, value); index is -1
    when no logit is a number. Synchronous."""
    import torch
    lib = load()
    v = logits.reshape(-1)
    if v.dtype != torch.float32 or not v.is_cuda or not v.is_contiguous():
        raise QlmError(1, "logits must be a contiguous CUDA float32 vector")
    out_i = torch.empty(1, dtype=torch.int32, device=v.device)
    out_v = torch.empty(1, dtype=torch.float32, device=v.device)
    st = _stream_ptr(stream) if stream is not None else torch.cuda.current_stream(v.device).cuda_stream
    with torch.cuda.device(v.device):
        _check(lib.qlm_argmax_f32(v.data_ptr(), v.numel(), int(col0), comm.handle if comm is not None else None,
                                  out_i.data_ptr(), out_v.data_ptr(), SYNC, st))
    return int(out_i.item()), float(out_v.item())


def _dev_f32(t, name):
    import torch
    if not (_is_torch(t) and t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()):
        raise QlmError(1, f"{name} must be a contiguous float32 CUDA tensor")
    return t


def _torch_stream(stream):
    import torch
    return _stream_ptr(stream) if stream is not None else torch.cuda.current_stream().cuda_stream


def rms_norm(x, w, eps: float, out=None, stream=None):
    """math::rms_norm on device rows of w.numel(): out = x * rsqrt(mean(x^2) + eps) * (1 + w)."""
    _dev_f32(x, "x"), _dev_f32(w, "w")
    size = w.numel()
    if x.numel() % size:
        raise QlmError(1, "x is not a whole number of rows")
    out = x.new_empty(x.shape) if out is None else _dev_f32(out, "out")
    _check(load().qlm_rms_norm(x.data_ptr(), w.data_ptr(), out.data_ptr(), x.numel() // size, size, eps,
                               _torch_stream(stream)))
    return out


def add_rms_norm(residual, delta, w, eps: float, out=None, stream=None):
    """math::add_rms_norm: residual += delta (in place); returns rms_norm(residual)."""
    _dev_f32(residual, "residual"), _dev_f32(delta, "delta"), _dev_f32(w, "w")
    size = w.numel()
    if residual.numel() % size or delta.numel() != residual.numel():
        raise QlmError(1, "residual/delta shapes do not match w")
    out = residual.new_empty(residual.shape) if out is None else _dev_f32(out, "out")
    _check(load().qlm_add_rms_norm(residual.data_ptr(), delta.data_ptr(), w.data_ptr(), out.data_ptr(),
                                   residual.numel() // size, size, eps, _torch_stream(stream)))
    return out


def add_then_rms_norm(residual, delta, w, eps: float, out=None, stream=None):
    """The decoder layer's unfused residual step (modules.hpp:228-231):
    math::elementwise_add(residual, delta) in place, then returns
    math::rms_norm(residual) — one launch, the bits of the two."""
    _dev_f32(residual, "residual"), _dev_f32(delta, "delta"), _dev_f32(w, "w")
    size = w.numel()
    if residual.numel() % size or delta.numel() != residual.numel():
        raise QlmError(1, "residual/delta shapes do not match w")
    out = residual.new_empty(residual.shape) if out is None else _dev_f32(out, "out")
    _check(load().qlm_add_then_rms_norm(residual.data_ptr(), delta.data_ptr(), w.data_ptr(), out.data_ptr(),
                                        residual.numel() // size, size, eps, _torch_stream(stream)))
    return out


def silu_mul(a, b, stream=None):
    """math::silu_mul: a = silu(a) * b in place (within 2 ulp of the reference)."""
    _dev_f32(a, "a"), _dev_f32(b, "b")
    if a.numel() != b.numel():
        raise QlmError(1, "a and b differ in size")
    _check(load().qlm_silu_mul(a.data_ptr(), b.data_ptr(), a.numel(), _torch_stream(stream)))
    return a


def silu(x, stream=None):
    """x = x / (1 + exp(-x)) in place (math::silu; within 2 ulp of the reference)."""
    _dev_f32(x, "x")
    _check(load().qlm_silu(x.data_ptr(), x.numel(), _torch_stream(stream)))
    return x


def conv1d_update_tapmajor(inp, state, oldest_tap: int, weight_t, out=None, stream=None):
    """One causal-conv step on a tap-major ring: state [ntaps, conv_dim], weight_t
    [ntaps + 1, conv_dim]; returns out [conv_dim]. The caller advances oldest_tap."""
    _dev_f32(inp, "input"), _dev_f32(state, "state"), _dev_f32(weight_t, "weight_t")
    conv_dim = inp.numel()
    ks = weight_t.shape[0]
    if weight_t.numel() != ks * conv_dim or state.numel() != (ks - 1) * conv_dim:
        raise QlmError(1, "state/weight_t shapes do not match the input")
    out = inp.new_empty(inp.shape) if out is None else _dev_f32(out, "out")
    _check(load().qlm_conv1d_update_tapmajor(inp.data_ptr(), state.data_ptr(), oldest_tap, weight_t.data_ptr(),
                                             out.data_ptr(), conv_dim, ks, _torch_stream(stream)))
    return out


def l2norm_heads(x, head_dim: int, eps: float = 1e-6, stream=None):
    """x_h /= sqrt(sumsq(x_h) + eps) in place for each head row of head_dim."""
    _dev_f32(x, "x")
    if x.numel() % head_dim:
        raise QlmError(1, "x is not a whole number of heads")
    _check(load().qlm_l2norm_heads(x.data_ptr(), x.numel() // head_dim, head_dim, eps, _torch_stream(stream)))
    return x


def gdn_gates(a_raw, b_raw, A_log, dt_bias, stream=None):
    """Per-head (decay, write gate) of the gated-delta-net step, as device tensors."""
    for t, nm in ((a_raw, "a_raw"), (b_raw, "b_raw"), (A_log, "A_log"), (dt_bias, "dt_bias")):
        _dev_f32(t, nm)
    heads = a_raw.numel()
    dec, beta = a_raw.new_empty(heads), a_raw.new_empty(heads)
    _check(load().qlm_gdn_gates(a_raw.data_ptr(), b_raw.data_ptr(), A_log.data_ptr(), dt_bias.data_ptr(),
                                dec.data_ptr(), beta.data_ptr(), heads, _torch_stream(stream)))
    return dec, beta


def gdn_recurrence(state, q, k, v, decay, beta, out=None, stream=None):
    """Gated delta rule for all heads: state [heads, d, d] updated in place; returns out [heads, d]."""
    for t, nm in ((state, "state"), (q, "q"), (k, "k"), (v, "v"), (decay, "decay"), (beta, "beta")):
        _dev_f32(t, nm)
    heads, d = state.shape[0], state.shape[-1]
    if state.numel() != heads * d * d or q.numel() != heads * d or k.numel() != heads * d or v.numel() != heads * d:
        raise QlmError(1, "state/q/k/v shapes do not match [heads, d, d] / [heads, d]")
    out = q.new_empty((heads, d)) if out is None else _dev_f32(out, "out")
    _check(load().qlm_gdn_recurrence(state.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), decay.data_ptr(),
                                     beta.data_ptr(), out.data_ptr(), heads, d, _torch_stream(stream)))
    return out


def rms_norm_gain(x, w, eps: float, out=None, stream=None):
    """rms_norm with a plain gain w (the gated-delta-net head norm)."""
    _dev_f32(x, "x"), _dev_f32(w, "w")
    size = w.numel()
    if x.numel() % size:
        raise QlmError(1, "x is not a whole number of rows")
    out = x.new_empty(x.shape) if out is None else _dev_f32(out, "out")
    _check(load().qlm_rms_norm_gain(x.data_ptr(), w.data_ptr(), out.data_ptr(), x.numel() // size, size, eps,
                                    _torch_stream(stream)))
    return out


def gqa_attend(q, k_cache, v_cache, pos: int, out=None, scratch=None, parallel: bool = True, stream=None):
    """GQA attention of one decode token: q [heads, q_stride] (query first), caches
    [T, kv_heads, d] with positions 0..pos valid; returns out [heads, d].
    parallel: spread over (head, position block) CTAs through a score scratch of
    heads * (pos + 1) floats (allocated when not given); same results."""
    for t, nm in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _dev_f32(t, nm)
    heads, q_stride = q.shape
    kv_heads, d = k_cache.shape[-2], k_cache.shape[-1]
    out = q.new_empty((heads, d)) if out is None else _dev_f32(out, "out")
    if parallel and scratch is None:
        scratch = q.new_empty(heads * (pos + 1))
    sp = scratch.data_ptr() if parallel else None
    _check(load().qlm_gqa_attend(q.data_ptr(), q_stride, k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(), pos,
                                 heads, kv_heads, d, sp, _torch_stream(stream)))
    return out


def rope_neox_tables(pos0: int, num_tokens: int, theta: float, rotary_dim: int):
    """Host cos/sin tables [num_tokens, rotary_dim/2] for positions pos0.., as the reference computes them."""
    c = np.empty((num_tokens, rotary_dim // 2), np.float32)
    s = np.empty_like(c)
    _check(load().qlm_rope_neox_tables(pos0, num_tokens, theta, rotary_dim, c.ctypes.data, s.ctypes.data))
    return c, s


def rope_neox(t, pos0: int, theta: float, rotary_dim: int, tables=None, stream=None):
    """math::apply_rope_neox in place on t [num_tokens, num_heads, head_dim] (token i at pos0 + i)."""
    import torch
    _dev_f32(t, "t")
    if t.dim() != 3:
        raise QlmError(1, "t must be [num_tokens, num_heads, head_dim]")
    n_tok, heads, head_dim = t.shape
    if tables is None:
        c, s = rope_neox_tables(pos0, n_tok, theta, rotary_dim)
        tables = (torch.from_numpy(c).to(t.device), torch.from_numpy(s).to(t.device))
    _check(load().qlm_rope_neox(t.data_ptr(), n_tok, heads, head_dim, rotary_dim, tables[0].data_ptr(),
                                tables[1].data_ptr(), _torch_stream(stream)))
    return t


def matmul_grouped(x, weights, ys=None, flags: int = 0, stream=None):
    """[x . W_g^T for W_g in weights] in one exact launch per 8 activation rows
    (weights that share x: q/k/v, gate/up; the int8 counterpart of QuickLM's
    bf16-only math::matmul_batched, ops/math_ops.cpp:902-954). x: CUDA float32
    [M, K]; weights: 1..8 Int8Weight on x's device with the same K; ys:
    optional list of CUDA float32 [M, rows_g] outputs. Bit-identical to
    matmul(x, W_g) for every g."""
    import torch
    lib = load()
    a2 = x if x.dim() == 2 else x.view(1, -1)
    if a2.dtype != torch.float32 or not a2.is_cuda or a2.stride(1) != 1:
        raise QlmError(1, "x must be a CUDA float32 matrix with unit column stride")
    if ys is None:
        ys = [torch.empty((a2.shape[0], w.rows), dtype=torch.float32, device=x.device) for w in weights]
    n = len(weights)
    hs = (ctypes.c_void_p * n)(*[w.handle for w in weights])
    yp = (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys])
    ld = (ctypes.c_int64 * n)(*[y.stride(0) for y in ys])
    st = _stream_ptr(stream) if stream is not None else torch.cuda.current_stream(x.device).cuda_stream
    _check(lib.qlm_linear_int8_grouped(a2.data_ptr(), a2.shape[0], a2.shape[1], a2.stride(0), hs, n, yp, ld, flags,
                                       st))
    return ys


class Model:
    """A QuickLM Qwen3.5-hybrid checkpoint decoded on the device (qlm_model_*):
    every activation stays in HBM; ``decode`` returns the greedy next token of
    each sequence (DecoderModel::forward + sample(logits, 0, 0),
    src/model/model.cpp:151-199, 259-272). ``batch`` sequences advance in
    lockstep (one position for all); each one's logits are bit-identical to
    decoding it alone."""

    def __init__(self, path: str, device: int = 0, max_seq: int = 2048, batch: int = 1):
        lib = load()
        h = ctypes.c_void_p()
        _check(lib.qlm_model_load_batch(os.fsencode(path), device, max_seq, batch, ctypes.byref(h)))
        self._h = h
        vals = [ctypes.c_int() for _ in range(5)]
        _check(lib.qlm_model_info(self._h, *[ctypes.byref(v) for v in vals]))
        self.vocab, self.hidden, self.layers, self.max_seq, self.batch = (v.value for v in vals)

    @property
    def handle(self):
        if not self._h:
            raise QlmError(1, "model already freed")
        return self._h

    def decode(self, tokens, pos: int, logits: bool = False):
        """One step at position ``pos``: tokens (``batch`` ints) in, the greedy
        next tokens out (and the logits [batch, vocab] when asked)."""
        toks = np.ascontiguousarray(np.asarray(tokens, np.int32).reshape(-1))
        if toks.size != self.batch:
            raise QlmError(1, f"{toks.size} tokens for a batch of {self.batch}")
        nxt = np.empty(self.batch, np.int32)
        lg = np.empty((self.batch, self.vocab), np.float32) if logits else None
        _check(load().qlm_model_decode_batch(self.handle, toks.ctypes.data, int(pos), nxt.ctypes.data,
                                             lg.ctypes.data if lg is not None else None))
        return (nxt, lg) if logits else nxt

    @property
    def stream(self) -> int:
        """The cudaStream_t (as an integer) every step runs on."""
        return int(load().qlm_model_stream(self.handle) or 0)

    def reset(self) -> None:
        """Clear the KV caches and recurrent states (DecoderModel::reset_states)."""
        _check(load().qlm_model_reset(self.handle))

    def free(self) -> None:
        if self._h:
            load().qlm_model_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
