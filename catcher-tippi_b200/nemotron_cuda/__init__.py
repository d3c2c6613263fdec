"""Python bindings of the B200 affine INT8 quantized linear (libcqlinear.so).

A thin ctypes layer over the C ABI in include/cqlinear.h, mirroring the
reference's Rust layer API (crates/nemotron-mlx/src/model/layers.rs:208-352
and crates/nemotron-mlx/src/backend/mod.rs:41-94) so the tests and the
benchmark read like the reference's own.  There is no CPU fallback: importing
works without a GPU (for ABI and validation tests), but every compute call
goes through the CUDA library and fails loudly if it cannot run.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcqlinear.so")

CQ_OK, CQ_INVALID_ARGUMENT, CQ_RUNTIME_ERROR = 0, -1, -3
DTYPES = {"f16": 0, "bf16": 1, "f32": 2}
ACTS = {"none": 0, "silu": 1, "relu": 2}

_lib = None


class CQError(RuntimeError):
    """A failed C-ABI call: `status` is the cq_status, str() the library's message."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing; run catcher-tippi_b200/build.py")
    L = ctypes.CDLL(LIB_PATH)
    vp, i32, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t
    pp = ctypes.POINTER(ctypes.c_void_p)
    sig = {
        "cq_last_error": ([], ctypes.c_char_p),
        "cq_version": ([], ctypes.c_char_p),
        "cq_is_device_available": ([], i32),
        "cq_linear_create": ([vp, vp, vp, vp, i32, i32, i32, i32, i32, pp], i32),
        "cq_linear_create_from_f32": ([vp, sz, i32, i32, vp, sz, i32, i32, i32, pp], i32),
        "cq_linear_concat": ([vp, i32, pp], i32),
        "cq_linear_forward": ([vp, vp, i32, vp, vp], i32),
        "cq_linear_forward_ex": ([vp, vp, i32, i32, vp, i32, i32, vp], i32),
        "cq_linear_forward_f32": ([vp, vp, sz, i32, vp, sz], i32),
        "cq_linear_reserve": ([vp, i32], i32),
        "cq_linear_forward_noalloc": ([vp, vp, i32, i32, vp, i32, i32, vp], i32),
        "cq_linear_prescale_activations": ([vp, vp, i32, i32, vp, vp, vp], i32),
        "cq_linear_forward_prescaled": ([vp, vp, vp, i32, vp, i32, i32, vp], i32),
        "cq_linear_input_dims": ([vp], i32),
        "cq_linear_output_dims": ([vp], i32),
        "cq_linear_group_size": ([vp], i32),
        "cq_linear_dtype": ([vp], i32),
        "cq_linear_device_arrays": ([vp, pp, pp, pp, pp], i32),
        "cq_linear_copy_arrays": ([vp, vp, vp, vp, vp], i32),
        "cq_linear_destroy": ([vp], None),
        "cq_quantized_matmul": ([vp, sz, sz, sz, vp, sz, sz, sz, vp, sz], i32),
        "cq_quantize": ([vp, i32, i32, i32, i32, i32, vp, vp, vp, vp], i32),
        "cq_dequantize": ([vp, vp, vp, i32, i32, i32, i32, vp, vp], i32),
        "cq_device_status": ([i32, ctypes.POINTER(ctypes.c_int32)], i32),
        "cq_device_watchdog_check": ([i32], i32),
        # streaming encoder (include/cqencoder.h)
        "cq_encoder_default_config": ([vp], None),
        "cq_encoder_create": ([vp, i32, i32, pp], i32),
        "cq_encoder_set_linear": ([vp, ctypes.c_char_p, vp, vp, vp, vp, i32, i32, i32], i32),
        "cq_encoder_set_tensor": ([vp, ctypes.c_char_p, vp, sz], i32),
        "cq_encoder_get_tensor": ([vp, ctypes.c_char_p, vp, sz], i32),
        "cq_encoder_linear": ([vp, ctypes.c_char_p], vp),
        "cq_encoder_init_random": ([vp, ctypes.c_uint64], i32),
        "cq_encoder_tensor_count": ([vp], i32),
        "cq_encoder_tensor_name": ([vp, i32], ctypes.c_char_p),
        "cq_encoder_destroy": ([vp], None),
        "cq_encoder_state_create": ([vp, i32, i32, pp], i32),
        "cq_encoder_state_set_prompts": ([vp, vp, i32], i32),
        "cq_encoder_state_output_frames": ([vp, i32], i32),
        "cq_encoder_encode_chunk": ([vp, vp, i32, vp, vp], i32),
        "cq_encoder_state_chunks": ([vp], i32),
        "cq_encoder_state_kernels_per_chunk": ([vp], i32),
        "cq_encoder_state_reset": ([vp], i32),
        "cq_encoder_state_set_pdl": ([vp, i32], i32),
        "cq_encoder_state_destroy": ([vp], None),
        # batched RNNT decoder (include/cqrnnt.h)
        "cq_rnnt_default_config": ([vp], None),
        "cq_rnnt_create": ([vp, i32, i32, pp], i32),
        "cq_rnnt_set_linear": ([vp, ctypes.c_char_p, vp, vp, vp, vp, i32, i32, i32], i32),
        "cq_rnnt_set_tensor": ([vp, ctypes.c_char_p, vp, sz], i32),
        "cq_rnnt_get_tensor": ([vp, ctypes.c_char_p, vp, sz], i32),
        "cq_rnnt_linear": ([vp, ctypes.c_char_p], vp),
        "cq_rnnt_init_random": ([vp, ctypes.c_uint64], i32),
        "cq_rnnt_set_fused_lstm": ([vp, i32], i32),
        "cq_rnnt_tensor_count": ([vp], i32),
        "cq_rnnt_tensor_name": ([vp, i32], ctypes.c_char_p),
        "cq_rnnt_destroy": ([vp], None),
        "cq_rnnt_state_create": ([vp, i32, i32, pp], i32),
        "cq_rnnt_state_capacity": ([vp], i32),
        "cq_rnnt_decode_chunk": ([vp, vp, i32, i32, vp, vp, vp, vp], i32),
        "cq_rnnt_state_kernels_per_chunk": ([vp], i32),
        "cq_rnnt_state_set_persistent": ([vp, i32], i32),
        "cq_rnnt_state_set_pdl": ([vp, i32], i32),
        "cq_rnnt_state_reset": ([vp], i32),
        "cq_rnnt_state_destroy": ([vp], None),
        # release artifacts (include/cqartifact.h)
        "cq_artifact_open": ([ctypes.c_char_p, pp], i32),
        "cq_artifact_close": ([vp], None),
        "cq_artifact_model_id": ([vp], ctypes.c_char_p),
        "cq_artifact_format_version": ([vp], i32),
        "cq_artifact_tensor_count": ([vp], i32),
        "cq_artifact_tensor_name": ([vp, i32], ctypes.c_char_p),
        "cq_artifact_tensor_info": ([vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int32),
                                     ctypes.POINTER(ctypes.c_int64), i32,
                                     ctypes.POINTER(ctypes.c_int32),
                                     ctypes.POINTER(ctypes.c_int32)], i32),
        "cq_artifact_f16_to_f32": ([vp, ctypes.c_char_p, vp, sz], i32),
        "cq_linear_from_artifact": ([vp, ctypes.c_char_p, ctypes.c_char_p, i32, i32, pp], i32),
        "cq_encoder_bind_artifact": ([vp, vp], i32),
        "cq_rnnt_bind_artifact": ([vp, vp], i32),
        # log-mel frontend (include/cqlogmel.h)
        "cq_logmel_create": ([i32, i32, i32, i32, i32, ctypes.c_float, i32, pp], i32),
        "cq_logmel_create_nemotron": ([i32, pp], i32),
        "cq_logmel_frames": ([vp, ctypes.c_int64, i32], ctypes.c_int64),
        "cq_logmel_mel_bins": ([vp], i32),
        "cq_logmel_window": ([vp, vp, sz], i32),
        "cq_logmel_filters": ([vp, vp, sz], i32),
        "cq_logmel_extract": ([vp, vp, i32, ctypes.c_int64, ctypes.c_int64, i32, vp, vp], i32),
        "cq_logmel_destroy": ([vp], None),
        # streaming scheduler and tokenizer (include/cqstream.h)
        "cq_chunk_scheduler_create": ([i32, pp], i32),
        "cq_chunk_scheduler_push": ([vp, vp, sz, ctypes.POINTER(ctypes.c_int32)], i32),
        "cq_chunk_scheduler_finish": ([vp, ctypes.POINTER(ctypes.c_int32)], i32),
        "cq_chunk_scheduler_window": ([vp, i32, vp, sz, ctypes.POINTER(ctypes.c_size_t),
                                       ctypes.POINTER(ctypes.c_int32),
                                       ctypes.POINTER(ctypes.c_int32)], i32),
        "cq_chunk_scheduler_reset": ([vp], i32),
        "cq_chunk_scheduler_destroy": ([vp], None),
        "cq_tokenizer_from_json": ([ctypes.c_char_p, ctypes.c_uint32, ctypes.c_uint32, pp], i32),
        "cq_tokenizer_decode": ([vp, vp, sz, i32, ctypes.POINTER(ctypes.c_char_p)], i32),
        "cq_tokenizer_destroy": ([vp], None),
        # transcription ABI (include/catcher.h)
        "catcher_create": ([ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_uint32], vp),
        "catcher_create_config": ([ctypes.c_char_p, ctypes.c_char_p, ctypes.c_uint32, vp, vp, i32,
                                   i32], vp),
        "catcher_start": ([vp], i32),
        "catcher_push_audio": ([vp, vp, sz], i32),
        "catcher_finish": ([vp], i32),
        "catcher_finish_before": ([vp, ctypes.c_uint64], i32),
        "catcher_text": ([vp], ctypes.c_char_p),
        "catcher_text_before": ([vp, ctypes.c_uint64], ctypes.c_char_p),
        "catcher_segments": ([vp], ctypes.c_char_p),
        "catcher_warning": ([vp], ctypes.c_char_p),
        "catcher_last_error": ([vp], ctypes.c_char_p),
        "catcher_destroy": ([vp], None),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def _check(status: int) -> None:
    if status != CQ_OK:
        raise CQError(status, lib().cq_last_error().decode())


def last_error() -> str:
    return lib().cq_last_error().decode()


def version() -> str:
    return lib().cq_version().decode()


def is_device_available() -> bool:
    return bool(lib().cq_is_device_available())


def _ptr(a) -> ctypes.c_void_p | None:
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return ctypes.c_void_p(a.ctypes.data)
    return ctypes.c_void_p(a.data_ptr())  # torch tensor


def _stream_ptr(stream) -> ctypes.c_void_p | None:
    if stream is None:
        import torch
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if isinstance(stream, int):
        return ctypes.c_void_p(stream)
    return ctypes.c_void_p(stream.cuda_stream)


def device_status(device: int = 0) -> int:
    """Reads and clears the device watchdog word (0 = clean)."""
    v = ctypes.c_int32(0)
    _check(lib().cq_device_status(device, ctypes.byref(v)))
    return int(v.value)


class QuantizedLinear:
    """Affine INT8 linear bound to one CUDA device (QuantizedLinear, layers.rs:208-319)."""

    def __init__(self, handle: ctypes.c_void_p):
        self._h = handle

    # -- construction -------------------------------------------------------
    @classmethod
    def from_packed(cls, qweight: np.ndarray, scales: np.ndarray, biases: np.ndarray,
                    bias: np.ndarray | None, group_size: int, dtype: str = "bf16",
                    device: int = 0) -> "QuantizedLinear":
        """Packed host arrays (u32 [N, K/4]; T bits [N, K/g]) -> device layer (from_artifact)."""
        q = np.ascontiguousarray(qweight, dtype=np.uint32)
        s = np.ascontiguousarray(scales)
        b = np.ascontiguousarray(biases)
        bb = None if bias is None else np.ascontiguousarray(bias)
        n, k4 = q.shape
        h = ctypes.c_void_p()
        _check(lib().cq_linear_create(_ptr(q), _ptr(s), _ptr(b), _ptr(bb), n, k4 * 4, group_size,
                                      DTYPES[dtype], device, ctypes.byref(h)))
        return cls(h)

    @classmethod
    def from_device(cls, qweight, scales, biases, bias, group_size: int, dtype: str = "bf16",
                    device: int = 0) -> "QuantizedLinear":
        """Packed torch device tensors (q int32/uint32 [N, K/4]; scales/biases T) -> layer copy."""
        n, k4 = qweight.shape
        h = ctypes.c_void_p()
        _check(lib().cq_linear_create(_ptr(qweight), _ptr(scales), _ptr(biases), _ptr(bias), n,
                                      k4 * 4, group_size, DTYPES[dtype], device, ctypes.byref(h)))
        return cls(h)

    @classmethod
    def from_artifact(cls, artifact, weight_name: str, bias_name: str | None = None,
                      dtype: str = "f16", device: int = 0) -> "QuantizedLinear":
        """QuantizedLinear::from_artifact (layers.rs:222-256) from an opened Artifact."""
        h = ctypes.c_void_p()
        _check(lib().cq_linear_from_artifact(artifact._h, weight_name.encode(),
                                             None if bias_name is None else bias_name.encode(),
                                             DTYPES[dtype], device, ctypes.byref(h)))
        return cls(h)

    @classmethod
    def from_f32(cls, weight, output_dims: int, input_dims: int, bias, group_size: int,
                 dtype: str = "f16", device: int = 0) -> "QuantizedLinear":
        """Quantise an f32 row-major weight on the device (from_f32, layers.rs:259-280)."""
        w = np.ascontiguousarray(np.asarray(weight, dtype=np.float32).reshape(-1))
        bb = np.ascontiguousarray(np.asarray(bias, dtype=np.float32).reshape(-1))
        h = ctypes.c_void_p()
        _check(lib().cq_linear_create_from_f32(_ptr(w), w.size, output_dims, input_dims, _ptr(bb),
                                               bb.size, group_size, DTYPES[dtype], device,
                                               ctypes.byref(h)))
        return cls(h)

    @classmethod
    def concat(cls, parts: list["QuantizedLinear"]) -> "QuantizedLinear":
        arr = (ctypes.c_void_p * len(parts))(*[p._h for p in parts])
        h = ctypes.c_void_p()
        _check(lib().cq_linear_concat(ctypes.cast(arr, ctypes.c_void_p), len(parts),
                                      ctypes.byref(h)))
        return cls(h)

    # -- properties ---------------------------------------------------------
    @property
    def input_dims(self) -> int:
        return int(lib().cq_linear_input_dims(self._h))

    @property
    def output_dims(self) -> int:
        return int(lib().cq_linear_output_dims(self._h))

    @property
    def group_size(self) -> int:
        return int(lib().cq_linear_group_size(self._h))

    @property
    def dtype(self) -> str:
        code = int(lib().cq_linear_dtype(self._h))
        return {v: k for k, v in DTYPES.items()}[code]

    def device_arrays(self) -> tuple[int, int, int, int]:
        ptrs = [ctypes.c_void_p() for _ in range(4)]
        _check(lib().cq_linear_device_arrays(self._h, *[ctypes.byref(p) for p in ptrs]))
        return tuple(int(p.value or 0) for p in ptrs)

    # -- compute ------------------------------------------------------------
    def forward(self, x, y=None, act: str = "none", stream=None, rows: int | None = None):
        """Device forward (forward_array): x torch [M, >=K] in T -> y torch [M, >=N] in T."""
        import torch
        m = x.shape[0] if rows is None else rows
        if y is None:
            y = torch.empty((m, self.output_dims), dtype=x.dtype, device=x.device)
        _check(lib().cq_linear_forward_ex(self._h, _ptr(x), x.stride(0), m, _ptr(y), y.stride(0),
                                          ACTS[act], _stream_ptr(stream)))
        return y

    def reserve(self, max_rows: int) -> None:
        """Allocate the batched-path workspace now (before graph capture)."""
        _check(lib().cq_linear_reserve(self._h, max_rows))

    def forward_raw(self, x_ptr: int, ldx: int, rows: int, y_ptr: int, ldy: int,
                    act: str = "none", stream: int = 0) -> None:
        _check(lib().cq_linear_forward_ex(self._h, ctypes.c_void_p(x_ptr), ldx, rows,
                                          ctypes.c_void_p(y_ptr), ldy, ACTS[act],
                                          ctypes.c_void_p(stream)))

    def prescale_activations(self, x, rows: int | None = None, stream=None):
        """The tensor-core GEMM's activation format for x bf16 [M, >=K] (bf16
        layers, M >= 256): returns (x16 f16 [M, K], row_scale f32 [M])."""
        import torch
        m = x.shape[0] if rows is None else rows
        x16 = torch.empty((m, self.input_dims), dtype=torch.float16, device=x.device)
        rs = torch.empty((m,), dtype=torch.float32, device=x.device)
        _check(lib().cq_linear_prescale_activations(self._h, _ptr(x), x.stride(0), m, _ptr(x16),
                                                    _ptr(rs), _stream_ptr(stream)))
        return x16, rs

    def forward_prescaled(self, x16, row_scale, y=None, act: str = "none", stream=None,
                          rows: int | None = None):
        """forward on activations from prescale_activations (bit-identical to forward)."""
        import torch
        m = x16.shape[0] if rows is None else rows
        if y is None:
            y = torch.empty((m, self.output_dims), dtype=torch.bfloat16, device=x16.device)
        _check(lib().cq_linear_forward_prescaled(self._h, _ptr(x16), _ptr(row_scale), m, _ptr(y),
                                                 y.stride(0), ACTS[act], _stream_ptr(stream)))
        return y

    def forward_f32(self, input, rows: int) -> np.ndarray:
        """Host f32 in / out (forward_f32, layers.rs:283-296)."""
        x = np.ascontiguousarray(np.asarray(input, dtype=np.float32).reshape(-1))
        out = np.empty(max(rows, 0) * self.output_dims, dtype=np.float32)
        _check(lib().cq_linear_forward_f32(self._h, _ptr(x), x.size, rows, _ptr(out), out.size))
        return out

    def close(self) -> None:
        if self._h:
            lib().cq_linear_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PointwiseConv1d:
    """Quantized 1x1 convolution over [batch, time, channels] (layers.rs:321-352)."""

    def __init__(self, linear: QuantizedLinear):
        self.linear = linear

    @classmethod
    def from_device(cls, qweight, scales, biases, bias, group_size: int, dtype: str = "bf16",
                    device: int = 0) -> "PointwiseConv1d":
        return cls(QuantizedLinear.from_device(qweight, scales, biases, bias, group_size, dtype,
                                               device))

    @classmethod
    def from_f32(cls, weight, output_dims, input_dims, bias, group_size, dtype="f16", device=0):
        return cls(QuantizedLinear.from_f32(weight, output_dims, input_dims, bias, group_size,
                                            dtype, device))

    def forward_f32(self, input, batch: int, time: int):
        values = self.linear.forward_f32(input, batch * time)
        return values.reshape(batch, time, self.linear.output_dims)


def quantized_matmul(input, rows: int, input_dims: int, weight, output_dims: int,
                     group_size: int) -> np.ndarray:
    """backend::quantized_matmul (backend/mod.rs:41-94): f32 in, f32 out."""
    x = np.ascontiguousarray(np.asarray(input, dtype=np.float32).reshape(-1))
    w = np.ascontiguousarray(np.asarray(weight, dtype=np.float32).reshape(-1))
    out = np.empty(max(rows * output_dims, 0), dtype=np.float32)
    _check(lib().cq_quantized_matmul(_ptr(x), x.size, rows, input_dims, _ptr(w), w.size,
                                     output_dims, group_size, _ptr(out), out.size))
    return out


def quantize(w, group_size: int, dtype: str, round_input: bool = True, stream=None):
    """Device affine quantisation of a torch f32 [N, K] tensor -> (q u32, scales, biases)."""
    import torch
    n, k = w.shape
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[dtype]
    q = torch.empty((n, k // 4), dtype=torch.int32, device=w.device)
    s = torch.empty((n, k // group_size), dtype=tdt, device=w.device)
    b = torch.empty_like(s)
    _check(lib().cq_quantize(_ptr(w), n, k, group_size, DTYPES[dtype], int(round_input), _ptr(q),
                             _ptr(s), _ptr(b), _stream_ptr(stream)))
    return q, s, b


def dequantize(q, s, b, group_size: int, dtype: str, stream=None):
    import torch
    n = q.shape[0]
    k = q.shape[1] * 4
    w = torch.empty((n, k), dtype=torch.float32, device=q.device)
    _check(lib().cq_dequantize(_ptr(q), _ptr(s), _ptr(b), n, k, group_size, DTYPES[dtype], _ptr(w),
                               _stream_ptr(stream)))
    return w
