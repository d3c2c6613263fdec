"""Python bindings of the batched RNNT greedy decoder (include/cqrnnt.h).

Mirrors the reference's StreamingRnntDecoder
(crates/nemotron-mlx/src/model/rnnt.rs:336-388): tensors bound by artifact
name, a state holding the prediction networks of several streams, and
``decode_chunk`` running the greedy loop of one chunk on the GPU.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import DTYPES, _check, _ptr, _stream_ptr, lib

CONFIG_FIELDS = ("enc_hidden", "pred_hidden", "joint_hidden", "vocab", "blank", "lstm_layers",
                 "max_symbols", "group_size")


class RnntConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in CONFIG_FIELDS]

    @classmethod
    def default(cls, **overrides) -> "RnntConfig":
        c = cls()
        lib().cq_rnnt_default_config(ctypes.byref(c))
        for k, v in overrides.items():
            setattr(c, k, int(v))
        if "vocab" in overrides and "blank" not in overrides:
            c.blank = c.vocab - 1
        return c


class Rnnt:
    def __init__(self, cfg: RnntConfig | None = None, dtype: str = "bf16", device: int = 0):
        self.cfg = cfg if cfg is not None else RnntConfig.default()
        self.dtype, self.device = dtype, device
        h = ctypes.c_void_p()
        _check(lib().cq_rnnt_create(ctypes.byref(self.cfg), DTYPES[dtype], device, ctypes.byref(h)))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                lib().cq_rnnt_destroy(h)
            except TypeError:  # interpreter shutdown
                pass
            self._h = None

    @classmethod
    def random(cls, cfg: RnntConfig | None = None, seed: int = 0, dtype: str = "bf16",
               device: int = 0) -> "Rnnt":
        r = cls(cfg, dtype, device)
        _check(lib().cq_rnnt_init_random(r._h, ctypes.c_uint64(seed)))
        return r

    def set_fused_lstm(self, enable: bool = True) -> None:
        """One launch per LSTM layer step, or separate ih / hh / cell launches
        (same bits); for states created afterwards."""
        _check(lib().cq_rnnt_set_fused_lstm(self._h, int(enable)))

    def bind_artifact(self, artifact) -> None:
        """Binds every tensor from an opened Artifact (from_artifact)."""
        _check(lib().cq_rnnt_bind_artifact(self._h, artifact._h))

    @classmethod
    def from_artifact(cls, artifact, cfg=None, dtype: str = "f16", device: int = 0) -> "Rnnt":
        m = cls(cfg, dtype, device)
        m.bind_artifact(artifact)
        return m

    def tensor_names(self) -> list[str]:
        n = lib().cq_rnnt_tensor_count(self._h)
        return [lib().cq_rnnt_tensor_name(self._h, i).decode() for i in range(n)]

    def set_linear(self, name: str, q, s, b, bias, group_size: int) -> None:
        q8 = np.ascontiguousarray(q).view(np.uint8)
        keep = [None if a is None else np.ascontiguousarray(a) for a in (q, s, b, bias)]
        _check(lib().cq_rnnt_set_linear(self._h, name.encode(), *[_ptr(a) for a in keep],
                                        q8.shape[0], q8.shape[1], group_size))

    def set_tensor(self, name: str, values) -> None:
        v = np.ascontiguousarray(np.asarray(values, dtype=np.float32).reshape(-1))
        _check(lib().cq_rnnt_set_tensor(self._h, name.encode(), _ptr(v), v.size))

    def get_tensor(self, name: str, size: int) -> np.ndarray:
        out = np.empty(size, dtype=np.float32)
        _check(lib().cq_rnnt_get_tensor(self._h, name.encode(), _ptr(out), size))
        return out

    def linear_arrays(self, name: str):
        h = lib().cq_rnnt_linear(self._h, name.encode())
        if not h:
            raise KeyError(name)
        h = ctypes.c_void_p(h)
        n, k, g = (lib().cq_linear_output_dims(h), lib().cq_linear_input_dims(h),
                   lib().cq_linear_group_size(h))
        q = np.empty((n, k // 4), np.uint32)
        s = np.empty((n, k // g), np.uint16)
        b = np.empty_like(s)
        bias = np.empty(n, np.uint16)
        _check(lib().cq_linear_copy_arrays(h, _ptr(q), _ptr(s), _ptr(b), _ptr(bias)))
        return q, s, b, bias

    def export_params(self, linear_names: dict, dense_names: dict) -> dict:
        params = {}
        for name, (_, _, has_bias) in linear_names.items():
            q, s, b, bias = self.linear_arrays(name)
            params[name] = (q, s, b, bias if has_bias else None)
        for name, shape in dense_names.items():
            params[name] = self.get_tensor(name, int(np.prod(shape))).reshape(shape)
        return params

    def state(self, streams: int, max_frames: int = 14) -> "RnntState":
        return RnntState(self, streams, max_frames)


class RnntState:
    def __init__(self, rnnt: Rnnt, streams: int, max_frames: int):
        self.rnnt, self.streams = rnnt, streams
        h = ctypes.c_void_p()
        _check(lib().cq_rnnt_state_create(rnnt._h, streams, max_frames, ctypes.byref(h)))
        self._h = h
        self.capacity = int(lib().cq_rnnt_state_capacity(h))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                lib().cq_rnnt_state_destroy(h)
            except TypeError:
                pass
            self._h = None

    @property
    def kernels_per_chunk(self) -> int:
        return int(lib().cq_rnnt_state_kernels_per_chunk(self._h))

    def set_persistent(self, enable: bool = True) -> None:
        """One persistent launch per chunk (early exit on all-blank frames)."""
        _check(lib().cq_rnnt_state_set_persistent(self._h, int(enable)))

    def reset(self) -> None:
        _check(lib().cq_rnnt_state_reset(self._h))

    def set_pdl(self, enable: bool = True) -> None:
        """Programmatic dependent launch between this state's kernels."""
        _check(lib().cq_rnnt_state_set_pdl(self._h, int(enable)))

    def decode_chunk_raw(self, encoded, frames: int, tokens, token_frames, counts, stream=None):
        """Device tensors in and out (no synchronisation)."""
        _check(lib().cq_rnnt_decode_chunk(self._h, _ptr(encoded), encoded.stride(0), frames,
                                          _ptr(tokens), _ptr(token_frames), _ptr(counts),
                                          _stream_ptr(stream)))

    def decode_chunk(self, encoded, frames: int, stream=None) -> list[list[tuple[int, int]]]:
        """encoded torch T [streams * frames, enc_hidden] -> per stream [(token, frame)]."""
        import torch
        dev = encoded.device
        tokens = torch.empty((self.streams, self.capacity), dtype=torch.int32, device=dev)
        token_frames = torch.empty_like(tokens)
        counts = torch.empty((self.streams,), dtype=torch.int32, device=dev)
        self.decode_chunk_raw(encoded, frames, tokens, token_frames, counts, stream)
        torch.cuda.synchronize()
        t, f, n = tokens.cpu().numpy(), token_frames.cpu().numpy(), counts.cpu().numpy()
        return [list(zip(t[s, :n[s]].tolist(), f[s, :n[s]].tolist())) for s in range(self.streams)]
