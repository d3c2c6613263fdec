"""Python bindings of the streaming FastConformer encoder (include/cqencoder.h).

Mirrors the reference's StreamingEncoder API
(crates/nemotron-mlx/src/model/encoder.rs:567-655): tensors are bound by their
artifact names, a state carries the streaming caches of several lock-step
streams, and ``encode_chunk`` runs one chunk of all of them on the GPU.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import DTYPES, _check, _ptr, _stream_ptr, lib

CONFIG_FIELDS = ("hidden", "ff", "layers", "heads", "conv_kernel", "sliding_window", "mel_bins",
                 "sub_channels", "num_prompts", "prompt_hidden", "group_size")


class EncoderConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in CONFIG_FIELDS]

    @classmethod
    def default(cls, **overrides) -> "EncoderConfig":
        c = cls()
        lib().cq_encoder_default_config(ctypes.byref(c))
        for k, v in overrides.items():
            setattr(c, k, int(v))
        return c

    def as_dict(self) -> dict:
        return {n: int(getattr(self, n)) for n in CONFIG_FIELDS}


def _bits_dtype(dtype: str):
    return np.uint16


class Encoder:
    """The encoder's weights on one device (StreamingEncoder::from_artifact)."""

    def __init__(self, cfg: EncoderConfig | None = None, dtype: str = "bf16", device: int = 0):
        self.cfg = cfg if cfg is not None else EncoderConfig.default()
        self.dtype = dtype
        self.device = device
        h = ctypes.c_void_p()
        _check(lib().cq_encoder_create(ctypes.byref(self.cfg), DTYPES[dtype], device, ctypes.byref(h)))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                lib().cq_encoder_destroy(h)
            except TypeError:  # interpreter shutdown: module globals already cleared
                pass
            self._h = None

    @classmethod
    def random(cls, cfg: EncoderConfig | None = None, seed: int = 0, dtype: str = "bf16",
               device: int = 0) -> "Encoder":
        e = cls(cfg, dtype, device)
        _check(lib().cq_encoder_init_random(e._h, ctypes.c_uint64(seed)))
        return e

    def bind_artifact(self, artifact) -> None:
        """Binds every tensor from an opened Artifact (from_artifact)."""
        _check(lib().cq_encoder_bind_artifact(self._h, artifact._h))

    @classmethod
    def from_artifact(cls, artifact, cfg=None, dtype: str = "f16", device: int = 0) -> "Encoder":
        m = cls(cfg, dtype, device)
        m.bind_artifact(artifact)
        return m

    def tensor_names(self) -> list[str]:
        n = lib().cq_encoder_tensor_count(self._h)
        return [lib().cq_encoder_tensor_name(self._h, i).decode() for i in range(n)]

    def set_linear(self, name: str, q, s, b, bias, group_size: int) -> None:
        q8 = np.ascontiguousarray(q).view(np.uint8) if isinstance(q, np.ndarray) else None
        out, inp = (q8.shape if q8 is not None else (q.shape[0], q.shape[1] * 4))
        keep = [np.ascontiguousarray(a) if isinstance(a, np.ndarray) else a for a in (q, s, b, bias)]
        _check(lib().cq_encoder_set_linear(self._h, name.encode(), *[_ptr(a) for a in keep],
                                           out, inp, group_size))

    def set_tensor(self, name: str, values) -> None:
        v = np.ascontiguousarray(np.asarray(values, dtype=np.float32).reshape(-1))
        _check(lib().cq_encoder_set_tensor(self._h, name.encode(), _ptr(v), v.size))

    def get_tensor(self, name: str, size: int) -> np.ndarray:
        out = np.empty(size, dtype=np.float32)
        _check(lib().cq_encoder_get_tensor(self._h, name.encode(), _ptr(out), size))
        return out

    def linear_arrays(self, name: str):
        """Host copies (q u32 [N, K/4], scales, biases, bias T bits or None) of a bound linear."""
        h = lib().cq_encoder_linear(self._h, name.encode())
        if not h:
            raise KeyError(name)
        h = ctypes.c_void_p(h)
        n = lib().cq_linear_output_dims(h)
        k = lib().cq_linear_input_dims(h)
        g = lib().cq_linear_group_size(h)
        q = np.empty((n, k // 4), np.uint32)
        s = np.empty((n, k // g), np.uint16)
        b = np.empty_like(s)
        bias = np.empty(n, np.uint16)
        _check(lib().cq_linear_copy_arrays(h, _ptr(q), _ptr(s), _ptr(b), _ptr(bias)))
        return q, s, b, bias, g

    def export_params(self, oracle_linear_names, oracle_dense_names) -> dict:
        """Every tensor in the oracle's parameter format (tests)."""
        params = {}
        for name, (_, _, has_bias) in oracle_linear_names.items():
            q, s, b, bias, _ = self.linear_arrays(name)
            params[name] = (q, s, b, bias if has_bias else None)
        for name, shape in oracle_dense_names.items():
            params[name] = self.get_tensor(name, int(np.prod(shape))).reshape(shape)
        return params

    def state(self, streams: int = 1, max_mel_frames: int = 112) -> "EncoderState":
        return EncoderState(self, streams, max_mel_frames)


class EncoderState:
    """Streaming caches of `streams` lock-step utterances (StreamingEncoderCache)."""

    def __init__(self, encoder: Encoder, streams: int, max_mel_frames: int):
        self.encoder = encoder
        self.streams = streams
        h = ctypes.c_void_p()
        _check(lib().cq_encoder_state_create(encoder._h, streams, max_mel_frames, ctypes.byref(h)))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                lib().cq_encoder_state_destroy(h)
            except TypeError:  # interpreter shutdown: module globals already cleared
                pass
            self._h = None

    def set_prompts(self, ids) -> None:
        a = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
        _check(lib().cq_encoder_state_set_prompts(self._h, _ptr(a), a.size))

    def output_frames(self, mel_frames: int) -> int:
        return int(lib().cq_encoder_state_output_frames(self._h, mel_frames))

    @property
    def chunks(self) -> int:
        return int(lib().cq_encoder_state_chunks(self._h))

    @property
    def kernels_per_chunk(self) -> int:
        return int(lib().cq_encoder_state_kernels_per_chunk(self._h))

    def reset(self) -> None:
        _check(lib().cq_encoder_state_reset(self._h))

    def set_pdl(self, enable: bool = True) -> None:
        """Programmatic dependent launch between this state's kernels."""
        _check(lib().cq_encoder_state_set_pdl(self._h, int(enable)))

    def encode_chunk(self, mel, out=None, stream=None):
        """mel torch f32 [streams, frames, mel_bins] on the device -> out torch T
        [streams * encoder_frames, hidden]."""
        import torch
        s, t, _ = mel.shape
        frames = self.output_frames(t)
        if out is None:
            tdt = torch.bfloat16 if self.encoder.dtype == "bf16" else torch.float16
            out = torch.empty((s * frames, self.encoder.cfg.hidden), dtype=tdt, device=mel.device)
        _check(lib().cq_encoder_encode_chunk(self._h, _ptr(mel), t, _ptr(out), _stream_ptr(stream)))
        return out
