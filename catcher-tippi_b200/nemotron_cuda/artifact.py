"""Python bindings of the release-artifact reader (include/cqartifact.h).

Mirrors the reference's Artifact (crates/nemotron-mlx/src/weights/
artifact.rs:156-252): ``Artifact(path)`` parses manifest.json and maps
weights.safetensors; ``tensor_info``/``f16_to_f32`` read it on the host, and
``Encoder.bind_artifact``/``Rnnt.bind_artifact``/``QuantizedLinear.from_artifact``
bind its tensors on a device.
"""
from __future__ import annotations

import ctypes
from typing import NamedTuple

import numpy as np

from . import _check, _ptr, lib

STORAGES = {0: "Int8Affine", 1: "F16", 2: "F32", 3: "I32"}


class TensorInfo(NamedTuple):
    shape: tuple
    storage: str
    group_size: int  # 0 unless Int8Affine


class Artifact:
    def __init__(self, path: str):
        h = ctypes.c_void_p()
        _check(lib().cq_artifact_open(str(path).encode(), ctypes.byref(h)))
        self._h = h

    def close(self) -> None:
        if getattr(self, "_h", None):
            try:
                lib().cq_artifact_close(self._h)
            except TypeError:  # interpreter shutdown
                pass
            self._h = None

    def __del__(self):
        self.close()

    def __enter__(self) -> "Artifact":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    @property
    def model_id(self) -> str:
        return lib().cq_artifact_model_id(self._h).decode()

    @property
    def format_version(self) -> int:
        return int(lib().cq_artifact_format_version(self._h))

    def tensor_names(self) -> list[str]:
        n = lib().cq_artifact_tensor_count(self._h)
        return [lib().cq_artifact_tensor_name(self._h, i).decode() for i in range(n)]

    def tensor_info(self, name: str) -> TensorInfo:
        rank, storage, group = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        shape = (ctypes.c_int64 * 8)()
        _check(lib().cq_artifact_tensor_info(self._h, name.encode(), ctypes.byref(rank), shape, 8,
                                             ctypes.byref(storage), ctypes.byref(group)))
        return TensorInfo(tuple(int(shape[i]) for i in range(min(rank.value, 8))),
                          STORAGES[storage.value], int(group.value))

    def f16_to_f32(self, name: str) -> np.ndarray:
        n = int(np.prod(self.tensor_info(name).shape))
        out = np.empty(n, dtype=np.float32)
        _check(lib().cq_artifact_f16_to_f32(self._h, name.encode(), _ptr(out), n))
        return out
