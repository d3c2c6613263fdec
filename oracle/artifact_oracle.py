"""CPU oracle of the MLX release artifact format -- TEST INFRASTRUCTURE ONLY.

Only tests/ may import this module.  It restates, in numpy:

* the artifact writer convert_tensors (crates/nemotron-mlx/src/weights/
  artifact.rs:258-330): every Int8Affine tensor is cast to f16 and
  affine-quantised with 8 bits (MLX quantize, restated by oracle.quantize) into
  "{name}.__qweight" (U32 [N, K/4]), "{name}.__scales" and "{name}.__biases"
  (F16 [N, K/g]); every F16 tensor is cast to f16 under its own name; the
  manifest records format_version 1, the model id and, per tensor, its
  artifact shape and storage (serde's external tagging: "F16" or
  {"Int8Affine": {"group_size": g}});
* the safetensors container MLX writes: an 8-byte little-endian header size, a
  JSON header {name: {dtype, shape, data_offsets}} padded with spaces to a
  multiple of 8 bytes, then the arrays back to back;
* the reader side (Artifact::load, quantized_arrays, f16_to_f32, f16_array;
  artifact.rs:156-252), used to hand the same tensors to the encoder and RNNT
  oracles that the CUDA loader binds.

Parity of this restatement is pinned by the reference's own artifact test
(crates/nemotron-mlx/tests/encoder_artifact.rs:14-242): the same tensor set,
shapes, storage policies and group size are written here and read back by both
this reader and the library.
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

import oracle as qo

FORMAT_VERSION = 1
WEIGHTS_FILE = "weights.safetensors"
MANIFEST_FILE = "manifest.json"

_ST_DTYPES = {np.dtype(np.float16): "F16", np.dtype(np.float32): "F32",
              np.dtype(np.uint32): "U32", np.dtype(np.int32): "I32"}
_NP_DTYPES = {v: k for k, v in _ST_DTYPES.items()}


def int8_affine(group_size: int) -> dict:
    return {"Int8Affine": {"group_size": int(group_size)}}


F16 = "F16"


def save_safetensors(path: str, arrays: dict) -> None:
    """The safetensors container (header, padding, data), arrays in name order."""
    header, blobs, offset = {}, [], 0
    for name in sorted(arrays):
        a = np.ascontiguousarray(arrays[name])
        raw = a.tobytes()
        header[name] = {"dtype": _ST_DTYPES[a.dtype], "shape": list(a.shape),
                        "data_offsets": [offset, offset + len(raw)]}
        blobs.append(raw)
        offset += len(raw)
    text = json.dumps(header, separators=(",", ":")).encode()
    text += b" " * ((-len(text)) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for raw in blobs:
            f.write(raw)


def load_safetensors(path: str) -> dict:
    with open(path, "rb") as f:
        data = f.read()
    (n,) = struct.unpack("<Q", data[:8])
    header = json.loads(data[8:8 + n])
    body = data[8 + n:]
    out = {}
    for name, e in header.items():
        if name == "__metadata__":
            continue
        b0, b1 = e["data_offsets"]
        out[name] = np.frombuffer(body[b0:b1], dtype=_NP_DTYPES[e["dtype"]]).reshape(e["shape"])
    return out


def convert_tensors(out_dir: str, model_id: str, specs: list) -> None:
    """convert_tensors: specs are (name, f32 source array, artifact_shape, storage)."""
    if os.path.exists(out_dir):
        raise FileExistsError(f"artifact output already exists: {out_dir}")
    os.makedirs(out_dir)
    arrays, tensors = {}, {}
    for name, source, shape, storage in specs:
        runtime = np.asarray(source, dtype=np.float32).reshape(shape)
        if isinstance(storage, dict):
            g = storage["Int8Affine"]["group_size"]
            q, s, b = qo.quantize(runtime, g, "f16")
            arrays[f"{name}.__qweight"] = q
            arrays[f"{name}.__scales"] = s.view(np.float16)
            arrays[f"{name}.__biases"] = b.view(np.float16)
        elif storage == F16:
            arrays[name] = runtime.astype(np.float16)
        else:
            raise ValueError(f"unsupported artifact storage for {name}: {storage}")
        tensors[name] = {"shape": [int(d) for d in shape], "storage": storage}
    save_safetensors(os.path.join(out_dir, WEIGHTS_FILE), arrays)
    manifest = {"format_version": FORMAT_VERSION, "model_id": model_id, "tensors": tensors}
    with open(os.path.join(out_dir, MANIFEST_FILE), "w") as f:
        json.dump(manifest, f, indent=2)


class Artifact:
    """Artifact::load and its accessors."""

    def __init__(self, path: str):
        with open(os.path.join(path, MANIFEST_FILE)) as f:
            self.manifest = json.load(f)
        self.arrays = load_safetensors(os.path.join(path, WEIGHTS_FILE))

    def tensor_info(self, name: str):
        return self.manifest["tensors"].get(name)

    def _require_tensor(self, name: str) -> dict:
        t = self.tensor_info(name)
        if t is None:
            raise KeyError(f"missing artifact tensor {name}")
        return t

    def _require_array(self, name: str) -> np.ndarray:
        if name not in self.arrays:
            raise KeyError(f"missing artifact array {name}")
        return self.arrays[name]

    def quantized_arrays(self, name: str):
        """(q u32 [N, K/4], scales f16 bits, biases f16 bits, group, shape)."""
        t = self._require_tensor(name)
        if not isinstance(t["storage"], dict):
            raise TypeError(f"tensor {name} has incompatible storage {t['storage']}")
        g = t["storage"]["Int8Affine"]["group_size"]
        return (self._require_array(f"{name}.__qweight"),
                self._require_array(f"{name}.__scales").view(np.uint16),
                self._require_array(f"{name}.__biases").view(np.uint16), g, t["shape"])

    def f16_array(self, name: str) -> np.ndarray:
        t = self._require_tensor(name)
        if t["storage"] != F16:
            raise TypeError(f"tensor {name} has incompatible storage {t['storage']}")
        return self._require_array(name)

    def f16_to_f32(self, name: str) -> np.ndarray:
        return self.f16_array(name).astype(np.float32).reshape(-1)


def _t_bits(bits_f16: np.ndarray, dtype: str) -> np.ndarray:
    """F16 bit patterns -> T bit patterns (bf16: round to nearest even)."""
    if dtype == "f16":
        return np.ascontiguousarray(bits_f16)
    return qo.to_t(bits_f16.view(np.float16).astype(np.float32), dtype)


def model_params(art: Artifact, linear_names: dict, dense_names: dict, dtype: str) -> dict:
    """The oracle parameter dict of a model bound from an artifact: linears as
    (q, scales, biases, output bias | None) in T, dense tensors as f32."""
    params = {}
    for name, (n, k, has_bias) in linear_names.items():
        q, s, b, g, shape = art.quantized_arrays(name)
        if list(shape) != [n, k]:
            raise ValueError(f"artifact tensor {name} is {shape}, expected {[n, k]}")
        bias = None
        if has_bias:
            bn = name[: -len(".weight")] + ".bias" if name.endswith(".weight") else name + ".bias"
            bias = _t_bits(art.f16_array(bn).view(np.uint16).reshape(-1), dtype)
        params[name] = (q, _t_bits(s, dtype), _t_bits(b, dtype), bias)
    for name in dense_names:
        params[name] = art.f16_to_f32(name).reshape(dense_names[name])
    return params


# ------------------------------------------------------------------ fixtures

def reference_fixture_specs(channels: int = 128) -> list:
    """The tensors of the reference's converted-artifact test
    (crates/nemotron-mlx/tests/encoder_artifact.rs:14-199): a one-block encoder
    of width `channels`, identity quantized matrices, constant F16 kernels,
    unit norms and zero biases, Int8Affine with group 128."""
    g8 = int8_affine(128)
    specs = []

    def f16(name, shape, value):
        specs.append((name, np.full(shape, value, np.float32), list(shape), F16))

    def eye(name, out, inp, source_shape=None):
        w = np.zeros((out, inp), np.float32)
        k = min(out, inp)
        w[np.arange(k), np.arange(k)] = 1.0
        specs.append((name, w.reshape(source_shape or (out, inp)), [out, inp], g8))

    c = channels
    f16("encoder.subsampling.conv_in.weight", (c, 1, 3, 3), 0.01)
    f16("encoder.subsampling.conv_in.bias", (c,), 0.0)
    eye("prompt_projector.linear_1.weight", c, c + 128)
    f16("prompt_projector.linear_1.bias", (c,), 0.0)
    eye("prompt_projector.linear_2.weight", c, c)
    f16("prompt_projector.linear_2.bias", (c,), 0.0)
    p = "encoder.layers.0"
    for ff in ("feed_forward1", "feed_forward2"):
        eye(f"{p}.{ff}.linear1.weight", c, c)
        eye(f"{p}.{ff}.linear2.weight", c, c)
    for norm in ("norm_feed_forward1", "norm_self_att", "norm_conv", "norm_feed_forward2",
                 "norm_out", "conv.norm"):
        f16(f"{p}.{norm}.weight", (c,), 1.0)
        f16(f"{p}.{norm}.bias", (c,), 0.0)
    eye(f"{p}.conv.pointwise_conv1.weight", 2 * c, c, (2 * c, c, 1))
    eye(f"{p}.conv.pointwise_conv2.weight", c, c, (c, c, 1))
    f16(f"{p}.conv.depthwise_conv.weight", (c, 1, 9), 0.01)
    for proj in ("q_proj", "k_proj", "v_proj", "o_proj", "relative_k_proj"):
        eye(f"{p}.self_attn.{proj}.weight", c, c)
    f16(f"{p}.self_attn.bias_u", (2, 64), 0.0)
    f16(f"{p}.self_attn.bias_v", (2, 64), 0.0)
    for layer in range(2):
        s = f"encoder.subsampling.layers.{layer}"
        f16(f"{s}.depthwise_conv.weight", (c, 1, 3, 3), 0.01)
        f16(f"{s}.depthwise_conv.bias", (c,), 0.0)
        eye(f"{s}.pointwise_conv.weight", c, c, (c, c, 1, 1))
        f16(f"{s}.pointwise_conv.bias", (c,), 0.0)
    specs.append(("encoder.subsampling.linear.weight", np.full((c, 2 * c), 0.01, np.float32),
                  [c, 2 * c], g8))
    f16("encoder.subsampling.linear.bias", (c,), 0.0)
    return specs


# StreamingEncoder::from_artifact_with_config(&artifact, config, 8, channels)
# in the same test: one block, two heads, window 4, 8 mel bins.
REFERENCE_FIXTURE_CONFIG = dict(hidden=128, ff=128, layers=1, heads=2, conv_kernel=9,
                                sliding_window=4, mel_bins=8, sub_channels=128, num_prompts=128,
                                prompt_hidden=128, group_size=128)


def _bias_name(weight_name: str) -> str:
    return weight_name[: -len(".weight")] + ".bias" if weight_name.endswith(".weight") \
        else weight_name + ".bias"


def random_specs(linear_names: dict, dense_names: dict, group: int, seed: int,
                 std: dict | None = None) -> list:
    """Seeded f32 source tensors for every linear (N(0, 0.02), or the std that
    `std` maps a name to), its F16 output bias, and every dense tensor (norm
    weights around 1, convolution kernels N(0, 1/9), the rest N(0, 0.02))."""
    rng = np.random.default_rng(seed)
    std = std or {}
    specs = []
    for name, (n, k, has_bias) in linear_names.items():
        w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(std.get(name, 0.02))
        specs.append((name, w, [n, k], int8_affine(group)))
        if has_bias:
            b = rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)
            specs.append((_bias_name(name), b, [n], F16))
    for name, shape in dense_names.items():
        if name.endswith("norm.weight") or (".norm_" in name and name.endswith(".weight")):
            v = 1.0 + 0.1 * rng.standard_normal(shape, dtype=np.float32)
        elif name.endswith("depthwise_conv.weight") or name.endswith("conv_in.weight"):
            v = rng.standard_normal(shape, dtype=np.float32) / np.float32(3.0)
        else:
            v = 0.02 * rng.standard_normal(shape, dtype=np.float32)
        specs.append((name, np.asarray(v, np.float32), list(shape), F16))
    return specs
