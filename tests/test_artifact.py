"""Release-artifact reader on the CPU: the manifest/safetensors restatement in
oracle/artifact_oracle.py against the reference's converted-artifact fixture
(crates/nemotron-mlx/tests/encoder_artifact.rs), and the library's host-side
reader (include/cqartifact.h) against that restatement -- shapes, storage
policies, F16 widening and the reference's error texts
(crates/nemotron-mlx/src/weights/artifact.rs:13-56).  Nothing here touches a
device: the checks that bind tensors on a GPU are in test_artifact_gpu.py.
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np
import pytest

import artifact_oracle as ao
import encoder_oracle as eo

FIXTURE_ID = "fixture/subsampling"


@pytest.fixture(scope="module")
def fixture_dir(tmp_path_factory, oracle_mod):
    out = str(tmp_path_factory.mktemp("art") / "artifact")
    ao.convert_tensors(out, FIXTURE_ID, ao.reference_fixture_specs())
    return out


def _oracle_cfg(d):
    return eo.EncoderConfig(hidden=d["hidden"], ff=d["ff"], layers=d["layers"], heads=d["heads"],
                            conv_kernel=d["conv_kernel"], sliding_window=d["sliding_window"],
                            mel_bins=d["mel_bins"], sub_channels=d["sub_channels"],
                            num_prompts=d["num_prompts"], prompt_hidden=d["prompt_hidden"],
                            group=d["group_size"])


def test_converter_writes_the_reference_layout(fixture_dir):
    with open(os.path.join(fixture_dir, "manifest.json")) as f:
        m = json.load(f)
    assert m["format_version"] == 1 and m["model_id"] == FIXTURE_ID
    lin = m["tensors"]["encoder.subsampling.linear.weight"]
    assert lin == {"shape": [128, 256], "storage": {"Int8Affine": {"group_size": 128}}}
    pw = m["tensors"]["encoder.layers.0.conv.pointwise_conv1.weight"]
    assert pw["shape"] == [256, 128]  # trailing unit dimension squeezed
    assert m["tensors"]["encoder.layers.0.conv.depthwise_conv.weight"] == \
        {"shape": [128, 1, 9], "storage": "F16"}
    arrays = ao.load_safetensors(os.path.join(fixture_dir, "weights.safetensors"))
    q = arrays["encoder.subsampling.linear.weight.__qweight"]
    assert q.dtype == np.uint32 and q.shape == (128, 64)
    s = arrays["encoder.subsampling.linear.weight.__scales"]
    assert s.dtype == np.float16 and s.shape == (128, 2)
    assert "encoder.subsampling.linear.weight" not in arrays
    # the header is padded to 8 bytes and the data follows it directly
    with open(os.path.join(fixture_dir, "weights.safetensors"), "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
    assert n % 8 == 0


def test_identity_matrices_survive_quantization(fixture_dir, oracle_mod):
    art = ao.Artifact(fixture_dir)
    q, s, b, g, shape = art.quantized_arrays("encoder.layers.0.self_attn.q_proj.weight")
    assert g == 128 and list(shape) == [128, 128]
    w = oracle_mod.dequantize(q, s, b, g, "f16")
    off = ~np.eye(128, dtype=bool)
    # each group's edge is its 1.0 (the bias, code 0): the diagonal is exact
    assert np.all(np.diag(w) == 1.0)
    # zeros take code 255 at scale f16(-1/255): 1 + 255 * scale, 2^-16 from 0
    s16 = np.float32(np.float16(np.float32(-1.0) / np.float32(255.0)))
    assert np.all(w[off] == np.float32(255.0) * s16 + np.float32(1.0))
    assert np.abs(w[off]).max() <= 2.0 ** -16


def test_oracle_encoder_binds_the_fixture(fixture_dir, oracle_mod):
    """The reference test's assertion: a 9-frame chunk of 0.25 through the
    one-block encoder gives [1, 2, 128]."""
    cfg = _oracle_cfg(ao.REFERENCE_FIXTURE_CONFIG)
    art = ao.Artifact(fixture_dir)
    params = ao.model_params(art, eo.linear_names(cfg), eo.dense_names(cfg), "f16")
    enc = eo.Encoder(cfg, params, "f16")
    out = enc.encode_chunk(np.full((9, 8), 0.25, np.float32), 101, enc.new_cache())
    assert out.shape == (2, 128)
    assert np.all(np.isfinite(out))


def test_library_reads_manifest_and_widens_f16(cq, fixture_dir):
    from nemotron_cuda.artifact import Artifact
    ref = ao.Artifact(fixture_dir)
    with Artifact(fixture_dir) as art:
        assert art.model_id == FIXTURE_ID and art.format_version == 1
        assert art.tensor_names() == sorted(ref.manifest["tensors"])
        info = art.tensor_info("encoder.subsampling.linear.weight")
        assert info.shape == (128, 256) and info.storage == "Int8Affine" and info.group_size == 128
        info = art.tensor_info("encoder.subsampling.conv_in.weight")
        assert info.shape == (128, 1, 3, 3) and info.storage == "F16" and info.group_size == 0
        for name in ("encoder.subsampling.conv_in.weight", "encoder.layers.0.norm_out.weight",
                     "encoder.layers.0.self_attn.bias_u"):
            np.testing.assert_array_equal(art.f16_to_f32(name), ref.f16_to_f32(name))


def test_library_errors_carry_the_reference_texts(cq, fixture_dir):
    from nemotron_cuda import CQError, QuantizedLinear
    from nemotron_cuda.artifact import Artifact
    art = Artifact(fixture_dir)
    with pytest.raises(CQError, match="^missing artifact tensor nope$"):
        art.tensor_info("nope")
    with pytest.raises(CQError, match=r"^tensor encoder.subsampling.linear.weight has incompatible "
                                      r"storage Int8Affine \{ group_size: 128 \}$"):
        art.f16_to_f32("encoder.subsampling.linear.weight")
    # QuantizedLinear::from_artifact validates the artifact before touching a device
    with pytest.raises(CQError, match="^tensor encoder.subsampling.conv_in.weight has "
                                      "incompatible storage F16$"):
        QuantizedLinear.from_artifact(art, "encoder.subsampling.conv_in.weight")
    with pytest.raises(CQError, match="^missing artifact tensor nope.weight$"):
        QuantizedLinear.from_artifact(art, "nope.weight")
    with pytest.raises(CQError, match="^missing artifact tensor nope.bias$"):
        QuantizedLinear.from_artifact(art, "encoder.subsampling.linear.weight", "nope.bias")
    with pytest.raises(CQError, match="incompatible storage Int8Affine"):
        QuantizedLinear.from_artifact(art, "encoder.subsampling.linear.weight",
                                      "encoder.layers.0.feed_forward1.linear1.weight")


def _copy_artifact(src, dst, manifest_edit=None, weights_edit=None):
    os.makedirs(dst)
    with open(os.path.join(src, "manifest.json")) as f:
        m = json.load(f)
    if manifest_edit:
        m = manifest_edit(m)
    with open(os.path.join(dst, "manifest.json"), "w") as f:
        f.write(m if isinstance(m, str) else json.dumps(m))
    with open(os.path.join(src, "weights.safetensors"), "rb") as f:
        w = f.read()
    if weights_edit:
        w = weights_edit(w)
    with open(os.path.join(dst, "weights.safetensors"), "wb") as f:
        f.write(w)
    return dst


def test_missing_arrays_and_malformed_files_are_rejected(cq, fixture_dir, tmp_path):
    from nemotron_cuda import CQError, QuantizedLinear
    from nemotron_cuda.artifact import Artifact

    def ghost(m):
        m["tensors"]["ghost.weight"] = {"shape": [128, 128],
                                        "storage": {"Int8Affine": {"group_size": 128}}}
        return m
    art = Artifact(_copy_artifact(fixture_dir, str(tmp_path / "ghost"), ghost))
    with pytest.raises(CQError, match="^missing artifact array ghost.weight.__qweight$"):
        QuantizedLinear.from_artifact(art, "ghost.weight")

    def wrong_shape(m):
        m["tensors"]["encoder.subsampling.linear.weight"]["shape"] = [128, 512]
        return m
    art = Artifact(_copy_artifact(fixture_dir, str(tmp_path / "shape"), wrong_shape))
    with pytest.raises(CQError, match="__qweight must be U32"):
        QuantizedLinear.from_artifact(art, "encoder.subsampling.linear.weight")

    with pytest.raises(CQError, match="cannot open"):
        Artifact(str(tmp_path / "absent"))
    with pytest.raises(CQError, match="invalid artifact manifest"):
        Artifact(_copy_artifact(fixture_dir, str(tmp_path / "json"), lambda m: "{\"tensors\": ["))

    def v2(m):
        m["format_version"] = 2
        return m
    with pytest.raises(CQError, match="unsupported artifact format_version 2"):
        Artifact(_copy_artifact(fixture_dir, str(tmp_path / "v2"), v2))
    with pytest.raises(CQError, match="outside the file"):
        Artifact(_copy_artifact(fixture_dir, str(tmp_path / "cut"), None, lambda w: w[:-64]))
    with pytest.raises(CQError, match="invalid safetensors header"):
        Artifact(_copy_artifact(fixture_dir, str(tmp_path / "hdr"), None,
                                lambda w: struct.pack("<Q", 1 << 40) + w[8:]))

    def offsets(first):
        def edit(w):
            (n,) = struct.unpack("<Q", w[:8])
            h = json.loads(w[8:8 + n])
            name = next(k for k in h if k != "__metadata__")
            h[name]["data_offsets"][0] = first
            text = json.dumps(h, separators=(",", ":")).encode()
            text += b" " * (-len(text) % 8)
            return struct.pack("<Q", len(text)) + text + w[8 + n:]
        return edit
    # negative, fractional and beyond-2^53 offsets are rejected before use;
    # the file mapping is released on every one of these errors
    for i, first in enumerate((-8, 0.5, 2.0 ** 60)):
        with pytest.raises(CQError, match="bad data_offsets"):
            Artifact(_copy_artifact(fixture_dir, str(tmp_path / f"off{i}"), None, offsets(first)))


def test_abi_rejects_null_arguments_without_a_device(cq):
    import ctypes
    L = cq.lib()
    h = ctypes.c_void_p()
    assert L.cq_artifact_open(None, ctypes.byref(h)) == cq.CQ_INVALID_ARGUMENT
    assert L.cq_artifact_tensor_count(None) == 0
    assert L.cq_artifact_tensor_name(None, 0) is None
    assert L.cq_encoder_bind_artifact(None, None) == cq.CQ_INVALID_ARGUMENT
    assert L.cq_rnnt_bind_artifact(None, None) == cq.CQ_INVALID_ARGUMENT
    L.cq_artifact_close(None)
