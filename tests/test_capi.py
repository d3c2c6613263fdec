"""C-ABI tests that need no GPU: the library loads, exports every symbol that
include/*.h declares, and rejects bad arguments with the reference's messages
before touching a device (crates/nemotron-mlx/tests/quantized_matmul.rs:49-75,
crates/nemotron-mlx/src/model/layers.rs:510-530)."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import ROOT


def declared_symbols() -> set[str]:
    names = set()
    inc = os.path.join(ROOT, "include")
    for f in os.listdir(inc):
        if not f.endswith(".h"):
            continue
        text = open(os.path.join(inc, f)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b((?:cq|catcher)_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_header_declares_the_boundary():
    names = declared_symbols()
    for required in ("cq_linear_create", "cq_linear_forward", "cq_linear_forward_f32",
                     "cq_linear_destroy", "cq_last_error", "cq_quantized_matmul",
                     "catcher_create", "catcher_push_audio", "catcher_finish", "catcher_text",
                     "catcher_last_error", "catcher_destroy"):
        assert required in names


def test_library_exports_every_declared_symbol(cq):
    lib = ctypes.CDLL(cq.LIB_PATH)
    missing = [n for n in sorted(declared_symbols()) if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", cq.LIB_PATH], capture_output=True,
                         text=True).stdout
    exported = set(re.findall(r" T ((?:cq|catcher)_[a-z0-9_]+)$", out, flags=re.M))
    assert declared_symbols() <= exported


def test_version_and_last_error(cq):
    assert "sm_100a" in cq.version()
    assert isinstance(cq.last_error(), str)


@pytest.mark.parametrize(
    "args,needle",
    [
        ((np.zeros(127), 1, 128, np.zeros(128), 1, 128), "input has 127 values"),
        ((np.zeros(128), 1, 128, np.zeros(127), 1, 128), "weight has 127 values"),
        ((np.zeros(128), 1, 128, np.zeros(128), 1, 96), "not divisible by group size 96"),
        ((np.zeros(128), 1, 128, np.zeros(128), 1, 0), "group size must be positive"),
    ],
)
def test_quantized_matmul_rejects_bad_shapes(cq, args, needle):
    """quantized_matmul.rs:49-75, through the C ABI, before any device work."""
    with pytest.raises(cq.CQError) as ei:
        cq.quantized_matmul(*args)
    assert ei.value.status == cq.CQ_INVALID_ARGUMENT
    assert needle in str(ei.value)
    assert str(ei.value).startswith("invalid matrix shape: ")


def test_quantized_matmul_rejects_unsupported_group(cq):
    with pytest.raises(cq.CQError) as ei:
        cq.quantized_matmul(np.zeros(16), 1, 16, np.zeros(16), 1, 16)
    assert "supported group sizes are 32, 64 and 128" in str(ei.value)


@pytest.mark.parametrize(
    "w_len,bias_len,group,needle",
    [
        (255, 2, 128, "linear weight/bias mismatch for 2x128"),
        (256, 3, 128, "linear weight/bias mismatch for 2x128"),
        (256, 2, 96, "linear input dimension 128 is incompatible with group size 96"),
        (256, 2, 0, "linear input dimension 128 is incompatible with group size 0"),
    ],
)
def test_from_f32_rejects_bad_shapes(cq, w_len, bias_len, group, needle):
    """validate_linear_shapes, crates/nemotron-mlx/src/model/layers.rs:510-530."""
    with pytest.raises(cq.CQError) as ei:
        cq.QuantizedLinear.from_f32(np.zeros(w_len), 2, 128, np.zeros(bias_len), group)
    assert ei.value.status == cq.CQ_INVALID_ARGUMENT
    assert needle in str(ei.value)


def test_create_rejects_null_and_bad_group(cq):
    lib = cq.lib()
    h = ctypes.c_void_p()
    st = lib.cq_linear_create(None, None, None, None, 4, 128, 64, 0, 0, ctypes.byref(h))
    assert st == cq.CQ_INVALID_ARGUMENT and "must not be null" in cq.last_error()
    q = np.zeros((4, 32), np.uint32)
    s = np.zeros((4, 2), np.uint16)
    st = lib.cq_linear_create(q.ctypes.data, s.ctypes.data, s.ctypes.data, None, 4, 128, 48, 0, 0,
                              ctypes.byref(h))
    assert st == cq.CQ_INVALID_ARGUMENT and "supported group sizes" in cq.last_error()
    st = lib.cq_linear_create(q.ctypes.data, s.ctypes.data, s.ctypes.data, None, 4, 128, 64, 7, 0,
                              ctypes.byref(h))
    assert st == cq.CQ_INVALID_ARGUMENT and "unknown dtype" in cq.last_error()


def test_null_handles_are_rejected(cq):
    lib = cq.lib()
    assert lib.cq_linear_forward(None, None, 1, None, None) == cq.CQ_INVALID_ARGUMENT
    assert "layer must not be null" in cq.last_error()
    assert lib.cq_linear_input_dims(None) == -1
    lib.cq_linear_destroy(None)  # no-op


def test_quantize_entry_validates_before_device_work(cq):
    lib = cq.lib()
    assert lib.cq_quantize(None, 4, 100, 64, 0, 1, None, None, None, None) == cq.CQ_INVALID_ARGUMENT
    assert "group size 64" in cq.last_error()
    assert lib.cq_dequantize(None, None, None, 4, 128, 24, 0, None, None) == cq.CQ_INVALID_ARGUMENT


def test_encoder_abi_rejects_null_arguments_without_a_device(cq):
    """cqencoder.h entry points validate their handles before any CUDA call."""
    from nemotron_cuda.encoder import EncoderConfig
    cfg = EncoderConfig.default()
    assert cfg.as_dict() == dict(hidden=1024, ff=4096, layers=24, heads=8, conv_kernel=9,
                                 sliding_window=57, mel_bins=128, sub_channels=256,
                                 num_prompts=128, prompt_hidden=2048, group_size=64)
    L = cq.lib()
    h = ctypes.c_void_p()
    assert L.cq_encoder_create(None, 1, 0, ctypes.byref(h)) == cq.CQ_INVALID_ARGUMENT
    assert "config must not be null" in cq.last_error()
    assert L.cq_encoder_set_tensor(None, b"x", None, 0) == cq.CQ_INVALID_ARGUMENT
    assert L.cq_encoder_encode_chunk(None, None, 112, None, None) == cq.CQ_INVALID_ARGUMENT
    assert L.cq_encoder_state_output_frames(None, 112) == 0
    assert L.cq_encoder_tensor_count(None) == -1
    assert L.cq_encoder_linear(None, b"x") is None
    assert L.cq_encoder_state_set_pdl(None, 0) == cq.CQ_INVALID_ARGUMENT
    assert L.cq_rnnt_state_set_pdl(None, 0) == cq.CQ_INVALID_ARGUMENT
    assert L.cq_rnnt_state_set_persistent(None, 1) == cq.CQ_INVALID_ARGUMENT
