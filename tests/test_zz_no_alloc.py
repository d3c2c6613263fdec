"""The no-allocation entry point, cq_linear_forward_noalloc.

Callers that cannot allocate device memory once a stream is running (a
transcriber fed from a real-time audio path, a host held to a fixed GPU memory
budget) use this entry: the scratch that batched bf16 calls stage their f16
activations in comes from an array in the library's device image instead of a
cudaMalloc.  Its results must match the regular entry point
(cq_linear_forward_ex) call for call.  This file is collected last so that a
run stopping at the first failure has run every other test before it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

from conftest import GEMM_FLOOR, assert_parity

pytestmark = pytest.mark.gpu

ROWS = 896  # 64 streams x 14 frames: the batched tensor-core path, which stages scratch


def _dev(torch, bits, dtype):
    a = np.ascontiguousarray(bits).view(np.int16)
    return torch.from_numpy(a).cuda().view(torch.bfloat16 if dtype == "bf16" else torch.float16)


def _bits(t):
    import torch
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _call_noalloc(cq, layer, x, y, act="none"):
    return cq.lib().cq_linear_forward_noalloc(
        layer._h, ctypes.c_void_p(x.data_ptr()), x.stride(0), x.shape[0],
        ctypes.c_void_p(y.data_ptr()), y.stride(0), cq.ACTS[act], None)


def test_noalloc_matches_regular_entry_on_two_calls(cq, oracle_mod):
    import torch
    assert torch.cuda.is_available()
    rng = np.random.default_rng(2024)
    n, k = 2048, 1024
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    q, s, b = oracle_mod.quantize(w, 64, "bf16")
    bias = oracle_mod.to_t((rng.standard_normal(n) * 0.1).astype(np.float32), "bf16")
    layer = cq.QuantizedLinear.from_packed(q, s, b, bias, 64, "bf16")
    for call in range(2):  # two calls in a row, different inputs
        x_bits = oracle_mod.to_t(rng.standard_normal((ROWS, k)).astype(np.float32), "bf16")
        x = _dev(torch, x_bits, "bf16")
        y_ref = torch.empty((ROWS, n), dtype=torch.bfloat16, device="cuda")
        y_na = torch.full((ROWS, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        layer.forward(x, y_ref, act="silu", stream=0)
        st = _call_noalloc(cq, layer, x, y_na, act="silu")
        assert st == cq.CQ_OK, cq.last_error()
        torch.cuda.synchronize()
        got, want = _bits(y_na), _bits(y_ref)
        assert_parity(got, want, "bf16", min_exact=0.97, bias_bits=bias, act="silu")
        assert np.array_equal(got, want), f"call {call}: same kernels, different scratch"
    assert cq.device_status(0) == 0


def test_noalloc_small_rows_and_f16(cq, oracle_mod):
    """Paths without scratch (the GEMV, f16 layers) run through the same entry."""
    import torch
    rng = np.random.default_rng(7)
    for dtype, rows in (("bf16", 14), ("f16", 300)):
        w = (rng.standard_normal((1024, 1024)) * 0.02).astype(np.float32)
        q, s, b = oracle_mod.quantize(w, 64, dtype)
        layer = cq.QuantizedLinear.from_packed(q, s, b, None, 64, dtype)
        x = _dev(torch, oracle_mod.to_t(rng.standard_normal((rows, 1024)).astype(np.float32), dtype),
                 dtype)
        tdt = torch.bfloat16 if dtype == "bf16" else torch.float16
        y_ref = torch.empty((rows, 1024), dtype=tdt, device="cuda")
        y_na = torch.empty((rows, 1024), dtype=tdt, device="cuda")
        layer.forward(x, y_ref, stream=0)
        assert _call_noalloc(cq, layer, x, y_na) == cq.CQ_OK, cq.last_error()
        torch.cuda.synchronize()
        assert np.array_equal(_bits(y_na), _bits(y_ref))


def test_noalloc_rejects_rows_beyond_the_limit(cq, oracle_mod):
    import torch
    rng = np.random.default_rng(9)
    w = (rng.standard_normal((512, 4096)) * 0.02).astype(np.float32)
    q, s, b = oracle_mod.quantize(w, 64, "bf16")
    layer = cq.QuantizedLinear.from_packed(q, s, b, None, 64, "bf16")
    rows = 1100  # 1100 x 4096 x 2 bytes > 8 MiB
    x = torch.zeros((rows, 4096), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((rows, 512), dtype=torch.bfloat16, device="cuda")
    st = _call_noalloc(cq, layer, x, y)
    assert st == cq.CQ_INVALID_ARGUMENT
    assert "exceeds the no-allocation scratch" in cq.last_error()


def test_noalloc_first_call_allocates_nothing_and_matches_the_oracle(cq, oracle_mod):
    """On a fresh layer the no-allocation call comes first: device free memory
    must not move (the regular entry would reserve a 1.8 MB workspace, which a
    cudaMalloc rounds to 2 MiB), and the output is checked against the oracle
    directly, not only against the regular entry."""
    import torch
    rng = np.random.default_rng(31)
    n, k = 2048, 1024

    def make_layer():
        w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        q, s, b = oracle_mod.quantize(w, 64, "bf16")
        return (q, s, b), cq.QuantizedLinear.from_packed(q, s, b, None, 64, "bf16")

    # warm-up on another layer of the same shape: loads the kernels and looks
    # the scratch array up, which the driver may back with memory lazily
    _, warm = make_layer()
    x_bits = oracle_mod.to_t(rng.standard_normal((ROWS, k)).astype(np.float32), "bf16")
    x = _dev(torch, x_bits, "bf16")
    y = torch.empty((ROWS, n), dtype=torch.bfloat16, device="cuda")
    assert _call_noalloc(cq, warm, x, y) == cq.CQ_OK, cq.last_error()
    torch.cuda.synchronize()

    (q, s, b), fresh = make_layer()
    y = torch.full((ROWS, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    assert _call_noalloc(cq, fresh, x, y) == cq.CQ_OK, cq.last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free0 - free1 < (1 << 20), f"device free memory fell by {free0 - free1} bytes"
    assert_parity(_bits(y), oracle_mod.qmatmul(x_bits, q, s, b, 64, "bf16"), "bf16",
                  min_exact=0.6, floor_frac=GEMM_FLOOR)
    assert cq.device_status(0) == 0


_CAPTURE_SCRIPT = textwrap.dedent("""
    import ctypes, sys
    import numpy as np
    import torch
    sys.path[:0] = sys.argv[1:3]
    import nemotron_cuda as cq
    import oracle
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((1024, 1024)) * 0.02).astype(np.float32)
    q, s, b = oracle.quantize(w, 64, "bf16")
    layer = cq.QuantizedLinear.from_packed(q, s, b, None, 64, "bf16")
    x = torch.zeros((512, 1024), dtype=torch.bfloat16, device="cuda")
    y = torch.zeros((512, 1024), dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        g.capture_begin()
        st = cq.lib().cq_linear_forward_noalloc(
            layer._h, ctypes.c_void_p(x.data_ptr()), 1024, 512, ctypes.c_void_p(y.data_ptr()),
            1024, 0, ctypes.c_void_p(stream.cuda_stream))
        g.capture_end()
    print(st, cq.last_error())
""")


def test_noalloc_first_call_during_capture_is_rejected():
    """The first call on a device looks the scratch address up; during a stream
    capture it fails with a clear message instead of a generic CUDA error.  Run
    in a fresh process so that this call really is the first."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _CAPTURE_SCRIPT, os.path.join(root, "catcher-tippi_b200"),
                        os.path.join(root, "oracle")], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    status, _, message = r.stdout.strip().splitlines()[-1].partition(" ")
    assert int(status) == -1, r.stdout
    assert "must not run during stream capture" in message, message
