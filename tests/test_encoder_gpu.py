"""Streaming encoder parity on the GPU: the CUDA chunk pipeline (subsampling,
FastConformer blocks, prompt projector, through include/cqencoder.h) against
the CPU restatement in oracle/encoder_oracle.py, chunk after chunk, so that
every streaming cache (subsampling time caches, attention window, depthwise
cache) is exercised across chunk boundaries.

Tolerances.  Both sides round to T at the same points, but their fp32 sums run
in different orders (tensor-core tiles against the oracle's sequential and
float64 sums), so single roundings of T flip and the flips propagate through
the LayerNorms and residual adds of every block.  Bounds, per chunk output:
relative L2 <= 2e-2 (bf16) / 4e-3 (f16) and max |diff| <= 8e-2 (bf16) /
1.6e-2 (f16) times max |reference|, several times the spread measured over
24 blocks.
"""
from __future__ import annotations

import numpy as np
import pytest

import encoder_oracle as eo

pytestmark = pytest.mark.gpu

TOL = {"bf16": (2e-2, 8e-2), "f16": (4e-3, 1.6e-2)}

SMALL = dict(hidden=256, ff=512, layers=2, heads=2, sliding_window=21, mel_bins=32,
             sub_channels=64, num_prompts=64, prompt_hidden=256, group_size=64)


def _oracle_cfg(d):
    return eo.EncoderConfig(hidden=d["hidden"], ff=d["ff"], layers=d["layers"], heads=d["heads"],
                            conv_kernel=d.get("conv_kernel", 9), sliding_window=d["sliding_window"],
                            mel_bins=d["mel_bins"], sub_channels=d["sub_channels"],
                            num_prompts=d["num_prompts"], prompt_hidden=d["prompt_hidden"],
                            group=d["group_size"])


def _compare(got_t, want, dtype, what):
    import torch
    got = got_t.float().cpu().numpy().astype(np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    assert np.all(np.isfinite(got)), what
    diff = np.abs(got - want)
    rel_l2 = float(np.sqrt((diff ** 2).sum() / max((want ** 2).sum(), 1e-30)))
    rel_max = float(diff.max() / max(np.abs(want).max(), 1e-30))
    l2_tol, max_tol = TOL[dtype]
    assert rel_l2 <= l2_tol and rel_max <= max_tol, (what, rel_l2, rel_max)
    _ = torch
    return rel_l2, rel_max


def _bind_params(cq_enc, params, cfg):
    for name, (n, k, has_bias) in eo.linear_names(cfg).items():
        q, s, b, bias = params[name]
        cq_enc.set_linear(name, q, s, b, bias if has_bias else None, cfg.group)
    for name in eo.dense_names(cfg):
        cq_enc.set_tensor(name, params[name])


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_small_encoder_matches_oracle_over_chunks(cq, oracle_mod, dtype):
    """Host-bound weights, two lock-step streams, five chunks (the window fills)."""
    import torch
    from nemotron_cuda.encoder import Encoder, EncoderConfig
    cfg = _oracle_cfg(SMALL)
    params = eo.random_params(cfg, 11, dtype)
    enc = Encoder(EncoderConfig.default(**SMALL), dtype)
    _bind_params(enc, params, cfg)
    ref = eo.Encoder(cfg, params, dtype)
    streams = 2
    state = enc.state(streams, 112)
    state.set_prompts([3, 7])
    caches = [ref.new_cache() for _ in range(streams)]
    rng = np.random.default_rng(5)
    for chunk in range(5):
        mel = rng.standard_normal((streams, 112, cfg.mel_bins)).astype(np.float32)
        out = state.encode_chunk(torch.from_numpy(mel).cuda())
        torch.cuda.synchronize()
        frames = out.shape[0] // streams
        assert frames == 14
        for s, pid in enumerate((3, 7)):
            want = ref.encode_chunk(mel[s], pid, caches[s])
            _compare(out[s * frames:(s + 1) * frames], want, dtype, f"chunk {chunk} stream {s}")
    assert state.chunks == 5
    assert cq.device_status(0) == 0


def test_full_encoder_random_weights_matches_oracle(cq, oracle_mod):
    """The checkpoint's shape (24 blocks, hidden 1024) with device-generated
    weights read back for the oracle; 112-frame chunks, the first four fill
    the 56-frame attention window."""
    import torch
    from nemotron_cuda.encoder import Encoder
    dtype = "bf16"
    enc = Encoder.random(None, seed=3, dtype=dtype)
    cfg = eo.EncoderConfig()
    params = enc.export_params(eo.linear_names(cfg), eo.dense_names(cfg))
    ref = eo.Encoder(cfg, params, dtype)
    cache = ref.new_cache()
    state = enc.state(1, 112)
    rng = np.random.default_rng(9)
    for chunk in range(5):
        mel = rng.standard_normal((1, 112, 128)).astype(np.float32)
        out = state.encode_chunk(torch.from_numpy(mel).cuda())
        torch.cuda.synchronize()
        want = ref.encode_chunk(mel[0], 101, cache)
        _compare(out, want, dtype, f"chunk {chunk}")
    assert cq.device_status(0) == 0


def test_streams_are_independent_and_reset_restarts(cq, oracle_mod):
    """A stream's output does not depend on its neighbours (up to the kernel
    choice, which follows the row count), and reset() replays the chunks bit
    for bit (the first chunk runs eagerly, later ones replay a graph)."""
    import torch
    from nemotron_cuda.encoder import Encoder, EncoderConfig
    enc = Encoder.random(EncoderConfig.default(**SMALL), seed=4, dtype="bf16")
    rng = np.random.default_rng(1)
    mels = [torch.from_numpy(rng.standard_normal((3, 112, SMALL["mel_bins"])).astype(np.float32)).cuda()
            for _ in range(3)]
    st3 = enc.state(3, 112)
    outs3 = [st3.encode_chunk(m).clone() for m in mels]
    st1 = enc.state(1, 112)
    outs1 = [st1.encode_chunk(m[1:2].contiguous()).clone() for m in mels]
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(zip(outs3, outs1)):
        _compare(a[14:28], b.float().cpu().numpy(), "bf16", f"chunk {i}")
    st1.reset()
    again = [st1.encode_chunk(m[1:2].contiguous()).clone() for m in mels]
    torch.cuda.synchronize()
    for a, b in zip(again, outs1):
        assert torch.equal(a, b)
    # without programmatic dependent launch: the same bits
    st1.set_pdl(False)
    st1.reset()
    no_pdl = [st1.encode_chunk(m[1:2].contiguous()).clone() for m in mels]
    torch.cuda.synchronize()
    for a, b in zip(no_pdl, outs1):
        assert torch.equal(a, b)


def test_sixteen_streams_match_one_stream_bit_for_bit(cq, oracle_mod):
    """Below 256 rows per linear every encoder kernel gives a row the same bits
    whatever the row count (the GEMV's reduction order follows K alone; the
    other kernels work per stream or per row), so each of 16 lock-step streams
    equals the same stream decoded alone, bit for bit, over chunks of 14 and
    13 frames."""
    import torch
    from nemotron_cuda.encoder import Encoder, EncoderConfig
    enc = Encoder.random(EncoderConfig.default(**SMALL), seed=8, dtype="bf16")
    rng = np.random.default_rng(3)
    S = 16
    mels = [torch.from_numpy(rng.standard_normal((S, n, SMALL["mel_bins"])).astype(np.float32)).cuda()
            for n in (112, 104, 112)]
    st = enc.state(S, 112)
    outs = [st.encode_chunk(m).clone() for m in mels]
    for k in (0, 7, 15):
        one = enc.state(1, 112)
        alone = [one.encode_chunk(m[k:k + 1].contiguous()).clone() for m in mels]
        torch.cuda.synchronize()
        for c, (a, b) in enumerate(zip(outs, alone)):
            q = b.shape[0]
            assert a.shape[0] == S * q
            assert torch.equal(a[k * q:(k + 1) * q], b), (k, c)
    assert cq.device_status(0) == 0


def test_prompt_changes_only_through_the_projector(cq, oracle_mod):
    import torch
    from nemotron_cuda.encoder import Encoder, EncoderConfig
    enc = Encoder.random(EncoderConfig.default(**SMALL), seed=6, dtype="bf16")
    mel = torch.randn((2, 112, SMALL["mel_bins"]), device="cuda")
    st = enc.state(2, 112)
    st.set_prompts([0, 5])
    out = st.encode_chunk(mel)
    torch.cuda.synchronize()
    st2 = enc.state(2, 112)
    st2.set_prompts([5, 5])
    out2 = st2.encode_chunk(torch.stack([mel[1], mel[1]]))
    torch.cuda.synchronize()
    assert torch.equal(out2[:14], out2[14:])
    assert torch.equal(out2[14:], out[14:])


def test_encoder_binding_errors(cq):
    from nemotron_cuda import CQError
    from nemotron_cuda.encoder import Encoder, EncoderConfig
    enc = Encoder(EncoderConfig.default(**SMALL), "bf16")
    with pytest.raises(CQError, match="unknown encoder tensor"):
        enc.set_tensor("encoder.layers.9.norm_out.weight", np.zeros(256))
    with pytest.raises(CQError, match="has 255 values, expected 256"):
        enc.set_tensor("encoder.layers.0.norm_out.weight", np.zeros(255))
    w = np.zeros((256, 256), np.float32)
    import oracle
    q, s, b = oracle.quantize(w, 64, "bf16")
    with pytest.raises(CQError, match="must be 512x256"):
        enc.set_linear("encoder.layers.0.feed_forward1.linear1.weight", q, s, b, None, 64)
    with pytest.raises(CQError, match="is not bound"):
        enc.state(1, 112)
    # the subsampling Conv2D keeps a thread on one group of 8 channels
    with pytest.raises(CQError, match="subsampling channels must be 8 times a power of two"):
        Encoder(EncoderConfig.default(**{**SMALL, "sub_channels": 72}), "bf16")
    names = enc.tensor_names()
    assert names[0] == "encoder.subsampling.layers.0.pointwise_conv.weight"
    assert "encoder.layers.1.self_attn.bias_v" in names
    assert len(names) == len(set(names)) == len(eo.linear_names(_oracle_cfg(SMALL))) + \
        len(eo.dense_names(_oracle_cfg(SMALL)))


def test_chunk_shapes_follow_the_subsampling(cq):
    """First chunks see one extra zero frame (encoder_streaming.rs:158-208):
    9 then 8 mel frames give 2 then 1 encoder frames, 112 give 14."""
    from nemotron_cuda.encoder import Encoder, EncoderConfig
    enc = Encoder.random(EncoderConfig.default(**SMALL), seed=2, dtype="f16")
    st = enc.state(1, 112)
    assert st.output_frames(9) == 2
    assert st.output_frames(112) == 14
    import torch
    st.encode_chunk(torch.zeros((1, 9, SMALL["mel_bins"]), device="cuda"))
    assert st.output_frames(8) == 1
    assert st.output_frames(112) == 14
