"""CPU restatement of the cache-aware streaming FastConformer encoder and the
prompt projector (TEST INFRASTRUCTURE).

Only the test suite, the smoke check and the benchmark's CPU-baseline leg use
this module; the CUDA library never calls it.  It restates, op by op and with
the reference's rounding points:

* ``crates/nemotron-mlx/src/model/encoder.rs``: ``RelativePositionAttention``
  (:183-259), ``softmax_in_place`` (:278-288), ``QuantizedFeedForward``
  (:323-336), ``ConformerConvolution`` (:376-397), ``FastConformerLayer::forward``
  (:498-535), ``residual_add`` (:538-552), ``silu_in_place`` (:554-558),
  ``StreamingEncoder::encode_chunk`` (:641-655), ``Conv2dSubsampling::forward``
  (:767-802), ``mask_invalid_time`` (:805-809), ``channel_frequency_flatten``
  (:812-833), ``relative_position_encoding`` (:864-884), ``relative_shift``
  (:887-906), ``SubsamplingCache::new`` (:12-35);
* ``crates/nemotron-mlx/src/model/layers.rs``: ``Fp16Conv2d`` (:37-205),
  ``DepthwiseConv1d::forward_f32`` (:418-455), ``LayerNorm::forward_f32``
  (:492-507);
* ``crates/nemotron-mlx/src/model/cache.rs``: ``CausalConv1dCache`` (:4-44),
  ``CausalConv2dCache`` (:47-118), ``AttentionKvCache::update`` (:155-208);
* ``crates/nemotron-mlx/src/model/prompt.rs``: ``PromptProjector::forward_f32``
  (:110-140).

Rounding points.  In the reference every tensor between ops is host f32.  Ops
run through MLX (quantized linears, LayerNorm, the depthwise and Conv2D
convolutions) cast their f32 input to T (f16 in the reference artifact; the
layer dtype here) and hand back T values; host ops (residual adds, SiLU, GLU,
the attention core, softmax) compute in f32.  This module keeps those points:
``rnd`` marks each cast to T.  The attention core and LayerNorm statistics are
computed in float64 here (a more exact value of the same expression; the
reference sums in f32); residual adds, SiLU and GLU use numpy float32, which is
IEEE single precision like the reference's host code.

Pinned by tests/test_encoder_oracle.py against the reference's own tests
(crates/nemotron-mlx/tests/encoder_streaming.rs, model_layers.rs:80-137).
"""
from __future__ import annotations

import dataclasses

import numpy as np

import oracle as qo


# ------------------------------------------------------------------ helpers


def rnd(x, dtype: str) -> np.ndarray:
    """Cast f32 values to T and back (T = "f16" or "bf16"; "f32" is a no-op)."""
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x.copy()
    return qo.np_from_t(qo.np_to_t(x, dtype), dtype)


def silu(x: np.ndarray) -> np.ndarray:
    """encoder.rs:554-558: v / (1 + exp(-v)) in f32."""
    x = np.asarray(x, dtype=np.float32)
    one = np.float32(1.0)
    with np.errstate(over="ignore"):
        return (x / (one + np.exp(-x))).astype(np.float32)


def relu(x: np.ndarray) -> np.ndarray:
    return np.maximum(np.asarray(x, dtype=np.float32), np.float32(0.0))


def residual_add(left: np.ndarray, right: np.ndarray, scale: float) -> np.ndarray:
    """encoder.rs:538-552: left + scale * right, f32."""
    return (left.astype(np.float32) + np.float32(scale) * right.astype(np.float32)).astype(np.float32)


class QLinear:
    """One affine INT8 linear (layers.rs:298-310) evaluated by the C oracle."""

    def __init__(self, q, s, b, bias_bits, group: int, dtype: str):
        self.q, self.s, self.b, self.bias = q, s, b, bias_bits
        self.group, self.dtype = group, dtype
        q8 = np.ascontiguousarray(q).view(np.uint8)
        self.output_dims, self.input_dims = q8.shape

    @classmethod
    def from_f32(cls, weight: np.ndarray, bias: np.ndarray | None, group: int, dtype: str):
        q, s, b = qo.quantize(np.asarray(weight, np.float32), group, dtype)
        bias_bits = None if bias is None else qo.to_t(np.asarray(bias, np.float32), dtype)
        return cls(q, s, b, bias_bits, group, dtype)

    def __call__(self, x: np.ndarray, act: str = "none") -> np.ndarray:
        """f32 [rows, K] -> f32 [rows, N] holding T values."""
        x = np.asarray(x, np.float32).reshape(-1, self.input_dims)
        xt = qo.to_t(x, self.dtype)
        y = qo.qmatmul(xt, self.q, self.s, self.b, self.group, self.dtype, self.bias, act)
        return qo.from_t(y, self.dtype)


def layer_norm(x: np.ndarray, weight: np.ndarray, bias: np.ndarray, eps: float,
               dtype: str) -> np.ndarray:
    """layers.rs:492-507: input and affine parameters in T, output T."""
    xt = rnd(x, dtype).astype(np.float64)
    mean = xt.mean(axis=-1, keepdims=True)
    var = ((xt - mean) ** 2).mean(axis=-1, keepdims=True)
    y = (xt - mean) / np.sqrt(var + eps) * weight.astype(np.float64) + bias.astype(np.float64)
    return rnd(y.astype(np.float32), dtype)


# ------------------------------------------------------------------ caches


class CausalConv1dCache:
    """cache.rs:4-44: left context of one causal depthwise convolution."""

    def __init__(self, channels: int, left_frames: int):
        self.channels, self.left_frames = channels, left_frames
        self.values = np.zeros(channels * left_frames, np.float32)

    def prepend_and_update(self, chunk: np.ndarray, frames: int) -> np.ndarray:
        chunk = np.asarray(chunk, np.float32).ravel()
        if chunk.size != frames * self.channels:
            raise ValueError(f"cache chunk has {chunk.size} values, expected {frames}x{self.channels}")
        combined = np.concatenate([self.values, chunk])
        keep = self.left_frames * self.channels
        self.values = combined[combined.size - keep:].copy()
        return combined


class CausalConv2dCache:
    """cache.rs:47-118: time context of one causal subsampling Conv2D."""

    def __init__(self, frequency_bins: int, channels: int, left_frames: int,
                 initial_extra_frames: int):
        self.frequency_bins, self.channels = frequency_bins, channels
        self.left_frames, self.initial_extra_frames = left_frames, initial_extra_frames
        self.first_chunk = True
        self.values = np.zeros((left_frames, frequency_bins, channels), np.float32)

    def prepend_and_update(self, chunk: np.ndarray) -> np.ndarray:
        chunk = np.asarray(chunk, np.float32)
        frames, freq, ch = chunk.shape
        if freq != self.frequency_bins or ch != self.channels:
            raise ValueError(f"conv2d cache expected [1,{frames},{self.frequency_bins},{self.channels}]")
        parts = []
        if self.first_chunk:
            parts.append(np.zeros((self.initial_extra_frames, freq, ch), np.float32))
        parts += [self.values, chunk]
        combined = np.concatenate(parts, axis=0)
        history = np.concatenate([self.values, chunk], axis=0)
        self.values = history[history.shape[0] - self.left_frames:].copy()
        self.first_chunk = False
        return combined


class AttentionKvCache:
    """cache.rs:120-208: per-head sliding window of keys and values."""

    def __init__(self, heads: int, head_dim: int, max_frames: int):
        self.heads, self.head_dim, self.max_frames = heads, head_dim, max_frames
        self.frames = 0
        self.keys = np.zeros((heads, 0, head_dim), np.float32)
        self.values = np.zeros((heads, 0, head_dim), np.float32)

    def update(self, current_keys: np.ndarray, current_values: np.ndarray, current_frames: int):
        """current_* [heads, frames, head_dim] -> (visible frames, keys, values)."""
        ck = np.asarray(current_keys, np.float32).reshape(self.heads, current_frames, self.head_dim)
        cv = np.asarray(current_values, np.float32).reshape(self.heads, current_frames, self.head_dim)
        keys = np.concatenate([self.keys, ck], axis=1)
        values = np.concatenate([self.values, cv], axis=1)
        total = keys.shape[1]
        retained = min(total, self.max_frames)
        drop = total - retained
        self.frames = retained
        self.keys = keys[:, drop:].copy()
        self.values = values[:, drop:].copy()
        return total, keys, values


# ------------------------------------------------------------------ convolutions


class DepthwiseConv1d:
    """layers.rs:357-455: f16 depthwise causal cross-correlation with a cache."""

    def __init__(self, weight: np.ndarray, bias: np.ndarray, dtype: str):
        self.weight = rnd(np.asarray(weight, np.float32), dtype)   # [channels, kernel]
        self.bias = rnd(np.asarray(bias, np.float32), dtype)
        self.channels, self.kernel = self.weight.shape
        self.dtype = dtype

    def forward(self, x: np.ndarray, cache: CausalConv1dCache) -> np.ndarray:
        time = x.shape[0]
        combined = cache.prepend_and_update(x, time).reshape(time + self.kernel - 1, self.channels)
        ct = rnd(combined, self.dtype)
        acc = np.zeros((time, self.channels), np.float32)
        for j in range(self.kernel):
            acc += self.weight[:, j][None, :] * ct[j:j + time]
        return rnd(rnd(acc, self.dtype) + self.bias[None, :], self.dtype)


class Conv2d:
    """layers.rs:26-205: ``Fp16Conv2d`` with causal time cache and NeMo's
    asymmetric frequency padding (left kernel-1, right stride-1)."""

    def __init__(self, weight_oihw: np.ndarray, bias: np.ndarray, stride: int, groups: int,
                 dtype: str):
        w = np.asarray(weight_oihw, np.float32)
        self.out_ch, self.cpg, self.kernel, k2 = w.shape
        assert self.kernel == k2
        self.in_ch = self.cpg * groups
        self.stride, self.groups, self.dtype = stride, groups, dtype
        self.weight = rnd(w, dtype)
        self.bias = rnd(np.asarray(bias, np.float32), dtype)

    def streaming_output_length(self, input_frames: int) -> int:
        left = self.kernel - self.stride
        if input_frames + left < self.kernel:
            return 0
        return (input_frames + left - self.kernel) // self.stride + 1

    def forward_causal(self, x: np.ndarray, cache: CausalConv2dCache) -> np.ndarray:
        """x [time, freq, in_ch] -> [out_time, out_freq, out_ch] (T values)."""
        combined = cache.prepend_and_update(x)
        tc, freq, ch = combined.shape
        k, s = self.kernel, self.stride
        padded = np.zeros((tc, freq + (k - 1) + (s - 1), ch), np.float32)
        padded[:, k - 1:k - 1 + freq] = combined
        xt = rnd(padded, self.dtype)
        tout = (tc - k) // s + 1
        fout = (padded.shape[1] - k) // s + 1
        opg = self.out_ch // self.groups
        w = self.weight.reshape(self.groups, opg, self.cpg, k, k)
        acc = np.zeros((max(tout, 0), fout, self.groups, opg), np.float32)
        for kt in range(k):
            for kf in range(k):
                sl = xt[kt:kt + s * (tout - 1) + 1:s, kf:kf + s * (fout - 1) + 1:s]
                sl = sl.reshape(tout, fout, self.groups, self.cpg)
                acc += np.einsum("tfgi,goi->tfgo", sl, w[:, :, :, kt, kf]).astype(np.float32)
        out = acc.reshape(tout, fout, self.out_ch)
        return rnd(rnd(out, self.dtype) + self.bias, self.dtype)


def mask_invalid_time(x: np.ndarray, valid_frames: int) -> np.ndarray:
    x = x.copy()
    x[min(valid_frames, x.shape[0]):] = 0.0
    return x


def channel_frequency_flatten(x: np.ndarray) -> np.ndarray:
    """encoder.rs:812-833: NHWC [time, freq, ch] -> [time, ch * freq] (channel-major)."""
    t, f, c = x.shape
    return np.ascontiguousarray(x.transpose(0, 2, 1)).reshape(t, c * f)


# ------------------------------------------------------------------ attention


def relative_position_encoding(hidden_size: int, total_frames: int) -> np.ndarray:
    """encoder.rs:864-884: positions L-1 .. -(L-1), sin/cos interleaved, f32."""
    if hidden_size == 0 or hidden_size % 2 or total_frames == 0:
        raise ValueError("relative positions require a positive even hidden size and nonzero frames")
    positions = np.arange(total_frames - 1, -total_frames, -1, dtype=np.float32)
    index = np.arange(hidden_size // 2, dtype=np.float32)
    exponent = (np.float32(2.0) * index / np.float32(hidden_size)).astype(np.float32)
    denom = np.power(np.float32(10000.0), exponent).astype(np.float32)
    angle = (positions[:, None] / denom[None, :]).astype(np.float32)
    out = np.empty((positions.size, hidden_size), np.float32)
    out[:, 0::2] = np.sin(angle)
    out[:, 1::2] = np.cos(angle)
    return out


def relative_shift(scores: np.ndarray, query_length: int, position_length: int) -> np.ndarray:
    """encoder.rs:887-906: pad one zero per row, flatten, drop the first Q entries."""
    scores = np.asarray(scores).ravel()
    if query_length == 0 or position_length == 0 or scores.size != query_length * position_length:
        raise ValueError("relative shift score dimensions are inconsistent")
    rows = scores.reshape(query_length, position_length)
    padded = np.concatenate([np.zeros((query_length, 1), scores.dtype), rows], axis=1).ravel()
    return padded[query_length:]


class RelPosAttention:
    """encoder.rs:183-259 with the K/V cache of cache.rs:155-208."""

    def __init__(self, q, k, v, o, pos, bias_u, bias_v, heads: int):
        self.q, self.k, self.v, self.o, self.pos = q, k, v, o, pos
        self.hidden = q.output_dims
        self.heads = heads
        self.head_dim = self.hidden // heads
        self.bias_u = np.asarray(bias_u, np.float32).ravel()
        self.bias_v = np.asarray(bias_v, np.float32).ravel()

    def forward(self, x: np.ndarray, cache: AttentionKvCache) -> np.ndarray:
        qf = x.shape[0]
        H, hd = self.heads, self.head_dim
        queries = self.q(x)
        keys = self.k(x).reshape(qf, H, hd).transpose(1, 0, 2)
        values = self.v(x).reshape(qf, H, hd).transpose(1, 0, 2)
        visible, vk, vv = cache.update(keys, values, qf)
        positions = relative_position_encoding(self.hidden, visible)
        pframes = positions.shape[0]
        relk = self.pos(positions)
        scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
        attended = np.zeros((qf, self.hidden), np.float64)
        for h in range(H):
            sl = slice(h * hd, (h + 1) * hd)
            qh = queries[:, sl].astype(np.float64)
            raw = (qh + self.bias_v[sl]) @ relk[:, sl].astype(np.float64).T      # [Q, P]
            shifted = relative_shift(raw, qf, pframes).reshape(qf, pframes)
            content = (qh + self.bias_u[sl]) @ vk[h].astype(np.float64).T         # [Q, V]
            scores = (content + shifted[:, :visible]) * scale
            scores = np.exp(scores - scores.max(axis=1, keepdims=True))
            probs = scores / scores.sum(axis=1, keepdims=True)
            attended[:, sl] = probs @ vv[h].astype(np.float64)
        return self.o(attended.astype(np.float32))


# ------------------------------------------------------------------ blocks


class FeedForward:
    """encoder.rs:323-336: linear1 -> SiLU -> linear2, no biases."""

    def __init__(self, linear1: QLinear, linear2: QLinear):
        self.linear1, self.linear2 = linear1, linear2

    def __call__(self, x: np.ndarray) -> np.ndarray:
        # SiLU on the T output of linear1, then the cast to T at linear2's input:
        # the C oracle's fused epilogue applies exactly that pair.
        return self.linear2(self.linear1(x, act="silu"))


class ConvModule:
    """encoder.rs:376-397: pw1 -> GLU -> depthwise (cache) -> LayerNorm -> SiLU -> pw2."""

    def __init__(self, pw1: QLinear, depthwise: DepthwiseConv1d, norm_w, norm_b, pw2: QLinear,
                 dtype: str):
        self.pw1, self.depthwise, self.pw2 = pw1, depthwise, pw2
        self.norm_w, self.norm_b = rnd(norm_w, dtype), rnd(norm_b, dtype)
        self.dtype = dtype

    def __call__(self, x: np.ndarray, cache: CausalConv1dCache) -> np.ndarray:
        c = x.shape[1]
        projected = self.pw1(x)
        first, gate = projected[:, :c], projected[:, c:]
        one = np.float32(1.0)
        with np.errstate(over="ignore"):
            gated = (first / (one + np.exp(-gate))).astype(np.float32)
        d = self.depthwise.forward(gated, cache)
        n = layer_norm(d, self.norm_w, self.norm_b, 1e-5, self.dtype)
        return self.pw2(silu(n))


class LayerCache:
    def __init__(self, heads: int, head_dim: int, max_cache_frames: int, hidden: int, kernel: int):
        self.attention = AttentionKvCache(heads, head_dim, max_cache_frames)
        self.convolution = CausalConv1dCache(hidden, kernel - 1)


class FastConformerLayer:
    """encoder.rs:498-535: macaron block with five LayerNorms."""

    NORMS = ("norm_feed_forward1", "norm_self_att", "norm_conv", "norm_feed_forward2", "norm_out")

    def __init__(self, ff1, attention, conv, ff2, norms: dict, dtype: str):
        self.ff1, self.attention, self.conv, self.ff2 = ff1, attention, conv, ff2
        self.norms = {k: (rnd(w, dtype), rnd(b, dtype)) for k, (w, b) in norms.items()}
        self.dtype = dtype

    def _ln(self, name, x):
        w, b = self.norms[name]
        return layer_norm(x, w, b, 1e-5, self.dtype)

    def forward(self, x: np.ndarray, cache: LayerCache) -> np.ndarray:
        hidden = residual_add(x, self.ff1(self._ln("norm_feed_forward1", x)), 0.5)
        hidden = residual_add(hidden, self.attention.forward(self._ln("norm_self_att", hidden),
                                                             cache.attention), 1.0)
        hidden = residual_add(hidden, self.conv(self._ln("norm_conv", hidden), cache.convolution), 1.0)
        hidden = residual_add(hidden, self.ff2(self._ln("norm_feed_forward2", hidden)), 0.5)
        return self._ln("norm_out", hidden)


class SubsamplingCache:
    """encoder.rs:12-35."""

    def __init__(self, mel_bins: int, channels: int, kernel: int = 3, stride: int = 2,
                 stages: int = 3):
        left = kernel - stride
        extra = kernel - 1 - left
        freq = mel_bins
        self.layers = []
        for stage in range(stages):
            self.layers.append(CausalConv2dCache(freq, 1 if stage == 0 else channels, left, extra))
            freq = (freq + (kernel - 1) + (stride - 1) - kernel) // stride + 1


class Subsampling:
    """encoder.rs:767-802: stem Conv2D, two depthwise-separable stages, output linear."""

    def __init__(self, stem: Conv2d, stages: list, output: QLinear):
        self.stem, self.stages, self.output = stem, stages, output

    def forward(self, x: np.ndarray, cache: SubsamplingCache) -> np.ndarray:
        time = x.shape[0]
        valid = time
        h = self.stem.forward_causal(x[:, :, None], cache.layers[0])
        valid = self.stem.streaming_output_length(valid)
        h = relu(mask_invalid_time(h, valid))
        for i, (dw, pw) in enumerate(self.stages):
            h = dw.forward_causal(h, cache.layers[i + 1])
            valid = dw.streaming_output_length(valid)
            t, f, c = h.shape
            h = pw(h.reshape(t * f, c)).reshape(t, f, pw.output_dims)
            h = relu(mask_invalid_time(h, valid))
        return self.output(channel_frequency_flatten(h))


class PromptProjector:
    """prompt.rs:110-140: [hidden | one-hot prompt] -> linear1 + ReLU -> linear2."""

    def __init__(self, linear1: QLinear, linear2: QLinear):
        self.linear1, self.linear2 = linear1, linear2
        self.hidden = linear2.output_dims
        self.num_prompts = linear1.input_dims - self.hidden

    def __call__(self, hidden: np.ndarray, prompt_id: int) -> np.ndarray:
        rows = hidden.shape[0]
        if prompt_id >= self.num_prompts:
            raise ValueError("prompt id out of range")
        fused = np.zeros((rows, self.hidden + self.num_prompts), np.float32)
        fused[:, :self.hidden] = hidden
        fused[:, self.hidden + prompt_id] = 1.0
        return self.linear2(self.linear1(fused, act="relu"))


# ------------------------------------------------------------------ model


@dataclasses.dataclass(frozen=True)
class EncoderConfig:
    """encoder.rs:937-955 (``EncoderConfig::nemotron_3_5``) plus the subsampling
    and prompt dimensions that ``StreamingEncoder::from_artifact`` binds."""
    hidden: int = 1024
    ff: int = 4096
    layers: int = 24
    heads: int = 8
    conv_kernel: int = 9
    sliding_window: int = 57          # cached frames = sliding_window - 1
    mel_bins: int = 128
    sub_channels: int = 256
    num_prompts: int = 128
    prompt_hidden: int = 2048
    group: int = 64

    @property
    def cache_frames(self) -> int:
        return self.sliding_window - 1

    @property
    def sub_freq(self) -> int:
        # three stride-2 kernel-3 stages, frequency padded by (kernel-1, stride-1)
        f = self.mel_bins
        for _ in range(3):
            f = (f + 2 + 1 - 3) // 2 + 1
        return f


def linear_names(cfg: EncoderConfig) -> dict[str, tuple[int, int, bool]]:
    """Quantized linears of the encoder: artifact name -> (out, in, has bias)."""
    d, f = cfg.hidden, cfg.ff
    names = {
        "encoder.subsampling.layers.0.pointwise_conv.weight": (cfg.sub_channels, cfg.sub_channels, True),
        "encoder.subsampling.layers.1.pointwise_conv.weight": (cfg.sub_channels, cfg.sub_channels, True),
        "encoder.subsampling.linear.weight": (d, cfg.sub_channels * cfg.sub_freq, True),
        "prompt_projector.linear_1.weight": (cfg.prompt_hidden, d + cfg.num_prompts, True),
        "prompt_projector.linear_2.weight": (d, cfg.prompt_hidden, True),
    }
    for i in range(cfg.layers):
        p = f"encoder.layers.{i}"
        for ffn in ("feed_forward1", "feed_forward2"):
            names[f"{p}.{ffn}.linear1.weight"] = (f, d, False)
            names[f"{p}.{ffn}.linear2.weight"] = (d, f, False)
        for proj in ("q_proj", "k_proj", "v_proj", "o_proj", "relative_k_proj"):
            names[f"{p}.self_attn.{proj}.weight"] = (d, d, False)
        names[f"{p}.conv.pointwise_conv1.weight"] = (2 * d, d, False)
        names[f"{p}.conv.pointwise_conv2.weight"] = (d, d, False)
    return names


def dense_names(cfg: EncoderConfig) -> dict[str, tuple[int, ...]]:
    """Unquantized tensors: artifact name -> shape."""
    d, c = cfg.hidden, cfg.sub_channels
    names = {
        "encoder.subsampling.conv_in.weight": (c, 1, 3, 3),
        "encoder.subsampling.conv_in.bias": (c,),
    }
    for s in range(2):
        names[f"encoder.subsampling.layers.{s}.depthwise_conv.weight"] = (c, 1, 3, 3)
        names[f"encoder.subsampling.layers.{s}.depthwise_conv.bias"] = (c,)
    for i in range(cfg.layers):
        p = f"encoder.layers.{i}"
        names[f"{p}.conv.depthwise_conv.weight"] = (d, 1, cfg.conv_kernel)
        for n in ("conv.norm",) + FastConformerLayer.NORMS:
            names[f"{p}.{n}.weight"] = (d,)
            names[f"{p}.{n}.bias"] = (d,)
        names[f"{p}.self_attn.bias_u"] = (cfg.heads, d // cfg.heads)
        names[f"{p}.self_attn.bias_v"] = (cfg.heads, d // cfg.heads)
    return names


def random_params(cfg: EncoderConfig, seed: int, dtype: str) -> dict:
    """Seeded synthetic weights: f32 dense tensors and quantized linears as
    (q, scales, biases, bias_bits | None) in T."""
    rng = np.random.default_rng(seed)
    params = {}
    for name, (n, k, has_bias) in linear_names(cfg).items():
        w = (rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02))
        q, s, b = qo.quantize(w, cfg.group, dtype)
        bias = qo.to_t(rng.standard_normal(n, dtype=np.float32) * np.float32(0.02), dtype) \
            if has_bias else None
        params[name] = (q, s, b, bias)
    for name, shape in dense_names(cfg).items():
        if name.endswith("norm.weight") or (".norm_" in name and name.endswith(".weight")):
            v = 1.0 + 0.1 * rng.standard_normal(shape, dtype=np.float32)
        elif name.endswith("depthwise_conv.weight") or name.endswith("conv_in.weight"):
            v = rng.standard_normal(shape, dtype=np.float32) / np.float32(3.0)
        else:
            v = 0.02 * rng.standard_normal(shape, dtype=np.float32)
        params[name] = np.asarray(v, np.float32)
    return params


class Encoder:
    """encoder.rs:567-655: subsampling -> FastConformer layers -> prompt projector."""

    def __init__(self, cfg: EncoderConfig, params: dict, dtype: str):
        self.cfg, self.dtype = cfg, dtype
        g = cfg.group

        def lin(name):
            q, s, b, bias = params[name]
            return QLinear(q, s, b, bias, g, dtype)

        c = cfg.sub_channels
        stem = Conv2d(params["encoder.subsampling.conv_in.weight"],
                      params["encoder.subsampling.conv_in.bias"], 2, 1, dtype)
        stages = []
        for s in range(2):
            p = f"encoder.subsampling.layers.{s}"
            stages.append((Conv2d(params[f"{p}.depthwise_conv.weight"], params[f"{p}.depthwise_conv.bias"],
                                  2, c, dtype), lin(f"{p}.pointwise_conv.weight")))
        self.subsampling = Subsampling(stem, stages, lin("encoder.subsampling.linear.weight"))
        self.layers = []
        for i in range(cfg.layers):
            p = f"encoder.layers.{i}"
            ff1 = FeedForward(lin(f"{p}.feed_forward1.linear1.weight"), lin(f"{p}.feed_forward1.linear2.weight"))
            ff2 = FeedForward(lin(f"{p}.feed_forward2.linear1.weight"), lin(f"{p}.feed_forward2.linear2.weight"))
            att = RelPosAttention(*(lin(f"{p}.self_attn.{n}.weight")
                                    for n in ("q_proj", "k_proj", "v_proj", "o_proj", "relative_k_proj")),
                                  rnd(params[f"{p}.self_attn.bias_u"], dtype),
                                  rnd(params[f"{p}.self_attn.bias_v"], dtype), cfg.heads)
            dw_w = params[f"{p}.conv.depthwise_conv.weight"].reshape(cfg.hidden, cfg.conv_kernel)
            conv = ConvModule(lin(f"{p}.conv.pointwise_conv1.weight"),
                              DepthwiseConv1d(dw_w, np.zeros(cfg.hidden, np.float32), dtype),
                              params[f"{p}.conv.norm.weight"], params[f"{p}.conv.norm.bias"],
                              lin(f"{p}.conv.pointwise_conv2.weight"), dtype)
            norms = {n: (params[f"{p}.{n}.weight"], params[f"{p}.{n}.bias"])
                     for n in FastConformerLayer.NORMS}
            self.layers.append(FastConformerLayer(ff1, att, conv, ff2, norms, dtype))
        self.prompt = PromptProjector(lin("prompt_projector.linear_1.weight"),
                                      lin("prompt_projector.linear_2.weight"))

    def new_cache(self):
        cfg = self.cfg
        return {
            "subsampling": SubsamplingCache(cfg.mel_bins, cfg.sub_channels),
            "layers": [LayerCache(cfg.heads, cfg.hidden // cfg.heads, cfg.cache_frames, cfg.hidden,
                                  cfg.conv_kernel) for _ in range(cfg.layers)],
        }

    def encode_chunk(self, features: np.ndarray, prompt_id: int, cache: dict,
                     trace: list | None = None) -> np.ndarray:
        """features f32 [time, mel_bins] -> f32 [frames, hidden] (T values)."""
        h = self.subsampling.forward(np.asarray(features, np.float32), cache["subsampling"])
        if trace is not None:
            trace.append(h)
        for layer, lc in zip(self.layers, cache["layers"]):
            h = layer.forward(h, lc)
            if trace is not None:
                trace.append(h)
        return self.prompt(h, prompt_id)


def chunk_audio_seconds(mel_frames: int) -> float:
    """10 ms mel hop: a chunk of N mel frames carries N * 10 ms of audio."""
    return mel_frames * 0.010

