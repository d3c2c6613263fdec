"""CPU restatement of the RNNT greedy decoder (TEST INFRASTRUCTURE).

Only the test suite, the smoke check and the benchmark's CPU-baseline leg use
this module; the CUDA library never calls it.  It restates
crates/nemotron-mlx/src/model/rnnt.rs:

* ``LstmCell::step_f32`` (:113-148): gates = ih(x) + hh(h) + bias with every
  MLX op rounding to T (the two linears' outputs, each add), PyTorch's
  i, f, g, o gate order, sigmoid / tanh results in T, c = f*c + i*g and
  h = o * tanh(c) with a T rounding after every product and sum;
* ``LstmCell::from_artifact`` (:86-111): bias = T(bias_ih) + T(bias_hh) in T;
* ``QuantizedEmbedding`` (:153-208): dequantised once to T, row lookup;
* ``PredictionNetwork::step`` (:273-290): a blank after initialisation returns
  the cached projector output without advancing the LSTMs;
* ``JointNetwork::score`` (:321-333): relu(enc + dec) in f32, the head linear
  in T, argmax (first maximum);
* ``StreamingRnntDecoder::decode_frames`` (:364-388) and ``GreedyRnnt``
  (:392-418): per frame, up to max_symbols emissions, stopping at blank.

Elementwise ops compute in f32 and round to T, standing in for MLX's f16 /
bf16 kernels (bit agreement with MLX's Metal math is unpinned).  Pinned by
tests/test_rnnt_oracle.py against crates/nemotron-mlx/tests/rnnt_decode.rs.
"""
from __future__ import annotations

import dataclasses

import numpy as np

import oracle as qo
from encoder_oracle import QLinear, rnd


def _sigmoid(x: np.ndarray) -> np.ndarray:
    one = np.float32(1.0)
    with np.errstate(over="ignore"):
        return (one / (one + np.exp(-x.astype(np.float32)))).astype(np.float32)


class LstmCell:
    def __init__(self, ih: QLinear, hh: QLinear, bias_ih, bias_hh, dtype: str):
        self.ih, self.hh, self.dtype = ih, hh, dtype
        self.hidden = ih.input_dims
        self.bias = rnd(rnd(bias_ih, dtype) + rnd(bias_hh, dtype), dtype)

    def step(self, x: np.ndarray, h: np.ndarray, c: np.ndarray):
        """x, h, c f32 [H] (T values) -> (h', c')."""
        T = self.dtype
        H = self.hidden
        gates = rnd(rnd(self.ih(x[None, :])[0] + self.hh(h[None, :])[0], T) + self.bias, T)
        i = rnd(_sigmoid(gates[:H]), T)
        f = rnd(_sigmoid(gates[H:2 * H]), T)
        g = rnd(np.tanh(gates[2 * H:3 * H]), T)
        o = rnd(_sigmoid(gates[3 * H:]), T)
        c_prev = rnd(c, T)
        c_new = rnd(rnd(f * c_prev, T) + rnd(i * g, T), T)
        h_new = rnd(o * rnd(np.tanh(c_new), T), T)
        return h_new, c_new


class PredictionNetwork:
    def __init__(self, embedding: np.ndarray, cells: list, projector: QLinear, blank: int):
        self.embedding = embedding  # [V, H] f32 of T values
        self.cells, self.projector, self.blank = cells, projector, blank

    def new_state(self):
        H = self.embedding.shape[1]
        return {"h": [np.zeros(H, np.float32) for _ in self.cells],
                "c": [np.zeros(H, np.float32) for _ in self.cells],
                "out": np.zeros(self.projector.output_dims, np.float32), "init": False}

    def step(self, token: int, st: dict) -> np.ndarray:
        if st["init"] and token == self.blank:
            return st["out"].copy()
        x = self.embedding[token]
        for l, cell in enumerate(self.cells):
            st["h"][l], st["c"][l] = cell.step(x, st["h"][l], st["c"][l])
            x = st["h"][l]
        st["out"] = self.projector(x[None, :])[0]
        st["init"] = True
        return st["out"].copy()


class Joint:
    def __init__(self, head: QLinear):
        self.head = head

    def logits(self, enc: np.ndarray, dec: np.ndarray) -> np.ndarray:
        fused = np.maximum((enc.astype(np.float32) + dec.astype(np.float32)).astype(np.float32),
                           np.float32(0.0))
        return self.head(fused[None, :])[0]

    def score(self, enc: np.ndarray, dec: np.ndarray) -> int:
        return int(np.argmax(self.logits(enc, dec)))


def greedy_decode_with(frame_count: int, blank: int, max_symbols: int, score):
    """rnnt.rs:392-418 (GreedyRnnt::decode_with)."""
    out = []
    for frame in range(frame_count):
        for symbol in range(max_symbols):
            token = score(frame, symbol)
            if token == blank:
                break
            out.append((token, frame))
    return out


@dataclasses.dataclass(frozen=True)
class RnntConfig:
    enc_hidden: int = 1024
    pred_hidden: int = 640
    joint_hidden: int = 640
    vocab: int = 1025
    layers: int = 2
    max_symbols: int = 10
    group: int = 64

    @property
    def blank(self) -> int:
        return self.vocab - 1


def linear_names(cfg: RnntConfig) -> dict:
    H = cfg.pred_hidden
    names = {
        "encoder_projector.weight": (cfg.joint_hidden, cfg.enc_hidden, True),
        "decoder.decoder_projector.weight": (cfg.joint_hidden, H, True),
        "joint.head.weight": (cfg.vocab, cfg.joint_hidden, True),
        "decoder.embedding.weight": (cfg.vocab, H, False),
    }
    for l in range(cfg.layers):
        names[f"decoder.lstm.weight_ih_l{l}"] = (4 * H, H, False)
        names[f"decoder.lstm.weight_hh_l{l}"] = (4 * H, H, False)
    return names


def dense_names(cfg: RnntConfig) -> dict:
    return {f"decoder.lstm.bias_{k}_l{l}": (4 * cfg.pred_hidden,)
            for l in range(cfg.layers) for k in ("ih", "hh")}


def random_params(cfg: RnntConfig, seed: int, dtype: str) -> dict:
    rng = np.random.default_rng(seed)
    params = {}
    for name, (n, k, has_bias) in linear_names(cfg).items():
        w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
        if name == "decoder.embedding.weight":
            w = rng.standard_normal((n, k), dtype=np.float32)
        q, s, b = qo.quantize(w, cfg.group, dtype)
        bias = qo.to_t(rng.standard_normal(n, dtype=np.float32) * np.float32(0.02), dtype) \
            if has_bias else None
        params[name] = (q, s, b, bias)
    for name, shape in dense_names(cfg).items():
        params[name] = (0.02 * rng.standard_normal(shape)).astype(np.float32)
    return params


# Wide-margin decoder ("trained-like").  Every structural weight is 255 * 2^-k,
# so in its group of zeros the scale (w / 255 with the edge/sign rule) is
# exact in f16 and bf16 and the zeros dequantise to exactly 0: nothing but the
# intended paths carries signal, and every greedy decision stays several logit
# units from the runner-up.
_ONE = 255.0 / 256.0     # one-hot embedding and encoder pass-through weight
_GATE_OPEN = 6.0         # input / output gate bias (sigmoid ~ 0.9975); forget gate -6
_LSTM_GAIN = 255.0 / 64.0  # g-gate weight: a one-hot input -> ~0.757 one-hot output per layer
_SUPPRESS_W = -255.0 / 32.0  # decoder projector: last token's unit -> its joint coordinate
_LIFT_W = 255.0 / 512.0  # decoder projector: "a token was emitted" unit -> blank's coordinate
_HEAD_GAIN = 255.0 / 64.0
_BLANK_BIAS = 1.5
_OTHER_BIAS = -8.0


def structured_params(cfg: RnntConfig, seed: int, dtype: str, active: int = 48):
    """Parameters of a decoder whose greedy decisions all have wide margins.

    It behaves like a trained transducer on synthetic "phone" frames: the
    encoder projector passes encoder channel c to joint coordinate c; active
    token i (vocabulary id tokens[i]) is embedded as prediction unit i plus a
    shared unit (the last one), which both LSTM layers carry through (input and
    output gates open, forget gate closed, g-gate = gain * identity); the
    decoder projector turns unit i into a push of about -6 on joint coordinate
    i (the last token is not repeated) and the shared unit into about +0.38 on
    blank's coordinate (the last joint unit); the head reads token i from
    coordinate i and blank from its own, with a blank bias.  So a frame
    carrying strength 2-4 on channel i emits token i once and then blank, a
    strength above about 6.8 repeats the token up to max_symbols, and two
    channels alternate up to the cap.  Head rows of the inactive tokens are
    N(0, 0.02) noise under a -8 bias.  Returns (params, tokens)."""
    rng = np.random.default_rng(seed)
    H, J, E, V = cfg.pred_hidden, cfg.joint_hidden, cfg.enc_hidden, cfg.vocab
    if not (active < min(H, J) - 1 and J <= E):
        raise ValueError("structured decoder needs active < hidden sizes and joint <= encoder")
    tokens = rng.choice(cfg.blank, size=active, replace=False).astype(np.int64)
    idx = np.arange(active)
    bc = J - 1  # blank's joint coordinate
    shared = H - 1  # prediction unit set by every active token
    f = np.float32
    params = {}

    def put(name, w, bias=None):
        q, s, b = qo.quantize(w, cfg.group, dtype)
        params[name] = (q, s, b, None if bias is None else qo.to_t(np.asarray(bias, f), dtype))

    w = np.zeros((J, E), f)
    w[np.arange(J), np.arange(J)] = _ONE
    put("encoder_projector.weight", w, np.zeros(J, f))
    w = np.zeros((V, H), f)
    w[tokens, idx] = _ONE
    w[tokens, shared] = _ONE
    put("decoder.embedding.weight", w)
    for l in range(cfg.layers):
        w = np.zeros((4 * H, H), f)
        w[2 * H + np.arange(H), np.arange(H)] = _LSTM_GAIN
        put(f"decoder.lstm.weight_ih_l{l}", w)
        put(f"decoder.lstm.weight_hh_l{l}", np.zeros((4 * H, H), f))
        params[f"decoder.lstm.bias_ih_l{l}"] = np.concatenate(
            [np.full(H, _GATE_OPEN), np.full(H, -_GATE_OPEN), np.zeros(H), np.full(H, _GATE_OPEN)]
        ).astype(f)
        params[f"decoder.lstm.bias_hh_l{l}"] = np.zeros(4 * H, f)
    w = np.zeros((J, H), f)
    w[idx, idx] = _SUPPRESS_W
    w[bc, shared] = _LIFT_W
    put("decoder.decoder_projector.weight", w, np.zeros(J, f))
    w = (rng.standard_normal((V, J)) * 0.02).astype(f)
    w[tokens] = 0.0
    w[cfg.blank] = 0.0
    w[tokens, idx] = _HEAD_GAIN
    w[cfg.blank, bc] = _HEAD_GAIN
    bias = np.full(V, _OTHER_BIAS, f)
    bias[tokens] = 0.0
    bias[cfg.blank] = _BLANK_BIAS
    put("joint.head.weight", w, bias)
    return params, tokens


def structured_frames(rng, streams: int, frames: int, enc_hidden: int, active: int) -> np.ndarray:
    """Encoder frames for structured_params: f32 [streams, frames, enc_hidden]
    of N(0, 0.02) noise where each frame is silence (30 %), one token of
    strength 2-4 (45 %: emits once, then blank), two tokens of strengths 3.5-4
    and 2-3 (15 %: alternate up to the cap) or one strong token of 8.5-9.5
    (10 %: repeats up to the cap)."""
    x = (rng.standard_normal((streams, frames, enc_hidden)) * 0.02).astype(np.float32)
    kind = rng.random((streams, frames))
    for s in range(streams):
        for t in range(frames):
            a, b = rng.choice(active, size=2, replace=False)
            if kind[s, t] < 0.30:
                continue
            if kind[s, t] < 0.75:
                x[s, t, a] += rng.uniform(2.0, 4.0)
            elif kind[s, t] < 0.90:
                x[s, t, a] += rng.uniform(3.5, 4.0)
                x[s, t, b] += rng.uniform(2.0, 3.0)
            else:
                x[s, t, a] += rng.uniform(8.5, 9.5)
    return x


class RnntDecoder:
    """rnnt.rs:336-388: encoder projector + prediction network + joint."""

    def __init__(self, cfg: RnntConfig, params: dict, dtype: str):
        self.cfg, self.dtype = cfg, dtype
        g = cfg.group

        def lin(name):
            q, s, b, bias = params[name]
            return QLinear(q, s, b, bias, g, dtype)

        self.enc_proj = lin("encoder_projector.weight")
        q, s, b, _ = params["decoder.embedding.weight"]
        emb = rnd(qo.dequantize(q, s, b, g, dtype), dtype)
        cells = [LstmCell(lin(f"decoder.lstm.weight_ih_l{l}"), lin(f"decoder.lstm.weight_hh_l{l}"),
                          params[f"decoder.lstm.bias_ih_l{l}"], params[f"decoder.lstm.bias_hh_l{l}"],
                          dtype) for l in range(cfg.layers)]
        self.prediction = PredictionNetwork(emb, cells, lin("decoder.decoder_projector.weight"),
                                            cfg.blank)
        self.joint = Joint(lin("joint.head.weight"))

    def new_state(self):
        return self.prediction.new_state()

    def decode_frames(self, encoded: np.ndarray, st: dict, margins: list | None = None):
        """encoded f32 [frames, enc_hidden] -> [(token, frame)] (frame local to the call).
        `margins` collects the top-1 / top-2 logit gap of every decision, in T
        ulps of the top logit."""
        dec = self.prediction.step(self.cfg.blank, st)
        enc_all = self.enc_proj(encoded)
        out = []
        for frame in range(encoded.shape[0]):
            for _ in range(self.cfg.max_symbols):
                logits = self.joint.logits(enc_all[frame], dec)
                token = int(np.argmax(logits))
                if margins is not None:
                    top = np.sort(logits)[-2:]
                    margins.append(float(top[1] - top[0]) / t_ulp(top[1], self.dtype))
                if token == self.cfg.blank:
                    break
                out.append((token, frame))
                dec = self.prediction.step(token, st)
        return out


def t_ulp(v: float, dtype: str) -> float:
    """Spacing of T at magnitude |v|."""
    mant = {"bf16": 7, "f16": 10}[dtype]
    m = max(abs(float(v)), 2.0 ** -14)
    return 2.0 ** (np.floor(np.log2(m)) - mant)


def check_path(dec: RnntDecoder, encoded: np.ndarray, st: dict, path: list, tol_ulps: float = 8.0):
    """Teacher-forced check of a decoded chunk: replays `path` [(token, frame)]
    (another implementation's greedy choices) through this decoder and, at
    every decision, compares the choice with this decoder's argmax.  A choice
    that differs counts as a near tie when its logit is within tol_ulps T ulps
    of the maximum, otherwise as a mismatch.  Advances `st` along the path."""
    cfg = dec.cfg
    stats = {"decisions": 0, "differ": 0, "mismatch": 0, "min_margin": np.inf}
    out = dec.prediction.step(cfg.blank, st)
    enc_all = dec.enc_proj(encoded)
    for frame in range(encoded.shape[0]):
        chosen = [t for t, f in path if f == frame]
        if len(chosen) > cfg.max_symbols:
            stats["mismatch"] += 1
        for k in range(cfg.max_symbols):
            logits = dec.joint.logits(enc_all[frame], out)
            best = int(np.argmax(logits))
            choice = chosen[k] if k < len(chosen) else cfg.blank
            top = np.sort(logits)[-2:]
            stats["min_margin"] = min(stats["min_margin"], float(top[1] - top[0]))
            stats["decisions"] += 1
            if choice != best:
                stats["differ"] += 1
                if logits[choice] < logits[best] - tol_ulps * t_ulp(logits[best], dec.dtype):
                    stats["mismatch"] += 1
            if choice == cfg.blank:
                break
            out = dec.prediction.step(choice, st)
    return stats
