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
        `margins` collects the top-1 / top-2 logit gap of every decision."""
        dec = self.prediction.step(self.cfg.blank, st)
        enc_all = self.enc_proj(encoded)
        out = []
        for frame in range(encoded.shape[0]):
            for _ in range(self.cfg.max_symbols):
                logits = self.joint.logits(enc_all[frame], dec)
                token = int(np.argmax(logits))
                if margins is not None:
                    top = np.sort(logits)[-2:]
                    margins.append(float(top[1] - top[0]))
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
