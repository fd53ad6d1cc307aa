"""CPU restatement of FunASR-GGML's audio encoder (SANM) and adaptor, the producer of
the decoder's prefill embeddings.

TEST INFRASTRUCTURE ONLY: imported by tests/ and bench.py's baseline legs as the
checker of the CUDA encoder; the product library never calls it.

What it restates (reference paths are relative to the FunASR-GGML tree):
  compute/encoder_ops.cpp:17-30    layer_norm = ggml_norm(x, 1e-5) * w + b
  compute/encoder_ops.cpp:35-44    linear_with_bias = W . x + b
  compute/encoder_ops.cpp:57-110   FSMN: out[c, t] = sum_k v[c, t + k - pad] w[c, k] + v[c, t]
                                   (depthwise, zero outside [0, T)), pad = (K - 1) / 2 - shift
  compute/encoder_ops.cpp:135-196  SANM attention: q, k, v projections, FSMN on v, 4-head
                                   bidirectional attention (q / sqrt(head_dim), softmax over
                                   keys), output projection, plus the FSMN memory
  compute/encoder_ops.cpp:210-240  layer: norm1 -> SANM -> residual (not in encoder0,
                                   560 -> 512), norm2 -> FFN (w1, ReLU, w2) -> residual
  compute/encoder_ops.cpp:255-290  encoder: x * sqrt(512), encoder0, 49 main layers,
                                   after_norm, 20 tp layers, tp_norm
  compute/adaptor_ops.cpp:11-149   adaptor: linear1 -> ReLU -> linear2, then 2 blocks of
                                   LayerNorm (eps 1e-12) -> 8-head attention -> residual,
                                   LayerNorm -> FFN (1024 -> 256 -> 1024, ReLU) -> residual
ggml_norm: (x - mean) / sqrt(mean((x - mean)^2) + eps) over the feature dimension.
Weights follow model/loader.cpp:21-80,135-200 (audio_encoder.*, audio_adaptor.*). Two
weight arithmetics, as for the decoder: exact dequantised weights, or (w16=True) the
weights rounded once to f16 as the CUDA path stores them. Activations are float64.
"""
from __future__ import annotations

import numpy as np

import oracle as _o

TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_BF16 = 0, 1, 8, 30

ENCODER = dict(input_dim=560, output_size=512, attention_heads=4, linear_units=2048, num_blocks=50,
               tp_blocks=20, kernel_size=11, sanm_shift=0)
ADAPTOR = dict(input_dim=512, hidden_dim=2048, output_dim=1024, num_blocks=2, attention_heads=8, ffn_dim=256)


def weight_f64(t, ne, arr, w16=True):
    """[ne1][ne0] float64 matrix (or vector) of a GGUF tensor."""
    n0 = int(ne[0])
    n1 = int(ne[1]) if len(ne) > 1 else 1
    if t == TYPE_Q8_0:
        w = _o.q8_0_dequant(np.ascontiguousarray(arr).reshape(n1, -1), n0)
        if w16:
            w = w.astype(np.float16).astype(np.float32)
    elif t == TYPE_BF16:
        w = _o.bf16_bits_to_f32(np.ascontiguousarray(arr, np.uint16).ravel())
        if w16:
            w = w.astype(np.float16).astype(np.float32)
    elif t == TYPE_F16:
        w = _o.f16_bits_to_f32(np.ascontiguousarray(arr, np.uint16).ravel())
    else:
        w = np.ascontiguousarray(arr, np.float32).ravel()
    w = np.asarray(w, np.float64).reshape(n1, n0)
    return w if n1 > 1 else w[0]


def layer_norm(x, w, b, eps):
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    return (x - mu) / np.sqrt(var + eps) * w + b


def fsmn(v, w, pad):
    """v [T][C], w [C][K]: depthwise conv over time plus v."""
    T, C = v.shape
    K = w.shape[1]
    out = v.copy()
    for k in range(K):
        s = k - pad
        if abs(s) >= T:
            continue
        if s >= 0:
            out[: T - s] += v[s:] * w[:, k]
        else:
            out[-s:] += v[: T + s] * w[:, k]
    return out


def mha(q, k, v, n_heads):
    T, D = q.shape
    hd = D // n_heads
    out = np.empty((T, v.shape[1]))
    vd = v.shape[1] // n_heads
    for h in range(n_heads):
        qh = q[:, h * hd:(h + 1) * hd] / np.sqrt(hd)
        s = qh @ k[:, h * hd:(h + 1) * hd].T
        s = np.exp(s - s.max(1, keepdims=True))
        s /= s.sum(1, keepdims=True)
        out[:, h * vd:(h + 1) * vd] = s @ v[:, h * vd:(h + 1) * vd]
    return out


class _W:
    def __init__(self, w, w16):
        self.w, self.w16 = w, w16

    def __call__(self, name):
        t, ne, arr = self.w[name]
        return weight_f64(t, ne, arr, self.w16)


def _linear(W, p, x):
    return x @ W(p + ".weight").T + W(p + ".bias")


def encoder_layer(W, p, x, cfg, residual):
    pad = (cfg["kernel_size"] - 1) // 2 - cfg["sanm_shift"]
    x1 = layer_norm(x, W(p + ".norm1.weight"), W(p + ".norm1.bias"), 1e-5)
    q = _linear(W, p + ".self_attn.linear_q", x1)
    k = _linear(W, p + ".self_attn.linear_k", x1)
    v = _linear(W, p + ".self_attn.linear_v", x1)
    fw = W(p + ".self_attn.fsmn_block.weight")           # [C][K] (ggml ne [K, 1, C])
    mem = fsmn(v, fw.reshape(v.shape[1], cfg["kernel_size"]), pad)
    att = _linear(W, p + ".self_attn.linear_out", mha(q, k, v, cfg["attention_heads"])) + mem
    x = x + att if residual else att
    x2 = layer_norm(x, W(p + ".norm2.weight"), W(p + ".norm2.bias"), 1e-5)
    h = np.maximum(_linear(W, p + ".feed_forward.w_1", x2), 0.0)
    return x + _linear(W, p + ".feed_forward.w_2", h)


def encoder_forward(w, x, cfg=ENCODER, w16=True):
    """x [T][560] LFR features -> [T][512]."""
    W = _W(w, w16)
    x = np.asarray(x, np.float64) * np.sqrt(cfg["output_size"])
    x = encoder_layer(W, "audio_encoder.encoders0.0", x, cfg, False)
    for i in range(cfg["num_blocks"] - 1):
        x = encoder_layer(W, f"audio_encoder.encoders.{i}", x, cfg, True)
    x = layer_norm(x, W("audio_encoder.after_norm.weight"), W("audio_encoder.after_norm.bias"), 1e-5)
    for i in range(cfg["tp_blocks"]):
        x = encoder_layer(W, f"audio_encoder.tp_encoders.{i}", x, cfg, True)
    return layer_norm(x, W("audio_encoder.tp_norm.weight"), W("audio_encoder.tp_norm.bias"), 1e-5)


def adaptor_forward(w, x, cfg=ADAPTOR, w16=True):
    """x [T][512] -> [T][1024] decoder input embeddings."""
    W = _W(w, w16)
    x = np.maximum(_linear(W, "audio_adaptor.linear1", np.asarray(x, np.float64)), 0.0)
    x = _linear(W, "audio_adaptor.linear2", x)
    for i in range(cfg["num_blocks"]):
        p = f"audio_adaptor.blocks.{i}"
        x1 = layer_norm(x, W(p + ".norm1.weight"), W(p + ".norm1.bias"), 1e-12)
        q = _linear(W, p + ".self_attn.linear_q", x1)
        k = _linear(W, p + ".self_attn.linear_k", x1)
        v = _linear(W, p + ".self_attn.linear_v", x1)
        x = x + _linear(W, p + ".self_attn.linear_out", mha(q, k, v, cfg["attention_heads"]))
        x2 = layer_norm(x, W(p + ".norm2.weight"), W(p + ".norm2.bias"), 1e-12)
        h = np.maximum(_linear(W, p + ".feed_forward.w_1", x2), 0.0)
        x = x + _linear(W, p + ".feed_forward.w_2", h)
    return x
