"""Generate encoder_small.npz, the fixture that pins the encoder + adaptor oracle
(oracle/encoder.py) against an independent formulation of the same graphs.

Run in the build container (needs torch and gguf-py):
    python tests/golden/make_encoder_golden.py

The formulation here follows the reference's graph definitions
(compute/encoder_ops.cpp:17-290, compute/adaptor_ops.cpp:11-149) with PyTorch's own
operators in float64, written apart from the oracle's numpy code:
  * Q8_0 weights dequantised by gguf-py's quantisation module (gguf.quants), not by the
    oracle's codec;
  * LayerNorm by torch.nn.functional.layer_norm (eps 1e-5 in the encoder, 1e-12 in the
    adaptor);
  * the FSMN memory as a depthwise Conv1d (groups = channels) over the value sequence
    zero-padded by (K-1)/2 - shift on the left and the rest on the right, plus the
    values themselves (compute/encoder_ops.cpp:57-110 builds it from shifted slices);
  * attention by torch.nn.functional.scaled_dot_product_attention (no mask: the encoder
    and adaptor attend both ways), heads split from the projection columns.
The weights are fa_synth.make_encoder_weights(seed) of a 3 + 2-layer encoder; the fixture
stores the seed, a checksum of the weights, the LFR inputs and both outputs for two
utterance lengths (5 frames, shorter than the FSMN kernel, and 21).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "funasr-ggml_b200"))
sys.path.insert(0, HERE)

import fa_synth  # noqa: E402
from make_golden import weights_checksum  # noqa: E402

ENC_CFG = dict(fa_synth.ENCODER, num_blocks=3, tp_blocks=2)
ENC_SEED = 4321
FRAMES = (5, 21)


def _tensor(w, name):
    """float64 torch tensor [ne1][ne0] (or [ne0]) of a GGUF-form weight."""
    import torch
    from gguf import GGMLQuantizationType
    from gguf.quants import dequantize
    t, ne, arr = w[name]
    n0 = int(ne[0])
    n1 = int(ne[1]) if len(ne) > 1 else 1
    if t == 8:
        a = dequantize(np.ascontiguousarray(arr).reshape(n1, -1), GGMLQuantizationType.Q8_0).astype(np.float64)
    elif t == 1:
        a = np.ascontiguousarray(arr, np.uint16).view(np.float16).astype(np.float64)
    elif t == 30:
        a = (np.ascontiguousarray(arr, np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    else:
        a = np.ascontiguousarray(arr, np.float32).astype(np.float64)
    a = torch.from_numpy(np.ascontiguousarray(a.reshape(n1, n0)))
    return a if n1 > 1 else a[0]


def _sanm_layer(w, p, x, cfg, residual):
    import torch
    import torch.nn.functional as F
    g = lambda n: _tensor(w, p + n)
    h = F.layer_norm(x, (x.shape[-1],), g(".norm1.weight"), g(".norm1.bias"), 1e-5)
    q = F.linear(h, g(".self_attn.linear_q.weight"), g(".self_attn.linear_q.bias"))
    k = F.linear(h, g(".self_attn.linear_k.weight"), g(".self_attn.linear_k.bias"))
    v = F.linear(h, g(".self_attn.linear_v.weight"), g(".self_attn.linear_v.bias"))
    T, C = v.shape
    K = cfg["kernel_size"]
    left = (K - 1) // 2 - cfg["sanm_shift"]
    taps = g(".self_attn.fsmn_block.weight").reshape(C, 1, K)
    conv = F.conv1d(F.pad(v.T.unsqueeze(0), (left, K - 1 - left)), taps, groups=C)[0].T
    mem = conv + v
    H = cfg["attention_heads"]
    split = lambda t: t.reshape(T, H, -1).transpose(0, 1)
    o = F.scaled_dot_product_attention(split(q), split(k), split(v)).transpose(0, 1).reshape(T, -1)
    att = F.linear(o, g(".self_attn.linear_out.weight"), g(".self_attn.linear_out.bias")) + mem
    x = x + att if residual else att
    h = F.layer_norm(x, (x.shape[-1],), g(".norm2.weight"), g(".norm2.bias"), 1e-5)
    f = F.linear(torch.relu(F.linear(h, g(".feed_forward.w_1.weight"), g(".feed_forward.w_1.bias"))),
                 g(".feed_forward.w_2.weight"), g(".feed_forward.w_2.bias"))
    return x + f


def encoder_torch(w, x, cfg):
    import torch
    import torch.nn.functional as F
    g = lambda n: _tensor(w, n)
    x = torch.from_numpy(np.asarray(x, np.float64)) * float(np.sqrt(cfg["output_size"]))
    x = _sanm_layer(w, "audio_encoder.encoders0.0", x, cfg, False)
    for i in range(cfg["num_blocks"] - 1):
        x = _sanm_layer(w, f"audio_encoder.encoders.{i}", x, cfg, True)
    x = F.layer_norm(x, (x.shape[-1],), g("audio_encoder.after_norm.weight"), g("audio_encoder.after_norm.bias"), 1e-5)
    for i in range(cfg["tp_blocks"]):
        x = _sanm_layer(w, f"audio_encoder.tp_encoders.{i}", x, cfg, True)
    return F.layer_norm(x, (x.shape[-1],), g("audio_encoder.tp_norm.weight"), g("audio_encoder.tp_norm.bias"), 1e-5)


def adaptor_torch(w, x, acfg=fa_synth.ADAPTOR):
    import torch
    import torch.nn.functional as F
    g = lambda n: _tensor(w, n)
    x = torch.relu(F.linear(x, g("audio_adaptor.linear1.weight"), g("audio_adaptor.linear1.bias")))
    x = F.linear(x, g("audio_adaptor.linear2.weight"), g("audio_adaptor.linear2.bias"))
    T = x.shape[0]
    H = acfg["attention_heads"]
    split = lambda t: t.reshape(T, H, -1).transpose(0, 1)
    for i in range(acfg["num_blocks"]):
        p = f"audio_adaptor.blocks.{i}"
        h = F.layer_norm(x, (x.shape[-1],), g(p + ".norm1.weight"), g(p + ".norm1.bias"), 1e-12)
        q, k, v = (F.linear(h, g(p + f".self_attn.{n}.weight"), g(p + f".self_attn.{n}.bias"))
                   for n in ("linear_q", "linear_k", "linear_v"))
        o = F.scaled_dot_product_attention(split(q), split(k), split(v)).transpose(0, 1).reshape(T, -1)
        x = x + F.linear(o, g(p + ".self_attn.linear_out.weight"), g(p + ".self_attn.linear_out.bias"))
        h = F.layer_norm(x, (x.shape[-1],), g(p + ".norm2.weight"), g(p + ".norm2.bias"), 1e-12)
        f = torch.relu(F.linear(h, g(p + ".feed_forward.w_1.weight"), g(p + ".feed_forward.w_1.bias")))
        x = x + F.linear(f, g(p + ".feed_forward.w_2.weight"), g(p + ".feed_forward.w_2.bias"))
    return x


def main():
    w = fa_synth.make_encoder_weights(ENC_CFG, seed=ENC_SEED)
    out = {"seed": ENC_SEED, "checksum": weights_checksum(w)}
    rng = np.random.default_rng(99)
    for T in FRAMES:
        x = fa_synth.lfr_features(rng, T)
        enc = encoder_torch(w, x, ENC_CFG)
        out[f"x{T}"] = x
        out[f"enc{T}"] = enc.numpy()
        out[f"ada{T}"] = adaptor_torch(w, enc).numpy()
    np.savez_compressed(os.path.join(HERE, "encoder_small.npz"), **out)
    print("encoder_small.npz")


if __name__ == "__main__":
    main()
