"""Seeded random-init decoder weights and synthetic inputs (no checkpoints, no datasets).

Weights follow the reference's Q8_0 build (tools/hf_convert_ggml_q8.py:312-320):
every 2-D projection and lm_head is Q8_0, embed_tokens and the norms BF16.
Q8_0 blocks are drawn directly: int8 values ~ U[-127, 127], f16 scales
~ U(0.001, 0.02). Tensor names follow model/loader.cpp:91-117,217-227.
"""
from __future__ import annotations

from typing import Dict, Tuple

import numpy as np

TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_BF16 = 0, 1, 8, 30

# Qwen3-0.6B decoder of FunASR-Nano (funasr_gguf.md header; core/config.hpp:119-136).
QWEN3_06B = dict(n_layers=28, hidden=1024, n_heads=16, n_kv_heads=8, head_dim=128, ffn=3072, vocab=151936,
                 eps=1e-5, rope_base=1e6)


def small_config(n_layers=2, hidden=256, ffn=512, vocab=2048):
    """Same attention geometry (16/8 heads x 128), fewer/smaller everything else."""
    return dict(QWEN3_06B, n_layers=n_layers, hidden=hidden, ffn=ffn, vocab=vocab)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def q8_0_random(rng: np.random.Generator, n: int, k: int, d_lo=0.001, d_hi=0.02) -> np.ndarray:
    """[n][k/32*34] uint8 Q8_0 rows with random int8 values and f16 scales."""
    nb = k // 32
    blocks = np.empty((n, nb, 34), np.uint8)
    d = rng.uniform(d_lo, d_hi, size=(n, nb)).astype(np.float16)
    blocks[:, :, :2] = d.view(np.uint8).reshape(n, nb, 2)
    blocks[:, :, 2:] = rng.integers(-127, 128, size=(n, nb, 32), dtype=np.int8).view(np.uint8)
    return blocks.reshape(n, nb * 34)


def make_weights(cfg: dict, seed: int = 0, d_range=(0.001, 0.02)) -> Dict[str, Tuple[int, Tuple[int, int], np.ndarray]]:
    """name -> (ggml type, ne (input dim first), data) for one random-init decoder.

    d_range is the range of the Q8_0 block scales. The default (0.001, 0.02) is the
    steady-state benchmark's; it gives logits of order +-150. (0.0002, 0.004) gives the
    +-25 logits of a trained Qwen3."""
    rng = np.random.default_rng(seed)
    lo, hi = d_range
    H, F, V = cfg["hidden"], cfg["ffn"], cfg["vocab"]
    QD = cfg["n_heads"] * cfg["head_dim"]
    KD = cfg["n_kv_heads"] * cfg["head_dim"]
    D = cfg["head_dim"]
    w = {}

    def bf16(shape, lo, hi):
        return f32_to_bf16_bits(rng.uniform(lo, hi, size=shape).astype(np.float32))

    w["llm.model.embed_tokens.weight"] = (TYPE_BF16, (H, V), f32_to_bf16_bits(
        (rng.standard_normal((V, H), dtype=np.float32) * 0.05)))
    w["llm.model.norm.weight"] = (TYPE_BF16, (H, 1), bf16(H, 0.8, 1.2))
    w["llm.lm_head.weight"] = (TYPE_Q8_0, (H, V), q8_0_random(rng, V, H, lo, hi))
    for i in range(cfg["n_layers"]):
        p = f"llm.model.layers.{i}."
        w[p + "self_attn.q_proj.weight"] = (TYPE_Q8_0, (H, QD), q8_0_random(rng, QD, H, lo, hi))
        w[p + "self_attn.k_proj.weight"] = (TYPE_Q8_0, (H, KD), q8_0_random(rng, KD, H, lo, hi))
        w[p + "self_attn.v_proj.weight"] = (TYPE_Q8_0, (H, KD), q8_0_random(rng, KD, H, lo, hi))
        w[p + "self_attn.o_proj.weight"] = (TYPE_Q8_0, (QD, H), q8_0_random(rng, H, QD, lo, hi))
        w[p + "mlp.gate_proj.weight"] = (TYPE_Q8_0, (H, F), q8_0_random(rng, F, H, lo, hi))
        w[p + "mlp.up_proj.weight"] = (TYPE_Q8_0, (H, F), q8_0_random(rng, F, H, lo, hi))
        w[p + "mlp.down_proj.weight"] = (TYPE_Q8_0, (F, H), q8_0_random(rng, H, F, lo, hi))
        w[p + "self_attn.q_norm.weight"] = (TYPE_BF16, (D, 1), bf16(D, 0.8, 1.2))
        w[p + "self_attn.k_norm.weight"] = (TYPE_BF16, (D, 1), bf16(D, 0.8, 1.2))
        w[p + "input_layernorm.weight"] = (TYPE_BF16, (H, 1), bf16(H, 0.8, 1.2))
        w[p + "post_attention_layernorm.weight"] = (TYPE_BF16, (H, 1), bf16(H, 0.8, 1.2))
    return w


def decoder_desc(cfg: dict, **over) -> dict:
    """Keyword arguments for fa_dec.Decoder from a config dict."""
    d = dict(n_layers=cfg["n_layers"], hidden=cfg["hidden"], ffn=cfg["ffn"], vocab=cfg["vocab"],
             rope_base=cfg.get("rope_base", 1e6), rms_eps=cfg.get("eps", 1e-5))
    d.update(over)
    return d


def audio_embeds(rng: np.random.Generator, n: int, hidden: int, scale: float = 1.0) -> np.ndarray:
    """Stand-in for adaptor output frames [n][hidden] (the encoder is out of scope)."""
    return (rng.standard_normal((n, hidden), dtype=np.float32) * scale).astype(np.float32)


# ------------------------------------------------------------ encoder --
ENCODER = dict(input_dim=560, output_size=512, attention_heads=4, linear_units=2048, num_blocks=50, tp_blocks=20,
               kernel_size=11, sanm_shift=0)
ADAPTOR = dict(input_dim=512, hidden_dim=2048, output_dim=1024, num_blocks=2, attention_heads=8, ffn_dim=256)


def make_encoder_weights(ecfg: dict = ENCODER, acfg: dict = ADAPTOR, seed: int = 0,
                         d_range=(0.0002, 0.001)) -> Dict[str, Tuple[int, Tuple[int, int], np.ndarray]]:
    """Random-init SANM encoder + adaptor weights in the reference's GGUF layout
    (model/loader.cpp:21-80,135-200) and types (tools/hf_convert_ggml_q8.py:308-323):
    2-D weights whose input dimension is a multiple of 32 are Q8_0, the others
    (encoder0's 560-wide projections) and the FSMN taps are F16, norms and biases F32.
    The default scales give weights of standard deviation ~1/sqrt(fan-in)."""
    rng = np.random.default_rng(seed)
    lo, hi = d_range
    w = {}

    def mat(name, n, k):
        if k % 32 == 0:
            w[name] = (TYPE_Q8_0, (k, n), q8_0_random(rng, n, k, lo, hi))
        else:
            x = (rng.standard_normal((n, k)) / np.sqrt(k)).astype(np.float16)
            w[name] = (TYPE_F16, (k, n), x.view(np.uint16))

    def vec(name, n, mean, std):
        w[name] = (TYPE_F32, (n, 1), (mean + std * rng.standard_normal(n)).astype(np.float32))

    def layer(p, d_in, d):
        vec(p + ".norm1.weight", d_in, 1.0, 0.1)
        vec(p + ".norm1.bias", d_in, 0.0, 0.1)
        for nm in ("linear_q", "linear_k", "linear_v"):
            mat(p + f".self_attn.{nm}.weight", d, d_in)
            vec(p + f".self_attn.{nm}.bias", d, 0.0, 0.05)
        mat(p + ".self_attn.linear_out.weight", d, d)
        vec(p + ".self_attn.linear_out.bias", d, 0.0, 0.05)
        taps = (rng.standard_normal((d, ecfg["kernel_size"])) * 0.1).astype(np.float16)
        w[p + ".self_attn.fsmn_block.weight"] = (TYPE_F16, (ecfg["kernel_size"], d), taps.view(np.uint16))
        vec(p + ".norm2.weight", d, 1.0, 0.1)
        vec(p + ".norm2.bias", d, 0.0, 0.1)
        mat(p + ".feed_forward.w_1.weight", ecfg["linear_units"], d)
        vec(p + ".feed_forward.w_1.bias", ecfg["linear_units"], 0.0, 0.05)
        mat(p + ".feed_forward.w_2.weight", d, ecfg["linear_units"])
        vec(p + ".feed_forward.w_2.bias", d, 0.0, 0.05)

    d = ecfg["output_size"]
    layer("audio_encoder.encoders0.0", ecfg["input_dim"], d)
    for i in range(ecfg["num_blocks"] - 1):
        layer(f"audio_encoder.encoders.{i}", d, d)
    for nm in ("after_norm", "tp_norm"):
        vec(f"audio_encoder.{nm}.weight", d, 1.0, 0.1)
        vec(f"audio_encoder.{nm}.bias", d, 0.0, 0.1)
    for i in range(ecfg["tp_blocks"]):
        layer(f"audio_encoder.tp_encoders.{i}", d, d)
    D = acfg["output_dim"]
    mat("audio_adaptor.linear1.weight", acfg["hidden_dim"], acfg["input_dim"])
    vec("audio_adaptor.linear1.bias", acfg["hidden_dim"], 0.0, 0.05)
    mat("audio_adaptor.linear2.weight", D, acfg["hidden_dim"])
    vec("audio_adaptor.linear2.bias", D, 0.0, 0.05)
    for i in range(acfg["num_blocks"]):
        p = f"audio_adaptor.blocks.{i}"
        vec(p + ".norm1.weight", D, 1.0, 0.1)
        vec(p + ".norm1.bias", D, 0.0, 0.1)
        for nm in ("linear_q", "linear_k", "linear_v", "linear_out"):
            mat(p + f".self_attn.{nm}.weight", D, D)
            vec(p + f".self_attn.{nm}.bias", D, 0.0, 0.05)
        vec(p + ".norm2.weight", D, 1.0, 0.1)
        vec(p + ".norm2.bias", D, 0.0, 0.1)
        mat(p + ".feed_forward.w_1.weight", acfg["ffn_dim"], D)
        vec(p + ".feed_forward.w_1.bias", acfg["ffn_dim"], 0.0, 0.05)
        mat(p + ".feed_forward.w_2.weight", D, acfg["ffn_dim"])
        vec(p + ".feed_forward.w_2.bias", D, 0.0, 0.05)
    return w


def lfr_features(rng: np.random.Generator, T: int, dim: int = 560) -> np.ndarray:
    """Stand-in for LFR-stacked log-mel frames [T][560] (the front end is out of scope)."""
    return (rng.standard_normal((T, dim)) * 2.0 - 4.0).astype(np.float32)
