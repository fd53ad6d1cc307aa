"""Generate the golden fixtures that pin the CPU oracle.

Run in the build container (needs the reference tree and transformers):
    python tests/golden/make_golden.py <path of the FunASR-GGML source tree>

1. q8_0_codec.npz — inputs and the bytes produced by the reference converter's own
   Q8_0 quantiser, FunAsr.quantize_q8_0 in tools/hf_convert_ggml_q8.py:354-381,
   imported from the reference tree and called unchanged.
2. qwen3_small.npz — logits of a 2-layer random-init Qwen3 decoder (16 query / 8 KV
   heads x 128, rms eps 1e-5 as compute/llm_ops_gpu.cpp:50, RoPE base 1e6) computed by
   the transformers Qwen3 implementation (the model family the reference converts from)
   in float64, with weights that are exactly the dequantised Q8_0 / BF16 values of
   fa_synth.make_weights(seed). The fixture stores the seed, a checksum of the weights
   and the inputs; tests regenerate the weights and check the checksum first.
3. ops.npz — RMSNorm (eps 1e-5) and NEOX RoPE outputs from the same implementation.
"""
from __future__ import annotations

import hashlib
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "funasr-ggml_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import fa_synth  # noqa: E402
import oracle  # noqa: E402

GOLDEN_CFG = dict(fa_synth.QWEN3_06B, n_layers=2, hidden=128, ffn=256, vocab=512)
GOLDEN_SEED = 1234


def weights_checksum(w) -> str:
    h = hashlib.sha256()
    for name in sorted(w):
        t, ne, arr = w[name]
        h.update(name.encode())
        h.update(np.ascontiguousarray(arr).tobytes())
    return h.hexdigest()


def q8_codec(ref_root: str):
    import torch
    spec = importlib.util.spec_from_file_location("ref_q8", os.path.join(ref_root, "tools", "hf_convert_ggml_q8.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    rng = np.random.default_rng(7)
    rows = [
        rng.standard_normal(32 * 64).astype(np.float32),
        (rng.standard_normal(32 * 64) * 1e-3).astype(np.float32),
        (rng.standard_normal(32 * 64) * 100).astype(np.float32),
        np.zeros(32 * 64, np.float32),                                  # d == 0 -> 1e-8 rule
        np.tile(np.array([127.0, -127.0, 63.5, -63.5, 0.5, -0.5, 1.5, 2.5] * 4, np.float32), 64),  # ties
        rng.uniform(-1, 1, 32 * 64).astype(np.float32),
    ]
    x = np.stack(rows)
    out = mod.FunAsr.quantize_q8_0(None, torch.from_numpy(x.copy()))
    out = np.asarray(out, np.uint8).reshape(x.shape[0], -1)
    np.savez_compressed(os.path.join(HERE, "q8_0_codec.npz"), x=x, q8=out)
    print("q8_0_codec.npz", x.shape, out.shape)


def hf_small():
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM

    cfg = GOLDEN_CFG
    w = fa_synth.make_weights(cfg, seed=GOLDEN_SEED)
    H, V, L = cfg["hidden"], cfg["vocab"], cfg["n_layers"]
    hcfg = Qwen3Config(hidden_size=H, intermediate_size=cfg["ffn"], num_hidden_layers=L,
                       num_attention_heads=16, num_key_value_heads=8, head_dim=128, vocab_size=V,
                       rms_norm_eps=1e-5, rope_theta=1e6, max_position_embeddings=4096,
                       tie_word_embeddings=False, attention_bias=False, hidden_act="silu")
    hcfg._attn_implementation = "eager"
    model = Qwen3ForCausalLM(hcfg).to(torch.float64).eval()

    def dq(name, n, k):
        t, ne, arr = w[name]
        return torch.from_numpy(oracle.q8_0_dequant(arr, k).reshape(n, k).astype(np.float64))

    def bf(name):
        t, ne, arr = w[name]
        return torch.from_numpy(oracle.bf16_bits_to_f32(arr).astype(np.float64).reshape(-1))

    sd = {}
    t, ne, emb = w["llm.model.embed_tokens.weight"]
    emb_f = oracle.bf16_bits_to_f32(emb).reshape(V, H).astype(np.float64)
    sd["model.embed_tokens.weight"] = torch.from_numpy(emb_f)
    sd["model.norm.weight"] = bf("llm.model.norm.weight")
    sd["lm_head.weight"] = dq("llm.lm_head.weight", V, H)
    for i in range(L):
        p, q = f"llm.model.layers.{i}.", f"model.layers.{i}."
        sd[q + "self_attn.q_proj.weight"] = dq(p + "self_attn.q_proj.weight", 2048, H)
        sd[q + "self_attn.k_proj.weight"] = dq(p + "self_attn.k_proj.weight", 1024, H)
        sd[q + "self_attn.v_proj.weight"] = dq(p + "self_attn.v_proj.weight", 1024, H)
        sd[q + "self_attn.o_proj.weight"] = dq(p + "self_attn.o_proj.weight", H, 2048)
        sd[q + "mlp.gate_proj.weight"] = dq(p + "mlp.gate_proj.weight", cfg["ffn"], H)
        sd[q + "mlp.up_proj.weight"] = dq(p + "mlp.up_proj.weight", cfg["ffn"], H)
        sd[q + "mlp.down_proj.weight"] = dq(p + "mlp.down_proj.weight", H, cfg["ffn"])
        sd[q + "self_attn.q_norm.weight"] = bf(p + "self_attn.q_norm.weight")
        sd[q + "self_attn.k_norm.weight"] = bf(p + "self_attn.k_norm.weight")
        sd[q + "input_layernorm.weight"] = bf(p + "input_layernorm.weight")
        sd[q + "post_attention_layernorm.weight"] = bf(p + "post_attention_layernorm.weight")
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected and all("rotary" in m for m in missing), (missing, unexpected)

    # prompt: 4 token ids, 8 audio-like embedding rows, 4 token ids, then 8 teacher-forced tokens
    rng = np.random.default_rng(99)
    pre = rng.integers(0, V, 4)
    audio = rng.standard_normal((8, H)).astype(np.float32)
    suf = rng.integers(0, V, 4)
    dec = rng.integers(0, V, 8)
    rows = [emb_f[t] for t in pre] + [a.astype(np.float64) for a in audio] + [emb_f[t] for t in suf] + \
           [emb_f[t] for t in dec]
    x = torch.from_numpy(np.stack(rows))[None]
    with torch.no_grad():
        logits = model(inputs_embeds=x).logits[0].numpy()
    np.savez_compressed(os.path.join(HERE, "qwen3_small.npz"), seed=GOLDEN_SEED,
                        cfg=np.array([cfg["n_layers"], H, cfg["ffn"], V]), checksum=weights_checksum(w),
                        pre=pre.astype(np.int32), audio=audio, suf=suf.astype(np.int32), dec=dec.astype(np.int32),
                        logits=logits.astype(np.float32))
    print("qwen3_small.npz", logits.shape, "checksum", weights_checksum(w)[:16])

    # single ops from the same implementation
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm, apply_rotary_pos_emb
    rs = np.random.default_rng(5)
    xn = rs.standard_normal((6, 128)).astype(np.float32) * 3
    wn = rs.uniform(0.5, 1.5, 128).astype(np.float32)
    norm = Qwen3RMSNorm(128, eps=1e-5).to(torch.float64)
    norm.weight.data = torch.from_numpy(wn.astype(np.float64))
    with torch.no_grad():
        yn = norm(torch.from_numpy(xn.astype(np.float64))).numpy()
    pos = np.array([0, 1, 15, 16, 2047, 40959], np.int64)
    qv = rs.standard_normal((1, 1, len(pos), 128))
    kv = rs.standard_normal((1, 1, len(pos), 128))
    inv = 1.0 / (1e6 ** (np.arange(0, 128, 2, dtype=np.float64) / 128))
    fr = pos[:, None].astype(np.float64) * inv[None]
    embp = np.concatenate([fr, fr], -1)
    cos, sin = torch.from_numpy(np.cos(embp))[None], torch.from_numpy(np.sin(embp))[None]
    qr, kr = apply_rotary_pos_emb(torch.from_numpy(qv), torch.from_numpy(kv), cos, sin)
    np.savez_compressed(os.path.join(HERE, "ops.npz"), xn=xn, wn=wn, yn=yn, pos=pos.astype(np.int32),
                        qv=qv[0, 0], qr=qr.numpy()[0, 0])
    print("ops.npz")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path of the FunASR-GGML source tree>")
    ref = sys.argv[1]
    q8_codec(ref)
    hf_small()
