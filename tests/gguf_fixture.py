"""Writes decoder weights as a GGUF model file with gguf-py (the GGUF library that
ships with llama.cpp / ggml, installed in this environment), in the layout of the
reference's converter (tools/hf_convert_ggml_q8.py): FunAsr.* hyper-parameter keys,
llm.* tensor names, Q8_0 projections, BF16 embedding and norms. Test helper only."""
from __future__ import annotations

import numpy as np

import fa_synth


def write_model_gguf(path: str, cfg: dict, w: dict, context_length: int = 40960) -> None:
    import gguf
    wr = gguf.GGUFWriter(path, arch="FunAsr")
    wr.add_uint32("FunAsr.block_count", cfg["n_layers"])
    wr.add_uint32("FunAsr.embedding_length", cfg["hidden"])
    wr.add_uint32("FunAsr.context_length", context_length)
    wr.add_uint32("FunAsr.feed_forward_length", cfg["ffn"])
    wr.add_uint32("FunAsr.attention.head_count", cfg["n_heads"])
    wr.add_uint32("FunAsr.attention.head_count_kv", cfg["n_kv_heads"])
    wr.add_float32("FunAsr.rope.freq_base", float(cfg.get("rope_base", 1e6)))
    wr.add_uint32("FunAsr.attention.key_length", cfg["head_dim"])
    wr.add_uint32("FunAsr.attention.value_length", cfg["head_dim"])
    wr.add_uint32("tokenizer.ggml.eos_token_id", 151645)
    # a tensor outside the decoder, as a full model file has (the encoder's), to be skipped
    wr.add_tensor("encoder.embed.weight", np.ones((4, 8), np.float32))
    for name, (t, ne, arr) in w.items():
        ne1 = int(ne[1]) if len(ne) > 1 else 1
        if t == fa_synth.TYPE_Q8_0:
            wr.add_tensor(name, np.ascontiguousarray(arr, np.uint8).reshape(ne1, -1),
                          raw_dtype=gguf.GGMLQuantizationType.Q8_0)
        elif t == fa_synth.TYPE_BF16:
            shape = (int(ne[0]),) if ne1 == 1 else (ne1, int(ne[0]))
            wr.add_tensor(name, np.ascontiguousarray(arr, np.uint16).reshape(shape).view(np.uint8)
                          .reshape(*shape[:-1], shape[-1] * 2), raw_dtype=gguf.GGMLQuantizationType.BF16)
        else:
            wr.add_tensor(name, np.ascontiguousarray(arr).reshape(ne1, -1) if ne1 > 1 else np.ascontiguousarray(arr))
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
