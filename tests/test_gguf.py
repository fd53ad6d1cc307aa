"""CPU tests of the GGUF model-file reader (fa_gguf_read_desc / fa_gguf_find_tensor)
against files written by gguf-py, an independent GGUF implementation."""
import os

import numpy as np
import pytest

import fa_dec
import fa_synth
from gguf_fixture import write_model_gguf

CFG = fa_synth.small_config(n_layers=2, hidden=256, ffn=512, vocab=2048)


@pytest.fixture(scope="module")
def model_file(tmp_path_factory):
    w = fa_synth.make_weights(CFG, seed=3)
    path = str(tmp_path_factory.mktemp("gguf") / "model.gguf")
    write_model_gguf(path, CFG, w, context_length=4096)
    return path, w


def test_geometry_from_funasr_keys(model_file):
    path, _ = model_file
    d = fa_dec.gguf_desc(path, max_seqs=3)
    got = (d.n_layers, d.hidden, d.ffn, d.vocab, d.n_heads, d.n_kv_heads, d.head_dim, d.rope_base, d.max_ctx)
    assert got == (2, 256, 512, 2048, 16, 8, 128, 1e6, 4096)
    assert d.max_seqs == 3          # runtime sizes are left to the caller


def test_every_decoder_tensor_located_byte_exact(model_file):
    path, w = model_file
    raw = np.fromfile(path, np.uint8)
    for name, (t, ne, arr) in w.items():
        typ, (ne0, rows), off, nb = fa_dec.gguf_find_tensor(path, name)
        assert typ == t and ne0 == ne[0] and rows == (ne[1] if len(ne) > 1 else 1)
        a = np.ascontiguousarray(arr).view(np.uint8).ravel()
        assert nb == a.size and np.array_equal(raw[off:off + nb], a), name


def test_missing_keys_tensors_and_bad_files_are_errors(model_file, tmp_path):
    path, _ = model_file
    with pytest.raises(fa_dec.FaError) as e:
        fa_dec.gguf_find_tensor(path, "llm.model.layers.9.mlp.up_proj.weight")
    assert e.value.code == fa_dec.FA_ERR_WEIGHTS
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUF" + b"\x07\x00\x00\x00" + bytes(64))            # version 7
    with pytest.raises(fa_dec.FaError, match="version"):
        fa_dec.gguf_desc(str(bad))
    trunc = tmp_path / "trunc.gguf"
    trunc.write_bytes(open(path, "rb").read()[:4000])                      # tensor data cut off
    with pytest.raises(fa_dec.FaError):
        fa_dec.gguf_desc(str(trunc))
    nokeys = tmp_path / "nokeys.gguf"
    import gguf
    wr = gguf.GGUFWriter(str(nokeys), arch="FunAsr")
    wr.add_uint32("FunAsr.block_count", 2)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    with pytest.raises(fa_dec.FaError, match="embedding_length"):
        fa_dec.gguf_desc(str(nokeys))
    with pytest.raises(fa_dec.FaError, match="cannot open"):
        fa_dec.gguf_desc(os.path.join(str(tmp_path), "absent.gguf"))
