"""The C++ host API (include/funasr_b200.hpp) driven by a C++ program written like the
reference's own GPU tests (tests/cpp/test_decoder_api.cpp): model loaded from a GGUF
file, warmup, prefill, greedy loop with GPURunner::argmax, cache views, a second stream
through BatchDecoder. Its outputs are checked against the oracle."""
import os
import subprocess

import numpy as np
import pytest

import fa_synth
import oracle
from gguf_fixture import write_model_gguf
from helpers import assert_close

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIBDIR = os.path.join(ROOT, "funasr-ggml_b200")
CFG = fa_synth.small_config(n_layers=2, hidden=256, ffn=512, vocab=2048)


@pytest.fixture(scope="module")
def program(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("cpp") / "test_decoder_api")
    cmd = ["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
           os.path.join(HERE, "cpp", "test_decoder_api.cpp"), "-L", LIBDIR, "-lfunasr_dec",
           f"-Wl,-rpath,{LIBDIR}", "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_host_f16_cast_matches_ieee(tmp_path):
    """KVCache::commit casts the reference's f32 K/V with funasr_b200::f32_to_f16_bits:
    round to nearest even, gradual underflow, overflow to infinity, NaN kept."""
    exe = str(tmp_path / "f16cast")
    r = subprocess.run(["g++", "-std=c++17", "-O2", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                        os.path.join(HERE, "cpp", "test_f16_cast.cpp"), "-o", exe], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    rng = np.random.default_rng(3)
    edge = np.array([0.0, -0.0, 1.0, -1.0, 65504.0, 65519.99, 65520.0, 1e9, -1e9, np.inf, -np.inf,
                     6.1035156e-05, 6.0975552e-05, 5.9604645e-08, 2.9802322e-08, 2.9802326e-08, 1e-12,
                     1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11, 2049.0, 2051.0, 0.1, 1 / 3], np.float32)
    ticks = (np.arange(1, 1 << 14, dtype=np.uint32) << 13).view(np.float32)   # exact ties and neighbours
    x = np.concatenate([edge, rng.standard_normal(200000).astype(np.float32) * 10,
                        rng.standard_normal(50000).astype(np.float32) * 1e-5, ticks, np.nextafter(ticks, 0)]
                       ).astype(np.float32)
    (tmp_path / "in.bin").write_bytes(x.tobytes())
    r = subprocess.run([exe, str(tmp_path / "in.bin"), str(tmp_path / "out.bin")], capture_output=True, timeout=60)
    assert r.returncode == 0
    got = np.frombuffer((tmp_path / "out.bin").read_bytes(), np.uint16)
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want), np.nonzero(got != want)[0][:10]
    nan = subprocess.run([exe, str(tmp_path / "nan.bin"), str(tmp_path / "nan_out.bin")], capture_output=True)
    assert nan.returncode == 2                                      # missing input file
    (tmp_path / "nan.bin").write_bytes(np.array([np.nan], np.float32).tobytes())
    subprocess.run([exe, str(tmp_path / "nan.bin"), str(tmp_path / "nan_out.bin")], check=True)
    h = int(np.frombuffer((tmp_path / "nan_out.bin").read_bytes(), np.uint16)[0])
    assert (h & 0x7c00) == 0x7c00 and (h & 0x3ff) != 0


def test_program_builds_and_reports_a_bad_model_path(program, tmp_path):
    r = subprocess.run([program, str(tmp_path / "absent.gguf"), "/dev/null", "1", "1", str(tmp_path / "o")],
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 2 and "cannot open" in r.stdout, r.stdout


@pytest.mark.gpu
def test_cpp_api_decode_matches_oracle(program, tmp_path, torch_cuda):
    w = fa_synth.make_weights(CFG, seed=21)
    model = str(tmp_path / "model.gguf")
    write_model_gguf(model, CFG, w, context_length=4096)
    n_prompt, n_new = 40, 16
    prompt = fa_synth.audio_embeds(np.random.default_rng(5), n_prompt, CFG["hidden"])
    prompt.tofile(str(tmp_path / "prompt.f32"))
    out = str(tmp_path / "out.bin")
    r = subprocess.run([program, model, str(tmp_path / "prompt.f32"), str(n_prompt), str(n_new), out],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr

    kvd = CFG["n_kv_heads"] * CFG["head_dim"]
    n_past = n_prompt + n_new
    raw = open(out, "rb").read()
    ids = np.frombuffer(raw, np.int32, n_new)
    off = 4 * n_new
    logits = np.frombuffer(raw, np.float32, CFG["vocab"], off)
    off += 4 * CFG["vocab"]
    k0 = np.frombuffer(raw, np.uint16, n_past * kvd, off).reshape(n_past, kvd)
    off += 2 * n_past * kvd
    v0 = np.frombuffer(raw, np.uint16, n_past * kvd, off).reshape(n_past, kvd)
    off += 2 * n_past * kvd
    ids2 = np.frombuffer(raw, np.int32, n_new, off)
    ids3 = np.frombuffer(raw, np.int32, n_new, off + 4 * n_new)

    od = oracle.OracleDecoder(CFG, w, n_pages=64, max_seqs=1, max_pages_per_seq=64, max_pos=4096,
                              mode=oracle.MODE_EXACT)
    od.seq_open(0)
    lg, nx = od.forward([0] * n_prompt, embeds=prompt)
    o_ids = []
    tok = int(nx[-1])
    for _ in range(n_new):
        o_ids.append(tok)
        lg, nx = od.forward([0], tokens=[tok])
        tok = int(nx[0])
    assert np.mean(ids == np.array(o_ids)) >= 0.99, (ids, o_ids)
    assert np.array_equal(ids2, ids), "BatchDecoder stream differs from GPURunner stream"
    assert np.array_equal(ids3, ids), "Scheduler stream differs from GPURunner stream"
    assert_close(logits, lg[0], what="last-step logits")
    # layer-0 cache in [pos][kv_dim] order from the oracle's pages
    pages = od.pool[0].reshape(-1, CFG["n_kv_heads"], 2, 16, CFG["head_dim"])
    bt = od.block_table[0]
    pos = np.arange(n_past)
    ref_k = pages[bt[pos // 16], :, 0, pos % 16].reshape(n_past, kvd)
    ref_v = pages[bt[pos // 16], :, 1, pos % 16].reshape(n_past, kvd)
    assert np.mean(k0 == ref_k) > 0.98 and np.mean(v0 == ref_v) > 0.98
