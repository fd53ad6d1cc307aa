"""The continuous-batching scheduler: its policy on CPU against a fake backend (C++
unit test of funasr-ggml_b200/csrc/sched_core.hpp), and on the GPU through the C ABI,
where every stream must produce the tokens it produces decoded alone."""
import os
import subprocess

import numpy as np
import pytest

import fa_dec
import fa_synth

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def test_sched_core_policy_against_fake_backend(tmp_path):
    exe = str(tmp_path / "test_sched_core")
    r = subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror",
                        "-I", os.path.join(ROOT, "funasr-ggml_b200", "csrc"),
                        os.path.join(HERE, "cpp", "test_sched_core.cpp"), "-o", exe], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout


def test_sched_rejects_bad_arguments_without_gpu():
    with pytest.raises(fa_dec.FaError):
        fa_dec.Scheduler(None)


@pytest.mark.gpu
def test_sched_streams_match_streams_decoded_alone(torch_cuda):
    cfg = fa_synth.small_config(n_layers=2, hidden=256, ffn=512, vocab=2048)
    w = fa_synth.make_weights(cfg, seed=51)
    rng = np.random.default_rng(8)
    streams = []
    for tag in range(12):
        n = int(rng.integers(5, 120))
        if tag % 3 == 0:
            streams.append((tag, None, fa_synth.audio_embeds(rng, n, cfg["hidden"]), int(rng.integers(1, 40))))
        else:
            streams.append((tag, rng.integers(0, cfg["vocab"], n).astype(np.int32), None, int(rng.integers(1, 40))))
    desc = fa_synth.decoder_desc(cfg, max_ctx=512, n_pages=80, max_seqs=6, max_rows=96)

    # each stream alone: prefill then greedy steps
    dec = fa_dec.Decoder(0, **desc)
    dec.load_weights(w)
    ref = {}
    for tag, ids, emb, max_new in streams:
        s = dec.seq_open(512)
        e = emb if emb is not None else fa_synth_embed(w, cfg, ids)
        first, _ = dec.prefill(s, e)
        toks = [int(first)]
        while len(toks) < max_new:
            n2, _ = dec.decode_step([s], [toks[-1]])
            toks.append(int(n2[0]))
        ref[tag] = toks
        dec.seq_close(s)
    dec.close()

    dec = fa_dec.Decoder(0, **desc)
    dec.load_weights(w)
    sch = fa_dec.Scheduler(dec, max_batch_rows=96, prefill_chunk=40, max_running=6, eos_id=-1)
    for tag, ids, emb, max_new in streams:
        sch.submit(tag, max_new, ids=ids, embeds=emb)
    got = {tag: [] for tag, *_ in streams}
    done = set()
    steps = 0
    while not sch.idle():
        for tag, tok, fin in sch.step():
            assert tag not in done and tok >= 0
            got[tag].append(tok)
            if fin:
                done.add(tag)
        steps += 1
        assert steps < 5000
    st = sch.stats()
    assert st["finished"] == len(streams) and st["running"] == 0
    assert dec.pool_info()[1] == dec.pool_info()[0]          # every page back in the pool
    total = sum(len(v) for v in ref.values())
    agree = sum(int(a == b) for t in ref for a, b in zip(ref[t], got[t]))
    assert all(len(got[t]) == len(ref[t]) for t in ref)
    assert agree / total >= 0.99, (agree, total)
    sch.close()
    dec.close()


def fa_synth_embed(w, cfg, ids):
    """Host embedding lookup (BF16 table -> f32), as the reference's prompt builder."""
    table = w["llm.model.embed_tokens.weight"][2].reshape(cfg["vocab"], cfg["hidden"])
    return (table[ids].astype(np.uint32) << 16).view(np.float32)
