"""The one-row decode step as one persistent kernel (k_row_step.cu) against the launch-per-op
step: same logits bits, same ids, same K/V page bytes, over contexts that take one and
several attention splits, with token and embedding inputs; and its bounded waits (a CTA
whose values never arrive makes the step fail with FA_ERR_TIMEOUT, and the context keeps
working). The step's agreement with the oracle is checked at full Qwen3-0.6B geometry by
test_gpu_decoder.test_qwen3_06b_greedy_decode_batch1, whose batch-1 steps run on it."""
import numpy as np
import pytest

import fa_dec
import fa_synth

pytestmark = pytest.mark.gpu

# the smallest shapes the kernel takes: hidden and ffn multiples of 512
CFG = fa_synth.small_config(n_layers=3, hidden=512, ffn=1024, vocab=4096)
MAX_CTX = 2048


@pytest.fixture(scope="module")
def w():
    return fa_synth.make_weights(CFG, seed=21)


def _decoder(w, row_step):
    dec = fa_dec.Decoder(0, **fa_synth.decoder_desc(CFG, max_ctx=MAX_CTX, n_pages=128, max_seqs=4, max_rows=512))
    dec.load_weights(w)
    dec.set_row_step(row_step)
    return dec


def _run(w, row_step, prompt_len, n_steps, seed):
    """prefill prompt_len token ids, then n_steps decode steps with logits, then 6 steps of
    generate: (logits per step, ids, generated ids, K/V bytes of every layer's pages,
    launches of the last decode step)."""
    rng = np.random.default_rng(seed)
    dec = _decoder(w, row_step)
    s = dec.seq_open(MAX_CTX)
    toks = rng.integers(0, CFG["vocab"], prompt_len)
    nxt, _ = dec.forward([s] * prompt_len, tokens=toks)
    tok = int(nxt[-1])
    lgs, ids = [], []
    for _ in range(n_steps):
        g, lg = dec.decode_step([s], [tok], want_logits=True)
        lgs.append(lg[0].copy())
        tok = int(g[0])
        ids.append(tok)
    launches = dec.step_launches()
    gen, _ = dec.generate([s], [tok], 6)
    pages = dec.block_table(s)
    kv = [dec.kv_read_pages(l, pages) for l in range(CFG["n_layers"])]
    dec.close()
    return np.stack(lgs), np.array(ids), np.asarray(gen).ravel(), kv, launches


@pytest.mark.parametrize("prompt_len,n_steps", [(40, 30), (292, 12)])
def test_row_step_gives_the_launch_path_bits(torch_cuda, w, prompt_len, n_steps):
    """40 + 30: one attention split (pages 3 -> 5, the token's page changing under the
    patch); 292 + 12: 19-20 pages in 5 splits of 4, merged by the split that ends last."""
    lg_a, ids_a, gen_a, kv_a, n_a = _run(w, True, prompt_len, n_steps, seed=prompt_len)
    lg_b, ids_b, gen_b, kv_b, n_b = _run(w, False, prompt_len, n_steps, seed=prompt_len)
    assert n_a == 1 and n_b > 3 * CFG["n_layers"], (n_a, n_b)
    assert np.array_equal(lg_a.view(np.uint32), lg_b.view(np.uint32)), np.abs(lg_a - lg_b).max()
    assert np.array_equal(ids_a, ids_b) and np.array_equal(gen_a, gen_b)
    for l in range(CFG["n_layers"]):
        assert np.array_equal(kv_a[l], kv_b[l]), f"layer {l} K/V pages differ"


def test_row_step_embedding_input(torch_cuda, w):
    """A row given as an embedding (the audio-frame rows of a prompt) enters layer 0 from x."""
    toks = np.random.default_rng(3).integers(0, CFG["vocab"], 20)
    e = np.random.default_rng(4).standard_normal((1, CFG["hidden"])).astype(np.float32)
    out = []
    for row_step in (True, False):
        dec = _decoder(w, row_step)
        s = dec.seq_open(MAX_CTX)
        dec.forward([s] * 20, tokens=toks)
        nxt, lg = dec.forward([s], embeds=e, want_logits=True)
        if row_step:
            assert dec.step_launches() == 1
        out.append((nxt.copy(), lg.copy()))
        dec.close()
    assert np.array_equal(out[0][0], out[1][0])
    assert np.array_equal(out[0][1].view(np.uint32), out[1][1].view(np.uint32))


def test_row_step_barrier_timeout_is_reported_and_recovers(torch_cuda, w):
    """CTA 5 leaves at once: the CTAs waiting for its rows give up after 50 ms, all leave,
    the step fails with FA_ERR_TIMEOUT and rolls back; the same step then runs normally and
    gives the launch path's bits."""
    rng = np.random.default_rng(8)
    toks = rng.integers(0, CFG["vocab"], 33)
    ref = _decoder(w, False)
    s = ref.seq_open(MAX_CTX)
    nxt, _ = ref.forward([s] * 33, tokens=toks)
    want_ids, want_lg = ref.decode_step([s], [int(nxt[-1])], want_logits=True)
    ref.close()

    dec = _decoder(w, True)
    s = dec.seq_open(MAX_CTX)
    nxt, _ = dec.forward([s] * 33, tokens=toks)
    dec.set_row_step_fault(5, 50000)
    with pytest.raises(fa_dec.FaError) as ei:
        dec.decode_step([s], [int(nxt[-1])])
    assert ei.value.code == -8, ei.value          # FA_ERR_TIMEOUT
    assert dec.seq_length(s) == 33
    dec.set_row_step_fault(-1)
    got_ids, got_lg = dec.decode_step([s], [int(nxt[-1])], want_logits=True)
    assert dec.step_launches() == 1
    assert np.array_equal(got_ids, want_ids)
    assert np.array_equal(got_lg.view(np.uint32), want_lg.view(np.uint32))
    dec.close()
