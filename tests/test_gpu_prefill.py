"""GPU parity of kernel (2b), the tensor-core prefill attention, against the oracle.

Tiles of up to 64 consecutive rows of one sequence attend causally to the paged
cache. The oracle computes each row's attention exactly (fp32 softmax, f16 pages);
the kernel's products are exact (f16 pairs for Q and P, f16 K/V) and accumulate in
fp32, so the bound is the fp32 one of the decode kernel: 1e-4 max-abs, 1e-5 rel-RMS.
"""
import math

import numpy as np
import pytest

import fa_dec
import oracle
from helpers import assert_close, dev

pytestmark = pytest.mark.gpu

PAGE_ELEMS = 8 * 2 * 16 * 128


def _case(torch, rng, chunks, n_pages=2048, q_scale=0.3, bad_page=False):
    """chunks: list of (first position, rows) of one sequence each."""
    rows_pos, rows_slot, tiles = [], [], []
    for s, (p0, n) in enumerate(chunks):
        for off in range(0, n, 64):
            k = min(64, n - off)
            tiles.append((len(rows_pos), k))
            rows_pos += list(range(p0 + off, p0 + off + k))
            rows_slot += [s] * k
    M = len(rows_pos)
    pos = np.array(rows_pos, np.int32)
    slot = np.array(rows_slot, np.int32)
    bt_stride = int(math.ceil((pos.max() + 1) / 16)) + 1
    bt = np.stack([rng.choice(n_pages, bt_stride, replace=False) for _ in chunks]).astype(np.int32)
    if bad_page:
        bt[0, 0] = n_pages + 5
    pool = oracle.f32_to_f16_bits(rng.standard_normal((n_pages, PAGE_ELEMS)).astype(np.float32))
    q = (rng.standard_normal((M, 16, 128)) * q_scale).astype(np.float32)
    d = [dev(torch, a) for a in (q, pos, slot, bt, np.ascontiguousarray(pool).view(np.int16),
                                 np.array(tiles, np.int32))]
    out32 = torch.zeros((M, 2048), dtype=torch.float32, device="cuda")
    out16 = torch.zeros((M, 2048), dtype=torch.int16, device="cuda")
    out_lo = torch.zeros((M, 2048), dtype=torch.int16, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    fa_dec.op_prefill_attention(d[0].data_ptr(), M, d[1].data_ptr(), d[2].data_ptr(), d[3].data_ptr(), bt_stride,
                                n_pages, d[4].data_ptr(), d[5].data_ptr(), len(tiles), out16=out16.data_ptr(),
                                out16_lo=out_lo.data_ptr(), out32=out32.data_ptr(), err=err.data_ptr())
    torch.cuda.synchronize()
    o32 = out32.cpu().numpy()
    hi = oracle.f16_bits_to_f32(out16.cpu().numpy().view(np.uint16))
    lo = oracle.f16_bits_to_f32(out_lo.cpu().numpy().view(np.uint16))
    ref = None if bad_page else oracle.paged_attention(q, slot, pos + 1, bt, pool)
    return o32, hi, lo, ref, int(err.item())


@pytest.mark.parametrize("chunks,q_scale", [
    ([(0, 64)], 0.3),                                   # one full tile from position 0
    ([(0, 17), (100, 64), (1000, 41), (2047, 1)], 0.3), # ragged tiles, mid-sequence chunks, one row
    ([(4000, 130)], 0.3),                               # long context, three tiles of one chunk
    ([(63, 2), (64, 64), (127, 3)], 0.3),               # block edges of the 64-key blocks
    ([(0, 64), (500, 64)], 2.0),                        # sharp softmax: many running-max rescales
])
def test_prefill_attention_matches_oracle(torch_cuda, chunks, q_scale):
    rng = np.random.default_rng(sum(p + n for p, n in chunks))
    o32, hi, lo, ref, err = _case(torch_cuda, rng, chunks, q_scale=q_scale)
    assert err == 0
    assert_close(o32, ref, max_abs_tol=1e-4, rel_rms_tol=1e-5, what="prefill attention f32")
    assert_close(hi + lo, ref, max_abs_tol=1e-4, rel_rms_tol=1e-5, what="prefill attention f16 pair")


def test_prefill_attention_flags_bad_page(torch_cuda):
    rng = np.random.default_rng(9)
    _, _, _, _, err = _case(torch_cuda, rng, [(10, 20)], bad_page=True)
    assert err & 2


def test_decoder_forward_with_prefill_tiles_matches_oracle(torch_cuda):
    """One fa_forward mixing a 150-row chunk (three tiles), a 20-row chunk (one tile)
    and single decode rows (decode kernel), then decode steps: logits against the
    oracle within 2e-2 / 1e-3, greedy ids >= 99 %, identical block tables."""
    import fa_synth
    cfg = fa_synth.small_config(n_layers=2, hidden=256, ffn=512, vocab=2048)
    w = fa_synth.make_weights(cfg, seed=31)
    dec = fa_dec.Decoder(0, **fa_synth.decoder_desc(cfg, max_ctx=1024, n_pages=256, max_seqs=8, max_rows=256))
    dec.load_weights(w)
    od = oracle.OracleDecoder(cfg, w, n_pages=256, max_seqs=8, max_pages_per_seq=64, max_pos=1024,
                              mode=oracle.MODE_EXACT)
    rng = np.random.default_rng(12)
    sids = [dec.seq_open(1024) for _ in range(3)]
    for s in sids:
        od.seq_open(s)
    # sequence 2 already holds 3 tokens
    pre = fa_synth.audio_embeds(rng, 3, cfg["hidden"])
    dec.forward([2] * 3, embeds=pre)
    od.forward([2] * 3, embeds=pre)
    rows = [0] * 150 + [1] * 20 + [2]
    emb = fa_synth.audio_embeds(rng, len(rows), cfg["hidden"])
    g_next, g_lg = dec.forward(rows, embeds=emb, want_logits=True)
    o_lg, o_next = od.forward(rows, embeds=emb)
    assert_close(g_lg, o_lg, what="mixed prefill logits")
    agree = [np.mean(g_next == o_next)]
    last = [149, 169, 170]
    toks = g_next[last]
    for _ in range(6):
        g_next, g_lg = dec.decode_step(sids, toks, want_logits=True)
        o_lg, o_next = od.forward(sids, tokens=toks)
        assert_close(g_lg, o_lg, what="decode after prefill")
        agree.append(np.mean(g_next == o_next))
        toks = g_next
    assert np.mean(agree) >= 0.99
    for s in sids:
        bt = dec.block_table(s)
        assert np.array_equal(bt, od.block_table[s, :len(bt)])
    dec.close()


def test_forward_rows_outputs_equal_full_forward(torch_cuda):
    """fa_forward_rows runs lm_head on the listed rows only; their next ids and logits
    equal those of a full fa_forward of the same rows (rows are independent in every
    kernel after attention), and n_out = 0 still appends every row."""
    import fa_synth
    cfg = fa_synth.small_config(n_layers=2, hidden=256, ffn=512, vocab=2048)
    w = fa_synth.make_weights(cfg, seed=41)
    dec = fa_dec.Decoder(0, **fa_synth.decoder_desc(cfg, max_ctx=512, n_pages=128, max_seqs=8, max_rows=128))
    dec.load_weights(w)
    rng = np.random.default_rng(3)
    a, b, c, d = (dec.seq_open(512) for _ in range(4))
    rows_a = [a] * 40 + [c] * 3
    rows_b = [b] * 40 + [d] * 3
    emb = fa_synth.audio_embeds(rng, len(rows_a), cfg["hidden"])
    n_full, lg_full = dec.forward(rows_a, embeds=emb, want_logits=True)
    sel = [39, 42, 0]
    n_sel, lg_sel = dec.forward_rows(rows_b, sel, embeds=emb, want_logits=True)
    assert np.array_equal(n_sel, n_full[sel])
    assert np.array_equal(lg_sel, lg_full[sel])
    n0, _ = dec.forward_rows([a] * 5, [], embeds=emb[:5])
    assert len(n0) == 0 and dec.seq_length(a) == 45
    dec.close()
