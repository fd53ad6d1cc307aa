"""GPU parity of the audio encoder (SANM) + adaptor against the oracle restatement of
compute/encoder_ops.cpp and compute/adaptor_ops.cpp (oracle/encoder.py), with the
weights rounded to f16 as the GPU stores them. The GPU computes in fp32 with f16-pair
GEMM inputs; the oracle in float64."""
import sys
import os

import numpy as np
import pytest

import fa_dec
import fa_synth
from helpers import rel_rms

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
import encoder as enc_oracle  # noqa: E402

pytestmark = pytest.mark.gpu

SMALL = dict(fa_synth.ENCODER, num_blocks=3, tp_blocks=2)


def _enc(cfg, w, max_frames=512):
    e = fa_dec.Encoder(0, num_blocks=cfg["num_blocks"], tp_blocks=cfg["tp_blocks"], max_frames=max_frames)
    e.load_weights(w)
    return e


@pytest.fixture(scope="module")
def small_w():
    return fa_synth.make_encoder_weights(SMALL, seed=5)


@pytest.mark.parametrize("T", [1, 7, 50, 130, 300])
def test_encoder_adaptor_match_oracle(torch_cuda, small_w, T):
    e = _enc(SMALL, small_w)
    x = fa_synth.lfr_features(np.random.default_rng(T), T)
    got = e.forward(x)
    ref = enc_oracle.adaptor_forward(small_w, enc_oracle.encoder_forward(small_w, x, SMALL))
    assert got.shape == (T, 1024) and np.isfinite(got).all()
    rr = rel_rms(got, ref)
    ma = float(np.abs(got - ref).max())
    assert rr < 1e-4 and ma < 1e-3 * float(np.abs(ref).max()), (rr, ma)
    e.close()


def test_full_encoder_70_layers(torch_cuda):
    w = fa_synth.make_encoder_weights(fa_synth.ENCODER, seed=6)
    e = _enc(fa_synth.ENCODER, w, max_frames=256)
    x = fa_synth.lfr_features(np.random.default_rng(1), 82)          # 5 s of audio
    got = e.forward(x)
    ref = enc_oracle.adaptor_forward(w, enc_oracle.encoder_forward(w, x, fa_synth.ENCODER))
    assert rel_rms(got, ref) < 1e-3, rel_rms(got, ref)
    # bad input size
    with pytest.raises(fa_dec.FaError):
        e.forward(np.zeros((257, 560), np.float32))
    e.close()


def test_encoder_output_feeds_prefill_from_device(torch_cuda, small_w):
    """Encoder output left on the device goes straight into fa_prefill; the result
    equals a prefill of the same embeddings from host memory."""
    torch = torch_cuda
    e = _enc(SMALL, small_w)
    T = 40
    x = fa_synth.lfr_features(np.random.default_rng(3), T)
    d_in = torch.from_numpy(x).cuda()
    d_out = torch.zeros((T, 1024), dtype=torch.float32, device="cuda")
    e.forward_dev(d_in.data_ptr(), T, d_out.data_ptr())
    host = d_out.cpu().numpy()
    cfg = fa_synth.small_config(n_layers=2, hidden=1024, ffn=512, vocab=2048)
    w = fa_synth.make_weights(cfg, seed=4)
    dec = fa_dec.Decoder(0, **fa_synth.decoder_desc(cfg, max_ctx=256, n_pages=32, max_seqs=2, max_rows=64))
    dec.load_weights(w)
    a, b = dec.seq_open(256), dec.seq_open(256)
    n_dev, lg_dev = prefill_ptr(dec, a, d_out.data_ptr(), T)
    n_host, lg_host = dec.prefill(b, host, want_logits=True)
    assert n_dev == n_host and np.array_equal(lg_dev, lg_host)
    dec.close()
    e.close()


def prefill_ptr(dec, sid, ptr, n):
    import ctypes
    nxt = ctypes.c_int()
    lg = np.zeros(dec.vocab, np.float32)
    fa_dec._check(fa_dec.lib().fa_prefill(dec.ctx, sid, ctypes.c_void_p(ptr), n, ctypes.byref(nxt),
                                          lg.ctypes.data_as(ctypes.c_void_p)), dec.ctx)
    return nxt.value, lg


def test_batch_of_512_rows_or_more_matches_oracle(torch_cuda, small_w):
    """A pass of >= 512 rows takes the warp-per-row LayerNorm and the 4-wide bias kernel;
    each utterance still matches the oracle and its own smaller pass."""
    e = _enc(SMALL, small_w, max_frames=1024)
    rng = np.random.default_rng(12)
    utts = [fa_synth.lfr_features(rng, n) for n in (150, 249, 3, 120, 91)]
    assert sum(len(u) for u in utts) >= 512
    batch = e.forward_batch(utts)
    for u, b in zip(utts, batch):
        ref = enc_oracle.adaptor_forward(small_w, enc_oracle.encoder_forward(small_w, u, SMALL))
        assert rel_rms(b, ref) < 1e-4
        assert rel_rms(b, e.forward(u)) < 1e-5
    e.close()


def test_batched_utterances_equal_separate_runs(torch_cuda, small_w):
    """Several utterances in one pass (block-diagonal attention, FSMN within each
    utterance) give each utterance's own result; graphs and direct launches agree."""
    e = _enc(SMALL, small_w)
    rng = np.random.default_rng(11)
    utts = [fa_synth.lfr_features(rng, n) for n in (1, 37, 16, 100, 17)]
    batch = e.forward_batch(utts)
    for u, b in zip(utts, batch):
        ref = enc_oracle.adaptor_forward(small_w, enc_oracle.encoder_forward(small_w, u, SMALL))
        assert rel_rms(b, ref) < 1e-4
        assert rel_rms(b, e.forward(u)) < 1e-5        # other split-K factors at other row counts
    e.set_graphs(False)
    direct = e.forward_batch(utts)
    assert all(np.array_equal(a, b) for a, b in zip(batch, direct))
    with pytest.raises(fa_dec.FaError):
        e.forward_batch([np.zeros((300, 560), np.float32)] * 2)   # 600 frames > max_frames 512
    e.close()
