"""CPU tests of the oracle: pinned against the golden fixtures, then self-consistency."""
import numpy as np
import pytest

import fa_synth
import make_golden
import oracle


def test_q8_0_codec_matches_reference_converter():
    g = np.load(make_golden.os.path.join(make_golden.HERE, "q8_0_codec.npz"))
    q = oracle.q8_0_quantize(g["x"])
    assert np.array_equal(q, g["q8"]), "Q8_0 bytes differ from tools/hf_convert_ggml_q8.py quantize_q8_0"


def test_q8_0_roundtrip_within_half_step():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((4, 1024)).astype(np.float32) * 5
    q = oracle.q8_0_quantize(x)
    y = oracle.q8_0_dequant(q, 1024)
    d = np.abs(x.reshape(-1, 32)).max(1) / 127
    err = np.abs(x - y).reshape(-1, 32).max(1)
    # half a step, plus the f16 rounding of the stored scale times |q| <= 127
    assert np.all(err <= d * 0.5 + 127 * d * 2.0 ** -11 + 1e-7)


def test_f16_conversion_matches_ieee():
    rng = np.random.default_rng(1)
    x = np.concatenate([
        rng.standard_normal(100000).astype(np.float32) * 1000,
        rng.standard_normal(10000).astype(np.float32) * 1e-6,      # subnormal range
        np.array([65504, 65519, 65520, 1e9, -1e9, 0.0, -0.0, 6.1035156e-05, 5.9604645e-08,
                  2.9802322e-08, 2.9802326e-08, np.inf, -np.inf], np.float32),
    ])
    mine = oracle.f32_to_f16_bits(x)
    ref = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(mine, ref)
    assert np.array_equal(oracle.f16_bits_to_f32(ref), ref.view(np.float16).astype(np.float32))


def test_rmsnorm_and_rope_match_qwen3_ops():
    o = np.load(make_golden.os.path.join(make_golden.HERE, "ops.npz"))
    yn = oracle.rmsnorm(o["xn"], o["wn"])
    assert np.abs(yn - o["yn"]).max() <= 1e-6 * np.abs(o["yn"]).max()
    cs = oracle.rope_table(40960)
    c, s = cs[o["pos"], :, 0], cs[o["pos"], :, 1]
    q = o["qv"].astype(np.float32)
    qr = np.concatenate([q[:, :64] * c - q[:, 64:] * s, q[:, :64] * s + q[:, 64:] * c], 1)
    assert np.abs(qr - o["qr"]).max() < 1e-5


def _golden_decoder(mode):
    h = np.load(make_golden.os.path.join(make_golden.HERE, "qwen3_small.npz"))
    cfg = make_golden.GOLDEN_CFG
    w = fa_synth.make_weights(cfg, seed=int(h["seed"]))
    assert make_golden.weights_checksum(w) == str(h["checksum"]), "synthetic weight stream changed"
    od = oracle.OracleDecoder(cfg, w, n_pages=64, max_seqs=4, max_pages_per_seq=16, max_pos=4096, mode=mode)
    return h, cfg, w, od


@pytest.mark.parametrize("mode,tol", [(oracle.MODE_EXACT, 1e-3), (oracle.MODE_W16, 2e-3)])
def test_decoder_logits_match_qwen3(mode, tol):
    h, cfg, w, od = _golden_decoder(mode)
    od.seq_open(0)
    emb = oracle.bf16_bits_to_f32(w["llm.model.embed_tokens.weight"][2]).reshape(cfg["vocab"], cfg["hidden"])
    rows = np.concatenate([emb[h["pre"]], h["audio"], emb[h["suf"]]], 0)
    lg, _ = od.forward([0] * 16, embeds=rows)
    outs = [lg] + [od.forward([0], tokens=[t])[0] for t in h["dec"]]
    L = np.concatenate(outs, 0)
    ref = h["logits"]
    rr = np.sqrt(((L - ref) ** 2).mean() / (ref ** 2).mean())
    assert rr < tol, rr
    assert np.array_equal(L.argmax(1), ref.argmax(1))


def test_prefill_equals_stepwise():
    h, cfg, w, od = _golden_decoder(oracle.MODE_W16)
    od2 = oracle.OracleDecoder(cfg, w, n_pages=64, max_seqs=4, max_pages_per_seq=16, max_pos=4096, mode=oracle.MODE_W16)
    toks = np.random.default_rng(3).integers(0, cfg["vocab"], 21)
    od.seq_open(1)
    od2.seq_open(1)
    a, _ = od.forward([1] * 21, tokens=toks)
    b = np.concatenate([od2.forward([1], tokens=[t])[0] for t in toks])
    assert np.abs(a - b).max() <= 1e-4 * np.abs(b).max()
    assert np.array_equal(od.pool, od2.pool)
    assert np.array_equal(od.block_table, od2.block_table)


def test_paged_attention_matches_dense():
    rng = np.random.default_rng(4)
    n_pages, PT, D = 40, 16, 128
    pool = oracle.f32_to_f16_bits(rng.standard_normal((n_pages, 8, 2, PT, D)).astype(np.float32))
    bt = np.stack([rng.permutation(n_pages)[:8] for _ in range(3)]).astype(np.int32)
    n_kv = np.array([1, 37, 128], np.int32)
    q = rng.standard_normal((3, 16, 128)).astype(np.float32) * 0.2
    out = oracle.paged_attention(q, [0, 1, 2], n_kv, bt, pool)
    P = oracle.f16_bits_to_f32(pool)
    for m in range(3):
        n = n_kv[m]
        toks = np.arange(n)
        pg = bt[m, toks // PT]
        for H in range(16):
            K = P[pg, H // 2, 0, toks % PT].astype(np.float64)
            V = P[pg, H // 2, 1, toks % PT].astype(np.float64)
            s = K @ q[m, H].astype(np.float64)
            p = np.exp(s - s.max())
            p /= p.sum()
            assert np.allclose(out[m, H * 128:(H + 1) * 128], p @ V, atol=1e-6)


def test_paged_append_then_gather_equals_contiguous_cache_view():
    """The reference keeps each layer's cache as one token-major slab [n_ctx][8*128],
    writes step n's K/V at row n (llm_ops_gpu.cpp:82-93) and reads [0, n_kv) back as
    [8][n_kv][128] (:97-105). Appending the same tokens to scattered pages and gathering
    them must give exactly that array."""
    rng = np.random.default_rng(11)
    L, n_pages, PT, D, H = 3, 64, 16, 128, 8
    lens = np.array([1, 16, 17, 70], np.int32)
    bt_stride = 6
    bt = rng.permutation(n_pages)[: 4 * bt_stride].reshape(4, bt_stride).astype(np.int32)
    pool = np.zeros((L, n_pages, H * 2 * PT * D), np.uint16)
    slabs_k = [np.zeros((L, int(n), H * D), np.uint16) for n in lens]
    slabs_v = [np.zeros((L, int(n), H * D), np.uint16) for n in lens]
    for step in range(int(lens.max())):
        live = np.nonzero(lens > step)[0]
        k = oracle.f32_to_f16_bits(rng.standard_normal((len(live), L, H, D)).astype(np.float32))
        v = oracle.f32_to_f16_bits(rng.standard_normal((len(live), L, H, D)).astype(np.float32))
        oracle.kv_append_raw(k, v, live.astype(np.int32), np.full(len(live), step, np.int32), bt, pool, L, n_pages)
        for i, m in enumerate(live):
            slabs_k[m][:, step] = k[i].reshape(L, H * D)
            slabs_v[m][:, step] = v[i].reshape(L, H * D)
    order = np.array([2, 0, 3, 1], np.int32)            # slots in any order, rows packed
    n_kv = lens[order]
    row0 = np.concatenate([[0], np.cumsum(n_kv)[:-1]]).astype(np.int32)
    gk, gv = oracle.kv_gather(pool, bt, order, n_kv, row0, int(n_kv.sum()))
    for i, m in enumerate(order):
        r = slice(row0[i], row0[i] + n_kv[i])
        want_k = slabs_k[m].reshape(L, -1, H, D).transpose(0, 2, 1, 3)
        want_v = slabs_v[m].reshape(L, -1, H, D).transpose(0, 2, 1, 3)
        assert np.array_equal(gk[:, :, r], want_k)
        assert np.array_equal(gv[:, :, r], want_v)


def test_ggml_cpu_mode_is_a_coarser_approximation():
    """The reference's CPU backend quantises activations to Q8_0; the oracle restates it
    (mode 2). It stays within a few percent of exact arithmetic on the golden model."""
    h, cfg, w, od = _golden_decoder(oracle.MODE_GGML_CPU)
    od.seq_open(0)
    emb = oracle.bf16_bits_to_f32(w["llm.model.embed_tokens.weight"][2]).reshape(cfg["vocab"], cfg["hidden"])
    rows = np.concatenate([emb[h["pre"]], h["audio"], emb[h["suf"]]], 0)
    lg, _ = od.forward([0] * 16, embeds=rows)
    ref = h["logits"][:16]
    rr = np.sqrt(((lg - ref) ** 2).mean() / (ref ** 2).mean())
    assert 1e-3 < rr < 0.1, rr


def test_allocator_and_compaction_restatement():
    a = oracle.PageAllocatorOracle(10)
    got = [a.alloc() for _ in range(6)]
    assert got == [0, 1, 2, 3, 4, 5]
    a.free(2)
    a.free(4)
    assert a.alloc() == 2
    live = [0, 1, 2, 3, 5]
    src, dst = oracle.compaction_plan(live, 10)
    assert (src, dst) == ([5], [4])


def test_f16_weights_stay_close_to_exact_weights():
    """Mode 1 (the CUDA path: weights rounded once to f16) against mode 0 (exact d*q)
    on the golden model: the fixed weight rounding moves the logits by far less than
    the reference's own Q8_0 activation quantisation (mode 2) does."""
    outs = {}
    for mode in (oracle.MODE_EXACT, oracle.MODE_W16, oracle.MODE_GGML_CPU):
        h, cfg, w, od = _golden_decoder(mode)
        od.seq_open(0)
        emb = oracle.bf16_bits_to_f32(w["llm.model.embed_tokens.weight"][2]).reshape(cfg["vocab"], cfg["hidden"])
        rows = np.concatenate([emb[h["pre"]], h["audio"], emb[h["suf"]]], 0)
        outs[mode], _ = od.forward([0] * 16, embeds=rows)
    ref = outs[oracle.MODE_EXACT]
    rr = lambda a: float(np.sqrt(((a - ref) ** 2).mean() / (ref ** 2).mean()))
    assert rr(outs[oracle.MODE_W16]) < 2e-3
    assert rr(outs[oracle.MODE_W16]) < 0.2 * rr(outs[oracle.MODE_GGML_CPU])


def test_encoder_oracle_matches_independent_torch_formulation():
    """oracle/encoder.py (numpy restatement of compute/encoder_ops.cpp:17-290 and
    compute/adaptor_ops.cpp:11-149) against the fixture of make_encoder_golden.py: the same
    graphs in PyTorch float64 with gguf-py's Q8_0 dequantiser, a depthwise Conv1d for the
    FSMN memory and scaled_dot_product_attention, on a 3 + 2-layer encoder at 5 and 21
    frames. Both are float64, so they agree to rounding."""
    import encoder
    import make_encoder_golden as g
    h = np.load(make_golden.os.path.join(make_golden.HERE, "encoder_small.npz"))
    w = fa_synth.make_encoder_weights(g.ENC_CFG, seed=int(h["seed"]))
    assert make_golden.weights_checksum(w) == str(h["checksum"]), "synthetic encoder weight stream changed"
    for T in g.FRAMES:
        enc = encoder.encoder_forward(w, h[f"x{T}"], g.ENC_CFG, w16=False)
        ada = encoder.adaptor_forward(w, enc, w16=False)
        for got, ref in ((enc, h[f"enc{T}"]), (ada, h[f"ada{T}"])):
            assert np.abs(got - ref).max() <= 1e-12 * np.abs(ref).max(), T
