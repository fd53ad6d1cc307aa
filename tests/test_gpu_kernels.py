"""GPU parity of the kernel-level C-ABI entry points against the CPU oracle.

Byte identity for the page writes (kernel 1 and the raw append), tolerance for the
floating-point attention and GEMM outputs, exact indices for the argmax.
"""
import math

import numpy as np
import pytest

import fa_dec
import fa_synth
import oracle
from helpers import assert_close, dev, max_abs, rel_rms

pytestmark = pytest.mark.gpu

PAGE_ELEMS = 8 * 2 * 16 * 128


def _bf16_vec(rng, n, lo, hi):
    return oracle.bf16_bits_to_f32(fa_synth.f32_to_bf16_bits(rng.uniform(lo, hi, n).astype(np.float32)))


def _i16(a):
    return np.ascontiguousarray(a, np.uint16).view(np.int16)


def _u16(t):
    return t.cpu().numpy().view(np.uint16)


# ------------------------------------------------------------------- kernel 1 --
def test_qknorm_rope_append_pages_byte_identical(torch_cuda):
    torch = torch_cuda
    rng = np.random.default_rng(10)
    n_pages, max_pos, n_seq = 2048, 4096, 8
    bt_stride = max_pos // 16
    bt = rng.permutation(n_pages)[: n_seq * bt_stride].reshape(n_seq, bt_stride).astype(np.int32)
    pairs = set()
    edge = [0, 15, 16, 17, 4095, 2047, 2048]
    rows = []
    for p in edge:
        rows.append((int(rng.integers(n_seq)), p))
    while len(rows) < 61:
        rows.append((int(rng.integers(n_seq)), int(rng.integers(max_pos))))
    rows = [r for r in rows if not (r in pairs or pairs.add(r))]
    slot = np.array([r[0] for r in rows], np.int32)
    pos = np.array([r[1] for r in rows], np.int32)
    M = len(rows)
    qkv = (rng.standard_normal((M, 32 * 128)) * 3).astype(np.float32)
    qn, kn = _bf16_vec(rng, 128, 0.8, 1.2), _bf16_vec(rng, 128, 0.8, 1.2)
    rope = oracle.rope_table(max_pos)
    pool0 = oracle.f32_to_f16_bits(rng.standard_normal((n_pages, PAGE_ELEMS)).astype(np.float32))

    d_pool = dev(torch, _i16(pool0))
    d_q = torch.zeros((M, 16 * 128), dtype=torch.float32, device="cuda")
    d_err = torch.zeros(1, dtype=torch.int32, device="cuda")
    args = [dev(torch, a) for a in (qkv, pos, slot, bt, qn, kn, rope)]
    fa_dec.op_qknorm_rope_append(args[0].data_ptr(), M, args[1].data_ptr(), args[2].data_ptr(), args[3].data_ptr(),
                                 bt_stride, n_pages, args[4].data_ptr(), args[5].data_ptr(), 1e-5,
                                 args[6].data_ptr(), max_pos, d_pool.data_ptr(), d_q.data_ptr(), d_err.data_ptr())
    torch.cuda.synchronize()
    pool_ref = pool0.copy()
    q_ref = oracle.qknorm_rope_append(qkv, slot, pos, bt, qn, kn, rope, pool_ref)
    assert int(d_err.item()) == 0
    got = _u16(d_pool)
    assert np.array_equal(got, pool_ref), f"{(got != pool_ref).sum()} f16 values differ"
    assert np.array_equal(d_q.cpu().numpy().view(np.uint32), q_ref.view(np.uint32))


def test_qknorm_rope_append_rejects_bad_page(torch_cuda):
    torch = torch_cuda
    n_pages = 4
    bt = np.array([[0, 1, 7, 2]], np.int32)       # page 7 is outside the pool
    pos = np.array([40], np.int32)                # page index 2 -> 7
    slot = np.zeros(1, np.int32)
    qkv = np.ones((1, 4096), np.float32)
    rope = oracle.rope_table(64)
    d_pool = torch.zeros((n_pages, PAGE_ELEMS), dtype=torch.int16, device="cuda")
    d_q = torch.zeros((1, 2048), dtype=torch.float32, device="cuda")
    d_err = torch.zeros(1, dtype=torch.int32, device="cuda")
    a = [dev(torch, x) for x in (qkv, pos, slot, bt, np.ones(128, np.float32), rope)]
    fa_dec.op_qknorm_rope_append(a[0].data_ptr(), 1, a[1].data_ptr(), a[2].data_ptr(), a[3].data_ptr(), 4, n_pages,
                                 a[4].data_ptr(), a[4].data_ptr(), 1e-5, a[5].data_ptr(), 64, d_pool.data_ptr(),
                                 d_q.data_ptr(), d_err.data_ptr())
    torch.cuda.synchronize()
    assert int(d_err.item()) & 2
    assert int(d_pool.abs().sum().item()) == 0


# ----------------------------------------------- raw append (page-table bench) --
def test_raw_append_cfg1_pages_byte_identical(torch_cuda):
    """28 layers x 8 heads x 128 f16, page 16, 32 sequences with contexts ~U[64,1024],
    block tables from a random permutation of a 4096-page pool, 256 append steps with
    K/V ~ N(0,1) cast to f16: the touched pages equal the oracle's byte for byte."""
    torch = torch_cuda
    rng = np.random.default_rng(2024)
    L, n_pages, n_seq, steps = 28, 4096, 32, 256
    ctx0 = rng.integers(64, 1025, n_seq).astype(np.int32)
    bt_stride = (1024 + steps + 15) // 16
    bt = rng.permutation(n_pages)[: n_seq * bt_stride].reshape(n_seq, bt_stride).astype(np.int32)
    d_pool = torch.zeros((L, n_pages, PAGE_ELEMS), dtype=torch.int16, device="cuda")
    pool_ref = np.zeros((L, n_pages, PAGE_ELEMS), np.uint16)
    d_bt = dev(torch, bt)
    slot = np.arange(n_seq, dtype=np.int32)
    d_slot = dev(torch, slot)
    d_err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for s in range(steps):
        pos = ctx0 + s
        k = oracle.f32_to_f16_bits(rng.standard_normal((n_seq, L, 8, 128)).astype(np.float32))
        v = oracle.f32_to_f16_bits(rng.standard_normal((n_seq, L, 8, 128)).astype(np.float32))
        dk, dv, dp = dev(torch, _i16(k)), dev(torch, _i16(v)), dev(torch, pos)
        fa_dec.op_kv_append(dk.data_ptr(), dv.data_ptr(), n_seq, L, dp.data_ptr(), d_slot.data_ptr(),
                            d_bt.data_ptr(), bt_stride, n_pages, d_pool.data_ptr(), d_err.data_ptr())
        oracle.kv_append_raw(k, v, slot, pos, bt, pool_ref, L, n_pages)
    torch.cuda.synchronize()
    assert int(d_err.item()) == 0
    touched = np.unique(np.concatenate([bt[i, ctx0[i] // 16:(ctx0[i] + steps - 1) // 16 + 1] for i in range(n_seq)]))
    idx = torch.from_numpy(touched.astype(np.int64)).cuda()
    got = d_pool.index_select(1, idx).cpu().numpy().view(np.uint16)
    assert np.array_equal(got, pool_ref[:, touched])
    # nothing outside the touched pages was written
    untouched = np.setdiff1d(np.arange(n_pages), touched)
    assert int(d_pool.index_select(1, torch.from_numpy(untouched.astype(np.int64)).cuda()).abs().sum().item()) == 0
    # the gather side of the same workload: 8 of the sequences read back over their whole
    # length, in head-major slabs, equal the oracle's gather of the oracle's pages
    pick = np.array([3, 0, 31, 17, 8, 22, 5, 12], np.int32)
    n_kv = (ctx0[pick] + steps).astype(np.int32)
    row0 = np.concatenate([[0], np.cumsum(n_kv)[:-1]]).astype(np.int32)
    total = int(n_kv.sum())
    d_k = torch.zeros((L, 8, total, 128), dtype=torch.int16, device="cuda")
    d_v = torch.zeros_like(d_k)
    d_pick, d_nkv, d_row0 = dev(torch, pick), dev(torch, n_kv), dev(torch, row0)
    fa_dec.op_kv_gather(d_pool.data_ptr(), L, n_pages, d_bt.data_ptr(), bt_stride, d_pick.data_ptr(),
                        d_nkv.data_ptr(), d_row0.data_ptr(), len(pick), bt_stride, total, d_k.data_ptr(),
                        d_v.data_ptr(), d_err.data_ptr())
    torch.cuda.synchronize()
    assert int(d_err.item()) == 0
    gk, gv = oracle.kv_gather(pool_ref, bt, pick, n_kv, row0, total)
    assert np.array_equal(_u16(d_k), gk)
    assert np.array_equal(_u16(d_v), gv)


def test_kv_gather_ragged_and_bounds(torch_cuda):
    """Lengths 0, 1, 15, 16, 17, 255, 256 and random ones, sequences gathered in any slot
    order into a slab with gaps: the rows equal the oracle's, the gaps keep their
    sentinel, and a length beyond max_pages or a page outside the pool sets its error bit
    and writes nothing for that sequence."""
    torch = torch_cuda
    rng = np.random.default_rng(77)
    L, n_pages, max_pages = 5, 600, 20
    lens = np.array([0, 1, 15, 16, 17, 255, 256, 320, 3, 100, 200, 33], np.int32)
    n_seq = len(lens)
    bt = rng.permutation(n_pages)[: n_seq * max_pages].reshape(n_seq, max_pages).astype(np.int32)
    pool = rng.integers(0, 1 << 16, (L, n_pages, PAGE_ELEMS), dtype=np.uint16)
    d_pool, d_bt = dev(torch, _i16(pool)), dev(torch, bt)
    order = rng.permutation(n_seq).astype(np.int32)
    n_kv = lens[order]
    row0 = (np.concatenate([[0], np.cumsum(n_kv + 5)[:-1]]) + 3).astype(np.int32)   # gaps of 5 rows
    total = int(row0[-1] + n_kv[-1] + 7)
    sentinel = 0x7C01                                           # an f16 NaN pattern nothing writes
    d_k = torch.full((L, 8, total, 128), sentinel, dtype=torch.int16, device="cuda")
    d_v = torch.full_like(d_k, sentinel)
    d_err = torch.zeros(1, dtype=torch.int32, device="cuda")
    a = [dev(torch, x) for x in (order, n_kv, row0)]
    fa_dec.op_kv_gather(d_pool.data_ptr(), L, n_pages, d_bt.data_ptr(), max_pages, a[0].data_ptr(), a[1].data_ptr(),
                        a[2].data_ptr(), n_seq, max_pages, total, d_k.data_ptr(), d_v.data_ptr(), d_err.data_ptr())
    torch.cuda.synchronize()
    assert int(d_err.item()) == 0
    want_k = np.full((L, 8, total, 128), sentinel, np.uint16)
    want_v = want_k.copy()
    oracle.kv_gather(pool, bt, order, n_kv, row0, total, out_k=want_k, out_v=want_v)
    assert np.array_equal(_u16(d_k), want_k)
    assert np.array_equal(_u16(d_v), want_v)

    # a length past max_pages * 16 (bit 8) and a page outside the pool (bit 2)
    bad_bt = bt.copy()
    bad_bt[1, 0] = n_pages + 3
    cases = [(np.array([0], np.int32), np.array([max_pages * 16 + 1], np.int32), bt, 8),
             (np.array([1], np.int32), np.array([1], np.int32), bad_bt, 2)]
    for slot_, nkv_, bt_, bit in cases:
        d_err.zero_()
        d_k.fill_(sentinel)
        b = [dev(torch, x) for x in (slot_, nkv_, np.zeros(1, np.int32), bt_)]
        fa_dec.op_kv_gather(d_pool.data_ptr(), L, n_pages, b[3].data_ptr(), max_pages, b[0].data_ptr(),
                            b[1].data_ptr(), b[2].data_ptr(), 1, max_pages, total, d_k.data_ptr(), d_v.data_ptr(),
                            d_err.data_ptr())
        torch.cuda.synchronize()
        assert int(d_err.item()) == bit
        assert bool((d_k == sentinel).all().item())


# ------------------------------------------------------------------- kernel 2 --
def _attention_case(torch, rng, n_kv, pps, n_splits=None, n_pages=1024, q_scale=0.3):
    M = len(n_kv)
    n_kv = np.asarray(n_kv, np.int32)
    max_pg = int(math.ceil(n_kv.max() / 16))
    bt_stride = max_pg + 1
    bt = np.stack([rng.choice(n_pages, bt_stride, replace=bt_stride > n_pages) for _ in range(M)]).astype(np.int32)
    pool = oracle.f32_to_f16_bits(rng.standard_normal((n_pages, PAGE_ELEMS)).astype(np.float32))
    q = (rng.standard_normal((M, 16, 128)) * q_scale).astype(np.float32)
    slot = np.arange(M, dtype=np.int32)
    pos = n_kv - 1
    if n_splits is None:
        n_splits = int(math.ceil(max_pg / pps))
    d = [dev(torch, a) for a in (q, pos, slot, bt, _i16(pool))]
    out32 = torch.zeros((M, 2048), dtype=torch.float32, device="cuda")
    out16 = torch.zeros((M, 2048), dtype=torch.int16, device="cuda")
    nb = fa_dec.op_attention_scratch_bytes(M, n_splits)
    scratch = torch.zeros(max(nb, 16), dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    fa_dec.op_paged_attention(d[0].data_ptr(), M, d[1].data_ptr(), d[2].data_ptr(), d[3].data_ptr(), bt_stride,
                              n_pages, d[4].data_ptr(), pps, n_splits, scratch.data_ptr(), out16.data_ptr(),
                              out32.data_ptr(), err.data_ptr())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = oracle.paged_attention(q, slot, n_kv, bt, pool)
    return out32.cpu().numpy(), oracle.f16_bits_to_f32(_u16(out16)), ref


@pytest.mark.parametrize("n_kv,pps,n_splits", [
    ([1, 2, 15, 16, 17, 31, 33, 100, 257], 4, None),      # ragged, partial pages, idle warps
    ([5, 64, 300], 20, 1),                                  # one split: direct output
    ([2048] * 6 + [1, 2049, 1000], 32, None),               # long contexts, split-K combine
    ([4000, 3], 64, None),
])
def test_paged_attention_matches_oracle(torch_cuda, n_kv, pps, n_splits):
    rng = np.random.default_rng(sum(n_kv) + pps)
    o32, o16, ref = _attention_case(torch_cuda, rng, n_kv, pps, n_splits)
    assert_close(o32, ref, max_abs_tol=1e-4, rel_rms_tol=1e-5, what="attention f32")
    assert_close(o16, ref, what="attention f16")


def test_paged_attention_sharp_softmax(torch_cuda):
    """Large scores (q scale 3): the online-softmax rescaling is exercised hard."""
    rng = np.random.default_rng(77)
    o32, o16, ref = _attention_case(torch_cuda, rng, [700, 1333, 50], 8, None, q_scale=3.0)
    assert_close(o32, ref, max_abs_tol=1e-3, rel_rms_tol=1e-5, what="attention f32")


@pytest.mark.parametrize("case", ["too_few_splits", "pos_past_block_table", "negative_pos"])
def test_paged_attention_rejects_bad_rows(torch_cuda, case):
    """A row the kernel cannot serve sets error bit 8 and keeps its old output; the other
    rows are still computed."""
    torch = torch_cuda
    rng = np.random.default_rng(12)
    n_pages, bt_stride = 256, 8
    M = 3
    n_kv = np.array([100, 37, 128], np.int32)            # 7, 3 and 8 pages
    pps, n_splits = 4, 2
    if case == "too_few_splits":
        pps = 3                                          # 6 pages covered; row 0 and 2 need more
    bt = np.stack([rng.choice(n_pages, bt_stride, replace=False) for _ in range(M)]).astype(np.int32)
    pool = oracle.f32_to_f16_bits(rng.standard_normal((n_pages, PAGE_ELEMS)).astype(np.float32))
    q = (rng.standard_normal((M, 16, 128)) * 0.3).astype(np.float32)
    slot = np.arange(M, dtype=np.int32)
    pos = n_kv - 1
    bad = {0, 2} if case == "too_few_splits" else {0}
    if case == "pos_past_block_table":
        pos[0] = bt_stride * 16                          # page 8 of an 8-entry row
    if case == "negative_pos":
        pos[0] = -5
    ref = oracle.paged_attention(q, slot, n_kv, bt, pool)
    d = [dev(torch, a) for a in (q, pos, slot, bt, _i16(pool))]
    out32 = torch.full((M, 2048), 3.0, dtype=torch.float32, device="cuda")
    scratch = torch.zeros(fa_dec.op_attention_scratch_bytes(M, n_splits), dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    fa_dec.op_paged_attention(d[0].data_ptr(), M, d[1].data_ptr(), d[2].data_ptr(), d[3].data_ptr(), bt_stride,
                              n_pages, d[4].data_ptr(), pps, n_splits, scratch.data_ptr(), 0, out32.data_ptr(),
                              err.data_ptr())
    torch.cuda.synchronize()
    assert int(err.item()) == 8
    got = out32.cpu().numpy()
    for m in range(M):
        if m in bad:
            assert (got[m] == 3.0).all(), m
        else:
            assert_close(got[m], ref[m], max_abs_tol=1e-4, rel_rms_tol=1e-5, what=f"row {m}")


def test_paged_attention_full_size_batch128_ctx2048(torch_cuda):
    """B=128 rows at 2048-2175 tokens (one layer of the steady-state decode shape); all
    rows checked for finiteness, 12 sampled rows against the oracle."""
    torch = torch_cuda
    rng = np.random.default_rng(5)
    M, n_pages = 128, 128 * 137
    n_kv = (2048 + rng.integers(0, 128, M)).astype(np.int32)
    bt_stride = 137
    bt = rng.permutation(n_pages).reshape(M, bt_stride).astype(np.int32)
    gen = torch.Generator(device="cuda").manual_seed(5)
    d_pool = (torch.randn((n_pages, PAGE_ELEMS), generator=gen, device="cuda", dtype=torch.float32) * 0.5)
    d_pool = d_pool.to(torch.float16).view(torch.int16)
    q = (rng.standard_normal((M, 16, 128)) * 0.3).astype(np.float32)
    slot = np.arange(M, dtype=np.int32)
    d = [dev(torch, a) for a in (q, n_kv - 1, slot, bt)] + [d_pool]
    pps, n_splits = 64, 3
    out32 = torch.zeros((M, 2048), dtype=torch.float32, device="cuda")
    scratch = torch.zeros(fa_dec.op_attention_scratch_bytes(M, n_splits), dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    fa_dec.op_paged_attention(d[0].data_ptr(), M, d[1].data_ptr(), d[2].data_ptr(), d[3].data_ptr(), bt_stride,
                              n_pages, d[4].data_ptr(), pps, n_splits, scratch.data_ptr(), 0, out32.data_ptr(),
                              err.data_ptr())
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    got = out32.cpu().numpy()
    assert np.isfinite(got).all()
    rows = rng.choice(M, 12, replace=False)
    used = np.unique(bt[rows])
    sub = d_pool.index_select(0, torch.from_numpy(used.astype(np.int64)).cuda()).cpu().numpy().view(np.uint16)
    remap = np.searchsorted(used, bt[rows]).astype(np.int32)
    ref = oracle.paged_attention(q[rows], np.arange(12, dtype=np.int32), n_kv[rows], remap, sub)
    assert_close(got[rows], ref, max_abs_tol=1e-4, rel_rms_tol=1e-5, what="attention full size")


# ------------------------------------------------------------------- kernel 4 --
def _q8_device(torch, rng, N, K):
    """Random Q8_0 weights: GGUF bytes on the host, f16(d * q) [N][K] on the device."""
    raw = fa_synth.q8_0_random(rng, N, K)
    d_raw = dev(torch, raw)
    w16 = torch.zeros((N, K), dtype=torch.int16, device="cuda")       # f16 bit patterns
    fa_dec.op_repack_q8(d_raw.data_ptr(), N, K, w16.data_ptr())
    return raw, w16


# The two weight forms the GEMMs read: "q8p", the decoder's Q8_0 planes (every weight the
# exact d*q, checked against the oracle's exact mode), and "f16", f16(d*q) (the encoder's
# form, checked against the oracle's W16 mode).
FORMS = ["q8p", "f16"]


def _weights(torch, raw, N, K, form):
    """Device weights of GGUF Q8_0 bytes `raw` [N][K/32*34] in `form`, and the oracle mode."""
    d_raw = dev(torch, raw)
    if form == "f16":
        w = torch.zeros((N, K), dtype=torch.int16, device="cuda")
        fa_dec.op_repack_q8(d_raw.data_ptr(), N, K, w.data_ptr())
        return w, oracle.MODE_W16
    w = torch.zeros(fa_dec.op_q8_planes_bytes(N, K), dtype=torch.uint8, device="cuda")
    fa_dec.op_repack_q8_planes(d_raw.data_ptr(), N, K, w.data_ptr())
    return w, oracle.MODE_EXACT


def _gemm(form, a_hi, a_lo, M, K, w, N, split, c, variant):
    f = fa_dec.op_q8p_gemm if form == "q8p" else fa_dec.op_q8_gemm
    f(a_hi, a_lo, M, K, w, N, split, c, variant)


def test_repack_planes_keep_every_gguf_byte(torch_cuda):
    """q [N][K], the scales block-major [K/32][N] and row-major [N][K/32]: the GGUF bytes moved."""
    torch = torch_cuda
    rng = np.random.default_rng(1)
    N, K = 192, 512
    raw = fa_synth.q8_0_random(rng, N, K)
    w, _ = _weights(torch, raw, N, K, "q8p")
    torch.cuda.synchronize()
    got = w.cpu().numpy()
    assert got.nbytes == N * K + N * (K // 32) * 4
    blocks = raw.reshape(N, K // 32, 34)
    d = blocks[:, :, :2].copy().view(np.uint16)[:, :, 0]
    assert np.array_equal(got[:N * K].view(np.int8).reshape(N, K), blocks[:, :, 2:].view(np.int8).reshape(N, K))
    d_t = got[N * K:N * K + N * K // 16].view(np.uint16).reshape(K // 32, N)
    d_r = got[N * K + N * K // 16:].view(np.uint16).reshape(N, K // 32)
    assert np.array_equal(d_t, d.T) and np.array_equal(d_r, d)


def test_repack_rounds_d_times_q_to_f16(torch_cuda):
    rng = np.random.default_rng(0)
    raw, w16 = _q8_device(torch_cuda, rng, 128, 256)
    torch_cuda.cuda.synchronize()
    blocks = raw.reshape(128, 8, 34)
    d = oracle.f16_bits_to_f32(blocks[:, :, :2].copy().view(np.uint16)[:, :, 0])
    q = blocks[:, :, 2:].view(np.int8).astype(np.float32)
    want = oracle.f32_to_f16_bits((d[:, :, None] * q).reshape(128, 256))
    assert np.array_equal(w16.cpu().numpy().view(np.uint16), want)


@pytest.mark.parametrize("form", FORMS)
def test_tcgen05_gemm_single_tile(torch_cuda, form):
    """One CTA (128 x 128 tile, K = 64) of the tcgen05 kernel: the smallest case."""
    torch = torch_cuda
    rng = np.random.default_rng(42)
    M, N, K = 128, 128, 64
    raw = fa_synth.q8_0_random(rng, N, K)
    w, mode = _weights(torch, raw, N, K, form)
    a = rng.standard_normal((M, K)).astype(np.float32)
    hi, lo, a_eff = _split_f16(a)
    d_hi, d_lo = dev(torch, _i16(hi)), dev(torch, _i16(lo))
    c = torch.zeros((1, M, N), dtype=torch.float32, device="cuda")
    _gemm(form, d_hi.data_ptr(), d_lo.data_ptr(), M, K, w.data_ptr(), N, 1, c.data_ptr(), 0)
    torch.cuda.synchronize()
    ref = oracle.gemm_q8(a_eff, raw, N, mode)
    got = c[0].cpu().numpy()
    assert rel_rms(got, ref) < 5e-6, rel_rms(got, ref)


def _split_f16(x):
    """x = hi + lo as two f16 arrays (the form the GEMM reads); returns (hi, lo, hi + lo)."""
    hi = oracle.f32_to_f16_bits(x)
    lo = oracle.f32_to_f16_bits(x - oracle.f16_bits_to_f32(hi))
    return hi, lo, oracle.f16_bits_to_f32(hi) + oracle.f16_bits_to_f32(lo)


@pytest.mark.parametrize("form", FORMS)
@pytest.mark.parametrize("variant", [0, 1, 2, 4])
@pytest.mark.parametrize("M,N,K,split", [
    (1, 1024, 1024, 1), (5, 4096, 1024, 4), (16, 1024, 2048, 8), (17, 2048, 1024, 2),
    (64, 6144, 1024, 4), (128, 1024, 3072, 12), (200, 1024, 1024, 1), (300, 512, 2048, 2),
    # prefill-size row counts, ragged last row tile
    (256, 4096, 1024, 1), (400, 6144, 1024, 2), (513, 1024, 3072, 4),
])
def test_q8_gemm_matches_oracle(torch_cuda, M, N, K, split, variant, form):
    if variant == 4 and M > 128 and form == "f16":
        pytest.skip("with f16 weights the swapped tcgen05 kernel takes at most 128 rows")
    torch = torch_cuda
    rng = np.random.default_rng(M * 7 + N + K)
    raw = fa_synth.q8_0_random(rng, N, K)
    w, mode = _weights(torch, raw, N, K, form)
    a = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    hi, lo, a_eff = _split_f16(a)
    d_hi, d_lo = dev(torch, _i16(hi)), dev(torch, _i16(lo))
    c = torch.zeros((split, M, N), dtype=torch.float32, device="cuda")
    _gemm(form, d_hi.data_ptr(), d_lo.data_ptr(), M, K, w.data_ptr(), N, split, c.data_ptr(), variant)
    torch.cuda.synchronize()
    got = c.sum(0).cpu().numpy()
    ref = oracle.gemm_q8(a_eff, raw, N, mode)
    # fp32 accumulation over K (up to 3072) against a double-precision sum: ~sqrt(K) * 2^-24
    assert rel_rms(got, ref) < 5e-6, rel_rms(got, ref)
    assert max_abs(got, ref) < 2e-5 * np.abs(ref).max()
    # without the lo plane the result is the f16-activation product
    c.zero_()
    _gemm(form, d_hi.data_ptr(), 0, M, K, w.data_ptr(), N, split, c.data_ptr(), variant)
    torch.cuda.synchronize()
    ref16 = oracle.gemm_q8(oracle.f16_bits_to_f32(hi), raw, N, mode)
    assert rel_rms(c.sum(0).cpu().numpy(), ref16) < 5e-6


@pytest.mark.parametrize("M,N,K", [
    (1, 4096, 1024), (2, 1024, 2048), (3, 6144, 1024), (4, 1024, 3072), (5, 4096, 1024), (8, 1024, 3072),
    (1, 768, 512), (6, 64, 256), (8, 2048, 4096), (2, 151936, 1024),
])
@pytest.mark.parametrize("form", FORMS)
def test_small_m_gemm_matches_oracle(torch_cuda, M, N, K, form):
    """The CUDA-core kernel (variant 3) on the decoder's shapes and odd ones: fp32 result
    against the oracle's double sum, with and without the lo plane."""
    torch = torch_cuda
    rng = np.random.default_rng(M * 11 + N + K)
    raw = fa_synth.q8_0_random(rng, N, K)
    w, mode = _weights(torch, raw, N, K, form)
    a = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    hi, lo, a_eff = _split_f16(a)
    d_hi, d_lo = dev(torch, _i16(hi)), dev(torch, _i16(lo))
    assert fa_dec.op_gemm_plan(M, N, K, variant=3) == 1
    c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    _gemm(form, d_hi.data_ptr(), d_lo.data_ptr(), M, K, w.data_ptr(), N, 1, c.data_ptr(), 3)
    torch.cuda.synchronize()
    got = c.cpu().numpy()
    ref = oracle.gemm_q8(a_eff, raw, N, mode)
    assert rel_rms(got, ref) < 5e-6, rel_rms(got, ref)
    assert max_abs(got, ref) < 2e-5 * np.abs(ref).max()
    c.zero_()
    _gemm(form, d_hi.data_ptr(), 0, M, K, w.data_ptr(), N, 1, c.data_ptr(), 3)
    torch.cuda.synchronize()
    ref16 = oracle.gemm_q8(oracle.f16_bits_to_f32(hi), raw, N, mode)
    assert rel_rms(c.cpu().numpy(), ref16) < 5e-6


@pytest.mark.parametrize("M,F,K", [(1, 3072, 1024), (2, 3072, 1024), (5, 512, 256), (8, 1536, 2048)])
@pytest.mark.parametrize("form", FORMS)
def test_small_m_gemm_swiglu_equals_separate_kernels(torch_cuda, M, F, K, form):
    """Gate/up GEMM with SwiGLU in its epilogue: the same bits as the small-M GEMM followed
    by the decoder's SwiGLU kernel, and within f16-pair precision of the oracle."""
    torch = torch_cuda
    rng = np.random.default_rng(M + F + K)
    raw = fa_synth.q8_0_random(rng, 2 * F, K)
    w, mode = _weights(torch, raw, 2 * F, K, form)
    hi, lo, a_eff = _split_f16(rng.standard_normal((M, K)).astype(np.float32))
    d_hi, d_lo = dev(torch, _i16(hi)), dev(torch, _i16(lo))
    h16 = torch.zeros((M, F), dtype=torch.int16, device="cuda")
    h_lo = torch.zeros_like(h16)
    sw = fa_dec.op_q8p_gemm_swiglu if form == "q8p" else fa_dec.op_q8_gemm_swiglu
    sw(d_hi.data_ptr(), d_lo.data_ptr(), M, K, w.data_ptr(), 2 * F, h16.data_ptr(), h_lo.data_ptr())
    c = torch.zeros((M, 2 * F), dtype=torch.float32, device="cuda")
    _gemm(form, d_hi.data_ptr(), d_lo.data_ptr(), M, K, w.data_ptr(), 2 * F, 1, c.data_ptr(), 3)
    r16 = torch.zeros_like(h16)
    r_lo = torch.zeros_like(h16)
    fa_dec.op_swiglu(c.data_ptr(), 1, M, F, r16.data_ptr(), r_lo.data_ptr())
    torch.cuda.synchronize()
    assert torch.equal(h16, r16) and torch.equal(h_lo, r_lo)
    gu = oracle.gemm_q8(a_eff, raw, 2 * F, mode).astype(np.float64)
    g, u = gu[:, :F], gu[:, F:]
    want = g / (1.0 + np.exp(-g)) * u
    got = oracle.f16_bits_to_f32(_u16(h16)).astype(np.float64) + oracle.f16_bits_to_f32(_u16(h_lo))
    assert rel_rms(got, want) < 5e-6, rel_rms(got, want)


@pytest.mark.parametrize("M,N,K", [(3, 4096, 1024), (16, 1024, 3072), (17, 6144, 1024), (32, 1024, 2048),
                                   (33, 4096, 1024), (64, 1024, 3072), (9, 256, 512), (65, 4096, 1024),
                                   (128, 1024, 3072), (100, 6144, 1024)])
@pytest.mark.parametrize("form", FORMS)
def test_few_row_tcgen05_gemm_matches_oracle(torch_cuda, M, N, K, form):
    """The swapped tcgen05 kernel (variant 4) at each activation tile width (16, 32, 64,
    128 rows) and the planner's split, against the oracle's double sum."""
    torch = torch_cuda
    rng = np.random.default_rng(M * 13 + N + K)
    raw = fa_synth.q8_0_random(rng, N, K)
    w, mode = _weights(torch, raw, N, K, form)
    hi, lo, a_eff = _split_f16((rng.standard_normal((M, K)) * 3).astype(np.float32))
    d_hi, d_lo = dev(torch, _i16(hi)), dev(torch, _i16(lo))
    split = fa_dec.op_gemm_plan(M, N, K, variant=4)
    c = torch.zeros((split, M, N), dtype=torch.float32, device="cuda")
    _gemm(form, d_hi.data_ptr(), d_lo.data_ptr(), M, K, w.data_ptr(), N, split, c.data_ptr(), 4)
    torch.cuda.synchronize()
    got = c.sum(0).cpu().numpy()
    ref = oracle.gemm_q8(a_eff, raw, N, mode)
    assert rel_rms(got, ref) < 5e-6, rel_rms(got, ref)
    assert max_abs(got, ref) < 2e-5 * np.abs(ref).max()


@pytest.mark.parametrize("form", FORMS)
def test_small_m_gemm_rows_do_not_depend_on_m(torch_cuda, form):
    """A row's result is the same bits whether it is computed alone or among 2..8 rows, so
    batching sequences together does not change any sequence's logits."""
    torch = torch_cuda
    rng = np.random.default_rng(5)
    N, K = 4096, 1024
    w, _ = _weights(torch, fa_synth.q8_0_random(rng, N, K), N, K, form)
    hi, lo, _ = _split_f16((rng.standard_normal((8, K)) * 3).astype(np.float32))
    d_hi, d_lo = dev(torch, _i16(hi)), dev(torch, _i16(lo))
    outs = {}
    for M in (1, 2, 3, 4, 8):
        c = torch.zeros((M, N), dtype=torch.float32, device="cuda")
        _gemm(form, d_hi.data_ptr(), d_lo.data_ptr(), M, K, w.data_ptr(), N, 1, c.data_ptr(), 3)
        torch.cuda.synchronize()
        outs[M] = c.cpu().numpy()
    for M in (2, 3, 4, 8):
        assert np.array_equal(outs[M][0].view(np.uint32), outs[1][0].view(np.uint32))
        assert np.array_equal(outs[M][:2].view(np.uint32), outs[2].view(np.uint32))


def test_small_m_gemm_rejects_shapes_it_does_not_take(torch_cuda):
    torch = torch_cuda
    a = torch.zeros((9, 1024), dtype=torch.int16, device="cuda")
    w = torch.zeros((1024, 1024), dtype=torch.int16, device="cuda")
    c = torch.zeros((9, 1024), dtype=torch.float32, device="cuda")
    for M, K, split in ((9, 1024, 1), (4, 320, 1), (4, 1024, 2)):
        with pytest.raises(RuntimeError):
            fa_dec.op_q8_gemm(a.data_ptr(), 0, M, K, w.data_ptr(), 1024, split, c.data_ptr(), 3)
    # variant 0 sends what the small-M kernel does not take to tcgen05
    fa_dec.op_q8_gemm(a.data_ptr(), 0, 4, 1024, w.data_ptr(), 1024, 2, c.data_ptr(), 0)
    torch.cuda.synchronize()


@pytest.mark.parametrize("form", FORMS)
@pytest.mark.parametrize("variant", [0, 1, 3, 4])
@pytest.mark.parametrize("M,N", [(7, 151936), (300, 4096), (1, 151936), (4, 151936), (40, 151936), (128, 151936)])
def test_lm_head_argmax_full_vocab(torch_cuda, variant, M, N, form):
    if (variant == 3 and M > 8) or (variant == 4 and M > 128 and form == "f16"):
        pytest.skip("outside the kernel's row range")
    torch = torch_cuda
    rng = np.random.default_rng(3)
    K = 1024
    raw = fa_synth.q8_0_random(rng, N, K)
    w, mode = _weights(torch, raw, N, K, form)
    hi, lo, a_eff = _split_f16(rng.standard_normal((M, K)).astype(np.float32))
    d_hi, d_lo = dev(torch, _i16(hi)), dev(torch, _i16(lo))
    scratch = torch.zeros(fa_dec.op_argmax_scratch_bytes(M, N), dtype=torch.uint8, device="cuda")
    nxt = torch.zeros(M, dtype=torch.int32, device="cuda")
    logits = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    am = fa_dec.op_q8p_gemm_argmax if form == "q8p" else fa_dec.op_q8_gemm_argmax
    am(d_hi.data_ptr(), d_lo.data_ptr(), M, K, w.data_ptr(), N, scratch.data_ptr(), nxt.data_ptr(),
       logits.data_ptr(), variant)
    torch.cuda.synchronize()
    ref = oracle.gemm_q8(a_eff, raw, N, mode)
    assert rel_rms(logits.cpu().numpy(), ref) < 5e-6
    assert np.array_equal(nxt.cpu().numpy(), oracle.argmax_rows(ref))
    # the kernel's argmax is the first maximum of its own logits
    assert np.array_equal(nxt.cpu().numpy(), oracle.argmax_rows(logits.cpu().numpy()))


@pytest.mark.parametrize("form", FORMS)
@pytest.mark.parametrize("variant", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("j1,j2", [(1000, 70000), (64 * 5 + 3, 64 * 5 + 40), (0, 151935), (64 * 7 + 31, 64 * 7 + 32)])
def test_lm_head_argmax_ties_pick_first(torch_cuda, j1, j2, variant, form):
    torch = torch_cuda
    M, N, K = 3, 151936, 1024
    nb = K // 32
    blocks = np.zeros((N, nb, 34), np.uint8)
    small = np.array([0.001], np.float16).view(np.uint8)
    blocks[:, :, 0:2] = small
    big = np.array([0.02], np.float16).view(np.uint8)
    for j in (j1, j2):
        blocks[j, :, 0:2] = big
        blocks[j, :, 2:] = np.uint8(127)
    raw = blocks.reshape(N, nb * 34)
    w, _ = _weights(torch, raw, N, K, form)
    a16 = oracle.f32_to_f16_bits(np.full((M, K), 0.5, np.float32))
    d_a = dev(torch, _i16(a16))
    scratch = torch.zeros(fa_dec.op_argmax_scratch_bytes(M, N), dtype=torch.uint8, device="cuda")
    nxt = torch.zeros(M, dtype=torch.int32, device="cuda")
    am = fa_dec.op_q8p_gemm_argmax if form == "q8p" else fa_dec.op_q8_gemm_argmax
    am(d_a.data_ptr(), 0, M, K, w.data_ptr(), N, scratch.data_ptr(), nxt.data_ptr(), 0, variant)
    torch.cuda.synchronize()
    assert nxt.cpu().numpy().tolist() == [j1] * M


# ------------------------------------------------------- failure detection --
def test_bounded_wait_gives_up_and_leaves_the_context_usable(torch_cuda):
    """An mbarrier wait that nothing completes gives up after its limit and reports a
    timeout in the kernel error word; the next kernel on the same context runs."""
    torch = torch_cuda
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    import time
    t0 = time.perf_counter()
    fa_dec.op_wait_selftest(20000, err.data_ptr())          # 20 ms
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert int(err.item()) & 1
    rng = np.random.default_rng(77)
    o32, _, ref = _attention_case(torch, rng, [40, 300], 8)
    assert_close(o32, ref, max_abs_tol=1e-4, rel_rms_tol=1e-5, what="attention after a timed-out wait")
