"""GPU test of fa_op_paged_attention_noalloc, the attention entry point for callers
that cannot allocate device memory (a runtime that owns every allocation, a process
that forbids cudaMalloc after start-up). It keeps its split-K scratch in a buffer
built into the library instead of taking one from the caller.

Its output must match the allocating entry point, fa_op_paged_attention, and the
oracle on the same inputs, on two calls in a row (the built-in buffer keeps the first
call's contents when the second one runs); the one-split path (no scratch used), the
f16 pair outputs, the capacity boundary and a split choice that does not cover a row
are checked too. This file is collected last so that a run which stops at the first
failure has already run every other test.
"""
import math

import numpy as np
import pytest

import fa_dec
import oracle
from helpers import assert_close, dev

pytestmark = pytest.mark.gpu

PAGE_ELEMS = 8 * 2 * 16 * 128


def _inputs(torch, rng, n_kv, n_pages=1024):
    M = len(n_kv)
    n_kv = np.asarray(n_kv, np.int32)
    bt_stride = int(math.ceil(n_kv.max() / 16)) + 1
    bt = np.stack([rng.choice(n_pages, bt_stride, replace=False) for _ in range(M)]).astype(np.int32)
    pool = oracle.f32_to_f16_bits(rng.standard_normal((n_pages, PAGE_ELEMS)).astype(np.float32))
    q = (rng.standard_normal((M, 16, 128)) * 0.3).astype(np.float32)
    slot = np.arange(M, dtype=np.int32)
    d = [dev(torch, a) for a in (q, n_kv - 1, slot, bt, np.ascontiguousarray(pool).view(np.int16))]
    ref = oracle.paged_attention(q, slot, n_kv, bt, pool)
    return M, bt_stride, n_pages, d, ref


def _run_both(torch, rng, n_kv, pps, n_splits=None, pair=False):
    """Both entry points on the same inputs: (noalloc f32, allocating f32, oracle, n_splits,
    noalloc f16 pair summed in f32 or None)."""
    M, bt_stride, n_pages, d, ref_o = _inputs(torch, rng, n_kv)
    if n_splits is None:
        n_splits = int(math.ceil(math.ceil(max(n_kv) / 16) / pps))
    args = (d[0].data_ptr(), M, d[1].data_ptr(), d[2].data_ptr(), d[3].data_ptr(), bt_stride, n_pages,
            d[4].data_ptr(), pps, n_splits)
    ref = torch.zeros((M, 2048), dtype=torch.float32, device="cuda")
    scratch = torch.zeros(max(fa_dec.op_attention_scratch_bytes(M, n_splits), 16), dtype=torch.uint8, device="cuda")
    err = torch.zeros(2, dtype=torch.int32, device="cuda")
    fa_dec.op_paged_attention(*args, scratch.data_ptr(), out32=ref.data_ptr(), err=err[0:1].data_ptr())
    got = torch.zeros((M, 2048), dtype=torch.float32, device="cuda")
    hi = lo = None
    if pair:
        hi = torch.zeros((M, 2048), dtype=torch.float16, device="cuda")
        lo = torch.zeros((M, 2048), dtype=torch.float16, device="cuda")
    fa_dec.op_paged_attention_noalloc(*args, out32=got.data_ptr(), err=err[1:2].data_ptr(),
                                      out16=hi.data_ptr() if pair else 0, out16_lo=lo.data_ptr() if pair else 0)
    torch.cuda.synchronize()
    assert err.cpu().numpy().tolist() == [0, 0]
    pair_sum = (hi.float() + lo.float()).cpu().numpy() if pair else None
    return got.cpu().numpy(), ref.cpu().numpy(), ref_o, n_splits, pair_sum


def test_noalloc_attention_matches_allocating_entry_point_twice(torch_cuda):
    rng = np.random.default_rng(2718)
    got, ref, ref_o, n_splits, _ = _run_both(torch_cuda, rng, [2048] * 6 + [1, 17, 700, 1333], pps=16)
    assert n_splits > 1
    assert_close(got, ref, max_abs_tol=1e-4, rel_rms_tol=1e-5, what="first call vs allocating entry point")
    assert_close(got, ref_o, max_abs_tol=1e-4, rel_rms_tol=1e-5, what="first call vs oracle")
    # second call: other rows, other split count, while the buffer still holds call one's partials
    got, ref, ref_o, n_splits, _ = _run_both(torch_cuda, rng, [300, 5, 4000, 64, 999], pps=8)
    assert n_splits > 1
    assert_close(got, ref, max_abs_tol=1e-4, rel_rms_tol=1e-5, what="second call vs allocating entry point")
    assert_close(got, ref_o, max_abs_tol=1e-4, rel_rms_tol=1e-5, what="second call vs oracle")


def test_noalloc_attention_one_split_and_f16_pair(torch_cuda):
    rng = np.random.default_rng(31)
    # one split: the kernel stores the output itself and the built-in buffer is not touched
    got, ref, ref_o, n_splits, pair = _run_both(torch_cuda, rng, [5, 64, 300, 1], pps=32, n_splits=1, pair=True)
    assert n_splits == 1
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    assert_close(got, ref_o, max_abs_tol=1e-4, rel_rms_tol=1e-5, what="one split vs oracle")
    # hi + lo carries about 22 bits: within the f32 bar of the oracle
    assert_close(pair, ref_o, max_abs_tol=1e-4, rel_rms_tol=1e-5, what="one split f16 pair")
    got, ref, ref_o, n_splits, pair = _run_both(torch_cuda, rng, [1500, 33, 2048], pps=16, pair=True)
    assert n_splits > 1
    assert_close(pair, ref_o, max_abs_tol=1e-4, rel_rms_tol=1e-5, what="split f16 pair")


def test_noalloc_attention_capacity_boundary(torch_cuda):
    """M * n_splits = 1008 fits the 8 MiB buffer exactly; 1009 does not."""
    torch = torch_cuda
    rng = np.random.default_rng(5)
    n_kv = [16 * 63] * 16                         # 63 pages per row, one page per split
    got, ref, ref_o, n_splits, _ = _run_both(torch, rng, n_kv, pps=1, n_splits=63)
    assert len(n_kv) * n_splits == 1008
    assert_close(got, ref_o, max_abs_tol=1e-4, rel_rms_tol=1e-5, what="1008 row-splits")
    t = torch.zeros(16, dtype=torch.int32, device="cuda")
    with pytest.raises(fa_dec.FaError) as e:
        fa_dec.op_paged_attention_noalloc(t.data_ptr(), 1, t.data_ptr(), t.data_ptr(), t.data_ptr(), 1, 1,
                                          t.data_ptr(), 1, 1009, out32=t.data_ptr())
    assert e.value.code == fa_dec.FA_ERR_CAPACITY
    with pytest.raises(fa_dec.FaError) as e:
        # 1000 rows x 64 splits need ~532 MB of partials, far above the built-in 8 MiB
        fa_dec.op_paged_attention_noalloc(t.data_ptr(), 1000, t.data_ptr(), t.data_ptr(), t.data_ptr(), 1, 1,
                                          t.data_ptr(), 4, 64, out32=t.data_ptr())
    assert e.value.code == fa_dec.FA_ERR_CAPACITY
    assert "8388608" in str(e.value)


def test_noalloc_attention_flags_rows_the_splits_do_not_cover(torch_cuda):
    """pages_per_split * n_splits below a row's page count: error bit 8, row left as it was."""
    torch = torch_cuda
    rng = np.random.default_rng(9)
    M, bt_stride, n_pages, d, ref_o = _inputs(torch, rng, [40 * 16, 16])
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.full((M, 2048), 7.0, dtype=torch.float32, device="cuda")
    fa_dec.op_paged_attention_noalloc(d[0].data_ptr(), M, d[1].data_ptr(), d[2].data_ptr(), d[3].data_ptr(),
                                      bt_stride, n_pages, d[4].data_ptr(), 8, 2, out32=out.data_ptr(),
                                      err=err.data_ptr())
    torch.cuda.synchronize()
    assert int(err.item()) & 8
    got = out.cpu().numpy()
    assert (got[0] == 7.0).all()                  # 40 pages, 16 covered: not written
    assert_close(got[1:], ref_o[1:], max_abs_tol=1e-4, rel_rms_tol=1e-5, what="covered row")
