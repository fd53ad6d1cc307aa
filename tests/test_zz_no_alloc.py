"""GPU test of fa_op_paged_attention_noalloc, the attention entry point for callers
that cannot allocate device memory (a runtime that owns every allocation, a process
that forbids cudaMalloc after start-up). It keeps its split-K scratch in a buffer
built into the library instead of taking one from the caller.

Its output must match the allocating entry point, fa_op_paged_attention, on the same
inputs, on two calls in a row (the built-in buffer keeps the first call's contents
when the second one runs). This file is collected last so that a run which stops at
the first failure has already run every other test.
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
    d = [dev(torch, a) for a in (q, n_kv - 1, np.arange(M, dtype=np.int32), bt,
                                 np.ascontiguousarray(pool).view(np.int16))]
    return M, bt_stride, n_pages, d


def _run_both(torch, rng, n_kv, pps):
    M, bt_stride, n_pages, d = _inputs(torch, rng, n_kv)
    n_splits = int(math.ceil(math.ceil(max(n_kv) / 16) / pps))
    args = (d[0].data_ptr(), M, d[1].data_ptr(), d[2].data_ptr(), d[3].data_ptr(), bt_stride, n_pages,
            d[4].data_ptr(), pps, n_splits)
    ref = torch.zeros((M, 2048), dtype=torch.float32, device="cuda")
    scratch = torch.zeros(max(fa_dec.op_attention_scratch_bytes(M, n_splits), 16), dtype=torch.uint8, device="cuda")
    err = torch.zeros(2, dtype=torch.int32, device="cuda")
    fa_dec.op_paged_attention(*args, scratch.data_ptr(), out32=ref.data_ptr(), err=err[0:1].data_ptr())
    got = torch.zeros((M, 2048), dtype=torch.float32, device="cuda")
    fa_dec.op_paged_attention_noalloc(*args, out32=got.data_ptr(), err=err[1:2].data_ptr())
    torch.cuda.synchronize()
    assert err.cpu().numpy().tolist() == [0, 0]
    return got.cpu().numpy(), ref.cpu().numpy(), n_splits


def test_noalloc_attention_matches_allocating_entry_point_twice(torch_cuda):
    rng = np.random.default_rng(2718)
    got, ref, n_splits = _run_both(torch_cuda, rng, [2048] * 6 + [1, 17, 700, 1333], pps=16)
    assert n_splits > 1
    assert_close(got, ref, max_abs_tol=1e-4, rel_rms_tol=1e-5, what="first call")
    # second call: other rows, other split count, while the buffer still holds call one's partials
    got, ref, n_splits = _run_both(torch_cuda, rng, [300, 5, 4000, 64, 999], pps=8)
    assert n_splits > 1
    assert_close(got, ref, max_abs_tol=1e-4, rel_rms_tol=1e-5, what="second call")


def test_noalloc_attention_rejects_requests_beyond_its_buffer(torch_cuda):
    torch = torch_cuda
    t = torch.zeros(16, dtype=torch.int32, device="cuda")
    with pytest.raises(fa_dec.FaError) as e:
        # 1000 rows x 64 splits need ~532 MB of partials, far above the built-in 8 MiB
        fa_dec.op_paged_attention_noalloc(t.data_ptr(), 1000, t.data_ptr(), t.data_ptr(), t.data_ptr(), 1, 1,
                                          t.data_ptr(), 4, 64, out32=t.data_ptr())
    assert e.value.code == fa_dec.FA_ERR_CAPACITY
    assert "8388608" in str(e.value)
