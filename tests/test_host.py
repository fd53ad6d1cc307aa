"""CPU tests of the C-ABI library: it loads, exports the header's symbols, rejects bad
descriptors, refuses to run without a GPU, and its page allocator follows the
restated policy of the oracle (lowest free page first; compaction moves)."""
import ctypes

import numpy as np
import pytest

import fa_dec
import oracle


def test_library_exports_every_declared_symbol():
    L = fa_dec.lib()
    names = fa_dec.header_functions()
    assert len(names) >= 35
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert b"sm_100a" in L.fa_version()


def test_desc_struct_layout_matches_header():
    # fa_model_desc: 10 ints/floats, one size_t (8-aligned), 2 ints
    assert ctypes.sizeof(fa_dec._Desc) == 64
    assert ctypes.sizeof(fa_dec._TensorView) == 48


@pytest.mark.parametrize("field,value", [("head_dim", 64), ("n_kv_heads", 4), ("hidden", 1000), ("max_rows", 0)])
def test_bad_descriptor_is_rejected_before_touching_the_gpu(field, value):
    d = fa_dec.default_desc(**{field: value})
    ctx = fa_dec.lib().fa_create(0, ctypes.byref(d))
    assert not ctx
    assert fa_dec.last_error(None)


def test_no_cpu_fallback_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible; covered by the GPU tests")
    with pytest.raises(fa_dec.FaError) as e:
        fa_dec.Decoder(0)
    assert "CUDA" in str(e.value) or "device" in str(e.value)


def test_op_entry_points_validate_arguments():
    with pytest.raises(fa_dec.FaError):
        fa_dec.op_q8_gemm(0, 0, 4, 100, 0, 0, 64, 1, 0, 0)
    assert fa_dec.op_attention_scratch_bytes(128, 1) == 0
    assert fa_dec.op_attention_scratch_bytes(128, 4) == 128 * 16 * 4 * 130 * 4


@pytest.mark.parametrize("call", [
    # gather: null pool, non-positive sizes, block-table stride below max_pages
    lambda: fa_dec.op_kv_gather(0, 28, 16, 8, 4, 8, 8, 8, 1, 4, 64, 8, 8),
    lambda: fa_dec.op_kv_gather(16, 28, 16, 8, 4, 8, 8, 8, 0, 4, 64, 16, 16),
    lambda: fa_dec.op_kv_gather(16, 28, 16, 8, 2, 8, 8, 8, 1, 4, 64, 16, 16),
    # gather: a pool or slab address that is not 16-byte aligned
    lambda: fa_dec.op_kv_gather(24, 28, 16, 8, 4, 8, 8, 8, 1, 4, 64, 16, 16),
    # split-K partials of the paged attention need a 16-byte aligned scratch
    lambda: fa_dec.op_paged_attention(16, 1, 16, 16, 16, 4, 16, 16, 4, 2, 24, out16=16),
    # a GEMM variant outside 0..4, and the plan of one
    lambda: fa_dec.op_gemm_plan(16, 1024, 1024, variant=5),
    # the fused SwiGLU GEMM and the SwiGLU kernel reject missing buffers before touching a GPU
    lambda: fa_dec.op_q8_gemm_swiglu(0, 0, 1, 1024, 16, 2048, 16, 16),
    lambda: fa_dec.op_swiglu(0, 1, 1, 1024, 16, 16),
])
def test_new_op_entry_points_reject_bad_arguments(call):
    with pytest.raises(fa_dec.FaError) as e:
        call()
    assert "INVALID_ARG" in str(e.value)


def test_allocator_matches_oracle_policy():
    rng = np.random.default_rng(0)
    n = 300
    mine = fa_dec.PageAllocator(n)
    ref = oracle.PageAllocatorOracle(n)
    live = []
    for step in range(5000):
        if live and (rng.random() < 0.45 or len(live) == n):
            p = live.pop(int(rng.integers(len(live))))
            mine.free(p)
            ref.free(p)
        else:
            a, b = mine.alloc(), ref.alloc()
            assert a == b, step
            live.append(a)
        assert mine.n_free() == ref.n_free()
    with pytest.raises(fa_dec.FaError):
        mine.free(live[0]) if False else mine.free(n + 5)


def test_allocator_exhaustion_and_double_free():
    a = fa_dec.PageAllocator(3)
    assert [a.alloc(), a.alloc(), a.alloc()] == [0, 1, 2]
    with pytest.raises(fa_dec.FaError) as e:
        a.alloc()
    assert e.value.code == fa_dec.FA_ERR_POOL_EXHAUSTED
    a.free(1)
    with pytest.raises(fa_dec.FaError):
        a.free(1)


def test_compaction_matches_oracle_plan():
    rng = np.random.default_rng(1)
    for trial in range(20):
        n = int(rng.integers(5, 200))
        mine = fa_dec.PageAllocator(n)
        pages = [mine.alloc() for _ in range(n)]
        freed = rng.choice(n, size=int(rng.integers(0, n)), replace=False)
        for p in freed:
            mine.free(int(p))
        live = sorted(set(pages) - set(int(p) for p in freed))
        src, dst = mine.compact_moves()
        assert (src, dst) == oracle.compaction_plan(live, n)
        after = sorted((set(live) - set(src)) | set(dst))
        assert after == list(range(len(live)))
        # the allocator now hands out exactly the tail
        assert mine.n_free() == n - len(live)
        if len(live) < n:
            assert mine.alloc() == len(live)


def test_gemm_planner_choices():
    """The split-K factors the decoder plans (host only): one row block per small-M step,
    the swapped-operand kernel's splits for the decode shapes, and large-M GEMMs kept
    whole once the epilogue is counted."""
    shapes = {"qkv": (4096, 1024), "o": (1024, 2048), "gu": (6144, 1024), "dn": (1024, 3072)}
    plan = lambda M, nm, v=0: fa_dec.op_gemm_plan(M, *shapes[nm], variant=v)
    # 1-2 rows: the CUDA-core kernel, no split
    assert [plan(1, nm) for nm in shapes] == [1, 1, 1, 1]
    assert [plan(2, nm) for nm in shapes] == [1, 1, 1, 1]
    # 128 rows: the decode step's splits (one unit per SM, 96 for gate/up)
    assert [plan(128, nm) for nm in shapes] == [4, 16, 2, 16]
    assert [plan(16, nm) for nm in shapes] == [4, 16, 2, 16]
    # 2048 and 4096 rows: whole K per unit
    assert [plan(2048, nm) for nm in shapes] == [1, 1, 1, 1]
    assert [plan(4096, nm) for nm in shapes] == [1, 1, 1, 1]
    # the small-M kernel alone (variant 3) also needs no split; mma.sync plans its own
    assert plan(8, "qkv", 3) == 1
    assert plan(128, "qkv", 1) >= 1


def test_attention_planner_choices():
    """Pages per CTA and splits of the decode attention: 128 rows at 2048 tokens split in
    three (seven waves of 3 CTAs per SM); a short single row is not split (a merge launch
    costs more than the pages it saves)."""
    pps, ns = fa_dec.op_attention_plan(np.full(128, 2048, np.int32))
    assert (pps, ns) == (44, 3)
    assert fa_dec.op_attention_plan(np.array([112], np.int32))[1] == 1
    pps, ns = fa_dec.op_attention_plan(np.array([4096], np.int32))
    assert ns > 1 and pps * ns >= 4096 // 16


def test_step_attention_plan_fuses_only_in_one_wave():
    """What the decode attention kernel finishes itself (host only): the split merge (bit 2 of
    the fused-op mask) and kernel (1) (bit 3) only when its CTAs fit in one wave. 128 rows at
    2048 tokens (3 splits x 8 KV heads x 128 rows = 3,072 CTAs, seven waves) keep both as
    launches; 16 rows at 1025 tokens (384 CTAs of 4 warps, 3 per SM on 148 SMs), 2 rows at
    257 and one row at 113 (8 warps, one CTA per SM) fuse; mask 6 leaves kernel (1) a launch."""
    plan = lambda M, n_kv, mask=14: fa_dec.step_attention_plan(np.full(M, n_kv, np.int32), mask=mask)
    p = plan(128, 2048)
    assert (p["pages_per_split"], p["n_splits"], p["warps"]) == (44, 3, 4)
    assert not p["merge"] and not p["append"]
    assert not plan(64, 2048)["append"]
    p = plan(16, 1025)
    assert p["n_splits"] == 3 and p["warps"] == 4 and p["merge"] and p["append"]
    p = plan(2, 257)
    assert p["merge"] and p["append"]
    p = plan(1, 113)
    assert (p["n_splits"], p["warps"]) == (1, 8) and not p["merge"] and p["append"]
    p = plan(16, 1025, mask=6)
    assert p["merge"] and not p["append"]
    assert not any(plan(16, 1025, mask=0)[k] for k in ("merge", "append"))
    for bad in (lambda: plan(4, 100, mask=16), lambda: plan(4, 0)):
        with pytest.raises(fa_dec.FaError):
            bad()

