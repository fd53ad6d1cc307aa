"""ctypes binding of libfunasr_dec.so (include/funasr_dec.h).

The library is the product: every call here goes to the CUDA path, and a
failure raises FaError; there is no CPU fallback. `Decoder` mirrors the
reference's GPUContext / GPURunner / KVCache roles (compute/gpu_context.hpp,
compute/gpu_runner.hpp, compute/kv_cache.hpp) over one fa_ctx.
"""
from __future__ import annotations

import ctypes
import os
import re
from typing import Dict, Optional, Sequence, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "libfunasr_dec.so")
HEADER = os.path.join(ROOT, "include", "funasr_dec.h")

FA_OK = 0
ERRORS = {
    -1: "INVALID_ARG", -2: "CUDA", -3: "OOM", -4: "POOL_EXHAUSTED", -5: "SEQ", -6: "CAPACITY",
    -7: "WEIGHTS", -8: "TIMEOUT", -9: "NOT_READY", -10: "DEVICE",
}
FA_ERR_INVALID_ARG = -1
FA_ERR_CUDA = -2
FA_ERR_POOL_EXHAUSTED = -4
FA_ERR_SEQ = -5
FA_ERR_CAPACITY = -6
FA_ERR_WEIGHTS = -7

TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_BF16 = 0, 1, 8, 30
PAGE_TOKENS = 16


class FaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class _Desc(ctypes.Structure):
    _fields_ = [
        ("n_layers", ctypes.c_int), ("hidden", ctypes.c_int), ("n_heads", ctypes.c_int),
        ("n_kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("ffn", ctypes.c_int),
        ("vocab", ctypes.c_int), ("rope_base", ctypes.c_float), ("rms_eps", ctypes.c_float),
        ("max_ctx", ctypes.c_int), ("n_pages", ctypes.c_int), ("kv_bytes", ctypes.c_size_t),
        ("max_seqs", ctypes.c_int), ("max_rows", ctypes.c_int),
    ]


class _TensorView(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("type", ctypes.c_int), ("ne", ctypes.c_int64 * 2),
                ("data", ctypes.c_void_p), ("nbytes", ctypes.c_size_t)]


class _EncoderDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in (
        "input_dim", "output_size", "attention_heads", "linear_units", "num_blocks", "tp_blocks", "kernel_size",
        "sanm_shift", "adaptor_hidden", "adaptor_output", "adaptor_blocks", "adaptor_heads", "adaptor_ffn",
        "max_frames")]


class _SchedConfig(ctypes.Structure):
    _fields_ = [("max_batch_rows", ctypes.c_int), ("prefill_chunk", ctypes.c_int), ("max_running", ctypes.c_int),
                ("eos_id", ctypes.c_int)]


class _SchedEvent(ctypes.Structure):
    _fields_ = [("tag", ctypes.c_int64), ("token", ctypes.c_int), ("finished", ctypes.c_int)]


class _SchedStats(ctypes.Structure):
    _fields_ = [("steps", ctypes.c_long), ("rows", ctypes.c_long), ("prompt_rows", ctypes.c_long),
                ("tokens", ctypes.c_long), ("finished", ctypes.c_long), ("waiting", ctypes.c_int),
                ("running", ctypes.c_int), ("reserved_pages", ctypes.c_long), ("total_pages", ctypes.c_long)]


_lib = None
_P = ctypes.c_void_p
_I = ctypes.c_int


def header_functions() -> list:
    """Names of every function the C header declares."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(fa_[a-z0-9_]+)\s*\(", text)))


def lib():
    """Load the library (build it first with funasr-ggml_b200/build.py)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise FaError(-2, f"{LIB_PATH} is missing; run `python funasr-ggml_b200/build.py`")
    L = ctypes.CDLL(LIB_PATH)
    sig = {
        "fa_version": ([], ctypes.c_char_p),
        "fa_last_error": ([_P], ctypes.c_char_p),
        "fa_default_desc": ([ctypes.POINTER(_Desc)], None),
        "fa_create": ([_I, ctypes.POINTER(_Desc)], _P),
        "fa_destroy": ([_P], None),
        "fa_load_weights": ([_P, ctypes.POINTER(_TensorView), _I], _I),
        "fa_set_stream": ([_P, _P], _I),
        "fa_set_graphs": ([_P, _I], _I),
        "fa_set_gemm_variant": ([_P, _I], _I),
        "fa_set_fused_epilogues": ([_P, _I], _I),
        "fa_set_pdl": ([_P, _I], _I),
        "fa_set_row_step": ([_P, _I], _I),
        "fa_profile_row_step": ([_P, _P], _I),
        "fa_set_row_step_fault": ([_P, _I, _I], _I),
        "fa_pool_info": ([_P, _P, _P, _P], _I),
        "fa_seq_open": ([_P, _I, _P], _I),
        "fa_seq_close": ([_P, _I], _I),
        "fa_seq_length": ([_P, _I, _P], _I),
        "fa_seq_truncate": ([_P, _I, _I], _I),
        "fa_seq_block_table": ([_P, _I, _P, _I, _P], _I),
        "fa_forward_rows": ([_P, _I, _P, _P, _P, _I, _P, _P, _P], _I),
        "fa_ctx_desc": ([_P, _P], _I),
        "fa_encoder_default_desc": ([_P], None),
        "fa_encoder_create": ([_I, _P], _P),
        "fa_encoder_destroy": ([_P], None),
        "fa_encoder_load_weights": ([_P, _P, _I], _I),
        "fa_encoder_forward": ([_P, _P, _I, _P], _I),
        "fa_encoder_forward_dev": ([_P, _P, _I, _P, _P], _I),
        "fa_encoder_forward_batch": ([_P, _I, _P, _P, _P, _P], _I),
        "fa_encoder_set_graphs": ([_P, _I], _I),
        "fa_sched_create": ([_P, _P], _P),
        "fa_sched_destroy": ([_P], None),
        "fa_sched_submit": ([_P, ctypes.c_int64, _P, _P, _I, _I], _I),
        "fa_sched_step": ([_P, _P, _I, _P], _I),
        "fa_sched_idle": ([_P], _I),
        "fa_sched_get_stats": ([_P, _P], _I),
        "fa_forward": ([_P, _I, _P, _P, _P, _P, _P], _I),
        "fa_prefill": ([_P, _I, _P, _I, _P, _P], _I),
        "fa_decode_step": ([_P, _I, _P, _P, _P, _P], _I),
        "fa_generate": ([_P, _I, _P, _P, _I, _P, _P], _I),
        "fa_kv_read_pages": ([_P, _I, _P, _I, _P], _I),
        "fa_kv_append": ([_P, _I, _P, _P, _P], _I),
        "fa_kv_fill_synthetic": ([_P, _I, _I, ctypes.c_uint64], _I),
        "fa_pool_compact": ([_P, _P], _I),
        "fa_profile": ([_P, _I], _I),
        "fa_profile_attention": ([_P, _P, _P], _I),
        "fa_step_launches": ([_P, _P], _I),
        "fa_op_qknorm_rope_append": ([_P, _I, _P, _P, _P, _I, _I, _P, _P, ctypes.c_float, _P, _I, _P, _P, _P, _P], _I),
        "fa_op_kv_append": ([_P, _P, _I, _I, _P, _P, _P, _I, _I, _P, _P, _P], _I),
        "fa_op_kv_gather": ([_P, _I, _I, _P, _I, _P, _P, _P, _I, _I, _I, _P, _P, _P, _P], _I),
        "fa_op_attention_scratch_bytes": ([_I, _I], ctypes.c_size_t),
        "fa_op_paged_attention": ([_P, _I, _P, _P, _P, _I, _I, _P, _I, _I, _P, _P, _P, _P, _P, _P], _I),
        "fa_gguf_read_desc": ([ctypes.c_char_p, _P], _I),
        "fa_load_gguf": ([_P, ctypes.c_char_p], _I),
        "fa_gguf_find_tensor": ([ctypes.c_char_p, ctypes.c_char_p, _P, _P, _P, _P], _I),
        "fa_op_attention_plan": ([_P, _I, _I, _P, _P], _I),
        "fa_step_attention_plan": ([_P, _I, _I, _I, _P, _P, _P, _P], _I),
        "fa_op_gemm_plan": ([_I, _I, _I, _I, _I, _P], _I),
        "fa_op_wait_selftest": ([_I, _P, _P], _I),
        "fa_op_prefill_attention": ([_P, _I, _P, _P, _P, _I, _I, _P, _P, _I, _P, _P, _P, _P, _P], _I),
        "fa_op_paged_attention_noalloc": ([_P, _I, _P, _P, _P, _I, _I, _P, _I, _I, _P, _P, _P, _P, _P], _I),
        "fa_op_repack_q8": ([_P, _I, _I, _P, _P], _I),
        "fa_op_q8_gemm": ([_P, _P, _I, _I, _P, _I, _I, _P, _I, _P], _I),
        "fa_op_argmax_scratch_bytes": ([_I, _I], ctypes.c_size_t),
        "fa_op_q8_gemm_argmax": ([_P, _P, _I, _I, _P, _I, _P, _P, _P, _I, _P], _I),
        "fa_op_q8_gemm_swiglu": ([_P, _P, _I, _I, _P, _I, _P, _P, _P], _I),
        "fa_op_swiglu": ([_P, _I, _I, _I, _P, _P, _P], _I),
        "fa_op_q8_planes_bytes": ([_I, _I], ctypes.c_size_t),
        "fa_op_repack_q8_planes": ([_P, _I, _I, _P, _P], _I),
        "fa_op_q8p_gemm": ([_P, _P, _I, _I, _P, _I, _I, _P, _I, _P], _I),
        "fa_op_q8p_gemm_argmax": ([_P, _P, _I, _I, _P, _I, _P, _P, _P, _I, _P], _I),
        "fa_op_q8p_gemm_swiglu": ([_P, _P, _I, _I, _P, _I, _P, _P, _P], _I),
        "fa_palloc_create": ([_I], _P),
        "fa_palloc_destroy": ([_P], None),
        "fa_palloc_alloc": ([_P], _I),
        "fa_palloc_free": ([_P, _I], _I),
        "fa_palloc_n_free": ([_P], _I),
        "fa_palloc_compact": ([_P, _P, _P, _I, _P], _I),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    _lib = L
    return L


def last_error(ctx=None) -> str:
    s = lib().fa_last_error(ctx)
    return s.decode() if s else ""


def _check(rc: int, ctx=None) -> int:
    if rc < 0:
        raise FaError(rc, last_error(ctx))
    return rc


def _p(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def default_desc(**over) -> _Desc:
    d = _Desc()
    lib().fa_default_desc(ctypes.byref(d))
    for k, v in over.items():
        setattr(d, k, v)
    return d


def gguf_desc(path: str, **over) -> _Desc:
    """Geometry of the decoder in a GGUF model file (fa_gguf_read_desc) plus runtime sizes."""
    d = default_desc()
    _check(lib().fa_gguf_read_desc(os.fsencode(path), ctypes.byref(d)))
    for k, v in over.items():
        setattr(d, k, v)
    return d


def gguf_find_tensor(path: str, name: str):
    """(ggml type, (ne0, rows), file offset, bytes) of one tensor of a GGUF file."""
    t = ctypes.c_int()
    ne = (ctypes.c_int64 * 2)()
    off, nb = ctypes.c_size_t(), ctypes.c_size_t()
    _check(lib().fa_gguf_find_tensor(os.fsencode(path), name.encode(), ctypes.byref(t), ne, ctypes.byref(off),
                                     ctypes.byref(nb)))
    return t.value, (ne[0], ne[1]), off.value, nb.value


# ------------------------------------------------------------------ Decoder --
class Decoder:
    """One fa_ctx on one GPU: weights, the paged KV pool, sequences and steps."""

    def __init__(self, device: int = 0, **desc):
        self.desc = default_desc(**desc)
        self.ctx = lib().fa_create(device, ctypes.byref(self.desc))
        if not self.ctx:
            raise FaError(-2, last_error(None))
        self.hidden = self.desc.hidden
        self.vocab = self.desc.vocab
        self.n_layers = self.desc.n_layers

    def close(self):
        if getattr(self, "ctx", None):
            lib().fa_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _c(self, rc):
        return _check(rc, self.ctx)

    # weights ----------------------------------------------------------------
    def load_weights(self, weights: Dict[str, Tuple[int, Sequence[int], np.ndarray]]):
        views = (_TensorView * len(weights))()
        keep = []
        for i, (name, (t, ne, arr)) in enumerate(weights.items()):
            arr = np.ascontiguousarray(arr)
            keep.append(arr)
            nb = name.encode()
            keep.append(nb)
            views[i].name = nb
            views[i].type = t
            views[i].ne[0] = int(ne[0])
            views[i].ne[1] = int(ne[1]) if len(ne) > 1 else 1
            views[i].data = arr.ctypes.data
            views[i].nbytes = arr.nbytes
        self._c(lib().fa_load_weights(self.ctx, views, len(weights)))

    def load_gguf(self, path: str):
        """Load the decoder tensors (llm.*) of a GGUF model file."""
        self._c(lib().fa_load_gguf(self.ctx, os.fsencode(path)))

    def set_stream(self, stream_ptr: Optional[int]):
        self._c(lib().fa_set_stream(self.ctx, stream_ptr))

    def set_gemm_variant(self, variant: int):
        """0 (default): small-M CUDA-core GEMM up to 2 rows, the swapped tcgen05 GEMM above (in
        128-row activation tiles); 1: mma.sync GEMM (cross-check); 2: 128-row-tile tcgen05 at
        every M; 3: small-M kernel up to 8 rows; 4: swapped tcgen05 at every M."""
        self._c(lib().fa_set_gemm_variant(self.ctx, int(variant)))

    def set_fused_epilogues(self, mask: int):
        """Mask of ops finished inside the kernel before them: 1 = QKV GEMM with per-head
        norm/RoPE/append, 2 = gate/up GEMM with SwiGLU, 4 = decode attention merging its
        splits itself when its CTAs fit in one wave, 8 = decode attention running the per-head
        norm/RoPE/append itself in one-wave steps of distinct sequences (default 14); 0 = separate
        kernels. Same bits either way."""
        self._c(lib().fa_set_fused_epilogues(self.ctx, int(mask)))

    def set_row_step(self, enable: bool):
        """One-row decode steps as one persistent kernel (default on; same bits as launch by
        launch)."""
        self._c(lib().fa_set_row_step(self.ctx, int(enable)))

    def set_row_step_fault(self, absent_cta: int, wait_us: int = 0):
        """Failure test: CTA absent_cta of the one-row step kernel never reaches its barriers,
        so the step gives up after wait_us and returns FA_ERR_TIMEOUT (-1: off)."""
        self._c(lib().fa_set_row_step_fault(self.ctx, int(absent_cta), int(wait_us)))

    def set_pdl(self, enable: bool):
        self._c(lib().fa_set_pdl(self.ctx, int(enable)))

    def set_graphs(self, enable: bool):
        self._c(lib().fa_set_graphs(self.ctx, int(enable)))

    def pool_info(self):
        n = ctypes.c_int(); f = ctypes.c_int(); b = ctypes.c_size_t()
        self._c(lib().fa_pool_info(self.ctx, ctypes.byref(n), ctypes.byref(f), ctypes.byref(b)))
        return n.value, f.value, b.value

    # sequences --------------------------------------------------------------
    def seq_open(self, max_tokens: int) -> int:
        sid = ctypes.c_int()
        self._c(lib().fa_seq_open(self.ctx, int(max_tokens), ctypes.byref(sid)))
        return sid.value

    def seq_close(self, sid: int):
        self._c(lib().fa_seq_close(self.ctx, int(sid)))

    def seq_length(self, sid: int) -> int:
        n = ctypes.c_int()
        self._c(lib().fa_seq_length(self.ctx, int(sid), ctypes.byref(n)))
        return n.value

    def seq_truncate(self, sid: int, n: int):
        self._c(lib().fa_seq_truncate(self.ctx, int(sid), int(n)))

    def block_table(self, sid: int) -> np.ndarray:
        n = ctypes.c_int()
        self._c(lib().fa_seq_block_table(self.ctx, int(sid), None, 0, ctypes.byref(n)))
        out = np.zeros(n.value, np.int32)
        self._c(lib().fa_seq_block_table(self.ctx, int(sid), _p(out), n.value, ctypes.byref(n)))
        return out

    # steps ------------------------------------------------------------------
    def forward(self, seq_ids, tokens=None, embeds=None, want_logits=False):
        sids = _i32(seq_ids)
        M = len(sids)
        tok = None if tokens is None else _i32(tokens)
        emb = None if embeds is None else np.ascontiguousarray(embeds, np.float32)
        nxt = np.zeros(M, np.int32)
        lg = np.zeros((M, self.vocab), np.float32) if want_logits else None
        self._c(lib().fa_forward(self.ctx, M, _p(sids), _p(tok), _p(emb), _p(nxt), _p(lg)))
        return nxt, lg

    def forward_rows(self, seq_ids, out_rows, tokens=None, embeds=None, want_logits=False):
        """forward() returning next ids (and logits) of the rows in out_rows only."""
        sids = _i32(seq_ids)
        M = len(sids)
        rows = _i32(out_rows)
        tok = None if tokens is None else _i32(tokens)
        emb = None if embeds is None else np.ascontiguousarray(embeds, np.float32)
        nxt = np.zeros(max(len(rows), 1), np.int32)
        lg = np.zeros((max(len(rows), 1), self.vocab), np.float32) if want_logits else None
        self._c(lib().fa_forward_rows(self.ctx, M, _p(sids), _p(tok), _p(emb), len(rows), _p(rows) if len(rows) else None,
                                      _p(nxt), _p(lg)))
        return nxt[:len(rows)], (lg[:len(rows)] if want_logits else None)

    def decode_step(self, seq_ids, tokens, want_logits=False):
        sids = _i32(seq_ids)
        tok = _i32(tokens)
        nxt = np.zeros(len(sids), np.int32)
        lg = np.zeros((len(sids), self.vocab), np.float32) if want_logits else None
        self._c(lib().fa_decode_step(self.ctx, len(sids), _p(sids), _p(tok), _p(nxt), _p(lg)))
        return nxt, lg

    def prefill(self, sid: int, embeds: np.ndarray, want_logits=False):
        emb = np.ascontiguousarray(embeds, np.float32)
        nxt = ctypes.c_int()
        lg = np.zeros(self.vocab, np.float32) if want_logits else None
        self._c(lib().fa_prefill(self.ctx, int(sid), _p(emb), emb.shape[0], ctypes.byref(nxt), _p(lg)))
        return nxt.value, lg

    def generate(self, seq_ids, first_tokens, n_steps: int):
        sids = _i32(seq_ids)
        tok = _i32(first_tokens)
        out = np.zeros((n_steps, len(sids)), np.int32)
        ms = ctypes.c_float()
        self._c(lib().fa_generate(self.ctx, len(sids), _p(sids), _p(tok), int(n_steps), _p(out), ctypes.byref(ms)))
        return out, ms.value

    # pages ------------------------------------------------------------------
    def kv_read_pages(self, layer: int, pages) -> np.ndarray:
        pg = _i32(pages)
        out = np.zeros((len(pg), 8 * 2 * PAGE_TOKENS * 128), np.uint16)
        self._c(lib().fa_kv_read_pages(self.ctx, int(layer), _p(pg), len(pg), _p(out)))
        return out

    def kv_append(self, seq_ids, k16: np.ndarray, v16: np.ndarray):
        sids = _i32(seq_ids)
        k16 = np.ascontiguousarray(k16, np.uint16)
        v16 = np.ascontiguousarray(v16, np.uint16)
        self._c(lib().fa_kv_append(self.ctx, len(sids), _p(sids), _p(k16), _p(v16)))

    def kv_fill_synthetic(self, sid: int, n_tokens: int, seed: int = 0):
        self._c(lib().fa_kv_fill_synthetic(self.ctx, int(sid), int(n_tokens), ctypes.c_uint64(seed)))

    def pool_compact(self) -> int:
        n = ctypes.c_int()
        self._c(lib().fa_pool_compact(self.ctx, ctypes.byref(n)))
        return n.value

    # measurement --------------------------------------------------------------
    def profile(self, enable: bool):
        self._c(lib().fa_profile(self.ctx, int(enable)))

    def profile_attention(self):
        ms = ctypes.c_float(); n = ctypes.c_int()
        self._c(lib().fa_profile_attention(self.ctx, ctypes.byref(ms), ctypes.byref(n)))
        return ms.value, n.value

    def profile_row_step(self) -> float:
        """Device ms of the persistent one-row step kernel in the last profiled step (0 if
        the step ran launch by launch)."""
        ms = ctypes.c_float()
        self._c(lib().fa_profile_row_step(self.ctx, ctypes.byref(ms)))
        return ms.value

    def step_launches(self) -> int:
        n = ctypes.c_int()
        self._c(lib().fa_step_launches(self.ctx, ctypes.byref(n)))
        return n.value


# ------------------------------------------------------- kernel-level ops --
def op_qknorm_rope_append(qkv, M, pos, slot, bt, bt_stride, n_pages, qn, kn, eps, rope, max_pos, pool, q_out,
                          err=0, stream=0):
    _check(lib().fa_op_qknorm_rope_append(qkv, M, pos, slot, bt, bt_stride, n_pages, qn, kn, eps, rope, max_pos,
                                          pool, q_out, err or None, stream or None))


def op_kv_append(k, v, M, n_layers, pos, slot, bt, bt_stride, n_pages, pool, err=0, stream=0):
    _check(lib().fa_op_kv_append(k, v, M, n_layers, pos, slot, bt, bt_stride, n_pages, pool, err or None,
                                 stream or None))


def op_kv_gather(pool, n_layers, n_pages, bt, bt_stride, slot, n_kv, row0, M, max_pages, total_rows, k_out, v_out,
                 err=0, stream=0):
    """Head-major K/V slabs [n_layers][8][total_rows][128] of the tokens [0, n_kv[m]) of
    sequences slot[m] (device pointers throughout)."""
    _check(lib().fa_op_kv_gather(pool, n_layers, n_pages, bt, bt_stride, slot, n_kv, row0, M, max_pages, total_rows,
                                 k_out, v_out, err or None, stream or None))


def op_attention_scratch_bytes(M, n_splits) -> int:
    return int(lib().fa_op_attention_scratch_bytes(M, n_splits))


def op_paged_attention(q, M, pos, slot, bt, bt_stride, n_pages, pool, pps, n_splits, scratch, out16=0, out32=0,
                       err=0, stream=0, out16_lo=0):
    _check(lib().fa_op_paged_attention(q, M, pos, slot, bt, bt_stride, n_pages, pool, pps, n_splits,
                                       scratch or None, out16 or None, out16_lo or None, out32 or None, err or None,
                                       stream or None))


def op_attention_plan(n_kv, n_sm=148):
    """(pages_per_split, n_splits) the decoder picks for rows with contexts n_kv."""
    a = np.ascontiguousarray(n_kv, np.int32)
    pps, ns = ctypes.c_int(), ctypes.c_int()
    _check(lib().fa_op_attention_plan(a.ctypes.data, len(a), n_sm, ctypes.byref(pps), ctypes.byref(ns)))
    return pps.value, ns.value


def step_attention_plan(n_kv, n_sm=148, mask=14):
    """The decoder's attention plan for a step of decode rows with contexts n_kv under fused
    mask `mask`: dict of pages_per_split, n_splits, warps, merge (the attention kernel merges
    its splits) and append (it runs kernel (1) for rows of distinct sequences)."""
    a = np.ascontiguousarray(n_kv, np.int32)
    pps, ns, w, f = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    _check(lib().fa_step_attention_plan(a.ctypes.data, len(a), n_sm, int(mask), ctypes.byref(pps),
                                        ctypes.byref(ns), ctypes.byref(w), ctypes.byref(f)))
    return dict(pages_per_split=pps.value, n_splits=ns.value, warps=w.value, merge=bool(f.value & 1),
                append=bool(f.value & 2))


def op_prefill_attention(q, M, pos, slot, bt, bt_stride, n_pages, pool, tiles, n_tiles, out16=0, out32=0, err=0,
                         stream=0, out16_lo=0):
    """Kernel (2b): causal tensor-core attention over prefill tiles (first row, rows)."""
    _check(lib().fa_op_prefill_attention(q, M, pos, slot, bt, bt_stride, n_pages, pool, tiles, n_tiles,
                                         out16 or None, out16_lo or None, out32 or None, err or None,
                                         stream or None))


def op_wait_selftest(limit_us, err, stream=0):
    """A bounded mbarrier wait that must run out (nothing completes the barrier)."""
    _check(lib().fa_op_wait_selftest(int(limit_us), err, stream or None))


def op_gemm_plan(M, N, K, variant=0, n_sm=148):
    """Split-K factor the decoder picks for an M x N x K GEMM."""
    s = ctypes.c_int()
    _check(lib().fa_op_gemm_plan(M, N, K, variant, n_sm, ctypes.byref(s)))
    return s.value


def op_paged_attention_noalloc(q, M, pos, slot, bt, bt_stride, n_pages, pool, pps, n_splits, out16=0, out32=0,
                               err=0, stream=0, out16_lo=0):
    """fa_op_paged_attention with the library's built-in scratch buffer (allocates nothing)."""
    _check(lib().fa_op_paged_attention_noalloc(q, M, pos, slot, bt, bt_stride, n_pages, pool, pps, n_splits,
                                               out16 or None, out16_lo or None, out32 or None, err or None,
                                               stream or None))


def op_repack_q8(raw, N, K, w16, stream=0):
    _check(lib().fa_op_repack_q8(raw, N, K, w16, stream or None))


def op_q8_gemm(a16, a16_lo, M, K, w16, N, n_split, c, variant=0, stream=0):
    _check(lib().fa_op_q8_gemm(a16, a16_lo or None, M, K, w16, N, n_split, c, variant, stream or None))


def op_q8_gemm_swiglu(a16, a16_lo, M, K, w16, N, h16, h_lo, stream=0):
    _check(lib().fa_op_q8_gemm_swiglu(a16, a16_lo or None, M, K, w16, N, h16, h_lo or None, stream or None))


def op_swiglu(part, n_part, M, ffn, h16, h_lo, stream=0):
    _check(lib().fa_op_swiglu(part, n_part, M, ffn, h16, h_lo or None, stream or None))


def op_argmax_scratch_bytes(M, N) -> int:
    return int(lib().fa_op_argmax_scratch_bytes(M, N))


def op_q8_gemm_argmax(a16, a16_lo, M, K, w16, N, scratch, nxt, logits=0, variant=0, stream=0):
    _check(lib().fa_op_q8_gemm_argmax(a16, a16_lo or None, M, K, w16, N, scratch, nxt, logits or None, variant,
                                      stream or None))


def op_q8_planes_bytes(N, K) -> int:
    """Bytes of the Q8_0 planes (q int8 [N][K], scales f16 [K/32][N] and [N][K/32])."""
    return int(lib().fa_op_q8_planes_bytes(N, K))


def op_repack_q8_planes(raw, N, K, planes, stream=0):
    """GGUF Q8_0 blocks [N][K/32][34 B] on the device -> the planes the decoder GEMMs read."""
    _check(lib().fa_op_repack_q8_planes(raw, N, K, planes, stream or None))


def op_q8p_gemm(a16, a16_lo, M, K, planes, N, n_split, c, variant=0, stream=0):
    _check(lib().fa_op_q8p_gemm(a16, a16_lo or None, M, K, planes, N, n_split, c, variant, stream or None))


def op_q8p_gemm_swiglu(a16, a16_lo, M, K, planes, N, h16, h_lo, stream=0):
    _check(lib().fa_op_q8p_gemm_swiglu(a16, a16_lo or None, M, K, planes, N, h16, h_lo or None, stream or None))


def op_q8p_gemm_argmax(a16, a16_lo, M, K, planes, N, scratch, nxt, logits=0, variant=0, stream=0):
    _check(lib().fa_op_q8p_gemm_argmax(a16, a16_lo or None, M, K, planes, N, scratch, nxt, logits or None, variant,
                                       stream or None))


# ---------------------------------------------------------------- encoder --
def _views(weights):
    views = (_TensorView * len(weights))()
    keep = []
    for i, (name, (t, ne, arr)) in enumerate(weights.items()):
        arr = np.ascontiguousarray(arr)
        nb = name.encode()
        keep += [arr, nb]
        views[i].name = nb
        views[i].type = t
        views[i].ne[0] = int(ne[0])
        views[i].ne[1] = int(ne[1]) if len(ne) > 1 else 1
        views[i].data = arr.ctypes.data
        views[i].nbytes = arr.nbytes
    return views, keep


class Encoder:
    """fa_encoder_*: SANM encoder + adaptor on one GPU, LFR features -> decoder embeddings."""

    def __init__(self, device: int = 0, **desc):
        self.desc = _EncoderDesc()
        lib().fa_encoder_default_desc(ctypes.byref(self.desc))
        for k, v in desc.items():
            setattr(self.desc, k, v)
        self.e = lib().fa_encoder_create(device, ctypes.byref(self.desc))
        if not self.e:
            raise FaError(FA_ERR_CUDA, last_error(None))

    def load_weights(self, weights):
        views, keep = _views(weights)
        _check(lib().fa_encoder_load_weights(self.e, views, len(weights)))

    def forward(self, lfr: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(lfr, np.float32)
        out = np.zeros((x.shape[0], self.desc.adaptor_output), np.float32)
        _check(lib().fa_encoder_forward(self.e, _p(x), x.shape[0], _p(out)))
        return out

    def forward_batch(self, utterances):
        """Several utterances in one pass: list of [T_i][input_dim] -> list of [T_i][adaptor_output]."""
        frames = np.array([len(u) for u in utterances], np.int32)
        x = np.ascontiguousarray(np.concatenate(utterances), np.float32)
        out = np.zeros((x.shape[0], self.desc.adaptor_output), np.float32)
        _check(lib().fa_encoder_forward_batch(self.e, len(frames), _p(frames), _p(x), _p(out), None))
        return np.split(out, np.cumsum(frames)[:-1])

    def set_graphs(self, enable: bool):
        _check(lib().fa_encoder_set_graphs(self.e, int(bool(enable))))

    def forward_dev(self, lfr_ptr: int, T: int, out_ptr: int, stream: int = 0):
        _check(lib().fa_encoder_forward_dev(self.e, lfr_ptr, T, out_ptr, stream or None))

    def close(self):
        if getattr(self, "e", None):
            lib().fa_encoder_destroy(self.e)
            self.e = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------ continuous batching --
class Scheduler:
    """fa_sched_*: streams submitted with a prompt (token ids or embeddings) and a
    token budget; each step() runs one batched forward and returns the generated
    (tag, token, finished) events."""

    def __init__(self, decoder, max_batch_rows=512, prefill_chunk=512, max_running=256, eos_id=-1,
                 max_events=4096):
        cfg = _SchedConfig(max_batch_rows, prefill_chunk, max_running, eos_id)
        self.dec = decoder
        ctx = decoder.ctx if decoder is not None else None
        self.s = lib().fa_sched_create(ctx, ctypes.byref(cfg))
        if not self.s:
            raise FaError(FA_ERR_INVALID_ARG, last_error(None))
        self._ev = (_SchedEvent * max_events)()
        self._n = max_events

    def submit(self, tag: int, max_new: int, ids=None, embeds=None):
        i = None if ids is None else _i32(ids)
        e = None if embeds is None else np.ascontiguousarray(embeds, np.float32)
        n = len(i) if i is not None else len(e)
        _check(lib().fa_sched_submit(self.s, int(tag), _p(i), _p(e), n, int(max_new)), self.dec.ctx)

    def step(self):
        n = ctypes.c_int()
        _check(lib().fa_sched_step(self.s, self._ev, self._n, ctypes.byref(n)), self.dec.ctx)
        return [(self._ev[k].tag, self._ev[k].token, bool(self._ev[k].finished)) for k in range(n.value)]

    def idle(self) -> bool:
        return bool(lib().fa_sched_idle(self.s))

    def stats(self) -> dict:
        st = _SchedStats()
        _check(lib().fa_sched_get_stats(self.s, ctypes.byref(st)))
        return {k: getattr(st, k) for k, _ in _SchedStats._fields_}

    def close(self):
        if getattr(self, "s", None):
            lib().fa_sched_destroy(self.s)
            self.s = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------ host page allocator --
class PageAllocator:
    """Host-only view of the library's page allocation policy (no GPU needed)."""

    def __init__(self, n_pages: int):
        self.n_pages = int(n_pages)
        self.h = lib().fa_palloc_create(int(n_pages))
        if not self.h:
            raise FaError(-1, last_error(None))

    def __del__(self):
        if getattr(self, "h", None):
            lib().fa_palloc_destroy(self.h)
            self.h = None

    def alloc(self) -> int:
        return _check(lib().fa_palloc_alloc(self.h))

    def free(self, page: int):
        _check(lib().fa_palloc_free(self.h, int(page)))

    def n_free(self) -> int:
        return _check(lib().fa_palloc_n_free(self.h))

    def compact_moves(self):
        """Apply compaction; returns the (src, dst) page moves in order."""
        src = np.zeros(self.n_pages, np.int32)
        dst = np.zeros_like(src)
        n = ctypes.c_int()
        _check(lib().fa_palloc_compact(self.h, _p(src), _p(dst), len(src), ctypes.byref(n)))
        return src[: n.value].tolist(), dst[: n.value].tolist()
