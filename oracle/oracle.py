"""ctypes/numpy front end of the CPU oracle (oracle/oracle.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference legs. It restates the reference decoder's
semantics on the CPU; the product library never calls it.

Besides the bindings, this module holds the oracle's restatement of the page
allocator policy (lowest free page first, pages taken when a sequence's length
reaches a multiple of 16, returned on close) and of page compaction, so that
block tables can be checked for byte identity against the CUDA library.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

# GEMM arithmetic modes of or_gemm_q8 / or_decoder_forward.
MODE_EXACT = 0      # f32 activations x exactly dequantised weights d*q: the decoder CUDA path
MODE_W16 = 1        # f32 activations x f16(d*q) weights: the f16 weight form (the encoder's GEMMs)
MODE_GGML_CPU = 2   # ggml CPU backend: Q8_0 activations, integer block dots

QK8_0 = 32
Q8_0_BYTES = 34


def build() -> str:
    """Compile liboracle.so with the committed Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float


def _declare(L):
    L.or_f32_to_f16.argtypes = [_P, _I64, _P]
    L.or_f16_to_f32.argtypes = [_P, _I64, _P]
    L.or_rope_table.argtypes = [_I, _I, ctypes.c_double, _P]
    L.or_q8_0_quantize.argtypes = [_P, _I64, _P]
    L.or_q8_0_dequant.argtypes = [_P, _I64, _P]
    L.or_rmsnorm.argtypes = [_P, _P, _I, _I, _F, _P]
    L.or_gemm_q8.argtypes = [_P, _I, _I, _P, _I, _I, _P]
    L.or_qknorm_rope_append.argtypes = [_P, _I, _P, _P, _P, _I, _P, _P, _I, _I, _I, _I, _F, _F, _P, _P, _P]
    L.or_kv_append_raw.argtypes = [_P, _P, _I, _I, _P, _P, _P, _I, _I, _I, _I, _I, _P]
    L.or_paged_attention.argtypes = [_P, _I, _P, _P, _P, _I, _P, _I, _I, _I, _I, _P]
    L.or_argmax_rows.argtypes = [_P, _I, _I, _P]
    L.or_decoder_forward.argtypes = [_P, _I, _I, _P, _P, _P, _P, _P, _I, _P, _P, _P, _P]
    L.or_num_threads.restype = _I
    L.or_set_num_threads.argtypes = [_I]


def _ptr(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ------------------------------------------------------------------ conversions --
def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().or_f32_to_f16(_ptr(x), x.size, _ptr(out))
    return out


def f16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    h = _c(h, np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().or_f16_to_f32(_ptr(h), h.size, _ptr(out))
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (_c(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bit patterns (finite inputs)."""
    u = _c(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


# ------------------------------------------------------------------- RoPE / Q8_0 --
def rope_table(max_pos: int, head_dim: int = 128, base: float = 1e6) -> np.ndarray:
    cs = np.empty((max_pos, head_dim // 2, 2), np.float32)
    lib().or_rope_table(max_pos, head_dim, base, _ptr(cs))
    return cs


def q8_0_quantize(x: np.ndarray) -> np.ndarray:
    """Q8_0 blocks of a [..., K] f32 array, as uint8 [..., K/32*34]."""
    x = _c(x, np.float32)
    assert x.shape[-1] % QK8_0 == 0
    out = np.empty(x.shape[:-1] + (x.shape[-1] // QK8_0 * Q8_0_BYTES,), np.uint8)
    lib().or_q8_0_quantize(_ptr(x), x.size, _ptr(out))
    return out


def q8_0_dequant(blocks: np.ndarray, k: int) -> np.ndarray:
    blocks = _c(blocks, np.uint8)
    n = blocks.size // Q8_0_BYTES * QK8_0
    out = np.empty(n, np.float32)
    lib().or_q8_0_dequant(_ptr(blocks), n, _ptr(out))
    return out.reshape(blocks.shape[:-1] + (k,))


# ------------------------------------------------------------------------- ops --
def rmsnorm(x: np.ndarray, w: Optional[np.ndarray], eps: float = 1e-5) -> np.ndarray:
    x = _c(x, np.float32)
    n = x.shape[-1]
    rows = x.size // n
    out = np.empty_like(x)
    lib().or_rmsnorm(_ptr(x), _ptr(None if w is None else _c(w, np.float32)), rows, n, eps, _ptr(out))
    return out


def gemm_q8(a: np.ndarray, w_q8: np.ndarray, n: int, mode: int = MODE_EXACT) -> np.ndarray:
    a = _c(a, np.float32)
    M, K = a.shape
    w_q8 = _c(w_q8, np.uint8)
    assert w_q8.size == n * K // QK8_0 * Q8_0_BYTES
    out = np.empty((M, n), np.float32)
    lib().or_gemm_q8(_ptr(a), M, K, _ptr(w_q8), n, mode, _ptr(out))
    return out


def qknorm_rope_append(qkv, slot, pos, block_table, qn_w, kn_w, rope_cs, pool_layer,
                       n_heads=16, n_kv_heads=8, head_dim=128, page_tokens=16, eps=1e-5):
    """Mutates pool_layer ([n_pages][Hkv][2][PT][D] uint16); returns q_out [M][Hq*D]."""
    qkv = _c(qkv, np.float32)
    M = qkv.shape[0]
    slot = _c(slot, np.int32); pos = _c(pos, np.int32)
    bt = _c(block_table, np.int32)
    assert pool_layer.dtype == np.uint16 and pool_layer.flags["C_CONTIGUOUS"]
    q_out = np.empty((M, n_heads * head_dim), np.float32)
    q_scale = np.float32(1.0) / np.sqrt(np.float32(head_dim))
    lib().or_qknorm_rope_append(_ptr(qkv), M, _ptr(slot), _ptr(pos), _ptr(bt), bt.shape[1],
                                _ptr(_c(qn_w, np.float32)), _ptr(_c(kn_w, np.float32)),
                                n_heads, n_kv_heads, head_dim, page_tokens, eps, float(q_scale),
                                _ptr(_c(rope_cs, np.float32)), _ptr(pool_layer), _ptr(q_out))
    return q_out


def kv_append_raw(k16, v16, slot, pos, block_table, pool, n_layers, n_pages,
                  n_kv_heads=8, head_dim=128, page_tokens=16):
    """k16/v16: [M][n_layers][Hkv][D] uint16; pool: [n_layers][n_pages][page] uint16 (mutated)."""
    k16 = _c(k16, np.uint16); v16 = _c(v16, np.uint16)
    bt = _c(block_table, np.int32)
    lib().or_kv_append_raw(_ptr(k16), _ptr(v16), k16.shape[0], n_layers, _ptr(_c(slot, np.int32)),
                           _ptr(_c(pos, np.int32)), _ptr(bt), bt.shape[1], n_pages,
                           n_kv_heads, head_dim, page_tokens, _ptr(pool))


def kv_gather(pool, block_table, slot, n_kv, row0, total_rows, out_k=None, out_v=None,
              n_kv_heads=8, head_dim=128, page_tokens=16):
    """Head-major K/V slabs of the tokens [0, n_kv[m]) of sequences slot[m].

    Restates compute/llm_ops_gpu.cpp:97-105: the view of a layer's cache over n_kv
    tokens ([n_kv][8*128], token-major), reshaped to [128, 8, n_kv] and made contiguous
    as [8][n_kv][128] (ggml_cont of the 0,2,1,3 permutation), here read through the
    block table. pool: [n_layers][n_pages][Hkv][2][16][128] uint16. Returns k, v
    [n_layers][Hkv][total_rows][128] uint16 with sequence m at rows row0[m]...; rows no
    sequence covers keep out_k / out_v's values (zeros when not given)."""
    pool = np.asarray(pool)
    L = pool.shape[0]
    P = pool.reshape(L, pool.shape[1], n_kv_heads, 2, page_tokens, head_dim)
    k = np.zeros((L, n_kv_heads, total_rows, head_dim), np.uint16) if out_k is None else out_k
    v = np.zeros((L, n_kv_heads, total_rows, head_dim), np.uint16) if out_v is None else out_v
    bt = np.asarray(block_table)
    for m in range(len(slot)):
        n = int(n_kv[m])
        toks = np.arange(n)
        pg = bt[slot[m], toks // page_tokens]
        r = slice(int(row0[m]), int(row0[m]) + n)
        # the split advanced indices come first: [n][L][Hkv][D] -> [L][Hkv][n][D]
        k[:, :, r] = P[:, pg, :, 0, toks % page_tokens].transpose(1, 2, 0, 3)
        v[:, :, r] = P[:, pg, :, 1, toks % page_tokens].transpose(1, 2, 0, 3)
    return k, v


def paged_attention(q, slot, n_kv, block_table, pool_layer, n_heads=16, n_kv_heads=8,
                    head_dim=128, page_tokens=16):
    q = _c(q, np.float32)
    M = q.shape[0]
    bt = _c(block_table, np.int32)
    out = np.empty((M, n_heads * head_dim), np.float32)
    lib().or_paged_attention(_ptr(q), M, _ptr(_c(slot, np.int32)), _ptr(_c(n_kv, np.int32)), _ptr(bt),
                             bt.shape[1], _ptr(_c(pool_layer, np.uint16)), n_heads, n_kv_heads,
                             head_dim, page_tokens, _ptr(out))
    return out


def argmax_rows(logits: np.ndarray) -> np.ndarray:
    logits = _c(logits, np.float32)
    M, N = logits.shape
    out = np.empty(M, np.int32)
    lib().or_argmax_rows(_ptr(logits), M, N, _ptr(out))
    return out


def num_threads() -> int:
    return int(lib().or_num_threads())


def set_num_threads(n: int) -> None:
    lib().or_set_num_threads(int(n))


# ------------------------------------------------------------------- full model --
class _Model(ctypes.Structure):
    _fields_ = [
        ("n_layers", _I), ("hidden", _I), ("n_heads", _I), ("n_kv_heads", _I), ("head_dim", _I),
        ("ffn", _I), ("vocab", _I), ("page_tokens", _I), ("n_pages", _I), ("max_pos", _I),
        ("eps", _F),
        ("embed_bf16", _P), ("final_norm", _P), ("lm_head", _P),
        ("wq", _P), ("wk", _P), ("wv", _P), ("wo", _P), ("wg", _P), ("wu", _P), ("wd", _P),
        ("in_norm", _P), ("post_norm", _P), ("q_norm", _P), ("k_norm", _P),
        ("rope_cs", _P),
    ]


class OracleDecoder:
    """Whole-decoder oracle over a paged f16 cache owned by this object.

    `weights` is a synthetic/loaded model in GGUF form (see the package's synth
    module): dict name -> (ggml_type, ne, ndarray). Norm weights may be BF16/F32.
    """

    def __init__(self, cfg, weights, n_pages: int, max_seqs: int, max_pages_per_seq: int,
                 max_pos: int, mode: int = MODE_EXACT):
        self.cfg = cfg
        self.mode = mode
        L = cfg["n_layers"]
        self.n_pages = n_pages
        self.page_elems = cfg["n_kv_heads"] * 2 * 16 * cfg["head_dim"]
        self.pool = np.zeros((L, n_pages, self.page_elems), np.uint16)
        self.block_table = np.zeros((max_seqs, max_pages_per_seq), np.int32)
        self.alloc = PageAllocatorOracle(n_pages)
        self.seq_len = {}
        self.seq_pages = {}
        self.rope = rope_table(max_pos, cfg["head_dim"], cfg.get("rope_base", 1e6))
        self._keep = []

        def f32(name):
            t, ne, arr = weights[name]
            a = bf16_bits_to_f32(arr) if t == 30 else (f16_bits_to_f32(arr) if t == 1 else _c(arr, np.float32))
            a = np.ascontiguousarray(a.reshape(-1), np.float32)
            self._keep.append(a)
            return a

        def raw(name):
            t, ne, arr = weights[name]
            a = np.ascontiguousarray(arr)
            self._keep.append(a)
            return a

        def parr(arrs):
            p = (ctypes.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
            self._keep.append(p)
            return ctypes.cast(p, ctypes.c_void_p)

        pre = "llm.model.layers.{}."
        m = _Model()
        m.n_layers = L; m.hidden = cfg["hidden"]; m.n_heads = cfg["n_heads"]; m.n_kv_heads = cfg["n_kv_heads"]
        m.head_dim = cfg["head_dim"]; m.ffn = cfg["ffn"]; m.vocab = cfg["vocab"]; m.page_tokens = 16
        m.n_pages = n_pages; m.max_pos = max_pos; m.eps = cfg.get("eps", 1e-5)
        t, ne, emb = weights["llm.model.embed_tokens.weight"]
        assert t == 30, "oracle expects a BF16 embedding table"
        emb = raw("llm.model.embed_tokens.weight")
        m.embed_bf16 = emb.ctypes.data
        m.final_norm = f32("llm.model.norm.weight").ctypes.data
        m.lm_head = raw("llm.lm_head.weight").ctypes.data
        names = {"wq": "self_attn.q_proj.weight", "wk": "self_attn.k_proj.weight", "wv": "self_attn.v_proj.weight",
                 "wo": "self_attn.o_proj.weight", "wg": "mlp.gate_proj.weight", "wu": "mlp.up_proj.weight",
                 "wd": "mlp.down_proj.weight"}
        for f, n in names.items():
            setattr(m, f, parr([raw(pre.format(i) + n) for i in range(L)]))
        norms = {"in_norm": "input_layernorm.weight", "post_norm": "post_attention_layernorm.weight",
                 "q_norm": "self_attn.q_norm.weight", "k_norm": "self_attn.k_norm.weight"}
        for f, n in norms.items():
            setattr(m, f, parr([f32(pre.format(i) + n) for i in range(L)]))
        m.rope_cs = self.rope.ctypes.data
        self.model = m

    # sequence bookkeeping (restated allocator policy)
    def seq_open(self, slot: int):
        self.seq_len[slot] = 0
        self.seq_pages[slot] = []

    def seq_close(self, slot: int):
        for p in self.seq_pages.pop(slot):
            self.alloc.free(p)
        self.seq_len.pop(slot)

    def _reserve(self, slot: int, new_len: int):
        pages = self.seq_pages[slot]
        while len(pages) * 16 < new_len:
            p = self.alloc.alloc()
            self.block_table[slot, len(pages)] = p
            pages.append(p)

    def adopt(self, slot: int, length: int, pages_by_layer):
        """Take over a cached sequence: `length` tokens whose pages (allocated here by the
        same lowest-first policy) get the given contents, pages_by_layer[l] = [n][page_elems]
        f16 bits in block-table order. Returns the slot's page ids."""
        self._reserve(slot, length)
        self.seq_len[slot] = length
        pages = self.seq_pages[slot]
        for l, arr in enumerate(pages_by_layer):
            self.pool[l, pages] = np.asarray(arr, np.uint16).reshape(len(pages), self.page_elems)
        return list(pages)

    def forward(self, slots: Sequence[int], tokens=None, embeds=None, want_logits=True):
        """One forward over rows; each row appends one token to its sequence."""
        slots = np.asarray(slots, np.int32)
        M = len(slots)
        pos = np.empty(M, np.int32)
        for i, s in enumerate(slots):
            pos[i] = self.seq_len[int(s)]
            self._reserve(int(s), pos[i] + 1)
            self.seq_len[int(s)] += 1
        V = self.cfg["vocab"]
        logits = np.empty((M, V), np.float32) if want_logits else None
        nxt = np.empty(M, np.int32)
        tok = None if tokens is None else _c(tokens, np.int32)
        emb = None if embeds is None else _c(embeds, np.float32)
        lib().or_decoder_forward(ctypes.byref(self.model), self.mode, M, _ptr(tok), _ptr(emb), _ptr(slots),
                                 _ptr(pos), _ptr(self.block_table), self.block_table.shape[1],
                                 _ptr(self.pool), _ptr(logits), _ptr(nxt), None)
        return logits, nxt


class PageAllocatorOracle:
    """Restated page allocation policy: the lowest free page id is handed out first."""

    def __init__(self, n_pages: int):
        self.free_set = np.ones(n_pages, bool)

    def alloc(self) -> int:
        idx = np.flatnonzero(self.free_set)
        if idx.size == 0:
            raise MemoryError("page pool exhausted")
        p = int(idx[0])
        self.free_set[p] = False
        return p

    def free(self, p: int) -> None:
        assert not self.free_set[p], "double free"
        self.free_set[p] = True

    def n_free(self) -> int:
        return int(self.free_set.sum())


def compaction_plan(live_pages: Sequence[int], n_pages: int):
    """Restated compaction: while the highest live page is above the lowest free
    page, move it there. Returns (src, dst) lists in move order."""
    live = set(int(p) for p in live_pages)
    free = sorted(p for p in range(n_pages) if p not in live)
    hi = sorted(live, reverse=True)
    src, dst = [], []
    fi = 0
    for p in hi:
        if fi >= len(free) or free[fi] > p:
            break
        src.append(p)
        dst.append(free[fi])
        fi += 1
    return src, dst
