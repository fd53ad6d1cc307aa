// The decode step of a single row (one sequence, one token: the one-utterance decode of
// the reference's gpu_decode_tokens loop, compute/llm_ops_gpu.cpp:155-207) as ONE
// persistent kernel.
//
// With one row every launch of the launch-per-op step is latency-bound: a layer's eight
// launches move 17 MB of Q8_0 weights (2.6 us at HBM rate) in ~34 us. Here one CTA per SM
// (a cooperative launch, so all CTAs are resident) runs every layer in five phases:
//
//   A  residual add + RMSNorm (every CTA, redundantly) -> QKV GEMV rows
//   B  per (split, KV head) item: q/k RMSNorm + RoPE, K/V append, paged attention
//      (+ split merge by the item that finishes last)
//   C  o_proj GEMV rows
//   D  residual add + RMSNorm -> gate|up GEMV rows + SwiGLU
//   E  down GEMV rows
//
// Every value one phase hands to the next travels as a 64-bit word {32-bit value, 32-bit
// tag}, written with one relaxed store; the tag is this launch's sequence number times
// the layer count plus the layer. A consumer polls the words it needs until each carries
// the tag it expects, so the data is its own signal: no grid barrier, no fence, one L2
// round trip per exchange (waits bounded in time; a CTA that gives up raises the abort
// flag that ends every other wait). One buffer per exchange suffices: a phase's words
// are rewritten only a layer later, after every consumer of the previous layer has used
// them (each phase needs every row of the one before). Each CTA keeps its own copy of
// the residual stream in shared memory.
//
// The weights of the next phase do not depend on its input: each warp loads its next rows
// into registers before it polls, and the attention items start their page copies (4-deep
// rings, barriers initialised once and their phases counted across layers) during the
// previous layer. The token's own K/V row, computed in phase B, is written to its page and
// patched into the page's shared-memory copy.
//
// Same arithmetic as the launch-per-op step with the CUDA-core GEMMs (k_gemv.cu): a GEMV
// unit is a block of 4 weight rows x 512 columns, lane l holding 16 int8 of each row, the
// same fp32 FMA chain per lane, the same xor-shuffle reduction, and the ks units of a row
// block summed in unit order from 0; the norms call residual_norm_row, attention runs the
// body of kernel (2) (k_attn_body.cuh) and kernel (1) is qkv_head_apply. The outputs are
// the same bits, which the tests check.
#include "fa_kernels.cuh"
#include "k_append.cuh"
#include "k_attn_body.cuh"
#include "k_norm.cuh"

#include <cstddef>

namespace fa {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kUnitsPerWarp = 4;
constexpr int kMaxUnits = kWarps * kUnitsPerWarp;
constexpr int kRowStages = 4;
constexpr int kWpl = 16;                 // int8 weights per lane per unit
constexpr int kSlice = 32 * kWpl;        // columns of a unit
constexpr int D = 128;
constexpr int kHq = 16, kHkv = 8;
constexpr int kQkvN = (kHq + 2 * kHkv) * D;
constexpr int kPollWords = 16;           // words one thread polls at a time
using ASmem = attn::Smem<kRowStages>;

struct RowSmem {
    ASmem att;
    float red[kMaxUnits][4];
    double sh[kWarps];
    __half newkv[2 * D];       // the token's K row then V row (f16), for the page patch
    int last;
    alignas(16) float buf[4];  // act [max(hidden, Hq * 128, ffn)], x [hidden], part [hidden]
};

__host__ __device__ inline size_t act_floats(int hidden, int ffn) {
    int k = hidden > ffn ? hidden : ffn;
    return (size_t)(k > kHq * D ? k : kHq * D);
}

// Weights of a warp's units for the next GEMV phase, held in registers while it polls.
struct WRegs {
    uint4 q[kUnitsPerWarp][4];
    float d[kUnitsPerWarp][4];
};

// The CTA's share of a GEMM: row blocks (or gate/up pairs) [b0, b0 + nb) and its units.
struct Span {
    int b0, nb, n_units;
};

__device__ __forceinline__ Span cta_span(const RowGemm& g, int cta, int G) {
    const int total = g.swiglu ? g.N / 8 : g.N / 4;
    Span s;
    s.b0 = (int)((long long)cta * total / G);
    s.nb = (int)((long long)(cta + 1) * total / G) - s.b0;
    s.n_units = s.nb * g.ks * (g.swiglu ? 2 : 1);
    return s;
}

// Unit u of the span -> first weight row n0 and K slice c. SwiGLU units run pair by pair:
// the ks units of the gate rows of output columns f0..f0+3, then those of their up rows
// (gate row f is weight row (f/64)*128 + f%64, its up row 64 further).
__device__ __forceinline__ void unit_rows(const RowGemm& g, const Span& s, int u, int& n0, int& c) {
    c = u % g.ks;
    if (!g.swiglu) {
        n0 = 4 * (s.b0 + u / g.ks);
    } else {
        const int pl = u / (2 * g.ks), which = (u / g.ks) & 1;
        const int f0 = 4 * (s.b0 + pl);
        n0 = (f0 / 64) * 128 + f0 % 64 + 64 * which;
    }
}

__device__ __forceinline__ void load_units(WRegs& w, const RowGemm& g, const Span& s, const unsigned char* planes,
                                           int warp, int lane) {
    const int8_t* q = reinterpret_cast<const int8_t*>(planes);
    const __half* dr = reinterpret_cast<const __half*>(planes + q8p_dr_offset(g.N, g.K));
#pragma unroll
    for (int i = 0; i < kUnitsPerWarp; ++i) {
        const int u = warp + kWarps * i;
        if (u >= s.n_units) break;
        int n0, c;
        unit_rows(g, s, u, n0, c);
        const int k0 = c * kSlice + lane * kWpl;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            w.q[i][r] = __ldg(reinterpret_cast<const uint4*>(q + (size_t)(n0 + r) * g.K + k0));
            w.d[i][r] = __half2float(dr[(size_t)(n0 + r) * (g.K / kQK) + k0 / kQK]);
        }
    }
}

// Every unit of the warp: 4 dot products of 512 columns with act (shared memory), the
// CUDA-core kernel's arithmetic; lane 0 leaves the 4 sums in red[u].
__device__ __forceinline__ void dot_units(const WRegs& w, const RowGemm& g, const Span& s, const float* act,
                                          float (*red)[4], int warp, int lane) {
#pragma unroll
    for (int i = 0; i < kUnitsPerWarp; ++i) {
        const int u = warp + kWarps * i;
        if (u >= s.n_units) break;
        int n0, c;
        unit_rows(g, s, u, n0, c);
        const int k0 = c * kSlice + lane * kWpl;
        float x[kWpl];
#pragma unroll
        for (int h = 0; h < kWpl / 4; ++h) {
            const float4 t = reinterpret_cast<const float4*>(act + k0)[h];
            x[4 * h] = t.x; x[4 * h + 1] = t.y; x[4 * h + 2] = t.z; x[4 * h + 3] = t.w;
        }
        float acc[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            // int8 -> f32 exactly: the byte q + 128 under the exponent of 2^23 reads as 2^23 + q + 128
            const uint32_t* wb = reinterpret_cast<const uint32_t*>(&w.q[i][r]);
            float wf[kWpl];
#pragma unroll
            for (int j4 = 0; j4 < kWpl / 4; ++j4) {
                const uint32_t v = wb[j4] ^ 0x80808080u;
#pragma unroll
                for (int b = 0; b < 4; ++b)
                    wf[4 * j4 + b] = __int_as_float((int)__byte_perm(v, 0x4B000000u, 0x7540u + (unsigned)b)) - 8388736.0f;
            }
            float sq = 0.0f;
#pragma unroll
            for (int j = 0; j < kWpl; ++j) sq = fmaf(wf[j], x[j], sq);
            acc[r] = 0.0f;
            acc[r] = fmaf(w.d[i][r], sq, acc[r]);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
        if (lane == 0)
#pragma unroll
            for (int r = 0; r < 4; ++r) red[u][r] = acc[r];
    }
}

// ------------------------------------------------------------------ words --
__device__ __forceinline__ void st_word(unsigned long long* p, uint32_t v, uint32_t tag) {
    const unsigned long long w = ((unsigned long long)tag << 32) | v;
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ unsigned long long ld_word(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t pack_pair(float y) {
    const __half h = __float2half_rn(y);
    const __half l = __float2half_rn(__fsub_rn(y, __half2float(h)));
    return (uint32_t)__half_as_ushort(h) | ((uint32_t)__half_as_ushort(l) << 16);
}

// The pair as the GEMMs read it: f32(hi) + f32(lo).
__device__ __forceinline__ float pair_sum(uint32_t w) {
    return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu))) +
           __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}

// The normed row as the GEMMs read it: the f16 pair hi = f16(y), lo = f16(y - hi), summed.
__device__ __forceinline__ float pair_value(float y) { return pair_sum(pack_pair(y)); }

__device__ __forceinline__ bool aborted(const RowCtl* ctl) {
    return *reinterpret_cast<const volatile int*>(&ctl->abort) != 0;
}

// One thread's wait for up to kPollWords words: ptr(u) gives word u's address (nullptr:
// none), f(u, value) receives each once all carry `tag`. False when the wait ran out (the
// abort flag is raised) or another CTA's did.
template <typename Ptr, typename F>
__device__ __forceinline__ bool poll_thread(const RowStepArgs& a, uint32_t tag, Ptr ptr, F f) {
    const unsigned long long* p[kPollWords];
    unsigned long long v[kPollWords];
#pragma unroll
    for (int u = 0; u < kPollWords; ++u) {
        p[u] = ptr(u);
        v[u] = p[u] ? ld_word(p[u]) : 0ull;
    }
    unsigned long long t0 = 0;
    for (int it = 0;; ++it) {
        bool all = true;
#pragma unroll
        for (int u = 0; u < kPollWords; ++u)
            if (p[u] && (uint32_t)(v[u] >> 32) != tag) all = false;
        if (all) break;
        const unsigned long long now = global_ns();
        if (it == 0) {
            t0 = now;
        } else if (now - t0 > a.wait_ns) {
            record_error(a.err, kDevErrTimeout);
            atomicExch(&a.ctl->abort, 1);
            return false;
        }
        if ((it & 7) == 7 && aborted(a.ctl)) return false;
#pragma unroll
        for (int u = 0; u < kPollWords; ++u)
            if (p[u] && (uint32_t)(v[u] >> 32) != tag) v[u] = ld_word(p[u]);
    }
#pragma unroll
    for (int u = 0; u < kPollWords; ++u)
        if (p[u]) f(u, (uint32_t)v[u]);
    return true;
}

// The CTA reads words [0, n) of src, word i going to f(i, value), once each carries tag;
// ends with a CTA barrier. False (for every thread) when a wait gave up.
template <typename F>
__device__ __forceinline__ bool poll_words(const RowStepArgs& a, const unsigned long long* src, int n, uint32_t tag,
                                           F f) {
    bool ok = true;
    for (int i0 = threadIdx.x; i0 < n && ok; i0 += kPollWords * kThreads)
        ok = poll_thread(a, tag,
                         [&](int u) -> const unsigned long long* {
                             const int i = i0 + u * kThreads;
                             return i < n ? src + i : nullptr;
                         },
                         [&](int u, uint32_t v) { f(i0 + u * kThreads, v); });
    return __syncthreads_or(!ok) == 0;
}

// Row sums over the ks units of each block, in unit order from 0 (after a CTA barrier),
// as tagged words: the result rows, or for SwiGLU the f16 pair of silu(gate) * up.
__device__ __forceinline__ void finish_units(const RowGemm& g, const Span& s, const float (*red)[4],
                                             unsigned long long* out, uint32_t tag) {
    for (int q = threadIdx.x; q < s.nb * 4; q += kThreads) {
        const int b = q >> 2, r = q & 3;
        if (!g.swiglu) {
            float v = 0.0f;
            for (int c = 0; c < g.ks; ++c) v += red[b * g.ks + c][r];
            st_word(out + 4 * (s.b0 + b) + r, __float_as_uint(v), tag);
        } else {
            float gv = 0.0f, uv = 0.0f;
            for (int c = 0; c < g.ks; ++c) gv += red[b * 2 * g.ks + c][r];
            for (int c = 0; c < g.ks; ++c) uv += red[b * 2 * g.ks + g.ks + c][r];
            st_word(out + 4 * (s.b0 + b) + r, pack_pair(silu_mul(gv, uv)), tag);
        }
    }
}

__device__ __forceinline__ void bar_sync_attn() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads, 1) row_step_kernel(const RowStepArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    RowSmem& S = *reinterpret_cast<RowSmem*>(smem_raw);
    const int Hd = a.hidden;
    float* act = S.buf;
    float* xr = S.buf + act_floats(a.hidden, a.ffn);   // this CTA's copy of the residual stream
    float* part = xr + Hd;                             // the sum the next norm adds to it
    const int cta = blockIdx.x, G = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (cta == a.absent_cta) return;    // failure test: the words of its rows never arrive
    const uint32_t seq = *reinterpret_cast<const volatile uint32_t*>(&a.ctl->seq);
    const uint32_t tag0 = (seq + 1u) * (uint32_t)a.n_layers;

    // ---- this CTA's attention item: split cta / 8 of KV head cta % 8
    AttnArgs at{};
    at.q = nullptr; at.block_table = a.block_table; at.bt_stride = a.bt_stride; at.n_pages = a.n_pages;
    at.slot = a.slot; at.pos = a.pos; at.rows = nullptr; at.M = 1; at.Hq = kHq; at.Hkv = kHkv;
    at.pages_per_split = a.pps; at.n_splits = a.n_splits; at.part_o = a.att_po; at.part_ml = a.att_pml;
    at.out16 = nullptr; at.out16_lo = nullptr; at.out32 = nullptr; at.err = a.err;
    const int split = cta / kHkv, h = cta % kHkv;
    const int pos = a.pos[0];
    const int n_kv = pos + 1;
    const int n_row_pages = (n_kv + kPageTokens - 1) / kPageTokens;
    const bool len_bad = attn::row_len_bad(at, n_kv, n_row_pages);
    if (len_bad && cta == 0 && threadIdx.x == 0) record_error(a.err, kDevErrBadLen);
    const int p_begin = split * a.pps;
    const int p_end = min(n_row_pages, p_begin + a.pps);
    const bool item = cta < a.n_splits * kHkv && !len_bad && p_begin < n_row_pages;
    const int n_valid = min(a.n_splits, (n_row_pages + a.pps - 1) / max(a.pps, 1));
    const int p_last = n_row_pages - 1;
    const bool owner = item && p_last >= p_begin && p_last < p_end;   // the token's page is in this split
    const int* bt = a.block_table + (size_t)a.slot[0] * a.bt_stride;
    const size_t page_elems = (size_t)kHkv * attn::TILE_HALVES;

    if (threadIdx.x == 0) {
        for (int w = 0; w < attn::WARPS; ++w)
            for (int s = 0; s < kRowStages; ++s) mbar_init(&S.att.bars[w][s], 1);
        fence_mbar_init();
    }
    // ---- layer 0's input row
    const bool embed_row = !a.x_ready && a.tok[0] != -1;
    if (embed_row) {
        const int tok = a.tok[0];
        const bool bad = tok < 0 || tok >= a.vocab;
        if (bad && cta == 0 && threadIdx.x == 0) record_error(a.err, kDevErrBadPage);
        const size_t off = (size_t)(bad ? 0 : tok) * Hd;
        for (int i = threadIdx.x; i < Hd; i += kThreads) {
            float v;
            if (bad) v = 0.0f;
            else if (a.embed_type == 30) v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.embed)[off + i]);
            else if (a.embed_type == 1) v = __half2float(reinterpret_cast<const __half*>(a.embed)[off + i]);
            else v = reinterpret_cast<const float*>(a.embed)[off + i];
            xr[i] = v;
        }
    } else {
        for (int i = threadIdx.x; i < Hd; i += kThreads) xr[i] = a.x_a[i];
    }
    __syncthreads();

    const Span sp_qkv = cta_span(a.gm[0], cta, G), sp_o = cta_span(a.gm[1], cta, G);
    const Span sp_gu = cta_span(a.gm[2], cta, G), sp_dn = cta_span(a.gm[3], cta, G);
    WRegs wr;
    load_units(wr, a.gm[0], sp_qkv, a.layers[0].w[0], warp, lane);

    auto emit_act = [&](int j, float y) { act[j] = pair_value(y); };
    auto to_part = [&](int i, uint32_t v) { part[i] = __uint_as_float(v); };
    // the page ring's barriers are initialised once; bit s = parity of stage s's next phase
    uint32_t ring_ph = 0u;
    int nw = 0, issued = 0;        // this warp's pages of the item and copies in flight
    // The item's page copies of layer l start (attention warps); the ring's shared memory
    // was last read and patched by generic accesses, hence the proxy fence.
    auto start_pages = [&](int l) {
        if (item && warp < attn::WARPS) {
            if (lane == 0) fence_proxy_async_smem();
            __syncwarp();
            const __half* hb = a.pool + (size_t)l * a.layer_stride + (size_t)h * attn::TILE_HALVES;
            nw = attn::warp_page_count(p_end - p_begin, warp);
            nw = attn::warp_check_pages(at, bt, p_begin, nw, warp, lane);
            issued = attn::warp_issue_first(S.att, bt, p_begin, nw, hb, page_elems, warp, lane);
        }
    };
    // nothing may land in shared memory after the CTA has left: wait (bounded) for the
    // copies in flight
    auto leave = [&]() {
        if (item && warp < attn::WARPS)
            for (int k = 0; k < issued; ++k) {
                const int st = k % kRowStages;
                const bool done = mbar_wait_bounded(&S.att.bars[warp][st],
                                                    ((uint32_t)(k / kRowStages) & 1u) ^ ((ring_ph >> st) & 1u));
                (void)__all_sync(0xffffffffu, done);
            }
    };
    start_pages(0);

    for (int l = 0; l < a.n_layers; ++l) {
        const RowLayer L = a.layers[l];
        const uint32_t tag = tag0 + (uint32_t)l;
        __half* pool_l = a.pool + (size_t)l * a.layer_stride;
        at.pool_layer = pool_l;
        const __half* head_base = pool_l + (size_t)h * attn::TILE_HALVES;

        // ---------------- A: norm + QKV (the item's page copies are in flight)
        if (l == 0) {
            residual_norm_row<8, false>(xr, nullptr, 0, 0, Hd, L.in_norm, a.eps, nullptr, S.sh, emit_act);
        } else {
            if (!poll_words(a, a.w_dn, Hd, tag - 1u, to_part)) return leave();
            residual_norm_row<8, false>(xr, reinterpret_cast<const float4*>(part), 0, 1, Hd, L.in_norm, a.eps, xr,
                                        S.sh, emit_act);
        }
        __syncthreads();
        dot_units(wr, a.gm[0], sp_qkv, act, S.red, warp, lane);
        __syncthreads();
        finish_units(a.gm[0], sp_qkv, S.red, a.w_qkv, tag);

        // ---------------- B: kernel (1) for the item's heads, then attention
        if (item) {
            bool ok = true;
            if (warp >= 4) {
                const int v = warp - 4;     // q heads 2h, 2h+1, then K and V of head h
                const int j = v < 2 ? 2 * h + v : (v == 2 ? kHq + h : kHq + kHkv + h);
                if (v < 2 || owner) {
                    float x[4];
                    ok = poll_thread(a, tag,
                                     [&](int u) -> const unsigned long long* {
                                         return u < 4 ? a.w_qkv + j * D + lane + 32 * u : nullptr;
                                     },
                                     [&](int u, uint32_t w) { x[u] = __fadd_rn(0.0f, __uint_as_float(w)); });
                    // the lanes poll their own words, but the head's norm shuffles over the
                    // whole warp: all lanes go on, or none
                    ok = __all_sync(0xffffffffu, ok);
                    if (ok) {
                        AppendArgs app{};
                        app.n_part = 1; app.M = 1; app.pos = a.pos; app.slot = a.slot;
                        app.block_table = a.block_table; app.bt_stride = a.bt_stride; app.n_pages = a.n_pages;
                        app.qn_w = L.q_norm; app.kn_w = L.k_norm; app.Hq = kHq; app.Hkv = kHkv; app.eps = a.eps;
                        app.q_scale = a.q_scale; app.rope = a.rope; app.max_pos = a.max_pos;
                        app.pool_layer = pool_l; app.q_out = nullptr; app.err = a.err;
                        const HeadRowMeta meta = qkv_head_meta(app, 0, j, lane);
                        qkv_head_apply(app, meta, 0, j, lane, x, v < 2 ? S.att.q[v] : nullptr,
                                       v < 2 ? nullptr : S.newkv + (v - 2) * D);
                    }
                }
            }
            if (__syncthreads_or(!ok)) return leave();
            if (warp < attn::WARPS) {
                const int t = threadIdx.x;
                S.att.q[0][t] = S.att.q[0][t] * attn::kLog2e;
                S.att.q[1][t] = S.att.q[1][t] * attn::kLog2e;
                bar_sync_attn();
                const int rel = p_last - p_begin;
                const int patch_i = owner && warp == rel % attn::WARPS ? rel / attn::WARPS : -1;
                attn::warp_pages(at, S.att, bt, p_begin, nw, issued, n_kv, head_base, page_elems,
                                 owner ? S.newkv : nullptr, patch_i, pos % kPageTokens, warp, lane, ring_ph);
                ring_ph = attn::ring_phase_after<kRowStages>(ring_ph, nw);
                issued = 0;
                bar_sync_attn();
                if (a.n_splits == 1) {
                    attn::merge_warps(S.att, t, [&](int hq, float, float Ls, float Os) {
                        st_word(a.w_att + (2 * h + hq) * D + t, pack_pair(Ls > 0.0f ? Os / Ls : 0.0f), tag);
                    });
                } else {
                    // partials to the scratch; the split that finishes last merges the head's
                    // splits and writes its words
                    attn::merge_warps(S.att, t, [&](int hq, float M, float Ls, float Os) {
                        attn::merge_store(at, split, h, 0, t, hq, M, Ls, Os);
                    });
                    bar_sync_attn();
                    if (t == 0) {
                        __threadfence();
                        const int old = atomicAdd(&a.ctl->att_cnt[h], 1);
                        S.last = old == n_valid - 1;
                        if (S.last) {
                            __threadfence();
                            a.ctl->att_cnt[h] = 0;
                        }
                    }
                    bar_sync_attn();
                    if (S.last && warp < 2) {
                        const int H = 2 * h + warp;
                        attn::combine_head<true>(at, 0, H, lane, [&](int d, float v) {
                            st_word(a.w_att + H * D + d, pack_pair(v), tag);
                        });
                    }
                }
            }
        }
        load_units(wr, a.gm[1], sp_o, L.w[1], warp, lane);

        // ---------------- C: o_proj
        if (!poll_words(a, a.w_att, kHq * D, tag, [&](int i, uint32_t v) { act[i] = pair_sum(v); })) return leave();
        dot_units(wr, a.gm[1], sp_o, act, S.red, warp, lane);
        __syncthreads();
        finish_units(a.gm[1], sp_o, S.red, a.w_o, tag);
        load_units(wr, a.gm[2], sp_gu, L.w[2], warp, lane);

        // ---------------- D: norm + gate|up + SwiGLU
        if (!poll_words(a, a.w_o, Hd, tag, to_part)) return leave();
        residual_norm_row<8, false>(xr, reinterpret_cast<const float4*>(part), 0, 1, Hd, L.post_norm, a.eps, xr, S.sh,
                                    emit_act);
        __syncthreads();
        dot_units(wr, a.gm[2], sp_gu, act, S.red, warp, lane);
        __syncthreads();
        finish_units(a.gm[2], sp_gu, S.red, a.w_h, tag);
        load_units(wr, a.gm[3], sp_dn, L.w[3], warp, lane);

        // ---------------- E: down
        if (!poll_words(a, a.w_h, a.ffn, tag, [&](int i, uint32_t v) { act[i] = pair_sum(v); })) return leave();
        dot_units(wr, a.gm[3], sp_dn, act, S.red, warp, lane);
        __syncthreads();
        finish_units(a.gm[3], sp_dn, S.red, a.w_dn, tag);
        if (l + 1 < a.n_layers) {
            load_units(wr, a.gm[0], sp_qkv, a.layers[l + 1].w[0], warp, lane);
            start_pages(l + 1);
        }
    }

    // ---------------- final norm: the lm_head's input pair (CTA 0)
    if (cta != 0) return;
    if (!poll_words(a, a.w_dn, Hd, tag0 + (uint32_t)a.n_layers - 1u, to_part)) return;
    residual_norm_row<8, false>(xr, reinterpret_cast<const float4*>(part), 0, 1, Hd, a.final_norm, a.eps, xr, S.sh,
                                [&](int j, float y) { split_store(y, a.xn16, a.xn_lo, (size_t)j); });
    __syncthreads();
    for (int i = threadIdx.x; i < Hd; i += kThreads) a.x_a[i] = xr[i];
    // every CTA read the sequence number at its start, long before this point (its rows
    // of every phase came before)
    if (threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(&a.ctl->seq) = seq + 1u;
}

}  // namespace

bool row_step_shapes(int hidden, int ffn, int grid, RowGemm* gm) {
    if (hidden <= 0 || hidden > 4096 || hidden % kSlice || ffn % kSlice || grid <= 0) return false;
    const int shapes[4][3] = {{kQkvN, hidden, kEpiStoreF32},
                              {hidden, kHq * D, kEpiStoreF32},
                              {2 * ffn, hidden, kEpiSwiglu},
                              {hidden, ffn, kEpiStoreF32}};
    for (int i = 0; i < 4; ++i) {
        int ks = 0, ns = 0;
        if (!gemv_q8_split(1, shapes[i][0], shapes[i][1], shapes[i][2], &ks, &ns) || ns != 1 || ks * kSlice != shapes[i][1])
            return false;
        RowGemm& g = gm[i];
        g.N = shapes[i][0];
        g.K = shapes[i][1];
        g.ks = ks;
        g.swiglu = shapes[i][2] == kEpiSwiglu;
        if (g.swiglu && (ffn % 64)) return false;
        const int total = g.swiglu ? g.N / 8 : g.N / 4;
        const int per_cta = (total + grid - 1) / grid;
        if (per_cta * ks * (g.swiglu ? 2 : 1) > kMaxUnits) return false;
    }
    return row_step_smem_bytes(hidden, ffn) <= 227 * 1024;
}

size_t row_step_smem_bytes(int hidden, int ffn) {
    return offsetof(RowSmem, buf) + sizeof(float) * (act_floats(hidden, ffn) + 2 * (size_t)hidden);
}

size_t row_step_words(int hidden, int ffn) {
    return (size_t)kQkvN + (size_t)kHq * D + 2 * (size_t)hidden + (size_t)ffn;
}

cudaError_t configure_row_step() {
    return cudaFuncSetAttribute(row_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

cudaError_t launch_row_step(const RowStepArgs& a, int grid, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = row_step_smem_bytes(a.hidden, a.ffn);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, row_step_kernel, a);
}

}  // namespace fa
