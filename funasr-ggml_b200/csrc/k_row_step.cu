// The decode step of a single row (one sequence, one token: the one-utterance decode of
// the reference's gpu_decode_tokens loop, compute/llm_ops_gpu.cpp:155-207) as ONE
// persistent kernel.
//
// With one row every launch of the launch-per-op step is latency-bound: a layer's eight
// launches move 17 MB of Q8_0 weights (2.6 us at HBM rate) in ~34 us. Here one CTA per SM
// (a cooperative launch, so all CTAs are resident) runs every layer in five phases, and
// then the final one:
//
//   A  residual add + RMSNorm (every CTA, redundantly) -> QKV GEMV rows
//   B  per (split, KV head) item: q/k RMSNorm + RoPE, K/V append, paged attention on all 8
//      warps (+ split merge by the item that finishes last)
//   C  o_proj GEMV rows
//   D  residual add + RMSNorm -> gate|up GEMV rows + SwiGLU
//   E  down GEMV rows
//   F  final norm (every CTA), lm_head rows of 64-row vocab tiles and their maxima, the
//      argmax by the CTA that finishes last (hidden 512 or 1024; otherwise the lm_head
//      runs as its own launch after the kernel)
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
// The weights of the next phase do not depend on its input: as soon as a phase's dot
// products are done, one thread stages the CTA's rows of the next GEMM into shared memory
// by bulk copies (so the copies leave the load/store unit free for the polls), the next
// norm's weights follow by cp.async, and the attention items start their page copies
// (2-deep rings on all 8 warps, barriers initialised once, their phases counted) during
// the previous layer. The token's own K/V row, computed in phase B, is written to its page and
// patched into the page's shared-memory copy.
//
// Same arithmetic as the launch-per-op step with the CUDA-core GEMMs (k_gemv.cu): a GEMV
// unit is a block of 4 weight rows x 512 columns, lane l holding 16 int8 of each row, the
// same fp32 FMA chain per lane, a warp reduction that pairs lanes as its xor-shuffle
// reduction does, and the ks units of a row block summed in unit order from 0; the norms call residual_norm_row, attention runs the
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
constexpr int kRowStages = 2;           // page ring depth: 16 pages per split in flight
constexpr int kWpl = 16;                 // int8 weights per lane per unit
constexpr int kSlice = 32 * kWpl;        // columns of a unit
constexpr int D = 128;
constexpr int kHq = 16, kHkv = 8;
constexpr int kQkvN = (kHq + 2 * kHkv) * D;
constexpr int kPollWords = 16;           // words one thread polls at a time
constexpr int kLmRows = 32;              // lm_head rows per staged chunk: one 4-row block per warp
constexpr int kLmSlots = 3;              // chunks in flight (in the attention ring's shared memory)
constexpr int kAttnNW = 8;               // the attention item's warps: the whole CTA
using ASmem = attn::Smem<kRowStages, kAttnNW>;

struct RowSmem {
    ASmem att;
    float red[kMaxUnits][4];
    double sh[kWarps];
    __half newkv[2 * D];       // the token's K row then V row (f16), for the page patch
    uint64_t wbar;             // completion of the staged weights' bulk copies
    uint64_t lmbar[kLmSlots];  // completion of the lm_head chunks
    float tilev[2][64];        // the logits of a 64-row vocab tile (two tiles alternate)
    float rv[kWarps];          // the argmax's per-warp results
    int ri[kWarps];
    int last;
    // act [max(hidden, Hq * 128, ffn)] (permuted, act_index), x [hidden], part [hidden],
    // norm weights [2][hidden], then the staged weights: q rows [rows][K] int8, then their
    // scales [rows][K / 32] f16
    alignas(128) float buf[4];
};

__host__ __device__ inline size_t act_floats(int hidden, int ffn) {
    int k = hidden > ffn ? hidden : ffn;
    return (size_t)(k > kHq * D ? k : kHq * D);
}

__host__ __device__ inline size_t stage_offset(int hidden, int ffn) {   // bytes from buf, 128-aligned
    return ((act_floats(hidden, ffn) + 4 * (size_t)hidden) * sizeof(float) + 127) / 128 * 128;
}

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

// The CTA's share of a GEMM as runs of consecutive weight rows: run(n, rr, cnt) for
// weight rows [n, n + cnt) that go to staged rows [rr, rr + cnt).
template <typename Run>
__device__ __forceinline__ void share_runs(const RowGemm& g, const Span& s, Run run) {
    if (!g.swiglu) {
        run(4 * s.b0, 0, 4 * s.nb);
        return;
    }
    // output columns f in [4 b0, 4 (b0 + nb)): gate row (f/64)*128 + f%64, up row 64 further;
    // consecutive f map to consecutive rows within a 64-block
    const int f0 = 4 * s.b0, f1 = 4 * (s.b0 + s.nb);
    for (int fa = f0; fa < f1;) {
        const int fb = min(f1, (fa / 64 + 1) * 64);
        for (int which = 0; which < 2; ++which)
            run((fa / 64) * 128 + fa % 64 + 64 * which, which * 4 * s.nb + (fa - f0), fb - fa);
        fa = fb;
    }
}

// Thread 0: one bulk copy per run of the CTA's share (q rows, then the same rows' scales)
// into the staging area, completion on bar.
__device__ __forceinline__ void stage_weights(const RowGemm& g, const Span& s, const unsigned char* planes,
                                              unsigned char* sq, __half* sd, uint64_t* bar) {
    const size_t dr_off = q8p_dr_offset(g.N, g.K);
    const uint32_t rows = (uint32_t)(s.nb * (g.swiglu ? 8 : 4));
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(bar, rows * (uint32_t)(g.K + g.K / 16));
    share_runs(g, s, [&](int n, int rr, int cnt) {
        bulk_copy_g2s(sq + (size_t)rr * g.K, planes + (size_t)n * g.K, (uint32_t)(cnt * g.K), bar);
        bulk_copy_g2s(sd + (size_t)rr * (g.K / kQK), planes + dr_off + (size_t)n * (g.K / 16),
                      (uint32_t)(cnt * (g.K / 16)), bar);
    });
}

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Thread 0: the CTA's shares of one layer's four GEMMs (and its norm weights) into L2, so
// that their staging copies a phase later find them there.
__device__ __forceinline__ void prefetch_layer(const RowStepArgs& a, const RowLayer* L, int cta, int G) {
    for (int i = 0; i < 4; ++i) {
        const RowGemm& g = a.gm[i];
        const unsigned char* w = L->w[i];
        const size_t dr_off = q8p_dr_offset(g.N, g.K);
        share_runs(g, cta_span(g, cta, G), [&](int n, int, int cnt) {
            prefetch_l2(w + (size_t)n * g.K, (uint32_t)(cnt * g.K));
            prefetch_l2(w + dr_off + (size_t)n * (g.K / 16), (uint32_t)(cnt * (g.K / 16)));
        });
    }
    prefetch_l2(L->in_norm, (uint32_t)a.hidden * 4);
    prefetch_l2(L->post_norm, (uint32_t)a.hidden * 4);
}

// The activation row in shared memory is stored permuted within each 512-column slice:
// column c*512 + l*16 + 4h + e (lane l's 16 values, piece h) sits at c*512 + h*128 + l*4 + e,
// so that the four 16 B loads of a warp's lanes read consecutive chunks (no bank conflict).
__device__ __forceinline__ int act_index(int j) {
    return (j & ~511) | (((j >> 2) & 3) << 7) | (((j >> 4) & 31) << 2) | (j & 3);
}

// Lane sums of unit u: for each of its 4 rows, this lane's 16 columns of the CUDA-core
// kernel's arithmetic (the fp32 FMA chain, then one multiply-add by the block's scale).
__device__ __forceinline__ void unit_lane_sums(const RowGemm& g, const Span& s, const unsigned char* sq,
                                               const __half* sd, const float* act, int u, int lane, float (&acc)[4]) {
    const int K = g.K;
    const int blk = u / g.ks;                 // row block (SwiGLU: gate or up block of a pair)
    const int c = u - blk * g.ks;             // K slice
    const int rr0 = g.swiglu ? (blk & 1) * 4 * s.nb + 4 * (blk >> 1) : 4 * blk;
    const int k0 = c * kSlice + lane * kWpl;
    uint4 q[4];
    float dsc[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        q[r] = lds128(sq + (size_t)(rr0 + r) * K + k0);
        dsc[r] = __half2float(sd[(size_t)(rr0 + r) * (K / kQK) + k0 / kQK]);
    }
    float x[kWpl];
#pragma unroll
    for (int h = 0; h < kWpl / 4; ++h) {
        const float4 t = *reinterpret_cast<const float4*>(act + c * kSlice + h * 128 + lane * 4);
        x[4 * h] = t.x; x[4 * h + 1] = t.y; x[4 * h + 2] = t.z; x[4 * h + 3] = t.w;
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        // int8 -> f32 exactly: the byte q + 128 under the exponent of 2^23 reads as 2^23 + q + 128
        const uint32_t wb[4] = {q[r].x, q[r].y, q[r].z, q[r].w};
        float wf[kWpl];
#pragma unroll
        for (int j4 = 0; j4 < kWpl / 4; ++j4) {
            const uint32_t v = wb[j4] ^ 0x80808080u;
#pragma unroll
            for (int b = 0; b < 4; ++b)
                wf[4 * j4 + b] = __int_as_float((int)__byte_perm(v, 0x4B000000u, 0x7540u + (unsigned)b)) - 8388736.0f;
        }
        float sq_ = 0.0f;
#pragma unroll
        for (int j = 0; j < kWpl; ++j) sq_ = fmaf(wf[j], x[j], sq_);
        acc[r] = 0.0f;
        acc[r] = fmaf(dsc[r], sq_, acc[r]);
    }
}

// Every unit of the warp: 4 dot products of 512 columns of the staged rows with act; the
// 4 sums of unit u land in red[u]. The unit's four rows are consecutive staged rows. The
// 4 lane sums are reduced over the warp by halving exchanges (16 and 8 lanes apart, each
// lane keeping half of the values it holds, then 4, 2, 1 apart): every partial sum pairs
// the same lanes in the same order as an xor-shuffle reduction of each value over 16, 8,
// 4, 2, 1 (the CUDA-core kernel's), so the totals are the same bits, with 6 shuffles
// instead of 20. Lane 8r ends with row r.
__device__ __forceinline__ void dot_units(const RowGemm& g, const Span& s, const unsigned char* sq, const __half* sd,
                                          const float* act, float (*red)[4], int warp, int lane) {
#pragma unroll 1
    for (int u = warp; u < s.n_units; u += kWarps) {
        float v[4];
        unit_lane_sums(g, s, sq, sd, act, u, lane, v);
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const bool b = lane & 16;
            const float keep = b ? v[k + 2] : v[k];
            const float send = b ? v[k] : v[k + 2];
            v[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
        {
            const bool b = lane & 8;
            const float keep = b ? v[1] : v[0];
            const float send = b ? v[0] : v[1];
            v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 4);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
        v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
        if ((lane & 7) == 0) red[u][lane >> 3] = v[0];
    }
}

// Norm weights [n] into shared memory by cp.async (waited for by the next poll).
__device__ __forceinline__ void prefetch_norm(float* dst, const float* src, int n) {
    for (int i = 4 * threadIdx.x; i < n; i += 4 * kThreads) cp_async16(dst + i, src + i, true);
    cp_async_commit();
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
    cp_async_wait<0>();     // this thread's norm-weight prefetch, if any
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


__global__ void __launch_bounds__(kThreads, 1) row_step_kernel(const RowStepArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    RowSmem& S = *reinterpret_cast<RowSmem*>(smem_raw);
    const int Hd = a.hidden;
    float* act = S.buf;
    float* xr = S.buf + act_floats(a.hidden, a.ffn);   // this CTA's copy of the residual stream
    float* part = xr + Hd;                             // the sum the next norm adds to it
    float* nrm_in = part + Hd;                         // the layer's norm weights, prefetched
    float* nrm_post = nrm_in + Hd;
    unsigned char* sq = reinterpret_cast<unsigned char*>(S.buf) + stage_offset(a.hidden, a.ffn);
    __half* sd = reinterpret_cast<__half*>(sq + a.stage_q_bytes);
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
    if (len_bad) {
        // the row's attention would be skipped, so its words would never come: flag the row
        // and leave before anything is written (the same for every CTA)
        if (cta == 0 && threadIdx.x == 0) record_error(a.err, kDevErrBadLen);
        return;
    }
    const int p_begin = split * a.pps;
    const int p_end = min(n_row_pages, p_begin + a.pps);
    const bool item = cta < a.n_splits * kHkv && !len_bad && p_begin < n_row_pages;
    const int n_valid = min(a.n_splits, (n_row_pages + a.pps - 1) / max(a.pps, 1));
    const int p_last = n_row_pages - 1;
    const bool owner = item && p_last >= p_begin && p_last < p_end;   // the token's page is in this split
    const int* bt = a.block_table + (size_t)a.slot[0] * a.bt_stride;
    const size_t page_elems = (size_t)kHkv * attn::TILE_HALVES;

    if (threadIdx.x == 0) {
        for (int w = 0; w < kAttnNW; ++w)
            for (int s = 0; s < kRowStages; ++s) mbar_init(&S.att.bars[w][s], 1);
        mbar_init(&S.wbar, 1);
        for (int k = 0; k < kLmSlots; ++k) mbar_init(&S.lmbar[k], 1);
        fence_mbar_init();
    }
    prefetch_norm(nrm_in, a.layers[0].in_norm, Hd);
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
    cp_async_wait<0>();
    __syncthreads();

    // the staged weights: issued by the last warp's lane 0 (whose warp has no share of the
    // phases' output rows, so the words go out without waiting for it) as soon as the
    // buffer is free, waited for by every thread before its dot products
    const bool issuer = threadIdx.x == kThreads - 32;
    uint32_t wpar = 0u;
    bool wpend = false;
    auto stage = [&](int gi, const unsigned char* planes) {
        if (issuer) stage_weights(a.gm[gi], cta_span(a.gm[gi], cta, G), planes, sq, sd, &S.wbar);
        wpend = true;
    };
    stage(0, a.layers[0].w[0]);
    if (issuer) prefetch_layer(a, a.layers, cta, G);

    auto emit_act = [&](int j, float y) { act[act_index(j)] = pair_value(y); };
    // the page ring's barriers are initialised once; bit s = parity of stage s's next phase
    uint32_t ring_ph = 0u;
    int nw = 0, issued = 0;        // this warp's pages of the item and copies in flight
    // The item's page copies of layer l start (attention warps); the ring's shared memory
    // was last read and patched by generic accesses, hence the proxy fence.
    auto start_pages = [&](int l) {
        if (item) {
            if (lane == 0) fence_proxy_async_smem();
            __syncwarp();
            const __half* hb = a.pool + (size_t)l * a.layer_stride + (size_t)h * attn::TILE_HALVES;
            nw = attn::warp_page_count(p_end - p_begin, warp, kAttnNW);
            nw = attn::warp_check_pages(at, bt, p_begin, nw, warp, lane, kAttnNW);
            issued = attn::warp_issue_first(S.att, bt, p_begin, nw, hb, page_elems, warp, lane);
        }
    };
    start_pages(0);

    // The layer loop. The four GEMV phases (A: QKV, C: o_proj, D: gate|up, E: down; GEMM gi =
    // 0..3) run one code path with CTA-uniform parameters, and B (attention) follows A inside
    // it, so that each piece of code appears once: the kernel's instructions then stay in
    // the SM's instruction cache from layer to layer.
    bool ok = true;
    for (int l = 0; l < a.n_layers && ok; ++l) {
        const RowLayer* Lp = a.layers + l;
        const uint32_t tag = tag0 + (uint32_t)l;
        __half* pool_l = a.pool + (size_t)l * a.layer_stride;
        at.pool_layer = pool_l;

        for (int gi = 0; gi < 4; ++gi) {
            // ---- the phase's input: the previous phase's words; the next norm's weights
            if (gi == 1) prefetch_norm(nrm_post, Lp->post_norm, Hd);
            if (gi == 3) {
                if (l + 1 < a.n_layers) prefetch_norm(nrm_in, Lp[1].in_norm, Hd);
                else if (cta == 0 || a.lm) prefetch_norm(nrm_in, a.final_norm, Hd);
            }
            const bool pairs = gi == 1 || gi == 3;   // attention output, SwiGLU output: f16 pairs
            if (gi != 0 || l > 0) {
                const unsigned long long* src = gi == 0 ? a.w_dn : gi == 1 ? a.w_att : gi == 2 ? a.w_o : a.w_h;
                const int n = gi == 1 ? kHq * D : gi == 3 ? a.ffn : Hd;
                ok = poll_words(a, src, n, gi == 0 ? tag - 1u : tag, [&](int i, uint32_t v) {
                    if (pairs) act[act_index(i)] = pair_sum(v);
                    else part[i] = __uint_as_float(v);
                });
                if (!ok) break;
            }
            if (gi == 0 || gi == 2) {
                const bool first = gi == 0 && l == 0;   // the embedding row: nothing to add
                residual_norm_row<8, false>(xr, first ? nullptr : reinterpret_cast<const float4*>(part), 0,
                                            first ? 0 : 1, Hd, gi == 0 ? nrm_in : nrm_post, a.eps,
                                            first ? nullptr : xr, S.sh, emit_act);
            }
            // ---- the staged weights, the dot products, the next staging, the words out
            {
                const bool got = mbar_wait_bounded(&S.wbar, wpar);
                wpar ^= 1u;
                wpend = false;
                if (__syncthreads_or(!got)) {
                    if (threadIdx.x == 0) {
                        record_error(a.err, kDevErrTimeout);
                        atomicExch(&a.ctl->abort, 1);
                    }
                    ok = false;
                    break;
                }
            }
            const RowGemm& g = a.gm[gi];
            const Span sp = cta_span(g, cta, G);
            dot_units(g, sp, sq, sd, act, S.red, warp, lane);
            __syncthreads();
            if (gi < 3) stage(gi + 1, Lp->w[gi + 1]);
            else if (l + 1 < a.n_layers) stage(0, Lp[1].w[0]);
            finish_units(g, sp, S.red, gi == 0 ? a.w_qkv : gi == 1 ? a.w_o : gi == 2 ? a.w_h : a.w_dn, tag);
            if (gi == 0 && issuer && l + 1 < a.n_layers) prefetch_layer(a, Lp + 1, cta, G);
            if (gi == 3 && l + 1 < a.n_layers) start_pages(l + 1);
            if (gi != 0 || !item) continue;

            // ---------------- B: kernel (1) for the item's heads, then attention
            bool hok = true;
            if (warp >= 4) {
                const int v = warp - 4;     // q heads 2h, 2h+1, then K and V of head h
                const int j = v < 2 ? 2 * h + v : (v == 2 ? kHq + h : kHq + kHkv + h);
                if (v < 2 || owner) {
                    AppendArgs app{};
                    app.n_part = 1; app.M = 1; app.pos = a.pos; app.slot = a.slot;
                    app.block_table = a.block_table; app.bt_stride = a.bt_stride; app.n_pages = a.n_pages;
                    app.qn_w = Lp->q_norm; app.kn_w = Lp->k_norm; app.Hq = kHq; app.Hkv = kHkv; app.eps = a.eps;
                    app.q_scale = a.q_scale; app.rope = a.rope; app.max_pos = a.max_pos;
                    app.pool_layer = pool_l; app.q_out = nullptr; app.err = a.err;
                    // the head's norm weights, rotation and page do not depend on the words
                    const HeadRowMeta meta = qkv_head_meta(app, 0, j, lane);
                    float x[4];
                    hok = poll_thread(a, tag,
                                      [&](int u) -> const unsigned long long* {
                                          return u < 4 ? a.w_qkv + j * D + lane + 32 * u : nullptr;
                                      },
                                      [&](int u, uint32_t w) { x[u] = __fadd_rn(0.0f, __uint_as_float(w)); });
                    // the lanes poll their own words, but the head's norm shuffles over the
                    // whole warp: all lanes go on, or none
                    hok = __all_sync(0xffffffffu, hok);
                    if (hok)
                        qkv_head_apply(app, meta, 0, j, lane, x, v < 2 ? S.att.q[v] : nullptr,
                                       v < 2 ? nullptr : S.newkv + (v - 2) * D);
                }
            }
            if (__syncthreads_or(!hok)) {
                ok = false;
                break;
            }
            // every warp of the CTA takes pages
            const int t = threadIdx.x;
            if (t < D) {
                S.att.q[0][t] = S.att.q[0][t] * attn::kLog2e;
                S.att.q[1][t] = S.att.q[1][t] * attn::kLog2e;
            }
            __syncthreads();
            const int rel = p_last - p_begin;
            const int patch_i = owner && warp == rel % kAttnNW ? rel / kAttnNW : -1;
            const __half* head_base = pool_l + (size_t)h * attn::TILE_HALVES;
            attn::warp_pages(at, S.att, bt, p_begin, nw, issued, n_kv, head_base, page_elems,
                             owner ? S.newkv : nullptr, patch_i, pos % kPageTokens, warp, lane, ring_ph);
            ring_ph = attn::ring_phase_after<kRowStages>(ring_ph, nw);
            issued = 0;
            __syncthreads();
            if (a.n_splits == 1) {
                if (t < D)
                    attn::merge_warps(S.att, t, [&](int hq, float, float Ls, float Os) {
                        st_word(a.w_att + (2 * h + hq) * D + t, pack_pair(Ls > 0.0f ? Os / Ls : 0.0f), tag);
                    });
            } else {
                // partials to the scratch; the split that finishes last merges the head's
                // splits and writes its words
                if (t < D)
                    attn::merge_warps(S.att, t, [&](int hq, float M, float Ls, float Os) {
                        attn::merge_store(at, split, h, 0, t, hq, M, Ls, Os);
                    });
                __syncthreads();
                if (t == 0) {
                    __threadfence();
                    const int old = atomicAdd(&a.ctl->att_cnt[h], 1);
                    S.last = old == n_valid - 1;
                    if (S.last) {
                        __threadfence();
                        a.ctl->att_cnt[h] = 0;
                    }
                }
                __syncthreads();
                if (S.last && warp < 2) {
                    const int H = 2 * h + warp;
                    attn::combine_head<true>(at, 0, H, lane, [&](int d, float v) {
                        st_word(a.w_att + H * D + d, pack_pair(v), tag);
                    });
                }
            }
        }
    }
    if (!ok) {
        // nothing may land in shared memory after the CTA has left: wait (bounded) for the
        // copies in flight
        cp_async_wait<0>();
        if (wpend) (void)mbar_wait_bounded(&S.wbar, wpar);
        if (item)
            for (int k = 0; k < issued; ++k) {
                const int st = k % kRowStages;
                const bool done = mbar_wait_bounded(&S.att.bars[warp][st],
                                                    ((uint32_t)(k / kRowStages) & 1u) ^ ((ring_ph >> st) & 1u));
                (void)__all_sync(0xffffffffu, done);
            }
        return;
    }

    // ---------------- F: the final norm, then (a.lm) the lm_head and the argmax
    const uint32_t tag_last = tag0 + (uint32_t)a.n_layers - 1u;
    if (!a.lm) {
        // the lm_head runs as its own launch: CTA 0 leaves the final norm's pair for it
        if (cta != 0) return;
        if (!poll_words(a, a.w_dn, Hd, tag_last, [&](int i, uint32_t v) { part[i] = __uint_as_float(v); })) return;
        residual_norm_row<8, false>(xr, reinterpret_cast<const float4*>(part), 0, 1, Hd, nrm_in, a.eps, xr, S.sh,
                                    [&](int j, float y) { split_store(y, a.xn16, a.xn_lo, (size_t)j); });
        __syncthreads();
        for (int i = threadIdx.x; i < Hd; i += kThreads) a.x_a[i] = xr[i];
        // every CTA read the sequence number at its start, long before this point (its rows
        // of every phase came before)
        if (threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(&a.ctl->seq) = seq + 1u;
        return;
    }
    // Every CTA normalises the row itself, then computes the logits of its 64-row vocab
    // tiles with the CUDA-core lm_head kernel's arithmetic (a warp per 4 rows over all of
    // K, its 512-column slices in order), streamed through kLmSlots chunks of kLmRows
    // rows in the attention ring's shared memory; each tile's first maximum goes to
    // amax_val / amax_idx, and the CTA that finishes last reduces them as the argmax
    // reduce kernel does.
    if (!poll_words(a, a.w_dn, Hd, tag_last, [&](int i, uint32_t v) { part[i] = __uint_as_float(v); })) return;
    residual_norm_row<8, false>(xr, reinterpret_cast<const float4*>(part), 0, 1, Hd, nrm_in, a.eps, xr, S.sh,
                                [&](int j, float y) {
                                    act[act_index(j)] = pair_value(y);
                                    if (cta == 0) split_store(y, a.xn16, a.xn_lo, (size_t)j);
                                });
    __syncthreads();
    if (cta == 0)
        for (int i = threadIdx.x; i < Hd; i += kThreads) a.x_a[i] = xr[i];
    {
        const int K = Hd;
        const int tile0 = (int)((long long)cta * a.lm_tiles / G);
        const int tile1 = (int)((long long)(cta + 1) * a.lm_tiles / G);
        const int n_chunks = 2 * (tile1 - tile0);
        const uint32_t slot_bytes = (uint32_t)(kLmRows * (K + K / 16));
        unsigned char* ring = reinterpret_cast<unsigned char*>(&S.att.tiles[0][0][0]);
        const size_t dr_off = q8p_dr_offset(a.vocab, K);
        auto issue = [&](int k) {
            unsigned char* slot = ring + (size_t)(k % kLmSlots) * slot_bytes;
            const size_t row0 = (size_t)64 * tile0 + (size_t)kLmRows * k;
            uint64_t* bar = &S.lmbar[k % kLmSlots];
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(bar, slot_bytes);
            bulk_copy_g2s(slot, a.lm_q + row0 * K, (uint32_t)(kLmRows * K), bar);
            bulk_copy_g2s(slot + kLmRows * K, a.lm_q + dr_off + row0 * (K / 16), (uint32_t)(kLmRows * K / 16), bar);
        };
        if (issuer)
            for (int k = 0; k < kLmSlots && k < n_chunks; ++k) issue(k);
        bool lok = true;
        int k = 0;
        for (; k < n_chunks; ++k) {
            const bool got = mbar_wait_bounded(&S.lmbar[k % kLmSlots], (uint32_t)(k / kLmSlots) & 1u);
            if (__syncthreads_or(!got)) {
                if (threadIdx.x == 0) record_error(a.err, kDevErrTimeout);
                lok = false;
                break;
            }
            const unsigned char* slot = ring + (size_t)(k % kLmSlots) * slot_bytes;
            const __half* dsl = reinterpret_cast<const __half*>(slot + kLmRows * K);
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 2
            for (int sl = 0; sl < K / kSlice; ++sl) {
                const int k0 = sl * kSlice + lane * kWpl;
                float x[kWpl];
#pragma unroll
                for (int hh = 0; hh < kWpl / 4; ++hh) {
                    const float4 t4 = *reinterpret_cast<const float4*>(act + sl * kSlice + hh * 128 + lane * 4);
                    x[4 * hh] = t4.x; x[4 * hh + 1] = t4.y; x[4 * hh + 2] = t4.z; x[4 * hh + 3] = t4.w;
                }
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int rr = 4 * warp + r;
                    const uint4 q = lds128(slot + (size_t)rr * K + k0);
                    const float dsc = __half2float(dsl[(size_t)rr * (K / kQK) + k0 / kQK]);
                    const uint32_t wb[4] = {q.x, q.y, q.z, q.w};
                    float wf[kWpl];
#pragma unroll
                    for (int j4 = 0; j4 < kWpl / 4; ++j4) {
                        const uint32_t v = wb[j4] ^ 0x80808080u;
#pragma unroll
                        for (int b = 0; b < 4; ++b)
                            wf[4 * j4 + b] =
                                __int_as_float((int)__byte_perm(v, 0x4B000000u, 0x7540u + (unsigned)b)) - 8388736.0f;
                    }
                    float sq_ = 0.0f;
#pragma unroll
                    for (int j = 0; j < kWpl; ++j) sq_ = fmaf(wf[j], x[j], sq_);
                    acc[r] = fmaf(dsc, sq_, acc[r]);
                }
            }
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
            const int tp = (k >> 1) & 1;
            if (lane == 0)
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    float v = 0.0f;
                    v += acc[r];
                    const int rt = (k & 1) * kLmRows + 4 * warp + r;   // row within the tile
                    S.tilev[tp][rt] = v;
                    if (a.logits) a.logits[(size_t)64 * tile0 + (size_t)kLmRows * k + 4 * warp + r] = v;
                }
            __syncthreads();   // the chunk's slot is free; the tile's values are complete
            if (issuer && k + kLmSlots < n_chunks) issue(k + kLmSlots);
            if ((k & 1) && warp == 0) {
                // the tile's first maximum (NaN never wins), ties to the lower index
                float bv = -INFINITY;
                int bi = 0x7fffffff;
                const int row_base = 64 * (tile0 + (k >> 1));
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const int rr = lane + 32 * hh;
                    const float v = S.tilev[tp][rr];
                    if (v > bv) { bv = v; bi = row_base + rr; }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
                }
                if (lane == 0) {
                    a.amax_val[tile0 + (k >> 1)] = bv;
                    a.amax_idx[tile0 + (k >> 1)] = bi;
                }
            }
        }
        if (!lok) {
            // wait (bounded) for the chunks still in flight before leaving
            const int issued_to = min(n_chunks, k + kLmSlots);
            for (int kk = k + 1; kk < issued_to; ++kk)
                (void)mbar_wait_bounded(&S.lmbar[kk % kLmSlots], (uint32_t)(kk / kLmSlots) & 1u);
            return;
        }
    }
    // the tile maxima are out: the CTA that finishes last reduces them
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const int old = atomicAdd(&a.ctl->lm_cnt, 1);
        S.last = old == G - 1;
        if (S.last) {
            __threadfence();
            a.ctl->lm_cnt = 0;
        }
    }
    __syncthreads();
    if (S.last) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int t = threadIdx.x; t < a.lm_tiles; t += kThreads) {
            const float v = __ldcg(a.amax_val + t);
            const int i = __ldcg(a.amax_idx + t);
            if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) { S.rv[warp] = bv; S.ri[warp] = bi; }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int w = 1; w < kWarps; ++w)
                if (S.rv[w] > bv || (S.rv[w] == bv && S.ri[w] < bi)) { bv = S.rv[w]; bi = S.ri[w]; }
            // all-NaN or empty rows fall back to index 0, as the reference's scan does
            if (bi == 0x7fffffff) bi = 0;
            a.next[0] = bi;
            if (a.feed_tok) a.feed_tok[0] = bi;
            if (a.feed_pos) a.feed_pos[0] += 1;
        }
    }
    if (cta == 0 && threadIdx.x == 0) *reinterpret_cast<volatile uint32_t*>(&a.ctl->seq) = seq + 1u;
}

}  // namespace

// Bytes of the largest share of q rows one CTA stages (its row blocks of one GEMM x K).
static size_t stage_q_bytes(const RowGemm* gm, int grid) {
    size_t m = 0;
    for (int i = 0; i < 4; ++i) {
        const int total = gm[i].swiglu ? gm[i].N / 8 : gm[i].N / 4;
        const size_t rows = (size_t)((total + grid - 1) / grid) * (gm[i].swiglu ? 8 : 4);
        m = rows * gm[i].K > m ? rows * gm[i].K : m;
    }
    return m;
}

static size_t smem_bytes(int hidden, int ffn, size_t sq_bytes) {
    return offsetof(RowSmem, buf) + stage_offset(hidden, ffn) + sq_bytes + sq_bytes / 16;
}

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
    return smem_bytes(hidden, ffn, stage_q_bytes(gm, grid)) <= 227 * 1024;
}

bool row_step_lm_fits(int hidden, int vocab) {
    // the CUDA-core lm_head's argmax form at one row: one warp per 4 rows over all of K, in
    // one or two slices of 512 columns
    return (hidden == 512 || hidden == 1024) && vocab % 64 == 0 &&
           (size_t)kLmSlots * kLmRows * (hidden + hidden / 16) <= sizeof(((ASmem*)nullptr)->tiles);
}

size_t row_step_words(int hidden, int ffn) {
    return (size_t)kQkvN + (size_t)kHq * D + 2 * (size_t)hidden + (size_t)ffn;
}

cudaError_t configure_row_step() {
    return cudaFuncSetAttribute(row_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
}

cudaError_t launch_row_step(const RowStepArgs& args, int grid, cudaStream_t s) {
    RowStepArgs a = args;
    a.stage_q_bytes = (int)stage_q_bytes(a.gm, grid);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem_bytes(a.hidden, a.ffn, (size_t)a.stage_q_bytes);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, row_step_kernel, a);
}

}  // namespace fa
