// The body of kernel (2), paged GQA decode attention for one (split, KV head, row), as
// device functions: the stand-alone kernel (k_attention.cu) and the one-row persistent
// step (k_row_step.cu) run the same code, so their outputs are the same bits.
//
// NW warps (4, or 8 for steps of at most two rows); warp w owns pages w, w+NW, ... of the
// split and streams them through a private STAGES-deep shared-memory ring: lane 0 issues
// one 8 KiB cp.async.bulk (K and V of this head in this page) per stage, completion is
// counted on an mbarrier and every wait is bounded in time. Compute per page (lane = (token parity par, 8-dim chunk c)):
//   QK  : 8 x 16 B shared loads, 16 fp32 FMAs each (two tokens side by side as packed
//         pairs), then a 16-lane transpose reduction leaves lane r of each half-warp with
//         the score of (token 2*(r/2)+par, head r%2)
//   softmax: max and sum by xor shuffles, running (max, sum) per head in log2 units
//   PV  : p broadcast through shared memory, 8 x 16 B loads, 16 FMAs each
// The NW warps then merge in shared memory; with several splits the un-normalised partials
// go to the scratch buffer and the split merge (combine_head) finishes them.
#pragma once

#include "fa_kernels.cuh"

namespace fa {
namespace attn {

constexpr int D = 128;
constexpr int TILE_HALVES = 2 * kPageTokens * D;   // K then V of one head in one page
constexpr uint32_t TILE_BYTES = TILE_HALVES * 2;   // 8192
constexpr float kLog2e = 1.4426950408889634f;

template <int STAGES, int NW>
struct Smem {
    __half tiles[NW][STAGES][TILE_HALVES];
    uint64_t bars[NW][STAGES];
    float q[2][D];
    float2 pbuf[NW][32];            // each p twice: the PV products take it as a packed pair
    float acc[NW][2][D];
    float ml[NW][4];
};

// Two fp32 fused multiply-adds in one instruction (sm_100 packs a pair of fp32 lanes): each
// half is the same correctly rounded fma as fmaf, so results do not change.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(r)
        : "l"(*reinterpret_cast<unsigned long long*>(&a)), "l"(*reinterpret_cast<unsigned long long*>(&b)),
          "l"(*reinterpret_cast<unsigned long long*>(&c)));
    return *reinterpret_cast<float2*>(&r);
}

__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    unsigned long long r;
    asm("mul.rn.f32x2 %0, %1, %2;"
        : "=l"(r)
        : "l"(*reinterpret_cast<unsigned long long*>(&a)), "l"(*reinterpret_cast<unsigned long long*>(&b)));
    return *reinterpret_cast<float2*>(&r);
}

__device__ __forceinline__ void load8(const __half* p, float (&f)[8]) {
    const uint4 v = lds128(p);
    float2 a = h2_to_f2(v.x), b = h2_to_f2(v.y), c = h2_to_f2(v.z), d = h2_to_f2(v.w);
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
    f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

// Reduce 16 values across the 16 lanes of a half-warp so that lane r ends with
// the total of value index r. Each stage halves the count kept per lane.
__device__ __forceinline__ float transpose_reduce16(float (&v)[16], int lane) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const bool b = lane & 8;
        const float keep = b ? v[k + 8] : v[k];
        const float send = b ? v[k] : v[k + 8];
        v[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const bool b = lane & 4;
        const float keep = b ? v[k + 4] : v[k];
        const float send = b ? v[k] : v[k + 4];
        v[k] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const bool b = lane & 2;
        const float keep = b ? v[k + 2] : v[k];
        const float send = b ? v[k] : v[k + 2];
        v[k] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    }
    {
        const bool b = lane & 1;
        const float keep = b ? v[1] : v[0];
        const float send = b ? v[0] : v[1];
        v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
    }
    return v[0];
}

// The row's context must be 1 .. bt_stride * 16 tokens and pages_per_split * n_splits
// must reach its last page; otherwise the kernel and the merge leave the row untouched.
__device__ __forceinline__ bool row_len_bad(const AttnArgs& a, int n_kv, int n_row_pages) {
    return n_kv <= 0 || n_row_pages > a.bt_stride ||
           (long long)a.pages_per_split * a.n_splits < (long long)n_row_pages;
}

// Output as f32 and/or as the (hi, lo) f16 pair the o_proj GEMM consumes.
__device__ __forceinline__ void store_out(const AttnArgs& a, size_t o, float v) {
    if (a.out16) {
        const __half h = __float2half_rn(v);
        a.out16[o] = h;
        if (a.out16_lo) a.out16_lo[o] = __float2half_rn(__fsub_rn(v, __half2float(h)));
    }
    if (a.out32) a.out32[o] = v;
}

// Pages warp `warp` of nwarps owns in a split of `span` pages.
__device__ __forceinline__ int warp_page_count(int span, int warp, int nwarps) {
    return span > warp ? (span - warp + nwarps - 1) / nwarps : 0;
}

// The warp's pages checked against the pool (all lanes call): 0 and an error flag when
// any block-table entry is outside it, else nw.
__device__ __forceinline__ int warp_check_pages(const AttnArgs& a, const int* bt, int p_begin, int nw, int warp,
                                                int lane, int nwarps) {
    bool bad = false;
    for (int i = lane; i < nw; i += 32) {
        const int pg = bt[p_begin + warp + nwarps * i];
        bad |= (pg < 0 || pg >= a.n_pages);
    }
    if (__any_sync(0xffffffffu, bad)) {
        if (lane == 0) record_error(a.err, kDevErrBadPage);
        return 0;
    }
    return nw;
}

// Lane 0 issues the copies of the warp's first min(STAGES, nw) pages; every lane gets
// the number issued.
template <int STAGES, int NW>
__device__ __forceinline__ int warp_issue_first(Smem<STAGES, NW>& S, const int* bt, int p_begin, int nw,
                                                const __half* head_base, size_t page_elems, int warp, int lane) {
    int issued = 0;
    if (lane == 0) {
        for (; issued < STAGES && issued < nw; ++issued) {
            const int pg = bt[p_begin + warp + NW * issued];
            mbar_arrive_expect_tx(&S.bars[warp][issued], TILE_BYTES);
            bulk_copy_g2s(S.tiles[warp][issued], head_base + (size_t)pg * page_elems, TILE_BYTES,
                          &S.bars[warp][issued]);
        }
    }
    return __shfl_sync(0xffffffffu, issued, 0);
}

// Phase parity of the next wait on each stage of a warp's ring (bit s), after a round of
// nw pages that began at ph0: every page completes one phase of its stage's barrier.
template <int STAGES>
__device__ __forceinline__ uint32_t ring_phase_after(uint32_t ph0, int nw) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
        const int uses = nw > s ? (nw - s + STAGES - 1) / STAGES : 0;
        ph0 ^= (uint32_t)(uses & 1) << s;
    }
    return ph0;
}

// One warp's pages: scores, online softmax and PV products, then the warp's partial
// (acc, max, sum) into S.acc[warp] / S.ml[warp]. q comes from S.q (the caller has
// synchronised after writing it); `issued` copies are in flight; the barrier of stage s
// next completes the phase of parity bit s of ph0 (0 for fresh barriers).
// patch (or nullptr): the K row then the V row (2 x 128 f16) of token patch_t of the
// warp's page patch_i, written over the page's shared-memory copy once it has landed.
template <int STAGES, int NW>
__device__ __forceinline__ void warp_pages(const AttnArgs& a, Smem<STAGES, NW>& S, const int* bt, int p_begin, int nw,
                                           int issued, int n_kv, const __half* head_base, size_t page_elems,
                                           const __half* patch, int patch_i, int patch_t, int warp, int lane,
                                           uint32_t ph0 = 0u) {
    const int c = lane & 15;
    const int par = lane >> 4;
    // q of both heads for this lane's 8 dims, each value twice: a QK product runs two
    // tokens' dot products side by side (packed fp32 pairs), in the same order as one at a time
    float2 q0[8], q1[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        q0[k] = make_float2(S.q[0][8 * c + k], S.q[0][8 * c + k]);
        q1[k] = make_float2(S.q[1][8 * c + k], S.q[1][8 * c + k]);
    }
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
    // PV accumulators of the lane's 8 dims as 4 packed pairs per head
    float2 acc0[4], acc1[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) { acc0[k] = make_float2(0.0f, 0.0f); acc1[k] = make_float2(0.0f, 0.0f); }

    int i = 0;
    bool ok = true;
    for (; i < nw; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = ((uint32_t)(i / STAGES) & 1u) ^ ((ph0 >> s) & 1u);
        const bool got = mbar_wait_bounded(&S.bars[warp][s], ph);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }

        const int t0 = (p_begin + warp + NW * i) * kPageTokens;
        const int nvalid = min(kPageTokens, n_kv - t0);
        __half* Kt = S.tiles[warp][s];
        const __half* Vt = Kt + kPageTokens * D;
        if (patch && i == patch_i) {
            // lanes 0-15 write the K row, 16-31 the V row, 16 B each
            const uint4 v = reinterpret_cast<const uint4*>(patch)[lane];
            __half* dst = Kt + (lane < 16 ? 0 : kPageTokens * D) + patch_t * D + 8 * (lane & 15);
            *reinterpret_cast<uint4*>(dst) = v;
            __syncwarp();
        }

        float part[16];
#pragma unroll
        for (int ii = 0; ii < 8; ii += 2) {
            // tokens 2ii+par and 2(ii+1)+par side by side
            float fa[8], fb[8];
            load8(Kt + (2 * ii + par) * D + 8 * c, fa);
            load8(Kt + (2 * ii + 2 + par) * D + 8 * c, fb);
            float2 s0 = make_float2(0.0f, 0.0f), s1 = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float2 kk = make_float2(fa[k], fb[k]);
                s0 = ffma2(q0[k], kk, s0);
                s1 = ffma2(q1[k], kk, s1);
            }
            part[2 * ii] = s0.x;
            part[2 * ii + 1] = s1.x;
            part[2 * ii + 2] = s0.y;
            part[2 * ii + 3] = s1.y;
        }
        const float tot = transpose_reduce16(part, lane);
        const int r = lane & 15;
        const int hh = r & 1;
        const int tt = 2 * (r >> 1) + par;
        const float sc = tt < nvalid ? tot : -INFINITY;

        float mx = sc;
#pragma unroll
        for (int o = 2; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float mxo = __shfl_xor_sync(0xffffffffu, mx, 1);
        const float mn0 = fmaxf(m0, hh ? mxo : mx);
        const float mn1 = fmaxf(m1, hh ? mx : mxo);
        const float al0 = exp2f(m0 - mn0);
        const float al1 = exp2f(m1 - mn1);
        const float p = exp2f(sc - (hh ? mn1 : mn0));
        float ps = p;
#pragma unroll
        for (int o = 2; o < 32; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
        const float pso = __shfl_xor_sync(0xffffffffu, ps, 1);
        l0 = l0 * al0 + (hh ? pso : ps);
        l1 = l1 * al1 + (hh ? ps : pso);
        m0 = mn0;
        m1 = mn1;

        S.pbuf[warp][lane] = make_float2(p, p);   // lane index = par*16 + 2*ii + hh
        __syncwarp();
        float2 pv[16];
        {
            const float4* pb = reinterpret_cast<const float4*>(&S.pbuf[warp][par * 16]);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float4 t = pb[k];
                pv[2 * k] = make_float2(t.x, t.y);
                pv[2 * k + 1] = make_float2(t.z, t.w);
            }
        }
        {
            const float2 a0 = make_float2(al0, al0), a1 = make_float2(al1, al1);
#pragma unroll
            for (int k = 0; k < 4; ++k) { acc0[k] = fmul2(acc0[k], a0); acc1[k] = fmul2(acc1[k], a1); }
        }
#pragma unroll
        for (int ii = 0; ii < 8; ++ii) {
            if (2 * ii + par < nvalid) {
                float f[8];
                load8(Vt + (2 * ii + par) * D + 8 * c, f);
                const float2 pa = pv[2 * ii], pb = pv[2 * ii + 1];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float2 vv = make_float2(f[2 * k], f[2 * k + 1]);
                    acc0[k] = ffma2(pa, vv, acc0[k]);
                    acc1[k] = ffma2(pb, vv, acc1[k]);
                }
            }
        }
        __syncwarp();
        if (lane == 0 && i + STAGES < nw) {
            fence_proxy_async_smem();
            const int pg = bt[p_begin + warp + NW * (i + STAGES)];
            mbar_arrive_expect_tx(&S.bars[warp][s], TILE_BYTES);
            bulk_copy_g2s(S.tiles[warp][s], head_base + (size_t)pg * page_elems, TILE_BYTES, &S.bars[warp][s]);
        }
        if (i + STAGES < nw) ++issued;
    }

    if (!ok) {
        // A wait gave up: flag it, then wait (bounded again) for this warp's
        // copies still in flight so none lands after the CTA has moved on.
        if (lane == 0) record_error(a.err, kDevErrTimeout);
        for (int k = i; k < issued; ++k) {
            const bool done = mbar_wait_bounded(&S.bars[warp][k % STAGES],
                                                ((uint32_t)(k / STAGES) & 1u) ^ ((ph0 >> (k % STAGES)) & 1u));
            (void)__all_sync(0xffffffffu, done);
        }
        m0 = m1 = -INFINITY;
        l0 = l1 = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) { acc0[k] = make_float2(0.0f, 0.0f); acc1[k] = make_float2(0.0f, 0.0f); }
    }

    float o0[8], o1[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        o0[2 * k] = acc0[k].x; o0[2 * k + 1] = acc0[k].y;
        o1[2 * k] = acc1[k].x; o1[2 * k + 1] = acc1[k].y;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        o0[k] += __shfl_xor_sync(0xffffffffu, o0[k], 16);
        o1[k] += __shfl_xor_sync(0xffffffffu, o1[k], 16);
    }
    if (lane < 16) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            S.acc[warp][0][8 * c + k] = o0[k];
            S.acc[warp][1][8 * c + k] = o1[k];
        }
    }
    if (lane == 0) {
        S.ml[warp][0] = m0; S.ml[warp][1] = m1;
        S.ml[warp][2] = l0; S.ml[warp][3] = l1;
    }
}

// Merge of the NW warps' partials (after a barrier over them), thread d < 128 owning dim
// d: for each of the two query heads hq, the maximum M, the sum L and the output O (warps
// in order), handed to epi(hq, M, L, O).
template <int STAGES, int NW, typename Epi>
__device__ __forceinline__ void merge_warps(const Smem<STAGES, NW>& S, int d, Epi epi) {
#pragma unroll
    for (int hq = 0; hq < 2; ++hq) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, S.ml[w][hq]);
        float L = 0.0f, O = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                const float sc = exp2f(S.ml[w][hq] - M);
                L = fmaf(S.ml[w][2 + hq], sc, L);
                O = fmaf(S.acc[w][hq][d], sc, O);
            }
        }
        epi(hq, M, L, O);
    }
}

// merge_warps' epilogue of kernel (2): the output of query head 2h + hq of row m (one
// split), or the split's partial.
__device__ __forceinline__ void merge_store(const AttnArgs& a, int split, int h, int m, int d, int hq, float M, float L,
                                            float O) {
    const int H = 2 * h + hq;
    if (a.n_splits == 1) {
        const float v = L > 0.0f ? O / L : 0.0f;
        store_out(a, (size_t)m * a.Hq * D + (size_t)H * D + d, v);
    } else {
        const size_t base = ((size_t)m * a.Hq + H) * a.n_splits + split;
        a.part_o[base * D + d] = O;
        if (d == 0) {
            a.part_ml[base * 2] = M;
            a.part_ml[base * 2 + 1] = L;
        }
    }
}

template <bool CG>
__device__ __forceinline__ float ld_part(const float* p) {
    if constexpr (CG) return __ldcg(p);
    else return *p;
}
template <bool CG>
__device__ __forceinline__ float4 ld_part4(const float4* p) {
    if constexpr (CG) return __ldcg(p);
    else return *p;
}

// Merge of the split partials of (row m, query head H) by one warp, lane l owning dims
// 4l..4l+3: the split maxima read by the lanes together, then every output sums its splits
// in split order (the same arithmetic as one thread per dim); out(d, value) for each of the
// lane's dims. CG: read the partials at L2 (they were written by other CTAs of the same
// kernel).
template <bool CG, typename Out>
__device__ __forceinline__ void combine_head(const AttnArgs& a, int m, int H, int lane, Out out) {
    const int n_kv = a.pos[m] + 1;
    const int n_row_pages = (n_kv + kPageTokens - 1) / kPageTokens;
    if (row_len_bad(a, n_kv, n_row_pages)) return;      // flagged by the attention kernel
    const int n_valid = min(a.n_splits, (n_row_pages + a.pages_per_split - 1) / a.pages_per_split);
    const size_t base = ((size_t)m * a.Hq + H) * a.n_splits;
    float M = -INFINITY;
    for (int s = lane; s < n_valid; s += 32) M = fmaxf(M, ld_part<CG>(a.part_ml + (base + s) * 2));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.0f;
    float O[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (M != -INFINITY) {
        for (int s = 0; s < n_valid; ++s) {
            const float sc = exp2f(ld_part<CG>(a.part_ml + (base + s) * 2) - M);
            L = fmaf(ld_part<CG>(a.part_ml + (base + s) * 2 + 1), sc, L);
            const float4 o4 = ld_part4<CG>(reinterpret_cast<const float4*>(a.part_o + (base + s) * D) + lane);
            O[0] = fmaf(o4.x, sc, O[0]);
            O[1] = fmaf(o4.y, sc, O[1]);
            O[2] = fmaf(o4.z, sc, O[2]);
            O[3] = fmaf(o4.w, sc, O[3]);
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) out(4 * lane + j, L > 0.0f ? O[j] / L : 0.0f);
}

}  // namespace attn
}  // namespace fa
