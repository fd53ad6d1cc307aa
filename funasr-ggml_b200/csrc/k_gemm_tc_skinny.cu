// Kernel (4), few-row form on the tensor cores: the Q8_0 weight GEMM of a step with up to
// 128 rows (a decode batch), with the operands swapped:
//
//     C^T[N][M] = W[N][K] . A[M][K]^T,   the MMA's M side = 128 weight rows,
//                                        its N side = the activation rows (16 ... 128)
//
// Two weight forms. The decoder's: Q8_0 planes (q int8 [N][K], block scales d_t), exact
// d*q expanded in shared memory into an f16 pair (W_hi + W_lo, q8_planes.cuh), so a
// product is W_hi*a_hi + W_hi*a_lo + W_lo*a_hi (the dropped W_lo*a_lo is below 2^-22 of
// it) and the kernel streams 34/32 B per weight from HBM. The encoder's: f16 weights
// [N][K] (one rounding at load), W*a_hi + W*a_lo. Accumulation is fp32 in TMEM; outputs
// are fp32 split-K partials [split][M][N] or per-64-column row maxima for the lm_head
// argmax. Why swap: with 128-row activation
// tiles a step of 16 rows still pays for a 128 x 128 fp32 accumulator per unit (64 KiB of
// epilogue and partials) and for 64 KiB of activation copies per stage pair; here a unit's
// accumulator is 128 x BNA (8-32 KiB up to 64 rows), a stage holds 16 KiB of weights and
// BNA rows of activations, so six stages fit and each SM keeps ~96 KiB of weights in flight.
//
// Persistent, one CTA per SM, units = (128 weight rows, K chunk). 6 warps (10 for Q8_0):
//   warp 0      TMA producer: the weight tile (64 K x 128 rows: f16 128 B swizzled, or
//               the q tile 64 B x 128 rows and its 2 x 128 scales) and the activation hi /
//               lo tiles (64 K x BNA rows; rows past M read as zeros) per stage; the first
//               stages' weight copies go out before the wait on the previous kernel
//   warp 1      TMEM (two BNA-column accumulators) and tcgen05.mma kind::f16, M=128,
//               N=BNA, K=16, every product of a stage into one accumulator
//   warps 2..5  epilogue: TMEM lanes 32*(warp%4).. are weight rows, columns are
//               activation rows; each warp writes 128 B runs of one activation row
//   warps 6..13 (Q8_0) expand each stage's q tile, half a weight row per thread, into the
//               W_hi / W_lo pair in a TMEM slot (tcgen05.st) that the MMAs read as their
//               A operand; the raw stage and the slot are released when those MMAs complete
// Every mbarrier wait is bounded; a wait that gives up records an error and the CTA
// drains its copies and MMAs before freeing TMEM.
#include "fa_kernels.cuh"
#include "k_append.cuh"
#include "tc_common.cuh"

#include <cuda.h>

#include <utility>

namespace fa {

namespace {

constexpr int WM = 128;             // weight rows per unit
constexpr int BK = 64;
constexpr int CONV_THREADS = 256;   // Q8_0: warps 6..13 expand q into the f16 pair

template <bool Q8>
__host__ __device__ constexpr int threads_for() {
    return Q8 ? 64 + 128 + CONV_THREADS : 64 + 128;
}

// f16 weights: one ring, 6 stages of 16 KiB weights + BNA-row activation pairs up to 64
// rows (at most 192 KiB), 4 at 128 rows (48 KiB each).
template <int BNA>
__host__ __device__ constexpr int stages_for() {
    return BNA <= 64 ? 6 : 4;
}
// Q8_0 weights: a shared-memory ring of raw stages (q 8 KiB + scales 512 B + activation
// pair), about 200 KiB deep, and the expanded W_hi / W_lo tiles in tensor memory (the MMA's
// A operand read from TMEM): 4 slots of 64 columns (32 for hi, 32 for lo: 128 rows x 64 K
// f16, two per column) above the accumulators.
template <int BNA>
__host__ __device__ constexpr int raw_stages_q8() {
    return BNA <= 16 ? 16 : BNA <= 32 ? 12 : BNA <= 64 ? 8 : 5;
}
constexpr int kConvSlots = 4;
constexpr uint32_t kConvCol0 = 256;             // first TMEM column of the expanded slots
constexpr uint32_t kConvSlotCols = 64;
constexpr uint32_t W_BYTES = WM * BK * 2;
constexpr uint32_t Q_BYTES = WM * BK;           // int8 q tile
constexpr uint32_t D_BYTES = 2 * WM * 2;        // f16 scales of 2 blocks x 128 rows

template <int BNA>
struct SkEpi {
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t drain;
    uint64_t rbar;                  // fused epilogues: the cluster peers' partial rows have arrived
    float amax_v[4][BNA];
    int amax_i[4][BNA];
    int got[4];                     // argmax epilogue: each warp's accumulator wait succeeded
    uint32_t tmem_base;
    int err;
    int issued;
    int consumed;
};

template <int BNA, bool Q8>
struct SkSmem;

template <int BNA>
struct SkSmem<BNA, false> {
    static constexpr int STAGES = stages_for<BNA>();
    __half w[STAGES][WM * BK];      // 16 KiB each; every operand buffer is a multiple of 1 KiB
    __half a_hi[STAGES][BNA * BK];
    __half a_lo[STAGES][BNA * BK];
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    SkEpi<BNA> e;
};

template <int BNA>
struct SkSmem<BNA, true> {
    static constexpr int STAGES = raw_stages_q8<BNA>();
    static constexpr int CSTAGES = kConvSlots;
    __half a_hi[STAGES][BNA * BK];
    __half a_lo[STAGES][BNA * BK];
    int8_t q[STAGES][WM * BK];      // 64 B rows, 64 B swizzle (conflict-free row reads)
    __half d[STAGES][2 * WM];
    uint64_t full[STAGES];          // raw stage landed (q, scales, activations)
    uint64_t empty[STAGES];         // its MMAs are done: the producer may refill it
    uint64_t cfull[CSTAGES];        // expanded slot written (128 converter arrivals)
    uint64_t cempty[CSTAGES];       // its MMAs are done: the converters may overwrite it
    SkEpi<BNA> e;
};

template <int BNA, bool Q8>
__host__ __device__ constexpr uint32_t tmem_cols() {
    return Q8 ? 512u : (2 * BNA < 32 ? 32u : (uint32_t)(2 * BNA));
}

// tcgen05.mma with the A operand (M = 128 rows, K = 16: 8 columns of f16 pairs) in TMEM.
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(db), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Half a row (32 of the stage's 64 K values, half h) of a raw stage -> the f16 pair of those
// weights in TMEM slot columns [col + 16h, col + 16h + 16) (hi) and [col + 32 + 16h, ...)
// (lo). The q row is read with the 64 B swizzle its TMA box was written with: chunk c of
// row r sits at chunk c ^ ((r >> 1) & 3).
__device__ __forceinline__ void q8_halfrow_to_tmem(const int8_t* q, const __half* d, int r, int h, uint32_t taddr) {
    uint32_t hi[16], lo[16];
    const unsigned char* row = reinterpret_cast<const unsigned char*>(q) + r * 64;
    const __half dv = d[h * WM + r];              // K [32h, 32h + 32) is Q8_0 block h of the stage
    const __half2 d2 = __halves2half2(dv, dv);
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
        const int c = 2 * h + cc;
        const uint4 v = lds128(row + ((c ^ ((r >> 1) & 3)) << 4));
        uint4 h0, l0, h1, l1;
        q8x8_to_hilo(v.x, v.y, d2, h0, l0);
        q8x8_to_hilo(v.z, v.w, d2, h1, l1);
        hi[8 * cc + 0] = h0.x; hi[8 * cc + 1] = h0.y; hi[8 * cc + 2] = h0.z; hi[8 * cc + 3] = h0.w;
        hi[8 * cc + 4] = h1.x; hi[8 * cc + 5] = h1.y; hi[8 * cc + 6] = h1.z; hi[8 * cc + 7] = h1.w;
        lo[8 * cc + 0] = l0.x; lo[8 * cc + 1] = l0.y; lo[8 * cc + 2] = l0.z; lo[8 * cc + 3] = l0.w;
        lo[8 * cc + 4] = l1.x; lo[8 * cc + 5] = l1.y; lo[8 * cc + 6] = l1.z; lo[8 * cc + 7] = l1.w;
    }
    TMEM_ST_X16(taddr + 16u * h, hi);
    TMEM_ST_X16(taddr + 32u + 16u * h, lo);
}

// Epilogue forms (template parameter EPI): fp32 split-K partials, lm_head per-tile argmax,
// and two that finish the product inside a cluster of the n_split CTAs of one weight tile
// (one unit per CTA): each CTA stages its partial tile in shared memory, the CTAs exchange
// the rows each finishes (bulk copies between their shared memories) and each sums its
// rows over the cluster's tiles in split order and applies the next op itself:
//   EPI_QKV     the tile is one head vector of the QKV projection: per-head RMSNorm, RoPE,
//               q to q_out, K / V into their pages (kernel (1), k_append.cuh)
//   EPI_SWIGLU  the tile is 64 gate rows and the 64 up rows of the same outputs: SwiGLU,
//               written as the down GEMM's f16 pair
constexpr int EPI_STORE = 0, EPI_ARGMAX = 1, EPI_QKV = 2, EPI_SWIGLU = 3;

struct SkArgs {
    int M, N, K, n_split, epilogue, has_lo;
    AppendArgs app;                 // EPI_QKV
    __half* H;                      // EPI_SWIGLU: [M][N/2] hi / lo
    __half* H_lo;
    int n_wtiles;                   // N / 128 weight tiles
    int n_units;                    // weight tiles x splits x activation tiles of BNA rows
    float* C;
    float* amax_val;
    int* amax_idx;
    int* err;
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// v[m] (m < 32): this lane's value (weight row n) for activation row m. Five butterfly rounds
// halve the rows each lane keeps, taking the first maximum (larger value, then lower row)
// of each pair; lane l ends with the maximum over the warp's 32 weight rows for activation
// row l. NaN never wins (it enters as -inf with an index no row has).
__device__ __forceinline__ void warp_argmax32_transpose(const uint32_t (&vb)[32], int n, int lane, float& out_v,
                                                        int& out_i) {
    float v[32];
    int ix[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) {
        v[k] = __uint_as_float(vb[k]);
        ix[k] = n;
        if (!(v[k] > -INFINITY)) { v[k] = -INFINITY; ix[k] = 0x7fffffff; }
    }
#pragma unroll
    for (int c = 16; c > 0; c >>= 1) {
        const bool b = (lane & c) != 0;
#pragma unroll
        for (int k = 0; k < c; ++k) {
            float keep = b ? v[k + c] : v[k];
            int keep_i = b ? ix[k + c] : ix[k];
            const float send = b ? v[k] : v[k + c];
            const int send_i = b ? ix[k] : ix[k + c];
            const float rv = __shfl_xor_sync(0xffffffffu, send, c);
            const int ri = __shfl_xor_sync(0xffffffffu, send_i, c);
            if (rv > keep || (rv == keep && ri < keep_i)) { keep = rv; keep_i = ri; }
            v[k] = keep;
            ix[k] = keep_i;
        }
    }
    out_v = v[0];
    out_i = ix[0];
}

// tm_w: the f16 weights [N][K] (128 B swizzle), or for Q8_0 the q plane [N][K] uint8;
// tm_d: Q8_0 only, the d_t plane [K/32][N] f16 (2 x 128 boxes).
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of `p` (this CTA's shared memory) in the shared memory of cluster CTA `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
    return out;
}

template <int BNA, bool Q8, int EPI>
__global__ void __launch_bounds__(threads_for<Q8>(), 1)
    q8_gemm_tc_skinny_kernel(const __grid_constant__ CUtensorMap tm_a_hi, const __grid_constant__ CUtensorMap tm_a_lo,
                             const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_d,
                             const SkArgs g) {
    extern __shared__ unsigned char smem_raw[];
    using Smem = SkSmem<BNA, Q8>;
    Smem& S = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    SkEpi<BNA>& E = S.e;
    constexpr uint32_t kIdesc = idesc_f16(WM, BNA, false, false);
    constexpr uint32_t TCOLS = tmem_cols<BNA, Q8>();
    constexpr int STAGES = Smem::STAGES;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int k_unit = g.K / g.n_split;
    const int n_iters = k_unit / BK;

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm_a_hi);
        tma_prefetch_desc(&tm_a_lo);
        tma_prefetch_desc(&tm_w);
        if constexpr (Q8) tma_prefetch_desc(&tm_d);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        if constexpr (Q8) {
            for (int s = 0; s < Smem::CSTAGES; ++s) {
                mbar_init(&S.cfull[s], CONV_THREADS);
                mbar_init(&S.cempty[s], 1);
            }
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&E.tfull[b], 1);
            mbar_init(&E.tempty[b], 128);
        }
        mbar_init(&E.drain, 1);
        mbar_init(&E.rbar, 1);
        E.err = 0;
        E.issued = 0;
        E.consumed = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&E.tmem_base)),
                     "r"(TCOLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = E.tmem_base;
    pdl_trigger();

    // EPI_QKV: the epilogue warps finish up to kPreRows rows each with the rows' metadata
    // (position, page, rotation, norm weights) loaded during the MMAs
    constexpr int kPreRows = 8;
    HeadRowMeta meta[kPreRows];
    const bool qkv_pre = EPI == EPI_QKV && (BNA / g.n_split + 3) / 4 <= kPreRows;

    int my_units = 0;
    for (int u = blockIdx.x; u < g.n_units; u += gridDim.x) ++my_units;
    const int total = my_units * n_iters;

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t a_bytes = (uint32_t)(BNA * BK * 2) * (g.has_lo ? 2u : 1u);
            const uint32_t bytes = (Q8 ? Q_BYTES + D_BYTES : W_BYTES) + a_bytes;
            auto coords = [&](int it, int& k, int& n0, int& m0) {
                const int u = blockIdx.x + (it / n_iters) * gridDim.x;
                const int t = u / g.n_split;
                k = (u % g.n_split) * k_unit + (it % n_iters) * BK;
                n0 = (t % g.n_wtiles) * WM;
                m0 = (t / g.n_wtiles) * BNA;
            };
            auto load_w = [&](int it, int s) {
                int k, n0, m0;
                coords(it, k, n0, m0);
                if constexpr (Q8) {
                    tma_load_2d(S.q[s], &tm_w, k, n0, &S.full[s]);
                    tma_load_2d(S.d[s], &tm_d, n0, k / kQK, &S.full[s]);
                } else {
                    tma_load_2d(S.w[s], &tm_w, k, n0, &S.full[s]);
                }
            };
            auto load_a = [&](int it, int s) {
                int k, n0, m0;
                coords(it, k, n0, m0);
                tma_load_2d(S.a_hi[s], &tm_a_hi, k, m0, &S.full[s]);
                if (g.has_lo) tma_load_2d(S.a_lo[s], &tm_a_lo, k, m0, &S.full[s]);
            };
            const int pre = total < STAGES ? total : STAGES;
            for (int it = 0; it < pre; ++it) {
                mbar_arrive_expect_tx(&S.full[it], bytes);
                load_w(it, it);
            }
            pdl_wait();
            for (int it = 0; it < pre; ++it) load_a(it, it);
            E.issued = pre;
            bool ok = true;
            for (int it = pre; it < total; ++it) {
                const int s = it % STAGES;
                if (!mbar_wait_bounded(&S.empty[s], (uint32_t)((it / STAGES) & 1) ^ 1u)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&S.full[s], bytes);
                load_w(it, s);
                load_a(it, s);
                E.issued = it + 1;
            }
            if (!ok) E.err = 1;
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = true;
            int it = 0, j = 0;
            for (int u = blockIdx.x; u < g.n_units && ok; u += gridDim.x, ++j) {
                const int buf = j & 1;
                if (j >= 2 && !mbar_wait_bounded(&E.tempty[buf], (uint32_t)((j >> 1) - 1) & 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem + (uint32_t)(buf * BNA);
                for (int i = 0; i < n_iters; ++i, ++it) {
                    const int s = it % STAGES;
                    if (!mbar_wait_bounded(&S.full[s], (uint32_t)(it / STAGES) & 1u)) { ok = false; break; }
                    if constexpr (Q8) {
                        const int cs = it % Smem::CSTAGES;
                        if (!mbar_wait_bounded(&S.cfull[cs], (uint32_t)(it / Smem::CSTAGES) & 1u)) {
                            ok = false;
                            break;
                        }
                        E.consumed = it + 1;
                        tc_fence_after();
                        const uint32_t w_hi = tmem + kConvCol0 + (uint32_t)cs * kConvSlotCols;
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk) {
                            const uint32_t koff = (uint32_t)(kk * 32) >> 4;   // bytes / 16
                            const uint32_t wh = w_hi + (uint32_t)(kk * 8);    // 8 columns per K16
                            const uint64_t dah = smem_desc_k128(S.a_hi[s]) + koff;
                            tc_mma_f16_ts(d_tmem, wh, dah, kIdesc, (i > 0 || kk > 0) ? 1u : 0u);
                            if (g.has_lo) tc_mma_f16_ts(d_tmem, wh, smem_desc_k128(S.a_lo[s]) + koff, kIdesc, 1u);
                            tc_mma_f16_ts(d_tmem, wh + 32, dah, kIdesc, 1u);
                        }
                        tc_commit(&S.empty[s]);
                        tc_commit(&S.cempty[cs]);
                    } else {
                        E.consumed = it + 1;
                        tc_fence_after();
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk) {
                            const uint32_t koff = (uint32_t)(kk * 32) >> 4;   // bytes / 16
                            const uint64_t dw = smem_desc_k128(S.w[s]) + koff;
                            tc_mma_f16(d_tmem, dw, smem_desc_k128(S.a_hi[s]) + koff, kIdesc,
                                       (i > 0 || kk > 0) ? 1u : 0u);
                            if (g.has_lo) tc_mma_f16(d_tmem, dw, smem_desc_k128(S.a_lo[s]) + koff, kIdesc, 1u);
                        }
                        tc_commit(&S.empty[s]);
                    }
                }
                if (!ok) break;
                tc_commit(&E.tfull[buf]);
            }
            if (!ok) E.err = 1;
            tc_commit(&E.drain);
            if (!mbar_wait_bounded(&E.drain, 0)) E.err = 1;
        }
        __syncwarp();
    } else if (warp >= 6) {
        if constexpr (Q8) {
            // converters: raw stage it (q, scales) -> TMEM slot it % CSTAGES; a warp may only
            // reach its own quarter of the lanes, so thread (warp w, lane l) expands half h =
            // (w - 6) / 4 (K values [32h, 32h + 32)) of weight row 32 * (w % 4) + l
            const int r = 32 * (warp & 3) + lane;
            const int half = (warp - 6) >> 2;
            const uint32_t lane_base = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
            for (int it = 0; it < total; ++it) {
                const int s = it % STAGES;
                const int cs = it % Smem::CSTAGES;
                bool got = mbar_wait_bounded(&S.full[s], (uint32_t)(it / STAGES) & 1u);
                if (got && it >= Smem::CSTAGES)
                    got = mbar_wait_bounded(&S.cempty[cs], (uint32_t)((it / Smem::CSTAGES) - 1) & 1u);
                if (!__all_sync(0xffffffffu, got)) {
                    if (lane == 0) E.err = 1;
                    break;
                }
                tc_fence_after();
                q8_halfrow_to_tmem(S.q[s], S.d[s], r, half, lane_base + kConvCol0 + (uint32_t)cs * kConvSlotCols);
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&S.cfull[cs]);
            }
        }
    } else {
        const int q = warp & 3;                 // TMEM lanes 32q..32q+31: weight rows of this warp
        if constexpr (EPI == EPI_QKV) {
            if (qkv_pre) {
                // the metadata may come from the previous kernels: wait for them first
                pdl_wait();
                const int rpr = BNA / g.n_split;
                const int t = blockIdx.x / g.n_split;
                const int mrow0 = (t / g.n_wtiles) * BNA + (int)cluster_rank() * rpr;
#pragma unroll
                for (int r = 0; r < kPreRows; ++r) {
                    const int i = (warp - 2) + 4 * r;
                    if (i < rpr && mrow0 + i < g.M) meta[r] = qkv_head_meta(g.app, mrow0 + i, (t % g.n_wtiles), lane);
                }
                // consume the values here, so the loads (and the ones that depend on them) are
                // issued and complete now, while the MMAs run, not where they are first used
#pragma unroll
                for (int r = 0; r < kPreRows; ++r)
                    asm volatile("" ::"r"(meta[r].pos), "r"(meta[r].page), "f"(meta[r].rot[0].x), "f"(meta[r].rot[0].y),
                                 "f"(meta[r].rot[1].x), "f"(meta[r].rot[1].y), "f"(meta[r].w[0]), "f"(meta[r].w[1]),
                                 "f"(meta[r].w[2]), "f"(meta[r].w[3]));
            }
        }
        int j = 0;
        for (int u = blockIdx.x; u < g.n_units; u += gridDim.x, ++j) {
            const int split = u % g.n_split;
            const int t = u / g.n_split;
            const int n0 = (t % g.n_wtiles) * WM;
            const int m0 = (t / g.n_wtiles) * BNA;
            const int rows = min(BNA, g.M - m0);  // activation rows of this unit
            const int buf = j & 1;
            const bool got = __all_sync(0xffffffffu, mbar_wait_bounded(&E.tfull[buf], (uint32_t)(j >> 1) & 1u));
            if (EPI == EPI_ARGMAX) {
                // the four warps meet at named barriers below: they leave together or not at all
                if (lane == 0) E.got[q] = got ? 1 : 0;
                epi_bar();
                if (!(E.got[0] & E.got[1] & E.got[2] & E.got[3])) {
                    if (lane == 0) E.err = 1;
                    break;
                }
            } else if (!got) {
                if (lane == 0) E.err = 1;
                break;
            }
            tc_fence_after();
            // 32 (or 16) accumulator columns = activation rows at a time; columns past M are zeros
            constexpr int CH = BNA < 32 ? BNA : 32;
            const int n = n0 + q * 32 + lane;
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BNA);
            constexpr bool FUSED = EPI == EPI_QKV || EPI == EPI_SWIGLU;
            float* out = !FUSED && g.C ? g.C + (EPI == EPI_ARGMAX ? 0 : (size_t)split * g.M * g.N) +
                                             (size_t)m0 * g.N + n
                                       : nullptr;
            // fused forms: the partial tile goes to shared memory [row][128 weight rows], over
            // the raw ring (every stage of this CTA's one unit has been consumed by now; the
            // proxy fence orders these writes after the tensor cores' reads of that memory)
            float* stage = reinterpret_cast<float*>(&S.a_hi[0][0]);
            if constexpr (FUSED) fence_proxy_async_smem();
#pragma unroll 1
            for (int c0 = 0; c0 < BNA && c0 < rows; c0 += CH) {
                uint32_t cur[CH];
                if constexpr (CH == 16) {
                    TMEM_LD_X16(tbase + c0, cur);
                } else {
                    TMEM_LD_X32(tbase + c0, cur);
                }
                tmem_wait_ld();
                if (out) {
#pragma unroll
                    for (int m = 0; m < CH; ++m)
                        if (c0 + m < rows) out[(size_t)(c0 + m) * g.N] = __uint_as_float(cur[m]);
                }
                if constexpr (FUSED) {
#pragma unroll
                    for (int m = 0; m < CH; ++m) stage[(c0 + m) * WM + q * 32 + lane] = __uint_as_float(cur[m]);
                }
                if constexpr (EPI == EPI_ARGMAX) {
                    if constexpr (CH == 32) {
                        // first maximum over this warp's 32 weight rows for all 32 activation
                        // rows at once: lane l ends with activation row c0 + l
                        float bv;
                        int bi;
                        warp_argmax32_transpose(cur, n, lane, bv, bi);
                        if (c0 + lane < rows) { E.amax_v[q][c0 + lane] = bv; E.amax_i[q][c0 + lane] = bi; }
                    } else {
#pragma unroll
                        for (int m = 0; m < CH; ++m) {
                            if (c0 + m >= rows) break;
                            float bv = __uint_as_float(cur[m]);
                            int bi = n;
                            if (!(bv > -INFINITY)) { bv = -INFINITY; bi = 0x7fffffff; }
#pragma unroll
                            for (int o = 16; o > 0; o >>= 1) {
                                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
                            }
                            if (lane == 0) { E.amax_v[q][c0 + m] = bv; E.amax_i[q][c0 + m] = bi; }
                        }
                    }
                }
            }
            if constexpr (FUSED) fence_proxy_async_smem();   // the staged tile is read by bulk copies
            tc_fence_before();
            mbar_arrive(&E.tempty[buf]);
            if (EPI == EPI_ARGMAX) {
                // then over the two warps of each 64-row half
                epi_bar();
                for (int tt = threadIdx.x - 64; tt < 2 * BNA; tt += 128) {
                    const int h = tt / BNA, m = tt % BNA;
                    if (m < rows) {
                        float bv = E.amax_v[2 * h][m];
                        int bi = E.amax_i[2 * h][m];
                        const float ov = E.amax_v[2 * h + 1][m];
                        const int oi = E.amax_i[2 * h + 1][m];
                        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
                        const int n_tiles = g.N / 64;
                        g.amax_val[(size_t)(m0 + m) * n_tiles + n0 / 64 + h] = bv;
                        g.amax_idx[(size_t)(m0 + m) * n_tiles + n0 / 64 + h] = bi;
                    }
                }
                epi_bar();
            }
        }
    }
    __syncthreads();
    if (E.err) {
        if (threadIdx.x == 0) {
            record_error(g.err, kDevErrTimeout);
            for (int it = E.consumed; it < E.issued; ++it)
                (void)mbar_wait_bounded(&S.full[it % STAGES], (uint32_t)(it / STAGES) & 1u);
        }
        __syncthreads();
    }
    if constexpr (EPI == EPI_QKV || EPI == EPI_SWIGLU) {
        static_assert(Q8 && Smem::STAGES >= 4, "the staged tile lives over the raw ring of the Q8_0 form");
        // Each CTA owns rows [rank, rank + 1) * rpr of the tile. After one cluster barrier
        // (every CTA has staged its partial tile and its MMAs are done with the ring), CTA s
        // pushes its partial rows of CTA r into r's receive slot s with one bulk copy; CTA r
        // waits (bounded) for the bytes, then sums the partials in split order from its own
        // shared memory. Every thread of every CTA passes the barrier, errors or not, and a
        // CTA leaves only after its outgoing copies have read their source and its incoming
        // copies have landed.
        const int cs = g.n_split;
        const uint32_t rank = cluster_rank();
        const int t = blockIdx.x / g.n_split;
        const int n0 = (t % g.n_wtiles) * WM;
        const int m0 = (t / g.n_wtiles) * BNA;
        const int rpr = BNA / cs;                          // rows this CTA finishes
        const uint32_t slot_bytes = (uint32_t)rpr * WM * 4;
        const float* stage = reinterpret_cast<const float*>(&S.a_hi[0][0]);
        float* recv = reinterpret_cast<float*>(&S.a_lo[0][0]);
        if (threadIdx.x == 0) mbar_arrive_expect_tx(&E.rbar, (uint32_t)(cs - 1) * slot_bytes);
        cluster_sync_all();
        if (threadIdx.x == 0) {
            for (int r = 1; r < cs; ++r) {
                const uint32_t peer = (rank + (uint32_t)r) % (uint32_t)cs;
                const uint32_t dst = dsmem_addr(recv + (size_t)rank * rpr * WM, peer);
                const uint32_t bar = dsmem_addr(&E.rbar, peer);
                asm volatile(
                    "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                        dst),
                    "r"(smem_u32(stage + (size_t)peer * rpr * WM)), "r"(slot_bytes), "r"(bar)
                    : "memory");
            }
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
        const bool got = mbar_wait_bounded(&E.rbar, 0);
        if (!got && lane == 0) E.err = 1;
        if (got && !E.err) {
            // partial s of local row i: this CTA's own staging for s == rank, else slot s
            auto row = [&](int sp, int i) -> const float* {
                return sp == (int)rank ? stage + (size_t)(rank * rpr + i) * WM : recv + (size_t)(sp * rpr + i) * WM;
            };
            if constexpr (EPI == EPI_QKV) {
                if (qkv_pre) {
                    if (warp >= 2 && warp < 6) {
                        // the warp's rows ew, ew + 4, ... two at a time, side by side; a rolled
                        // loop: this code runs once per launch, so its size costs instruction
                        // fetches from L2, and a second unrolled copy would cost them again
                        const int ew = warp - 2;
                        constexpr int RB = 2;
#pragma unroll 1
                        for (int r0 = 0; r0 < kPreRows; r0 += RB) {
                            float x[RB][4];
                            int mr[RB];
                            bool live[RB];
#pragma unroll
                            for (int r = 0; r < RB; ++r) {
                                const int i = ew + 4 * (r0 + r);
                                mr[r] = m0 + (int)rank * rpr + i;
                                live[r] = i < rpr && mr[r] < g.M;
#pragma unroll
                                for (int k = 0; k < 4; ++k) x[r][k] = 0.0f;
                                if (!live[r]) continue;
                                for (int sp = 0; sp < cs; ++sp) {
                                    const float* src = row(sp, i) + lane;
#pragma unroll
                                    for (int k = 0; k < 4; ++k) x[r][k] = __fadd_rn(x[r][k], src[32 * k]);
                                }
                            }
                            qkv_head_apply_rows<RB>(g.app, &meta[r0], mr, n0 / WM, lane, x, live);
                        }
                    }
                } else {
                    for (int i = warp; i < rpr && m0 + (int)rank * rpr + i < g.M; i += threads_for<Q8>() / 32) {
                        float x[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                        for (int sp = 0; sp < cs; ++sp) {
                            const float* src = row(sp, i) + lane;
#pragma unroll
                            for (int k = 0; k < 4; ++k) x[k] = __fadd_rn(x[k], src[32 * k]);
                        }
                        qkv_head_finish(g.app, m0 + (int)rank * rpr + i, n0 / WM, lane, x);
                    }
                }
            } else {
                const int F = g.N / 2;
                for (int i = warp; i < rpr && m0 + (int)rank * rpr + i < g.M; i += threads_for<Q8>() / 32) {
                    float gs[2] = {0.0f, 0.0f}, us[2] = {0.0f, 0.0f};
                    for (int sp = 0; sp < cs; ++sp) {
                        const float* src = row(sp, i) + lane;
#pragma unroll
                        for (int k = 0; k < 2; ++k) {
                            gs[k] = __fadd_rn(gs[k], src[32 * k]);
                            us[k] = __fadd_rn(us[k], src[64 + 32 * k]);
                        }
                    }
                    const size_t o = (size_t)(m0 + (int)rank * rpr + i) * F + n0 / 2 + lane;
#pragma unroll
                    for (int k = 0; k < 2; ++k) split_store(silu_mul(gs[k], us[k]), g.H, g.H_lo, o + 32 * k);
                }
            }
        }
        if (threadIdx.x == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        __syncthreads();
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS) : "memory");
    }
}

template <int BNA, bool Q8>
size_t skinny_smem() {
    return sizeof(SkSmem<BNA, Q8>) + 1024;
}

// launch_k with a cluster of `cluster` CTAs along x (and programmatic dependent launch when
// the step enables it)
template <typename... KArgs, typename... Args>
cudaError_t launch_clustered(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                             int cluster, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    int n = 0;
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = (unsigned)cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
    if (launch_pdl_enabled()) {
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    cfg.attrs = attr;
    cfg.numAttrs = n;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

template <int BNA, bool Q8>
bool launch_bna(const GemmArgs& g, int* err, cudaStream_t s, int n_sm) {
    CUtensorMap ta, tl, tw, td;
    if (!make_map(&ta, g.A, g.K, g.M, BK, BNA, true)) return false;
    if (!make_map(&tl, g.A_lo ? g.A_lo : g.A, g.K, g.M, BK, BNA, true)) return false;
    if constexpr (Q8) {
        if (!make_map_u8(&tw, g.W8.q, g.K, g.N, BK, WM, true)) return false;
        if (!make_map(&td, g.W8.d_t, g.N, g.K / kQK, WM, 2, false)) return false;
    } else {
        if (!make_map(&tw, g.Wh, g.K, g.N, BK, WM, true)) return false;
        td = tw;
    }
    SkArgs a{};
    a.M = g.M; a.N = g.N; a.K = g.K; a.n_split = g.n_split; a.epilogue = g.epilogue; a.has_lo = g.A_lo != nullptr;
    a.n_wtiles = g.N / WM;
    a.n_units = a.n_wtiles * g.n_split * ((g.M + BNA - 1) / BNA);
    a.C = g.C; a.amax_val = g.amax_val; a.amax_idx = g.amax_idx; a.err = err;
    const int grid = a.n_units < n_sm ? a.n_units : n_sm;
    const dim3 blk(threads_for<Q8>());
    const size_t sm = skinny_smem<BNA, Q8>();
    if (g.epilogue == kEpiArgmax) {
        launch_k(q8_gemm_tc_skinny_kernel<BNA, Q8, EPI_ARGMAX>, dim3(grid), blk, sm, s, ta, tl, tw, td, a);
    } else if (g.epilogue == kEpiStoreF32) {
        launch_k(q8_gemm_tc_skinny_kernel<BNA, Q8, EPI_STORE>, dim3(grid), blk, sm, s, ta, tl, tw, td, a);
    } else if constexpr (Q8) {
        // fused forms: one unit per CTA, clusters of the n_split CTAs of each weight tile
        if (!skinny_fusable(g.M, g.N, g.K, g.n_split, n_sm)) return false;
        if (g.epilogue == kEpiQkvAppend) {
            if (!g.app) return false;
            a.app = *g.app;
            launch_clustered(q8_gemm_tc_skinny_kernel<BNA, Q8, EPI_QKV>, dim3(a.n_units), blk, sm, s, g.n_split, ta,
                             tl, tw, td, a);
        } else if (g.epilogue == kEpiSwiglu) {
            if (!g.H || !g.swiglu_interleave64) return false;
            a.H = g.H;
            a.H_lo = g.H_lo;
            launch_clustered(q8_gemm_tc_skinny_kernel<BNA, Q8, EPI_SWIGLU>, dim3(a.n_units), blk, sm, s, g.n_split,
                             ta, tl, tw, td, a);
        } else {
            return false;
        }
    } else {
        return false;
    }
    return true;
}

template <bool Q8>
bool launch_rows(const GemmArgs& g, int* err, cudaStream_t s, int sms) {
    switch (Q8 ? skinny_tile_rows(g.M) : (g.M <= 16 ? 16 : g.M <= 32 ? 32 : g.M <= 64 ? 64 : 128)) {
        case 16: return launch_bna<16, Q8>(g, err, s, sms);
        case 32: return launch_bna<32, Q8>(g, err, s, sms);
        case 64: return launch_bna<64, Q8>(g, err, s, sms);
        default: return launch_bna<128, Q8>(g, err, s, sms);
    }
}

template <int BNA, bool Q8>
void set_smem_attr() {
    static_assert(sizeof(SkSmem<BNA, Q8>) + 1024 <= 232448, "shared memory per CTA");
    cudaFuncSetAttribute(q8_gemm_tc_skinny_kernel<BNA, Q8, EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)skinny_smem<BNA, Q8>());
    cudaFuncSetAttribute(q8_gemm_tc_skinny_kernel<BNA, Q8, EPI_ARGMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)skinny_smem<BNA, Q8>());
    if constexpr (Q8) {
        cudaFuncSetAttribute(q8_gemm_tc_skinny_kernel<BNA, Q8, EPI_QKV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)skinny_smem<BNA, Q8>());
        cudaFuncSetAttribute(q8_gemm_tc_skinny_kernel<BNA, Q8, EPI_SWIGLU>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)skinny_smem<BNA, Q8>());
    }
}

}  // namespace

// Whether the fused epilogues take a GEMM: Q8_0 weights, one activation tile (M <= 128),
// one unit per CTA (weight tiles x n_split <= SMs) and a cluster of n_split CTAs (1 to 8)
// that divides the tile's rows.
bool skinny_fusable(int M, int N, int K, int n_split, int n_sm) {
    if (M < 1 || M > kSkinnyMaxRows || N % WM || K % BK || n_split < 1 || n_split > 8 || (K / n_split) % BK)
        return false;
    if (n_split & (n_split - 1)) return false;
    const int bna = skinny_tile_rows(M);
    return (N / WM) * n_split <= n_sm && bna % n_split == 0;
}

// Activation rows per tile for Q8_0 weights: the smallest of 16 / 32 / 64 / 128 that holds
// M, and 128-row tiles above 128 rows. (Two 64-row tiles at 65-128 rows, which would halve
// the split-K partials, measured slower: the weight tile is then expanded twice.)
int skinny_tile_rows(int M) {
    return M <= 16 ? 16 : M <= 32 ? 32 : M <= 64 ? 64 : 128;
}

void configure_gemm_tc_skinny() {
    set_smem_attr<16, false>();
    set_smem_attr<32, false>();
    set_smem_attr<64, false>();
    set_smem_attr<128, false>();
    set_smem_attr<16, true>();
    set_smem_attr<32, true>();
    set_smem_attr<64, true>();
    set_smem_attr<128, true>();
}

bool gemm_tc_skinny_supported(const GemmArgs& g) {
    const bool w_ok = g.W8.q ? (g.W8.d_t != nullptr) : (g.Wh != nullptr);
    // f16 weights: one activation tile of up to 128 rows; Q8_0 planes: any number of
    // 128-row activation tiles (the units then cover every (weight tile, activation tile))
    return w_ok && g.A != nullptr && g.M >= 1 && (g.W8.q || g.M <= kSkinnyMaxRows) && g.N % WM == 0 &&
           g.K % BK == 0 && g.n_split > 0 && (g.K / g.n_split) % BK == 0 &&
           (g.epilogue == kEpiStoreF32    ? g.C != nullptr
            : g.epilogue == kEpiArgmax    ? g.n_split == 1 && g.amax_val && g.amax_idx
            : g.epilogue == kEpiQkvAppend ? g.W8.q && g.app != nullptr
            : g.epilogue == kEpiSwiglu    ? g.W8.q && g.H && g.swiglu_interleave64
                                          : false) &&
           tensor_maps_available();
}

// Split-K factor: the divisor S of K/64 (K/S >= 128) minimising rounds * (32-wide K blocks
// per unit + 2 fill + epilogue), rounds = ceil(units / SMs), units = N/128 * S * activation
// tiles. The epilogue counts 2 blocks for one activation tile (a decode step) and 8 when
// there are several (a prefill forward), where split partials of full tiles cost more than
// the waves they save.
int gemm_tc_skinny_pick_split(int M, int N, int K, int n_sm) {
    const int bna = skinny_tile_rows(M);
    const int m_tiles = (M + bna - 1) / bna;
    const int tiles = N / WM * m_tiles;
    const int epi = M > kSkinnyMaxRows ? 8 : 2;
    const int kb = K / BK;
    int best = 1;
    long best_cost = -1;
    for (int sp = 1; sp <= kb; ++sp) {
        if (kb % sp || (sp > 1 && K / sp < 128)) continue;
        const long units = (long)tiles * sp;
        const long rounds = (units + n_sm - 1) / n_sm;
        const long cost = rounds * (K / sp / kQK + 2 + epi);
        if (best_cost < 0 || cost < best_cost) { best = sp; best_cost = cost; }
    }
    return best;
}

bool launch_q8_gemm_tc_skinny(const GemmArgs& g, int* err, cudaStream_t s) {
    if (!gemm_tc_skinny_supported(g)) return false;
    static int n_sm[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && n_sm[dev] == 0) cudaDeviceGetAttribute(&n_sm[dev], cudaDevAttrMultiProcessorCount, dev);
    const int sms = (dev >= 0 && dev < 64 && n_sm[dev] > 0) ? n_sm[dev] : 148;
    return g.W8.q ? launch_rows<true>(g, err, s, sms) : launch_rows<false>(g, err, s, sms);
}

}  // namespace fa
