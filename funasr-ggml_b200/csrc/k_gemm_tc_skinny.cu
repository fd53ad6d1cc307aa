// Kernel (4), few-row form on the tensor cores: the Q8_0 weight GEMM of a step with up to
// 128 rows (a decode batch), with the operands swapped:
//
//     C^T[N][M] = W[N][K] . A[M][K]^T,   the MMA's M side = 128 weight rows,
//                                        its N side = the activation rows (16 ... 128)
//
// Same arithmetic as k_gemm_tc.cu (f16(d*q) weights, the activation as an f16 hi/lo pair,
// fp32 accumulation in TMEM) and the same outputs (fp32 split-K partials [split][M][N],
// or per-64-column row maxima for the lm_head argmax). Why swap: with 128-row activation
// tiles a step of 16 rows still pays for a 128 x 128 fp32 accumulator per unit (64 KiB of
// epilogue and partials) and for 64 KiB of activation copies per stage pair; here a unit's
// accumulator is 128 x BNA (8-32 KiB up to 64 rows), a stage holds 16 KiB of weights and
// BNA rows of activations, so six stages fit and each SM keeps ~96 KiB of weights in flight.
//
// Persistent, one CTA per SM, units = (128 weight rows, K chunk). 6 warps:
//   warp 0      TMA producer: the weight tile (64 K x 128 rows) and the activation hi /
//               lo tiles (64 K x BNA rows; rows past M read as zeros) per stage, 128 B
//               swizzled; the first stages' weight copies go out before the wait on the
//               previous kernel
//   warp 1      TMEM (two BNA-column accumulators) and tcgen05.mma kind::f16, M=128,
//               N=BNA, K=16, hi and lo into one accumulator
//   warps 2..5  epilogue: TMEM lanes 32*(warp%4).. are weight rows, columns are
//               activation rows; each warp writes 128 B runs of one activation row
// Every mbarrier wait is bounded; a wait that gives up records an error and the CTA
// drains its copies and MMAs before freeing TMEM.
#include "fa_kernels.cuh"
#include "tc_common.cuh"

#include <cuda.h>

namespace fa {

namespace {

constexpr int WM = 128;             // weight rows per unit
constexpr int BK = 64;
constexpr int THREADS = 64 + 128;

// stages of the ring: 6 of 16 KiB weights + BNA-row activation pairs up to 64 rows (at
// most 192 KiB), 4 at 128 rows (48 KiB each)
template <int BNA>
__host__ __device__ constexpr int stages_for() {
    return BNA <= 64 ? 6 : 4;
}
constexpr uint32_t W_BYTES = WM * BK * 2;

template <int BNA, int STAGES = stages_for<BNA>()>
struct SkSmem {
    __half w[STAGES][WM * BK];      // 16 KiB each; every operand buffer is a multiple of 1 KiB
    __half a_hi[STAGES][BNA * BK];
    __half a_lo[STAGES][BNA * BK];
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t drain;
    float amax_v[4][BNA];
    int amax_i[4][BNA];
    int got[4];                     // argmax epilogue: each warp's accumulator wait succeeded
    uint32_t tmem_base;
    int err;
    int issued;
    int consumed;
};

template <int BNA>
__host__ __device__ constexpr uint32_t tmem_cols() {
    return 2 * BNA < 32 ? 32u : (uint32_t)(2 * BNA);
}

struct SkArgs {
    int M, N, K, n_split, epilogue, has_lo;
    int n_units;
    float* C;
    float* amax_val;
    int* amax_idx;
    int* err;
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int BNA>
__global__ void __launch_bounds__(THREADS, 1)
    q8_gemm_tc_skinny_kernel(const __grid_constant__ CUtensorMap tm_a_hi, const __grid_constant__ CUtensorMap tm_a_lo,
                             const __grid_constant__ CUtensorMap tm_w, const SkArgs g) {
    extern __shared__ unsigned char smem_raw[];
    SkSmem<BNA>& S =
        *reinterpret_cast<SkSmem<BNA>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr uint32_t kIdesc = idesc_f16(WM, BNA, false, false);
    constexpr uint32_t TCOLS = tmem_cols<BNA>();
    constexpr int STAGES = stages_for<BNA>();
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int k_unit = g.K / g.n_split;
    const int n_iters = k_unit / BK;

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm_a_hi);
        tma_prefetch_desc(&tm_a_lo);
        tma_prefetch_desc(&tm_w);
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&S.tfull[b], 1);
            mbar_init(&S.tempty[b], 128);
        }
        mbar_init(&S.drain, 1);
        S.err = 0;
        S.issued = 0;
        S.consumed = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem_base)),
                     "r"(TCOLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;
    pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t bytes = W_BYTES + (uint32_t)(BNA * BK * 2) * (g.has_lo ? 2u : 1u);
            int my_units = 0;
            for (int u = blockIdx.x; u < g.n_units; u += gridDim.x) ++my_units;
            const int total = my_units * n_iters;
            auto coords = [&](int it, int& k, int& n0) {
                const int u = blockIdx.x + (it / n_iters) * gridDim.x;
                k = (u % g.n_split) * k_unit + (it % n_iters) * BK;
                n0 = (u / g.n_split) * WM;
            };
            const int pre = total < STAGES ? total : STAGES;
            for (int it = 0; it < pre; ++it) {
                int k, n0;
                coords(it, k, n0);
                mbar_arrive_expect_tx(&S.full[it], bytes);
                tma_load_2d(S.w[it], &tm_w, k, n0, &S.full[it]);
            }
            pdl_wait();
            for (int it = 0; it < pre; ++it) {
                int k, n0;
                coords(it, k, n0);
                tma_load_2d(S.a_hi[it], &tm_a_hi, k, 0, &S.full[it]);
                if (g.has_lo) tma_load_2d(S.a_lo[it], &tm_a_lo, k, 0, &S.full[it]);
            }
            S.issued = pre;
            bool ok = true;
            for (int it = pre; it < total; ++it) {
                const int s = it % STAGES;
                if (!mbar_wait_bounded(&S.empty[s], (uint32_t)((it / STAGES) & 1) ^ 1u)) {
                    ok = false;
                    break;
                }
                int k, n0;
                coords(it, k, n0);
                mbar_arrive_expect_tx(&S.full[s], bytes);
                tma_load_2d(S.w[s], &tm_w, k, n0, &S.full[s]);
                tma_load_2d(S.a_hi[s], &tm_a_hi, k, 0, &S.full[s]);
                if (g.has_lo) tma_load_2d(S.a_lo[s], &tm_a_lo, k, 0, &S.full[s]);
                S.issued = it + 1;
            }
            if (!ok) S.err = 1;
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = true;
            int it = 0, j = 0;
            for (int u = blockIdx.x; u < g.n_units && ok; u += gridDim.x, ++j) {
                const int buf = j & 1;
                if (j >= 2 && !mbar_wait_bounded(&S.tempty[buf], (uint32_t)((j >> 1) - 1) & 1u)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem + (uint32_t)(buf * BNA);
                for (int i = 0; i < n_iters; ++i, ++it) {
                    const int s = it % STAGES;
                    if (!mbar_wait_bounded(&S.full[s], (uint32_t)(it / STAGES) & 1u)) { ok = false; break; }
                    S.consumed = it + 1;
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint32_t koff = (uint32_t)(kk * 32) >> 4;   // bytes / 16
                        const uint64_t dw = smem_desc_k128(S.w[s]) + koff;
                        tc_mma_f16(d_tmem, dw, smem_desc_k128(S.a_hi[s]) + koff, kIdesc, (i > 0 || kk > 0) ? 1u : 0u);
                        if (g.has_lo) tc_mma_f16(d_tmem, dw, smem_desc_k128(S.a_lo[s]) + koff, kIdesc, 1u);
                    }
                    tc_commit(&S.empty[s]);
                }
                if (!ok) break;
                tc_commit(&S.tfull[buf]);
            }
            if (!ok) S.err = 1;
            tc_commit(&S.drain);
            if (!mbar_wait_bounded(&S.drain, 0)) S.err = 1;
        }
        __syncwarp();
    } else {
        const int q = warp & 3;                 // TMEM lanes 32q..32q+31: weight rows of this warp
        int j = 0;
        for (int u = blockIdx.x; u < g.n_units; u += gridDim.x, ++j) {
            const int split = u % g.n_split;
            const int n0 = (u / g.n_split) * WM;
            const int buf = j & 1;
            const bool got = __all_sync(0xffffffffu, mbar_wait_bounded(&S.tfull[buf], (uint32_t)(j >> 1) & 1u));
            if (g.epilogue == kEpiArgmax) {
                // the four warps meet at named barriers below: they leave together or not at all
                if (lane == 0) S.got[q] = got ? 1 : 0;
                epi_bar();
                if (!(S.got[0] & S.got[1] & S.got[2] & S.got[3])) {
                    if (lane == 0) S.err = 1;
                    break;
                }
            } else if (!got) {
                if (lane == 0) S.err = 1;
                break;
            }
            tc_fence_after();
            // 32 (or 16) accumulator columns = activation rows at a time; columns past M are zeros
            constexpr int CH = BNA < 32 ? BNA : 32;
            const int n = n0 + q * 32 + lane;
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BNA);
            float* out = g.C ? g.C + (g.epilogue == kEpiStoreF32 ? (size_t)split * g.M * g.N : 0) + n : nullptr;
#pragma unroll 1
            for (int c0 = 0; c0 < BNA && c0 < g.M; c0 += CH) {
                uint32_t v[CH];
                if constexpr (CH == 16) {
                    TMEM_LD_X16(tbase + c0, v);
                } else {
                    TMEM_LD_X32(tbase + c0, v);
                }
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (out) {
#pragma unroll
                    for (int m = 0; m < CH; ++m)
                        if (c0 + m < g.M) out[(size_t)(c0 + m) * g.N] = __uint_as_float(v[m]);
                }
                if (g.epilogue == kEpiArgmax) {
                    // per activation row: first maximum over this warp's 32 weight rows; NaN never wins
#pragma unroll
                    for (int m = 0; m < CH; ++m) {
                        if (c0 + m >= g.M) break;
                        float bv = __uint_as_float(v[m]);
                        int bi = n;
                        if (!(bv > -INFINITY)) { bv = -INFINITY; bi = 0x7fffffff; }
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) {
                            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
                        }
                        if (lane == 0) { S.amax_v[q][c0 + m] = bv; S.amax_i[q][c0 + m] = bi; }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&S.tempty[buf]);
            if (g.epilogue == kEpiArgmax) {
                // then over the two warps of each 64-row half
                epi_bar();
                for (int t = threadIdx.x - 64; t < 2 * BNA; t += 128) {
                    const int h = t / BNA, m = t % BNA;
                    if (m < g.M) {
                        float bv = S.amax_v[2 * h][m];
                        int bi = S.amax_i[2 * h][m];
                        const float ov = S.amax_v[2 * h + 1][m];
                        const int oi = S.amax_i[2 * h + 1][m];
                        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
                        const int n_tiles = g.N / 64;
                        g.amax_val[(size_t)m * n_tiles + n0 / 64 + h] = bv;
                        g.amax_idx[(size_t)m * n_tiles + n0 / 64 + h] = bi;
                    }
                }
                epi_bar();
            }
        }
    }
    __syncthreads();
    if (S.err) {
        if (threadIdx.x == 0) {
            record_error(g.err, kDevErrTimeout);
            for (int it = S.consumed; it < S.issued; ++it)
                (void)mbar_wait_bounded(&S.full[it % STAGES], (uint32_t)(it / STAGES) & 1u);
        }
        __syncthreads();
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS) : "memory");
    }
}

template <int BNA>
size_t skinny_smem() {
    return sizeof(SkSmem<BNA>) + 1024;
}

template <int BNA>
bool launch_bna(const GemmArgs& g, int* err, cudaStream_t s, int n_sm) {
    CUtensorMap ta, tl, tw;
    if (!make_map(&ta, g.A, g.K, g.M, BK, BNA, true)) return false;
    if (!make_map(&tl, g.A_lo ? g.A_lo : g.A, g.K, g.M, BK, BNA, true)) return false;
    if (!make_map(&tw, g.Wh, g.K, g.N, BK, WM, true)) return false;
    SkArgs a{};
    a.M = g.M; a.N = g.N; a.K = g.K; a.n_split = g.n_split; a.epilogue = g.epilogue; a.has_lo = g.A_lo != nullptr;
    a.n_units = (g.N / WM) * g.n_split;
    a.C = g.C; a.amax_val = g.amax_val; a.amax_idx = g.amax_idx; a.err = err;
    const int grid = a.n_units < n_sm ? a.n_units : n_sm;
    launch_k(q8_gemm_tc_skinny_kernel<BNA>, dim3(grid), dim3(THREADS), skinny_smem<BNA>(), s, ta, tl, tw, a);
    return true;
}

}  // namespace

void configure_gemm_tc_skinny() {
    cudaFuncSetAttribute(q8_gemm_tc_skinny_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)skinny_smem<16>());
    cudaFuncSetAttribute(q8_gemm_tc_skinny_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)skinny_smem<32>());
    cudaFuncSetAttribute(q8_gemm_tc_skinny_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)skinny_smem<64>());
    cudaFuncSetAttribute(q8_gemm_tc_skinny_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)skinny_smem<128>());
}

bool gemm_tc_skinny_supported(const GemmArgs& g) {
    return g.Wh != nullptr && g.A != nullptr && g.M >= 1 && g.M <= kSkinnyMaxRows && g.N % WM == 0 &&
           g.K % BK == 0 && g.n_split > 0 && (g.K / g.n_split) % BK == 0 &&
           (g.epilogue == kEpiStoreF32 ? g.C != nullptr
                                       : g.epilogue == kEpiArgmax && g.n_split == 1 && g.amax_val && g.amax_idx) &&
           tensor_maps_available();
}

// Split-K factor: the divisor S of K/64 (K/S >= 128) minimising rounds * (32-wide K blocks
// per unit + 2 fill + 2 epilogue), rounds = ceil(units / SMs), units = N/128 * S.
int gemm_tc_skinny_pick_split(int M, int N, int K, int n_sm) {
    (void)M;
    const int tiles = N / WM;
    const int kb = K / BK;
    int best = 1;
    long best_cost = -1;
    for (int sp = 1; sp <= kb; ++sp) {
        if (kb % sp || (sp > 1 && K / sp < 128)) continue;
        const long units = (long)tiles * sp;
        const long rounds = (units + n_sm - 1) / n_sm;
        const long cost = rounds * (K / sp / kQK + 2 + 2);
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
    if (g.M <= 16) return launch_bna<16>(g, err, s, sms);
    if (g.M <= 32) return launch_bna<32>(g, err, s, sms);
    if (g.M <= 64) return launch_bna<64>(g, err, s, sms);
    return launch_bna<128>(g, err, s, sms);
}

}  // namespace fa
