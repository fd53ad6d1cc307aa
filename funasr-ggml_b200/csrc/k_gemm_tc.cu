// Kernel (4), Blackwell path: Q8_0 weight GEMM on the 5th-generation tensor cores.
//
//     C[M][N] = A[M][K] . W[N][K]^T,   W[n][k] = d[k/32][n] * q[n][k]
//
// Same arithmetic as the mma.sync kernel in k_gemm.cu (and the oracle's exact
// GEMM mode): A arrives as an f16 pair (hi, lo), q enters the MMA as exact f16
// integers, and each 32-wide Q8_0 block's partial sum is scaled by its d in
// fp32 before it joins the fp32 accumulator - ggml's block-scaled dot without
// rounding either operand.
//
// Persistent kernel: one CTA per SM walks the work units u = blockIdx.x,
// blockIdx.x + gridDim.x, ... where a unit is one 128 x 128 output tile times one
// K chunk (split-K). The pipeline never drains between units: the producer runs
// ahead into the next unit, and the epilogue of one unit overlaps the next
// unit's MMAs. 10 warps, one role each:
//   warp 0      TMA producer: cp.async.bulk.tensor 2-D loads per stage of A hi,
//               A lo (128 x 64 f16), W (128 x 64 f16), all 128 B swizzled, and the
//               stage's block scales (2 x 128 f16); 4-stage ring
//   warp 1      allocates 256 TMEM columns; one lane issues tcgen05.mma
//               (cta_group::1, kind::f16, M=128, N=128, K=16) for one Q8_0 block
//               (2 k-steps x hi/lo) into TMEM buffer (block & 1) and commits it
//   warps 2..9  epilogue: warp w reads TMEM lanes 32*(w%4).. (its rows) and
//               columns 64*((w-2)/4).. ; per block acc += partial * d, then the
//               buffer (and, after a stage's second block, the stage) is released;
//               at a unit's end the fp32 partials or the tile's row argmax go out
// A stage is free again when the MMAs that read it have completed (tcgen05.commit)
// and all 8 epilogue warps have read its scales. Every mbarrier wait is bounded in
// time; a wait that gives up records an error and the CTA drains its copies and
// MMAs before freeing TMEM.
#include "fa_kernels.cuh"

#include <cuda.h>

#include <mutex>

namespace fa {

namespace {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int BK = 64;              // K per stage: two Q8_0 blocks
constexpr int STAGES = 4;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t A_BYTES = BM * BK * 2;
constexpr uint32_t B_BYTES = BN * BK * 2;
constexpr uint32_t SC_BYTES = 2 * BN * 2;
constexpr uint32_t TMEM_COLS = 2 * BN;  // two fp32 accumulators of 128 columns

struct TcSmem {
    __half a_hi[STAGES][BM * BK];   // 16 KiB each, 1 KiB aligned (128 B swizzle atoms)
    __half a_lo[STAGES][BM * BK];
    __half b[STAGES][BN * BK];      // 16 KiB each
    __half scale[STAGES][2][BN];    // d of the stage's two K blocks for the tile's columns
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int err;
    int issued;
    int consumed;
};

// UMMA shared-memory descriptor: K-major tile of 128 B rows in 128 B swizzle
// atoms (8 rows x 128 B = 1 KiB apart), descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc(const void* p) {
    const uint32_t a = smem_u32(p);
    uint64_t d = 0;
    d |= (uint64_t)((a & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;                 // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset: next 8-row group
    d |= (uint64_t)1 << 46;                 // descriptor version
    d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
    return d;
}

// Instruction descriptor: kind::f16, A/B f16 K-major, D f32, M=128, N=128.
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

#define TMEM_LD_X32(taddr, v)                                                                                  \
    asm volatile(                                                                                              \
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"       \
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                             \
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),       \
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), \
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]),           \
          "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),           \
          "=r"(v[30]), "=r"(v[31])                                                                             \
        : "r"(taddr))

struct TcArgs {
    int M, N, K, n_split, epilogue, has_lo;
    int n_tiles_n, n_units;
    float* C;
    float* amax_val;
    int* amax_idx;
    int* err;
};

struct Unit {
    int m0, n0, split, k_begin;
};

__device__ __forceinline__ Unit unit_of(const TcArgs& g, int u) {
    Unit r;
    r.split = u % g.n_split;
    const int t = u / g.n_split;
    r.n0 = (t % g.n_tiles_n) * BN;
    r.m0 = (t / g.n_tiles_n) * BM;
    r.k_begin = r.split * (g.K / g.n_split);
    return r;
}

__global__ void __launch_bounds__(THREADS, 1)
    q8_gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a_hi, const __grid_constant__ CUtensorMap tm_a_lo,
                      const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_sc,
                      const TcArgs g) {
    extern __shared__ unsigned char smem_raw[];
    TcSmem& S = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int k_len = g.K / g.n_split;
    const int n_iters = k_len / BK;     // stages per unit
    const int n_blk = k_len / kQK;      // Q8_0 blocks per unit

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1 + EPI_WARPS);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&S.tfull[b], 1);
            mbar_init(&S.tempty[b], 32 * EPI_WARPS);
        }
        mbar_init(&S.drain, 1);
        S.err = 0;
        S.issued = 0;
        S.consumed = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem_base)),
                     "r"(TMEM_COLS)
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
            const uint32_t bytes = A_BYTES * (g.has_lo ? 2 : 1) + B_BYTES + SC_BYTES;
            int my_units = 0;
            for (int u = blockIdx.x; u < g.n_units; u += gridDim.x) ++my_units;
            const int total = my_units * n_iters;
            auto coords = [&](int it, int& k, int& m0, int& n0) {
                const Unit w = unit_of(g, blockIdx.x + (it / n_iters) * gridDim.x);
                k = w.k_begin + (it % n_iters) * BK;
                m0 = w.m0;
                n0 = w.n0;
            };
            // The weights and scales do not depend on the previous kernel: the first
            // stages' copies go out before waiting for it; the activations after.
            const int pre = total < STAGES ? total : STAGES;
            for (int it = 0; it < pre; ++it) {
                int k, m0, n0;
                coords(it, k, m0, n0);
                mbar_arrive_expect_tx(&S.full[it], bytes);
                tma_load_2d(S.b[it], &tm_b, k, n0, &S.full[it]);
                tma_load_2d(S.scale[it], &tm_sc, n0, k / kQK, &S.full[it]);
            }
            pdl_wait();
            for (int it = 0; it < pre; ++it) {
                int k, m0, n0;
                coords(it, k, m0, n0);
                tma_load_2d(S.a_hi[it], &tm_a_hi, k, m0, &S.full[it]);
                if (g.has_lo) tma_load_2d(S.a_lo[it], &tm_a_lo, k, m0, &S.full[it]);
            }
            S.issued = pre;
            bool ok = true;
            for (int it = pre; it < total; ++it) {
                const int s = it % STAGES;
                if (!mbar_wait_bounded(&S.empty[s], (uint32_t)((it / STAGES) & 1) ^ 1u)) {
                    ok = false;
                    break;
                }
                int k, m0, n0;
                coords(it, k, m0, n0);
                mbar_arrive_expect_tx(&S.full[s], bytes);
                tma_load_2d(S.a_hi[s], &tm_a_hi, k, m0, &S.full[s]);
                if (g.has_lo) tma_load_2d(S.a_lo[s], &tm_a_lo, k, m0, &S.full[s]);
                tma_load_2d(S.b[s], &tm_b, k, n0, &S.full[s]);
                tma_load_2d(S.scale[s], &tm_sc, n0, k / kQK, &S.full[s]);
                S.issued = it + 1;
            }
            if (!ok) S.err = 1;
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = true;
            int it = 0, j = 0;
            for (int u = blockIdx.x; u < g.n_units && ok; u += gridDim.x) {
                for (int b = 0; b < n_blk; ++b, ++j) {
                    const int half = b & 1, s = it % STAGES;
                    if (half == 0) {
                        if (!mbar_wait_bounded(&S.full[s], (uint32_t)(it / STAGES) & 1u)) { ok = false; break; }
                        S.consumed = it + 1;
                    }
                    const int buf = j & 1;
                    if (j >= 2 && !mbar_wait_bounded(&S.tempty[buf], (uint32_t)((j >> 1) - 1) & 1u)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem + (uint32_t)(buf * BN);
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk) {
                        const uint32_t koff = (uint32_t)(half * 64 + kk * 32) >> 4;   // bytes / 16
                        const uint64_t db = smem_desc(S.b[s]) + koff;
                        tc_mma(d_tmem, smem_desc(S.a_hi[s]) + koff, db, kk > 0 ? 1u : 0u);
                        if (g.has_lo) tc_mma(d_tmem, smem_desc(S.a_lo[s]) + koff, db, 1u);
                    }
                    tc_commit(&S.tfull[buf]);
                    if (half == 1) {
                        tc_commit(&S.empty[s]);
                        ++it;
                    }
                }
            }
            if (!ok) S.err = 1;
            // every MMA issued so far completes before TMEM can be released
            tc_commit(&S.drain);
            if (!mbar_wait_bounded(&S.drain, 0)) S.err = 1;
        }
        __syncwarp();
    } else {
        const int q = warp & 3;                 // TMEM lanes 32q..32q+31 belong to this warp
        const int ch = (warp - 2) >> 2;         // column half of the tile
        const int row = q * 32 + lane;          // accumulator row
        int it = 0, j = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < g.n_units && ok; u += gridDim.x) {
            const Unit w = unit_of(g, u);
            float acc[64];
#pragma unroll
            for (int c = 0; c < 64; ++c) acc[c] = 0.0f;
            for (int b = 0; b < n_blk; ++b, ++j) {
                const int buf = j & 1, half = b & 1, s = it % STAGES;
                const bool got = mbar_wait_bounded(&S.tfull[buf], (uint32_t)(j >> 1) & 1u);
                if (!__all_sync(0xffffffffu, got)) {
                    if (lane == 0) S.err = 1;
                    ok = false;
                    break;
                }
                tc_fence_after();
                uint32_t v[64];
                const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN + ch * 64);
                TMEM_LD_X32(taddr, v);
                TMEM_LD_X32(taddr + 32, (v + 32));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                tc_fence_before();
                mbar_arrive(&S.tempty[buf]);
                const __half2* sc = reinterpret_cast<const __half2*>(&S.scale[s][half][ch * 64]);
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const float2 d = __half22float2(sc[c]);
                    acc[2 * c] = fmaf(__uint_as_float(v[2 * c]), d.x, acc[2 * c]);
                    acc[2 * c + 1] = fmaf(__uint_as_float(v[2 * c + 1]), d.y, acc[2 * c + 1]);
                }
                if (half == 1) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&S.empty[s]);   // this warp is done with the stage's scales
                    ++it;
                }
            }
            if (!ok) break;
            const int gm = w.m0 + row;
            const int c0 = w.n0 + ch * 64;
            if (gm < g.M) {
                if (g.C) {
                    float* out = g.C + (g.epilogue == kEpiStoreF32 ? (size_t)w.split * g.M * g.N : 0) +
                                 (size_t)gm * g.N + c0;
#pragma unroll
                    for (int c = 0; c < 64; c += 4)
                        *reinterpret_cast<float4*>(out + c) = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
                }
                if (g.epilogue == kEpiArgmax) {
                    // first maximum of the row within this 64-column half; NaN never wins
                    float bv = -INFINITY;
                    int bi = 0x7fffffff;
#pragma unroll
                    for (int c = 0; c < 64; ++c)
                        if (acc[c] > bv) { bv = acc[c]; bi = c0 + c; }
                    const int n_tiles = g.N / 64;
                    g.amax_val[(size_t)gm * n_tiles + c0 / 64] = bv;
                    g.amax_idx[(size_t)gm * n_tiles + c0 / 64] = bi;
                }
            }
        }
    }
    __syncthreads();
    if (S.err) {
        // drain: every bulk tensor copy issued but not consumed lands before exit
        if (threadIdx.x == 0) {
            record_error(g.err, kDevErrTimeout);
            for (int it = S.consumed; it < S.issued; ++it)
                (void)mbar_wait_bounded(&S.full[it % STAGES], (uint32_t)(it / STAGES) & 1u);
        }
        __syncthreads();
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// ------------------------------------------------------------- tensor maps --
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 2-D f16 row-major [rows][cols] map with a (box_cols x box_rows) box.
bool make_map(CUtensorMap* tm, const void* base, int cols, int rows, int box_cols, int box_rows, bool swizzle) {
    EncodeTiledFn enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

size_t gemm_tc_smem_bytes() { return sizeof(TcSmem) + 1024; }

void configure_gemm_tc() {
    cudaFuncSetAttribute(q8_gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_tc_smem_bytes());
}

// Split-K factor for the persistent kernel: the divisor S of K/64 (with K/S >= 128)
// that minimises rounds * (Q8_0 blocks per unit + 2), rounds = ceil(units / SMs).
int gemm_tc_pick_split(int M, int N, int K, int n_sm) {
    const int tiles = (N / BN) * ((M + BM - 1) / BM);
    const int kb = K / BK;
    int best = 1;
    long best_cost = -1;
    for (int sp = 1; sp <= kb; ++sp) {
        if (kb % sp || (sp > 1 && K / sp < 128)) continue;
        const long units = (long)tiles * sp;
        const long rounds = (units + n_sm - 1) / n_sm;
        const long cost = rounds * (K / sp / kQK + 2);
        if (best_cost < 0 || cost < best_cost) { best = sp; best_cost = cost; }
    }
    return best;
}

bool gemm_tc_supported(const GemmArgs& g) {
    return g.Wqh != nullptr && g.N % BN == 0 && g.K % BK == 0 && g.n_split > 0 && (g.K / g.n_split) % BK == 0 &&
           encoder() != nullptr;
}

// Returns false when the tensor maps cannot be built (the caller reports it).
bool launch_q8_gemm_tc(const GemmArgs& g, int* err, cudaStream_t s) {
    static int n_sm[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && n_sm[dev] == 0) cudaDeviceGetAttribute(&n_sm[dev], cudaDevAttrMultiProcessorCount, dev);
    CUtensorMap ta, tl, tb, tsc;
    if (!make_map(&ta, g.A, g.K, g.M, BK, BM, true)) return false;
    if (!make_map(&tl, g.A_lo ? g.A_lo : g.A, g.K, g.M, BK, BM, true)) return false;
    if (!make_map(&tb, g.Wqh, g.K, g.N, BK, BN, true)) return false;
    if (!make_map(&tsc, g.Wd, g.N, g.K / kQK, BN, 2, false)) return false;
    TcArgs a{};
    a.M = g.M; a.N = g.N; a.K = g.K; a.n_split = g.n_split; a.epilogue = g.epilogue; a.has_lo = g.A_lo != nullptr;
    a.n_tiles_n = g.N / BN;
    a.n_units = a.n_tiles_n * ((g.M + BM - 1) / BM) * g.n_split;
    a.C = g.C; a.amax_val = g.amax_val; a.amax_idx = g.amax_idx; a.err = err;
    const int sms = (dev >= 0 && dev < 64 && n_sm[dev] > 0) ? n_sm[dev] : 148;
    const int grid = a.n_units < sms ? a.n_units : sms;
    launch_k(q8_gemm_tc_kernel, dim3(grid), dim3(THREADS), gemm_tc_smem_bytes(), s, ta, tl, tb, tsc, a);
    return true;
}

}  // namespace fa
