// Kernel (4), Blackwell path: Q8_0 weight GEMM on the 5th-generation tensor cores.
//
//     C[M][N] = A[M][K] . W[N][K]^T,   W = f16(d * q) per Q8_0 block, made at load time
//
// Arithmetic (the oracle's GEMM mode 1): A arrives as an f16 pair (hi, lo) with
// hi + lo = x to ~22 bits, so the product is a smooth function of the
// activations; the weights are the Q8_0 values d*q rounded once to f16 (relative
// error <= 2^-11, fixed per weight); products are exact and accumulate in fp32 in
// TMEM over the whole K range of a work unit.
//
// Persistent kernel: one CTA per SM walks the work units u = blockIdx.x,
// blockIdx.x + gridDim.x, ... where a unit is one 128 x 128 output tile times one
// K chunk (split-K). The pipeline never drains between units: the producer runs
// ahead into the next unit, and the epilogue of one unit (TMEM buffer u & 1)
// overlaps the MMAs of the next. 10 warps, one role each:
//   warp 0      TMA producer: cp.async.bulk.tensor 2-D loads per stage of A hi,
//               A lo (128 x 64 f16) and W (128 x 64 f16), 128 B swizzled; 4-stage
//               ring. The first stages' weight copies go out before the wait on
//               the previous kernel (programmatic dependent launch).
//   warp 1      allocates 256 TMEM columns; one lane issues tcgen05.mma
//               (cta_group::1, kind::f16, M=128, N=128, K=16; hi and lo) and
//               commits stages back to the producer and units to the epilogue
//   warps 2..9  epilogue: warp w reads TMEM lanes 32*(w%4).. (its rows) and
//               columns 64*((w-2)/4).. of the unit's accumulator, releases the
//               buffer, and writes fp32 split-K partials or the tile's row argmax
// Every mbarrier wait is bounded in time; a wait that gives up records an error
// and the CTA drains its copies and MMAs before freeing TMEM.
#include "fa_kernels.cuh"
#include "tc_common.cuh"

#include <cuda.h>

#include <mutex>

namespace fa {

namespace {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int BK = 64;              // K per stage
constexpr int STAGES = 4;
constexpr int EPI_WARPS = 8;
constexpr int CONV_THREADS = 128;   // Q8_0: warps 10..13 expand q into the f16 pair
constexpr uint32_t A_BYTES = BM * BK * 2;
constexpr uint32_t B_BYTES = BN * BK * 2;
constexpr uint32_t Q_BYTES = BN * BK;       // int8 q tile
constexpr uint32_t D_BYTES = 2 * BN * 2;    // f16 scales of 2 blocks x 128 rows
constexpr uint32_t TMEM_COLS = 2 * BN;      // two fp32 accumulators of 128 columns

template <bool Q8>
__host__ __device__ constexpr int threads_for() {
    return 64 + 32 * EPI_WARPS + (Q8 ? CONV_THREADS : 0);
}

struct TcEpi {
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int err;
    int issued;
    int consumed;
};

template <bool Q8>
struct TcSmem;

template <>
struct TcSmem<false> {
    static constexpr int RS = STAGES;
    __half a_hi[STAGES][BM * BK];   // 16 KiB each, 1 KiB aligned (128 B swizzle atoms)
    __half a_lo[STAGES][BM * BK];
    __half b[STAGES][BN * BK];      // 16 KiB each
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    TcEpi e;
};

// Q8_0: 3 raw stages (activation pair 32 KiB + q 8 KiB + scales), 2 expanded weight stages.
template <>
struct TcSmem<true> {
    static constexpr int RS = 3;
    static constexpr int CS = 2;
    __half a_hi[RS][BM * BK];
    __half a_lo[RS][BM * BK];
    __half b_hi[CS][BN * BK];
    __half b_lo[CS][BN * BK];
    int8_t q[RS][BN * BK];
    __half d[RS][2 * BN];
    uint64_t full[RS];
    uint64_t empty[RS];
    uint64_t cfull[CS];
    uint64_t cempty[CS];
    TcEpi e;
};

__device__ __forceinline__ uint64_t smem_desc(const void* p) { return smem_desc_k128(p); }

// Instruction descriptor: kind::f16, A/B f16 K-major, D f32, M=128, N=128.
constexpr uint32_t kIdesc = idesc_f16(BM, BN, false, false);

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    tc_mma_f16(tmem_d, da, db, kIdesc, accumulate);
}

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

// tm_b: the f16 weights [N][K] (128 B swizzle), or for Q8_0 the q plane [N][K] uint8;
// tm_d: Q8_0 only, the d_t plane [K/32][N] f16 (2 x 128 boxes).
template <bool Q8>
__global__ void __launch_bounds__(threads_for<Q8>(), 1)
    q8_gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a_hi, const __grid_constant__ CUtensorMap tm_a_lo,
                      const __grid_constant__ CUtensorMap tm_b, const __grid_constant__ CUtensorMap tm_d,
                      const TcArgs g) {
    extern __shared__ unsigned char smem_raw[];
    using Smem = TcSmem<Q8>;
    Smem& S = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    TcEpi& E = S.e;
    constexpr int RS = Smem::RS;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int n_iters = (g.K / g.n_split) / BK;     // stages per unit

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm_a_hi);
        tma_prefetch_desc(&tm_a_lo);
        tma_prefetch_desc(&tm_b);
        if constexpr (Q8) tma_prefetch_desc(&tm_d);
        for (int s = 0; s < RS; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        if constexpr (Q8) {
            for (int s = 0; s < Smem::CS; ++s) {
                mbar_init(&S.cfull[s], CONV_THREADS);
                mbar_init(&S.cempty[s], 1);
            }
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&E.tfull[b], 1);
            mbar_init(&E.tempty[b], 32 * EPI_WARPS);
        }
        mbar_init(&E.drain, 1);
        E.err = 0;
        E.issued = 0;
        E.consumed = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&E.tmem_base)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = E.tmem_base;
    pdl_trigger();

    int my_units = 0;
    for (int u = blockIdx.x; u < g.n_units; u += gridDim.x) ++my_units;
    const int total = my_units * n_iters;

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t bytes = A_BYTES * (g.has_lo ? 2 : 1) + (Q8 ? Q_BYTES + D_BYTES : B_BYTES);
            auto coords = [&](int it, int& k, int& m0, int& n0) {
                const Unit w = unit_of(g, blockIdx.x + (it / n_iters) * gridDim.x);
                k = w.k_begin + (it % n_iters) * BK;
                m0 = w.m0;
                n0 = w.n0;
            };
            auto load_b = [&](int it, int s) {
                int k, m0, n0;
                coords(it, k, m0, n0);
                if constexpr (Q8) {
                    tma_load_2d(S.q[s], &tm_b, k, n0, &S.full[s]);
                    tma_load_2d(S.d[s], &tm_d, n0, k / kQK, &S.full[s]);
                } else {
                    tma_load_2d(S.b[s], &tm_b, k, n0, &S.full[s]);
                }
            };
            auto load_a = [&](int it, int s) {
                int k, m0, n0;
                coords(it, k, m0, n0);
                tma_load_2d(S.a_hi[s], &tm_a_hi, k, m0, &S.full[s]);
                if (g.has_lo) tma_load_2d(S.a_lo[s], &tm_a_lo, k, m0, &S.full[s]);
            };
            // The weights do not depend on the previous kernel: the first stages'
            // weight copies go out before waiting for it; the activations after.
            const int pre = total < RS ? total : RS;
            for (int it = 0; it < pre; ++it) {
                mbar_arrive_expect_tx(&S.full[it], bytes);
                load_b(it, it);
            }
            pdl_wait();
            for (int it = 0; it < pre; ++it) load_a(it, it);
            E.issued = pre;
            bool ok = true;
            for (int it = pre; it < total; ++it) {
                const int s = it % RS;
                if (!mbar_wait_bounded(&S.empty[s], (uint32_t)((it / RS) & 1) ^ 1u)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&S.full[s], bytes);
                load_a(it, s);
                load_b(it, s);
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
                const uint32_t d_tmem = tmem + (uint32_t)(buf * BN);
                for (int i = 0; i < n_iters; ++i, ++it) {
                    const int s = it % RS;
                    if (!mbar_wait_bounded(&S.full[s], (uint32_t)(it / RS) & 1u)) { ok = false; break; }
                    if constexpr (Q8) {
                        const int cs = it % Smem::CS;
                        if (!mbar_wait_bounded(&S.cfull[cs], (uint32_t)(it / Smem::CS) & 1u)) {
                            ok = false;
                            break;
                        }
                        E.consumed = it + 1;
                        tc_fence_after();
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk) {
                            const uint32_t koff = (uint32_t)(kk * 32) >> 4;   // bytes / 16
                            const uint64_t dbh = smem_desc(S.b_hi[cs]) + koff;
                            const uint64_t dah = smem_desc(S.a_hi[s]) + koff;
                            tc_mma(d_tmem, dah, dbh, (i > 0 || kk > 0) ? 1u : 0u);
                            if (g.has_lo) tc_mma(d_tmem, smem_desc(S.a_lo[s]) + koff, dbh, 1u);
                            tc_mma(d_tmem, dah, smem_desc(S.b_lo[cs]) + koff, 1u);
                        }
                        tc_commit(&S.empty[s]);
                        tc_commit(&S.cempty[cs]);
                    } else {
                        E.consumed = it + 1;
                        tc_fence_after();
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk) {
                            const uint32_t koff = (uint32_t)(kk * 32) >> 4;   // bytes / 16
                            const uint64_t db = smem_desc(S.b[s]) + koff;
                            tc_mma(d_tmem, smem_desc(S.a_hi[s]) + koff, db, (i > 0 || kk > 0) ? 1u : 0u);
                            if (g.has_lo) tc_mma(d_tmem, smem_desc(S.a_lo[s]) + koff, db, 1u);
                        }
                        tc_commit(&S.empty[s]);
                    }
                }
                if (!ok) break;
                tc_commit(&E.tfull[buf]);
            }
            if (!ok) E.err = 1;
            // every MMA issued so far completes before TMEM can be released
            tc_commit(&E.drain);
            if (!mbar_wait_bounded(&E.drain, 0)) E.err = 1;
        }
        __syncwarp();
    } else if (warp >= 2 + EPI_WARPS) {
        if constexpr (Q8) {
            // converters: raw stage it (q, scales) -> expanded ring slot it % CS
            const int t = threadIdx.x - 32 * (2 + EPI_WARPS);
            for (int it = 0; it < total; ++it) {
                const int s = it % RS;
                const int cs = it % Smem::CS;
                bool got = mbar_wait_bounded(&S.full[s], (uint32_t)(it / RS) & 1u);
                if (got && it >= Smem::CS)
                    got = mbar_wait_bounded(&S.cempty[cs], (uint32_t)((it / Smem::CS) - 1) & 1u);
                if (!__all_sync(0xffffffffu, got)) {
                    if (lane == 0) E.err = 1;
                    break;
                }
                q8_stage_to_hilo<BN>(S.q[s], S.d[s], BN, S.b_hi[cs], S.b_lo[cs], t, CONV_THREADS);
                fence_proxy_async_smem();
                mbar_arrive(&S.cfull[cs]);
            }
        }
    } else {
        const int q = warp & 3;                 // TMEM lanes 32q..32q+31 belong to this warp
        const int ch = (warp - 2) >> 2;         // column half of the tile
        const int row = q * 32 + lane;          // accumulator row
        int j = 0;
        for (int u = blockIdx.x; u < g.n_units; u += gridDim.x, ++j) {
            const Unit w = unit_of(g, u);
            const int buf = j & 1;
            const bool got = mbar_wait_bounded(&E.tfull[buf], (uint32_t)(j >> 1) & 1u);
            if (!__all_sync(0xffffffffu, got)) {
                if (lane == 0) E.err = 1;
                break;
            }
            tc_fence_after();
            uint32_t v[64];
            const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN + ch * 64);
            TMEM_LD_X32(taddr, v);
            TMEM_LD_X32(taddr + 32, (v + 32));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            tc_fence_before();
            mbar_arrive(&E.tempty[buf]);
            const int gm = w.m0 + row;
            const int c0 = w.n0 + ch * 64;
            if (gm < g.M) {
                if (g.C) {
                    float* out = g.C + (g.epilogue == kEpiStoreF32 ? (size_t)w.split * g.M * g.N : 0) +
                                 (size_t)gm * g.N + c0;
#pragma unroll
                    for (int c = 0; c < 64; c += 4)
                        *reinterpret_cast<float4*>(out + c) =
                            make_float4(__uint_as_float(v[c]), __uint_as_float(v[c + 1]), __uint_as_float(v[c + 2]),
                                        __uint_as_float(v[c + 3]));
                }
                if (g.epilogue == kEpiArgmax) {
                    // first maximum of the row within this 64-column half; NaN never wins
                    float bv = -INFINITY;
                    int bi = 0x7fffffff;
#pragma unroll
                    for (int c = 0; c < 64; ++c)
                        if (__uint_as_float(v[c]) > bv) { bv = __uint_as_float(v[c]); bi = c0 + c; }
                    const int n_tiles = g.N / 64;
                    g.amax_val[(size_t)gm * n_tiles + c0 / 64] = bv;
                    g.amax_idx[(size_t)gm * n_tiles + c0 / 64] = bi;
                }
            }
        }
    }
    __syncthreads();
    if (E.err) {
        // drain: every bulk tensor copy issued but not consumed lands before exit
        if (threadIdx.x == 0) {
            record_error(g.err, kDevErrTimeout);
            for (int it = E.consumed; it < E.issued; ++it)
                (void)mbar_wait_bounded(&S.full[it % RS], (uint32_t)(it / RS) & 1u);
        }
        __syncthreads();
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

}  // namespace

// ------------------------------------------------------------- tensor maps --
namespace {

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
}  // namespace

static bool make_map_elem(CUtensorMap* tm, CUtensorMapDataType type, int elem_bytes, const void* base, int cols,
                          long long rows, int box_cols, int box_rows, bool swizzle) {
    EncodeTiledFn enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * (cuuint64_t)elem_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(tm, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map(CUtensorMap* tm, const void* base, int cols, long long rows, int box_cols, int box_rows, bool swizzle) {
    return make_map_elem(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, cols, rows, box_cols, box_rows, swizzle);
}

bool make_map_u8(CUtensorMap* tm, const void* base, int cols, long long rows, int box_cols, int box_rows,
                 bool swizzle64) {
    EncodeTiledFn enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tensor_maps_available() { return encoder() != nullptr; }

template <bool Q8>
static size_t tc_smem_bytes() {
    static_assert(sizeof(TcSmem<Q8>) + 1024 <= 232448, "shared memory per CTA");
    return sizeof(TcSmem<Q8>) + 1024;
}

size_t gemm_tc_smem_bytes() { return tc_smem_bytes<false>(); }

void configure_gemm_tc() {
    cudaFuncSetAttribute(q8_gemm_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)tc_smem_bytes<false>());
    cudaFuncSetAttribute(q8_gemm_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)tc_smem_bytes<true>());
}

// Split-K factor for the persistent kernel: the divisor S of K/64 (with K/S >= 128)
// that minimises rounds * (32-wide K blocks per unit + 2 + 8), rounds = ceil(units / SMs):
// a unit costs its K blocks, about 2 blocks of pipeline fill and about 8 of epilogue
// (a 128 x 128 fp32 tile out of TMEM and to memory). Without the epilogue term the model
// split large-M GEMMs that run faster whole (gate/up at 2048 rows: 593 TFLOP/s at split 2,
// 672 at 1024 rows unsplit); the decode shapes at 128 rows keep their splits.
int gemm_tc_pick_split(int M, int N, int K, int n_sm) {
    const int tiles = (N / BN) * ((M + BM - 1) / BM);
    const int kb = K / BK;
    int best = 1;
    long best_cost = -1;
    for (int sp = 1; sp <= kb; ++sp) {
        if (kb % sp || (sp > 1 && K / sp < 128)) continue;
        const long units = (long)tiles * sp;
        const long rounds = (units + n_sm - 1) / n_sm;
        const long cost = rounds * (K / sp / kQK + 2 + 8);
        if (best_cost < 0 || cost < best_cost) { best = sp; best_cost = cost; }
    }
    return best;
}

bool gemm_tc_supported(const GemmArgs& g) {
    const bool w_ok = g.W8.q ? (g.W8.d_t != nullptr) : (g.Wh != nullptr);
    return w_ok && g.N % BN == 0 && g.K % BK == 0 && g.n_split > 0 && (g.K / g.n_split) % BK == 0 &&
           encoder() != nullptr;
}

// Returns false when the tensor maps cannot be built (the caller reports it).
bool launch_q8_gemm_tc(const GemmArgs& g, int* err, cudaStream_t s) {
    static int n_sm[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && n_sm[dev] == 0) cudaDeviceGetAttribute(&n_sm[dev], cudaDevAttrMultiProcessorCount, dev);
    CUtensorMap ta, tl, tb, td;
    if (!make_map(&ta, g.A, g.K, g.M, BK, BM, true)) return false;
    if (!make_map(&tl, g.A_lo ? g.A_lo : g.A, g.K, g.M, BK, BM, true)) return false;
    const bool q8 = g.W8.q != nullptr;
    if (q8) {
        if (!make_map_u8(&tb, g.W8.q, g.K, g.N, BK, BN, false)) return false;
        if (!make_map(&td, g.W8.d_t, g.N, g.K / kQK, BN, 2, false)) return false;
    } else {
        if (!make_map(&tb, g.Wh, g.K, g.N, BK, BN, true)) return false;
        td = tb;
    }
    TcArgs a{};
    a.M = g.M; a.N = g.N; a.K = g.K; a.n_split = g.n_split; a.epilogue = g.epilogue; a.has_lo = g.A_lo != nullptr;
    a.n_tiles_n = g.N / BN;
    a.n_units = a.n_tiles_n * ((g.M + BM - 1) / BM) * g.n_split;
    a.C = g.C; a.amax_val = g.amax_val; a.amax_idx = g.amax_idx; a.err = err;
    const int sms = (dev >= 0 && dev < 64 && n_sm[dev] > 0) ? n_sm[dev] : 148;
    const int grid = a.n_units < sms ? a.n_units : sms;
    if (q8)
        launch_k(q8_gemm_tc_kernel<true>, dim3(grid), dim3(threads_for<true>()), tc_smem_bytes<true>(), s, ta, tl, tb,
                 td, a);
    else
        launch_k(q8_gemm_tc_kernel<false>, dim3(grid), dim3(threads_for<false>()), tc_smem_bytes<false>(), s, ta, tl,
                 tb, td, a);
    return true;
}

}  // namespace fa
