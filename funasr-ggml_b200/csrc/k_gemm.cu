// Kernel (4): Q8_0 weight GEMM for the decode projections and lm_head.
//
// Replaces the reference's ggml_mul_mat(Q8_0 weight, f32 activations) calls
// (compute/llm_ops_gpu.cpp:53-55 QKV, :149 o_proj, :177-180 gate/up/down,
// :206 lm_head). At decode batch B the weight stream is read once per step for
// all B rows, so the op is a skinny GEMM C[B][N] = A[B][K] . W[N][K]^T.
//
// Arithmetic (same as k_gemm_tc.cu): activations arrive as an f16 pair (hi, lo)
// with hi + lo = x to ~22 bits, so the product is a smooth function of them (a
// single f16 rounding of the activations makes the decoder output jump by ~3e-4
// relative under 1e-7 input noise, which no parity tolerance survives). Weights
// are the decoder's Q8_0 planes, each stage's q tile expanded into the exact f16
// pair W_hi + W_lo = d*q (q8_planes.cuh; three MMAs per product: Wh.ah, Wh.al,
// Wl.ah), or the encoder's f16 weights (two MMAs); products accumulate in fp32.
//
// This is the legacy-tensor-core (mma.sync m16n8k16) implementation, kept as the
// cross-check of the tcgen05 kernel in k_gemm_tc.cu, which is the default.
// Pipeline: 3-stage cp.async ring for the A tiles (BM x 64 f16, hi and lo) and
// the weight tile (64 x 64 f16); ldmatrix feeds the MMAs (2 per k16 step). Split-K over grid.z writes fp32
// partials that the next fused kernel (RoPE/append, residual+RMSNorm, SwiGLU)
// sums in a fixed order, so results are deterministic.
// Epilogue kEpiArgmax (lm_head): per-row maximum and its first column over the
// CTA's 64 columns; launch_argmax_reduce picks the first global maximum, the
// tie rule of the reference's argmax (compute/gpu_runner.hpp:108-118).
#include "fa_kernels.cuh"

#include <algorithm>

namespace fa {

namespace {

constexpr int BN = 64;
constexpr int BK = 64;
constexpr int STAGES = 3;
constexpr int A_LD = BK + 8;    // halves; 144 B rows keep ldmatrix conflict-free
constexpr int B_LD = BK + 8;

template <int BM, int WM, int WN>
struct Cfg {
    static constexpr int THREADS = 32 * WM * WN;
    static constexpr int WTM = BM / WM;
    static constexpr int WTN = BN / WN;
    static constexpr int MT = WTM / 16;
    static constexpr int NT = WTN / 8;
    static constexpr int A_STAGE = BM * A_LD;        // halves
    static constexpr int Q_STAGE = 2 * BN * B_LD * 2;   // bytes (f16 weight tile hi, then lo; padded rows)
    static constexpr size_t SMEM = (size_t)STAGES * (2 * A_STAGE * 2 + Q_STAGE) + (size_t)BM * WN * 8;
    static_assert(WTM % 16 == 0 && WTN % 8 == 0, "warp tile");
    static_assert(NT % 2 == 0, "B fragments are loaded two n8 tiles at a time");
};

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int BM, int WM, int WN, bool Q8>
__global__ void __launch_bounds__(Cfg<BM, WM, WN>::THREADS) q8_gemm_kernel(const GemmArgs g) {
    using C = Cfg<BM, WM, WN>;
    extern __shared__ __align__(128) unsigned char smem[];
    pdl_trigger();
    pdl_wait();
    // A stage st: hi tile at As + (2*st) * A_STAGE, lo tile right after it
    __half* As = reinterpret_cast<__half*>(smem);
    unsigned char* Qs = smem + (size_t)STAGES * 2 * C::A_STAGE * 2;
    const bool has_lo = g.A_lo != nullptr;
    float* red_v = reinterpret_cast<float*>(smem + (size_t)STAGES * (2 * C::A_STAGE * 2 + C::Q_STAGE));
    int* red_i = reinterpret_cast<int*>(red_v + BM * WN);

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int wm = warp / WN, wn = warp % WN;
    const int n0 = blockIdx.x * BN;
    const int m0 = blockIdx.y * BM;
    const int k_len = g.K / g.n_split;
    const int k_begin = blockIdx.z * k_len;
    const int n_iter = k_len / BK;

    auto load_stage = [&](int it, int st) {
        const int k0 = k_begin + it * BK;
        __half* a_dst = As + 2 * st * C::A_STAGE;
        for (int ch = tid; ch < BM * 8 * (has_lo ? 2 : 1); ch += C::THREADS) {
            const int pl = ch / (BM * 8);
            const int r = (ch >> 3) % BM, cc = ch & 7;
            const int gm = m0 + r;
            const bool ok = gm < g.M;
            const __half* src = (pl ? g.A_lo : g.A) + (size_t)(ok ? gm : 0) * g.K + k0 + cc * 8;
            cp_async16(a_dst + pl * C::A_STAGE + r * A_LD + cc * 8, src, ok);
        }
        __half* q_dst = reinterpret_cast<__half*>(Qs + st * C::Q_STAGE);
        for (int ch = tid; ch < BN * 8; ch += C::THREADS) {
            const int r = ch >> 3, cc = ch & 7;
            if constexpr (Q8) {
                // 8 int8 values of one block and its scale -> the exact f16 pair, stored directly
                const uint2 qv = __ldg(reinterpret_cast<const uint2*>(g.W8.q + (size_t)(n0 + r) * g.K + k0 + cc * 8));
                const __half dv = g.W8.d_r[(size_t)(n0 + r) * (g.K / kQK) + (k0 + cc * 8) / kQK];
                uint4 h, l;
                q8x8_to_hilo(qv.x, qv.y, __halves2half2(dv, dv), h, l);
                *reinterpret_cast<uint4*>(q_dst + r * B_LD + cc * 8) = h;
                *reinterpret_cast<uint4*>(q_dst + BN * B_LD + r * B_LD + cc * 8) = l;
            } else {
                cp_async16(q_dst + r * B_LD + cc * 8, g.Wh + (size_t)(n0 + r) * g.K + k0 + cc * 8, true);
            }
        }
    };

    float acc[C::MT][C::NT][4];
#pragma unroll
    for (int i = 0; i < C::MT; ++i)
#pragma unroll
        for (int j = 0; j < C::NT; ++j)
#pragma unroll
            for (int k = 0; k < 4; ++k) acc[i][j][k] = 0.0f;

#pragma unroll
    for (int st = 0; st < STAGES - 1; ++st) {
        if (st < n_iter) load_stage(st, st);
        cp_async_commit();
    }

    for (int it = 0; it < n_iter; ++it) {
        const int st = it % STAGES;
        cp_async_wait<STAGES - 2>();
        __syncthreads();
        {
            const int nx = it + STAGES - 1;
            if (nx < n_iter) load_stage(nx, nx % STAGES);
            cp_async_commit();
        }
        const __half* Bs = reinterpret_cast<const __half*>(Qs + st * C::Q_STAGE);
        const __half* a_hi = As + 2 * st * C::A_STAGE;
        const __half* a_lo = a_hi + C::A_STAGE;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
            uint32_t ah[C::MT][4], al[C::MT][4];
#pragma unroll
            for (int mt = 0; mt < C::MT; ++mt) {
                const int r = wm * C::WTM + mt * 16 + (lane & 15);
                ldmatrix_x4(ah[mt], a_hi + r * A_LD + kk * 16 + (lane >> 4) * 8);
                if (has_lo) ldmatrix_x4(al[mt], a_lo + r * A_LD + kk * 16 + (lane >> 4) * 8);
            }
#pragma unroll
            for (int np = 0; np < C::NT / 2; ++np) {
                uint32_t bf[4], bl[4];
                const int r = wn * C::WTN + np * 16 + (lane & 7) + ((lane >> 4) << 3);
                ldmatrix_x4(bf, Bs + r * B_LD + kk * 16 + ((lane >> 3) & 1) * 8);
                if constexpr (Q8) ldmatrix_x4(bl, Bs + BN * B_LD + r * B_LD + kk * 16 + ((lane >> 3) & 1) * 8);
#pragma unroll
                for (int mt = 0; mt < C::MT; ++mt) {
                    mma16816(acc[mt][2 * np], ah[mt], bf[0], bf[1]);
                    mma16816(acc[mt][2 * np + 1], ah[mt], bf[2], bf[3]);
                    if (has_lo) {
                        mma16816(acc[mt][2 * np], al[mt], bf[0], bf[1]);
                        mma16816(acc[mt][2 * np + 1], al[mt], bf[2], bf[3]);
                    }
                    if constexpr (Q8) {
                        mma16816(acc[mt][2 * np], ah[mt], bl[0], bl[1]);
                        mma16816(acc[mt][2 * np + 1], ah[mt], bl[2], bl[3]);
                    }
                }
            }
        }
    }
    cp_async_wait<0>();

    const int gq = lane >> 2, tq = lane & 3;
    if (g.epilogue == kEpiStoreF32 || g.C != nullptr) {
        float* out = g.C + (g.epilogue == kEpiStoreF32 ? (size_t)blockIdx.z * g.M * g.N : 0);
#pragma unroll
        for (int mt = 0; mt < C::MT; ++mt) {
#pragma unroll
            for (int nt = 0; nt < C::NT; ++nt) {
                const int col = n0 + wn * C::WTN + nt * 8 + 2 * tq;
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const int row = m0 + wm * C::WTM + mt * 16 + gq + hf * 8;
                    if (row < g.M)
                        *reinterpret_cast<float2*>(out + (size_t)row * g.N + col) =
                            make_float2(acc[mt][nt][2 * hf], acc[mt][nt][2 * hf + 1]);
                }
            }
        }
    }
    if (g.epilogue == kEpiArgmax) {
#pragma unroll
        for (int mt = 0; mt < C::MT; ++mt) {
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                float bv = -INFINITY;
                int bi = 0x7fffffff;
#pragma unroll
                for (int nt = 0; nt < C::NT; ++nt) {
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const float v = acc[mt][nt][2 * hf + e];
                        const int col = n0 + wn * C::WTN + nt * 8 + 2 * tq + e;
                        if (v > bv || (v == bv && col < bi)) { bv = v; bi = col; }
                    }
                }
#pragma unroll
                for (int o = 1; o < 4; o <<= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
                }
                if (tq == 0) {
                    const int rl = wm * C::WTM + mt * 16 + gq + hf * 8;
                    red_v[rl * WN + wn] = bv;
                    red_i[rl * WN + wn] = bi;
                }
            }
        }
        __syncthreads();
        for (int rl = tid; rl < BM; rl += C::THREADS) {
            const int row = m0 + rl;
            if (row >= g.M) continue;
            float bv = red_v[rl * WN];
            int bi = red_i[rl * WN];
            for (int w = 1; w < WN; ++w) {
                const float v = red_v[rl * WN + w];
                const int ix = red_i[rl * WN + w];
                if (v > bv || (v == bv && ix < bi)) { bv = v; bi = ix; }
            }
            const int n_tiles = g.N / BN;
            g.amax_val[(size_t)row * n_tiles + blockIdx.x] = bv;
            g.amax_idx[(size_t)row * n_tiles + blockIdx.x] = bi;
        }
    }
}

template <int BM, int WM, int WN>
void launch_cfg(const GemmArgs& g, cudaStream_t s) {
    using C = Cfg<BM, WM, WN>;
    dim3 grid(g.N / BN, (g.M + BM - 1) / BM, g.n_split);
    if (g.W8.q) launch_k(q8_gemm_kernel<BM, WM, WN, true>, grid, dim3(C::THREADS), C::SMEM, s, g);
    else launch_k(q8_gemm_kernel<BM, WM, WN, false>, grid, dim3(C::THREADS), C::SMEM, s, g);
}

template <int BM, int WM, int WN>
void configure_cfg() {
    cudaFuncSetAttribute(q8_gemm_kernel<BM, WM, WN, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)Cfg<BM, WM, WN>::SMEM);
    cudaFuncSetAttribute(q8_gemm_kernel<BM, WM, WN, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)Cfg<BM, WM, WN>::SMEM);
}

}  // namespace

// Opt every tile configuration into its dynamic shared memory on the current device.
void configure_gemm() {
    configure_cfg<16, 1, 4>();
    configure_cfg<32, 2, 4>();
    configure_cfg<64, 2, 4>();
    configure_cfg<128, 4, 2>();
}

int gemm_pick_split(int M, int N, int K, int n_sm) {
    const int bm = M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : 128));
    const int tiles = (N / BN) * ((M + bm - 1) / bm);
    const int kb = K / BK;
    int best = 1;
    for (int s = 1; s <= kb; ++s) {
        if (kb % s) continue;
        if (K / s < 128 && s > 1) break;
        best = s;
        if (tiles * s >= 2 * n_sm) break;
    }
    return best;
}

void launch_q8_gemm(const GemmArgs& g, cudaStream_t s) {
    if (g.M <= 16) launch_cfg<16, 1, 4>(g, s);
    else if (g.M <= 32) launch_cfg<32, 2, 4>(g, s);
    else if (g.M <= 64) launch_cfg<64, 2, 4>(g, s);
    else launch_cfg<128, 4, 2>(g, s);
}

}  // namespace fa
