// Kernel (4), small-M form: the Q8_0 GEMM of a decode step with at most 8 rows, on the
// CUDA cores. C[m][n] = sum_k x[m][k] * W[n][k], x = hi + lo (the activation pair the
// tcgen05 kernel reads; their f32 sum is exact).
//
// Weights: the decoder's Q8_0 planes (q int8 [N][K] and the row-major scales d_r
// [N][K/32], q8_planes.cuh): a lane loads 16 (or 8) int8 values of a row, all in one Q8_0
// block, and accumulates sum_k q*x of them in fp32 before one multiply by the block's d,
// so every weight is the exact d * q and the kernel streams 34/32 B per weight. The
// encoder's f16 weights [N][K] take the same structure with 8 f16 per lane.
//
// Same role as the tcgen05 kernel (compute/llm_ops_gpu.cpp:53-55,149,177-180,206: every
// ggml_mul_mat of the decoder), same epilogues: fp32 results [M][N] (one "partial"), or
// per-64-column row maxima for the lm_head argmax; and one of its own, SwiGLU of the
// stacked gate / up product written as the next GEMM's f16 pair (compute/llm_ops_gpu.cpp:
// 177-180, ggml_silu(gate) * up), which saves the separate SwiGLU launch.
//
// Why a second kernel: with one token per sequence and few sequences the product is a
// matrix-vector product. Its floor is the weight read (2-7 MB of Q8_0 per layer GEMM,
// about a microsecond at HBM rate), and the tcgen05 kernel's fixed costs (TMEM
// allocation, barrier set-up, a 128-row tile pipeline, a split-K partial round trip)
// dominate it. Here a warp owns a block of 4 weight rows x (K / ks) columns: it issues
// all of its weight loads before waiting on the previous kernel (the weights do not
// depend on it), then reads the activations, accumulates 4 x M dot products in fp32,
// reduces them over its lanes, and ks warps of one row block add their sums in a fixed
// order, so results do not depend on timing.
#include "fa_kernels.cuh"

#include <type_traits>

namespace fa {

namespace {

constexpr int kRowsPerWarp = 4;
constexpr int kMaxWarps = 16;

struct GemvArgs {
    const __half* A;
    const __half* A_lo;
    const __half* W;                 // f16 weights, or nullptr
    const int8_t* Wq;                // Q8_0 planes: q [N][K] and d_r [N][K/32]
    const __half* Wd;
    int M, N, K;
    int ks;                          // warps sharing one row block's K range
    int G;                           // row blocks per CTA
    int epilogue;
    int interleave64;                // SwiGLU: gate / up rows stacked in blocks of 64 each
    float* C;
    float* amax_val;
    int* amax_idx;
    __half* H;
    __half* H_lo;
};

__device__ __forceinline__ void h8_to_f32(const uint4& u, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 t = __half22float2(h[j]);
        f[2 * j] = t.x;
        f[2 * j + 1] = t.y;
    }
}

// Weights per lane per slice: WPL = 8 (f16: one 16 B load; Q8_0: 8 B) or 16 (Q8_0: 16 B).
// A slice is the 32 * WPL columns one warp-wide load covers.
template <bool Q8, int WPL>
struct WLoad {
    using T = typename std::conditional<(!Q8 || WPL == 16), uint4, uint2>::type;
};

// MM: rows of activations the registers hold (>= a.M); NS: K slices per warp
template <int MM, int NS, bool Q8, int WPL>
__global__ void __launch_bounds__(kMaxWarps * 32) gemv_kernel(const GemvArgs a) {
    using WT = typename WLoad<Q8, WPL>::T;
    constexpr int kSlice = 32 * WPL;
    __shared__ float red[kMaxWarps * kRowsPerWarp * MM];
    pdl_trigger();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = warp % a.ks, g = warp / a.ks;
    // SwiGLU: the first G/2 row blocks are gate rows, the others the up rows of the same columns
    const bool swiglu = a.epilogue == kEpiSwiglu;
    const int half_g = a.G / 2;
    // (with interleave64: output column f of the gate rows is weight row (f/64)*128 + f%64,
    // its up row 64 further; a block of 4 rows never crosses a 64-row boundary)
    const int f0 = (blockIdx.x * half_g + (g < half_g ? g : g - half_g)) * kRowsPerWarp;
    const int n0 = !swiglu ? blockIdx.x * (a.G * kRowsPerWarp) + g * kRowsPerWarp
                 : a.interleave64 ? (f0 / 64) * 128 + f0 % 64 + (g < half_g ? 0 : 64)
                 : g < half_g ? f0 : a.N / 2 + f0;
    const int k0 = c * (NS * kSlice) + lane * WPL;

    WT w[NS][kRowsPerWarp];
    float dsc[NS][kRowsPerWarp];
#pragma unroll
    for (int s = 0; s < NS; ++s)
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) {
            const size_t e = (size_t)(n0 + r) * a.K + k0 + s * kSlice;
            if constexpr (Q8) {
                w[s][r] = __ldg(reinterpret_cast<const WT*>(a.Wq + e));
                dsc[s][r] = __half2float(a.Wd[(size_t)(n0 + r) * (a.K / kQK) + (k0 + s * kSlice) / kQK]);
            } else {
                w[s][r] = __ldg(reinterpret_cast<const WT*>(a.W + e));
                dsc[s][r] = 1.0f;
            }
        }
    pdl_wait();

    float acc[kRowsPerWarp][MM];
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
        for (int m = 0; m < MM; ++m) acc[r][m] = 0.0f;
    constexpr int XV = Q8 ? WPL : 8;     // activation values per lane per slice
#pragma unroll
    for (int s = 0; s < NS; ++s) {
        float wf[kRowsPerWarp][XV];
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r) {
            if constexpr (Q8) {
                // int8 -> f32 exactly without the (quarter-rate) integer conversion: the byte
                // q + 128 under the exponent of 2^23 reads as 2^23 + q + 128
                const uint32_t* wb = reinterpret_cast<const uint32_t*>(&w[s][r]);
#pragma unroll
                for (int j4 = 0; j4 < XV / 4; ++j4) {
                    const uint32_t u = wb[j4] ^ 0x80808080u;
#pragma unroll
                    for (int b = 0; b < 4; ++b)
                        wf[r][4 * j4 + b] =
                            __int_as_float((int)__byte_perm(u, 0x4B000000u, 0x7540u + (unsigned)b)) - 8388736.0f;
                }
            } else {
                h8_to_f32(w[s][r], wf[r]);
            }
        }
#pragma unroll
        for (int m = 0; m < MM; ++m) {
            if (m < a.M) {
                const size_t off = (size_t)m * a.K + k0 + s * kSlice;
                float x[XV];
#pragma unroll
                for (int h = 0; h < XV / 8; ++h) {
                    h8_to_f32(*reinterpret_cast<const uint4*>(a.A + off + 8 * h), x + 8 * h);
                    if (a.A_lo) {
                        float xl[8];
                        h8_to_f32(*reinterpret_cast<const uint4*>(a.A_lo + off + 8 * h), xl);
#pragma unroll
                        for (int j = 0; j < 8; ++j) x[8 * h + j] += xl[j];
                    }
                }
#pragma unroll
                for (int r = 0; r < kRowsPerWarp; ++r) {
                    float sq = 0.0f;
#pragma unroll
                    for (int j = 0; j < XV; ++j) sq = fmaf(wf[r][j], x[j], sq);
                    acc[r][m] = Q8 ? fmaf(dsc[s][r], sq, acc[r][m]) : acc[r][m] + sq;
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
        for (int m = 0; m < MM; ++m)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[r][m] += __shfl_xor_sync(0xffffffffu, acc[r][m], o);
    if (lane == 0)
#pragma unroll
        for (int r = 0; r < kRowsPerWarp; ++r)
#pragma unroll
            for (int m = 0; m < MM; ++m) red[((g * a.ks + c) * kRowsPerWarp + r) * MM + m] = acc[r][m];
    __syncthreads();

    // sums over the ks warps of each row block, in warp order; kept in red[] slot c = 0
    const int rows = a.G * kRowsPerWarp;
    const int row_base = blockIdx.x * rows;
    for (int t = threadIdx.x; t < rows * a.M; t += blockDim.x) {
        const int m = t % a.M, rr = t / a.M;
        const int gg = rr / kRowsPerWarp, r = rr % kRowsPerWarp;
        float v = 0.0f;
        for (int cc = 0; cc < a.ks; ++cc) v += red[((gg * a.ks + cc) * kRowsPerWarp + r) * MM + m];
        if (a.C) a.C[(size_t)m * a.N + row_base + rr] = v;
        if (a.ks > 1) red[(gg * a.ks * kRowsPerWarp + r) * MM + m] = v;
    }
    if (a.epilogue == kEpiStoreF32) return;
    __syncthreads();
    if (swiglu) {
        const int F = a.N / 2;
        for (int t = threadIdx.x; t < half_g * kRowsPerWarp * a.M; t += blockDim.x) {
            const int m = t % a.M, rr = t / a.M;
            const int gg = rr / kRowsPerWarp, r = rr % kRowsPerWarp;
            const float gv = red[(gg * a.ks * kRowsPerWarp + r) * MM + m];
            const float uv = red[((gg + half_g) * a.ks * kRowsPerWarp + r) * MM + m];
            split_store(silu_mul(gv, uv), a.H, a.H_lo, (size_t)m * F + (blockIdx.x * half_g + gg) * kRowsPerWarp + r);
        }
        return;
    }
    // rows == 64: the first maximum of each activation row over these 64 columns; NaN never wins
    if (warp < a.M) {
        const int m = warp;
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int rr = lane + 32 * h;
            const int gg = rr / kRowsPerWarp, r = rr % kRowsPerWarp;
            const float v = red[(gg * a.ks * kRowsPerWarp + r) * MM + m];
            if (v > bv) { bv = v; bi = row_base + rr; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) {
            const int n_tiles = a.N / 64;
            a.amax_val[(size_t)m * n_tiles + blockIdx.x] = bv;
            a.amax_idx[(size_t)m * n_tiles + blockIdx.x] = bi;
        }
    }
}

template <int MM, bool Q8, int WPL>
void launch_mm(const GemvArgs& a, int ns, cudaStream_t s) {
    const dim3 grid(a.N / (a.G * kRowsPerWarp)), block(a.ks * a.G * 32);   // SwiGLU: N / 2 over G / 2 blocks
    if (ns == 1) launch_k(gemv_kernel<MM, 1, Q8, WPL>, grid, block, 0, s, a);
    else if (ns == 2) launch_k(gemv_kernel<MM, 2, Q8, WPL>, grid, block, 0, s, a);
    else launch_k(gemv_kernel<MM, 4, Q8, WPL>, grid, block, 0, s, a);
}

template <bool Q8, int WPL>
void launch_form(const GemvArgs& a, int ns, cudaStream_t s) {
    if (a.M == 1) launch_mm<1, Q8, WPL>(a, ns, s);
    else if (a.M == 2) launch_mm<2, Q8, WPL>(a, ns, s);
    else if (a.M <= 4) launch_mm<4, Q8, WPL>(a, ns, s);
    else launch_mm<8, Q8, WPL>(a, ns, s);
}

}  // namespace

// Weights per lane per slice: 8 f16, or 16 int8 of Q8_0 when K allows (8 otherwise).
static int wpl_for(bool q8, int K) { return q8 && K % 512 == 0 ? 16 : 8; }

// Chooses (ks, G, slices per warp) for a shape, or returns false when the kernel does not
// take it. Store epilogue: the fewest warps per row block that still give >= 4096 warps
// (enough loads in flight to cover HBM latency), else the most the shape allows.
// Argmax epilogue: 64 rows per CTA (16 row blocks) and one warp per row block.
static bool shape_config(int M, int N, int K, int epilogue, bool q8, int* ks_out, int* G_out, int* ns_out) {
    const int kSlice = 32 * wpl_for(q8, K);
    if (M < 1 || M > kGemvMaxRows || N <= 0 || K <= 0 || K % kSlice) return false;
    const int n_sl = K / kSlice;
    if (epilogue == kEpiArgmax) {
        if (N % 64 || (n_sl != 1 && n_sl != 2 && n_sl != 4)) return false;
        *ks_out = 1; *G_out = 16; *ns_out = n_sl;
        return true;
    }
    if (N % kRowsPerWarp) return false;
    static const int cand[] = {1, 2, 3, 4, 6, 8, 12, 16};
    int best = 0;
    for (int ks : cand) {
        if (n_sl % ks) continue;
        const int ns = n_sl / ks;
        if (ns != 1 && ns != 2 && ns != 4) continue;
        best = ks;
        if ((long)(N / kRowsPerWarp) * ks >= 4096) break;
    }
    if (!best) return false;
    if (epilogue == kEpiSwiglu) {
        // gate and up row blocks in pairs: G even, (N / 2) a multiple of the CTA's G / 2 blocks
        while (best > 8) {
            int next = 0;
            for (int ks : cand)
                if (ks < best && n_sl % ks == 0 && (n_sl / ks == 1 || n_sl / ks == 2 || n_sl / ks == 4)) next = ks;
            if (!next) return false;
            best = next;
        }
        int G = best >= 8 ? 2 : 8 / best;
        while (G > 2 && (N / 2) % (G / 2 * kRowsPerWarp)) G >>= 1;
        if (N % 2 || (N / 2) % (G / 2 * kRowsPerWarp)) return false;
        *ks_out = best; *G_out = G; *ns_out = n_sl / best;
        return true;
    }
    int G = best >= 8 ? 1 : 8 / best;
    while (G > 1 && N % (G * kRowsPerWarp)) G >>= 1;
    *ks_out = best; *G_out = G; *ns_out = n_sl / best;
    return true;
}

static bool gemv_config(const GemmArgs& g, int* ks, int* G, int* ns) {
    const bool q8 = g.W8.q != nullptr;
    if (g.n_split != 1 || !g.A || (q8 ? !g.W8.d_r : !g.Wh)) return false;
    if (g.epilogue == kEpiArgmax ? (!g.amax_val || !g.amax_idx) : g.epilogue == kEpiSwiglu ? !g.H : !g.C)
        return false;
    return shape_config(g.M, g.N, g.K, g.epilogue, q8, ks, G, ns);
}

bool gemv_shape_supported(int M, int N, int K, int epilogue, bool q8) {
    int ks, G, ns;
    return shape_config(M, N, K, epilogue, q8, &ks, &G, &ns);
}

bool gemv_q8_split(int M, int N, int K, int epilogue, int* ks, int* ns) {
    int G;
    if (wpl_for(true, K) != 16) return false;
    return shape_config(M, N, K, epilogue, true, ks, &G, ns);
}

bool launch_q8_gemv(const GemmArgs& g, cudaStream_t s) {
    int ks, G, ns;
    if (!gemv_config(g, &ks, &G, &ns)) return false;
    GemvArgs a{};
    a.A = g.A; a.A_lo = g.A_lo; a.W = g.Wh; a.Wq = g.W8.q; a.Wd = g.W8.d_r;
    a.M = g.M; a.N = g.N; a.K = g.K; a.ks = ks; a.G = G;
    a.epilogue = g.epilogue; a.interleave64 = g.swiglu_interleave64;
    a.C = g.epilogue == kEpiSwiglu ? nullptr : g.C; a.amax_val = g.amax_val;
    a.amax_idx = g.amax_idx; a.H = g.H; a.H_lo = g.H_lo;
    if (!g.W8.q) launch_form<false, 8>(a, ns, s);
    else if (wpl_for(true, g.K) == 16) launch_form<true, 16>(a, ns, s);
    else launch_form<true, 8>(a, ns, s);
    return true;
}

}  // namespace fa
