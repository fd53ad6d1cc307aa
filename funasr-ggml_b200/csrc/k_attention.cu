// Kernel (2): paged GQA decode attention over the f16 page pool.
//
// Replaces the reference's attention subgraph (compute/llm_ops_gpu.cpp:98-143):
// the full-cache views, three cont(permute) copies and two ggml_repeat 8->16 GQA
// expansions of K and V, scores = K.q/sqrt(128), diag_mask_inf, soft_max and the
// V^T.p matmul. Here each KV head is read from HBM once and serves both of its
// query heads (query head H uses KV head H/2, as the reference's repeat/permute
// order gives), and the softmax is an online softmax in fp32.
//
// Work split: one CTA per (split of `pages_per_split` pages, KV head, row).
// 4 warps; warp w owns pages w, w+4, ... of the split. Each warp streams its
// pages through a private kAttnStages-deep (2) shared-memory ring: lane 0 issues one
// 8 KiB cp.async.bulk (TMA bulk copy, K and V of this head in this page) per stage,
// completion is counted on an mbarrier, every wait is bounded in time.
// Compute per page (lane = (token parity par, 8-dim chunk c)):
//   QK  : 8 x 16 B shared loads, 16 fp32 FMAs each, then a 16-lane transpose
//         reduction leaves lane r of each half-warp with the score of
//         (token 2*(r/2)+par, head r%2)
//   softmax: max and sum by xor shuffles, running (max, sum) per head in log2 units
//   PV  : p broadcast through 128 B of shared memory, 8 x 16 B loads, 16 FMAs each
// The 4 warps merge in shared memory; with several splits the un-normalised
// partials go to the scratch buffer and attn_combine merges them.
//
// Roofline: HBM. Algorithmic bytes per (row, layer) = n_kv * 8 heads * 2 * 128 * 2 B
// = n_kv * 4096 B; compute is 4 flop per byte read.
#include "fa_kernels.cuh"
#include "funasr_dec.h"

#include <cmath>
#include <mutex>
#include <string>

namespace fa {

namespace {

constexpr int D = 128;
constexpr int WARPS = 4;
constexpr int STAGES = kAttnStages;
constexpr int TILE_HALVES = 2 * kPageTokens * D;   // K then V of one head in one page
constexpr uint32_t TILE_BYTES = TILE_HALVES * 2;   // 8192
constexpr float kLog2e = 1.4426950408889634f;

struct AttnSmem {
    __half tiles[WARPS][STAGES][TILE_HALVES];
    uint64_t bars[WARPS][STAGES];
    float q[2][D];
    float2 pbuf[WARPS][32];         // each p twice: the PV products take it as a packed pair
    float acc[WARPS][2][D];
    float ml[WARPS][4];
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

__global__ void __launch_bounds__(128, kAttnCtasPerSm) paged_attn_kernel(const AttnArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    AttnSmem& S = *reinterpret_cast<AttnSmem*>(smem_raw);
    const int split = blockIdx.x;
    const int h = blockIdx.y;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    pdl_trigger();
    pdl_wait();
    const int m = a.rows ? a.rows[blockIdx.z] : (int)blockIdx.z;

    const int n_kv = a.pos[m] + 1;
    const int n_row_pages = (n_kv + kPageTokens - 1) / kPageTokens;
    // A row whose position is negative, whose pages run past its block-table row, or
    // whose pages the splits do not all cover is an argument error: flag it (once, from
    // split 0) and write nothing for the row.
    if (row_len_bad(a, n_kv, n_row_pages)) {
        if (split == 0 && threadIdx.x == 0) record_error(a.err, kDevErrBadLen);
        return;
    }
    const int p_begin = split * a.pages_per_split;
    if (p_begin >= n_row_pages) return;                 // uniform for the CTA
    const int p_end = min(n_row_pages, p_begin + a.pages_per_split);
    const int* bt = a.block_table + (size_t)a.slot[m] * a.bt_stride;

    if (threadIdx.x == 0) {
        for (int w = 0; w < WARPS; ++w)
            for (int s = 0; s < STAGES; ++s) mbar_init(&S.bars[w][s], 1);
        fence_mbar_init();
    }
    {
        const float* qg = a.q + ((size_t)m * a.Hq + 2 * h) * D;
        S.q[0][threadIdx.x] = qg[threadIdx.x] * kLog2e;
        S.q[1][threadIdx.x] = qg[D + threadIdx.x] * kLog2e;
    }
    __syncthreads();

    const int span = p_end - p_begin;
    int nw = span > warp ? (span - warp + WARPS - 1) / WARPS : 0;
    {
        bool bad = false;
        for (int i = lane; i < nw; i += 32) {
            const int pg = bt[p_begin + warp + WARPS * i];
            bad |= (pg < 0 || pg >= a.n_pages);
        }
        if (__any_sync(0xffffffffu, bad)) {
            if (lane == 0) record_error(a.err, kDevErrBadPage);
            nw = 0;
        }
    }

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

    const size_t page_elems = (size_t)a.Hkv * TILE_HALVES;
    const __half* head_base = a.pool_layer + (size_t)h * TILE_HALVES;
    int issued = 0;
    if (lane == 0) {
        for (; issued < STAGES && issued < nw; ++issued) {
            const int pg = bt[p_begin + warp + WARPS * issued];
            mbar_arrive_expect_tx(&S.bars[warp][issued], TILE_BYTES);
            bulk_copy_g2s(S.tiles[warp][issued], head_base + (size_t)pg * page_elems, TILE_BYTES,
                          &S.bars[warp][issued]);
        }
    }
    issued = __shfl_sync(0xffffffffu, issued, 0);

    int i = 0;
    bool ok = true;
    for (; i < nw; ++i) {
        const int s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        const bool got = mbar_wait_bounded(&S.bars[warp][s], ph);
        if (!__all_sync(0xffffffffu, got)) { ok = false; break; }

        const int t0 = (p_begin + warp + WARPS * i) * kPageTokens;
        const int nvalid = min(kPageTokens, n_kv - t0);
        const __half* Kt = S.tiles[warp][s];
        const __half* Vt = Kt + kPageTokens * D;

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
            const int pg = bt[p_begin + warp + WARPS * (i + STAGES)];
            mbar_arrive_expect_tx(&S.bars[warp][s], TILE_BYTES);
            bulk_copy_g2s(S.tiles[warp][s], head_base + (size_t)pg * page_elems, TILE_BYTES, &S.bars[warp][s]);
        }
        if (i + STAGES < nw) ++issued;
    }

    if (!ok) {
        // A wait gave up: flag it, then wait (bounded again) for this warp's
        // copies still in flight so none lands after the CTA has exited.
        if (lane == 0) record_error(a.err, kDevErrTimeout);
        for (int k = i; k < issued; ++k) {
            const bool done = mbar_wait_bounded(&S.bars[warp][k % STAGES], (uint32_t)(k / STAGES) & 1u);
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
    __syncthreads();

    const int d = threadIdx.x;
#pragma unroll
    for (int hq = 0; hq < 2; ++hq) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < WARPS; ++w) M = fmaxf(M, S.ml[w][hq]);
        float L = 0.0f, O = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < WARPS; ++w) {
                const float sc = exp2f(S.ml[w][hq] - M);
                L += S.ml[w][2 + hq] * sc;
                O += S.acc[w][hq][d] * sc;
            }
        }
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
}

// Merge of the split partials: a warp per (row, query head), lane l owning dims 4l..4l+3.
// The split maxima are read by the lanes together; every output then sums its splits in
// split order, the same arithmetic as one thread per dim.
__global__ void __launch_bounds__(256) attn_combine_kernel(const AttnArgs a) {
    pdl_trigger();
    pdl_wait();
    const int w = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= a.M * a.Hq) return;
    const int m = a.rows ? a.rows[w / a.Hq] : w / a.Hq;
    const int H = w % a.Hq;
    const int n_kv = a.pos[m] + 1;
    const int n_row_pages = (n_kv + kPageTokens - 1) / kPageTokens;
    if (row_len_bad(a, n_kv, n_row_pages)) return;      // flagged by the attention kernel
    const int n_valid = min(a.n_splits, (n_row_pages + a.pages_per_split - 1) / a.pages_per_split);
    const size_t base = ((size_t)m * a.Hq + H) * a.n_splits;
    float M = -INFINITY;
    for (int s = lane; s < n_valid; s += 32) M = fmaxf(M, a.part_ml[(base + s) * 2]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float L = 0.0f;
    float O[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (M != -INFINITY) {
        for (int s = 0; s < n_valid; ++s) {
            const float sc = exp2f(a.part_ml[(base + s) * 2] - M);
            L += a.part_ml[(base + s) * 2 + 1] * sc;
            const float4 o4 = reinterpret_cast<const float4*>(a.part_o + (base + s) * D)[lane];
            O[0] += o4.x * sc;
            O[1] += o4.y * sc;
            O[2] += o4.z * sc;
            O[3] += o4.w * sc;
        }
    }
    const size_t o = (size_t)m * a.Hq * D + (size_t)H * D + 4 * lane;
#pragma unroll
    for (int j = 0; j < 4; ++j) store_out(a, o + j, L > 0.0f ? O[j] / L : 0.0f);
}

}  // namespace

size_t attn_smem_bytes() { return sizeof(AttnSmem); }

// Opt the kernel into its dynamic shared memory on the current device.
cudaError_t configure_attention() {
    return cudaFuncSetAttribute(paged_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)sizeof(AttnSmem));
}

void launch_paged_attention(const AttnArgs& a, cudaStream_t s) {
    dim3 grid(a.n_splits, a.Hkv, a.M);
    launch_k(paged_attn_kernel, grid, dim3(128), sizeof(AttnSmem), s, a);
}

void launch_attn_combine(const AttnArgs& a, cudaStream_t s) {
    launch_k(attn_combine_kernel, dim3((a.M * a.Hq + 7) / 8), dim3(256), 0, s, a);
}

// ---------------------------------------------------- allocation-free variant --
// For callers that may not allocate device memory themselves (a host runtime that
// owns every allocation through its own pool, a plugin loaded into a process that
// forbids cudaMalloc after start-up, code that must not allocate while a graph is
// being built around it): the split-K partials live in one buffer compiled into the
// library. Every GPU that loads the library holds it until the process exits.
constexpr size_t kNoAllocScratchBytes = (size_t)8 << 20;   // 8 MiB: M * n_splits <= 1008

int report_op_error(int code, const char* msg);   // fa_api.cu

static __device__ __align__(256) unsigned char g_attn_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};   // device address of g_attn_scratch per device
}  // namespace

}  // namespace fa

// The first call on a device looks up the buffer's device address there
// (cudaGetSymbolAddress) and sets the kernel's shared-memory limit; make that first
// call before any stream capture. The address is cached per device for the life of
// the process: a cudaDeviceReset() destroys the context it belongs to, so do not
// call this entry point on a device after resetting it. All calls share the one
// buffer, so calls whose work overlaps on the GPU (other streams, other host
// threads) race on it. Nothing in it needs to start at zero: a call writes every
// partial it later reads.
extern "C" FA_API int fa_op_paged_attention_noalloc(const float* q, int M, const int* pos, const int* slot,
                                                    const int* bt, int bt_stride, int n_pages,
                                                    const uint16_t* pool_layer, int pps, int n_splits,
                                                    uint16_t* out16, uint16_t* out16_lo, float* out32, int* err,
                                                    void* stream) {
    using namespace fa;
    if (!q || !pos || !slot || !bt || !pool_layer || M <= 0 || pps <= 0 || n_splits <= 0 || (!out16 && !out32))
        return report_op_error(FA_ERR_INVALID_ARG, "null or non-positive argument");
    const int Hq = 16, Hkv = 8;
    const size_t need = n_splits > 1 ? (size_t)M * Hq * n_splits * (D + 2) * sizeof(float) : 0;
    if (need > kNoAllocScratchBytes) {
        const std::string msg = "fa_op_paged_attention_noalloc: " + std::to_string(M) + " rows x " +
                                std::to_string(n_splits) + " splits need " + std::to_string(need) +
                                " bytes of split-K scratch; the built-in buffer holds " +
                                std::to_string(kNoAllocScratchBytes) + " (M * n_splits <= 1008)";
        return report_op_error(FA_ERR_CAPACITY, msg.c_str());
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return report_op_error(FA_ERR_CUDA, "fa_op_paged_attention_noalloc: no current CUDA device");
    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_ptr[dev]) {
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
            if (e != cudaSuccess || !p) {
                const std::string msg = std::string("fa_op_paged_attention_noalloc: cudaGetSymbolAddress: ") +
                                        cudaGetErrorString(e);
                return report_op_error(FA_ERR_CUDA, msg.c_str());
            }
            const cudaError_t ec = configure_attention();
            if (ec != cudaSuccess) {
                cudaGetLastError();
                const std::string msg = std::string("fa_op_paged_attention_noalloc: shared-memory limit: ") +
                                        cudaGetErrorString(ec);
                return report_op_error(FA_ERR_CUDA, msg.c_str());
            }
            g_noalloc_ptr[dev] = p;   // cached only once both set-up calls succeeded
        }
        base = g_noalloc_ptr[dev];
    }
    AttnArgs a{};
    a.q = q; a.pool_layer = reinterpret_cast<const __half*>(pool_layer); a.block_table = bt; a.bt_stride = bt_stride;
    a.n_pages = n_pages; a.slot = slot; a.pos = pos; a.M = M; a.Hq = Hq; a.Hkv = Hkv; a.pages_per_split = pps;
    a.n_splits = n_splits;
    a.part_o = reinterpret_cast<float*>(base);
    a.part_ml = a.part_o + (size_t)M * Hq * n_splits * D;
    a.out16 = reinterpret_cast<__half*>(out16); a.out16_lo = reinterpret_cast<__half*>(out16_lo);
    a.out32 = out32; a.err = err;
    launch_paged_attention(a, (cudaStream_t)stream);
    if (n_splits > 1) launch_attn_combine(a, (cudaStream_t)stream);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        const std::string msg = std::string("fa_op_paged_attention_noalloc: launch: ") + cudaGetErrorString(e);
        return report_op_error(FA_ERR_CUDA, msg.c_str());
    }
    return FA_OK;
}
