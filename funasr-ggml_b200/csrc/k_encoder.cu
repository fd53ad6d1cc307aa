// Audio encoder (SANM) and adaptor kernels: the elementwise, normalisation, FSMN and
// attention steps around the tensor-core GEMMs of compute/encoder_ops.cpp and
// compute/adaptor_ops.cpp. Rows are frames: x [T][d] row-major, fp32 residual stream;
// GEMM inputs leave their producer as an f16 pair (hi, lo) like the decoder's.
#include "fa_kernels.cuh"

#include <algorithm>
#include <cmath>

namespace fa {

namespace {

__device__ __forceinline__ void split_store_h(float v, __half* hi, __half* lo, size_t o) {
    const __half h = __float2half_rn(v);
    hi[o] = h;
    lo[o] = __float2half_rn(__fsub_rn(v, __half2float(h)));
}

// Four consecutive values as f16 pairs: hi[o..o+3], lo[o..o+3] in one 8-byte store each
// (o a multiple of 4).
__device__ __forceinline__ void split_store_h4(float4 v, __half* hi, __half* lo, size_t o) {
    const __half h0 = __float2half_rn(v.x), h1 = __float2half_rn(v.y);
    const __half h2 = __float2half_rn(v.z), h3 = __float2half_rn(v.w);
    const __half2 hh[2] = {__halves2half2(h0, h1), __halves2half2(h2, h3)};
    const __half2 ll[2] = {__halves2half2(__float2half_rn(__fsub_rn(v.x, __half2float(h0))),
                                          __float2half_rn(__fsub_rn(v.y, __half2float(h1)))),
                           __halves2half2(__float2half_rn(__fsub_rn(v.z, __half2float(h2))),
                                          __float2half_rn(__fsub_rn(v.w, __half2float(h3))))};
    *reinterpret_cast<uint2*>(hi + o) = *reinterpret_cast<const uint2*>(hh);
    *reinterpret_cast<uint2*>(lo + o) = *reinterpret_cast<const uint2*>(ll);
}

template <int NT>
__device__ __forceinline__ double block_sum_d(double v, double* sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) sh[w] = v;
    __syncthreads();
    double t = 0.0;
    for (int i = 0; i < NT / 32; ++i) t += sh[i];
    return t;
}

// x[t] = scale * in[t] (d columns), zero columns d..ld-1 of the padded copy.
__global__ void __launch_bounds__(256) enc_scale_kernel(const float* in, int d, int ld, float scale, float* x) {
    const int t = blockIdx.x;
    for (int i = threadIdx.x; i < ld; i += 256)
        x[(size_t)t * ld + i] = i < d ? in[(size_t)t * d + i] * scale : 0.0f;
}

// One CTA per row. With n_part >= 0 the row is first updated:
//   x = (residual ? x : 0) + sum_s part[s] + bias (+ mem)
// Then, with ln_w, y = LayerNorm(x) * w + b (ggml_norm: mean and variance over the d
// columns, eps inside the root), written back into x when ln_in_place, and as an f16
// pair [T][ld_out] when out_hi. Without ln_w the pair holds x itself.
__global__ void __launch_bounds__(256) enc_resid_ln_kernel(float* x, int d, int ld_x, const float* part, int n_part,
                                                           int T, const float* bias, const float* mem, int residual,
                                                           const float* ln_w, const float* ln_b, float eps,
                                                           int ln_in_place, __half* out_hi, __half* out_lo,
                                                           int ld_out) {
    __shared__ double sh[8];
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x;
    float* xr = x + (size_t)t * ld_x;
    constexpr int PER = 8;   // columns per thread (d <= 2048)
    float v[PER];
    double s = 0.0;
#pragma unroll
    for (int c = 0; c < PER; ++c) {
        const int i = threadIdx.x + 256 * c;
        v[c] = 0.0f;
        if (i >= d) continue;
        float a = xr[i];
        if (n_part >= 0) {
            float acc = residual ? a : 0.0f;
            for (int p = 0; p < n_part; ++p) acc = __fadd_rn(acc, part[((size_t)p * T + t) * d + i]);
            if (bias) acc = __fadd_rn(acc, bias[i]);
            if (mem) acc = __fadd_rn(acc, mem[(size_t)t * d + i]);
            a = acc;
            if (!ln_w || !ln_in_place) xr[i] = a;
        }
        v[c] = a;
        s += (double)a;
    }
    if (!ln_w) {
        if (out_hi)
#pragma unroll
            for (int c = 0; c < PER; ++c) {
                const int i = threadIdx.x + 256 * c;
                if (i < d) split_store_h(v[c], out_hi, out_lo, (size_t)t * ld_out + i);
            }
        return;
    }
    s = block_sum_d<256>(s, sh);
    const double mean = s / d;
    double q = 0.0;
#pragma unroll
    for (int c = 0; c < PER; ++c) {
        const int i = threadIdx.x + 256 * c;
        if (i < d) q += ((double)v[c] - mean) * ((double)v[c] - mean);
    }
    q = block_sum_d<256>(q, sh);
    const float inv = (float)(1.0 / sqrt(q / d + (double)eps));
    const float mf = (float)mean;
#pragma unroll
    for (int c = 0; c < PER; ++c) {
        const int i = threadIdx.x + 256 * c;
        if (i >= d) continue;
        const float y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c], mf), inv), ln_w[i]), ln_b[i]);
        if (ln_in_place) xr[i] = y;
        if (out_hi) split_store_h(y, out_hi, out_lo, (size_t)t * ld_out + i);
    }
}

// The same row update and LayerNorm with one warp per row (d a multiple of 4, at most
// 32 * 4 * NV): lane l owns the float4 groups l, l + 32, ...; sums in double over the
// warp's shuffles instead of a CTA's barriers.
template <int NV>
__global__ void __launch_bounds__(256) enc_resid_ln_warp_kernel(float* x, int d, int ld_x, const float* part,
                                                                int n_part, int T, const float* bias, const float* mem,
                                                                int residual, const float* ln_w, const float* ln_b,
                                                                float eps, int ln_in_place, __half* out_hi,
                                                                __half* out_lo, int ld_out) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= T) return;
    const int d4 = d / 4;
    float4* xr = reinterpret_cast<float4*>(x + (size_t)t * ld_x);
    float4 v[NV];
    double s = 0.0;
#pragma unroll
    for (int c = 0; c < NV; ++c) {
        const int i = lane + 32 * c;
        v[c] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i >= d4) continue;
        float4 a = xr[i];
        if (n_part >= 0) {
            float4 acc = residual ? a : make_float4(0.f, 0.f, 0.f, 0.f);
            for (int p = 0; p < n_part; ++p) {
                const float4 q = reinterpret_cast<const float4*>(part + ((size_t)p * T + t) * d)[i];
                acc.x = __fadd_rn(acc.x, q.x); acc.y = __fadd_rn(acc.y, q.y);
                acc.z = __fadd_rn(acc.z, q.z); acc.w = __fadd_rn(acc.w, q.w);
            }
            if (bias) {
                const float4 b = reinterpret_cast<const float4*>(bias)[i];
                acc.x = __fadd_rn(acc.x, b.x); acc.y = __fadd_rn(acc.y, b.y);
                acc.z = __fadd_rn(acc.z, b.z); acc.w = __fadd_rn(acc.w, b.w);
            }
            if (mem) {
                const float4 m = reinterpret_cast<const float4*>(mem + (size_t)t * d)[i];
                acc.x = __fadd_rn(acc.x, m.x); acc.y = __fadd_rn(acc.y, m.y);
                acc.z = __fadd_rn(acc.z, m.z); acc.w = __fadd_rn(acc.w, m.w);
            }
            a = acc;
            if (!ln_w || !ln_in_place) xr[i] = a;
        }
        v[c] = a;
        s += (double)a.x + (double)a.y + (double)a.z + (double)a.w;
    }
    const size_t orow = (size_t)t * ld_out;
    if (!ln_w) {
        if (out_hi)
#pragma unroll
            for (int c = 0; c < NV; ++c) {
                const int i = lane + 32 * c;
                if (i < d4) split_store_h4(v[c], out_hi, out_lo, orow + 4 * i);
            }
        return;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const double mean = s / d;
    double q = 0.0;
#pragma unroll
    for (int c = 0; c < NV; ++c) {
        const int i = lane + 32 * c;
        if (i >= d4) continue;
        const double a0 = (double)v[c].x - mean, a1 = (double)v[c].y - mean;
        const double a2 = (double)v[c].z - mean, a3 = (double)v[c].w - mean;
        q += a0 * a0 + a1 * a1 + a2 * a2 + a3 * a3;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float inv = (float)(1.0 / sqrt(q / d + (double)eps));
    const float mf = (float)mean;
#pragma unroll
    for (int c = 0; c < NV; ++c) {
        const int i = lane + 32 * c;
        if (i >= d4) continue;
        const float4 w = reinterpret_cast<const float4*>(ln_w)[i];
        const float4 b = reinterpret_cast<const float4*>(ln_b)[i];
        float4 y;
        y.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c].x, mf), inv), w.x), b.x);
        y.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c].y, mf), inv), w.y), b.y);
        y.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c].z, mf), inv), w.z), b.z);
        y.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c].w, mf), inv), w.w), b.w);
        if (ln_in_place) xr[i] = y;
        if (out_hi) split_store_h4(y, out_hi, out_lo, orow + 4 * i);
    }
}

// y = sum_s part[s] + bias, optionally ReLU; to fp32 (y32) and/or an f16 pair.
__global__ void __launch_bounds__(256) enc_bias_act_kernel(const float* part, int n_part, int T, int n,
                                                           const float* bias, int relu, float* y32, __half* y_hi,
                                                           __half* y_lo) {
    pdl_trigger();
    pdl_wait();
    const size_t total = (size_t)T * n;
    for (size_t e = blockIdx.x * (size_t)256 + threadIdx.x; e < total; e += (size_t)gridDim.x * 256) {
        const int i = (int)(e % n);
        float acc = 0.0f;
        for (int p = 0; p < n_part; ++p) acc = __fadd_rn(acc, part[(size_t)p * total + e]);
        acc = __fadd_rn(acc, bias[i]);
        if (relu) acc = fmaxf(acc, 0.0f);
        if (y32) y32[e] = acc;
        if (y_hi) split_store_h(acc, y_hi, y_lo, e);
    }
}

// The same with a thread per 4 consecutive columns (n a multiple of 4), the form used from
// 512 rows up.
__global__ void __launch_bounds__(256) enc_bias_act4_kernel(const float* part, int n_part, int T, int n,
                                                           const float* bias, int relu, float* y32, __half* y_hi,
                                                           __half* y_lo) {
    pdl_trigger();
    pdl_wait();
    const int n4 = n / 4;
    const int total4 = T * n4;
    const float4* p4 = reinterpret_cast<const float4*>(part);
    const float4* b4 = reinterpret_cast<const float4*>(bias);
    for (int e4 = blockIdx.x * 256 + threadIdx.x; e4 < total4; e4 += gridDim.x * 256) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int p = 0; p < n_part; ++p) {
            const float4 v = p4[(size_t)p * total4 + e4];
            acc.x = __fadd_rn(acc.x, v.x); acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z); acc.w = __fadd_rn(acc.w, v.w);
        }
        const float4 b = b4[e4 % n4];
        acc.x = __fadd_rn(acc.x, b.x); acc.y = __fadd_rn(acc.y, b.y);
        acc.z = __fadd_rn(acc.z, b.z); acc.w = __fadd_rn(acc.w, b.w);
        if (relu) {
            acc.x = fmaxf(acc.x, 0.0f); acc.y = fmaxf(acc.y, 0.0f);
            acc.z = fmaxf(acc.z, 0.0f); acc.w = fmaxf(acc.w, 0.0f);
        }
        if (y32) reinterpret_cast<float4*>(y32)[e4] = acc;
        if (y_hi) split_store_h4(acc, y_hi, y_lo, 4 * (size_t)e4);
    }
}

// FSMN memory on v = qkv[:, 2d:3d]: mem[t][c] = v[t][c] + sum_k v[t + k - pad][c] * w[c][k]
// (zero outside the row's utterance, rows [seg[t].x, seg[t].y)); taps w [d][K].
__global__ void __launch_bounds__(256) enc_fsmn_kernel(const float* qkv, const int2* seg, int d, const float* w, int K,
                                                       int pad, float* mem) {
    pdl_trigger();
    pdl_wait();
    const int t = blockIdx.x;
    const int2 sg = seg[t];
    for (int c = threadIdx.x; c < d; c += 256) {
        const float* vcol = qkv + 2 * d + c;
        float acc = vcol[(size_t)t * 3 * d];
        for (int k = 0; k < K; ++k) {
            const int s = t + k - pad;
            if (s >= sg.x && s < sg.y) acc = fmaf(vcol[(size_t)s * 3 * d], w[(size_t)c * K + k], acc);
        }
        mem[(size_t)t * d + c] = acc;
    }
}

// Bidirectional multi-head attention within each utterance, head_dim 128. CTA = (tile,
// head), 8 warps; a tile (first row, rows <= 16, utterance start, utterance length) lies
// in one utterance. One pass over the utterance's keys in chunks of 32 with an online
// softmax: the keys and values of the next NST chunks are in flight (cp.async into a ring)
// while a chunk is used. Warp w scores rows w and w+8 against the chunk (lane = key),
// updates each row's running max and sum and leaves the chunk's probabilities in shared
// memory; thread t then rescales output dim t % 128 of rows 8 (t / 128) .. +7 and adds the
// chunk's values. fp32 throughout; exp of scores minus the running max. (Shared memory
// allows two CTAs per SM: 8 warps instead of 4 keep twice the loads in flight, with every
// product, sum and rescale computed in the same order as with 4.)
constexpr int ATT_ROWS = 16;
constexpr int ATT_WARPS = 8;
constexpr int ATT_THREADS = 32 * ATT_WARPS;
constexpr int HD = 128;
constexpr int QK_ROWS = ATT_ROWS / ATT_WARPS;            // rows a warp scores
constexpr int PV_ROWS = ATT_ROWS * HD / ATT_THREADS;     // rows a thread accumulates
constexpr int KCH = 32;                  // keys per chunk
constexpr int KLD = HD + 4;              // padded row of a staged key / value (floats)
constexpr int NST = 3;                   // chunks in flight

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool full) {
    // 16 bytes from global to shared memory; with full == false the destination is zeroed
    const int n = full ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(n)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_older() {
    asm volatile("cp.async.wait_group %0;" ::"n"(NST - 1) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(ATT_THREADS) enc_attention_kernel(const float* qkv, const int4* tiles, int d,
                                                            __half* out_hi, __half* out_lo, int max_T) {
    extern __shared__ __align__(16) float sm[];
    float* qs = sm;                                  // [16][128] scaled queries
    float* ks = qs + ATT_ROWS * HD;                  // [NST][32][KLD] keys
    float* vs = ks + NST * KCH * KLD;                // [NST][32][KLD] values
    float* ps = vs + NST * KCH * KLD;                // [16][32] the chunk's probabilities
    float* al = ps + ATT_ROWS * KCH;                 // [16] rescale of the running output
    float* ls = al + ATT_ROWS;                       // [16] final row sums
    (void)max_T;
    pdl_trigger();
    pdl_wait();
    const int h = blockIdx.y;
    const int4 tl = tiles[blockIdx.x];
    const int r0 = tl.x;
    const int nr = tl.y;
    const int k0 = tl.z;                             // the utterance's rows [k0, k0 + T)
    const int T = tl.w;
    const int ld = 3 * d;
    const float scale = 1.0f / sqrtf((float)HD);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_chunks = (T + KCH - 1) / KCH;

    // chunk c into ring slot c % NST (rows past the utterance read as zeros); one copy
    // group per call, empty past the last chunk, so group counts stay uniform
    auto issue = [&](int c) {
        if (c < n_chunks) {
            const int slot = c % NST, c0 = c * KCH;
            for (int e = threadIdx.x; e < KCH * (HD / 4); e += ATT_THREADS) {
                const int kk = e / (HD / 4), j4 = e % (HD / 4);
                const bool ok = c0 + kk < T;
                const float* src = qkv + (size_t)(k0 + (ok ? c0 + kk : 0)) * ld + h * HD + 4 * j4;
                cp_async16(ks + (slot * KCH + kk) * KLD + 4 * j4, src + d, ok);
                cp_async16(vs + (slot * KCH + kk) * KLD + 4 * j4, src + 2 * d, ok);
            }
        }
        cp_async_commit();
    };
    for (int c = 0; c < NST; ++c) issue(c);
    for (int e = threadIdx.x; e < ATT_ROWS * HD; e += ATT_THREADS) {
        const int r = e / HD, j = e % HD;
        qs[e] = r < nr ? qkv[(size_t)(r0 + r) * ld + h * HD + j] * scale : 0.0f;
    }

    float m_run[QK_ROWS], l_run[QK_ROWS];            // rows warp + 8i; every lane holds the same values
#pragma unroll
    for (int i = 0; i < QK_ROWS; ++i) {
        m_run[i] = -INFINITY;
        l_run[i] = 0.0f;
    }
    const int j = threadIdx.x & (HD - 1);            // output dim of this thread
    const int rb = (threadIdx.x / HD) * PV_ROWS;     // its first output row
    float acc[PV_ROWS];
#pragma unroll
    for (int r = 0; r < PV_ROWS; ++r) acc[r] = 0.0f;

    for (int c = 0; c < n_chunks; ++c) {
        cp_async_wait_older();                       // this thread's copies of chunk c have landed
        __syncthreads();                             // ... and every thread's; the queries too
        const int slot = c % NST, nk = min(KCH, T - c * KCH);
        float sc[QK_ROWS];
#pragma unroll
        for (int i = 0; i < QK_ROWS; ++i) sc[i] = 0.0f;
        const float* kr = ks + (slot * KCH + lane) * KLD;
#pragma unroll 4
        for (int jj = 0; jj < HD; jj += 4) {
            const float4 k4 = *reinterpret_cast<const float4*>(kr + jj);
#pragma unroll
            for (int i = 0; i < QK_ROWS; ++i) {
                const float4 q4 = *reinterpret_cast<const float4*>(qs + (warp + ATT_WARPS * i) * HD + jj);
                sc[i] = fmaf(q4.x, k4.x, fmaf(q4.y, k4.y, fmaf(q4.z, k4.z, fmaf(q4.w, k4.w, sc[i]))));
            }
        }
#pragma unroll
        for (int i = 0; i < QK_ROWS; ++i) {
            const int r = warp + ATT_WARPS * i;
            const float sv = lane < nk ? sc[i] : -INFINITY;
            float cm = sv;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
            const float mn = fmaxf(m_run[i], cm);    // finite: every chunk holds at least one key
            const float a = m_run[i] == -INFINITY ? 0.0f : expf(m_run[i] - mn);
            const float p = lane < nk ? expf(sv - mn) : 0.0f;
            float psum = p;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
            l_run[i] = l_run[i] * a + psum;
            m_run[i] = mn;
            ps[r * KCH + lane] = p;
            if (lane == 0) al[r] = a;
        }
        __syncthreads();
        const float* vr = vs + slot * KCH * KLD + j;
#pragma unroll
        for (int r = 0; r < PV_ROWS; ++r) acc[r] *= al[rb + r];
        // four keys at a time: each row's four probabilities in one 16 B load (the same
        // address in every thread of the warp), the FMAs still in key order
        int kk = 0;
        for (; kk + 4 <= nk; kk += 4) {
            const float v0 = vr[kk * KLD], v1 = vr[(kk + 1) * KLD], v2 = vr[(kk + 2) * KLD], v3 = vr[(kk + 3) * KLD];
#pragma unroll
            for (int r = 0; r < PV_ROWS; ++r) {
                const float4 p4 = *reinterpret_cast<const float4*>(ps + (rb + r) * KCH + kk);
                acc[r] = fmaf(p4.w, v3, fmaf(p4.z, v2, fmaf(p4.y, v1, fmaf(p4.x, v0, acc[r]))));
            }
        }
        for (; kk < nk; ++kk) {
            const float v = vr[kk * KLD];
#pragma unroll
            for (int r = 0; r < PV_ROWS; ++r) acc[r] = fmaf(ps[(rb + r) * KCH + kk], v, acc[r]);
        }
        __syncthreads();                             // every thread is done with slot c % NST
        issue(c + NST);
    }
    cp_async_wait_all();                             // only empty groups remain; none outlives the CTA
    if (lane == 0)
#pragma unroll
        for (int i = 0; i < QK_ROWS; ++i) ls[warp + ATT_WARPS * i] = l_run[i];
    __syncthreads();
#pragma unroll
    for (int r = 0; r < PV_ROWS; ++r)
        if (rb + r < nr)
            split_store_h(acc[r] / ls[rb + r], out_hi, out_lo, (size_t)(r0 + rb + r) * d + h * HD + j);
}

}  // namespace

void launch_enc_scale(const float* in, int T, int d, int ld, float scale, float* x, cudaStream_t s) {
    enc_scale_kernel<<<T, 256, 0, s>>>(in, d, ld, scale, x);
}

void launch_enc_resid_ln(float* x, int d, int ld_x, const float* part, int n_part, int T, const float* bias,
                         const float* mem, int residual, const float* ln_w, const float* ln_b, float eps,
                         int ln_in_place, __half* out_hi, __half* out_lo, int ld_out, cudaStream_t s) {
    // a warp per row for batches of >= 512 rows (800 rows: the encoder pass 1 ms faster),
    // where the row's float4 groups fit 8 per lane (d <= 1024) and every row and output
    // stays 16-byte aligned; a CTA per row otherwise (at 82 rows the warp form left most
    // SMs idle and made the pass 1 ms slower)
    const bool warp_rows =
        T >= 512 && d % 4 == 0 && d <= 1024 && ld_x % 4 == 0 && (!out_hi || ld_out % 4 == 0);
    if (warp_rows && d <= 512)
        launch_k(enc_resid_ln_warp_kernel<4>, dim3((T + 7) / 8), dim3(256), 0, s, x, d, ld_x, part, n_part, T, bias,
                 mem, residual, ln_w, ln_b, eps, ln_in_place, out_hi, out_lo, ld_out);
    else if (warp_rows)
        launch_k(enc_resid_ln_warp_kernel<8>, dim3((T + 7) / 8), dim3(256), 0, s, x, d, ld_x, part, n_part, T, bias,
                 mem, residual, ln_w, ln_b, eps, ln_in_place, out_hi, out_lo, ld_out);
    else
        launch_k(enc_resid_ln_kernel, dim3(T), dim3(256), 0, s, x, d, ld_x, part, n_part, T, bias, mem, residual,
                 ln_w, ln_b, eps, ln_in_place, out_hi, out_lo, ld_out);
}

void launch_enc_bias_act(const float* part, int n_part, int T, int n, const float* bias, int relu, float* y32,
                         __half* y_hi, __half* y_lo, int n_sm, cudaStream_t s) {
    // a thread per element below 512 rows, per 4 elements above: measured on one B200,
    // 82 rows x 70 layers took 0.8 ms longer with the 4-wide form (5.3 vs 4.5 ms a pass),
    // 800 rows x 70 layers 2 ms less
    if (T >= 512 && n % 4 == 0) {
        const size_t total4 = (size_t)T * n / 4;
        int blocks = (int)std::min<size_t>((total4 + 255) / 256, (size_t)n_sm * 8);
        if (blocks < 1) blocks = 1;
        launch_k(enc_bias_act4_kernel, dim3(blocks), dim3(256), 0, s, part, n_part, T, n, bias, relu, y32, y_hi,
                 y_lo);
        return;
    }
    const size_t total = (size_t)T * n;
    int blocks = (int)std::min<size_t>((total + 255) / 256, (size_t)n_sm * 8);
    if (blocks < 1) blocks = 1;
    launch_k(enc_bias_act_kernel, dim3(blocks), dim3(256), 0, s, part, n_part, T, n, bias, relu, y32, y_hi, y_lo);
}

void launch_enc_fsmn(const float* qkv, int T, const int2* seg, int d, const float* w, int K, int pad, float* mem,
                     cudaStream_t s) {
    launch_k(enc_fsmn_kernel, dim3(T), dim3(256), 0, s, qkv, seg, d, w, K, pad, mem);
}

size_t enc_attention_smem(int max_T) {
    (void)max_T;   // the online softmax keeps no per-key scores
    return sizeof(float) * ((size_t)ATT_ROWS * HD + 2 * NST * KCH * KLD + ATT_ROWS * KCH + 2 * ATT_ROWS);
}

// The attention kernel's shared memory (queries, the key / value ring, one chunk's
// probabilities: 109 KiB) does not depend on the utterance length; opt in once per device.
void configure_encoder(int) {
    cudaFuncSetAttribute(enc_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)enc_attention_smem(kEncMaxFrames));
}

void launch_enc_attention(const float* qkv, const int4* tiles, int n_tiles, int d, int n_heads, __half* out_hi,
                          __half* out_lo, int max_T, cudaStream_t s) {
    launch_k(enc_attention_kernel, dim3(n_tiles, n_heads), dim3(ATT_THREADS), enc_attention_smem(max_T), s, qkv, tiles, d,
             out_hi, out_lo, max_T);
}

}  // namespace fa
