// The residual add + RMSNorm of one activation row (ggml_add residual,
// compute/llm_ops_gpu.cpp:172,182, then gpu_rms_norm * w, :16-25) in the one order the
// decoder uses (residual_rmsnorm_kernel, k_small.cu): a kernel that normalises rows
// itself calls it to give the same bits.
#pragma once

#include "fa_kernels.cuh"

namespace fa {

// Sum of v over the first NT threads of the block (the others must pass 0): xor-shuffle
// within each warp, then over the NT / 32 warp sums. sh holds one double per warp of the
// block. Every thread of the block calls it; all get the sum.
template <int NT>
__device__ __forceinline__ double block_sum_double(double v, double* sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x < 32) {
        t = threadIdx.x < NT / 32 ? sh[threadIdx.x] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        if (threadIdx.x == 0) sh[0] = t;
    }
    __syncthreads();
    t = sh[0];
    __syncthreads();
    return t;
}

// Sum of n_part split-K partials of one float4 column group, in partial order; the
// loads of a group of G partials are all issued before the first add (the same sum for
// every G; a larger G shortens the chain of load rounds and costs registers).
// CG: load at L2 (ld.global.cg), for partials written by other CTAs of the same kernel.
template <int G = 8, bool CG = false>
__device__ __forceinline__ float4 sum_parts4(const float4* p, size_t stride4, int n_part) {
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < n_part; s0 += G) {
        float4 t[G];
#pragma unroll
        for (int u = 0; u < G; ++u)
            if (s0 + u < n_part) {
                if constexpr (CG) t[u] = __ldcg(p + (size_t)(s0 + u) * stride4);
                else t[u] = p[(size_t)(s0 + u) * stride4];
            }
#pragma unroll
        for (int u = 0; u < G; ++u)
            if (s0 + u < n_part) {
                o.x = __fadd_rn(o.x, t[u].x); o.y = __fadd_rn(o.y, t[u].y);
                o.z = __fadd_rn(o.z, t[u].z); o.w = __fadd_rn(o.w, t[u].w);
            }
    }
    return o;
}

// One row: a = x_row + sum over n_part partials (part4 points at this row's first float4
// of partial 0, stride4 floats4 between partials); x_out_row (may be null, may equal
// x_row) receives a; then y = (a * scale) * w, scale = 1 / sqrt(mean(a^2) + eps) with the
// squares summed in double, and emit(j, y) for every column j. Threads [0, 256) each own
// the float4 groups t, t + 256, ... (hidden <= 4096, a multiple of 4); every thread of the
// block must call it (it synchronises), and sh needs one double per warp. CG: x_row (a
// global address then) and the partials are read at L2, for values other CTAs of the same
// kernel wrote.
template <int G = 8, bool CG = false, typename Emit>
__device__ __forceinline__ void residual_norm_row(const float* x_row, const float4* part4, size_t stride4, int n_part,
                                                  int hidden, const float* w, float eps, float* x_out_row, double* sh,
                                                  Emit emit) {
    const int n4 = hidden / 4;
    const bool owner = threadIdx.x < 256;
    float4 v[4];
    double ss = 0.0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const int i = threadIdx.x + 256 * c;
        if (!owner || i >= n4) break;
        float4 a;
        if constexpr (CG) a = __ldcg(reinterpret_cast<const float4*>(x_row) + i);
        else a = reinterpret_cast<const float4*>(x_row)[i];
        if (n_part > 0) {
            const float4 o = sum_parts4<G, CG>(part4 + i, stride4, n_part);
            a.x = __fadd_rn(a.x, o.x); a.y = __fadd_rn(a.y, o.y);
            a.z = __fadd_rn(a.z, o.z); a.w = __fadd_rn(a.w, o.w);
        }
        if (x_out_row) reinterpret_cast<float4*>(x_out_row)[i] = a;
        v[c] = a;
        ss += (double)__fmul_rn(a.x, a.x) + (double)__fmul_rn(a.y, a.y) + (double)__fmul_rn(a.z, a.z) +
              (double)__fmul_rn(a.w, a.w);
    }
    ss = block_sum_double<256>(ss, sh);
    const float mean = (float)(ss / (double)hidden);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        const int i = threadIdx.x + 256 * c;
        if (!owner || i >= n4) break;
        const float4 ww = reinterpret_cast<const float4*>(w)[i];
        emit(4 * i, __fmul_rn(__fmul_rn(v[c].x, scale), ww.x));
        emit(4 * i + 1, __fmul_rn(__fmul_rn(v[c].y, scale), ww.y));
        emit(4 * i + 2, __fmul_rn(__fmul_rn(v[c].z, scale), ww.z));
        emit(4 * i + 3, __fmul_rn(__fmul_rn(v[c].w, scale), ww.w));
    }
}

}  // namespace fa
