// The end of kernel (1) for one (row, head vector), shared by the append kernel and by
// the QKV GEMM's fused epilogue: given the head vector's split-K sum x (lane l holding
// dims l, l+32, l+64, l+96), apply per-head RMSNorm and NEOX RoPE to q and k heads and
// write q (scaled) to q_out, or K (rotated) / V into the page of the row's token
// (compute/llm_ops_gpu.cpp:16-25,57-96). Explicit round-to-nearest intrinsics keep the K
// page bytes equal to the CPU oracle's given the same x:
//   ss    = sum over 128 of (double)(x*x)      (ggml CPU rms_norm sums in double)
//   scale = 1 / sqrt((float)(ss/128) + eps)     (correctly rounded div and sqrt)
//   y     = (x * scale) * w
//   rope  : y0' = y0*c - y1*s, y1' = y0*s + y1*c, no fused multiply-add
//   K, V  : f32 -> f16 round-to-nearest-even
// Every lane of the warp calls it (the norm reduces over the warp).
#pragma once

#include "fa_kernels.cuh"

namespace fa {

// What one lane needs from global memory for a (row, head vector): the row's position,
// the page its K / V goes to, the rotation pairs and the norm weights of its dims. Split
// out so a caller can issue these loads for several rows before using any of them.
struct HeadRowMeta {
    int pos;
    int page;
    float2 rot[2];
    float w[4];
};

__device__ __forceinline__ HeadRowMeta qkv_head_meta(const AppendArgs& a, int m, int j, int lane) {
    constexpr int D = 128;
    HeadRowMeta h{};
    h.pos = a.pos[m];
    const bool is_q = j < a.Hq;
    const bool is_k = !is_q && j < a.Hq + a.Hkv;
    if (h.pos < 0 || h.pos >= a.max_pos) return h;
    if (is_q || is_k) {
        const float* w = is_q ? a.qn_w : a.kn_w;
#pragma unroll
        for (int k = 0; k < 4; ++k) h.w[k] = w[lane + 32 * k];
        const float2* cs = a.rope + (size_t)h.pos * (D / 2);
        h.rot[0] = cs[lane];
        h.rot[1] = cs[lane + 32];
    }
    if (!is_q) h.page = a.block_table[(size_t)a.slot[m] * a.bt_stride + h.pos / kPageTokens];
    return h;
}

// q_dst (optional): where a q head goes instead of a.q_out (128 floats, any address space);
// kv_dst (optional): a second copy of a K / V head's 128 f16 values besides the page.
__device__ __forceinline__ void qkv_head_apply(const AppendArgs& a, const HeadRowMeta& h, int m, int j, int lane,
                                               float (&x)[4], float* q_dst = nullptr, __half* kv_dst = nullptr) {
    constexpr int D = 128;
    const int pos = h.pos;
    const bool is_q = j < a.Hq;
    const bool is_k = !is_q && j < a.Hq + a.Hkv;
    if (pos < 0 || pos >= a.max_pos) {
        if (lane == 0) record_error(a.err, kDevErrBadPos);
        return;
    }

    if (is_q || is_k) {
        double ss = 0.0;
#pragma unroll
        for (int k = 0; k < 4; ++k) ss += (double)__fmul_rn(x[k], x[k]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float mean = (float)(ss * (1.0 / D));      // D = 128: exactly ss / D
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
        float y[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) y[k] = __fmul_rn(__fmul_rn(x[k], scale), h.w[k]);
        // pair (y[0], y[2]) uses rotation index lane, pair (y[1], y[3]) index lane + 32
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const float2 r = h.rot[k];
            const float x0 = y[k], x1 = y[k + 2];
            y[k] = __fsub_rn(__fmul_rn(x0, r.x), __fmul_rn(x1, r.y));
            y[k + 2] = __fadd_rn(__fmul_rn(x0, r.y), __fmul_rn(x1, r.x));
        }
        if (is_q) {
            float* dst = q_dst ? q_dst : a.q_out + ((size_t)m * a.Hq + j) * D;
#pragma unroll
            for (int k = 0; k < 4; ++k) dst[lane + 32 * k] = __fmul_rn(y[k], a.q_scale);
            return;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) x[k] = y[k];
    }

    // K (rotated) or V (as projected) into the page of this row's token.
    const int hh = is_k ? (j - a.Hq) : (j - a.Hq - a.Hkv);
    const int kv = is_k ? 0 : 1;
    const int page = h.page;
    if (page < 0 || page >= a.n_pages) {
        if (lane == 0) record_error(a.err, kDevErrBadPage);
        return;
    }
    __half* dst = a.pool_layer + (size_t)page * a.Hkv * 2 * kPageTokens * D +
                  ((size_t)(hh * 2 + kv) * kPageTokens + pos % kPageTokens) * D;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const __half v = __float2half_rn(x[k]);
        dst[lane + 32 * k] = v;
        if (kv_dst) kv_dst[lane + 32 * k] = v;
    }
}

// qkv_head_apply for R rows of the same head vector at once (row r live when live[r]): the
// same operations per row, written side by side so that the rows' dependency chains (the
// double-precision sum of squares across the warp, the correctly rounded divide and
// square root) overlap.
template <int R>
__device__ __forceinline__ void qkv_head_apply_rows(const AppendArgs& a, const HeadRowMeta* h, const int* m, int j,
                                                    int lane, float (&x)[R][4], const bool* live) {
    constexpr int D = 128;
    const bool is_q = j < a.Hq;
    const bool is_k = !is_q && j < a.Hq + a.Hkv;
    bool ok[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        ok[r] = live[r] && h[r].pos >= 0 && h[r].pos < a.max_pos;
        if (live[r] && !ok[r] && lane == 0) record_error(a.err, kDevErrBadPos);
    }
    if (is_q || is_k) {
        double ss[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            ss[r] = 0.0;
#pragma unroll
            for (int k = 0; k < 4; ++k) ss[r] += (double)__fmul_rn(x[r][k], x[r][k]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int r = 0; r < R; ++r) ss[r] += __shfl_xor_sync(0xffffffffu, ss[r], o);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float mean = (float)(ss[r] * (1.0 / D));
            const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
            float y[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) y[k] = __fmul_rn(__fmul_rn(x[r][k], scale), h[r].w[k]);
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const float2 rr = h[r].rot[k];
                const float x0 = y[k], x1 = y[k + 2];
                y[k] = __fsub_rn(__fmul_rn(x0, rr.x), __fmul_rn(x1, rr.y));
                y[k + 2] = __fadd_rn(__fmul_rn(x0, rr.y), __fmul_rn(x1, rr.x));
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) x[r][k] = y[k];
        }
        if (is_q) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (!ok[r]) continue;
                float* dst = a.q_out + ((size_t)m[r] * a.Hq + j) * D;
#pragma unroll
                for (int k = 0; k < 4; ++k) dst[lane + 32 * k] = __fmul_rn(x[r][k], a.q_scale);
            }
            return;
        }
    }
    const int hh = is_k ? (j - a.Hq) : (j - a.Hq - a.Hkv);
    const int kv = is_k ? 0 : 1;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        if (!ok[r]) continue;
        const int page = h[r].page;
        if (page < 0 || page >= a.n_pages) {
            if (lane == 0) record_error(a.err, kDevErrBadPage);
            continue;
        }
        __half* dst = a.pool_layer + (size_t)page * a.Hkv * 2 * kPageTokens * D +
                      ((size_t)(hh * 2 + kv) * kPageTokens + h[r].pos % kPageTokens) * D;
#pragma unroll
        for (int k = 0; k < 4; ++k) dst[lane + 32 * k] = __float2half_rn(x[r][k]);
    }
}

// The head vector j of row m summed over the QKV GEMM's split-K partials, in partial
// order with 8 partials' loads in flight at a time (lane l: dims l, l+32, l+64, l+96):
// kernel (1)'s input, wherever kernel (1) runs.
__device__ __forceinline__ void qkv_head_sum(const AppendArgs& a, int m, int j, int lane, float (&x)[4]) {
    constexpr int D = 128;
    const int W = (a.Hq + 2 * a.Hkv) * D;
#pragma unroll
    for (int k = 0; k < 4; ++k) x[k] = 0.0f;
    const float* base = a.qkv_part + (size_t)m * W + (size_t)j * D + lane;
    const size_t stride = (size_t)a.M * W;
    for (int s0 = 0; s0 < a.n_part; s0 += 8) {
        float t[8][4];
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (s0 + u < a.n_part)
#pragma unroll
                for (int k = 0; k < 4; ++k) t[u][k] = base[(size_t)(s0 + u) * stride + 32 * k];
#pragma unroll
        for (int u = 0; u < 8; ++u)
            if (s0 + u < a.n_part)
#pragma unroll
                for (int k = 0; k < 4; ++k) x[k] = __fadd_rn(x[k], t[u][k]);
    }
}

__device__ __forceinline__ void qkv_head_finish(const AppendArgs& a, int m, int j, int lane, float (&x)[4]) {
    const HeadRowMeta h = qkv_head_meta(a, m, j, lane);
    qkv_head_apply(a, h, m, j, lane, x);
}

}  // namespace fa
