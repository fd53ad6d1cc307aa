// Small fused kernels around the three big ones:
//   embed            : token -> f32 hidden row (pipeline/prompt_builder.hpp:93-113, BF16/F16/F32
//                      tables), done on the device instead of on the host per token
//   residual_rmsnorm : x += sum of split-K partials of the previous projection
//                      (ggml_add residual, compute/llm_ops_gpu.cpp:172,182), then
//                      f16(rms_norm(x) * w) for the next GEMM (gpu_rms_norm, :16-25)
//   swiglu           : f16(silu(gate) * up) from the gate/up GEMM partials (:177-180)
//   argmax_reduce    : first maximum over lm_head tiles (compute/gpu_runner.hpp:108-118)
//   repack_q8        : GGUF Q8_0 blocks -> f16(d * q) weight matrix (the encoder's weights)
//   repack_q8_planes : GGUF Q8_0 blocks -> the q / d_t / d_r planes the decoder GEMMs read
//   page_copy / fill_random / read_pages / apply_bt_updates : page-pool maintenance
#include "fa_kernels.cuh"
#include "q8_planes.cuh"
#include "k_norm.cuh"

namespace fa {

namespace {

__global__ void __launch_bounds__(256) embed_kernel(const void* table, int table_type, int hidden,
                                                    const int* tokens, const float* embeds, int vocab,
                                                    float* x, int* err) {
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.x;
    float* dst = x + (size_t)m * hidden;
    if (embeds) {
        for (int i = threadIdx.x; i < hidden; i += blockDim.x) dst[i] = embeds[(size_t)m * hidden + i];
        return;
    }
    const int tok = tokens[m];
    if (tok == -1) return;   // the row was loaded from embeddings
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0) record_error(err, kDevErrBadPage);
        for (int i = threadIdx.x; i < hidden; i += blockDim.x) dst[i] = 0.0f;
        return;
    }
    const size_t off = (size_t)tok * hidden;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        float v;
        if (table_type == 30) v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(table)[off + i]);
        else if (table_type == 1) v = __half2float(reinterpret_cast<const __half*>(table)[off + i]);
        else v = reinterpret_cast<const float*>(table)[off + i];
        dst[i] = v;
    }
}

// One CTA per row (residual_norm_row's 256-thread order); G partials' loads in flight per
// round (16 for the decode step's split-16 projections, 8 otherwise: 136 vs ~80 registers).
template <int G>
__global__ void __launch_bounds__(256) residual_rmsnorm_kernel(float* x, const float* part, int n_part, int M,
                                                               int hidden, const float* w, float eps,
                                                               __half* xn_hi, __half* xn_lo, const int* rows) {
    __shared__ double sh[8];
    pdl_trigger();
    pdl_wait();
    const int m = rows ? rows[blockIdx.x] : (int)blockIdx.x;   // source row; output row blockIdx.x
    const int n4 = hidden / 4;
    float* xr = x + (size_t)m * hidden;
    const size_t o = (size_t)blockIdx.x * hidden;
    residual_norm_row<G>(xr, reinterpret_cast<const float4*>(part) + (size_t)m * n4, (size_t)M * n4, n_part, hidden, w,
                      eps, n_part > 0 ? xr : nullptr, sh,
                      [&](int j, float y) { split_store(y, xn_hi, xn_lo, o + j); });
}

// Thread per float4 group of one row's ffn outputs. Columns of a partial row: gate
// [0, ffn) then up [ffn, 2 ffn), or with interleave64 blocks of 64 gate columns followed by
// the 64 up columns of the same outputs (the decoder's stacking of the gate/up weights).
__global__ void __launch_bounds__(256) swiglu_kernel(const float* part, int n_part, int M, int ffn,
                                                     __half* h_hi, __half* h_lo, int interleave64) {
    pdl_trigger();
    pdl_wait();
    const size_t idx = (size_t)blockIdx.x * 256 + threadIdx.x;
    const int f4 = ffn / 4;
    if (idx >= (size_t)M * f4) return;
    const int m = (int)(idx / f4), j = (int)(idx % f4);
    const float4* p = reinterpret_cast<const float4*>(part) + (size_t)m * 2 * f4;
    const size_t stride4 = (size_t)M * 2 * f4;
    const int gj = interleave64 ? (j / 16) * 32 + j % 16 : j;
    const int uj = interleave64 ? gj + 16 : f4 + j;
    const float4 g = sum_parts4(p + gj, stride4, n_part);
    const float4 u = sum_parts4(p + uj, stride4, n_part);
    const size_t o = (size_t)m * ffn + 4 * (size_t)j;
    split_store(silu_mul(g.x, u.x), h_hi, h_lo, o);
    split_store(silu_mul(g.y, u.y), h_hi, h_lo, o + 1);
    split_store(silu_mul(g.z, u.z), h_hi, h_lo, o + 2);
    split_store(silu_mul(g.w, u.w), h_hi, h_lo, o + 3);
}

__global__ void __launch_bounds__(256) argmax_reduce_kernel(const float* val, const int* idx, int n_tiles,
                                                            int* next, int* feed_tokens, int* feed_pos) {
    __shared__ float sv[8];
    __shared__ int si[8];
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.x;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int t = threadIdx.x; t < n_tiles; t += 256) {
        const float v = val[(size_t)m * n_tiles + t];
        const int i = idx[(size_t)m * n_tiles + t];
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
        // all-NaN or empty rows fall back to index 0, as the reference's scan does
        if (bi == 0x7fffffff) bi = 0;
        next[m] = bi;
        if (feed_tokens) feed_tokens[m] = bi;
        if (feed_pos) feed_pos[m] += 1;
    }
}

__global__ void apply_bt_updates_kernel(int* bt, const int* upd_idx, const int* upd_page, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) bt[upd_idx[i]] = upd_page[i];
}

__global__ void repack_q8_kernel(const uint8_t* raw, int N, int K, int r0, __half* dst_w) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int nb = K / kQK;
    if (i >= (size_t)N * nb) return;
    const int n = (int)(i / nb), b = (int)(i % nb);
    const uint8_t* blk = raw + i * kQBytes;
    const float d = __half2float(__ushort_as_half((uint16_t)blk[0] | ((uint16_t)blk[1] << 8)));
    __half* w = dst_w + (size_t)(r0 + n) * K + (size_t)b * kQK;
#pragma unroll
    for (int j = 0; j < kQK; ++j) w[j] = __float2half_rn(__fmul_rn(d, (float)(int8_t)blk[2 + j]));
}

// One thread per Q8_0 block: the 32 values go to q row r0 + n, the scale to both
// scale planes (block-major d_t with row length n_total, row-major d_r).
__global__ void repack_q8_planes_kernel(const uint8_t* raw, int N, int K, int r0, int n_total, int8_t* q,
                                        __half* d_t, __half* d_r, int ileave) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int nb = K / kQK;
    if (i >= (size_t)N * nb) return;
    const int n_src = (int)(i / nb), b = (int)(i % nb);
    // row n_src lands at r0 + n_src, or with ileave at r0 + blocks of ileave rows spaced 2 * ileave
    const int n = ileave ? (n_src / ileave) * 2 * ileave + n_src % ileave : n_src;
    const uint8_t* blk = raw + i * kQBytes;
    const __half d = __ushort_as_half((uint16_t)blk[0] | ((uint16_t)blk[1] << 8));
    d_t[(size_t)b * n_total + r0 + n] = d;
    d_r[(size_t)(r0 + n) * nb + b] = d;
    int8_t* dst = q + (size_t)(r0 + n) * K + (size_t)b * kQK;
#pragma unroll
    for (int j = 0; j < kQK; ++j) dst[j] = (int8_t)blk[2 + j];
}

__global__ void __launch_bounds__(256) page_copy_kernel(__half* pool, size_t layer_stride, const int* src,
                                                        const int* dst, size_t page_elems) {
    const int i = blockIdx.x, l = blockIdx.y;
    const uint4* s = reinterpret_cast<const uint4*>(pool + l * layer_stride + (size_t)src[i] * page_elems);
    uint4* d = reinterpret_cast<uint4*>(pool + l * layer_stride + (size_t)dst[i] * page_elems);
    const size_t n16 = page_elems * 2 / 16;
    for (size_t k = threadIdx.x; k < n16; k += 256) d[k] = s[k];
}

__device__ __forceinline__ uint32_t hash32(uint64_t x) {
    x ^= x >> 33;
    x *= 0xff51afd7ed558ccdull;
    x ^= x >> 33;
    x *= 0xc4ceb9fe1a85ec53ull;
    x ^= x >> 33;
    return (uint32_t)x;
}

// Fills whole pages with deterministic values in [-2, 2): synthetic steady-state cache.
__global__ void __launch_bounds__(256) fill_random_kernel(__half* pool, size_t layer_stride, const int* pages,
                                                          size_t page_elems, unsigned long long seed) {
    const int i = blockIdx.x, l = blockIdx.y;
    __half* d = pool + l * layer_stride + (size_t)pages[i] * page_elems;
    for (size_t k = threadIdx.x; k < page_elems; k += 256) {
        const uint32_t h = hash32(seed ^ ((((uint64_t)l << 40) | ((uint64_t)pages[i] << 20)) + k * 0x9e3779b97f4a7c15ull));
        d[k] = __float2half_rn((float)(h >> 8) * (4.0f / 16777216.0f) - 2.0f);
    }
}

__global__ void __launch_bounds__(256) read_pages_kernel(const __half* pool_layer, const int* pages,
                                                         size_t page_elems, __half* out) {
    const int i = blockIdx.x;
    const uint4* s = reinterpret_cast<const uint4*>(pool_layer + (size_t)pages[i] * page_elems);
    uint4* d = reinterpret_cast<uint4*>(out + (size_t)i * page_elems);
    const size_t n16 = page_elems * 2 / 16;
    for (size_t k = threadIdx.x; k < n16; k += 256) d[k] = s[k];
}

// Self-test of the bounded waits every pipelined kernel uses: one CTA arms an
// mbarrier for a byte count that no copy will ever deliver and waits on it with a
// short limit. The wait must give up, record kDevErrTimeout and let the kernel
// return normally, leaving the context usable.
__global__ void wait_selftest_kernel(int* err, unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(&bar, 16);   // 16 bytes that never arrive
    }
    __syncthreads();
    const bool got = mbar_wait_bounded(&bar, 0, limit_ns);
    if (!got && threadIdx.x == 0) record_error(err, kDevErrTimeout);
}

}  // namespace

void launch_embed(const void* table, int table_type, int hidden, const int* tokens, const float* embeds, int M,
                  int vocab, float* x, int* err, cudaStream_t s) {
    launch_k(embed_kernel, dim3(M), dim3(256), 0, s, table, table_type, hidden, tokens, embeds, vocab, x, err);
}

void launch_residual_rmsnorm(float* x, const float* part, int n_part, int M, int hidden, const float* w, float eps,
                             __half* xn_hi, __half* xn_lo, cudaStream_t s, int n_out, const int* rows) {
    if (n_out < 0) n_out = M;
    if (n_part > 8)
        launch_k(residual_rmsnorm_kernel<16>, dim3(n_out), dim3(256), 0, s, x, part, n_part, M, hidden, w, eps, xn_hi,
                 xn_lo, rows);
    else
        launch_k(residual_rmsnorm_kernel<8>, dim3(n_out), dim3(256), 0, s, x, part, n_part, M, hidden, w, eps, xn_hi,
                 xn_lo, rows);
}

void launch_swiglu(const float* part, int n_part, int M, int ffn, __half* h_hi, __half* h_lo, cudaStream_t s,
                   bool interleave64) {
    const size_t n = (size_t)M * (ffn / 4);
    launch_k(swiglu_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, part, n_part, M, ffn, h_hi, h_lo,
             interleave64 ? 1 : 0);
}

void launch_argmax_reduce(const float* val, const int* idx, int M, int n_tiles, int* next, int* feed_tokens,
                          int* feed_pos, cudaStream_t s) {
    launch_k(argmax_reduce_kernel, dim3(M), dim3(256), 0, s, val, idx, n_tiles, next, feed_tokens, feed_pos);
}

void launch_apply_bt_updates(int* block_table, const int* upd_idx, const int* upd_page, int n, cudaStream_t s) {
    if (n <= 0) return;
    apply_bt_updates_kernel<<<(n + 255) / 256, 256, 0, s>>>(block_table, upd_idx, upd_page, n);
}

void launch_repack_q8(const uint8_t* raw, int N, int K, int r0, __half* dst_w, cudaStream_t s) {
    const size_t n = (size_t)N * (K / kQK);
    repack_q8_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(raw, N, K, r0, dst_w);
}

void launch_repack_q8_planes(const uint8_t* raw, int N, int K, int r0, int n_total, void* planes, cudaStream_t s,
                             int interleave) {
    const size_t n = (size_t)N * (K / kQK);
    unsigned char* b = static_cast<unsigned char*>(planes);
    repack_q8_planes_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
        raw, N, K, r0, n_total, reinterpret_cast<int8_t*>(b), reinterpret_cast<__half*>(b + q8p_dt_offset(n_total, K)),
        reinterpret_cast<__half*>(b + q8p_dr_offset(n_total, K)), interleave);
}

void launch_page_copy(__half* pool, size_t layer_stride, int n_layers, const int* src, const int* dst, int n,
                      cudaStream_t s) {
    if (n <= 0) return;
    const size_t page_elems = (size_t)8 * 2 * kPageTokens * 128;
    page_copy_kernel<<<dim3(n, n_layers), 256, 0, s>>>(pool, layer_stride, src, dst, page_elems);
}

void launch_fill_random(__half* pool, size_t layer_stride, int n_layers, const int* pages, int n_pages_list,
                        unsigned long long seed, cudaStream_t s) {
    if (n_pages_list <= 0) return;
    const size_t page_elems = (size_t)8 * 2 * kPageTokens * 128;
    fill_random_kernel<<<dim3(n_pages_list, n_layers), 256, 0, s>>>(pool, layer_stride, pages, page_elems, seed);
}

void launch_read_pages(const __half* pool_layer, const int* pages, int n, __half* out, cudaStream_t s) {
    if (n <= 0) return;
    const size_t page_elems = (size_t)8 * 2 * kPageTokens * 128;
    read_pages_kernel<<<n, 256, 0, s>>>(pool_layer, pages, page_elems, out);
}

void launch_wait_selftest(int* err, unsigned long long limit_ns, cudaStream_t s) {
    wait_selftest_kernel<<<1, 32, 0, s>>>(err, limit_ns);
}

}  // namespace fa
