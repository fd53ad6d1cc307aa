// Kernel (1): fused per-head Q/K RMSNorm + NEOX RoPE + paged f16 K/V append.
//
// Replaces, per layer and step, the ggml node chain of the reference's
// gpu_gqa_forward (compute/llm_ops_gpu.cpp:57-96): reshape, gpu_rms_norm on q/k
// (ggml_rms_norm + cast + mul, :16-25), ggml_rope_ext mode 2 (:72-75), and the
// ggml_cpy of K/V into the f32 cache slot (:84-96). The cache here is paged f16.
//
// Arithmetic is written with explicit round-to-nearest intrinsics so that the
// K page bytes equal those of the CPU oracle given the same f32 inputs:
//   ss    = sum over 128 of (double)(x*x)      (ggml CPU rms_norm sums in double)
//   scale = 1 / sqrt((float)(ss/128) + eps)     (correctly rounded div and sqrt)
//   y     = (x * scale) * w
//   rope  : y0' = y0*c - y1*s, y1' = y0*s + y1*c, no fused multiply-add
//   K, V  : f32 -> f16 round-to-nearest-even
//
// Grid: (M rows, (Hq + 2*Hkv) / 8 head groups); 8 warps, one warp per 128-wide
// head vector, lane l owning dims {l, l+32, l+64, l+96} so both NEOX pairs
// (l, l+64) and (l+32, l+96) stay in one lane. Memory-bound on nothing: a few KB
// per row; it exists to avoid ~10 ggml launches and the f32 cache round trip.
#include "fa_kernels.cuh"
#include "k_append.cuh"

namespace fa {

namespace {

constexpr int D = 128;

__global__ void __launch_bounds__(256) qknorm_rope_append_kernel(AppendArgs a) {
    pdl_trigger();
    pdl_wait();
    const int m = blockIdx.x;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int j = blockIdx.y * 8 + warp;          // head vector index in the qkv row
    const int n_vec = a.Hq + 2 * a.Hkv;
    if (j >= n_vec) return;
    float x[4];
    qkv_head_sum(a, m, j, lane, x);
    qkv_head_finish(a, m, j, lane, x);
}

// Raw append: one warp copies one (row, layer, head) pair of 256 B K and 256 B V rows.
__global__ void __launch_bounds__(256) kv_append_raw_kernel(RawAppendArgs a) {
    const int gw = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int total = a.M * a.n_layers * a.Hkv;
    if (gw >= total) return;
    const int h = gw % a.Hkv;
    const int l = (gw / a.Hkv) % a.n_layers;
    const int m = gw / (a.Hkv * a.n_layers);
    const int pos = a.pos[m];
    const int page = a.block_table[(size_t)a.slot[m] * a.bt_stride + pos / kPageTokens];
    if (pos < 0 || page < 0 || page >= a.n_pages) {
        if (lane == 0) record_error(a.err, kDevErrBadPage);
        return;
    }
    const size_t page_elems = (size_t)a.Hkv * 2 * kPageTokens * D;
    __half* pg = a.pool + ((size_t)l * a.n_pages + page) * page_elems;
    const size_t src = (((size_t)m * a.n_layers + l) * a.Hkv + h) * D;
    const int t = pos % kPageTokens;
    // 128 halves = 16 x 16 B; lanes 0..15 copy K, lanes 16..31 copy V
    const int c = lane & 15;
    const __half* s = (lane < 16 ? a.k : a.v) + src;
    __half* d = pg + ((size_t)(h * 2 + (lane < 16 ? 0 : 1)) * kPageTokens + t) * D;
    reinterpret_cast<uint4*>(d)[c] = reinterpret_cast<const uint4*>(s)[c];
}

// Gather: one CTA copies one page of one sequence in one layer (64 KiB: 8 heads x K|V x
// 16 tokens x 128) into the head-major slabs. Each (head, K|V) part of a page is 4 KiB of
// consecutive tokens and lands as 4 KiB of consecutive rows, so every warp access is 512 B
// contiguous on both sides; a thread issues its 16 loads before any store.
__global__ void __launch_bounds__(256) kv_gather_kernel(GatherArgs a) {
    const int pi = blockIdx.x, m = blockIdx.y, l = blockIdx.z;
    const int n_kv = a.n_kv[m], row0 = a.row0[m];
    if (n_kv < 0 || n_kv > a.max_pages * kPageTokens || row0 < 0 || row0 + n_kv > a.total_rows) {
        if (pi == 0 && l == 0 && threadIdx.x == 0) record_error(a.err, kDevErrBadLen);
        return;
    }
    const int t0 = pi * kPageTokens;
    if (t0 >= n_kv) return;
    const int page = a.block_table[(size_t)a.slot[m] * a.bt_stride + pi];
    if (page < 0 || page >= a.n_pages) {
        if (threadIdx.x == 0) record_error(a.err, kDevErrBadPage);
        return;
    }
    const int nt = min(kPageTokens, n_kv - t0);
    const int t = threadIdx.x >> 4;         // token within the page
    const int c = threadIdx.x & 15;         // 16 B column within the 256 B row
    const size_t page_vec = (size_t)a.Hkv * 2 * kPageTokens * D / 8;
    const uint4* src = reinterpret_cast<const uint4*>(a.pool) + ((size_t)l * a.n_pages + page) * page_vec;
    if (t >= nt) return;
    uint4 r[16];
#pragma unroll
    for (int j = 0; j < 16; ++j)
        if (j < 2 * a.Hkv) r[j] = src[(size_t)j * kPageTokens * (D / 8) + threadIdx.x];
    const size_t row = (size_t)row0 + t0 + t;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        if (j >= 2 * a.Hkv) break;
        const int h = j >> 1;
        __half* out = (j & 1) ? a.v_out : a.k_out;
        uint4* dst = reinterpret_cast<uint4*>(out + (((size_t)l * a.Hkv + h) * a.total_rows + row) * D);
        dst[c] = r[j];
    }
}

}  // namespace

void launch_kv_gather(const GatherArgs& a, cudaStream_t s) {
    dim3 grid(a.max_pages, a.M, a.n_layers);
    kv_gather_kernel<<<grid, 256, 0, s>>>(a);
}

void launch_qknorm_rope_append(const AppendArgs& a, cudaStream_t s) {
    const int n_vec = a.Hq + 2 * a.Hkv;
    dim3 grid(a.M, (n_vec + 7) / 8);
    launch_k(qknorm_rope_append_kernel, grid, dim3(256), 0, s, a);
}

void launch_kv_append_raw(const RawAppendArgs& a, cudaStream_t s) {
    const int total = a.M * a.n_layers * a.Hkv;
    kv_append_raw_kernel<<<(total + 7) / 8, 256, 0, s>>>(a);
}

}  // namespace fa
