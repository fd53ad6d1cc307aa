// Kernel (2): paged GQA decode attention over the f16 page pool.
//
// Replaces the reference's attention subgraph (compute/llm_ops_gpu.cpp:98-143):
// the full-cache views, three cont(permute) copies and two ggml_repeat 8->16 GQA
// expansions of K and V, scores = K.q/sqrt(128), diag_mask_inf, soft_max and the
// V^T.p matmul. Here each KV head is read from HBM once and serves both of its
// query heads (query head H uses KV head H/2, as the reference's repeat/permute
// order gives), and the softmax is an online softmax in fp32.
//
// Work split: one CTA per (split of `pages_per_split` pages, KV head, row); the CTA's
// four warps run the body in k_attn_body.cuh (page ring, scores, online softmax, PV,
// merge of the warps). With several splits the un-normalised partials go to the scratch
// buffer and are merged either by the split of each (row, KV head) that finishes last
// (AttnArgs::merge_cnt given: the decoder's steps) or by attn_combine (the op entry points).
//
// Roofline: HBM. Algorithmic bytes per (row, layer) = n_kv * 8 heads * 2 * 128 * 2 B
// = n_kv * 4096 B; compute is 4 flop per byte read.
#include "fa_kernels.cuh"
#include "k_append.cuh"
#include "k_attn_body.cuh"
#include "funasr_dec.h"

#include <cmath>
#include <mutex>
#include <string>

namespace fa {

namespace {

using attn::D;
template <int NW>
using AttnSmem = attn::Smem<kAttnStages, NW>;

// NW warps per CTA: 4 (3 CTAs per SM) in general, 8 for steps of at most kAttnWideRows rows,
// whose few CTAs would otherwise leave each warp several pages in a row. APPEND: the form
// that runs kernel (1) itself (AttnArgs::fuse_append); a separate instance, so that the
// plain form's page loop carries no patch branch.
template <int NW, bool APPEND>
__global__ void __launch_bounds__(NW * 32, NW == 4 ? kAttnCtasPerSm : 1) paged_attn_kernel(const AttnArgs a) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    AttnSmem<NW>& S = *reinterpret_cast<AttnSmem<NW>*>(smem_raw);
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
    if (attn::row_len_bad(a, n_kv, n_row_pages)) {
        if (split == 0 && threadIdx.x == 0) record_error(a.err, kDevErrBadLen);
        return;
    }
    const int p_begin = split * a.pages_per_split;
    if (p_begin >= n_row_pages) return;                 // uniform for the CTA
    const int p_end = min(n_row_pages, p_begin + a.pages_per_split);
    const int* bt = a.block_table + (size_t)a.slot[m] * a.bt_stride;

    if (threadIdx.x == 0) {
        for (int w = 0; w < NW; ++w)
            for (int s = 0; s < kAttnStages; ++s) mbar_init(&S.bars[w][s], 1);
        fence_mbar_init();
    }
    if (!APPEND && threadIdx.x < D) {
        const float* qg = a.q + ((size_t)m * a.Hq + 2 * h) * D;
        S.q[0][threadIdx.x] = qg[threadIdx.x] * attn::kLog2e;
        S.q[1][threadIdx.x] = qg[D + threadIdx.x] * attn::kLog2e;
    }
    __syncthreads();

    int nw = attn::warp_page_count(p_end - p_begin, warp, NW);
    nw = attn::warp_check_pages(a, bt, p_begin, nw, warp, lane, NW);
    const size_t page_elems = (size_t)a.Hkv * attn::TILE_HALVES;
    const __half* head_base = a.pool_layer + (size_t)h * attn::TILE_HALVES;
    const int issued = attn::warp_issue_first(S, bt, p_begin, nw, head_base, page_elems, warp, lane);
    const __half* patch = nullptr;
    int patch_i = -1, patch_t = 0;
    if constexpr (APPEND) {
        // kernel (1) for this KV head while the first pages are in flight: warps 0 and 1
        // the two query heads (into shared memory), warps 2 and 3 the K and V heads when
        // this split holds the token's page (written to the page, and kept to patch this
        // CTA's copy of it, which may have been taken before the write)
        __shared__ __align__(16) __half newkv[2 * D];
        const int p_last = n_row_pages - 1;
        const bool owner = p_last >= p_begin && p_last < p_end;
        if (warp < 4 && (warp < 2 || owner)) {
            const int j = warp < 2 ? 2 * h + warp : (warp == 2 ? a.Hq + h : a.Hq + a.Hkv + h);
            float x[4];
            qkv_head_sum(a.app, m, j, lane, x);
            const HeadRowMeta meta = qkv_head_meta(a.app, m, j, lane);
            qkv_head_apply(a.app, meta, m, j, lane, x, warp < 2 ? S.q[warp] : nullptr,
                           warp < 2 ? nullptr : newkv + (warp - 2) * D);
        }
        __syncthreads();
        if (threadIdx.x < D) {
            S.q[0][threadIdx.x] = S.q[0][threadIdx.x] * attn::kLog2e;
            S.q[1][threadIdx.x] = S.q[1][threadIdx.x] * attn::kLog2e;
        }
        __syncthreads();
        if (owner) {
            const int rel = p_last - p_begin;
            patch = newkv;
            patch_i = warp == rel % NW ? rel / NW : -1;
            patch_t = (n_kv - 1) % kPageTokens;
        }
    }
    attn::warp_pages(a, S, bt, p_begin, nw, issued, n_kv, head_base, page_elems, patch, patch_i, patch_t, warp,
                     lane);
    __syncthreads();
    if (threadIdx.x < D)
        attn::merge_warps(S, threadIdx.x, [&](int hq, float M, float L, float O) {
            attn::merge_store(a, split, h, m, threadIdx.x, hq, M, L, O);
        });
    if (!a.merge_cnt || a.n_splits == 1) return;
    // The split merge here: the CTA that counts its (row, KV head) last merges the splits
    // of both query heads (the partials it reads are at L2; the count is reset for the next
    // launch). No CTA waits for another.
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
        const int n_valid = min(a.n_splits, (n_row_pages + a.pages_per_split - 1) / a.pages_per_split);
        int* cnt = a.merge_cnt + (size_t)m * a.Hkv + h;
        __threadfence();
        last = atomicAdd(cnt, 1) == n_valid - 1;
        if (last) {
            __threadfence();
            *cnt = 0;
        }
    }
    __syncthreads();
    if (last && warp < 2) {
        const int H = 2 * h + warp;
        const size_t o = (size_t)m * a.Hq * D + (size_t)H * D;
        attn::combine_head<true>(a, m, H, lane, [&](int d, float v) { attn::store_out(a, o + d, v); });
    }
}

// Merge of the split partials: a warp per (row, query head).
__global__ void __launch_bounds__(256) attn_combine_kernel(const AttnArgs a) {
    pdl_trigger();
    pdl_wait();
    const int w = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= a.M * a.Hq) return;
    const int m = a.rows ? a.rows[w / a.Hq] : w / a.Hq;
    const int H = w % a.Hq;
    const size_t o = (size_t)m * a.Hq * D + (size_t)H * D;
    attn::combine_head<false>(a, m, H, lane, [&](int d, float v) { attn::store_out(a, o + d, v); });
}

}  // namespace

size_t attn_smem_bytes() { return sizeof(AttnSmem<4>); }

int attn_warps(int M) { return M <= kAttnWideRows ? 8 : 4; }

// Opt the kernels into their dynamic shared memory on the current device.
cudaError_t configure_attention() {
    cudaError_t e = cudaFuncSetAttribute(paged_attn_kernel<4, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(AttnSmem<4>));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(paged_attn_kernel<4, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)sizeof(AttnSmem<4>));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(paged_attn_kernel<8, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)sizeof(AttnSmem<8>));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(paged_attn_kernel<8, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)sizeof(AttnSmem<8>));
    return e;
}

void launch_paged_attention(const AttnArgs& a, cudaStream_t s) {
    dim3 grid(a.n_splits, a.Hkv, a.M);
    const int warps = a.warps ? a.warps : attn_warps(a.M);
    if (warps == 8) {
        if (a.fuse_append) launch_k(paged_attn_kernel<8, true>, grid, dim3(256), sizeof(AttnSmem<8>), s, a);
        else launch_k(paged_attn_kernel<8, false>, grid, dim3(256), sizeof(AttnSmem<8>), s, a);
    } else {
        if (a.fuse_append) launch_k(paged_attn_kernel<4, true>, grid, dim3(128), sizeof(AttnSmem<4>), s, a);
        else launch_k(paged_attn_kernel<4, false>, grid, dim3(128), sizeof(AttnSmem<4>), s, a);
    }
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
