// C ABI of libfunasr_dec: context, weights, page pool, sequences, the batched
// decoder forward (captured as CUDA graphs), greedy generation and the
// kernel-level entry points. See include/funasr_dec.h for the contract.
//
// One forward over M rows launches, per layer:
//   residual_rmsnorm  (x += down-proj partials of the previous layer; f16 norm)
//   q8_gemm   QKV     (Wq|Wk|Wv concatenated: N = 4096)      -> split-K partials
//   qknorm_rope_append (sums the partials, writes q and the f16 K/V pages)
//   paged_attention (+ split combine)                         -> f16 [M][2048]
//   q8_gemm   o_proj                                          -> partials
//   residual_rmsnorm  (x += o; f16 post-attention norm)
//   q8_gemm   gate|up (N = 2*ffn)                             -> partials
//   swiglu                                                    -> f16 [M][ffn]
//   q8_gemm   down                                            -> partials
// then the final residual_rmsnorm, the lm_head GEMM with a fused argmax and
// the argmax reduce. This is the node list of the reference's per-token ggml
// graph (compute/llm_ops_gpu.cpp:155-207) with the copies removed and every
// elementwise op folded into a neighbour.
#include "fa_kernels.cuh"
#include "page_alloc.hpp"
#include "nvtx_range.hpp"
#include "funasr_dec.h"

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

namespace {

thread_local std::string g_err;

// Q8_0 weights on the device as q / d_t / d_r planes (q8_planes.cuh), one buffer per
// (stacked) matrix: the GGUF bytes rearranged, nothing rounded.
struct LayerW {
    unsigned char* qkv_q = nullptr;
    unsigned char* o_q = nullptr;
    unsigned char* gu_q = nullptr;
    unsigned char* dn_q = nullptr;
    float* in_norm = nullptr;
    float* post_norm = nullptr;
    float* q_norm = nullptr;
    float* k_norm = nullptr;
};

struct Seq {
    bool open = false;
    int len = 0;
    int max_tokens = 0;
    std::vector<int> pages;
};

constexpr int kD = 128;
constexpr int kHq = 16;
constexpr int kHkv = 8;
constexpr size_t kPageElems = (size_t)kHkv * 2 * fa::kPageTokens * kD;

std::mutex g_cfg_mu;
bool g_configured[64] = {};

}  // namespace

namespace fa {
namespace {
thread_local bool t_launch_pdl = false;
}
bool launch_pdl_enabled() { return t_launch_pdl; }
void set_launch_pdl(bool on) { t_launch_pdl = on; }
}  // namespace fa

// Kernel attribute set-up, once per device (before any graph capture).
namespace fa {
cudaError_t configure_attention();
void configure_gemm();
void configure_gemm_tc();
void configure_gemm_tc_skinny();
}  // namespace fa

static int ensure_configured() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return FA_ERR_CUDA;
    std::lock_guard<std::mutex> lk(g_cfg_mu);
    if (dev >= 0 && dev < 64 && !g_configured[dev]) {
        fa::configure_attention();
        fa::configure_gemm();
        fa::configure_gemm_tc();
        fa::configure_gemm_tc_skinny();
        fa::configure_prefill_attention();
        fa::configure_row_step();
        g_configured[dev] = true;
    }
    return FA_OK;
}

namespace fa {
// Kernel attributes (dynamic shared memory) of the current device, set once.
int ensure_device_configured() { return ensure_configured(); }
}  // namespace fa

struct fa_ctx {
    int device = 0;
    fa_model_desc d{};
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    int n_sm = 148;
    std::string err;

    bool loaded = false;
    std::vector<LayerW> L;
    void* embed = nullptr;
    int embed_type = FA_TYPE_BF16;
    float* final_norm = nullptr;
    unsigned char* lm_q = nullptr;
    std::vector<void*> dev_allocs;

    __half* pool = nullptr;
    size_t layer_stride = 0;   // elements between layers of the pool
    int n_pages = 0;
    int* bt_dev = nullptr;
    int bt_stride = 0;
    float2* rope = nullptr;
    fa::PageAllocator palloc;
    std::vector<Seq> seqs;

    // step buffers
    float* x = nullptr;
    __half* xn16 = nullptr;     // GEMM input activations: hi plane, lo plane at xn_lo
    __half* xn_lo = nullptr;
    float* part = nullptr;
    size_t part_elems = 0;
    float* q_rot = nullptr;
    __half* attn16 = nullptr;
    __half* attn_lo = nullptr;
    __half* h16 = nullptr;
    __half* h_lo = nullptr;
    float* att_po = nullptr;
    float* att_pml = nullptr;
    int* att_cnt = nullptr;        // [rows][Hkv] split counters of the in-kernel split merge
    int att_max_splits = 0;
    float* amax_v = nullptr;
    int* amax_i = nullptr;
    float* logits_dev = nullptr;
    int* row_tok = nullptr;
    int* row_slot = nullptr;
    int* row_pos = nullptr;
    int* next_dev = nullptr;
    int* upd_idx = nullptr;
    int* upd_page = nullptr;
    int max_updates = 0;
    int* err_dev = nullptr;
    int* scratch_ints = nullptr;   // compaction / synthetic-fill page lists
    int scratch_ints_n = 0;

    // pinned host staging
    int* h_rows = nullptr;     // tok | slot | pos | upd_idx | upd_page
    int* h_next = nullptr;
    int* h_err = nullptr;

    bool use_graphs = true;
    // bit 0: QKV + kernel (1), bit 1: gate/up + SwiGLU, finished in the tcgen05 GEMM's
    // clusters; bit 2: split merge inside the attention kernel; bit 3: kernel (1) inside the
    // attention kernel. Bit 0 is off: the QKV form measured slower (its per-row norm / RoPE /
    // append tail runs on 4 warps per SM, where the other forms spread it over every SM)
    int fuse_epilogues = 14;
    bool enqueue_failed = false; // a planned launch declined its arguments while a step was enqueued
    bool use_pdl = true;       // programmatic dependent launch between the step's kernels
    // one-row steps as one persistent kernel (k_row_step.cu) when the shapes allow it
    bool row_step_on = true;
    bool row_ready = false;    // buffers and the layer table below exist
    fa::RowGemm row_gm[4] = {};
    fa::RowLayer* row_layers = nullptr;
    unsigned long long* row_words = nullptr;   // the phases' tagged words (row_step_words)
    size_t row_words_n = 0;
    fa::RowCtl* row_ctl = nullptr;
    int row_absent_cta = -1;   // failure test (fa_set_row_step_fault)
    unsigned long long row_wait_ns = fa::kWaitLimitNs;
    std::string enqueue_msg;   // why a planned launch failed while a step was enqueued
    int gemm_variant = 0;      // 0: CUDA-core kernel up to 2 rows, swapped tcgen05 up to 128 (lm_head: 32),
                               // 128-row-tile tcgen05 above; 1: mma.sync; 2: 128-row-tile tcgen05;
                               // 3: CUDA-core up to 8 rows, else 2; 4: swapped tcgen05 up to 128, else 2
    struct GraphEntry {
        cudaGraphExec_t exec;
        int launches;
    };
    std::map<std::array<int, 12>, GraphEntry> graphs;
    // prefill tiles (first row, rows) and the rows left to the decode kernel
    int2* pf_tiles = nullptr;
    int* dec_rows = nullptr;
    int* out_rows = nullptr;     // rows whose next id / logits a step returns (when not all)
    CUtensorMap pool_map{};
    bool pool_map_ok = false;

    bool prof = false;
    std::vector<cudaEvent_t> prof_ev;   // pairs per attention launch
    int prof_n = 0;
    bool prof_row = false;     // the last profiled step ran the one-row step kernel
    int last_launches = 0;
    cudaEvent_t ev_t0 = nullptr, ev_t1 = nullptr;
};

#define FA_CK(call)                                                                    \
    do {                                                                               \
        cudaError_t e_ = (call);                                                       \
        if (e_ != cudaSuccess) {                                                       \
            return set_err(ctx, FA_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
        }                                                                              \
    } while (0)

static int set_err(const fa_ctx* cctx, int code, const std::string& msg) {
    if (cctx) const_cast<fa_ctx*>(cctx)->err = msg;
    g_err = msg;
    return code;
}

namespace fa {
// Records a context-free error (read back with fa_last_error(NULL)) for entry points
// defined in other translation units.
int report_op_error(int code, const char* msg) { return set_err(nullptr, code, msg); }
int report_ctx_error(const fa_ctx* ctx, int code, const char* msg) { return set_err(ctx, code, msg); }
int ensure_device_configured();
}  // namespace fa

template <typename T>
static int dev_alloc(fa_ctx* ctx, T** p, size_t bytes) {
    void* v = nullptr;
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(&v, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_err(ctx, FA_ERR_OOM, "cudaMalloc(" + std::to_string(bytes) + " B): " + cudaGetErrorString(e));
    }
    ctx->dev_allocs.push_back(v);
    *p = reinterpret_cast<T*>(v);
    return FA_OK;
}

// ------------------------------------------------------------------ basics --
extern "C" const char* fa_version(void) { return "funasr_dec sm_100a 0.1"; }

extern "C" const char* fa_last_error(const fa_ctx* ctx) { return ctx ? ctx->err.c_str() : g_err.c_str(); }

extern "C" void fa_default_desc(fa_model_desc* d) {
    if (!d) return;
    std::memset(d, 0, sizeof(*d));
    d->n_layers = 28;
    d->hidden = 1024;
    d->n_heads = 16;
    d->n_kv_heads = 8;
    d->head_dim = 128;
    d->ffn = 3072;
    d->vocab = 151936;
    d->rope_base = 1000000.0f;
    d->rms_eps = 1e-5f;
    d->max_ctx = 40960;
    d->n_pages = 0;
    d->kv_bytes = (size_t)4 << 30;
    d->max_seqs = 256;
    d->max_rows = 512;
}

static int validate_desc(const fa_model_desc* d) {
    if (!d) return set_err(nullptr, FA_ERR_INVALID_ARG, "desc is NULL");
    if (d->head_dim != kD || d->n_heads != kHq || d->n_kv_heads != kHkv)
        return set_err(nullptr, FA_ERR_INVALID_ARG,
                       "kernels are built for head_dim 128, 16 query heads, 8 KV heads");
    if (d->n_layers <= 0 || d->hidden <= 0 || d->hidden % 64 || d->ffn <= 0 || d->ffn % 64 || d->vocab <= 0 ||
        d->vocab % 64)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "n_layers > 0; hidden, ffn, vocab multiples of 64 required");
    if (d->hidden > 4096)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "hidden above 4096 is not supported by the norm kernel");
    if (d->max_ctx <= 0 || d->max_seqs <= 0 || d->max_rows <= 0 || d->max_rows > 4096)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "max_ctx, max_seqs > 0 and 0 < max_rows <= 4096 required");
    if (!(d->rms_eps > 0.0f) || !(d->rope_base > 0.0f))
        return set_err(nullptr, FA_ERR_INVALID_ARG, "rms_eps and rope_base must be positive");
    return FA_OK;
}

static int max_split_for(int K) { return std::max(1, K / 128); }

extern "C" fa_ctx* fa_create(int device, const fa_model_desc* desc) {
    if (validate_desc(desc) != FA_OK) return nullptr;
    int n_dev = 0;
    cudaError_t e = cudaGetDeviceCount(&n_dev);
    if (e != cudaSuccess || n_dev == 0) {
        set_err(nullptr, FA_ERR_CUDA, std::string("no CUDA device: ") + cudaGetErrorString(e));
        cudaGetLastError();
        return nullptr;
    }
    if (device < 0 || device >= n_dev) {
        set_err(nullptr, FA_ERR_INVALID_ARG, "device " + std::to_string(device) + " out of range");
        return nullptr;
    }
    if (cudaSetDevice(device) != cudaSuccess) {
        set_err(nullptr, FA_ERR_CUDA, "cudaSetDevice failed");
        return nullptr;
    }
    cudaDeviceProp prop{};
    cudaGetDeviceProperties(&prop, device);
    if (prop.major != 10) {
        set_err(nullptr, FA_ERR_CUDA,
                std::string("this library is built for sm_100a (B200); device is ") + prop.name);
        return nullptr;
    }
    if (ensure_configured() != FA_OK) {
        set_err(nullptr, FA_ERR_CUDA, "kernel configuration failed");
        return nullptr;
    }
    fa_ctx* ctx = new fa_ctx();
    ctx->device = device;
    ctx->d = *desc;
    ctx->n_sm = prop.multiProcessorCount;
    auto fail = [&](void) -> fa_ctx* {
        g_err = ctx->err;
        fa_destroy(ctx);
        return nullptr;
    };
    if (cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking) != cudaSuccess) {
        set_err(ctx, FA_ERR_CUDA, "cudaStreamCreate failed");
        return fail();
    }
    ctx->stream = ctx->own_stream;
    const fa_model_desc& d = ctx->d;

    // page pool
    const size_t page_bytes_all = kPageElems * 2 * (size_t)d.n_layers;
    int n_pages = d.n_pages;
    if (n_pages <= 0) n_pages = (int)std::max<size_t>(1, d.kv_bytes / page_bytes_all);
    ctx->n_pages = n_pages;
    ctx->layer_stride = (size_t)n_pages * kPageElems;
    if (dev_alloc(ctx, &ctx->pool, page_bytes_all * n_pages)) return fail();
    ctx->palloc.init(n_pages);
    ctx->bt_stride = (d.max_ctx + fa::kPageTokens - 1) / fa::kPageTokens;
    if (dev_alloc(ctx, &ctx->bt_dev, sizeof(int) * (size_t)d.max_seqs * ctx->bt_stride)) return fail();
    if (cudaMemset(ctx->bt_dev, 0, sizeof(int) * (size_t)d.max_seqs * ctx->bt_stride) != cudaSuccess) {
        set_err(ctx, FA_ERR_CUDA, "memset block table");
        return fail();
    }
    ctx->seqs.resize(d.max_seqs);

    // RoPE table: theta = pos * base^(-2i/128) in double, cos/sin in double, f32 once.
    {
        std::vector<float2> tab((size_t)d.max_ctx * (kD / 2));
        double inv[kD / 2];
        for (int i = 0; i < kD / 2; ++i) inv[i] = std::pow((double)d.rope_base, -2.0 * i / (double)kD);
        for (int p = 0; p < d.max_ctx; ++p)
            for (int i = 0; i < kD / 2; ++i) {
                const double th = (double)p * inv[i];
                tab[(size_t)p * (kD / 2) + i] = make_float2((float)std::cos(th), (float)std::sin(th));
            }
        if (dev_alloc(ctx, &ctx->rope, sizeof(float2) * tab.size())) return fail();
        if (cudaMemcpy(ctx->rope, tab.data(), sizeof(float2) * tab.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaDeviceSynchronize() != cudaSuccess) {
            set_err(ctx, FA_ERR_CUDA, "rope table upload");
            return fail();
        }
    }

    // step buffers
    const int R = d.max_rows;
    const int qkv_n = (kHq + 2 * kHkv) * kD;
    const size_t part_cols = std::max({(size_t)qkv_n * max_split_for(d.hidden), (size_t)d.hidden * max_split_for(kHq * kD),
                                       (size_t)2 * d.ffn * max_split_for(d.hidden), (size_t)d.hidden * max_split_for(d.ffn)});
    ctx->part_elems = part_cols * R;
    ctx->att_max_splits = 64;
    ctx->max_updates = R + 64;
    if (dev_alloc(ctx, &ctx->x, sizeof(float) * R * d.hidden) ||
        dev_alloc(ctx, &ctx->xn16, sizeof(__half) * 2 * R * std::max(d.hidden, d.ffn)) ||
        dev_alloc(ctx, &ctx->part, sizeof(float) * ctx->part_elems) ||
        dev_alloc(ctx, &ctx->q_rot, sizeof(float) * R * kHq * kD) ||
        dev_alloc(ctx, &ctx->attn16, sizeof(__half) * 2 * R * kHq * kD) ||
        dev_alloc(ctx, &ctx->h16, sizeof(__half) * 2 * R * d.ffn) ||
        dev_alloc(ctx, &ctx->att_po, sizeof(float) * (size_t)R * kHq * ctx->att_max_splits * kD) ||
        dev_alloc(ctx, &ctx->att_pml, sizeof(float) * (size_t)R * kHq * ctx->att_max_splits * 2) ||
        dev_alloc(ctx, &ctx->att_cnt, sizeof(int) * (size_t)R * kHkv) ||
        dev_alloc(ctx, &ctx->amax_v, sizeof(float) * (size_t)R * (d.vocab / 64)) ||
        dev_alloc(ctx, &ctx->amax_i, sizeof(int) * (size_t)R * (d.vocab / 64)) ||
        dev_alloc(ctx, &ctx->row_tok, sizeof(int) * R) || dev_alloc(ctx, &ctx->row_slot, sizeof(int) * R) ||
        dev_alloc(ctx, &ctx->row_pos, sizeof(int) * R) || dev_alloc(ctx, &ctx->next_dev, sizeof(int) * R) ||
        dev_alloc(ctx, &ctx->upd_idx, sizeof(int) * ctx->max_updates * 64) ||
        dev_alloc(ctx, &ctx->upd_page, sizeof(int) * ctx->max_updates * 64) ||
        dev_alloc(ctx, &ctx->err_dev, sizeof(int)) || dev_alloc(ctx, &ctx->pf_tiles, sizeof(int2) * R) ||
        dev_alloc(ctx, &ctx->dec_rows, sizeof(int) * R) || dev_alloc(ctx, &ctx->out_rows, sizeof(int) * R))
        return fail();
    ctx->pool_map_ok = fa::make_pool_map(&ctx->pool_map, ctx->pool,
                                         (long long)d.n_layers * n_pages * kHkv * 2 * fa::kPageTokens);
    ctx->max_updates *= 64;
    ctx->xn_lo = ctx->xn16 + (size_t)R * std::max(d.hidden, d.ffn);
    ctx->attn_lo = ctx->attn16 + (size_t)R * kHq * kD;
    ctx->h_lo = ctx->h16 + (size_t)R * d.ffn;
    if (cudaMemset(ctx->err_dev, 0, sizeof(int)) != cudaSuccess ||
        cudaMemset(ctx->att_cnt, 0, sizeof(int) * (size_t)R * kHkv) != cudaSuccess) {
        set_err(ctx, FA_ERR_CUDA, "memset err");
        return fail();
    }
    // tok | slot | pos | tiles (2R) | decode rows | output rows | updates
    const size_t h_ints = 7 * (size_t)R + 2 * (size_t)ctx->max_updates;
    if (cudaMallocHost(&ctx->h_rows, sizeof(int) * h_ints) != cudaSuccess ||
        cudaMallocHost(&ctx->h_next, sizeof(int) * (size_t)R * 4096) != cudaSuccess ||
        cudaMallocHost(&ctx->h_err, sizeof(int)) != cudaSuccess) {
        set_err(ctx, FA_ERR_OOM, "cudaMallocHost failed");
        return fail();
    }
    if (cudaEventCreate(&ctx->ev_t0) != cudaSuccess || cudaEventCreate(&ctx->ev_t1) != cudaSuccess) {
        set_err(ctx, FA_ERR_CUDA, "event create");
        return fail();
    }
    return ctx;
}

static void clear_graphs(fa_ctx* ctx) {
    for (auto& kv : ctx->graphs) cudaGraphExecDestroy(kv.second.exec);
    ctx->graphs.clear();
}

extern "C" void fa_destroy(fa_ctx* ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    clear_graphs(ctx);
    for (void* p : ctx->dev_allocs) cudaFree(p);
    if (ctx->logits_dev) cudaFree(ctx->logits_dev);
    if (ctx->scratch_ints) cudaFree(ctx->scratch_ints);
    if (ctx->h_rows) cudaFreeHost(ctx->h_rows);
    if (ctx->h_next) cudaFreeHost(ctx->h_next);
    if (ctx->h_err) cudaFreeHost(ctx->h_err);
    for (auto e : ctx->prof_ev) cudaEventDestroy(e);
    if (ctx->ev_t0) cudaEventDestroy(ctx->ev_t0);
    if (ctx->ev_t1) cudaEventDestroy(ctx->ev_t1);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
}

extern "C" int fa_set_stream(fa_ctx* ctx, void* stream) {
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    cudaSetDevice(ctx->device);
    FA_CK(cudaStreamSynchronize(ctx->stream));
    ctx->stream = stream ? (cudaStream_t)stream : ctx->own_stream;
    return FA_OK;
}

extern "C" int fa_set_gemm_variant(fa_ctx* ctx, int variant) {
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    if (variant < 0 || variant > 4) return set_err(ctx, FA_ERR_INVALID_ARG, "variant must be 0 to 4");
    ctx->gemm_variant = variant;
    clear_graphs(ctx);
    return FA_OK;
}

extern "C" int fa_set_fused_epilogues(fa_ctx* ctx, int enable) {
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    if (enable < 0 || enable > 15) return set_err(ctx, FA_ERR_INVALID_ARG, "fused epilogue mask must be 0 to 15");
    ctx->fuse_epilogues = enable;
    clear_graphs(ctx);
    return FA_OK;
}

extern "C" int fa_set_row_step(fa_ctx* ctx, int enable) {
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    ctx->row_step_on = enable != 0;
    clear_graphs(ctx);
    return FA_OK;
}

extern "C" int fa_set_row_step_fault(fa_ctx* ctx, int absent_cta, int wait_us) {
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    ctx->row_absent_cta = absent_cta < 0 ? -1 : absent_cta;
    ctx->row_wait_ns = wait_us > 0 ? (unsigned long long)wait_us * 1000ull : fa::kWaitLimitNs;
    clear_graphs(ctx);
    return FA_OK;
}

extern "C" int fa_set_graphs(fa_ctx* ctx, int enable) {
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    ctx->use_graphs = enable != 0;
    return FA_OK;
}

extern "C" int fa_set_pdl(fa_ctx* ctx, int enable) {
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    ctx->use_pdl = enable != 0;
    clear_graphs(ctx);
    return FA_OK;
}

extern "C" int fa_ctx_desc(const fa_ctx* ctx, fa_model_desc* desc) {
    if (!ctx || !desc) return set_err(ctx, FA_ERR_INVALID_ARG, "fa_ctx_desc: bad argument");
    *desc = ctx->d;
    return FA_OK;
}

extern "C" int fa_pool_info(const fa_ctx* ctx, int* n_pages, int* n_free, size_t* page_bytes) {
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    if (n_pages) *n_pages = ctx->n_pages;
    if (n_free) *n_free = ctx->palloc.n_free();
    if (page_bytes) *page_bytes = kPageElems * 2 * (size_t)ctx->d.n_layers;
    return FA_OK;
}

// ----------------------------------------------------------------- weights --
namespace {

struct TensorSpec {
    const fa_tensor_view* v = nullptr;
};

float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

float f16_to_f32_host(uint16_t h) {
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}

}  // namespace

static int find_tensor(fa_ctx* ctx, const std::unordered_map<std::string, const fa_tensor_view*>& m,
                       const std::string& name, int type_q8, int64_t ne0, int64_t ne1,
                       const fa_tensor_view** out) {
    auto it = m.find(name);
    if (it == m.end()) return set_err(ctx, FA_ERR_WEIGHTS, "missing tensor " + name);
    const fa_tensor_view* v = it->second;
    if (v->ne[0] != ne0 || (ne1 > 0 && v->ne[1] != ne1))
        return set_err(ctx, FA_ERR_WEIGHTS,
                       name + ": shape [" + std::to_string(v->ne[0]) + ", " + std::to_string(v->ne[1]) +
                           "], expected [" + std::to_string(ne0) + ", " + std::to_string(ne1) + "]");
    if (type_q8 && v->type != FA_TYPE_Q8_0)
        return set_err(ctx, FA_ERR_WEIGHTS, name + ": expected Q8_0 (type 8), got type " + std::to_string(v->type));
    if (!type_q8 && v->type != FA_TYPE_F32 && v->type != FA_TYPE_F16 && v->type != FA_TYPE_BF16)
        return set_err(ctx, FA_ERR_WEIGHTS, name + ": expected F32/F16/BF16");
    const size_t elems = (size_t)v->ne[0] * (size_t)(v->ne[1] > 0 ? v->ne[1] : 1);
    const size_t want = type_q8 ? elems / 32 * 34 : elems * (v->type == FA_TYPE_F32 ? 4 : 2);
    if (v->nbytes != want || !v->data)
        return set_err(ctx, FA_ERR_WEIGHTS, name + ": " + std::to_string(v->nbytes) + " bytes, expected " +
                                                std::to_string(want));
    *out = v;
    return FA_OK;
}

static int upload_vec_f32(fa_ctx* ctx, const fa_tensor_view* v, float** dst) {
    const size_t n = (size_t)v->ne[0];
    std::vector<float> h(n);
    for (size_t i = 0; i < n; ++i) {
        if (v->type == FA_TYPE_F32) h[i] = reinterpret_cast<const float*>(v->data)[i];
        else if (v->type == FA_TYPE_BF16) h[i] = bf16_to_f32(reinterpret_cast<const uint16_t*>(v->data)[i]);
        else h[i] = f16_to_f32_host(reinterpret_cast<const uint16_t*>(v->data)[i]);
    }
    if (int rc = dev_alloc(ctx, dst, sizeof(float) * n)) return rc;
    FA_CK(cudaMemcpy(*dst, h.data(), sizeof(float) * n, cudaMemcpyHostToDevice));
    return FA_OK;
}

// Split a GGUF Q8_0 tensor with N rows of K into the planes of a stacked matrix of
// n_total rows, at row offset r0.
static int upload_q8(fa_ctx* ctx, const fa_tensor_view* v, uint8_t* staging, int N, int K, int r0, int n_total,
                     unsigned char* planes, int interleave = 0) {
    FA_CK(cudaMemcpyAsync(staging, v->data, v->nbytes, cudaMemcpyHostToDevice, ctx->stream));
    fa::launch_repack_q8_planes(staging, N, K, r0, n_total, planes, ctx->stream, interleave);
    FA_CK(cudaGetLastError());
    FA_CK(cudaStreamSynchronize(ctx->stream));
    return FA_OK;
}

// Buffers and the per-layer weight table of the one-row step kernel, when it takes the
// model's shapes (else one-row steps run launch by launch).
static int setup_row_step(fa_ctx* ctx) {
    const fa_model_desc& d = ctx->d;
    if (!fa::row_step_shapes(d.hidden, d.ffn, ctx->n_sm, ctx->row_gm)) return FA_OK;
    int attr = 0;
    if (cudaDeviceGetAttribute(&attr, cudaDevAttrCooperativeLaunch, ctx->device) != cudaSuccess || !attr) {
        cudaGetLastError();
        return FA_OK;
    }
    std::vector<fa::RowLayer> tab(d.n_layers);
    for (int l = 0; l < d.n_layers; ++l) {
        const LayerW& w = ctx->L[l];
        tab[l].w[0] = w.qkv_q; tab[l].w[1] = w.o_q; tab[l].w[2] = w.gu_q; tab[l].w[3] = w.dn_q;
        tab[l].in_norm = w.in_norm; tab[l].post_norm = w.post_norm; tab[l].q_norm = w.q_norm; tab[l].k_norm = w.k_norm;
    }
    int r;
    if ((r = dev_alloc(ctx, &ctx->row_layers, sizeof(fa::RowLayer) * tab.size())) ||
        (r = dev_alloc(ctx, &ctx->row_words, sizeof(unsigned long long) * fa::row_step_words(d.hidden, d.ffn))) ||
        (r = dev_alloc(ctx, &ctx->row_ctl, sizeof(fa::RowCtl))))
        return r;
    FA_CK(cudaMemcpy(ctx->row_layers, tab.data(), sizeof(fa::RowLayer) * tab.size(), cudaMemcpyHostToDevice));
    ctx->row_words_n = fa::row_step_words(d.hidden, d.ffn);
    FA_CK(cudaMemset(ctx->row_ctl, 0, sizeof(fa::RowCtl)));
    FA_CK(cudaMemset(ctx->row_words, 0, sizeof(unsigned long long) * ctx->row_words_n));
    ctx->row_ready = true;
    return FA_OK;
}

extern "C" int fa_load_weights(fa_ctx* ctx, const fa_tensor_view* tensors, int n) {
    if (!ctx || (!tensors && n > 0)) return set_err(ctx, FA_ERR_INVALID_ARG, "bad arguments");
    if (ctx->loaded) return set_err(ctx, FA_ERR_INVALID_ARG, "weights already loaded");
    cudaSetDevice(ctx->device);
    const fa_model_desc& d = ctx->d;
    std::unordered_map<std::string, const fa_tensor_view*> m;
    for (int i = 0; i < n; ++i)
        if (tensors[i].name) m[tensors[i].name] = &tensors[i];
    const int H = d.hidden, F = d.ffn, V = d.vocab, QD = kHq * kD, KD = kHkv * kD;

    // validate everything first
    const fa_tensor_view *emb, *fnorm, *lm;
    int rc;
    if ((rc = find_tensor(ctx, m, "llm.model.embed_tokens.weight", 0, H, V, &emb))) return rc;
    if ((rc = find_tensor(ctx, m, "llm.model.norm.weight", 0, H, 0, &fnorm))) return rc;
    if ((rc = find_tensor(ctx, m, "llm.lm_head.weight", 1, H, V, &lm))) return rc;
    struct LV { const fa_tensor_view *q, *k, *v, *o, *g, *u, *dn, *qn, *kn, *in, *post; };
    std::vector<LV> lv(d.n_layers);
    for (int l = 0; l < d.n_layers; ++l) {
        const std::string p = "llm.model.layers." + std::to_string(l) + ".";
        LV& t = lv[l];
        if ((rc = find_tensor(ctx, m, p + "self_attn.q_proj.weight", 1, H, QD, &t.q))) return rc;
        if ((rc = find_tensor(ctx, m, p + "self_attn.k_proj.weight", 1, H, KD, &t.k))) return rc;
        if ((rc = find_tensor(ctx, m, p + "self_attn.v_proj.weight", 1, H, KD, &t.v))) return rc;
        if ((rc = find_tensor(ctx, m, p + "self_attn.o_proj.weight", 1, QD, H, &t.o))) return rc;
        if ((rc = find_tensor(ctx, m, p + "mlp.gate_proj.weight", 1, H, F, &t.g))) return rc;
        if ((rc = find_tensor(ctx, m, p + "mlp.up_proj.weight", 1, H, F, &t.u))) return rc;
        if ((rc = find_tensor(ctx, m, p + "mlp.down_proj.weight", 1, F, H, &t.dn))) return rc;
        if ((rc = find_tensor(ctx, m, p + "self_attn.q_norm.weight", 0, kD, 0, &t.qn))) return rc;
        if ((rc = find_tensor(ctx, m, p + "self_attn.k_norm.weight", 0, kD, 0, &t.kn))) return rc;
        if ((rc = find_tensor(ctx, m, p + "input_layernorm.weight", 0, H, 0, &t.in))) return rc;
        if ((rc = find_tensor(ctx, m, p + "post_attention_layernorm.weight", 0, H, 0, &t.post))) return rc;
    }

    size_t max_q8 = lm->nbytes;
    for (auto& t : lv)
        for (auto* v : {t.q, t.k, t.v, t.o, t.g, t.u, t.dn}) max_q8 = std::max(max_q8, v->nbytes);
    uint8_t* staging = nullptr;
    {
        cudaError_t e = cudaMalloc(&staging, max_q8);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return set_err(ctx, FA_ERR_OOM, "weight staging buffer");
        }
    }
    auto run = [&]() -> int {
        ctx->L.resize(d.n_layers);
        const int QKV = QD + 2 * KD;
        for (int l = 0; l < d.n_layers; ++l) {
            LayerW& w = ctx->L[l];
            LV& t = lv[l];
            int r;
            if ((r = dev_alloc(ctx, &w.qkv_q, fa::q8p_bytes(QKV, H))) || (r = dev_alloc(ctx, &w.o_q, fa::q8p_bytes(H, QD))) ||
                (r = dev_alloc(ctx, &w.gu_q, fa::q8p_bytes(2 * F, H))) || (r = dev_alloc(ctx, &w.dn_q, fa::q8p_bytes(H, F))))
                return r;
            if ((r = upload_q8(ctx, t.q, staging, QD, H, 0, QKV, w.qkv_q)) ||
                (r = upload_q8(ctx, t.k, staging, KD, H, QD, QKV, w.qkv_q)) ||
                (r = upload_q8(ctx, t.v, staging, KD, H, QD + KD, QKV, w.qkv_q)) ||
                (r = upload_q8(ctx, t.o, staging, H, QD, 0, H, w.o_q)) ||
                // gate and up rows in blocks of 64: rows [128 b, 128 b + 64) are gate rows
                // [64 b, 64 b + 64), the next 64 the up rows of the same outputs
                (r = upload_q8(ctx, t.g, staging, F, H, 0, 2 * F, w.gu_q, 64)) ||
                (r = upload_q8(ctx, t.u, staging, F, H, 64, 2 * F, w.gu_q, 64)) ||
                (r = upload_q8(ctx, t.dn, staging, H, F, 0, H, w.dn_q)))
                return r;
            if ((r = upload_vec_f32(ctx, t.qn, &w.q_norm)) || (r = upload_vec_f32(ctx, t.kn, &w.k_norm)) ||
                (r = upload_vec_f32(ctx, t.in, &w.in_norm)) || (r = upload_vec_f32(ctx, t.post, &w.post_norm)))
                return r;
        }
        int r;
        if ((r = dev_alloc(ctx, &ctx->lm_q, fa::q8p_bytes(V, H)))) return r;
        if ((r = upload_q8(ctx, lm, staging, V, H, 0, V, ctx->lm_q))) return r;
        if ((r = upload_vec_f32(ctx, fnorm, &ctx->final_norm))) return r;
        if ((r = dev_alloc(ctx, (uint8_t**)&ctx->embed, emb->nbytes))) return r;
        FA_CK(cudaMemcpy(ctx->embed, emb->data, emb->nbytes, cudaMemcpyHostToDevice));
        ctx->embed_type = emb->type;
        return setup_row_step(ctx);
    };
    rc = run();
    // host -> device copies from pageable memory can return before their DMA lands, and
    // the library's stream does not order after them: wait for every copy here
    if (cudaDeviceSynchronize() != cudaSuccess && rc == FA_OK) rc = set_err(ctx, FA_ERR_CUDA, "weight upload");
    cudaFree(staging);
    if (rc == FA_OK) ctx->loaded = true;
    return rc;
}

// --------------------------------------------------------------- sequences --
static int check_seq(const fa_ctx* ctx, int seq_id) {
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    if (seq_id < 0 || seq_id >= (int)ctx->seqs.size() || !ctx->seqs[seq_id].open)
        return set_err(ctx, FA_ERR_SEQ, "sequence " + std::to_string(seq_id) + " is not open");
    return FA_OK;
}

extern "C" int fa_seq_open(fa_ctx* ctx, int max_tokens, int* seq_id) {
    if (!ctx || !seq_id) return set_err(ctx, FA_ERR_INVALID_ARG, "bad arguments");
    if (max_tokens <= 0 || max_tokens > ctx->d.max_ctx)
        return set_err(ctx, FA_ERR_CAPACITY, "max_tokens must be in [1, max_ctx]");
    for (int i = 0; i < (int)ctx->seqs.size(); ++i) {
        if (!ctx->seqs[i].open) {
            Seq& s = ctx->seqs[i];
            s.open = true;
            s.len = 0;
            s.max_tokens = max_tokens;
            s.pages.clear();
            *seq_id = i;
            return FA_OK;
        }
    }
    return set_err(ctx, FA_ERR_SEQ, "no free sequence slot (max_seqs reached)");
}

extern "C" int fa_seq_close(fa_ctx* ctx, int seq_id) {
    if (int rc = check_seq(ctx, seq_id)) return rc;
    Seq& s = ctx->seqs[seq_id];
    for (int p : s.pages) ctx->palloc.release(p);
    s.pages.clear();
    s.open = false;
    s.len = 0;
    return FA_OK;
}

extern "C" int fa_seq_length(const fa_ctx* ctx, int seq_id, int* n_tokens) {
    if (int rc = check_seq(ctx, seq_id)) return rc;
    if (n_tokens) *n_tokens = ctx->seqs[seq_id].len;
    return FA_OK;
}

extern "C" int fa_seq_truncate(fa_ctx* ctx, int seq_id, int n_tokens) {
    if (int rc = check_seq(ctx, seq_id)) return rc;
    Seq& s = ctx->seqs[seq_id];
    if (n_tokens < 0 || n_tokens > s.len)
        return set_err(ctx, FA_ERR_INVALID_ARG, "truncate length must be in [0, current length]");
    const size_t keep = (size_t)(n_tokens + fa::kPageTokens - 1) / fa::kPageTokens;
    while (s.pages.size() > keep) {
        ctx->palloc.release(s.pages.back());
        s.pages.pop_back();
    }
    s.len = n_tokens;
    return FA_OK;
}

extern "C" int fa_seq_block_table(const fa_ctx* ctx, int seq_id, int* pages, int max_pages, int* n_pages) {
    if (int rc = check_seq(ctx, seq_id)) return rc;
    const Seq& s = ctx->seqs[seq_id];
    if (n_pages) *n_pages = (int)s.pages.size();
    if (pages)
        for (int i = 0; i < (int)s.pages.size() && i < max_pages; ++i) pages[i] = s.pages[i];
    return FA_OK;
}

// Reserve pages so that every sequence in `need` can hold its new length. Records
// block-table updates; on exhaustion returns every page taken here.
static int reserve_pages(fa_ctx* ctx, const std::vector<std::pair<int, int>>& need, std::vector<int>& upd_idx,
                         std::vector<int>& upd_page) {
    std::vector<std::pair<int, int>> taken;   // (seq, page)
    for (auto& sn : need) {
        Seq& s = ctx->seqs[sn.first];
        const size_t want = (size_t)(sn.second + fa::kPageTokens - 1) / fa::kPageTokens;
        while (s.pages.size() < want) {
            const int p = ctx->palloc.alloc();
            if (p < 0) {
                for (auto it = taken.rbegin(); it != taken.rend(); ++it) {
                    ctx->seqs[it->first].pages.pop_back();
                    ctx->palloc.release(it->second);
                }
                upd_idx.clear();
                upd_page.clear();
                return set_err(ctx, FA_ERR_POOL_EXHAUSTED, "KV page pool exhausted");
            }
            upd_idx.push_back(sn.first * ctx->bt_stride + (int)s.pages.size());
            upd_page.push_back(p);
            s.pages.push_back(p);
            taken.push_back({sn.first, p});
        }
    }
    return FA_OK;
}

static int upload_updates(fa_ctx* ctx, const std::vector<int>& ui, const std::vector<int>& up) {
    size_t off = 0;
    while (off < ui.size()) {
        const int n = (int)std::min<size_t>(ui.size() - off, (size_t)ctx->max_updates);
        int* hi = ctx->h_rows + 7 * ctx->d.max_rows;
        std::memcpy(hi, ui.data() + off, sizeof(int) * n);
        std::memcpy(hi + ctx->max_updates, up.data() + off, sizeof(int) * n);
        FA_CK(cudaMemcpyAsync(ctx->upd_idx, hi, sizeof(int) * n, cudaMemcpyHostToDevice, ctx->stream));
        FA_CK(cudaMemcpyAsync(ctx->upd_page, hi + ctx->max_updates, sizeof(int) * n, cudaMemcpyHostToDevice,
                              ctx->stream));
        fa::launch_apply_bt_updates(ctx->bt_dev, ctx->upd_idx, ctx->upd_page, n, ctx->stream);
        FA_CK(cudaGetLastError());
        off += n;
        if (off < ui.size()) FA_CK(cudaStreamSynchronize(ctx->stream));   // staging reuse
    }
    return FA_OK;
}

// ----------------------------------------------------------------- forward --
namespace {

struct StepPlan {
    int M = 0;
    int s_qkv = 1, s_o = 1, s_gu = 1, s_dn = 1;
    int pps = 32;        // attention pages per split (decode kernel)
    int n_splits = 1;
    int att_warps = 4;   // warps per attention CTA
    int n_dec = 0;       // rows for the decode kernel (all M rows when there are no tiles)
    int n_tiles = 0;     // prefill tiles for the tensor-core kernel
    int n_out = -1;      // rows through lm_head: -1 all (with token feedback), else the listed rows
    bool embeds = false; // input rows already in x
    bool logits = false;
    bool prof = false;
    bool fuse_swiglu = false;  // gate/up GEMM on the small-M kernel writes SwiGLU's output itself
    bool fuse_gu_tc = false;   // gate/up GEMM on the tcgen05 kernel finishes SwiGLU in its clusters
    bool fuse_qkv = false;     // QKV GEMM on the tcgen05 kernel finishes kernel (1) in its clusters
    bool row_step = false;     // one row: the persistent step kernel, then lm_head and argmax
    bool att_merge = false;    // the attention kernel merges its splits itself (no combine launch)
    bool att_append = false;   // ... and runs kernel (1) for its KV heads (no kernel (1) launch)
    std::array<int, 12> key() const {
        return {M, s_qkv, s_o, s_gu, s_dn, pps * 16 + att_warps, n_splits, n_dec, n_tiles, n_out,
                (int)att_append * 128 + (int)att_merge * 64 + (int)row_step * 32 + (int)fuse_qkv * 16 + (int)fuse_gu_tc * 8 +
                    (int)fuse_swiglu * 4 + (int)embeds * 2 + (int)logits,
                (int)prof};
    }
};

// Rows of one sequence at consecutive positions that form a run at least this long
// go to the tensor-core prefill kernel in tiles of up to 64 rows.
constexpr int kPrefillMinRun = 16;

}  // namespace

// Attention work split for rows of row_pages[i] pages each: the CTA form (warps per CTA)
// and pages per CTA (a multiple of 4) that minimise the estimated time
//   waves * (4 * ceil(pps / warps) + 2) + (8 if any row is split)
// where waves = ceil(CTAs / (CTAs per SM * n_sm)) (3 CTAs of 4 warps or one of 8 per SM), a
// CTA costs its rounds of pages (one per warp each) plus about 2 pages' worth of set-up, and
// merging split partials costs a launch of its own, about 8 pages' worth (a unit is
// ~0.5 us: 128 rows x 2048 tokens run 7 waves of 46 in 173 us; the merge launch takes
// 4-6 us); at most max_splits splits per row. warps_in = 0 lets the model choose (8 for one
// row, either form up to kAttnPlanWideRows rows, 4 above); 4 or 8 fixes it.
static void attention_split(const std::vector<int>& row_pages, int n_sm, int max_splits, int* pps_out,
                            int* n_splits_out, int* warps_out = nullptr, int warps_in = 0) {
    int max_pages = 1;
    for (int pg : row_pages) max_pages = std::max(max_pages, pg);
    const int rows = (int)row_pages.size();
    int forms[2] = {4, 8}, n_forms = 2;
    if (warps_in) { forms[0] = warps_in; n_forms = 1; }
    else if (rows == 1) { forms[0] = 8; n_forms = 1; }
    else if (rows > fa::kAttnPlanWideRows) { forms[0] = 4; n_forms = 1; }
    long long best_cost = -1;
    int best = 0, best_w = forms[0];
    for (int fi = 0; fi < n_forms; ++fi) {
        const int warps = forms[fi];
        const long long slots = (long long)(warps == 4 ? fa::kAttnCtasPerSm : 1) * n_sm;
        for (int pps = 4; pps <= 256; pps += 4) {
            const int n_splits = (max_pages + pps - 1) / pps;
            if (n_splits > max_splits) continue;
            long long ctas = 0;
            for (int pg : row_pages) ctas += (long long)kHkv * ((std::max(pg, 1) + pps - 1) / pps);
            const long long waves = (ctas + slots - 1) / slots;
            const long long cost = waves * (4 * ((pps + warps - 1) / warps) + 2) + (n_splits > 1 ? 8 : 0);
            if (best_cost < 0 || cost < best_cost) {
                best_cost = cost;
                best = pps;
                best_w = warps;
            }
            if (n_splits == 1) break;   // larger pps change nothing
        }
    }
    if (!best) best = (max_pages + max_splits - 1) / max_splits;   // unreachable with pps up to 256
    *pps_out = best;
    *n_splits_out = (max_pages + best - 1) / best;
    if (warps_out) *warps_out = best_w;
}

// The decode attention of a step with rows of row_pages[i] pages: the split (attention_split,
// CTA form chosen by the cost model) and what the attention kernel finishes itself under the
// fused-op mask. Both fusions are taken only when the attention CTAs fit in one wave:
//   merge  (bit 2): the split that counts its (row, KV head) last merges the splits; over
//          several waves each CTA's count and the last split's merge hold back the next wave
//          (measured: 4 rows x 2048 tokens 1.49 -> 1.45 ms per step, 16 x 1024 1.64 -> 1.61;
//          64 and 128 rows x 2048 2-4 % slower);
//   append (bit 3): kernel (1) for each CTA's KV head, whose per-CTA work then overlaps the
//          first page copies once, where over several waves every wave repeats it (measured:
//          2 rows x 256 tokens 1.094 -> 1.045 ms per step, 16 x 1024 1.615 -> 1.587; 128 x 2048
//          no gain, the attention launch 5.6 us longer). The step adds its own conditions.
struct AttnChoice {
    int pps = 0, n_splits = 0, warps = 4;
    bool merge = false, append = false;
};
static AttnChoice plan_attention(const std::vector<int>& row_pages, int n_sm, int max_splits, int mask) {
    AttnChoice c;
    attention_split(row_pages, n_sm, max_splits, &c.pps, &c.n_splits, &c.warps);
    long long ctas = 0;
    for (int pg : row_pages) ctas += (long long)kHkv * ((std::max(pg, 1) + c.pps - 1) / c.pps);
    const long long slots = (long long)(c.warps == 4 ? fa::kAttnCtasPerSm : 1) * n_sm;
    const bool one_wave = ctas <= slots;
    c.merge = c.n_splits > 1 && (mask & 4) && one_wave;
    c.append = (mask & 8) && one_wave;
    return c;
}

// Whether a GEMM of M rows goes to the CUDA-core kernel under a GEMM variant.
static bool gemv_rows(int variant, int M) {
    return (variant == 0 && M <= fa::kGemvAutoRows) || (variant == 3 && M <= fa::kGemvMaxRows);
}

// Whether a GEMM of M rows goes to the swapped tcgen05 kernel. With Q8_0 planes (the
// decoder's weights) it takes every M above the CUDA-core kernel's rows, in 128-row
// activation tiles; with f16 weights it takes one tile of up to 128 rows.
static bool skinny_rows(int variant, int M, int epilogue = fa::kEpiStoreF32, bool q8 = true) {
    if (q8) return (variant == 0 && M > fa::kGemvAutoRows) || variant == 4;
    const int auto_rows = epilogue == fa::kEpiArgmax ? fa::kSkinnyArgmaxAutoRows : fa::kSkinnyAutoRows;
    return (variant == 0 && M > fa::kGemvAutoRows && M <= auto_rows) || (variant == 4 && M <= fa::kSkinnyMaxRows);
}

// row_len: context length of each row given to the decode kernel (all rows, or the
// rows outside prefill tiles); n_tiles: prefill tiles of the step; distinct: every row
// belongs to a sequence of its own.
static StepPlan make_plan(fa_ctx* ctx, int M, const std::vector<int>& row_len, bool embeds, bool logits,
                          int n_tiles = 0, bool distinct = false) {
    const fa_model_desc& d = ctx->d;
    StepPlan p;
    p.M = M;
    auto pick = [&](int n, int k) {
        if (gemv_rows(ctx->gemm_variant, M) && fa::gemv_shape_supported(M, n, k, fa::kEpiStoreF32)) return 1;
        if (skinny_rows(ctx->gemm_variant, M) && n % 128 == 0) return fa::gemm_tc_skinny_pick_split(M, n, k, ctx->n_sm);
        return ctx->gemm_variant != 1 && n % 128 == 0 ? fa::gemm_tc_pick_split(M, n, k, ctx->n_sm)
                                                       : fa::gemm_pick_split(M, n, k, ctx->n_sm);
    };
    p.s_qkv = pick((kHq + 2 * kHkv) * kD, d.hidden);
    p.s_o = pick(d.hidden, kHq * kD);
    p.s_gu = pick(2 * d.ffn, d.hidden);
    p.s_dn = pick(d.hidden, d.ffn);
    p.fuse_swiglu = gemv_rows(ctx->gemm_variant, M) && fa::gemv_shape_supported(M, 2 * d.ffn, d.hidden, fa::kEpiSwiglu);
    // one-tile steps on the tcgen05 kernel: QKV finishes kernel (1) and gate/up finishes
    // SwiGLU inside clusters of their split CTAs (no partials, no separate launches)
    const bool tc = !gemv_rows(ctx->gemm_variant, M) && skinny_rows(ctx->gemm_variant, M);
    p.fuse_qkv = tc && (ctx->fuse_epilogues & 1) &&
                 fa::skinny_fusable(M, (kHq + 2 * kHkv) * kD, d.hidden, p.s_qkv, ctx->n_sm);
    p.fuse_gu_tc = tc && (ctx->fuse_epilogues & 2) && fa::skinny_fusable(M, 2 * d.ffn, d.hidden, p.s_gu, ctx->n_sm);
    p.n_dec = (int)row_len.size();
    p.n_tiles = n_tiles;
    if (p.n_dec > 0) {
        std::vector<int> row_pages(row_len.size());
        for (size_t i = 0; i < row_len.size(); ++i)
            row_pages[i] = (row_len[i] + fa::kPageTokens - 1) / fa::kPageTokens;
        const AttnChoice c = plan_attention(row_pages, ctx->n_sm, ctx->att_max_splits, ctx->fuse_epilogues);
        p.pps = c.pps;
        p.n_splits = c.n_splits;
        p.att_warps = c.warps;
        p.att_merge = c.merge;
        // kernel (1) inside the attention kernel: steps of decode rows of distinct sequences
        // only (prefill tiles need q of every row; a row attends over the K / V that earlier
        // rows of its sequence append in the same step, which another CTA would be writing),
        // when the QKV GEMM does not finish kernel (1) itself
        p.att_append = c.append && n_tiles == 0 && p.n_dec == M && distinct && !p.fuse_qkv;
    }
    p.embeds = embeds;
    p.logits = logits;
    p.prof = ctx->prof;
    // one decode row, CUDA-core GEMM arithmetic, every attention item on its own SM
    p.row_step = ctx->row_ready && ctx->row_step_on && M == 1 && n_tiles == 0 && p.n_dec == 1 &&
                 gemv_rows(ctx->gemm_variant, 1) && p.att_warps == 8 && p.n_splits * kHkv <= ctx->n_sm;
    return p;
}

static int ensure_logits(fa_ctx* ctx) {
    if (ctx->logits_dev) return FA_OK;
    void* v = nullptr;
    if (cudaMalloc(&v, sizeof(float) * (size_t)ctx->d.max_rows * ctx->d.vocab) != cudaSuccess) {
        cudaGetLastError();
        return set_err(ctx, FA_ERR_OOM, "logits buffer");
    }
    ctx->logits_dev = (float*)v;
    return FA_OK;
}

static int ensure_prof_events(fa_ctx* ctx) {
    const size_t want = 2 * (size_t)ctx->d.n_layers;
    while (ctx->prof_ev.size() < want) {
        cudaEvent_t e;
        FA_CK(cudaEventCreate(&e));
        ctx->prof_ev.push_back(e);
    }
    return FA_OK;
}

static void record_prof(fa_ctx* ctx, int idx, bool capturing) {
    if (capturing) cudaEventRecordWithFlags(ctx->prof_ev[idx], ctx->stream, cudaEventRecordExternal);
    else cudaEventRecord(ctx->prof_ev[idx], ctx->stream);
}

// One Q8_0 GEMM launch on the selected implementation: the CUDA-core kernel for a few
// rows (variants 0 and 3, make_plan gives those shapes n_split 1), else tcgen05; the
// mma.sync cross-check kernel for variant 1 or a shape outside both.
static void run_gemm(fa_ctx* ctx, const fa::GemmArgs& g) {
    const int v = ctx->gemm_variant;
    if (v != 1) {
        if (gemv_rows(v, g.M) && fa::launch_q8_gemv(g, ctx->stream)) return;
        if (skinny_rows(v, g.M, g.epilogue, g.W8.q != nullptr) &&
            fa::launch_q8_gemm_tc_skinny(g, ctx->err_dev, ctx->stream))
            return;
        if (fa::gemm_tc_supported(g) && fa::launch_q8_gemm_tc(g, ctx->err_dev, ctx->stream)) return;
    }
    fa::launch_q8_gemm(g, ctx->stream);
}

static int enqueue_row_step(fa_ctx* ctx, const StepPlan& p, bool capturing);
static int enqueue_lm_head(fa_ctx* ctx, const StepPlan& p, int Mo);

// Enqueue the kernels of one forward step. Returns the number of launches.
static int enqueue_step(fa_ctx* ctx, const StepPlan& p, bool capturing) {
    if (p.row_step) return enqueue_row_step(ctx, p, capturing);
    const fa_model_desc& d = ctx->d;
    cudaStream_t s = ctx->stream;
    const int M = p.M, H = d.hidden, F = d.ffn;
    const int QKV = (kHq + 2 * kHkv) * kD;
    int n = 0;
    if (!p.embeds) {
        fa::launch_embed(ctx->embed, ctx->embed_type, H, ctx->row_tok, nullptr, M, d.vocab, ctx->x, ctx->err_dev, s);
        ++n;
    }
    const float* prev_part = nullptr;
    int prev_n = 0;
    for (int l = 0; l < d.n_layers; ++l) {
        const LayerW& w = ctx->L[l];
        __half* pool_l = ctx->pool + (size_t)l * ctx->layer_stride;
        fa::launch_residual_rmsnorm(ctx->x, prev_part, prev_n, M, H, w.in_norm, d.rms_eps, ctx->xn16, ctx->xn_lo, s);
        fa::GemmArgs g{};
        fa::AppendArgs a{};
        a.qkv_part = ctx->part; a.n_part = p.s_qkv; a.M = M; a.pos = ctx->row_pos; a.slot = ctx->row_slot;
        a.block_table = ctx->bt_dev; a.bt_stride = ctx->bt_stride; a.n_pages = ctx->n_pages;
        a.qn_w = w.q_norm; a.kn_w = w.k_norm; a.Hq = kHq; a.Hkv = kHkv; a.eps = d.rms_eps;
        a.q_scale = 1.0f / std::sqrt((float)kD);
        a.rope = ctx->rope; a.max_pos = d.max_ctx; a.pool_layer = pool_l; a.q_out = ctx->q_rot; a.err = ctx->err_dev;
        g.A = ctx->xn16; g.A_lo = ctx->xn_lo; g.W8 = fa::q8p_view(w.qkv_q, QKV, H); g.M = M; g.N = QKV; g.K = H;
        g.n_split = p.s_qkv;
        if (p.fuse_qkv) {
            g.epilogue = fa::kEpiQkvAppend; g.app = &a;
            if (!fa::launch_q8_gemm_tc_skinny(g, ctx->err_dev, s)) ctx->enqueue_failed = true;
            --n;
        } else {
            g.epilogue = fa::kEpiStoreF32; g.C = ctx->part;
            run_gemm(ctx, g);
            if (p.att_append) --n;   // kernel (1) runs inside the attention kernel
            else fa::launch_qknorm_rope_append(a, s);
        }
        const bool prof_l = p.prof && (l == 0 || l == d.n_layers / 2 || l == d.n_layers - 1);
        if (prof_l) record_prof(ctx, 2 * l, capturing);
        if (p.n_dec > 0) {
            fa::AttnArgs at{};
            at.q = ctx->q_rot; at.pool_layer = pool_l; at.block_table = ctx->bt_dev; at.bt_stride = ctx->bt_stride;
            at.n_pages = ctx->n_pages; at.slot = ctx->row_slot; at.pos = ctx->row_pos; at.M = p.n_dec;
            at.rows = p.n_tiles > 0 ? ctx->dec_rows : nullptr; at.Hq = kHq;
            at.Hkv = kHkv; at.pages_per_split = p.pps; at.n_splits = p.n_splits; at.warps = p.att_warps;
            at.part_o = ctx->att_po;
            at.part_ml = ctx->att_pml; at.out16 = ctx->attn16; at.out16_lo = ctx->attn_lo; at.out32 = nullptr;
            at.err = ctx->err_dev;
            at.merge_cnt = p.att_merge ? ctx->att_cnt : nullptr;
            if (p.att_append) {
                at.fuse_append = 1;
                at.app = a;
            }
            fa::launch_paged_attention(at, s);
            ++n;
            if (p.n_splits > 1 && !p.att_merge) {
                fa::launch_attn_combine(at, s);
                ++n;
            }
        }
        if (p.n_tiles > 0) {
            fa::PrefillAttnArgs pa{};
            pa.q = ctx->q_rot; pa.block_table = ctx->bt_dev; pa.bt_stride = ctx->bt_stride; pa.n_pages = ctx->n_pages;
            pa.slot = ctx->row_slot; pa.pos = ctx->row_pos; pa.M = M; pa.Hq = kHq; pa.Hkv = kHkv;
            pa.tiles = ctx->pf_tiles; pa.n_tiles = p.n_tiles;
            pa.pool_row0 = l * ctx->n_pages * kHkv * 2 * fa::kPageTokens;
            pa.out16 = ctx->attn16; pa.out16_lo = ctx->attn_lo; pa.out32 = nullptr; pa.err = ctx->err_dev;
            fa::launch_prefill_attention(ctx->pool_map, pa, s);
            ++n;
        }
        if (prof_l) record_prof(ctx, 2 * l + 1, capturing);
        g = fa::GemmArgs{};
        g.A = ctx->attn16; g.A_lo = ctx->attn_lo; g.W8 = fa::q8p_view(w.o_q, H, kHq * kD); g.M = M; g.N = H;
        g.K = kHq * kD;
        g.n_split = p.s_o; g.epilogue = fa::kEpiStoreF32; g.C = ctx->part;
        run_gemm(ctx, g);
        fa::launch_residual_rmsnorm(ctx->x, ctx->part, p.s_o, M, H, w.post_norm, d.rms_eps, ctx->xn16, ctx->xn_lo, s);
        g = fa::GemmArgs{};
        g.A = ctx->xn16; g.A_lo = ctx->xn_lo; g.W8 = fa::q8p_view(w.gu_q, 2 * F, H); g.M = M; g.N = 2 * F; g.K = H;
        g.n_split = p.s_gu;
        g.swiglu_interleave64 = 1;     // gate / up rows stacked in blocks of 64 (upload_q8)
        if (p.fuse_swiglu || p.fuse_gu_tc) {
            g.epilogue = fa::kEpiSwiglu; g.H = ctx->h16; g.H_lo = ctx->h_lo;
            const bool ok = p.fuse_swiglu ? fa::launch_q8_gemv(g, s) : fa::launch_q8_gemm_tc_skinny(g, ctx->err_dev, s);
            if (!ok) ctx->enqueue_failed = true;
            --n;
        } else {
            g.epilogue = fa::kEpiStoreF32; g.C = ctx->part;
            run_gemm(ctx, g);
            fa::launch_swiglu(ctx->part, p.s_gu, M, F, ctx->h16, ctx->h_lo, s, true);
        }
        g = fa::GemmArgs{};
        g.A = ctx->h16; g.A_lo = ctx->h_lo; g.W8 = fa::q8p_view(w.dn_q, H, F); g.M = M; g.N = H; g.K = F;
        g.n_split = p.s_dn; g.epilogue = fa::kEpiStoreF32; g.C = ctx->part;
        run_gemm(ctx, g);
        n += 8;
        prev_part = ctx->part;
        prev_n = p.s_dn;
    }
    // final norm and lm_head: all rows (feeding each row's argmax back as its next
    // token), or only the listed rows, compacted, or none
    const bool all = p.n_out < 0;
    const int Mo = all ? M : p.n_out;
    if (Mo == 0) return n;
    fa::launch_residual_rmsnorm(ctx->x, prev_part, prev_n, M, H, ctx->final_norm, d.rms_eps, ctx->xn16, ctx->xn_lo, s,
                                Mo, all ? nullptr : ctx->out_rows);
    n += 1 + enqueue_lm_head(ctx, p, Mo);
    return n;
}

// The final lm_head GEMM (fused per-tile argmax, logits when asked) and the argmax reduce
// of the Mo output rows, from the final norm's pair in xn16 / xn_lo.
static int enqueue_lm_head(fa_ctx* ctx, const StepPlan& p, int Mo) {
    const fa_model_desc& d = ctx->d;
    const bool all = p.n_out < 0;
    fa::GemmArgs g{};
    g.A = ctx->xn16; g.A_lo = ctx->xn_lo; g.W8 = fa::q8p_view(ctx->lm_q, d.vocab, d.hidden); g.M = Mo; g.N = d.vocab;
    g.K = d.hidden;
    g.n_split = 1; g.epilogue = fa::kEpiArgmax; g.C = p.logits ? ctx->logits_dev : nullptr;
    g.amax_val = ctx->amax_v; g.amax_idx = ctx->amax_i;
    run_gemm(ctx, g);
    fa::launch_argmax_reduce(ctx->amax_v, ctx->amax_i, Mo, d.vocab / 64, ctx->next_dev, all ? ctx->row_tok : nullptr,
                             all ? ctx->row_pos : nullptr, ctx->stream);
    return 2;
}

// One row: the persistent step kernel (embedding, every layer, the final norm and, for
// hidden 1024, the lm_head and the argmax) as a cooperative launch; otherwise the lm_head
// and the argmax reduce follow as launches of their own. Profiling brackets the persistent
// kernel with events 0 and 1.
static int enqueue_row_step(fa_ctx* ctx, const StepPlan& p, bool capturing) {
    const fa_model_desc& d = ctx->d;
    fa::RowStepArgs a{};
    a.layers = ctx->row_layers; a.n_layers = d.n_layers; a.hidden = d.hidden; a.ffn = d.ffn;
    for (int i = 0; i < 4; ++i) a.gm[i] = ctx->row_gm[i];
    a.eps = d.rms_eps; a.q_scale = 1.0f / std::sqrt((float)kD);
    a.embed = ctx->embed; a.embed_type = ctx->embed_type; a.vocab = d.vocab; a.x_ready = p.embeds ? 1 : 0;
    a.tok = ctx->row_tok; a.slot = ctx->row_slot; a.pos = ctx->row_pos;
    a.block_table = ctx->bt_dev; a.bt_stride = ctx->bt_stride; a.n_pages = ctx->n_pages;
    a.pool = ctx->pool; a.layer_stride = ctx->layer_stride; a.rope = ctx->rope; a.max_pos = d.max_ctx;
    a.x_a = ctx->x;
    a.w_qkv = ctx->row_words; a.w_att = a.w_qkv + (kHq + 2 * kHkv) * kD; a.w_o = a.w_att + kHq * kD;
    a.w_h = a.w_o + d.hidden; a.w_dn = a.w_h + d.ffn;
    a.att_po = ctx->att_po; a.att_pml = ctx->att_pml; a.pps = p.pps; a.n_splits = p.n_splits;
    a.final_norm = ctx->final_norm; a.xn16 = ctx->xn16; a.xn_lo = ctx->xn_lo;
    a.ctl = ctx->row_ctl; a.err = ctx->err_dev;
    a.wait_ns = ctx->row_wait_ns; a.absent_cta = ctx->row_absent_cta;
    const int Mo = p.n_out < 0 ? 1 : p.n_out;
    const bool lm_here = fa::row_step_lm_fits(d.hidden, d.vocab);
    a.lm = lm_here && Mo > 0;
    a.lm_q = ctx->lm_q; a.lm_tiles = d.vocab / 64; a.logits = p.logits ? ctx->logits_dev : nullptr;
    a.amax_val = ctx->amax_v; a.amax_idx = ctx->amax_i; a.next = ctx->next_dev;
    a.feed_tok = p.n_out < 0 ? ctx->row_tok : nullptr; a.feed_pos = p.n_out < 0 ? ctx->row_pos : nullptr;
    const bool pdl = fa::launch_pdl_enabled();
    fa::set_launch_pdl(false);
    if (p.prof) record_prof(ctx, 0, capturing);
    const cudaError_t e = fa::launch_row_step(a, ctx->n_sm, ctx->stream);
    if (p.prof) record_prof(ctx, 1, capturing);
    fa::set_launch_pdl(pdl);
    if (e != cudaSuccess) {
        ctx->enqueue_failed = true;
        ctx->enqueue_msg = std::string("one-row step kernel launch: ") + cudaGetErrorString(e);
        return 1;
    }
    return 1 + (Mo > 0 && !lm_here ? enqueue_lm_head(ctx, p, Mo) : 0);
}

// enqueue_step with programmatic dependent launch between its kernels when enabled
static int enqueue_step_pdl(fa_ctx* ctx, const StepPlan& p, bool capturing) {
    fa::set_launch_pdl(ctx->use_pdl);
    ctx->enqueue_failed = false;
    ctx->enqueue_msg.clear();
    const int n = enqueue_step(ctx, p, capturing);
    fa::set_launch_pdl(false);
    return n;
}

static std::string enqueue_error(const fa_ctx* ctx) {
    return ctx->enqueue_msg.empty() ? std::string("a fused GEMM launch declined its arguments") : ctx->enqueue_msg;
}

static int run_step(fa_ctx* ctx, const StepPlan& p) {
    fa::NvtxRange nv("fa step");
    if (p.prof)
        if (int rc = ensure_prof_events(ctx)) return rc;
    if (!ctx->use_graphs) {
        ctx->last_launches = enqueue_step_pdl(ctx, p, false);
        if (ctx->enqueue_failed) return set_err(ctx, FA_ERR_CUDA, enqueue_error(ctx));
        FA_CK(cudaGetLastError());
        ctx->prof_n = p.prof && !p.row_step ? ctx->d.n_layers : 0;
        ctx->prof_row = p.prof && p.row_step;
        return FA_OK;
    }
    auto it = ctx->graphs.find(p.key());
    if (it == ctx->graphs.end()) {
        fa::NvtxRange nv_cap("fa step graph capture");
        FA_CK(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
        const int n = enqueue_step_pdl(ctx, p, true);
        cudaGraph_t graph = nullptr;
        cudaError_t e = cudaStreamEndCapture(ctx->stream, &graph);
        if (e != cudaSuccess || ctx->enqueue_failed) {
            if (graph) cudaGraphDestroy(graph);
            return set_err(ctx, FA_ERR_CUDA, ctx->enqueue_failed ? enqueue_error(ctx)
                                                                  : std::string("graph capture: ") + cudaGetErrorString(e));
        }
        cudaGraphExec_t exec = nullptr;
        e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (e != cudaSuccess) return set_err(ctx, FA_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(e));
        if (ctx->graphs.size() > 64) clear_graphs(ctx);
        it = ctx->graphs.emplace(p.key(), fa_ctx::GraphEntry{exec, n}).first;
    }
    ctx->last_launches = it->second.launches;
    FA_CK(cudaGraphLaunch(it->second.exec, ctx->stream));
    ctx->prof_n = p.prof && !p.row_step ? ctx->d.n_layers : 0;
    ctx->prof_row = p.prof && p.row_step;
    return FA_OK;
}

static int check_device_error(fa_ctx* ctx) {
    FA_CK(cudaMemcpyAsync(ctx->h_err, ctx->err_dev, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
    FA_CK(cudaStreamSynchronize(ctx->stream));
    if (*ctx->h_err) {
        const int e = *ctx->h_err;
        cudaMemsetAsync(ctx->err_dev, 0, sizeof(int), ctx->stream);
        // a one-row step that gave up leaves words of its sequence number behind: clear
        // them and start the numbering afresh
        if (ctx->row_ctl) {
            cudaMemsetAsync(ctx->row_ctl, 0, sizeof(fa::RowCtl), ctx->stream);
            cudaMemsetAsync(ctx->row_words, 0, sizeof(unsigned long long) * ctx->row_words_n, ctx->stream);
        }
        // and the split counters of a step whose attention stopped part-way
        cudaMemsetAsync(ctx->att_cnt, 0, sizeof(int) * (size_t)ctx->d.max_rows * kHkv, ctx->stream);
        cudaStreamSynchronize(ctx->stream);
        if (e & fa::kDevErrTimeout) return set_err(ctx, FA_ERR_TIMEOUT, "a bounded device wait gave up");
        return set_err(ctx, FA_ERR_DEVICE, "kernel reported error bits " + std::to_string(e) +
                                               " (2: bad page, 4: bad position / token)");
    }
    return FA_OK;
}

extern "C" int fa_forward(fa_ctx* ctx, int n_rows, const int* seq_ids, const int* token_ids, const float* embeds,
                          int* next_ids, float* logits) {
    return fa_forward_rows(ctx, n_rows, seq_ids, token_ids, embeds, -1, nullptr, next_ids, logits);
}

extern "C" int fa_forward_rows(fa_ctx* ctx, int n_rows, const int* seq_ids, const int* token_ids, const float* embeds,
                               int n_out, const int* out_rows, int* next_ids, float* logits) {
    fa::NvtxRange nv("fa_forward_rows");
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    if (!ctx->loaded) return set_err(ctx, FA_ERR_NOT_READY, "weights not loaded");
    if (n_rows <= 0 || n_rows > ctx->d.max_rows || !seq_ids)
        return set_err(ctx, FA_ERR_CAPACITY, "n_rows must be in [1, max_rows]");
    if (!token_ids && !embeds) return set_err(ctx, FA_ERR_INVALID_ARG, "give token_ids and/or embeds");
    if (n_out > n_rows || (n_out > 0 && !out_rows))
        return set_err(ctx, FA_ERR_INVALID_ARG, "n_out must be <= n_rows, with out_rows when n_out > 0");
    for (int k = 0; k < n_out; ++k)
        if (out_rows[k] < 0 || out_rows[k] >= n_rows)
            return set_err(ctx, FA_ERR_INVALID_ARG, "out_rows entry outside [0, n_rows)");
    cudaSetDevice(ctx->device);
    const fa_model_desc& d = ctx->d;
    const int M = n_rows;
    const int Mo = n_out < 0 ? M : n_out;
    // positions: consecutive per sequence in row order
    std::unordered_map<int, int> extra;
    std::vector<int> pos(M), row_len(M);
    for (int i = 0; i < M; ++i) {
        if (int rc = check_seq(ctx, seq_ids[i])) return rc;
        if (token_ids && !(token_ids[i] == -1 && embeds) && (token_ids[i] < 0 || token_ids[i] >= d.vocab))
            return set_err(ctx, FA_ERR_INVALID_ARG, "token id out of range");
        const Seq& s = ctx->seqs[seq_ids[i]];
        const int k = extra[seq_ids[i]]++;
        pos[i] = s.len + k;
        row_len[i] = pos[i] + 1;
        if (pos[i] >= s.max_tokens || pos[i] >= d.max_ctx)
            return set_err(ctx, FA_ERR_CAPACITY, "sequence " + std::to_string(seq_ids[i]) + " is full");
    }
    std::vector<std::pair<int, int>> need;
    for (int i = 0; i < M; ++i) need.push_back({seq_ids[i], pos[i] + 1});
    std::vector<int> ui, up;
    if (int rc = reserve_pages(ctx, need, ui, up)) return rc;
    if (logits)
        if (int rc = ensure_logits(ctx)) return rc;

    int* h = ctx->h_rows;
    for (int i = 0; i < M; ++i) {
        h[i] = token_ids ? token_ids[i] : 0;
        h[M + i] = seq_ids[i];
        h[2 * M + i] = pos[i];
    }
    // runs of >= kPrefillMinRun rows of one sequence at consecutive positions become
    // tensor-core prefill tiles; the other rows stay with the decode kernel
    int* h_tiles = h + 3 * M;
    int* h_dec = h + 5 * M;
    int* h_out = h + 6 * M;
    for (int k = 0; k < n_out; ++k) h_out[k] = out_rows[k];
    int n_tiles = 0, n_dec = 0;
    std::vector<int> dec_len;
    for (int i = 0; i < M;) {
        int j = i + 1;
        while (j < M && seq_ids[j] == seq_ids[i] && pos[j] == pos[j - 1] + 1) ++j;
        if (ctx->pool_map_ok && j - i >= kPrefillMinRun) {
            for (int t = i; t < j; t += 64) {
                h_tiles[2 * n_tiles] = t;
                h_tiles[2 * n_tiles + 1] = std::min(64, j - t);
                ++n_tiles;
            }
        } else {
            for (int t = i; t < j; ++t) {
                h_dec[n_dec++] = t;
                dec_len.push_back(row_len[t]);
            }
        }
        i = j;
    }
    int rc = FA_OK;
    auto body = [&]() -> int {
        FA_CK(cudaMemcpyAsync(ctx->row_tok, h, sizeof(int) * M, cudaMemcpyHostToDevice, ctx->stream));
        FA_CK(cudaMemcpyAsync(ctx->row_slot, h + M, sizeof(int) * M, cudaMemcpyHostToDevice, ctx->stream));
        FA_CK(cudaMemcpyAsync(ctx->row_pos, h + 2 * M, sizeof(int) * M, cudaMemcpyHostToDevice, ctx->stream));
        if (n_tiles > 0) {
            FA_CK(cudaMemcpyAsync(ctx->pf_tiles, h_tiles, sizeof(int2) * n_tiles, cudaMemcpyHostToDevice, ctx->stream));
            if (n_dec > 0)
                FA_CK(cudaMemcpyAsync(ctx->dec_rows, h_dec, sizeof(int) * n_dec, cudaMemcpyHostToDevice, ctx->stream));
        }
        if (n_out > 0)
            FA_CK(cudaMemcpyAsync(ctx->out_rows, h_out, sizeof(int) * n_out, cudaMemcpyHostToDevice, ctx->stream));
        if (int r = upload_updates(ctx, ui, up)) return r;
        if (embeds)
            FA_CK(cudaMemcpyAsync(ctx->x, embeds, sizeof(float) * M * d.hidden, cudaMemcpyDefault, ctx->stream));
        // embeddings only: x is the input; with token ids too, rows with id -1 keep their embedding
        const bool x_ready = embeds && !token_ids;
        StepPlan p = n_tiles > 0 ? make_plan(ctx, M, dec_len, x_ready, logits != nullptr, n_tiles)
                                 : make_plan(ctx, M, row_len, x_ready, logits != nullptr, 0, (int)extra.size() == M);
        p.n_out = n_out < 0 ? -1 : n_out;
        if (int r = run_step(ctx, p)) return r;
        if (Mo > 0)
            FA_CK(cudaMemcpyAsync(ctx->h_next, ctx->next_dev, sizeof(int) * Mo, cudaMemcpyDeviceToHost, ctx->stream));
        if (logits && Mo > 0)
            FA_CK(cudaMemcpyAsync(logits, ctx->logits_dev, sizeof(float) * Mo * d.vocab, cudaMemcpyDeviceToHost,
                                  ctx->stream));
        return check_device_error(ctx);
    };
    rc = body();
    if (rc != FA_OK) {
        // roll back the page reservations of this call
        for (size_t k = ui.size(); k-- > 0;) {
            const int seq = ui[k] / ctx->bt_stride;
            ctx->seqs[seq].pages.pop_back();
            ctx->palloc.release(up[k]);
        }
        return rc;
    }
    for (int i = 0; i < M; ++i) ctx->seqs[seq_ids[i]].len += 1;
    if (next_ids && Mo > 0) std::memcpy(next_ids, ctx->h_next, sizeof(int) * Mo);
    return FA_OK;
}

extern "C" int fa_prefill(fa_ctx* ctx, int seq_id, const float* embeds, int n_tok, int* next_id, float* last_logits) {
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    if (int rc = check_seq(ctx, seq_id)) return rc;
    if (!embeds || n_tok <= 0) return set_err(ctx, FA_ERR_INVALID_ARG, "embeds and n_tok > 0 required");
    const int R = ctx->d.max_rows;
    std::vector<int> ids(R, seq_id);
    for (int off = 0; off < n_tok; off += R) {
        const int m = std::min(R, n_tok - off);
        const bool last = off + m == n_tok;
        const int last_row = m - 1;
        int nx = 0;
        // lm_head only for the last row of the last chunk
        if (int rc = fa_forward_rows(ctx, m, ids.data(), nullptr, embeds + (size_t)off * ctx->d.hidden, last ? 1 : 0,
                                     last ? &last_row : nullptr, &nx, last ? last_logits : nullptr))
            return rc;
        if (last && next_id) *next_id = nx;
    }
    return FA_OK;
}

extern "C" int fa_decode_step(fa_ctx* ctx, int n_seq, const int* seq_ids, const int* token_ids, int* next_ids,
                              float* logits) {
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    if (!seq_ids || !token_ids) return set_err(ctx, FA_ERR_INVALID_ARG, "seq_ids and token_ids required");
    for (int i = 0; i < n_seq; ++i)
        for (int j = 0; j < i; ++j)
            if (seq_ids[i] == seq_ids[j]) return set_err(ctx, FA_ERR_INVALID_ARG, "decode rows must be distinct sequences");
    return fa_forward(ctx, n_seq, seq_ids, token_ids, nullptr, next_ids, logits);
}

extern "C" int fa_generate(fa_ctx* ctx, int n_seq, const int* seq_ids, const int* first_tokens, int n_steps,
                           int* out_ids, float* device_ms) {
    fa::NvtxRange nv("fa_generate");
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    if (!ctx->loaded) return set_err(ctx, FA_ERR_NOT_READY, "weights not loaded");
    if (n_seq <= 0 || n_seq > ctx->d.max_rows || !seq_ids || !first_tokens || n_steps <= 0)
        return set_err(ctx, FA_ERR_INVALID_ARG, "bad arguments");
    if ((size_t)n_seq * n_steps > (size_t)ctx->d.max_rows * 4096)
        return set_err(ctx, FA_ERR_CAPACITY, "n_seq * n_steps exceeds the output staging buffer");
    cudaSetDevice(ctx->device);
    const fa_model_desc& d = ctx->d;
    std::vector<int> base(n_seq);
    std::vector<std::pair<int, int>> need;
    for (int i = 0; i < n_seq; ++i) {
        if (int rc = check_seq(ctx, seq_ids[i])) return rc;
        for (int j = 0; j < i; ++j)
            if (seq_ids[i] == seq_ids[j]) return set_err(ctx, FA_ERR_INVALID_ARG, "rows must be distinct sequences");
        if (first_tokens[i] < 0 || first_tokens[i] >= d.vocab) return set_err(ctx, FA_ERR_INVALID_ARG, "token id out of range");
        const Seq& s = ctx->seqs[seq_ids[i]];
        base[i] = s.len;
        if (s.len + n_steps > s.max_tokens || s.len + n_steps > d.max_ctx)
            return set_err(ctx, FA_ERR_CAPACITY, "sequence " + std::to_string(seq_ids[i]) + " would overflow");
        need.push_back({seq_ids[i], s.len + n_steps});
    }
    std::vector<int> ui, up;
    if (int rc = reserve_pages(ctx, need, ui, up)) return rc;
    int* h = ctx->h_rows;
    for (int i = 0; i < n_seq; ++i) {
        h[i] = first_tokens[i];
        h[n_seq + i] = seq_ids[i];
        h[2 * n_seq + i] = base[i];
    }
    auto body = [&]() -> int {
        FA_CK(cudaMemcpyAsync(ctx->row_tok, h, sizeof(int) * n_seq, cudaMemcpyHostToDevice, ctx->stream));
        FA_CK(cudaMemcpyAsync(ctx->row_slot, h + n_seq, sizeof(int) * n_seq, cudaMemcpyHostToDevice, ctx->stream));
        FA_CK(cudaMemcpyAsync(ctx->row_pos, h + 2 * n_seq, sizeof(int) * n_seq, cudaMemcpyHostToDevice, ctx->stream));
        if (int r = upload_updates(ctx, ui, up)) return r;
        FA_CK(cudaEventRecord(ctx->ev_t0, ctx->stream));
        std::vector<int> row_len(n_seq);
        for (int k = 0; k < n_steps; ++k) {
            for (int i = 0; i < n_seq; ++i) row_len[i] = base[i] + k + 1;
            StepPlan p = make_plan(ctx, n_seq, row_len, false, false, 0, true);   // distinct: checked above
            if (int r = run_step(ctx, p)) return r;
            FA_CK(cudaMemcpyAsync(ctx->h_next + (size_t)k * n_seq, ctx->next_dev, sizeof(int) * n_seq,
                                  cudaMemcpyDeviceToHost, ctx->stream));
        }
        FA_CK(cudaEventRecord(ctx->ev_t1, ctx->stream));
        return check_device_error(ctx);
    };
    int rc = body();
    if (rc != FA_OK) {
        for (size_t k = ui.size(); k-- > 0;) {
            const int seq = ui[k] / ctx->bt_stride;
            ctx->seqs[seq].pages.pop_back();
            ctx->palloc.release(up[k]);
        }
        return rc;
    }
    for (int i = 0; i < n_seq; ++i) ctx->seqs[seq_ids[i]].len += n_steps;
    if (out_ids) std::memcpy(out_ids, ctx->h_next, sizeof(int) * (size_t)n_seq * n_steps);
    if (device_ms) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, ctx->ev_t0, ctx->ev_t1);
        *device_ms = ms;
    }
    return FA_OK;
}

// ------------------------------------------------------------------- pages --
static int ensure_scratch_ints(fa_ctx* ctx, int n) {
    if (ctx->scratch_ints_n >= n) return FA_OK;
    if (ctx->scratch_ints) cudaFree(ctx->scratch_ints);
    ctx->scratch_ints = nullptr;
    ctx->scratch_ints_n = 0;
    void* v = nullptr;
    if (cudaMalloc(&v, sizeof(int) * (size_t)n) != cudaSuccess) {
        cudaGetLastError();
        return set_err(ctx, FA_ERR_OOM, "page list buffer");
    }
    ctx->scratch_ints = (int*)v;
    ctx->scratch_ints_n = n;
    return FA_OK;
}

extern "C" int fa_kv_read_pages(fa_ctx* ctx, int layer, const int* pages, int n, uint16_t* out) {
    if (!ctx || !pages || !out || n < 0) return set_err(ctx, FA_ERR_INVALID_ARG, "bad arguments");
    if (layer < 0 || layer >= ctx->d.n_layers) return set_err(ctx, FA_ERR_INVALID_ARG, "layer out of range");
    for (int i = 0; i < n; ++i)
        if (pages[i] < 0 || pages[i] >= ctx->n_pages) return set_err(ctx, FA_ERR_INVALID_ARG, "page out of range");
    if (n == 0) return FA_OK;
    cudaSetDevice(ctx->device);
    if (int rc = ensure_scratch_ints(ctx, n)) return rc;
    __half* buf = nullptr;
    FA_CK(cudaMalloc(&buf, kPageElems * 2 * (size_t)n));
    int rc = FA_OK;
    auto body = [&]() -> int {
        FA_CK(cudaMemcpyAsync(ctx->scratch_ints, pages, sizeof(int) * n, cudaMemcpyHostToDevice, ctx->stream));
        fa::launch_read_pages(ctx->pool + (size_t)layer * ctx->layer_stride, ctx->scratch_ints, n, buf, ctx->stream);
        FA_CK(cudaGetLastError());
        FA_CK(cudaMemcpyAsync(out, buf, kPageElems * 2 * (size_t)n, cudaMemcpyDeviceToHost, ctx->stream));
        FA_CK(cudaStreamSynchronize(ctx->stream));
        return FA_OK;
    };
    rc = body();
    cudaFree(buf);
    return rc;
}

extern "C" int fa_kv_append(fa_ctx* ctx, int n_rows, const int* seq_ids, const uint16_t* k, const uint16_t* v) {
    if (!ctx || !seq_ids || !k || !v || n_rows <= 0) return set_err(ctx, FA_ERR_INVALID_ARG, "bad arguments");
    cudaSetDevice(ctx->device);
    const int L = ctx->d.n_layers;
    std::unordered_map<int, int> extra;
    std::vector<int> pos(n_rows);
    std::vector<std::pair<int, int>> need;
    for (int i = 0; i < n_rows; ++i) {
        if (int rc = check_seq(ctx, seq_ids[i])) return rc;
        const Seq& s = ctx->seqs[seq_ids[i]];
        pos[i] = s.len + extra[seq_ids[i]]++;
        if (pos[i] >= s.max_tokens) return set_err(ctx, FA_ERR_CAPACITY, "sequence full");
        need.push_back({seq_ids[i], pos[i] + 1});
    }
    std::vector<int> ui, up;
    if (int rc = reserve_pages(ctx, need, ui, up)) return rc;
    const size_t bytes = (size_t)n_rows * L * kHkv * kD * 2;
    __half *kd = nullptr, *vd = nullptr;
    int *pd = nullptr;
    auto body = [&]() -> int {
        FA_CK(cudaMalloc(&kd, bytes));
        FA_CK(cudaMalloc(&vd, bytes));
        FA_CK(cudaMalloc(&pd, sizeof(int) * 2 * n_rows));
        FA_CK(cudaMemcpyAsync(kd, k, bytes, cudaMemcpyHostToDevice, ctx->stream));
        FA_CK(cudaMemcpyAsync(vd, v, bytes, cudaMemcpyHostToDevice, ctx->stream));
        std::vector<int> hp(2 * n_rows);
        for (int i = 0; i < n_rows; ++i) { hp[i] = pos[i]; hp[n_rows + i] = seq_ids[i]; }
        FA_CK(cudaMemcpyAsync(pd, hp.data(), sizeof(int) * 2 * n_rows, cudaMemcpyHostToDevice, ctx->stream));
        if (int r = upload_updates(ctx, ui, up)) return r;
        fa::RawAppendArgs a{};
        a.k = kd; a.v = vd; a.M = n_rows; a.n_layers = L; a.Hkv = kHkv; a.pos = pd; a.slot = pd + n_rows;
        a.block_table = ctx->bt_dev; a.bt_stride = ctx->bt_stride; a.n_pages = ctx->n_pages; a.pool = ctx->pool;
        a.err = ctx->err_dev;
        fa::launch_kv_append_raw(a, ctx->stream);
        FA_CK(cudaGetLastError());
        return check_device_error(ctx);
    };
    int rc = body();
    if (kd) cudaFree(kd);
    if (vd) cudaFree(vd);
    if (pd) cudaFree(pd);
    if (rc != FA_OK) {
        for (size_t q = ui.size(); q-- > 0;) {
            ctx->seqs[ui[q] / ctx->bt_stride].pages.pop_back();
            ctx->palloc.release(up[q]);
        }
        return rc;
    }
    for (int i = 0; i < n_rows; ++i) ctx->seqs[seq_ids[i]].len += 1;
    return FA_OK;
}

extern "C" int fa_kv_fill_synthetic(fa_ctx* ctx, int seq_id, int n_tokens, uint64_t seed) {
    if (int rc = check_seq(ctx, seq_id)) return rc;
    if (n_tokens < 0) return set_err(ctx, FA_ERR_INVALID_ARG, "n_tokens < 0");
    Seq& s = ctx->seqs[seq_id];
    if (s.len % fa::kPageTokens)
        return set_err(ctx, FA_ERR_INVALID_ARG, "synthetic fill starts on a page boundary (length % 16 == 0)");
    if (s.len + n_tokens > s.max_tokens) return set_err(ctx, FA_ERR_CAPACITY, "sequence would overflow");
    cudaSetDevice(ctx->device);
    const size_t first_new = s.pages.size();
    std::vector<int> ui, up;
    if (int rc = reserve_pages(ctx, {{seq_id, s.len + n_tokens}}, ui, up)) return rc;
    std::vector<int> fill(s.pages.begin() + first_new, s.pages.end());
    auto body = [&]() -> int {
        if (int r = upload_updates(ctx, ui, up)) return r;
        if (!fill.empty()) {
            if (int r = ensure_scratch_ints(ctx, (int)fill.size())) return r;
            FA_CK(cudaMemcpyAsync(ctx->scratch_ints, fill.data(), sizeof(int) * fill.size(), cudaMemcpyHostToDevice,
                                  ctx->stream));
            fa::launch_fill_random(ctx->pool, ctx->layer_stride, ctx->d.n_layers, ctx->scratch_ints, (int)fill.size(),
                                   seed, ctx->stream);
            FA_CK(cudaGetLastError());
        }
        FA_CK(cudaStreamSynchronize(ctx->stream));
        return FA_OK;
    };
    int rc = body();
    if (rc != FA_OK) {
        for (size_t q = ui.size(); q-- > 0;) {
            s.pages.pop_back();
            ctx->palloc.release(up[q]);
        }
        return rc;
    }
    s.len += n_tokens;
    return FA_OK;
}

extern "C" int fa_pool_compact(fa_ctx* ctx, int* n_moved) {
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    cudaSetDevice(ctx->device);
    std::vector<int> src, dst;
    ctx->palloc.compact(src, dst);
    if (n_moved) *n_moved = (int)src.size();
    if (src.empty()) return FA_OK;
    std::unordered_map<int, int> remap;
    for (size_t i = 0; i < src.size(); ++i) remap[src[i]] = dst[i];
    std::vector<int> ui, up;
    for (int sid = 0; sid < (int)ctx->seqs.size(); ++sid) {
        Seq& s = ctx->seqs[sid];
        if (!s.open) continue;
        for (size_t k = 0; k < s.pages.size(); ++k) {
            auto it = remap.find(s.pages[k]);
            if (it != remap.end()) {
                s.pages[k] = it->second;
                ui.push_back(sid * ctx->bt_stride + (int)k);
                up.push_back(it->second);
            }
        }
    }
    const int n = (int)src.size();
    if (int rc = ensure_scratch_ints(ctx, 2 * n)) return rc;
    std::vector<int> both(src);
    both.insert(both.end(), dst.begin(), dst.end());
    FA_CK(cudaMemcpyAsync(ctx->scratch_ints, both.data(), sizeof(int) * 2 * n, cudaMemcpyHostToDevice, ctx->stream));
    fa::launch_page_copy(ctx->pool, ctx->layer_stride, ctx->d.n_layers, ctx->scratch_ints, ctx->scratch_ints + n, n,
                         ctx->stream);
    FA_CK(cudaGetLastError());
    if (int rc = upload_updates(ctx, ui, up)) return rc;
    FA_CK(cudaStreamSynchronize(ctx->stream));
    return FA_OK;
}

// ------------------------------------------------------------- measurement --
extern "C" int fa_profile(fa_ctx* ctx, int enable) {
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    ctx->prof = enable != 0;
    return FA_OK;
}

extern "C" int fa_profile_attention(fa_ctx* ctx, float* total_ms, int* n_launches) {
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    FA_CK(cudaStreamSynchronize(ctx->stream));
    float tot = 0.0f;
    int n = 0;
    if (ctx->prof_n > 0) {
        const int L = ctx->d.n_layers;
        const int layers[3] = {0, L / 2, L - 1};
        for (int i = 0; i < 3; ++i) {
            if (i > 0 && layers[i] == layers[i - 1]) continue;
            float ms = 0.0f;
            FA_CK(cudaEventElapsedTime(&ms, ctx->prof_ev[2 * layers[i]], ctx->prof_ev[2 * layers[i] + 1]));
            tot += ms;
            ++n;
        }
    }
    if (total_ms) *total_ms = tot;
    if (n_launches) *n_launches = n;
    return FA_OK;
}

extern "C" int fa_profile_row_step(fa_ctx* ctx, float* ms) {
    if (!ctx || !ms) return set_err(ctx, FA_ERR_INVALID_ARG, "bad arguments");
    FA_CK(cudaStreamSynchronize(ctx->stream));
    *ms = 0.0f;
    if (ctx->prof_row) FA_CK(cudaEventElapsedTime(ms, ctx->prof_ev[0], ctx->prof_ev[1]));
    return FA_OK;
}

extern "C" int fa_step_launches(const fa_ctx* ctx, int* n) {
    if (!ctx) return set_err(nullptr, FA_ERR_INVALID_ARG, "ctx is NULL");
    if (n) *n = ctx->last_launches;
    return FA_OK;
}

// ------------------------------------------------------------ kernel ops --
#define OP_CK(call)                                                                                     \
    do {                                                                                                \
        cudaError_t e_ = (call);                                                                        \
        if (e_ != cudaSuccess) return set_err(nullptr, FA_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

extern "C" int fa_op_qknorm_rope_append(const float* qkv, int M, const int* pos, const int* slot, const int* bt,
                                        int bt_stride, int n_pages, const float* qn, const float* kn, float eps,
                                        const float* rope, int max_pos, uint16_t* pool_layer, float* q_out, int* err,
                                        void* stream) {
    if (!qkv || !pos || !slot || !bt || !qn || !kn || !rope || !pool_layer || !q_out || M <= 0)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "null argument");
    if (int rc = ensure_configured()) return rc;
    fa::AppendArgs a{};
    a.qkv_part = qkv; a.n_part = 1; a.M = M; a.pos = pos; a.slot = slot; a.block_table = bt; a.bt_stride = bt_stride;
    a.n_pages = n_pages; a.qn_w = qn; a.kn_w = kn; a.Hq = kHq; a.Hkv = kHkv; a.eps = eps;
    a.q_scale = 1.0f / std::sqrt((float)kD); a.rope = reinterpret_cast<const float2*>(rope); a.max_pos = max_pos;
    a.pool_layer = reinterpret_cast<__half*>(pool_layer); a.q_out = q_out; a.err = err;
    fa::launch_qknorm_rope_append(a, (cudaStream_t)stream);
    OP_CK(cudaGetLastError());
    return FA_OK;
}

extern "C" int fa_op_kv_append(const uint16_t* k, const uint16_t* v, int M, int n_layers, const int* pos,
                               const int* slot, const int* bt, int bt_stride, int n_pages, uint16_t* pool, int* err,
                               void* stream) {
    if (!k || !v || !pos || !slot || !bt || !pool || M <= 0 || n_layers <= 0)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "null argument");
    fa::RawAppendArgs a{};
    a.k = reinterpret_cast<const __half*>(k); a.v = reinterpret_cast<const __half*>(v); a.M = M;
    a.n_layers = n_layers; a.Hkv = kHkv; a.pos = pos; a.slot = slot; a.block_table = bt; a.bt_stride = bt_stride;
    a.n_pages = n_pages; a.pool = reinterpret_cast<__half*>(pool); a.err = err;
    fa::launch_kv_append_raw(a, (cudaStream_t)stream);
    OP_CK(cudaGetLastError());
    return FA_OK;
}

extern "C" int fa_op_kv_gather(const uint16_t* pool, int n_layers, int n_pages, const int* bt, int bt_stride,
                               const int* slot, const int* n_kv, const int* row0, int M, int max_pages,
                               int total_rows, uint16_t* k_out, uint16_t* v_out, int* err, void* stream) {
    if (!pool || !bt || !slot || !n_kv || !row0 || !k_out || !v_out || M <= 0 || n_layers <= 0 ||
        n_pages <= 0 || max_pages <= 0 || total_rows <= 0 || bt_stride < max_pages)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "null or non-positive argument, or bt_stride < max_pages");
    if (M > 65535 || n_layers > 65535)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "M and n_layers are limited to 65535");
    if ((reinterpret_cast<uintptr_t>(pool) & 15) || (reinterpret_cast<uintptr_t>(k_out) & 15) ||
        (reinterpret_cast<uintptr_t>(v_out) & 15))
        return set_err(nullptr, FA_ERR_INVALID_ARG, "pool and outputs must be 16-byte aligned");
    fa::GatherArgs a{};
    a.pool = reinterpret_cast<const __half*>(pool); a.n_layers = n_layers; a.n_pages = n_pages; a.Hkv = kHkv;
    a.block_table = bt; a.bt_stride = bt_stride; a.slot = slot; a.n_kv = n_kv; a.row0 = row0; a.M = M;
    a.max_pages = max_pages; a.total_rows = total_rows; a.k_out = reinterpret_cast<__half*>(k_out);
    a.v_out = reinterpret_cast<__half*>(v_out); a.err = err;
    fa::launch_kv_gather(a, (cudaStream_t)stream);
    OP_CK(cudaGetLastError());
    return FA_OK;
}

extern "C" int fa_op_prefill_attention(const float* q, int M, const int* pos, const int* slot, const int* bt,
                                       int bt_stride, int n_pages, const uint16_t* pool_layer, const int* tiles,
                                       int n_tiles, uint16_t* out16, uint16_t* out16_lo, float* out32, int* err,
                                       void* stream) {
    if (!q || !pos || !slot || !bt || !pool_layer || !tiles || M <= 0 || n_tiles <= 0 || n_pages <= 0 ||
        bt_stride <= 0 || (!out16 && !out32))
        return set_err(nullptr, FA_ERR_INVALID_ARG, "null or non-positive argument");
    if ((reinterpret_cast<uintptr_t>(pool_layer) & 15) || (reinterpret_cast<uintptr_t>(tiles) & 7) ||
        (reinterpret_cast<uintptr_t>(out16) & 15) || (reinterpret_cast<uintptr_t>(out16_lo) & 15) ||
        (reinterpret_cast<uintptr_t>(out32) & 15) || (reinterpret_cast<uintptr_t>(q) & 15))
        return set_err(nullptr, FA_ERR_INVALID_ARG, "q, pool and outputs must be 16-byte, tiles 8-byte aligned");
    if (int rc = ensure_configured()) return rc;
    CUtensorMap tm;
    if (!fa::make_pool_map(&tm, pool_layer, (long long)n_pages * kHkv * 2 * fa::kPageTokens))
        return set_err(nullptr, FA_ERR_CUDA, "cannot build the page-pool tensor map");
    fa::PrefillAttnArgs a{};
    a.q = q; a.block_table = bt; a.bt_stride = bt_stride; a.n_pages = n_pages; a.slot = slot; a.pos = pos;
    a.M = M; a.Hq = kHq; a.Hkv = kHkv; a.tiles = reinterpret_cast<const int2*>(tiles); a.n_tiles = n_tiles;
    a.pool_row0 = 0;
    a.out16 = reinterpret_cast<__half*>(out16); a.out16_lo = reinterpret_cast<__half*>(out16_lo);
    a.out32 = out32; a.err = err;
    fa::launch_prefill_attention(tm, a, (cudaStream_t)stream);
    OP_CK(cudaGetLastError());
    return FA_OK;
}

extern "C" int fa_op_wait_selftest(int limit_us, int* err_dev, void* stream) {
    if (limit_us <= 0 || limit_us > 1000000 || !err_dev)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "limit_us in (0, 1e6] and err_dev required");
    fa::launch_wait_selftest(err_dev, (unsigned long long)limit_us * 1000ull, (cudaStream_t)stream);
    OP_CK(cudaGetLastError());
    return FA_OK;
}

extern "C" int fa_op_attention_plan(const int* n_kv, int M, int n_sm, int* pages_per_split, int* n_splits) {
    if (!n_kv || M <= 0 || n_sm <= 0 || !pages_per_split || !n_splits)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "fa_op_attention_plan: bad argument");
    std::vector<int> row_pages((size_t)M);
    for (int i = 0; i < M; ++i) {
        if (n_kv[i] <= 0) return set_err(nullptr, FA_ERR_INVALID_ARG, "fa_op_attention_plan: n_kv must be > 0");
        row_pages[i] = (n_kv[i] + fa::kPageTokens - 1) / fa::kPageTokens;
    }
    attention_split(row_pages, n_sm, 64, pages_per_split, n_splits, nullptr, fa::attn_warps(M));
    return FA_OK;
}

extern "C" int fa_step_attention_plan(const int* n_kv, int M, int n_sm, int mask, int* pages_per_split,
                                      int* n_splits, int* warps, int* fused) {
    if (!n_kv || M <= 0 || n_sm <= 0 || mask < 0 || mask > 15 || !pages_per_split || !n_splits || !warps || !fused)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "fa_step_attention_plan: bad argument");
    std::vector<int> row_pages((size_t)M);
    for (int i = 0; i < M; ++i) {
        if (n_kv[i] <= 0) return set_err(nullptr, FA_ERR_INVALID_ARG, "fa_step_attention_plan: n_kv must be > 0");
        row_pages[i] = (n_kv[i] + fa::kPageTokens - 1) / fa::kPageTokens;
    }
    const AttnChoice c = plan_attention(row_pages, n_sm, 64, mask);
    *pages_per_split = c.pps;
    *n_splits = c.n_splits;
    *warps = c.warps;
    *fused = (c.merge ? 1 : 0) | (c.append ? 2 : 0);
    return FA_OK;
}

extern "C" size_t fa_op_attention_scratch_bytes(int M, int n_splits) {
    if (M <= 0 || n_splits <= 1) return 0;
    return (size_t)M * kHq * n_splits * (kD + 2) * sizeof(float);
}

extern "C" int fa_op_paged_attention(const float* q, int M, const int* pos, const int* slot, const int* bt,
                                     int bt_stride, int n_pages, const uint16_t* pool_layer, int pps, int n_splits,
                                     void* scratch, uint16_t* out16, uint16_t* out16_lo, float* out32, int* err,
                                     void* stream) {
    if (!q || !pos || !slot || !bt || !pool_layer || M <= 0 || pps <= 0 || n_splits <= 0 || (!out16 && !out32))
        return set_err(nullptr, FA_ERR_INVALID_ARG, "null or non-positive argument");
    if (n_splits > 1 && !scratch) return set_err(nullptr, FA_ERR_INVALID_ARG, "scratch required when n_splits > 1");
    if (n_splits > 1 && (reinterpret_cast<uintptr_t>(scratch) & 15))
        return set_err(nullptr, FA_ERR_INVALID_ARG, "scratch must be 16-byte aligned");
    if (int rc = ensure_configured()) return rc;
    fa::AttnArgs a{};
    a.q = q; a.pool_layer = reinterpret_cast<const __half*>(pool_layer); a.block_table = bt; a.bt_stride = bt_stride;
    a.n_pages = n_pages; a.slot = slot; a.pos = pos; a.M = M; a.Hq = kHq; a.Hkv = kHkv; a.pages_per_split = pps;
    a.n_splits = n_splits;
    a.part_o = reinterpret_cast<float*>(scratch);
    a.part_ml = a.part_o ? a.part_o + (size_t)M * kHq * n_splits * kD : nullptr;
    a.out16 = reinterpret_cast<__half*>(out16); a.out16_lo = reinterpret_cast<__half*>(out16_lo);
    a.out32 = out32; a.err = err;
    fa::launch_paged_attention(a, (cudaStream_t)stream);
    if (n_splits > 1) fa::launch_attn_combine(a, (cudaStream_t)stream);
    OP_CK(cudaGetLastError());
    return FA_OK;
}

extern "C" int fa_op_repack_q8(const uint8_t* raw, int N, int K, uint16_t* w16, void* stream) {
    if (!raw || !w16 || N <= 0 || K <= 0 || K % 32) return set_err(nullptr, FA_ERR_INVALID_ARG, "bad arguments");
    fa::launch_repack_q8(raw, N, K, 0, reinterpret_cast<__half*>(w16), (cudaStream_t)stream);
    OP_CK(cudaGetLastError());
    return FA_OK;
}

static int op_gemm(const fa::GemmArgs& g, int variant, cudaStream_t s) {
    if (variant < 0 || variant > 4) return set_err(nullptr, FA_ERR_INVALID_ARG, "variant must be 0 to 4");
    if (variant == 1) {
        fa::launch_q8_gemm(g, s);
    } else if (variant == 3) {
        if (!fa::launch_q8_gemv(g, s)) return set_err(nullptr, FA_ERR_INVALID_ARG, "shape outside the CUDA-core kernel");
    } else if (variant == 4) {
        if (!fa::launch_q8_gemm_tc_skinny(g, nullptr, s))
            return set_err(nullptr, FA_ERR_INVALID_ARG, "shape outside the few-row tcgen05 kernel");
    } else if (variant == 0 && gemv_rows(0, g.M) && fa::launch_q8_gemv(g, s)) {
        // taken by the CUDA-core kernel
    } else if (variant == 0 && skinny_rows(0, g.M, g.epilogue, g.W8.q != nullptr) &&
               fa::launch_q8_gemm_tc_skinny(g, nullptr, s)) {
        // taken by the few-row tcgen05 kernel
    } else {
        if (!fa::gemm_tc_supported(g)) return set_err(nullptr, FA_ERR_INVALID_ARG, "shape outside the tcgen05 kernel");
        if (!fa::launch_q8_gemm_tc(g, nullptr, s)) return set_err(nullptr, FA_ERR_CUDA, "tensor map encoding failed");
    }
    OP_CK(cudaGetLastError());
    return FA_OK;
}

extern "C" int fa_op_gemm_plan(int M, int N, int K, int variant, int n_sm, int* n_split) {
    if (M <= 0 || N <= 0 || K <= 0 || N % 64 || K % 64 || n_sm <= 0 || !n_split || variant < 0 || variant > 4)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "fa_op_gemm_plan: bad argument");
    if (gemv_rows(variant, M) && fa::gemv_shape_supported(M, N, K, fa::kEpiStoreF32)) *n_split = 1;
    else if (skinny_rows(variant, M) && N % 128 == 0) *n_split = fa::gemm_tc_skinny_pick_split(M, N, K, n_sm);
    else if (variant != 1 && N % 128 == 0) *n_split = fa::gemm_tc_pick_split(M, N, K, n_sm);
    else *n_split = fa::gemm_pick_split(M, N, K, n_sm);
    return FA_OK;
}

extern "C" int fa_op_q8_gemm(const uint16_t* a16, const uint16_t* a16_lo, int M, int K, const uint16_t* w16,
                             int N, int n_split, float* c, int variant, void* stream) {
    if (!a16 || !w16 || !c || M <= 0 || N <= 0 || K <= 0 || N % 64 || K % 64 || n_split <= 0 ||
        (K / 64) % n_split)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "need N, K multiples of 64 and n_split dividing K/64");
    if (int rc = ensure_configured()) return rc;
    fa::GemmArgs g{};
    g.A = reinterpret_cast<const __half*>(a16); g.A_lo = reinterpret_cast<const __half*>(a16_lo);
    g.Wh = reinterpret_cast<const __half*>(w16);
    g.M = M; g.N = N; g.K = K; g.n_split = n_split; g.epilogue = fa::kEpiStoreF32; g.C = c;
    return op_gemm(g, variant, (cudaStream_t)stream);
}

extern "C" int fa_op_q8_gemm_swiglu(const uint16_t* a16, const uint16_t* a16_lo, int M, int K, const uint16_t* w16,
                                    int N, uint16_t* h16, uint16_t* h_lo, void* stream) {
    if (!a16 || !w16 || !h16 || M <= 0 || N <= 0 || K <= 0)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "null or non-positive argument");
    if (int rc = ensure_configured()) return rc;
    fa::GemmArgs g{};
    g.A = reinterpret_cast<const __half*>(a16); g.A_lo = reinterpret_cast<const __half*>(a16_lo);
    g.Wh = reinterpret_cast<const __half*>(w16);
    g.M = M; g.N = N; g.K = K; g.n_split = 1; g.epilogue = fa::kEpiSwiglu;
    g.H = reinterpret_cast<__half*>(h16); g.H_lo = reinterpret_cast<__half*>(h_lo);
    if (!fa::launch_q8_gemv(g, (cudaStream_t)stream))
        return set_err(nullptr, FA_ERR_INVALID_ARG, "shape outside the small-M kernel");
    OP_CK(cudaGetLastError());
    return FA_OK;
}

extern "C" int fa_op_swiglu(const float* part, int n_part, int M, int ffn, uint16_t* h16, uint16_t* h_lo,
                            void* stream) {
    if (!part || !h16 || n_part <= 0 || M <= 0 || ffn <= 0 || ffn % 4)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "need partials, n_part > 0, M > 0 and ffn a multiple of 4");
    fa::launch_swiglu(part, n_part, M, ffn, reinterpret_cast<__half*>(h16), reinterpret_cast<__half*>(h_lo),
                      (cudaStream_t)stream);
    OP_CK(cudaGetLastError());
    return FA_OK;
}

extern "C" size_t fa_op_argmax_scratch_bytes(int M, int N) {
    if (M <= 0 || N <= 0) return 0;
    return (size_t)M * (N / 64) * (sizeof(float) + sizeof(int));
}

extern "C" int fa_op_q8_gemm_argmax(const uint16_t* a16, const uint16_t* a16_lo, int M, int K, const uint16_t* w16,
                                    int N, void* scratch, int* next, float* logits, int variant, void* stream) {
    if (!a16 || !w16 || !scratch || !next || M <= 0 || N % 64 || K % 64)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "bad arguments");
    if (int rc = ensure_configured()) return rc;
    fa::GemmArgs g{};
    g.A = reinterpret_cast<const __half*>(a16); g.A_lo = reinterpret_cast<const __half*>(a16_lo);
    g.Wh = reinterpret_cast<const __half*>(w16);
    g.M = M; g.N = N; g.K = K; g.n_split = 1; g.epilogue = fa::kEpiArgmax; g.C = logits;
    g.amax_val = reinterpret_cast<float*>(scratch);
    g.amax_idx = reinterpret_cast<int*>(g.amax_val + (size_t)M * (N / 64));
    if (int rc = op_gemm(g, variant, (cudaStream_t)stream)) return rc;
    fa::launch_argmax_reduce(g.amax_val, g.amax_idx, M, N / 64, next, nullptr, nullptr, (cudaStream_t)stream);
    OP_CK(cudaGetLastError());
    return FA_OK;
}

// Q8_0 planes (the decoder's weight form): the same GEMMs reading q / d_t / d_r.
extern "C" size_t fa_op_q8_planes_bytes(int N, int K) {
    if (N <= 0 || K <= 0 || N % 4 || K % 64) return 0;
    return fa::q8p_bytes(N, K);
}

extern "C" int fa_op_repack_q8_planes(const uint8_t* raw, int N, int K, void* planes, void* stream) {
    if (!raw || !planes || N <= 0 || K <= 0 || N % 4 || K % 64)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "need N a multiple of 4 and K of 64");
    if (reinterpret_cast<uintptr_t>(planes) & 255)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "planes must be 256-byte aligned");
    fa::launch_repack_q8_planes(raw, N, K, 0, N, planes, (cudaStream_t)stream);
    OP_CK(cudaGetLastError());
    return FA_OK;
}

static int q8p_args(const void* a16, const void* planes, int M, int N, int K, fa::GemmArgs* g) {
    if (!a16 || !planes || M <= 0 || N <= 0 || K <= 0 || N % 64 || K % 64)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "need N, K multiples of 64");
    if (reinterpret_cast<uintptr_t>(planes) & 255)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "planes must be 256-byte aligned");
    *g = fa::GemmArgs{};
    g->A = reinterpret_cast<const __half*>(a16);
    g->W8 = fa::q8p_view(planes, N, K);
    g->M = M; g->N = N; g->K = K;
    return FA_OK;
}

extern "C" int fa_op_q8p_gemm(const uint16_t* a16, const uint16_t* a16_lo, int M, int K, const void* planes, int N,
                              int n_split, float* c, int variant, void* stream) {
    fa::GemmArgs g;
    if (int rc = q8p_args(a16, planes, M, N, K, &g)) return rc;
    if (!c || n_split <= 0 || (K / 64) % n_split)
        return set_err(nullptr, FA_ERR_INVALID_ARG, "need an output and n_split dividing K/64");
    if (int rc = ensure_configured()) return rc;
    g.A_lo = reinterpret_cast<const __half*>(a16_lo);
    g.n_split = n_split; g.epilogue = fa::kEpiStoreF32; g.C = c;
    return op_gemm(g, variant, (cudaStream_t)stream);
}

extern "C" int fa_op_q8p_gemm_swiglu(const uint16_t* a16, const uint16_t* a16_lo, int M, int K, const void* planes,
                                     int N, uint16_t* h16, uint16_t* h_lo, void* stream) {
    fa::GemmArgs g;
    if (int rc = q8p_args(a16, planes, M, N, K, &g)) return rc;
    if (!h16) return set_err(nullptr, FA_ERR_INVALID_ARG, "h16 is NULL");
    if (int rc = ensure_configured()) return rc;
    g.A_lo = reinterpret_cast<const __half*>(a16_lo);
    g.n_split = 1; g.epilogue = fa::kEpiSwiglu;
    g.H = reinterpret_cast<__half*>(h16); g.H_lo = reinterpret_cast<__half*>(h_lo);
    if (!fa::launch_q8_gemv(g, (cudaStream_t)stream))
        return set_err(nullptr, FA_ERR_INVALID_ARG, "shape outside the small-M kernel");
    OP_CK(cudaGetLastError());
    return FA_OK;
}

extern "C" int fa_op_q8p_gemm_argmax(const uint16_t* a16, const uint16_t* a16_lo, int M, int K, const void* planes,
                                     int N, void* scratch, int* next, float* logits, int variant, void* stream) {
    fa::GemmArgs g;
    if (int rc = q8p_args(a16, planes, M, N, K, &g)) return rc;
    if (!scratch || !next) return set_err(nullptr, FA_ERR_INVALID_ARG, "bad arguments");
    if (int rc = ensure_configured()) return rc;
    g.A_lo = reinterpret_cast<const __half*>(a16_lo);
    g.n_split = 1; g.epilogue = fa::kEpiArgmax; g.C = logits;
    g.amax_val = reinterpret_cast<float*>(scratch);
    g.amax_idx = reinterpret_cast<int*>(g.amax_val + (size_t)M * (N / 64));
    if (int rc = op_gemm(g, variant, (cudaStream_t)stream)) return rc;
    fa::launch_argmax_reduce(g.amax_val, g.amax_idx, M, N / 64, next, nullptr, nullptr, (cudaStream_t)stream);
    OP_CK(cudaGetLastError());
    return FA_OK;
}

// ------------------------------------------------------- host allocator --
struct fa_palloc {
    fa::PageAllocator a;
};

extern "C" fa_palloc* fa_palloc_create(int n_pages) {
    if (n_pages <= 0) {
        set_err(nullptr, FA_ERR_INVALID_ARG, "n_pages must be positive");
        return nullptr;
    }
    fa_palloc* p = new fa_palloc();
    p->a.init(n_pages);
    return p;
}

extern "C" void fa_palloc_destroy(fa_palloc* pa) { delete pa; }

extern "C" int fa_palloc_alloc(fa_palloc* pa) {
    if (!pa) return set_err(nullptr, FA_ERR_INVALID_ARG, "NULL allocator");
    const int p = pa->a.alloc();
    if (p < 0) return set_err(nullptr, FA_ERR_POOL_EXHAUSTED, "page pool exhausted");
    return p;
}

extern "C" int fa_palloc_free(fa_palloc* pa, int page) {
    if (!pa) return set_err(nullptr, FA_ERR_INVALID_ARG, "NULL allocator");
    if (!pa->a.release(page)) return set_err(nullptr, FA_ERR_INVALID_ARG, "page out of range or already free");
    return FA_OK;
}

extern "C" int fa_palloc_n_free(const fa_palloc* pa) { return pa ? pa->a.n_free() : FA_ERR_INVALID_ARG; }

extern "C" int fa_palloc_compact(fa_palloc* pa, int* src, int* dst, int max_moves, int* n_moves) {
    if (!pa) return set_err(nullptr, FA_ERR_INVALID_ARG, "NULL allocator");
    std::vector<int> s, d;
    pa->a.compact(s, d);
    if (n_moves) *n_moves = (int)s.size();
    for (int i = 0; i < (int)s.size() && i < max_moves; ++i) {
        if (src) src[i] = s[i];
        if (dst) dst[i] = d[i];
    }
    return (int)s.size() <= max_moves || (!src && !dst) ? FA_OK
                                                        : set_err(nullptr, FA_ERR_CAPACITY, "more moves than max_moves");
}
