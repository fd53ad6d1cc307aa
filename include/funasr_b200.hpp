// funasr_b200.hpp — C++17 host API of the B200 decoder path, over the C ABI of
// funasr_dec.h. Header only; link libfunasr_dec.so.
//
// The classes keep the reference's names, argument meanings and conventions (bool
// results, last_error() strings, n_past bookkeeping) for the decoder's KV-cache path,
// so a caller of the reference switches by changing includes:
//   LLMConfig    core/config.hpp:119-136
//   GPUKVCache   compute/gpu_context.hpp:66-78         n_ctx, n_past, n_layers, kv_dim, initialized
//   GPUContext   compute/gpu_context.hpp:84-181        init, clear_kv_cache, kv_cache, config, cleanup
//   GPURunner    compute/gpu_runner.hpp:22-236         warmup, forward, argmax, is_warmed_up
//   KVCache      compute/kv_cache.hpp:25-168           init, clear, free, n_past, n_ctx, n_layers,
//                                                      kv_dim, is_initialized, set_n_past
//   GPUEncoderAdaptorRunner compute/encoder_adaptor_gpu.hpp:27-191  init, forward_on_gpu
// Deviations, all forced by ggml's absence or by the paged cache:
//   - weights come as GGUF tensor views or a GGUF file path instead of LLMWeights
//     (ggml_tensor pointers);
//   - KVCache::k_tensor()/v_tensor() (ggml views of the f32 cache) become
//     read_layer(), which returns the f16 cache of one layer as [n_past][kv_dim];
//   - GPURunner::forward_tokens() adds the embedding lookup on the device.
// BatchDecoder and Scheduler are new: many sequences on one GPU, one batched step for
// all of them (Scheduler adds admission, prompt chunking and page release).
//
// Not thread-safe per GPUContext; use one host thread per GPU, as the reference does.
#ifndef FUNASR_B200_HPP
#define FUNASR_B200_HPP

#include "funasr_dec.h"

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

namespace funasr_b200 {

struct LLMConfig {
    int block_count = 28;
    int embedding_length = 1024;
    int context_length = 40960;
    int feed_forward_length = 3072;
    int head_count = 16;
    int head_count_kv = 8;
    int key_length = 128;
    int value_length = 128;
    float rope_freq_base = 1000000.0f;
    int vocab_size = 151936;

    int head_dim() const { return key_length; }
    int q_dim() const { return head_count * head_dim(); }
    int kv_dim() const { return head_count_kv * head_dim(); }
    int gqa_groups() const { return head_count / head_count_kv; }
};

// Geometry of a descriptor from any struct with LLMConfig's field names (this one or
// the reference's own).
template <typename Cfg>
inline void apply_config(const Cfg& cfg, fa_model_desc& d) {
    d.n_layers = cfg.block_count;
    d.hidden = cfg.embedding_length;
    d.n_heads = cfg.head_count;
    d.n_kv_heads = cfg.head_count_kv;
    d.head_dim = cfg.key_length;
    d.ffn = cfg.feed_forward_length;
    d.vocab = cfg.vocab_size;
    d.rope_base = cfg.rope_freq_base;
    d.max_ctx = cfg.context_length;
}

inline LLMConfig config_of(const fa_model_desc& d) {
    LLMConfig c;
    c.block_count = d.n_layers;
    c.embedding_length = d.hidden;
    c.head_count = d.n_heads;
    c.head_count_kv = d.n_kv_heads;
    c.key_length = c.value_length = d.head_dim;
    c.feed_forward_length = d.ffn;
    c.vocab_size = d.vocab;
    c.rope_freq_base = d.rope_base;
    c.context_length = d.max_ctx;
    return c;
}

struct GPUKVCache {
    int n_ctx = 0;
    int n_past = 0;
    int n_layers = 0;
    int kv_dim = 0;
    bool initialized = false;
};

// Runtime sizes that the reference's single-sequence cache did not need.
struct PoolOptions {
    int max_seqs = 1;        // sequence slots (GPUContext's own sequence included)
    int max_rows = 512;      // tokens per forward call (prefill chunk / decode batch)
    int n_pages = 0;         // 0: enough for max_seqs sequences of n_ctx tokens
    size_t kv_bytes = 0;     // pool budget instead of n_pages
};

class GPUContext {
public:
    GPUContext() = default;
    ~GPUContext() { cleanup(); }
    GPUContext(const GPUContext&) = delete;
    GPUContext& operator=(const GPUContext&) = delete;

    // GPUContext::init(const LLMWeights&, const LLMConfig&, n_ctx, gpu_id) with the
    // weights as GGUF tensor views (names of model/loader.cpp, host memory).
    template <typename Cfg>
    bool init(const std::vector<fa_tensor_view>& weights, const Cfg& cfg, int n_ctx = 2048, int gpu_id = 0,
              const PoolOptions& opt = PoolOptions()) {
        fa_model_desc d;
        fa_default_desc(&d);
        apply_config(cfg, d);
        if (!create(d, n_ctx, gpu_id, opt)) return false;
        if (fa_load_weights(ctx_, weights.data(), (int)weights.size()) != FA_OK) return fail(fa_last_error(ctx_));
        return open_own_sequence(n_ctx);
    }

    // The model-file path (Recognizer::init + init_gpu): geometry and decoder tensors
    // from a GGUF file.
    bool init(const std::string& gguf_path, int n_ctx = 2048, int gpu_id = 0,
              const PoolOptions& opt = PoolOptions()) {
        fa_model_desc d;
        fa_default_desc(&d);
        if (fa_gguf_read_desc(gguf_path.c_str(), &d) != FA_OK) return fail(fa_last_error(nullptr));
        if (!create(d, n_ctx, gpu_id, opt)) return false;
        if (fa_load_gguf(ctx_, gguf_path.c_str()) != FA_OK) return fail(fa_last_error(ctx_));
        return open_own_sequence(n_ctx);
    }

    // Every utterance starts here: the cache is emptied (its pages go back to the pool).
    void clear_kv_cache() {
        if (!kv_cache_.initialized) return;
        fa_seq_truncate(ctx_, seq_, 0);
        kv_cache_.n_past = 0;
    }

    void cleanup() {
        if (ctx_) fa_destroy(ctx_);
        ctx_ = nullptr;
        seq_ = -1;
        kv_cache_ = GPUKVCache();
        initialized_ = false;
    }

    bool is_initialized() const { return initialized_; }
    GPUKVCache& kv_cache() { return kv_cache_; }
    const GPUKVCache& kv_cache() const { return kv_cache_; }
    const LLMConfig& config() const { return cfg_; }
    const std::string& last_error() const { return err_; }

    fa_ctx* handle() const { return ctx_; }
    int seq() const { return seq_; }       // the sequence behind kv_cache()
    int gpu_id() const { return gpu_id_; }

private:
    bool fail(const std::string& m) {
        err_ = m;
        return false;
    }

    bool create(fa_model_desc d, int n_ctx, int gpu_id, const PoolOptions& opt) {
        cleanup();
        if (n_ctx <= 0) return fail("n_ctx must be > 0");
        if (d.max_ctx < n_ctx) d.max_ctx = n_ctx;
        d.max_seqs = opt.max_seqs;
        d.max_rows = opt.max_rows;
        d.n_pages = opt.n_pages;
        d.kv_bytes = opt.kv_bytes;
        if (!d.n_pages && !d.kv_bytes) d.n_pages = opt.max_seqs * ((n_ctx + FA_PAGE_TOKENS - 1) / FA_PAGE_TOKENS + 1);
        ctx_ = fa_create(gpu_id, &d);
        if (!ctx_) return fail(fa_last_error(nullptr));
        cfg_ = config_of(d);
        gpu_id_ = gpu_id;
        return true;
    }

    bool open_own_sequence(int n_ctx) {
        if (fa_seq_open(ctx_, n_ctx, &seq_) != FA_OK) return fail(fa_last_error(ctx_));
        kv_cache_.n_ctx = n_ctx;
        kv_cache_.n_past = 0;
        kv_cache_.n_layers = cfg_.block_count;
        kv_cache_.kv_dim = cfg_.kv_dim();
        kv_cache_.initialized = true;
        initialized_ = true;
        return true;
    }

    fa_ctx* ctx_ = nullptr;
    int seq_ = -1;
    int gpu_id_ = 0;
    bool initialized_ = false;
    LLMConfig cfg_;
    GPUKVCache kv_cache_;
    std::string err_;
};

class GPURunner {
public:
    explicit GPURunner(GPUContext& ctx) : gpu_ctx_(ctx) {}
    GPURunner(const GPURunner&) = delete;
    GPURunner& operator=(const GPURunner&) = delete;

    // Runs one prefill of max_prefill_len rows and one decode step on dummy input so
    // that the step plans and CUDA graphs of both shapes exist, then empties the cache.
    bool warmup(int max_prefill_len = 500, int max_past = 2048) {
        const GPUKVCache& kv = gpu_ctx_.kv_cache();
        const int n = std::min(max_prefill_len, std::min(max_past, kv.n_ctx - 1));
        if (n < 1) return fail("warmup: cache too small");
        std::vector<float> embeds((size_t)n * gpu_ctx_.config().embedding_length, 0.0f);
        std::vector<float> logits;
        if (!forward(embeds.data(), n, 0, logits) || !forward(embeds.data(), 1, n, logits)) return false;
        gpu_ctx_.clear_kv_cache();
        warmed_up_ = true;
        return true;
    }

    // Appends seq_len rows of input embeddings ([seq_len][embedding_length] f32) at
    // positions n_past.. and returns the last row's logits. n_past below the cached
    // length rewinds the cache first (as the reference's position argument does).
    bool forward(const float* input_embeds, int seq_len, int n_past, std::vector<float>& logits_out) {
        if (!input_embeds || seq_len <= 0) return fail("forward: no input");
        if (!rewind(n_past)) return false;
        logits_out.resize((size_t)gpu_ctx_.config().vocab_size);
        if (fa_prefill(gpu_ctx_.handle(), gpu_ctx_.seq(), input_embeds, seq_len, &next_id_, logits_out.data()) !=
            FA_OK)
            return fail(fa_last_error(gpu_ctx_.handle()));
        gpu_ctx_.kv_cache().n_past = n_past + seq_len;
        return true;
    }

    // forward() with token ids: the embedding rows are gathered on the device.
    bool forward_tokens(const int* token_ids, int seq_len, int n_past, std::vector<float>& logits_out) {
        if (!token_ids || seq_len <= 0) return fail("forward_tokens: no input");
        if (!rewind(n_past)) return false;
        const GPUContext& c = gpu_ctx_;
        logits_out.resize((size_t)seq_len * c.config().vocab_size);
        std::vector<int> seqs((size_t)seq_len, c.seq()), next((size_t)seq_len);
        if (fa_forward(c.handle(), seq_len, seqs.data(), token_ids, nullptr, next.data(), logits_out.data()) != FA_OK)
            return fail(fa_last_error(c.handle()));
        logits_out.erase(logits_out.begin(), logits_out.end() - c.config().vocab_size);
        next_id_ = next.back();
        gpu_ctx_.kv_cache().n_past = n_past + seq_len;
        return true;
    }

    // First index of the maximum (compute/gpu_runner.hpp:108-118).
    static int argmax(const std::vector<float>& logits) {
        int best = 0;
        for (size_t i = 1; i < logits.size(); ++i)
            if (logits[i] > logits[(size_t)best]) best = (int)i;
        return best;
    }

    // The argmax of the last forward's last row, computed on the device.
    int last_next_id() const { return next_id_; }
    bool is_warmed_up() const { return warmed_up_; }
    const std::string& last_error() const { return err_; }

private:
    bool fail(const std::string& m) {
        err_ = m;
        std::printf("[GPURunner] %s\n", m.c_str());
        return false;
    }

    bool rewind(int n_past) {
        int len = 0;
        if (fa_seq_length(gpu_ctx_.handle(), gpu_ctx_.seq(), &len) != FA_OK)
            return fail(fa_last_error(gpu_ctx_.handle()));
        if (n_past < 0 || n_past > len)
            return fail("n_past " + std::to_string(n_past) + " outside the cached 0.." + std::to_string(len));
        if (n_past < len && fa_seq_truncate(gpu_ctx_.handle(), gpu_ctx_.seq(), n_past) != FA_OK)
            return fail(fa_last_error(gpu_ctx_.handle()));
        return true;
    }

    GPUContext& gpu_ctx_;
    bool warmed_up_ = false;
    int next_id_ = -1;
    std::string err_;
};

// The CPU KVCache's interface (compute/kv_cache.hpp) over one paged sequence of a
// GPUContext: a second utterance stream next to the context's own.
// IEEE binary32 -> binary16 bits, round to nearest, ties to even (the cast the cache
// applies to every K/V value), with overflow to infinity and gradual underflow.
inline uint16_t f32_to_f16_bits(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));   // inf, nan
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);                                        // rounds past max
    if (ax < 0x38800000u) {                                                                          // f16 subnormal
        if (ax < 0x33000000u) return (uint16_t)sign;                                                  // below half the least
        const int shift = 126 - (int)(ax >> 23);             // 14 ... 24
        const uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        uint32_t r = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1u))) ++r;
        return (uint16_t)(sign | r);
    }
    uint32_t r = ((ax - 0x38000000u) >> 13);                 // rebias exponent, keep 10 mantissa bits
    const uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;    // may carry into the exponent: still correct
    return (uint16_t)(sign | r);
}

// What k_tensor() / v_tensor() return. The reference hands out ggml tensors of its
// contiguous f32 cache; ggml is absent here and the cache lives in device pages, so this
// is a handle on one sequence's K (or V) pages: read(layer) copies a layer out as the
// reference laid it out, [n_past][kv_dim] (f16 bits).
class KVCache;
struct KVTensorView {
    const KVCache* cache = nullptr;
    bool is_v = false;
    bool read(int layer, std::vector<uint16_t>& out) const;
};

class KVCache {
public:
    KVCache() = default;
    ~KVCache() { free(); }
    KVCache(const KVCache&) = delete;
    KVCache& operator=(const KVCache&) = delete;

    bool init(GPUContext& ctx, int n_ctx) {
        free();
        if (!ctx.is_initialized() || fa_seq_open(ctx.handle(), n_ctx, &seq_) != FA_OK) return false;
        ctx_ = &ctx;
        n_ctx_ = n_ctx;
        return true;
    }
    void clear() {
        if (ctx_) fa_seq_truncate(ctx_->handle(), seq_, 0);
        pending_.assign(pending_.size(), Pending{});
    }
    void free() {
        if (ctx_) fa_seq_close(ctx_->handle(), seq_);
        pending_.clear();
        ctx_ = nullptr;
        seq_ = -1;
    }
    int n_past() const {
        int n = 0;
        if (ctx_) fa_seq_length(ctx_->handle(), seq_, &n);
        return n;
    }
    int n_ctx() const { return n_ctx_; }
    int n_layers() const { return ctx_ ? ctx_->config().block_count : 0; }
    int kv_dim() const { return ctx_ ? ctx_->config().kv_dim() : 0; }
    bool is_initialized() const { return ctx_ != nullptr; }
    // Rewinds only: positions past the cached length were never written.
    void set_n_past(int n) {
        if (ctx_ && n >= 0 && n <= n_past()) fa_seq_truncate(ctx_->handle(), seq_, n);
    }
    int seq_id() const { return seq_; }

    // The step's K and V of one layer as the reference's forward hands them over
    // (compute/kv_cache.hpp:68-74): host f32 [seq_len][kv_dim], held until commit().
    void set_pending(int layer, const float* k, const float* v) {
        if (layer < 0 || layer >= n_layers()) return;
        if ((int)pending_.size() < n_layers()) pending_.resize((size_t)n_layers());
        pending_[(size_t)layer] = {k, v};
    }
    // Writes the pending K/V of every layer at positions [n_past, n_past + seq_len)
    // (compute/kv_cache.hpp:80-97) and drops the pending pointers: each value cast to
    // f16 (round to nearest even) into the sequence's pages. The cache must hold at least
    // n_past tokens; later ones are dropped first (the pages are appended in order). A
    // layer with nothing pending gets zeros there, the value the reference's cleared cache
    // holds. False when the context reports an error (fa_last_error).
    bool commit(int n_past, int seq_len) {
        if (!ctx_ || seq_len <= 0 || n_past < 0 || n_past > this->n_past()) return false;
        if (n_past < this->n_past() && fa_seq_truncate(ctx_->handle(), seq_, n_past) != FA_OK) return false;
        const int L = n_layers(), kvd = kv_dim();
        std::vector<uint16_t> k((size_t)seq_len * L * kvd, 0), v((size_t)seq_len * L * kvd, 0);
        for (int l = 0; l < L && l < (int)pending_.size(); ++l) {
            const Pending& p = pending_[(size_t)l];
            if (!p.k || !p.v) continue;
            for (int t = 0; t < seq_len; ++t)
                for (int i = 0; i < kvd; ++i) {
                    const size_t o = ((size_t)t * L + l) * kvd + i;
                    k[o] = f32_to_f16_bits(p.k[(size_t)t * kvd + i]);
                    v[o] = f32_to_f16_bits(p.v[(size_t)t * kvd + i]);
                }
        }
        pending_.assign(pending_.size(), Pending{});
        const std::vector<int> rows((size_t)seq_len, seq_);
        return fa_kv_append(ctx_->handle(), seq_len, rows.data(), k.data(), v.data()) == FA_OK;
    }
    // The reference's tensor accessors (compute/kv_cache.hpp:146-147), as device views.
    KVTensorView k_tensor() const { return {this, false}; }
    KVTensorView v_tensor() const { return {this, true}; }

    std::vector<int> block_table() const {
        std::vector<int> pages;
        int n = 0;
        if (!ctx_ || fa_seq_block_table(ctx_->handle(), seq_, nullptr, 0, &n) != FA_OK) return pages;
        pages.resize((size_t)n);
        fa_seq_block_table(ctx_->handle(), seq_, pages.data(), n, &n);
        return pages;
    }

    // The layer's cache as the reference laid it out, [n_past][kv_dim] (f16 bits here,
    // f32 there): k[pos][h * head_dim + i].
    bool read_layer(int layer, std::vector<uint16_t>& k, std::vector<uint16_t>& v) const {
        if (!ctx_) return false;
        return read_sequence_layer(*ctx_, seq_, n_past(), layer, k, v);
    }

    static bool read_sequence_layer(const GPUContext& ctx, int seq, int n_tok, int layer, std::vector<uint16_t>& k,
                                    std::vector<uint16_t>& v) {
        const int hd = ctx.config().head_dim(), hk = ctx.config().head_count_kv, kvd = hk * hd;
        int n_pages = 0;
        if (fa_seq_block_table(ctx.handle(), seq, nullptr, 0, &n_pages) != FA_OK) return false;
        std::vector<int> pages((size_t)n_pages);
        if (fa_seq_block_table(ctx.handle(), seq, pages.data(), n_pages, &n_pages) != FA_OK) return false;
        const size_t page_elems = (size_t)hk * 2 * FA_PAGE_TOKENS * hd;
        std::vector<uint16_t> raw(page_elems * (size_t)n_pages);
        if (n_pages && fa_kv_read_pages(ctx.handle(), layer, pages.data(), n_pages, raw.data()) != FA_OK) return false;
        k.assign((size_t)n_tok * kvd, 0);
        v.assign((size_t)n_tok * kvd, 0);
        for (int p = 0; p < n_tok; ++p) {
            const uint16_t* page = raw.data() + page_elems * (size_t)(p / FA_PAGE_TOKENS);
            const int t = p % FA_PAGE_TOKENS;
            for (int h = 0; h < hk; ++h) {
                const uint16_t* kp = page + ((size_t)(h * 2 + 0) * FA_PAGE_TOKENS + t) * hd;
                const uint16_t* vp = page + ((size_t)(h * 2 + 1) * FA_PAGE_TOKENS + t) * hd;
                std::copy(kp, kp + hd, k.begin() + (size_t)p * kvd + (size_t)h * hd);
                std::copy(vp, vp + hd, v.begin() + (size_t)p * kvd + (size_t)h * hd);
            }
        }
        return true;
    }

private:
    struct Pending {
        const float* k = nullptr;
        const float* v = nullptr;
    };
    GPUContext* ctx_ = nullptr;
    int seq_ = -1;
    int n_ctx_ = 0;
    std::vector<Pending> pending_;
};

inline bool KVTensorView::read(int layer, std::vector<uint16_t>& out) const {
    std::vector<uint16_t> k, v;
    if (!cache || !cache->read_layer(layer, k, v)) return false;
    out = is_v ? std::move(v) : std::move(k);
    return true;
}

// Many utterance streams on one GPU: open a sequence per stream, prefill it, then
// advance every live stream by one greedy token per step() call.
class BatchDecoder {
public:
    explicit BatchDecoder(GPUContext& ctx) : ctx_(ctx) {}

    int open(int max_tokens) {
        int id = -1;
        if (fa_seq_open(ctx_.handle(), max_tokens, &id) != FA_OK) {
            err_ = fa_last_error(ctx_.handle());
            return -1;
        }
        return id;
    }
    bool close(int seq) { return check(fa_seq_close(ctx_.handle(), seq)); }
    // Prefills embeds [n_tok][embedding_length]; *next_id = greedy token after the last row.
    bool prefill(int seq, const float* embeds, int n_tok, int* next_id) {
        return check(fa_prefill(ctx_.handle(), seq, embeds, n_tok, next_id, nullptr));
    }
    // tokens[i] is appended to seqs[i]; next[i] is its greedy successor.
    bool step(const std::vector<int>& seqs, const std::vector<int>& tokens, std::vector<int>& next) {
        if (seqs.size() != tokens.size()) {
            err_ = "step: seqs and tokens differ in length";
            return false;
        }
        next.resize(seqs.size());
        return check(fa_decode_step(ctx_.handle(), (int)seqs.size(), seqs.data(), tokens.data(), next.data(),
                                    nullptr));
    }
    int free_pages() const {
        int n = 0, f = 0;
        size_t b = 0;
        fa_pool_info(ctx_.handle(), &n, &f, &b);
        return f;
    }
    const std::string& last_error() const { return err_; }

private:
    bool check(int rc) {
        if (rc == FA_OK) return true;
        err_ = fa_last_error(ctx_.handle());
        return false;
    }
    GPUContext& ctx_;
    std::string err_;
};

// The audio encoder + adaptor (compute/encoder_adaptor_gpu.hpp:27-677): LFR features
// [frames][input_dim] -> decoder input embeddings [frames][adaptor_output], kept on the
// device (forward_on_gpu, the reference's name) or copied to the host (forward).
class GPUEncoderAdaptorRunner {
public:
    GPUEncoderAdaptorRunner() = default;
    ~GPUEncoderAdaptorRunner() { release(); }
    GPUEncoderAdaptorRunner(const GPUEncoderAdaptorRunner&) = delete;
    GPUEncoderAdaptorRunner& operator=(const GPUEncoderAdaptorRunner&) = delete;

    // weights: the audio_encoder.* and audio_adaptor.* GGUF tensors (host memory)
    bool init(const std::vector<fa_tensor_view>& weights, int max_frames = 1024, int gpu_id = 0) {
        release();
        fa_encoder_desc d;
        fa_encoder_default_desc(&d);
        d.max_frames = max_frames;
        e_ = fa_encoder_create(gpu_id, &d);
        if (!e_) return fail();
        if (fa_encoder_load_weights(e_, weights.data(), (int)weights.size()) != FA_OK) return fail();
        desc_ = d;
        return true;
    }
    // embeds_dev: frames x adaptor_output f32 on the device (e.g. straight into fa_prefill)
    bool forward_on_gpu(const float* lfr_dev, int input_dim, int frames, float* embeds_dev, int& out_frames) {
        out_frames = 0;
        if (!e_ || input_dim != desc_.input_dim) return false;
        if (fa_encoder_forward_dev(e_, lfr_dev, frames, embeds_dev, nullptr) != FA_OK) return fail();
        out_frames = frames;
        return true;
    }
    bool forward(const float* lfr, int input_dim, int frames, std::vector<float>& embeds) {
        if (!e_ || input_dim != desc_.input_dim) return false;
        embeds.resize((size_t)frames * desc_.adaptor_output);
        return fa_encoder_forward(e_, lfr, frames, embeds.data()) == FA_OK || fail();
    }
    int output_dim() const { return desc_.adaptor_output; }
    const std::string& last_error() const { return err_; }

private:
    bool fail() {
        err_ = fa_last_error(nullptr);
        return false;
    }
    void release() {
        if (e_) fa_encoder_destroy(e_);
        e_ = nullptr;
    }
    fa_encoder* e_ = nullptr;
    fa_encoder_desc desc_{};
    std::string err_;
};

// Continuous batching over a GPUContext's sequence slots and page pool (fa_sched_*):
// streams are submitted with a prompt and a token budget; each step() runs one batched
// forward and returns the tokens it produced as (tag, token, finished) events.
class Scheduler {
public:
    struct Config {
        int max_batch_rows = 512;
        int prefill_chunk = 512;
        int max_running = 256;
        int eos_id = 151645;   // tokenizer.ggml.eos_token_id of the FunASR model; -1: none
    };

    Scheduler(GPUContext& ctx, const Config& cfg) : ctx_(ctx) {
        fa_sched_config c{cfg.max_batch_rows, cfg.prefill_chunk, cfg.max_running, cfg.eos_id};
        s_ = fa_sched_create(ctx.handle(), &c);
        if (!s_) err_ = fa_last_error(nullptr);
    }
    ~Scheduler() {
        if (s_) fa_sched_destroy(s_);
    }
    Scheduler(const Scheduler&) = delete;
    Scheduler& operator=(const Scheduler&) = delete;

    bool ok() const { return s_ != nullptr; }
    bool submit_tokens(int64_t tag, const std::vector<int>& ids, int max_new) {
        return check(fa_sched_submit(s_, tag, ids.data(), nullptr, (int)ids.size(), max_new));
    }
    // embeds: n_prompt rows of embedding_length f32 (e.g. the adaptor's output)
    bool submit_embeds(int64_t tag, const float* embeds, int n_prompt, int max_new) {
        return check(fa_sched_submit(s_, tag, nullptr, embeds, n_prompt, max_new));
    }
    bool step(std::vector<fa_sched_event>& events, int max_events = 4096) {
        events.resize((size_t)max_events);
        int n = 0;
        if (!check(fa_sched_step(s_, events.data(), max_events, &n))) {
            events.clear();
            return false;
        }
        events.resize((size_t)n);
        return true;
    }
    bool idle() const { return fa_sched_idle(s_) == 1; }
    fa_sched_stats stats() const {
        fa_sched_stats st{};
        fa_sched_get_stats(s_, &st);
        return st;
    }
    const std::string& last_error() const { return err_; }

private:
    bool check(int rc) {
        if (rc == FA_OK) return true;
        err_ = fa_last_error(ctx_.handle());
        return false;
    }
    GPUContext& ctx_;
    fa_sched* s_ = nullptr;
    std::string err_;
};

}  // namespace funasr_b200

#endif  // FUNASR_B200_HPP
