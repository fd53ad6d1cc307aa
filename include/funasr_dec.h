/* funasr_dec.h — C ABI of the B200 (sm_100a) FunASR LLM-decoder hot path.
 *
 * The library replaces the reference's decoder KV-cache path:
 *   compute/kv_cache.hpp                 KVCache (f32 [layer][pos][1024], one sequence)
 *   compute/gpu_context.hpp:66-78,98-122,220-349
 *                                        GPUKVCache, weight upload, KV alloc/clear
 *   compute/llm_ops_gpu.cpp:34-207       Qwen3 decoder graph (ggml-cuda)
 *   compute/gpu_runner.hpp:44-236        warmup / forward / argmax
 *   pipeline/pipeline.cpp:434-451        greedy decode loop
 * with a paged f16 KV cache shared by many sequences, batched forwards over
 * rows (one row = one token of one sequence) and hand-written CUDA kernels.
 *
 * Conventions
 *   - Every call returns FA_OK (0) or a negative FA_ERR_* code; the message of the
 *     last failure is fa_last_error(ctx) (fa_last_error(NULL) for calls without a
 *     context). There is no CPU fallback: without a usable GPU, fa_create fails.
 *   - Host pointers unless the name says _dev. Shapes are row-major C arrays.
 *   - One fa_ctx per GPU. A context is not thread-safe; use one host thread per
 *     context (the reference also drives one GPURunner from one thread).
 *   - Model geometry fixed by the kernels: head_dim 128, 16 query heads, 8 KV heads
 *     (Qwen3-0.6B as used by FunASR-Nano). n_layers, hidden, ffn, vocab are free
 *     (hidden, ffn, vocab multiples of 64).
 */
#ifndef FUNASR_DEC_H
#define FUNASR_DEC_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FA_API __attribute__((visibility("default")))
#else
#define FA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FA_OK 0
#define FA_ERR_INVALID_ARG (-1)
#define FA_ERR_CUDA (-2)
#define FA_ERR_OOM (-3)            /* device allocation failed */
#define FA_ERR_POOL_EXHAUSTED (-4) /* no free KV page; nothing of the call was applied */
#define FA_ERR_SEQ (-5)            /* unknown / closed sequence, or no free slot */
#define FA_ERR_CAPACITY (-6)       /* beyond max_rows, a sequence's max_tokens or max_ctx */
#define FA_ERR_WEIGHTS (-7)        /* missing tensor, wrong type or shape */
#define FA_ERR_TIMEOUT (-8)        /* a bounded device wait gave up */
#define FA_ERR_NOT_READY (-9)      /* weights not loaded */
#define FA_ERR_DEVICE (-10)        /* a kernel reported a bad page / position / token */

#define FA_PAGE_TOKENS 16

/* GGML tensor type ids accepted in fa_tensor_view.type. */
#define FA_TYPE_F32 0
#define FA_TYPE_F16 1
#define FA_TYPE_Q8_0 8
#define FA_TYPE_BF16 30

/* Decoder geometry and runtime sizes. Mirrors LLMConfig (core/config.hpp:119-136)
 * plus the cache sizing that replaces n_ctx (compute/gpu_context.hpp:315-349). */
typedef struct fa_model_desc {
    int n_layers;    /* block_count, 28 */
    int hidden;      /* embedding_length, 1024 */
    int n_heads;     /* head_count, 16 */
    int n_kv_heads;  /* head_count_kv, 8 */
    int head_dim;    /* key_length, 128 */
    int ffn;         /* feed_forward_length, 3072 */
    int vocab;       /* vocab_size, 151936 */
    float rope_base; /* rope_freq_base, 1e6 */
    float rms_eps;   /* 1e-5 (compute/llm_ops_gpu.cpp:50) */
    int max_ctx;     /* longest sequence (RoPE table length), e.g. 40960 */
    int n_pages;     /* KV page pool size; 0 = derive from kv_bytes */
    size_t kv_bytes; /* pool budget in bytes when n_pages == 0 */
    int max_seqs;    /* sequence slots */
    int max_rows;    /* rows (tokens) per forward call: decode batch + prefill chunk */
} fa_model_desc;

/* One tensor in GGUF naming and ggml order: ne[0] is the input (fastest) dim.
 * Replaces the host->device copies of GPUContext::load_weights
 * (compute/gpu_context.hpp:220-310); names as model/loader.cpp:91-117,217-227. */
typedef struct fa_tensor_view {
    const char* name;
    int type;          /* FA_TYPE_* */
    int64_t ne[2];     /* ne[1] = 1 for vectors */
    const void* data;  /* host memory in GGUF layout (Q8_0: rows of [f16 d][32 x int8]) */
    size_t nbytes;
} fa_tensor_view;

typedef struct fa_ctx fa_ctx;

/* Qwen3-0.6B decoder of FunASR-Nano with n_ctx 2048-style defaults. */
FA_API void fa_default_desc(fa_model_desc* desc);

/* ---- context: GPUContext::init / cleanup (compute/gpu_context.hpp:98-169) ---- */
FA_API fa_ctx* fa_create(int device, const fa_model_desc* desc); /* NULL on failure: fa_last_error(NULL) */
FA_API void fa_destroy(fa_ctx* ctx);
FA_API const char* fa_last_error(const fa_ctx* ctx);
FA_API int fa_load_weights(fa_ctx* ctx, const fa_tensor_view* tensors, int n);
/* ---- GGUF model files (decoder part of core/gguf_reader.hpp, ModelConfig::load_from_gguf
 *      core/config.hpp:191-228 and ModelLoader::load_llm model/loader.cpp:91-117,210-227) ---- */
/* Fill the geometry fields of *desc (n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn,
 * vocab, rope_base, max_ctx) from a GGUF file's FunAsr.* keys; the runtime sizes (pages,
 * sequences, rows) are left as they were. Host only. vocab comes from llm.lm_head.weight
 * (151936 when the file has none, as the reference fixes it). */
FA_API int fa_gguf_read_desc(const char* path, fa_model_desc* desc);
/* Where a tensor sits in a GGUF file: ggml type, ne[0] and the product of the other
 * dims, byte offset from the start of the file, bytes (0 for types the decoder does not
 * take). Host only. */
FA_API int fa_gguf_find_tensor(const char* path, const char* name, int* type, int64_t* ne, size_t* file_offset,
                               size_t* nbytes);
/* Map a GGUF file and load its llm.* tensors as fa_load_weights does. */
FA_API int fa_load_gguf(fa_ctx* ctx, const char* path);
/* Run the library's work on `cuda_stream` (a cudaStream_t of this device); NULL restores
 * the library's own stream. */
FA_API int fa_set_stream(fa_ctx* ctx, void* cuda_stream);
/* GEMM implementation: 0 = default: the CUDA-core small-M kernel for steps of up to 2
 * rows, the tcgen05 kernel with swapped operands (weights on the MMA's 128-row side,
 * expanded from Q8_0 into TMEM) above, in 128-row activation tiles; 1 = mma.sync kernel
 * (same arithmetic; kept to cross-check); 2 = the 128-row-tile tcgen05 kernel at every M;
 * 3 = the small-M kernel up to 8 rows, else as 2; 4 = the swapped tcgen05 kernel at every
 * M. */
FA_API int fa_set_gemm_variant(fa_ctx* ctx, int variant);
/* Which ops of a step finish inside the kernel before them (a mask): bit 0 = the QKV
 * projection of steps of up to 128 rows on the swapped tcgen05 kernel finishes kernel (1)
 * (per-head norm, RoPE, K/V append) in clusters of its split-K CTAs; bit 1 = the gate/up
 * projection finishes SwiGLU the same way; bit 2 = decode attention with several splits
 * per row merges them in the attention kernel (the split that finishes last for a row and
 * KV head merges both query heads) instead of a merge launch; bit 3 = steps of decode rows
 * of distinct sequences whose attention CTAs fit in one wave run kernel (1) inside the
 * attention kernel (every split computes its KV head's query heads, the split holding the
 * token's page appends K and V). Default
 * 14; 0 = separate
 * kernels. The results are the same bits either way. No counterpart in the reference
 * (ggml runs each node separately, compute/llm_ops_gpu.cpp:53-96,135-143,177-180). */
FA_API int fa_set_fused_epilogues(fa_ctx* ctx, int mask);
/* 1 = programmatic dependent launch between a step's kernels (default): each kernel's
 * prologue overlaps the previous kernel's tail. 0 = plain stream order. */
FA_API int fa_set_pdl(fa_ctx* ctx, int enable);
/* 1 (default) = a step of one decode row (one sequence, one token) runs as one persistent
 * kernel over every SM (embedding, all layers, final norm; a layer's phases hand their
 * values on as tagged words that the next phase polls) followed by the lm_head and argmax
 * launches, when the model's shapes allow it and
 * the GEMM variant is 0 or 3; 0 = launch by launch. Same bits either way. Replaces the
 * reference's per-token graph launch of compute/llm_ops_gpu.cpp:155-207 for one stream. */
FA_API int fa_set_row_step(fa_ctx* ctx, int enable);
/* Failure test of the one-row step kernel's waits: with absent_cta >= 0 that CTA leaves
 * at once, so the values of its rows never arrive and the other CTAs' waits run out after
 * wait_us microseconds (<= 0: the default 2 s); every CTA then leaves, the step returns
 * FA_ERR_TIMEOUT and the context stays usable. absent_cta = -1 turns it off. No reference
 * counterpart. */
FA_API int fa_set_row_step_fault(fa_ctx* ctx, int absent_cta, int wait_us);
/* 1 = launch each step as a captured CUDA graph (default), 0 = direct launches. */
FA_API int fa_set_graphs(fa_ctx* ctx, int enable);
/* The descriptor the context runs with (n_pages resolved from kv_bytes). */
FA_API int fa_ctx_desc(const fa_ctx* ctx, fa_model_desc* desc);
/* Pool geometry: pages, free pages, bytes of one page across all layers. */
FA_API int fa_pool_info(const fa_ctx* ctx, int* n_pages, int* n_free, size_t* page_bytes_all_layers);

/* ---- sequences: KVCache::init / clear / n_past / set_n_past (compute/kv_cache.hpp:38-151),
 *      GPUContext::clear_kv_cache (compute/gpu_context.hpp:116-122) ---- */
FA_API int fa_seq_open(fa_ctx* ctx, int max_tokens, int* seq_id);
FA_API int fa_seq_close(fa_ctx* ctx, int seq_id);     /* returns the sequence's pages to the pool */
FA_API int fa_seq_length(const fa_ctx* ctx, int seq_id, int* n_tokens);
/* Roll back to n_tokens <= current length (KVCache::set_n_past); whole pages past it are freed. */
FA_API int fa_seq_truncate(fa_ctx* ctx, int seq_id, int n_tokens);
/* Copies up to max_pages entries of the sequence's block table; *n_pages = its page count. */
FA_API int fa_seq_block_table(const fa_ctx* ctx, int seq_id, int* pages, int max_pages, int* n_pages);

/* ---- forward: GPURunner::forward / forward_gpu_tensor (compute/gpu_runner.hpp:82-105,136-236)
 * One call appends one token per row to its sequence and runs the decoder over all rows.
 * Rows of one sequence take consecutive positions in row order (chunked prefill);
 * every row's K/V is in the cache before any row's attention, so a prefill chunk is
 * causal within itself. Inputs: token_ids [n_rows] (embedding lookup on the device) or
 * embeds [n_rows][hidden] f32 (audio frames; exactly one of the two), in host or device
 * memory (the encoder's output can be passed as it is).
 * Outputs (optional): next_ids [n_rows] = argmax of each row's logits (first maximum),
 * logits [n_rows][vocab] f32. */
FA_API int fa_forward(fa_ctx* ctx, int n_rows, const int* seq_ids, const int* token_ids, const float* embeds,
               int* next_ids, float* logits);
/* fa_forward returning the outputs of selected rows only: next_ids [n_out] and logits
 * [n_out][vocab] belong to rows out_rows[0..n_out); only those rows go through the final
 * norm and lm_head. n_out = 0: no outputs (a prefill chunk whose last row is not the
 * sequence's last); n_out = -1: all rows, as fa_forward. Token ids and embeddings may
 * be mixed: with both given, a row whose token id is -1 takes its embeds row (a stream's
 * audio frames next to other streams' tokens in one batch). */
FA_API int fa_forward_rows(fa_ctx* ctx, int n_rows, const int* seq_ids, const int* token_ids, const float* embeds,
                           int n_out, const int* out_rows, int* next_ids, float* logits);
/* Prefill n_tok embedding rows of one sequence in chunks of max_rows
 * (pipeline/pipeline.cpp:405 -> GPURunner::forward_gpu_tensor); next_id/last_logits
 * describe the last row. */
FA_API int fa_prefill(fa_ctx* ctx, int seq_id, const float* embeds, int n_tok, int* next_id, float* last_logits);
/* One greedy decode step for n_seq distinct sequences (pipeline/pipeline.cpp:434-451,
 * batched): token_ids[i] is appended to seq_ids[i]. */
FA_API int fa_decode_step(fa_ctx* ctx, int n_seq, const int* seq_ids, const int* token_ids, int* next_ids,
                   float* logits);
/* n_steps greedy steps with the argmax fed back on the device (no host round trip per
 * token; EOS is not checked). out_ids [n_steps][n_seq]. device_ms (optional) = time of the
 * n_steps steps on the device, CUDA events on the library stream, H2D/D2H excluded. */
FA_API int fa_generate(fa_ctx* ctx, int n_seq, const int* seq_ids, const int* first_tokens, int n_steps, int* out_ids,
                float* device_ms);

/* ---- continuous batching: many streams, one forward per step ----
 * New (the reference decodes one utterance at a time, pipeline/pipeline.cpp:434-451).
 * Streams are admitted first come first served when a sequence slot is free and the
 * page pool can hold the whole stream (prompt + max_new tokens), so a running stream
 * never meets an exhausted pool. Each step runs one forward over one decode row per
 * stream past its prompt plus prompt chunks (prefill_chunk rows per stream) of streams
 * still in prefill, up to max_batch_rows; a stream ends after max_new tokens or at
 * eos_id, and its pages return to the pool. The scheduler uses the context's sequence
 * slots and the pages free when it is created. One host thread per scheduler. */
typedef struct fa_sched fa_sched;
typedef struct fa_sched_config {
    int max_batch_rows;  /* rows per forward, <= the context's max_rows */
    int prefill_chunk;   /* prompt rows of one stream per forward */
    int max_running;     /* streams admitted at once, <= max_seqs */
    int eos_id;          /* end-of-sequence id (151645 for Qwen3), -1 to ignore */
} fa_sched_config;
typedef struct fa_sched_event {
    int64_t tag;         /* the stream's tag from fa_sched_submit */
    int token;           /* generated token id; -1 when the stream failed */
    int finished;        /* 1 on the stream's last event */
} fa_sched_event;
typedef struct fa_sched_stats {
    long steps, rows, prompt_rows, tokens, finished;
    int waiting, running;
    long reserved_pages, total_pages;
} fa_sched_stats;
FA_API fa_sched* fa_sched_create(fa_ctx* ctx, const fa_sched_config* cfg);
FA_API void fa_sched_destroy(fa_sched* s);
/* Queue a stream: prompt as token ids or as embedding rows [n_prompt][hidden] (one of the two). */
FA_API int fa_sched_submit(fa_sched* s, int64_t tag, const int* prompt_ids, const float* prompt_embeds, int n_prompt,
                           int max_new);
/* Run one step (when no undelivered events remain) and deliver up to max_events events. */
FA_API int fa_sched_step(fa_sched* s, fa_sched_event* events, int max_events, int* n_events);
/* 1 when no stream is waiting or running and every event was delivered. */
FA_API int fa_sched_idle(const fa_sched* s);
FA_API int fa_sched_get_stats(const fa_sched* s, fa_sched_stats* out);

/* ---- pages ---- */
/* Copy pages of one layer ([n][kv_heads][2][16][head_dim] f16 bit patterns) to the host. */
FA_API int fa_kv_read_pages(fa_ctx* ctx, int layer, const int* pages, int n, uint16_t* out);
/* Append given f16 K/V for all layers: k, v [n_rows][n_layers][kv_heads][head_dim]
 * (the raw-append microbenchmark; positions follow the sequences' lengths). */
FA_API int fa_kv_append(fa_ctx* ctx, int n_rows, const int* seq_ids, const uint16_t* k, const uint16_t* v);
/* Extend a sequence by n_tokens of synthetic cache content (deterministic values in
 * [-2, 2) from seed) without running the model: steady-state decode benchmarks. */
FA_API int fa_kv_fill_synthetic(fa_ctx* ctx, int seq_id, int n_tokens, uint64_t seed);
/* Move live pages down into the lowest free ids (highest live page first) and rewrite
 * the block tables; afterwards the live pages are exactly [0, n_live). */
FA_API int fa_pool_compact(fa_ctx* ctx, int* n_moved);

/* ---- measurement ---- */
/* 1 = bracket the attention launches of layers 0, L/2 and L-1 with CUDA events, or in a
 * one-row step the persistent step kernel (events taken into graphs when captured). */
FA_API int fa_profile(fa_ctx* ctx, int enable);
/* Those attention launches of the last forward/generate step: summed device ms and count
 * (paged-attention kernel plus its split combine); 0 launches after a one-row step. */
FA_API int fa_profile_attention(fa_ctx* ctx, float* total_ms, int* n_launches);
/* Device ms of the persistent step kernel in the last profiled step; 0 when that step was
 * not a one-row step. */
FA_API int fa_profile_row_step(fa_ctx* ctx, float* ms);
/* Kernels launched by the last forward step (all of this library's kernels). */
FA_API int fa_step_launches(const fa_ctx* ctx, int* n_launches);

/* ---- kernel-level entry points (device pointers, caller's stream) ----
 * These are the kernels of one decoder layer, exposed for parity tests and
 * microbenchmarks. `stream` is a cudaStream_t or NULL (legacy default stream). */

/* Kernel (1): per-head Q/K RMSNorm + NEOX RoPE + paged f16 K/V append
 * (compute/llm_ops_gpu.cpp:57-96). qkv_dev [M][(16+2*8)*128] f32; rope_dev
 * [max_pos][64][2] f32 (cos, sin); pool_layer_dev [n_pages][8][2][16][128] f16;
 * q_out_dev [M][16][128] f32 (scaled by 1/sqrt(128)). */
FA_API int fa_op_qknorm_rope_append(const float* qkv_dev, int M, const int* pos_dev, const int* slot_dev,
                             const int* block_table_dev, int bt_stride, int n_pages, const float* q_norm_dev,
                             const float* k_norm_dev, float eps, const float* rope_dev, int max_pos,
                             uint16_t* pool_layer_dev, float* q_out_dev, int* err_dev, void* stream);
/* Raw f16 append for n_layers layers: k/v [M][n_layers][8][128]; pool [n_layers][n_pages][page]. */
FA_API int fa_op_kv_append(const uint16_t* k_dev, const uint16_t* v_dev, int M, int n_layers, const int* pos_dev,
                    const int* slot_dev, const int* block_table_dev, int bt_stride, int n_pages,
                    uint16_t* pool_dev, int* err_dev, void* stream);
/* KV gather (compute/llm_ops_gpu.cpp:97-105: the view of a layer's cache over n_kv
 * tokens, reshaped to [128, 8, n_kv] and made contiguous as [8][n_kv][128]). Copies
 * tokens [0, n_kv[m]) of sequence slot[m] in every layer from the pool into k_out_dev /
 * v_out_dev [n_layers][8][total_rows][128] f16, sequence m at rows [row0[m],
 * row0[m] + n_kv[m]) of each head plane; rows no sequence covers are left as they are.
 * n_kv[m] <= 16 * max_pages. Bad lengths or row ranges set error bit 8, bad pages bit 2. */
FA_API int fa_op_kv_gather(const uint16_t* pool_dev, int n_layers, int n_pages, const int* block_table_dev,
                           int bt_stride, const int* slot_dev, const int* n_kv_dev, const int* row0_dev, int M,
                           int max_pages, int total_rows, uint16_t* k_out_dev, uint16_t* v_out_dev, int* err_dev,
                           void* stream);
/* Kernel (2): paged GQA decode attention (compute/llm_ops_gpu.cpp:98-143). Row m attends
 * to tokens [0, pos[m]] of sequence slot[m]. q [M][16][128] f32 (pre-scaled).
 * Output [M][2048] as f32 and/or as an f16 pair (out16 = f16(o), out16_lo = f16(o - out16),
 * the form the next GEMM reads). scratch_dev holds the split-K partials:
 * fa_op_attention_scratch_bytes(M, n_splits) bytes, 16-byte aligned (may be NULL when
 * n_splits == 1). A row with pos < 0, with more pages than bt_stride, or whose pages
 * pages_per_split * n_splits does not cover sets error bit 8 and is not written; a page
 * id outside [0, n_pages) sets bit 2. */
FA_API size_t fa_op_attention_scratch_bytes(int M, int n_splits);
/* The split for fa_op_paged_attention's CTA form (8 warps for up to 2 rows, else 4) and rows
 * with contexts n_kv[M] on n_sm SMs (host only). */
FA_API int fa_op_attention_plan(const int* n_kv, int M, int n_sm, int* pages_per_split, int* n_splits);
/* The decoder's attention plan for a step of M decode rows with contexts n_kv[M] on n_sm SMs
 * under fused-op mask `mask` (fa_set_fused_epilogues; host only): pages per split, splits,
 * warps per CTA (the cost model picks 4 or 8 up to 64 rows), and in *fused bit 0 whether the
 * attention kernel merges its splits itself, bit 1 whether it runs kernel (1) itself (for
 * rows of distinct sequences, unless the QKV GEMM finishes kernel (1)). Both fusions need the
 * attention CTAs to fit in one wave. No counterpart in the reference (ggml plans nothing of
 * this: compute/llm_ops_gpu.cpp:98-143 builds one attention subgraph per token). */
FA_API int fa_step_attention_plan(const int* n_kv, int M, int n_sm, int mask, int* pages_per_split, int* n_splits,
                                  int* warps, int* fused);
FA_API int fa_op_paged_attention(const float* q_dev, int M, const int* pos_dev, const int* slot_dev,
                          const int* block_table_dev, int bt_stride, int n_pages, const uint16_t* pool_layer_dev,
                          int pages_per_split, int n_splits, void* scratch_dev, uint16_t* out16_dev,
                          uint16_t* out16_lo_dev, float* out32_dev, int* err_dev, void* stream);
/* Kernel (2b): causal attention of prefill tiles on the tensor cores (tcgen05, TMEM,
 * TMA). tiles_dev holds n_tiles pairs (first row, rows) of rows of the q/pos/slot
 * arrays: up to 64 consecutive rows of one sequence with non-decreasing positions;
 * each row m attends to tokens [0, pos[m]] of sequence slot[m]. Output as for
 * fa_op_paged_attention. A bad tile or position sets FA error bit 4 (kernel error
 * word) and that tile writes nothing. q, pool and outputs 16-byte aligned. */
FA_API int fa_op_prefill_attention(const float* q_dev, int M, const int* pos_dev, const int* slot_dev,
                                   const int* block_table_dev, int bt_stride, int n_pages,
                                   const uint16_t* pool_layer_dev, const int* tiles_dev, int n_tiles,
                                   uint16_t* out16_dev, uint16_t* out16_lo_dev, float* out32_dev, int* err_dev,
                                   void* stream);
/* fa_op_paged_attention without the scratch argument: nothing is allocated, by the
 * library or the caller. No counterpart in the reference; it exists for callers that
 * cannot call cudaMalloc (an embedding runtime that owns all device memory, a process
 * that forbids allocation once started). The split-K partials go to one 8 MiB buffer
 * built into the library (held on every GPU that loads it until exit), so
 * M * n_splits <= 1008 (FA_ERR_CAPACITY otherwise). The first call on a device sets
 * the buffer up; make it before any stream capture (and not after a cudaDeviceReset
 * of that device: the cached address belongs to the destroyed context). Calls share
 * the buffer: calls that overlap on the GPU race. Row and page checks as for
 * fa_op_paged_attention. */
FA_API int fa_op_paged_attention_noalloc(const float* q_dev, int M, const int* pos_dev, const int* slot_dev,
                                         const int* block_table_dev, int bt_stride, int n_pages,
                                         const uint16_t* pool_layer_dev, int pages_per_split, int n_splits,
                                         uint16_t* out16_dev, uint16_t* out16_lo_dev, float* out32_dev, int* err_dev,
                                         void* stream);
/* Kernel (4): Q8_0 GEMM C = A . W^T (compute/llm_ops_gpu.cpp:53-55,149,177-180,206).
 * A [M][K] as an f16 pair a16 + a16_lo (a16_lo may be NULL: plain f16 activations).
 * Two weight forms. fa_op_q8p_*: the decoder's, Q8_0 planes built by
 * fa_op_repack_q8_planes from GGUF blocks [N][K/32][34 B] (tools/hf_convert_ggml_q8.py:
 * 354-381): q int8 [N][K], then the block scales twice, f16 [K/32][N] and f16 [N][K/32],
 * in one 256-byte aligned buffer of fa_op_q8_planes_bytes(N, K) bytes (N a multiple of
 * 4, K of 64); every weight is the exact d * q. fa_op_q8_gemm*: W [N][K] f16, e.g.
 * f16(d * q) from fa_op_repack_q8 (the encoder's form).
 * n_split > 1 writes partials [n_split][M][N] (their sum is C).
 * variant: 0 = the small-M CUDA-core kernel when M <= 2 and n_split == 1 (K a multiple of
 * 256), the swapped tcgen05 kernel when M <= 128 (with argmax M <= 32), else the 128-row-
 * tile tcgen05 kernel (N a multiple of 128); 1 = mma.sync kernel; 2 = 128-row-tile tcgen05
 * kernel; 3 = small-M kernel (M <= 8, n_split 1, K a multiple of 256, N of 4; with argmax N
 * of 64 and K <= 1024); 4 = swapped tcgen05 kernel (M <= 128, N a multiple of 128). */
FA_API int fa_op_repack_q8(const uint8_t* gguf_q8_dev, int N, int K, uint16_t* w16_dev, void* stream);
/* The split-K factor the decoder uses for an M x N x K GEMM of `variant` on n_sm SMs (host only). */
FA_API int fa_op_gemm_plan(int M, int N, int K, int variant, int n_sm, int* n_split);
FA_API int fa_op_q8_gemm(const uint16_t* a16_dev, const uint16_t* a16_lo_dev, int M, int K, const uint16_t* w16_dev,
                         int N, int n_split, float* c_dev, int variant, void* stream);
/* Gate/up GEMM with SwiGLU in its epilogue (compute/llm_ops_gpu.cpp:177-180), small-M
 * kernel only (M <= 8, K a multiple of 256): w16 stacks the gate rows [0, N/2) over the up
 * rows [N/2, N); h16 / h_lo [M][N/2] receive the f16 pair of silu(gate) * up. */
FA_API int fa_op_q8_gemm_swiglu(const uint16_t* a16_dev, const uint16_t* a16_lo_dev, int M, int K,
                                const uint16_t* w16_dev, int N, uint16_t* h16_dev, uint16_t* h_lo_dev, void* stream);
/* SwiGLU of split-K partials part [n_part][M][2*ffn] (gate columns then up columns) into the
 * f16 pair h16 / h_lo [M][ffn]: the decoder's separate SwiGLU kernel. */
FA_API int fa_op_swiglu(const float* part_dev, int n_part, int M, int ffn, uint16_t* h16_dev, uint16_t* h_lo_dev,
                        void* stream);
/* lm_head with fused argmax: next [M] = first column of each row's maximum; logits optional. */
FA_API size_t fa_op_argmax_scratch_bytes(int M, int N);
FA_API int fa_op_q8_gemm_argmax(const uint16_t* a16_dev, const uint16_t* a16_lo_dev, int M, int K,
                                const uint16_t* w16_dev, int N, void* scratch_dev, int* next_dev, float* logits_dev,
                                int variant, void* stream);
/* The same three GEMMs on Q8_0 planes (the form the decoder's layers and lm_head use). */
FA_API size_t fa_op_q8_planes_bytes(int N, int K);
FA_API int fa_op_repack_q8_planes(const uint8_t* gguf_q8_dev, int N, int K, void* planes_dev, void* stream);
FA_API int fa_op_q8p_gemm(const uint16_t* a16_dev, const uint16_t* a16_lo_dev, int M, int K, const void* planes_dev,
                          int N, int n_split, float* c_dev, int variant, void* stream);
FA_API int fa_op_q8p_gemm_swiglu(const uint16_t* a16_dev, const uint16_t* a16_lo_dev, int M, int K,
                                 const void* planes_dev, int N, uint16_t* h16_dev, uint16_t* h_lo_dev, void* stream);
FA_API int fa_op_q8p_gemm_argmax(const uint16_t* a16_dev, const uint16_t* a16_lo_dev, int M, int K,
                                 const void* planes_dev, int N, void* scratch_dev, int* next_dev, float* logits_dev,
                                 int variant, void* stream);

/* ---- host-only page allocator (no GPU needed): the policy behind fa_seq_* ----
 * Lowest free page id first; compaction moves the highest live page into the lowest
 * free id until the live pages are [0, n_live). */
typedef struct fa_palloc fa_palloc;
FA_API fa_palloc* fa_palloc_create(int n_pages);
FA_API void fa_palloc_destroy(fa_palloc* pa);
FA_API int fa_palloc_alloc(fa_palloc* pa);              /* page id, or FA_ERR_POOL_EXHAUSTED */
FA_API int fa_palloc_free(fa_palloc* pa, int page);     /* FA_ERR_INVALID_ARG on double free / range */
FA_API int fa_palloc_n_free(const fa_palloc* pa);
/* Applies compaction to the allocator and returns the moves (src[i] -> dst[i]); *n_moves. */
FA_API int fa_palloc_compact(fa_palloc* pa, int* src, int* dst, int max_moves, int* n_moves);

/* Failure detection without a fault: one CTA waits, with a limit of limit_us
 * microseconds, on an mbarrier that nothing completes, the same bounded wait every
 * pipelined kernel uses. The wait gives up, sets bit 1 (timeout) in *err_dev and the
 * kernel returns, leaving the context usable. */
FA_API int fa_op_wait_selftest(int limit_us, int* err_dev, void* stream);

/* ---- audio encoder (SANM) + adaptor: the producer of the prefill embeddings ----
 * Replaces compute/encoder_adaptor_gpu.hpp:27-677 (GPUEncoderAdaptorRunner::forward_on_gpu
 * :88-191) with the graphs of compute/encoder_ops.cpp:17-290 and compute/adaptor_ops.cpp:11-149.
 * Input: LFR features [T][input_dim] f32 (the front end's output); output: decoder input
 * embeddings [T][adaptor_output] f32, ready for fa_prefill / fa_forward (which accept
 * device pointers too). Weights: audio_encoder.* and audio_adaptor.* tensors
 * (model/loader.cpp:21-80,135-200), 2-D ones Q8_0, F16, BF16 or F32. */
typedef struct fa_encoder fa_encoder;
typedef struct fa_encoder_desc {
    int input_dim;       /* 560 = 80 mels x LFR 7 */
    int output_size;     /* 512, attention_heads x 128 */
    int attention_heads; /* 4 */
    int linear_units;    /* 2048 */
    int num_blocks;      /* 50: encoder0 + 49 */
    int tp_blocks;       /* 20 */
    int kernel_size;     /* FSMN taps, 11 */
    int sanm_shift;      /* 0 */
    int adaptor_hidden;  /* 2048 */
    int adaptor_output;  /* 1024 = decoder hidden, adaptor_heads x 128 */
    int adaptor_blocks;  /* 2 */
    int adaptor_heads;   /* 8 */
    int adaptor_ffn;     /* 256 */
    int max_frames;      /* frames per call (one utterance or a batch), <= 3000 */
} fa_encoder_desc;
FA_API void fa_encoder_default_desc(fa_encoder_desc* desc);
FA_API fa_encoder* fa_encoder_create(int device, const fa_encoder_desc* desc); /* NULL: fa_last_error(NULL) */
FA_API void fa_encoder_destroy(fa_encoder* e);
FA_API int fa_encoder_load_weights(fa_encoder* e, const fa_tensor_view* tensors, int n);
/* Host in, host out; synchronous. */
FA_API int fa_encoder_forward(fa_encoder* e, const float* lfr, int T, float* embeds);
/* Device (or host) pointers, on `stream` (NULL: the encoder's stream); returns when done. */
FA_API int fa_encoder_forward_dev(fa_encoder* e, const float* lfr_dev, int T, float* embeds_dev, void* stream);
/* n_utt utterances at once (frames[i] rows each, concatenated in lfr and embeds; host or
 * device pointers): every kernel runs over all rows, attention and the FSMN stay within
 * each utterance. Sum of frames <= max_frames. Each row layout is captured once as a
 * CUDA graph and replayed. */
FA_API int fa_encoder_forward_batch(fa_encoder* e, int n_utt, const int* frames, const float* lfr, float* embeds,
                                    void* stream);
/* 1 = replay captured CUDA graphs (default), 0 = direct launches. */
FA_API int fa_encoder_set_graphs(fa_encoder* e, int enable);

/* Library version string. */
FA_API const char* fa_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FUNASR_DEC_H */
