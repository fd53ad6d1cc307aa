// Launchers of the decoder kernels (one translation unit each) used by fa_api.cu.
#pragma once

#include "fa_common.cuh"
#include "q8_planes.cuh"

#include <cuda.h>

namespace fa {

// ---------------------------------------------------------------- k_append.cu --
// Kernel (1): per-head Q/K RMSNorm + NEOX RoPE + paged f16 K/V append.
struct AppendArgs {
    const float* qkv_part;   // [n_part][M][(Hq + 2*Hkv) * 128] f32 split-K partials of Wqkv . x
    int n_part;
    int M;
    const int* pos;          // [M] token position of each row
    const int* slot;         // [M] sequence slot of each row
    const int* block_table;  // [slots][bt_stride]
    int bt_stride;
    int n_pages;
    const float* qn_w;       // [128]
    const float* kn_w;       // [128]
    int Hq, Hkv;
    float eps, q_scale;
    const float2* rope;      // [max_pos][64]
    int max_pos;
    __half* pool_layer;      // [n_pages][Hkv][2][16][128]
    float* q_out;            // [M][Hq][128]
    int* err;
};
void launch_qknorm_rope_append(const AppendArgs& a, cudaStream_t s);

// Raw append of given f16 K/V for several layers (page-table microbenchmark).
struct RawAppendArgs {
    const __half* k;         // [M][n_layers][Hkv][128]
    const __half* v;
    int M, n_layers, Hkv;
    const int* pos;
    const int* slot;
    const int* block_table;
    int bt_stride;
    int n_pages;
    __half* pool;            // [n_layers][n_pages][Hkv][2][16][128]
    int* err;
};
void launch_kv_append_raw(const RawAppendArgs& a, cudaStream_t s);

// KV gather: tokens [0, n_kv[m]) of sequence slot[m], every layer, from the pages into
// head-major slabs k_out / v_out [n_layers][Hkv][total_rows][128], sequence m at rows
// [row0[m], row0[m] + n_kv[m]) of each head's plane. Hkv <= 8.
struct GatherArgs {
    const __half* pool;      // [n_layers][n_pages][Hkv][2][16][128]
    int n_layers, n_pages, Hkv;
    const int* block_table;
    int bt_stride;
    const int* slot;         // [M]
    const int* n_kv;         // [M]
    const int* row0;         // [M]
    int M, max_pages, total_rows;
    __half* k_out;
    __half* v_out;
    int* err;
};
void launch_kv_gather(const GatherArgs& a, cudaStream_t s);

// ------------------------------------------------------------- k_attention.cu --
// Kernel (2): paged GQA decode attention (head_dim 128, 2 query heads per KV head).
struct AttnArgs {
    const float* q;          // [M][Hq][128], already scaled by 1/sqrt(128)
    const __half* pool_layer;
    const int* block_table;
    int bt_stride;
    int n_pages;
    const int* slot;         // [M]
    const int* pos;          // [rows]; row m attends to tokens [0, pos[m]]
    const int* rows;         // [M] rows to attend (grid.z index -> row), or nullptr: rows 0..M-1
    int M, Hq, Hkv;
    int pages_per_split;     // pages one CTA reads
    int n_splits;            // grid.x; splits beyond a row's length exit at once
    int warps;               // 4 or 8 warps per CTA; 0: attn_warps(M)
    float* part_o;           // [M][Hq][n_splits][128] un-normalised partial outputs
    float* part_ml;          // [M][Hq][n_splits][2]   (running max in log2 units, sum)
    __half* out16;           // [M][Hq*128] final output as f16 hi part, or nullptr
    __half* out16_lo;        // [M][Hq*128] f16 remainder (out - hi), or nullptr
    float* out32;            // [M][Hq*128] final output (f32) or nullptr
    int* err;
    int* merge_cnt;          // [rows][Hkv] splits done per (row, KV head), zero between launches:
                             // the split that finishes last merges the head's splits itself;
                             // nullptr: the merge is launch_attn_combine's
    int fuse_append;         // kernel (1) of the rows' KV heads runs here, from app (q unused,
    AppendArgs app;          // rows 0..M-1): q of both query heads into shared memory, the token's
                             // K / V into its page by the split that holds the page
};
size_t attn_smem_bytes();
void launch_paged_attention(const AttnArgs& a, cudaStream_t s);
// Pipeline depth of each warp's page ring and the CTAs that fit on one SM (shared
// memory: 4 warps x kAttnStages x 8 KiB per CTA).
constexpr int kAttnStages = 2;
constexpr int kAttnCtasPerSm = 3;
// Steps of at most this many rows run 8 warps per CTA (one CTA per SM) unless AttnArgs::warps
// says otherwise, so that a split's pages spread over twice the warps; attn_warps gives that
// default for M rows (the decoder's planner picks 4 or 8 by its cost model up to
// kAttnPlanWideRows rows, 8 for one row).
constexpr int kAttnWideRows = 2;
constexpr int kAttnPlanWideRows = 64;
int attn_warps(int M);
// Split combine; only needed when n_splits > 1.
void launch_attn_combine(const AttnArgs& a, cudaStream_t s);

// ------------------------------------------------------------ k_prefill_attn.cu --
// Kernel (2b): causal attention of prefill tiles on the tensor cores. A tile is up to
// 64 consecutive rows of one sequence with non-decreasing positions; each CTA takes
// one (KV head, tile) and attends its rows to keys [0, pos[row]].
struct PrefillAttnArgs {
    const float* q;          // [M][Hq][128], already scaled by 1/sqrt(128)
    const int* block_table;
    int bt_stride;
    int n_pages;
    const int* slot;         // [M]
    const int* pos;          // [M]
    int M, Hq, Hkv;
    const int2* tiles;       // [n_tiles] (first row, rows <= 64)
    int n_tiles;
    int pool_row0;           // row of this layer's page 0 in the pool tensor map
    __half* out16;
    __half* out16_lo;
    float* out32;
    int* err;
};
size_t prefill_attn_smem_bytes();
void configure_prefill_attention();
// Tensor map over a page pool viewed as [total_rows][128] f16 (one row = one token of
// one head's K or V), 16-row x 64-column boxes, 128 B swizzle.
bool make_pool_map(CUtensorMap* tm, const void* pool, long long total_rows);
void launch_prefill_attention(const CUtensorMap& tm_pool, const PrefillAttnArgs& a, cudaStream_t s);

// --------------------------------------------------------------- k_encoder.cu --
// Audio encoder / adaptor steps around the GEMMs (x rows are frames).
void launch_enc_scale(const float* in, int T, int d, int ld, float scale, float* x, cudaStream_t s);
void launch_enc_resid_ln(float* x, int d, int ld_x, const float* part, int n_part, int T, const float* bias,
                         const float* mem, int residual, const float* ln_w, const float* ln_b, float eps,
                         int ln_in_place, __half* out_hi, __half* out_lo, int ld_out, cudaStream_t s);
void launch_enc_bias_act(const float* part, int n_part, int T, int n, const float* bias, int relu, float* y32,
                         __half* y_hi, __half* y_lo, int n_sm, cudaStream_t s);
// seg[t] = (first, end) rows of row t's utterance
void launch_enc_fsmn(const float* qkv, int T, const int2* seg, int d, const float* w, int K, int pad, float* mem,
                     cudaStream_t s);
size_t enc_attention_smem(int max_T);
void configure_encoder(int max_T);
// tiles[i] = (first row, rows <= 16, utterance's first row, utterance length <= max_T)
void launch_enc_attention(const float* qkv, const int4* tiles, int n_tiles, int d, int n_heads, __half* out_hi,
                          __half* out_lo, int max_T, cudaStream_t s);
constexpr int kEncAttRows = 16;
constexpr int kEncMaxFrames = 3000;   // frames per utterance and per batched pass (the encoder's row buffers)

// ------------------------------------------------------------------ k_gemm.cu --
// Kernel (4): Q8_0 weight GEMM on the tensor cores.  C[M][N] = A[M][K] . W[N][K]^T
// kEpiSwiglu (small-M kernel only): W stacks gate rows [0, N/2) over up rows [N/2, N) and
// the result is written as the f16 pair of silu(gate) * up, [M][N/2].
// kEpiQkvAppend (swapped tcgen05 kernel, Q8_0, skinny_fusable shapes): the QKV GEMM finishes
// kernel (1) itself (per-head RMSNorm, RoPE, q out, K / V into the pages) from *app.
// kEpiSwiglu on the swapped kernel needs swiglu_interleave64 and skinny_fusable shapes.
enum GemmEpilogue { kEpiStoreF32 = 0, kEpiArgmax = 1, kEpiSwiglu = 2, kEpiQkvAppend = 3 };
struct GemmArgs {
    const __half* A;         // [M][K] f16 activations (hi part)
    const __half* A_lo;      // [M][K] f16 remainder x - hi, or nullptr (plain f16 activations)
    const __half* Wh;        // [N][K] f16 weights (the encoder's f16(d * q)), read when W8.q is null
    Q8Planes W8;             // Q8_0 weights as q / d_t / d_r planes (the decoder's): exact d * q
    int M, N, K;
    int n_split;             // split-K factor (grid.z); K/n_split multiple of 64
    int epilogue;
    float* C;                // kEpiStoreF32: [n_split][M][N] partials (n_split == 1: the result)
    float* amax_val;         // kEpiArgmax: [M][N/64] per-tile row maxima
    int* amax_idx;           //             [M][N/64] first column holding them
    __half* H;               // kEpiSwiglu: [M][N/2] hi part
    __half* H_lo;            //             [M][N/2] lo part (may be nullptr)
    int swiglu_interleave64; // kEpiSwiglu: W stacks blocks of 64 gate rows and the 64 up rows of
                             // the same columns (the decoder's layout) instead of gate over up
    const struct AppendArgs* app;   // kEpiQkvAppend: kernel (1)'s arguments (qkv_part unused)
};
// mma.sync (m16n8k16) implementation; the cross-check variant.
void launch_q8_gemm(const GemmArgs& g, cudaStream_t s);
int gemm_pick_split(int M, int N, int K, int n_sm);
// tcgen05 / TMEM / TMA implementation (k_gemm_tc.cu); the default.
bool gemm_tc_supported(const GemmArgs& g);
int gemm_tc_pick_split(int M, int N, int K, int n_sm);
bool launch_q8_gemm_tc(const GemmArgs& g, int* err, cudaStream_t s);
size_t gemm_tc_smem_bytes();
// tcgen05 kernel with the operands swapped for steps of up to kSkinnyMaxRows rows
// (k_gemm_tc_skinny.cu): weights on the MMA's 128-row side, activations on its N side.
constexpr int kSkinnyMaxRows = 128;
// The default GEMM choice uses it up to this many rows (layer GEMMs: 10-25 % faster than the
// 128-row-tile kernel at 4-128 rows), and for the lm_head argmax only up to 32 rows (its
// per-row warp reductions make it slower than the 128-row-tile epilogue above that).
constexpr int kSkinnyAutoRows = 128;
constexpr int kSkinnyArgmaxAutoRows = 32;
bool gemm_tc_skinny_supported(const GemmArgs& g);
int skinny_tile_rows(int M);      // activation rows per tile the kernel takes for Q8_0 weights
bool skinny_fusable(int M, int N, int K, int n_split, int n_sm);   // the fused epilogues apply
int gemm_tc_skinny_pick_split(int M, int N, int K, int n_sm);
bool launch_q8_gemm_tc_skinny(const GemmArgs& g, int* err, cudaStream_t s);
// CUDA-core small-M kernel (k_gemv.cu): M <= kGemvMaxRows, n_split 1, K a multiple of 256;
// the store epilogue needs N a multiple of 4, the argmax epilogue N a multiple of 64 and
// K <= 1024 (f16 weights) or K <= 2048 (Q8_0 planes, K a multiple of 512) or K == 256. The
// decoder uses it by default up to kGemvAutoRows rows.
constexpr int kGemvMaxRows = 8;
constexpr int kGemvAutoRows = 2;
bool gemv_shape_supported(int M, int N, int K, int epilogue, bool q8 = true);
bool launch_q8_gemv(const GemmArgs& g, cudaStream_t s);   // false: shape or pointers not taken
// How the CUDA-core kernel splits a Q8_0 GEMM with 16 weights per lane (K a multiple of 512):
// ks warps share a block of 4 weight rows, each taking ns slices of 512 columns. False when
// the kernel would not take the shape that way.
bool gemv_q8_split(int M, int N, int K, int epilogue, int* ks, int* ns);

// --------------------------------------------------------------- k_row_step.cu --
// The decode step of one row (one sequence, one token) as one persistent cooperative
// kernel: embedding, every layer and the final norm; the lm_head GEMV and the argmax
// reduce follow as ordinary launches. Same arithmetic, same bits as the launch-per-op step
// with the CUDA-core GEMMs.
struct RowLayer {
    const unsigned char* w[4];   // Q8_0 planes of QKV, o_proj, gate|up (64-row blocks), down
    const float* in_norm;
    const float* post_norm;
    const float* q_norm;
    const float* k_norm;
};
struct RowGemm {
    int N, K, ks;                // ks warps x 512 columns cover K (one slice each)
    int swiglu;                  // gate / up pairs, 64-row interleave, SwiGLU output
};
struct RowCtl {
    unsigned int seq;            // launches completed: tags of launch k are (k + 1) * layers + layer
    int abort;                   // a wait ran out: every CTA leaves
    int att_cnt[8];              // attention splits finished per KV head (reset by the last one)
    int lm_cnt;                  // CTAs done with their lm_head tiles (reset by the last one)
};
struct RowStepArgs {
    const RowLayer* layers;
    int n_layers, hidden, ffn;
    RowGemm gm[4];
    float eps, q_scale;
    const void* embed;
    int embed_type, vocab;
    int x_ready;                 // x_a already holds the row's input (embeddings given)
    const int* tok;
    const int* slot;
    const int* pos;
    const int* block_table;
    int bt_stride, n_pages;
    __half* pool;
    size_t layer_stride;         // elements between layers of the pool
    const float2* rope;
    int max_pos;
    float* x_a;                  // the row's input (x_ready), and the final residual on exit
    // tagged words {value, tag} the phases hand on (row_step_words of them, in this order)
    unsigned long long* w_qkv;   // [(Hq + 2 Hkv) * 128] f32
    unsigned long long* w_att;   // [Hq * 128] f16 pair
    unsigned long long* w_o;     // [hidden] f32
    unsigned long long* w_h;     // [ffn] f16 pair
    unsigned long long* w_dn;    // [hidden] f32
    float* att_po;               // split partials (n_splits > 1)
    float* att_pml;
    int pps, n_splits;
    const float* final_norm;
    __half* xn16;                // final norm output, the lm_head's input pair
    __half* xn_lo;
    // lm (row_step_lm_fits): the lm_head and the argmax run in the kernel too
    int lm;
    const unsigned char* lm_q;   // lm_head Q8_0 planes [vocab][hidden]
    int lm_tiles;                // vocab / 64
    float* logits;               // [vocab] or nullptr
    float* amax_val;             // [lm_tiles] per-tile maxima and their rows
    int* amax_idx;
    int* next;                   // [1] the argmax
    int* feed_tok;               // or nullptr: the token fed back for the next step
    int* feed_pos;               //             and its position + 1
    RowCtl* ctl;
    int* err;
    unsigned long long wait_ns;  // limit of one wait for a word
    int absent_cta;              // failure test: this CTA leaves at once (its words never come); -1 = none
    int stage_q_bytes;           // set by launch_row_step
};
size_t row_step_words(int hidden, int ffn);
bool row_step_lm_fits(int hidden, int vocab);
// Fills gm[] for a model's shapes; false when the kernel does not take them.
bool row_step_shapes(int hidden, int ffn, int grid, RowGemm* gm);
cudaError_t configure_row_step();
// grid: one CTA per SM (a cooperative launch: all CTAs resident, or the launch fails)
cudaError_t launch_row_step(const RowStepArgs& a, int grid, cudaStream_t s);

// ----------------------------------------------------------------- k_small.cu --
void launch_embed(const void* table, int table_type, int hidden, const int* tokens, const float* embeds,
                  int M, int vocab, float* x, int* err, cudaStream_t s);
// Activations for the GEMMs leave their producer as an f16 pair: hi = f16(y), lo = f16(y - hi).
// x[m] += sum_s part[s][m] (n_part may be 0); (hi, lo)[m] = split(rmsnorm(x[m]) * w).
// With rows: only rows[k] (k < n_out) are processed and written to output row k.
void launch_residual_rmsnorm(float* x, const float* part, int n_part, int M, int hidden, const float* w,
                             float eps, __half* xn_hi, __half* xn_lo, cudaStream_t s, int n_out = -1,
                             const int* rows = nullptr);
// (hi, lo)[m][j] = split(silu(g) * u), g and u summed over n_part partials of the gate|up GEMM:
// gate columns [0, ffn) and up columns [ffn, 2 ffn), or with interleave64 the decoder's
// stacking, 64 gate columns then the 64 up columns of the same outputs, block after block
void launch_swiglu(const float* part, int n_part, int M, int ffn, __half* h_hi, __half* h_lo, cudaStream_t s,
                   bool interleave64 = false);
// next[m] = first column of the row maximum over n_tiles partial maxima; optional feedback
// of the token into tokens[m] and pos[m] += 1 for device-fed generation.
void launch_argmax_reduce(const float* val, const int* idx, int M, int n_tiles, int* next, int* feed_tokens,
                          int* feed_pos, cudaStream_t s);
void launch_apply_bt_updates(int* block_table, const int* upd_idx, const int* upd_page, int n, cudaStream_t s);
// One CTA waits on an mbarrier that is never completed, for limit_ns: sets kDevErrTimeout.
void launch_wait_selftest(int* err, unsigned long long limit_ns, cudaStream_t s);
// GGUF Q8_0 rows [N][K/32][34 B] -> W [N][K] f16 with W = f16(f32(d) * q), rows landing at
// destination row r0 + n (Wq, Wk, Wv and gate, up are stacked that way).
void launch_repack_q8(const uint8_t* raw, int N, int K, int r0, __half* dst_w, cudaStream_t s);
void launch_page_copy(__half* pool, size_t layer_stride, int n_layers, const int* src, const int* dst, int n,
                      cudaStream_t s);
void launch_fill_random(__half* pool, size_t layer_stride, int n_layers, const int* pages, int n_pages_list,
                        unsigned long long seed, cudaStream_t s);
void launch_read_pages(const __half* pool_layer, const int* pages, int n, __half* out, cudaStream_t s);

}  // namespace fa
