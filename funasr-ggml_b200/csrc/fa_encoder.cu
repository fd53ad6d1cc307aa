// Audio encoder (SANM, 50 + 20 layers) and adaptor on the GPU: the producer of the
// decoder's prefill embeddings, exported as fa_encoder_*.
//
// Replaces compute/encoder_adaptor_gpu.hpp:27-677 (GPUEncoderAdaptorRunner, in
// particular forward_on_gpu :88-191) and the graphs of compute/encoder_ops.cpp:17-290
// and compute/adaptor_ops.cpp:11-149. Per encoder layer (rows are frames):
//   LayerNorm -> QKV GEMM (q, k, v stacked, 1536 x d_in) -> + bias -> FSMN on v
//   -> 4-head bidirectional attention -> output GEMM -> + bias + FSMN memory
//   (+ residual) -> LayerNorm -> FFN GEMM (2048) -> + bias, ReLU -> GEMM -> + bias
//   + residual
// The GEMMs are the decoder's tcgen05 kernel (f16(d*q) weights, activations as an
// f16 pair); encoder0's 560-wide input is zero-padded to 576 columns.
#include "nvtx_range.hpp"
#include "fa_kernels.cuh"
#include "funasr_dec.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <unordered_map>
#include <vector>

namespace fa {
int report_op_error(int code, const char* msg);   // fa_api.cu
int ensure_device_configured();                     // fa_api.cu
}  // namespace fa

namespace {

struct Lin {
    __half* w = nullptr;   // [n][kp] f16
    float* b = nullptr;    // [n]
    int n = 0, k = 0, kp = 0;
};

struct EncLayer {
    float *n1w = nullptr, *n1b = nullptr, *n2w = nullptr, *n2b = nullptr;
    Lin qkv, out, w1, w2;
    float* fsmn = nullptr;   // [d][K]
    int d_in = 0;
};

struct AdaBlock {
    float *n1w = nullptr, *n1b = nullptr, *n2w = nullptr, *n2b = nullptr;
    Lin qkv, out, w1, w2;
};

int pad64(int k) { return (k + 63) / 64 * 64; }

float bf16f(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

float f16f(uint16_t h) {
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}

}  // namespace

struct fa_encoder {
    int device = 0;
    fa_encoder_desc d{};
    cudaStream_t stream = nullptr;
    int n_sm = 148;
    bool loaded = false;
    std::vector<void*> allocs;
    EncLayer e0;
    std::vector<EncLayer> main_l, tp_l;
    float *after_w = nullptr, *after_b = nullptr, *tp_w = nullptr, *tp_b = nullptr;
    Lin lin1, lin2;
    std::vector<AdaBlock> blocks;
    // activations
    float *in_raw = nullptr, *in0 = nullptr, *x = nullptr, *qkv = nullptr, *mem = nullptr, *part = nullptr;
    __half *xn = nullptr, *xn_lo = nullptr, *att = nullptr, *att_lo = nullptr, *hid = nullptr, *hid_lo = nullptr;
    __half *xn0 = nullptr, *xn0_lo = nullptr;   // encoder0's padded input pair: its pad columns stay zero
    size_t part_elems = 0;
    int* err_dev = nullptr;
    int* h_err = nullptr;
    // utterance layout of the rows: seg[t] = (first, end) row of row t's utterance;
    // attention tiles (first row, rows, utterance start, utterance length)
    int2* seg_dev = nullptr;
    int4* tiles_dev = nullptr;
    int2* h_seg = nullptr;
    int4* h_tiles = nullptr;
    int max_tiles = 0;
    bool use_graphs = true;
    std::map<std::pair<int, int>, cudaGraphExec_t> graphs;   // (rows, tiles) -> the whole forward

    template <typename T>
    int alloc(T** p, size_t bytes) {
        void* v = nullptr;
        if (cudaMalloc(&v, bytes ? bytes : 16) != cudaSuccess) {
            cudaGetLastError();
            return fa::report_op_error(FA_ERR_OOM, ("encoder: cudaMalloc of " + std::to_string(bytes) + " B").c_str());
        }
        allocs.push_back(v);
        *p = reinterpret_cast<T*>(v);
        return FA_OK;
    }
    ~fa_encoder() {
        if (device >= 0) cudaSetDevice(device);
        for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
        for (void* p : allocs) cudaFree(p);
        if (h_err) cudaFreeHost(h_err);
        if (h_seg) cudaFreeHost(h_seg);
        if (h_tiles) cudaFreeHost(h_tiles);
        if (stream) cudaStreamDestroy(stream);
    }
};

namespace {

int fail(const std::string& m, int code = FA_ERR_WEIGHTS) { return fa::report_op_error(code, m.c_str()); }

// Split-K factor of an encoder GEMM of T rows (the kernel gemm() picks for it)
int enc_split(int T, int n, int kp, int n_sm) {
    if (n % 128) return fa::gemm_pick_split(T, n, kp, n_sm);
    return T <= fa::kSkinnyAutoRows ? fa::gemm_tc_skinny_pick_split(T, n, kp, n_sm)
                                    : fa::gemm_tc_pick_split(T, n, kp, n_sm);
}

using TMap = std::unordered_map<std::string, const fa_tensor_view*>;

const fa_tensor_view* get(const TMap& m, const std::string& name, std::string& err) {
    auto it = m.find(name);
    if (it == m.end()) {
        err = "missing tensor " + name;
        return nullptr;
    }
    return it->second;
}

// Host f32 copy of a 1-D tensor of n values (any of F32 / F16 / BF16).
bool host_vec(const fa_tensor_view* v, int n, std::vector<float>& out, std::string& err) {
    const size_t cnt = (size_t)v->ne[0] * (size_t)(v->ne[1] > 0 ? v->ne[1] : 1);
    if ((int)cnt != n) {
        err = std::string(v->name) + ": " + std::to_string(cnt) + " values, expected " + std::to_string(n);
        return false;
    }
    out.resize(n);
    for (int i = 0; i < n; ++i) {
        if (v->type == FA_TYPE_F32) out[i] = reinterpret_cast<const float*>(v->data)[i];
        else if (v->type == FA_TYPE_F16) out[i] = f16f(reinterpret_cast<const uint16_t*>(v->data)[i]);
        else if (v->type == FA_TYPE_BF16) out[i] = bf16f(reinterpret_cast<const uint16_t*>(v->data)[i]);
        else {
            err = std::string(v->name) + ": unsupported type " + std::to_string(v->type);
            return false;
        }
    }
    return true;
}

int upload_vec(fa_encoder* e, const TMap& m, const std::string& name, int n, float** dst, int off = 0,
               float* existing = nullptr) {
    std::string err;
    const fa_tensor_view* v = get(m, name, err);
    std::vector<float> h;
    if (!v || !host_vec(v, n, h, err)) return fail(err);
    float* p = existing;
    if (!p && e->alloc(&p, sizeof(float) * n)) return FA_ERR_OOM;
    // copies from pageable memory can return before their DMA lands: order and wait on the stream
    if (cudaMemcpyAsync(p + off, h.data(), sizeof(float) * n, cudaMemcpyHostToDevice, e->stream) != cudaSuccess ||
        cudaStreamSynchronize(e->stream) != cudaSuccess)
        return fail("upload " + name, FA_ERR_CUDA);
    if (dst) *dst = p;
    return FA_OK;
}

// A 2-D weight [n][k] (GGUF ne = {k, n}) into rows r0.. of an f16 [rows][kp] matrix.
int upload_mat(fa_encoder* e, const fa_tensor_view* v, int n, int k, int kp, __half* dst, int r0, uint8_t* staging) {
    if (v->ne[0] != k || v->ne[1] != n)
        return fail(std::string(v->name) + ": shape [" + std::to_string(v->ne[0]) + ", " + std::to_string(v->ne[1]) +
                    "], expected [" + std::to_string(k) + ", " + std::to_string(n) + "]");
    if (v->type == FA_TYPE_Q8_0 && kp == k) {
        if (v->nbytes != (size_t)n * (k / 32) * 34) return fail(std::string(v->name) + ": byte size");
        // the copy and the repack on one stream: a copy from pageable memory may return
        // before its DMA has landed
        if (cudaMemcpyAsync(staging, v->data, v->nbytes, cudaMemcpyHostToDevice, e->stream) != cudaSuccess)
            return fail("upload " + std::string(v->name), FA_ERR_CUDA);
        fa::launch_repack_q8(staging, n, k, r0, dst, e->stream);
        if (cudaStreamSynchronize(e->stream) != cudaSuccess) return fail("repack", FA_ERR_CUDA);
        return FA_OK;
    }
    std::vector<__half> h((size_t)n * kp, __float2half(0.0f));
    for (int r = 0; r < n; ++r)
        for (int c = 0; c < k; ++c) {
            const size_t i = (size_t)r * k + c;
            float f;
            if (v->type == FA_TYPE_F32) f = reinterpret_cast<const float*>(v->data)[i];
            else if (v->type == FA_TYPE_F16) f = f16f(reinterpret_cast<const uint16_t*>(v->data)[i]);
            else if (v->type == FA_TYPE_BF16) f = bf16f(reinterpret_cast<const uint16_t*>(v->data)[i]);
            else return fail(std::string(v->name) + ": Q8_0 needs a width that is a multiple of 64");
            h[(size_t)r * kp + c] = __float2half_rn(f);
        }
    if (cudaMemcpyAsync(dst + (size_t)r0 * kp, h.data(), sizeof(__half) * h.size(), cudaMemcpyHostToDevice,
                        e->stream) != cudaSuccess ||
        cudaStreamSynchronize(e->stream) != cudaSuccess)
        return fail("upload " + std::string(v->name), FA_ERR_CUDA);
    return FA_OK;
}

int load_lin(fa_encoder* e, const TMap& m, const std::vector<std::string>& names, int n_each, int k, Lin& L,
             uint8_t* staging) {
    L.n = n_each * (int)names.size();
    L.k = k;
    L.kp = pad64(k);
    if (e->alloc(&L.w, sizeof(__half) * (size_t)L.n * L.kp) || e->alloc(&L.b, sizeof(float) * L.n)) return FA_ERR_OOM;
    for (size_t i = 0; i < names.size(); ++i) {
        std::string err;
        const fa_tensor_view* v = get(m, names[i] + ".weight", err);
        if (!v) return fail(err);
        if (int rc = upload_mat(e, v, n_each, k, L.kp, L.w, (int)i * n_each, staging)) return rc;
        float* bp = L.b;
        if (int rc = upload_vec(e, m, names[i] + ".bias", n_each, nullptr, (int)i * n_each, bp)) return rc;
    }
    return FA_OK;
}

int load_enc_layer(fa_encoder* e, const TMap& m, const std::string& p, int d_in, EncLayer& L, uint8_t* staging) {
    const fa_encoder_desc& d = e->d;
    L.d_in = d_in;
    int rc;
    if ((rc = upload_vec(e, m, p + ".norm1.weight", d_in, &L.n1w)) || (rc = upload_vec(e, m, p + ".norm1.bias", d_in, &L.n1b)) ||
        (rc = upload_vec(e, m, p + ".norm2.weight", d.output_size, &L.n2w)) ||
        (rc = upload_vec(e, m, p + ".norm2.bias", d.output_size, &L.n2b)))
        return rc;
    const std::string a = p + ".self_attn.";
    if ((rc = load_lin(e, m, {a + "linear_q", a + "linear_k", a + "linear_v"}, d.output_size, d_in, L.qkv, staging)) ||
        (rc = load_lin(e, m, {a + "linear_out"}, d.output_size, d.output_size, L.out, staging)) ||
        (rc = load_lin(e, m, {p + ".feed_forward.w_1"}, d.linear_units, d.output_size, L.w1, staging)) ||
        (rc = load_lin(e, m, {p + ".feed_forward.w_2"}, d.output_size, d.linear_units, L.w2, staging)))
        return rc;
    return upload_vec(e, m, a + "fsmn_block.weight", d.output_size * d.kernel_size, &L.fsmn);
}

int load_ada_block(fa_encoder* e, const TMap& m, const std::string& p, AdaBlock& B, uint8_t* staging) {
    const fa_encoder_desc& d = e->d;
    const int D = d.adaptor_output;
    int rc;
    if ((rc = upload_vec(e, m, p + ".norm1.weight", D, &B.n1w)) || (rc = upload_vec(e, m, p + ".norm1.bias", D, &B.n1b)) ||
        (rc = upload_vec(e, m, p + ".norm2.weight", D, &B.n2w)) || (rc = upload_vec(e, m, p + ".norm2.bias", D, &B.n2b)))
        return rc;
    const std::string a = p + ".self_attn.";
    if ((rc = load_lin(e, m, {a + "linear_q", a + "linear_k", a + "linear_v"}, D, D, B.qkv, staging)) ||
        (rc = load_lin(e, m, {a + "linear_out"}, D, D, B.out, staging)) ||
        (rc = load_lin(e, m, {p + ".feed_forward.w_1"}, d.adaptor_ffn, D, B.w1, staging)) ||
        (rc = load_lin(e, m, {p + ".feed_forward.w_2"}, D, d.adaptor_ffn, B.w2, staging)))
        return rc;
    return FA_OK;
}

// C[split][T][n] = A[T][kp] . W^T on the tensor cores: the swapped-operand kernel up to
// 128 rows (one utterance of up to ~13 s), the 128-row-tile kernel above, the mma.sync
// kernel when N is not a multiple of 128; returns the split count.
int gemm(fa_encoder* e, const __half* a, const __half* a_lo, int T, const Lin& L) {
    fa::GemmArgs g{};
    g.A = a; g.A_lo = a_lo; g.Wh = L.w; g.M = T; g.N = L.n; g.K = L.kp; g.epilogue = fa::kEpiStoreF32; g.C = e->part;
    g.n_split = enc_split(T, L.n, L.kp, e->n_sm);
    const bool tc = L.n % 128 == 0;
    if (tc && T <= fa::kSkinnyAutoRows && fa::launch_q8_gemm_tc_skinny(g, e->err_dev, e->stream)) return g.n_split;
    if (!(tc && fa::gemm_tc_supported(g) && fa::launch_q8_gemm_tc(g, e->err_dev, e->stream)))
        fa::launch_q8_gemm(g, e->stream);
    return g.n_split;
}

// The LayerNorm that follows a layer's last residual add, applied by the same launch: the
// next layer's norm1 (into xn, x kept), or after_norm / tp_norm in place of x. The launch
// normalises the f32 row it has just written, the values a separate launch would read
// back, so the results are the same bits with one launch fewer per layer.
struct LnTail {
    const float* w = nullptr;
    const float* b = nullptr;
    float eps = 0.0f;
    int in_place = 0;
    bool to_xn = false;      // the f16 pair into xn / xn_lo
};

void enc_layer(fa_encoder* e, const EncLayer& L, int T, int n_tiles, bool residual, const float* x_in, int ld_in,
               bool ln1_done, const LnTail& tail) {
    const fa_encoder_desc& d = e->d;
    const int D = d.output_size;
    cudaStream_t s = e->stream;
    // norm1 of the layer input (encoder0: the scaled features, 560 of 576 columns), unless
    // the previous layer's last launch left it in xn
    const bool padded = L.qkv.kp != L.d_in;
    __half* in_hi = padded ? e->xn0 : e->xn;
    __half* in_lo = padded ? e->xn0_lo : e->xn_lo;
    if (!ln1_done)
        fa::launch_enc_resid_ln(const_cast<float*>(x_in), L.d_in, ld_in, nullptr, -1, T, nullptr, nullptr, 0, L.n1w,
                                L.n1b, 1e-5f, 0, in_hi, in_lo, L.qkv.kp, s);
    int sp = gemm(e, in_hi, in_lo, T, L.qkv);
    fa::launch_enc_bias_act(e->part, sp, T, L.qkv.n, L.qkv.b, 0, e->qkv, nullptr, nullptr, e->n_sm, s);
    fa::launch_enc_fsmn(e->qkv, T, e->seg_dev, D, L.fsmn, d.kernel_size, (d.kernel_size - 1) / 2 - d.sanm_shift,
                        e->mem, s);
    fa::launch_enc_attention(e->qkv, e->tiles_dev, n_tiles, D, d.attention_heads, e->att, e->att_lo, d.max_frames, s);
    sp = gemm(e, e->att, e->att_lo, T, L.out);
    // x = (x) + out + bias + memory, then norm2
    fa::launch_enc_resid_ln(e->x, D, D, e->part, sp, T, L.out.b, e->mem, residual ? 1 : 0, L.n2w, L.n2b, 1e-5f, 0,
                            e->xn, e->xn_lo, D, s);
    sp = gemm(e, e->xn, e->xn_lo, T, L.w1);
    fa::launch_enc_bias_act(e->part, sp, T, L.w1.n, L.w1.b, 1, nullptr, e->hid, e->hid_lo, e->n_sm, s);
    sp = gemm(e, e->hid, e->hid_lo, T, L.w2);
    fa::launch_enc_resid_ln(e->x, D, D, e->part, sp, T, L.w2.b, nullptr, 1, tail.w, tail.b, tail.eps, tail.in_place,
                            tail.to_xn ? e->xn : nullptr, tail.to_xn ? e->xn_lo : nullptr, tail.to_xn ? D : 0, s);
}

void ada_block(fa_encoder* e, const AdaBlock& B, int T, int n_tiles, bool ln1_done, const LnTail& tail) {
    const fa_encoder_desc& d = e->d;
    const int D = d.adaptor_output;
    cudaStream_t s = e->stream;
    if (!ln1_done)
        fa::launch_enc_resid_ln(e->x, D, D, nullptr, -1, T, nullptr, nullptr, 0, B.n1w, B.n1b, 1e-12f, 0, e->xn,
                                e->xn_lo, D, s);
    int sp = gemm(e, e->xn, e->xn_lo, T, B.qkv);
    fa::launch_enc_bias_act(e->part, sp, T, B.qkv.n, B.qkv.b, 0, e->qkv, nullptr, nullptr, e->n_sm, s);
    fa::launch_enc_attention(e->qkv, e->tiles_dev, n_tiles, D, d.adaptor_heads, e->att, e->att_lo, d.max_frames, s);
    sp = gemm(e, e->att, e->att_lo, T, B.out);
    fa::launch_enc_resid_ln(e->x, D, D, e->part, sp, T, B.out.b, nullptr, 1, B.n2w, B.n2b, 1e-12f, 0, e->xn, e->xn_lo,
                            D, s);
    sp = gemm(e, e->xn, e->xn_lo, T, B.w1);
    fa::launch_enc_bias_act(e->part, sp, T, B.w1.n, B.w1.b, 1, nullptr, e->hid, e->hid_lo, e->n_sm, s);
    sp = gemm(e, e->hid, e->hid_lo, T, B.w2);
    fa::launch_enc_resid_ln(e->x, D, D, e->part, sp, T, B.w2.b, nullptr, 1, tail.w, tail.b, tail.eps, tail.in_place,
                            tail.to_xn ? e->xn : nullptr, tail.to_xn ? e->xn_lo : nullptr, tail.to_xn ? D : 0, s);
}

}  // namespace

extern "C" void fa_encoder_default_desc(fa_encoder_desc* d) {
    if (!d) return;
    d->input_dim = 560;
    d->output_size = 512;
    d->attention_heads = 4;
    d->linear_units = 2048;
    d->num_blocks = 50;
    d->tp_blocks = 20;
    d->kernel_size = 11;
    d->sanm_shift = 0;
    d->adaptor_hidden = 2048;
    d->adaptor_output = 1024;
    d->adaptor_blocks = 2;
    d->adaptor_heads = 8;
    d->adaptor_ffn = 256;
    d->max_frames = 1024;
}

extern "C" fa_encoder* fa_encoder_create(int device, const fa_encoder_desc* desc) {
    if (!desc) {
        fail("fa_encoder_create: NULL descriptor", FA_ERR_INVALID_ARG);
        return nullptr;
    }
    const fa_encoder_desc& d = *desc;
    if (d.output_size != d.attention_heads * 128 || d.adaptor_output != d.adaptor_heads * 128 || d.num_blocks < 1 ||
        d.tp_blocks < 0 || d.kernel_size < 1 || d.max_frames < 1 || d.max_frames > fa::kEncMaxFrames || d.input_dim < 1 ||
        d.input_dim > 2048 || d.output_size % 128 || d.linear_units % 128 || d.adaptor_hidden % 128 ||
        d.adaptor_ffn % 128 || d.output_size > 2048 || d.adaptor_output > 2048) {
        fail("fa_encoder_create: unsupported geometry (head_dim 128, widths multiples of 128, <= 3000 frames)",
             FA_ERR_INVALID_ARG);
        return nullptr;
    }
    int n_dev = 0;
    if (cudaGetDeviceCount(&n_dev) != cudaSuccess || device < 0 || device >= n_dev) {
        cudaGetLastError();
        fail("fa_encoder_create: no CUDA device " + std::to_string(device), FA_ERR_CUDA);
        return nullptr;
    }
    cudaSetDevice(device);
    if (fa::ensure_device_configured() != FA_OK) {
        fail("fa_encoder_create: kernel configuration", FA_ERR_CUDA);
        return nullptr;
    }
    fa::configure_encoder(d.max_frames);
    fa_encoder* e = new fa_encoder;
    e->device = device;
    e->d = d;
    cudaDeviceGetAttribute(&e->n_sm, cudaDevAttrMultiProcessorCount, device);
    if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete e;
        fail("fa_encoder_create: stream", FA_ERR_CUDA);
        return nullptr;
    }
    const int T = d.max_frames;
    const int kin = pad64(d.input_dim);
    const int wide = std::max({kin, d.output_size, d.adaptor_output});
    const int nmax = std::max({3 * d.output_size, 3 * d.adaptor_output, d.linear_units, d.adaptor_hidden});
    // split-K partials: the largest split * rows * width any GEMM of the model uses
    size_t part = 0;
    const int shapes[][2] = {{3 * d.output_size, kin}, {3 * d.output_size, d.output_size}, {d.output_size, d.output_size},
                             {d.linear_units, d.output_size}, {d.output_size, d.linear_units},
                             {d.adaptor_hidden, d.output_size}, {d.adaptor_output, d.adaptor_hidden},
                             {3 * d.adaptor_output, d.adaptor_output}, {d.adaptor_output, d.adaptor_output},
                             {d.adaptor_ffn, d.adaptor_output}, {d.adaptor_output, d.adaptor_ffn}};
    for (int m = 1; m <= T; ++m)
        for (const auto& sh : shapes) {
            const int kp = pad64(sh[1]);
            const int sp = enc_split(m, sh[0], kp, e->n_sm);
            part = std::max(part, (size_t)sp * m * sh[0]);
        }
    e->part_elems = part;
    e->max_tiles = 2 * T;
    if (e->alloc(&e->in_raw, sizeof(float) * (size_t)T * d.input_dim) || e->alloc(&e->in0, sizeof(float) * (size_t)T * kin) ||
        e->alloc(&e->x, sizeof(float) * (size_t)T * std::max(d.output_size, d.adaptor_output)) ||
        e->alloc(&e->qkv, sizeof(float) * (size_t)T * nmax) || e->alloc(&e->mem, sizeof(float) * (size_t)T * d.output_size) ||
        e->alloc(&e->part, sizeof(float) * part) || e->alloc(&e->xn, sizeof(__half) * (size_t)T * wide) ||
        e->alloc(&e->xn_lo, sizeof(__half) * (size_t)T * wide) ||
        e->alloc(&e->att, sizeof(__half) * (size_t)T * std::max(d.output_size, d.adaptor_output)) ||
        e->alloc(&e->att_lo, sizeof(__half) * (size_t)T * std::max(d.output_size, d.adaptor_output)) ||
        e->alloc(&e->hid, sizeof(__half) * (size_t)T * std::max(d.linear_units, d.adaptor_hidden)) ||
        e->alloc(&e->hid_lo, sizeof(__half) * (size_t)T * std::max(d.linear_units, d.adaptor_hidden)) ||
        e->alloc(&e->xn0, sizeof(__half) * (size_t)T * kin) || e->alloc(&e->xn0_lo, sizeof(__half) * (size_t)T * kin) ||
        e->alloc(&e->seg_dev, sizeof(int2) * (size_t)T) || e->alloc(&e->tiles_dev, sizeof(int4) * (size_t)2 * T) ||
        cudaMallocHost(&e->h_seg, sizeof(int2) * (size_t)T) != cudaSuccess ||
        cudaMallocHost(&e->h_tiles, sizeof(int4) * (size_t)2 * T) != cudaSuccess ||
        e->alloc(&e->err_dev, sizeof(int)) || cudaMallocHost(&e->h_err, sizeof(int)) != cudaSuccess) {
        delete e;
        return nullptr;
    }
    // encoder0's pad columns stay zero (only its norm1 writes that buffer)
    if (cudaMemset(e->xn0, 0, sizeof(__half) * (size_t)T * kin) != cudaSuccess ||
        cudaMemset(e->xn0_lo, 0, sizeof(__half) * (size_t)T * kin) != cudaSuccess ||
        cudaMemset(e->err_dev, 0, sizeof(int)) != cudaSuccess) {
        delete e;
        fail("fa_encoder_create: memset", FA_ERR_CUDA);
        return nullptr;
    }
    return e;
}

extern "C" void fa_encoder_destroy(fa_encoder* e) { delete e; }

extern "C" int fa_encoder_load_weights(fa_encoder* e, const fa_tensor_view* tensors, int n) {
    if (!e || (!tensors && n > 0)) return fail("fa_encoder_load_weights: bad argument", FA_ERR_INVALID_ARG);
    if (e->loaded) return fail("encoder weights already loaded", FA_ERR_INVALID_ARG);
    cudaSetDevice(e->device);
    TMap m;
    for (int i = 0; i < n; ++i)
        if (tensors[i].name) m[tensors[i].name] = &tensors[i];
    const fa_encoder_desc& d = e->d;
    size_t max_q8 = 0;
    for (int i = 0; i < n; ++i)
        if (tensors[i].type == FA_TYPE_Q8_0) max_q8 = std::max(max_q8, tensors[i].nbytes);
    uint8_t* staging = nullptr;
    if (max_q8 && cudaMalloc(&staging, max_q8) != cudaSuccess) {
        cudaGetLastError();
        return fail("encoder weight staging", FA_ERR_OOM);
    }
    auto run = [&]() -> int {
        int rc;
        if ((rc = load_enc_layer(e, m, "audio_encoder.encoders0.0", d.input_dim, e->e0, staging))) return rc;
        e->main_l.resize(d.num_blocks - 1);
        for (int i = 0; i < d.num_blocks - 1; ++i)
            if ((rc = load_enc_layer(e, m, "audio_encoder.encoders." + std::to_string(i), d.output_size, e->main_l[i],
                                     staging)))
                return rc;
        e->tp_l.resize(d.tp_blocks);
        for (int i = 0; i < d.tp_blocks; ++i)
            if ((rc = load_enc_layer(e, m, "audio_encoder.tp_encoders." + std::to_string(i), d.output_size, e->tp_l[i],
                                     staging)))
                return rc;
        if ((rc = upload_vec(e, m, "audio_encoder.after_norm.weight", d.output_size, &e->after_w)) ||
            (rc = upload_vec(e, m, "audio_encoder.after_norm.bias", d.output_size, &e->after_b)) ||
            (rc = upload_vec(e, m, "audio_encoder.tp_norm.weight", d.output_size, &e->tp_w)) ||
            (rc = upload_vec(e, m, "audio_encoder.tp_norm.bias", d.output_size, &e->tp_b)))
            return rc;
        if ((rc = load_lin(e, m, {"audio_adaptor.linear1"}, d.adaptor_hidden, d.output_size, e->lin1, staging)) ||
            (rc = load_lin(e, m, {"audio_adaptor.linear2"}, d.adaptor_output, d.adaptor_hidden, e->lin2, staging)))
            return rc;
        e->blocks.resize(d.adaptor_blocks);
        for (int i = 0; i < d.adaptor_blocks; ++i)
            if ((rc = load_ada_block(e, m, "audio_adaptor.blocks." + std::to_string(i), e->blocks[i], staging)))
                return rc;
        return FA_OK;
    };
    int rc = run();
    if (cudaStreamSynchronize(e->stream) != cudaSuccess && rc == FA_OK) rc = fail("weight upload", FA_ERR_CUDA);
    if (staging) cudaFree(staging);
    if (rc == FA_OK) e->loaded = true;
    return rc;
}

// The whole encoder + adaptor over the rows in in_raw (T rows, n_tiles attention tiles
// in tiles_dev), leaving the embeddings in x. Launch order only; no synchronisation.
static void enqueue(fa_encoder* e, int T, int n_tiles, cudaStream_t s) {
    const fa_encoder_desc& d = e->d;
    const int kin = pad64(d.input_dim);
    cudaStream_t saved = e->stream;
    e->stream = s;
    fa::set_launch_pdl(true);
    fa::launch_enc_scale(e->in_raw, T, d.input_dim, kin, std::sqrt((float)d.output_size), e->in0, s);
    // each layer's last launch also applies the norm that comes next: the following layer's
    // norm1, after_norm (in place) after the main layers, tp_norm (in place, and the
    // adaptor's f16 input) after the tp layers
    auto norm1_of = [](const EncLayer& L) { return LnTail{L.n1w, L.n1b, 1e-5f, 0, true}; };
    const LnTail after{e->after_w, e->after_b, 1e-5f, 1, false};
    const LnTail tp{e->tp_w, e->tp_b, 1e-5f, 1, true};
    const size_t n_main = e->main_l.size(), n_tp = e->tp_l.size();
    enc_layer(e, e->e0, T, n_tiles, false, e->in0, kin, false, n_main ? norm1_of(e->main_l[0]) : after);
    for (size_t i = 0; i < n_main; ++i)
        enc_layer(e, e->main_l[i], T, n_tiles, true, e->x, d.output_size, true,
                  i + 1 < n_main ? norm1_of(e->main_l[i + 1]) : after);
    if (n_tp == 0)   // tp_norm on its own
        fa::launch_enc_resid_ln(e->x, d.output_size, d.output_size, nullptr, -1, T, nullptr, nullptr, 0, e->tp_w,
                                e->tp_b, 1e-5f, 1, e->xn, e->xn_lo, d.output_size, s);
    for (size_t i = 0; i < n_tp; ++i)   // the first one normalises after_norm's output itself
        enc_layer(e, e->tp_l[i], T, n_tiles, true, e->x, d.output_size, i > 0,
                  i + 1 < n_tp ? norm1_of(e->tp_l[i + 1]) : tp);
    int sp = gemm(e, e->xn, e->xn_lo, T, e->lin1);
    fa::launch_enc_bias_act(e->part, sp, T, e->lin1.n, e->lin1.b, 1, nullptr, e->hid, e->hid_lo, e->n_sm, s);
    sp = gemm(e, e->hid, e->hid_lo, T, e->lin2);
    // x = lin2 output, then the first block's norm1 in the same launch
    const size_t n_blk = e->blocks.size();
    auto ada_norm1 = [](const AdaBlock& B) { return LnTail{B.n1w, B.n1b, 1e-12f, 0, true}; };
    const LnTail none{};
    const LnTail t0 = n_blk ? ada_norm1(e->blocks[0]) : none;
    fa::launch_enc_resid_ln(e->x, d.adaptor_output, d.adaptor_output, e->part, sp, T, e->lin2.b, nullptr, 0, t0.w,
                            t0.b, t0.eps, 0, t0.to_xn ? e->xn : nullptr, t0.to_xn ? e->xn_lo : nullptr,
                            t0.to_xn ? d.adaptor_output : 0, s);
    for (size_t i = 0; i < n_blk; ++i)
        ada_block(e, e->blocks[i], T, n_tiles, true, i + 1 < n_blk ? ada_norm1(e->blocks[i + 1]) : none);
    fa::set_launch_pdl(false);
    e->stream = saved;
}

// n_utt utterances of frames[i] rows each, concatenated: lfr [sum][input_dim] f32 in, embeds
// [sum][adaptor_output] f32 out; host or device pointers. The forward of a row layout
// (rows, tiles) is captured once as a CUDA graph and replayed.
extern "C" int fa_encoder_forward_batch(fa_encoder* e, int n_utt, const int* frames, const float* lfr, float* embeds,
                                        void* stream) {
    fa::NvtxRange nv("fa_encoder_forward_batch");
    if (!e || n_utt < 1 || !frames || !lfr || !embeds)
        return fail("fa_encoder_forward_batch: bad argument", FA_ERR_INVALID_ARG);
    if (!e->loaded) return fail("encoder weights not loaded", FA_ERR_NOT_READY);
    long total = 0;
    for (int i = 0; i < n_utt; ++i) {
        if (frames[i] < 1) return fail("fa_encoder_forward_batch: every utterance needs >= 1 frame", FA_ERR_INVALID_ARG);
        total += frames[i];
    }
    if (total > e->d.max_frames)
        return fail("fa_encoder_forward_batch: " + std::to_string(total) + " frames in all, max_frames = " +
                        std::to_string(e->d.max_frames),
                    FA_ERR_CAPACITY);
    cudaSetDevice(e->device);
    const fa_encoder_desc& d = e->d;
    const int T = (int)total;
    int n_tiles = 0;
    for (int i = 0, r = 0; i < n_utt; r += frames[i], ++i) {
        for (int t = 0; t < frames[i]; ++t) e->h_seg[r + t] = make_int2(r, r + frames[i]);
        for (int t = 0; t < frames[i]; t += fa::kEncAttRows)
            e->h_tiles[n_tiles++] = make_int4(r + t, std::min(fa::kEncAttRows, frames[i] - t), r, frames[i]);
    }
    cudaStream_t s = stream ? (cudaStream_t)stream : e->stream;
    cudaError_t ce = cudaMemcpyAsync(e->seg_dev, e->h_seg, sizeof(int2) * T, cudaMemcpyHostToDevice, s);
    if (ce == cudaSuccess)
        ce = cudaMemcpyAsync(e->tiles_dev, e->h_tiles, sizeof(int4) * n_tiles, cudaMemcpyHostToDevice, s);
    if (ce == cudaSuccess)
        ce = cudaMemcpyAsync(e->in_raw, lfr, sizeof(float) * (size_t)T * d.input_dim, cudaMemcpyDefault, s);
    if (ce != cudaSuccess) return fail(std::string("encoder input: ") + cudaGetErrorString(ce), FA_ERR_CUDA);
    if (e->use_graphs) {
        auto key = std::make_pair(T, n_tiles);
        auto it = e->graphs.find(key);
        if (it == e->graphs.end()) {
            cudaGraph_t g = nullptr;
            ce = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
            if (ce == cudaSuccess) {
                enqueue(e, T, n_tiles, s);
                ce = cudaStreamEndCapture(s, &g);
            }
            cudaGraphExec_t ex = nullptr;
            if (ce == cudaSuccess) ce = cudaGraphInstantiate(&ex, g, 0);
            if (g) cudaGraphDestroy(g);
            if (ce != cudaSuccess) return fail(std::string("encoder graph: ") + cudaGetErrorString(ce), FA_ERR_CUDA);
            if (e->graphs.size() >= 32) {
                for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
                e->graphs.clear();
            }
            it = e->graphs.emplace(key, ex).first;
        }
        ce = cudaGraphLaunch(it->second, s);
    } else {
        enqueue(e, T, n_tiles, s);
        ce = cudaGetLastError();
    }
    if (ce == cudaSuccess)
        ce = cudaMemcpyAsync(embeds, e->x, sizeof(float) * (size_t)T * d.adaptor_output, cudaMemcpyDefault, s);
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(e->h_err, e->err_dev, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
    if (ce != cudaSuccess) return fail(std::string("encoder forward: ") + cudaGetErrorString(ce), FA_ERR_CUDA);
    if (*e->h_err) {
        cudaMemsetAsync(e->err_dev, 0, sizeof(int), s);
        cudaStreamSynchronize(s);
        return fail("encoder: a bounded device wait gave up", FA_ERR_TIMEOUT);
    }
    return FA_OK;
}

// One utterance, device (or host) pointers, on `stream` (NULL: the encoder's stream);
// returns when done.
extern "C" int fa_encoder_forward_dev(fa_encoder* e, const float* lfr_dev, int T, float* embeds_dev, void* stream) {
    if (T < 1) return fail("fa_encoder_forward: T must be >= 1", FA_ERR_INVALID_ARG);
    return fa_encoder_forward_batch(e, 1, &T, lfr_dev, embeds_dev, stream);
}

// One utterance, host in, host out.
extern "C" int fa_encoder_forward(fa_encoder* e, const float* lfr, int T, float* embeds) {
    return fa_encoder_forward_dev(e, lfr, T, embeds, nullptr);
}

extern "C" int fa_encoder_set_graphs(fa_encoder* e, int enable) {
    if (!e) return fail("fa_encoder_set_graphs: NULL encoder", FA_ERR_INVALID_ARG);
    e->use_graphs = enable != 0;
    return FA_OK;
}
