// Q8_0 weights as the GEMM kernels read them: the GGUF blocks split into planes.
//
// A GGUF Q8_0 matrix [N][K] is N rows of K/32 blocks of 34 B: an f16 scale d and 32
// int8 values q, weight = d * q (tools/hf_convert_ggml_q8.py:354-381). On the device
// the same numbers live in three planes of one buffer, losslessly:
//   q    int8 [N][K]        the block values, row-major (TMA tiles, 16 B vector loads)
//   d_t  f16  [K/32][N]     the block scales, block-major: one TMA box carries the
//                           scales of 128 consecutive rows for a run of blocks
//   d_r  f16  [N][K/32]     the same scales row-major, for the CUDA-core kernel, whose
//                           warps walk one row's blocks
// A kernel reads q and one of the two scale planes, so the bytes it streams per weight
// are the GGUF file's 34/32. Stacked matrices (Wq|Wk|Wv, gate|up) are stacked along N in
// every plane.
//
// Exact dequantisation for the tensor cores: d*q has at most 11 + 7 significant bits, so
// it is the sum of two f16 values, hi = f16(d*q) and lo = d*q - hi, both exact (lo is a
// multiple of d's last place and at most 2^6 of them, representable down to the f16
// subnormals). The tensor-core kernels expand a tile of q into an f16 (hi, lo) pair (in TMEM
// as the MMA's A operand, or in shared memory) and multiply it with the activation pair; the
// CUDA-core kernels sum q * x in fp32 and multiply by d once. No weight is rounded.
#pragma once

#include "fa_common.cuh"

namespace fa {

struct Q8Planes {
    const int8_t* q = nullptr;
    const __half* d_t = nullptr;
    const __half* d_r = nullptr;
};

// Byte offsets of the planes inside one buffer (256 B aligned for N % 4 == 0, K % 64 == 0).
__host__ __device__ inline size_t q8p_dt_offset(int N, int K) { return (size_t)N * K; }
__host__ __device__ inline size_t q8p_dr_offset(int N, int K) { return (size_t)N * K + (size_t)N * (K / kQK) * 2; }
__host__ __device__ inline size_t q8p_bytes(int N, int K) { return (size_t)N * K + (size_t)N * (K / kQK) * 4; }

inline Q8Planes q8p_view(const void* base, int N, int K) {
    Q8Planes p;
    const unsigned char* b = static_cast<const unsigned char*>(base);
    p.q = reinterpret_cast<const int8_t*>(b);
    p.d_t = reinterpret_cast<const __half*>(b + q8p_dt_offset(N, K));
    p.d_r = reinterpret_cast<const __half*>(b + q8p_dr_offset(N, K));
    return p;
}

// 8 consecutive int8 values (two 32-bit words) times their block scale d (both halves of
// d2) -> 8 f16 hi = f16(d*q) and 8 f16 lo = d*q - hi, exactly. int8 -> f16 by the
// exponent trick: the byte q + 128 under the f16 exponent of 1024 reads as 1024 + q + 128,
// and subtracting 1152 leaves q. hi is the correctly rounded product; the fused
// multiply-add forms d*q - hi before its single rounding, and that difference is
// representable, so lo is exact.
__device__ __forceinline__ void q8x8_to_hilo(uint32_t w0, uint32_t w1, __half2 d2, uint4& hi, uint4& lo) {
    const uint32_t v0 = w0 ^ 0x80808080u, v1 = w1 ^ 0x80808080u;
    uint32_t h[4];
    h[0] = __byte_perm(v0, 0x64646464u, 0x4140);
    h[1] = __byte_perm(v0, 0x64646464u, 0x4342);
    h[2] = __byte_perm(v1, 0x64646464u, 0x4140);
    h[3] = __byte_perm(v1, 0x64646464u, 0x4342);
    const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));   // 1152
    uint32_t oh[4], ol[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __half2 qv = __hsub2(*reinterpret_cast<const __half2*>(&h[j]), bias);
        const __half2 p = __hmul2(qv, d2);
        const __half2 r = __hfma2(qv, d2, __hneg2(p));
        oh[j] = *reinterpret_cast<const uint32_t*>(&p);
        ol[j] = *reinterpret_cast<const uint32_t*>(&r);
    }
    hi = make_uint4(oh[0], oh[1], oh[2], oh[3]);
    lo = make_uint4(ol[0], ol[1], ol[2], ol[3]);
}

// Byte offset of 16-byte chunk c (0..7) of row r in a K-major tile of 128 B rows stored
// in 128 B swizzle atoms (8 rows x 128 B, chunk index XOR row % 8): the layout a TMA
// SWIZZLE_128B box has and the UMMA descriptor of smem_desc_k128 reads.
__device__ __forceinline__ uint32_t swz128_off(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void sts128(void* p, const uint4& v) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(smem_u32(p)), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ uint2 lds64(const void* p) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(smem_u32(p)));
    return v;
}

// Expands one stage of q [rows][64] int8 (plain 64 B rows) with scales d [2][d_ld] (block
// b of row r at d[b * d_ld + r]) into 128 B-swizzled f16 tiles w_hi / w_lo [rows][64].
// `t` is the caller's index among `n_threads` cooperating threads; rows * 8 chunks of 8
// values are shared out so that each warp reads 256 contiguous bytes of q per step.
template <int ROWS>
__device__ __forceinline__ void q8_stage_to_hilo(const int8_t* q, const __half* d, int d_ld, __half* w_hi,
                                                 __half* w_lo, int t, int n_threads) {
    unsigned char* hi = reinterpret_cast<unsigned char*>(w_hi);
    unsigned char* lo = reinterpret_cast<unsigned char*>(w_lo);
    for (int id = t; id < ROWS * 8; id += n_threads) {
        const int r = id >> 3, c = id & 7;
        const uint2 qv = lds64(q + r * 64 + c * 8);
        const __half dv = d[(c >> 2) * d_ld + r];
        uint4 h, l;
        q8x8_to_hilo(qv.x, qv.y, __halves2half2(dv, dv), h, l);
        const uint32_t off = swz128_off(r, c);
        sts128(hi + off, h);
        sts128(lo + off, l);
    }
}

// Host: repack GGUF Q8_0 blocks [N][K/32][34 B] into the planes of a stacked matrix of
// n_total rows at row offset r0 (k_small.cu); with interleave > 0 source row n goes to
// r0 + (n / interleave) * 2 * interleave + n % interleave (two matrices in alternating blocks).
void launch_repack_q8_planes(const uint8_t* raw, int N, int K, int r0, int n_total, void* planes, cudaStream_t s,
                             int interleave = 0);

}  // namespace fa
