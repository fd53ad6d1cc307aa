// Shared definitions for the sm_100a decoder kernels of libfunasr_dec.
//
// Data layout in HBM (one decoder, one GPU):
//   KV page pool   : [layer][page][kv_head][K|V][token 16][head_dim] f16.
//                    One page holds 16 tokens of one sequence for every KV head:
//                    8 * 2 * 16 * 128 * 2 B = 64 KiB per layer. The (K,V) pair of one
//                    head in one page is one contiguous 8 KiB run, so a single bulk
//                    copy moves it.
//   block table    : int32 [seq_slot][page_index]; token p of slot s sits in page
//                    block_table[s][p / 16] at in-page token p % 16.
//   Q8_0 weights   : the GGUF blocks ([f16 d][32 x int8]) split into planes, nothing rounded
//                    (q8_planes.cuh): q int8 [N][K], scales f16 [K/32][N] and [N][K/32].
//                    The encoder's weights are f16(d * q) [N][K], row-major, TMA-able.
//   RoPE table     : float2 [pos][head_dim/2] = (cos, sin), computed on the host in double.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <utility>

namespace fa {

constexpr int kPageTokens = 16;
constexpr int kQK = 32;            // Q8_0 block length
constexpr int kQBytes = 34;        // Q8_0 block bytes

// Device error codes written to the per-context error word.
constexpr int kDevErrTimeout = 1;     // a bounded mbarrier wait gave up
constexpr int kDevErrBadPage = 2;     // block table entry outside the pool
constexpr int kDevErrBadPos = 4;      // position outside the RoPE table
constexpr int kDevErrBadLen = 8;      // sequence length or output row range outside its bounds

// Upper bound for one mbarrier wait, in nanoseconds of %globaltimer.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase. Returns false (and leaves the barrier as
// is) once limit_ns (kWaitLimitNs unless given) has passed without the phase
// completing.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  unsigned long long limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > limit_ns) return false;
    }
}

// One bulk (non-tensor) global -> shared copy whose completion is counted on `bar`.
// dst, src 16 B aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ uint4 lds128(const void* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_u32(p)));
    return v;
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t u) {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    return __half22float2(h);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
    const int n = pred ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(n)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// y as the f16 pair the GEMMs read: hi = f16(y), lo = f16(y - hi) (lo may be omitted)
__device__ __forceinline__ void split_store(float y, __half* hi, __half* lo, size_t i) {
    const __half h = __float2half_rn(y);
    hi[i] = h;
    if (lo) lo[i] = __float2half_rn(__fsub_rn(y, __half2float(h)));
}

// SwiGLU of one gate / up pair: silu(g) * u = g / (1 + exp(-g)) * u
__device__ __forceinline__ float silu_mul(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

__device__ __forceinline__ void record_error(int* err, int code) {
    if (err) atomicOr(err, code);
}

// Programmatic dependent launch. pdl_trigger lets the next kernel of the stream
// start its prologue once every CTA of this one has started; pdl_wait blocks
// until the previous kernel has completed and its writes are visible. Both are
// no-ops for a kernel launched without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Host: launches of the decode-step kernels go through launch_k, which adds the
// programmatic-serialization attribute while launch_pdl_enabled() is set (the
// step enqueue sets it for its own launches; everything else launches plainly).
bool launch_pdl_enabled();
void set_launch_pdl(bool on);

template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = launch_pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace fa
