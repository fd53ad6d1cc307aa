// Kernel (2b): causal paged GQA attention for prefill chunks on the 5th-generation
// tensor cores.
//
// Replaces, for rows of a prefill chunk (seq_len > 1 in compute/llm_ops_gpu.cpp:
// 98-143), the per-row decode kernel, which reads a sequence's whole context once for
// every row. Here a CTA takes a tile of up to 64 consecutive rows of one sequence and
// one KV head: its 128 query vectors (64 rows x the 2 query heads of the KV head) form
// the M = 128 side of every MMA, so each K/V page of the context is read once per tile
// instead of once per row.
//
// Per key block of 64 tokens (4 pages):
//   S  = Q . K^T       tcgen05.mma kind::f16, M 128, N 64, K 128, f32 accumulator in TMEM
//   P  = exp2(S*log2e - m)    one query vector per thread, fp32, causal mask key <= pos
//   O += P . V         tcgen05.mma, M 128, N 128 (head dims), K 64 (tokens), V MN-major
// Q and P enter the MMAs as f16 pairs (hi = f16(x), lo = f16(x - hi)), two MMAs into
// one accumulator, so products carry ~22 bits of the fp32 operands; K and V are the f16
// cache values themselves. Softmax is online with a lazy running maximum: O and the sum
// are rescaled only when a block's maximum exceeds the running one by more than 2^8,
// so most blocks never touch O (P stays <= 256, exact as an f16 pair).
//
// Roles (192 threads): warp 0 issues TMA loads of the K/V pages (2-D tensor map over
// the page pool, 16-row x 64-column boxes, 128 B swizzle) into a 3-stage ring; warp 1
// allocates TMEM (two 64-column S buffers + a 128-column O accumulator) and issues the
// MMAs; warps 2-5 stage Q, run the softmax and write the outputs. Every mbarrier wait
// is bounded; on a timeout the CTA records the error, drains its copies and MMAs and
// frees TMEM.
//
// Roofline: tensor pipe. Per tile and KV head, 4 x 2 x 128 x 128 x n_kv flops (QK and
// PV, hi and lo) against n_kv x 512 B of K/V read.
#include "fa_kernels.cuh"
#include "tc_common.cuh"

namespace fa {

namespace {

constexpr int D = 128;
constexpr int KB = 64;                    // keys per block
constexpr int PST = 3;                    // K/V ring stages
constexpr int THREADS = 192;
constexpr uint32_t BOX_BYTES = 16 * 64 * 2;             // one page, one 64-dim half
constexpr uint32_t STAGE_BYTES = 4 * 2 * 2 * BOX_BYTES; // 4 pages x (K, V) x 2 halves = 32 KiB
constexpr uint32_t TMEM_COLS = 256;                     // S0 [0,64) S1 [64,128) O [128,256)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescale = 8.0f;                        // lazy-max threshold, log2 units
constexpr int PAGE_LIST = 2048;                         // block-table entries staged in shared memory

struct PfSmem {
    __half q_hi[2][128 * 64];       // [dim half][128 query vectors][64 dims], swizzled
    __half q_lo[2][128 * 64];
    __half k[PST][2][KB * 64];      // [stage][dim half][64 tokens][64 dims]
    __half v[PST][2][KB * 64];
    __half p_hi[128 * 64];          // [128 query vectors][64 tokens]
    __half p_lo[128 * 64];
    int pages[PAGE_LIST];           // the tile's block-table entries [0, last page]
    uint64_t kv_full[PST];
    uint64_t kv_empty[PST];
    uint64_t s_full[2];
    uint64_t p_ready;
    uint64_t o_done;
    uint64_t q_ready;
    uint64_t drain;
    uint32_t tmem_base;
    int err;
    int issued;
    int consumed;
};

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` in a [rows][128 B] tile
// with 128 B swizzle (chunk index XOR row within the 8-row atom).
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
    return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

// Eight consecutive outputs from offset o (a multiple of 8): 16 B stores of the f16
// pair and/or two 16 B stores of f32.
__device__ __forceinline__ void store_pf8(const PrefillAttnArgs& a, size_t o, const float (&v)[8]) {
    if (a.out16) {
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const __half h0 = __float2half_rn(v[2 * e]), h1 = __float2half_rn(v[2 * e + 1]);
            hi[e] = pack_h2(h0, h1);
            lo[e] = pack_h2(__float2half_rn(__fsub_rn(v[2 * e], __half2float(h0))),
                            __float2half_rn(__fsub_rn(v[2 * e + 1], __half2float(h1))));
        }
        *reinterpret_cast<uint4*>(a.out16 + o) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        if (a.out16_lo) *reinterpret_cast<uint4*>(a.out16_lo + o) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    if (a.out32) {
        *reinterpret_cast<float4*>(a.out32 + o) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(a.out32 + o + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
}

__global__ void __launch_bounds__(THREADS, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tm_pool, const PrefillAttnArgs a) {
    extern __shared__ unsigned char smem_raw[];
    PfSmem& S = *reinterpret_cast<PfSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int h = blockIdx.x;                       // KV head

    if (threadIdx.x == 0) {
        tma_prefetch_desc(&tm_pool);
        for (int s = 0; s < PST; ++s) {
            mbar_init(&S.kv_full[s], 1);
            mbar_init(&S.kv_empty[s], 1);
        }
        mbar_init(&S.s_full[0], 1);
        mbar_init(&S.s_full[1], 1);
        mbar_init(&S.p_ready, 128);
        mbar_init(&S.o_done, 1);
        mbar_init(&S.q_ready, 128);
        mbar_init(&S.drain, 1);
        S.err = 0;
        S.issued = 0;
        S.consumed = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&S.tmem_base)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;
    pdl_trigger();
    pdl_wait();

    const int2 tile = a.tiles[blockIdx.y];          // (first row, rows)
    const int row0 = tile.x;
    const int n_rows = tile.y;
    const bool bad_tile = row0 < 0 || n_rows < 1 || n_rows > 64 || row0 + n_rows > a.M;
    // keys [0, pos of the tile's last row]
    const int pos_last = bad_tile ? 0 : a.pos[row0 + n_rows - 1];
    const bool bad = bad_tile || pos_last < 0 || pos_last / kPageTokens >= a.bt_stride;
    const int n_blocks = pos_last / KB + 1;
    const int slot = bad ? 0 : a.slot[row0];
    if (bad && threadIdx.x == 0) record_error(a.err, kDevErrBadPos);

    if (bad) {
        // nothing issued: fall through to the TMEM release
    } else if (warp == 0) {
        const int* bt = a.block_table + (size_t)slot * a.bt_stride;
        const int last_page = pos_last / kPageTokens;
        for (int i = lane; i <= last_page && i < PAGE_LIST; i += 32) S.pages[i] = bt[i];
        __syncwarp();
        if (lane == 0) {
            bool ok = true;
            for (int j = 0; j < n_blocks; ++j) {
                const int s = j % PST;
                if (j >= PST && !mbar_wait_bounded(&S.kv_empty[s], (uint32_t)((j / PST) - 1) & 1u)) {
                    ok = false;
                    break;
                }
                mbar_arrive_expect_tx(&S.kv_full[s], STAGE_BYTES);
                for (int q = 0; q < 4; ++q) {
                    // pages past the last one repeat it: finite data under a zero weight
                    const int pi = min(j * 4 + q, last_page);
                    int pg = pi < PAGE_LIST ? S.pages[pi] : bt[pi];
                    if (pg < 0 || pg >= a.n_pages) {
                        record_error(a.err, kDevErrBadPage);
                        pg = 0;
                    }
                    const int y = a.pool_row0 + ((pg * a.Hkv + h) * 2) * kPageTokens;
                    tma_load_2d(&S.k[s][0][q * 16 * 64], &tm_pool, 0, y, &S.kv_full[s]);
                    tma_load_2d(&S.k[s][1][q * 16 * 64], &tm_pool, 64, y, &S.kv_full[s]);
                    tma_load_2d(&S.v[s][0][q * 16 * 64], &tm_pool, 0, y + kPageTokens, &S.kv_full[s]);
                    tma_load_2d(&S.v[s][1][q * 16 * 64], &tm_pool, 64, y + kPageTokens, &S.kv_full[s]);
                }
                S.issued = j + 1;
            }
            if (!ok) S.err = 1;
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t kIdS = idesc_f16(128, KB, false, false);
            constexpr uint32_t kIdPV = idesc_f16(128, D, false, true);
            bool ok = mbar_wait_bounded(&S.q_ready, 0);
            for (int j = 0; ok && j <= n_blocks; ++j) {
                if (j < n_blocks) {
                    const int s = j % PST;
                    if (!mbar_wait_bounded(&S.kv_full[s], (uint32_t)(j / PST) & 1u)) { ok = false; break; }
                    S.consumed = j + 1;
                    tc_fence_after();
                    const uint32_t d_s = tmem + (uint32_t)((j & 1) * KB);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const int hf = kk >> 2;
                        const uint32_t off = (uint32_t)((kk & 3) * 32) >> 4;
                        const uint64_t db = smem_desc_k128(S.k[s][hf]) + off;
                        tc_mma_f16(d_s, smem_desc_k128(S.q_hi[hf]) + off, db, kIdS, kk > 0 ? 1u : 0u);
                        tc_mma_f16(d_s, smem_desc_k128(S.q_lo[hf]) + off, db, kIdS, 1u);
                    }
                    tc_commit(&S.s_full[j & 1]);
                }
                if (j >= 1) {
                    const int jp = j - 1;
                    const int sp = jp % PST;
                    if (!mbar_wait_bounded(&S.p_ready, (uint32_t)jp & 1u)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t d_o = tmem + 128;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t db = smem_desc_mn128(&S.v[sp][0][kk * 16 * 64], 64 * 64 * 2);
                        const uint32_t off = (uint32_t)(kk * 32) >> 4;
                        tc_mma_f16(d_o, smem_desc_k128(S.p_hi) + off, db, kIdPV, (jp > 0 || kk > 0) ? 1u : 0u);
                        tc_mma_f16(d_o, smem_desc_k128(S.p_lo) + off, db, kIdPV, 1u);
                    }
                    tc_commit(&S.kv_empty[sp]);
                    tc_commit(&S.o_done);
                }
            }
            if (!ok) S.err = 1;
            tc_commit(&S.drain);
            if (!mbar_wait_bounded(&S.drain, 0)) S.err = 1;
        }
        __syncwarp();
    } else {
        // softmax / epilogue: thread t owns TMEM lane t = query vector t (a warp may
        // only touch TMEM lanes 32 * (warp % 4) ..)
        const int q = warp & 3;
        const int t = 32 * q + lane;
        const int r = t & 63;                         // row within the tile
        const int hq = t >> 6;                        // query head 2h + hq
        const bool live = r < n_rows;
        const int row = row0 + r;
        const int pos_r = live ? a.pos[row] : -1;
        const int H = 2 * h + hq;
        // stage Q (pre-scaled by 1/sqrt(128)) as an f16 pair, swizzled K-major: each
        // warp loads its 32 query vectors, one 512 B vector per instruction (lane l
        // takes dims 4l..4l+3), eight loads in flight at a time
        {
            const int hf = lane >> 4;               // dims 64*hf ..
            const int chunk = (lane & 15) >> 1;     // 16 B chunk within the 128 B row
            const uint32_t sub = (uint32_t)(lane & 1) * 8;
#pragma unroll 1
            for (int v0 = 0; v0 < 32; v0 += 8) {
                float4 x[8];
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int tv = 32 * q + v0 + k;            // query vector = TMEM lane
                    const int rr = tv & 63;
                    x[k] = rr < n_rows ? *reinterpret_cast<const float4*>(
                                             a.q + ((size_t)(row0 + rr) * a.Hq + 2 * h + (tv >> 6)) * D + 4 * lane)
                                       : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                }
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const int tv = 32 * q + v0 + k;
                    const __half h0 = __float2half_rn(x[k].x), h1 = __float2half_rn(x[k].y);
                    const __half h2 = __float2half_rn(x[k].z), h3 = __float2half_rn(x[k].w);
                    const uint2 hi = make_uint2(pack_h2(h0, h1), pack_h2(h2, h3));
                    const uint2 lo = make_uint2(pack_h2(__float2half_rn(__fsub_rn(x[k].x, __half2float(h0))),
                                                        __float2half_rn(__fsub_rn(x[k].y, __half2float(h1)))),
                                                pack_h2(__float2half_rn(__fsub_rn(x[k].z, __half2float(h2))),
                                                        __float2half_rn(__fsub_rn(x[k].w, __half2float(h3)))));
                    const uint32_t off = sw128(tv, chunk) + sub;
                    *reinterpret_cast<uint2*>(reinterpret_cast<unsigned char*>(S.q_hi[hf]) + off) = hi;
                    *reinterpret_cast<uint2*>(reinterpret_cast<unsigned char*>(S.q_lo[hf]) + off) = lo;
                }
            }
            fence_proxy_async_smem();
            mbar_arrive(&S.q_ready);
        }

        float m_run = -INFINITY, l_run = 0.0f;
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        bool ok = true;
        for (int j = 0; j < n_blocks; ++j) {
            const bool got = mbar_wait_bounded(&S.s_full[j & 1], (uint32_t)(j >> 1) & 1u);
            if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
            tc_fence_after();
            uint32_t sv[64];
            const uint32_t ts = tmem + lane_base + (uint32_t)((j & 1) * KB);
            TMEM_LD_X32(ts, sv);
            TMEM_LD_X32(ts + 32, (sv + 32));
            tmem_wait_ld();
            // scores in log2 units with the causal mask
            const int key0 = j * KB;
            float bmax = -INFINITY;
#pragma unroll
            for (int c = 0; c < 64; ++c) {
                const float x = key0 + c <= pos_r ? __uint_as_float(sv[c]) * kLog2e : -INFINITY;
                sv[c] = __float_as_uint(x);
                bmax = fmaxf(bmax, x);
            }
            float alpha = 1.0f;
            bool rescale = false;
            if (m_run == -INFINITY) {
                m_run = bmax;                        // first block with a key (O still empty)
            } else if (bmax > m_run + kRescale) {
                alpha = exp2f(m_run - bmax);
                m_run = bmax;
                rescale = true;
            }
            // P as f16 pairs, row t of the swizzled [128][64] tiles
            float psum = 0.0f;
            uint32_t ph[32], pl[32];
#pragma unroll
            for (int c = 0; c < 64; c += 2) {
                const float x0 = __uint_as_float(sv[c]), x1 = __uint_as_float(sv[c + 1]);
                const float p0 = m_run == -INFINITY ? 0.0f : exp2f(x0 - m_run);
                const float p1 = m_run == -INFINITY ? 0.0f : exp2f(x1 - m_run);
                psum += p0 + p1;
                const __half h0 = __float2half_rn(p0), h1 = __float2half_rn(p1);
                ph[c >> 1] = pack_h2(h0, h1);
                pl[c >> 1] = pack_h2(__float2half_rn(__fsub_rn(p0, __half2float(h0))),
                                     __float2half_rn(__fsub_rn(p1, __half2float(h1))));
            }
            l_run = l_run * alpha + psum;
            // O and the P tile are free once the previous block's P.V has completed
            if (j >= 1) {
                const bool od = mbar_wait_bounded(&S.o_done, (uint32_t)(j - 1) & 1u);
                if (!__all_sync(0xffffffffu, od)) { ok = false; break; }
                tc_fence_after();
                if (__any_sync(0xffffffffu, rescale)) {
                    const uint32_t to = tmem + lane_base + 128;
#pragma unroll 1
                    for (int c = 0; c < 128; c += 32) {
                        uint32_t ov[32];
                        TMEM_LD_X32(to + c, ov);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * alpha);
                        TMEM_ST_X32(to + c, ov);
                    }
                    tmem_wait_st();
                }
            }
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const uint32_t off = sw128(t, c);
                *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(S.p_hi) + off) =
                    make_uint4(ph[4 * c], ph[4 * c + 1], ph[4 * c + 2], ph[4 * c + 3]);
                *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(S.p_lo) + off) =
                    make_uint4(pl[4 * c], pl[4 * c + 1], pl[4 * c + 2], pl[4 * c + 3]);
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(&S.p_ready);
        }
        if (ok) {
            const bool od = mbar_wait_bounded(&S.o_done, (uint32_t)(n_blocks - 1) & 1u);
            if (!__all_sync(0xffffffffu, od)) ok = false;
        }
        if (!ok) {
            if (lane == 0) S.err = 1;
        } else {
            tc_fence_after();
            const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
            const uint32_t to = tmem + lane_base + 128;
            const size_t obase = ((size_t)row * a.Hq + H) * D;
#pragma unroll 1
            for (int c = 0; c < 128; c += 32) {
                uint32_t ov[32];
                TMEM_LD_X32(to + c, ov);
                tmem_wait_ld();
                if (live) {
#pragma unroll
                    for (int e = 0; e < 32; e += 8) {
                        float o[8];
#pragma unroll
                        for (int k = 0; k < 8; ++k) o[k] = __uint_as_float(ov[e + k]) * inv;
                        store_pf8(a, obase + c + e, o);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (S.err) {
        if (threadIdx.x == 0) {
            record_error(a.err, kDevErrTimeout);
            for (int j = S.consumed; j < S.issued; ++j)
                (void)mbar_wait_bounded(&S.kv_full[j % PST], (uint32_t)(j / PST) & 1u);
        }
        __syncthreads();
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

}  // namespace

size_t prefill_attn_smem_bytes() { return sizeof(PfSmem) + 1024; }

void configure_prefill_attention() {
    cudaFuncSetAttribute(prefill_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)prefill_attn_smem_bytes());
}

bool make_pool_map(CUtensorMap* tm, const void* pool, long long total_rows) {
    return make_map(tm, pool, D, total_rows, 64, kPageTokens, true);
}

void launch_prefill_attention(const CUtensorMap& tm_pool, const PrefillAttnArgs& a, cudaStream_t s) {
    launch_k(prefill_attn_kernel, dim3(a.Hkv, a.n_tiles), dim3(THREADS), prefill_attn_smem_bytes(), s, tm_pool, a);
}

}  // namespace fa
