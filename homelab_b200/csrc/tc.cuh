// tc.cuh - FP8 GEMV/GEMM for decode batches on the 5th-generation tensor cores.
//
// y[t, n] = sum_k x[t, k] * e4m3(q[n, k]) * scale(n, k), fp32 accumulation: the
// arithmetic of the reference's gemv_impl<T, true> (ops.cu:338-440); only the
// summation order differs.
//
// The weights never pass through registers: TMA copies 128 x 128 e4m3 tiles of
// q (row-major) into a shared-memory ring in the canonical K-major 128-byte
// swizzled layout, and tcgen05.mma (kind::f8f6f4, M = 128, K = 32) reads them
// from there.  The activations enter as the B operand: every 128-column block of
// x[t] is split exactly into e4m3 terms with power-of-two scales,
//   x = s1 * q1 + s2 * q2 (+ s3 * q3 + s4 * q4 for fp32 x),
// q_i = e4m3(residual / s_i), s_i chosen so the block's largest residual lands
// in [128, 256).  A bf16 value has 8 significant bits and an e4m3 term carries
// 4, so two terms reproduce every bf16 activation within 2^14 of its block's
// largest exactly (smaller ones to within 2^-20 of the largest); fp32
// activations take four terms (16 bits).  Each (token, term) is one column of
// B (a token owns TS = 2 or 4 consecutive columns), so one MMA gives every
// term's partial dot product for a 128-row tile.  Accumulators live in tensor
// memory one K block (128 columns, one weight scale) at a time, up to four
// tiles in flight; an epilogue warpgroup folds each block into fp32 registers,
//   acc = fma(w_scale, ((s1 * D1 + s2 * D2) (+ s3 * D3) (+ s4 * D4)), acc),
// K blocks in order.
// Tiles (row block, K block) are split contiguously over the CTAs (stream-K);
// a row block split over several CTAs is summed by the last CTA to finish, in
// CTA order (deterministic), through a caller workspace.
//
// Warp roles (10 warps): 0 TMA producer, 1 MMA issuer and tensor-memory owner,
// 2-5 epilogue (warp w reads tensor-memory lanes 32*(w%4)..+31), 6-9 activation
// splitters (tile i goes to splitter (i - first tile) % 4, which streams the
// tile's 128-column slices of every token into its own shared-memory ring with
// bulk copies, its ring's depth ahead).
// Every wait is bounded and records an error code.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace oomb {

constexpr int kTcThreads = 320;
constexpr int kTcSplitters = 4;
constexpr int kTcTile = 128;                 // rows of a weight tile, and columns of a K block
constexpr int kTcTileBytes = kTcTile * kTcTile;
constexpr int kTcMaxStages = 8;              // ring depth; at least kTcSplitters (see tc_plan)
constexpr int kTcMaxT = 64;                  // tokens per launch
constexpr int kTcSplitGroup = 16;            // tokens a splitter converts at once
constexpr int kTcKSteps = kTcTile / 32;      // MMAs (K = 32 each) per tile
constexpr int kTcAccBufs = 4;                // tensor-memory accumulator buffers (tiles in flight)

enum : unsigned {
    ERR_TC_WAIT = 0x500,  // a tensor-core pipeline wait ran out (+ the waiting role)
};

struct TcParams {
    const void* x;       // [T, K] bf16 or fp32
    int T, K, nrows;
    const float* scale;  // 1x128: [nrows, K/128]; 128x128: [nrows/128, K/128]
    int layout;
    void* y;             // [T, nrows] bf16 or fp32
    int y_bf16;
    float* partial;      // [grid][2][T][128] split-K partial sums
    unsigned* counters;  // [nrows/128][4] arrivals per (row block, tensor-memory lane quarter)
    int tiles, kblocks;  // (nrows/128) * (K/128), K/128
    int q_tiles;         // q is in the packed tile layout (oomb_pack_fp8_tiles), else row-major
    int nmma;            // MMA N = T * TS rounded up to 8
    int stages;
    int nbufs;           // tensor-memory accumulator buffers in use (<= kTcAccBufs)
    int xdepth;          // x slots per splitter in use (<= kTcXDepth)
    int tmem_cols;
    unsigned* err;
};

__host__ __device__ constexpr int tc_ts(bool x_bf16) { return x_bf16 ? 2 : 4; }
__host__ __device__ constexpr int tc_terms(bool x_bf16) { return x_bf16 ? 2 : 4; }

constexpr int kTcXDepth = 2;  // x slots per splitter (at most)

// Shared memory (after aligning the base to 1024 bytes):
// [A ring: stages x 16 KB][B ring: stages x nmma*128]
// [x rings: 4 splitters x kTcXDepth x T x 128 x xbytes][x scales: stages x T*TS floats]
// [barriers][tensor-memory address]
struct TcSmem {
    size_t a_off, b_off, x_off, x_stage, sx_off, bar_off, total;
};

__host__ __device__ inline TcSmem tc_smem(int stages, int nmma, int T, int ts, int xbytes, int xdepth) {
    TcSmem m{};
    m.a_off = 0;
    m.b_off = static_cast<size_t>(stages) * kTcTileBytes;
    m.x_off = m.b_off + static_cast<size_t>(stages) * nmma * 128;
    m.x_stage = static_cast<size_t>(T) * kTcTile * xbytes;
    m.sx_off = m.x_off + static_cast<size_t>(kTcSplitters) * xdepth * m.x_stage;
    m.bar_off = (m.sx_off + static_cast<size_t>(stages) * T * ts * 4 + 7) & ~static_cast<size_t>(7);
    // a_full, a_empty, b_full, b_empty [kTcMaxStages]; x_full [4][kTcMaxStages] (kTcXDepth used);
    // mma_done, tmem_empty [kTcAccBufs]; tensor-memory address
    m.total = m.bar_off + ((4 + kTcSplitters) * kTcMaxStages + 2 * kTcAccBufs) * 8 + 16;
    return m;
}

// ---- PTX wrappers ------------------------------------------------------------------------

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_addr(dst)),
        "l"(map), "r"(smem_addr(bar)), "r"(x), "r"(y), "l"(policy)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major operand in the 128-byte swizzled
// canonical layout: 128-byte rows, 8-row groups 1024 bytes apart (stride byte
// offset 64 x 16 B), descriptor version 1, layout type 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t tc_smem_desc(uint32_t addr) {
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}

// Instruction descriptor: D fp32, A and B e4m3, both K-major, N = n, M = 128.
__host__ __device__ inline uint32_t tc_idesc(int n) {
    return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       int accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives on `bar` once every tcgen05 operation this thread issued has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                   "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Two floats to packed e4m3 (lo in the low byte), round to nearest even, saturating.
__device__ __forceinline__ uint32_t e4m3x2_from_f32(float lo, float hi) {
    unsigned short r;
    asm("{\n .reg .b16 t;\n cvt.rn.satfinite.e4m3x2.f32 t, %1, %2;\n mov.b16 %0, t;\n}" : "=h"(r) : "f"(hi), "f"(lo));
    return r;
}

// e = floor(log2(m)) - 7 (so m / 2^e lies in [128, 256)), or 0 when m == 0;
// returns 2^e and sets inv = 2^-e.
__device__ __forceinline__ float tc_term_scale(float m, float& inv) {
    int e = 0;
    if (m > 0.0f) e = max(-100, min(100, static_cast<int>((__float_as_uint(m) >> 23) & 0xff) - 127 - 7));
    inv = __int_as_float((127 - e) << 23);
    return __int_as_float((127 + e) << 23);
}

// Byte offset of (row n, K byte c) in a K-major 128-byte swizzled tile with a
// 1024-aligned base: 16-byte chunk index XOR (row mod 8).
__device__ __forceinline__ int sw128_offset(int n, int c) {
    return (n >> 3) * 1024 + (n & 7) * 128 + ((((c >> 4) ^ (n & 7)) & 7) << 4) + (c & 15);
}

// Tiles [lo, hi) of CTA c, and the CTA owning a tile.
__device__ __forceinline__ int tc_lo(int tiles, int c, int grid) {
    return static_cast<int>(static_cast<int64_t>(c) * tiles / grid);
}
__device__ __forceinline__ int tc_owner(int tiles, int tile, int grid) {
    int c = static_cast<int>(static_cast<int64_t>(tile) * grid / tiles);
    while (c + 1 < grid && tc_lo(tiles, c + 1, grid) <= tile) c++;
    while (c > 0 && tc_lo(tiles, c, grid) > tile) c--;
    return c;
}

// Row-major e4m3 q [n, k] to the packed tile layout: tile (rb, kb) of 128 x 128
// bytes is contiguous at (rb * k/128 + kb) * 16 KB, its rows 128 bytes apart.
// One CTA per tile, 16 bytes a thread.
__global__ void pack_fp8_tiles_kernel(const uint8_t* q, int k, uint8_t* tiles) {
    const int kblocks = k / kTcTile;
    const int tile = blockIdx.x, rb = tile / kblocks, kb = tile - rb * kblocks;
    for (int c = threadIdx.x; c < kTcTileBytes / 16; c += blockDim.x) {
        const int r = c / 8, col = (c % 8) * 16;
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(q + static_cast<int64_t>(rb * kTcTile + r) * k +
                                                             kb * kTcTile + col));
        *reinterpret_cast<uint4*>(tiles + static_cast<int64_t>(tile) * kTcTileBytes + r * kTcTile + col) = v;
    }
}

template <int MAXT>
__device__ __forceinline__ void tc_store_row(const TcParams& p, const float (&acc)[MAXT], int rb, int r) {
#pragma unroll
    for (int t = 0; t < MAXT; t++) {
        if (t < p.T) {
            const int64_t yi = static_cast<int64_t>(t) * p.nrows + rb * kTcTile + r;
            if (p.y_bf16) static_cast<__nv_bfloat16*>(p.y)[yi] = __float2bfloat16_rn(acc[t]);
            else static_cast<float*>(p.y)[yi] = acc[t];
        }
    }
}

template <bool XBF16, int MAXT>
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                 const TcParams p) {
    constexpr int TS = tc_ts(XBF16), TERMS = tc_terms(XBF16);
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int XB = XBF16 ? 2 : 4;
    const TcSmem L = tc_smem(p.stages, p.nmma, p.T, TS, XB, p.xdepth);
    uint8_t* a_ring = smem + L.a_off;
    uint8_t* b_ring = smem + L.b_off;
    uint8_t* x_ring = smem + L.x_off;
    float* sx_ring = reinterpret_cast<float*>(smem + L.sx_off);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar_off);
    uint64_t* a_full = bars;
    uint64_t* a_empty = bars + kTcMaxStages;
    uint64_t* b_full = bars + 2 * kTcMaxStages;
    uint64_t* b_empty = bars + 3 * kTcMaxStages;
    uint64_t* x_full = bars + 4 * kTcMaxStages;  // [splitter][x slot]
    uint64_t* mma_done = bars + (4 + kTcSplitters) * kTcMaxStages;
    uint64_t* tmem_empty = mma_done + kTcAccBufs;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_empty + kTcAccBufs);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.stages, T = p.T, nmma = p.nmma, grid = gridDim.x;
    const int lo = tc_lo(p.tiles, blockIdx.x, grid), hi = tc_lo(p.tiles, blockIdx.x + 1, grid);

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; i++) {
            mbar_init(&a_full[i], 1);
            mbar_init(&a_empty[i], 1);
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 4);
            for (int w = 0; w < kTcSplitters; w++) mbar_init(&x_full[w * kTcMaxStages + i], 1);
        }
        for (int i = 0; i < p.nbufs; i++) {
            mbar_init(&mma_done[i], 1);
            mbar_init(&tmem_empty[i], 4);
        }
        fence_barrier_init();
    }
    // B rows past the real (token, term) columns stay zero for the whole kernel
    for (int i = threadIdx.x; i < S * nmma * 32; i += kTcThreads) reinterpret_cast<uint32_t*>(b_ring)[i] = 0u;
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(p.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_launch_dependents();

    if (warp == 0) {
        // ================= TMA producer: weight tiles (independent of the previous kernel) =================
        if (lane == 0) {
            const uint64_t pol = make_evict_first_policy();
            for (int i = lo; i < hi; i++) {
                const int s = (i - lo) % S, it = (i - lo) / S;
                if (!mbar_wait(&a_empty[s], (it & 1) ^ 1, p.err, ERR_TC_WAIT + 1)) break;
                const int rb = i / p.kblocks, kb = i - rb * p.kblocks;
                mbar_arrive_expect_tx(&a_full[s], kTcTileBytes);
                if (p.q_tiles)
                    tma_load_2d(a_ring + s * kTcTileBytes, &qmap, 0, i * kTcTile, &a_full[s], pol);
                else
                    tma_load_2d(a_ring + s * kTcTileBytes, &qmap, kb * kTcTile, rb * kTcTile, &a_full[s], pol);
            }
        }
    } else if (warp >= 6) {
        // ================= activation splitters: B tiles and their term scales =================
        constexpr int SG = MAXT < kTcSplitGroup ? MAXT : kTcSplitGroup;
        const int sw = warp - 6, XD = p.xdepth;
        uint64_t* xf = x_full + sw * kTcMaxStages;
        uint8_t* xr = x_ring + static_cast<size_t>(sw) * XD * L.x_stage;
        // this splitter's m-th tile, and the bulk copies of its 128-column slices of every token
        auto my_tile = [&](int m) { return lo + sw + m * kTcSplitters; };
        auto fetch = [&](int m) {
            const int i = my_tile(m);
            if (lane == 0 && i < hi) {
                const int slot = m % XD, kb = i % p.kblocks;
                mbar_arrive_expect_tx(&xf[slot], static_cast<unsigned>(T * kTcTile * XB));
                for (int t = 0; t < T; t++) {
                    const uint8_t* src = static_cast<const uint8_t*>(p.x) +
                                         (static_cast<int64_t>(t) * p.K + static_cast<int64_t>(kb) * kTcTile) * XB;
                    bulk_g2s_plain(xr + slot * L.x_stage + t * kTcTile * XB, src, kTcTile * XB, &xf[slot]);
                }
            }
        };
        pdl_wait();
        for (int m = 0; m < XD; m++) fetch(m);
        for (int m = 0; my_tile(m) < hi; m++) {
            const int i = my_tile(m);
            const int s = (i - lo) % S, it = (i - lo) / S;
            if (!mbar_wait(&b_empty[s], (it & 1) ^ 1, p.err, ERR_TC_WAIT + 2)) break;
            if (!mbar_wait(&xf[m % XD], (m / XD) & 1, p.err, ERR_TC_WAIT + 7)) break;
            uint8_t* bt = b_ring + s * nmma * 128;
            float* sx = sx_ring + s * T * TS;
            const uint8_t* xs = xr + (m % XD) * L.x_stage;
            for (int g = 0; g < T; g += SG) {
                // lane l holds columns 4l .. 4l+3 of tokens g .. g+SG-1
                float v[SG][4];
#pragma unroll
                for (int u = 0; u < SG; u++) {
                    const int t = g + u;
                    if (t < T) {
                        if (XBF16) {
                            const uint2 w = *reinterpret_cast<const uint2*>(xs + (t * kTcTile + lane * 4) * 2);
                            v[u][0] = __uint_as_float(w.x << 16);
                            v[u][1] = __uint_as_float(w.x & 0xffff0000u);
                            v[u][2] = __uint_as_float(w.y << 16);
                            v[u][3] = __uint_as_float(w.y & 0xffff0000u);
                        } else {
                            const float4 w = *reinterpret_cast<const float4*>(xs + (t * kTcTile + lane * 4) * 4);
                            v[u][0] = w.x;
                            v[u][1] = w.y;
                            v[u][2] = w.z;
                            v[u][3] = w.w;
                        }
                    } else {
                        v[u][0] = v[u][1] = v[u][2] = v[u][3] = 0.0f;
                    }
                }
#pragma unroll
                for (int term = 0; term < TERMS; term++) {
                    float mx[SG];
#pragma unroll
                    for (int u = 0; u < SG; u++)
                        mx[u] = fmaxf(fmaxf(fabsf(v[u][0]), fabsf(v[u][1])), fmaxf(fabsf(v[u][2]), fabsf(v[u][3])));
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                        for (int u = 0; u < SG; u++) mx[u] = fmaxf(mx[u], __shfl_xor_sync(0xffffffffu, mx[u], o));
#pragma unroll
                    for (int u = 0; u < SG; u++) {
                        const int t = g + u;
                        if (t < T) {
                            float inv;
                            const float sc = tc_term_scale(mx[u], inv);
                            const uint32_t lo2 = e4m3x2_from_f32(v[u][0] * inv, v[u][1] * inv);
                            const uint32_t hi2 = e4m3x2_from_f32(v[u][2] * inv, v[u][3] * inv);
                            *reinterpret_cast<uint32_t*>(bt + sw128_offset(t * TS + term, lane * 4)) =
                                lo2 | (hi2 << 16);
                            if (lane == 0) sx[t * TS + term] = sc;
                            if (term + 1 < TERMS) {
                                // residual for the next term: exact, since q * sc carries at most 4 significant bits
                                const float2 a = e4m3x2_to_float2(static_cast<unsigned short>(lo2));
                                const float2 b = e4m3x2_to_float2(static_cast<unsigned short>(hi2));
                                v[u][0] -= a.x * sc;
                                v[u][1] -= a.y * sc;
                                v[u][2] -= b.x * sc;
                                v[u][3] -= b.y * sc;
                            }
                        }
                    }
                }
            }
            // the x slot is read and B is written: order both against the async proxy, refill the
            // x slot with this splitter's tile one ring depth ahead, hand B to the MMA
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            fetch(m + XD);
            if (lane == 0) mbar_arrive(&b_full[s]);
        }
    } else if (warp == 1) {
        // ================= MMA issuer =================
        if (lane == 0) {
            const uint32_t idesc = tc_idesc(nmma);
            for (int i = lo; i < hi; i++) {
                const int s = (i - lo) % S, it = (i - lo) / S;
                const int j = i - lo, buf = j % p.nbufs, use = j / p.nbufs;
                if (!mbar_wait(&a_full[s], it & 1, p.err, ERR_TC_WAIT + 3)) break;
                if (!mbar_wait(&b_full[s], it & 1, p.err, ERR_TC_WAIT + 4)) break;
                if (!mbar_wait(&tmem_empty[buf], (use & 1) ^ 1, p.err, ERR_TC_WAIT + 5)) break;
                tc_fence_after();
                const uint32_t a_addr = smem_addr(a_ring + s * kTcTileBytes);
                const uint32_t b_addr = smem_addr(b_ring + s * nmma * 128);
                const uint32_t d = tmem_base + static_cast<uint32_t>(buf * nmma);
#pragma unroll
                for (int k = 0; k < kTcKSteps; k++)
                    tc_mma(d, tc_smem_desc(a_addr + 32 * k), tc_smem_desc(b_addr + 32 * k), idesc, k > 0);
                tc_commit(&a_empty[s]);
                tc_commit(&mma_done[buf]);
            }
        }
    } else {
        // ================= epilogue warpgroup (warps 2..5) =================
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;  // row of the tile this thread owns
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        float acc[MAXT];
#pragma unroll
        for (int t = 0; t < MAXT; t++) acc[t] = 0.0f;
        // weight scales of this thread's row, fetched four tiles ahead
        auto tile_scale = [&](int i) {
            const int rb = i / p.kblocks, kb = i - rb * p.kblocks;
            return p.layout ? __ldg(p.scale + static_cast<int64_t>(rb) * p.kblocks + kb)
                            : __ldg(p.scale + static_cast<int64_t>(rb * kTcTile + r) * p.kblocks + kb);
        };
        float ws_ring[4];
#pragma unroll
        for (int u = 0; u < 4; u++) ws_ring[u] = lo + u < hi ? tile_scale(lo + u) : 0.0f;
        for (int i = lo; i < hi; i++) {
            const int s = (i - lo) % S;
            const int j = i - lo, buf = j % p.nbufs;
            const int rb = i / p.kblocks;
            if (!mbar_wait(&mma_done[buf], (j / p.nbufs) & 1, p.err, ERR_TC_WAIT + 6)) break;
            tc_fence_after();
            const float* sx = sx_ring + s * T * TS;
            const float ws = ws_ring[0];
            ws_ring[0] = ws_ring[1];
            ws_ring[1] = ws_ring[2];
            ws_ring[2] = ws_ring[3];
            ws_ring[3] = i + 4 < hi ? tile_scale(i + 4) : 0.0f;
            // 8 columns per load: 8 / TS tokens
#pragma unroll
            for (int c0 = 0; c0 < MAXT * TS; c0 += 8) {
                if (c0 < T * TS) {
                    float d[8];
                    tc_ld8(tmem_base + lane_base + static_cast<uint32_t>(buf * nmma + c0), d);
                    tc_wait_ld();
#pragma unroll
                    for (int q = 0; q < 8; q += TS) {
                        const int t = (c0 + q) / TS;
                        if (t < T) {
                            float u = sx[t * TS] * d[q];
#pragma unroll
                            for (int term = 1; term < TERMS; term++) u = __fadd_rn(u, sx[t * TS + term] * d[q + term]);
                            acc[t] = fmaf(ws, u, acc[t]);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&tmem_empty[buf]);
                mbar_arrive(&b_empty[s]);
            }
            // end of this CTA's part of row block rb: write it, or hand it to the split-K fix-up
            if (i + 1 == hi || (i + 1) % p.kblocks == 0) {
                const int rb0 = rb * p.kblocks;
                if ((i + 1) % p.kblocks == 0 && lo <= rb0) {
                    tc_store_row<MAXT>(p, acc, rb, r);
                } else {
                    // partial slot 0 when rb is where this CTA starts, else 1; each warp
                    // fixes up its own 32 rows (counters per row block and lane quarter)
                    const int side = lo / p.kblocks == rb ? 0 : 1;
                    float* pp = p.partial + (static_cast<int64_t>(blockIdx.x) * 2 + side) * T * kTcTile;
#pragma unroll
                    for (int t = 0; t < MAXT; t++)
                        if (t < T) pp[t * kTcTile + r] = acc[t];
                    __threadfence();
                    __syncwarp();
                    const int c_first = tc_owner(p.tiles, rb0, grid);
                    const int c_last = tc_owner(p.tiles, rb0 + p.kblocks - 1, grid);
                    unsigned prev = 0;
                    if (lane == 0) prev = atomicAdd(p.counters + rb * 4 + quarter, 1u);
                    prev = __shfl_sync(0xffffffffu, prev, 0);
                    if (prev == static_cast<unsigned>(c_last - c_first)) {
                        __threadfence();
                        float sum[MAXT];
#pragma unroll
                        for (int t = 0; t < MAXT; t++) sum[t] = 0.0f;
                        for (int c = c_first; c <= c_last; c++) {
                            const int sd = tc_lo(p.tiles, c, grid) / p.kblocks == rb ? 0 : 1;
                            const float* q = p.partial + (static_cast<int64_t>(c) * 2 + sd) * T * kTcTile + r;
#pragma unroll
                            for (int t = 0; t < MAXT; t++)
                                if (t < T) sum[t] += __ldcg(q + t * kTcTile);
                        }
                        tc_store_row<MAXT>(p, sum, rb, r);
                        if (lane == 0) p.counters[rb * 4 + quarter] = 0u;
                    }
                }
#pragma unroll
                for (int t = 0; t < MAXT; t++) acc[t] = 0.0f;
            }
        }
    }
    // the producer and MMA roles ran on lane 0 alone: reconverge every warp
    // before the CTA barrier (an aligned barrier must not be reached diverged)
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(p.tmem_cols)
                     : "memory");
    }
}

}  // namespace oomb
