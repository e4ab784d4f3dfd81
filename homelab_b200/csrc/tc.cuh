// tc.cuh - FP8 GEMV/GEMM for decode batches on the 5th-generation tensor cores.
//
// y[t, n] = sum_k x[t, k] * e4m3(q[n, k]) * scale(n, k), fp32 accumulation: the
// arithmetic of the reference's gemv_impl<T, true> (ops.cu:338-440); only the
// summation order differs.
//
// The weights never pass through registers: TMA copies 128 x 128 e4m3 tiles of
// q (row-major, or the packed tile layout) into a shared-memory ring in the
// canonical K-major 128-byte swizzled layout, and tcgen05.mma (kind::f8f6f4,
// M = 128, K = 32) reads them from there.  The activations enter as the B
// operand, split once per call by xsplit_kernel: every 128-column block of an
// activation row is written as TS e4m3 terms with power-of-two scales,
//   x = s1 * q1 + s2 * q2 + ... + s_TS * q_TS,
// q_i = e4m3(residual / s_i), s_i chosen so the block's largest residual lands
// in [128, 256).  An e4m3 term carries 4 significant bits of each value, so the
// largest residual shrinks by 2^-4 per term: two terms reproduce every bf16
// activation (8 significant bits) within 2^14 of its block's largest exactly,
// and fp32 activations take six terms, which keep every value to within
// 2^-24 of its block's largest (24 significant bits, the fp32 mantissa).
// The terms land in a workspace image [rows = assignment * TS + term, K] that
// TMA copies tile by tile (nmma rows x 128 bytes, 128-byte swizzle) into the B
// ring beside the weights, with the tile's term scales; so the split costs one
// pass over x per call instead of one per weight tile.  Each (token, term) is
// one column of B, so one MMA gives every term's partial dot product for a
// 128-row tile.  Accumulators live in tensor memory one K block (128 columns,
// one weight scale) at a time, up to four tiles in flight; an epilogue
// warpgroup folds each block into fp32 registers,
//   acc = fma(w_scale, s1 * D1 + s2 * D2 + ... + s_TS * D_TS, acc),
// K blocks in order.
// Tiles (row block, K block) are split contiguously over the CTAs (stream-K);
// a row block split over several CTAs is summed by the last CTA to finish, in
// CTA order (deterministic), through a caller workspace.
//
// Warp roles (11 warps): 0 weight TMA producer, 1 MMA issuer and tensor-memory
// owner, 2-5 and 7-10 two epilogue warpgroups (warp w reads tensor-memory lanes
// 32*(w%4)..+31; with 8 or more token slots each warpgroup folds half of the
// tokens), 6 the B loader (split activations and term scales, after the
// dependency wait).
// Every wait is bounded and records an error code.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace oomb {

constexpr int kTcThreads = 352;             // 11 warps: TMA producer, MMA, 2 x 4 epilogue, B loader
constexpr int kTcTile = 128;                 // rows of a weight tile, and columns of a K block
constexpr int kTcTileBytes = kTcTile * kTcTile;
constexpr int kTcMaxStages = 8;              // ring depth
constexpr int kTcMinStages = 3;
constexpr int kTcMaxT = 64;                  // tokens per launch (bf16 x; 32 for fp32 x)
constexpr int kTcKSteps = kTcTile / 32;      // MMAs (K = 32 each) per tile
constexpr int kTcAccBufs = 4;                // tensor-memory accumulator buffers (tiles in flight)
constexpr int kTcMaxN = 256;                 // largest MMA N (M = 128)

enum : unsigned {
    ERR_TC_WAIT = 0x500,  // a tensor-core pipeline wait ran out (+ the waiting role)
};

// e4m3 terms per activation value: 2 reproduce bf16, 6 keep 24 bits of fp32.
__host__ __device__ constexpr int tc_ts(bool x_bf16) { return x_bf16 ? 2 : 6; }

// Row stride (floats) of the term-scale image: its rows' aligned 16-byte
// supersets stay inside the row.
__host__ __device__ inline int tc_sx_stride(int rows) { return ((rows + 3) & ~3) + 4; }

struct TcParams {
    int T, K, nrows;
    const float* scale;  // 1x128: [nrows, K/128]; 128x128: [nrows/128, K/128]
    int layout;
    void* y;             // [T, nrows] bf16 or fp32
    int y_bf16;
    float* partial;      // [grid][2][T][128] split-K partial sums
    unsigned* counters;  // [nrows/128][4] arrivals per (row block, tensor-memory lane quarter)
    const float* sx;     // term scales of the split activations [K/128][sx_stride]
    int sx_stride;
    int tiles, kblocks;  // (nrows/128) * (K/128), K/128
    int q_tiles;         // q is in the packed tile layout (oomb_pack_fp8_tiles), else row-major
    int nmma;            // MMA N = T * TS rounded up to 8
    int stages;
    int nbufs;           // tensor-memory accumulator buffers in use (<= kTcAccBufs)
    int tmem_cols;
    unsigned* err;
};

// Shared memory (after aligning the base to 1024 bytes):
// [A ring: stages x 16 KB][B ring: stages x nmma*128][term scales: stages x (nmma + 8) floats]
// [barriers][tensor-memory address]
struct TcSmem {
    size_t a_off, b_off, sx_off, sx_slot, bar_off, total;
};

__host__ __device__ inline TcSmem tc_smem(int stages, int nmma) {
    TcSmem m{};
    m.a_off = 0;
    m.b_off = static_cast<size_t>(stages) * kTcTileBytes;
    m.sx_off = m.b_off + static_cast<size_t>(stages) * nmma * 128;
    m.sx_slot = static_cast<size_t>(nmma + 8);
    m.bar_off = (m.sx_off + static_cast<size_t>(stages) * m.sx_slot * 4 + 7) & ~static_cast<size_t>(7);
    // a_full, a_empty, b_full, b_empty [kTcMaxStages]; mma_done, tmem_empty [kTcAccBufs]; tensor-memory address
    m.total = m.bar_off + (4 * kTcMaxStages + 2 * kTcAccBufs) * 8 + 16;
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

__device__ __forceinline__ void tc_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

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

// ---- the activation split (one pass per call) ------------------------------------------

struct XsParams {
    const void* x;         // [*, K] bf16 or fp32
    const int32_t* rows;   // [A] activation row of each assignment, or null (row = assignment)
    const int32_t* first;  // device word holding the first assignment to split (the first CSR offset), or null: 0
    const int32_t* count;  // device word holding A (the last CSR offset), or null: A = a_host
    const int32_t* count_idx;  // with count: A = count[*count_idx] (a CSR whose group count is on the device)
    int a_host;
    int a_cover;           // assignments the grid covers (>= A)
    int zero_pad;          // rows of assignments in [A, a_cover) are written as zero terms
    int K, kblocks;
    uint8_t* xs;           // [rows_alloc, K] e4m3 terms, row = assignment * TS + term
    int rows_alloc;
    float* sx;             // [kblocks][sx_stride] term scales, same row index
    int sx_stride;
};

// One warp per (assignment, K block): lane l splits columns 4l .. 4l+3 of the
// block into TS terms (the block's largest residual sets each term's scale).
template <bool XBF16>
__global__ void __launch_bounds__(256) xsplit_kernel(const XsParams p) {
    constexpr int TS = tc_ts(XBF16);
    pdl_wait();  // x, rows and the count come from earlier kernels; xs / sx may still be read by one
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int64_t w = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
    if (w >= static_cast<int64_t>(p.a_cover) * p.kblocks) return;
    const int a = static_cast<int>(w / p.kblocks), kb = static_cast<int>(w - static_cast<int64_t>(a) * p.kblocks);
    const int A = p.count ? __ldcg(p.count + (p.count_idx ? __ldcg(p.count_idx) : 0)) : p.a_host;
    if ((a >= A && !p.zero_pad) || (p.first && a < __ldcg(p.first))) return;
    float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (a < A) {
        const int row = p.rows ? __ldcg(p.rows + a) : a;
        const int64_t idx = static_cast<int64_t>(row) * p.K + static_cast<int64_t>(kb) * kTcTile + lane * 4;
        if (XBF16) {
            const uint2 u = __ldcg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p.x) + idx));
            v[0] = __uint_as_float(u.x << 16);
            v[1] = __uint_as_float(u.x & 0xffff0000u);
            v[2] = __uint_as_float(u.y << 16);
            v[3] = __uint_as_float(u.y & 0xffff0000u);
        } else {
            const float4 u = __ldcg(reinterpret_cast<const float4*>(static_cast<const float*>(p.x) + idx));
            v[0] = u.x;
            v[1] = u.y;
            v[2] = u.z;
            v[3] = u.w;
        }
    }
#pragma unroll
    for (int term = 0; term < TS; term++) {
        float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float inv;
        const float sc = tc_term_scale(mx, inv);
        const uint32_t lo2 = e4m3x2_from_f32(v[0] * inv, v[1] * inv);
        const uint32_t hi2 = e4m3x2_from_f32(v[2] * inv, v[3] * inv);
        const int r = a * TS + term;
        if (r < p.rows_alloc) {
            *reinterpret_cast<uint32_t*>(p.xs + static_cast<int64_t>(r) * p.K + static_cast<int64_t>(kb) * kTcTile +
                                         lane * 4) = lo2 | (hi2 << 16);
            if (lane == 0) p.sx[static_cast<int64_t>(kb) * p.sx_stride + r] = sc;
        }
        if (term + 1 < TS) {
            // exact residual: q * sc carries at most 4 significant bits
            const float2 qa = e4m3x2_to_float2(static_cast<unsigned short>(lo2));
            const float2 qb = e4m3x2_to_float2(static_cast<unsigned short>(hi2));
            v[0] -= qa.x * sc;
            v[1] -= qa.y * sc;
            v[2] -= qb.x * sc;
            v[3] -= qb.y * sc;
        }
    }
}

// Folds one K block from tensor memory into acc for tokens [t0, t0 + NT) of
// the n present: column c = t * TS + term of the buffer at taddr, term scales
// sx[c]:  acc[t - t0] = fma(ws, s_0 D_0 + s_1 D_1 + ... (left to right), acc).
// Columns are read 32 at a time (one wait per 32), the tail 8 at a time, never
// past the last 8-column group holding a present token (t0 * TS must be a
// multiple of 8 when t0 > 0).  Entries of acc past the present tokens take
// whatever the read columns hold and are never stored.  Called by every lane
// of a warp with the same n.
template <int TS, int NT>
__device__ __forceinline__ void tc_fold(uint32_t taddr, const float* sx, int t0, int n, float ws, float (&acc)[NT]) {
    const int nt = n - t0 < NT ? n - t0 : NT;
    if (nt <= 0) return;
    const int base = t0 * TS;
    const int ncol = (nt * TS + 7) & ~7;
    const float* sxb = sx + base;
    constexpr int NC = NT * TS;
    constexpr int LG = NC % 32 == 0 ? 32 : 8;  // columns a tensor-memory load brings
    if constexpr (NC % 8 == 0 && TS % 2 == 0) {
        if (nt == NT) {
            // every column present: all tensor-memory loads in flight before one
            // wait, and each token's term pairs multiplied two at a time (each
            // product rounded as alone, so the same sums as one at a time)
            float d[NC / LG][LG];
#pragma unroll
            for (int g = 0; g < NC / LG; g++) {
                if constexpr (LG == 32) tc_ld32(taddr + static_cast<uint32_t>(base + LG * g), d[g]);
                else tc_ld8(taddr + static_cast<uint32_t>(base + LG * g), d[g]);
            }
            tc_wait_ld();
#pragma unroll
            for (int t = 0; t < NT; t++) {
                float u = 0.0f;
#pragma unroll
                for (int q = 0; q < TS; q += 2) {
                    const int c = t * TS + q;  // even: the pair (c, c + 1) shares token t and a load group
                    const float2 sp = *reinterpret_cast<const float2*>(sxb + c);
                    const float2 pr = fmul2(sp, make_float2(d[c / LG][c % LG], d[c / LG][c % LG + 1]));
                    u = q == 0 ? __fadd_rn(pr.x, pr.y) : __fadd_rn(__fadd_rn(u, pr.x), pr.y);
                }
                acc[t] = fmaf(ws, u, acc[t]);
            }
            return;
        }
    }
    float u = 0.0f;
    auto fold = [&](int c, float d) {
        const int t = c / TS, term = c - (c / TS) * TS;
        if (t < NT) {
            const float v = __fmul_rn(sxb[c], d);
            u = term == 0 ? v : __fadd_rn(u, v);
            if (term == TS - 1) acc[t] = fmaf(ws, u, acc[t]);
        }
    };
#pragma unroll
    for (int c0 = 0; c0 < NT * TS; c0 += 32) {
        if (c0 < ncol) {
            if (c0 + 32 <= ncol) {
                float d[32];
                tc_ld32(taddr + static_cast<uint32_t>(base + c0), d);
                tc_wait_ld();
#pragma unroll
                for (int q = 0; q < 32; q++) fold(c0 + q, d[q]);
            } else {
#pragma unroll
                for (int c1 = c0; c1 < c0 + 32 && c1 < NT * TS; c1 += 8) {
                    if (c1 < ncol) {
                        float d[8];
                        tc_ld8(taddr + static_cast<uint32_t>(base + c1), d);
                        tc_wait_ld();
#pragma unroll
                        for (int q = 0; q < 8; q++) fold(c1 + q, d[q]);
                    }
                }
            }
        }
    }
}

// The epilogue's token split: with at least 8 token slots the two warpgroups
// take halves (their first column, HALF * TS, a multiple of 8), else warpgroup 0
// takes all and warpgroup 1 idles.
template <int MAXN>
struct EpiSplit {
    static constexpr int HALF = MAXN >= 8 ? MAXN / 2 : MAXN;
    static constexpr bool SPLIT = MAXN >= 8;
    static constexpr int WARPS = SPLIT ? 8 : 4;                    // epilogue warps launched
    static constexpr int THREADS = SPLIT ? kTcThreads : 7 * 32;  // without the split: warps 0-6 only
};

template <bool XBF16, int MAXT>
__global__ void __launch_bounds__(kTcThreads, 1) tc_gemm_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                 const __grid_constant__ CUtensorMap xmap,
                                                                 const TcParams p) {
    constexpr int TS = tc_ts(XBF16);
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const TcSmem L = tc_smem(p.stages, p.nmma);
    uint8_t* a_ring = smem + L.a_off;
    uint8_t* b_ring = smem + L.b_off;
    float* sx_ring = reinterpret_cast<float*>(smem + L.sx_off);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bar_off);
    uint64_t* a_full = bars;
    uint64_t* a_empty = bars + kTcMaxStages;
    uint64_t* b_full = bars + 2 * kTcMaxStages;
    uint64_t* b_empty = bars + 3 * kTcMaxStages;
    uint64_t* mma_done = bars + 4 * kTcMaxStages;
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
            mbar_init(&b_empty[i], EpiSplit<MAXT>::WARPS);
        }
        for (int i = 0; i < p.nbufs; i++) {
            mbar_init(&mma_done[i], 1);
            mbar_init(&tmem_empty[i], EpiSplit<MAXT>::WARPS);
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(p.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
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
    } else if (warp == 6) {
        // ================= B loader: the split activations of each tile's K block, and their term scales =================
        if (lane == 0) {
            pdl_wait();  // written by xsplit_kernel, the previous launch
            const uint64_t keep = make_evict_last_policy();  // read once per row block
            const int sxa = (T * TS + 3) & ~3;
            const unsigned bytes = static_cast<unsigned>(nmma * 128 + sxa * 4);
            for (int i = lo; i < hi; i++) {
                const int s = (i - lo) % S, it = (i - lo) / S, kb = i % p.kblocks;
                if (!mbar_wait(&b_empty[s], (it & 1) ^ 1, p.err, ERR_TC_WAIT + 2)) break;
                mbar_arrive_expect_tx(&b_full[s], bytes);
                tma_load_2d(b_ring + s * nmma * 128, &xmap, kb * kTcTile, 0, &b_full[s], keep);
                bulk_g2s_plain(sx_ring + s * L.sx_slot, p.sx + static_cast<int64_t>(kb) * p.sx_stride,
                               static_cast<unsigned>(sxa * 4), &b_full[s]);
            }
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
        // ================= epilogue warpgroups (warps 2..5 and 7..10) =================
        using SP = EpiSplit<MAXT>;
        const int wg = warp >= 7 ? 1 : 0;
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;  // row of the tile this thread owns
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        const int t0 = wg * SP::HALF;       // this warpgroup's first token
        const bool idle = wg == 1 && !SP::SPLIT;
        float acc[SP::HALF];
#pragma unroll
        for (int t = 0; t < SP::HALF; t++) acc[t] = 0.0f;
        // weight scales of this thread's row, fetched four tiles ahead
        auto tile_scale = [&](int i) {
            const int rb = i / p.kblocks, kb = i - rb * p.kblocks;
            return p.layout ? __ldg(p.scale + static_cast<int64_t>(rb) * p.kblocks + kb)
                            : __ldg(p.scale + static_cast<int64_t>(rb * kTcTile + r) * p.kblocks + kb);
        };
        float ws_ring[4];
#pragma unroll
        for (int u = 0; u < 4; u++) ws_ring[u] = lo + u < hi ? tile_scale(lo + u) : 0.0f;
        // stores this warpgroup's tokens of row r of row block rb from v
        auto store_row = [&](const float (&v)[SP::HALF], int rb) {
#pragma unroll
            for (int t = 0; t < SP::HALF; t++) {
                if (t0 + t < p.T) {
                    const int64_t yi = static_cast<int64_t>(t0 + t) * p.nrows + rb * kTcTile + r;
                    if (p.y_bf16) static_cast<__nv_bfloat16*>(p.y)[yi] = __float2bfloat16_rn(v[t]);
                    else static_cast<float*>(p.y)[yi] = v[t];
                }
            }
        };
        for (int i = lo; i < hi; i++) {
            const int s = (i - lo) % S;
            const int j = i - lo, buf = j % p.nbufs;
            const int rb = i / p.kblocks;
            const float ws = ws_ring[0];
            ws_ring[0] = ws_ring[1];
            ws_ring[1] = ws_ring[2];
            ws_ring[2] = ws_ring[3];
            ws_ring[3] = i + 4 < hi ? tile_scale(i + 4) : 0.0f;
            if (!mbar_wait(&mma_done[buf], (j / p.nbufs) & 1, p.err, ERR_TC_WAIT + 6)) break;
            tc_fence_after();
            if (!idle)
                tc_fold<TS, SP::HALF>(tmem_base + lane_base + static_cast<uint32_t>(buf * nmma), sx_ring + s * L.sx_slot,
                                      t0, T, ws, acc);
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
                    if (!idle) store_row(acc, rb);
                } else {
                    // partial slot 0 when rb is where this CTA starts, else 1; each warp
                    // writes its tokens of its 32 rows, and the last of the 2 x (CTAs of the
                    // row block) warps of its lane quarter to arrive sums every token
                    const int side = lo / p.kblocks == rb ? 0 : 1;
                    float* pp = p.partial + (static_cast<int64_t>(blockIdx.x) * 2 + side) * T * kTcTile;
                    if (!idle) {
#pragma unroll
                        for (int t = 0; t < SP::HALF; t++)
                            if (t0 + t < T) pp[(t0 + t) * kTcTile + r] = acc[t];
                    }
                    __threadfence();
                    __syncwarp();
                    const int c_first = tc_owner(p.tiles, rb0, grid);
                    const int c_last = tc_owner(p.tiles, rb0 + p.kblocks - 1, grid);
                    unsigned prev = 0;
                    if (lane == 0) prev = atomicAdd(p.counters + rb * 4 + quarter, 1u);
                    prev = __shfl_sync(0xffffffffu, prev, 0);
                    constexpr unsigned PER_CTA = SP::SPLIT ? 2u : 1u;  // arrivals per CTA and lane quarter
                    if (prev == PER_CTA * static_cast<unsigned>(c_last - c_first + 1) - 1u) {
                        __threadfence();
                        // sums in CTA order; 16 tokens of up to 4 CTAs are loaded at once, so a
                        // row block costs ceil(T / 16) * ceil(CTAs / 4) L2 round trips
                        for (int tt = 0; tt < T; tt += 16) {
                            float sum[16];
#pragma unroll
                            for (int u = 0; u < 16; u++) sum[u] = 0.0f;
                            for (int c0 = c_first; c0 <= c_last; c0 += 4) {
                                float v[4][16];
#pragma unroll
                                for (int cc = 0; cc < 4; cc++) {
                                    const int c = c0 + cc;
                                    const bool have = c <= c_last;
                                    const int sd = have && tc_lo(p.tiles, c, grid) / p.kblocks == rb ? 0 : 1;
                                    const float* q =
                                        p.partial + (static_cast<int64_t>(have ? c : c0) * 2 + sd) * T * kTcTile + r;
#pragma unroll
                                    for (int u = 0; u < 16; u++)
                                        v[cc][u] = have && tt + u < T ? __ldcg(q + (tt + u) * kTcTile) : 0.0f;
                                }
#pragma unroll
                                for (int cc = 0; cc < 4; cc++)
                                    if (c0 + cc <= c_last)
#pragma unroll
                                        for (int u = 0; u < 16; u++) sum[u] += v[cc][u];
                            }
#pragma unroll
                            for (int u = 0; u < 16; u++) {
                                if (tt + u < T) {
                                    const int64_t yi = static_cast<int64_t>(tt + u) * p.nrows + rb * kTcTile + r;
                                    if (p.y_bf16) static_cast<__nv_bfloat16*>(p.y)[yi] = __float2bfloat16_rn(sum[u]);
                                    else static_cast<float*>(p.y)[yi] = sum[u];
                                }
                            }
                        }
                        if (lane == 0) p.counters[rb * 4 + quarter] = 0u;
                    }
                }
#pragma unroll
                for (int t = 0; t < SP::HALF; t++) acc[t] = 0.0f;
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
