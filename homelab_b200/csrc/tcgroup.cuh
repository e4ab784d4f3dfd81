// tcgroup.cuh - grouped FP8 expert GEMM on the 5th-generation tensor cores: the
// large-step path of the routed experts (the reference's moe_tiled,
// crates/oominf-cuda/kernels/moe.cu:204-335, launched from Moe::run_group,
// crates/oominf-models-qwen/src/moe.rs:650,746-758).
//
// One projection per launch, over every group of a CSR grouping:
//   y[a, r] = sum_k x[row(a), k] * e4m3(W_e[r, k]) * scale_e(r, k)
// for a in [off[e], off[e+1]), row(a) = rows ? rows[a] : a, W_e the e4m3
// matrix [N, K] at byte offset w_off of record recs[e] and scale_e its fp32
// block scales at s_off (1x128 or 128x128).  fp32 accumulation, fp32 y [A, N].
//
// Work units are (group chunk, 128-row block): every group is cut into chunks
// of at most CH assignments, and the units are spread over a persistent grid
// (CTA b takes units b, b + grid, ...), each unit's K blocks in order inside one
// CTA - no split-K fix-up.  Units of one row block of one expert are
// consecutive, so the CTAs working at the same time read the same weight tiles
// and the chunks after the first find them in L2.
//
// The arithmetic is the dense tensor-core kernel's (tc.cuh): xsplit_kernel
// first splits every assignment's activation row (gathered through `rows`)
// into e4m3 terms with power-of-two scales (two terms for bf16 x, six for fp32
// x), once per launch, into a workspace image whose row a * TS + term is one
// column of the B operand; per tile, TMA copies the chunk's rows of that image
// (nmma rows from row a0 * TS) into the B ring beside the weights.
// tcgen05.mma (kind::f8f6f4, M = 128, K = 32) accumulates one K block per
// tensor-memory buffer and the epilogue folds
//   acc = fma(w_scale, sum_term s_term * D_term, acc)
// K blocks in order.  The MMA's N is the chunk's own column count (rounded up
// to 16), so a chunk of 4 assignments costs a 16-column MMA; an output's bits
// do not depend on the chunking.
//
// Weights: records live at arbitrary addresses (resident, staged or received),
// so no tensor map can name them.  The copy warp moves each 128 x 128 weight
// tile with 16-byte cp.async straight into the 128-byte swizzled K-major layout
// the MMA reads (every lane 32 chunks of 16 bytes: 4 rows of 128 bytes per warp
// instruction, coalesced), commits one group per tile and releases a tile to the
// MMA kTgLag tiles later, after cp.async.wait_group and a proxy fence.
//
// Warp roles (11 warps): 0 weight copies, 1 MMA issuer and tensor-memory owner,
// 2-5 and 7-10 epilogue (two warpgroups, each a half of a chunk's assignments),
// 6 the B loader.  Every wait is bounded and records an error code.
#pragma once

#include "tc.cuh"

namespace oomb {

constexpr int kTgMaxExperts = 4096;  // groups per launch (their chunk prefix sits in shared memory)
#ifndef OOMB_TG_LAG
#define OOMB_TG_LAG 3
#endif
// weight tiles in flight before the oldest is released (< stages); measured on
// B200 with 6: config-5 batch 128 2.55 -> 2.88 ms, batch 1024 4.12 -> 5.67 ms (the
// deeper ring also forces smaller chunks), so 3
constexpr int kTgLag = OOMB_TG_LAG;

enum : unsigned {
    ERR_TG_WAIT = 0x580,  // a grouped tensor-core pipeline wait ran out (+ the waiting role)
};

struct TgParams {
    const uint64_t* recs;  // [n_experts] record addresses
    const int32_t* off;    // [n_experts + 1] CSR offsets of the groups
    int n_experts;         // groups (an upper bound when n_dev is set)
    const int32_t* n_dev;  // device word holding the group count, or null: n_experts
    int a_max;             // assignments the split covered (off[n_experts] must not exceed it)
    int K, N;
    int64_t w_off, s_off;  // byte offsets of the projection's e4m3 weights and fp32 scales in a record
    int layout;            // OOMB_SCALE_1X128 (0) or OOMB_SCALE_128X128 (1)
    float* y;              // [A, N] fp32
    const float* sx;       // term scales of the split activations [K/128][sx_stride]
    int sx_stride;
    int chunk;             // assignments per unit (the kernel's CH)
    int rblocks, kblocks;  // N / 128, K / 128
    int nmma;              // B rows per stage (CH * TS), and the accumulator stride in tensor memory
    int stages, nbufs, tmem_cols;
    unsigned* err;
};

// Shared memory: the dense kernel's layout, then the chunk prefix.
__host__ __device__ inline size_t tg_smem_bytes(int stages, int nmma, int n_experts) {
    const TcSmem m = tc_smem(stages, nmma);
    return ((m.total + 15) & ~static_cast<size_t>(15)) + 4 * static_cast<size_t>(n_experts + 1);
}

struct TgUnit {
    int e, rb, a0, nt;
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <bool XBF16, int CH>
__global__ void __launch_bounds__(kTcThreads, 1) tc_group_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                  const TgParams p) {
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
    int* cs = reinterpret_cast<int*>(smem + ((L.total + 15) & ~static_cast<size_t>(15)));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.stages, KB = p.kblocks;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; i++) {
            mbar_init(&a_full[i], 1);
            mbar_init(&a_empty[i], 1);
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], EpiSplit<CH>::WARPS);
        }
        for (int i = 0; i < p.nbufs; i++) {
            mbar_init(&mma_done[i], 1);
            mbar_init(&tmem_empty[i], EpiSplit<CH>::WARPS);
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(p.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // the grouping (off) and the split activations come from earlier kernels
    pdl_wait();
    if (warp == 0) {
        // cs[e] = chunks of the groups before e (exclusive prefix), cs[n_experts] = all chunks
        const int E = p.n_dev ? min(max(__ldcg(p.n_dev), 0), p.n_experts) : p.n_experts, per = (E + 31) / 32;
        const int e0 = min(E, lane * per), e1 = min(E, e0 + per);
        int mine = 0;
        for (int e = e0; e < e1; e++) {
            const int c = __ldcg(p.off + e + 1) - __ldcg(p.off + e);
            mine += c > 0 ? (c + p.chunk - 1) / p.chunk : 0;
        }
        int incl = mine;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int run = incl - mine;
        for (int e = e0; e < e1; e++) {
            cs[e] = run;
            const int c = __ldcg(p.off + e + 1) - __ldcg(p.off + e);
            run += c > 0 ? (c + p.chunk - 1) / p.chunk : 0;
        }
        // more assignments than the split covered: do nothing, report it
        if (__ldcg(p.off + E) > p.a_max) {
            if (lane == 31) record_error(p.err, ERR_BAD_TABLE);
            incl = 0;
        }
        // groups past the device count (when it is on the device) hold no chunk
        incl = __shfl_sync(0xffffffffu, incl, 31);
        for (int e = E + lane; e <= p.n_experts; e += 32) cs[e] = incl;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_launch_dependents();

    const int grid = gridDim.x;
    const int units = cs[p.n_experts] * p.rblocks;
    const int my_units = static_cast<int>(blockIdx.x) < units ? (units - static_cast<int>(blockIdx.x) + grid - 1) / grid : 0;
    const int ntiles = my_units * KB;
    // the unit of this CTA's j-th tile
    auto unit_of = [&](int j) {
        const int u = static_cast<int>(blockIdx.x) + (j / KB) * grid;
        const int g = u / p.rblocks;
        int lo = 0, hi = p.n_experts;  // cs[lo] <= g < cs[hi]
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (cs[mid] <= g) lo = mid;
            else hi = mid;
        }
        TgUnit U;
        U.e = lo;
        U.rb = u - g * p.rblocks;
        U.a0 = __ldcg(p.off + lo) + (g - cs[lo]) * p.chunk;
        U.nt = min(p.chunk, __ldcg(p.off + lo + 1) - U.a0);
        return U;
    };

    if (warp == 0) {
        // ================= weight copies: 16-byte cp.async into the swizzled ring =================
        int j = 0;
        const uint8_t* wrow = nullptr;
        for (; j < ntiles; j++) {
            const int s = j % S, it = j / S, kb = j % KB;
            int ok = 1;
            if (lane == 0) ok = mbar_wait(&a_empty[s], (it & 1) ^ 1, p.err, ERR_TG_WAIT + 1);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            if (kb == 0) {
                const TgUnit U = unit_of(j);
                wrow = reinterpret_cast<const uint8_t*>(__ldg(reinterpret_cast<const unsigned long long*>(p.recs) + U.e)) +
                       p.w_off + static_cast<int64_t>(U.rb) * kTcTile * p.K;
                if (reinterpret_cast<uintptr_t>(wrow) & 15u) {
                    // a record address the 16-byte copies cannot take: skip the work, report it
                    if (lane == 0) record_error(p.err, ERR_BAD_TABLE);
                    break;
                }
            }
            uint8_t* dst = a_ring + s * kTcTileBytes;
            const uint8_t* src = wrow + kb * kTcTile;
#pragma unroll 8
            for (int i = 0; i < kTcTileBytes / 16 / 32; i++) {
                const int q = lane + 32 * i, r = q >> 3, c = (q & 7) * 16;
                cp_async16(dst + sw128_offset(r, c), src + static_cast<int64_t>(r) * p.K + c);
            }
            cp_async_commit();
            if (j >= kTgLag) {
                // tile j - kTgLag has landed for this lane; make it visible to the tensor cores
                cp_async_wait<kTgLag>();
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_full[(j - kTgLag) % S]);
            }
        }
        cp_async_wait<0>();
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0)
            for (int i = j > kTgLag ? j - kTgLag : 0; i < j; i++) mbar_arrive(&a_full[i % S]);
    } else if (warp == 6) {
        // ================= B loader: the chunk's split activations and term scales per tile =================
        if (lane == 0) {
            const uint64_t keep = make_evict_last_policy();  // read once per row block of the expert
            TgUnit U{};
            for (int j = 0; j < ntiles; j++) {
                const int s = j % S, it = j / S, kb = j % KB;
                if (kb == 0) U = unit_of(j);
                const int e0 = U.a0 * TS, e0a = e0 & ~3, e1a = (e0 + U.nt * TS + 3) & ~3;
                if (!mbar_wait(&b_empty[s], (it & 1) ^ 1, p.err, ERR_TG_WAIT + 2)) break;
                mbar_arrive_expect_tx(&b_full[s], static_cast<unsigned>(p.nmma * 128 + (e1a - e0a) * 4));
                tma_load_2d(b_ring + s * p.nmma * 128, &xmap, kb * kTcTile, e0, &b_full[s], keep);
                bulk_g2s_plain(sx_ring + s * L.sx_slot, p.sx + static_cast<int64_t>(kb) * p.sx_stride + e0a,
                               static_cast<unsigned>((e1a - e0a) * 4), &b_full[s]);
            }
        }
    } else if (warp == 1) {
        // ================= MMA issuer =================
        if (lane == 0) {
            int nt = 0;
            for (int j = 0; j < ntiles; j++) {
                const int s = j % S, it = j / S;
                const int buf = j % p.nbufs, use = j / p.nbufs;
                if (j % KB == 0) nt = unit_of(j).nt;
                const int n = (nt * TS + 15) / 16 * 16;  // this chunk's columns, a valid MMA N (16..nmma)
                if (!mbar_wait(&a_full[s], it & 1, p.err, ERR_TG_WAIT + 3)) break;
                if (!mbar_wait(&b_full[s], it & 1, p.err, ERR_TG_WAIT + 4)) break;
                if (!mbar_wait(&tmem_empty[buf], (use & 1) ^ 1, p.err, ERR_TG_WAIT + 5)) break;
                tc_fence_after();
                const uint32_t a_addr = smem_addr(a_ring + s * kTcTileBytes);
                const uint32_t b_addr = smem_addr(b_ring + s * p.nmma * 128);
                const uint32_t d = tmem_base + static_cast<uint32_t>(buf * p.nmma);
                const uint32_t idesc = tc_idesc(n);
#pragma unroll
                for (int k = 0; k < kTcKSteps; k++)
                    tc_mma(d, tc_smem_desc(a_addr + 32 * k), tc_smem_desc(b_addr + 32 * k), idesc, k > 0);
                tc_commit(&a_empty[s]);
                tc_commit(&mma_done[buf]);
            }
        }
    } else {
        // ================= epilogue warpgroups (warps 2..5 and 7..10) =================
        using SP = EpiSplit<CH>;
        const int wg = warp >= 7 ? 1 : 0;
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;  // row of the tile this thread owns
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        const int t0 = wg * SP::HALF;       // this warpgroup's first assignment of a chunk
        const bool idle = wg == 1 && !SP::SPLIT;
        float acc[SP::HALF];
#pragma unroll
        for (int t = 0; t < SP::HALF; t++) acc[t] = 0.0f;
        TgUnit U{};
        const float* sp = nullptr;
        for (int j = 0; j < ntiles; j++) {
            const int s = j % S, buf = j % p.nbufs, kb = j % KB;
            if (kb == 0) {
                U = unit_of(j);
                sp = reinterpret_cast<const float*>(
                    reinterpret_cast<const uint8_t*>(__ldg(reinterpret_cast<const unsigned long long*>(p.recs) + U.e)) +
                    p.s_off);
            }
            // the weight scale of this thread's row for this K block (its load overlaps the wait)
            const float ws = p.layout ? __ldg(sp + static_cast<int64_t>(U.rb) * KB + kb)
                                      : __ldg(sp + static_cast<int64_t>(U.rb * kTcTile + r) * KB + kb);
            if (!mbar_wait(&mma_done[buf], (j / p.nbufs) & 1, p.err, ERR_TG_WAIT + 6)) break;
            tc_fence_after();
            if (!idle)
                tc_fold<TS, SP::HALF>(tmem_base + lane_base + static_cast<uint32_t>(buf * p.nmma),
                                      sx_ring + s * L.sx_slot + ((U.a0 * TS) & 3), t0, U.nt, ws, acc);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&tmem_empty[buf]);
                mbar_arrive(&b_empty[s]);
            }
            if (kb == KB - 1) {
#pragma unroll
                for (int t = 0; t < SP::HALF; t++) {
                    if (!idle && t0 + t < U.nt) p.y[static_cast<int64_t>(U.a0 + t0 + t) * p.N + U.rb * kTcTile + r] = acc[t];
                    acc[t] = 0.0f;
                }
            }
        }
    }
    // the copy-side roles ran on lane 0 alone in places: reconverge before the CTA barrier
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(p.tmem_cols)
                     : "memory");
    }
}

// h[i] = silu(g[i]) * u[i] for i in [start, end), silu(v) = v / (1 + exp(-v)):
// the reference's moe_swiglu (moe.cu:335-339) between the tiled gate and up
// projections and the tiled down projection.
__global__ void swiglu_range_kernel(const float* g, const float* u, float* h, int64_t start, int64_t end) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t i = start + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= end) return;
    const float v = __ldcg(g + i);
    h[i] = v / (1.0f + expf(-v)) * __ldcg(u + i);
}

}  // namespace oomb
