// gemv_fp8.cuh - FP8 e4m3 block-scaled GEMV for decode steps (t <= 4 per launch).
//
// y[t, n] = sum_k x[t, k] * e4m3(q[n, k]) * scale(n, k), fp32 accumulation.
// The arithmetic of the reference's gemv_impl<T, true> (ops.cu:338-440): each
// weight decoded exactly, fp32 products and sums; only the summation order
// differs.
//
// Structure (one CTA per SM, persistent over a contiguous range of row groups):
//   - warp 8 (producer) streams "stages" of RG rows x KC columns of q into a
//     ring of shared-memory buffers with cp.async.bulk, each completed on an
//     mbarrier; consumers hand buffers back through a second mbarrier;
//   - warps 0..7 (consumers) split a stage into 4-row x 512-column tasks; lane l
//     of a task covers 16 columns (one 16-byte chunk per row), decodes e4m3 to
//     fp32 and accumulates with packed FMAs; activations for its columns live in
//     registers (loaded once per K-range, reused across all rows of the pass);
//   - per pass of up to MAXG row groups the warps reduce their partials
//     (multi-value butterfly), combine slabs through shared memory in slab
//     order (deterministic) and write y.
// The kernel signals dependents at entry and streams weights before
// griddepcontrol.wait, so consecutive launches overlap their weight streams.
#pragma once

#include "common.cuh"

namespace oomb {

constexpr int kGemvConsumerWarps = 8;
constexpr int kGemvThreads = (kGemvConsumerWarps + 1) * 32;
constexpr int kGemvStageBytes = 16 * 1024;
constexpr int kGemvStages = 6;
constexpr int kGemvMaxTokens = 4;  // tokens per launch

struct GemvPlan {
    int rg;      // rows per group (multiple of 4, <= 32)
    int kc;      // columns per stage (<= 4096; == k when one stage holds whole rows)
    int ks;      // stages per row group along K
    int nsl;     // 512-column slabs per stage
    int groups;  // row groups
    int grid;    // CTAs
    int maxg;    // row groups per reduction pass
};

struct GemvParams {
    const void* x;
    const uint8_t* q;
    const float* scale;
    void* y;
    int n, k, t;  // t: real tokens (<= template T)
    int layout;   // 0: 1x128, 1: 128x128
    int y_bf16;
    int rg, kc, ks, nsl, groups;
    unsigned* err;
};

// Padded token count of a launch: 1, 2 or 4.
inline int gemv_tpad(int t) { return t <= 1 ? 1 : (t <= 2 ? 2 : 4); }

inline GemvPlan gemv_plan(int n, int k, int tpad, int num_sms) {
    GemvPlan p{};
    const int nsl_full = (k + 511) / 512;
    if (nsl_full >= 8) {
        p.kc = 4096;
        p.rg = 4;
    } else {
        p.kc = k;
        p.rg = 4 * (8 / nsl_full);
    }
    p.ks = (k + p.kc - 1) / p.kc;
    p.nsl = ((p.kc < k ? p.kc : k) + 511) / 512;
    p.groups = (n + p.rg - 1) / p.rg;
    p.grid = p.groups < num_sms ? p.groups : num_sms;
    // With several K-stages per group, a pass covers MAXG groups K-stage by
    // K-stage so activations are reused across MAXG * RG rows; keep
    // MAXG * 4 * T <= 32 partials per lane.
    p.maxg = p.ks == 1 ? 1 : (tpad == 1 ? 4 : (tpad == 2 ? 4 : 2));
    return p;
}

__device__ __forceinline__ const float* scale_ptr(const float* scale, int layout, int k, int row,
                                                  int col) {
    const int nb = (k + 127) >> 7;
    const int r = layout ? (row >> 7) : row;
    return scale + static_cast<int64_t>(r) * nb + (col >> 7);
}

// Stage s of a CTA whose groups are [g0, g1): group, K-stage, slot in the pass.
struct StageCoord {
    int g, ks, gi, pass_first, pass_n;
    bool pass_last;
};

template <int MAXG>
__device__ __forceinline__ StageCoord stage_coord(int s, int g0, int g1, int KS) {
    StageCoord c;
    if (MAXG == 1) {
        c.g = g0 + s / KS;
        c.ks = s % KS;
        c.gi = 0;
        c.pass_first = c.g;
        c.pass_n = 1;
        c.pass_last = c.ks == KS - 1;
    } else {
        const int per_pass = MAXG * KS;
        const int pass = s / per_pass;
        const int within = s - pass * per_pass;
        c.pass_first = g0 + pass * MAXG;
        c.pass_n = min(MAXG, g1 - c.pass_first);
        c.ks = within / c.pass_n;
        c.gi = within - c.ks * c.pass_n;
        c.g = c.pass_first + c.gi;
        c.pass_last = (c.ks == KS - 1) && (c.gi == c.pass_n - 1);
    }
    return c;
}

// Loads the four block scales of a task (rows sg*4 .. +3 of stage coordinate c).
__device__ __forceinline__ void task_scales(const GemvParams& p, const StageCoord& c, int sg,
                                            int col, float (&sc)[4]) {
    const int row0 = c.g * p.rg + sg * 4;
    const int kcol = c.ks * p.kc + col;
#pragma unroll
    for (int i = 0; i < 4; i++)
        sc[i] = row0 + i < p.n ? __ldg(scale_ptr(p.scale, p.layout, p.k, row0 + i, kcol)) : 0.0f;
}

template <int T, bool XBF16, int MAXG>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_fp8_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* stage_buf = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kGemvStages * kGemvStageBytes);
    uint64_t* empty = full + kGemvStages;
    constexpr int V = MAXG * 4 * T;  // partial sums per lane per pass (<= 32)
    static_assert(V <= 32, "too many partials per lane");
    float* red = reinterpret_cast<float*>(empty + kGemvStages);  // [2][warps][V]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g0 = static_cast<int>((static_cast<int64_t>(blockIdx.x) * p.groups) / gridDim.x);
    const int g1 = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * p.groups) / gridDim.x);
    const int KS = p.ks;
    const int nstages = (g1 - g0) * KS;
    const int kcs = min(p.kc, p.k);  // shared-memory row stride of a stage

    if (threadIdx.x == 0) {
        for (int i = 0; i < kGemvStages; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kGemvConsumerWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kGemvConsumerWarps) {
        // ---------------- producer ----------------
        if (lane == 0 && nstages > 0) {
            // Pull this CTA's block scales into L2 ahead of the consumers.
            {
                const int nb = (p.k + 127) >> 7;
                const int r0 = g0 * p.rg, r1 = min(p.n, g1 * p.rg);
                const int s0 = p.layout ? (r0 >> 7) : r0;
                const int s1 = p.layout ? ((r1 - 1) >> 7) + 1 : r1;
                uintptr_t a = reinterpret_cast<uintptr_t>(p.scale + static_cast<int64_t>(s0) * nb);
                uintptr_t b = reinterpret_cast<uintptr_t>(p.scale + static_cast<int64_t>(s1) * nb);
                // Round inward: the prefetch never touches bytes outside the array.
                a = (a + 15) & ~static_cast<uintptr_t>(15);
                b &= ~static_cast<uintptr_t>(15);
                if (b > a)
                    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a),
                                 "r"(static_cast<unsigned>(b - a))
                                 : "memory");
            }
            const uint64_t pol = make_evict_first_policy();
            bool ok = true;
            int s = 0;
            for (; s < nstages; s++) {
                const int slot = s % kGemvStages;
                ok = mbar_wait(&empty[slot], ((s / kGemvStages) & 1) ^ 1, p.err, ERR_EMPTY_WAIT);
                if (!ok) break;
                const StageCoord c = stage_coord<MAXG>(s, g0, g1, KS);
                const int row0 = c.g * p.rg;
                const int nrows = min(p.rg, p.n - row0);
                const int kc0 = c.ks * p.kc;
                const int kcl = min(p.kc, p.k - kc0);
                uint8_t* dst = stage_buf + slot * kGemvStageBytes;
                mbar_arrive_expect_tx(&full[slot], static_cast<unsigned>(nrows * kcl));
                const uint8_t* src = p.q + static_cast<int64_t>(row0) * p.k + kc0;
                if (kcl == p.k) {
                    bulk_g2s(dst, src, static_cast<unsigned>(nrows * kcl), &full[slot], pol);
                } else {
                    for (int r = 0; r < nrows; r++)
                        bulk_g2s(dst + r * kcs, src + static_cast<int64_t>(r) * p.k,
                                 static_cast<unsigned>(kcl), &full[slot], pol);
                }
            }
            if (!ok) {
                // Wait (bounded) for every stage already issued to land, so no copy
                // targets this CTA's shared memory after it exits.
                for (int d = (s > kGemvStages ? s - kGemvStages : 0); d < s; d++)
                    mbar_wait(&full[d % kGemvStages], (d / kGemvStages) & 1, p.err, ERR_DRAIN_WAIT);
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    const int rsg = p.rg >> 2;
    const int tasks = rsg * p.nsl;
    const bool active = warp < tasks;
    const int sg = active ? warp / p.nsl : 0;
    const int sl = active ? warp % p.nsl : 0;
    const int col = sl * 512 + lane * 16;  // column inside a stage

    // Weights and scales do not depend on the previous kernel in the stream;
    // the activations may, so wait for it before reading x.
    pdl_wait();

    float acc[MAXG][4][T];
    float2 xr[T][8];
    int x_ks = -1;
    int pass_parity = 0;
    float sc[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sc_next[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (nstages > 0 && active) {
        const StageCoord c0 = stage_coord<MAXG>(0, g0, g1, KS);
        if (col < min(p.kc, p.k - c0.ks * p.kc)) task_scales(p, c0, sg, col, sc_next);
    }

    for (int s = 0; s < nstages; s++) {
        const StageCoord c = stage_coord<MAXG>(s, g0, g1, KS);
        const int slot = s % kGemvStages;
        const int row0 = c.g * p.rg;
        const int nrows = min(p.rg, p.n - row0);
        const int kc0 = c.ks * p.kc;
        const int kcl = min(p.kc, p.k - kc0);
        const bool col_ok = active && col < kcl;

#pragma unroll
        for (int i = 0; i < 4; i++) sc[i] = sc_next[i];
        if (s + 1 < nstages && active) {  // prefetch the next stage's scales
            const StageCoord cn = stage_coord<MAXG>(s + 1, g0, g1, KS);
            if (col < min(p.kc, p.k - cn.ks * p.kc)) task_scales(p, cn, sg, col, sc_next);
        }
        if (c.gi == 0 && c.ks == 0) {
#pragma unroll
            for (int g = 0; g < MAXG; g++)
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int t = 0; t < T; t++) acc[g][i][t] = 0.0f;
        }
        if (col_ok && x_ks != c.ks) {
#pragma unroll
            for (int t = 0; t < T; t++) {
                if (t < p.t) {
                    load_x16<XBF16>(p.x, static_cast<int64_t>(t) * p.k + kc0 + col, xr[t]);
                } else {
#pragma unroll
                    for (int j = 0; j < 8; j++) xr[t][j] = make_float2(0.0f, 0.0f);
                }
            }
            x_ks = c.ks;
        }

        if (!mbar_wait(&full[slot], (s / kGemvStages) & 1, p.err, ERR_FULL_WAIT)) return;
        if (col_ok) {
            const uint8_t* base = stage_buf + slot * kGemvStageBytes + (sg * 4) * kcs + col;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                if (sg * 4 + i < nrows) {
                    const uint4 w = *reinterpret_cast<const uint4*>(base + i * kcs);
#pragma unroll
                    for (int g = 0; g < MAXG; g++) {
                        if (g == c.gi) {
#pragma unroll
                            for (int t = 0; t < T; t++)
                                acc[g][i][t] = fmaf(dot16_e4m3(w, xr[t]), sc[i], acc[g][i][t]);
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);

        if (c.pass_last) {
            float v[V];
#pragma unroll
            for (int g = 0; g < MAXG; g++)
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int t = 0; t < T; t++) v[(g * 4 + i) * T + t] = acc[g][i][t];
            float* rb = red + pass_parity * kGemvConsumerWarps * V;
            warp_reduce_multi<V>(v, lane);
            // 32 / V lanes hold each total; the lowest of them writes it.
            if ((lane & (32 / V - 1)) == 0) rb[warp * V + reduce_index<V>(lane, 0)] = v[0];
            asm volatile("bar.sync 1, %0;" ::"r"(kGemvConsumerWarps * 32) : "memory");
            const int outs = c.pass_n * p.rg * T;
            for (int o = threadIdx.x; o < outs; o += kGemvConsumerWarps * 32) {
                const int t = o % T;
                const int rr = o / T;
                const int gi = rr / p.rg;
                const int r = rr % p.rg;
                const int row = (c.pass_first + gi) * p.rg + r;
                if (row >= p.n || t >= p.t) continue;
                const int task0 = (r >> 2) * p.nsl;
                const int vi = (gi * 4 + (r & 3)) * T + t;
                float sum = 0.0f;
                for (int q = 0; q < p.nsl; q++) sum += rb[(task0 + q) * V + vi];
                const int64_t yi = static_cast<int64_t>(t) * p.n + row;
                if (p.y_bf16)
                    static_cast<__nv_bfloat16*>(p.y)[yi] = __float2bfloat16_rn(sum);
                else
                    static_cast<float*>(p.y)[yi] = sum;
            }
            pass_parity ^= 1;
        }
    }
}

inline size_t gemv_smem_bytes(int maxg, int tpad) {
    const int v = maxg * 4 * tpad;
    return static_cast<size_t>(kGemvStages) * kGemvStageBytes + 2 * kGemvStages * sizeof(uint64_t) +
           2 * kGemvConsumerWarps * v * sizeof(float);
}

}  // namespace oomb
