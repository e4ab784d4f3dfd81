// moe_fp8.cuh - routed-expert FFN kernels over FP8 e4m3 expert records.
//
// gate/up: h[a, j] = silu(x[tok(a)] . Wg[j]) * (x[tok(a)] . Wu[j])
// down:    y[a, r] = h[a] . Wd[r]
// for every assignment a of expert group i (assignments [off[i], off[i+1]),
// record at recs[i]).  The structure of the reference's moe_gate_up / moe_down
// (crates/oominf-cuda/kernels/moe.cu:52-151): weights decoded once per group of
// assignments, fp32 activations and accumulation, SwiGLU fused into gate/up,
// silu(v) = v / (1 + exp(-v)) (moe.cu:50).
//
// Work is a flat list of units (expert group, row group): a CTA takes a
// contiguous slice of it, so any number of active experts spreads evenly over
// the SMs.  Each unit is one stage: RG rows of the projection(s) streamed into
// shared memory with cp.async.bulk (gate/up: RG/2 gate rows then the matching
// RG/2 up rows; down: RG rows).  Assignments of a unit are processed in chunks
// of TB tokens against the stage held in shared memory.
#pragma once

#include "common.cuh"
#include "gemv_fp8.cuh"

namespace oomb {

constexpr int kMoeTB = 4;  // assignments per chunk when an expert may get several

struct MoeParams {
    const uint64_t* recs;       // [n_e] record addresses
    const int32_t* off;         // [n_e + 1]
    const int32_t* assign_tok;  // [A] token of each assignment (gate/up only)
    const int32_t* n_e_dev;     // number of groups on the device, or null
    int n_e_host;               // number of groups when n_e_dev is null
    const void* x;              // gate/up: activations [*, kdim]; down: h [A, kdim] fp32
    float* out;                 // gate/up: h [A, nrows]; down: y [A, nrows]
    int kdim;                   // columns (hidden for gate/up, inter for down)
    int nrows;                  // rows per projection (inter for gate/up, hidden for down)
    int64_t w_off[2], s_off[2]; // part offsets in a record (gate, up) or (down, -)
    int layout;
    int rgp;                    // rows per part per unit
    int nsl;                    // 512-column slabs per stage
    int gpe;                    // units per expert = ceil(nrows / rgp)
    unsigned* err;
};

inline void moe_plan(int kdim, int parts, int* rgp, int* nsl) {
    *nsl = (kdim + 511) / 512;
    const int rg = 4 * (8 / *nsl);  // stage rows; requires kdim <= 4096
    *rgp = rg / parts;
}

__device__ __forceinline__ int ld_cg_i32(const int32_t* p) { return __ldcg(p); }

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + expf(-v)); }

// PARTS = 2: gate/up with fused SwiGLU; PARTS = 1: down.  XBF16: activations
// are bf16 (gate/up only).  EARLY: the producer reads the routing tables before
// griddepcontrol.wait (only valid when the kernel two launches back wrote them
// and the previous one triggered its dependents after waiting for it).
template <int PARTS, bool XBF16, bool EARLY, int TB>
__global__ void __launch_bounds__(kGemvThreads, 1) moe_fp8_kernel(const MoeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* stage_buf = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kGemvStages * kGemvStageBytes);
    uint64_t* empty = full + kGemvStages;
    constexpr int V = 4 * TB;
    float* red = reinterpret_cast<float*>(empty + kGemvStages);  // [2][warps][V]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rg = PARTS * p.rgp;
    const int stride = p.kdim;  // shared-memory row stride (whole rows per stage)

    if (threadIdx.x == 0) {
        for (int i = 0; i < kGemvStages; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], kGemvConsumerWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kGemvConsumerWarps) {
        // ---------------- producer ----------------
        if (!EARLY) pdl_wait();
        pdl_launch_dependents();
        if (lane != 0) return;
        const int n_e = p.n_e_dev ? ld_cg_i32(p.n_e_dev) : p.n_e_host;
        const int units = n_e * p.gpe;
        const int u0 = static_cast<int>((static_cast<int64_t>(blockIdx.x) * units) / gridDim.x);
        const int u1 = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * units) / gridDim.x);
        const uint64_t pol = make_evict_first_policy();
        bool ok = true;
        int s = 0;
        for (int u = u0; u < u1; u++, s++) {
            const int slot = s % kGemvStages;
            ok = mbar_wait(&empty[slot], ((s / kGemvStages) & 1) ^ 1, p.err, ERR_EMPTY_WAIT);
            if (!ok) break;
            const int ei = u / p.gpe, g = u - ei * p.gpe;
            const int row0 = g * p.rgp;
            const int nr = min(p.rgp, p.nrows - row0);
            const uint8_t* rec = reinterpret_cast<const uint8_t*>(__ldcg(
                reinterpret_cast<const unsigned long long*>(p.recs) + ei));
            uint8_t* dst = stage_buf + slot * kGemvStageBytes;
            const unsigned bytes = static_cast<unsigned>(nr * p.kdim);
            mbar_arrive_expect_tx(&full[slot], bytes * PARTS);
#pragma unroll
            for (int part = 0; part < PARTS; part++)
                bulk_g2s(dst + part * p.rgp * stride,
                         rec + p.w_off[part] + static_cast<int64_t>(row0) * p.kdim, bytes,
                         &full[slot], pol);
        }
        if (!ok) {
            for (int d = (s > kGemvStages ? s - kGemvStages : 0); d < s; d++)
                mbar_wait(&full[d % kGemvStages], (d / kGemvStages) & 1, p.err, ERR_DRAIN_WAIT);
        }
        return;
    }

    // ---------------- consumers ----------------
    pdl_wait();
    pdl_launch_dependents();
    const int n_e = p.n_e_dev ? ld_cg_i32(p.n_e_dev) : p.n_e_host;
    const int units = n_e * p.gpe;
    const int u0 = static_cast<int>((static_cast<int64_t>(blockIdx.x) * units) / gridDim.x);
    const int u1 = static_cast<int>((static_cast<int64_t>(blockIdx.x + 1) * units) / gridDim.x);

    const int rsg = rg >> 2;
    const int tasks = rsg * p.nsl;
    const bool active = warp < tasks;
    const int sg = active ? warp / p.nsl : 0;
    const int sl = active ? warp % p.nsl : 0;
    const int col = sl * 512 + lane * 16;
    const bool col_ok = active && col < p.kdim;
    // Stage row sg*4 + i belongs to part (row / rgp), projection row (row % rgp).
    int prow[4], ppart[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        ppart[i] = (sg * 4 + i) / p.rgp;
        prow[i] = (sg * 4 + i) - ppart[i] * p.rgp;
    }

    // Per-unit metadata, fetched one unit ahead so its L2 latency overlaps the
    // current unit's compute.
    struct Meta {
        int a_begin, a_end;
        float sc[4];
    };
    auto fetch = [&](int u, Meta& m) {
        const int ei = u / p.gpe, g = u - ei * p.gpe;
        const int row0 = g * p.rgp;
        const int nr = min(p.rgp, p.nrows - row0);
        const uint8_t* rec = reinterpret_cast<const uint8_t*>(
            __ldcg(reinterpret_cast<const unsigned long long*>(p.recs) + ei));
        m.a_begin = ld_cg_i32(p.off + ei);
        m.a_end = ld_cg_i32(p.off + ei + 1);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            m.sc[i] = 0.0f;
            if (col_ok && prow[i] < nr) {
                const float* sp = reinterpret_cast<const float*>(rec + (ppart[i] ? p.s_off[1] : p.s_off[0]));
                m.sc[i] = __ldg(scale_ptr(sp, p.layout, p.kdim, row0 + prow[i], col));
            }
        }
    };

    float2 xr[TB][8];
    int x_expert = -1, x_a0 = -1;
    int parity = 0;
    Meta cur, nxt;
    if (u0 < u1) fetch(u0, nxt);

    for (int u = u0, s = 0; u < u1; u++, s++) {
        const int slot = s % kGemvStages;
        const int ei = u / p.gpe, g = u - ei * p.gpe;
        const int row0 = g * p.rgp;
        const int nr = min(p.rgp, p.nrows - row0);
        cur = nxt;
        if (u + 1 < u1) fetch(u + 1, nxt);
        if (!mbar_wait(&full[slot], (s / kGemvStages) & 1, p.err, ERR_FULL_WAIT)) return;
        const uint8_t* base = stage_buf + slot * kGemvStageBytes + col;

        for (int a0 = cur.a_begin; a0 < cur.a_end; a0 += TB) {
            const int nb = min(TB, cur.a_end - a0);
            if (col_ok && (x_expert != ei || x_a0 != a0)) {
#pragma unroll
                for (int b = 0; b < TB; b++) {
                    if (b < nb) {
                        if (PARTS == 2) {
                            const int tok = ld_cg_i32(p.assign_tok + a0 + b);
                            load_x16<XBF16>(p.x, static_cast<int64_t>(tok) * p.kdim + col, xr[b]);
                        } else {
                            load_x16_cg<false>(p.x, static_cast<int64_t>(a0 + b) * p.kdim + col, xr[b]);
                        }
                    }
                }
                x_expert = ei;
                x_a0 = a0;
            }
            float v[V];
#pragma unroll
            for (int i = 0; i < V; i++) v[i] = 0.0f;
            if (col_ok) {
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    if (prow[i] < nr) {
                        const uint4 w = *reinterpret_cast<const uint4*>(base + (sg * 4 + i) * stride);
#pragma unroll
                        for (int b = 0; b < TB; b++)
                            if (b < nb) v[i * TB + b] = dot16_e4m3(w, xr[b]) * cur.sc[i];
                    }
                }
            }
            float* rb = red + parity * kGemvConsumerWarps * V;
            warp_reduce_multi<V>(v, lane);
            if ((lane & (32 / V - 1)) == 0) rb[warp * V + reduce_index<V>(lane, 0)] = v[0];
            asm volatile("bar.sync 1, %0;" ::"r"(kGemvConsumerWarps * 32) : "memory");
            // Outputs of this chunk: nr rows x nb assignments.
            for (int o = threadIdx.x; o < nr * nb; o += kGemvConsumerWarps * 32) {
                const int b = o % nb, r = o / nb;
                float res[PARTS];
#pragma unroll
                for (int part = 0; part < PARTS; part++) {
                    const int srow = part * p.rgp + r;  // stage row
                    const int task0 = (srow >> 2) * p.nsl;
                    const int vi = (srow & 3) * TB + b;
                    float sum = 0.0f;
                    for (int q = 0; q < p.nsl; q++) sum += rb[(task0 + q) * V + vi];
                    res[part] = sum;
                }
                const float val = PARTS == 2 ? silu_f(res[0]) * res[PARTS - 1] : res[0];
                p.out[static_cast<int64_t>(a0 + b) * p.nrows + row0 + r] = val;
            }
            parity ^= 1;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
}

inline size_t moe_smem_bytes() {
    return static_cast<size_t>(kGemvStages) * kGemvStageBytes + 2 * kGemvStages * sizeof(uint64_t) +
           2 * kGemvConsumerWarps * (4 * kMoeTB) * sizeof(float);
}

// Assignments per chunk for a step of t tokens: an expert gets at most one
// assignment per token, so single-token steps need one.
inline int moe_tb(int t) { return t <= 1 ? 1 : kMoeTB; }

// out[t, c] = sum_s w[t, s] * y[slot[t, s], c], in slot order with fmaf
// (moe.cu:155-164).  Four columns per thread.
template <bool OUT_BF16>
__global__ void combine_slots_kernel(const float* y, const int32_t* slot, const float* w, void* out,
                                     int T, int H, int K) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i >= static_cast<int64_t>(T) * H) return;
    const int t = static_cast<int>(i / H), c = static_cast<int>(i % H);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < K; s++) {
        const float ws = __ldcg(w + t * K + s);
        const int a = __ldcg(slot + t * K + s);
        const float4 v = __ldcg(reinterpret_cast<const float4*>(y + static_cast<int64_t>(a) * H + c));
        acc.x = fmaf(ws, v.x, acc.x);
        acc.y = fmaf(ws, v.y, acc.y);
        acc.z = fmaf(ws, v.z, acc.z);
        acc.w = fmaf(ws, v.w, acc.w);
    }
    if (OUT_BF16) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
        __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
        uint2 pk;
        pk.x = *reinterpret_cast<unsigned*>(&lo);
        pk.y = *reinterpret_cast<unsigned*>(&hi);
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + i) = pk;
    } else {
        *reinterpret_cast<float4*>(static_cast<float*>(out) + i) = acc;
    }
}

// out = routed + sigmoid(gate_logit[t]) * shared (ops.cu:311-316).
__global__ void moe_combine_kernel(const float* routed, const float* shared, const float* gate_logit,
                                   float* out, int T, int H) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(T) * H) return;
    const float g = gate_logit[i / H];
    out[i] = routed[i] + (1.0f / (1.0f + expf(-g))) * shared[i];
}

}  // namespace oomb
