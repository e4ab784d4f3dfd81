// ep.cuh - expert parallelism: the device side of dispatch and combine.
//
// Experts are sharded over G ranks, expert e on rank e / epr (epr = experts per
// rank).  A step on every rank: route the rank's T tokens (replicated router);
// ep_meta_kernel writes, for every destination rank g, meta[g][t][s] = the
// local id on g of the expert of slot s of token t, or -1 when that expert
// lives elsewhere; the rank's activations and meta go to every rank (fixed-size
// all-to-all, no host round trip); ep_group_kernel groups the received
// assignments by local expert in (source rank, token, slot) order - the order
// the single-GPU path gives the same assignments - and lists the active experts
// and their records; the expert kernels run on that grouping;
// ep_scatter_kernel puts each output row at its slot's place in the return
// buffer of its source rank, [G][T*K][H]; after the reverse all-to-all,
// ep_combine_kernel sums each token's slots in slot order with fused
// multiply-adds (moe_combine_slots, moe.cu:155-164), reading slot s from the
// rank that owns its expert.  Every expert output is computed by the same
// arithmetic as on one GPU, so the combined result is bit-identical to it.
#pragma once

#include "common.cuh"

namespace oomb {

constexpr int kEpThreads = 256;

// meta[g][t][s] for g < G: local expert id of ids[t][s] on rank g, or -1.
__global__ void ep_meta_kernel(const int32_t* ids, int T, int K, int epr, int G, int32_t* meta, unsigned* err) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t n = static_cast<int64_t>(G) * T * K;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int g = static_cast<int>(i / (static_cast<int64_t>(T) * K));
        const int ts = static_cast<int>(i - static_cast<int64_t>(g) * T * K);
        const int e = __ldcg(ids + ts);
        if (e < 0 || e >= G * epr) {
            record_error(err, ERR_BAD_TABLE);
            meta[i] = -1;
        } else {
            meta[i] = e / epr == g ? e - g * epr : -1;
        }
    }
}

// Groups the received assignments rmeta[g][t][s] (local expert or -1) by local
// expert, ordered by (g, t, s) within an expert.  One CTA.  Outputs as the
// route kernel's grouping: n_active, off[n_active + 1], assign_row[A] (row
// g * T + t of the received activations), assign_ret[A] (row g * T*K + t*K + s
// of the return buffer), recs_active[n_active] = recs_local[expert].
// Shared memory: counts [epr] and base [epr] ints.
__global__ void __launch_bounds__(kEpThreads) ep_group_kernel(const int32_t* rmeta, int G, int T, int K, int epr,
                                                             const uint64_t* recs_local, int32_t* n_active,
                                                             int32_t* off, int32_t* assign_row, int32_t* assign_ret,
                                                             uint64_t* recs_active, unsigned* err) {
    extern __shared__ int32_t ep_sm[];
    int32_t* counts = ep_sm;
    int32_t* base = ep_sm + epr;
    // the records table is the layer's: fetch it before waiting on the previous kernel
    pdl_wait();
    pdl_launch_dependents();
    const int n = G * T * K;
    for (int e = threadIdx.x; e < epr; e += blockDim.x) counts[e] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int e = __ldcg(rmeta + i);
        if (e >= epr) record_error(err, ERR_BAD_TABLE);
        else if (e >= 0) atomicAdd(&counts[e], 1);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        // exclusive scans over local experts: assignment start and active index
        const int lane = threadIdx.x;
        int run_a = 0, run_n = 0;
        for (int e0 = 0; e0 < epr; e0 += 32) {
            const int e = e0 + lane;
            const int c = e < epr ? counts[e] : 0;
            int inc_a = c, inc_n = c > 0 ? 1 : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int va = __shfl_up_sync(0xffffffffu, inc_a, o);
                const int vn = __shfl_up_sync(0xffffffffu, inc_n, o);
                if (lane >= o) {
                    inc_a += va;
                    inc_n += vn;
                }
            }
            const int start = run_a + inc_a - c;
            const int idx = run_n + inc_n - (c > 0 ? 1 : 0);
            if (e < epr && c > 0) {
                base[e] = start;
                off[idx] = start;
                recs_active[idx] = recs_local[e];
            }
            run_a += __shfl_sync(0xffffffffu, inc_a, 31);
            run_n += __shfl_sync(0xffffffffu, inc_n, 31);
        }
        if (lane == 0) {
            off[run_n] = run_a;
            *n_active = run_n;
        }
        // ranks within an expert in (g, t, s) order, 32 entries at a time
        for (int i0 = 0; i0 < n; i0 += 32) {
            const int i = i0 + lane;
            const int e0v = i < n ? __ldcg(rmeta + i) : -1;
            const int e = (e0v >= 0 && e0v < epr) ? e0v : -1 - lane;  // unique dummies for idle lanes
            const unsigned peers = __match_any_sync(0xffffffffu, e);
            const int rank = __popc(peers & ((1u << lane) - 1u));
            if (e >= 0) {
                const int a = base[e] + rank;
                const int g = i / (T * K), ts = i - g * T * K;
                assign_row[a] = g * T + ts / K;
                assign_ret[a] = i;
            }
            __syncwarp();
            if (e >= 0 && (peers >> lane) == 1u) base[e] += rank + 1;
            __syncwarp();
        }
    }
}

// ret[assign_ret[a]][:] = y[a][:] for a < A (A read from off[n_active]).
__global__ void ep_scatter_kernel(const float* y, const int32_t* n_active, const int32_t* off,
                                  const int32_t* assign_ret, int H, float* ret) {
    pdl_wait();
    pdl_launch_dependents();
    const int A = __ldcg(off + __ldcg(n_active));
    const int per_row = H / 4;
    const int64_t n = static_cast<int64_t>(A) * per_row;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int a = static_cast<int>(i / per_row), c = static_cast<int>(i - static_cast<int64_t>(a) * per_row);
        const int r = __ldcg(assign_ret + a);
        const float4 v = __ldcg(reinterpret_cast<const float4*>(y + static_cast<int64_t>(a) * H) + c);
        reinterpret_cast<float4*>(ret + static_cast<int64_t>(r) * H)[c] = v;
    }
}

// out[t, c] = sum_s w[t, s] * back[owner(ids[t, s])][t*K + s][c] in slot order
// with fmaf, owner(e) = e / epr.  back: [G][T*K][H] fp32 (the returned rows).
template <bool OUT_BF16>
__global__ void ep_combine_kernel(const float* back, const int32_t* ids, const float* w, int T, int K, int H, int epr,
                                  int G, void* out) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i >= static_cast<int64_t>(T) * H) return;
    const int t = static_cast<int>(i / H), c = static_cast<int>(i % H);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < K; s++) {
        const int e = __ldcg(ids + t * K + s);
        const float ws = __ldcg(w + t * K + s);
        const int g = min(max(e / epr, 0), G - 1);
        const float4 v = __ldcg(reinterpret_cast<const float4*>(
            back + (static_cast<int64_t>(g) * T * K + static_cast<int64_t>(t) * K + s) * H + c));
        acc.x = fmaf(ws, v.x, acc.x);
        acc.y = fmaf(ws, v.y, acc.y);
        acc.z = fmaf(ws, v.z, acc.z);
        acc.w = fmaf(ws, v.w, acc.w);
    }
    if (OUT_BF16) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
        uint2 pk;
        pk.x = *reinterpret_cast<unsigned*>(&lo);
        pk.y = *reinterpret_cast<unsigned*>(&hi);
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + i) = pk;
    } else {
        *reinterpret_cast<float4*>(static_cast<float*>(out) + i) = acc;
    }
}

}  // namespace oomb
