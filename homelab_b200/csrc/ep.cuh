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
// counts, base: epr ints of shared memory each.
__device__ void ep_group_body(const int32_t* rmeta, int G, int T, int K, int epr, const uint64_t* recs_local,
                              int32_t* n_active, int32_t* off, int32_t* assign_row, int32_t* assign_ret,
                              uint64_t* recs_active, unsigned* err, int32_t* counts, int32_t* base) {
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

// Shared memory: counts [epr] and base [epr] ints.
__global__ void __launch_bounds__(kEpThreads) ep_group_kernel(const int32_t* rmeta, int G, int T, int K, int epr,
                                                             const uint64_t* recs_local, int32_t* n_active,
                                                             int32_t* off, int32_t* assign_row, int32_t* assign_ret,
                                                             uint64_t* recs_active, unsigned* err) {
    extern __shared__ int32_t ep_sm[];
    pdl_wait();
    pdl_launch_dependents();
    ep_group_body(rmeta, G, T, K, epr, recs_local, n_active, off, assign_row, assign_ret, recs_active, err, ep_sm,
                  ep_sm + epr);
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

// ---- exchange through peer memory ----------------------------------------------
//
// The fixed-size all-to-alls of a step, done by the kernels themselves over
// NVLink instead of by a collective library: every rank has a mailbox (the same
// layout on every rank, mapped into every peer through CUDA IPC); a sender
// stores its chunk straight into the destination rank's mailbox (plain peer
// stores; chunks packed with the step's token count, the same on every rank),
// then - after a system-scope fence - stores the step's epoch into
// the destination's flag for this source; a receiver polls its own flags
// (acquire) before it reads.  The epoch is the mailbox's step counter + 1; the
// combine's last block advances the counter at the end of the step.  One set
// of buffers suffices: a rank can dispatch step n + 1 only after its combine of
// step n has every peer's return, which each peer sends after it has finished
// reading its step-n inputs.

struct EpMailbox {
    size_t counter, tickets, flags_dispatch, flags_return, meta, x, back, back_words, meta_words, x_words, total;
};

// Layout for `ranks` ranks of up to t_max tokens, top-k slots, hidden h,
// activation element size xb.
__host__ __device__ inline EpMailbox ep_mailbox(int ranks, int t_max, int k, int h, int xb) {
    auto up = [](size_t v) { return (v + 255) & ~static_cast<size_t>(255); };
    EpMailbox m{};
    size_t o = 0;
    m.counter = o; o += 4;
    m.tickets = o; o = up(o + 8);
    m.flags_dispatch = o; o = up(o + static_cast<size_t>(ranks) * 4);
    m.flags_return = o; o = up(o + static_cast<size_t>(ranks) * 4);
    m.meta = o; o = up(o + static_cast<size_t>(ranks) * t_max * k * 4);
    m.x = o; o = up(o + static_cast<size_t>(ranks) * t_max * h * xb);
    m.back = o; o = up(o + static_cast<size_t>(ranks) * t_max * k * static_cast<size_t>(h) * 4);
    // the one-launch step's returned rows: (epoch, value) words, [ranks][t * k][h]
    m.back_words = o; o = up(o + static_cast<size_t>(ranks) * t_max * k * static_cast<size_t>(h) * 8);
    // the one-launch step's dispatch: (epoch, meta) and (epoch, 4 bytes of x) words
    m.meta_words = o; o = up(o + static_cast<size_t>(ranks) * t_max * k * 8);
    m.x_words = o; o = up(o + static_cast<size_t>(ranks) * t_max * static_cast<size_t>(h) * xb * 2);
    m.total = o;
    return m;
}

struct EpPeer {
    const unsigned long long* peers;  // [ranks] mailbox base of every rank (own rank: the local mailbox)
    uint8_t* mailbox;                 // the local mailbox
    int ranks, rank, t_max, k, h, xb;
    unsigned* err;
};

__device__ __forceinline__ unsigned ep_ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// A release fence at system scope: the writes this thread has made or observed
// (through a CTA barrier, for the other threads' writes) are ordered before its
// later writes as every GPU of the node sees them.  With a relaxed flag store
// after it and the reader's acquire load, it is the release pattern the
// hand-offs need; no store-to-load ordering is needed, so not the sequentially
// consistent fence (__threadfence_system), which measured ~8 us a hand-off on
// B200 with every CTA of a launch fencing.
__device__ __forceinline__ void ep_fence_release_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void ep_st_relaxed_sys(unsigned* p, unsigned v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ep_epoch(const EpPeer& q) {
    return __ldcg(reinterpret_cast<const unsigned*>(q.mailbox + ep_mailbox(q.ranks, q.t_max, q.k, q.h, q.xb).counter)) +
           1u;
}

// Threads 0 .. ranks-1 wait for the local flags of every source rank to carry
// `epoch` (bounded); then the CTA synchronises.  False in every thread when a
// wait ran out.
__device__ __forceinline__ bool ep_wait_flags(const unsigned* flags, int ranks, unsigned epoch, unsigned* err,
                                              unsigned code) {
    __shared__ int failed;
    if (threadIdx.x == 0) failed = 0;
    __syncthreads();
    for (int g = threadIdx.x; g < ranks; g += blockDim.x) {
        if (ep_ld_acquire_sys(flags + g) != epoch) {
            const unsigned long long t0 = global_ns(), limit = wait_limit();
            while (ep_ld_acquire_sys(flags + g) != epoch) {
                if (global_ns() - t0 > limit) {
                    record_error(err, code);
                    failed = 1;
                    break;
                }
            }
        }
    }
    __syncthreads();
    return failed == 0;
}

// 16-byte copy of n bytes (n % 16 == 0, both 16-byte aligned) by the CTA.
__device__ __forceinline__ void ep_copy16(uint8_t* dst, const uint8_t* src, size_t n) {
    for (size_t i = static_cast<size_t>(threadIdx.x) * 16; i < n; i += static_cast<size_t>(blockDim.x) * 16)
        *reinterpret_cast<uint4*>(dst + i) = __ldcg(reinterpret_cast<const uint4*>(src + i));
}

enum : unsigned { ERR_EP_DISPATCH_WAIT = 0x700, ERR_EP_RETURN_WAIT = 0x710 };

// Dispatch: block g writes, into rank g's mailbox, this rank's meta for g (the
// local id on g of each slot's expert, or -1) and its T activation rows, then
// raises this rank's dispatch flag there.
__global__ void __launch_bounds__(kEpThreads) ep_dispatch_kernel(EpPeer q, const int32_t* ids, int T, int epr,
                                                                 const void* x) {
    pdl_wait();
    pdl_launch_dependents();
    const int g = blockIdx.x;
    const EpMailbox m = ep_mailbox(q.ranks, q.t_max, q.k, q.h, q.xb);
    uint8_t* dst = reinterpret_cast<uint8_t*>(q.peers[g]);
    const unsigned epoch = ep_epoch(q);
    int32_t* meta = reinterpret_cast<int32_t*>(dst + m.meta) + static_cast<size_t>(q.rank) * T * q.k;
    for (int i = threadIdx.x; i < T * q.k; i += blockDim.x) {
        const int e = __ldcg(ids + i);
        if (e < 0 || e >= q.ranks * epr) {
            record_error(q.err, ERR_BAD_TABLE);
            meta[i] = -1;
        } else {
            meta[i] = e / epr == g ? e - g * epr : -1;
        }
    }
    ep_copy16(dst + m.x + static_cast<size_t>(q.rank) * T * q.h * q.xb, static_cast<const uint8_t*>(x),
              static_cast<size_t>(T) * q.h * q.xb);
    __syncthreads();
    if (threadIdx.x == 0) {
        ep_fence_release_sys();
        ep_st_relaxed_sys(reinterpret_cast<unsigned*>(dst + m.flags_dispatch) + q.rank, epoch);
    }
}

// The grouping of ep_group_kernel over the mailbox's received meta, after every
// source rank's dispatch flag carries this step's epoch.  One CTA; shared
// memory as ep_group_kernel.
__global__ void __launch_bounds__(kEpThreads) ep_group_peer_kernel(EpPeer q, int T, int epr,
                                                                  const uint64_t* recs_local, int32_t* n_active,
                                                                  int32_t* off, int32_t* assign_row,
                                                                  int32_t* assign_ret, uint64_t* recs_active) {
    extern __shared__ int32_t ep_sm[];
    pdl_wait();
    pdl_launch_dependents();
    const EpMailbox m = ep_mailbox(q.ranks, q.t_max, q.k, q.h, q.xb);
    if (!ep_wait_flags(reinterpret_cast<const unsigned*>(q.mailbox + m.flags_dispatch), q.ranks, ep_epoch(q), q.err,
                       ERR_EP_DISPATCH_WAIT)) {
        if (threadIdx.x == 0) {
            *n_active = 0;  // nothing runs on a failed step; the error word says why
            off[0] = 0;
        }
        return;
    }
    ep_group_body(reinterpret_cast<const int32_t*>(q.mailbox + m.meta), q.ranks, T, q.k, epr, recs_local, n_active,
                  off, assign_row, assign_ret, recs_active, q.err, ep_sm, ep_sm + epr);
}

// Return: each output row goes straight to its source rank's mailbox, row
// (this rank, slot) of the returned rows; the last block to finish raises this
// rank's return flag on every rank.
__global__ void ep_return_kernel(EpPeer q, const float* y, const int32_t* n_active, const int32_t* off,
                                 const int32_t* assign_ret, int T) {
    pdl_wait();
    pdl_launch_dependents();
    const EpMailbox m = ep_mailbox(q.ranks, q.t_max, q.k, q.h, q.xb);
    const unsigned epoch = ep_epoch(q);
    const int A = __ldcg(off + __ldcg(n_active));
    const int per_row = q.h / 4;
    const int64_t n = static_cast<int64_t>(A) * per_row;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int a = static_cast<int>(i / per_row), c = static_cast<int>(i - static_cast<int64_t>(a) * per_row);
        const int r = __ldcg(assign_ret + a);  // g * T*K + t*K + s
        const int g = r / (T * q.k), ts = r - g * T * q.k;
        float* back = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(q.peers[g]) + m.back);
        const float4 v = __ldcg(reinterpret_cast<const float4*>(y + static_cast<int64_t>(a) * q.h) + c);
        reinterpret_cast<float4*>(back + (static_cast<int64_t>(q.rank) * T * q.k + ts) * q.h)[c] = v;
    }
    __syncthreads();
    __shared__ bool last;
    unsigned* ticket = reinterpret_cast<unsigned*>(q.mailbox + m.tickets);
    if (threadIdx.x == 0) {
        ep_fence_release_sys();
        last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    if (threadIdx.x == 0) *ticket = 0u;
    ep_fence_release_sys();
    for (int g = threadIdx.x; g < q.ranks; g += blockDim.x)
        ep_st_relaxed_sys(reinterpret_cast<unsigned*>(reinterpret_cast<uint8_t*>(q.peers[g]) + m.flags_return) + q.rank,
                          epoch);
}

// ep_combine_kernel over the mailbox's returned rows, after every rank's return
// flag carries this step's epoch; the last block advances the step counter.
template <bool OUT_BF16>
__global__ void ep_combine_peer_kernel(EpPeer q, const int32_t* ids, const float* w, int T, int epr, void* out) {
    pdl_wait();
    pdl_launch_dependents();
    const EpMailbox m = ep_mailbox(q.ranks, q.t_max, q.k, q.h, q.xb);
    const unsigned epoch = ep_epoch(q);
    const bool ok = ep_wait_flags(reinterpret_cast<const unsigned*>(q.mailbox + m.flags_return), q.ranks, epoch,
                                  q.err, ERR_EP_RETURN_WAIT);
    const float* back = reinterpret_cast<const float*>(q.mailbox + m.back);
    const int K = q.k, H = q.h;
    if (ok) {
        for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < static_cast<int64_t>(T) * H;
             i += static_cast<int64_t>(gridDim.x) * blockDim.x * 4) {
            const int t = static_cast<int>(i / H), c = static_cast<int>(i % H);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int s = 0; s < K; s++) {
                const int e = __ldcg(ids + t * K + s);
                const float ws = __ldcg(w + t * K + s);
                const int g = min(max(e / epr, 0), q.ranks - 1);
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
    }
    // every block has read the epoch: the last one advances the step counter
    __syncthreads();
    __shared__ bool last;
    unsigned* ticket = reinterpret_cast<unsigned*>(q.mailbox + m.tickets) + 1;
    if (threadIdx.x == 0) last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    if (last && threadIdx.x == 0) {
        *ticket = 0u;
        *reinterpret_cast<unsigned*>(q.mailbox + m.counter) = epoch;
    }
}

}  // namespace oomb
