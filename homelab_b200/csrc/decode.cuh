// decode.cuh - one routed-MoE decode step (router GEMV, softmax top-k, grouping,
// gate/up+SiLU, down, slot-order combine) in one persistent launch.
//
// The routed half of Moe::forward (crates/oominf-models-qwen/src/moe.rs:254-366
// with begin_routed / finish_routed, moe.rs:532-582, 638-659) for a layer whose
// experts are all resident, with the arithmetic of the separate kernels
// (route.cuh, stream.cuh, combine.cuh): every output is bit-identical to the
// chain route_kernel -> gate/up -> down -> combine_slots.
//
// Every CTA of the grid (one or two per SM, all resident at once) runs:
//   1. before the dependency wait: its router rows land in shared memory by
//      bulk copy, and the layer's record table is fetched;
//   2. CTA c < ceil(E / 8) computes the logits of router rows 8c .. 8c + 7 (a
//      warp each) for every token (activations staged by one bulk copy after
//      the wait, when they fit; few CTAs read them, so their lines are not a
//      hot spot), writes them to global memory; a grid barrier, then every
//      CTA loads all T x E logits into shared memory;
//   3. softmax top-k and grouping of all tokens from the logits, the same in
//      every CTA (deterministic), into shared-memory routing tables: no
//      second hand-off through global memory.  From two tokens (p.singles) every
//      slot is a group of its own, so the streaming phases keep their one-token
//      form (an expert picked twice streams twice; measured on B200 at config 2,
//      8 tokens: 95 us a step against 158 grouped by expert with two-token units);
//   4. the streaming engine over the CTA's slice of gate/up units, then of down
//      units, through one weight ring: the copy producer runs straight on from
//      gate/up into down, so the down weights stream in while gate/up finishes
//      and the consumers wait at the second grid barrier (down reads every h row
//      of its expert);
//   5. per down row group a counter; the CTA whose unit completes a group (the
//      last of the n_e experts) combines that group's rows of every token in
//      slot order and writes the output.
// The two grid barriers count arrivals in a slot of a ring indexed by a launch
// epoch, so a CTA that starts late (launches overlap under programmatic
// dependent launch) cannot disturb a count it does not own: every CTA reads
// the epoch word after the dependency wait and uses epoch + 1; CTA 0 zeroes the
// slot two launches ahead (last used by a launch that has completed, next used
// by one that cannot start before this one completes) and stores the epoch
// back once every CTA has arrived at the second barrier (so all have read it).
// An arrival is a release add, a wait one thread per CTA polling the count with
// acquire loads: a single hot word, polled by one thread of each CTA.  All
// waits are bounded.  The row-group counters are reset by the CTA that
// completes the group.  The host launches only a grid that fits on the GPU at
// once.
#pragma once

#include "ep.cuh"
#include "route.cuh"
#include "stream.cuh"

namespace oomb {

constexpr int kDecodeMaxT = 16;         // tokens per launch
// Stages each CTA keeps in flight (0: the whole ring).  All CTAs start streaming
// at once after routing; with the whole ring requested, every CTA's stages land
// together at the end of a ~28 MB burst and its consumers start late.  One stage
// per CTA (2 per SM, ~9.5 MB in flight) still keeps HBM busy, and consumption
// follows arrival: measured on B200, config 2 batch 1, 27.33 us per step with the
// whole ring, 26.97 with two stages, 26.02 with one.
#ifndef OOMB_DECODE_LAG
#define OOMB_DECODE_LAG 1
#endif
constexpr int kDecodeLag = OOMB_DECODE_LAG;
// The same for the one-token down phase's weight stages (they do not depend on
// h, so they can go out as soon as gate/up frees ring slots; 0: no limit).
#ifndef OOMB_DECODE_DOWN_LAG
#define OOMB_DECODE_DOWN_LAG OOMB_DECODE_LAG
#endif
constexpr int kDecodeDownLag = OOMB_DECODE_DOWN_LAG;
constexpr int kDecodeMaxGroups = 512;   // down row groups (combine counters, bitmap bits)
// sync-area words: the launch epoch; a ring of 4 slots of the grid barriers'
// arrival counts (slot epoch % 4, three counts 32 words apart); the row-group counters
constexpr int kSyncSlot = 3 * 32;
constexpr int kSyncEpoch = 0, kSyncBars = 32, kSyncGroups = kSyncBars + 4 * kSyncSlot;
constexpr int kSyncWords = kSyncGroups + kDecodeMaxGroups;

enum : unsigned {
    ERR_GRID_WAIT = 0x600,    // a grid barrier ran out (CTAs not resident together)
    ERR_ROUTER_WAIT = 0x610,  // the router rows never landed in shared memory
};

struct DecodeParams {
    RouteParams r;        // x, x_bf16, w, logits (scratch), T, H, E, K, recs_all, err
    StreamParams gu, dn;  // planned phases: gu.x = x, gu.y = h; dn.x = h, dn.y = y
    unsigned* sync;       // kSyncWords words, zero before first use
    int32_t* ids_out;     // [T, K]
    float* w_out;         // [T, K]
    void* out;            // [T, H]
    int out_bf16;
    int stages, slot_bytes, meta_stride;
    int off_bars, off_red, off_meta, off_chunk, off_tabs;  // shared-memory layout (bytes)
    int x_off;  // ring offset (bytes) of the staged activations, or -1 to read them from global memory
    // expert parallelism (EP kernels): the mailboxes, experts per rank; r.recs_all
    // then holds this rank's epr records, gu.x the mailbox's received activations
    EpPeer ep;
    int epr;
    int dn1;  // one token: the down phase and the combine run per row group in one CTA (down1_*)
    int singles;  // every slot a group of its own (the one-token streaming form for a few tokens)
};

// Routing tables in shared memory (byte offsets from the table area).
struct DecodeTabs {
    int recs, recs_active, rbar, xbar, lg, ids, w, counts, base, active, off, assign_tok, slot_assign, n_active, cbits,
        rmeta, aret, total;
};

// T: this rank's tokens; TA: tokens whose slots are grouped (T, or ranks * T
// with expert parallelism, where every received slot is a group of its own).
__host__ __device__ inline DecodeTabs decode_tabs(int T, int K, int E, int TA) {
    DecodeTabs d{};
    const int A = TA * K;
    const int NG = E > A ? E : A;  // groups at most: experts, or (expert parallelism) received slots
    int o = 0;
    d.recs = o; o += E * 8;
    d.recs_active = o; o += NG * 8;
    d.rbar = o; o += 8;
    d.xbar = o; o += 8;
    d.lg = o; o += T * E * 4;
    d.rmeta = o; o += A * 4;
    d.aret = o; o += A * 4;
    d.ids = o; o += A * 4;
    d.w = o; o += A * 4;
    d.counts = o; o += E * 4;
    d.base = o; o += E * 4;
    d.active = o; o += NG * 4;
    d.off = o; o += (NG + 1) * 4;
    d.assign_tok = o; o += A * 4;
    d.slot_assign = o; o += A * 4;
    d.n_active = o; o += 4;
    d.cbits = o; o += (kDecodeMaxGroups / 32) * 4;
    d.total = (o + 15) & ~15;
    return d;
}

// Bytes of the ring that the routing phase borrows: the CTA's router rows (and
// the staged activations after them), later the softmax probabilities and
// picks.
__host__ __device__ inline size_t decode_ring_borrow(int T, int H, int E, int K, int rows_per_cta, size_t x_bytes) {
    const size_t rows = static_cast<size_t>(rows_per_cta) * H * 2 + x_bytes;
    const size_t ranks = (static_cast<size_t>(T) * E + 2 * static_cast<size_t>(T) * K) * 4;
    return rows > ranks ? rows : ranks;
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_relaxed_u32(unsigned* p, unsigned v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One thread per CTA, after a CTA barrier that follows the writes to publish:
// a release add to the arrival count at ctr.
__device__ __forceinline__ void bar_arrive(unsigned* ctr) {
    fence_acq_rel_gpu();
    asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
}

// One thread per CTA: polls the arrival count at ctr (acquire) until it reaches
// n.  False when the wait ran out (the error code is recorded).
// Pause between polls of a grid barrier's count: one thread of every CTA polls
// the same line that every CTA's arrival updates.  Measured on B200, config 2
// batch 1: 23.50 us a step polling back to back, 23.15 with 64 or 200 ns.
#ifndef OOMB_BAR_BACKOFF_NS
#define OOMB_BAR_BACKOFF_NS 64
#endif
__device__ __forceinline__ bool bar_wait(const unsigned* ctr, unsigned n, unsigned* err, unsigned code) {
    if (ld_acquire_u32(ctr) >= n) return true;
    const unsigned long long t0 = global_ns(), limit = wait_limit();
    while (ld_acquire_u32(ctr) < n) {
        if (OOMB_BAR_BACKOFF_NS > 0) __nanosleep(OOMB_BAR_BACKOFF_NS);
        if (global_ns() - t0 > limit) {
            record_error(err, code);
            return false;
        }
    }
    return true;
}

// Expert parallelism: every received slot of a local expert (meta entry >= 0;
// -1 marks another rank's) becomes a group of its own, in (source rank, token,
// slot) order: assign_tok = the received token row, assign_ret = the slot's return
// index.  Every group then holds one assignment, so the streaming phases run their
// one-token form (an expert picked by two slots streams twice: rare at the batch
// sizes this step serves).  One warp; all its lanes call this.
__device__ void group_singletons(const RouteParams& p, const GroupOut& g, const int32_t* meta,
                                 const uint64_t* recs_sm) {
    const int lane = threadIdx.x & 31;
    const int n = p.T * p.K;
    int run = 0;
    for (int i0 = 0; i0 < n; i0 += 32) {
        const int i = i0 + lane;
        const int e = i < n ? meta[i] : -1;
        const bool valid = e >= 0 && e < p.E;
        if (e >= p.E) record_error(p.err, ERR_BAD_TABLE);
        const unsigned vm = __ballot_sync(0xffffffffu, valid);
        if (valid) {
            const int idx = run + __popc(vm & ((1u << lane) - 1u));
            g.active[idx] = e;
            g.off[idx] = idx;
            g.assign_tok[idx] = i / p.K;
            g.assign_ret[idx] = i;
            g.recs_active[idx] = recs_sm[e];
        }
        run += __popc(vm);
    }
    if (lane == 0) {
        g.off[run] = run;
        *g.n_active = run;
    }
}

// Every slot of the step a group of its own, in slot order (one warp; all its
// lanes call this): group i = slot i, so each group holds one assignment and the
// streaming phases run their one-token form; an expert picked by two slots
// streams twice.  A slot with an invalid expert id is recorded as an error and
// left out.
__device__ void group_slots(const RouteParams& p, const GroupOut& g, const int32_t* ids_sm, const uint64_t* recs_sm) {
    const int lane = threadIdx.x & 31;
    const int n = p.T * p.K;
    int run = 0;
    for (int i0 = 0; i0 < n; i0 += 32) {
        const int i = i0 + lane;
        const int e = i < n ? ids_sm[i] : -1;
        const bool valid = i < n && e >= 0 && e < p.E;
        if (i < n && !valid) record_error(p.err, ERR_BAD_TABLE);
        const unsigned vm = __ballot_sync(0xffffffffu, valid);
        const int idx = run + __popc(vm & ((1u << lane) - 1u));
        if (valid) {
            g.active[idx] = e;
            g.off[idx] = idx;
            g.assign_tok[idx] = i / p.K;
            g.recs_active[idx] = recs_sm[e];
        }
        if (i < n) g.slot_assign[i] = valid ? idx : 0;
        run += __popc(vm);
    }
    if (lane == 0) {
        g.off[run] = run;
        *g.n_active = run;
    }
}

__device__ __forceinline__ void consumers_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kWarps * 32) : "memory"); }

// Logits of router row e (bf16, in shared memory) for tokens [t0, t0 + nt):
// the canonical order of router_row_dot (per lane one fmaf chain over columns
// 256*i + 8*lane + j, i ascending, then the xor tree).  Activations from
// global memory, or staged in shared memory (XSM, rows of p.H).  The logits go
// to p.logits.  Written as short loops (one token at a time): this code runs
// once per launch, so its instruction fetch costs more than its arithmetic.
template <bool XBF16, bool XSM>
__device__ __forceinline__ void logits_row(const RouteParams& p, const uint8_t* wrow, const uint8_t* xsm, int e, int t0,
                                           int nt, int lane) {
#pragma unroll 1
    for (int t = t0; t < t0 + nt; t++) {
        float acc = 0.0f;
#pragma unroll 2
        for (int base = lane * 8; base < p.H; base += 256) {
            const uint4 wv = *reinterpret_cast<const uint4*>(wrow + static_cast<size_t>(base) * 2);
            const unsigned ww[4] = {wv.x, wv.y, wv.z, wv.w};
            const int64_t xi = static_cast<int64_t>(t) * p.H + base;
            float xv[8];
            if (XBF16) {
                const uint4* xp = XSM ? reinterpret_cast<const uint4*>(xsm + xi * 2)
                                      : reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.x) + xi);
                const uint4 a = XSM ? *xp : __ldcg(xp);
                const unsigned aa[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    xv[2 * q] = __uint_as_float(aa[q] << 16);
                    xv[2 * q + 1] = __uint_as_float(aa[q] & 0xffff0000u);
                }
            } else {
                const float4* xp = XSM ? reinterpret_cast<const float4*>(xsm + xi * 4)
                                       : reinterpret_cast<const float4*>(static_cast<const float*>(p.x) + xi);
                const float4 a = XSM ? xp[0] : __ldcg(xp), b = XSM ? xp[1] : __ldcg(xp + 1);
                xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w;
                xv[4] = b.x; xv[5] = b.y; xv[6] = b.z; xv[7] = b.w;
            }
#pragma unroll
            for (int q = 0; q < 4; q++) {
                acc = __fmaf_rn(xv[2 * q], __uint_as_float(ww[q] << 16), acc);
                acc = __fmaf_rn(xv[2 * q + 1], __uint_as_float(ww[q] & 0xffff0000u), acc);
            }
        }
        const float v = xor_tree32(acc);
        if (lane == 0) p.logits[static_cast<int64_t>(t) * p.E + e] = v;
    }
}

// ---- one token: down and combine per row group ----
// With one token the step's K assignments are its K slots, one per expert.  A
// CTA owns row groups of 8 output rows.  For each it streams the group's 8 rows
// of every slot's down matrix (stages of `spp` slots), warp w computes the 8
// outputs of slots w, w + kWarps, ... with the arithmetic of the stand-alone
// down kernel (the same 16-column lane slices of 512-column slabs, block scales,
// fp32 dot products, lane tree and slab order, so every y is bit-identical to
// it), and the CTA combines the group's slots in slot order right away: no y
// rows through L2, no counters between CTAs, no last-arriver hand-off.
#ifndef OOMB_DECODE_DOWN1
#define OOMB_DECODE_DOWN1 1
#endif
struct Down1 {
    int spp, nst;  // slots per stage, stages per row group
};
__host__ __device__ inline Down1 down1_plan(int K, int I, int slot_bytes) {
    Down1 d;
    d.spp = slot_bytes / (8 * I);
    if (d.spp > K) d.spp = K;
    d.nst = d.spp > 0 ? (K + d.spp - 1) / d.spp : 0;
    return d;
}

// Copy producer: row groups [g0, g1) from ring position s on.
__device__ bool down1_copy(const StreamParams& dn, const int32_t* ids_sm, const uint64_t* recs_sm, int K,
                           const Ring& rg, int g0, int g1, int& s, int lag) {
    const int S = rg.stages, I = dn.k;
    const Down1 d = down1_plan(K, I, rg.slot_bytes);
    const unsigned rows8 = static_cast<unsigned>(8 * I);
    const uint64_t pol = make_evict_first_policy();
    const int s_begin = s;
    bool ok = true;
    for (int g = g0; g < g1 && ok; g++) {
        for (int q = 0; q < d.nst; q++, s++) {
            const int slot = s % S;
            ok = mbar_wait(&rg.empty[slot], ((s / S) & 1) ^ 1, dn.err, ERR_EMPTY_WAIT);
            if (ok && lag > 0 && lag < S && s >= lag)
                ok = mbar_wait(&rg.full[(s - lag) % S], ((s - lag) / S) & 1, dn.err, ERR_EMPTY_WAIT);
            if (!ok) break;
            const int s0 = q * d.spp, ns = min(d.spp, K - s0);
            mbar_arrive_expect_tx(&rg.full[slot], static_cast<unsigned>(ns) * rows8);
            uint8_t* dst = rg.stage_buf + slot * rg.slot_bytes;
            for (int i = 0; i < ns; i++) {
                const uint8_t* rec = reinterpret_cast<const uint8_t*>(recs_sm[ids_sm[s0 + i]]);
                bulk_g2s(dst + i * rows8, rec + dn.w_off[0] + static_cast<int64_t>(g) * rows8, rows8, &rg.full[slot],
                         pol);
            }
        }
    }
    if (!ok) {
        for (int t = max(s_begin, s - S); t < s; t++) mbar_wait(&rg.full[t % S], (t / S) & 1, dn.err, ERR_DRAIN_WAIT);
    }
    return ok;
}

// Consumers: row groups [g0, g1) from ring position pos.s on; V: partials per
// lane (8 rows x slabs, rounded up to a power of two).  ysm: K x 8 floats.
template <bool BLK, int V>
__device__ bool down1_consume(const DecodeParams& p, const int32_t* ids_sm, const float* w_sm, const int32_t* slot_sm,
                              const uint64_t* recs_sm, int K, const Ring& rg, int g0, int g1, RingPos& pos, float* ysm) {
    const StreamParams& dn = p.dn;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = rg.stages, I = dn.k;
    const Down1 d = down1_plan(K, I, rg.slot_bytes);
    const int nsl = (I + 511) / 512;
    constexpr int VS = V / 8;  // partials per row
    const uint64_t keep = make_evict_last_policy();
    const float* h = static_cast<const float*>(dn.x);
    int s = pos.s;
    for (int g = g0; g < g1; g++, s += d.nst) {
        const int row0 = g * 8;
        for (int si = warp; si < K; si += kWarps) {
            const uint8_t* rec = reinterpret_cast<const uint8_t*>(recs_sm[ids_sm[si]]);
            const float* scl = reinterpret_cast<const float*>(rec + dn.s_off[0]);
            const int64_t hrow = static_cast<int64_t>(slot_sm[si]) * I;
            const int q = si / d.spp, st = s + q, slot = st % S;
            float v[V];
#pragma unroll
            for (int i = 0; i < V; i++) v[i] = 0.0f;
            // the activation slice and block scales of slab qs (h rows come from L2)
            auto load = [&](int qs, XSlice<false>& xs, float (&sc)[8]) {
                const int col = qs * 512 + lane * 16;
                const bool col_ok = col < I;
                const int kb = (col_ok ? col : 0) >> 7;
                if (col_ok) xs.load(h, hrow + col);
                else xs.zero();
                if (BLK) {
                    const float s0 = ld_scale(scl + static_cast<int64_t>(row0 >> 7) * dn.nb + kb, keep);
#pragma unroll
                    for (int j = 0; j < 8; j++) sc[j] = s0;
                } else {
#pragma unroll
                    for (int j = 0; j < 8; j++) sc[j] = ld_scale(scl + static_cast<int64_t>(row0 + j) * dn.nb + kb, keep);
                }
            };
            auto dot8 = [&](int qs, const XSlice<false>& xs, const float (&sc)[8]) {
                const int col = qs * 512 + lane * 16;
                const int ccol = col < I ? col : 0;
                const uint8_t* base = rg.stage_buf + slot * rg.slot_bytes + (si - q * d.spp) * 8 * I + ccol;
                uint4 raw[8];
#pragma unroll
                for (int j = 0; j < 8; j++) raw[j] = *reinterpret_cast<const uint4*>(base + j * I);
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    WDec<false> w;
                    w.decode(raw[j]);
                    v[j * VS + qs] = fmaf(xs.dot(w), sc[j] * xs.scale(), 0.0f);
                }
            };
            if constexpr (VS <= 2) {
                // every slab's loads in flight before the stage wait
                XSlice<false> xs[VS];
                float sc[VS][8];
#pragma unroll
                for (int qs = 0; qs < VS; qs++)
                    if (qs < nsl) load(qs, xs[qs], sc[qs]);
                if (!mbar_wait(&rg.full[slot], (st / S) & 1, dn.err, ERR_FULL_WAIT)) return false;
#pragma unroll
                for (int qs = 0; qs < VS; qs++)
                    if (qs < nsl) dot8(qs, xs[qs], sc[qs]);
            } else {
#pragma unroll
                for (int qs = 0; qs < VS; qs++) {
                    if (qs >= nsl) break;
                    XSlice<false> xs;
                    float sc[8];
                    load(qs, xs, sc);
                    if (!mbar_wait(&rg.full[slot], (st / S) & 1, dn.err, ERR_FULL_WAIT)) return false;
                    dot8(qs, xs, sc);
                }
            }
            warp_reduce_multi<V>(v, lane);
            // value i's total sits in lane i * (32 / V); row j adds its slabs in slab order
            float y = 0.0f;
#pragma unroll
            for (int qs = 0; qs < VS; qs++) {
                const float t = __shfl_sync(0xffffffffu, v[0], ((lane & 7) * VS + qs) * (32 / V));
                if (qs < nsl) y += t;
            }
            if (lane < 8) ysm[si * 8 + lane] = y;
        }
        // every warp releases every stage of the group (its producer waits for all kWarps)
        __syncwarp();
        if (lane == 0)
            for (int q = 0; q < d.nst; q++) mbar_arrive(&rg.empty[(s + q) % S]);
        consumers_sync();
        if (threadIdx.x < 8) {
            float acc = 0.0f;
            for (int si = 0; si < K; si++) acc = fmaf(w_sm[si], ysm[si * 8 + threadIdx.x], acc);
            const int64_t oi = row0 + threadIdx.x;
            if (p.out_bf16) static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(acc);
            else static_cast<float*>(p.out)[oi] = acc;
        }
        consumers_sync();
    }
    pos.s = s;
    return true;
}

// XBF16: activations bf16 (else fp32).  BLK: 128x128 block scales.  TB, P: the
// token slots and units per pass of both streaming phases (as the stand-alone
// kernels would take them for at most T assignments per expert).  EP: expert
// parallelism, this rank holding experts [rank * epr, (rank + 1) * epr):
//   after top-k, CTA g < ranks stores this rank's meta and activations into
//   rank g's mailbox as (epoch, payload) words, then unpacks source g's
//   activation words into the plain layout and counts it in (GPU scope); every
//   CTA polls all sources' meta words and groups the received slots (local
//   expert ids, -1 for another rank's; every slot a group of its own) in
//   (source, token, slot) order, and its consumers wait for the activations of
//   every source before gate/up; the streaming phases run
//   over the local experts, down's reduction storing each output value into its
//   source rank's mailbox as an (epoch, value) word over NVLink; the combine of
//   each rank polls the words of its tokens' slots (bounded) and adds them in
//   slot order: no barrier, fence or flag on the return.
template <bool XBF16, bool BLK, int TB, int P, bool EP>
__global__ void __launch_bounds__(kThreads, OOMB_STREAM_CTAS_PER_SM) decode_kernel(const DecodeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_fail;
    __shared__ unsigned s_epoch, s_ep_epoch;
    Ring rg;
    rg.stages = p.stages;
    rg.slot_bytes = p.slot_bytes;
    rg.stage_buf = smem;
    rg.full = reinterpret_cast<uint64_t*>(smem + p.off_bars);
    rg.empty = rg.full + kMaxStages;
    rg.mfull = rg.empty + kMaxStages;
    rg.mempty = rg.mfull + kMetaBufs;
    rg.red = reinterpret_cast<float*>(smem + p.off_red);
    rg.meta = reinterpret_cast<int*>(smem + p.off_meta);
    rg.meta_stride = p.meta_stride;
    rg.chunk_hdr = reinterpret_cast<int*>(smem + p.off_chunk);

    const int T = p.r.T, H = p.r.H, E = p.r.E, K = p.r.K, A = T * K;
    const int G = EP ? p.ep.ranks : 1;
    const int nrec = EP ? p.epr : E;  // entries of the record table r.recs_all
    const DecodeTabs dt = decode_tabs(T, K, E, G * T);
    uint8_t* tabs = smem + p.off_tabs;
    uint64_t* recs_sm = reinterpret_cast<uint64_t*>(tabs + dt.recs);
    uint64_t* recs_active = reinterpret_cast<uint64_t*>(tabs + dt.recs_active);
    uint64_t* rbar = reinterpret_cast<uint64_t*>(tabs + dt.rbar);
    int32_t* ids_sm = reinterpret_cast<int32_t*>(tabs + dt.ids);
    float* w_sm = reinterpret_cast<float*>(tabs + dt.w);
    int32_t* off_sm = reinterpret_cast<int32_t*>(tabs + dt.off);
    int32_t* assign_tok = reinterpret_cast<int32_t*>(tabs + dt.assign_tok);
    int32_t* slot_sm = reinterpret_cast<int32_t*>(tabs + dt.slot_assign);
    int32_t* n_active = reinterpret_cast<int32_t*>(tabs + dt.n_active);
    unsigned* cbits = reinterpret_cast<unsigned*>(tabs + dt.cbits);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    uint64_t* xbar = reinterpret_cast<uint64_t*>(tabs + dt.xbar);
    float* lg = reinterpret_cast<float*>(tabs + dt.lg);
    // This CTA's router rows: [kWarps * blockIdx.x, + nrow), row i landing at i * H * 2.
    const int row0 = kWarps * static_cast<int>(blockIdx.x);
    const int nrow = max(0, min(kWarps, E - row0));
    const unsigned x_bytes = static_cast<unsigned>(T * H * (XBF16 ? 2 : 4));
    const bool xsm = p.x_off >= 0;

    // ---- 1. before the dependency wait: only weights and the record table ----
    if (threadIdx.x == 0) {
        s_fail = 0;
        ring_init(rg);
        mbar_init(rbar, 1);
        mbar_init(xbar, 1);
        fence_barrier_init();
        if (nrow > 0) {
            mbar_arrive_expect_tx(rbar, static_cast<unsigned>(nrow * H * 2));
            bulk_g2s_plain(smem, p.r.w + static_cast<int64_t>(row0) * H, static_cast<unsigned>(nrow * H * 2), rbar);
        }
    }
    const unsigned long long rec_pre =
        static_cast<int>(threadIdx.x) < nrec
            ? ld_prefetch_u64(reinterpret_cast<const unsigned long long*>(p.r.recs_all) + threadIdx.x)
            : 0ull;
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x == 0) {
        // every launch on this workspace before this one has completed
        s_epoch = ld_relaxed_u32(p.sync + kSyncEpoch) + 1u;
        if (blockIdx.x == 0) {
            unsigned* ahead = p.sync + kSyncBars + ((s_epoch + 2u) & 3u) * kSyncSlot;
            ahead[0] = 0u;
            ahead[32] = 0u;
            ahead[64] = 0u;
        }
        if (EP) s_ep_epoch = ep_epoch(p.ep);
        if (xsm && nrow > 0) {
            // the activations may come from the previous kernel: staged after the wait
            mbar_arrive_expect_tx(xbar, x_bytes);
            bulk_g2s_plain(smem + p.x_off, p.r.x, x_bytes, xbar);
        }
    }
    if (static_cast<int>(threadIdx.x) < nrec) recs_sm[threadIdx.x] = rec_pre;
    if (threadIdx.x < kDecodeMaxGroups / 32) cbits[threadIdx.x] = 0u;
    __syncthreads();
    const unsigned epoch = s_epoch;

    // ---- 2. router logits of this CTA's rows, grid barrier, all logits into shared memory ----
    if (warp < nrow) {
        const bool ok = mbar_wait(rbar, 0, p.r.err, ERR_ROUTER_WAIT) &&
                        (!xsm || mbar_wait(xbar, 0, p.r.err, ERR_ROUTER_WAIT));
        if (ok) {
            const int e = row0 + warp;
            const uint8_t* wrow = smem + static_cast<size_t>(warp) * H * 2;
            for (int t0 = 0; t0 < T; t0 += kRouteTT) {
                if (xsm) logits_row<XBF16, true>(p.r, wrow, smem + p.x_off, e, t0, min(kRouteTT, T - t0), lane);
                else logits_row<XBF16, false>(p.r, wrow, nullptr, e, t0, min(kRouteTT, T - t0), lane);
            }
        } else {
            s_fail = 1;
        }
    }
    __syncthreads();
    // the CTAs with router rows publish their logits; every CTA waits for all of them
    unsigned* bars = p.sync + kSyncBars + (epoch & 3u) * kSyncSlot;
    if (threadIdx.x == 0) {
        if (nrow > 0 && !s_fail) bar_arrive(bars);
        const unsigned writers = static_cast<unsigned>((E + kWarps - 1) / kWarps);
        if (!s_fail && !bar_wait(bars, writers, p.r.err, ERR_GRID_WAIT)) s_fail = 1;
    }
    __syncthreads();
    if (s_fail) return;
    for (int o = threadIdx.x; o < T * E; o += kThreads) lg[o] = __ldcg(p.r.logits + o);
    __syncthreads();

    // ---- 3. top-k and grouping of every token, in every CTA ----
    {
        if (E <= 128) topk_warps<kThreads, true, 4>(p.r, lg, 0, T, ids_sm, w_sm);
        else topk_warps<kThreads, true, kRouteSmallE / 32>(p.r, lg, 0, T, ids_sm, w_sm);
        __syncthreads();
        if (blockIdx.x == 0) {
            for (int o = threadIdx.x; o < A; o += kThreads) {
                p.ids_out[o] = ids_sm[o];
                p.w_out[o] = w_sm[o];
            }
        }
        if constexpr (EP) {
            const EpMailbox mb = ep_mailbox(p.ep.ranks, p.ep.t_max, p.ep.k, p.ep.h, p.ep.xb);
            const unsigned ep_ep = s_ep_epoch;
            // every CTA read the mailbox epoch before the logits barrier: hand it to the next step
            if (blockIdx.x == 0 && threadIdx.x == 0) *reinterpret_cast<unsigned*>(p.ep.mailbox + mb.counter) = ep_ep;
            const unsigned long long* meta_w =
                reinterpret_cast<const unsigned long long*>(p.ep.mailbox + mb.meta_words);
            const int xw_n = T * H * p.ep.xb / 4;  // 4-byte words of one rank's activations
            if (static_cast<int>(blockIdx.x) < G) {
                // dispatch to rank g as (epoch, payload) words: the meta (local expert
                // ids on g, -1 elsewhere), then the activations, 4 bytes a word; no
                // fence or flag (a word that shows this step's epoch holds its payload)
                const int g = blockIdx.x;
                uint8_t* dst = reinterpret_cast<uint8_t*>(p.ep.peers[g]);
                unsigned long long* mw =
                    reinterpret_cast<unsigned long long*>(dst + mb.meta_words) + static_cast<size_t>(p.ep.rank) * A;
                for (int i = threadIdx.x; i < A; i += kThreads) {
                    const int e = ids_sm[i];
                    st_word32_sys(mw + i, ep_ep, static_cast<unsigned>(e / p.epr == g ? e - g * p.epr : -1));
                }
                unsigned long long* xw =
                    reinterpret_cast<unsigned long long*>(dst + mb.x_words) + static_cast<size_t>(p.ep.rank) * xw_n;
                const unsigned* xs = static_cast<const unsigned*>(p.r.x);
                for (int i = threadIdx.x; i < xw_n; i += kThreads) st_word32_sys(xw + i, ep_ep, __ldcg(xs + i));
                // and receive source g's activations: unpack its words into the plain
                // layout the gate/up phase reads, then count this source in (GPU scope)
                const unsigned long long* xr =
                    reinterpret_cast<const unsigned long long*>(p.ep.mailbox + mb.x_words) + static_cast<size_t>(g) * xw_n;
                unsigned* xo = reinterpret_cast<unsigned*>(p.ep.mailbox + mb.x) + static_cast<size_t>(g) * xw_n;
                for (int i = threadIdx.x; i < xw_n && !s_fail; i += kThreads) {
                    unsigned long long w = ld_word_sys(xr + i);
                    if (static_cast<unsigned>(w >> 32) != ep_ep) {
                        const unsigned long long t0 = global_ns(), limit = wait_limit();
                        while (static_cast<unsigned>((w = ld_word_sys(xr + i)) >> 32) != ep_ep) {
                            if (global_ns() - t0 > limit) {
                                record_error(p.r.err, ERR_EP_DISPATCH_WAIT);
                                s_fail = 1;
                                break;
                            }
                        }
                    }
                    xo[i] = static_cast<unsigned>(w);
                }
                __syncthreads();
                if (threadIdx.x == 0 && !s_fail) bar_arrive(bars + 64);
            }
            // every source rank's slots for this rank's experts, from their meta words
            int32_t* rmeta = reinterpret_cast<int32_t*>(tabs + dt.rmeta);
            for (int i = threadIdx.x; i < G * A && !s_fail; i += kThreads) {
                unsigned long long w = ld_word_sys(meta_w + i);
                if (static_cast<unsigned>(w >> 32) != ep_ep) {
                    const unsigned long long t0 = global_ns(), limit = wait_limit();
                    while (static_cast<unsigned>((w = ld_word_sys(meta_w + i)) >> 32) != ep_ep) {
                        if (global_ns() - t0 > limit) {
                            record_error(p.r.err, ERR_EP_DISPATCH_WAIT);
                            s_fail = 1;
                            break;
                        }
                    }
                }
                rmeta[i] = static_cast<int32_t>(static_cast<unsigned>(w));
            }
            __syncthreads();
            if (s_fail) return;
            RouteParams rq = p.r;
            rq.T = G * T;
            rq.E = p.epr;
            const GroupOut go{n_active, reinterpret_cast<int32_t*>(tabs + dt.active), off_sm, assign_tok, slot_sm,
                              recs_active, reinterpret_cast<int32_t*>(tabs + dt.aret)};
            if (warp == 0) group_singletons(rq, go, rmeta, recs_sm);
        } else {
            const GroupOut go{n_active, reinterpret_cast<int32_t*>(tabs + dt.active), off_sm, assign_tok, slot_sm,
                              recs_active, nullptr};
            if (p.singles) {
                if (warp == 0) group_slots(p.r, go, ids_sm, recs_sm);
            } else if (A <= 32) {
                if (warp == 0) group_warp(p.r, go, ids_sm, recs_sm);
            } else {
                group_assignments<kThreads>(p.r, go, ids_sm, reinterpret_cast<int32_t*>(tabs + dt.counts),
                                            reinterpret_cast<int32_t*>(tabs + dt.base), recs_sm);
            }
        }
        __syncthreads();
    }

    // ---- 4. gate/up then down through one ring ----
    const int n_e = *n_active;
    const Tables tgu{recs_active, off_sm, assign_tok, n_e, nullptr};
    const Tables tdn{recs_active, off_sm, nullptr, n_e, EP ? reinterpret_cast<const int32_t*>(tabs + dt.aret) : nullptr,
                     EP ? s_ep_epoch : 0u};
    int gu0, gu1, dn0, dn1, g10 = 0, g11 = 0;
    cta_units(n_e, p.gu.gpe, gu0, gu1);
    cta_units(n_e, p.dn.gpe, dn0, dn1);
    constexpr bool D1 = TB == 1 && !EP;  // one token (TB == 1 only for a one-token step)
    if (D1 && p.dn1) cta_units(1, H / 8, g10, g11);

    if (warp == kWarps) {
        if (lane != 0) return;
        int s = 0;
        if (stream_copy<2, P, true, true>(p.gu, tgu, rg, gu0, gu1, s, kDecodeLag)) {
            if (D1 && p.dn1) down1_copy(p.dn, ids_sm, recs_sm, K, rg, g10, g11, s, kDecodeDownLag);
            else stream_copy<1, P, true, true>(p.dn, tdn, rg, dn0, dn1, s, kDecodeLag);
        }
        return;
    }
    if (warp == kWarps + 1) {
        int q = 0;
        if (stream_meta<2, P, true, true>(p.gu, tgu, rg, gu0, gu1, q) && !(D1 && p.dn1))
            stream_meta<1, P, true, true>(p.dn, tdn, rg, dn0, dn1, q);
        return;
    }

    RingPos pos{0, 0, 0};
    if constexpr (EP) {
        // the activations of every source rank are unpacked (CTAs 0 .. ranks - 1)
        if (threadIdx.x == 0 && !bar_wait(bars + 64, static_cast<unsigned>(G), p.r.err, ERR_GRID_WAIT)) s_fail = 1;
        consumers_sync();
        if (s_fail) return;
    }
    if (!stream_consume<2, TB, P, XBF16, true, BLK, true>(p.gu, tgu, rg, gu0, gu1, pos)) s_fail = 1;
    consumers_sync();  // the CTA's h rows are written
    if (threadIdx.x == 0 && !s_fail) {
        bar_arrive(bars + 32);
        if (!bar_wait(bars + 32, gridDim.x, p.r.err, ERR_GRID_WAIT)) s_fail = 1;
    }
    consumers_sync();
    if (s_fail) return;
    if (threadIdx.x == 0) {
        // every CTA has read the epoch: hand it to the next launch
        if (blockIdx.x == 0) st_relaxed_u32(p.sync + kSyncEpoch, epoch);
    }
    if constexpr (D1) {
        if (p.dn1) {
            // one token: down and combine per row group, then done
            bool ok;
            if (((p.dn.k + 511) / 512) <= 2)
                ok = down1_consume<BLK, 16>(p, ids_sm, w_sm, slot_sm, recs_sm, K, rg, g10, g11, pos, rg.red);
            else
                ok = down1_consume<BLK, 32>(p, ids_sm, w_sm, slot_sm, recs_sm, K, rg, g10, g11, pos, rg.red);
            (void)ok;
            return;
        }
    }
    if (!stream_consume<1, TB, P, false, true, BLK, true, EP>(p.dn, tdn, rg, dn0, dn1, pos)) s_fail = 1;
    consumers_sync();  // the CTA's y rows are written
    if (s_fail) return;

    if constexpr (EP) {
        // ---- 5 (expert parallel). every output row of this rank's tokens arrives in
        // its mailbox as (epoch, value) words, stored by the down phase of the expert's
        // rank: the combine polls the words of its slots (bounded) and adds them in
        // slot order as they are valid; no barrier, fence or flag between the ranks ----
        const EpMailbox mb = ep_mailbox(p.ep.ranks, p.ep.t_max, p.ep.k, p.ep.h, p.ep.xb);
        const unsigned ep_ep = s_ep_epoch;
        const unsigned long long* words = reinterpret_cast<const unsigned long long*>(p.ep.mailbox + mb.back_words);
        for (int o = blockIdx.x * (kWarps * 32) + threadIdx.x; o < T * H; o += gridDim.x * (kWarps * 32)) {
            const int t = o / H, c = o - t * H;
            float acc = 0.0f;
            for (int s0 = 0; s0 < K; s0 += 8) {
                // slot s from expert rank g: word (g * T * K + t * K + s) * H + c
                const unsigned long long* wp[8];
                unsigned long long w[8];
                unsigned pending = 0u;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const int s = s0 + j;
                    wp[j] = nullptr;
                    w[j] = 0ull;
                    if (s < K) {
                        const int g = min(max(ids_sm[t * K + s] / p.epr, 0), G - 1);
                        wp[j] = words + (static_cast<int64_t>(g) * A + static_cast<int64_t>(t) * K + s) * H + c;
                        w[j] = ld_word_sys(wp[j]);
                        if (static_cast<unsigned>(w[j] >> 32) != ep_ep) pending |= 1u << j;
                    }
                }
                if (pending) {
                    const unsigned long long t0 = global_ns(), limit = wait_limit();
                    while (pending) {
#pragma unroll
                        for (int j = 0; j < 8; j++)
                            if ((pending >> j) & 1u) {
                                w[j] = ld_word_sys(wp[j]);
                                if (static_cast<unsigned>(w[j] >> 32) == ep_ep) pending &= ~(1u << j);
                            }
                        if (!pending) break;
                        __nanosleep(32);
                        if (global_ns() - t0 > limit) {
                            record_error(p.r.err, ERR_EP_RETURN_WAIT);
                            return;  // this thread's outputs stay unwritten
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < 8; j++)
                    if (s0 + j < K) acc = fmaf(w_sm[t * K + s0 + j], __uint_as_float(static_cast<unsigned>(w[j])), acc);
            }
            if (p.out_bf16) static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(acc);
            else static_cast<float*>(p.out)[o] = acc;
        }
    }

    if constexpr (!EP) {
        // ---- 5. slot-order combine of the row groups this CTA completes ----
        for (int i = threadIdx.x; i < dn1 - dn0; i += kWarps * 32) {
            const int g = (dn0 + i) % p.dn.gpe;
            fence_acq_rel_gpu();  // release the CTA's y rows before counting the unit
            const unsigned old = atomicAdd(p.sync + kSyncGroups + g, 1u);
            if (old == static_cast<unsigned>(n_e - 1)) {
                p.sync[kSyncGroups + g] = 0u;  // every expert's unit of the group has arrived
                atomicOr(&cbits[g >> 5], 1u << (g & 31));
            }
        }
        consumers_sync();
        fence_acq_rel_gpu();  // acquire: the other CTAs' y rows of the completed groups
        const float* y = static_cast<const float*>(p.dn.y);
        const int rpp = p.dn.rpp;
        for (int wd = 0; wd < (p.dn.gpe + 31) / 32; wd++) {
            unsigned bits = cbits[wd];
            while (bits) {
                const int g = wd * 32 + __ffs(bits) - 1;
                bits &= bits - 1;
                const int row0 = g * rpp, nr = min(rpp, H - row0);
                for (int o = threadIdx.x; o < nr * T; o += kWarps * 32) {
                    const int t = o / nr, row = row0 + (o - t * nr);
                    float acc = 0.0f;
                    for (int s0 = 0; s0 < K; s0 += 8) {
                        float v[8], ws[8];
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            const bool ok = s0 + j < K;
                            ws[j] = ok ? w_sm[t * K + s0 + j] : 0.0f;
                            v[j] = ok ? __ldcg(y + static_cast<int64_t>(slot_sm[t * K + s0 + j]) * H + row) : 0.0f;
                        }
#pragma unroll
                        for (int j = 0; j < 8; j++)
                            if (s0 + j < K) acc = fmaf(ws[j], v[j], acc);
                    }
                    const int64_t oi = static_cast<int64_t>(t) * H + row;
                    if (p.out_bf16) static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(acc);
                    else static_cast<float*>(p.out)[oi] = acc;
                }
            }
        }
    }
}

}  // namespace oomb
