// stream.cuh - the weight-streaming engine behind the FP8 GEMV and expert kernels.
//
// Computes y[row] = sum_c x[c] * e4m3(q[row, c]) * scale(row, c) for a stream of
// row groups of one or two FP8 matrices, with fp32 accumulation: the arithmetic
// of the reference's gemv_impl<T, true> (ops.cu:338-440) and moe_gate_up /
// moe_down (moe.cu:52-151); only the summation order differs.
//
// Two CTAs fit per SM, and the stand-alone kernels launch two per SM, both
// computing at once (measured faster than one per SM with the next kernel of a
// dependent-launch chain streaming beside it).  Every CTA is persistent over
// a contiguous slice of "units" (a unit is one row group: RPP rows of each part,
// all K columns).
// Warp roles:
//   warp 8 (copy producer, one lane): streams each unit's rows (contiguous in
//     row-major q) into a ring of shared-memory stages (up to 32 KB each, as
//     many as fit the CTA's half of shared memory) with cp.async.bulk,
//     completed on mbarriers; consumers release stages through a second set of
//     mbarriers.
//   warp 9 (metadata producer): for every pass of P units it loads the units'
//     assignment ranges and block-scale rows into a ring of shared tables,
//     handshaked with mbarriers, so consumers never wait on L2 for them.
//   warps 0..7 (consumers): warp w owns 512-column slab w % NSL and row
//     partition w / NSL and takes eight rows of every stage (four gate and four
//     up rows of a fused SwiGLU unit, else rows rp + j*RP).  Lane l covers 16
//     columns: one 16-byte load of e4m3 per row, decoded to f16 (exact) and
//     multiplied with the activations by the mixed-precision fma.rn.f32.f16
//     (exact products, fp32 sums).  bf16 activations become f16 after an exact
//     power-of-two scaling chosen per 16-value chunk, undone in the block-scale
//     multiply; fp32 activations take the fp32 path (decode to fp32, packed
//     fma.rn.f32x2).
//   Partial sums stay in registers over a pass of P units; then each warp
//   reduces them (a multi-value butterfly, the same lane tree for every value),
//   the slabs are added in slab order through shared memory, and the pass's
//   outputs are written: each output's arithmetic is fixed whatever else shares
//   its launch.
// Kernels signal dependents at entry; the dense GEMV and the EARLY expert
// variant stream weights and load their unit tables before griddepcontrol.wait.
#pragma once

#include "common.cuh"

namespace oomb {

#ifndef OOMB_STREAM_WARPS
#define OOMB_STREAM_WARPS 8
#endif
#ifndef OOMB_STREAM_ROWS
#define OOMB_STREAM_ROWS 8
#endif
#ifndef OOMB_STREAM_STAGES
#define OOMB_STREAM_STAGES 6
#endif
#ifndef OOMB_STREAM_CTAS_PER_SM
#define OOMB_STREAM_CTAS_PER_SM 2
#endif
constexpr int kWarps = OOMB_STREAM_WARPS;    // consumer warps
constexpr int kThreads = (kWarps + 2) * 32;  // + copy producer + metadata producer
constexpr int kRows = OOMB_STREAM_ROWS;      // rows per consumer warp per stage
constexpr int kStageBytes = 32 * 1024;  // largest stage
constexpr int kMaxStages = OOMB_STREAM_STAGES;  // ring depth limit (smaller stages get more of them)
constexpr int kRedV = 16;  // partials per lane per pass (kRows x P x TB)
// A stage holds kRows rows of every consumer warp's 512-column slab.
static_assert(kWarps * kRows * 512 <= kStageBytes, "a stage must fit its shared-memory slot");
constexpr int kMetaBufs = 3;  // per-pass tables in flight (the metadata warp runs two passes ahead)
constexpr int kSmemLimit = OOMB_STREAM_CTAS_PER_SM == 2 ? 110 * 1024 : 227 * 1024;  // two CTAs per SM

struct StreamPlan {
    int kc;      // columns per stage (== k when a stage holds whole rows; else 4096)
    int ks;      // stages per unit along K
    int nsl;     // 512-column slabs per stage
    int rp;      // row partitions (warps per slab)
    int rpp;     // rows per part per unit
    int nb;      // 128-column scale blocks per row
    int sr;      // scale rows kept per unit and part (one block row for 128x128, RPP rows for 1x128)
    int stages;  // ring depth
    int stage_bytes;  // bytes one unit's K-stage occupies (<= kStageBytes)
    int slot_bytes;   // ring slot: stage_bytes rounded up to 1 KB
    size_t smem;
};

// Shared-memory layout: [stages x slot_bytes][full][empty][meta_full][meta_empty]
// [red 2 x kWarps x kRedV][meta kMetaBufs x (P x 4 ints + P x PARTS x SR x NB floats)]
// [chunk headers 2 x 4 ints]
inline size_t stream_meta_bytes(int P, int parts, int sr, int nb) {
    return static_cast<size_t>(P) * 4 * sizeof(int) + static_cast<size_t>(P) * parts * sr * nb * sizeof(float);
}

inline StreamPlan stream_plan(int k, int parts, int P, int layout) {
    StreamPlan p{};
    const int nsl_full = (k + 511) / 512;
    p.kc = nsl_full > 8 ? 4096 : k;
    p.ks = (k + p.kc - 1) / p.kc;
    p.nsl = ((p.kc < k ? p.kc : k) + 511) / 512;
    p.rp = kWarps / p.nsl;
    p.rpp = parts == 2 ? (kRows / 2) * p.rp : kRows * p.rp;
    p.nb = (k + 127) / 128;
    p.sr = layout ? 1 : p.rpp;  // unit sizes divide 128: one block row per unit
    p.stage_bytes = parts * p.rpp * (p.kc < k ? p.kc : k);
    p.slot_bytes = (p.stage_bytes + 1023) & ~1023;
    const size_t fixed = (2 * kMaxStages + 2 * kMetaBufs) * sizeof(uint64_t) + 2 * kWarps * kRedV * sizeof(float) +
                         kMetaBufs * stream_meta_bytes(P, parts, p.sr, p.nb) + 8 * sizeof(int) + 128;
    // as many slots as fit the CTA's share of shared memory
    p.stages = kMaxStages;
    while (p.stages > 2 && static_cast<size_t>(p.stages) * p.slot_bytes + fixed > kSmemLimit) p.stages--;
    p.smem = static_cast<size_t>(p.stages) * p.slot_bytes + fixed;
    return p;
}

struct StreamParams {
    // dense matrix (MOE == false)
    const uint8_t* q;
    const float* scale;
    // expert groups (MOE == true)
    const uint64_t* recs;
    const int32_t* off;
    const int32_t* assign_tok;  // gate/up: token of each assignment
    const int32_t* n_e_dev;     // group count on the device, or null
    int n_e_host;
    int64_t w_off[2], s_off[2];
    int layout;  // 0: 1x128, 1: 128x128
    // shape and plan
    int k, nrows;  // columns; rows per part
    int kc, ks, nsl, rp, rpp, nb, sr, stages, slot_bytes;
    int gpe;  // units per expert group (dense: units in total)
    // activations and outputs
    const void* x;  // dense: [t, k]; gate/up: [*, k] rows picked by assign_tok; down: h [A, k] fp32
    int t;          // dense: tokens of this launch
    void* y;        // dense: [t, nrows] (y_bf16 ? bf16 : fp32); MoE: [A, nrows] fp32
    int y_bf16;
    unsigned* err;
    // expert-parallel outputs (decode kernel): the output of assignment a, return
    // index aret[a] = source rank g * ep_tk + slot, goes to rank g's mailbox at
    // ep_back_off, word (ep_rank * ep_tk + slot) * nrows + row of [*, nrows]
    // (epoch, value) words, stored over NVLink
    const unsigned long long* ep_peers;
    int64_t ep_back_off;
    int ep_rank, ep_tk;
};

// ---- activation slices in registers ----------------------------------------------------

// 16 bf16 activations as f16 pairs scaled by 2^-s (s from the largest
// magnitude, so the largest lands in [2^14, 2^15)); returns 2^s.  Read through
// L2: the activations may come from a kernel of the same dependent-launch chain.
__device__ __forceinline__ float load_x16_f16(const uint16_t* p, unsigned (&xh)[8]) {
    const uint4 a = __ldcg(reinterpret_cast<const uint4*>(p));
    const uint4 b = __ldcg(reinterpret_cast<const uint4*>(p) + 1);
    const unsigned w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    unsigned m = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) m = __vmaxu2(m, w[i] & 0x7fff7fffu);
    m = max(m & 0xffffu, m >> 16);
    int s = m ? static_cast<int>((m >> 7) & 0xff) - 127 - 14 : 0;
    s = max(-100, min(100, s));
    const float inv = __int_as_float((127 - s) << 23);
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float lo = __uint_as_float(w[i] << 16) * inv;
        const float hi = __uint_as_float(w[i] & 0xffff0000u) * inv;
        unsigned r;
        asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
        xh[i] = r;
    }
    return __int_as_float((127 + s) << 23);
}

// 16 e4m3 weights (one 16-byte chunk) decoded once per row and shared by every
// token slot: exact f16 pairs, or exact fp32 pairs.
template <bool F16>
struct WDec;

template <>
struct WDec<true> {
    unsigned h[8];
    __device__ __forceinline__ void decode(uint4 w) {
        const unsigned words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h[2 * i]) : "h"(static_cast<unsigned short>(words[i] & 0xffffu)));
            asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h[2 * i + 1]) : "h"(static_cast<unsigned short>(words[i] >> 16)));
        }
    }
};

template <>
struct WDec<false> {
    float2 f[8];
    __device__ __forceinline__ void decode(uint4 w) {
        const unsigned words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            f[2 * i] = e4m3x2_to_float2(static_cast<unsigned short>(words[i] & 0xffffu));
            f[2 * i + 1] = e4m3x2_to_float2(static_cast<unsigned short>(words[i] >> 16));
        }
    }
};

// Activation slice of one token: f16 form (bf16 inputs; exact products with
// the mixed-precision fma.rn.f32.f16, fp32 sums) or fp32 form (packed fp32 FMA).
template <bool XBF16>
struct XSlice;

template <>
struct XSlice<true> {
    unsigned h[8];
    float s;  // 2^s undoing the f16 scaling
    __device__ __forceinline__ void load(const void* base, int64_t idx) {
        s = load_x16_f16(static_cast<const uint16_t*>(base) + idx, h);
    }
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int i = 0; i < 8; i++) h[i] = 0u;
        s = 0.0f;
    }
    __device__ __forceinline__ float dot(const WDec<true>& w) const {
        float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // four short chains
#pragma unroll
        for (int i = 0; i < 8; i++)
            asm("{\n .reg .b16 wa, wb, xa, xb;\n mov.b32 {wa, wb}, %2;\n mov.b32 {xa, xb}, %3;\n"
                " fma.rn.f32.f16 %0, wa, xa, %0;\n fma.rn.f32.f16 %1, wb, xb, %1;\n}"
                : "+f"(a[(i & 1) * 2]), "+f"(a[(i & 1) * 2 + 1])
                : "r"(w.h[i]), "r"(h[i]));
        return (a[0] + a[1]) + (a[2] + a[3]);
    }
    __device__ __forceinline__ float scale() const { return s; }
};

template <>
struct XSlice<false> {
    float2 f[8];
    __device__ __forceinline__ void load(const void* base, int64_t idx) { load_x16_cg<false>(base, idx, f); }
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int i = 0; i < 8; i++) f[i] = make_float2(0.0f, 0.0f);
    }
    __device__ __forceinline__ float dot(const WDec<false>& w) const {
        float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int i = 0; i < 8; i++) acc = ffma2(w.f[i], f[i], acc);
        return acc.x + acc.y;
    }
    __device__ __forceinline__ float scale() const { return 1.0f; }
};

// ---- units and routing tables ---------------------------------------------------------------

// The routing tables a MoE launch streams from: record address of each expert
// group, assignment ranges off[n_e + 1], token of each assignment, group count.
// They live in global memory (written by an earlier kernel) or, in the fused
// decode kernel, in this CTA's shared memory (TSMEM).
struct Tables {
    const uint64_t* recs;
    const int32_t* off;
    const int32_t* assign_tok;
    int n_e;
    const int32_t* assign_ret;  // expert-parallel outputs: return index of each assignment
    unsigned epoch;             // expert-parallel outputs: the step epoch stored with every value
};

template <bool TSMEM>
__device__ __forceinline__ int tab_i32(const int32_t* a) {
    if constexpr (TSMEM) return *a;
    else return __ldcg(a);
}

template <bool TSMEM>
__device__ __forceinline__ unsigned long long tab_u64(const uint64_t* a) {
    if constexpr (TSMEM) return *reinterpret_cast<const unsigned long long*>(a);
    else return __ldcg(reinterpret_cast<const unsigned long long*>(a));
}

// The tables of a stand-alone launch (dense launches: one group, no tables).
__device__ __forceinline__ Tables global_tables(const StreamParams& p, bool moe) {
    Tables tb{p.recs, p.off, p.assign_tok, 1, nullptr};
    if (moe) tb.n_e = p.n_e_dev ? __ldcg(p.n_e_dev) : p.n_e_host;
    return tb;
}

// The CTA's slice [u0, u1) of the flat list of n_e * gpe units (32-bit
// arithmetic: units * (grid + 1) < 2^32 for every launch the host plans).
__device__ __forceinline__ void cta_units(int n_e, int gpe, int& u0, int& u1) {
    const unsigned units = static_cast<unsigned>(n_e * gpe);
    u0 = static_cast<int>((blockIdx.x * units) / gridDim.x);
    u1 = static_cast<int>(((blockIdx.x + 1) * units) / gridDim.x);
}

// Stage row (part-major) of the warp's slot j: for PARTS == 2 the first half
// of the slots are gate rows H*rpi .. H*rpi+H-1 (H = kRows/2) and the second
// half the same up rows; else rpi + j*RP.
template <int PARTS>
__device__ __forceinline__ int slot_row(int rpi, int rp, int j) {
    constexpr int H = kRows / 2;
    return PARTS == 2 ? (j / H) * (H * rp) + H * rpi + (j % H) : rpi + j * rp;
}

// The shared-memory rings of a streaming CTA: weight stages with their
// full/empty mbarriers, per-pass unit tables with theirs, the reduction
// buffers and the chunk headers.  `meta_stride` (ints) holds the largest pass
// table of any phase the CTA runs.
struct Ring {
    uint8_t* stage_buf;
    uint64_t* full;
    uint64_t* empty;
    uint64_t* mfull;
    uint64_t* mempty;
    float* red;      // [2][kWarps][kRedV]
    int* meta;       // [kMetaBufs][meta_stride]
    int* chunk_hdr;  // [2][4]
    int stages, slot_bytes, meta_stride;
};

// Positions in the rings, carried from one phase to the next within a launch:
// s counts stages, q pass tables, rparity the reduction buffer in use.
struct RingPos {
    int s, q, rparity;
};

// ---- per-pass reduction and output ----------------------------------------------------------

// hdr[pi] = {a_begin, a_end, row0, nr} of the pass's units (shared memory).
// EPOUT: MoE outputs go to the mailboxes of the ranks whose assignments they
// are (aret: return index of each assignment) as (epoch, value) words; else to p.y.
template <int PARTS, int TB, int P, bool MOE, bool EPOUT = false>
__device__ __forceinline__ void reduce_write(const StreamParams& p, const float (&acc)[P][kRows][TB], float* rb,
                                             const int* hdr, int pn, int warp, int lane, const int32_t* aret = nullptr,
                                             unsigned epoch = 0u) {
    // The multi-value butterfly sums every partial over the 32 lanes by the same
    // tree (pairs at lane distance 16, then 8, 4, 2, 1; addition commutes), so
    // an output's arithmetic does not depend on its position in the pass: results
    // are identical however the assignments are grouped into launches.
    float v[kRedV];
#pragma unroll
    for (int a = 0; a < P; a++)
#pragma unroll
        for (int j = 0; j < kRows; j++)
#pragma unroll
            for (int b = 0; b < TB; b++) v[(a * kRows + j) * TB + b] = acc[a][j][b];
#pragma unroll
    for (int j = kRows * P * TB; j < kRedV; j++) v[j] = 0.0f;
    warp_reduce_multi<kRedV>(v, lane);
    if ((lane & 1) == 0) rb[warp * kRedV + reduce_index<kRedV>(lane, 0)] = v[0];
    asm volatile("bar.sync 1, %0;" ::"r"(kWarps * 32) : "memory");
    // outputs of the pass: unit pi, output row r (of RPP), token b
    const int outs = pn * p.rpp * TB;
    for (int o = threadIdx.x; o < outs; o += kWarps * 32) {
        const int b = o % TB;
        const int rr = o / TB;
        const int pi = rr / p.rpp, r = rr - pi * p.rpp;
        const int a_begin = hdr[pi * 4 + 0], a_end = hdr[pi * 4 + 1];
        const int row0 = hdr[pi * 4 + 2], nr = hdr[pi * 4 + 3];
        if (r >= nr || b >= a_end - a_begin) continue;
        float res[2];
#pragma unroll
        for (int part = 0; part < PARTS; part++) {
            // stage row of (part, r) -> owning row partition and slot
            int rpi, j;
            if (PARTS == 2) {
                rpi = r / (kRows / 2);
                j = part * (kRows / 2) + r % (kRows / 2);
            } else {
                j = r / p.rp;
                rpi = r - j * p.rp;
            }
            const int vi = (pi * kRows + j) * TB + b;
            float sum = 0.0f;
            for (int q = 0; q < p.nsl; q++) sum += rb[(rpi * p.nsl + q) * kRedV + vi];
            res[part] = sum;
        }
        const int row = row0 + r;
        if (MOE) {
            const float val = PARTS == 2 ? res[0] / (1.0f + expf(-res[0])) * res[PARTS - 1] : res[0];
            if (EPOUT) {
                const int r = aret[a_begin + b];
                const int g = r / p.ep_tk, ts = r - g * p.ep_tk;
                unsigned long long* dst = reinterpret_cast<unsigned long long*>(
                    reinterpret_cast<uint8_t*>(p.ep_peers[g]) + p.ep_back_off);
                st_word_sys(dst + (static_cast<int64_t>(p.ep_rank) * p.ep_tk + ts) * p.nrows + row, epoch, val);
            } else {
                static_cast<float*>(p.y)[static_cast<int64_t>(a_begin + b) * p.nrows + row] = val;
            }
        } else {
            const int64_t yi = static_cast<int64_t>(a_begin + b) * p.nrows + row;
            if (p.y_bf16) static_cast<__nv_bfloat16*>(p.y)[yi] = __float2bfloat16_rn(res[0]);
            else static_cast<float*>(p.y)[yi] = res[0];
        }
    }
}

// ---- the three roles --------------------------------------------------------------------

// Copy producer (one lane): streams units [u0, u1) into the stage ring,
// continuing at ring position s.  With lag > 0 at most `lag` stages are in
// flight: stage s is requested once stage s - lag has landed, so when every CTA
// requests at once, each CTA's first stages are served first instead of all of
// its ring landing together at the end of the burst.  After a wait that ran out
// it drains its copies in flight and returns false.
template <int PARTS, int P, bool MOE, bool TSMEM>
__device__ bool stream_copy(const StreamParams& p, const Tables& tb, const Ring& rg, int u0, int u1, int& s,
                            int lag = 0) {
    if (u1 <= u0) return true;
    const int S = rg.stages, KS = p.ks;
    const int kcs = min(p.kc, p.k);  // shared-memory row stride
    const uint64_t pol = make_evict_first_policy();
    int ei = u0 / p.gpe;
    const uint8_t* rec = MOE ? reinterpret_cast<const uint8_t*>(tab_u64<TSMEM>(tb.recs + ei)) : p.q;
    const uint8_t* rec_next =
        (MOE && ei + 1 < tb.n_e) ? reinterpret_cast<const uint8_t*>(tab_u64<TSMEM>(tb.recs + ei + 1)) : rec;
    int rec_ei = ei;
    bool ok = true;
    const int s_begin = s;
    for (int pf = u0; pf < u1 && ok; pf += P) {
        const int pn = min(P, u1 - pf);
        for (int ks = 0; ks < KS && ok; ks++) {
            for (int pi = 0; pi < pn; pi++, s++) {
                const int slot = s % S;
                ok = mbar_wait(&rg.empty[slot], ((s / S) & 1) ^ 1, p.err, ERR_EMPTY_WAIT);
                if (ok && lag > 0 && lag < S && s >= lag)
                    ok = mbar_wait(&rg.full[(s - lag) % S], ((s - lag) / S) & 1, p.err, ERR_EMPTY_WAIT);
                if (!ok) break;
                const int u = pf + pi;
                const int uei = u / p.gpe, g = u - uei * p.gpe;
                if (MOE && uei != rec_ei) {
                    rec = uei == rec_ei + 1 ? rec_next : reinterpret_cast<const uint8_t*>(tab_u64<TSMEM>(tb.recs + uei));
                    rec_ei = uei;
                    if (uei + 1 < tb.n_e) rec_next = reinterpret_cast<const uint8_t*>(tab_u64<TSMEM>(tb.recs + uei + 1));
                }
                const int row0 = g * p.rpp;
                const int nr = min(p.rpp, p.nrows - row0);
                const int kc0 = ks * p.kc;
                const int kcl = min(p.kc, p.k - kc0);
                uint8_t* dst = rg.stage_buf + slot * rg.slot_bytes;
                mbar_arrive_expect_tx(&rg.full[slot], static_cast<unsigned>(PARTS * nr * kcl));
#pragma unroll
                for (int part = 0; part < PARTS; part++) {
                    const uint8_t* src = (MOE ? rec + (part ? p.w_off[1] : p.w_off[0]) : rec) +
                                         static_cast<int64_t>(row0) * p.k + kc0;
                    uint8_t* d = dst + part * p.rpp * kcs;
                    if (kcl == p.k) {
                        bulk_g2s(d, src, static_cast<unsigned>(nr * kcl), &rg.full[slot], pol);
                    } else {
                        for (int r = 0; r < nr; r++)
                            bulk_g2s(d + r * kcs, src + static_cast<int64_t>(r) * p.k, static_cast<unsigned>(kcl),
                                     &rg.full[slot], pol);
                    }
                }
            }
        }
    }
    if (!ok) {
        // copies issued from this phase's stages that may still be in flight
        for (int d = max(s_begin, s - S); d < s; d++) mbar_wait(&rg.full[d % S], (d / S) & 1, p.err, ERR_DRAIN_WAIT);
    }
    return ok;
}

// Metadata producer (one warp): for every pass of P units of [u0, u1) loads
// the unit headers and block-scale rows into the table ring, continuing at
// table position q.
template <int PARTS, int P, bool MOE, bool TSMEM>
__device__ bool stream_meta(const StreamParams& p, const Tables& tb, const Ring& rg, int u0, int u1, int& q) {
    const int lane = threadIdx.x & 31;
    const int meta_ints = P * 4;
    const int pair_floats = p.sr * p.nb;  // scale table of one (unit, part)
    const uint64_t keep = make_evict_last_policy();
    for (int pf = u0; pf < u1; pf += P, q++) {
        const int buf = q % kMetaBufs;
        if (!mbar_wait(&rg.mempty[buf], ((q / kMetaBufs) & 1) ^ 1, p.err, ERR_EMPTY_WAIT)) return false;
        const int pn = min(P, u1 - pf);
        int* hdr = rg.meta + buf * rg.meta_stride;
        float* sc = reinterpret_cast<float*>(hdr + meta_ints);
        // unit headers and record addresses: lane pi holds unit pi's
        unsigned long long urec = reinterpret_cast<unsigned long long>(p.q);
        int urow0 = 0;
        if (lane < pn) {
            const int u = pf + lane;
            const int ei = u / p.gpe, g = u - ei * p.gpe;
            urow0 = g * p.rpp;
            if (MOE) urec = tab_u64<TSMEM>(tb.recs + ei);
            hdr[lane * 4 + 0] = MOE ? tab_i32<TSMEM>(tb.off + ei) : 0;
            hdr[lane * 4 + 1] = MOE ? tab_i32<TSMEM>(tb.off + ei + 1) : p.t;
            hdr[lane * 4 + 2] = urow0;
            hdr[lane * 4 + 3] = min(p.rpp, p.nrows - urow0);
        }
        // scale tables, one per (unit, part): 128x128 keeps the unit's block row
        // (unit sizes divide 128), 1x128 its RPP rows; NB blocks per row.  All loads
        // of a batch (8 per lane, across every (unit, part) of the pass) are
        // issued before any store, so a pass costs one L2 round trip.
        const int total = pn * PARTS * pair_floats;
        for (int e0 = 0; e0 < total; e0 += 8 * 32) {
            float v[8];
#pragma unroll
            for (int m = 0; m < 8; m++) {
                const int e = e0 + m * 32 + lane;
                const int ec = e < total ? e : 0;
                const int pair = ec / pair_floats, ep = ec - pair * pair_floats;
                const int pi = pair / PARTS, part = pair - pi * PARTS;
                const unsigned long long rb = __shfl_sync(0xffffffffu, urec, pi);
                const int row0 = __shfl_sync(0xffffffffu, urow0, pi);
                v[m] = 0.0f;
                if (e < total) {
                    const float* sp = MOE ? reinterpret_cast<const float*>(
                                                reinterpret_cast<const uint8_t*>(rb) + (part ? p.s_off[1] : p.s_off[0]))
                                          : p.scale;
                    const int r = ep / p.nb, kb = ep - r * p.nb;
                    const int srow = p.layout ? (row0 >> 7) + r : row0 + r;
                    if ((p.layout ? srow * 128 : srow) < p.nrows) v[m] = ld_scale(sp + static_cast<int64_t>(srow) * p.nb + kb, keep);
                }
            }
#pragma unroll
            for (int m = 0; m < 8; m++) {
                const int e = e0 + m * 32 + lane;
                if (e < total) sc[e] = v[m];
            }
        }
        mbar_arrive(&rg.mfull[buf]);  // release: this lane's header and table writes
    }
    return true;
}

// Consumer warps: the arithmetic of units [u0, u1) from the rings, continuing
// at ring positions `pos`.  Returns false when a wait ran out.
template <int PARTS, int TB, int P, bool XBF16, bool MOE, bool BLK, bool TSMEM, bool EPOUT = false>
__device__ bool stream_consume(const StreamParams& p, const Tables& tb, const Ring& rg, int u0, int u1,
                               RingPos& pos) {
    static_assert(kRows * P * TB <= kRedV, "too many partials per lane");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = rg.stages, KS = p.ks;
    const int kcs = min(p.kc, p.k);  // shared-memory row stride
    const int meta_ints = P * 4;
    const int pair_floats = p.sr * p.nb;

    const bool active = warp < p.rp * p.nsl;  // warp-uniform
    const int sl = active ? warp % p.nsl : 0;
    const int rpi = active ? warp / p.nsl : 0;
    const int col = sl * 512 + lane * 16;
    const int kc = p.kc, kdim = p.k, nb_k = p.nb;
    // byte offset of each of the warp's rows in a stage and its row within its part
    int roff[kRows], rin[kRows];
#pragma unroll
    for (int j = 0; j < kRows; j++) {
        const int srow = slot_row<PARTS>(rpi, p.rp, j);
        roff[j] = srow * kcs;
        rin[j] = PARTS == 2 ? srow - (j / (kRows / 2)) * p.rpp : srow;
    }

    XSlice<XBF16> xs[TB];
    int x_key0 = -1, x_key1 = -1;  // (expert or K-stage, first assignment) the slices hold
    if constexpr (MOE && PARTS == 2 && TB == 1 && TSMEM) {
        // tables in shared memory: the first unit's token is known without its pass
        // table, so its activation slice is requested before the first table wait
        if (u0 < u1) {
            const int tok = tb.assign_tok[tb.off[u0 / p.gpe]];
            if (active && col < min(p.kc, p.k)) xs[0].load(p.x, static_cast<int64_t>(tok) * p.k + col);
            else xs[0].zero();
            x_key0 = 0;
            x_key1 = tok;
        }
    }
    int s = pos.s, q = pos.q, rparity = pos.rparity;

    for (int pf = u0; pf < u1; pf += P, q++) {
        const int pn = min(P, u1 - pf);
        const int buf = q % kMetaBufs;
        if (!mbar_wait(&rg.mfull[buf], (q / kMetaBufs) & 1, p.err, ERR_FULL_WAIT)) return false;
        const int* hdr = rg.meta + buf * rg.meta_stride;
        const float* sct = reinterpret_cast<const float*>(hdr + meta_ints);
        float acc[P][kRows][TB];
#pragma unroll
        for (int a = 0; a < P; a++)
#pragma unroll
            for (int j = 0; j < kRows; j++)
#pragma unroll
                for (int b = 0; b < TB; b++) acc[a][j][b] = 0.0f;
        bool chunked_any = false;
        for (int ks = 0; ks < KS; ks++) {
            const int kc0 = ks * kc;
            const int kcl = min(kc, kdim - kc0);
            const bool col_ok = active && col < kcl;
            // lanes past the end read column 0 of the stage with zero activations
            const int ccol = col_ok ? col : 0;
            const int kb = (kc0 + ccol) >> 7;
#pragma unroll
            for (int pi = 0; pi < P; pi++) {
                if (pi < pn) {
                    const int a_begin = hdr[pi * 4 + 0];
                    int a_end = hdr[pi * 4 + 1];
                    const int nr = hdr[pi * 4 + 3];
                    if (P > 1 && a_end - a_begin > TB) {
                        record_error(p.err, ERR_BAD_TABLE);  // the host promised at most TB per unit
                        a_end = a_begin + TB;
                    }
                    const bool chunked = P == 1 && a_end - a_begin > TB;
                    chunked_any |= chunked;
                    // block scales: with 128x128 blocks every row of a unit lies in
                    // one block row (unit sizes divide 128), so one per part
                    float sc[kRows];
                    const float* st = sct + pi * PARTS * pair_floats + kb;
                    if (BLK) {
                        const float s0 = st[0];
                        const float s1 = PARTS == 2 ? st[pair_floats] : s0;
#pragma unroll
                        for (int j = 0; j < kRows; j++) sc[j] = (PARTS == 2 && j >= kRows / 2) ? s1 : s0;
                    } else {
#pragma unroll
                        for (int j = 0; j < kRows; j++)
                            sc[j] = st[(PARTS == 2 ? j / (kRows / 2) : 0) * pair_floats + rin[j] * nb_k];
                    }
                    // Activation slices: gate/up the assignment's token, down the
                    // assignment's h row, dense the token.  They are reloaded only when
                    // their key changes: (K stage, first assignment of the chunk), or
                    // with one token slot in gate/up the token itself, which every
                    // expert of that token shares.
                    const int key0 = MOE ? 0 : ks;
                    auto ensure_x = [&](int a0, int nb) {
                        const int key1 = (MOE && PARTS == 2 && TB == 1) ? tab_i32<TSMEM>(tb.assign_tok + a0) : a0;
                        if (x_key0 == key0 && x_key1 == key1) return;
#pragma unroll
                        for (int b = 0; b < TB; b++) {
                            if (b < nb && col_ok) {
                                const int64_t xr = (MOE && PARTS == 2) ? tab_i32<TSMEM>(tb.assign_tok + a0 + b) : a0 + b;
                                xs[b].load(p.x, xr * kdim + kc0 + col);
                            } else {
                                xs[b].zero();
                            }
                        }
                        x_key0 = key0;
                        x_key1 = key1;
                    };
                    // the first chunk's activations are requested before the stage wait,
                    // so their latency overlaps the stage's
                    if (a_begin < a_end) ensure_x(a_begin, min(TB, a_end - a_begin));
                    const int slot = s % S;
                    if (!mbar_wait(&rg.full[slot], (s / S) & 1, p.err, ERR_FULL_WAIT)) return false;
                    const uint8_t* base = rg.stage_buf + slot * rg.slot_bytes + ccol;
                    for (int a0 = a_begin; a0 < a_end; a0 += TB) {
                        const int nb = min(TB, a_end - a0);
                        if (a0 != a_begin) ensure_x(a0, nb);
                        if (active) {
                            float sx[kRows][TB];
#pragma unroll
                            for (int j = 0; j < kRows; j++)
#pragma unroll
                                for (int b = 0; b < TB; b++) sx[j][b] = sc[j] * xs[b].scale();
                            // every row's 16 bytes first, then decode and multiply
                            uint4 raw[kRows];
#pragma unroll
                            for (int j = 0; j < kRows; j++) raw[j] = *reinterpret_cast<const uint4*>(base + roff[j]);
#pragma unroll
                            for (int j = 0; j < kRows; j++) {
                                WDec<XBF16> w;
                                w.decode(raw[j]);
#pragma unroll
                                for (int b = 0; b < TB; b++) acc[pi][j][b] = fmaf(xs[b].dot(w), sx[j][b], acc[pi][j][b]);
                            }
                        }
                        if (chunked) {
                            // more assignments than token slots: reduce and write this chunk now
                            int* ch = rg.chunk_hdr + rparity * 4;
                            if (threadIdx.x == 0) {
                                ch[0] = a0;
                                ch[1] = a0 + nb;
                                ch[2] = hdr[pi * 4 + 2];
                                ch[3] = nr;
                            }
                            reduce_write<PARTS, TB, P, MOE, EPOUT>(p, acc, rg.red + rparity * kWarps * kRedV, ch, 1,
                                                                   warp, lane, tb.assign_ret, tb.epoch);
                            rparity ^= 1;
#pragma unroll
                            for (int j = 0; j < kRows; j++)
#pragma unroll
                                for (int b = 0; b < TB; b++) acc[pi][j][b] = 0.0f;
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&rg.empty[slot]);
                    s++;
                }
            }
        }
        if (!chunked_any) {
            reduce_write<PARTS, TB, P, MOE, EPOUT>(p, acc, rg.red + rparity * kWarps * kRedV, hdr, pn, warp, lane,
                                                   tb.assign_ret, tb.epoch);
            rparity ^= 1;
        }
        // this warp is done with the pass's table: hand it back
        __syncwarp();
        if (lane == 0) mbar_arrive(&rg.mempty[buf]);
    }
    pos.s = s;
    pos.q = q;
    pos.rparity = rparity;
    return true;
}

// Initialises the ring's mbarriers (one thread).
__device__ __forceinline__ void ring_init(const Ring& rg) {
    for (int i = 0; i < rg.stages; i++) {
        mbar_init(&rg.full[i], 1);
        mbar_init(&rg.empty[i], kWarps);
    }
    for (int i = 0; i < kMetaBufs; i++) {
        mbar_init(&rg.mfull[i], 32);
        mbar_init(&rg.mempty[i], kWarps);
    }
}

// ---- the stand-alone kernel -----------------------------------------------------------------

// PARTS: 2 = fused gate/up + SwiGLU (expert records), 1 = one matrix.
// TB: token slots per unit.  P: units per reduction pass (kRows * P * TB <= 16).
//   With P > 1 every unit has at most TB assignments (the host guarantees it);
//   with P == 1 a unit may have more, processed in chunks of TB against the
//   stage held in shared memory.
// MOE: units come from expert groups (recs/off); else from the dense q.
// EARLY: the copy producer reads the routing tables before griddepcontrol.wait
//   (valid only two launches after the kernel that wrote them, see capi.cu).
// BLK: 128x128 scale blocks (p.layout == 1), else 1x128.
//
// Shared-memory layout: [stages x slot_bytes][full][empty][meta_full][meta_empty]
// [red 2 x kWarps x kRedV][meta kMetaBufs x (P x 4 ints + P x PARTS x SR x NB floats)]
// [chunk headers 2 x 4 ints]
template <int PARTS, int TB, int P, bool XBF16, bool MOE, bool EARLY, bool BLK>
__global__ void __launch_bounds__(kThreads, OOMB_STREAM_CTAS_PER_SM) stream_kernel(const StreamParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    Ring rg;
    rg.stages = p.stages;
    rg.slot_bytes = p.slot_bytes;
    rg.stage_buf = smem;
    rg.full = reinterpret_cast<uint64_t*>(smem + p.stages * p.slot_bytes);
    rg.empty = rg.full + kMaxStages;
    rg.mfull = rg.empty + kMaxStages;
    rg.mempty = rg.mfull + kMetaBufs;
    rg.red = reinterpret_cast<float*>(rg.mempty + kMetaBufs);
    rg.meta = reinterpret_cast<int*>(rg.red + 2 * kWarps * kRedV);
    rg.meta_stride = P * 4 + P * PARTS * p.sr * p.nb;
    rg.chunk_hdr = rg.meta + kMetaBufs * rg.meta_stride;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        ring_init(rg);
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kWarps) {
        // ================= copy producer =================
        // weights and (dense, or tables written two launches back) unit tables do
        // not depend on the previous kernel
        if (MOE && !EARLY) pdl_wait();
        pdl_launch_dependents();
        if (lane != 0) return;
        const Tables tb = global_tables(p, MOE);
        int u0, u1;
        cta_units(tb.n_e, p.gpe, u0, u1);
        int s = 0;
        stream_copy<PARTS, P, MOE, false>(p, tb, rg, u0, u1, s);
        return;
    }

    if (warp == kWarps + 1) {
        // ================= metadata producer =================
        // block scales are weights; the unit tables are as ready as for the copy producer
        if (MOE && !EARLY) pdl_wait();
        pdl_launch_dependents();
        const Tables tb = global_tables(p, MOE);
        int u0, u1;
        cta_units(tb.n_e, p.gpe, u0, u1);
        int q = 0;
        stream_meta<PARTS, P, MOE, false>(p, tb, rg, u0, u1, q);
        return;
    }

    // ================= consumers =================
    pdl_wait();
    pdl_launch_dependents();
    const Tables tb = global_tables(p, MOE);
    int u0, u1;
    cta_units(tb.n_e, p.gpe, u0, u1);
    if (u1 <= u0) return;
    RingPos pos{0, 0, 0};
    stream_consume<PARTS, TB, P, XBF16, MOE, BLK, false>(p, tb, rg, u0, u1, pos);
}

}  // namespace oomb
