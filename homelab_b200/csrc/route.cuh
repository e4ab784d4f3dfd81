// route.cuh - router GEMV, softmax top-k and on-device grouping by expert.
//
// Bit-exact contract with the CPU oracle (oracle/oomb_oracle.c):
//   - logits: logit[t, e] = xor-tree over 32 lanes of lane l's fmaf chain over
//     columns 256*i + 8*l + j (i ascending, j = 0..7) of x[t] * bf16(W[e]);
//   - softmax: max over the row, exp by oomb_expf (the same Cody-Waite + Taylor
//     arithmetic as oo_expf), sum = xor-tree of 32 lane partials (lane l adds
//     experts l, l+32, ... in order), p = exp / sum (IEEE division);
//   - top-k: k rounds of argmax over p, ties to the lower id, picked entries set
//     to -2 (ops.cu:234-294); weights = p / (sum of picked p in pick order).
// Grouping (Moe::begin_routed / finish_routed, moe.rs:532-582, 638-659, all
// experts resident): assignments ordered by expert id, each expert's slots in
// slot order; off[n_e + 1], assign_tok[A], slot_assign[A], active[n_e] and the
// active experts' record addresses.
#pragma once

#include "common.cuh"

namespace oomb {

// exp(x) by Cody & Waite (1980) argument reduction x = n ln2 + r with ln2 split
// into a 16-bit head and an fp32 tail, the degree-7 Taylor polynomial of exp(r)
// on |r| <= ln2/2 in Horner form (fused multiply-adds), and 2^n applied in two
// exact power-of-two steps.  Identical arithmetic to oo_expf in the oracle.
__device__ __forceinline__ float oomb_expf(float x) {
    if (x != x) return x;
    if (x < -104.0f) return 0.0f;
    if (x > 88.5f) return __int_as_float(0x7f800000);
    const float n = rintf(__fmul_rn(x, 1.44269504088896341f));
    float r = __fmaf_rn(-n, 0.693145751953125f, x);
    r = __fmaf_rn(-n, 1.42860682030941723212e-6f, r);
    float p = 1.98412698412698413e-4f;
    p = __fmaf_rn(p, r, 1.38888888888888889e-3f);
    p = __fmaf_rn(p, r, 8.33333333333333333e-3f);
    p = __fmaf_rn(p, r, 4.16666666666666667e-2f);
    p = __fmaf_rn(p, r, 1.66666666666666667e-1f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ni = static_cast<int>(n);
    const int n1 = ni / 2, n2 = ni - n1;
    const float s1 = __int_as_float((n1 + 127) << 23);
    const float s2 = __int_as_float((n2 + 127) << 23);
    return __fmul_rn(__fmul_rn(p, s1), s2);
}

__device__ __forceinline__ float xor_tree32(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

struct RouteParams {
    const void* x;            // [T, H] activations
    int x_bf16;
    const uint16_t* w;        // bf16 router [E, H]
    float* logits;            // [T, E]
    int T, H, E, K;
    // top-k outputs
    int32_t* ids;             // [T, K]
    float* weights;           // [T, K]
    // grouping outputs (null to skip)
    const uint64_t* recs_all; // [E] record addresses of the layer (null: no recs_active)
    int32_t* n_active;        // [1]
    int32_t* active;          // [E]
    int32_t* off;             // [E + 1]
    int32_t* assign_tok;      // [T*K]
    int32_t* slot_assign;     // [T*K]
    uint64_t* recs_active;    // [E]
    unsigned* ticket;         // self-resetting arrival counter (zero before first use)
    int do_logits, do_topk, do_group;
    unsigned* err;
};

constexpr int kRouteThreads = 256;
constexpr int kRouteTT = 4;        // tokens per warp task in the logits phase
constexpr int kRouteMaxH = 4096;   // router rows held in registers up to this width
constexpr int kRouteSmallE = 256;  // experts whose probabilities fit 8 per lane
constexpr size_t kRouteXTileBytes = 64 * 1024;  // shared-memory tile of activations
constexpr int kRouteRecsSmem = 1024;  // layers with at most this many experts stage their record table

// One router row in registers: lane l holds columns 256*i + 8*l + j.
struct RouterRow {
    uint4 w[kRouteMaxH / 256];
};

// A 16-byte load kept in program order with the dependency wait: issued
// before griddepcontrol.wait, it overlaps the wait; its result is used after.
__device__ __forceinline__ uint4 ld_prefetch_v4(const void* ptr) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(ptr));
    return v;
}

__device__ __forceinline__ unsigned long long ld_prefetch_u64(const void* ptr) {
    unsigned long long v;
    asm volatile("ld.global.nc.u64 %0, [%1];" : "=l"(v) : "l"(ptr));
    return v;
}

__device__ __forceinline__ void router_row_load(const RouteParams& p, int e, int lane, RouterRow& r) {
    const uint16_t* wr = p.w + static_cast<int64_t>(e) * p.H;
#pragma unroll
    for (int i = 0; i < kRouteMaxH / 256; i++) {
        const int base = i * 256 + lane * 8;
        r.w[i] = base < p.H ? ld_prefetch_v4(wr + base) : make_uint4(0, 0, 0, 0);
    }
}

// Logits of row e for tokens [t0, t0 + nt) (nt <= kRouteTT) in the canonical
// order: per lane one fmaf chain over its columns in ascending order, then the
// xor tree.  The activations come from the CTA's shared-memory tile `xs`
// (tokens from `xt0`, row stride p.H).
template <bool XBF16>
__device__ __forceinline__ void router_row_dot(const RouteParams& p, const RouterRow& r, const uint8_t* xs,
                                               int xt0, int e, int t0, int nt, int lane) {
    float acc[kRouteTT];
#pragma unroll
    for (int j = 0; j < kRouteTT; j++) acc[j] = 0.0f;
#pragma unroll
    for (int i = 0; i < kRouteMaxH / 256; i++) {
        const int base = i * 256 + lane * 8;
        if (base < p.H) {
            const unsigned ww[4] = {r.w[i].x, r.w[i].y, r.w[i].z, r.w[i].w};
            float wf[8];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                wf[2 * q] = __uint_as_float(ww[q] << 16);
                wf[2 * q + 1] = __uint_as_float(ww[q] & 0xffff0000u);
            }
#pragma unroll
            for (int j = 0; j < kRouteTT; j++) {
                if (j < nt) {
                    float xv[8];
                    const int xi = (t0 + j - xt0) * p.H + base;
                    if (XBF16) {
                        const uint4 a = *reinterpret_cast<const uint4*>(xs + static_cast<size_t>(xi) * 2);
                        const unsigned aa[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                        for (int q = 0; q < 4; q++) {
                            xv[2 * q] = __uint_as_float(aa[q] << 16);
                            xv[2 * q + 1] = __uint_as_float(aa[q] & 0xffff0000u);
                        }
                    } else {
                        const float4* xp = reinterpret_cast<const float4*>(xs + static_cast<size_t>(xi) * 4);
                        const float4 a = xp[0], b = xp[1];
                        xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w;
                        xv[4] = b.x; xv[5] = b.y; xv[6] = b.z; xv[7] = b.w;
                    }
#pragma unroll
                    for (int q = 0; q < 8; q++) acc[j] = __fmaf_rn(xv[q], wf[q], acc[j]);
                }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kRouteTT; j++) {
        const float v = xor_tree32(acc[j]);
        if (j < nt && lane == 0) p.logits[static_cast<int64_t>(t0 + j) * p.E + e] = v;
    }
}

// Wide routers (hidden > kRouteMaxH): the same order streamed from memory.
template <bool XBF16>
__device__ __forceinline__ void router_row_wide(const RouteParams& p, int e, int t0, int nt, int lane) {
    float acc[kRouteTT];
#pragma unroll
    for (int j = 0; j < kRouteTT; j++) acc[j] = 0.0f;
    const uint16_t* wr = p.w + static_cast<int64_t>(e) * p.H;
    for (int base = lane * 8; base < p.H; base += 256) {
        const uint4 wv = __ldg(reinterpret_cast<const uint4*>(wr + base));
        const unsigned ww[4] = {wv.x, wv.y, wv.z, wv.w};
        float wf[8];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            wf[2 * q] = __uint_as_float(ww[q] << 16);
            wf[2 * q + 1] = __uint_as_float(ww[q] & 0xffff0000u);
        }
#pragma unroll
        for (int j = 0; j < kRouteTT; j++) {
            if (j < nt) {
                float xv[8];
                const int64_t xi = static_cast<int64_t>(t0 + j) * p.H + base;
                if (XBF16) {
                    const uint4 a = __ldcg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.x) + xi));
                    const unsigned aa[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        xv[2 * q] = __uint_as_float(aa[q] << 16);
                        xv[2 * q + 1] = __uint_as_float(aa[q] & 0xffff0000u);
                    }
                } else {
                    const float4* xp = reinterpret_cast<const float4*>(static_cast<const float*>(p.x) + xi);
                    const float4 a = __ldcg(xp), b = __ldcg(xp + 1);
                    xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w;
                    xv[4] = b.x; xv[5] = b.y; xv[6] = b.z; xv[7] = b.w;
                }
#pragma unroll
                for (int q = 0; q < 8; q++) acc[j] = __fmaf_rn(xv[q], wf[q], acc[j]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kRouteTT; j++) {
        const float v = xor_tree32(acc[j]);
        if (j < nt && lane == 0) p.logits[static_cast<int64_t>(t0 + j) * p.E + e] = v;
    }
}

// Softmax top-k of one token by one warp.  Lane l owns experts l, l+32, ...;
// with E <= 256 their probabilities stay in registers.
__device__ __forceinline__ void topk_token(const RouteParams& p, int t, int lane, int32_t* ids_sm) {
    const float* l = p.logits + static_cast<int64_t>(t) * p.E;
    const float NEG_INF = -__int_as_float(0x7f800000);
    int my_id = 0;
    float my_p = 0.0f, psum = 0.0f;
    if (p.E <= kRouteSmallE) {
        float pe[kRouteSmallE / 32];
        float mx = NEG_INF;
#pragma unroll
        for (int j = 0; j < kRouteSmallE / 32; j++) {
            const int e = lane + 32 * j;
            pe[j] = e < p.E ? __ldcg(l + e) : NEG_INF;
            mx = fmaxf(mx, pe[j]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < kRouteSmallE / 32; j++) {
            if (lane + 32 * j < p.E) {
                pe[j] = oomb_expf(__fsub_rn(pe[j], mx));
                s = __fadd_rn(s, pe[j]);
            }
        }
        const float sum = xor_tree32(s);
#pragma unroll
        for (int j = 0; j < kRouteSmallE / 32; j++) pe[j] = lane + 32 * j < p.E ? __fdiv_rn(pe[j], sum) : -3.0f;
        for (int r = 0; r < p.K; r++) {
            float bv = -3.0f;
            int bi = 0x7fffffff;
#pragma unroll
            for (int j = 0; j < kRouteSmallE / 32; j++)
                if (pe[j] > bv) { bv = pe[j]; bi = lane + 32 * j; }  // ascending ids: ties keep the lower
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
#pragma unroll
            for (int j = 0; j < kRouteSmallE / 32; j++)
                if (lane + 32 * j == bi) pe[j] = -2.0f;  // used entries sit below every probability
            if (lane == r) { my_id = bi; my_p = bv; }
            psum = __fadd_rn(psum, bv);
        }
    } else {
        float mx = NEG_INF;
        for (int i = lane; i < p.E; i += 32) mx = fmaxf(mx, __ldcg(l + i));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float s = 0.0f;
        for (int i = lane; i < p.E; i += 32) s = __fadd_rn(s, oomb_expf(__fsub_rn(__ldcg(l + i), mx)));
        const float sum = xor_tree32(s);
        unsigned long long picked_mask = 0;  // picks found in this lane's experts: bit j for expert lane+32j (j < 64)
        int picked_far[32];
        int nfar = 0;
        for (int r = 0; r < p.K; r++) {
            float bv = -3.0f;
            int bi = 0x7fffffff;
            for (int i = lane, j = 0; i < p.E; i += 32, j++) {
                bool used = j < 64 ? ((picked_mask >> j) & 1ull) != 0 : false;
                for (int q = 0; q < nfar; q++) used |= picked_far[q] == i;
                const float pi = used ? -2.0f : __fdiv_rn(oomb_expf(__fsub_rn(__ldcg(l + i), mx)), sum);
                if (pi > bv) { bv = pi; bi = i; }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
            if ((bi & 31) == lane) {
                const int j = bi >> 5;
                if (j < 64) picked_mask |= 1ull << j;
                else picked_far[nfar++] = bi;
            }
            if (lane == r) { my_id = bi; my_p = bv; }
            psum = __fadd_rn(psum, bv);
        }
    }
    if (lane < p.K) {
        p.ids[static_cast<int64_t>(t) * p.K + lane] = my_id;
        p.weights[static_cast<int64_t>(t) * p.K + lane] = __fdiv_rn(my_p, psum);
        if (ids_sm) ids_sm[t * p.K + lane] = my_id;
    }
}

// Softmax top-k of tokens [t0, t1) by the whole CTA, E <= kRouteSmallE.
// 1. Each warp computes the softmax of whole tokens in the canonical order
//    of topk_token (lane l owns experts l, l+32, ...) into prob[token][E]
//    (shared memory; NaN stored as -3, below every probability).
// 2. Every warp takes candidates of each token and counts, over its lanes, the
//    experts that beat the candidate: e beats i when p_e > p_i, or p_e == p_i
//    and e < i.  The candidate beaten by exactly r others is the r-th pick of k
//    argmax rounds with ties to the lower id (ops.cu:234-294).
// 3. weights = p / (sum of the picked p in pick order).
// Writes ids_out / w_out ([T, K], indexed by global token) and, if non-null,
// ids_sm.  prob: (t1 - t0) * E floats; pick_id / pick_p: (t1 - t0) * K entries.
// NT: the CTA's threads (all of them call this).  logits: [T, E] in global
// memory, or in this CTA's shared memory (LSM).
template <int NT, bool LSM = false>
__device__ void topk_block(const RouteParams& p, const float* logits, int t0, int t1, float* prob, int32_t* pick_id,
                           float* pick_p, int32_t* ids_out, float* w_out, int32_t* ids_sm) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int nwarps = NT / 32;
    constexpr int NJ = kRouteSmallE / 32;
    const int nt = t1 - t0, E = p.E;
    const float NEG_INF = -__int_as_float(0x7f800000);
    for (int tl = warp; tl < nt; tl += nwarps) {
        const float* l = logits + static_cast<int64_t>(t0 + tl) * E;
        float pe[NJ];
        float mx = NEG_INF;
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int e = lane + 32 * j;
            pe[j] = e < E ? (LSM ? l[e] : __ldcg(l + e)) : NEG_INF;
            mx = fmaxf(mx, pe[j]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            if (lane + 32 * j < E) {
                pe[j] = oomb_expf(__fsub_rn(pe[j], mx));
                s = __fadd_rn(s, pe[j]);
            }
        }
        const float sum = xor_tree32(s);
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int e = lane + 32 * j;
            if (e < E) {
                const float v = __fdiv_rn(pe[j], sum);
                prob[tl * E + e] = v == v ? v : -3.0f;
            }
        }
    }
    __syncthreads();
    // Ranks: lane l holds the token's probabilities of experts l + 32 j (absent
    // experts -5, below every stored value); warp w takes candidates w, w + nwarps,
    // ... and counts the experts that beat each over the warp.
    for (int tl = 0; tl < nt; tl++) {
        const float* pt = prob + tl * E;
        float pv[NJ];
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int e = lane + 32 * j;
            pv[j] = e < E ? pt[e] : -5.0f;
        }
        // four candidates at a time, so their load-compare-reduce chains overlap
        for (int i0 = warp; i0 < E; i0 += 4 * nwarps) {
            float pi[4];
            unsigned b[4];
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int i = i0 + c * nwarps;
                pi[c] = pt[i < E ? i : 0];
                b[c] = 0;
            }
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int i = i0 + c * nwarps;
#pragma unroll
                for (int j = 0; j < NJ; j++) b[c] += (pv[j] > pi[c] || (pv[j] == pi[c] && lane + 32 * j < i)) ? 1u : 0u;
            }
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int i = i0 + c * nwarps;
                const unsigned beats = __reduce_add_sync(0xffffffffu, b[c]);
                if (lane == 0 && i < E && beats < static_cast<unsigned>(p.K)) {
                    pick_id[tl * p.K + beats] = i;
                    pick_p[tl * p.K + beats] = pi[c];
                }
            }
        }
    }
    __syncthreads();
    for (int o = threadIdx.x; o < nt * p.K; o += NT) {
        const int tl = o / p.K, r = o - tl * p.K;
        float psum = 0.0f;
        for (int q = 0; q < p.K; q++) psum = __fadd_rn(psum, pick_p[tl * p.K + q]);
        const int64_t gi = static_cast<int64_t>(t0 + tl) * p.K + r;
        ids_out[gi] = pick_id[o];
        w_out[gi] = __fdiv_rn(pick_p[o], psum);
        if (ids_sm) ids_sm[(t0 + tl) * p.K + r] = pick_id[o];
    }
}

// Softmax top-k of tokens [t0, t1) with one warp per token (E <= kRouteSmallE):
// the same picks and weights as topk_block.  Each warp computes the token's
// canonical softmax (NaN stored as -3), then k argmax rounds over (p desc,
// id asc): exactly the first k of the order topk_block ranks by.  A round is
// two warp reductions (max of an order key, then min of the ids holding it).  The
// weights are p / (sum of the picks in pick order).  logits: [T, E] in global
// memory, or in this CTA's shared memory (LSM).  For a few tokens per warp this
// is far shorter than the block-wide ranking.
// NJ: probabilities per lane (E <= 32 NJ).
template <int NT, bool LSM, int NJ>
__device__ void topk_warps(const RouteParams& p, const float* logits, int t0, int t1, int32_t* ids_out, float* w_out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int nwarps = NT / 32;
    const int E = p.E, K = p.K;
    const float NEG_INF = -__int_as_float(0x7f800000);
    for (int t = t0 + warp; t < t1; t += nwarps) {
        const float* l = logits + static_cast<int64_t>(t) * E;
        float pe[NJ];
        float mx = NEG_INF;
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            const int e = lane + 32 * j;
            pe[j] = e < E ? (LSM ? l[e] : __ldcg(l + e)) : NEG_INF;
            mx = fmaxf(mx, pe[j]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            if (lane + 32 * j < E) {
                pe[j] = oomb_expf(__fsub_rn(pe[j], mx));
                s = __fadd_rn(s, pe[j]);
            }
        }
        const float sum = xor_tree32(s);
#pragma unroll
        for (int j = 0; j < NJ; j++) {
            if (lane + 32 * j < E) {
                const float v = __fdiv_rn(pe[j], sum);
                pe[j] = v == v ? v : -3.0f;
            } else {
                pe[j] = -5.0f;
            }
        }
        // Order keys: a probability's bits + 2 (non-negative floats order as
        // their bits), 1 for NaN (-3), 0 for an absent or picked expert.
        unsigned key[NJ];
#pragma unroll
        for (int j = 0; j < NJ; j++) key[j] = pe[j] >= 0.0f ? (__float_as_uint(pe[j]) & 0x7fffffffu) + 2u : (pe[j] == -3.0f ? 1u : 0u);
        int my_id = 0;
        float my_p = 0.0f, psum = 0.0f;
        for (int r = 0; r < K; r++) {
            unsigned bk = 0u, bi = 0xffffffffu;
#pragma unroll
            for (int j = 0; j < NJ; j++)
                if (key[j] > bk) {  // ascending ids within the lane: ties keep the lower
                    bk = key[j];
                    bi = static_cast<unsigned>(lane + 32 * j);
                }
            const unsigned mk = __reduce_max_sync(0xffffffffu, bk);
            const unsigned mi = __reduce_min_sync(0xffffffffu, bk == mk ? bi : 0xffffffffu);
#pragma unroll
            for (int j = 0; j < NJ; j++)
                if (static_cast<unsigned>(lane + 32 * j) == mi) key[j] = 0u;
            const float bv = mk >= 2u ? __uint_as_float(mk - 2u) : -3.0f;
            if (lane == r) {
                my_id = static_cast<int>(mi);
                my_p = bv;
            }
            psum = __fadd_rn(psum, bv);
        }
        if (lane < K) {
            ids_out[static_cast<int64_t>(t) * K + lane] = my_id;
            w_out[static_cast<int64_t>(t) * K + lane] = __fdiv_rn(my_p, psum);
        }
    }
}

// Where grouping writes its tables: the caller's global buffers (route_kernel)
// or shared memory (decode_kernel).
struct GroupOut {
    int32_t* n_active;
    int32_t* active;
    int32_t* off;
    int32_t* assign_tok;
    int32_t* slot_assign;
    uint64_t* recs_active;
    int32_t* assign_ret;  // optional: the slot (flat index) of each assignment
};

// Groups the T*K assignments by expert (counting sort, stable in slot order).
// SKIP_NEG: entries of -1 are another rank's (expert parallelism) and are
// skipped without an error.  Runs on one CTA of NT threads; ids in shared memory.  counts, base: E ints of
// shared scratch; recs_sm: the layer's record addresses staged in shared
// memory, or null to read them from p.recs_all.
template <int NT, bool SKIP_NEG = false>
__device__ void group_assignments(const RouteParams& p, const GroupOut& g, const int32_t* ids_sm, int32_t* counts,
                                  int32_t* base, const uint64_t* recs_sm) {
    const int A = p.T * p.K;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int e = threadIdx.x; e < p.E; e += blockDim.x) counts[e] = 0;
    __syncthreads();
    for (int s = threadIdx.x; s < A; s += blockDim.x) {
        const int e = ids_sm[s];
        if (e >= 0 && e < p.E) atomicAdd(&counts[e], 1);
        else if (!(SKIP_NEG && e < 0)) record_error(p.err, ERR_BAD_TABLE);
    }
    __syncthreads();
    if (p.E <= NT) {
        // One expert per thread: exclusive scans of the assignment counts and of
        // the active flags over the CTA (warp scans, then the warp totals).
        __shared__ int wtot_a[NT / 32], wtot_n[NT / 32];
        const int e = threadIdx.x;
        const int c = e < p.E ? counts[e] : 0;
        int inc_a = c, inc_n = c > 0 ? 1 : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int va = __shfl_up_sync(0xffffffffu, inc_a, o);
            const int vn = __shfl_up_sync(0xffffffffu, inc_n, o);
            if (lane >= o) { inc_a += va; inc_n += vn; }
        }
        if (lane == 31) { wtot_a[warp] = inc_a; wtot_n[warp] = inc_n; }
        __syncthreads();
        int pre_a = 0, pre_n = 0;
        for (int w = 0; w < warp; w++) { pre_a += wtot_a[w]; pre_n += wtot_n[w]; }
        const int start = pre_a + inc_a - c;
        const int idx = pre_n + inc_n - (c > 0 ? 1 : 0);
        if (c > 0) {
            base[e] = start;
            g.active[idx] = e;
            g.off[idx] = start;
            if (p.recs_all) g.recs_active[idx] = recs_sm ? recs_sm[e] : __ldcg(p.recs_all + e);
        }
        if (threadIdx.x == NT - 1) {
            g.off[pre_n + inc_n] = pre_a + inc_a;
            *g.n_active = pre_n + inc_n;
        }
        __syncthreads();
    } else if (threadIdx.x < 32) {
        // Exclusive scans over experts, 32 at a time: assignment start and active index.
        int run_a = 0, run_n = 0;
        for (int e0 = 0; e0 < p.E; e0 += 32) {
            const int e = e0 + lane;
            const int c = e < p.E ? counts[e] : 0;
            int inc_a = c, inc_n = c > 0 ? 1 : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int va = __shfl_up_sync(0xffffffffu, inc_a, o);
                const int vn = __shfl_up_sync(0xffffffffu, inc_n, o);
                if (lane >= o) { inc_a += va; inc_n += vn; }
            }
            const int start = run_a + inc_a - c;
            const int idx = run_n + inc_n - (c > 0 ? 1 : 0);
            if (e < p.E && c > 0) {
                base[e] = start;
                g.active[idx] = e;
                g.off[idx] = start;
                if (p.recs_all) g.recs_active[idx] = recs_sm ? recs_sm[e] : __ldcg(p.recs_all + e);
            }
            run_a += __shfl_sync(0xffffffffu, inc_a, 31);
            run_n += __shfl_sync(0xffffffffu, inc_n, 31);
        }
        if (lane == 0) {
            g.off[run_n] = run_a;
            *g.n_active = run_n;
        }
    }
    if (threadIdx.x < 32) {
        // Ranks in slot order, 32 slots at a time.
        for (int s0 = 0; s0 < A; s0 += 32) {
            const int s = s0 + lane;
            const int e = s < A ? ids_sm[s] : -1 - lane;  // unique dummies for idle lanes
            const unsigned peers = __match_any_sync(0xffffffffu, e);
            const int rank = __popc(peers & ((1u << lane) - 1u));
            if (s < A && e >= 0 && e < p.E) {
                const int a = base[e] + rank;
                g.assign_tok[a] = s / p.K;
                g.slot_assign[s] = a;
                if (g.assign_ret) g.assign_ret[a] = s;
            }
            __syncwarp();
            // the highest lane of each peer group advances the expert's base
            if (s < A && e >= 0 && e < p.E && (peers >> lane) == 1u) base[e] += rank + 1;
            __syncwarp();
        }
    }
}

// The tables of group_assignments for at most 32 assignments, by one warp (all
// its lanes call this): lane s holds assignment s; its position in (expert,
// slot) order is the count of assignments of smaller experts plus the earlier
// slots of its own expert; the first slot of each expert leads the expert's
// group, whose index is the count of leaders of smaller experts.
template <bool SKIP_NEG = false>
__device__ void group_warp(const RouteParams& p, const GroupOut& g, const int32_t* ids_sm, const uint64_t* recs_sm) {
    const int lane = threadIdx.x & 31;
    const int A = p.T * p.K;
    int key = 0x7fffffff;
    bool valid = false;
    if (lane < A) {
        const int e = ids_sm[lane];
        valid = e >= 0 && e < p.E;
        if (valid) key = e;
        else if (!(SKIP_NEG && e < 0)) record_error(p.err, ERR_BAD_TABLE);
    }
    int lt = 0, before = 0;
#pragma unroll 4
    for (int q = 0; q < A; q++) {
        const int kq = __shfl_sync(0xffffffffu, key, q);
        lt += kq < key ? 1 : 0;
        before += (kq == key && q < lane) ? 1 : 0;
    }
    const bool leader = valid && before == 0;
    const unsigned lead = __ballot_sync(0xffffffffu, leader);
    const unsigned vmask = __ballot_sync(0xffffffffu, valid);
    int idx = 0;
#pragma unroll 4
    for (int q = 0; q < A; q++) {
        const int kq = __shfl_sync(0xffffffffu, key, q);
        idx += (((lead >> q) & 1u) && kq < key) ? 1 : 0;
    }
    if (valid) {
        const int a = lt + before;
        g.assign_tok[a] = lane / p.K;
        g.slot_assign[lane] = a;
        if (g.assign_ret) g.assign_ret[a] = lane;
    }
    if (leader) {
        g.active[idx] = key;
        g.off[idx] = lt;
        if (p.recs_all) g.recs_active[idx] = recs_sm ? recs_sm[key] : __ldcg(p.recs_all + key);
    }
    if (lane == 0) {
        const int n = __popc(lead);
        g.off[n] = __popc(vmask);
        *g.n_active = n;
    }
}

// Shared memory of route_kernel:
//   [x tile][recs E u64][pick ids PT*K][pick p PT*K][prob PT*E][ids T*K][counts E][base E]
// (PT: tokens one CTA ranks: all T when it also groups, else kRouteThreads/32).
struct RouteSmem {
    int xtile_tokens;  // tokens of x staged per tile (narrow routers), 0 otherwise
    size_t x_bytes, recs_off, pick_off, ids_off, total;
};

__host__ __device__ inline RouteSmem route_smem(int T, int H, int E, int K, bool x_bf16, bool logits, bool topk,
                                                bool group) {
    RouteSmem m{};
    const size_t xb = x_bf16 ? 2 : 4;
    if (logits && H <= kRouteMaxH) {
        int tt = static_cast<int>(kRouteXTileBytes / (static_cast<size_t>(H) * xb)) / kRouteTT * kRouteTT;
        if (tt < kRouteTT) tt = kRouteTT;
        m.xtile_tokens = T < tt ? T : tt;
        m.x_bytes = (static_cast<size_t>(m.xtile_tokens) * H * xb + 15) & ~static_cast<size_t>(15);
    }
    m.recs_off = m.x_bytes;
    const size_t recs = group && E <= kRouteRecsSmem ? static_cast<size_t>(E) * 8 : 0;
    m.pick_off = m.recs_off + recs;
    const size_t pt = group ? static_cast<size_t>(T) : static_cast<size_t>(kRouteThreads / 32);
    const size_t picks = topk && E <= kRouteSmallE ? (2 * pt * K + pt * E) * 4 : 0;
    m.ids_off = m.pick_off + picks;
    m.total = m.ids_off + (group ? (static_cast<size_t>(T) * K + 2 * static_cast<size_t>(E)) * 4 : 0);
    return m;
}

// Logits phase: warp w of CTA c owns router row c*8 + w (one row per warp: the
// host launches ceil(E/8) CTAs), fetched into registers before the dependency
// wait.  After the wait the CTA stages the activations of a tile of tokens in
// shared memory with one cooperative load and every warp takes its row's
// dot products from there.  The last CTA to finish (atomic ticket) runs the
// softmax top-k of every token and the grouping, with the layer's record
// addresses already staged by every CTA before the wait.
template <bool XBF16>
__global__ void __launch_bounds__(kRouteThreads) route_kernel(const RouteParams p) {
    extern __shared__ __align__(16) uint8_t rsm[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int nwarps = kRouteThreads / 32;
    const RouteSmem sm = route_smem(p.T, p.H, p.E, p.K, XBF16, p.do_logits != 0, p.do_topk != 0, p.do_group != 0);
    const bool ranked = p.E <= kRouteSmallE;
    int32_t* pick_id = reinterpret_cast<int32_t*>(rsm + sm.pick_off);
    const int pt = p.do_group ? p.T : nwarps;
    float* pick_p = reinterpret_cast<float*>(rsm + sm.pick_off) + pt * p.K;
    float* prob = pick_p + pt * p.K;
    uint64_t* recs_sm = (p.do_group && p.recs_all && p.E <= kRouteRecsSmem)
                            ? reinterpret_cast<uint64_t*>(rsm + sm.recs_off) : nullptr;
    int32_t* ids_sm = p.do_group ? reinterpret_cast<int32_t*>(rsm + sm.ids_off) : nullptr;

    // The layer's record addresses do not depend on the previous kernel: every
    // CTA fetches them before waiting (only the last CTA will use them).
    uint64_t rec_pre[kRouteRecsSmem / kRouteThreads];
    if (recs_sm) {
#pragma unroll
        for (int m = 0; m < kRouteRecsSmem / kRouteThreads; m++) {
            const int e = threadIdx.x + m * kRouteThreads;
            rec_pre[m] = e < p.E ? ld_prefetch_u64(reinterpret_cast<const unsigned long long*>(p.recs_all) + e) : 0ull;
        }
    }

    if (p.do_logits) {
        const int e = blockIdx.x * nwarps + warp;
        const bool has_row = e < p.E;
        const bool narrow = p.H <= kRouteMaxH;
        // The router row does not depend on the previous kernel either.
        RouterRow row;
        if (narrow && has_row) router_row_load(p, e, lane, row);
        pdl_wait();
        pdl_launch_dependents();
        if (narrow) {
            const int xb = XBF16 ? 2 : 4;
            for (int xt0 = 0; xt0 < p.T; xt0 += sm.xtile_tokens) {
                const int xn = min(sm.xtile_tokens, p.T - xt0);
                // x rows [xt0, xt0 + xn) are contiguous: copy them 16 bytes a thread
                const int chunks = xn * p.H * xb / 16;
                const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.x) +
                                                                  static_cast<size_t>(xt0) * p.H * xb);
                uint4* dst = reinterpret_cast<uint4*>(rsm);
                for (int c = threadIdx.x; c < chunks; c += kRouteThreads) dst[c] = __ldcg(src + c);
                __syncthreads();
                if (has_row)
                    for (int t0 = xt0; t0 < xt0 + xn; t0 += kRouteTT)
                        router_row_dot<XBF16>(p, row, rsm, xt0, e, t0, min(kRouteTT, xt0 + xn - t0), lane);
                __syncthreads();
            }
        } else if (has_row) {
            for (int t0 = 0; t0 < p.T; t0 += kRouteTT) router_row_wide<XBF16>(p, e, t0, min(kRouteTT, p.T - t0), lane);
        }
        if (!p.do_topk) return;
        // The last CTA to finish its logits runs the rest (deterministic: the
        // work it does depends only on the logits, not on which CTA it is).
        __shared__ bool last;
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) last = atomicAdd(p.ticket, 1u) == gridDim.x - 1;
        __syncthreads();
        if (!last) return;
        __threadfence();
        if (threadIdx.x == 0) {
            *p.ticket = 0u;
        }
    } else {
        pdl_wait();
        pdl_launch_dependents();
    }
    if (p.do_group) {
        if (recs_sm) {
#pragma unroll
            for (int m = 0; m < kRouteRecsSmem / kRouteThreads; m++) {
                const int e = threadIdx.x + m * kRouteThreads;
                if (e < p.E) recs_sm[e] = rec_pre[m];
            }
        }
        // grouping needs every token's picks in one CTA
        if (ranked) {
            topk_block<kRouteThreads>(p, p.logits, 0, p.T, prob, pick_id, pick_p, p.ids, p.weights, ids_sm);
        } else {
            for (int t = warp; t < p.T; t += nwarps) topk_token(p, t, lane, ids_sm);
        }
        __syncthreads();
        const GroupOut go{p.n_active, p.active, p.off, p.assign_tok, p.slot_assign, p.recs_active, nullptr};
        group_assignments<kRouteThreads>(p, go, ids_sm, ids_sm + p.T * p.K, ids_sm + p.T * p.K + p.E, recs_sm);
    } else if (ranked) {
        for (int t0 = blockIdx.x * nwarps; t0 < p.T; t0 += gridDim.x * nwarps) {
            topk_block<kRouteThreads>(p, p.logits, t0, min(p.T, t0 + nwarps), prob, pick_id, pick_p, p.ids, p.weights,
                                      nullptr);
            __syncthreads();
        }
    } else {
        for (int t = blockIdx.x * nwarps + warp; t < p.T; t += gridDim.x * nwarps) topk_token(p, t, lane, nullptr);
    }
}

}  // namespace oomb
