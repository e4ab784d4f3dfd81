// attn.cuh - grouped-query decode attention over a bf16 KV cache (split-K flash-decode).
//
// For every sequence b (one query token each) and query head h of kv head
// h / G (G = heads / kv_heads query heads share a kv head):
//   out[b, h, :] = sum_j softmax_j(scale * q[b, h, :] . K[b, j, h / G, :]) V[b, j, h / G, :],
// j < kv_len[b], fp32 softmax and accumulation.  The decode case of the
// reference's Attention::attention (crates/oominf-core/src/backend.rs:551-568)
// as its flash-decode kernels compute it (attn_decode_partial_g12 +
// attn_decode_combine, crates/oominf-cuda/kernels/attention.cu:592-700): each
// worker keeps an online-softmax partial (running max m, sum l, unnormalised
// accumulator) over its share of the positions, and the partials merge as
//   out = sum_w e^(m_w - M) acc_w / sum_w e^(m_w - M) l_w,  M = max_w m_w.
// Here the cache is bf16 (the reference's is fp32 with hd 256 and G = 12), the
// merge runs in the same launch, and the layout is the reference's: row j of
// kv head c at ((j * kv_heads + c) * D) elements from the sequence's base.
//
// Bound: HBM (every K and V byte read once; 2 * kv_len * kv_heads * D * 2
// bytes per sequence).  Grid (splits, kv_heads, batch), 4 warps per CTA; warp
// w of split s takes a contiguous share of the positions and walks it in
// chunks of CP = min(32 / G, 8) positions: lane l owns elements [l * E, l * E + E) of a
// row (E = D / 32), so a warp reads each 2D-byte row with one coalesced load;
// the CP x G partial dot products of a chunk are summed over the lanes by one
// multi-value butterfly (lane l ends with the score of (position l / G, head
// l % G)); the chunk's softmax runs one score per lane; the weights reach
// every lane through shared memory for the V update.  The CTA merges its
// warps' partials in shared memory (warp order) and writes one partial to the
// workspace; the last CTA of a (sequence, kv head) to finish (an arrival
// counter that resets itself) merges the splits' partials in split order and
// writes the output: deterministic.
#pragma once

#include "common.cuh"

namespace oomb {

constexpr int kAttnWarps = 4;
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kAttnMaxSplits = 32;  // CTAs per (sequence, kv head): the last one merges at most this many (64 measured slower at batch 1: 17.5 -> 24.0 us)

enum : unsigned {
    ERR_ATTN_LEN = 0x800,  // a kv_len entry was outside [0, kv_max] (clamped)
};

struct AttnParams {
    const void* q;         // [B, H, D] fp32 or bf16
    int q_bf16;
    const uint16_t* k;     // bf16 K cache: sequence b at b * seq_stride elements, row j of kv head c at (j * Hkv + c) * D
    const uint16_t* v;     // bf16 V cache, same layout
    int64_t seq_stride;
    const int32_t* kv_len; // [B] visible positions per sequence (device), or null: kv_len_host for all
    int kv_len_host;
    void* out;             // [B, H, D] fp32 or bf16
    int out_bf16;
    int B, H, Hkv, kv_max;
    int splits;            // CTAs per (sequence, kv head)
    float scale;
    float* part;           // [B][Hkv][splits][G][D + 4]: acc, m, l of each CTA (rows 16-byte aligned)
    unsigned* counters;    // [B * Hkv] arrivals, zero between launches
    unsigned* err;
};

__device__ __forceinline__ void bf16x4_to_f32(uint2 w, float (&f)[4]) {
    f[0] = __uint_as_float(w.x << 16);
    f[1] = __uint_as_float(w.x & 0xffff0000u);
    f[2] = __uint_as_float(w.y << 16);
    f[3] = __uint_as_float(w.y & 0xffff0000u);
}

template <int G, int D>
__global__ void __launch_bounds__(kAttnThreads, G <= 4 ? 4 : 3) attn_decode_kernel(const AttnParams p) {
    static_assert(D == 128, "lanes own four elements of a row");
    static_assert(G >= 1 && G <= 32 && (32 % G) == 0, "G must divide 32");
    constexpr int E = D / 32;
    constexpr int CP = 32 / G < 8 ? 32 / G : 8;  // positions per chunk: CP * G <= 32 scores, one per lane
    constexpr int PS = D + 4;                      // floats per partial row: acc[D], m, l, padding
    __shared__ float2 ebuf[kAttnWarps][32];
    __shared__ float2 cbuf[kAttnWarps][32];
    __shared__ bool last;
    const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    pdl_wait();  // q (and the cache rows just appended) come from earlier kernels
    pdl_launch_dependents();
    int L = p.kv_len ? __ldcg(p.kv_len + b) : p.kv_len_host;
    if (L < 0 || L > p.kv_max) {
        if (threadIdx.x == 0) record_error(p.err, ERR_ATTN_LEN);
        L = max(0, min(L, p.kv_max));
    }
    const int W = p.splits * kAttnWarps, wi = split * kAttnWarps + warp;  // this warp's share of [0, L)
    const int j0 = static_cast<int>(static_cast<int64_t>(L) * wi / W);
    const int j1 = static_cast<int>(static_cast<int64_t>(L) * (wi + 1) / W);

    // this lane's elements of the G query heads, scaled, as pairs (elements 0,1 and 2,3)
    float2 qp[G][2];
#pragma unroll
    for (int g = 0; g < G; g++) {
        const int64_t qi = (static_cast<int64_t>(b) * p.H + kvh * G + g) * D + lane * E;
        float f[4];
        if (p.q_bf16) {
            bf16x4_to_f32(__ldcg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(p.q) + qi)), f);
        } else {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(static_cast<const float*>(p.q) + qi));
            f[0] = v.x;
            f[1] = v.y;
            f[2] = v.z;
            f[3] = v.w;
        }
        qp[g][0] = make_float2(f[0] * p.scale, f[1] * p.scale);
        qp[g][1] = make_float2(f[2] * p.scale, f[3] * p.scale);
    }
    // unnormalised accumulators of the lane's four elements, per head, as pairs
    float2 acc[G][2];
#pragma unroll
    for (int g = 0; g < G; g++) acc[g][0] = acc[g][1] = make_float2(0.0f, 0.0f);
    // running max and sum of the lane's head (lane % G); the same in every lane of that head
    float m_run = -INFINITY, l_run = 0.0f;
    const int64_t row_stride = static_cast<int64_t>(p.Hkv) * D;
    const uint16_t* kb = p.k + static_cast<int64_t>(b) * p.seq_stride + static_cast<int64_t>(kvh) * D + lane * E;
    const uint16_t* vb = p.v + static_cast<int64_t>(b) * p.seq_stride + static_cast<int64_t>(kvh) * D + lane * E;

    uint2 kr[CP];
    auto load_k = [&](int j) {
#pragma unroll
        for (int c = 0; c < CP; c++)
            kr[c] = j + c < j1 ? __ldcs(reinterpret_cast<const uint2*>(kb + (j + c) * row_stride)) : make_uint2(0u, 0u);
    };
    if (j0 < j1) load_k(j0);
    for (int j = j0; j < j1; j += CP) {
        const int n = min(CP, j1 - j);
        uint2 vr[CP];
#pragma unroll
        for (int c = 0; c < CP; c++)
            vr[c] = c < n ? __ldcs(reinterpret_cast<const uint2*>(vb + (j + c) * row_stride)) : make_uint2(0u, 0u);
        // partial scores: value c * G + g = this lane's share of q_g . k_c (two
        // element pairs at once, then the pair's halves added)
        float s[32];
#pragma unroll
        for (int i = CP * G; i < 32; i++) s[i] = 0.0f;
#pragma unroll
        for (int c = 0; c < CP; c++) {
            const float2 k01 = make_float2(__uint_as_float(kr[c].x << 16), __uint_as_float(kr[c].x & 0xffff0000u));
            const float2 k23 = make_float2(__uint_as_float(kr[c].y << 16), __uint_as_float(kr[c].y & 0xffff0000u));
#pragma unroll
            for (int g = 0; g < G; g++) {
                const float2 d2 = ffma2(qp[g][1], k23, fmul2(qp[g][0], k01));
                s[c * G + g] = __fadd_rn(d2.x, d2.y);
            }
        }
        if (j + CP < j1) load_k(j + CP);  // the next chunk's keys load under this chunk's math
        warp_reduce_multi<32>(s, lane);   // lane l: the score of (position l / G, head l % G)
        const int c_l = lane / G;  // lanes past CP * G hold padding: c_l >= CP >= n
        const float sc = c_l < n ? s[0] : -INFINITY;
        float cmax = sc;
#pragma unroll
        for (int o = G; o < 32; o <<= 1) cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, o));
        const float m_new = fmaxf(m_run, cmax);
        const float corr = __expf(m_run - m_new);
        const float e = c_l < n ? __expf(sc - m_new) : 0.0f;
        float esum = e;
#pragma unroll
        for (int o = G; o < 32; o <<= 1) esum += __shfl_xor_sync(0xffffffffu, esum, o);
        l_run = fmaf(l_run, corr, esum);
        m_run = m_new;
        ebuf[warp][lane] = make_float2(e, e);  // as pairs: one load gives both lanes of a packed FMA
        cbuf[warp][lane] = make_float2(corr, corr);
        __syncwarp();
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float2 cg = cbuf[warp][g];
            acc[g][0] = fmul2(acc[g][0], cg);
            acc[g][1] = fmul2(acc[g][1], cg);
        }
#pragma unroll
        for (int c = 0; c < CP; c++) {
            const float2 v01 = make_float2(__uint_as_float(vr[c].x << 16), __uint_as_float(vr[c].x & 0xffff0000u));
            const float2 v23 = make_float2(__uint_as_float(vr[c].y << 16), __uint_as_float(vr[c].y & 0xffff0000u));
#pragma unroll
            for (int g = 0; g < G; g++) {
                const float2 w = ebuf[warp][c * G + g];
                acc[g][0] = ffma2(w, v01, acc[g][0]);
                acc[g][1] = ffma2(w, v23, acc[g][1]);
            }
        }
        __syncwarp();
    }

    // ---- the CTA's partial: its warps' partials merged in warp order ----
    __shared__ float wm[kAttnWarps][G], wl[kAttnWarps][G];
    __shared__ __align__(16) float wacc[kAttnWarps][G][D];
    if (lane < G) {
        wm[warp][lane] = m_run;  // lane g holds head g's running max and sum
        wl[warp][lane] = l_run;
    }
#pragma unroll
    for (int g = 0; g < G; g++)
        *reinterpret_cast<float4*>(&wacc[warp][g][lane * E]) =
            make_float4(acc[g][0].x, acc[g][0].y, acc[g][1].x, acc[g][1].y);
    __syncthreads();
    const int64_t pbase = (static_cast<int64_t>(b) * p.Hkv + kvh) * p.splits;
    float* mine = p.part + (pbase + split) * G * PS;
    for (int o = threadIdx.x; o < G * D; o += kAttnThreads) {
        const int g = o / D, d = o - g * D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kAttnWarps; w++) M = fmaxf(M, wm[w][g]);
        float a = 0.0f, l = 0.0f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kAttnWarps; w++) {
                if (wm[w][g] == -INFINITY) continue;
                const float f = __expf(wm[w][g] - M);
                a = fmaf(f, wacc[w][g][d], a);
                l = fmaf(f, wl[w][g], l);
            }
        }
        mine[g * PS + d] = a;
        if (d == 0) {
            mine[g * PS + D] = M;
            mine[g * PS + D + 1] = l;
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(p.counters + b * p.Hkv + kvh, 1u);
        last = prev == static_cast<unsigned>(p.splits - 1);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    // ---- the last CTA of the (sequence, kv head): merge the splits' partials in split order ----
    constexpr int kMaxSplitsSmem = kAttnWarps * D;  // factors e^(m_s - M) staged per head in wacc
    const float* all = p.part + pbase * G * PS;
    float* fac = &wacc[0][0][0];  // [G][splits]
    for (int g = warp; g < G; g += kAttnWarps) {
        float M = -INFINITY;
        for (int s2 = lane; s2 < p.splits; s2 += 32) M = fmaxf(M, __ldcg(all + (static_cast<int64_t>(s2) * G + g) * PS + D));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        for (int s2 = lane; s2 < p.splits && s2 < kMaxSplitsSmem / G; s2 += 32) {
            const float ms = __ldcg(all + (static_cast<int64_t>(s2) * G + g) * PS + D);
            fac[g * (kMaxSplitsSmem / G) + s2] = (M == -INFINITY || ms == -INFINITY) ? 0.0f : __expf(ms - M);
        }
    }
    __syncthreads();
    for (int o = threadIdx.x; o < G * D; o += kAttnThreads) {
        const int g = o / D, d = o - g * D;
        const float* fg = fac + g * (kMaxSplitsSmem / G);
        float num = 0.0f, den = 0.0f;
#pragma unroll 8
        for (int s2 = 0; s2 < p.splits; s2++) {
            const float* pr = all + (static_cast<int64_t>(s2) * G + g) * PS;
            const float f = fg[s2];
            num = fmaf(f, __ldcg(pr + d), num);
            den = fmaf(f, __ldcg(pr + D + 1), den);
        }
        const float r = den > 0.0f ? num / den : 0.0f;  // no visible position: zeros
        const int64_t oi = (static_cast<int64_t>(b) * p.H + kvh * G + g) * D + d;
        if (p.out_bf16) static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(r);
        else static_cast<float*>(p.out)[oi] = r;
    }
    if (threadIdx.x == 0) p.counters[b * p.Hkv + kvh] = 0u;
}

// Appends t tokens of one kind (keys or values) per sequence to a bf16 cache:
// cache[b][start(b) + i][c][:] = bf16(src row (b * t + i), kv head c) for i < t,
// src rows src_row_stride elements apart, each [kv_heads, D] (fp32 or bf16).
// Eight elements a thread (one 16-byte store).
struct KvAppendParams {
    const void* src;
    int src_bf16;
    int64_t src_row_stride;
    uint16_t* cache;
    int64_t seq_stride;
    const int32_t* start;  // [B] first position to write, or null: start_all
    int start_all;
    int B, t, Hkv, D, kv_max;
    unsigned* err;
};

__global__ void kv_append_kernel(const KvAppendParams p) {
    pdl_wait();
    pdl_launch_dependents();
    const int per_row = p.Hkv * p.D / 8;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(p.B) * p.t * per_row) return;
    const int64_t row = i / per_row;
    const int c8 = static_cast<int>(i - row * per_row) * 8;
    const int b = static_cast<int>(row / p.t), ti = static_cast<int>(row - static_cast<int64_t>(b) * p.t);
    const int pos = (p.start ? __ldcg(p.start + b) : p.start_all) + ti;
    if (pos < 0 || pos >= p.kv_max) {
        record_error(p.err, ERR_ATTN_LEN);
        return;
    }
    float v[8];
    if (p.src_bf16) {
        const uint4 w = __ldcg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.src) + row * p.src_row_stride + c8));
        const unsigned ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
            v[2 * q] = __uint_as_float(ww[q] << 16);
            v[2 * q + 1] = __uint_as_float(ww[q] & 0xffff0000u);
        }
    } else {
        const float* sp = static_cast<const float*>(p.src) + row * p.src_row_stride + c8;
        const float4 a = __ldcg(reinterpret_cast<const float4*>(sp)), b4 = __ldcg(reinterpret_cast<const float4*>(sp) + 1);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b4.x, v[5] = b4.y, v[6] = b4.z, v[7] = b4.w;
    }
    uint4 o;
    unsigned* ow = reinterpret_cast<unsigned*>(&o);
#pragma unroll
    for (int q = 0; q < 4; q++) {
        __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * q], v[2 * q + 1]);
        ow[q] = *reinterpret_cast<unsigned*>(&h);
    }
    *reinterpret_cast<uint4*>(p.cache + static_cast<int64_t>(b) * p.seq_stride + static_cast<int64_t>(pos) * p.Hkv * p.D + c8) = o;
}

}  // namespace oomb
