/*
 * oomb_oracle.c - CPU restatement of oom-inference's FP8 decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path, never part of it.
 * Built with -ffp-contract=off so that every fused multiply-add below is an
 * explicit fmaf() and every other operation rounds on its own, as the CUDA
 * kernels it is compared against bit-for-bit do.
 *
 * References are to projects/oom-inference/ in jomcgi-org/homelab.
 */
#include "oomb_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------------- */
/* codecs                                                                  */
/* ---------------------------------------------------------------------- */

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* crates/oominf-core/src/fp8.rs:4-27: nearest e4m3 code, ties to even,
 * saturating at +-448 (0x7e / 0xfe); NaN saturates too. */
uint8_t oo_e4m3_from_f32(float x) {
    uint8_t sign = signbit(x) ? 0x80 : 0;
    float a = fabsf(x);
    if (isnan(a) || a >= 448.0f) return sign | 0x7e;
    if (a < ldexpf(1.0f, -6)) {
        /* subnormal: steps of 2^-9; 8 steps is the smallest normal, code 0x08 */
        return sign | (uint8_t)nearbyintf(a * 512.0f);
    }
    int e = (int)((f2u(a) >> 23) & 0xff) - 127;
    float m = nearbyintf((a / ldexpf(1.0f, e) - 1.0f) * 8.0f);
    int mi = (int)m;
    if (mi == 8) { mi = 0; e += 1; }
    int biased = e + 7;
    if (biased > 15 || (biased == 15 && mi == 7)) return sign | 0x7e;
    return sign | (uint8_t)(biased << 3) | (uint8_t)mi;
}

/* fp8.rs:29-43: exact value; 0x7f/0xff (NaN, never produced) read as 448. */
float oo_e4m3_to_f32(uint8_t b) {
    float s = (b & 0x80) ? -1.0f : 1.0f;
    int e = (b >> 3) & 0xf;
    float m = (float)(b & 7);
    float v;
    if (e == 0) v = m / 8.0f * ldexpf(1.0f, -6);
    else if (e == 15 && m == 7.0f) v = 448.0f;
    else v = (1.0f + m / 8.0f) * ldexpf(1.0f, e - 7);
    return s * v;
}

/* oominf-cpu/src/kernel.rs:14-27: as above but S.1111.111 is NaN. */
float oo_e4m3_to_f32_nan(uint8_t b) {
    if ((b & 0x7f) == 0x7f) return NAN;
    return oo_e4m3_to_f32(b);
}

/* Round to nearest even (crates/oominf-cuda/tests/gemv.rs:24-28); NaN kept quiet. */
uint16_t oo_bf16_from_f32(float v) {
    uint32_t b = f2u(v);
    if ((b & 0x7fffffff) > 0x7f800000) return (uint16_t)((b >> 16) | 0x40);
    return (uint16_t)((b + 0x7fff + ((b >> 16) & 1)) >> 16);
}

float oo_bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

/* ---------------------------------------------------------------------- */
/* quantizer                                                               */
/* ---------------------------------------------------------------------- */

#define OO_BLOCK 128 /* fp8.rs:46 */

int64_t oo_scale_count(int64_t n, int64_t k, int layout) {
    int64_t nb = (k + OO_BLOCK - 1) / OO_BLOCK;
    if (layout == OO_SCALE_128X128) return ((n + OO_BLOCK - 1) / OO_BLOCK) * nb;
    return n * nb;
}

float oo_scale_at(const float* scale, int layout, int64_t k, int64_t r, int64_t c) {
    int64_t nb = (k + OO_BLOCK - 1) / OO_BLOCK;
    int64_t row = layout == OO_SCALE_128X128 ? r / OO_BLOCK : r;
    return scale[row * nb + c / OO_BLOCK];
}

/* fp8.rs:52-88.  For 1x128 each (row, block) takes its own amax; for 128x128
 * the amax runs over the whole 2-D block.  scale = amax / 448 (1 when the block
 * is all zero), q = e4m3(w / scale) with an fp32 divide. */
void oo_quantize_blocks(const uint16_t* w, int64_t n, int64_t k, int layout, uint8_t* q,
                        float* scale) {
    int64_t nb = (k + OO_BLOCK - 1) / OO_BLOCK;
    int64_t rows_per = layout == OO_SCALE_128X128 ? OO_BLOCK : 1;
    int64_t nr = (n + rows_per - 1) / rows_per;
    for (int64_t br = 0; br < nr; br++) {
        int64_t r0 = br * rows_per, r1 = r0 + rows_per < n ? r0 + rows_per : n;
        for (int64_t b = 0; b < nb; b++) {
            int64_t c0 = b * OO_BLOCK, c1 = c0 + OO_BLOCK < k ? c0 + OO_BLOCK : k;
            float amax = 0.0f;
            for (int64_t r = r0; r < r1; r++)
                for (int64_t c = c0; c < c1; c++) {
                    float v = fabsf(oo_bf16_to_f32(w[r * k + c]));
                    /* f32::max ignores NaN (fp8.rs:74-77); fmaxf does the same. */
                    amax = fmaxf(amax, v);
                }
            float s = amax > 0.0f ? amax / 448.0f : 1.0f;
            scale[br * nb + b] = s;
            for (int64_t r = r0; r < r1; r++)
                for (int64_t c = c0; c < c1; c++)
                    q[r * k + c] = oo_e4m3_from_f32(oo_bf16_to_f32(w[r * k + c]) / s);
        }
    }
}

/* ---------------------------------------------------------------------- */
/* GEMV                                                                    */
/* ---------------------------------------------------------------------- */

void oo_gemv_fp8_f64(const float* x, int64_t t, const uint8_t* q, const float* scale, int layout,
                     int64_t n, int64_t k, double* y, double* mag) {
    for (int64_t r = 0; r < n; r++) {
        for (int64_t tt = 0; tt < t; tt++) {
            double s = 0.0, m = 0.0;
            for (int64_t c = 0; c < k; c++) {
                double w = (double)oo_e4m3_to_f32(q[r * k + c]) *
                           (double)oo_scale_at(scale, layout, k, r, c);
                double p = (double)x[tt * k + c] * w;
                s += p;
                m += fabs(p);
            }
            y[tt * n + r] = s;
            if (mag) mag[tt * n + r] = m;
        }
    }
}

/* linear.rs:259-290: GEMV_R=4 rows per warp, step 512 (FP8), want = ceil(2048 /
 * row_groups) clamped to [1, kchunks], smem_min = ceil(tp*k*4 / 48 KiB),
 * klen = ceil(ceil(k / splits0) / 512) * 512, splits = ceil(k / klen). */
int64_t oo_gemv_ref_plan(int64_t t, int64_t n, int64_t k, int64_t* klen) {
    const int64_t step = 512, smem = 48 * 1024;
    int64_t row_groups = (n + 3) / 4;
    int64_t kchunks = (k + step - 1) / step;
    int64_t tp = t <= 4 ? t : (t <= 8 ? 8 : 16);
    int64_t want = (2048 + row_groups - 1) / row_groups;
    if (want < 1) want = 1;
    if (want > kchunks) want = kchunks;
    int64_t smem_min = (tp * k * 4 + smem - 1) / smem;
    int64_t s0 = want > smem_min ? want : smem_min;
    if (s0 > kchunks) s0 = kchunks;
    int64_t kl = ((k + s0 - 1) / s0 + step - 1) / step * step;
    *klen = kl;
    return (k + kl - 1) / kl;
}

static float xor_tree32(float v[32]) {
    for (int o = 16; o > 0; o >>= 1) {
        float nv[32];
        for (int l = 0; l < 32; l++) nv[l] = v[l] + v[l ^ o];
        memcpy(v, nv, sizeof(nv));
    }
    return v[0];
}

/* ops.cu:338-440 (FP8 branch) under the plan above.  Lane l of the warp owning
 * row r covers kb = l*16 + 512*i inside the split's range; per 16-byte load it
 * decodes 16 weights, multiplies each by the block scale (an fp32 multiply,
 * ops.cu:382-383) and accumulates acc += x * w (contracted to an fma by nvcc,
 * ops.cu:399).  The warp sum is the xor-shuffle tree (ops.cu:402-406); split
 * partials are summed in split order starting from 0 (ops.cu:435-437). */
void oo_gemv_fp8_reforder(const float* x, int64_t t, const uint8_t* q, const float* scale,
                          int64_t n, int64_t k, float* y) {
    int64_t klen;
    int64_t splits = oo_gemv_ref_plan(t, n, k, &klen);
    int64_t nbk = (k + OO_BLOCK - 1) / OO_BLOCK;
    float* part = (float*)malloc(sizeof(float) * (size_t)splits);
    for (int64_t r = 0; r < n; r++) {
        for (int64_t tt = 0; tt < t; tt++) {
            for (int64_t s = 0; s < splits; s++) {
                int64_t k0 = s * klen;
                int64_t k1 = k0 + klen < k ? k0 + klen : k;
                int64_t kl = k1 - k0;
                float lanes[32];
                for (int l = 0; l < 32; l++) {
                    float acc = 0.0f;
                    for (int64_t kb = (int64_t)l * 16; kb < kl; kb += 512) {
                        float sc = scale[r * nbk + (k0 + kb) / OO_BLOCK];
                        for (int i = 0; i < 16; i++) {
                            float w = oo_e4m3_to_f32(q[r * k + k0 + kb + i]) * sc;
                            acc = fmaf(x[tt * k + k0 + kb + i], w, acc);
                        }
                    }
                    lanes[l] = acc;
                }
                part[s] = xor_tree32(lanes);
            }
            if (splits == 1) {
                y[tt * n + r] = part[0];
            } else {
                float sum = 0.0f;
                for (int64_t s = 0; s < splits; s++) sum += part[s];
                y[tt * n + r] = sum;
            }
        }
    }
    free(part);
}

void oo_gemv_bf16_f64(const float* x, int64_t t, const uint16_t* w, int64_t n, int64_t k,
                      double* y) {
    for (int64_t r = 0; r < n; r++)
        for (int64_t tt = 0; tt < t; tt++) {
            double s = 0.0;
            for (int64_t c = 0; c < k; c++)
                s += (double)x[tt * k + c] * (double)oo_bf16_to_f32(w[r * k + c]);
            y[tt * n + r] = s;
        }
}

/* ---------------------------------------------------------------------- */
/* router                                                                  */
/* ---------------------------------------------------------------------- */

/* Cody & Waite (1980) argument reduction with ln2 = LN2_HI + LN2_LO, LN2_HI
 * holding 16 significant bits so n * LN2_HI is exact for |n| < 2^8; exp(r) on
 * |r| <= ln2/2 by the Taylor series to degree 7 (truncation < 6e-9 relative,
 * under a tenth of an fp32 ulp) in Horner form; 2^n applied in two exact
 * power-of-two steps so results that land in the subnormal range round once.
 * Inputs below -104 give 0 and above 88.5 give +inf. */
#define OO_LOG2E 1.44269504088896341f
#define OO_LN2_HI 0.693145751953125f          /* 0x3f317200 */
#define OO_LN2_LO 1.42860682030941723212e-6f  /* ln2 - LN2_HI */
float oo_expf(float x) {
    if (x != x) return x;
    if (x < -104.0f) return 0.0f;
    if (x > 88.5f) return INFINITY;
    float n = nearbyintf(x * OO_LOG2E);
    float r = fmaf(-n, OO_LN2_HI, x);
    r = fmaf(-n, OO_LN2_LO, r);
    float p = 1.98412698412698413e-4f; /* 1/5040 */
    p = fmaf(p, r, 1.38888888888888889e-3f); /* 1/720 */
    p = fmaf(p, r, 8.33333333333333333e-3f); /* 1/120 */
    p = fmaf(p, r, 4.16666666666666667e-2f); /* 1/24 */
    p = fmaf(p, r, 1.66666666666666667e-1f); /* 1/6 */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;
    int n1 = ni / 2, n2 = ni - n1;
    float s1 = u2f((uint32_t)(n1 + 127) << 23);
    float s2 = u2f((uint32_t)(n2 + 127) << 23);
    return (p * s1) * s2;
}

void oo_router_logits(const float* x, int64_t t, const uint16_t* w, int64_t e, int64_t hdim,
                      float* logits) {
    for (int64_t tt = 0; tt < t; tt++)
        for (int64_t r = 0; r < e; r++) {
            float lanes[32];
            for (int l = 0; l < 32; l++) {
                float acc = 0.0f;
                for (int64_t base = (int64_t)l * 8; base < hdim; base += 256)
                    for (int j = 0; j < 8; j++)
                        acc = fmaf(x[tt * hdim + base + j], oo_bf16_to_f32(w[r * hdim + base + j]),
                                   acc);
                lanes[l] = acc;
            }
            logits[tt * e + r] = xor_tree32(lanes);
        }
}

/* ops.cu:230-294 with the canonical sum order: max over all logits (exact),
 * p_unnorm[i] = exp(l[i] - max), sum = xor tree of 32 lane partials where lane
 * l adds i = l, l+32, ... in order, p[i] = p_unnorm[i] / sum; k rounds pick the
 * largest p, ties to the lower id; weights = p / (p_0 + p_1 + ... in pick order). */
void oo_router_topk(const float* logits, int64_t t, int64_t e, int64_t k, int32_t* ids,
                    float* weights) {
    float* p = (float*)malloc(sizeof(float) * (size_t)e);
    float* chosen_p = (float*)malloc(sizeof(float) * (size_t)k);
    for (int64_t tt = 0; tt < t; tt++) {
        const float* l = logits + tt * e;
        float mx = -INFINITY;
        for (int64_t i = 0; i < e; i++) mx = fmaxf(mx, l[i]);
        float lanes[32];
        for (int ln = 0; ln < 32; ln++) {
            float s = 0.0f;
            for (int64_t i = ln; i < e; i += 32) s += oo_expf(l[i] - mx);
            lanes[ln] = s;
        }
        float sum = xor_tree32(lanes);
        for (int64_t i = 0; i < e; i++) p[i] = oo_expf(l[i] - mx) / sum;
        for (int64_t r = 0; r < k; r++) {
            float bv = -3.0f;
            int64_t bi = 0x7fffffff;
            for (int64_t i = 0; i < e; i++)
                if (p[i] > bv || (p[i] == bv && i < bi)) { bv = p[i]; bi = i; }
            ids[tt * k + r] = (int32_t)bi;
            chosen_p[r] = bv;
            p[bi] = -2.0f; /* used entries sit below every probability (ops.cu:279-281) */
        }
        float ps = 0.0f;
        for (int64_t r = 0; r < k; r++) ps += chosen_p[r];
        for (int64_t r = 0; r < k; r++) weights[tt * k + r] = chosen_p[r] / ps;
    }
    free(p);
    free(chosen_p);
}

/* ---------------------------------------------------------------------- */
/* routed experts                                                          */
/* ---------------------------------------------------------------------- */

int64_t oo_group_assignments(const int32_t* ids, int64_t t, int64_t k, int64_t e, int32_t* active,
                             int32_t* off, int32_t* assign_tok, int32_t* slot_assign) {
    int64_t a_total = t * k;
    int32_t* count = (int32_t*)calloc((size_t)e, sizeof(int32_t));
    for (int64_t s = 0; s < a_total; s++) {
        if (ids[s] < 0 || ids[s] >= e) { free(count); return -1; }
        count[ids[s]]++;
    }
    int64_t n_e = 0, a = 0;
    for (int64_t ex = 0; ex < e; ex++) {
        if (!count[ex]) continue;
        active[n_e] = (int32_t)ex;
        off[n_e] = (int32_t)a;
        for (int64_t s = 0; s < a_total; s++)
            if (ids[s] == ex) {
                assign_tok[a] = (int32_t)(s / k);
                slot_assign[s] = (int32_t)a;
                a++;
            }
        n_e++;
    }
    off[n_e] = (int32_t)a;
    free(count);
    return n_e;
}

static double rec_weight(const uint8_t* rec, int64_t w_off, int64_t s_off, int layout, int64_t k,
                         int64_t r, int64_t c) {
    const uint8_t* q = rec + w_off;
    const float* sc = (const float*)(rec + s_off);
    return (double)oo_e4m3_to_f32(q[r * k + c]) * (double)oo_scale_at(sc, layout, k, r, c);
}

void oo_moe_experts_f64(const uint8_t* const* recs, const oo_fp8_record* geo, const int32_t* off,
                        const int32_t* assign_tok, int64_t n_e, const float* x, double* y) {
    int64_t H = geo->hidden, I = geo->inter;
    double* h = (double*)malloc(sizeof(double) * (size_t)I);
    for (int64_t ei = 0; ei < n_e; ei++) {
        const uint8_t* rec = recs[ei];
        for (int64_t a = off[ei]; a < off[ei + 1]; a++) {
            const float* xr = x + (int64_t)assign_tok[a] * H;
            for (int64_t j = 0; j < I; j++) {
                double g = 0.0, u = 0.0;
                for (int64_t c = 0; c < H; c++) {
                    g += (double)xr[c] *
                         rec_weight(rec, geo->gate_weight, geo->gate_scale, geo->layout, H, j, c);
                    u += (double)xr[c] *
                         rec_weight(rec, geo->up_weight, geo->up_scale, geo->layout, H, j, c);
                }
                h[j] = g / (1.0 + exp(-g)) * u;
            }
            for (int64_t r = 0; r < H; r++) {
                double s = 0.0;
                for (int64_t j = 0; j < I; j++)
                    s += h[j] *
                         rec_weight(rec, geo->down_weight, geo->down_scale, geo->layout, I, r, j);
                y[a * H + r] = s;
            }
        }
    }
    free(h);
}

void oo_combine_slots(const float* y, const int32_t* slot_assign, const float* w, int64_t t,
                      int64_t h, int64_t k, float* out) {
    for (int64_t tt = 0; tt < t; tt++)
        for (int64_t c = 0; c < h; c++) {
            float acc = 0.0f;
            for (int64_t s = 0; s < k; s++)
                acc = fmaf(w[tt * k + s], y[(int64_t)slot_assign[tt * k + s] * h + c], acc);
            out[tt * h + c] = acc;
        }
}

void oo_combine_slots_f64(const double* y, const int32_t* slot_assign, const float* w, int64_t t,
                          int64_t h, int64_t k, double* out) {
    for (int64_t tt = 0; tt < t; tt++)
        for (int64_t c = 0; c < h; c++) {
            double acc = 0.0;
            for (int64_t s = 0; s < k; s++)
                acc += (double)w[tt * k + s] * y[(int64_t)slot_assign[tt * k + s] * h + c];
            out[tt * h + c] = acc;
        }
}

/* ---------------------------------------------------------------------- */
/* generators                                                              */
/* ---------------------------------------------------------------------- */

static uint64_t splitmix64(uint64_t* s) {
    uint64_t z = (*s += 0x9e3779b97f4a7c15ULL);
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

static void normals(uint64_t seed, float mu, float sigma, float* out, int64_t n) {
    uint64_t s = seed;
    for (int64_t i = 0; i < n; i += 2) {
        double u1 = ((splitmix64(&s) >> 11) + 1) * (1.0 / 9007199254740993.0);
        double u2 = (splitmix64(&s) >> 11) * (1.0 / 9007199254740992.0);
        double rr = sqrt(-2.0 * log(u1));
        out[i] = (float)(mu + sigma * rr * cos(6.283185307179586 * u2));
        if (i + 1 < n) out[i + 1] = (float)(mu + sigma * rr * sin(6.283185307179586 * u2));
    }
}

void oo_fill_normal_f32(uint64_t seed, float mu, float sigma, float* out, int64_t n) {
    normals(seed, mu, sigma, out, n);
}

void oo_fill_normal_bf16(uint64_t seed, float mu, float sigma, uint16_t* out, int64_t n) {
    float* tmp = (float*)malloc(sizeof(float) * (size_t)n);
    normals(seed, mu, sigma, tmp, n);
    for (int64_t i = 0; i < n; i++) out[i] = oo_bf16_from_f32(tmp[i]);
    free(tmp);
}
