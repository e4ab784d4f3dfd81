/*
 * oomb_oracle.h - CPU restatement of oom-inference's FP8 decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker the parity tests,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg compare the CUDA
 * path against.  The product (homelab_b200/liboomb.so) never links, loads or
 * calls it.
 *
 * Every function cites the reference file:line it restates.  Paths are
 * relative to projects/oom-inference/ in jomcgi-org/homelab.
 *
 * Parity pins (see tests/test_oracle.py and tests/test_ref_pin.py):
 *   - e4m3 codec and quantize_blocks: the known-answer tests of
 *     crates/oominf-core/src/fp8.rs:90-139 and
 *     crates/oominf-cpu/src/kernel.rs:531-539, byte for byte.
 *   - oo_gemv_fp8_reforder / oo_router_topk_ref: bit-exact (resp. id-exact)
 *     against the reference's own CUDA kernels (ops.cu gemv_fp8_t*, router_topk)
 *     compiled from source into oracle/_ref and run on a B200.
 */
#ifndef OOMB_ORACLE_H
#define OOMB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Scale layouts of a block-scaled FP8 matrix [n, k]. */
#define OO_SCALE_1X128 0   /* scale[r * ceil(k/128) + c/128]          (fp8.rs:46-88) */
#define OO_SCALE_128X128 1 /* scale[(r/128) * ceil(k/128) + c/128]                    */

/* ---- codecs ---------------------------------------------------------- */
uint8_t oo_e4m3_from_f32(float x);      /* fp8.rs:4-27 */
float oo_e4m3_to_f32(uint8_t b);        /* fp8.rs:29-43 (NaN codes read as 448) */
float oo_e4m3_to_f32_nan(uint8_t b);    /* oominf-cpu/src/kernel.rs:14-27 (NaN codes are NaN) */
uint16_t oo_bf16_from_f32(float v);     /* RNE, as crates/oominf-cuda/tests/gemv.rs:24-28 */
float oo_bf16_to_f32(uint16_t b);

/* ---- quantizer ------------------------------------------------------- */
/* fp8.rs:52-88 for layout 1x128 (byte-identical).  Layout 128x128 takes the
 * block's absolute maximum over the 2-D 128x128 block instead of a 1x128 row
 * segment; everything else (amax/448, 1 for an all-zero block, e4m3(w/scale))
 * is unchanged. */
void oo_quantize_blocks(const uint16_t* w_bf16, int64_t n, int64_t k, int layout, uint8_t* q,
                        float* scale);
int64_t oo_scale_count(int64_t n, int64_t k, int layout);
float oo_scale_at(const float* scale, int layout, int64_t k, int64_t r, int64_t c);

/* ---- dense GEMV ------------------------------------------------------ */
/* Truth: y[t, r] = sum_c x[t, c] * (e4m3(q[r, c]) * scale(r, c)), products and
 * sum in double; mag[t, r] = sum |x * w| (the reference's error scale,
 * crates/oominf-cuda/tests/moe_tiled.rs:190-211).  x is fp32 [t, k]. */
void oo_gemv_fp8_f64(const float* x, int64_t t, const uint8_t* q, const float* scale, int layout,
                     int64_t n, int64_t k, double* y, double* mag);

/* The reference's FP8 GEMV arithmetic in its exact fp32 order: gemv_impl<T,true>
 * (crates/oominf-cuda/kernels/ops.cu:338-440) under the split-K plan of
 * Gpu::gemv_at (crates/oominf-cuda/src/linear.rs:259-350), 1x128 scales,
 * t <= 4.  Per lane l: weights k0 + l*16 + 512*i, w = e4m3 * scale (fp32
 * multiply), acc = fma(x, w, acc); xor-shuffle tree over 32 lanes; per-split
 * partials summed in split order. */
void oo_gemv_fp8_reforder(const float* x, int64_t t, const uint8_t* q, const float* scale,
                          int64_t n, int64_t k, float* y);
/* The split plan gemv_at picks (linear.rs:270-287): returns splits, sets *klen. */
int64_t oo_gemv_ref_plan(int64_t t, int64_t n, int64_t k, int64_t* klen);

/* bf16 weights [n, k] (router), truth in double. */
void oo_gemv_bf16_f64(const float* x, int64_t t, const uint16_t* w, int64_t n, int64_t k,
                      double* y);

/* ---- router ---------------------------------------------------------- */
/* The exp shared by the oracle and the CUDA router: Cody-Waite reduction
 * x = n*ln2 + r (ln2 split into a 16-bit head and an fp32 tail), exp(r) by its
 * degree-7 Taylor polynomial in Horner form with fused multiply-adds, 2^n by
 * exponent construction.  Same source arithmetic as the device copy in
 * homelab_b200/csrc/oomb_math.cuh, so both give identical bits. */
float oo_expf(float x);

/* Canonical router logits (the order the CUDA router GEMV uses, so logits are
 * bit-identical): logit[t, e] = xor-tree over 32 lanes of the per-lane fma
 * chain over columns h = 256*i + 8*l + j (i ascending, j = 0..7).
 * x is fp32 [t, hdim] (bf16 inputs widened exactly), w bf16 [e, hdim]. */
void oo_router_logits(const float* x, int64_t t, const uint16_t* w, int64_t e, int64_t hdim,
                      float* logits);

/* Softmax over e logits, k rounds of argmax (ties to the lower id), weights
 * renormalised over the picks: ops.cu:230-294 / backend.rs:814-824, with the
 * canonical sum order of the CUDA router (32 lane partials, lane l summing
 * experts l, l+32, ... in order, then the xor tree) and oo_expf.  Bit-exact
 * with the CUDA router. */
void oo_router_topk(const float* logits, int64_t t, int64_t e, int64_t k, int32_t* ids,
                    float* weights);

/* ---- routed experts -------------------------------------------------- */
/* Grouping of a step's assignments by expert, in expert order, each expert's
 * slots in slot order: Moe::begin_routed (crates/oominf-models-qwen/src/moe.rs:
 * 532-582, all experts resident) and the meta table of finish_routed
 * (moe.rs:638-649).  Returns the number of active experts n_e and fills
 * active[n_e] (expert ids), off[n_e + 1], assign_tok[t*k], slot_assign[t*k].
 * Returns -1 if an id is out of range (moe.rs:545-547 bails). */
int64_t oo_group_assignments(const int32_t* ids, int64_t t, int64_t k, int64_t e, int32_t* active,
                             int32_t* off, int32_t* assign_tok, int32_t* slot_assign);

/* One FP8 expert record, all offsets in bytes from the record start.  gate/up
 * are [inter, hidden] (or fused [2*inter, hidden] with up = gate + inter rows),
 * down [hidden, inter], each with its own scales in `layout`. */
typedef struct {
    int64_t hidden, inter;
    int64_t gate_weight, gate_scale, up_weight, up_scale, down_weight, down_scale;
    int32_t layout;
    int32_t pad_;
} oo_fp8_record;

/* Expert FFN truth in double (moe.cu:52-151 structure, oominf-cpu/src/lib.rs:
 * 176-323): for assignment a of expert e (record recs[e]) and token tok(a):
 * g = x.Wg, u = x.Wu, h = silu(g) * u with silu(v) = v / (1 + exp(-v)),
 * y[a] = h . Wd.  Writes y [A, hidden] (double). */
void oo_moe_experts_f64(const uint8_t* const* recs, const oo_fp8_record* geo, const int32_t* off,
                        const int32_t* assign_tok, int64_t n_e, const float* x, double* y);

/* moe_combine_slots (moe.cu:155-164): out[t, c] = sum_s w[t, s] * y[slot_assign[t, s], c]
 * in slot order with fused multiply-adds, fp32 (bit-exact with the device). */
void oo_combine_slots(const float* y, const int32_t* slot_assign, const float* w, int64_t t,
                      int64_t h, int64_t k, float* out);
/* Same in double from double expert outputs (truth). */
void oo_combine_slots_f64(const double* y, const int32_t* slot_assign, const float* w, int64_t t,
                          int64_t h, int64_t k, double* out);

/* ---- deterministic generators --------------------------------------- */
/* splitmix64 stream; oo_fill_normal_bf16 draws N(mu, sigma) by Box-Muller and
 * rounds to bf16 (RNE).  Same seed, same bits, on every machine. */
void oo_fill_normal_bf16(uint64_t seed, float mu, float sigma, uint16_t* out, int64_t n);
void oo_fill_normal_f32(uint64_t seed, float mu, float sigma, float* out, int64_t n);

#ifdef __cplusplus
}
#endif
#endif
