/*
 * oomb.h - C ABI of the B200 (sm_100a) FP8 decode path of oom-inference.
 *
 * Each entry point replaces the launch body of one method of the engine's
 * Rust backend traits (projects/oom-inference/crates/oominf-core/src/backend.rs),
 * cited beside it.  Conventions, as in the reference backend:
 *   - every call is stream-ordered on the `stream` it is given and enqueues no
 *     implicit synchronisation; host reads of results sync through the stream;
 *   - the caller owns every device buffer (inputs, outputs, workspace); the
 *     library allocates nothing on the call path;
 *   - shapes and alignment are checked before launch, as Gpu::check does
 *     (crates/oominf-cuda/src/lib.rs:157-160): an unsupported shape returns
 *     OOMB_E_SHAPE / OOMB_E_ALIGN and launches nothing;
 *   - device pointers are plain addresses; the library needs the CUDA
 *     runtime and an sm_100a device, and fails loudly (OOMB_E_DEVICE) elsewhere.
 * Device-side waits are bounded: a wait that runs out records a code readable
 * with oomb_device_error() and the kernel returns instead of hanging.
 */
#ifndef OOMB_H
#define OOMB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A cudaStream_t (0 = the legacy default stream). */
typedef struct CUstream_st* oomb_stream;

/* Status codes (0 = success). */
#define OOMB_OK 0
#define OOMB_E_SHAPE (-1)     /* "buffer too small or shape unsupported" (lib.rs:157-160) */
#define OOMB_E_ALIGN (-2)     /* a pointer or stride is not 16-byte aligned */
#define OOMB_E_LAUNCH (-3)    /* the CUDA launch failed */
#define OOMB_E_TIMEOUT (-4)   /* a bounded device wait ran out (see oomb_device_error) */
#define OOMB_E_ARG (-5)       /* null pointer or bad enum */
#define OOMB_E_DEVICE (-6)    /* no usable sm_100 device */
#define OOMB_E_WORKSPACE (-7) /* workspace smaller than the *_workspace_bytes figure */

/* Flags of the expert entry points.  OOMB_TABLES_READY: recs, off and
 * assign_tok were written before the kernel preceding this call in the stream
 * started (by the host, or earlier), so the kernel may read them and start
 * streaming weights before that kernel finishes. */
#define OOMB_TABLES_READY 1

/* Element types of activations and outputs. */
#define OOMB_F32 0
#define OOMB_BF16 1

/* Scale layouts of a block-scaled FP8 e4m3 matrix q[n, k] (row-major):
 *   OOMB_SCALE_1X128:   w[r, c] = scale[r * ceil(k/128) + c/128] * e4m3(q[r, c])
 *                       (Weight::Fp8, backend.rs:162-170; fp8.rs:46-88)
 *   OOMB_SCALE_128X128: w[r, c] = scale[(r/128) * ceil(k/128) + c/128] * e4m3(q[r, c]) */
#define OOMB_SCALE_1X128 0
#define OOMB_SCALE_128X128 1

/* Byte layout of an FP8 expert record (layout tag "fp8-e4m3-b128x128" or
 * "fp8-e4m3-b1x128"), the FP8 counterpart of Nvfp4Record / Bf16Record
 * (backend.rs:783-807): gate and up e4m3 [inter, hidden], down e4m3
 * [hidden, inter], each with its own fp32 scales in `layout`.  Offsets are in
 * bytes from the record start and must be multiples of 16.  The record format
 * of experts.bin (docs/dev/format.md:37-76): parts at OOMB_PART_ALIGN offsets
 * in the order gate.weight, up.weight, down.weight, gate.weight_scale,
 * up.weight_scale, down.weight_scale, the stride rounded up to
 * OOMB_RECORD_ALIGN (oomb_fp8_record_layout computes it). */
#define OOMB_PART_ALIGN 256
#define OOMB_RECORD_ALIGN 4096
typedef struct {
    int64_t hidden;
    int64_t inter;
    int64_t gate_weight, gate_scale;
    int64_t up_weight, up_scale;
    int64_t down_weight, down_scale;
    int32_t layout;
    int32_t pad_;
} oomb_fp8_record;

/* A resident MoE layer for the fused decode path: the bf16 router [experts,
 * hidden] (routers stay bf16, crates/oominf-models-qwen/src/util.rs:48-60)
 * and one device record address per expert. */
typedef struct {
    int32_t hidden;
    int32_t experts;
    int32_t top_k;
    int32_t pad_;
    const uint16_t* router_w;
    const uint64_t* recs;
    oomb_fp8_record geo;
} oomb_moe_layer;

/* ---- library -------------------------------------------------------- */
const char* oomb_version(void);
const char* oomb_status_string(int status);
/* The first bounded-wait failure recorded on the current device since the
 * last clear (0 if none); `clear` != 0 resets it, and then also zeroes the
 * sync words of the no-alloc decode's fixed scratch on this device (see
 * oomb_moe_decode_fp8_noalloc).  Synchronises the device.  No counterpart in
 * the reference, whose kernels never wait on one another. */
int oomb_device_error(int* code, int clear);
/* Sets how long a bounded device wait polls before it gives up and records
 * its code, in nanoseconds, on the current device (0 restores the default of
 * 2 s).  Takes effect for kernels launched after it returns.  A diagnostic
 * knob: a short limit makes a wait that nothing will satisfy (a peer that
 * never raises its flag) end within milliseconds, so the failure path can be
 * exercised without hanging anything.  No counterpart in the reference. */
int oomb_set_wait_limit(uint64_t ns);

/* ---- Linear ------------------------------------------------------------ */
/* y[t, n] = x[t, k] . W[n, k]^T for FP8 e4m3 W with block scales, fp32
 * accumulation.  Replaces Linear::gemm_fp8 (backend.rs:199-209; launch body
 * Gpu::gemm_fp8 / gemv / gemv_at, crates/oominf-cuda/src/linear.rs:35-81,
 * 223-350).  x and y are fp32 or bf16.  k % 16 == 0; q, scale, x and y
 * 16-byte aligned.  One launch streams the weights once for all t tokens
 * (CUDA cores; t <= 16 is the decode/verify range of linear.rs:131-134); for
 * k > 4096 tokens go in launches of 2.  Workspace: optional.  With t >= 2 and a
 * workspace of at least oomb_gemm_fp8_workspace_bytes(t, n, k, x_dtype) bytes
 * (zeroed once), shapes the tensor-core path takes (n, k multiples of 128,
 * t <= 64) run there instead (oomb_gemm_fp8_tc); otherwise pass NULL, 0. */
int oomb_gemm_fp8(const void* x, int x_dtype, const uint8_t* q, const float* scale,
                  int scale_layout, void* y, int y_dtype, int t, int n, int k, void* workspace,
                  size_t workspace_bytes, oomb_stream stream);

/* The same product on the tensor cores (tcgen05, kind::f8f6f4): the weights go
 * from HBM to shared memory by TMA and straight into the MMA.  A first small
 * kernel splits x once into e4m3 terms with power-of-two scales per 128-column
 * block (two terms for bf16 x, exact; six for fp32 x, which keep every value
 * to within 2^-24 of its block's largest magnitude: 24 significant bits) into
 * the workspace; the terms form the MMA's B operand, and the per-block weight
 * and term scales are applied in fp32 as each 128-column block completes.
 * Needs n % 128 == 0, k % 128 == 0, 1 <= t <= 64 (bf16 x) or <= 32 (fp32 x),
 * and a workspace of oomb_gemm_fp8_workspace_bytes(t, n, k, x_dtype) bytes
 * (split-K partial sums, self-resetting counters, the split activations)
 * zeroed once before first use.  Returns OOMB_E_SHAPE for other shapes (use
 * oomb_gemm_fp8).  Calls sharing a workspace must be ordered on one stream. */
#define OOMB_Q_ROWS 0  /* q row-major [n, k] (Weight::Fp8) */
#define OOMB_Q_TILES 1 /* q in the packed tile layout of oomb_pack_fp8_tiles */
size_t oomb_gemm_fp8_workspace_bytes(int t, int n, int k, int x_dtype);
int oomb_gemm_fp8_tc(const void* x, int x_dtype, const uint8_t* q, int q_format, const float* scale,
                     int scale_layout, void* y, int y_dtype, int t, int n, int k, void* workspace,
                     size_t workspace_bytes, oomb_stream stream);

/* SwiGLU on stacked rows: y[r, i] = silu(gu[r, i]) * gu[r, n + i] with
 * silu(v) = v / (1 + exp(-v)); gu fp32 [rows, 2n], y fp32 or bf16 [rows, n],
 * n % 4 == 0.  The reference's silu_mul_rows (ops.cu:302-309), used between
 * the fused gate/up projection and the down projection of a dense MLP. */
int oomb_silu_mul_rows(const float* gu, void* y, int y_dtype, int rows, int n, oomb_stream stream);

/* Load-time repack of a row-major e4m3 matrix q [n, k] (n, k multiples of 128)
 * into 128 x 128-byte tiles, tile (rb, kb) contiguous at (rb * k/128 + kb) *
 * 16 KiB: the tensor-core path then streams each tile as one contiguous 16 KiB
 * read instead of 128 rows of 128 bytes.  tiles: n * k bytes. */
int oomb_pack_fp8_tiles(const uint8_t* q, int n, int k, uint8_t* tiles, oomb_stream stream);

/* logits[t, e] = x[t, :] . W[e, :] for a bf16 router W [e, hidden], in the
 * canonical order the oracle restates bit for bit (fp32 fma per lane over
 * columns 256*i + 8*lane + j, xor-tree over 32 lanes).  The router GEMV of
 * Moe::forward (crates/oominf-models-qwen/src/moe.rs:289-298). */
int oomb_router_logits(const void* x, int x_dtype, const uint16_t* w, float* logits, int t,
                       int e, int hidden, oomb_stream stream);

/* ---- Experts ------------------------------------------------------------ */
/* Softmax over e logits per row, top k (ties to the lower id), weights
 * renormalised over the picks.  Replaces Experts::router_topk (backend.rs:
 * 816-824; crates/oominf-cuda/src/experts.rs:10-38; ops.cu:234-294).
 * k <= 32, k <= e <= 8192. */
int oomb_router_topk(const float* logits, int32_t* ids, float* weights, int t, int e, int k,
                     oomb_stream stream);

/* h[a, :] = silu(x[tok(a)] . Wg^T) * (x[tok(a)] . Wu^T) for every assignment a
 * of the n_experts groups: expert i owns assignments [off[i], off[i+1]) and
 * its record is at recs[i]; tok(a) = assign_tok[a].  Replaces
 * Experts::moe_gate_up (backend.rs:827-836; experts.rs:43-93; moe.cu:55-106)
 * for FP8 records.  x: [*, hidden] fp32 or bf16; h: [A, inter] fp32.
 * hidden <= 4096, hidden % 16 == 0, inter % 16 == 0.  max_per_expert: the
 * largest assignment count of any group (Moe::run_group computes it for
 * moe_tiled, moe.rs:739-740), or 0 if unknown; 1 selects the fastest path.
 * flags: 0 or OOMB_TABLES_READY. */
int oomb_moe_gate_up_fp8(const uint64_t* recs, const int32_t* off, const int32_t* assign_tok,
                         int n_experts, const void* x, int x_dtype, float* h,
                         const oomb_fp8_record* geo, int max_per_expert, int flags,
                         oomb_stream stream);

/* y[a, :] = h[a, :] . Wd^T for every assignment.  Replaces Experts::moe_down
 * (backend.rs:860-868; experts.rs:174-209; moe.cu:110-151).  inter <= 4096;
 * max_per_expert and flags as for oomb_moe_gate_up_fp8. */
int oomb_moe_down_fp8(const uint64_t* recs, const int32_t* off, int n_experts, const float* h,
                      float* y, const oomb_fp8_record* geo, int max_per_expert, int flags,
                      oomb_stream stream);

/* out[t, c] = sum_s w[t, s] * y[slot_assign[t, s], c], summed in slot order
 * with fused multiply-adds (deterministic).  Replaces Experts::moe_combine_slots
 * (backend.rs:898-907; experts.rs:303-329; moe.cu:155-164).  out fp32 or bf16. */
int oomb_moe_combine_slots(const float* y, const int32_t* slot_assign, const float* w, void* out,
                           int out_dtype, int t, int h, int k, oomb_stream stream);

/* out = routed + sigmoid(gate_logit[t]) * shared.  Replaces Experts::moe_combine
 * (backend.rs:909-917; ops.cu:311-316).  All fp32 [t, h]; gate_logit [t]. */
int oomb_moe_combine(const float* routed, const float* shared, const float* gate_logit,
                     float* out, int t, int h, oomb_stream stream);

/* Grouped FP8 expert GEMM on the tensor cores (tcgen05) for large steps:
 * y[a, :] = x[row(a), :] . W_e^T for every assignment a of group e (a in
 * [off[e], off[e+1])), row(a) = rows[a], or a when rows is NULL; W_e the e4m3
 * matrix [n, k] at byte offset w_off of record recs[e], its fp32 block scales
 * (scale_layout) at s_off.  Replaces Experts::moe_tiled (backend.rs:873-886;
 * crates/oominf-cuda/src/experts.rs:211-266; moe.cu:204-335) for FP8 records:
 * the projection (w_off, s_off, s2_idx) becomes (w_off, s_off, scale_layout),
 * and the result is the Exact precision's: every activation row is split once
 * into e4m3 terms (bf16 x: two terms, exact; fp32 x: six terms, 24 significant
 * bits of each 128-column block, as the reference's three exact bf16 terms),
 * fp32 accumulate.  x: [*, k] fp32 or bf16; y: [A, n] fp32.  n, k multiples of
 * 128; n_experts <= 4096; w_off % 16 == 0.  max_per_expert picks the chunk size
 * (assignments per MMA, <= 64 for bf16 x and <= 32 for fp32 x); any group size
 * is correct, 0 if unknown.  max_assignments bounds A = off[n_experts] (it is
 * read on the device) and sizes the workspace: at least
 * oomb_moe_tiled_fp8_workspace_bytes(max_assignments, k, x_dtype) bytes, which
 * hold the split activations (no zeroing needed).  Calls sharing a workspace
 * must be ordered on one stream. */
size_t oomb_moe_tiled_fp8_workspace_bytes(int max_assignments, int k, int x_dtype);
int oomb_moe_tiled_fp8(const uint64_t* recs, const int32_t* off, const int32_t* rows, int n_experts,
                       int max_per_expert, int max_assignments, const void* x, int x_dtype, float* y, int n,
                       int k, int64_t w_off, int64_t s_off, int scale_layout, void* workspace,
                       size_t workspace_bytes, oomb_stream stream);

/* h[i] = silu(g[i]) * u[i] for i in [start, end), silu(v) = v / (1 + exp(-v)).
 * Replaces Experts::moe_swiglu_range (backend.rs; experts.rs:269-297;
 * moe.cu:337-341), the step between the tiled gate/up and down projections. */
int oomb_moe_swiglu_range(const float* g, const float* u, float* h, int64_t start, int64_t end,
                          oomb_stream stream);

/* ---- decode attention ------------------------------------------------------ */
/* Grouped-query attention of one query token per sequence over a bf16 KV
 * cache (flash-decode, split over the positions, merged in the same launch):
 *   out[b, h, :] = sum_j softmax_j(scale * q[b, h, :] . K[b, j, h / G, :]) V[b, j, h / G, :]
 * for j < kv_len[b], G = heads / kv_heads, fp32 softmax and accumulation.  The
 * decode case of Attention::attention (backend.rs:551-568; reference kernels
 * attn_decode_partial_g12 + attn_decode_combine, crates/oominf-cuda/kernels/
 * attention.cu:592-700) with a bf16 cache (a KvFormat beside the reference's
 * fp32 one) and every position below kv_len visible (the causal mask of a
 * decode step).  q, out: [batch, heads, head_dim] (fp32 or bf16).  Cache:
 * sequence b at b * seq_stride elements of k_cache / v_cache, row j of kv head
 * c at (j * kv_heads + c) * head_dim elements (the reference's row layout),
 * rows 0 .. kv_max - 1 allocated.  kv_len: device int32 [batch], or NULL to
 * use kv_len_all for every sequence; a sequence with no visible position gets
 * zeros.  head_dim 128; G in {1, 2, 4, 8}.  Workspace: at least
 * oomb_attention_decode_workspace_bytes(...) bytes (partials and self-resetting
 * arrival counters) zeroed once before first use; calls sharing it must be
 * ordered on one stream. */
size_t oomb_attention_decode_workspace_bytes(int batch, int heads, int kv_heads, int head_dim, int kv_max);
int oomb_attention_decode(const void* q, int q_dtype, const uint16_t* k_cache, const uint16_t* v_cache,
                          int64_t seq_stride, const int32_t* kv_len, int kv_len_all, void* out, int out_dtype,
                          int batch, int heads, int kv_heads, int head_dim, int kv_max, float scale,
                          void* workspace, size_t workspace_bytes, oomb_stream stream);

/* Appends t tokens of keys (or values) per sequence to a bf16 cache laid out as
 * oomb_attention_decode reads it: cache[b][start[b] + i][c][:] = bf16 of source
 * row b * t + i, kv head c, i < t.  Source rows (fp32 or bf16, [kv_heads,
 * head_dim] each) are src_row_stride elements apart, so keys and values can be
 * read straight out of a fused projection's output.  start: device int32
 * [batch] (the sequences' lengths before the step), or NULL for start_all.
 * Attention::kv_append (backend.rs:518-531) for a bf16 cache, batched over
 * sequences.  Positions outside [0, kv_max) are skipped and recorded in the
 * device error word. */
int oomb_kv_append(const void* src, int src_dtype, int64_t src_row_stride, uint16_t* cache, int64_t seq_stride,
                   const int32_t* start, int start_all, int batch, int t, int kv_heads, int head_dim, int kv_max,
                   oomb_stream stream);

/* ---- fused decode step of one resident MoE layer ------------------------ */
/* Router GEMV, softmax top-k, grouping of the step's assignments by expert
 * (expert order, slots in slot order: Moe::begin_routed / finish_routed,
 * moe.rs:532-582, 638-659), gate/up+SiLU, down and the slot-order combine, as
 * one stream-ordered sequence of kernels with no host round trip.  Same
 * results as calling the separate entry points in that order.
 *   x: [t, hidden] (x_dtype); out: [t, hidden] (out_dtype);
 *   ids, weights: optional [t, top_k] copies of the routing (NULL to skip).
 * x and out may be pinned host memory (cudaHostAlloc / cudaHostRegister): the
 * step then reads x over the bus into the workspace with one small kernel
 * after the stream's previous work, and stores out straight into host memory,
 * with no separate copies; pageable host memory is refused (OOMB_E_ARG).  The
 * workspace, ids and weights are device memory.
 * The workspace must hold oomb_moe_decode_workspace_bytes(t, layer) bytes and
 * be zeroed once before first use (oomb_workspace_clear), and again after a
 * device error (oomb_device_error); calls that share a workspace must be
 * ordered on one stream.  Paths: up to 16 tokens (up to 256 experts) the step
 * is one persistent launch on the CUDA cores (from 2 tokens every slot streams
 * as a group of its own); from 17 tokens, when hidden and
 * intermediate are multiples of 128 and hidden >= 2 * intermediate, it is the
 * grouped tensor-core path (route, the token rows split once into e4m3 terms,
 * gate and up, SwiGLU, down, combine: the same bits as oomb_moe_tiled_fp8 for
 * gate, up and down, oomb_moe_swiglu_range and oomb_moe_combine_slots on the
 * same routing); otherwise the chain of CUDA-core kernels.  The environment
 * variable OOMB_DECODE_CHAIN=1 selects the CUDA-core chain for every batch
 * (the bits of the one-launch step and of the expert-parallel ranks), and
 * OOMB_DECODE_TILED_MIN_T=n moves the tensor-core threshold to n tokens. */
size_t oomb_moe_decode_workspace_bytes(int t, const oomb_moe_layer* layer);
int oomb_moe_decode_fp8(const oomb_moe_layer* layer, const void* x, int x_dtype, int t, void* out,
                        int out_dtype, int32_t* ids, float* weights, void* workspace,
                        size_t workspace_bytes, oomb_stream stream);
int oomb_workspace_clear(void* workspace, size_t bytes, oomb_stream stream);

/* ---- a whole MoE layer: shared expert(s) + routed experts ----------------- */
/* The shared expert(s) of a layer in FP8: all shared experts side by side as
 * one SwiGLU MLP of width `inter` (gate rows then up rows of gate_up_q
 * [2 * inter, hidden], down_q [hidden, inter], block scales in scale_layout),
 * and the bf16 gate-logit row gate_w [1, hidden] (NULL: no gate). */
typedef struct {
    int32_t hidden;
    int32_t inter;
    int32_t scale_layout;
    int32_t pad_;
    const uint8_t* gate_up_q;
    const float* gate_up_scale;
    const uint8_t* down_q;
    const float* down_scale;
    const uint16_t* gate_w;
} oomb_shared_expert;

/* One MoE layer's decode step: the shared expert (gate/up GEMV, SwiGLU, down
 * GEMV, gate logit: Moe::shared, crates/oominf-models-qwen/src/moe.rs:
 * 498-527), the routed experts (as oomb_moe_decode_fp8) and the combine
 * out = routed + sigmoid(gate) * shared (Experts::moe_combine, backend.rs:
 * 909-917; ops.cu:311-316; out = routed + shared without a gate): the body of
 * Moe::forward (moe.rs:479-495) as one stream-ordered sequence, no host round
 * trip.  x and out are device memory ([t, hidden]); ids / weights optional as
 * for oomb_moe_decode_fp8.  The shared GEMVs run on the tensor cores from two
 * tokens.  Workspace: oomb_moe_layer_workspace_bytes(t, layer, shared, x_dtype)
 * bytes, zeroed once before first use (and after a device error); calls
 * sharing it must be ordered on one stream.  Bit-identical to calling
 * oomb_gemm_fp8, oomb_silu_mul_rows, oomb_gemm_fp8, oomb_router_logits,
 * oomb_moe_decode_fp8 and oomb_moe_combine in that order. */
size_t oomb_moe_layer_workspace_bytes(int t, const oomb_moe_layer* layer, const oomb_shared_expert* shared,
                                      int x_dtype);
int oomb_moe_layer_decode_fp8(const oomb_moe_layer* layer, const oomb_shared_expert* shared, const void* x,
                              int x_dtype, int t, void* out, int out_dtype, int32_t* ids, float* weights,
                              void* workspace, size_t workspace_bytes, oomb_stream stream);

/* ---- fused decode step that allocates nothing --------------------------- */
/* No counterpart in the reference: an addition of this library.  For callers
 * that cannot allocate or hold device memory where they call the decode step:
 * cudaMalloc and cudaFree may synchronise the device, which a decode loop must
 * not do, and some hosts (an engine whose device budget is fixed at start-up,
 * an FFI caller with no device allocator) have no workspace to pass.  The step
 * computes exactly what oomb_moe_decode_fp8 computes, with its scratch in one
 * fixed device array of OOMB_NOALLOC_SCRATCH_BYTES per device inside this
 * library; it calls no allocator.
 *   - Limit: a call fits when oomb_moe_decode_workspace_bytes(t, layer) <=
 *     OOMB_NOALLOC_SCRATCH_BYTES (8 MiB; with hidden 2048, 128 experts, top-8
 *     and intermediate 768 that is t <= 43); larger calls return
 *     OOMB_E_WORKSPACE before any launch.
 *   - The first call on each device, made with that device current, does a
 *     one-time set-up: it looks up the array's device address and zeroes the
 *     array's first 4096 bytes on `stream` (one cudaMemsetAsync): the kernel
 *     chain's self-resetting arrival counter (256 bytes) and the one-launch
 *     kernel's sync words (launch epoch, grid-barrier counts, row-group
 *     counters).  Make that first call before any stream capture.  If the
 *     set-up fails the call returns OOMB_E_DEVICE and the next call retries it.
 *   - All calls on one device share the array: they must be ordered (one
 *     stream, or otherwise serialised).  Overlapping calls race on the
 *     scratch and corrupt each other's results.
 *   - After a bounded device wait has run out (oomb_device_error reports a
 *     code), clearing the error with oomb_device_error(&code, 1) zeroes those
 *     4096 bytes again, so the next call starts from clean sync words. */
#define OOMB_NOALLOC_SCRATCH_BYTES (8 * 1024 * 1024)
int oomb_moe_decode_fp8_noalloc(const oomb_moe_layer* layer, const void* x, int x_dtype, int t, void* out,
                                int out_dtype, int32_t* ids, float* weights, oomb_stream stream);

/* ---- routed experts with device-side group counts ----------------------- */
/* gate/up+SiLU then down over n_active[0] (on the device) expert groups:
 * expert i owns assignments [off[i], off[i+1]), record recs_active[i], the
 * assignment's activation row assign_tok[a] of x.  h: [A, inter] fp32
 * scratch, y: [A, hidden] fp32.  max_active bounds n_active (launch size);
 * max_per_expert bounds any group (0 if unknown).  The same kernels and
 * arithmetic as oomb_moe_gate_up_fp8 / oomb_moe_down_fp8: an assignment's
 * output does not depend on which other assignments share the launch. */
int oomb_moe_experts_fp8(const uint64_t* recs_active, const int32_t* off, const int32_t* assign_tok,
                         const int32_t* n_active, int max_active, const void* x, int x_dtype, float* h, float* y,
                         const oomb_fp8_record* geo, int max_per_expert, oomb_stream stream);

/* The same step on the tensor cores, for many assignments per expert (the
 * reference's Moe::run_group takes its tiled branch there, moe.rs:746-758): the
 * activation rows split once into e4m3 terms, gate and up by oomb_moe_tiled_fp8's
 * kernel (into y, which needs hidden >= 2 * intermediate), SwiGLU into h, h split,
 * down into y.  The groups' count stays on the device (n_active); max_assignments
 * bounds off[n_active] and sizes the workspace
 * (oomb_moe_experts_tiled_fp8_workspace_bytes); max_per_expert bounds any group
 * (> 0).  hidden and intermediate are multiples of 128.  Within the tensor-core
 * path's tolerance of oomb_moe_experts_fp8 (another summation order); an output's
 * bits do not depend on the other assignments of the launch. */
size_t oomb_moe_experts_tiled_fp8_workspace_bytes(int max_assignments, const oomb_fp8_record* geo, int x_dtype);
int oomb_moe_experts_tiled_fp8(const uint64_t* recs_active, const int32_t* off, const int32_t* assign_tok,
                               const int32_t* n_active, int max_active, int max_assignments, const void* x,
                               int x_dtype, float* h, float* y, const oomb_fp8_record* geo, int max_per_expert,
                               void* workspace, size_t workspace_bytes, oomb_stream stream);

/* ---- expert parallelism (experts sharded over ranks) --------------------- */
/* No counterpart in the reference, which runs on one device (its experts are
 * tiered, not sharded).  Expert e lives on rank e / experts_per_rank.  A step:
 * route on every rank; oomb_ep_meta; all-to-all of meta and of the tokens'
 * activations (fixed sizes, no host round trip); oomb_ep_group;
 * oomb_moe_experts_fp8; oomb_ep_scatter; reverse all-to-all; oomb_ep_combine.
 * The expert outputs and the slot-order combine are the single-GPU path's
 * arithmetic, so every rank's output is bit-identical to one GPU's.
 *
 * meta[g][t][s] (ranks x t x k int32): local id on rank g of ids[t][s]'s
 * expert, or -1. */
int oomb_ep_meta(const int32_t* ids, int t, int k, int experts_per_rank, int ranks, int32_t* meta,
                 oomb_stream stream);
/* Groups the received recv_meta[g][t][s] by local expert in (g, t, s) order
 * (one CTA): n_active[0], off[n_active + 1], assign_row[A] = g * t + t_src
 * (row of the received activations [ranks * t, hidden]), assign_ret[A] =
 * g * t*k + t_src * k + s (row of the return buffer), recs_active[n_active] =
 * recs_local[local expert].  A <= ranks * t * k. */
int oomb_ep_group(const int32_t* recv_meta, int ranks, int t, int k, int experts_per_rank, const uint64_t* recs_local,
                  int32_t* n_active, int32_t* off, int32_t* assign_row, int32_t* assign_ret, uint64_t* recs_active,
                  oomb_stream stream);
/* ret[assign_ret[a]] = y[a] for the A grouped assignments; ret: [ranks * t*k, h]
 * fp32 (rows of absent slots are left as they are); max_rows bounds A. */
int oomb_ep_scatter(const float* y, const int32_t* n_active, const int32_t* off, const int32_t* assign_ret, int h,
                    int max_rows, float* ret, oomb_stream stream);
/* out[t] = sum_s w[t, s] * back[ids[t, s] / experts_per_rank][t*k + s] in slot
 * order with fused multiply-adds; back: [ranks][t*k][h] fp32 (the returned
 * rows); out fp32 or bf16 [t, h]. */
int oomb_ep_combine(const float* back, const int32_t* ids, const float* w, int t, int k, int h, int experts_per_rank,
                    int ranks, void* out, int out_dtype, oomb_stream stream);

/* Expert parallelism with the all-to-alls done by the kernels over NVLink:
 * every rank owns a mailbox (cudaMalloc'd by oomb_ep_mailbox_alloc, zeroed;
 * mapped into every peer through CUDA IPC), and the dispatch and return
 * kernels store straight into the destination rank's mailbox, then raise a
 * per-source flag there carrying the step's epoch (the mailbox's step counter
 * + 1); the grouping and combine kernels wait for every source's flag (bounded
 * waits; a wait that runs out records OOMB device error 0x700 / 0x710).  A step:
 * route; oomb_ep_dispatch_peer; oomb_ep_group_peer; oomb_moe_experts_fp8 over
 * the mailbox's received activations; oomb_ep_return_peer; oomb_ep_combine_peer
 * (which advances the step counter).  Every rank runs the same steps with the
 * same t; the arithmetic is the NCCL path's, bit-identical to one GPU. */
typedef struct oomb_ep_peer {
    const uint64_t* peers; /* device array [ranks]: every rank's mailbox in this process (own rank: mailbox) */
    void* mailbox;         /* this rank's mailbox */
    int ranks, rank;
    int t_max;             /* tokens per rank the mailbox holds */
    int top_k, hidden;
    int x_dtype;           /* OOMB_BF16 or OOMB_F32 activations */
} oomb_ep_peer;

/* The one-launch decode step (as oomb_moe_decode_fp8, up to 16 tokens per rank
 * and 256 experts) with expert parallelism: layer->recs holds this rank's
 * experts [rank * E/ranks, (rank + 1) * E/ranks), layer->router_w the whole
 * router.  Route, dispatch to the mailboxes, grouping of the received slots,
 * gate/up and down over the local experts (every received slot a group of its
 * own) with each output value stored into its source rank's mailbox as an
 * (epoch, value) 64-bit word, and the slot-order combine polling those words,
 * in one kernel per rank; every rank runs the step with the same t.  x and out
 * may be pinned host memory, as for oomb_moe_decode_fp8.  Bit-identical to one
 * GPU. */
size_t oomb_moe_decode_ep_workspace_bytes(int t, int ranks, const oomb_moe_layer* layer);
int oomb_moe_decode_ep_fp8(const oomb_moe_layer* layer, const oomb_ep_peer* peer, const void* x, int x_dtype, int t,
                           void* out, int out_dtype, int32_t* ids, float* weights, void* workspace,
                           size_t workspace_bytes, oomb_stream stream);

#define OOMB_IPC_HANDLE_BYTES 64
size_t oomb_ep_mailbox_bytes(int ranks, int t_max, int top_k, int hidden, int x_dtype);
/* Byte offset of the received activations [ranks * t, hidden] in a mailbox. */
size_t oomb_ep_mailbox_x_offset(int ranks, int t_max, int top_k, int hidden, int x_dtype);
int oomb_ep_mailbox_alloc(size_t bytes, void** mailbox);  /* cudaMalloc + zero */
int oomb_ep_mailbox_free(void* mailbox);
int oomb_ipc_handle(const void* dev_ptr, void* handle);    /* cudaIpcGetMemHandle of an allocation base */
int oomb_ipc_open(const void* handle, void** dev_ptr);     /* cudaIpcOpenMemHandle (lazy peer access) */
int oomb_ipc_close(void* dev_ptr);
/* ids [t, k] (experts of this rank's tokens), x [t, hidden]. */
int oomb_ep_dispatch_peer(const oomb_ep_peer* q, const int32_t* ids, int t, int experts_per_rank, const void* x,
                          oomb_stream stream);
/* As oomb_ep_group over the mailbox's received meta. */
int oomb_ep_group_peer(const oomb_ep_peer* q, int t, int experts_per_rank, const uint64_t* recs_local,
                       int32_t* n_active, int32_t* off, int32_t* assign_row, int32_t* assign_ret,
                       uint64_t* recs_active, oomb_stream stream);
/* Sends y[a] to its source rank's mailbox (row (this rank, slot)); max_rows bounds A. */
int oomb_ep_return_peer(const oomb_ep_peer* q, const float* y, const int32_t* n_active, const int32_t* off,
                        const int32_t* assign_ret, int t, int max_rows, oomb_stream stream);
/* As oomb_ep_combine over the mailbox's returned rows; out fp32 or bf16 [t, hidden]. */
int oomb_ep_combine_peer(const oomb_ep_peer* q, const int32_t* ids, const float* w, int t, int experts_per_rank,
                         void* out, int out_dtype, oomb_stream stream);

/* ---- offload staging ---------------------------------------------------- */
/* Copies that run beside compute, from pinned host memory or within the
 * device, ordered against compute with events: the Transfer trait
 * (crates/oominf-core/src/backend.rs:945-1018; CUDA body
 * crates/oominf-cuda/src/memory.rs:300-398) as used by TieredExperts to bring
 * cold expert records into device slots (crates/oominf-tiers/src/tiered.rs).
 * A copy queue is a non-blocking stream; events carry no timing.  Each record
 * is one cudaMemcpyAsync. */
typedef struct oomb_copy_queue_st* oomb_copy_queue;
typedef struct oomb_event_st* oomb_event;
int oomb_copy_queue_create(oomb_copy_queue* queue);   /* Transfer::copy_queue */
int oomb_copy_queue_destroy(oomb_copy_queue queue);
int oomb_pin_host(void* ptr, size_t len);            /* Transfer::pin_host (portable registration) */
int oomb_unpin_host(void* ptr);                      /* Transfer::unpin_host */
int oomb_copy_to_device(oomb_copy_queue queue, void* dst, const void* src, size_t len); /* copy_to_device */
int oomb_copy_on_device(oomb_copy_queue queue, void* dst, const void* src, size_t len); /* copy_on_device */
int oomb_record_compute(oomb_stream compute, oomb_event* ev); /* completes with the compute issued so far */
int oomb_record_copies(oomb_copy_queue queue, oomb_event* ev); /* completes with the copies queued so far */
int oomb_copies_wait(oomb_copy_queue queue, oomb_event ev);   /* later copies wait for ev */
int oomb_compute_wait(oomb_stream compute, oomb_event ev);    /* later compute waits for ev */
int oomb_event_done(oomb_event ev);                           /* 1 done, 0 pending, < 0 error */
int oomb_event_wait(oomb_event ev);                           /* blocks the host */
int oomb_event_destroy(oomb_event ev);
int oomb_copies_sync(oomb_copy_queue queue);                  /* blocks the host */

/* ---- expert tiers: the two-phase fetch over device slots ----------------- */
/* Replacement policy of an expert cache (crates/oominf-tiers/src/policy.rs:
 * 9-129, the Policy trait: touch / remove / victim).  Keys are layer *
 * experts + expert.  spec: "lru", "lfu" (LRFU with half-life 1e12) or
 * "lrfu:<half_life>" (each access adds 2^(now / half_life) to a key's score;
 * the lowest score is the victim).  Host-only: needs no GPU. */
typedef struct oomb_policy_st* oomb_policy;
int oomb_policy_create(const char* spec, oomb_policy* policy);
int oomb_policy_destroy(oomb_policy policy);
int oomb_policy_touch(oomb_policy policy, uint32_t key, uint64_t now);
int oomb_policy_remove(oomb_policy policy, uint32_t key);
/* The best victim among resident keys not in pinned[0 .. n_pinned), or -1. */
int64_t oomb_policy_victim(oomb_policy policy, const uint32_t* pinned, int n_pinned);

/* A device tier of expert records: `slots` records of record_stride bytes at
 * device_slots (caller-owned device memory), filled on demand from the pinned
 * host arena (record (layer, e) at host_arena + (layer * experts + e) *
 * record_stride; cudaHostAlloc / oomb_pin_host memory), victims chosen by the
 * policy `policy` (as oomb_policy_create).  The ExpertSource two-phase fetch
 * (crates/oominf-core/src/experts.rs:12-41) as TieredExperts drives its device
 * tier (crates/oominf-tiers/src/tiered.rs:1155-1421, 1494-1510):
 *   oomb_tier_begin_fetch: addrs[i] = the device address of experts[i]'s
 *     record of `layer`, ready[i] = 1 if compute issued now may read it (it was
 *     resident), 0 if its copy was queued (the copy queue first waits for the
 *     compute issued on `compute` so far: a kernel issued earlier may still
 *     read the victim's slot).  Victims are never records this fetch wants.
 *     Returns OOMB_E_SHAPE when the slots cannot hold one fetch's experts.
 *   oomb_tier_finish_fetch: compute issued on `compute` after it may read
 *     every record of the last begin_fetch (one stream wait on the copies).
 * Work on the ready records, issued between the two calls, overlaps the
 * copies.  A begin_fetch while a fetch is open finishes it first.  One host
 * thread per tier.  stats: requests, hits, misses, evictions, bytes copied. */
typedef struct oomb_tier_st* oomb_tier;
int oomb_tier_create(const void* host_arena, size_t record_stride, int layers, int experts, void* device_slots,
                     int slots, const char* policy, oomb_tier* tier);
int oomb_tier_destroy(oomb_tier tier);
int oomb_tier_begin_fetch(oomb_tier tier, oomb_stream compute, int layer, const int32_t* experts, int n,
                          uint64_t* addrs, uint8_t* ready);
int oomb_tier_finish_fetch(oomb_tier tier, oomb_stream compute);
int oomb_tier_stats(oomb_tier tier, uint64_t* stats5);

/* ---- weight preparation ------------------------------------------------- */
/* The record layout of an FP8 expert (hidden, inter multiples of 16): part
 * offsets into *geo, the record stride (bytes) into *stride. */
int oomb_fp8_record_layout(int64_t hidden, int64_t inter, int scale_layout, oomb_fp8_record* geo, size_t* stride);
/* Load-time conversion of one expert into its record on the device: bf16
 * gate, up [inter, hidden] and down [hidden, inter] quantized (as
 * oomb_quantize_fp8) into the parts of `record` laid out by *geo.  Padding
 * bytes are left as they are (zero the record first for a file image).  The
 * converter adapter's per-expert step (crates/oominf-convert). */
int oomb_quantize_fp8_record(const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                             const oomb_fp8_record* geo, uint8_t* record, oomb_stream stream);
/* The load-time quantizer on the device, byte-identical to fp8::quantize_blocks
 * (crates/oominf-core/src/fp8.rs:52-88) for OOMB_SCALE_1X128 and to its 2-D
 * block generalisation for OOMB_SCALE_128X128.  w: bf16 [n, k]. */
int oomb_quantize_fp8(const uint16_t* w, int n, int k, int scale_layout, uint8_t* q, float* scale,
                      oomb_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* OOMB_H */
