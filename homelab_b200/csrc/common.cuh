// common.cuh - sm_100a device helpers shared by the oomb kernels.
//
// Bulk copies (cp.async.bulk) into shared memory completed on mbarriers,
// bounded mbarrier waits that record an error code instead of hanging,
// programmatic dependent launch (griddepcontrol), FP8 e4m3 decode and the
// packed fp32 FMA of sm_100 (fma.rn.f32x2).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace oomb {

// Error codes a kernel writes to the device error word (first one wins).
enum : unsigned {
    ERR_NONE = 0,
    ERR_FULL_WAIT = 0x100,   // consumer gave up waiting for a stage to land
    ERR_EMPTY_WAIT = 0x200,  // producer gave up waiting for a stage to be released
    ERR_DRAIN_WAIT = 0x300,  // producer gave up draining its copies after an error
    ERR_BAD_TABLE = 0x400,   // a routing table entry was out of range (work skipped)
};

// A bounded wait gives up after this long (globaltimer nanoseconds): orders of
// magnitude above any legitimate stage wait, short enough that a lost copy
// ends the kernel with an error instead of hanging the GPU.  The limit in
// force lives in a device word (one per device), so a caller can shorten it
// (oomb_set_wait_limit) to make a wait that nothing will satisfy run out fast.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;
__device__ unsigned long long g_wait_limit_ns = kWaitLimitNs;

// The limit in force, read once when a wait did not succeed at once.
__device__ __forceinline__ unsigned long long wait_limit() {
    return *const_cast<volatile unsigned long long*>(&g_wait_limit_ns);
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void record_error(unsigned* err, unsigned code) {
    if (err) atomicCAS(err, 0u, code);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier --------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

// Makes mbarrier initialisation visible to the async (bulk copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile(
        "{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
    asm volatile(
        "{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(
            smem_addr(bar)),
        "r"(bytes)
        : "memory");
}

// try_wait returns once the phase completes or, without it, after a time the
// hardware chooses; OOMB_MBAR_SUSPEND_NS > 0 passes that time as a hint (the
// thread still wakes as soon as the phase completes), so waiting warps re-issue
// their poll less often.  Measured on B200 with a 10 us hint: no kernel faster
// (the config-3 batch-4 MLP 71.0 -> 74.6 us), so no hint by default.
#ifndef OOMB_MBAR_SUSPEND_NS
#define OOMB_MBAR_SUSPEND_NS 0
#endif
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
    unsigned ok;
#if OOMB_MBAR_SUSPEND_NS > 0
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(static_cast<unsigned>(OOMB_MBAR_SUSPEND_NS))
        : "memory");
#else
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
#endif
    return ok != 0;
}

// Waits for the phase of `bar` with the given parity to complete.  Gives up
// after wait_limit() nanoseconds, records `code` and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, unsigned* err,
                                          unsigned code) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns(), limit = wait_limit();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > limit) {
            record_error(err, code);
            return false;
        }
    }
}

// ---- bulk copies -------------------------------------------------------------

// Copies `bytes` (a multiple of 16; both addresses 16-byte aligned) from global
// memory into this CTA's shared memory; completion is counted in bytes on `bar`.
// `policy` is an L2 cache policy from make_evict_first_policy().
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// As bulk_g2s, with the default L2 policy (activations another kernel may read again).
__device__ __forceinline__ void bulk_g2s_plain(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Block scales are read again every step and are 0.4 % of the weight bytes:
// loaded with evict-last priority they stay in L2 under the streamed weights, so
// a step's scale reads do not queue in HBM behind its weight copies.
#ifndef OOMB_SCALE_KEEP
#define OOMB_SCALE_KEEP 1
#endif
__device__ __forceinline__ uint64_t make_evict_last_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ float ld_scale(const float* a, uint64_t keep) {
#if OOMB_SCALE_KEEP
    float v;
    asm("ld.global.nc.L2::cache_hint.f32 %0, [%1], %2;" : "=f"(v) : "l"(a), "l"(keep));
    return v;
#else
    return __ldg(a);
#endif
}

// Weights are streamed once per step: mark them evict-first so they do not push
// activations and routing tables out of L2.
__device__ __forceinline__ uint64_t make_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ---- programmatic dependent launch -----------------------------------------

// Blocks until the grids this one depends on have completed and their memory
// is visible.  A no-op when the launch had no programmatic dependency.
// A value and the step epoch that validates it, in one 8-byte word: an aligned
// 64-bit store is single-copy atomic, so a reader that sees the epoch sees the
// value stored with it, with no fence or flag between writer and reader.
__device__ __forceinline__ void st_word_sys(unsigned long long* p, unsigned epoch, float v) {
    const unsigned long long w = (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void st_word32_sys(unsigned long long* p, unsigned epoch, unsigned v) {
    const unsigned long long w = (static_cast<unsigned long long>(epoch) << 32) | v;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_word_sys(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Lets the next kernel in the stream start launching its CTAs.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- arithmetic --------------------------------------------------------------

// d = a * b + c on two fp32 lanes at once (sm_100 packed FMA), each lane
// rounded as fmaf.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n .reg .b64 ra, rb, rc, rd;\n"
        " mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mov.b64 rc, {%6, %7};\n"
        " fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// d = a * b on two fp32 lanes at once (sm_100 packed multiply), each lane
// rounded as __fmul_rn.
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    float2 d;
    asm("{\n .reg .b64 ra, rb, rd;\n"
        " mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
        " mul.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// Two e4m3 codes (low byte first) to their exact values.
__device__ __forceinline__ float2 e4m3x2_to_float2(unsigned short pair) {
    __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3);
    return __half22float2(*reinterpret_cast<const __half2*>(&hr));
}

__device__ __forceinline__ float bf16_bits_to_float(unsigned short b) {
    return __uint_as_float(static_cast<unsigned>(b) << 16);
}

// Sixteen consecutive activations as fp32, from fp32 or bf16 storage.
template <bool BF16>
__device__ __forceinline__ void load_x16(const void* base, int64_t idx, float2 (&x)[8]) {
    if constexpr (BF16) {
        const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + idx);
        uint4 a = __ldg(p), b = __ldg(p + 1);
        const unsigned w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 8; i++)
            x[i] = make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
    } else {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + idx);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float4 v = __ldg(p + i);
            x[2 * i] = make_float2(v.x, v.y);
            x[2 * i + 1] = make_float2(v.z, v.w);
        }
    }
}

// Same, for activations another kernel of this step wrote (bypasses the
// non-coherent read-only path).
template <bool BF16>
__device__ __forceinline__ void load_x16_cg(const void* base, int64_t idx, float2 (&x)[8]) {
    if constexpr (BF16) {
        const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + idx);
        uint4 a = __ldcg(p), b = __ldcg(p + 1);
        const unsigned w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 8; i++)
            x[i] = make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
    } else {
        const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + idx);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float4 v = __ldcg(p + i);
            x[2 * i] = make_float2(v.x, v.y);
            x[2 * i + 1] = make_float2(v.z, v.w);
        }
    }
}

// Dot product of 16 e4m3 weights (one 16-byte chunk) with 16 activations, as
// two interleaved fp32 FMA chains (even / odd columns) summed at the end.
__device__ __forceinline__ float dot16_e4m3(uint4 w, const float2 (&x)[8]) {
    const unsigned words[4] = {w.x, w.y, w.z, w.w};
    float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float2 lo = e4m3x2_to_float2(static_cast<unsigned short>(words[i] & 0xffffu));
        float2 hi = e4m3x2_to_float2(static_cast<unsigned short>(words[i] >> 16));
        acc = ffma2(lo, x[2 * i], acc);
        acc = ffma2(hi, x[2 * i + 1], acc);
    }
    return acc.x + acc.y;
}

// Sums `V` values per lane over the 32 lanes of a warp.  Afterwards lane l
// holds, in v[0 .. V/32) (or v[0] when V <= 32), the totals of the value
// indices given by reduce_index(): each halving step keeps half of the values
// and adds the partner lane's copy of them, so V values cost V - 1 shuffles
// (plus one per remaining level) instead of 5 V.
template <int V>
__device__ __forceinline__ void warp_reduce_multi(float (&v)[V], int lane) {
    static_assert((V & (V - 1)) == 0, "V must be a power of two");
    int n = V;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        if (n > 1) {
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < V / 2; i++) {
                if (i < n / 2) {
                    float send = upper ? v[i] : v[i + n / 2];
                    float keep = upper ? v[i + n / 2] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
            n >>= 1;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
        }
    }
}

// Index of the value whose warp total lane `lane` holds in v[j] after
// warp_reduce_multi<V>.
template <int V>
__device__ __forceinline__ int reduce_index(int lane, int j) {
    // Each halving step at offset o moves lanes with bit o set to the upper half.
    int idx = 0, n = V;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        if (n > 1) {
            n >>= 1;
            if (lane & o) idx += n;
        }
    }
    // When V > 32 each lane keeps V/32 values: v[j] is index idx + j.
    return idx + j;
}

}  // namespace oomb
