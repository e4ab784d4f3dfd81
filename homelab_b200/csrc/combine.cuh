// combine.cuh - slot-order weighted combine and the shared-expert combine.
#pragma once

#include "common.cuh"

namespace oomb {

// Copies n16 16-byte words of activations from pinned host memory, read at
// its mapped device address (.cv: fetched again, never a stale cached line),
// into device memory once the previous kernel of the stream has completed, so
// the kernels after it read a device copy.
__global__ void __launch_bounds__(256) stage_host_kernel(uint4* dst, const uint4* src, int64_t n16) {
    pdl_wait();
    pdl_launch_dependents();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; i < n16;
         i += static_cast<int64_t>(gridDim.x) * 256)
        dst[i] = __ldcv(src + i);
}

// out[t, c] = sum_s w[t, s] * y[slot[t, s], c] in slot order with fmaf
// (moe_combine_slots, moe.cu:155-164).  Four columns per thread; the slot
// indices and weights of a group of 8 slots are loaded before their rows so the
// row loads are in flight together.
template <bool OUT_BF16>
__global__ void combine_slots_kernel(const float* y, const int32_t* slot, const float* w, void* out,
                                     int T, int H, int K) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i >= static_cast<int64_t>(T) * H) return;
    const int t = static_cast<int>(i / H), c = static_cast<int>(i % H);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < K; s0 += 8) {
        int a[8];
        float ws[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const bool ok = s0 + j < K;
            a[j] = ok ? __ldcg(slot + t * K + s0 + j) : 0;
            ws[j] = ok ? __ldcg(w + t * K + s0 + j) : 0.0f;
        }
        float4 v[8];
#pragma unroll
        for (int j = 0; j < 8; j++)
            v[j] = s0 + j < K ? __ldcg(reinterpret_cast<const float4*>(y + static_cast<int64_t>(a[j]) * H + c))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 8; j++) {
            if (s0 + j < K) {
                acc.x = fmaf(ws[j], v[j].x, acc.x);
                acc.y = fmaf(ws[j], v[j].y, acc.y);
                acc.z = fmaf(ws[j], v[j].z, acc.z);
                acc.w = fmaf(ws[j], v[j].w, acc.w);
            }
        }
    }
    if (OUT_BF16) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
        __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
        uint2 pk;
        pk.x = *reinterpret_cast<unsigned*>(&lo);
        pk.y = *reinterpret_cast<unsigned*>(&hi);
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + i) = pk;
    } else {
        *reinterpret_cast<float4*>(static_cast<float*>(out) + i) = acc;
    }
}

// SwiGLU on stacked rows (silu_mul_rows, ops.cu:302-309): y[r, i] =
// silu(gu[r, i]) * gu[r, n + i], silu(v) = v / (1 + exp(-v)); gu fp32 [rows, 2n],
// y fp32 or bf16 [rows, n].  Four columns per thread (n % 4 == 0).
template <bool OUT_BF16>
__global__ void silu_mul_rows_kernel(const float* gu, void* y, int rows, int n) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i >= static_cast<int64_t>(rows) * n) return;
    const int r = static_cast<int>(i / n), c = static_cast<int>(i % n);
    const float4 g = __ldcg(reinterpret_cast<const float4*>(gu + static_cast<int64_t>(r) * 2 * n + c));
    const float4 u = __ldcg(reinterpret_cast<const float4*>(gu + static_cast<int64_t>(r) * 2 * n + n + c));
    const float o0 = g.x / (1.0f + expf(-g.x)) * u.x, o1 = g.y / (1.0f + expf(-g.y)) * u.y;
    const float o2 = g.z / (1.0f + expf(-g.z)) * u.z, o3 = g.w / (1.0f + expf(-g.w)) * u.w;
    if (OUT_BF16) {
        __nv_bfloat162 lo = __floats2bfloat162_rn(o0, o1), hi = __floats2bfloat162_rn(o2, o3);
        uint2 pk;
        pk.x = *reinterpret_cast<unsigned*>(&lo);
        pk.y = *reinterpret_cast<unsigned*>(&hi);
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(y) + i) = pk;
    } else {
        *reinterpret_cast<float4*>(static_cast<float*>(y) + i) = make_float4(o0, o1, o2, o3);
    }
}

// out = routed + sigmoid(gate_logit[t]) * shared (ops.cu:311-316); with no
// gate_logit (a shared expert without a gate) out = routed + shared.  out fp32
// or bf16 (RN of the fp32 sum).
template <bool OUT_BF16>
__global__ void moe_combine_kernel(const float* routed, const float* shared, const float* gate_logit, void* out,
                                   int T, int H) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= static_cast<int64_t>(T) * H) return;
    const float r = __ldcg(routed + i), sh = __ldcg(shared + i);
    float v;
    if (gate_logit) {
        const float g = __ldcg(gate_logit + i / H);
        v = r + (1.0f / (1.0f + expf(-g))) * sh;
    } else {
        v = r + sh;
    }
    if (OUT_BF16) static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
    else static_cast<float*>(out)[i] = v;
}

}  // namespace oomb
