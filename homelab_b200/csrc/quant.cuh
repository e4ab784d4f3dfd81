// quant.cuh - load-time FP8 block quantizer on the device.
//
// Byte-identical to fp8::quantize_blocks (crates/oominf-core/src/fp8.rs:52-88)
// for 1x128 blocks: scale = amax(|w|) / 448 (1 for an all-zero block), q =
// e4m3(w / scale) rounded to nearest even and saturated at +-448 (NaN -> the
// saturated code, as e4m3_from_f32 does).  For 128x128 blocks the amax runs
// over the 2-D block.
#pragma once

#include "common.cuh"

namespace oomb {

__device__ __forceinline__ uint8_t e4m3_from_f32_rne(float v) {
    if (v != v) return (__float_as_uint(v) >> 24 & 0x80) | 0x7e;
    return static_cast<uint8_t>(__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3));
}

// One CTA of 128 threads per scale block; thread c owns column c0 + c.
__global__ void __launch_bounds__(128) quantize_blocks_kernel(const uint16_t* w, int n, int k,
                                                              int layout, uint8_t* q,
                                                              float* scale) {
    const int nb = (k + 127) >> 7;
    const int br = blockIdx.x / nb, b = blockIdx.x % nb;
    const int rows_per = layout ? 128 : 1;
    const int r0 = br * rows_per, r1 = min(n, r0 + rows_per);
    const int c = b * 128 + threadIdx.x;
    float amax = 0.0f;
    if (c < k)
        for (int r = r0; r < r1; r++)
            amax = fmaxf(amax, fabsf(bf16_bits_to_float(w[static_cast<int64_t>(r) * k + c])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    __shared__ float wmax[4];
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = fmaxf(fmaxf(wmax[0], wmax[1]), fmaxf(wmax[2], wmax[3]));
    const float s = amax > 0.0f ? __fdiv_rn(amax, 448.0f) : 1.0f;
    if (threadIdx.x == 0) scale[static_cast<int64_t>(br) * nb + b] = s;
    if (c < k)
        for (int r = r0; r < r1; r++) {
            const int64_t i = static_cast<int64_t>(r) * k + c;
            q[i] = e4m3_from_f32_rne(__fdiv_rn(bf16_bits_to_float(w[i]), s));
        }
}

}  // namespace oomb
