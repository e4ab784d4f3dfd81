// Launcher for the reference's own CUDA kernels (test infrastructure only).
//
// The reference compiles every kernels/*.cu of crates/oominf-cuda to a module
// and launches the kernels by name through the driver API (build.rs:42-60,
// lib.rs:143-156).  This file does the same for the kernels on the decode hot
// path so the tests can run them beside the sm_100a path on identical device
// buffers.  Launch geometry follows the reference host code:
//   gemv_fp8_t{1..4}   Gpu::gemv_at          (src/linear.rs:260-349)
//   router_topk        Experts::router_topk  (src/experts.rs:10-37)
//   moe_gate_up_bf16   Experts::moe_gate_up_bf16 (src/experts.rs:95-140)
//   moe_down_bf16      Experts::moe_down_bf16
//   moe_combine_slots  Experts::moe_combine_slots (src/experts.rs:303-329)
//   fp8_dequantize_blocks, f32_to_bf16, silu_mul_rows   the dense path above 16
//                      tokens (Linear::gemm_fp8, src/linear.rs:35-81, 140-205) and the
//                      SwiGLU between its two GEMMs (src/elementwise.rs:56-70); one
//                      thread per element, grid(n, 256)
// The modules (ops.cubin, moe.cubin) are built from the reference sources by
// oracle/ref/Makefile; libcuda is opened at run time so this library loads on
// machines without a GPU.
#include <dlfcn.h>

#include <cstdint>
#include <cstdio>
#include <string>

namespace {

using CUresult = int;
using CUdevice = int;
using CUcontext = void*;
using CUmodule = void*;
using CUfunction = void*;
using CUstream = void*;

constexpr int kMaxDynamicSmemAttr = 8;  // CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES

struct Driver {
    CUresult (*init)(unsigned);
    CUresult (*ctx_get_current)(CUcontext*);
    CUresult (*module_load)(CUmodule*, const char*);
    CUresult (*module_get_function)(CUfunction*, CUmodule, const char*);
    CUresult (*func_set_attribute)(CUfunction, int, int);
    CUresult (*launch)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned,
                       CUstream, void**, void**);
};

Driver g_drv;
bool g_open = false;
CUfunction g_gemv[4], g_router, g_gate_up_bf16, g_down_bf16, g_combine, g_dequant, g_to_bf16, g_silu_rows;

template <class F>
bool sym(void* h, const char* name, F& f) {
    f = reinterpret_cast<F>(dlsym(h, name));
    return f != nullptr;
}

// Gpu::gemv_at split plan for FP8 weights and t <= 4 tokens (linear.rs:270-285).
void gemv_plan(int t, int n, int k, int* splits, int* klen, int* tiles) {
    const int step = 512, smem = 48 * 1024, warps = 8, rows_per_warp = 4;
    int row_groups = (n + rows_per_warp - 1) / rows_per_warp;
    int kchunks = (k + step - 1) / step;
    int want = (2048 + row_groups - 1) / row_groups;
    if (want < 1) want = 1;
    if (want > kchunks) want = kchunks;
    int smem_min = (t * k * 4 + smem - 1) / smem;
    int s0 = want > smem_min ? want : smem_min;
    if (s0 > kchunks) s0 = kchunks;
    *klen = ((k + s0 - 1) / s0 + step - 1) / step * step;
    *splits = (k + *klen - 1) / *klen;
    *tiles = (row_groups + warps - 1) / warps;
}

}  // namespace

extern "C" {

// Loads the modules from `dir` into the calling thread's current context.
// Returns 0, or a negative code: -1 no libcuda, -2 no current context,
// -3 a module or kernel is missing.
int orl_open(const char* dir) {
    if (g_open) return 0;
    void* h = dlopen("libcuda.so.1", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return -1;
    if (!sym(h, "cuInit", g_drv.init) || !sym(h, "cuCtxGetCurrent", g_drv.ctx_get_current) ||
        !sym(h, "cuModuleLoad", g_drv.module_load) ||
        !sym(h, "cuModuleGetFunction", g_drv.module_get_function) ||
        !sym(h, "cuFuncSetAttribute", g_drv.func_set_attribute) || !sym(h, "cuLaunchKernel", g_drv.launch))
        return -1;
    if (g_drv.init(0) != 0) return -2;
    CUcontext ctx = nullptr;
    if (g_drv.ctx_get_current(&ctx) != 0 || ctx == nullptr) return -2;
    CUmodule ops = nullptr, moe = nullptr;
    std::string d(dir);
    if (g_drv.module_load(&ops, (d + "/ops.cubin").c_str()) != 0) return -3;
    if (g_drv.module_load(&moe, (d + "/moe.cubin").c_str()) != 0) return -3;
    const char* gemv_names[4] = {"gemv_fp8_t1", "gemv_fp8_t2", "gemv_fp8_t3", "gemv_fp8_t4"};
    for (int i = 0; i < 4; i++)
        if (g_drv.module_get_function(&g_gemv[i], ops, gemv_names[i]) != 0) return -3;
    if (g_drv.module_get_function(&g_router, ops, "router_topk") != 0) return -3;
    if (g_drv.module_get_function(&g_gate_up_bf16, moe, "moe_gate_up_bf16") != 0) return -3;
    if (g_drv.module_get_function(&g_down_bf16, moe, "moe_down_bf16") != 0) return -3;
    if (g_drv.module_get_function(&g_combine, moe, "moe_combine_slots") != 0) return -3;
    if (g_drv.module_get_function(&g_dequant, ops, "fp8_dequantize_blocks") != 0) return -3;
    if (g_drv.module_get_function(&g_to_bf16, ops, "f32_to_bf16") != 0) return -3;
    if (g_drv.module_get_function(&g_silu_rows, ops, "silu_mul_rows") != 0) return -3;
    g_open = true;
    return 0;
}

// Sizes of the caller-owned split-K buffers for a gemv of t tokens:
// partial floats = splits * t * n, tickets (u32, zeroed once) = tiles.
void orl_gemv_plan(int t, int n, int k, int* splits, int* klen, int* tiles) {
    gemv_plan(t, n, k, splits, klen, tiles);
}

// y[t, n] = x[t, k] . dequant(W)[n, k]^T with the reference's FP8 gemv
// (x fp32, W e4m3, scale fp32 [n, ceil(k/128)]).  t in 1..4, k % 16 == 0.
int orl_gemv_fp8(const float* x, const uint8_t* w, const float* scale, float* y, float* partial,
                 unsigned* tickets, int t, int n, int k, void* stream) {
    if (!g_open || t < 1 || t > 4 || n < 1 || k < 16 || k % 16) return -5;
    int splits, klen, tiles;
    gemv_plan(t, n, k, &splits, &klen, &tiles);
    int smem = t * (klen < k ? klen : k) * 4;
    CUfunction f = g_gemv[t - 1];
    if (smem > 47 * 1024 && g_drv.func_set_attribute(f, kMaxDynamicSmemAttr, smem) != 0) return -3;
    float* pp = splits == 1 ? nullptr : partial;
    unsigned* tp = splits == 1 ? nullptr : tickets;
    void* args[] = {&x, &w, &scale, &y, &pp, &tp, &n, &k, &klen};
    return g_drv.launch(f, tiles, splits, 1, 256, 1, 1, smem, stream, args, nullptr) == 0 ? 0 : -3;
}

// Softmax top-k over E logits per token, ties to the lower id, renormalised.
int orl_router_topk(const float* logits, int* ids, float* weights, int t, int e, int k, void* stream) {
    if (!g_open || t < 1 || k < 1 || k > 32 || e < k || e > 8192) return -5;
    void* args[] = {&logits, &ids, &weights, &e, &k};
    return g_drv.launch(g_router, t, 1, 1, 256, 1, 1, e * 4, stream, args, nullptr) == 0 ? 0 : -3;
}

// h[a, j] = silu(x[tok(a)] . Wg[j]) * (x[tok(a)] . Wu[j]) over bf16 expert records.
int orl_moe_gate_up_bf16(const uint64_t* recs, const int* off, const int* assign_tok, int n_experts,
                         const float* x, float* h, int hidden, int inter, long long gw_off, long long uw_off,
                         void* stream) {
    if (!g_open || n_experts < 1 || hidden % 8 || inter % 8) return -5;
    void* args[] = {&recs, &off, &assign_tok, &x, &h, &hidden, &inter, &gw_off, &uw_off};
    return g_drv.launch(g_gate_up_bf16, (inter + 7) / 8, n_experts, 1, 256, 1, 1, 0, stream, args, nullptr) == 0
               ? 0
               : -3;
}

// y[a, r] = h[a] . Wd[r] over bf16 expert records.
int orl_moe_down_bf16(const uint64_t* recs, const int* off, int n_experts, const float* h, float* y, int hidden,
                      int inter, long long dw_off, void* stream) {
    if (!g_open || n_experts < 1 || hidden % 8 || inter % 8) return -5;
    void* args[] = {&recs, &off, &h, &y, &hidden, &inter, &dw_off};
    return g_drv.launch(g_down_bf16, (hidden + 7) / 8, n_experts, 1, 256, 1, 1, 0, stream, args, nullptr) == 0
               ? 0
               : -3;
}

// out[t, c] = sum_s w[t, s] * y[slot_assign[t, s], c] in slot order.
int orl_moe_combine_slots(const float* y, const int* slot_assign, const float* w, float* out, int t, int hidden,
                          int k, void* stream) {
    if (!g_open || t < 1 || hidden < 1 || k < 1) return -5;
    long long total = static_cast<long long>(t) * hidden;
    unsigned blocks = static_cast<unsigned>((total + 255) / 256);
    void* args[] = {&y, &slot_assign, &w, &out, &t, &hidden, &k};
    return g_drv.launch(g_combine, blocks, 1, 1, 256, 1, 1, 0, stream, args, nullptr) == 0 ? 0 : -3;
}

// W[n, k] bf16 = e4m3 q[n, k] * scale[n, ceil(k/128)] (1x128 blocks).
int orl_dequant_fp8(const uint8_t* q, const float* scale, void* w, int n, int k, void* stream) {
    if (!g_open || n < 1 || k < 1) return -5;
    const long long total = static_cast<long long>(n) * k;
    if ((total + 255) / 256 > 0x7fffffffLL) return -5;
    const unsigned blocks = static_cast<unsigned>((total + 255) / 256);
    void* args[] = {&q, &scale, &w, &n, &k};
    return g_drv.launch(g_dequant, blocks, 1, 1, 256, 1, 1, 0, stream, args, nullptr) == 0 ? 0 : -3;
}

// y[i] = bf16(x[i]), i < n.
int orl_f32_to_bf16(const float* x, void* y, int n, void* stream) {
    if (!g_open || n < 1) return -5;
    void* args[] = {&x, &y, &n};
    return g_drv.launch(g_to_bf16, static_cast<unsigned>((n + 255) / 256), 1, 1, 256, 1, 1, 0, stream, args,
                        nullptr) == 0
               ? 0
               : -3;
}

// y[r, i] = silu(gu[r, i]) * gu[r, n + i], gu [rows, 2n] fp32.
int orl_silu_mul_rows(const float* gu, float* y, int rows, int n, void* stream) {
    if (!g_open || rows < 1 || n < 1) return -5;
    const long long total = static_cast<long long>(rows) * n;
    if (total > 0x7fffffffLL) return -5;
    void* args[] = {&gu, &y, &rows, &n};
    return g_drv.launch(g_silu_rows, static_cast<unsigned>((total + 255) / 256), 1, 1, 256, 1, 1, 0, stream, args,
                        nullptr) == 0
               ? 0
               : -3;
}

}  // extern "C"
