// capi.cu - the extern "C" entry points of liboomb.so (declared in include/oomb.h).
//
// Shape and alignment checks run on the host before any launch (as Gpu::check,
// crates/oominf-cuda/src/lib.rs:157-160).  Every kernel is launched with
// programmatic stream serialization so a kernel's weight stream can start while
// the previous kernel in the stream drains; each kernel waits
// (griddepcontrol.wait) before it reads anything its predecessor writes.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <mutex>
#include <unordered_map>

#include "../../include/oomb.h"
#include "attn.cuh"
#include "combine.cuh"
#include "decode.cuh"
#include "ep.cuh"
#include "quant.cuh"
#include "route.cuh"
#include "stream.cuh"
#include "tc.cuh"
#include "tcgroup.cuh"
#include "tiers.h"

// CTAs per SM of a stand-alone dense GEMV launch.  Two: both CTAs' consumers
// work at once (twice the warps hiding shared-memory and FMA latency), at the
// cost of the next launch of a dependent chain no longer fitting beside this one
// to stream its weights early; measured on B200, config 1 (4096 x 4096, batch 1,
// back-to-back): 6.08 us with one CTA per SM, 5.33 with two.
#ifndef OOMB_DENSE_CTAS_PER_SM
#define OOMB_DENSE_CTAS_PER_SM 2
#endif
// The same for the stand-alone expert kernels (gate/up, down): two, measured on
// B200 at config 2 (gate/up+SiLU over 8 experts, back-to-back): 9.62 us with one
// CTA per SM (the next kernel streaming beside it), 8.24 with two.  Either is
// correct: an expert kernel lets its dependent launch only after its own
// dependency wait, so a kernel reading tables two launches back finds them
// complete whatever the occupancy.
// Single-GPU one-launch steps of 2 .. OOMB_DECODE_SINGLES_MAX_T tokens group every
// slot on its own (see fused_decode_plan).
#ifndef OOMB_DECODE_SINGLES_MAX_T
#define OOMB_DECODE_SINGLES_MAX_T 16
#endif
#ifndef OOMB_MOE_CTAS_PER_SM
#define OOMB_MOE_CTAS_PER_SM 2
#endif

namespace oomb {
namespace {

// Device error word: bounded waits that run out record a code here.
__device__ unsigned g_device_error;

constexpr int kMaxDevices = 64;

struct DeviceState {
    bool init = false;
    bool ok = false;
    int sms = 0;
    unsigned* err = nullptr;
};

DeviceState g_dev[kMaxDevices];
std::mutex g_dev_mu;

// Per-device state: SM count, error-word address, sm_100 check.
const DeviceState* device_state() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DeviceState& d = g_dev[dev];
    if (!d.init) {
        d.init = true;
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, dev) == cudaSuccess && prop.major == 10) {
            d.sms = prop.multiProcessorCount;
            void* p = nullptr;
            if (cudaGetSymbolAddress(&p, g_device_error) == cudaSuccess) {
                d.err = static_cast<unsigned*>(p);
                d.ok = true;
            }
        }
    }
    return d.ok ? &d : nullptr;
}

// Opts a kernel into more than 48 KB of dynamic shared memory, once per
// (kernel, device): calls made later (for instance during CUDA graph capture)
// find it done and touch nothing but the stream.
std::mutex g_attr_mu;
std::unordered_map<const void*, size_t> g_attr_done[kMaxDevices];

template <typename Kernel>
bool set_smem(Kernel k, size_t bytes) {
    // the default limit covers static and dynamic shared memory together
    if (bytes <= 40 * 1024) return true;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return false;
    const void* key = reinterpret_cast<const void*>(k);
    std::lock_guard<std::mutex> lk(g_attr_mu);
    auto it = g_attr_done[dev].find(key);
    if (it != g_attr_done[dev].end() && it->second >= bytes) return true;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)) !=
        cudaSuccess)
        return false;
    g_attr_done[dev][key] = bytes;
    return true;
}

template <typename Kernel, typename... Args>
int launch(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args... args) {
    if (!set_smem(kernel, smem)) return OOMB_E_LAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...) == cudaSuccess ? OOMB_OK : OOMB_E_LAUNCH;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Where a caller's buffer lives.  Pinned host memory (cudaHostAlloc,
// cudaHostRegister) is reachable from kernels at its mapped device address;
// pageable host memory and unknown pointers are reachable by no kernel.
enum class Mem { none, device, host };
Mem mem_kind(const void* p, const void** dev) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        (void)cudaGetLastError();
        return Mem::none;
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
        *dev = p;
        return Mem::device;
    }
    if (a.type == cudaMemoryTypeHost && a.devicePointer) {
        *dev = a.devicePointer;
        return Mem::host;
    }
    return Mem::none;
}

// ---- streaming kernels ----------------------------------------------------------

// Token slots for units with at most `maxn` assignments (0: unknown), and
// whether more than TB may occur (then P = 1 and chunks of TB are reduced one
// by one against the stage in shared memory).
struct TbP {
    int tb;
    bool chunked;
};
TbP tb_p(int maxn) {
    if (maxn == 1) return {1, false};
    if (maxn == 2) return {2, false};
    return {2, true};
}

// Completes the plan for (PARTS, P) and launches OOMB_MOE_CTAS_PER_SM (expert
// kernels) or OOMB_DENSE_CTAS_PER_SM (dense) CTAs per SM, or one per unit when
// there are fewer.  `groups` bounds the expert groups the kernel can
// see (their count may live on the device); dense launches pass 1.
template <int PARTS, int TB, int P, bool XB, bool MOE, bool EARLY>
int stream_launch_tp(const DeviceState* d, int groups, StreamParams sp, cudaStream_t s) {
    const StreamPlan pl = stream_plan(sp.k, PARTS, P, sp.layout);
    if (pl.stage_bytes > kStageBytes || pl.smem > static_cast<size_t>(kSmemLimit)) return OOMB_E_SHAPE;
    sp.kc = pl.kc;
    sp.ks = pl.ks;
    sp.nsl = pl.nsl;
    sp.rp = pl.rp;
    sp.rpp = pl.rpp;
    sp.nb = pl.nb;
    sp.sr = pl.sr;
    sp.stages = pl.stages;
    sp.slot_bytes = pl.slot_bytes;
    sp.gpe = (sp.nrows + pl.rpp - 1) / pl.rpp;
    const int64_t units = static_cast<int64_t>(groups) * sp.gpe;
    // fp32 activations keep one CTA per SM for a dense launch: measured on B200 at config 1
    // with 1x128 scales, 7.57 us with one, 8.74 with two (bf16: 6.08 with one, 5.33 with two)
    const int max_grid = d->sms * (MOE ? OOMB_MOE_CTAS_PER_SM : (XB ? OOMB_DENSE_CTAS_PER_SM : 1));
    const int grid = units < max_grid ? static_cast<int>(units > 0 ? units : 1) : max_grid;
    if (units * (grid + 1) >= (int64_t{1} << 32)) return OOMB_E_SHAPE;  // the kernel splits units in 32 bits
    if (sp.layout == OOMB_SCALE_128X128)
        return launch(stream_kernel<PARTS, TB, P, XB, MOE, EARLY, true>, dim3(grid), dim3(kThreads), pl.smem, s, sp);
    return launch(stream_kernel<PARTS, TB, P, XB, MOE, EARLY, false>, dim3(grid), dim3(kThreads), pl.smem, s, sp);
}

// Units per pass: as many as kRedV partials per lane allow.
template <int TB>
constexpr int pass_len() {
    return kRedV / (kRows * TB) > 0 ? kRedV / (kRows * TB) : 1;
}

template <int PARTS, bool XB, bool MOE, bool EARLY>
int stream_launch(const DeviceState* d, TbP tp, int groups, const StreamParams& sp, cudaStream_t s) {
    if (tp.chunked) return stream_launch_tp<PARTS, 2, 1, XB, MOE, EARLY>(d, groups, sp, s);
    if (tp.tb == 1) return stream_launch_tp<PARTS, 1, pass_len<1>(), XB, MOE, EARLY>(d, groups, sp, s);
    return stream_launch_tp<PARTS, 2, pass_len<2>(), XB, MOE, EARLY>(d, groups, sp, s);
}

// gate/up + SwiGLU over expert groups; the group count is n_e or *n_e_dev
// (then at most max_groups)
int launch_gate_up(const DeviceState* d, const uint64_t* recs, const int32_t* off, const int32_t* assign_tok,
                   const int32_t* n_e_dev, int n_e, int max_groups, const void* x, bool xbf16, float* h,
                   const oomb_fp8_record* geo, int maxn, bool early, cudaStream_t stream) {
    StreamParams sp{};
    sp.recs = recs;
    sp.off = off;
    sp.assign_tok = assign_tok;
    sp.n_e_dev = n_e_dev;
    sp.n_e_host = n_e;
    sp.w_off[0] = geo->gate_weight;
    sp.w_off[1] = geo->up_weight;
    sp.s_off[0] = geo->gate_scale;
    sp.s_off[1] = geo->up_scale;
    sp.layout = geo->layout;
    sp.k = static_cast<int>(geo->hidden);
    sp.nrows = static_cast<int>(geo->inter);
    sp.x = x;
    sp.y = h;
    sp.err = d->err;
    const int groups = n_e_dev ? max_groups : n_e;
    const TbP tp = tb_p(maxn);
    if (early)
        return xbf16 ? stream_launch<2, true, true, true>(d, tp, groups, sp, stream)
                     : stream_launch<2, false, true, true>(d, tp, groups, sp, stream);
    return xbf16 ? stream_launch<2, true, true, false>(d, tp, groups, sp, stream)
                 : stream_launch<2, false, true, false>(d, tp, groups, sp, stream);
}

// down projection over expert groups
int launch_down(const DeviceState* d, const uint64_t* recs, const int32_t* off, const int32_t* n_e_dev, int n_e,
                int max_groups, const float* h, float* y, const oomb_fp8_record* geo, int maxn, bool early,
                cudaStream_t stream) {
    StreamParams sp{};
    sp.recs = recs;
    sp.off = off;
    sp.n_e_dev = n_e_dev;
    sp.n_e_host = n_e;
    sp.w_off[0] = sp.w_off[1] = geo->down_weight;
    sp.s_off[0] = sp.s_off[1] = geo->down_scale;
    sp.layout = geo->layout;
    sp.k = static_cast<int>(geo->inter);
    sp.nrows = static_cast<int>(geo->hidden);
    sp.x = h;
    sp.y = y;
    sp.err = d->err;
    const int groups = n_e_dev ? max_groups : n_e;
    const TbP tp = tb_p(maxn);
    return early ? stream_launch<1, false, true, true>(d, tp, groups, sp, stream)
                 : stream_launch<1, false, true, false>(d, tp, groups, sp, stream);
}

// ---- tensor-core path ------------------------------------------------------------

// cuTensorMapEncodeTiled, fetched once from the driver through the runtime (the
// library links only the CUDA runtime).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<EncodeTiledFn>(nullptr);
        return reinterpret_cast<EncodeTiledFn>(f);
    }();
    return fn;
}

// Tensor map of a byte matrix [rows, k] (row-major) in boxes of 128 bytes x
// box_rows rows with the 128-byte swizzle the MMA descriptors expect: e4m3
// weights (box 128 x 128; packed tiles are a [tiles * 128, 128] matrix) and the
// split activation images (box 128 x nmma).
bool encode_u8_tiles(CUtensorMap* map, const uint8_t* q, int rows, int k, int box_rows) {
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(k)};
    const cuuint32_t box[2] = {kTcTile, static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(q), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    // As CUTLASS does for drivers up to 13.1 on tensors under 128 KiB.
    int drv = 0;
    if (cudaDriverGetVersion(&drv) == cudaSuccess && drv <= 13010 && static_cast<size_t>(rows) * k < 131072)
        reinterpret_cast<uint64_t*>(map)[1] &= ~(1ull << 21);
    return true;
}

bool encode_fp8_tiles(CUtensorMap* map, const uint8_t* q, int rows, int k) {
    return encode_u8_tiles(map, q, rows, k, kTcTile);
}

size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

// The activation split of one call: terms image [rows_alloc, k] and term scales
// [k/128][tc_sx_stride(rows_alloc)] at the given workspace offsets.
struct XsLayout {
    size_t xs_off, sx_off, end;
    int rows_alloc, sx_stride;
};

XsLayout xs_layout(size_t base, int rows_alloc, int k) {
    XsLayout x{};
    x.rows_alloc = rows_alloc;
    x.sx_stride = tc_sx_stride(rows_alloc);
    x.xs_off = align256(base);
    x.sx_off = align256(x.xs_off + static_cast<size_t>(rows_alloc) * k);
    x.end = align256(x.sx_off + static_cast<size_t>(k / kTcTile) * x.sx_stride * 4);
    return x;
}

int launch_xsplit(bool x_bf16, const XsParams& xp, cudaStream_t s) {
    const int64_t warps = static_cast<int64_t>(xp.a_cover) * xp.kblocks;
    const int64_t blocks = (warps + 7) / 8;
    if (blocks <= 0 || blocks > 0x7fffffff) return OOMB_E_SHAPE;
    return x_bf16 ? launch(xsplit_kernel<true>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, xp)
                  : launch(xsplit_kernel<false>, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, s, xp);
}

struct TcPlan {
    int grid, tiles, kblocks, nmma, stages, nbufs, tmem_cols;
    size_t smem, counters_off, partial_off, ws_bytes;
    XsLayout xs;
};

// Up to 4 tokens two CTAs fit on an SM (registers and shared memory), so the next
// launch of a dependent chain can start streaming; larger batches take one.
constexpr size_t kTcSmemLimit2 = 110 * 1024, kTcSmemLimit1 = 210 * 1024;
constexpr int kTcMinTokens = 2;  // oomb_gemm_fp8 takes the tensor cores from this batch size
constexpr int kTcMaxTF32 = 32;   // fp32 x: six terms a token, at most 192 MMA columns

bool tc_plan(const DeviceState* d, int t, int n, int k, bool x_bf16, TcPlan& pl) {
    if (t < 1 || t > (x_bf16 ? kTcMaxT : kTcMaxTF32) || n % kTcTile != 0 || k % kTcTile != 0 || n <= 0 || k <= 0)
        return false;
    const int ts = tc_ts(x_bf16);
    pl.kblocks = k / kTcTile;
    pl.tiles = (n / kTcTile) * pl.kblocks;
    pl.grid = pl.tiles < d->sms ? pl.tiles : d->sms;
    pl.nmma = (t * ts + 7) / 8 * 8;
    if (pl.nmma > kTcMaxN) return false;
    pl.nbufs = kTcAccBufs;
    while (pl.nbufs > 2 && pl.nbufs * pl.nmma > 512) pl.nbufs /= 2;
    int cols = 32;
    while (cols < pl.nbufs * pl.nmma) cols *= 2;
    if (cols > 512) return false;
    pl.tmem_cols = cols;
    const size_t limit = t <= 4 ? kTcSmemLimit2 : kTcSmemLimit1;
    auto total = [&](int st) { return tc_smem(st, pl.nmma).total + 1024; };
    pl.stages = kTcMaxStages;
    while (pl.stages > kTcMinStages && total(pl.stages) > limit) pl.stages--;
    pl.smem = total(pl.stages);
    if (pl.smem > 227 * 1024) return false;
    pl.counters_off = 0;
    pl.partial_off = align256(static_cast<size_t>(n / kTcTile) * 4 * 4);
    pl.xs = xs_layout(pl.partial_off + static_cast<size_t>(pl.grid) * 2 * t * kTcTile * 4, pl.nmma, k);
    pl.ws_bytes = pl.xs.end;
    return true;
}

template <bool XB, int MAXT>
int tc_launch_t(const TcPlan& pl, const CUtensorMap& qmap, const CUtensorMap& xmap, const TcParams& tp,
                cudaStream_t s) {
    return launch(tc_gemm_kernel<XB, MAXT>, dim3(pl.grid), dim3(EpiSplit<MAXT>::THREADS), pl.smem, s, qmap, xmap, tp);
}

template <bool XB>
int tc_launch(int t, const TcPlan& pl, const CUtensorMap& qmap, const CUtensorMap& xmap, const TcParams& tp,
              cudaStream_t s) {
    if (t <= 1) return tc_launch_t<XB, 1>(pl, qmap, xmap, tp, s);
    if (t <= 2) return tc_launch_t<XB, 2>(pl, qmap, xmap, tp, s);
    if (t <= 4) return tc_launch_t<XB, 4>(pl, qmap, xmap, tp, s);
    if (t <= 8) return tc_launch_t<XB, 8>(pl, qmap, xmap, tp, s);
    if (t <= 16) return tc_launch_t<XB, 16>(pl, qmap, xmap, tp, s);
    if (t <= 32) return tc_launch_t<XB, 32>(pl, qmap, xmap, tp, s);
    if constexpr (XB) return tc_launch_t<XB, 64>(pl, qmap, xmap, tp, s);
    return OOMB_E_SHAPE;
}

// Grouped tensor-core plan: the chunk (assignments per unit) is the smallest of
// 8, 16, 32, 64 that holds max_per_expert (at most 32 for fp32 x, whose six
// terms a column make 192 B rows), shrunk until the rings fit one CTA per SM;
// 512 tensor-memory columns hold nbufs accumulators of nmma columns.
bool tg_plan(int max_per_expert, bool x_bf16, int n_experts, TgParams& tp, size_t& smem) {
    const int ts = tc_ts(x_bf16);
    const int want = max_per_expert > 0 ? max_per_expert : 64;
    const int ch_max = x_bf16 ? 64 : 32;
    int ch = 8;
    while (ch < want && ch < ch_max) ch *= 2;
    for (; ch >= 8; ch /= 2) {
        const int nmma = ch * ts;
        if (nmma > kTcMaxN) continue;
        int nbufs = kTcAccBufs;
        while (nbufs > 2 && nbufs * nmma > 512) nbufs /= 2;
        if (nbufs * nmma > 512) continue;
        int cols = 32;
        while (cols < nbufs * nmma) cols *= 2;
        int stages = kTcMaxStages;
        auto total = [&](int st) { return tg_smem_bytes(st, nmma, n_experts) + 1024; };
        // the weight-copy warp keeps kTgLag tiles unreleased: the ring needs one more
        while (stages > kTgLag + 1 && total(stages) > kTcSmemLimit1) stages--;
        if (total(stages) > 227 * 1024) continue;
        tp.chunk = ch;
        tp.nmma = nmma;
        tp.nbufs = nbufs;
        tp.tmem_cols = cols;
        tp.stages = stages;
        smem = total(stages);
        return true;
    }
    return false;
}

template <bool XB>
int tg_launch(const TgParams& tp, const CUtensorMap& xmap, int grid, size_t smem, cudaStream_t s) {
    switch (tp.chunk) {
        case 8: return launch(tc_group_kernel<XB, 8>, dim3(grid), dim3(EpiSplit<8>::THREADS), smem, s, xmap, tp);
        case 16: return launch(tc_group_kernel<XB, 16>, dim3(grid), dim3(EpiSplit<16>::THREADS), smem, s, xmap, tp);
        case 32: return launch(tc_group_kernel<XB, 32>, dim3(grid), dim3(EpiSplit<32>::THREADS), smem, s, xmap, tp);
        default:
            if constexpr (XB)
                return launch(tc_group_kernel<XB, 64>, dim3(grid), dim3(EpiSplit<64>::THREADS), smem, s, xmap, tp);
            return OOMB_E_SHAPE;
    }
}


// One projection of the grouped tensor-core GEMM over split activations already
// in ws (layout xl, terms of the activation dtype x_bf16): y[a] = x[row(a)] .
// W_e^T for every assignment of the groups; the group count is n_dev[0] (on the
// device, at most n_experts) or n_experts.
int tiled_projection(const DeviceState* d, const uint64_t* recs, const int32_t* off, const int32_t* n_dev,
                     int n_experts, int max_per_expert, int a_max, bool x_bf16, uint8_t* ws, const XsLayout& xl,
                     float* y, int n, int k, int64_t w_off, int64_t s_off, int layout, cudaStream_t stream) {
    TgParams tp{};
    size_t smem = 0;
    if (!tg_plan(max_per_expert, x_bf16, n_experts, tp, smem)) return OOMB_E_SHAPE;
    CUtensorMap xmap;
    if (!encode_u8_tiles(&xmap, ws + xl.xs_off, xl.rows_alloc, k, tp.nmma)) return OOMB_E_LAUNCH;
    tp.recs = recs;
    tp.off = off;
    tp.n_experts = n_experts;
    tp.n_dev = n_dev;
    tp.a_max = a_max;
    tp.K = k;
    tp.N = n;
    tp.w_off = w_off;
    tp.s_off = s_off;
    tp.layout = layout;
    tp.y = y;
    tp.sx = reinterpret_cast<const float*>(ws + xl.sx_off);
    tp.sx_stride = xl.sx_stride;
    tp.rblocks = n / kTcTile;
    tp.kblocks = k / kTcTile;
    tp.err = d->err;
    return x_bf16 ? tg_launch<true>(tp, xmap, d->sms, smem, stream) : tg_launch<false>(tp, xmap, d->sms, smem, stream);
}

// The one-launch decode (decode.cuh) for up to kDecodeMaxT tokens and routers of
// at most kRouteSmallE experts: its plan, or false when the layer or batch is
// outside what it covers (the chain of kernels serves those).
struct FusedDecode {
    DecodeParams prm;
    size_t smem;
    int grid, tb, p;
};

std::mutex g_occ_mu;
std::unordered_map<const void*, int> g_occ[kMaxDevices];

// CTAs of `kernel` one SM holds at once with `smem` bytes of dynamic shared memory.
template <typename Kernel>
int resident_ctas(Kernel kernel, size_t smem) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
    const void* key = reinterpret_cast<const void*>(kernel);
    {
        std::lock_guard<std::mutex> lk(g_occ_mu);
        auto it = g_occ[dev].find(key);
        if (it != g_occ[dev].end() && (it->second >> 20) == static_cast<int>(smem >> 10)) return it->second & 0xff;
    }
    if (!set_smem(kernel, smem)) return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kThreads, smem) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lk(g_occ_mu);
    g_occ[dev][key] = (static_cast<int>(smem >> 10) << 20) | (n & 0xff);
    return n;
}

template <bool XB, bool BLK, int TB, int P, bool EP>
auto decode_kernel_ptr() {
    return decode_kernel<XB, BLK, TB, P, EP>;
}

template <bool XB, bool BLK, bool EP>
int fused_resident(int tb, size_t smem) {
    return tb == 1 ? resident_ctas(decode_kernel_ptr<XB, BLK, 1, pass_len<1>(), EP>(), smem)
                   : resident_ctas(decode_kernel_ptr<XB, BLK, 2, 1, EP>(), smem);
}

template <bool EP>
int fused_resident_any(bool xbf16, int layout, int tb, size_t smem) {
    return xbf16 ? (layout ? fused_resident<true, true, EP>(tb, smem) : fused_resident<true, false, EP>(tb, smem))
                 : (layout ? fused_resident<false, true, EP>(tb, smem) : fused_resident<false, false, EP>(tb, smem));
}

// ranks > 0: the expert-parallel kernel, this rank's experts E / ranks of them.
bool fused_decode_plan(const DeviceState* d, const oomb_moe_layer* L, int t, bool xbf16, FusedDecode& f,
                       int ranks = 0) {
    const char* env = getenv("OOMB_DECODE_CHAIN");
    if (ranks == 0 && env && env[0] == '1') return false;
    const int E = L->experts, K = L->top_k, H = static_cast<int>(L->geo.hidden), I = static_cast<int>(L->geo.inter);
    const int layout = L->geo.layout;
    if (t < 1 || t > kDecodeMaxT || E > kRouteSmallE || H > kRouteMaxH) return false;
    const int TA = ranks > 0 ? ranks * t : t;  // tokens whose slots this rank groups
    if (ranks > 0 && (E % ranks || E / ranks > kThreads)) return false;
    // expert parallelism groups every received slot on its own, and so does a
    // single-GPU step of up to OOMB_DECODE_SINGLES_MAX_T tokens: one assignment per group
    const bool singles = ranks == 0 && t > 1 && t <= OOMB_DECODE_SINGLES_MAX_T;
    const TbP tp = ranks > 0 || singles ? TbP{1, false} : tb_p(TA);
    f.tb = tp.chunked ? 2 : tp.tb;
    f.p = f.tb == 1 ? pass_len<1>() : 1;
    const StreamPlan pg = stream_plan(H, 2, f.p, layout), pd = stream_plan(I, 1, f.p, layout);
    if (pg.stage_bytes > kStageBytes || pd.stage_bytes > kStageBytes) return false;
    const int gpe_g = (I + pg.rpp - 1) / pg.rpp, gpe_d = (H + pd.rpp - 1) / pd.rpp;
    const int64_t groups_max = static_cast<int64_t>(TA) * K > E ? static_cast<int64_t>(TA) * K : E;
    if (gpe_d > kDecodeMaxGroups || groups_max * (gpe_g > gpe_d ? gpe_g : gpe_d) * 1025 >= (int64_t{1} << 32))
        return false;
    const int slot = pg.slot_bytes > pd.slot_bytes ? pg.slot_bytes : pd.slot_bytes;
    const int ms_g = f.p * 4 + f.p * 2 * pg.sr * pg.nb, ms_d = f.p * 4 + f.p * pd.sr * pd.nb;
    const int meta_stride = ms_g > ms_d ? ms_g : ms_d;
    const DecodeTabs dt = decode_tabs(t, K, E, TA);
    // [ring][bars][red][meta][chunk][tables]
    const size_t bars = (2 * kMaxStages + 2 * kMetaBufs) * sizeof(uint64_t);
    const size_t red = 2 * kWarps * kRedV * sizeof(float);
    const size_t meta = static_cast<size_t>(kMetaBufs) * meta_stride * 4;
    const size_t fixed = bars + red + ((meta + 15) & ~static_cast<size_t>(15)) + 8 * sizeof(int) + dt.total;
    int stages = kMaxStages;
    while (stages > 2 && static_cast<size_t>(stages) * slot + fixed > static_cast<size_t>(kSmemLimit)) stages--;
    const size_t ring = static_cast<size_t>(stages) * slot;
    if (ring + fixed > static_cast<size_t>(kSmemLimit)) return false;
    f.smem = ring + fixed;
    // every CTA must be resident at once (grid barriers)
    const int occ = ranks > 0 ? fused_resident_any<true>(xbf16, layout, f.tb, f.smem)
                              : fused_resident_any<false>(xbf16, layout, f.tb, f.smem);
    if (occ < 1) return false;
    f.grid = d->sms * (occ < OOMB_STREAM_CTAS_PER_SM ? occ : OOMB_STREAM_CTAS_PER_SM);
    // router rows: kWarps per CTA (one per consumer warp) on the first ceil(E / kWarps) CTAs
    const int rows_per_cta = E < kWarps ? E : kWarps;
    if ((E + kWarps - 1) / kWarps > f.grid || ring < decode_ring_borrow(t, H, E, K, rows_per_cta, 0)) return false;
    // the activations are staged in the ring after the router rows when they fit
    const size_t x_bytes = static_cast<size_t>(t) * H * (xbf16 ? 2 : 4);
    const bool x_staged = ring >= decode_ring_borrow(t, H, E, K, rows_per_cta, x_bytes);

    DecodeParams& q = f.prm;
    q = DecodeParams{};
    q.stages = stages;
    q.slot_bytes = slot;
    q.meta_stride = meta_stride;
    q.off_bars = static_cast<int>(ring);
    q.off_red = static_cast<int>(ring + bars);
    q.off_meta = static_cast<int>(ring + bars + red);
    q.off_chunk = static_cast<int>(q.off_meta + ((meta + 15) & ~static_cast<size_t>(15)));
    q.off_tabs = q.off_chunk + 8 * static_cast<int>(sizeof(int));
    q.x_off = x_staged ? rows_per_cta * H * 2 : -1;
    auto fill = [&](StreamParams& sp, const StreamPlan& pl, int k, int nrows, int gpe) {
        sp.layout = layout;
        sp.k = k;
        sp.nrows = nrows;
        sp.kc = pl.kc;
        sp.ks = pl.ks;
        sp.nsl = pl.nsl;
        sp.rp = pl.rp;
        sp.rpp = pl.rpp;
        sp.nb = pl.nb;
        sp.sr = pl.sr;
        sp.stages = stages;
        sp.slot_bytes = slot;
        sp.gpe = gpe;
        sp.err = d->err;
    };
    fill(q.gu, pg, H, I, gpe_g);
    q.gu.w_off[0] = L->geo.gate_weight;
    q.gu.w_off[1] = L->geo.up_weight;
    q.gu.s_off[0] = L->geo.gate_scale;
    q.gu.s_off[1] = L->geo.up_scale;
    fill(q.dn, pd, I, H, gpe_d);
    q.dn.w_off[0] = q.dn.w_off[1] = L->geo.down_weight;
    q.dn.s_off[0] = q.dn.s_off[1] = L->geo.down_scale;
    // one token: down and combine per row group of 8 rows (intermediate up to 2048:
    // at most four 512-column slabs; a slot's 8 rows fit a ring slot; a group's
    // stages fit the ring at once, since its consumers release them together)
    const Down1 d1 = down1_plan(K, I, slot);
    q.dn1 = OOMB_DECODE_DOWN1 && ranks == 0 && t == 1 && I <= 2048 && d1.spp >= 1 && d1.nst <= stages;
    q.singles = singles ? 1 : 0;
    return true;
}

template <bool XB, bool BLK, bool EP>
int fused_launch(const FusedDecode& f, cudaStream_t s) {
    if (f.tb == 1)
        return launch(decode_kernel<XB, BLK, 1, pass_len<1>(), EP>, dim3(f.grid), dim3(kThreads), f.smem, s, f.prm);
    return launch(decode_kernel<XB, BLK, 2, 1, EP>, dim3(f.grid), dim3(kThreads), f.smem, s, f.prm);
}

template <bool EP>
int fused_launch_any(bool xbf16, int layout, const FusedDecode& f, cudaStream_t s) {
    if (xbf16) return layout ? fused_launch<true, true, EP>(f, s) : fused_launch<true, false, EP>(f, s);
    return layout ? fused_launch<false, true, EP>(f, s) : fused_launch<false, false, EP>(f, s);
}

}  // namespace
}  // namespace oomb

using namespace oomb;

namespace {
// Zeroes the sync words of the no-alloc entry point's fixed scratch on the
// current device (defined with that entry point, at the end of this file).
bool noalloc_reset_sync();
}  // namespace

extern "C" {

int oomb_silu_mul_rows(const float* gu, void* y, int y_dtype, int rows, int n, oomb_stream stream) {
    if (!gu || !y) return OOMB_E_ARG;
    if (y_dtype != OOMB_F32 && y_dtype != OOMB_BF16) return OOMB_E_ARG;
    if (rows < 0 || n <= 0 || n % 4 != 0) return OOMB_E_SHAPE;
    if (!aligned16(gu) || !aligned16(y)) return OOMB_E_ALIGN;
    if (rows == 0) return OOMB_OK;
    if (!device_state()) return OOMB_E_DEVICE;
    const int64_t quads = static_cast<int64_t>(rows) * n / 4;
    const dim3 grid(static_cast<unsigned>((quads + 255) / 256));
    return y_dtype == OOMB_BF16 ? launch(silu_mul_rows_kernel<true>, grid, dim3(256), 0, stream, gu, y, rows, n)
                                : launch(silu_mul_rows_kernel<false>, grid, dim3(256), 0, stream, gu, y, rows, n);
}

size_t oomb_gemm_fp8_workspace_bytes(int t, int n, int k, int x_dtype) {
    const DeviceState* d = device_state();
    TcPlan pl{};
    if (!d || (x_dtype != OOMB_F32 && x_dtype != OOMB_BF16) || !tc_plan(d, t, n, k, x_dtype == OOMB_BF16, pl))
        return 0;
    return pl.ws_bytes;
}

int oomb_pack_fp8_tiles(const uint8_t* q, int n, int k, uint8_t* tiles, oomb_stream stream) {
    if (!q || !tiles) return OOMB_E_ARG;
    if (n <= 0 || k <= 0 || n % kTcTile || k % kTcTile) return OOMB_E_SHAPE;
    if (!aligned16(q) || !aligned16(tiles)) return OOMB_E_ALIGN;
    if (!device_state()) return OOMB_E_DEVICE;
    pack_fp8_tiles_kernel<<<static_cast<unsigned>((n / kTcTile) * (k / kTcTile)), 256, 0, stream>>>(q, k, tiles);
    return cudaGetLastError() == cudaSuccess ? OOMB_OK : OOMB_E_LAUNCH;
}

int oomb_gemm_fp8_tc(const void* x, int x_dtype, const uint8_t* q, int q_format, const float* scale,
                     int scale_layout, void* y, int y_dtype, int t, int n, int k, void* workspace,
                     size_t workspace_bytes, oomb_stream stream) {
    if (q_format != OOMB_Q_ROWS && q_format != OOMB_Q_TILES) return OOMB_E_ARG;
    if (!x || !q || !scale || !y || !workspace) return OOMB_E_ARG;
    if ((x_dtype != OOMB_F32 && x_dtype != OOMB_BF16) || (y_dtype != OOMB_F32 && y_dtype != OOMB_BF16) ||
        (scale_layout != OOMB_SCALE_1X128 && scale_layout != OOMB_SCALE_128X128))
        return OOMB_E_ARG;
    if (!aligned16(x) || !aligned16(q) || !aligned16(scale) || !aligned16(y) || !aligned16(workspace))
        return OOMB_E_ALIGN;
    if (t == 0) return OOMB_OK;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    const bool xb = x_dtype == OOMB_BF16;
    TcPlan pl{};
    if (!tc_plan(d, t, n, k, xb, pl)) return OOMB_E_SHAPE;
    if (workspace_bytes < pl.ws_bytes) return OOMB_E_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    CUtensorMap qmap, xmap;
    const bool packed = q_format == OOMB_Q_TILES;
    if (!(packed ? encode_fp8_tiles(&qmap, q, pl.tiles * kTcTile, kTcTile) : encode_fp8_tiles(&qmap, q, n, k)) ||
        !encode_u8_tiles(&xmap, ws + pl.xs.xs_off, pl.xs.rows_alloc, k, pl.nmma))
        return OOMB_E_LAUNCH;
    // 1. split x once into e4m3 terms (rows past t * TS are zero terms)
    XsParams xp{};
    xp.x = x;
    xp.a_host = t;
    xp.a_cover = (pl.nmma + tc_ts(xb) - 1) / tc_ts(xb);
    xp.zero_pad = 1;
    xp.K = k;
    xp.kblocks = pl.kblocks;
    xp.xs = ws + pl.xs.xs_off;
    xp.rows_alloc = pl.xs.rows_alloc;
    xp.sx = reinterpret_cast<float*>(ws + pl.xs.sx_off);
    xp.sx_stride = pl.xs.sx_stride;
    int rc = launch_xsplit(xb, xp, stream);
    if (rc) return rc;
    // 2. the GEMM, its weight stream starting under the split
    TcParams tp{};
    tp.T = t;
    tp.K = k;
    tp.nrows = n;
    tp.scale = scale;
    tp.layout = scale_layout;
    tp.y = y;
    tp.y_bf16 = y_dtype == OOMB_BF16;
    tp.counters = reinterpret_cast<unsigned*>(ws + pl.counters_off);
    tp.partial = reinterpret_cast<float*>(ws + pl.partial_off);
    tp.sx = xp.sx;
    tp.sx_stride = xp.sx_stride;
    tp.tiles = pl.tiles;
    tp.kblocks = pl.kblocks;
    tp.q_tiles = packed;
    tp.nmma = pl.nmma;
    tp.stages = pl.stages;
    tp.nbufs = pl.nbufs;
    tp.tmem_cols = pl.tmem_cols;
    tp.err = d->err;
    return xb ? tc_launch<true>(t, pl, qmap, xmap, tp, stream) : tc_launch<false>(t, pl, qmap, xmap, tp, stream);
}

size_t oomb_moe_tiled_fp8_workspace_bytes(int max_assignments, int k, int x_dtype) {
    if (max_assignments <= 0 || k <= 0 || k % kTcTile || (x_dtype != OOMB_F32 && x_dtype != OOMB_BF16)) return 0;
    return xs_layout(0, max_assignments * tc_ts(x_dtype == OOMB_BF16), k).end;
}

int oomb_moe_tiled_fp8(const uint64_t* recs, const int32_t* off, const int32_t* rows, int n_experts,
                       int max_per_expert, int max_assignments, const void* x, int x_dtype, float* y, int n, int k,
                       int64_t w_off, int64_t s_off, int scale_layout, void* workspace, size_t workspace_bytes,
                       oomb_stream stream) {
    if (!recs || !off || !x || !y || !workspace) return OOMB_E_ARG;
    if ((x_dtype != OOMB_F32 && x_dtype != OOMB_BF16) ||
        (scale_layout != OOMB_SCALE_1X128 && scale_layout != OOMB_SCALE_128X128) || max_per_expert < 0)
        return OOMB_E_ARG;
    if (n <= 0 || k <= 0 || n % kTcTile || k % kTcTile || n_experts < 0 || n_experts > kTgMaxExperts ||
        max_assignments <= 0)
        return OOMB_E_SHAPE;
    if (!aligned16(x) || !aligned16(y) || !aligned16(workspace) || (w_off & 15) || (s_off & 3) || w_off < 0 ||
        s_off < 0)
        return OOMB_E_ALIGN;
    if (n_experts == 0) return OOMB_OK;
    const bool xb = x_dtype == OOMB_BF16;
    const XsLayout xl = xs_layout(0, max_assignments * tc_ts(xb), k);
    if (workspace_bytes < xl.end) return OOMB_E_WORKSPACE;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    TgParams probe{};
    size_t smem = 0;
    if (!tg_plan(max_per_expert, xb, n_experts, probe, smem)) return OOMB_E_SHAPE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    // 1. split every assignment's row (through `rows`) once into e4m3 terms;
    //    the assignment count is off[n_experts], on the device
    XsParams xp{};
    xp.x = x;
    xp.rows = rows;
    xp.first = off;
    xp.count = off + n_experts;
    xp.a_cover = max_assignments;
    xp.zero_pad = 0;
    xp.K = k;
    xp.kblocks = k / kTcTile;
    xp.xs = ws + xl.xs_off;
    xp.rows_alloc = xl.rows_alloc;
    xp.sx = reinterpret_cast<float*>(ws + xl.sx_off);
    xp.sx_stride = xl.sx_stride;
    int rc = launch_xsplit(xb, xp, stream);
    if (rc) return rc;
    // 2. the grouped GEMM
    return tiled_projection(d, recs, off, nullptr, n_experts, max_per_expert, max_assignments, xb, ws, xl, y, n, k,
                            w_off, s_off, scale_layout, stream);
}

int oomb_moe_swiglu_range(const float* g, const float* u, float* h, int64_t start, int64_t end,
                          oomb_stream stream) {
    if (!g || !u || !h) return OOMB_E_ARG;
    if (start < 0 || end < start) return OOMB_E_SHAPE;
    if (start == end) return OOMB_OK;
    if (!device_state()) return OOMB_E_DEVICE;
    const int64_t blocks = (end - start + 255) / 256;
    if (blocks > 0x7fffffff) return OOMB_E_SHAPE;
    return launch(swiglu_range_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream, g, u, h, start,
                  end);
}


const char* oomb_version(void) { return "oomb 0.1 (sm_100a)"; }

const char* oomb_status_string(int status) {
    switch (status) {
        case OOMB_OK: return "ok";
        case OOMB_E_SHAPE: return "buffer too small or shape unsupported";
        case OOMB_E_ALIGN: return "pointer or stride not 16-byte aligned";
        case OOMB_E_LAUNCH: return "CUDA launch failed";
        case OOMB_E_TIMEOUT: return "a bounded device wait ran out";
        case OOMB_E_ARG: return "null pointer or bad enum";
        case OOMB_E_DEVICE: return "no usable sm_100 device";
        case OOMB_E_WORKSPACE: return "workspace too small";
        default: return "unknown status";
    }
}

int oomb_device_error(int* code, int clear) {
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    unsigned v = 0;
    if (cudaMemcpy(&v, d->err, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return OOMB_E_LAUNCH;
    if (code) *code = static_cast<int>(v);
    if (clear && v) {
        const unsigned z = 0;
        if (cudaMemcpy(d->err, &z, sizeof(z), cudaMemcpyHostToDevice) != cudaSuccess) return OOMB_E_LAUNCH;
        // a wait that ran out can leave counts behind in the sync words of the
        // library's own decode scratch, which no caller can reach: zero them too
        if (!noalloc_reset_sync()) return OOMB_E_LAUNCH;
    }
    return v ? OOMB_E_TIMEOUT : OOMB_OK;
}

int oomb_set_wait_limit(uint64_t ns) {
    if (!device_state()) return OOMB_E_DEVICE;
    const unsigned long long v = ns ? static_cast<unsigned long long>(ns) : kWaitLimitNs;
    return cudaMemcpyToSymbol(g_wait_limit_ns, &v, sizeof(v)) == cudaSuccess ? OOMB_OK : OOMB_E_LAUNCH;
}

int oomb_gemm_fp8(const void* x, int x_dtype, const uint8_t* q, const float* scale,
                  int scale_layout, void* y, int y_dtype, int t, int n, int k, void* workspace,
                  size_t workspace_bytes, oomb_stream stream) {
    if (!x || !q || !scale || !y) return OOMB_E_ARG;
    if ((x_dtype != OOMB_F32 && x_dtype != OOMB_BF16) || (y_dtype != OOMB_F32 && y_dtype != OOMB_BF16) ||
        (scale_layout != OOMB_SCALE_1X128 && scale_layout != OOMB_SCALE_128X128))
        return OOMB_E_ARG;
    if (t < 0 || n <= 0 || k <= 0 || k % 16 != 0) return OOMB_E_SHAPE;
    if (!aligned16(x) || !aligned16(q) || !aligned16(scale) || !aligned16(y)) return OOMB_E_ALIGN;
    if (t == 0) return OOMB_OK;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    // Batches of two or more tokens go to the tensor cores when the caller gave a
    // workspace and the shape allows (the CUDA-core stream is faster at one token).
    if (t >= kTcMinTokens && workspace) {
        TcPlan pl{};
        if (tc_plan(d, t, n, k, x_dtype == OOMB_BF16, pl) && workspace_bytes >= pl.ws_bytes && aligned16(workspace))
            return oomb_gemm_fp8_tc(x, x_dtype, q, OOMB_Q_ROWS, scale, scale_layout, y, y_dtype, t, n, k, workspace,
                                    workspace_bytes, stream);
    }
    // Token chunks are reduced per stage, which needs whole rows in a stage:
    // with K split over several stages (k > 4096) run 2-token launches.
    const bool k_split = (k + 511) / 512 > 8;
    const int per = k_split ? 2 : t;
    const size_t xs = x_dtype == OOMB_BF16 ? 2 : 4, ys = y_dtype == OOMB_BF16 ? 2 : 4;
    for (int t0 = 0; t0 < t; t0 += per) {
        const int tc = t - t0 < per ? t - t0 : per;
        StreamParams sp{};
        sp.q = q;
        sp.scale = scale;
        sp.layout = scale_layout;
        sp.k = k;
        sp.nrows = n;
        sp.x = static_cast<const uint8_t*>(x) + static_cast<size_t>(t0) * k * xs;
        sp.t = tc;
        sp.y = static_cast<uint8_t*>(y) + static_cast<size_t>(t0) * n * ys;
        sp.y_bf16 = y_dtype == OOMB_BF16;
        sp.err = d->err;
        const TbP tp = tb_p(tc);
        const int rc = x_dtype == OOMB_BF16 ? stream_launch<1, true, false, false>(d, tp, 1, sp, stream)
                                            : stream_launch<1, false, false, false>(d, tp, 1, sp, stream);
        if (rc) return rc;
    }
    return OOMB_OK;
}

int oomb_router_logits(const void* x, int x_dtype, const uint16_t* w, float* logits, int t, int e,
                       int hidden, oomb_stream stream) {
    if (!x || !w || !logits) return OOMB_E_ARG;
    if (x_dtype != OOMB_F32 && x_dtype != OOMB_BF16) return OOMB_E_ARG;
    if (t < 0 || e <= 0 || hidden <= 0 || hidden % 8 != 0) return OOMB_E_SHAPE;
    if (!aligned16(x) || !aligned16(w)) return OOMB_E_ALIGN;
    if (t == 0) return OOMB_OK;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    RouteParams p{};
    p.x = x;
    p.x_bf16 = x_dtype == OOMB_BF16;
    p.w = w;
    p.logits = logits;
    p.T = t;
    p.H = hidden;
    p.E = e;
    p.do_logits = 1;
    p.err = d->err;
    // one router row per warp
    const int grid = (e + kRouteThreads / 32 - 1) / (kRouteThreads / 32);
    const size_t smem = route_smem(t, hidden, e, 0, p.x_bf16 != 0, true, false, false).total;
    return p.x_bf16 ? launch(route_kernel<true>, dim3(grid), dim3(kRouteThreads), smem, stream, p)
                    : launch(route_kernel<false>, dim3(grid), dim3(kRouteThreads), smem, stream, p);
}

int oomb_router_topk(const float* logits, int32_t* ids, float* weights, int t, int e, int k,
                     oomb_stream stream) {
    if (!logits || !ids || !weights) return OOMB_E_ARG;
    if (t < 0 || k <= 0 || k > 32 || e > 8192 || k > e) return OOMB_E_SHAPE;
    if (t == 0) return OOMB_OK;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    RouteParams p{};
    p.logits = const_cast<float*>(logits);
    p.T = t;
    p.E = e;
    p.K = k;
    p.ids = ids;
    p.weights = weights;
    p.do_topk = 1;
    p.err = d->err;
    const int grid = (t + 7) / 8;
    const size_t smem = route_smem(t, 0, e, k, false, false, true, false).total;
    return launch(route_kernel<false>, dim3(grid), dim3(kRouteThreads), smem, stream, p);
}

int oomb_moe_gate_up_fp8(const uint64_t* recs, const int32_t* off, const int32_t* assign_tok,
                         int n_experts, const void* x, int x_dtype, float* h,
                         const oomb_fp8_record* geo, int max_per_expert, int flags,
                         oomb_stream stream) {
    if (!recs || !off || !assign_tok || !x || !h || !geo) return OOMB_E_ARG;
    if (flags & ~OOMB_TABLES_READY) return OOMB_E_ARG;
    if (x_dtype != OOMB_F32 && x_dtype != OOMB_BF16) return OOMB_E_ARG;
    if (geo->layout != OOMB_SCALE_1X128 && geo->layout != OOMB_SCALE_128X128) return OOMB_E_ARG;
    if (n_experts < 0 || max_per_expert < 0 || geo->hidden <= 0 || geo->inter <= 0 || geo->hidden % 16 ||
        geo->inter % 16 || geo->hidden > 4096)
        return OOMB_E_SHAPE;
    if ((geo->gate_weight | geo->up_weight | geo->gate_scale | geo->up_scale) & 15) return OOMB_E_ALIGN;
    if (!aligned16(x)) return OOMB_E_ALIGN;
    if (n_experts == 0) return OOMB_OK;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    return launch_gate_up(d, recs, off, assign_tok, nullptr, n_experts, n_experts, x, x_dtype == OOMB_BF16, h, geo,
                          max_per_expert, (flags & OOMB_TABLES_READY) != 0, stream);
}

int oomb_moe_down_fp8(const uint64_t* recs, const int32_t* off, int n_experts, const float* h,
                      float* y, const oomb_fp8_record* geo, int max_per_expert, int flags,
                      oomb_stream stream) {
    if (!recs || !off || !h || !y || !geo) return OOMB_E_ARG;
    if (flags & ~OOMB_TABLES_READY) return OOMB_E_ARG;
    if (geo->layout != OOMB_SCALE_1X128 && geo->layout != OOMB_SCALE_128X128) return OOMB_E_ARG;
    if (n_experts < 0 || max_per_expert < 0 || geo->hidden <= 0 || geo->inter <= 0 || geo->hidden % 16 ||
        geo->inter % 16 || geo->inter > 4096)
        return OOMB_E_SHAPE;
    if ((geo->down_weight | geo->down_scale) & 15) return OOMB_E_ALIGN;
    if (!aligned16(h)) return OOMB_E_ALIGN;
    if (n_experts == 0) return OOMB_OK;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    return launch_down(d, recs, off, nullptr, n_experts, n_experts, h, y, geo, max_per_expert,
                       (flags & OOMB_TABLES_READY) != 0, stream);
}

int oomb_moe_combine_slots(const float* y, const int32_t* slot_assign, const float* w, void* out,
                           int out_dtype, int t, int h, int k, oomb_stream stream) {
    if (!y || !slot_assign || !w || !out) return OOMB_E_ARG;
    if (out_dtype != OOMB_F32 && out_dtype != OOMB_BF16) return OOMB_E_ARG;
    if (t < 0 || h <= 0 || k <= 0 || h % 4) return OOMB_E_SHAPE;
    if (!aligned16(y) || !aligned16(out)) return OOMB_E_ALIGN;
    if (t == 0) return OOMB_OK;
    if (!device_state()) return OOMB_E_DEVICE;
    const int64_t quads = static_cast<int64_t>(t) * h / 4;
    const dim3 grid(static_cast<unsigned>((quads + 255) / 256));
    return out_dtype == OOMB_BF16
               ? launch(combine_slots_kernel<true>, grid, dim3(256), 0, stream, y, slot_assign, w, out, t, h, k)
               : launch(combine_slots_kernel<false>, grid, dim3(256), 0, stream, y, slot_assign, w, out, t, h, k);
}

int oomb_moe_combine(const float* routed, const float* shared, const float* gate_logit, float* out,
                     int t, int h, oomb_stream stream) {
    if (!routed || !shared || !gate_logit || !out) return OOMB_E_ARG;
    if (t < 0 || h <= 0) return OOMB_E_SHAPE;
    if (t == 0) return OOMB_OK;
    if (!device_state()) return OOMB_E_DEVICE;
    const int64_t n = static_cast<int64_t>(t) * h;
    return launch(moe_combine_kernel<false>, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, stream,
                  routed, shared, gate_logit, static_cast<void*>(out), t, h);
}

// ---- decode attention ----------------------------------------------------------

namespace {
struct AttnPlan {
    int splits;
    size_t counters_off, part_off, ws_bytes;
};

bool attn_plan(const DeviceState* d, int batch, int heads, int kv_heads, int head_dim, int kv_max, AttnPlan& pl) {
    if (batch <= 0 || heads <= 0 || kv_heads <= 0 || heads % kv_heads || head_dim != 128 || kv_max < 0) return false;
    const int G = heads / kv_heads;
    if (G != 1 && G != 2 && G != 4 && G != 8) return false;
    const int64_t pairs = static_cast<int64_t>(batch) * kv_heads;
    if (pairs > 65535LL * 65535LL) return false;
    // as many CTAs as are resident at once (four per SM by registers, three at
    // G = 8), rounded down to whole splits so the grid is one wave: a grid just
    // past one wave runs a second wave as long as the first; each warp at least
    // one chunk of positions
    const int resident = G <= 4 ? 4 : 3;
    const int64_t want = static_cast<int64_t>(d->sms) * resident / pairs;
    const int cp = 32 / G < 8 ? 32 / G : 8;
    const int64_t most = (static_cast<int64_t>(kv_max) + cp * kAttnWarps - 1) / (cp * kAttnWarps);
    pl.splits = static_cast<int>(want < most ? want : (most > 0 ? most : 1));
    if (pl.splits < 1) pl.splits = 1;
    if (pl.splits > kAttnMaxSplits) pl.splits = kAttnMaxSplits;  // the merge stages a factor per split
    pl.counters_off = 0;
    pl.part_off = (static_cast<size_t>(pairs) * 4 + 255) & ~static_cast<size_t>(255);
    pl.ws_bytes = pl.part_off + static_cast<size_t>(pairs) * pl.splits * G * (head_dim + 4) * 4;
    return true;
}
}  // namespace

size_t oomb_attention_decode_workspace_bytes(int batch, int heads, int kv_heads, int head_dim, int kv_max) {
    const DeviceState* d = device_state();
    AttnPlan pl{};
    if (!d || !attn_plan(d, batch, heads, kv_heads, head_dim, kv_max, pl)) return 0;
    return pl.ws_bytes;
}

int oomb_attention_decode(const void* q, int q_dtype, const uint16_t* k_cache, const uint16_t* v_cache,
                          int64_t seq_stride, const int32_t* kv_len, int kv_len_all, void* out, int out_dtype,
                          int batch, int heads, int kv_heads, int head_dim, int kv_max, float scale, void* workspace,
                          size_t workspace_bytes, oomb_stream stream) {
    if (!q || !k_cache || !v_cache || !out || !workspace) return OOMB_E_ARG;
    if ((q_dtype != OOMB_F32 && q_dtype != OOMB_BF16) || (out_dtype != OOMB_F32 && out_dtype != OOMB_BF16))
        return OOMB_E_ARG;
    if (batch < 0 || kv_max < 0 || seq_stride < 0 || (!kv_len && (kv_len_all < 0 || kv_len_all > kv_max)))
        return OOMB_E_SHAPE;
    if (batch > 1 && seq_stride < static_cast<int64_t>(kv_max) * kv_heads * head_dim) return OOMB_E_SHAPE;
    if (!aligned16(q) || !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(out) || !aligned16(workspace) ||
        (seq_stride % 8))
        return OOMB_E_ALIGN;
    if (batch == 0) return OOMB_OK;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    AttnPlan pl{};
    if (!attn_plan(d, batch, heads, kv_heads, head_dim, kv_max, pl)) return OOMB_E_SHAPE;
    if (workspace_bytes < pl.ws_bytes) return OOMB_E_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    AttnParams p{};
    p.q = q;
    p.q_bf16 = q_dtype == OOMB_BF16;
    p.k = k_cache;
    p.v = v_cache;
    p.seq_stride = seq_stride;
    p.kv_len = kv_len;
    p.kv_len_host = kv_len_all;
    p.out = out;
    p.out_bf16 = out_dtype == OOMB_BF16;
    p.B = batch;
    p.H = heads;
    p.Hkv = kv_heads;
    p.kv_max = kv_max;
    p.splits = pl.splits;
    p.scale = scale;
    p.part = reinterpret_cast<float*>(ws + pl.part_off);
    p.counters = reinterpret_cast<unsigned*>(ws + pl.counters_off);
    p.err = d->err;
    const dim3 grid(static_cast<unsigned>(pl.splits), static_cast<unsigned>(kv_heads), static_cast<unsigned>(batch));
    switch (heads / kv_heads) {
        case 1: return launch(attn_decode_kernel<1, 128>, grid, dim3(kAttnThreads), 0, stream, p);
        case 2: return launch(attn_decode_kernel<2, 128>, grid, dim3(kAttnThreads), 0, stream, p);
        case 4: return launch(attn_decode_kernel<4, 128>, grid, dim3(kAttnThreads), 0, stream, p);
        default: return launch(attn_decode_kernel<8, 128>, grid, dim3(kAttnThreads), 0, stream, p);
    }
}

int oomb_kv_append(const void* src, int src_dtype, int64_t src_row_stride, uint16_t* cache, int64_t seq_stride,
                   const int32_t* start, int start_all, int batch, int t, int kv_heads, int head_dim, int kv_max,
                   oomb_stream stream) {
    if (!src || !cache) return OOMB_E_ARG;
    if (src_dtype != OOMB_F32 && src_dtype != OOMB_BF16) return OOMB_E_ARG;
    if (batch < 0 || t < 0 || kv_heads <= 0 || head_dim <= 0 || kv_max <= 0 || (kv_heads * head_dim) % 8 ||
        src_row_stride < static_cast<int64_t>(kv_heads) * head_dim ||
        (batch > 1 && seq_stride < static_cast<int64_t>(kv_max) * kv_heads * head_dim))
        return OOMB_E_SHAPE;
    if (!start && (start_all < 0 || start_all + t > kv_max)) return OOMB_E_SHAPE;
    if (!aligned16(src) || !aligned16(cache) || (src_row_stride % 8) || (seq_stride % 8)) return OOMB_E_ALIGN;
    if (batch == 0 || t == 0) return OOMB_OK;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    KvAppendParams p{};
    p.src = src;
    p.src_bf16 = src_dtype == OOMB_BF16;
    p.src_row_stride = src_row_stride;
    p.cache = cache;
    p.seq_stride = seq_stride;
    p.start = start;
    p.start_all = start_all;
    p.B = batch;
    p.t = t;
    p.Hkv = kv_heads;
    p.D = head_dim;
    p.kv_max = kv_max;
    p.err = d->err;
    const int64_t n = static_cast<int64_t>(batch) * t * kv_heads * head_dim / 8;
    return launch(kv_append_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, stream, p);
}

// ---- fused decode ------------------------------------------------------------

namespace {
struct DecodeLayout {
    size_t ticket, sync, logits, ids, weights, n_active, active, off, assign_tok, slot_assign, recs_active,
        h, y, xs, xs_bytes, total;
};

// Batches from this size take the grouped tensor-core path in oomb_moe_decode_fp8
// (route, split x once, gate and up, SwiGLU, split h, down, combine) when the
// layer's shapes allow it; below it the one-launch kernel (or the CUDA-core chain).
// The environment variable OOMB_DECODE_TILED_MIN_T overrides it (>= 2).
// Measured on B200 with the one-launch kernel grouping every slot on its own: config 2
// at 16 tokens 205 us one launch vs 265 us tensor cores, config 4 401 vs 430 us at 14 and
// a tie at 16; so the tensor cores from 17 tokens, where the one-launch kernel ends.
constexpr int kDecodeTiledMinT = 17;

int decode_tiled_min_t() {
    const char* env = getenv("OOMB_DECODE_TILED_MIN_T");
    if (env && env[0]) {
        const int v = atoi(env);
        if (v >= 2) return v;
    }
    return kDecodeTiledMinT;
}

size_t up256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

// ranks > 1: the expert-parallel kernel, whose h holds the slots of every rank's tokens.
// y [A, H] fp32 also holds the device copy of activations passed in host memory
// (T x H, at most 4 bytes each): a step writes y only after its last read of x.
DecodeLayout decode_layout(int t, const oomb_moe_layer* L, int ranks = 1) {
    DecodeLayout d{};
    const size_t T = t, E = L->experts, K = L->top_k, A = T * K, AH = static_cast<size_t>(ranks) * A;
    const size_t H = L->geo.hidden, I = L->geo.inter;
    size_t o = 0;
    d.ticket = o; o += 256;
    d.sync = o; o = up256(o + kSyncWords * 4);
    d.logits = o; o = up256(o + T * E * 4);
    d.ids = o; o = up256(o + A * 4);
    d.weights = o; o = up256(o + A * 4);
    d.n_active = o; o += 256;
    d.active = o; o = up256(o + E * 4);
    d.off = o; o = up256(o + (E + 1) * 4);
    d.assign_tok = o; o = up256(o + A * 4);
    d.slot_assign = o; o = up256(o + A * 4);
    d.recs_active = o; o = up256(o + E * 8);
    d.h = o; o = up256(o + AH * I * 4);
    d.y = o; o = up256(o + A * H * 4);
    d.xs = o;
    d.xs_bytes = 0;
    if (ranks == 1 && t >= 2 && H % kTcTile == 0 && I % kTcTile == 0) {
        // the grouped tensor-core path's split activations: x (up to six terms, fp32 x) for
        // gate and up, then h (fp32, six terms) for down, one after the other in one region
        const size_t a = xs_layout(0, static_cast<int>(A) * tc_ts(false), static_cast<int>(H)).end;
        const size_t b = xs_layout(0, static_cast<int>(A) * tc_ts(false), static_cast<int>(I)).end;
        d.xs_bytes = a > b ? a : b;
        o = up256(o + d.xs_bytes);
    }
    d.total = o;
    return d;
}

int check_layer(const oomb_moe_layer* L) {
    if (!L || !L->router_w || !L->recs) return OOMB_E_ARG;
    const oomb_fp8_record& g = L->geo;
    if (g.layout != OOMB_SCALE_1X128 && g.layout != OOMB_SCALE_128X128) return OOMB_E_ARG;
    if (L->hidden != g.hidden || L->experts <= 0 || L->experts > 8192 || L->top_k <= 0 ||
        L->top_k > 32 || L->top_k > L->experts)
        return OOMB_E_SHAPE;
    if (g.hidden <= 0 || g.inter <= 0 || g.hidden % 16 || g.inter % 16 || g.hidden > 4096 || g.inter > 4096)
        return OOMB_E_SHAPE;
    if ((g.gate_weight | g.up_weight | g.down_weight | g.gate_scale | g.up_scale | g.down_scale) & 15)
        return OOMB_E_ALIGN;
    return OOMB_OK;
}
}  // namespace

size_t oomb_moe_decode_workspace_bytes(int t, const oomb_moe_layer* layer) {
    if (t <= 0 || check_layer(layer) != OOMB_OK) return 0;
    return decode_layout(t, layer).total;
}

int oomb_workspace_clear(void* workspace, size_t bytes, oomb_stream stream) {
    if (!workspace) return OOMB_E_ARG;
    return cudaMemsetAsync(workspace, 0, bytes, stream) == cudaSuccess ? OOMB_OK : OOMB_E_LAUNCH;
}

int oomb_moe_decode_fp8(const oomb_moe_layer* L, const void* x, int x_dtype, int t, void* out,
                        int out_dtype, int32_t* ids, float* weights, void* workspace,
                        size_t workspace_bytes, oomb_stream stream) {
    int rc = check_layer(L);
    if (rc) return rc;
    if (!x || !out || !workspace) return OOMB_E_ARG;
    if ((x_dtype != OOMB_F32 && x_dtype != OOMB_BF16) || (out_dtype != OOMB_F32 && out_dtype != OOMB_BF16))
        return OOMB_E_ARG;
    if (t < 0) return OOMB_E_SHAPE;
    if (!aligned16(x) || !aligned16(out) || !aligned16(workspace) || !aligned16(L->router_w))
        return OOMB_E_ALIGN;
    if (t == 0) return OOMB_OK;
    const DecodeLayout lay = decode_layout(t, L);
    if (workspace_bytes < lay.total) return OOMB_E_WORKSPACE;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const int E = L->experts, K = L->top_k, H = L->hidden;
    const int A = t * K;
    // x and out may be pinned host memory; the workspace, ids and weights are device memory
    const void* xv = nullptr;
    const void* ov = nullptr;
    const void* unused = nullptr;
    const Mem xk = mem_kind(x, &xv), ok = mem_kind(out, &ov);
    if (xk == Mem::none || ok == Mem::none || mem_kind(workspace, &unused) != Mem::device ||
        (ids && mem_kind(ids, &unused) != Mem::device) || (weights && mem_kind(weights, &unused) != Mem::device))
        return OOMB_E_ARG;
    out = const_cast<void*>(ov);
    if (xk == Mem::host) {
        // staged into the y region, which the step writes only after its last read of x
        const int64_t n16 = static_cast<int64_t>(t) * H * (x_dtype == OOMB_BF16 ? 2 : 4) / 16;
        const int64_t blocks = (n16 + 255) / 256;
        rc = launch(stage_host_kernel, dim3(static_cast<unsigned>(blocks < d->sms ? blocks : d->sms)), dim3(256), 0,
                    stream, reinterpret_cast<uint4*>(ws + lay.y), static_cast<const uint4*>(xv), n16);
        if (rc) return rc;
        x = ws + lay.y;
    } else {
        x = xv;
    }

    const bool xb = x_dtype == OOMB_BF16;
    const int I = static_cast<int>(L->geo.inter);
    bool tiled = t >= decode_tiled_min_t() && lay.xs_bytes > 0 && H >= 2 * I && E <= kTgMaxExperts &&
                 (getenv("OOMB_DECODE_CHAIN") == nullptr || getenv("OOMB_DECODE_CHAIN")[0] != '1');
    if (tiled) {
        const size_t need = xs_layout(0, A * tc_ts(xb), H).end;
        TgParams probe{};
        size_t smem = 0;
        tiled = need <= lay.xs_bytes && tg_plan(t, xb, A < E ? A : E, probe, smem) &&
                tg_plan(t, false, A < E ? A : E, probe, smem);
    }
    FusedDecode f;
    if (!tiled && fused_decode_plan(d, L, t, x_dtype == OOMB_BF16, f)) {
        // the whole step in one persistent launch
        DecodeParams& q = f.prm;
        q.r.x = x;
        q.r.x_bf16 = x_dtype == OOMB_BF16;
        q.r.w = L->router_w;
        q.r.logits = reinterpret_cast<float*>(ws + lay.logits);
        q.r.T = t;
        q.r.H = H;
        q.r.E = E;
        q.r.K = K;
        q.r.recs_all = L->recs;
        q.r.err = d->err;
        q.gu.x = x;
        q.gu.y = ws + lay.h;
        q.dn.x = ws + lay.h;
        q.dn.y = ws + lay.y;
        q.sync = reinterpret_cast<unsigned*>(ws + lay.sync);
        q.ids_out = ids ? ids : reinterpret_cast<int32_t*>(ws + lay.ids);
        q.w_out = weights ? weights : reinterpret_cast<float*>(ws + lay.weights);
        q.out = out;
        q.out_bf16 = out_dtype == OOMB_BF16;
        return fused_launch_any<false>(x_dtype == OOMB_BF16, L->geo.layout, f, stream);
    }

    // 1. router logits + top-k + grouping (one launch; the last CTA groups)
    RouteParams rp{};
    rp.x = x;
    rp.x_bf16 = x_dtype == OOMB_BF16;
    rp.w = L->router_w;
    rp.logits = reinterpret_cast<float*>(ws + lay.logits);
    rp.T = t;
    rp.H = H;
    rp.E = E;
    rp.K = K;
    rp.ids = ids ? ids : reinterpret_cast<int32_t*>(ws + lay.ids);
    rp.weights = weights ? weights : reinterpret_cast<float*>(ws + lay.weights);
    rp.recs_all = L->recs;
    rp.n_active = reinterpret_cast<int32_t*>(ws + lay.n_active);
    rp.active = reinterpret_cast<int32_t*>(ws + lay.active);
    rp.off = reinterpret_cast<int32_t*>(ws + lay.off);
    rp.assign_tok = reinterpret_cast<int32_t*>(ws + lay.assign_tok);
    rp.slot_assign = reinterpret_cast<int32_t*>(ws + lay.slot_assign);
    rp.recs_active = reinterpret_cast<uint64_t*>(ws + lay.recs_active);
    rp.ticket = reinterpret_cast<unsigned*>(ws + lay.ticket);
    rp.do_logits = rp.do_topk = rp.do_group = 1;
    rp.err = d->err;
    {
        // one router row per warp; the last CTA to finish runs top-k and grouping
        const int grid = (E + kRouteThreads / 32 - 1) / (kRouteThreads / 32);
        const size_t smem = route_smem(t, H, E, K, rp.x_bf16 != 0, true, true, true).total;
        if (smem > 200 * 1024) return OOMB_E_SHAPE;
        rc = rp.x_bf16 ? launch(route_kernel<true>, dim3(grid), dim3(kRouteThreads), smem, stream, rp)
                       : launch(route_kernel<false>, dim3(grid), dim3(kRouteThreads), smem, stream, rp);
        if (rc) return rc;
    }
    const int max_e = A < E ? A : E;
    float* h = reinterpret_cast<float*>(ws + lay.h);
    float* y = reinterpret_cast<float*>(ws + lay.y);
    if (tiled) {
        // The grouped tensor-core path (Moe::run_group's tiled branch, moe.rs:746-758):
        // x rows split once for gate and up, g and u in the y region (x staged there
        // from host memory is dead once split), SwiGLU into h, h split, down into y.
        // An expert gets at most one assignment per token: at most t per group.
        uint8_t* xsr = ws + lay.xs;
        float* g = y;
        float* u = y + static_cast<size_t>(A) * I;
        const XsLayout xl1 = xs_layout(0, A * tc_ts(xb), H);
        XsParams xp{};
        xp.x = x;
        xp.rows = rp.assign_tok;
        xp.a_host = A;
        xp.a_cover = A;
        xp.K = H;
        xp.kblocks = H / kTcTile;
        xp.xs = xsr + xl1.xs_off;
        xp.rows_alloc = xl1.rows_alloc;
        xp.sx = reinterpret_cast<float*>(xsr + xl1.sx_off);
        xp.sx_stride = xl1.sx_stride;
        if ((rc = launch_xsplit(xb, xp, stream))) return rc;
        if ((rc = tiled_projection(d, rp.recs_active, rp.off, rp.n_active, max_e, t, A, xb, xsr, xl1, g, I, H,
                                   L->geo.gate_weight, L->geo.gate_scale, L->geo.layout, stream)))
            return rc;
        if ((rc = tiled_projection(d, rp.recs_active, rp.off, rp.n_active, max_e, t, A, xb, xsr, xl1, u, I, H,
                                   L->geo.up_weight, L->geo.up_scale, L->geo.layout, stream)))
            return rc;
        const int64_t n_h = static_cast<int64_t>(A) * I;
        if ((rc = launch(swiglu_range_kernel, dim3(static_cast<unsigned>((n_h + 255) / 256)), dim3(256), 0, stream,
                         static_cast<const float*>(g), static_cast<const float*>(u), h, int64_t{0}, n_h)))
            return rc;
        const XsLayout xl2 = xs_layout(0, A * tc_ts(false), I);
        xp = XsParams{};
        xp.x = h;
        xp.a_host = A;
        xp.a_cover = A;
        xp.K = I;
        xp.kblocks = I / kTcTile;
        xp.xs = xsr + xl2.xs_off;
        xp.rows_alloc = xl2.rows_alloc;
        xp.sx = reinterpret_cast<float*>(xsr + xl2.sx_off);
        xp.sx_stride = xl2.sx_stride;
        if ((rc = launch_xsplit(false, xp, stream))) return rc;
        if ((rc = tiled_projection(d, rp.recs_active, rp.off, rp.n_active, max_e, t, A, false, xsr, xl2, y, H, I,
                                   L->geo.down_weight, L->geo.down_scale, L->geo.layout, stream)))
            return rc;
    } else {
    // 2. gate/up + SiLU over the active experts (an expert gets at most one
    //    assignment per token, so at most t)
    rc = launch_gate_up(d, rp.recs_active, rp.off, rp.assign_tok, rp.n_active, 0, max_e, x, rp.x_bf16 != 0, h,
                        &L->geo, t, false, stream);
    if (rc) return rc;
    // 3. down; its producer starts streaming weights while gate/up finishes
    rc = launch_down(d, rp.recs_active, rp.off, rp.n_active, 0, max_e, h, y, &L->geo, t, true, stream);
    if (rc) return rc;
    }
    // 4. slot-order combine
    const int64_t quads = static_cast<int64_t>(t) * H / 4;
    const dim3 cgrid(static_cast<unsigned>((quads + 255) / 256));
    return out_dtype == OOMB_BF16
               ? launch(combine_slots_kernel<true>, cgrid, dim3(256), 0, stream, static_cast<const float*>(y),
                        static_cast<const int32_t*>(rp.slot_assign), static_cast<const float*>(rp.weights), out, t, H, K)
               : launch(combine_slots_kernel<false>, cgrid, dim3(256), 0, stream, static_cast<const float*>(y),
                        static_cast<const int32_t*>(rp.slot_assign), static_cast<const float*>(rp.weights), out, t, H, K);
}

// ---- a whole MoE layer: shared expert + routed experts --------------------------

namespace {
struct LayerLayout {
    size_t dec, routed, gu, sact, shared, gate, tc1, tc2, total;
    size_t dec_bytes, tc1_bytes, tc2_bytes;
};

int check_shared(const oomb_shared_expert* S, const oomb_moe_layer* L) {
    if (!S || !S->gate_up_q || !S->gate_up_scale || !S->down_q || !S->down_scale) return OOMB_E_ARG;
    if (S->scale_layout != OOMB_SCALE_1X128 && S->scale_layout != OOMB_SCALE_128X128) return OOMB_E_ARG;
    if (S->hidden != L->hidden || S->inter <= 0 || S->inter % 16) return OOMB_E_SHAPE;
    if (!aligned16(S->gate_up_q) || !aligned16(S->gate_up_scale) || !aligned16(S->down_q) ||
        !aligned16(S->down_scale) || (S->gate_w && !aligned16(S->gate_w)))
        return OOMB_E_ALIGN;
    return OOMB_OK;
}

bool layer_layout(const DeviceState* d, int t, const oomb_moe_layer* L, const oomb_shared_expert* S, bool x_bf16,
                  LayerLayout& w) {
    const size_t T = t, H = L->hidden, SI = S->inter;
    w = LayerLayout{};
    w.dec_bytes = decode_layout(t, L).total;
    TcPlan p1{}, p2{};
    // the shared expert's two GEMVs take the tensor cores from two tokens when the shapes allow
    if (t >= kTcMinTokens && tc_plan(d, t, static_cast<int>(2 * SI), static_cast<int>(H), x_bf16, p1))
        w.tc1_bytes = p1.ws_bytes;
    if (t >= kTcMinTokens && tc_plan(d, t, static_cast<int>(H), static_cast<int>(SI), false, p2))
        w.tc2_bytes = p2.ws_bytes;
    size_t o = 0;
    w.dec = o; o = up256(o + w.dec_bytes);
    w.tc1 = o; o = up256(o + w.tc1_bytes);
    w.tc2 = o; o = up256(o + w.tc2_bytes);
    w.routed = o; o = up256(o + T * H * 4);
    w.gu = o; o = up256(o + T * 2 * SI * 4);
    w.sact = o; o = up256(o + T * SI * 4);
    w.shared = o; o = up256(o + T * H * 4);
    w.gate = o; o = up256(o + T * 4);
    w.total = o;
    return true;
}
}  // namespace

size_t oomb_moe_layer_workspace_bytes(int t, const oomb_moe_layer* layer, const oomb_shared_expert* shared,
                                      int x_dtype) {
    if (t <= 0 || check_layer(layer) != OOMB_OK || check_shared(shared, layer) != OOMB_OK) return 0;
    if (x_dtype != OOMB_F32 && x_dtype != OOMB_BF16) return 0;
    const DeviceState* d = device_state();
    LayerLayout w;
    if (!d || !layer_layout(d, t, layer, shared, x_dtype == OOMB_BF16, w)) return 0;
    return w.total;
}

int oomb_moe_layer_decode_fp8(const oomb_moe_layer* L, const oomb_shared_expert* S, const void* x, int x_dtype,
                              int t, void* out, int out_dtype, int32_t* ids, float* weights, void* workspace,
                              size_t workspace_bytes, oomb_stream stream) {
    int rc = check_layer(L);
    if (rc) return rc;
    if ((rc = check_shared(S, L))) return rc;
    if (!x || !out || !workspace) return OOMB_E_ARG;
    if ((x_dtype != OOMB_F32 && x_dtype != OOMB_BF16) || (out_dtype != OOMB_F32 && out_dtype != OOMB_BF16))
        return OOMB_E_ARG;
    if (t < 0) return OOMB_E_SHAPE;
    if (!aligned16(x) || !aligned16(out) || !aligned16(workspace)) return OOMB_E_ALIGN;
    if (t == 0) return OOMB_OK;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    LayerLayout w;
    if (!layer_layout(d, t, L, S, x_dtype == OOMB_BF16, w)) return OOMB_E_SHAPE;
    if (workspace_bytes < w.total) return OOMB_E_WORKSPACE;
    const void* unused = nullptr;
    if (mem_kind(x, &unused) != Mem::device || mem_kind(out, &unused) != Mem::device) return OOMB_E_ARG;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const int H = L->hidden, SI = S->inter;
    float* gu = reinterpret_cast<float*>(ws + w.gu);
    float* sact = reinterpret_cast<float*>(ws + w.sact);
    float* shared = reinterpret_cast<float*>(ws + w.shared);
    float* gate = reinterpret_cast<float*>(ws + w.gate);
    float* routed = reinterpret_cast<float*>(ws + w.routed);
    // 1. the shared expert (gate/up GEMV, SwiGLU, down GEMV) and its gate logit
    //    (Moe::shared, crates/oominf-models-qwen/src/moe.rs:498-527), queued first
    rc = oomb_gemm_fp8(x, x_dtype, S->gate_up_q, S->gate_up_scale, S->scale_layout, gu, OOMB_F32, t, 2 * SI, H,
                       w.tc1_bytes ? ws + w.tc1 : nullptr, w.tc1_bytes, stream);
    if (rc) return rc;
    rc = oomb_silu_mul_rows(gu, sact, OOMB_F32, t, SI, stream);
    if (rc) return rc;
    rc = oomb_gemm_fp8(sact, OOMB_F32, S->down_q, S->down_scale, S->scale_layout, shared, OOMB_F32, t, H, SI,
                       w.tc2_bytes ? ws + w.tc2 : nullptr, w.tc2_bytes, stream);
    if (rc) return rc;
    if (S->gate_w) {
        rc = oomb_router_logits(x, x_dtype, S->gate_w, gate, t, 1, H, stream);
        if (rc) return rc;
    }
    // 2. the routed experts: the fused decode step, fp32 out
    rc = oomb_moe_decode_fp8(L, x, x_dtype, t, routed, OOMB_F32, ids, weights, ws + w.dec, w.dec_bytes, stream);
    if (rc) return rc;
    // 3. out = routed + sigmoid(gate) * shared (moe_combine, ops.cu:311-316)
    const int64_t n = static_cast<int64_t>(t) * H;
    const dim3 grid(static_cast<unsigned>((n + 255) / 256));
    const float* g = S->gate_w ? gate : nullptr;
    return out_dtype == OOMB_BF16
               ? launch(moe_combine_kernel<true>, grid, dim3(256), 0, stream, static_cast<const float*>(routed),
                        static_cast<const float*>(shared), g, out, t, H)
               : launch(moe_combine_kernel<false>, grid, dim3(256), 0, stream, static_cast<const float*>(routed),
                        static_cast<const float*>(shared), g, out, t, H);
}

namespace {
int ep_xb(int x_dtype) { return x_dtype == OOMB_BF16 ? 2 : (x_dtype == OOMB_F32 ? 4 : 0); }

bool ep_peer_of(const oomb_ep_peer* q, EpPeer& p) {
    if (!q || !q->peers || !q->mailbox || q->ranks <= 0 || q->rank < 0 || q->rank >= q->ranks || q->t_max <= 0 ||
        q->top_k <= 0 || q->hidden <= 0 || q->hidden % 16 || ep_xb(q->x_dtype) == 0 || !aligned16(q->mailbox))
        return false;
    p.peers = reinterpret_cast<const unsigned long long*>(q->peers);
    p.mailbox = static_cast<uint8_t*>(q->mailbox);
    p.ranks = q->ranks;
    p.rank = q->rank;
    p.t_max = q->t_max;
    p.k = q->top_k;
    p.h = q->hidden;
    p.xb = ep_xb(q->x_dtype);
    p.err = nullptr;
    return true;
}
}  // namespace

size_t oomb_moe_decode_ep_workspace_bytes(int t, int ranks, const oomb_moe_layer* layer) {
    if (t <= 0 || ranks <= 0 || check_layer(layer) != OOMB_OK) return 0;
    return decode_layout(t, layer, ranks).total;
}

int oomb_moe_decode_ep_fp8(const oomb_moe_layer* L, const oomb_ep_peer* q, const void* x, int x_dtype, int t,
                           void* out, int out_dtype, int32_t* ids, float* weights, void* workspace,
                           size_t workspace_bytes, oomb_stream stream) {
    int rc = check_layer(L);
    if (rc) return rc;
    EpPeer ep;
    if (!ep_peer_of(q, ep) || !x || !out || !workspace) return OOMB_E_ARG;
    if ((x_dtype != OOMB_F32 && x_dtype != OOMB_BF16) || (out_dtype != OOMB_F32 && out_dtype != OOMB_BF16) ||
        x_dtype != q->x_dtype)
        return OOMB_E_ARG;
    if (q->hidden != L->hidden || q->top_k != L->top_k || L->experts % q->ranks) return OOMB_E_SHAPE;
    if (t <= 0 || t > q->t_max) return OOMB_E_SHAPE;
    if (!aligned16(x) || !aligned16(out) || !aligned16(workspace) || !aligned16(L->router_w)) return OOMB_E_ALIGN;
    const DecodeLayout lay = decode_layout(t, L, q->ranks);
    if (workspace_bytes < lay.total) return OOMB_E_WORKSPACE;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    ep.err = d->err;
    // x and out may be pinned host memory (as for oomb_moe_decode_fp8)
    const void* xv = nullptr;
    const void* ov = nullptr;
    const void* unused = nullptr;
    const Mem xk = mem_kind(x, &xv), okind = mem_kind(out, &ov);
    if (xk == Mem::none || okind == Mem::none || mem_kind(workspace, &unused) != Mem::device ||
        (ids && mem_kind(ids, &unused) != Mem::device) || (weights && mem_kind(weights, &unused) != Mem::device))
        return OOMB_E_ARG;
    out = const_cast<void*>(ov);
    if (xk == Mem::host) {
        // staged into the y region (unused by the expert-parallel step) once the previous kernel has completed
        const int64_t n16 = static_cast<int64_t>(t) * L->hidden * (x_dtype == OOMB_BF16 ? 2 : 4) / 16;
        const int64_t blocks = (n16 + 255) / 256;
        const int rs = launch(stage_host_kernel, dim3(static_cast<unsigned>(blocks < d->sms ? blocks : d->sms)),
                              dim3(256), 0, stream, reinterpret_cast<uint4*>(static_cast<uint8_t*>(workspace) + lay.y),
                              static_cast<const uint4*>(xv), n16);
        if (rs) return rs;
        x = static_cast<uint8_t*>(workspace) + lay.y;
    } else {
        x = xv;
    }
    FusedDecode f;
    if (!fused_decode_plan(d, L, t, x_dtype == OOMB_BF16, f, q->ranks)) return OOMB_E_SHAPE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const EpMailbox mb = ep_mailbox(q->ranks, q->t_max, q->top_k, q->hidden, ep.xb);
    DecodeParams& p = f.prm;
    p.r.x = x;
    p.r.x_bf16 = x_dtype == OOMB_BF16;
    p.r.w = L->router_w;
    p.r.logits = reinterpret_cast<float*>(ws + lay.logits);
    p.r.T = t;
    p.r.H = L->hidden;
    p.r.E = L->experts;
    p.r.K = L->top_k;
    p.r.recs_all = L->recs;  // this rank's records
    p.r.err = d->err;
    p.gu.x = static_cast<uint8_t*>(q->mailbox) + mb.x;  // every rank's activations, as received
    p.gu.y = ws + lay.h;
    p.dn.x = ws + lay.h;
    p.dn.y = nullptr;
    p.dn.ep_peers = reinterpret_cast<const unsigned long long*>(q->peers);
    p.dn.ep_back_off = static_cast<int64_t>(mb.back_words);
    p.dn.ep_rank = q->rank;
    p.dn.ep_tk = t * L->top_k;
    p.sync = reinterpret_cast<unsigned*>(ws + lay.sync);
    p.ids_out = ids ? ids : reinterpret_cast<int32_t*>(ws + lay.ids);
    p.w_out = weights ? weights : reinterpret_cast<float*>(ws + lay.weights);
    p.out = out;
    p.out_bf16 = out_dtype == OOMB_BF16;
    p.ep = ep;
    p.epr = L->experts / q->ranks;
    return fused_launch_any<true>(x_dtype == OOMB_BF16, L->geo.layout, f, stream);
}

// ---- expert parallelism -------------------------------------------------------

int oomb_ep_meta(const int32_t* ids, int t, int k, int experts_per_rank, int ranks, int32_t* meta,
                 oomb_stream stream) {
    if (!ids || !meta) return OOMB_E_ARG;
    if (t < 0 || k <= 0 || k > 32 || experts_per_rank <= 0 || ranks <= 0) return OOMB_E_SHAPE;
    if (t == 0) return OOMB_OK;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    const int64_t n = static_cast<int64_t>(ranks) * t * k;
    const unsigned grid = static_cast<unsigned>(n / kEpThreads + 1 < 1024 ? n / kEpThreads + 1 : 1024);
    return launch(ep_meta_kernel, dim3(grid), dim3(kEpThreads), 0, stream, ids, t, k, experts_per_rank, ranks, meta,
                  d->err);
}

int oomb_ep_group(const int32_t* recv_meta, int ranks, int t, int k, int experts_per_rank, const uint64_t* recs_local,
                  int32_t* n_active, int32_t* off, int32_t* assign_row, int32_t* assign_ret, uint64_t* recs_active,
                  oomb_stream stream) {
    if (!recv_meta || !recs_local || !n_active || !off || !assign_row || !assign_ret || !recs_active)
        return OOMB_E_ARG;
    if (ranks <= 0 || t <= 0 || k <= 0 || k > 32 || experts_per_rank <= 0 || experts_per_rank > 8192)
        return OOMB_E_SHAPE;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    const size_t smem = 2 * static_cast<size_t>(experts_per_rank) * 4;
    return launch(ep_group_kernel, dim3(1), dim3(kEpThreads), smem, stream, recv_meta, ranks, t, k, experts_per_rank,
                  recs_local, n_active, off, assign_row, assign_ret, recs_active, d->err);
}

int oomb_moe_experts_fp8(const uint64_t* recs_active, const int32_t* off, const int32_t* assign_tok,
                         const int32_t* n_active, int max_active, const void* x, int x_dtype, float* h, float* y,
                         const oomb_fp8_record* geo, int max_per_expert, oomb_stream stream) {
    if (!recs_active || !off || !assign_tok || !n_active || !x || !h || !y || !geo) return OOMB_E_ARG;
    if (x_dtype != OOMB_F32 && x_dtype != OOMB_BF16) return OOMB_E_ARG;
    if (geo->layout != OOMB_SCALE_1X128 && geo->layout != OOMB_SCALE_128X128) return OOMB_E_ARG;
    if (max_active <= 0 || geo->hidden <= 0 || geo->inter <= 0 || geo->hidden % 16 || geo->inter % 16 ||
        geo->hidden > 4096 || geo->inter > 4096)
        return OOMB_E_SHAPE;
    if (!aligned16(x) || !aligned16(h) || !aligned16(y)) return OOMB_E_ALIGN;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    const int maxn = max_per_expert > 0 ? max_per_expert : 0;
    int rc = launch_gate_up(d, recs_active, off, assign_tok, n_active, 0, max_active, x, x_dtype == OOMB_BF16, h, geo,
                            maxn, false, stream);
    if (rc) return rc;
    return launch_down(d, recs_active, off, n_active, 0, max_active, h, y, geo, maxn, true, stream);
}

size_t oomb_moe_experts_tiled_fp8_workspace_bytes(int max_assignments, const oomb_fp8_record* geo, int x_dtype) {
    if (max_assignments <= 0 || !geo || (x_dtype != OOMB_F32 && x_dtype != OOMB_BF16)) return 0;
    const int H = static_cast<int>(geo->hidden), I = static_cast<int>(geo->inter);
    if (H <= 0 || I <= 0 || H % kTcTile || I % kTcTile || H < 2 * I) return 0;
    // x split for gate and up, then h (fp32: six terms) for down, one after the other
    const size_t a = xs_layout(0, max_assignments * tc_ts(x_dtype == OOMB_BF16), H).end;
    const size_t b = xs_layout(0, max_assignments * tc_ts(false), I).end;
    return a > b ? a : b;
}

int oomb_moe_experts_tiled_fp8(const uint64_t* recs_active, const int32_t* off, const int32_t* assign_tok,
                               const int32_t* n_active, int max_active, int max_assignments, const void* x,
                               int x_dtype, float* h, float* y, const oomb_fp8_record* geo, int max_per_expert,
                               void* workspace, size_t workspace_bytes, oomb_stream stream) {
    if (!recs_active || !off || !assign_tok || !n_active || !x || !h || !y || !geo || !workspace) return OOMB_E_ARG;
    if (x_dtype != OOMB_F32 && x_dtype != OOMB_BF16) return OOMB_E_ARG;
    if (geo->layout != OOMB_SCALE_1X128 && geo->layout != OOMB_SCALE_128X128) return OOMB_E_ARG;
    const int H = static_cast<int>(geo->hidden), I = static_cast<int>(geo->inter);
    if (max_active <= 0 || max_active > kTgMaxExperts || max_assignments <= 0 || max_per_expert <= 0 || H <= 0 ||
        I <= 0 || H % kTcTile || I % kTcTile || H < 2 * I || H > 4096 || I > 4096)
        return OOMB_E_SHAPE;
    if (!aligned16(x) || !aligned16(h) || !aligned16(y) || !aligned16(workspace)) return OOMB_E_ALIGN;
    const size_t need = oomb_moe_experts_tiled_fp8_workspace_bytes(max_assignments, geo, x_dtype);
    if (need == 0) return OOMB_E_SHAPE;
    if (workspace_bytes < need) return OOMB_E_WORKSPACE;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    const bool xb = x_dtype == OOMB_BF16;
    const int A = max_assignments;
    uint8_t* xsr = static_cast<uint8_t*>(workspace);
    // g and u in y (H >= 2I), whose rows down overwrites only after SwiGLU has read them;
    // the assignment count is off[*n_active] on the device: the splits cover A rows and
    // skip the ones past it
    float* g = y;
    float* u = y + static_cast<size_t>(A) * I;
    const XsLayout xl1 = xs_layout(0, A * tc_ts(xb), H);
    XsParams xp{};
    xp.x = x;
    xp.rows = assign_tok;
    xp.count = off;
    xp.count_idx = n_active;
    xp.a_host = A;
    xp.a_cover = A;
    xp.K = H;
    xp.kblocks = H / kTcTile;
    xp.xs = xsr + xl1.xs_off;
    xp.rows_alloc = xl1.rows_alloc;
    xp.sx = reinterpret_cast<float*>(xsr + xl1.sx_off);
    xp.sx_stride = xl1.sx_stride;
    int rc = launch_xsplit(xb, xp, stream);
    if (rc) return rc;
    if ((rc = tiled_projection(d, recs_active, off, n_active, max_active, max_per_expert, A, xb, xsr, xl1, g, I, H,
                               geo->gate_weight, geo->gate_scale, geo->layout, stream)))
        return rc;
    if ((rc = tiled_projection(d, recs_active, off, n_active, max_active, max_per_expert, A, xb, xsr, xl1, u, I, H,
                               geo->up_weight, geo->up_scale, geo->layout, stream)))
        return rc;
    const int64_t n_h = static_cast<int64_t>(A) * I;
    if ((rc = launch(swiglu_range_kernel, dim3(static_cast<unsigned>((n_h + 255) / 256)), dim3(256), 0, stream,
                     static_cast<const float*>(g), static_cast<const float*>(u), h, int64_t{0}, n_h)))
        return rc;
    const XsLayout xl2 = xs_layout(0, A * tc_ts(false), I);
    xp = XsParams{};
    xp.x = h;
    xp.count = off;
    xp.count_idx = n_active;
    xp.a_host = A;
    xp.a_cover = A;
    xp.K = I;
    xp.kblocks = I / kTcTile;
    xp.xs = xsr + xl2.xs_off;
    xp.rows_alloc = xl2.rows_alloc;
    xp.sx = reinterpret_cast<float*>(xsr + xl2.sx_off);
    xp.sx_stride = xl2.sx_stride;
    if ((rc = launch_xsplit(false, xp, stream))) return rc;
    return tiled_projection(d, recs_active, off, n_active, max_active, max_per_expert, A, false, xsr, xl2, y, H, I,
                            geo->down_weight, geo->down_scale, geo->layout, stream);
}

int oomb_ep_scatter(const float* y, const int32_t* n_active, const int32_t* off, const int32_t* assign_ret, int h,
                    int max_rows, float* ret, oomb_stream stream) {
    if (!y || !n_active || !off || !assign_ret || !ret) return OOMB_E_ARG;
    if (h <= 0 || h % 4 || max_rows < 0) return OOMB_E_SHAPE;
    if (!aligned16(y) || !aligned16(ret)) return OOMB_E_ALIGN;
    if (max_rows == 0) return OOMB_OK;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    const int64_t n = static_cast<int64_t>(max_rows) * (h / 4);
    const unsigned grid = static_cast<unsigned>(n / 256 + 1 < 4 * d->sms ? n / 256 + 1 : 4 * d->sms);
    return launch(ep_scatter_kernel, dim3(grid), dim3(256), 0, stream, y, n_active, off, assign_ret, h, ret);
}

int oomb_ep_combine(const float* back, const int32_t* ids, const float* w, int t, int k, int h, int experts_per_rank,
                    int ranks, void* out, int out_dtype, oomb_stream stream) {
    if (!back || !ids || !w || !out) return OOMB_E_ARG;
    if (out_dtype != OOMB_F32 && out_dtype != OOMB_BF16) return OOMB_E_ARG;
    if (t < 0 || k <= 0 || h <= 0 || h % 4 || experts_per_rank <= 0 || ranks <= 0) return OOMB_E_SHAPE;
    if (!aligned16(back) || !aligned16(out)) return OOMB_E_ALIGN;
    if (t == 0) return OOMB_OK;
    if (!device_state()) return OOMB_E_DEVICE;
    const int64_t quads = static_cast<int64_t>(t) * h / 4;
    const dim3 grid(static_cast<unsigned>((quads + 255) / 256));
    return out_dtype == OOMB_BF16
               ? launch(ep_combine_kernel<true>, grid, dim3(256), 0, stream, back, ids, w, t, k, h, experts_per_rank,
                        ranks, out)
               : launch(ep_combine_kernel<false>, grid, dim3(256), 0, stream, back, ids, w, t, k, h, experts_per_rank,
                        ranks, out);
}

// ---- expert parallelism through peer memory ------------------------------------



size_t oomb_ep_mailbox_bytes(int ranks, int t_max, int top_k, int hidden, int x_dtype) {
    if (ranks <= 0 || t_max <= 0 || top_k <= 0 || hidden <= 0 || ep_xb(x_dtype) == 0) return 0;
    return ep_mailbox(ranks, t_max, top_k, hidden, ep_xb(x_dtype)).total;
}

size_t oomb_ep_mailbox_x_offset(int ranks, int t_max, int top_k, int hidden, int x_dtype) {
    if (ranks <= 0 || t_max <= 0 || top_k <= 0 || hidden <= 0 || ep_xb(x_dtype) == 0) return 0;
    return ep_mailbox(ranks, t_max, top_k, hidden, ep_xb(x_dtype)).x;
}

int oomb_ep_mailbox_alloc(size_t bytes, void** mailbox) {
    if (!mailbox || bytes == 0) return OOMB_E_ARG;
    *mailbox = nullptr;
    if (cudaMalloc(mailbox, bytes) != cudaSuccess) return OOMB_E_DEVICE;
    if (cudaMemset(*mailbox, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(*mailbox);
        *mailbox = nullptr;
        return OOMB_E_DEVICE;
    }
    return OOMB_OK;
}

int oomb_ep_mailbox_free(void* mailbox) {
    if (!mailbox) return OOMB_E_ARG;
    return cudaFree(mailbox) == cudaSuccess ? OOMB_OK : OOMB_E_DEVICE;
}

int oomb_ipc_handle(const void* dev_ptr, void* handle) {
    if (!dev_ptr || !handle) return OOMB_E_ARG;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)) != cudaSuccess) return OOMB_E_DEVICE;
    static_assert(sizeof(h) <= OOMB_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    return OOMB_OK;
}

int oomb_ipc_open(const void* handle, void** dev_ptr) {
    if (!handle || !dev_ptr) return OOMB_E_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *dev_ptr = nullptr;
    return cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? OOMB_OK : OOMB_E_DEVICE;
}

int oomb_ipc_close(void* dev_ptr) {
    if (!dev_ptr) return OOMB_E_ARG;
    return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? OOMB_OK : OOMB_E_DEVICE;
}

int oomb_ep_dispatch_peer(const oomb_ep_peer* q, const int32_t* ids, int t, int experts_per_rank, const void* x,
                          oomb_stream stream) {
    EpPeer p;
    if (!ep_peer_of(q, p) || !ids || !x || experts_per_rank <= 0) return OOMB_E_ARG;
    if (t <= 0 || t > q->t_max) return OOMB_E_SHAPE;
    if (!aligned16(x)) return OOMB_E_ALIGN;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    p.err = d->err;
    return launch(ep_dispatch_kernel, dim3(q->ranks), dim3(kEpThreads), 0, stream, p, ids, t, experts_per_rank, x);
}

int oomb_ep_group_peer(const oomb_ep_peer* q, int t, int experts_per_rank, const uint64_t* recs_local,
                       int32_t* n_active, int32_t* off, int32_t* assign_row, int32_t* assign_ret,
                       uint64_t* recs_active, oomb_stream stream) {
    EpPeer p;
    if (!ep_peer_of(q, p) || !recs_local || !n_active || !off || !assign_row || !assign_ret || !recs_active ||
        experts_per_rank <= 0)
        return OOMB_E_ARG;
    if (t <= 0 || t > q->t_max) return OOMB_E_SHAPE;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    p.err = d->err;
    const size_t smem = 2 * static_cast<size_t>(experts_per_rank) * sizeof(int32_t);
    if (smem > 200 * 1024) return OOMB_E_SHAPE;
    return launch(ep_group_peer_kernel, dim3(1), dim3(kEpThreads), smem, stream, p, t, experts_per_rank, recs_local,
                  n_active, off, assign_row, assign_ret, recs_active);
}

int oomb_ep_return_peer(const oomb_ep_peer* q, const float* y, const int32_t* n_active, const int32_t* off,
                        const int32_t* assign_ret, int t, int max_rows, oomb_stream stream) {
    EpPeer p;
    if (!ep_peer_of(q, p) || !y || !n_active || !off || !assign_ret) return OOMB_E_ARG;
    if (t <= 0 || t > q->t_max || max_rows <= 0) return OOMB_E_SHAPE;
    if (!aligned16(y)) return OOMB_E_ALIGN;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    p.err = d->err;
    const int64_t quads = static_cast<int64_t>(max_rows) * (q->hidden / 4);
    int grid = static_cast<int>((quads + 255) / 256);
    if (grid > 2 * d->sms) grid = 2 * d->sms;
    return launch(ep_return_kernel, dim3(grid > 0 ? grid : 1), dim3(256), 0, stream, p, y, n_active, off, assign_ret, t);
}

int oomb_ep_combine_peer(const oomb_ep_peer* q, const int32_t* ids, const float* w, int t, int experts_per_rank,
                         void* out, int out_dtype, oomb_stream stream) {
    EpPeer p;
    if (!ep_peer_of(q, p) || !ids || !w || !out || experts_per_rank <= 0) return OOMB_E_ARG;
    if (out_dtype != OOMB_F32 && out_dtype != OOMB_BF16) return OOMB_E_ARG;
    if (t <= 0 || t > q->t_max) return OOMB_E_SHAPE;
    if (!aligned16(out)) return OOMB_E_ALIGN;
    const DeviceState* d = device_state();
    if (!d) return OOMB_E_DEVICE;
    p.err = d->err;
    const int64_t quads = static_cast<int64_t>(t) * q->hidden / 4;
    int grid = static_cast<int>((quads + 255) / 256);
    if (grid > 2 * d->sms) grid = 2 * d->sms;
    return out_dtype == OOMB_BF16
               ? launch(ep_combine_peer_kernel<true>, dim3(grid), dim3(256), 0, stream, p, ids, w, t, experts_per_rank,
                        out)
               : launch(ep_combine_peer_kernel<false>, dim3(grid), dim3(256), 0, stream, p, ids, w, t,
                        experts_per_rank, out);
}

// ---- offload staging (Transfer, crates/oominf-core/src/backend.rs:945-1018) --------

int oomb_copy_queue_create(oomb_copy_queue* queue) {
    if (!queue) return OOMB_E_ARG;
    if (!device_state()) return OOMB_E_DEVICE;
    cudaStream_t s = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return OOMB_E_LAUNCH;
    *queue = reinterpret_cast<oomb_copy_queue>(s);
    return OOMB_OK;
}

int oomb_copy_queue_destroy(oomb_copy_queue queue) {
    if (!queue) return OOMB_E_ARG;
    return cudaStreamDestroy(reinterpret_cast<cudaStream_t>(queue)) == cudaSuccess ? OOMB_OK : OOMB_E_LAUNCH;
}

int oomb_pin_host(void* ptr, size_t len) {
    if (!ptr || len == 0) return OOMB_E_ARG;
    if (!device_state()) return OOMB_E_DEVICE;
    return cudaHostRegister(ptr, len, cudaHostRegisterPortable) == cudaSuccess ? OOMB_OK : OOMB_E_LAUNCH;
}

int oomb_unpin_host(void* ptr) {
    if (!ptr) return OOMB_E_ARG;
    return cudaHostUnregister(ptr) == cudaSuccess ? OOMB_OK : OOMB_E_LAUNCH;
}

int oomb_copy_to_device(oomb_copy_queue queue, void* dst, const void* src, size_t len) {
    if (!queue || !dst || !src) return OOMB_E_ARG;
    if (len == 0) return OOMB_OK;
    return cudaMemcpyAsync(dst, src, len, cudaMemcpyHostToDevice, reinterpret_cast<cudaStream_t>(queue)) == cudaSuccess
               ? OOMB_OK
               : OOMB_E_LAUNCH;
}

int oomb_copy_on_device(oomb_copy_queue queue, void* dst, const void* src, size_t len) {
    if (!queue || !dst || !src) return OOMB_E_ARG;
    if (len == 0) return OOMB_OK;
    return cudaMemcpyAsync(dst, src, len, cudaMemcpyDeviceToDevice, reinterpret_cast<cudaStream_t>(queue)) ==
                   cudaSuccess
               ? OOMB_OK
               : OOMB_E_LAUNCH;
}

namespace {
int record_on(cudaStream_t s, oomb_event* ev) {
    if (!ev) return OOMB_E_ARG;
    cudaEvent_t e = nullptr;
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return OOMB_E_LAUNCH;
    if (cudaEventRecord(e, s) != cudaSuccess) {
        cudaEventDestroy(e);
        return OOMB_E_LAUNCH;
    }
    *ev = reinterpret_cast<oomb_event>(e);
    return OOMB_OK;
}
}  // namespace

int oomb_record_compute(oomb_stream compute, oomb_event* ev) { return record_on(compute, ev); }

int oomb_record_copies(oomb_copy_queue queue, oomb_event* ev) {
    if (!queue) return OOMB_E_ARG;
    return record_on(reinterpret_cast<cudaStream_t>(queue), ev);
}

int oomb_copies_wait(oomb_copy_queue queue, oomb_event ev) {
    if (!queue || !ev) return OOMB_E_ARG;
    return cudaStreamWaitEvent(reinterpret_cast<cudaStream_t>(queue), reinterpret_cast<cudaEvent_t>(ev), 0) ==
                   cudaSuccess
               ? OOMB_OK
               : OOMB_E_LAUNCH;
}

int oomb_compute_wait(oomb_stream compute, oomb_event ev) {
    if (!ev) return OOMB_E_ARG;
    return cudaStreamWaitEvent(compute, reinterpret_cast<cudaEvent_t>(ev), 0) == cudaSuccess ? OOMB_OK
                                                                                             : OOMB_E_LAUNCH;
}

int oomb_event_done(oomb_event ev) {
    if (!ev) return OOMB_E_ARG;
    const cudaError_t r = cudaEventQuery(reinterpret_cast<cudaEvent_t>(ev));
    if (r == cudaSuccess) return 1;
    if (r == cudaErrorNotReady) return 0;
    return OOMB_E_LAUNCH;
}

int oomb_event_wait(oomb_event ev) {
    if (!ev) return OOMB_E_ARG;
    return cudaEventSynchronize(reinterpret_cast<cudaEvent_t>(ev)) == cudaSuccess ? OOMB_OK : OOMB_E_LAUNCH;
}

int oomb_event_destroy(oomb_event ev) {
    if (!ev) return OOMB_E_ARG;
    return cudaEventDestroy(reinterpret_cast<cudaEvent_t>(ev)) == cudaSuccess ? OOMB_OK : OOMB_E_LAUNCH;
}

int oomb_copies_sync(oomb_copy_queue queue) {
    if (!queue) return OOMB_E_ARG;
    return cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(queue)) == cudaSuccess ? OOMB_OK : OOMB_E_LAUNCH;
}

// ---- expert tiers: device slots over a pinned host arena --------------------------

struct oomb_policy_st {
    oomb::TierPolicy* p;
};

int oomb_policy_create(const char* spec, oomb_policy* policy) {
    if (!policy) return OOMB_E_ARG;
    *policy = nullptr;
    TierPolicy* p = make_policy(spec);
    if (!p) return OOMB_E_ARG;
    *policy = new oomb_policy_st{p};
    return OOMB_OK;
}

int oomb_policy_destroy(oomb_policy policy) {
    if (!policy) return OOMB_E_ARG;
    delete policy->p;
    delete policy;
    return OOMB_OK;
}

int oomb_policy_touch(oomb_policy policy, uint32_t key, uint64_t now) {
    if (!policy) return OOMB_E_ARG;
    policy->p->touch(key, now);
    return OOMB_OK;
}

int oomb_policy_remove(oomb_policy policy, uint32_t key) {
    if (!policy) return OOMB_E_ARG;
    policy->p->remove(key);
    return OOMB_OK;
}

int64_t oomb_policy_victim(oomb_policy policy, const uint32_t* pinned, int n_pinned) {
    if (!policy || n_pinned < 0 || (n_pinned > 0 && !pinned)) return OOMB_E_ARG;
    std::set<uint32_t> pin(pinned, pinned + n_pinned);
    return policy->p->victim([&](uint32_t k) { return pin.count(k) != 0; });
}

struct oomb_tier_st {
    oomb::Tier t;
};

int oomb_tier_create(const void* host_arena, size_t record_stride, int layers, int experts, void* device_slots,
                     int slots, const char* policy, oomb_tier* tier) {
    if (!tier) return OOMB_E_ARG;
    *tier = nullptr;
    if (!host_arena || !device_slots || record_stride == 0 || layers <= 0 || experts <= 0 || slots <= 0)
        return OOMB_E_ARG;
    if (static_cast<int64_t>(layers) * experts > 0xffffffffLL) return OOMB_E_SHAPE;
    if (!device_state()) return OOMB_E_DEVICE;
    const void* unused = nullptr;
    if (mem_kind(host_arena, &unused) != Mem::host || mem_kind(device_slots, &unused) != Mem::device)
        return OOMB_E_ARG;
    TierPolicy* p = make_policy(policy);
    if (!p) return OOMB_E_ARG;
    auto* st = new oomb_tier_st{};
    Tier& t = st->t;
    t.host_base = static_cast<const uint8_t*>(host_arena);
    t.device_base = static_cast<uint8_t*>(device_slots);
    t.stride = record_stride;
    t.layers = layers;
    t.experts = experts;
    t.slots = slots;
    t.policy = p;
    t.key_of.assign(slots, -1);
    for (int i = slots - 1; i >= 0; i--) t.free_slots.push_back(i);
    if (cudaStreamCreateWithFlags(&t.queue, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&t.compute_ev, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&t.copies_ev, cudaEventDisableTiming) != cudaSuccess) {
        if (t.queue) cudaStreamDestroy(t.queue);
        if (t.compute_ev) cudaEventDestroy(t.compute_ev);
        delete p;
        delete st;
        return OOMB_E_LAUNCH;
    }
    *tier = st;
    return OOMB_OK;
}

int oomb_tier_destroy(oomb_tier tier) {
    if (!tier) return OOMB_E_ARG;
    Tier& t = tier->t;
    cudaStreamSynchronize(t.queue);
    cudaEventDestroy(t.compute_ev);
    cudaEventDestroy(t.copies_ev);
    cudaStreamDestroy(t.queue);
    delete t.policy;
    delete tier;
    return OOMB_OK;
}

int oomb_tier_finish_fetch(oomb_tier tier, oomb_stream compute) {
    if (!tier) return OOMB_E_ARG;
    Tier& t = tier->t;
    if (!t.open) return OOMB_OK;
    t.open = false;
    if (cudaEventRecord(t.copies_ev, t.queue) != cudaSuccess) return OOMB_E_LAUNCH;
    return cudaStreamWaitEvent(compute, t.copies_ev, 0) == cudaSuccess ? OOMB_OK : OOMB_E_LAUNCH;
}

int oomb_tier_begin_fetch(oomb_tier tier, oomb_stream compute, int layer, const int32_t* experts, int n,
                          uint64_t* addrs, uint8_t* ready) {
    if (!tier || (n > 0 && (!experts || !addrs || !ready)) || n < 0) return OOMB_E_ARG;
    Tier& t = tier->t;
    if (layer < 0 || layer >= t.layers) return OOMB_E_SHAPE;
    for (int i = 0; i < n; i++)
        if (experts[i] < 0 || experts[i] >= t.experts) return OOMB_E_SHAPE;
    int rc = oomb_tier_finish_fetch(tier, compute);
    if (rc) return rc;
    std::set<uint32_t> wanted;
    for (int i = 0; i < n; i++) wanted.insert(static_cast<uint32_t>(layer) * t.experts + experts[i]);
    // refuse before touching anything when the slots cannot hold the fetch: its
    // missing records need free slots or residents it does not want
    size_t resident_wanted = 0;
    for (uint32_t k : wanted) resident_wanted += t.slot_of.count(k);
    const size_t missing = wanted.size() - resident_wanted;
    if (missing > t.free_slots.size() + (t.slot_of.size() - resident_wanted)) return OOMB_E_SHAPE;
    // every slot this fetch fills may still be read by compute issued before it
    if (cudaEventRecord(t.compute_ev, compute) != cudaSuccess || cudaStreamWaitEvent(t.queue, t.compute_ev, 0) != cudaSuccess)
        return OOMB_E_LAUNCH;
    std::unordered_map<uint32_t, bool> placed;  // keys filled by this fetch (not ready yet)
    for (int i = 0; i < n; i++) {
        const uint32_t key = static_cast<uint32_t>(layer) * t.experts + experts[i];
        t.stats.requests++;
        auto it = t.slot_of.find(key);
        if (it != t.slot_of.end()) {
            const bool fresh = placed.count(key) != 0;
            if (!fresh) t.stats.hits++;
            addrs[i] = reinterpret_cast<uint64_t>(t.device_base + static_cast<size_t>(it->second) * t.stride);
            ready[i] = fresh ? 0 : 1;
            t.policy->touch(key, t.now++);
            continue;
        }
        int slot;
        if (!t.free_slots.empty()) {
            slot = t.free_slots.back();
            t.free_slots.pop_back();
        } else {
            const int64_t v = t.policy->victim([&](uint32_t k) { return wanted.count(k) != 0; });
            if (v < 0) return OOMB_E_SHAPE;  // unreachable after the capacity check
            const uint32_t vk = static_cast<uint32_t>(v);
            slot = t.slot_of[vk];
            t.slot_of.erase(vk);
            t.policy->remove(vk);
            t.stats.evictions++;
        }
        t.slot_of[key] = slot;
        t.key_of[slot] = key;
        placed[key] = true;
        t.stats.misses++;
        uint8_t* dst = t.device_base + static_cast<size_t>(slot) * t.stride;
        const uint8_t* src = t.host_base + static_cast<size_t>(key) * t.stride;
        if (cudaMemcpyAsync(dst, src, t.stride, cudaMemcpyHostToDevice, t.queue) != cudaSuccess) return OOMB_E_LAUNCH;
        t.stats.bytes_copied += t.stride;
        addrs[i] = reinterpret_cast<uint64_t>(dst);
        ready[i] = 0;
        t.policy->touch(key, t.now++);
    }
    t.open = true;
    return OOMB_OK;
}

int oomb_tier_stats(oomb_tier tier, uint64_t* out5) {
    if (!tier || !out5) return OOMB_E_ARG;
    const TierStats& s = tier->t.stats;
    out5[0] = s.requests;
    out5[1] = s.hits;
    out5[2] = s.misses;
    out5[3] = s.evictions;
    out5[4] = s.bytes_copied;
    return OOMB_OK;
}

// ---- FP8 expert records: layout and load-time conversion ----------------------

int oomb_fp8_record_layout(int64_t hidden, int64_t inter, int scale_layout, oomb_fp8_record* geo, size_t* stride) {
    if (!geo || !stride) return OOMB_E_ARG;
    if (scale_layout != OOMB_SCALE_1X128 && scale_layout != OOMB_SCALE_128X128) return OOMB_E_ARG;
    if (hidden <= 0 || inter <= 0 || hidden % 16 || inter % 16) return OOMB_E_SHAPE;
    auto up = [](int64_t v, int64_t a) { return (v + a - 1) / a * a; };
    auto sbytes = [&](int64_t n, int64_t k) {
        const int64_t rows = scale_layout == OOMB_SCALE_128X128 ? (n + 127) / 128 : n;
        return rows * ((k + 127) / 128) * 4;
    };
    const int64_t H = hidden, I = inter;
    int64_t o = 0;
    oomb_fp8_record g{};
    g.hidden = H;
    g.inter = I;
    g.layout = scale_layout;
    g.gate_weight = o; o = up(o + I * H, OOMB_PART_ALIGN);
    g.up_weight = o; o = up(o + I * H, OOMB_PART_ALIGN);
    g.down_weight = o; o = up(o + H * I, OOMB_PART_ALIGN);
    g.gate_scale = o; o = up(o + sbytes(I, H), OOMB_PART_ALIGN);
    g.up_scale = o; o = up(o + sbytes(I, H), OOMB_PART_ALIGN);
    g.down_scale = o; o = up(o + sbytes(H, I), OOMB_PART_ALIGN);
    *geo = g;
    *stride = static_cast<size_t>(up(o, OOMB_RECORD_ALIGN));
    return OOMB_OK;
}

int oomb_quantize_fp8_record(const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                             const oomb_fp8_record* geo, uint8_t* record, oomb_stream stream) {
    if (!gate || !up || !down || !geo || !record) return OOMB_E_ARG;
    if (geo->layout != OOMB_SCALE_1X128 && geo->layout != OOMB_SCALE_128X128) return OOMB_E_ARG;
    if (geo->hidden <= 0 || geo->inter <= 0 || geo->hidden > 0x7fffffff || geo->inter > 0x7fffffff) return OOMB_E_SHAPE;
    if (!aligned16(record) || ((geo->gate_weight | geo->up_weight | geo->down_weight | geo->gate_scale |
                                geo->up_scale | geo->down_scale) & 15))
        return OOMB_E_ALIGN;
    const int H = static_cast<int>(geo->hidden), I = static_cast<int>(geo->inter);
    int rc = oomb_quantize_fp8(gate, I, H, geo->layout, record + geo->gate_weight,
                               reinterpret_cast<float*>(record + geo->gate_scale), stream);
    if (rc) return rc;
    rc = oomb_quantize_fp8(up, I, H, geo->layout, record + geo->up_weight,
                           reinterpret_cast<float*>(record + geo->up_scale), stream);
    if (rc) return rc;
    return oomb_quantize_fp8(down, H, I, geo->layout, record + geo->down_weight,
                             reinterpret_cast<float*>(record + geo->down_scale), stream);
}

int oomb_quantize_fp8(const uint16_t* w, int n, int k, int scale_layout, uint8_t* q, float* scale,
                      oomb_stream stream) {
    if (!w || !q || !scale) return OOMB_E_ARG;
    if (scale_layout != OOMB_SCALE_1X128 && scale_layout != OOMB_SCALE_128X128) return OOMB_E_ARG;
    if (n <= 0 || k <= 0) return OOMB_E_SHAPE;
    if (!device_state()) return OOMB_E_DEVICE;
    const int nb = (k + 127) / 128;
    const int nr = scale_layout == OOMB_SCALE_128X128 ? (n + 127) / 128 : n;
    quantize_blocks_kernel<<<static_cast<unsigned>(nr) * nb, 128, 0, stream>>>(w, n, k, scale_layout, q, scale);
    return cudaGetLastError() == cudaSuccess ? OOMB_OK : OOMB_E_LAUNCH;
}

}  // extern "C"

// ---- fused decode step without a caller workspace -----------------------------
//
// The same kernels as oomb_moe_decode_fp8, with their scratch in a fixed
// device array instead of caller memory, so the call allocates nothing.
namespace {

__device__ __align__(256) uint8_t g_noalloc_scratch[OOMB_NOALLOC_SCRATCH_BYTES];

// The part of the array that must be zero before a call and that the kernels
// keep consistent from call to call: the chain's self-resetting arrival
// counter (the first 256 bytes) and the one-launch kernel's sync words after
// it (launch epoch, barrier counts, row-group counters).
constexpr size_t kNoallocSyncBytes = 256 + ((static_cast<size_t>(kSyncWords) * 4 + 255) & ~static_cast<size_t>(255));

struct NoallocState {
    bool ok = false;
    uint8_t* scratch = nullptr;
};

NoallocState g_noalloc[kMaxDevices];
std::mutex g_noalloc_mu;

// Set-up per device, with that device current, done by the first call that
// succeeds in it: look up the array's device address and zero its sync words.
// A set-up that failed (for instance a first call made during stream capture)
// leaves the state untouched, so a later call retries.  Returns nullptr on
// failure.
uint8_t* noalloc_scratch(oomb_stream stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoallocState& s = g_noalloc[dev];
    if (!s.ok) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) {
            (void)cudaGetLastError();
            return nullptr;
        }
        if (cudaMemsetAsync(p, 0, kNoallocSyncBytes, stream) != cudaSuccess) {
            (void)cudaGetLastError();
            return nullptr;
        }
        s.scratch = static_cast<uint8_t*>(p);
        s.ok = true;
    }
    return s.scratch;
}

bool noalloc_reset_sync() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return false;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    const NoallocState& s = g_noalloc[dev];
    if (!s.ok) return true;  // never set up: the next call's set-up zeroes them
    return cudaMemset(s.scratch, 0, kNoallocSyncBytes) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
}

}  // namespace

extern "C" int oomb_moe_decode_fp8_noalloc(const oomb_moe_layer* layer, const void* x, int x_dtype, int t,
                                           void* out, int out_dtype, int32_t* ids, float* weights,
                                           oomb_stream stream) {
    const int rc = check_layer(layer);
    if (rc) return rc;
    if (t < 0) return OOMB_E_SHAPE;
    if (t > 0 && decode_layout(t, layer).total > static_cast<size_t>(OOMB_NOALLOC_SCRATCH_BYTES))
        return OOMB_E_WORKSPACE;
    if (!device_state()) return OOMB_E_DEVICE;
    uint8_t* scratch = noalloc_scratch(stream);
    if (!scratch) return OOMB_E_DEVICE;
    return oomb_moe_decode_fp8(layer, x, x_dtype, t, out, out_dtype, ids, weights, scratch,
                               OOMB_NOALLOC_SCRATCH_BYTES, stream);
}
