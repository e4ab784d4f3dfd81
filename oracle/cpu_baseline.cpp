// cpu_baseline.cpp - the reference's host expert path, restated in C++ with FP8
// weights: the timed CPU baseline (bench.py cpu_baseline leg and
// `bench.py --impl reference`).  TEST/BENCH INFRASTRUCTURE ONLY.
//
// Follows projects/oom-inference/crates/oominf-cpu:
//   - row kernel: kernel.rs:378-441 (per output row, 16-wide FMA over columns,
//     up to MAX_TOKENS = 4 activation rows in registers, kernel.rs:74);
//     the NVFP4 LUT decode is replaced by an exact e4m3 decode times the
//     block scale (the e4m3 table of kernel.rs:14-32, computed with
//     integer ops instead of a gather);
//   - worker pool: lib.rs:176-323 (gate/up in GATE_ROWS = 32 row items, SiLU*up,
//     down in DOWN_ROWS = 128 row items, lib.rs:47-48), std::thread workers
//     pulling items from a shared counter in place of rayon;
//   - router: the bf16 row kernel (kernel.rs:417-441) over the router matrix,
//     then softmax / top-k / renormalise as ops.cu:234-294.
#include <immintrin.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace {

constexpr int MAX_TOKENS = 4;    // kernel.rs:74
constexpr int GATE_ROWS = 32;    // lib.rs:47
constexpr int DOWN_ROWS = 128;   // lib.rs:48

float e4m3_scalar(uint8_t b) {
    float s = (b & 0x80) ? -1.0f : 1.0f;
    int e = (b >> 3) & 0xf, m = b & 7;
    if (e == 15 && m == 7) return NAN;
    float mag = e == 0 ? (float)m / 8.0f * ldexpf(1.0f, -6) : (1.0f + (float)m / 8.0f) * ldexpf(1.0f, e - 7);
    return s * mag;
}

// A pool of workers that run a list of items; the caller joins in.
class Pool {
  public:
    explicit Pool(int threads) : n_(std::max(1, threads)) {
        for (int i = 1; i < n_; i++) workers_.emplace_back([this] { loop(); });
    }
    ~Pool() {
        {
            std::lock_guard<std::mutex> g(m_);
            stop_ = true;
            gen_++;
        }
        cv_.notify_all();
        for (auto& w : workers_) w.join();
    }
    int threads() const { return n_; }
    // Runs fn(i) for i in [0, items) on every worker.
    void run(int64_t items, const std::function<void(int64_t)>& fn) {
        if (items <= 0) return;
        {
            std::lock_guard<std::mutex> g(m_);
            fn_ = &fn;
            items_ = items;
            next_.store(0);
            active_ = n_ - 1;
            gen_++;
        }
        cv_.notify_all();
        work();
        std::unique_lock<std::mutex> lk(m_);
        done_cv_.wait(lk, [this] { return active_ == 0; });
        fn_ = nullptr;
    }

  private:
    void work() {
        for (;;) {
            int64_t i = next_.fetch_add(1);
            if (i >= items_) break;
            (*fn_)(i);
        }
    }
    void loop() {
        uint64_t seen = 0;
        for (;;) {
            {
                std::unique_lock<std::mutex> lk(m_);
                cv_.wait(lk, [&] { return gen_ != seen; });
                seen = gen_;
                if (stop_) return;
            }
            work();
            {
                std::lock_guard<std::mutex> g(m_);
                if (--active_ == 0) done_cv_.notify_all();
            }
        }
    }
    int n_;
    std::vector<std::thread> workers_;
    std::mutex m_;
    std::condition_variable cv_, done_cv_;
    const std::function<void(int64_t)>* fn_ = nullptr;
    int64_t items_ = 0;
    std::atomic<int64_t> next_{0};
    int active_ = 0;
    uint64_t gen_ = 0;
    bool stop_ = false;
};

struct Fp8Matrix {
    const uint8_t* q;
    const float* scale;
    int layout;  // 0: 1x128, 1: 128x128
    int64_t cols;
    float scale_at(int64_t r, int64_t c) const {
        int64_t nb = (cols + 127) / 128;
        return scale[(layout ? r / 128 : r) * nb + c / 128];
    }
};

// out[r * nt + t] = W[row0 + r] . xs[t], nt <= MAX_TOKENS (kernel.rs:332-372 contract).
__attribute__((target("avx512f,avx512bw"))) void fp8_rows_avx512(const Fp8Matrix& m, int64_t row0,
                                                                  int64_t n_rows,
                                                                  const float* const* xs, int nt,
                                                                  float* out) {
    const __m512i k7f = _mm512_set1_epi32(0x7f), k80 = _mm512_set1_epi32(0x80);
    const __m512i bias = _mm512_set1_epi32(120 << 23);
    const __m512 sub_scale = _mm512_set1_ps(1.0f / 512.0f);
    const int64_t groups = m.cols / 16;
    for (int64_t r = 0; r < n_rows; r++) {
        int64_t row = row0 + r;
        const uint8_t* qr = m.q + row * m.cols;
        __m512 acc[MAX_TOKENS];
        for (int t = 0; t < MAX_TOKENS; t++) acc[t] = _mm512_setzero_ps();
        for (int64_t g = 0; g < groups; g++) {
            __m512i v = _mm512_cvtepu8_epi32(_mm_loadu_si128((const __m128i*)(qr + g * 16)));
            __m512i em = _mm512_and_si512(v, k7f);
            // normal codes: exponent rebased by 120, mantissa in place; subnormal
            // codes (exponent field 0): m * 2^-9.  Exact either way.
            __m512 fn = _mm512_castsi512_ps(_mm512_add_epi32(_mm512_slli_epi32(em, 20), bias));
            __m512 fs = _mm512_mul_ps(_mm512_cvtepi32_ps(em), sub_scale);
            __mmask16 sub = _mm512_cmplt_epi32_mask(em, _mm512_set1_epi32(8));
            __m512 f = _mm512_mask_blend_ps(sub, fn, fs);
            f = _mm512_castsi512_ps(_mm512_or_si512(_mm512_castps_si512(f),
                                                    _mm512_slli_epi32(_mm512_and_si512(v, k80), 24)));
            __m512 w = _mm512_mul_ps(f, _mm512_set1_ps(m.scale_at(row, g * 16)));
            for (int t = 0; t < nt; t++)
                acc[t] = _mm512_fmadd_ps(w, _mm512_loadu_ps(xs[t] + g * 16), acc[t]);
        }
        for (int t = 0; t < nt; t++) out[r * nt + t] = _mm512_reduce_add_ps(acc[t]);
    }
}

void fp8_rows_scalar(const Fp8Matrix& m, int64_t row0, int64_t n_rows, const float* const* xs,
                     int nt, float* out) {
    for (int64_t r = 0; r < n_rows; r++) {
        int64_t row = row0 + r;
        for (int t = 0; t < nt; t++) {
            float acc = 0.0f;
            for (int64_t c = 0; c < m.cols; c++)
                acc += e4m3_scalar(m.q[row * m.cols + c]) * m.scale_at(row, c) * xs[t][c];
            out[r * nt + t] = acc;
        }
    }
}

__attribute__((target("avx512f,avx512bw"))) void bf16_rows_avx512(const uint16_t* w, int64_t cols,
                                                                  int64_t row0, int64_t n_rows,
                                                                  const float* const* xs, int nt,
                                                                  float* out) {
    for (int64_t r = 0; r < n_rows; r++) {
        const uint16_t* row = w + (row0 + r) * cols;
        __m512 acc[MAX_TOKENS];
        for (int t = 0; t < MAX_TOKENS; t++) acc[t] = _mm512_setzero_ps();
        for (int64_t g = 0; g < cols / 16; g++) {
            __m256i words = _mm256_loadu_si256((const __m256i*)(row + g * 16));
            __m512 wv = _mm512_castsi512_ps(_mm512_slli_epi32(_mm512_cvtepu16_epi32(words), 16));
            for (int t = 0; t < nt; t++)
                acc[t] = _mm512_fmadd_ps(wv, _mm512_loadu_ps(xs[t] + g * 16), acc[t]);
        }
        for (int t = 0; t < nt; t++) out[r * nt + t] = _mm512_reduce_add_ps(acc[t]);
    }
}

void bf16_rows_scalar(const uint16_t* w, int64_t cols, int64_t row0, int64_t n_rows,
                      const float* const* xs, int nt, float* out) {
    for (int64_t r = 0; r < n_rows; r++)
        for (int t = 0; t < nt; t++) {
            float acc = 0.0f;
            for (int64_t c = 0; c < cols; c++) {
                uint32_t b = (uint32_t)w[(row0 + r) * cols + c] << 16;
                float f;
                memcpy(&f, &b, 4);
                acc += f * xs[t][c];
            }
            out[r * nt + t] = acc;
        }
}

bool has_avx512() {
    static const bool v = __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw");
    return v;
}

void fp8_rows(const Fp8Matrix& m, int64_t row0, int64_t n_rows, const float* const* xs, int nt,
              float* out) {
    if (has_avx512() && m.cols % 16 == 0) fp8_rows_avx512(m, row0, n_rows, xs, nt, out);
    else fp8_rows_scalar(m, row0, n_rows, xs, nt, out);
}

void bf16_rows(const uint16_t* w, int64_t cols, int64_t row0, int64_t n_rows,
               const float* const* xs, int nt, float* out) {
    if (has_avx512() && cols % 16 == 0) bf16_rows_avx512(w, cols, row0, n_rows, xs, nt, out);
    else bf16_rows_scalar(w, cols, row0, n_rows, xs, nt, out);
}

float silu(float x) { return x / (1.0f + expf(-x)); }  // lib.rs:152-154

}  // namespace

extern "C" {

// Record geometry: byte offsets of each part inside a record.
typedef struct {
    int64_t hidden, inter;
    int64_t gate_weight, gate_scale, up_weight, up_scale, down_weight, down_scale;
    int32_t layout;
    int32_t pad_;
} ocb_fp8_record;

void* ocb_pool_create(int threads) { return new Pool(threads); }
void ocb_pool_destroy(void* p) { delete static_cast<Pool*>(p); }
int ocb_pool_threads(void* p) { return static_cast<Pool*>(p)->threads(); }
int ocb_has_avx512(void) { return has_avx512() ? 1 : 0; }

// Dense FP8 GEMV y[t, n] = x[t, k] . W^T in items of GATE_ROWS rows, tokens in
// groups of MAX_TOKENS.
void ocb_gemv_fp8(void* pool, const float* x, int64_t t, const uint8_t* q, const float* scale,
                  int layout, int64_t n, int64_t k, float* y) {
    Pool* p = static_cast<Pool*>(pool);
    Fp8Matrix m{q, scale, layout, k};
    int64_t items = (n + GATE_ROWS - 1) / GATE_ROWS;
    for (int64_t t0 = 0; t0 < t; t0 += MAX_TOKENS) {
        int nt = (int)std::min<int64_t>(MAX_TOKENS, t - t0);
        p->run(items, [&](int64_t it) {
            int64_t r0 = it * GATE_ROWS, nr = std::min<int64_t>(GATE_ROWS, n - r0);
            const float* xs[MAX_TOKENS];
            for (int i = 0; i < nt; i++) xs[i] = x + (t0 + i) * k;
            float out[GATE_ROWS * MAX_TOKENS];
            fp8_rows(m, r0, nr, xs, nt, out);
            for (int64_t r = 0; r < nr; r++)
                for (int i = 0; i < nt; i++) y[(t0 + i) * n + r0 + r] = out[r * nt + i];
        });
    }
}

// One MoE layer step on the host: router logits (bf16 rows), softmax top-k,
// then every routed expert as HostExperts::run does (lib.rs:176-323) and the
// slot-order weighted combine (moe.cu:155-164).  recs[e] points at expert e's
// record.  x: [t, hidden] fp32; out: [t, hidden] fp32.  Returns 0, or -1 for a
// shape this port does not take.
int ocb_moe_layer(void* pool, const float* x, int64_t t, const uint16_t* router_w, int64_t e,
                  int64_t k, const uint8_t* const* recs, const ocb_fp8_record* geo, float* out) {
    Pool* p = static_cast<Pool*>(pool);
    const int64_t H = geo->hidden, I = geo->inter;
    if (k > 32 || k > e || H % 16 || I % 16) return -1;
    // Router: one item per GATE_ROWS experts.
    std::vector<float> logits(t * e);
    for (int64_t t0 = 0; t0 < t; t0 += MAX_TOKENS) {
        int nt = (int)std::min<int64_t>(MAX_TOKENS, t - t0);
        p->run((e + GATE_ROWS - 1) / GATE_ROWS, [&](int64_t it) {
            int64_t r0 = it * GATE_ROWS, nr = std::min<int64_t>(GATE_ROWS, e - r0);
            const float* xs[MAX_TOKENS];
            for (int i = 0; i < nt; i++) xs[i] = x + (t0 + i) * H;
            float o[GATE_ROWS * MAX_TOKENS];
            bf16_rows(router_w, H, r0, nr, xs, nt, o);
            for (int64_t r = 0; r < nr; r++)
                for (int i = 0; i < nt; i++) logits[(t0 + i) * e + r0 + r] = o[r * nt + i];
        });
    }
    // Top-k per token (ops.cu:234-294 arithmetic, serial).
    std::vector<int32_t> ids(t * k);
    std::vector<float> wts(t * k);
    std::vector<float> pr(e);
    for (int64_t tt = 0; tt < t; tt++) {
        const float* l = &logits[tt * e];
        float mx = -INFINITY, sum = 0.0f;
        for (int64_t i = 0; i < e; i++) mx = fmaxf(mx, l[i]);
        for (int64_t i = 0; i < e; i++) sum += expf(l[i] - mx);
        for (int64_t i = 0; i < e; i++) pr[i] = expf(l[i] - mx) / sum;
        float ps = 0.0f, cp[32];
        for (int64_t r = 0; r < k; r++) {
            int64_t bi = 0;
            for (int64_t i = 1; i < e; i++)
                if (pr[i] > pr[bi]) bi = i;
            ids[tt * k + r] = (int32_t)bi;
            cp[r] = pr[bi];
            ps += pr[bi];
            pr[bi] = -2.0f;
        }
        for (int64_t r = 0; r < k; r++) wts[tt * k + r] = cp[r] / ps;
    }
    // Jobs: one per distinct expert, tokens in slot order (moe.rs:541-551).
    struct Job { int64_t expert; std::vector<int64_t> tokens, slots; };
    std::vector<Job> jobs;
    {
        std::vector<int64_t> pos(e, -1);
        for (int64_t s = 0; s < t * k; s++) {
            int64_t ex = ids[s];
            if (pos[ex] < 0) { pos[ex] = (int64_t)jobs.size(); jobs.push_back({ex, {}, {}}); }
            jobs[pos[ex]].tokens.push_back(s / k);
            jobs[pos[ex]].slots.push_back(s);
        }
        std::sort(jobs.begin(), jobs.end(), [](const Job& a, const Job& b) { return a.expert < b.expert; });
    }
    // Gate/up + SiLU: items of GATE_ROWS rows per (job, token group).
    struct Item { int64_t job, row0, t0; };
    std::vector<std::vector<float>> acts(jobs.size());
    std::vector<Item> items;
    for (size_t j = 0; j < jobs.size(); j++) {
        acts[j].assign(jobs[j].tokens.size() * I, 0.0f);
        for (int64_t t0 = 0; t0 < (int64_t)jobs[j].tokens.size(); t0 += MAX_TOKENS)
            for (int64_t r0 = 0; r0 < I; r0 += GATE_ROWS) items.push_back({(int64_t)j, r0, t0});
    }
    p->run((int64_t)items.size(), [&](int64_t ii) {
        const Item& it = items[ii];
        const Job& jb = jobs[it.job];
        const uint8_t* rec = recs[jb.expert];
        Fp8Matrix g{rec + geo->gate_weight, (const float*)(rec + geo->gate_scale), geo->layout, H};
        Fp8Matrix u{rec + geo->up_weight, (const float*)(rec + geo->up_scale), geo->layout, H};
        int nt = (int)std::min<int64_t>(MAX_TOKENS, (int64_t)jb.tokens.size() - it.t0);
        int64_t nr = std::min<int64_t>(GATE_ROWS, I - it.row0);
        const float* xs[MAX_TOKENS];
        for (int i = 0; i < nt; i++) xs[i] = x + jb.tokens[it.t0 + i] * H;
        float go[GATE_ROWS * MAX_TOKENS], uo[GATE_ROWS * MAX_TOKENS];
        fp8_rows(g, it.row0, nr, xs, nt, go);
        fp8_rows(u, it.row0, nr, xs, nt, uo);
        for (int64_t r = 0; r < nr; r++)
            for (int i = 0; i < nt; i++)
                acts[it.job][(it.t0 + i) * I + it.row0 + r] = silu(go[r * nt + i]) * uo[r * nt + i];
    });
    // Down: items of DOWN_ROWS rows per (job, token group).
    std::vector<std::vector<float>> downs(jobs.size());
    items.clear();
    for (size_t j = 0; j < jobs.size(); j++) {
        downs[j].assign(jobs[j].tokens.size() * H, 0.0f);
        for (int64_t t0 = 0; t0 < (int64_t)jobs[j].tokens.size(); t0 += MAX_TOKENS)
            for (int64_t r0 = 0; r0 < H; r0 += DOWN_ROWS) items.push_back({(int64_t)j, r0, t0});
    }
    p->run((int64_t)items.size(), [&](int64_t ii) {
        const Item& it = items[ii];
        const Job& jb = jobs[it.job];
        const uint8_t* rec = recs[jb.expert];
        Fp8Matrix d{rec + geo->down_weight, (const float*)(rec + geo->down_scale), geo->layout, I};
        int nt = (int)std::min<int64_t>(MAX_TOKENS, (int64_t)jb.tokens.size() - it.t0);
        int64_t nr = std::min<int64_t>(DOWN_ROWS, H - it.row0);
        const float* xs[MAX_TOKENS];
        for (int i = 0; i < nt; i++) xs[i] = &acts[it.job][(it.t0 + i) * I];
        std::vector<float> o(DOWN_ROWS * MAX_TOKENS);
        fp8_rows(d, it.row0, nr, xs, nt, o.data());
        for (int64_t r = 0; r < nr; r++)
            for (int i = 0; i < nt; i++) downs[it.job][(it.t0 + i) * H + it.row0 + r] = o[r * nt + i];
    });
    // Slot-order combine.
    std::vector<const float*> slot_row(t * k);
    for (size_t j = 0; j < jobs.size(); j++)
        for (size_t i = 0; i < jobs[j].slots.size(); i++) slot_row[jobs[j].slots[i]] = &downs[j][i * H];
    for (int64_t tt = 0; tt < t; tt++)
        for (int64_t c = 0; c < H; c++) {
            float acc = 0.0f;
            for (int64_t s = 0; s < k; s++) acc += wts[tt * k + s] * slot_row[tt * k + s][c];
            out[tt * H + c] = acc;
        }
    return 0;
}

}  // extern "C"
