// oracle.cpp -- CPU restatement of Opure-VoxelEngine's decode path.
//
// TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA path (see oracle.h for
// who may load it and how it is pinned). Scalar, double accumulation, no SIMD
// reordering of any sum, exactly as src/engine/Opure_CpuReference.cpp computes.
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <vector>

namespace {

// ---------------------------------------------------------------------------
// fp16 <-> fp32 from the IEEE 754 binary16 definition.
float f16_to_f32(uint16_t h) {
    // Same case split as Opure_Streamer.cpp:49-84 (zero, subnormal, inf/NaN, normal),
    // except the subnormal exponent: that file writes 127-15-e (:66), which halves
    // every fp16 subnormal; the IEEE value needs 127-15-e+1 after e normalising shifts.
    const uint32_t sign = uint32_t(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            uint32_t e = 0;
            while ((man & 0x400u) == 0) { man <<= 1; ++e; }
            man &= 0x3FFu;
            bits = sign | ((127u - 15u + 1u - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

uint16_t f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xFFu;
    const uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFF) return uint16_t(sign | (man ? 0x7E00u : 0x7C00u));
    const int e = int(exp) - 112;  // rebias 127 -> 15
    if (e >= 31) return uint16_t(sign | 0x7C00u);
    if (e <= 0) {
        // Result is subnormal (or zero): value = M * 2^(exp-150), unit 2^-24.
        const int s = 14 - e;                 // bits to drop from the 24-bit significand
        if (s > 24) return uint16_t(sign);
        const uint32_t M = man | 0x800000u;
        uint32_t q = M >> s;
        const uint32_t rem = M & ((1u << s) - 1u);
        const uint32_t half = 1u << (s - 1);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return uint16_t(sign | q);
    }
    uint32_t q = (uint32_t(e) << 10) | (man >> 13);
    const uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;  // carry may reach inf: correct
    return uint16_t(sign | q);
}

struct F16Lut {
    float v[65536];
    F16Lut() { for (uint32_t i = 0; i < 65536; ++i) v[i] = f16_to_f32(uint16_t(i)); }
};
const F16Lut &lut() {
    static const F16Lut t;
    return t;
}

float bf16_to_f32(uint16_t h) {
    const uint32_t bits = uint32_t(h) << 16;
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

int g_threads = 1;

// Persistent worker pool: run(n, fn) calls fn(i) for i in [0, n), split into
// contiguous static chunks. Each index is computed by exactly one thread with the
// same arithmetic as a serial loop, so results do not depend on the thread count.
class Pool {
public:
    ~Pool() { resize(0); }
    void resize(int n) {
        {
            std::unique_lock<std::mutex> lk(mu_);
            stop_ = true;
            ++gen_;
        }
        cv_.notify_all();
        for (auto &t : workers_) t.join();
        workers_.clear();
        stop_ = false;
        for (int i = 0; i < n; ++i) workers_.emplace_back([this, i] { loop(i); });
    }
    int size() const { return int(workers_.size()); }
    void run(int64_t n, const std::function<void(int64_t)> &fn) {
        const int nt = size() + 1;
        if (nt == 1 || n < 2) {
            for (int64_t i = 0; i < n; ++i) fn(i);
            return;
        }
        {
            std::unique_lock<std::mutex> lk(mu_);
            fn_ = &fn;
            n_ = n;
            pending_ = size();
            ++gen_;
        }
        cv_.notify_all();
        chunk(0, nt, fn);
        std::unique_lock<std::mutex> lk(mu_);
        done_.wait(lk, [this] { return pending_ == 0; });
        fn_ = nullptr;
    }

private:
    void chunk(int who, int nt, const std::function<void(int64_t)> &fn) {
        const int64_t b = n_ * who / nt, e = n_ * (who + 1) / nt;
        for (int64_t i = b; i < e; ++i) fn(i);
    }
    void loop(int i) {
        uint64_t seen;
        {
            std::unique_lock<std::mutex> lk(mu_);
            seen = gen_;
        }
        for (;;) {
            const std::function<void(int64_t)> *fn;
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return gen_ != seen; });
                seen = gen_;
                if (stop_) return;
                fn = fn_;
            }
            chunk(i + 1, size() + 1, *fn);
            std::unique_lock<std::mutex> lk(mu_);
            if (--pending_ == 0) done_.notify_one();
        }
    }
    std::vector<std::thread> workers_;
    std::mutex mu_;
    std::condition_variable cv_, done_;
    const std::function<void(int64_t)> *fn_ = nullptr;
    int64_t n_ = 0;
    int pending_ = 0;
    uint64_t gen_ = 0;
    bool stop_ = false;
};

Pool &pool() {
    static Pool p;
    return p;
}

// Threads that run whole sequences of their own (orc_generate_batch workers, or callers
// that asked with orc_thread_serial) compute serially and never touch the shared pool.
thread_local bool t_serial = false;

// Runs fn over [0, n), in parallel when the work (n * cost) is large enough.
void parallel_for(int64_t n, uint64_t cost, const std::function<void(int64_t)> &fn) {
    if (!t_serial && g_threads > 1 && uint64_t(n) * cost > (1u << 16)) {
        pool().run(n, fn);
    } else {
        for (int64_t i = 0; i < n; ++i) fn(i);
    }
}

// Weight matrix in whichever storage the file had. Accumulation is identical.
struct Matrix {
    int dtype = -1;                 // ORC_F16 / ORC_F32 / ORC_I8 (BF16 is widened to F32)
    uint32_t rows = 0, cols = 0;
    std::vector<uint16_t> h;
    std::vector<float> f;
    std::vector<int8_t> q;
    float scale = 1.0f;
    bool present() const { return dtype >= 0; }
};

// y[o] = float(sum double(W[o][i]) * double(x[i])) -- Opure_CpuReference.cpp:151-161.
void gemv_rows(const Matrix &W, const float *x, float *y) {
    const uint32_t rows = W.rows, cols = W.cols;
    std::vector<double> xd(cols);
    for (uint32_t i = 0; i < cols; ++i) xd[i] = double(x[i]);
    const float *L = lut().v;
    parallel_for(rows, cols, [&](int64_t o) {
        double acc = 0.0;
        if (W.dtype == ORC_F16) {
            const uint16_t *row = W.h.data() + size_t(o) * cols;
            for (uint32_t i = 0; i < cols; ++i) acc += double(L[row[i]]) * xd[i];
            y[o] = float(acc);
        } else if (W.dtype == ORC_F32) {
            const float *row = W.f.data() + size_t(o) * cols;
            for (uint32_t i = 0; i < cols; ++i) acc += double(row[i]) * xd[i];
            y[o] = float(acc);
        } else {
            const int8_t *row = W.q.data() + size_t(o) * cols;
            for (uint32_t i = 0; i < cols; ++i) acc += double(row[i]) * xd[i];
            // Opure_GEMV_Quant.usf:92 applies scaleW * scaleX (scaleX = 1, :206 of the
            // engine) after the sum.
            y[o] = float(acc * double(W.scale));
        }
    });
}

void rmsnorm(const float *x, const float *g, float *y, uint32_t d, float eps) {
    // Opure_CpuReference.cpp:163-169.
    double ss = 0.0;
    for (uint32_t i = 0; i < d; ++i) ss += double(x[i]) * double(x[i]);
    const double inv = 1.0 / std::sqrt(ss / d + eps);
    for (uint32_t i = 0; i < d; ++i) y[i] = float(double(x[i]) * inv * double(g[i]));
}

void rope(float *vec, uint32_t nheads, uint32_t hd, uint32_t pos, double theta, int literal) {
    // Structure of Opure_CpuReference.cpp:171-189. The exponent follows the shader
    // (Opure_RoPE.usf:56, pair index) unless `literal` asks for the CPU file's
    // element index.
    for (uint32_t head = 0; head < nheads; ++head) {
        float *row = vec + size_t(head) * hd;
        for (uint32_t i = 0; i + 1 < hd; i += 2) {
            const double ex = literal ? double(i) : double(i / 2);
            const double freq = std::pow(theta, -2.0 * ex / double(hd));
            const double t = double(pos) * freq;
            const double ct = std::cos(t), st = std::sin(t);
            const double e0 = row[i], e1 = row[i + 1];
            row[i] = float(e0 * ct - e1 * st);
            row[i + 1] = float(e0 * st + e1 * ct);
        }
    }
}

void swiglu(const float *g, const float *u, float *h, uint32_t n) {
    // Opure_CpuReference.cpp:191-198 (float arithmetic, unbranched sigmoid).
    for (uint32_t i = 0; i < n; ++i) {
        const float s = 1.0f / (1.0f + std::exp(-g[i]));
        h[i] = (g[i] * s) * u[i];
    }
}

// One query head over `seq_len` keys: Opure_CpuReference.cpp:259-305.
// krow(s)/vrow(s) return fp16 rows of hd elements.
inline double widen(uint16_t h) { return double(lut().v[h]); }
inline double widen(float f) { return double(f); }

template <class KRow, class VRow>
void attend_head(const float *qrow, uint32_t seq_len, uint32_t hd, float scale, KRow krow,
                 VRow vrow, float *orow, std::vector<double> &scores) {
    scores.resize(seq_len);
    double m = -1e300;
    for (uint32_t s = 0; s < seq_len; ++s) {
        const auto *k = krow(s);
        double sc = 0.0;
        for (uint32_t d = 0; d < hd; ++d) sc += double(qrow[d]) * widen(k[d]);
        sc *= double(scale);
        scores[s] = sc;
        if (sc > m) m = sc;
    }
    double sum = 0.0;
    for (uint32_t s = 0; s < seq_len; ++s) {
        const double e = std::exp(scores[s] - m);
        scores[s] = e;
        sum += e;
    }
    for (uint32_t d = 0; d < hd; ++d) orow[d] = 0.0f;
    for (uint32_t s = 0; s < seq_len; ++s) {
        const auto *v = vrow(s);
        const double w = scores[s];
        for (uint32_t d = 0; d < hd; ++d) orow[d] = float(double(orow[d]) + w * widen(v[d]));
    }
    const double inv = 1.0 / (sum > 0.0 ? sum : 1.0);
    for (uint32_t d = 0; d < hd; ++d) orow[d] = float(double(orow[d]) * inv);
}

// Softmax probabilities in double, max-shifted.
void softmax_d(const float *logits, uint32_t n, std::vector<double> &p) {
    p.resize(n);
    double mx = -std::numeric_limits<double>::infinity();
    for (uint32_t i = 0; i < n; ++i) if (double(logits[i]) > mx) mx = logits[i];
    double z = 0.0;
    for (uint32_t i = 0; i < n; ++i) { p[i] = std::exp(double(logits[i]) - mx); z += p[i]; }
    for (uint32_t i = 0; i < n; ++i) p[i] /= z;
}

uint32_t inverse_cdf(const std::vector<double> &w, double u) {
    double z = 0.0;
    for (double x : w) z += x;
    const double thr = u * z;
    double c = 0.0;
    for (uint32_t i = 0; i < w.size(); ++i) {
        c += w[i];
        if (c > thr) return i;
    }
    // u*Z at the very top (rounding): the last index with non-zero weight.
    for (uint32_t i = uint32_t(w.size()); i-- > 0;) if (w[i] > 0.0) return i;
    return 0;
}

uint32_t argmax1(const float *x, uint32_t n, float *val) {
    float best = -std::numeric_limits<float>::infinity();
    uint32_t bi = 0;
    bool any = false;
    for (uint32_t i = 0; i < n; ++i) {
        if (x[i] > best || (!any && x[i] == best)) { best = x[i]; bi = i; any = true; }
    }
    if (val) *val = best;
    return bi;
}

}  // namespace

// ===========================================================================
extern "C" {

void orc_rng_u32_stream(uint64_t seed, uint64_t n, uint32_t *out) {
    uint64_t s = seed ? seed : 1;
    for (uint64_t i = 0; i < n; ++i) {
        s ^= s << 13; s ^= s >> 7; s ^= s << 17;
        out[i] = uint32_t(s >> 32);
    }
}

uint16_t orc_f32_to_f16(float f) { return f32_to_f16(f); }
float orc_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
void orc_f32_to_f16_n(const float *src, uint16_t *dst, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) dst[i] = f32_to_f16(src[i]);
}
void orc_f16_to_f32_n(const uint16_t *src, float *dst, uint64_t n) {
    const float *L = lut().v;
    for (uint64_t i = 0; i < n; ++i) dst[i] = L[src[i]];
}

void orc_gemv_f16(const uint16_t *w, const float *x, float *y, uint32_t rows, uint32_t cols,
                  uint32_t nvec) {
    Matrix M;
    M.dtype = ORC_F16; M.rows = rows; M.cols = cols;
    M.h.assign(w, w + size_t(rows) * cols);
    for (uint32_t v = 0; v < nvec; ++v) gemv_rows(M, x + size_t(v) * cols, y + size_t(v) * rows);
}

void orc_gemv_f32(const float *w, const float *x, float *y, uint32_t rows, uint32_t cols,
                  uint32_t nvec) {
    Matrix M;
    M.dtype = ORC_F32; M.rows = rows; M.cols = cols;
    M.f.assign(w, w + size_t(rows) * cols);
    for (uint32_t v = 0; v < nvec; ++v) gemv_rows(M, x + size_t(v) * cols, y + size_t(v) * rows);
}

void orc_gemv_q8(const int8_t *q, float scale_w, float scale_x, const float *x, float *y,
                 uint32_t rows, uint32_t cols, uint32_t nvec) {
    Matrix M;
    M.dtype = ORC_I8; M.rows = rows; M.cols = cols;
    M.q.assign(q, q + size_t(rows) * cols);
    M.scale = 1.0f;
    const double s = double(scale_w) * double(scale_x);
    std::vector<float> tmp(rows);
    for (uint32_t v = 0; v < nvec; ++v) {
        // The unscaled sum, then the two scales in double (the shader applies them in
        // float after its fp32 sum; the oracle keeps the CPU path's double).
        const float *xv = x + size_t(v) * cols;
        float *yv = y + size_t(v) * rows;
        std::vector<double> xd(cols);
        for (uint32_t i = 0; i < cols; ++i) xd[i] = xv[i];
        parallel_for(rows, cols, [&](int64_t o) {
            double acc = 0.0;
            const int8_t *row = q + size_t(o) * cols;
            for (uint32_t i = 0; i < cols; ++i) acc += double(row[i]) * xd[i];
            yv[o] = float(acc * s);
        });
    }
}

void orc_quantize_q8(const uint16_t *w_f16, uint64_t n, int8_t *q, float *scale) {
    const float *L = lut().v;
    float amax = 0.0f;
    for (uint64_t i = 0; i < n; ++i) amax = std::fmax(amax, std::fabs(L[w_f16[i]]));
    const float s = amax > 0.0f ? amax / 127.0f : 1.0f;
    for (uint64_t i = 0; i < n; ++i) {
        const float r = std::nearbyint(L[w_f16[i]] / s);  // default rounding mode: half-even
        q[i] = int8_t(r > 127.0f ? 127 : (r < -127.0f ? -127 : int(r)));
    }
    *scale = s;
}

void orc_rmsnorm(const float *x, const float *g, float *y, uint32_t d, float eps) {
    rmsnorm(x, g, y, d, eps);
}

void orc_rope(float *vec, uint32_t nheads, uint32_t hd, uint32_t pos, double theta, int lit) {
    rope(vec, nheads, hd, pos, theta, lit);
}

void orc_swiglu(const float *g, const float *u, float *h, uint32_t n) { swiglu(g, u, h, n); }

void orc_argmax(const float *x, uint32_t n, uint32_t rows, uint32_t *idx, float *val) {
    for (uint32_t r = 0; r < rows; ++r)
        idx[r] = argmax1(x + size_t(r) * n, n, val ? val + r : nullptr);
}

void orc_attention_paged(const float *q, const uint16_t *pool, const int32_t *page_table,
                         const uint32_t *seq_lens, uint32_t nseq, uint32_t nq,
                         uint32_t max_pages, uint32_t P, uint32_t nH, uint32_t nKV,
                         uint32_t hd, float scale, float *out) {
    const uint32_t group = nH / nKV;
    const int64_t jobs = int64_t(nseq) * nq * nH;
    parallel_for(jobs, uint64_t(max_pages) * P * hd, [&](int64_t job) {
        std::vector<double> scores;
        {
            const uint32_t h = uint32_t(job % nH);
            const uint32_t j = uint32_t((job / nH) % nq);
            const uint32_t b = uint32_t(job / (int64_t(nH) * nq));
            const uint32_t g = h / group;
            const int32_t *pt = page_table + size_t(b) * max_pages;
            auto at = [&](uint32_t s, uint32_t kv) {
                const size_t page = size_t(pt[s / P]);
                return pool + ((page * 2 + kv) * nKV + g) * size_t(P) * hd + size_t(s % P) * hd;
            };
            const size_t qo = ((size_t(b) * nq + j) * nH + h) * hd;
            attend_head(q + qo, seq_lens[b] + j, hd, scale,
                        [&](uint32_t s) { return at(s, 0); },
                        [&](uint32_t s) { return at(s, 1); }, out + qo, scores);
        }
    });
}

void orc_attention_f32(const float *q, const float *k_plane, const float *v_plane,
                       uint32_t nH, uint32_t nKV, uint32_t hd, uint32_t max_seq,
                       uint32_t seq_len, float scale, float *out) {
    const uint32_t group = nH / nKV;
    std::vector<double> scores;
    for (uint32_t h = 0; h < nH; ++h) {
        const size_t base = size_t(h / group) * max_seq * hd;
        attend_head(q + size_t(h) * hd, seq_len, hd, scale,
                    [&](uint32_t s) { return k_plane + base + size_t(s) * hd; },
                    [&](uint32_t s) { return v_plane + base + size_t(s) * hd; },
                    out + size_t(h) * hd, scores);
    }
}

uint32_t orc_sample_softmax(const float *logits, uint32_t vocab, float u) {
    std::vector<double> p;
    softmax_d(logits, vocab, p);
    return inverse_cdf(p, double(u));
}

namespace {
// Orderable key of (value, index): larger value first, then lower index; 0 for NaN.
uint64_t sample_key(float v, uint32_t i) {
    if (v != v) return 0;
    uint32_t b;
    std::memcpy(&b, &v, 4);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (uint64_t(b) << 32) | (0xffffffffu - i);
}
}  // namespace

uint32_t orc_sample_filtered(const float *logits, uint32_t V, float T, uint32_t top_k, float top_p, float rep,
                             const int32_t *hist, uint32_t hist_len, float u) {
    std::vector<float> lp(logits, logits + V);
    if (rep != 1.0f && hist) {
        std::vector<char> seen(V, 0);
        for (uint32_t i = 0; i < hist_len; ++i)
            if (hist[i] >= 0 && uint32_t(hist[i]) < V) seen[hist[i]] = 1;
        for (uint32_t i = 0; i < V; ++i)
            if (seen[i]) lp[i] = lp[i] > 0.f ? lp[i] / rep : lp[i] * rep;
    }
    std::vector<uint32_t> order;
    for (uint32_t i = 0; i < V; ++i)
        if (sample_key(lp[i], i)) order.push_back(i);
    if (order.empty()) return 0;
    std::sort(order.begin(), order.end(),
              [&](uint32_t a, uint32_t b) { return sample_key(lp[a], a) > sample_key(lp[b], b); });
    if (!(T > 0.f) || top_k == 1) return order[0];
    const double inv_t = 1.0 / double(T);
    const double zmax = double(lp[order[0]]) * inv_t;
    if (top_k > 1 && top_k < V && order.size() > top_k) order.resize(top_k);
    std::vector<uint64_t> mass(V, 0);
    for (uint32_t i : order) {
        const double e = std::exp(double(lp[i]) * inv_t - zmax);
        mass[i] = e > 0.0 ? uint64_t(std::nearbyint(e * 1099511627776.0)) : 0;  // NaN (inf - inf): 0
    }
    if (top_p < 1.0f) {
        uint64_t z = 0;
        for (uint32_t i : order) z += mass[i];
        const double tgt = std::ceil(double(top_p) * double(z));
        const uint64_t target = tgt < 1.0 ? 1 : uint64_t(tgt);
        if (target < z) {
            uint64_t cum = 0;
            size_t keep = order.size();
            for (size_t j = 0; j < order.size(); ++j) {
                cum += mass[order[j]];
                if (cum >= target) {
                    keep = j + 1;
                    break;
                }
            }
            order.resize(keep);
        }
    }
    std::vector<char> kept(V, 0);
    uint64_t total = 0;
    for (uint32_t i : order) {
        kept[i] = 1;
        total += mass[i];
    }
    if (total == 0) return order[0];  // no mass at all (an infinite logit): the greedy token
    uint64_t thr = uint64_t(std::floor(double(u) * double(total)));
    if (thr >= total) thr = total - 1;
    uint64_t c = 0;
    for (uint32_t i = 0; i < V; ++i) {
        if (!kept[i]) continue;
        c += mass[i];
        if (c > thr) return i;
    }
    return order.back();
}

void orc_logit_stats(const float *l, uint32_t V, float *out) {
    double ss = 0.0;
    uint64_t best = 0;
    for (uint32_t i = 0; i < V; ++i) {
        ss += double(l[i]) * double(l[i]);
        best = std::max(best, sample_key(l[i], i));
    }
    float mx = -std::numeric_limits<float>::infinity();
    if (best) mx = l[0xffffffffu - uint32_t(best & 0xffffffffu)];
    double se = 0.0;
    for (uint32_t i = 0; i < V; ++i) se += std::exp(double(l[i] - mx));
    double ent = 0.0;
    if (se > 0.0) {
        const double inv = 1.0 / se;
        for (uint32_t i = 0; i < V; ++i) {
            const double p = std::exp(double(l[i] - mx)) * inv;
            if (p > 0.0) ent -= p * std::log(p);
        }
    }
    out[0] = mx;
    out[1] = float(std::sqrt(ss));
    out[2] = float(ent);
    out[3] = float(double(mx) + std::log(se));
}

int orc_spec_accept_greedy(const float *tl, const uint32_t *draft, uint32_t k, uint32_t V,
                           uint32_t *out) {
    uint32_t a = 0;
    while (a < k && argmax1(tl + size_t(a) * V, V, nullptr) == draft[a]) {
        out[a] = draft[a];
        ++a;
    }
    out[a] = argmax1(tl + size_t(a) * V, V, nullptr);
    return int(a);
}

int orc_spec_accept_rejection(const float *tl, const float *dl, const uint32_t *draft,
                              const float *u_accept, float u_final, uint32_t k, uint32_t V,
                              uint32_t *out) {
    std::vector<double> p, q;
    for (uint32_t i = 0; i < k; ++i) {
        softmax_d(tl + size_t(i) * V, V, p);
        softmax_d(dl + size_t(i) * V, V, q);
        const uint32_t d = draft[i];
        if (double(u_accept[i]) * q[d] <= p[d]) {
            out[i] = d;
            continue;
        }
        std::vector<double> r(V);
        double z = 0.0;
        for (uint32_t x = 0; x < V; ++x) { r[x] = p[x] > q[x] ? p[x] - q[x] : 0.0; z += r[x]; }
        out[i] = inverse_cdf(z > 0.0 ? r : p, double(u_final));
        return int(i);
    }
    softmax_d(tl + size_t(k) * V, V, p);
    out[k] = inverse_cdf(p, double(u_final));
    return int(k);
}

void orc_set_threads(int n) {
    g_threads = n > 0 ? n : 1;
    pool().resize(g_threads - 1);
}
int orc_get_threads(void) { return g_threads; }

}  // extern "C"

// ===========================================================================
// Whole model
// ===========================================================================
struct orc_model {
    orc_config c{};
    Matrix embed, lm_head;
    std::vector<float> final_norm;
    struct Layer {
        std::vector<float> in_norm, post_norm;
        Matrix wq, wk, wv, wo, gate, up, down;
    };
    std::vector<Layer> layers;
};

struct orc_state {
    uint32_t max_pos = 0, len = 0;
    uint32_t win_page = 0, win_ring = 0;  // sliding window (orc_state_set_window)
    uint32_t L = 0, nKV = 0, hd = 0;
    std::vector<uint16_t> kv;  // [L][2][nKV][max_pos][hd]
    uint16_t *at(uint32_t l, uint32_t kvsel, uint32_t g, uint32_t pos) {
        return kv.data() + ((((size_t(l) * 2 + kvsel) * nKV + g) * max_pos + pos) * hd);
    }
    const uint16_t *at(uint32_t l, uint32_t kvsel, uint32_t g, uint32_t pos) const {
        return kv.data() + ((((size_t(l) * 2 + kvsel) * nKV + g) * max_pos + pos) * hd);
    }
};

namespace {

bool load_matrix(Matrix &M, int dtype, const void *data, uint64_t n, uint32_t rows,
                 uint32_t cols, float scale) {
    if (n != uint64_t(rows) * cols) return false;
    M.rows = rows; M.cols = cols; M.scale = scale;
    if (dtype == ORC_F16) {
        M.dtype = ORC_F16;
        M.h.assign(static_cast<const uint16_t *>(data), static_cast<const uint16_t *>(data) + n);
    } else if (dtype == ORC_F32) {
        M.dtype = ORC_F32;
        M.f.assign(static_cast<const float *>(data), static_cast<const float *>(data) + n);
    } else if (dtype == ORC_BF16) {
        M.dtype = ORC_F32;
        M.f.resize(n);
        for (uint64_t i = 0; i < n; ++i) M.f[i] = bf16_to_f32(static_cast<const uint16_t *>(data)[i]);
    } else if (dtype == ORC_I8) {
        M.dtype = ORC_I8;
        M.q.assign(static_cast<const int8_t *>(data), static_cast<const int8_t *>(data) + n);
    } else {
        return false;
    }
    return true;
}

bool load_vector(std::vector<float> &v, int dtype, const void *data, uint64_t n, uint32_t d) {
    if (n != d) return false;
    v.resize(n);
    if (dtype == ORC_F16) {
        orc_f16_to_f32_n(static_cast<const uint16_t *>(data), v.data(), n);
    } else if (dtype == ORC_F32) {
        std::memcpy(v.data(), data, n * 4);
    } else if (dtype == ORC_BF16) {
        for (uint64_t i = 0; i < n; ++i) v[i] = bf16_to_f32(static_cast<const uint16_t *>(data)[i]);
    } else {
        return false;
    }
    return true;
}

void embed_row(const Matrix &E, uint32_t tok, float *x) {
    const size_t off = size_t(tok) * E.cols;
    if (E.dtype == ORC_F16) {
        const float *L = lut().v;
        for (uint32_t i = 0; i < E.cols; ++i) x[i] = L[E.h[off + i]];
    } else if (E.dtype == ORC_F32) {
        std::memcpy(x, E.f.data() + off, size_t(E.cols) * 4);
    } else {
        for (uint32_t i = 0; i < E.cols; ++i) x[i] = float(E.q[off + i]) * E.scale;
    }
}

}  // namespace

extern "C" {

orc_model *orc_model_create(const orc_config *cfg) {
    if (!cfg || cfg->heads == 0 || cfg->kv_heads == 0 || cfg->heads % cfg->kv_heads != 0 ||
        cfg->hidden % cfg->heads != 0)
        return nullptr;
    auto *m = new orc_model;
    m->c = *cfg;
    m->layers.resize(cfg->layers);
    return m;
}

int orc_model_set_tensor(orc_model *m, int role, int layer, int dtype, const void *data,
                         uint64_t n, float scale) {
    if (!m || !data) return -1;
    const orc_config &c = m->c;
    const uint32_t h = c.hidden, ff = c.inter, kvh = c.kv_heads * (c.hidden / c.heads);
    if (role >= ORC_IN_NORM && (layer < 0 || uint32_t(layer) >= c.layers)) return -1;
    auto *Ly = role >= ORC_IN_NORM ? &m->layers[size_t(layer)] : nullptr;
    bool ok = false;
    switch (role) {
        case ORC_EMBED: ok = load_matrix(m->embed, dtype, data, n, c.vocab, h, scale); break;
        case ORC_LM_HEAD: ok = load_matrix(m->lm_head, dtype, data, n, c.vocab, h, scale); break;
        case ORC_FINAL_NORM: ok = load_vector(m->final_norm, dtype, data, n, h); break;
        case ORC_IN_NORM: ok = load_vector(Ly->in_norm, dtype, data, n, h); break;
        case ORC_POST_NORM: ok = load_vector(Ly->post_norm, dtype, data, n, h); break;
        case ORC_WQ: ok = load_matrix(Ly->wq, dtype, data, n, h, h, scale); break;
        case ORC_WK: ok = load_matrix(Ly->wk, dtype, data, n, kvh, h, scale); break;
        case ORC_WV: ok = load_matrix(Ly->wv, dtype, data, n, kvh, h, scale); break;
        case ORC_WO: ok = load_matrix(Ly->wo, dtype, data, n, h, h, scale); break;
        case ORC_GATE: ok = load_matrix(Ly->gate, dtype, data, n, ff, h, scale); break;
        case ORC_UP: ok = load_matrix(Ly->up, dtype, data, n, ff, h, scale); break;
        case ORC_DOWN: ok = load_matrix(Ly->down, dtype, data, n, h, ff, scale); break;
        default: ok = false;
    }
    return ok ? 0 : -1;
}

int orc_model_ready(const orc_model *m) {
    if (!m || !m->embed.present() || m->final_norm.empty()) return -1;
    for (const auto &L : m->layers) {
        if (L.in_norm.empty() || L.post_norm.empty() || !L.wq.present() || !L.wk.present() ||
            !L.wv.present() || !L.wo.present() || !L.gate.present() || !L.up.present() ||
            !L.down.present())
            return -1;
    }
    return 0;
}

void orc_model_free(orc_model *m) { delete m; }

orc_state *orc_state_create(const orc_model *m, uint32_t max_pos) {
    if (!m || max_pos == 0) return nullptr;
    auto *s = new orc_state;
    s->max_pos = max_pos;
    s->L = m->c.layers;
    s->nKV = m->c.kv_heads;
    s->hd = m->c.hidden / m->c.heads;
    s->kv.assign(size_t(s->L) * 2 * s->nKV * max_pos * s->hd, 0);
    return s;
}

void orc_state_free(orc_state *s) { delete s; }
uint32_t orc_state_len(const orc_state *s) { return s ? s->len : 0; }
void orc_state_set_window(orc_state *s, uint32_t page_size, uint32_t ring) {
    if (!s) return;
    s->win_page = ring ? page_size : 0;
    s->win_ring = ring;
}
void orc_state_truncate(orc_state *s, uint32_t len) {
    if (s && len < s->len) s->len = len;
}

int orc_state_load_kv(orc_state *s, const uint16_t *kv, uint32_t len) {
    if (!s || len > s->max_pos) return -1;
    for (uint32_t l = 0; l < s->L; ++l)
        for (uint32_t sel = 0; sel < 2; ++sel)
            for (uint32_t g = 0; g < s->nKV; ++g) {
                const uint16_t *src = kv + (((size_t(l) * 2 + sel) * s->nKV + g) * len) * s->hd;
                std::memcpy(s->at(l, sel, g, 0), src, size_t(len) * s->hd * 2);
            }
    s->len = len;
    return 0;
}

int orc_forward(const orc_model *m, orc_state *s, uint32_t tok, float *logits, float *trace) {
    if (!m || !s) return -1;
    const orc_config &c = m->c;
    if (tok >= c.vocab || s->len >= s->max_pos) return -1;
    const uint32_t h = c.hidden, ff = c.inter, hd = h / c.heads;
    const uint32_t kvd = c.kv_heads * hd, group = c.heads / c.kv_heads;
    const uint32_t t = s->len;

    std::vector<float> x(h), normed(h), q(h), k(kvd), v(kvd), attn(h), proj(h), n2(h);
    std::vector<float> g(ff), u(ff), hh(ff);
    embed_row(m->embed, tok, x.data());

    for (uint32_t Li = 0; Li < c.layers; ++Li) {
        const orc_model::Layer &P = m->layers[Li];
        rmsnorm(x.data(), P.in_norm.data(), normed.data(), h, c.eps);
        gemv_rows(P.wq, normed.data(), q.data());
        gemv_rows(P.wk, normed.data(), k.data());
        gemv_rows(P.wv, normed.data(), v.data());
        rope(q.data(), c.heads, hd, t, c.theta, c.rope_cpu_literal);
        rope(k.data(), c.kv_heads, hd, t, c.theta, c.rope_cpu_literal);
        // Append at position t ([kvHead][pos][dim], Opure_CpuReference.cpp:244-257),
        // rounded to the fp16 the CUDA path's cache holds.
        for (uint32_t g2 = 0; g2 < c.kv_heads; ++g2) {
            uint16_t *kd = s->at(Li, 0, g2, t);
            uint16_t *vd = s->at(Li, 1, g2, t);
            for (uint32_t d = 0; d < hd; ++d) {
                kd[d] = f32_to_f16(k[g2 * hd + d]);
                vd[d] = f32_to_f16(v[g2 * hd + d]);
            }
        }
        // Positions [w0, t]: all of them, or under a sliding window of win_ring pages of
        // win_page tokens the last win_ring - 1 whole pages and the current one.
        uint32_t w0 = 0;
        if (s->win_ring && t / s->win_page + 1 > s->win_ring) w0 = (t / s->win_page + 1 - s->win_ring) * s->win_page;
        const uint32_t seq_len = t + 1 - w0;
        parallel_for(c.heads, uint64_t(seq_len) * hd * 2, [&](int64_t hq) {
            std::vector<double> scores;
            {
                const uint32_t kvh = uint32_t(hq) / group;
                attend_head(q.data() + size_t(hq) * hd, seq_len, hd, c.attn_scale,
                            [&](uint32_t sp) { return static_cast<const orc_state *>(s)->at(Li, 0, kvh, w0 + sp); },
                            [&](uint32_t sp) { return static_cast<const orc_state *>(s)->at(Li, 1, kvh, w0 + sp); },
                            attn.data() + size_t(hq) * hd, scores);
            }
        });
        gemv_rows(P.wo, attn.data(), proj.data());
        for (uint32_t i = 0; i < h; ++i) x[i] = x[i] + proj[i];

        rmsnorm(x.data(), P.post_norm.data(), n2.data(), h, c.eps);
        gemv_rows(P.gate, n2.data(), g.data());
        gemv_rows(P.up, n2.data(), u.data());
        swiglu(g.data(), u.data(), hh.data(), ff);
        gemv_rows(P.down, hh.data(), proj.data());
        for (uint32_t i = 0; i < h; ++i) x[i] = x[i] + proj[i];
        if (trace) std::memcpy(trace + size_t(Li) * h, x.data(), size_t(h) * 4);
    }
    s->len = t + 1;
    if (logits) {
        // Final norm in place, then the (tied unless given) LM head, :338-345.
        rmsnorm(x.data(), m->final_norm.data(), x.data(), h, c.eps);
        gemv_rows(m->lm_head.present() ? m->lm_head : m->embed, x.data(), logits);
    }
    return 0;
}

int orc_generate(const orc_model *m, const uint32_t *prompt, uint32_t n_prompt,
                 uint32_t budget, uint32_t max_pos, uint32_t *out, float *margins) {
    if (!m || n_prompt == 0 || n_prompt > max_pos) return -1;
    orc_state *s = orc_state_create(m, max_pos);
    std::vector<float> logits(m->c.vocab);
    auto top = [&](float *margin) {
        float v1;
        const uint32_t i1 = argmax1(logits.data(), m->c.vocab, &v1);
        if (margin) {
            float v2 = -std::numeric_limits<float>::infinity();
            for (uint32_t i = 0; i < m->c.vocab; ++i)
                if (i != i1 && logits[i] > v2) v2 = logits[i];
            *margin = v1 - v2;
        }
        return i1;
    };
    for (uint32_t i = 0; i < n_prompt; ++i)
        orc_forward(m, s, prompt[i], i + 1 == n_prompt ? logits.data() : nullptr, nullptr);
    float mg = 0.0f;
    uint32_t next = top(&mg);
    int n = 0;
    for (uint32_t i = 0; i < budget; ++i) {
        out[n] = next;
        if (margins) margins[n] = mg;
        ++n;
        if (s->len + 1 >= max_pos) break;
        orc_forward(m, s, next, logits.data(), nullptr);
        next = top(&mg);
    }
    orc_state_free(s);
    return n;
}

}  // extern "C"

// ===========================================================================
// Stop rules, independent sequences, seeded synthetic inputs
// ===========================================================================
namespace {

// xorshift64 of Opure_TestHarness.cpp:36-47 (seed 0 behaves as seed 1).
struct Xorshift {
    uint64_t s;
    explicit Xorshift(uint64_t seed) : s(seed ? seed : 1) {}
    uint32_t next() {
        s ^= s << 13; s ^= s >> 7; s ^= s << 17;
        return uint32_t(s >> 32);
    }
    double open01() { return (double(next()) + 0.5) / 4294967296.0; }
};

// Standard normals by Box-Muller (Box & Muller 1958) on pairs of open uniforms u1, u2:
// r = sqrt(-2 ln u1), a = 2 pi u2; r cos(a) first, then r sin(a).
struct BoxMuller {
    Xorshift r;
    double spare = 0.0;
    bool has = false;
    explicit BoxMuller(uint64_t seed) : r(seed) {}
    double next() {
        if (has) {
            has = false;
            return spare;
        }
        const double u1 = r.open01(), u2 = r.open01();
        const double rad = std::sqrt(-2.0 * std::log(u1)), a = 2.0 * M_PI * u2;
        spare = rad * std::sin(a);
        has = true;
        return rad * std::cos(a);
    }
    // out[i] = float(next() * scale) for the next n draws; whole pairs run in blocks on the
    // worker pool, each block's xorshift state found by stepping the generator alone.
    void fill(uint64_t n, double scale, float *out) {
        uint64_t i = 0;
        if (has && n) {
            out[i++] = float(spare * scale);
            has = false;
        }
        constexpr uint64_t kPairs = 1 << 16;
        const uint64_t pairs = (n - i) / 2, blocks = (pairs + kPairs - 1) / kPairs;
        std::vector<uint64_t> starts(blocks);
        for (uint64_t b = 0; b < blocks; ++b) {
            starts[b] = r.s;
            const uint64_t m = std::min(kPairs, pairs - b * kPairs);
            for (uint64_t k = 0; k < 2 * m; ++k) r.next();
        }
        float *o = out + i;
        parallel_for(int64_t(blocks), 2 * kPairs * 64, [&](int64_t b) {
            BoxMuller g(1);
            g.r.s = starts[size_t(b)];
            const uint64_t m = std::min(kPairs, pairs - uint64_t(b) * kPairs);
            for (uint64_t k = 0; k < 2 * m; ++k) o[uint64_t(b) * 2 * kPairs + k] = float(g.next() * scale);
        });
        i += 2 * pairs;
        if (i < n) out[i] = float(next() * scale);
    }
};

uint16_t q8_round_store(float w, float scale) {
    float r = std::nearbyint(w / scale);
    r = std::fmin(127.f, std::fmax(-127.f, r));
    return uint16_t(uint8_t(int8_t(r)));
}

// Greedy generation of one sequence with the reference's stop rules
// (VoxelEngine::Generate, Opure_VoxelEngine.cpp:894-958): the token predicted from the last
// prompt position is pushed first; after each push the loop ends when it was the stop id
// (:925-930) or when seqLen + 1 >= maxPos (:932); otherwise one decode step follows.
int generate_one(const orc_model *m, const uint32_t *prompt, uint32_t n_prompt, uint32_t budget,
                 uint32_t max_pos, int64_t eos, uint32_t *out, float *margins, int *hit_stop,
                 uint32_t *second = nullptr) {
    if (!m || n_prompt == 0 || n_prompt > max_pos) return -1;
    orc_state *s = orc_state_create(m, max_pos);
    std::vector<float> logits(m->c.vocab);
    uint32_t i2 = 0;  // runner-up of the last top() (lowest index among equal values)
    auto top = [&](float *margin) {
        float v1;
        const uint32_t i1 = argmax1(logits.data(), m->c.vocab, &v1);
        float v2 = -std::numeric_limits<float>::infinity();
        i2 = i1;
        for (uint32_t i = 0; i < m->c.vocab; ++i)
            if (i != i1 && logits[i] > v2) {
                v2 = logits[i];
                i2 = i;
            }
        if (margin) *margin = v1 - v2;
        return i1;
    };
    for (uint32_t i = 0; i < n_prompt; ++i)
        orc_forward(m, s, prompt[i], i + 1 == n_prompt ? logits.data() : nullptr, nullptr);
    float mg = 0.0f;
    uint32_t next = top(&mg);
    int n = 0;
    if (hit_stop) *hit_stop = 0;
    for (uint32_t i = 0; i < budget; ++i) {
        out[n] = next;
        if (margins) margins[n] = mg;
        if (second) second[n] = i2;
        ++n;
        if (eos >= 0 && next == uint32_t(eos)) {
            if (hit_stop) *hit_stop = 1;
            break;
        }
        if (s->len + 1 >= max_pos) break;
        orc_forward(m, s, next, logits.data(), nullptr);
        next = top(&mg);
    }
    orc_state_free(s);
    return n;
}

}  // namespace

extern "C" {

void orc_thread_serial(int on) { t_serial = on != 0; }

int orc_generate_stop(const orc_model *m, const uint32_t *prompt, uint32_t n_prompt, uint32_t budget,
                      uint32_t max_pos, int64_t eos, uint32_t *out, float *margins, int *hit_stop) {
    return generate_one(m, prompt, n_prompt, budget, max_pos, eos, out, margins, hit_stop);
}

int orc_generate_batch(const orc_model *m, const uint32_t *prompts, const uint32_t *prompt_lens,
                       uint32_t n_seq, uint32_t budget, uint32_t max_pos, int64_t eos, int threads,
                       uint32_t *out, uint32_t *counts, float *margins, uint32_t *second) {
    if (!m || n_seq == 0) return -1;
    std::vector<size_t> off(n_seq + 1, 0);
    for (uint32_t i = 0; i < n_seq; ++i) off[i + 1] = off[i] + prompt_lens[i];
    const uint32_t nt = uint32_t(std::max(1, std::min<int>(threads, int(n_seq))));
    std::vector<int> rc(n_seq, 0);
    auto work = [&](uint32_t who) {
        t_serial = true;
        for (uint32_t i = who; i < n_seq; i += nt) {
            const int n = generate_one(m, prompts + off[i], prompt_lens[i], budget, max_pos, eos,
                                       out + size_t(i) * budget, margins ? margins + size_t(i) * budget : nullptr,
                                       nullptr, second ? second + size_t(i) * budget : nullptr);
            rc[i] = n;
            if (counts) counts[i] = n < 0 ? 0u : uint32_t(n);
        }
    };
    std::vector<std::thread> ts;
    for (uint32_t t = 1; t < nt; ++t) ts.emplace_back(work, t);
    work(0);
    for (auto &t : ts) t.join();
    for (int r : rc)
        if (r < 0) return -1;
    return 0;
}

void orc_synth_normal_f16(uint64_t seed, float stddev, uint64_t n, uint16_t *out) {
    // Pairs of normals come from pairs of draws, so the stream splits into chunks of whole
    // pairs: the generator state at each chunk start is found by stepping the (cheap)
    // xorshift alone, then the chunks (the costly transcendentals) run on the worker pool.
    constexpr uint64_t kPairs = 1 << 16;
    const uint64_t pairs = (n + 1) / 2, chunks = (pairs + kPairs - 1) / kPairs;
    std::vector<uint64_t> starts(chunks);
    Xorshift r(seed);
    for (uint64_t c = 0; c < chunks; ++c) {
        starts[c] = r.s;
        for (uint64_t i = 0; i < 2 * kPairs; ++i) r.next();
    }
    parallel_for(int64_t(chunks), 2 * kPairs * 64, [&](int64_t c) {
        BoxMuller g(1);
        g.r.s = starts[size_t(c)];
        const uint64_t i0 = uint64_t(c) * 2 * kPairs, i1 = std::min(n, i0 + 2 * kPairs);
        for (uint64_t i = i0; i < i1; ++i) out[i] = f32_to_f16(float(g.next() * stddev));
    });
}

void orc_synth_prompt(uint64_t seed, uint32_t vocab, uint32_t n, int32_t *out) {
    Xorshift r(seed);
    for (uint32_t i = 0; i < n; ++i) out[i] = int32_t(r.next() % vocab);
}

void orc_synth_permutation(uint64_t seed, uint32_t n, int32_t *out) {
    for (uint32_t i = 0; i < n; ++i) out[i] = int32_t(i);
    Xorshift r(seed);
    for (uint32_t i = n; i > 1; --i) std::swap(out[i - 1], out[r.next() % i]);
}

void orc_synth_uniforms(uint64_t seed, uint64_t n, float *out) {
    Xorshift r(seed);
    for (uint64_t i = 0; i < n; ++i) out[i] = float(double(r.next()) / 4294967296.0);
}

orc_model *orc_model_create_synth(const orc_config *cfg, const orc_synth *sp) {
    if (!sp) return nullptr;
    orc_model *m = orc_model_create(cfg);
    if (!m) return nullptr;
    const orc_config &c = m->c;
    const uint32_t h = c.hidden, ff = c.inter, kvh = c.kv_heads * (c.hidden / c.heads);
    BoxMuller g(sp->seed), noise(sp->noise_seed);
    std::vector<uint16_t> w;
    std::vector<int8_t> q;
    // One matrix in file order: fp16(N(0, std)), plus fp16-rounded N(0, noise_std) noise for
    // draft models; int8 (absmax / 127, round half to even, clamp +-127) when asked.
    std::vector<float> draws, noises;
    auto matrix = [&](int role, int layer, uint32_t rows, uint32_t cols, bool quantizable) {
        const uint64_t n = uint64_t(rows) * cols;
        w.resize(n);
        draws.resize(n);
        g.fill(n, double(sp->std), draws.data());
        if (sp->noise_std > 0.f) {
            noises.resize(n);
            noise.fill(n, double(sp->noise_std), noises.data());
        }
        for (uint64_t i = 0; i < n; ++i) {
            float v = f16_to_f32(f32_to_f16(draws[i]));
            if (sp->noise_std > 0.f) v = v + noises[i];
            w[i] = f32_to_f16(v);
        }
        if (sp->int8 && quantizable) {
            float amax = 0.f;
            for (uint16_t x : w) amax = std::fmax(amax, std::fabs(f16_to_f32(x)));
            const float scale = amax > 0.f ? amax / 127.0f : 1.0f;
            q.resize(w.size());
            for (size_t i = 0; i < w.size(); ++i) q[i] = int8_t(uint8_t(q8_round_store(f16_to_f32(w[i]), scale)));
            return orc_model_set_tensor(m, role, layer, ORC_I8, q.data(), q.size(), scale);
        }
        return orc_model_set_tensor(m, role, layer, ORC_F16, w.data(), w.size(), 1.0f);
    };
    const std::vector<uint16_t> ones(h, 0x3C00);
    int rc = matrix(ORC_EMBED, 0, c.vocab, h, false);
    for (uint32_t l = 0; l < c.layers && rc == 0; ++l) {
        const int L = int(l);
        rc |= orc_model_set_tensor(m, ORC_IN_NORM, L, ORC_F16, ones.data(), h, 1.f);
        rc |= matrix(ORC_WQ, L, h, h, true);
        rc |= matrix(ORC_WK, L, kvh, h, true);
        rc |= matrix(ORC_WV, L, kvh, h, true);
        rc |= matrix(ORC_WO, L, h, h, true);
        rc |= orc_model_set_tensor(m, ORC_POST_NORM, L, ORC_F16, ones.data(), h, 1.f);
        rc |= matrix(ORC_GATE, L, ff, h, true);
        rc |= matrix(ORC_UP, L, ff, h, true);
        rc |= matrix(ORC_DOWN, L, h, ff, true);
    }
    rc |= orc_model_set_tensor(m, ORC_FINAL_NORM, 0, ORC_F16, ones.data(), h, 1.f);
    if (!sp->tied) rc |= matrix(ORC_LM_HEAD, 0, c.vocab, h, false);
    if (rc != 0 || orc_model_ready(m) != 0) {
        orc_model_free(m);
        return nullptr;
    }
    return m;
}

}  // extern "C"
