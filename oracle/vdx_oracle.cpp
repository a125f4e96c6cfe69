// vdx_oracle.cpp - TEST INFRASTRUCTURE ONLY (see vdx_oracle.h).
//
// A line-by-line CPU restatement of TVdxSampler, src/VindexLLM.Sampler.pas. Each
// function cites the reference lines it follows. Two tie modes:
//   VDXS_TIES_FAITHFUL  - the reference's K-slot min-buffer (Sampler.pas:341-383) and
//                         its stable insertion sort (Sampler.pas:416-429).
//   VDXS_TIES_CANONICAL - top-k = the k largest values with ties to the lowest index;
//                         draw order = (probability desc, index asc).
// Floating-point convention (not pinned by any reference test): Single operands are
// evaluated in Double and rounded to Single on store; Exp is C's double exp.

#include "vdx_oracle.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <numeric>
#include <thread>
#include <vector>

namespace {

// ---- PRNG: xoshiro256** seeded by SplitMix64 (Sampler.pas:157-248) -------------
// WrapAdd/WrapMul (Sampler.pas:160-190) spell out mod-2^64 add and multiply so that
// Delphi's overflow checks do not trap; C++ unsigned arithmetic is already mod 2^64.
inline uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

uint64_t splitmix64(uint64_t& st) {  // Sampler.pas:194-201
    st += 0x9E3779B97F4A7C15ull;
    uint64_t r = st;
    r = (r ^ (r >> 30)) * 0xBF58476D1CE4E5B9ull;
    r = (r ^ (r >> 27)) * 0x94D049BB133111EBull;
    return r ^ (r >> 31);
}

struct Prng {
    uint64_t s0 = 0, s1 = 0, s2 = 0, s3 = 0;
    void seed(int64_t seed) {  // Sampler.pas:224-241
        uint64_t st;
        if (seed == 0)  // QueryPerformanceCounter: a non-deterministic timer value
            st = (uint64_t)std::chrono::steady_clock::now().time_since_epoch().count();
        else
            st = (uint64_t)seed;
        s0 = splitmix64(st);
        s1 = splitmix64(st);
        s2 = splitmix64(st);
        s3 = splitmix64(st);
    }
    uint64_t next() {  // Sampler.pas:208-222
        uint64_t result = rotl64(s1 * 5, 7) * 9;
        uint64_t t = s1 << 17;
        s2 ^= s0;
        s3 ^= s1;
        s1 ^= s2;
        s0 ^= s3;
        s2 ^= t;
        s3 = rotl64(s3, 45);
        return result;
    }
    float next_float() {  // Sampler.pas:243-248: upper 24 bits / 2^24
        return (float)((double)(next() >> 40) / 16777216.0);
    }
};

// ---- helpers ----------------------------------------------------------------------
inline float f32(double v) { return (float)v; }

inline float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// Exponent e of a positive finite float such that its ulp is 2^(e-23); subnormals
// count as e = -126 (they are multiples of 2^-149).
inline int float_exp(float p) {
    int e;
    std::frexp(p, &e);  // p = m * 2^e, m in [0.5, 1)
    e -= 1;
    return e < -126 ? -126 : e;
}

// True when every partial sum of the non-zero probabilities, in any order, is exact
// in double. All terms are multiples of 2^(emin-23) and every partial sum is at most
// n*pmax < 2^(E+1) with E = floor(log2(n*pmax)); such sums fit 53 bits iff
// emin >= E - 29. n*pmax is exact in double, so the GPU evaluates the same bound.
bool sums_exact(const float* p, int n_total) {
    int n = 0, emin = 1 << 20;
    float pmax = 0.0f;
    for (int i = 0; i < n_total; ++i)
        if (p[i] > 0.0f) {
            ++n;
            emin = std::min(emin, float_exp(p[i]));
            pmax = std::max(pmax, p[i]);
        }
    if (n == 0) return true;
    int E;
    std::frexp((double)n * (double)pmax, &E);
    E -= 1;
    return emin >= E - 29;
}

struct Workspace {
    std::vector<float> buf, pre, probs, row;
    std::vector<int32_t> idx, order;
};

struct Diag {
    uint32_t flags = 0;
    int32_t* out_idx = nullptr;
    float* out_prob = nullptr;
    int32_t out_k = 0;
};

// Repetition penalty, Sampler.pas:285-303 (applied once per ring slot, duplicates
// compound; value 0 unchanged; ids outside [0, V) skipped).
void apply_penalty(const vdxs_config& cfg, float* x, int V, const int32_t* hist, int hcount) {
    if (!(cfg.repeat_penalty != 1.0f) || hcount <= 0 || hist == nullptr) return;
    for (int li = 0; li < hcount; ++li) {
        int id = hist[li];
        if (id >= 0 && id < V) {
            float v = x[id];
            if (v > 0.0f)
                x[id] = f32((double)v / (double)cfg.repeat_penalty);
            else if (v < 0.0f)
                x[id] = f32((double)v * (double)cfg.repeat_penalty);
        }
    }
}

// Greedy, Sampler.pas:305-322: first (lowest index) maximum with strict '>'.
int32_t greedy(const float* x, int V) {
    int32_t best = 0;
    float score = x[0];
    for (int i = 1; i < V; ++i)
        if (x[i] > score) {
            best = i;
            score = x[i];
        }
    return best;
}

void fill_diag_walk(Diag* dg, const float* pre, const int32_t* idx, int K) {
    if (!dg) return;
    for (int j = 0; j < dg->out_k; ++j) {
        if (dg->out_idx) dg->out_idx[j] = j < K ? idx[j] : -1;
        if (dg->out_prob) dg->out_prob[j] = j < K ? pre[j] : 0.0f;
    }
}

// Draw diagnostics shared by both tie modes. `pre` = walk-ordered probabilities
// before the top-p cut; `post` = after it; pos = drawn walk position (K-1 on fallback).
void draw_flags(Diag* dg, const float* pre, const float* post, int K, int pos, bool fallback,
                double t, double lsum, bool sorted_walk) {
    if (!dg) return;
    if (fallback) dg->flags |= VDXS_FLAG_FALLBACK;
    if (sorted_walk && K > 1) {
        bool run = (pos > 0 && pre[pos - 1] == pre[pos]) || (pos + 1 < K && pre[pos + 1] == pre[pos]);
        if (run) dg->flags |= VDXS_FLAG_DRAW_TIE_RUN;
    }
    double before = 0.0;
    for (int i = 0; i < pos; ++i) before += post[i];
    double after = before + post[pos];
    double eps = 1e-6 * lsum;
    if (fallback || (t - before) <= eps || (after - t) <= eps) dg->flags |= VDXS_FLAG_NEAR_BOUNDARY;
}

// Boundary-tie class: more elements equal to the k-th largest value than slots left.
void boundary_flag(Diag* dg, const float* x, int V, int K, float kth) {
    if (!dg) return;
    long gt = 0, eq = 0;
    for (int i = 0; i < V; ++i) {
        if (x[i] > kth) ++gt;
        else if (x[i] == kth) ++eq;
    }
    if (gt + eq > K) dg->flags |= VDXS_FLAG_BOUNDARY_TIE;
}

// ---- top-k path, faithful: Sampler.pas:327-459 -------------------------------------
int32_t topk_faithful(const vdxs_config& cfg, const float* x, int V, float u, Workspace& ws,
                      Diag* dg) {
    const int K = cfg.top_k;
    const float inv_temp = f32(1.0 / (double)cfg.temperature);  // :325
    std::vector<float>& buf = ws.buf;
    std::vector<int32_t>& idx = ws.idx;
    buf.resize(K);
    idx.resize(K);

    // Pass 1 (:341-383): running max plus the K-slot min-buffer.
    float maxv = x[0];
    int min_idx = 0;
    float min_val = -1e30f;
    for (int i = 0; i < V; ++i) {
        float v = x[i];
        if (v > maxv) maxv = v;
        if (i < K) {
            buf[i] = v;
            idx[i] = i;
            if (i == K - 1) {
                min_idx = 0;
                min_val = buf[0];
                for (int j = 1; j < K; ++j)
                    if (buf[j] < min_val) {
                        min_idx = j;
                        min_val = buf[j];
                    }
            }
        } else if (v > min_val) {
            buf[min_idx] = v;
            idx[min_idx] = i;
            min_idx = 0;
            min_val = buf[0];
            for (int j = 1; j < K; ++j)
                if (buf[j] < min_val) {
                    min_idx = j;
                    min_val = buf[j];
                }
        }
    }
    if (dg) boundary_flag(dg, x, V, K, min_val);

    // Pass 2 (:385-391): temperature + exp, Double sum in slot order.
    double lsum = 0.0;
    for (int i = 0; i < K; ++i) {
        buf[i] = f32(std::exp(((double)buf[i] - (double)maxv) * (double)inv_temp));
        lsum += buf[i];
    }
    // Min-P (:393-410).
    if (cfg.min_p > 0.0f) {
        float best = buf[0];
        for (int i = 1; i < K; ++i)
            if (buf[i] > best) best = buf[i];
        float thr = f32((double)best * (double)cfg.min_p);
        lsum = 0.0;
        for (int i = 0; i < K; ++i)
            if (buf[i] < thr)
                buf[i] = 0.0f;
            else
                lsum += buf[i];
    }
    if (dg && !sums_exact(buf.data(), K)) dg->flags |= VDXS_FLAG_INEXACT_SUM;
    // Top-P (:412-445): stable insertion sort descending, then keep while below target.
    bool sorted = false;
    if (cfg.top_p < 1.0f) {
        for (int i = 1; i < K; ++i) {
            float v = buf[i];
            int32_t ti = idx[i];
            int j = i - 1;
            while (j >= 0 && buf[j] < v) {
                buf[j + 1] = buf[j];
                idx[j + 1] = idx[j];
                --j;
            }
            buf[j + 1] = v;
            idx[j + 1] = ti;
        }
        sorted = true;
    }
    if (dg) ws.pre.assign(buf.begin(), buf.end());
    if (sorted) {
        double target = (double)cfg.top_p * lsum;
        double cum = 0.0;
        lsum = 0.0;
        for (int i = 0; i < K; ++i) {
            if (cum < target && buf[i] > 0.0f) {
                cum += buf[i];
                lsum += buf[i];
            } else
                buf[i] = 0.0f;
        }
    } else if (dg && K > 1) {
        dg->flags |= VDXS_FLAG_SLOT_ORDER;
    }
    // Draw (:447-459).
    double t = (double)u * lsum;
    double cum = 0.0;
    int32_t result = idx[K - 1];
    int pos = K - 1;
    bool fallback = true;
    for (int i = 0; i < K; ++i) {
        cum += buf[i];
        if (cum > t) {
            result = idx[i];
            pos = i;
            fallback = false;
            break;
        }
    }
    if (dg) {
        draw_flags(dg, ws.pre.data(), buf.data(), K, pos, fallback, t, lsum, sorted);
        fill_diag_walk(dg, ws.pre.data(), idx.data(), K);
    }
    return result;
}

// ---- top-k path, canonical ----------------------------------------------------------
// Same arithmetic as Sampler.pas:385-459 on the canonical survivor set, walked in
// (probability desc, index asc) order for every top_p.
int32_t topk_canonical(const vdxs_config& cfg, const float* x, int V, float u, Workspace& ws,
                       Diag* dg) {
    const int K = cfg.top_k;
    const float inv_temp = f32(1.0 / (double)cfg.temperature);
    std::vector<int32_t>& order = ws.order;
    order.resize(V);
    std::iota(order.begin(), order.end(), 0);
    auto better = [x](int32_t a, int32_t b) { return x[a] > x[b] || (x[a] == x[b] && a < b); };
    std::nth_element(order.begin(), order.begin() + (K - 1), order.end(), better);
    std::sort(order.begin(), order.begin() + K, better);
    std::vector<float>& buf = ws.buf;
    std::vector<int32_t>& idx = ws.idx;
    buf.resize(K);
    idx.resize(K);
    for (int s = 0; s < K; ++s) {
        idx[s] = order[s];
        buf[s] = x[order[s]];
    }
    const float maxv = buf[0];
    if (dg) boundary_flag(dg, x, V, K, buf[K - 1]);
    for (int i = 0; i < K; ++i)
        buf[i] = f32(std::exp(((double)buf[i] - (double)maxv) * (double)inv_temp));
    if (cfg.min_p > 0.0f) {
        float best = buf[0];
        for (int i = 1; i < K; ++i)
            if (buf[i] > best) best = buf[i];
        float thr = f32((double)best * (double)cfg.min_p);
        for (int i = 0; i < K; ++i)
            if (buf[i] < thr) buf[i] = 0.0f;
    }
    if (dg && !sums_exact(buf.data(), K)) dg->flags |= VDXS_FLAG_INEXACT_SUM;
    // Sort by (p desc, idx asc).
    std::vector<int32_t> perm(K);
    std::iota(perm.begin(), perm.end(), 0);
    std::sort(perm.begin(), perm.end(), [&](int a, int b) {
        return buf[a] > buf[b] || (buf[a] == buf[b] && idx[a] < idx[b]);
    });
    std::vector<float> p(K);
    std::vector<int32_t> id(K);
    for (int i = 0; i < K; ++i) {
        p[i] = buf[perm[i]];
        id[i] = idx[perm[i]];
    }
    double lsum = 0.0;
    for (int i = 0; i < K; ++i) lsum += p[i];
    if (dg) ws.pre.assign(p.begin(), p.end());
    if (cfg.top_p < 1.0f) {
        double target = (double)cfg.top_p * lsum;
        double cum = 0.0;
        lsum = 0.0;
        for (int i = 0; i < K; ++i) {
            if (cum < target && p[i] > 0.0f) {
                cum += p[i];
                lsum += p[i];
            } else
                p[i] = 0.0f;
        }
    } else if (dg && K > 1) {
        dg->flags |= VDXS_FLAG_SLOT_ORDER;
    }
    double t = (double)u * lsum;
    double cum = 0.0;
    int32_t result = id[K - 1];
    int pos = K - 1;
    bool fallback = true;
    for (int i = 0; i < K; ++i) {
        cum += p[i];
        if (cum > t) {
            result = id[i];
            pos = i;
            fallback = false;
            break;
        }
    }
    if (dg) {
        draw_flags(dg, ws.pre.data(), p.data(), K, pos, fallback, t, lsum, true);
        fill_diag_walk(dg, ws.pre.data(), id.data(), K);
    }
    return result;
}

// ---- full-softmax path: Sampler.pas:461-527 --------------------------------------------
int32_t full_path(const vdxs_config& cfg, const float* x, int V, float u, Workspace& ws,
                  Diag* dg) {
    const float inv_temp = f32(1.0 / (double)cfg.temperature);
    std::vector<float>& pr = ws.probs;  // EnsureWorkspace (:250-263)
    pr.resize(V);
    float maxv = f32((double)x[0] * (double)inv_temp);  // :468
    for (int i = 0; i < V; ++i) {                         // :469-476
        float v = f32((double)x[i] * (double)inv_temp);
        pr[i] = v;
        if (v > maxv) maxv = v;
    }
    double lsum = 0.0;  // :479-486
    for (int i = 0; i < V; ++i) {
        float v = f32(std::exp((double)pr[i] - (double)maxv));
        pr[i] = v;
        lsum += v;
    }
    if (cfg.min_p > 0.0f) {  // :489-511
        float best = pr[0];
        for (int i = 1; i < V; ++i)
            if (pr[i] > best) best = pr[i];
        float thr = f32((double)best * (double)cfg.min_p);
        lsum = 0.0;
        for (int i = 0; i < V; ++i) {
            float v = pr[i];
            if (v < thr)
                pr[i] = 0.0f;
            else
                lsum += v;
        }
    }
    double t = (double)u * lsum;  // :514-526
    double cum = 0.0;
    int32_t result = V - 1;
    bool fallback = true;
    double before = 0.0;
    for (int i = 0; i < V; ++i) {
        before = cum;
        cum += pr[i];
        if (cum > t) {
            result = i;
            fallback = false;
            break;
        }
    }
    if (dg) {
        dg->flags |= VDXS_FLAG_FULL;
        if (!sums_exact(pr.data(), V)) dg->flags |= VDXS_FLAG_INEXACT_SUM;
        if (fallback) dg->flags |= VDXS_FLAG_FALLBACK;
        double eps = 1e-6 * lsum;
        if (fallback || (t - before) <= eps || (cum - t) <= eps) dg->flags |= VDXS_FLAG_NEAR_BOUNDARY;
        for (int j = 0; j < dg->out_k; ++j) {
            if (dg->out_idx) dg->out_idx[j] = -1;
            if (dg->out_prob) dg->out_prob[j] = 0.0f;
        }
    }
    return result;
}

// Process after the penalty (Sampler.pas:305-527) with the uniform supplied.
int32_t process_core(const vdxs_config& cfg, int tie_mode, const float* x, int V, float u,
                     Workspace& ws, Diag* dg) {
    if (cfg.temperature == 0.0f) {  // :306
        if (dg) {
            dg->flags |= VDXS_FLAG_GREEDY;
            for (int j = 0; j < dg->out_k; ++j) {
                if (dg->out_idx) dg->out_idx[j] = -1;
                if (dg->out_prob) dg->out_prob[j] = 0.0f;
            }
        }
        int32_t g = greedy(x, V);
        if (dg && dg->out_k > 0 && dg->out_idx) dg->out_idx[0] = g;
        return g;
    }
    if (cfg.top_k > 0 && cfg.top_k < V) {  // :327
        if (dg) dg->flags |= VDXS_FLAG_TOPK;
        return tie_mode == VDXS_TIES_CANONICAL ? topk_canonical(cfg, x, V, u, ws, dg)
                                               : topk_faithful(cfg, x, V, u, ws, dg);
    }
    return full_path(cfg, x, V, u, ws, dg);
}

vdxs_config default_config() {  // Sampler.pas:100-109
    vdxs_config c;
    c.temperature = 0.0f;
    c.top_k = 0;
    c.top_p = 1.0f;
    c.min_p = 0.0f;
    c.repeat_penalty = 1.0f;
    c.repeat_window = 64;
    c.seed = 0;
    return c;
}

}  // namespace

struct vdxo_sampler {
    vdxs_config cfg;
    Prng prng;
    std::vector<int32_t> history;  // FHistory (:48)
    int32_t hist_pos = 0, hist_count = 0;
    Workspace ws;
};

extern "C" {

vdxo_sampler* vdxo_create(void) {  // Sampler.pas:111-122
    vdxo_sampler* s = new vdxo_sampler();
    s->cfg = default_config();
    s->history.assign((size_t)std::max(0, s->cfg.repeat_window), 0);
    s->prng.seed(0);
    return s;
}

void vdxo_destroy(vdxo_sampler* s) { delete s; }

void vdxo_default_config(vdxs_config* out) { *out = default_config(); }

void vdxo_set_config(vdxo_sampler* s, const vdxs_config* cfg) {  // Sampler.pas:132-150
    bool seed_changed = cfg->seed != s->cfg.seed;
    s->cfg = *cfg;
    // SetLength with a non-positive window leaves an empty ring.
    size_t want = (size_t)std::max(0, s->cfg.repeat_window);
    if (s->history.size() != want) {
        s->history.assign(want, 0);
        s->hist_pos = 0;
        s->hist_count = 0;
    }
    if (seed_changed) s->prng.seed(s->cfg.seed);
}

void vdxo_get_config(const vdxo_sampler* s, vdxs_config* out) { *out = s->cfg; }

void vdxo_add_to_history(vdxo_sampler* s, int32_t token) {  // Sampler.pas:530-539
    if (s->cfg.repeat_window <= 0) return;
    s->history[s->hist_pos] = token;
    s->hist_pos = (s->hist_pos + 1) % s->cfg.repeat_window;
    if (s->hist_count < s->cfg.repeat_window) ++s->hist_count;
}

void vdxo_reset_history(vdxo_sampler* s) {  // Sampler.pas:541-549
    s->hist_pos = 0;
    s->hist_count = 0;
    if (s->cfg.seed > 0) s->prng.seed(s->cfg.seed);
}

int32_t vdxo_get_history(const vdxo_sampler* s, int32_t* ids, int32_t cap, int32_t* count,
                         int32_t* pos) {
    *count = s->hist_count;
    *pos = s->hist_pos;
    int n = std::min(cap, s->hist_count);
    for (int i = 0; i < n; ++i) ids[i] = s->history[i];
    return n;
}

int32_t vdxo_process(vdxo_sampler* s, float* logits, int32_t vocab) {  // Sampler.pas:265-528
    if (vocab <= 0 || logits == nullptr) return -1;
    apply_penalty(s->cfg, logits, vocab, s->history.data(), s->hist_count);
    // Greedy draws nothing; every other path draws exactly one NextFloat (:448, :514)
    // and nothing else touches the PRNG, so drawing it here is equivalent.
    float u = 0.0f;
    if (s->cfg.temperature != 0.0f) u = s->prng.next_float();
    return process_core(s->cfg, VDXS_TIES_FAITHFUL, logits, vocab, u, s->ws, nullptr);
}

uint64_t vdxo_next_uint64(vdxo_sampler* s) { return s->prng.next(); }
float vdxo_next_float(vdxo_sampler* s) { return s->prng.next_float(); }
void vdxo_get_state(const vdxo_sampler* s, uint64_t out[4]) {
    out[0] = s->prng.s0;
    out[1] = s->prng.s1;
    out[2] = s->prng.s2;
    out[3] = s->prng.s3;
}
void vdxo_set_state(vdxo_sampler* s, const uint64_t st[4]) {
    s->prng.s0 = st[0];
    s->prng.s1 = st[1];
    s->prng.s2 = st[2];
    s->prng.s3 = st[3];
}
uint64_t vdxo_splitmix64(uint64_t* state) { return splitmix64(*state); }

int32_t vdxo_process_row(const vdxs_config* cfg, int32_t tie_mode, float* logits, int32_t vocab,
                         const int32_t* history, int32_t history_count, float uniform,
                         uint32_t* out_flags, int32_t* out_idx, float* out_prob,
                         int32_t out_k) {
    if (!cfg || !logits || vocab <= 0) return -1;
    Workspace ws;
    Diag dg;
    dg.out_idx = out_idx;
    dg.out_prob = out_prob;
    dg.out_k = out_k;
    apply_penalty(*cfg, logits, vocab, history, history_count);
    int32_t tok = process_core(*cfg, tie_mode, logits, vocab, uniform, ws, &dg);
    if (out_flags) *out_flags = dg.flags;
    return tok;
}

int32_t vdxo_sample_batch(const vdxs_config* cfg, int32_t tie_mode, const void* logits,
                          int32_t dtype, int32_t batch, int32_t vocab, int64_t row_stride,
                          const int32_t* history, int64_t history_stride,
                          const int32_t* history_count, const float* uniform,
                          int32_t* out_tokens, uint32_t* out_flags, int32_t* out_idx,
                          float* out_prob, int32_t out_k, int32_t nthreads) {
    if (!cfg || !logits || !out_tokens || batch <= 0 || vocab <= 0 || row_stride < vocab)
        return -1;
    if (dtype != VDXS_DTYPE_F32 && dtype != VDXS_DTYPE_BF16) return -1;
    if (nthreads <= 0) nthreads = 1;
    nthreads = std::min(nthreads, batch);
    const bool want_diag = out_flags || out_idx || out_prob;
    const bool penalty = cfg->repeat_penalty != 1.0f && history && history_count;

    auto work = [&](int tid) {
        Workspace ws;
        for (int r = tid; r < batch; r += nthreads) {
            const float* x;
            int hcount = history_count ? history_count[r] : 0;
            bool copy = dtype == VDXS_DTYPE_BF16 || (penalty && hcount > 0);
            if (copy) {
                ws.row.resize(vocab);
                if (dtype == VDXS_DTYPE_BF16) {
                    const uint16_t* src = (const uint16_t*)logits + (size_t)r * row_stride;
                    for (int i = 0; i < vocab; ++i) ws.row[i] = bf16_to_f32(src[i]);
                } else {
                    const float* src = (const float*)logits + (size_t)r * row_stride;
                    std::memcpy(ws.row.data(), src, sizeof(float) * vocab);
                }
                if (penalty)
                    apply_penalty(*cfg, ws.row.data(), vocab, history + (size_t)r * history_stride,
                                  hcount);
                x = ws.row.data();
            } else {
                x = (const float*)logits + (size_t)r * row_stride;
            }
            float u = uniform ? uniform[r] : 0.0f;
            if (want_diag) {
                Diag dg;
                dg.out_idx = out_idx ? out_idx + (size_t)r * out_k : nullptr;
                dg.out_prob = out_prob ? out_prob + (size_t)r * out_k : nullptr;
                dg.out_k = (out_idx || out_prob) ? out_k : 0;
                out_tokens[r] = process_core(*cfg, tie_mode, x, vocab, u, ws, &dg);
                if (out_flags) out_flags[r] = dg.flags;
            } else {
                out_tokens[r] = process_core(*cfg, tie_mode, x, vocab, u, ws, nullptr);
            }
        }
    };
    if (nthreads == 1) {
        work(0);
    } else {
        std::vector<std::thread> th;
        th.reserve(nthreads);
        for (int t = 0; t < nthreads; ++t) th.emplace_back(work, t);
        for (auto& t : th) t.join();
    }
    return 0;
}

}  // extern "C"

// ---- unembedding: shaders/matvec_q4_0.comp:45-88 -------------------------------------
namespace {

// IEEE binary16 -> binary32 (unpackHalf2x16, exact for every encoding).
float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t ex = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    uint32_t bits;
    if (ex == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: normalise
            int e = -1;
            uint32_t m = man;
            do {
                ++e;
                m <<= 1;
            } while ((m & 0x400u) == 0);
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (ex == 0x1F) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((ex + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// One output row (matvec_q4_0.comp:45-88): 64 invocations each accumulate the elements
// tid, tid + 64, ... in order (acc += qval * scale * x, evaluated left to right with
// every operation rounded to float), then the shared-memory tree over strides 32..1.
float matvec_q4_0_row(const uint8_t* w, const float* x, int in_dim, int row) {
    const size_t blocks_per_row = (size_t)in_dim >> 5;
    const size_t row_byte_off = (size_t)row * blocks_per_row * 18u;
    float partial[64];
    for (int tid = 0; tid < 64; ++tid) {
        float acc = 0.0f;
        for (int elem = tid; elem < in_dim; elem += 64) {
            const size_t blk_off = row_byte_off + (size_t)(elem >> 5) * 18u;
            const int in_blk = elem & 31;
            const int byte_idx = in_blk & 15;
            const int is_high = in_blk >> 4;
            const float scale = half_to_float((uint16_t)(w[blk_off] | (w[blk_off + 1] << 8)));
            const uint32_t raw = w[blk_off + 2 + byte_idx];
            const uint32_t nibble = (raw >> (is_high * 4)) & 0x0Fu;
            const float qval = (float)((int)nibble - 8);
            const float qs = qval * scale;  // exact: a 4-bit integer times an fp16 value
            const float t = qs * x[elem];
            acc = acc + t;
        }
        partial[tid] = acc;
    }
    for (int stride = 32; stride > 0; stride >>= 1)
        for (int tid = 0; tid < stride; ++tid) partial[tid] = partial[tid] + partial[tid + stride];
    return partial[0];
}

}  // namespace

int32_t vdxo_matvec_q4_0(const uint8_t* weights, const float* x, int32_t batch, int32_t in_dim,
                         int32_t out_dim, float* out, int32_t nthreads) {
    if (!weights || !x || !out || batch <= 0 || in_dim <= 0 || (in_dim & 31) || out_dim <= 0) return -1;
    if (nthreads <= 0) nthreads = 1;
    auto work = [&](int t) {
        for (int r = t; r < out_dim; r += nthreads)
            for (int b = 0; b < batch; ++b)
                out[(size_t)b * out_dim + r] = matvec_q4_0_row(weights, x + (size_t)b * in_dim, in_dim, r);
    };
    std::vector<std::thread> th;
    for (int t = 1; t < nthreads; ++t) th.emplace_back(work, t);
    work(0);
    for (auto& h : th) h.join();
    return 0;
}
