// noetic_oracle.cpp -- CPU oracle: a C++ restatement of the reference's f32
// token-loop path, used ONLY by the tests, the smoke check and the benchmark's
// CPU-baseline leg as the checker.  Never linked into the product library.
//
// Parity status: pinned by the reference's known-answer and property tests
// (see noetic_oracle.h); RNG / seeded-init bit-exactness is unpinned (no
// known-answer vectors exist in the reference and it cannot be built here).
//
// Numerics rules followed throughout (the reference is Rust, which performs no
// FMA contraction and calls the platform libm for exp/ln/powf):
//   * build with -ffp-contract=off -fno-fast-math, f32 arithmetic in f32;
//   * f64 only where the reference uses f64 (sample_token's total and draw);
//   * identical loop and accumulation order in every reduction.

#include "noetic_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <set>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace {

thread_local std::string g_last_error;

void set_error(const std::string &m) { g_last_error = m; }

// ---------------------------------------------------------------- rng.rs
// splitmix64 follows rng.rs:9-15; Rng::new rng.rs:25-38; next_u64 rng.rs:46-56.
inline uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

uint64_t splitmix(uint64_t *state) {
    *state += 0x9E3779B97F4A7C15ull;
    uint64_t z = *state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

void rng_new(orc_rng *r, uint64_t seed) {
    uint64_t z = seed ^ 0xA0761D6478BD642Full;
    for (int i = 0; i < 4; ++i) r->s[i] = splitmix(&z);
    if (r->s[0] == 0 && r->s[1] == 0 && r->s[2] == 0 && r->s[3] == 0) r->s[0] = 0x9E3779B97F4A7C15ull;
    r->spare = 0.0f;
    r->has_spare = 0;
}

uint64_t next_u64(orc_rng *r) {
    uint64_t *s = r->s;
    const uint64_t result = rotl(s[0] + s[3], 23) + s[0];
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl(s[3], 45);
    return result;
}

// rng.rs:65-67: 24 high bits scaled by 2^-24.
float f32_unit(orc_rng *r) { return (float)(next_u64(r) >> 40) * (1.0f / 16777216.0f); }

// rng.rs:70-72
float uniform(orc_rng *r, float lo, float hi) { return lo + (hi - lo) * f32_unit(r); }

// rng.rs:75-90: Lemire threshold rejection, then modulo.
uint64_t below(orc_rng *r, uint64_t n) {
    if (n == 0) throw std::runtime_error("Rng::below requires a positive bound");
    if (n == 1) return 0;
    const uint64_t threshold = (0 - n) % n;
    for (;;) {
        uint64_t v = next_u64(r);
        if (v >= threshold) return v % n;
    }
}

// rng.rs:93-109: Marsaglia polar with one cached spare.
float normal(orc_rng *r) {
    if (r->has_spare) {
        r->has_spare = 0;
        return r->spare;
    }
    for (;;) {
        float u = uniform(r, -1.0f, 1.0f);
        float v = uniform(r, -1.0f, 1.0f);
        float s = u * u + v * v;
        if (s > 0.0f && s < 1.0f) {
            float f = std::sqrt(-2.0f * std::log(s) / s);
            r->spare = v * f;
            r->has_spare = 1;
            return u * f;
        }
    }
}

// ---------------------------------------------------------------- tensor.rs
const uint64_t MIN_WORK_PER_THREAD = 128 * 1024;  // tensor.rs:20

uint64_t worker_count(uint64_t requested, uint64_t jobs, uint64_t total_work) {  // tensor.rs:22-28
    if (jobs < 2 || total_work < MIN_WORK_PER_THREAD) return 1;
    uint64_t useful = std::max<uint64_t>(total_work / MIN_WORK_PER_THREAD, 1);
    return std::min(std::min(std::max<uint64_t>(requested, 1), jobs), useful);
}

// tensor.rs:247-273: four strided accumulators, ((s0+s1)+(s2+s3)), tail, bias.
void kern_matvec(const float *w, const float *bias, const float *x, float *out, uint64_t r0,
                 uint64_t rows, uint64_t din) {
    for (uint64_t i = 0; i < rows; ++i) {
        const uint64_t o = r0 + i;
        const float *wr = w + o * din;
        float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
        uint64_t p = 0;
        while (p + 4 <= din) {
            s0 += wr[p] * x[p];
            s1 += wr[p + 1] * x[p + 1];
            s2 += wr[p + 2] * x[p + 2];
            s3 += wr[p + 3] * x[p + 3];
            p += 4;
        }
        float s = (s0 + s1) + (s2 + s3);
        while (p < din) {
            s += wr[p] * x[p];
            ++p;
        }
        if (bias) s += bias[o];
        out[i] = s;
    }
}

// tensor.rs:221-245: row split over scoped threads (one spawn per call).
void matvec_nt(const float *w, const float *bias, const float *x, float *out, uint64_t dout,
               uint64_t din, uint64_t threads) {
    if (dout == 0) return;
    uint64_t nt = worker_count(threads, dout, dout * din);
    if (nt == 1) {
        kern_matvec(w, bias, x, out, 0, dout, din);
        return;
    }
    uint64_t rows = 1 + (dout - 1) / nt;
    std::vector<std::thread> pool;
    for (uint64_t r0 = 0; r0 < dout; r0 += rows) {
        uint64_t cnt = std::min(rows, dout - r0);
        pool.emplace_back([=] { kern_matvec(w, bias, x, out + r0, r0, cnt, din); });
    }
    for (auto &t : pool) t.join();
}

// tensor.rs:125-151
void kern_nt(const float *a, const float *b, float *c, uint64_t r0, uint64_t rows, uint64_t k,
             uint64_t n) {
    for (uint64_t i = 0; i < rows; ++i) {
        const float *ar = a + (r0 + i) * k;
        float *cr = c + i * n;
        for (uint64_t j = 0; j < n; ++j) {
            const float *br = b + j * k;
            float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
            uint64_t p = 0;
            while (p + 4 <= k) {
                s0 += ar[p] * br[p];
                s1 += ar[p + 1] * br[p + 1];
                s2 += ar[p + 2] * br[p + 2];
                s3 += ar[p + 3] * br[p + 3];
                p += 4;
            }
            float s = (s0 + s1) + (s2 + s3);
            while (p < k) {
                s += ar[p] * br[p];
                ++p;
            }
            cr[j] = s;
        }
    }
}

// tensor.rs:101-123
void gemm_nt(const float *a, const float *b, float *c, uint64_t m, uint64_t k, uint64_t n,
             uint64_t threads) {
    if (m == 0 || n == 0) return;
    uint64_t nt = worker_count(threads, m, m * k * n);
    if (nt == 1) {
        kern_nt(a, b, c, 0, m, k, n);
        return;
    }
    uint64_t rows = 1 + (m - 1) / nt;
    std::vector<std::thread> pool;
    for (uint64_t r0 = 0; r0 < m; r0 += rows) {
        uint64_t cnt = std::min(rows, m - r0);
        pool.emplace_back([=] { kern_nt(a, b, c + r0 * n, r0, cnt, k, n); });
    }
    for (auto &t : pool) t.join();
}

// tensor.rs:276-288: branchy stable sigmoid; silu = x * sigmoid(x).
inline float sigmoid(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + std::exp(-x));
    float e = std::exp(x);
    return e / (1.0f + e);
}
inline float silu(float x) { return x * sigmoid(x); }

// tensor.rs:298-312
void rms_norm_vec(const float *x, const float *w, float eps, float *out, uint64_t d) {
    float ms = 0.0f;
    for (uint64_t i = 0; i < d; ++i) ms += x[i] * x[i];
    float r = 1.0f / std::sqrt(ms / (float)d + eps);
    for (uint64_t i = 0; i < d; ++i) out[i] = x[i] * r * w[i];
}

// tensor.rs:314-352
void softmax_inplace(float *x, uint64_t n) {
    uint64_t pos_inf = 0;
    for (uint64_t i = 0; i < n; ++i)
        if (x[i] == INFINITY) ++pos_inf;
    if (pos_inf > 0) {
        float p = 1.0f / (float)pos_inf;
        for (uint64_t i = 0; i < n; ++i) x[i] = (x[i] == INFINITY) ? p : 0.0f;
        return;
    }
    float mx = -INFINITY;
    for (uint64_t i = 0; i < n; ++i)
        if (std::isfinite(x[i]) && x[i] > mx) mx = x[i];
    if (mx == -INFINITY) {
        for (uint64_t i = 0; i < n; ++i) x[i] = 1.0f / (float)n;
        return;
    }
    float s = 0.0f;
    for (uint64_t i = 0; i < n; ++i) {
        float e = std::isfinite(x[i]) ? std::exp(x[i] - mx) : 0.0f;
        x[i] = e;
        s += e;
    }
    if (!std::isfinite(s) || s <= 0.0f) {
        for (uint64_t i = 0; i < n; ++i) x[i] = 1.0f / (float)n;
        return;
    }
    float inv = 1.0f / s;
    for (uint64_t i = 0; i < n; ++i) x[i] *= inv;
}

// tensor.rs:354-365: first index of the strict maximum, NaN skipped.
uint64_t argmax(const float *x, uint64_t n) {
    uint64_t best = 0;
    float bv = std::isnan(x[0]) ? -INFINITY : x[0];
    for (uint64_t i = 1; i < n; ++i)
        if (!std::isnan(x[i]) && x[i] > bv) {
            bv = x[i];
            best = i;
        }
    return best;
}

// f32::total_cmp as a sortable integer key (IEEE total order).
inline int32_t total_key(float f) {
    int32_t b;
    std::memcpy(&b, &f, 4);
    return b ^ (int32_t)((uint32_t)(b >> 31) >> 1);
}

// ---------------------------------------------------------------- scan.rs
const float DECAY_FLOOR = 1e-30f;  // scan.rs:27

void kern_scan_seq(const float *a, const float *b, float *h, uint64_t b0, uint64_t batch,
                   uint64_t t, uint64_t d) {  // scan.rs:59-77
    std::vector<float> carry(d);
    for (uint64_t bi = 0; bi < batch; ++bi) {
        uint64_t gbase = (b0 + bi) * t * d, lbase = bi * t * d;
        std::fill(carry.begin(), carry.end(), 0.0f);
        for (uint64_t ti = 0; ti < t; ++ti) {
            uint64_t g = gbase + ti * d, l = lbase + ti * d;
            for (uint64_t j = 0; j < d; ++j) {
                float v = a[g + j] * carry[j] + b[g + j];
                carry[j] = v;
                h[l + j] = v;
            }
        }
    }
}

void scan_sequential(const float *a, const float *b, float *h, uint64_t batch, uint64_t t,
                     uint64_t d, uint64_t threads) {  // scan.rs:35-57
    uint64_t n = batch * t * d;
    if (n == 0) return;
    uint64_t nt = worker_count(threads, batch, n);
    if (nt == 1) {
        kern_scan_seq(a, b, h, 0, batch, t, d);
        return;
    }
    uint64_t per = 1 + (batch - 1) / nt;
    std::vector<std::thread> pool;
    for (uint64_t b0 = 0; b0 < batch; b0 += per) {
        uint64_t cnt = std::min(per, batch - b0);
        pool.emplace_back([=] { kern_scan_seq(a, b, h + b0 * t * d, b0, cnt, t, d); });
    }
    for (auto &th : pool) th.join();
}

// scan.rs:98-225.  Three passes over the same time chunking as the reference
// (per = 1 + (t-1)/nt); jobs are independent so they run serially here.
void scan_chunked(const float *a, const float *b, float *h, uint64_t batch, uint64_t t,
                  uint64_t d, uint64_t threads) {
    uint64_t n = batch * t * d;
    if (n == 0) return;
    uint64_t span = t * d;
    uint64_t nt = worker_count(threads, t, n);
    if (nt == 1 || t < 2) {
        scan_sequential(a, b, h, batch, t, d, threads);
        return;
    }
    uint64_t per = 1 + (t - 1) / nt;
    uint64_t chunks = 1 + (t - 1) / per;
    std::vector<float> chunk_decay(batch * chunks * d, 0.0f), carry_in(batch * chunks * d, 0.0f);
    std::vector<float> carry(d);
    // pass 1
    for (uint64_t bi = 0; bi < batch; ++bi) {
        for (uint64_t ci = 0; ci < chunks; ++ci) {
            uint64_t base = bi * span + ci * per * d;
            uint64_t rows = std::min(per, t - ci * per);
            float *dc = &chunk_decay[(bi * chunks + ci) * d];
            std::fill(carry.begin(), carry.end(), 0.0f);
            std::fill(dc, dc + d, 1.0f);
            bool last_chunk = ci + 1 == chunks;
            for (uint64_t i = 0; i < rows; ++i) {
                uint64_t g = base + i * d;
                for (uint64_t j = 0; j < d; ++j) {
                    float v = a[g + j] * carry[j] + b[g + j];
                    carry[j] = v;
                    h[g + j] = v;
                }
                if (last_chunk) continue;
                for (uint64_t j = 0; j < d; ++j) {
                    float p = dc[j] * a[g + j];
                    dc[j] = std::fabs(p) < DECAY_FLOOR ? 0.0f : p;
                }
            }
        }
    }
    // pass 2
    for (uint64_t bi = 0; bi < batch; ++bi)
        for (uint64_t ci = 1; ci < chunks; ++ci) {
            uint64_t prev = (bi * chunks + ci - 1) * d, cur = (bi * chunks + ci) * d;
            uint64_t last_row = bi * span + (ci * per - 1) * d;
            for (uint64_t j = 0; j < d; ++j)
                carry_in[cur + j] = h[last_row + j] + chunk_decay[prev + j] * carry_in[prev + j];
        }
    // pass 3
    std::vector<float> product(d);
    for (uint64_t bi = 0; bi < batch; ++bi)
        for (uint64_t ci = 1; ci < chunks; ++ci) {
            uint64_t base = bi * span + ci * per * d;
            uint64_t rows = std::min(per, t - ci * per);
            const float *cc = &carry_in[(bi * chunks + ci) * d];
            std::copy(cc, cc + d, product.begin());
            for (uint64_t i = 0; i < rows; ++i) {
                uint64_t g = base + i * d;
                bool alive = false;
                for (uint64_t j = 0; j < d; ++j) {
                    float s = product[j] * a[g + j];
                    s = std::fabs(s) < DECAY_FLOOR ? 0.0f : s;
                    product[j] = s;
                    h[g + j] += s;
                    alive |= s != 0.0f;
                }
                if (!alive) break;
            }
        }
}

// ---------------------------------------------------------------- model.rs / nn.rs
struct Tensor {
    std::string name;
    std::vector<uint64_t> shape;
    std::vector<float> val;
};

struct LayerIds {
    int n1, in_w, in_b, conv_w, conv_b, out_w, out_b, n2, up_w, up_b, down_w, down_b;
};

std::string config_error(const orc_config &c) {  // model.rs:37-76
    if (c.vocab == 0) return "vocabulary size must be positive";
    if (c.vocab > 0xFFFFFFFFull) return "vocabulary exceeds the u32 token-id space";
    if (c.d_model == 0) return "d_model must be positive";
    if (c.n_layer == 0) return "n_layer must be positive";
    if (c.expand == 0) return "expand must be positive";
    if (c.conv_k == 0) return "conv_k must be positive";
    if (c.mlp_mult == 0) return "mlp_mult must be positive";
    if (!std::isfinite(c.eps) || c.eps <= 0.0f) return "RMSNorm epsilon must be finite and positive";
    if (!std::isfinite(c.tau_max) || c.tau_max < 1.0f) return "tau_max must be finite and at least one";
    return "";
}

}  // namespace

struct orc_model {
    orc_config cfg;
    uint64_t threads = 1;
    std::vector<Tensor> tensors;  // creation order == checkpoint order
    int emb = -1, norm_f = -1;
    std::vector<LayerIds> layers;

    uint64_t d() const { return cfg.d_model; }
    uint64_t e() const { return cfg.d_model * cfg.expand; }
    uint64_t hidden() const { return cfg.d_model * cfg.mlp_mult; }
    uint64_t k() const { return cfg.conv_k; }
    uint64_t vocab() const { return cfg.vocab; }
    const float *v(int id) const { return tensors[id].val.data(); }

    int add(const std::string &name, std::vector<uint64_t> shape, std::vector<float> val) {
        tensors.push_back(Tensor{name, std::move(shape), std::move(val)});
        return (int)tensors.size() - 1;
    }
};

namespace {

std::vector<float> fill_normal(orc_rng *rng, uint64_t n, float std_) {  // nn.rs:8-15
    std::vector<float> v(n);
    for (uint64_t i = 0; i < n; ++i) v[i] = normal(rng) * std_;
    return v;
}

float init_std(uint64_t fan_in) { return std::sqrt(2.0f / (float)std::max<uint64_t>(fan_in, 1)); }

// Linear::new, nn.rs:31-39: weight draws, then a zero bias.
void linear_new(orc_model *m, orc_rng *rng, const std::string &name, uint64_t din, uint64_t dout,
                float std_, int *w, int *b) {
    std::vector<float> wv = fill_normal(rng, dout * din, std_);
    *w = m->add(name + ".w", {dout, din}, std::move(wv));
    *b = m->add(name + ".b", {dout}, std::vector<float>(dout, 0.0f));
}

// Lm::new, model.rs:183-206 (with SsmLayer::new model.rs:111-146 and
// SwiGlu::new nn.rs:80-88), drawing from one rng in creation order.
void lm_init(orc_model *m, orc_rng *rng) {
    const orc_config &c = m->cfg;
    const uint64_t d = c.d_model, e = m->e(), hidden = m->hidden(), k = c.conv_k;
    {
        std::vector<float> emb(c.vocab * d);
        for (auto &x : emb) x = normal(rng) * 0.02f;
        m->emb = m->add("emb", {c.vocab, d}, std::move(emb));
    }
    const float depth_scale = 1.0f / std::sqrt(2.0f * (float)c.n_layer);
    for (uint64_t layer = 0; layer < c.n_layer; ++layer) {
        LayerIds L{};
        std::string name = "blk" + std::to_string(layer);
        L.n1 = m->add(name + ".n1.gain", {d}, std::vector<float>(d, 1.0f));
        std::string ssm = name + ".ssm";
        linear_new(m, rng, ssm + ".in_proj", d, 3 * e, init_std(d), &L.in_w, &L.in_b);
        {
            float *bias = m->tensors[L.in_b].val.data();
            for (uint64_t j = 0; j < e; ++j) {
                float fraction = e > 1 ? (float)j / (float)(e - 1) : 0.0f;
                float tau = std::pow(c.tau_max, fraction);
                float decay = std::exp(-1.0f / tau);
                decay = std::min(std::max(decay, 0.001f), 0.9999f);
                bias[e + j] = std::log(decay / (1.0f - decay));
            }
        }
        {
            std::vector<float> conv(k * e, 0.0f);
            for (uint64_t j = 0; j < e; ++j) conv[j] = 1.0f;
            for (uint64_t q = 1; q < k; ++q)
                for (uint64_t j = 0; j < e; ++j) conv[q * e + j] = normal(rng) * 0.1f;
            L.conv_w = m->add(ssm + ".conv_w", {k, e}, std::move(conv));
            L.conv_b = m->add(ssm + ".conv_b", {e}, std::vector<float>(e, 0.0f));
        }
        linear_new(m, rng, ssm + ".out_proj", e, d, init_std(e) * depth_scale, &L.out_w, &L.out_b);
        L.n2 = m->add(name + ".n2.gain", {d}, std::vector<float>(d, 1.0f));
        linear_new(m, rng, name + ".mlp.up", d, 2 * hidden, init_std(d), &L.up_w, &L.up_b);
        linear_new(m, rng, name + ".mlp.down", hidden, d, init_std(hidden) * depth_scale, &L.down_w,
                   &L.down_b);
        m->layers.push_back(L);
    }
    m->norm_f = m->add("norm_f.gain", {d}, std::vector<float>(d, 1.0f));
}

// ---------------------------------------------------------------- autograd.rs forward
// dwconv, autograd.rs:550-575: y[b,t,j] = bias[j] + sum_{q<min(t+1,k)} w[q,j] x[b,t-q,j].
void dwconv(const float *x, const float *w, const float *bias, float *out, uint64_t batch,
            uint64_t t, uint64_t d, uint64_t k) {
    for (uint64_t bi = 0; bi < batch; ++bi) {
        uint64_t base = bi * t * d;
        for (uint64_t ti = 0; ti < t; ++ti) {
            uint64_t o = base + ti * d;
            for (uint64_t j = 0; j < d; ++j) out[o + j] = bias[j];
            uint64_t qmax = ti + 1 < k ? ti + 1 : k;
            for (uint64_t q = 0; q < qmax; ++q) {
                uint64_t src = base + (ti - q) * d;
                for (uint64_t j = 0; j < d; ++j) out[o + j] += w[q * d + j] * x[src + j];
            }
        }
    }
}

// rms_norm (autograd.rs:458-483) followed by mul_row (autograd.rs:376-392).
void rms_norm_rows(const float *x, const float *gain, float eps, float *out, uint64_t rows,
                   uint64_t d) {
    for (uint64_t i = 0; i < rows; ++i) {
        float ms = 0.0f;
        for (uint64_t j = 0; j < d; ++j) ms += x[i * d + j] * x[i * d + j];
        float r = 1.0f / std::sqrt(ms / (float)d + eps);
        for (uint64_t j = 0; j < d; ++j) out[i * d + j] = x[i * d + j] * r;
        for (uint64_t j = 0; j < d; ++j) out[i * d + j] = out[i * d + j] * gain[j];
    }
}

// Linear::forward, nn.rs:41-47: matmul_nt then add_row.
void linear_rows(const orc_model *m, int w, int b, const float *x, float *y, uint64_t rows,
                 uint64_t din, uint64_t dout) {
    gemm_nt(x, m->v(w), y, rows, din, dout, m->threads);
    const float *bias = m->v(b);
    for (uint64_t i = 0; i < rows; ++i)
        for (uint64_t j = 0; j < dout; ++j) y[i * dout + j] = y[i * dout + j] + bias[j];
}

bool chunked_scan_wanted(int policy, uint64_t threads, uint64_t batch, uint64_t t, uint64_t d) {
    // autograd.rs:539-545; policy 0 = Auto, 1 = Sequential, 2 = Chunked.
    if (policy == 1) return false;
    if (policy == 2) return true;
    return threads > 1 && batch * 2 <= threads && t >= 512 && batch * t * d >= (1u << 16);
}

// Lm::logits, model.rs:209-226, optionally capturing the decoder state left
// after the last position (infer.rs:32, 157-159; autograd.rs:564).
void lm_forward(const orc_model *m, const uint32_t *ids, uint64_t batch, uint64_t t, int policy,
                float *logits, float *state_out, uint32_t *heads_out, float *last_logits) {
    const uint64_t d = m->d(), e = m->e(), hidden = m->hidden(), k = m->k(), V = m->vocab();
    const uint64_t rows = batch * t;
    std::vector<float> x(rows * d), h1(rows * d), u(rows * 3 * e), vv(rows * e), z(rows * e),
        o(rows * e), conv(rows * e), a(rows * e), bb(rows * e), hs(rows * e), y(rows * e),
        r(rows * d), up(rows * 2 * hidden), s(rows * hidden);
    for (uint64_t i = 0; i < rows; ++i) {
        if (ids[i] >= V) throw std::runtime_error("embed: token out of range");
        std::memcpy(&x[i * d], m->v(m->emb) + (uint64_t)ids[i] * d, d * sizeof(float));
    }
    const uint64_t per_stream = m->cfg.n_layer * (k + 1) * e;
    for (uint64_t li = 0; li < m->cfg.n_layer; ++li) {
        const LayerIds &L = m->layers[li];
        rms_norm_rows(x.data(), m->v(L.n1), m->cfg.eps, h1.data(), rows, d);
        linear_rows(m, L.in_w, L.in_b, h1.data(), u.data(), rows, d, 3 * e);
        for (uint64_t i = 0; i < rows; ++i)
            for (uint64_t j = 0; j < e; ++j) {
                vv[i * e + j] = u[i * 3 * e + j];
                z[i * e + j] = u[i * 3 * e + e + j];
                o[i * e + j] = u[i * 3 * e + 2 * e + j];
            }
        dwconv(vv.data(), m->v(L.conv_w), m->v(L.conv_b), conv.data(), batch, t, e, k);
        for (uint64_t i = 0; i < rows * e; ++i) {
            float value = silu(conv[i]);
            float decay = sigmoid(z[i]);
            float update = 1.0f - decay;
            a[i] = decay;
            bb[i] = update * value;
        }
        if (chunked_scan_wanted(policy, m->threads, batch, t, e))
            scan_chunked(a.data(), bb.data(), hs.data(), batch, t, e, m->threads);
        else
            scan_sequential(a.data(), bb.data(), hs.data(), batch, t, e, m->threads);
        for (uint64_t i = 0; i < rows * e; ++i) y[i] = hs[i] * silu(o[i]);
        if (state_out) {
            for (uint64_t bi = 0; bi < batch; ++bi) {
                float *st = state_out + bi * per_stream + li * (k + 1) * e;
                uint64_t head = (k - 1 + t) % k;
                std::fill(st, st + k * e, 0.0f);
                for (uint64_t q = 0; q < std::min(t, k); ++q) {
                    uint64_t slot = (head + k - q) % k;
                    std::memcpy(st + slot * e, &vv[(bi * t + t - 1 - q) * e], e * sizeof(float));
                }
                std::memcpy(st + k * e, &hs[(bi * t + t - 1) * e], e * sizeof(float));
                if (heads_out) heads_out[bi] = (uint32_t)head;
            }
        }
        linear_rows(m, L.out_w, L.out_b, y.data(), r.data(), rows, e, d);
        for (uint64_t i = 0; i < rows * d; ++i) x[i] = x[i] + r[i];
        rms_norm_rows(x.data(), m->v(L.n2), m->cfg.eps, h1.data(), rows, d);
        linear_rows(m, L.up_w, L.up_b, h1.data(), up.data(), rows, d, 2 * hidden);
        for (uint64_t i = 0; i < rows; ++i)
            for (uint64_t j = 0; j < hidden; ++j)
                s[i * hidden + j] = silu(up[i * 2 * hidden + j]) * up[i * 2 * hidden + hidden + j];
        linear_rows(m, L.down_w, L.down_b, s.data(), r.data(), rows, hidden, d);
        for (uint64_t i = 0; i < rows * d; ++i) x[i] = x[i] + r[i];
    }
    rms_norm_rows(x.data(), m->v(m->norm_f), m->cfg.eps, h1.data(), rows, d);
    if (logits) gemm_nt(h1.data(), m->v(m->emb), logits, rows, d, V, m->threads);
    if (last_logits) {
        for (uint64_t bi = 0; bi < batch; ++bi)
            gemm_nt(&h1[(bi * t + t - 1) * d], m->v(m->emb), last_logits + bi * V, 1, d, V,
                    m->threads);
    }
}

}  // namespace

// ---------------------------------------------------------------- infer.rs
struct orc_state {
    uint64_t n_layer, k, e;
    std::vector<std::vector<float>> conv, h;
    uint64_t head;
};

namespace {
struct Scratch {
    std::vector<float> x, norm, proj, conv_value, gated, residual, up, gated_mlp;
};

// infer.rs:106-200 step_with_scratch
void step_impl(const orc_model *m, orc_state *st, uint32_t token, float *logits) {
    const uint64_t d = m->d(), e = m->e(), k = m->k(), hidden = m->hidden(), V = m->vocab();
    if (token >= V) throw std::runtime_error("streaming token is outside the vocabulary");
    thread_local Scratch s;
    s.x.resize(d);
    s.norm.resize(d);
    s.proj.resize(3 * e);
    s.conv_value.resize(e);
    s.gated.resize(e);
    s.residual.resize(d);
    s.up.resize(2 * hidden);
    s.gated_mlp.resize(hidden);
    std::memcpy(s.x.data(), m->v(m->emb) + (uint64_t)token * d, d * sizeof(float));
    const uint64_t threads = m->threads;
    // All layers share one head advance per token (every layer's conv_head
    // moves in lockstep in the reference, infer.rs:157).
    const uint64_t head = (st->head + 1) % k;
    for (uint64_t li = 0; li < m->cfg.n_layer; ++li) {
        const LayerIds &L = m->layers[li];
        float *ring = st->conv[li].data();
        float *hh = st->h[li].data();
        rms_norm_vec(s.x.data(), m->v(L.n1), m->cfg.eps, s.norm.data(), d);
        matvec_nt(m->v(L.in_w), m->v(L.in_b), s.norm.data(), s.proj.data(), 3 * e, d, threads);
        std::memcpy(ring + head * e, s.proj.data(), e * sizeof(float));
        const float *cw = m->v(L.conv_w), *cb = m->v(L.conv_b);
        for (uint64_t j = 0; j < e; ++j) {
            float sum = cb[j];
            for (uint64_t q = 0; q < k; ++q) {
                uint64_t slot = (head + k - q) % k;
                sum += cw[q * e + j] * ring[slot * e + j];
            }
            s.conv_value[j] = silu(sum);
        }
        for (uint64_t j = 0; j < e; ++j) {
            float decay = sigmoid(s.proj[e + j]);
            hh[j] = decay * hh[j] + (1.0f - decay) * s.conv_value[j];
            s.gated[j] = hh[j] * silu(s.proj[2 * e + j]);
        }
        matvec_nt(m->v(L.out_w), m->v(L.out_b), s.gated.data(), s.residual.data(), d, e, threads);
        for (uint64_t j = 0; j < d; ++j) s.x[j] += s.residual[j];
        rms_norm_vec(s.x.data(), m->v(L.n2), m->cfg.eps, s.norm.data(), d);
        matvec_nt(m->v(L.up_w), m->v(L.up_b), s.norm.data(), s.up.data(), 2 * hidden, d, threads);
        for (uint64_t j = 0; j < hidden; ++j) s.gated_mlp[j] = silu(s.up[j]) * s.up[hidden + j];
        matvec_nt(m->v(L.down_w), m->v(L.down_b), s.gated_mlp.data(), s.residual.data(), d, hidden,
                  threads);
        for (uint64_t j = 0; j < d; ++j) s.x[j] += s.residual[j];
    }
    st->head = head;
    rms_norm_vec(s.x.data(), m->v(m->norm_f), m->cfg.eps, s.norm.data(), d);
    matvec_nt(m->v(m->emb), nullptr, s.norm.data(), logits, V, d, threads);
}

// infer.rs:228-305 sample_token (plus margin diagnostics).
uint32_t sample_impl(float *logits, uint64_t vocab, const orc_sample_cfg *cfg,
                     const uint32_t *history, uint64_t n_hist, orc_rng *rng,
                     orc_sample_info *info) {
    if (vocab == 0) throw std::runtime_error("cannot sample from an empty vocabulary");
    orc_sample_info local{};
    local.order_margin = INFINITY;
    if (std::isfinite(cfg->rep_penalty) && cfg->rep_penalty > 1.0f && cfg->rep_window > 0) {
        uint64_t start = n_hist > cfg->rep_window ? n_hist - cfg->rep_window : 0;
        for (uint64_t i = start; i < n_hist; ++i) {
            uint32_t tok = history[i];
            if (tok >= vocab) continue;
            bool seen = false;
            for (uint64_t q = start; q < i; ++q)
                if (history[q] == tok) {
                    seen = true;
                    break;
                }
            if (seen) continue;
            if (logits[tok] > 0.0f)
                logits[tok] /= cfg->rep_penalty;
            else
                logits[tok] *= cfg->rep_penalty;
        }
    }
    if (cfg->greedy) {
        uint64_t best = argmax(logits, vocab);
        float second = -INFINITY;
        for (uint64_t i = 0; i < vocab; ++i)
            if (i != best && !std::isnan(logits[i]) && logits[i] > second) second = logits[i];
        local.token = (uint32_t)best;
        local.top2_margin = (double)logits[best] - (double)second;
        if (info) *info = local;
        return (uint32_t)best;
    }
    float temperature =
        (std::isfinite(cfg->temperature) && cfg->temperature > 1e-4f) ? cfg->temperature : 1e-4f;
    for (uint64_t i = 0; i < vocab; ++i) logits[i] /= temperature;
    softmax_inplace(logits, vocab);
    uint64_t keep = (cfg->top_k == 0 || cfg->top_k > vocab) ? vocab : cfg->top_k;
    std::vector<uint32_t> idx(vocab);
    for (uint64_t i = 0; i < vocab; ++i) idx[i] = (uint32_t)i;
    auto before = [&](uint32_t l, uint32_t r) {
        int32_t kl = total_key(logits[l]), kr = total_key(logits[r]);
        if (kl != kr) return kl > kr;  // descending probability
        return l < r;                  // ascending index on ties
    };
    // select_nth + truncate + sort under a strict total order is the first
    // `keep` entries of the full sort.
    std::sort(idx.begin(), idx.end(), before);
    idx.resize(keep);
    float top_p = std::isfinite(cfg->top_p) ? std::min(std::max(cfg->top_p, 0.0f), 1.0f) : 1.0f;
    float cumulative = 0.0f, previous = 0.0f;
    uint64_t kept = 0;
    for (uint32_t i : idx) {
        previous = cumulative;
        cumulative += logits[i];
        ++kept;
        if (cumulative >= top_p) break;
    }
    // Distance of top_p to the cumulative sums on both sides of the cut: a
    // slightly different sum moves the cut one entry either way.
    local.cut_margin = std::fabs((double)cumulative - (double)top_p);
    if (kept >= 2) local.cut_margin = std::min(local.cut_margin, std::fabs((double)previous - (double)top_p));
    uint64_t n_cand = std::max<uint64_t>(kept, 1);
    local.kept = (uint32_t)n_cand;
    double total = 0.0;
    for (uint64_t c = 0; c < n_cand; ++c) total += (double)logits[idx[c]];
    local.total = total;
    if (!std::isfinite(total) || total <= 0.0) {
        uint32_t t = idx[below(rng, n_cand)];
        local.token = t;
        local.used_below = 1;
        local.cdf_margin = INFINITY;
        if (info) *info = local;
        return t;
    }
    double draw = (double)f32_unit(rng) * total;
    local.draw = draw;
    double margin = INFINITY;
    uint32_t chosen = idx[n_cand - 1];
    bool found = false;
    double walk = draw;
    for (uint64_t c = 0; c < n_cand; ++c) {
        double before_sub = walk;
        walk -= (double)logits[idx[c]];
        margin = std::min(margin, std::min(std::fabs(before_sub), std::fabs(walk)));
        if (walk <= 0.0) {
            chosen = idx[c];
            found = true;
            break;
        }
    }
    (void)found;
    local.cdf_margin = margin / total;
    local.token = chosen;
    {
        uint64_t c = 0;
        while (c + 1 < n_cand && idx[c] != chosen) ++c;
        const double pc = (double)logits[idx[c]];
        double om = INFINITY;
        if (pc > 0.0) {
            if (c > 0) om = std::min(om, ((double)logits[idx[c - 1]] - pc) / pc);
            if (c + 1 < n_cand) om = std::min(om, (pc - (double)logits[idx[c + 1]]) / pc);
        }
        local.order_margin = om;
    }
    if (info) *info = local;
    return chosen;
}

// Graph::softmax_ce forward (autograd.rs:579-624): per row the maximum, the
// sequential f32 sum of exp(v - max), probabilities scaled by 1/max(sum,
// 1e-30); the loss subtracts ln(max(p[target], 1e-20)) in f64 and is the mean
// over rows whose target is not u32::MAX (1 when there are none).
float softmax_ce(const float *logits, uint64_t rows, uint64_t vocab, const uint32_t *targets) {
    if (vocab == 0) throw std::invalid_argument("softmax_ce: vocabulary must be positive");
    std::vector<float> probs(vocab);
    double loss = 0.0;
    uint64_t cnt = 0;
    for (uint64_t i = 0; i < rows; ++i) {
        const float *row = logits + i * vocab;
        float mx = -INFINITY;
        for (uint64_t j = 0; j < vocab; ++j) {
            if (!std::isfinite(row[j])) throw std::invalid_argument("softmax_ce: logits must be finite");
            if (row[j] > mx) mx = row[j];
        }
        float s = 0.0f;
        for (uint64_t j = 0; j < vocab; ++j) {
            const float e = expf(row[j] - mx);
            probs[j] = e;
            s += e;
        }
        const float inv = 1.0f / std::max(s, 1e-30f);
        for (uint64_t j = 0; j < vocab; ++j) probs[j] *= inv;
        const uint32_t t = targets[i];
        if (t != 0xFFFFFFFFu) {
            if (t >= vocab) throw std::invalid_argument("softmax_ce: target out of range");
            const float p = std::max(probs[t], 1e-20f);
            loss -= std::log((double)p);
            ++cnt;
        }
    }
    const double denom = cnt == 0 ? 1.0 : (double)cnt;
    return (float)(loss / denom);
}

template <class F>
int guarded(F &&f) {
    try {
        f();
        return 0;
    } catch (const std::exception &ex) {
        set_error(ex.what());
        return -1;
    }
}

}  // namespace

// ================================================================ C API
extern "C" {

const char *orc_last_error(void) { return g_last_error.c_str(); }

uint64_t orc_splitmix64(uint64_t *state) { return splitmix(state); }
void orc_rng_new(orc_rng *r, uint64_t seed) { rng_new(r, seed); }
uint64_t orc_rng_next_u64(orc_rng *r) { return next_u64(r); }
float orc_rng_f32_unit(orc_rng *r) { return f32_unit(r); }
uint64_t orc_rng_below(orc_rng *r, uint64_t n) { return n == 0 ? 0 : below(r, n); }
float orc_rng_normal(orc_rng *r) { return normal(r); }

uint64_t orc_worker_count(uint64_t requested, uint64_t jobs, uint64_t total_work) {
    return worker_count(requested, jobs, total_work);
}
void orc_matvec_nt(const float *w, const float *bias, const float *x, float *out, uint64_t dout,
                   uint64_t din, uint64_t threads) {
    matvec_nt(w, bias, x, out, dout, din, threads);
}
void orc_gemm_nt(const float *a, const float *b, float *c, uint64_t m, uint64_t k, uint64_t n,
                 uint64_t threads) {
    gemm_nt(a, b, c, m, k, n, threads);
}
void orc_rms_norm_vec(const float *x, const float *w, float eps, float *out, uint64_t d) {
    rms_norm_vec(x, w, eps, out, d);
}
float orc_sigmoid(float x) { return sigmoid(x); }
float orc_silu(float x) { return silu(x); }
void orc_softmax_inplace(float *x, uint64_t n) {
    if (n) softmax_inplace(x, n);
}
uint64_t orc_argmax(const float *x, uint64_t n) { return n ? argmax(x, n) : 0; }

void orc_scan_sequential(const float *a, const float *b, float *h, uint64_t batch, uint64_t t,
                         uint64_t d, uint64_t threads) {
    scan_sequential(a, b, h, batch, t, d, threads);
}
void orc_scan_chunked(const float *a, const float *b, float *h, uint64_t batch, uint64_t t,
                      uint64_t d, uint64_t threads) {
    scan_chunked(a, b, h, batch, t, d, threads);
}

int orc_config_check(const orc_config *cfg) {
    std::string e = config_error(*cfg);
    if (!e.empty()) {
        set_error(e);
        return -1;
    }
    return 0;
}

orc_model *orc_model_new(const orc_config *cfg, orc_rng *rng) {
    std::string err = config_error(*cfg);
    if (!err.empty()) {
        set_error(err);
        return nullptr;
    }
    orc_model *m = new orc_model();
    m->cfg = *cfg;
    lm_init(m, rng);
    return m;
}
void orc_model_free(orc_model *m) { delete m; }
uint64_t orc_model_tensor_count(const orc_model *m) { return m->tensors.size(); }
const char *orc_model_tensor_name(const orc_model *m, uint64_t i) {
    return m->tensors[i].name.c_str();
}
uint64_t orc_model_tensor_rank(const orc_model *m, uint64_t i) { return m->tensors[i].shape.size(); }
uint64_t orc_model_tensor_dim(const orc_model *m, uint64_t i, uint64_t axis) {
    return m->tensors[i].shape[axis];
}
float *orc_model_tensor_data(orc_model *m, uint64_t i) { return m->tensors[i].val.data(); }
uint64_t orc_model_tensor_numel(const orc_model *m, uint64_t i) { return m->tensors[i].val.size(); }
void orc_model_set_threads(orc_model *m, uint64_t threads) { m->threads = std::max<uint64_t>(threads, 1); }

int orc_lm_logits(const orc_model *m, const uint32_t *ids, uint64_t batch, uint64_t t,
                  int scan_policy, float *logits_out) {
    return guarded([&] {
        lm_forward(m, ids, batch, t, scan_policy, logits_out, nullptr, nullptr, nullptr);
    });
}

// scan_adjoint (scan.rs:235-260): per batch row, walking time down from a
// zero carry: c = g + carry; carry = a * c.
void orc_scan_adjoint(const float *a, const float *g, float *c, uint64_t batch, uint64_t t, uint64_t d) {
    std::vector<float> carry(d);
    for (uint64_t bi = 0; bi < batch; ++bi) {
        const uint64_t base = bi * t * d;
        std::fill(carry.begin(), carry.end(), 0.0f);
        for (uint64_t ti = t; ti > 0;) {
            --ti;
            const uint64_t idx = base + ti * d;
            for (uint64_t j = 0; j < d; ++j) {
                const float cv = g[idx + j] + carry[j];
                c[idx + j] = cv;
                carry[j] = a[idx + j] * cv;
            }
        }
    }
}

// ---- training-side ops (the backward pass and the optimiser around the scan)

// kern_tn (tensor.rs:179-198): C[m,n] = sum_q A[q,m] * B[q,n], one row of C
// at a time, q ascending, a product then an add (no fused multiply-add), and
// a zero A element skips its row of B.
void orc_gemm_tn(const float *a, const float *b, float *c, uint64_t p, uint64_t m, uint64_t n) {
    for (uint64_t i = 0; i < m; ++i) {
        float *cr = c + i * n;
        for (uint64_t j = 0; j < n; ++j) cr[j] = 0.0f;
        for (uint64_t q = 0; q < p; ++q) {
            const float av = a[q * m + i];
            if (av == 0.0f) continue;
            const float *br = b + q * n;
            for (uint64_t j = 0; j < n; ++j) cr[j] += av * br[j];
        }
    }
}

// Op::DwConv backward (autograd.rs:1050-1097): the three gradients
// accumulate into gx / gw / gb (each nullable) in the reference's loop order.
void orc_dwconv_backward(const float *x, const float *w, const float *go, float *gx, float *gw, float *gb,
                         uint64_t batch, uint64_t t, uint64_t d, uint64_t k) {
    if (gx)
        for (uint64_t bi = 0; bi < batch; ++bi) {
            const uint64_t base = bi * t * d;
            for (uint64_t ti = 0; ti < t; ++ti) {
                const uint64_t o = base + ti * d, qmax = ti + 1 < k ? ti + 1 : k;
                for (uint64_t q = 0; q < qmax; ++q) {
                    const uint64_t src = base + (ti - q) * d;
                    for (uint64_t j = 0; j < d; ++j) gx[src + j] += go[o + j] * w[q * d + j];
                }
            }
        }
    if (gw)
        for (uint64_t bi = 0; bi < batch; ++bi) {
            const uint64_t base = bi * t * d;
            for (uint64_t ti = 0; ti < t; ++ti) {
                const uint64_t o = base + ti * d, qmax = ti + 1 < k ? ti + 1 : k;
                for (uint64_t q = 0; q < qmax; ++q) {
                    const uint64_t src = base + (ti - q) * d;
                    for (uint64_t j = 0; j < d; ++j) gw[q * d + j] += go[o + j] * x[src + j];
                }
            }
        }
    if (gb)
        for (uint64_t i = 0; i < batch * t; ++i)
            for (uint64_t j = 0; j < d; ++j) gb[j] += go[i * d + j];
}

// AdamW::step (optim.rs:33-72) for one parameter tensor.  t is the step
// counter after its increment; decay is the parameter's Param::decay.  The
// bias corrections use powf exactly as the reference; every update is a
// product or a sum in f32 (no fused multiply-add).  A non-finite gradient
// or parameter stops the pass with an error, as the reference's assertion.
int orc_adamw_step(float *val, const float *grad, float *m, float *v, uint64_t n, float lr, float b1, float b2,
                   float eps, float wd, uint64_t t, int decay) {
    return guarded([&] {
        if (!(std::isfinite(lr) && lr >= 0.0f)) throw std::runtime_error("AdamW learning rate must be finite and non-negative");
        if (!(std::isfinite(b1) && b1 >= 0.0f && b1 < 1.0f)) throw std::runtime_error("AdamW beta1 must be in [0, 1)");
        if (!(std::isfinite(b2) && b2 >= 0.0f && b2 < 1.0f)) throw std::runtime_error("AdamW beta2 must be in [0, 1)");
        if (!(std::isfinite(eps) && eps > 0.0f)) throw std::runtime_error("AdamW epsilon must be finite and positive");
        if (!(std::isfinite(wd) && wd >= 0.0f)) throw std::runtime_error("AdamW weight decay must be finite and non-negative");
        if (t == 0) throw std::runtime_error("AdamW step counter must be at least 1");
        const float tf = (float)t;
        const float bc1 = 1.0f - powf(b1, tf), bc2 = 1.0f - powf(b2, tf);
        const float inv_bc1 = 1.0f / bc1, inv_bc2 = 1.0f / bc2;
        for (uint64_t i = 0; i < n; ++i) {
            const float gr = grad[i];
            if (!std::isfinite(gr)) throw std::runtime_error("AdamW received a non-finite gradient");
            if (!std::isfinite(val[i])) throw std::runtime_error("AdamW received a non-finite parameter");
            const float mi = b1 * m[i] + (1.0f - b1) * gr;
            const float vi = b2 * v[i] + (1.0f - b2) * gr * gr;
            m[i] = mi;
            v[i] = vi;
            const float mh = mi * inv_bc1, vh = vi * inv_bc2;
            float upd = mh / (sqrtf(vh) + eps);
            if (decay && wd != 0.0f) upd += wd * val[i];
            val[i] -= lr * upd;
        }
    });
}

int orc_softmax_ce(const float *logits, uint64_t rows, uint64_t vocab, const uint32_t *targets, float *loss_out) {
    return guarded([&] { *loss_out = softmax_ce(logits, rows, vocab, targets); });
}

int orc_lm_loss(const orc_model *m, const uint32_t *ids, const uint32_t *targets, uint64_t batch, uint64_t t,
                int scan_policy, float *loss_out, float *logits_out) {
    return guarded([&] {
        const uint64_t rows = batch * t, V = m->cfg.vocab;
        std::vector<float> own;
        float *lg = logits_out;
        if (!lg) {
            own.resize(rows * V);
            lg = own.data();
        }
        lm_forward(m, ids, batch, t, scan_policy, lg, nullptr, nullptr, nullptr);
        *loss_out = softmax_ce(lg, rows, V, targets);
    });
}

int orc_lm_prefill_state(const orc_model *m, const uint32_t *ids, uint64_t batch, uint64_t t,
                         float *state_out, uint32_t *heads_out, float *last_logits_out) {
    return guarded([&] {
        lm_forward(m, ids, batch, t, 1, nullptr, state_out, heads_out, last_logits_out);
    });
}

orc_state *orc_state_new(const orc_model *m) {
    orc_state *s = new orc_state();
    s->n_layer = m->cfg.n_layer;
    s->k = m->k();
    s->e = m->e();
    s->conv.assign(s->n_layer, std::vector<float>(s->k * s->e, 0.0f));
    s->h.assign(s->n_layer, std::vector<float>(s->e, 0.0f));
    s->head = s->k - 1;  // infer.rs:32
    return s;
}
void orc_state_free(orc_state *s) { delete s; }
void orc_state_reset(orc_state *s) {  // infer.rs:37-44
    for (auto &c : s->conv) std::fill(c.begin(), c.end(), 0.0f);
    for (auto &h : s->h) std::fill(h.begin(), h.end(), 0.0f);
    s->head = s->k - 1;
}
uint64_t orc_state_numel(const orc_state *s) { return s->n_layer * (s->k + 1) * s->e; }
void orc_state_get(const orc_state *s, float *out, uint32_t *head) {
    for (uint64_t l = 0; l < s->n_layer; ++l) {
        float *dst = out + l * (s->k + 1) * s->e;
        std::memcpy(dst, s->conv[l].data(), s->k * s->e * sizeof(float));
        std::memcpy(dst + s->k * s->e, s->h[l].data(), s->e * sizeof(float));
    }
    if (head) *head = (uint32_t)s->head;
}
void orc_state_set(orc_state *s, const float *in, uint32_t head) {
    for (uint64_t l = 0; l < s->n_layer; ++l) {
        const float *src = in + l * (s->k + 1) * s->e;
        std::memcpy(s->conv[l].data(), src, s->k * s->e * sizeof(float));
        std::memcpy(s->h[l].data(), src + s->k * s->e, s->e * sizeof(float));
    }
    s->head = head % s->k;
}

int orc_step(const orc_model *m, orc_state *s, uint32_t token, float *logits_out) {
    return guarded([&] { step_impl(m, s, token, logits_out); });
}

uint32_t orc_sample_token(float *logits, uint64_t vocab, const orc_sample_cfg *cfg,
                          const uint32_t *history, uint64_t n_history, orc_rng *rng,
                          orc_sample_info *info) {
    uint32_t out = 0;
    guarded([&] { out = sample_impl(logits, vocab, cfg, history, n_history, rng, info); });
    return out;
}

int orc_generate(const orc_model *m, const uint32_t *prompt, uint64_t n_prompt, uint64_t n,
                 const orc_sample_cfg *cfg, orc_rng *rng, uint32_t *out_tokens) {
    return guarded([&] {  // cli.rs:470-518 on ids
        orc_state *st = orc_state_new(m);
        std::vector<float> logits(m->vocab());
        std::vector<uint32_t> ids(prompt, prompt + n_prompt);
        if (ids.empty()) ids.push_back(10);
        for (uint32_t id : ids) step_impl(m, st, id, logits.data());
        uint64_t limit = cfg->rep_window;
        uint64_t hstart = ids.size() > limit ? ids.size() - limit : 0;
        std::vector<uint32_t> history(ids.begin() + hstart, ids.end());
        for (uint64_t g = 0; g < n; ++g) {
            uint32_t tok = sample_impl(logits.data(), m->vocab(), cfg, history.data(),
                                       history.size(), rng, nullptr);
            out_tokens[g] = tok;
            if (limit > 0) {
                if (history.size() < limit)
                    history.push_back(tok);
                else {
                    std::rotate(history.begin(), history.begin() + 1, history.end());
                    history[limit - 1] = tok;
                }
            }
            if (g + 1 < n) step_impl(m, st, tok, logits.data());
        }
        orc_state_free(st);
    });
}

// ---------------------------------------------------------------- ckpt.rs
uint32_t orc_crc32(const uint8_t *data, uint64_t n) {  // ckpt.rs:35-54
    uint32_t table[256];
    for (uint32_t i = 0; i < 256; ++i) {
        uint32_t c = i;
        for (int b = 0; b < 8; ++b) c = (c & 1) ? (0xEDB88320u ^ (c >> 1)) : (c >> 1);
        table[i] = c;
    }
    uint32_t crc = 0xFFFFFFFFu;
    for (uint64_t i = 0; i < n; ++i) crc = table[(crc ^ data[i]) & 0xFF] ^ (crc >> 8);
    return crc ^ 0xFFFFFFFFu;
}

static void put_u32(std::vector<uint8_t> &b, uint32_t v) {
    for (int i = 0; i < 4; ++i) b.push_back((uint8_t)(v >> (8 * i)));
}
static void put_str(std::vector<uint8_t> &b, const std::string &s) {
    put_u32(b, (uint32_t)s.size());
    b.insert(b.end(), s.begin(), s.end());
}

int orc_ckpt_save(const orc_model *m, const char *path, const char *const *keys,
                  const char *const *values, uint64_t n_meta) {
    return guarded([&] {  // ckpt.rs:132-200 (no aux tensors)
        std::vector<uint8_t> buf;
        const char magic[8] = {'N', 'O', 'E', 'T', 'I', 'C', 0, 1};
        buf.insert(buf.end(), magic, magic + 8);
        put_u32(buf, 1);
        put_u32(buf, (uint32_t)n_meta);
        for (uint64_t i = 0; i < n_meta; ++i) {
            put_str(buf, keys[i]);
            put_str(buf, values[i]);
        }
        put_u32(buf, (uint32_t)m->tensors.size());
        for (const Tensor &t : m->tensors) {
            put_str(buf, t.name);
            put_u32(buf, (uint32_t)t.shape.size());
            for (uint64_t dim : t.shape) put_u32(buf, (uint32_t)dim);
            put_u32(buf, (uint32_t)t.val.size());
            for (float f : t.val) {
                if (!std::isfinite(f)) throw std::runtime_error("checkpoint tensors must contain only finite values");
                uint32_t bits;
                std::memcpy(&bits, &f, 4);
                put_u32(buf, bits);
            }
        }
        put_u32(buf, orc_crc32(buf.data(), buf.size()));
        std::string tmp = std::string(path) + ".tmp";
        {
            std::ofstream f(tmp, std::ios::binary);
            if (!f) throw std::runtime_error("cannot open checkpoint for writing");
            f.write((const char *)buf.data(), (std::streamsize)buf.size());
            if (!f) throw std::runtime_error("checkpoint write failed");
        }
        if (std::rename(tmp.c_str(), path) != 0) throw std::runtime_error("checkpoint rename failed");
    });
}

orc_model *orc_ckpt_load_model(const char *path, orc_rng *rng) {
    orc_model *result = nullptr;
    guarded([&] {  // ckpt.rs:299-383, cli.rs:909-956, ckpt.rs:410-436
        std::ifstream f(path, std::ios::binary);
        if (!f) throw std::runtime_error("cannot open checkpoint");
        std::vector<uint8_t> raw((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
        if (raw.size() < 24) throw std::runtime_error("checkpoint too small");
        uint64_t body = raw.size() - 4;
        uint32_t want = raw[body] | (raw[body + 1] << 8) | (raw[body + 2] << 16) | ((uint32_t)raw[body + 3] << 24);
        if (orc_crc32(raw.data(), body) != want) throw std::runtime_error("checkpoint CRC mismatch (corrupt file)");
        uint64_t off = 0;
        auto take = [&](uint64_t n) {
            if (off + n > body) throw std::runtime_error("checkpoint truncated");
            const uint8_t *p = raw.data() + off;
            off += n;
            return p;
        };
        auto u32 = [&] {
            const uint8_t *p = take(4);
            return (uint32_t)p[0] | (p[1] << 8) | (p[2] << 16) | ((uint32_t)p[3] << 24);
        };
        auto str = [&] {
            uint32_t n = u32();
            const uint8_t *p = take(n);
            return std::string((const char *)p, n);
        };
        const uint8_t *mg = take(8);
        const uint8_t magic[8] = {'N', 'O', 'E', 'T', 'I', 'C', 0, 1};
        if (std::memcmp(mg, magic, 8) != 0) throw std::runtime_error("not a noetic checkpoint");
        if (u32() != 1) throw std::runtime_error("unsupported checkpoint version");
        uint32_t n_meta = u32();
        std::map<std::string, std::string> meta;
        for (uint32_t i = 0; i < n_meta; ++i) {
            std::string k = str(), v = str();
            if (k.empty() || meta.count(k)) throw std::runtime_error("checkpoint metadata contains an empty or duplicate key");
            meta[k] = v;
        }
        uint32_t n_t = u32();
        std::map<std::string, std::pair<std::vector<uint64_t>, std::vector<float>>> ts;
        for (uint32_t i = 0; i < n_t; ++i) {
            std::string name = str();
            if (name.empty() || ts.count(name)) throw std::runtime_error("checkpoint contains an empty or duplicate tensor name");
            uint32_t rank = u32();
            if (rank > 32 || rank > (body - off) / 4) throw std::runtime_error("checkpoint tensor rank is invalid");
            std::vector<uint64_t> shape(rank);
            uint64_t numel_expect = 1;
            for (auto &dim : shape) {
                dim = u32();
                numel_expect *= dim;
            }
            uint32_t numel = u32();
            if (numel > (body - off) / 4) throw std::runtime_error("checkpoint tensor payload is truncated");
            if (numel_expect != numel) throw std::runtime_error("checkpoint tensor shape does not match its element count");
            std::vector<float> vals(numel);
            const uint8_t *p = take(4ull * numel);
            std::memcpy(vals.data(), p, 4ull * numel);
            for (float v : vals)
                if (!std::isfinite(v)) throw std::runtime_error("checkpoint tensor contains a non-finite value");
            ts[name] = {shape, vals};
        }
        if (off != body) throw std::runtime_error("checkpoint has trailing data");
        auto req = [&](const char *k) -> uint64_t {
            auto it = meta.find(k);
            if (it == meta.end()) throw std::runtime_error(std::string("checkpoint metadata is missing '") + k + "'");
            return std::stoull(it->second);
        };
        orc_config c{};
        c.vocab = req("vocab");
        c.d_model = req("d_model");
        c.n_layer = req("n_layer");
        c.expand = req("expand");
        c.conv_k = req("conv_k");
        c.mlp_mult = req("mlp_mult");
        c.eps = meta.count("eps") ? std::stof(meta["eps"]) : 1e-5f;
        if (!meta.count("tau_max")) throw std::runtime_error("checkpoint metadata is missing 'tau_max'");
        c.tau_max = std::stof(meta["tau_max"]);
        std::string err = config_error(c);
        if (!err.empty()) throw std::runtime_error(err);
        orc_model *m = new orc_model();
        m->cfg = c;
        lm_init(m, rng);
        uint64_t model_tensors = 0;
        for (auto &kv : ts)
            if (kv.first.rfind("aux.", 0) != 0) ++model_tensors;
        if (model_tensors != m->tensors.size()) {
            delete m;
            throw std::runtime_error("checkpoint tensor set does not exactly match the model");
        }
        for (auto &t : m->tensors) {
            auto it = ts.find(t.name);
            if (it == ts.end() || it->second.first != t.shape) {
                delete m;
                throw std::runtime_error("checkpoint tensor '" + t.name + "' is missing or has the wrong shape");
            }
        }
        for (auto &t : m->tensors) t.val = ts[t.name].second;
        result = m;
    });
    return result;
}

}  // extern "C"
