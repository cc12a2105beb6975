// runtime.cu -- host runtime and C ABI of the B200 token loop.
//
// Owns: model parameters (host copy + one device allocation), the seeded
// initialiser (rng.rs / nn.rs / model.rs), the checkpoint format (ckpt.rs),
// and the decoder (infer.rs Decoder over S streams, cli.rs generate loop).
// Every entry point returns nk_status and records a thread-local message.

#include <algorithm>
#include <functional>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <mutex>
#include <thread>
#include <atomic>
#include <string>
#include <vector>

#include <cuda_runtime.h>
#include <fcntl.h>
#include <unistd.h>

#include "../../include/noetic_gpu.h"
#include "nk_kernels.h"
#include "nk_tc.h"

namespace {

thread_local std::string g_err;

struct NkError {
    nk_status code;
    std::string msg;
};

[[noreturn]] void fail(nk_status code, const std::string &msg) { throw NkError{code, msg}; }

void cuda_check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail(e == cudaErrorMemoryAllocation ? NK_ERR_OOM : NK_ERR_CUDA,
             std::string(what) + ": " + cudaGetErrorString(e));
    }
}

template <class F>
nk_status guard(F &&f) {
    try {
        f();
        return NK_OK;
    } catch (const NkError &e) {
        g_err = e.msg;
        return e.code;
    } catch (const std::bad_alloc &) {
        g_err = "host allocation failed";
        return NK_ERR_OOM;
    } catch (const std::exception &e) {
        g_err = e.what();
        return NK_ERR_INVALID;
    }
}

// ---------------------------------------------------------------- rng.rs
// splitmix64 (rng.rs:9-15), Rng::new (rng.rs:25-38), xoshiro256++
// (rng.rs:46-56), f32_unit (rng.rs:65-67), uniform (rng.rs:70-72) and the
// Marsaglia polar normal with its cached spare (rng.rs:93-109).
struct HostRng {
    uint64_t s[4];
    float spare = 0.0f;
    bool has_spare = false;

    static uint64_t splitmix(uint64_t &z) {
        z += 0x9E3779B97F4A7C15ull;
        uint64_t r = z;
        r = (r ^ (r >> 30)) * 0xBF58476D1CE4E5B9ull;
        r = (r ^ (r >> 27)) * 0x94D049BB133111EBull;
        return r ^ (r >> 31);
    }
    explicit HostRng(uint64_t seed) {
        uint64_t z = seed ^ 0xA0761D6478BD642Full;
        for (auto &w : s) w = splitmix(z);
        if (!s[0] && !s[1] && !s[2] && !s[3]) s[0] = 0x9E3779B97F4A7C15ull;
    }
    static uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }
    uint64_t next() {
        const uint64_t r = rotl(s[0] + s[3], 23) + s[0];
        const uint64_t t = s[1] << 17;
        s[2] ^= s[0];
        s[3] ^= s[1];
        s[1] ^= s[2];
        s[0] ^= s[3];
        s[2] ^= t;
        s[3] = rotl(s[3], 45);
        return r;
    }
    float unit() { return (float)(next() >> 40) * (1.0f / 16777216.0f); }
    float uniform(float lo, float hi) { return lo + (hi - lo) * unit(); }
    float normal() {
        if (has_spare) {
            has_spare = false;
            return spare;
        }
        for (;;) {
            const float u = uniform(-1.0f, 1.0f);
            const float v = uniform(-1.0f, 1.0f);
            const float q = u * u + v * v;
            if (q > 0.0f && q < 1.0f) {
                const float f = std::sqrt(-2.0f * std::log(q) / q);
                spare = v * f;
                has_spare = true;
                return u * f;
            }
        }
    }
};

// ---------------------------------------------------------------- config
std::string config_error(const nk_config &c) {  // model.rs:37-76
    if (c.vocab == 0) return "vocabulary size must be positive";
    if (c.vocab > 0xFFFFFFFFull) return "vocabulary exceeds the u32 token-id space";
    if (c.d_model == 0) return "d_model must be positive";
    if (c.n_layer == 0) return "n_layer must be positive";
    if (c.expand == 0) return "expand must be positive";
    if (c.conv_k == 0) return "conv_k must be positive";
    if (c.mlp_mult == 0) return "mlp_mult must be positive";
    if (!std::isfinite(c.eps) || c.eps <= 0.0f) return "RMSNorm epsilon must be finite and positive";
    if (!std::isfinite(c.tau_max) || c.tau_max < 1.0f) return "tau_max must be finite and at least one";
    const uint64_t lim = 1ull << 40;
    if (c.d_model > lim / c.expand || c.d_model > lim / c.mlp_mult || c.vocab > lim / c.d_model)
        return "model width overflow";
    return "";
}

// Sizes this build supports on the device (int indexing inside kernels).
std::string device_limits_error(const nk_config &c) {
    const uint64_t d = c.d_model, e = d * c.expand, h = d * c.mlp_mult;
    if (d > (1u << 16) || e > (1u << 16) || h > (1u << 17)) return "model width exceeds the device kernels' limit";
    if (c.conv_k > 64) return "conv_k above 64 is not supported by the device kernels";
    if (c.vocab * d > (1ull << 34)) return "embedding table exceeds the device kernels' limit";
    return "";
}

struct Tensor {
    std::string name;
    std::vector<uint64_t> shape;
    std::vector<float> host;
    size_t dev_off = 0;  // float offset into the device arena
    uint64_t numel() const {
        uint64_t n = 1;
        for (auto d : shape) n *= d;
        return n;
    }
};

struct LayerIx {
    int n1, in_w, in_b, conv_w, conv_b, out_w, out_b, n2, up_w, up_b, down_w, down_b;
};

}  // namespace

struct nk_model {
    nk_config cfg{};
    int device = 0;
    std::vector<Tensor> tensors;
    std::map<std::string, int> by_name;
    int emb = -1, norm_f = -1;
    std::vector<LayerIx> layers;
    float *arena = nullptr;
    size_t arena_floats = 0;
    bool dirty = true;
    // false after a direct checkpoint load: the device arena holds the
    // weights and the host copies are filled on demand (ensure_host)
    bool host_valid = true;
    nk::TcWeights tc;  // tensor-core operand forms (built with the arena)
    // out_w and down_w of every layer stored transposed ([E][d], [H][d] per
    // layer) for the persistent step kernel, built on first use
    float *wT = nullptr;

    uint64_t d() const { return cfg.d_model; }
    uint64_t e() const { return cfg.d_model * cfg.expand; }
    uint64_t hidden() const { return cfg.d_model * cfg.mlp_mult; }
    uint64_t k() const { return cfg.conv_k; }
    const float *dp(int id) const { return arena + tensors[id].dev_off; }

    int add(const std::string &name, std::vector<uint64_t> shape) {
        Tensor t;
        t.name = name;
        t.shape = std::move(shape);
        if (host_valid) t.host.assign(t.numel(), 0.0f);
        tensors.push_back(std::move(t));
        by_name[name] = (int)tensors.size() - 1;
        return (int)tensors.size() - 1;
    }

    // Parameter set in Lm::new creation order (model.rs:183-206,
    // model.rs:111-146, nn.rs:23-99) -- also the checkpoint order.
    void build_layout() {
        const uint64_t d = this->d(), e = this->e(), hd = hidden(), k = this->k();
        emb = add("emb", {cfg.vocab, d});
        for (uint64_t l = 0; l < cfg.n_layer; ++l) {
            const std::string b = "blk" + std::to_string(l);
            LayerIx L{};
            L.n1 = add(b + ".n1.gain", {d});
            L.in_w = add(b + ".ssm.in_proj.w", {3 * e, d});
            L.in_b = add(b + ".ssm.in_proj.b", {3 * e});
            L.conv_w = add(b + ".ssm.conv_w", {k, e});
            L.conv_b = add(b + ".ssm.conv_b", {e});
            L.out_w = add(b + ".ssm.out_proj.w", {d, e});
            L.out_b = add(b + ".ssm.out_proj.b", {d});
            L.n2 = add(b + ".n2.gain", {d});
            L.up_w = add(b + ".mlp.up.w", {2 * hd, d});
            L.up_b = add(b + ".mlp.up.b", {2 * hd});
            L.down_w = add(b + ".mlp.down.w", {d, hd});
            L.down_b = add(b + ".mlp.down.b", {d});
            layers.push_back(L);
        }
        norm_f = add("norm_f.gain", {d});
    }

    // Lm::new's draws, in order, from one generator (Appendix of the
    // reference's model: emb N(0,1)*0.02; per layer in_proj.w, conv taps
    // q>=1, out_proj.w, up.w, down.w; deterministic gains/biases).
    void init_random(HostRng &rng) {
        if (!host_valid) {  // every tensor is rewritten below
            for (auto &t : tensors) t.host.assign(t.numel(), 0.0f);
            host_valid = true;
        }
        const uint64_t d = this->d(), e = this->e(), hd = hidden(), k = this->k();
        for (auto &t : tensors) std::fill(t.host.begin(), t.host.end(), 0.0f);
        for (auto &x : tensors[emb].host) x = rng.normal() * 0.02f;
        const float depth_scale = 1.0f / std::sqrt(2.0f * (float)cfg.n_layer);
        auto init_std = [](uint64_t fan_in) { return std::sqrt(2.0f / (float)std::max<uint64_t>(fan_in, 1)); };
        auto fill = [&](int id, float sd) {
            for (auto &x : tensors[id].host) x = rng.normal() * sd;
        };
        for (uint64_t l = 0; l < cfg.n_layer; ++l) {
            const LayerIx &L = layers[l];
            std::fill(tensors[L.n1].host.begin(), tensors[L.n1].host.end(), 1.0f);
            fill(L.in_w, init_std(d));
            float *bias = tensors[L.in_b].host.data();
            for (uint64_t j = 0; j < e; ++j) {  // model.rs:116-128
                const float fraction = e > 1 ? (float)j / (float)(e - 1) : 0.0f;
                const float tau = std::pow(cfg.tau_max, fraction);
                float decay = std::exp(-1.0f / tau);
                decay = std::min(std::max(decay, 0.001f), 0.9999f);
                bias[e + j] = std::log(decay / (1.0f - decay));
            }
            float *cw = tensors[L.conv_w].host.data();  // model.rs:130-142
            for (uint64_t j = 0; j < e; ++j) cw[j] = 1.0f;
            for (uint64_t q = 1; q < k; ++q)
                for (uint64_t j = 0; j < e; ++j) cw[q * e + j] = rng.normal() * 0.1f;
            fill(L.out_w, init_std(e) * depth_scale);
            std::fill(tensors[L.n2].host.begin(), tensors[L.n2].host.end(), 1.0f);
            fill(L.up_w, init_std(d));
            fill(L.down_w, init_std(hd) * depth_scale);
        }
        std::fill(tensors[norm_f].host.begin(), tensors[norm_f].host.end(), 1.0f);
        dirty = true;
    }

    void ensure_arena() {
        if (arena) return;
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        size_t off = 0;
        for (auto &t : tensors) {
            t.dev_off = off;
            off += (t.numel() + 63) & ~size_t(63);  // 256-byte aligned tensors
        }
        arena_floats = off;
        cuda_check(cudaMalloc(&arena, arena_floats * sizeof(float)), "cudaMalloc(weights)");
    }

    // Host copies of every tensor from the device arena (after a direct load).
    void ensure_host() {
        if (host_valid) return;
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        for (auto &t : tensors) {
            t.host.resize(t.numel());
            cuda_check(cudaMemcpy(t.host.data(), arena + t.dev_off, t.numel() * sizeof(float), cudaMemcpyDeviceToHost),
                       "download weights");
        }
        host_valid = true;
    }

    void upload() {
        if (!dirty) return;
        if (!host_valid) fail(NK_ERR_INVALID, "model host copies are stale");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        ensure_arena();
        for (auto &t : tensors)
            cuda_check(cudaMemcpy(arena + t.dev_off, t.host.data(), t.numel() * sizeof(float),
                                  cudaMemcpyHostToDevice),
                       "cudaMemcpy(weights)");
        nk::tc_weights_free(tc);
        free_transposed();
        dirty = false;
    }

    void free_transposed() {
        if (wT) cudaFree(wT);
        wT = nullptr;
    }
    size_t wT_layer_floats() const { return (size_t)(e() + hidden()) * d(); }

    ~nk_model() {
        if (arena) {
            cudaSetDevice(device);
            cudaFree(arena);
        }
        free_transposed();
        if (device < 0) return;
        nk::tc_weights_free(tc);
    }
};

// ---------------------------------------------------------------- ckpt.rs
namespace {

const uint8_t MAGIC[8] = {'N', 'O', 'E', 'T', 'I', 'C', 0, 1};
const uint64_t MAX_CKPT_BYTES = 8ull << 30;

uint32_t crc32(const uint8_t *p, size_t n) {  // ckpt.rs:35-54
    static uint32_t table[256];
    static bool ready = false;
    if (!ready) {
        for (uint32_t i = 0; i < 256; ++i) {
            uint32_t c = i;
            for (int b = 0; b < 8; ++b) c = (c & 1) ? (0xEDB88320u ^ (c >> 1)) : (c >> 1);
            table[i] = c;
        }
        ready = true;
    }
    uint32_t crc = 0xFFFFFFFFu;
    for (size_t i = 0; i < n; ++i) crc = table[(crc ^ p[i]) & 0xFF] ^ (crc >> 8);
    return crc ^ 0xFFFFFFFFu;
}

// ---- the same CRC-32, fast: slicing by 8 (eight table lookups per 8
// bytes), and the CRC of a concatenation from the CRCs of its parts.
struct Crc8Tables {
    uint32_t t[8][256];
    Crc8Tables() {
        for (uint32_t i = 0; i < 256; ++i) {
            uint32_t c = i;
            for (int b = 0; b < 8; ++b) c = (c & 1) ? (0xEDB88320u ^ (c >> 1)) : (c >> 1);
            t[0][i] = c;
        }
        for (int k = 1; k < 8; ++k)
            for (uint32_t i = 0; i < 256; ++i) t[k][i] = (t[k - 1][i] >> 8) ^ t[0][t[k - 1][i] & 0xFF];
    }
};

uint32_t crc32_fast(const uint8_t *p, size_t n) {
    static const Crc8Tables T;
    uint32_t crc = 0xFFFFFFFFu;
    while (n >= 8) {
        uint32_t lo, hi;
        std::memcpy(&lo, p, 4);
        std::memcpy(&hi, p + 4, 4);
        lo ^= crc;
        crc = T.t[7][lo & 0xFF] ^ T.t[6][(lo >> 8) & 0xFF] ^ T.t[5][(lo >> 16) & 0xFF] ^ T.t[4][lo >> 24] ^
              T.t[3][hi & 0xFF] ^ T.t[2][(hi >> 8) & 0xFF] ^ T.t[1][(hi >> 16) & 0xFF] ^ T.t[0][hi >> 24];
        p += 8;
        n -= 8;
    }
    while (n--) crc = T.t[0][(crc ^ *p++) & 0xFF] ^ (crc >> 8);
    return crc ^ 0xFFFFFFFFu;
}

// Product of two polynomials modulo the CRC polynomial, in the reflected
// representation the CRC uses (bit 31 is x^0).
uint32_t crc_mulmod(uint32_t a, uint32_t b) {
    uint32_t prod = 0;
    for (uint32_t m = 1u << 31; m; m >>= 1) {
        if (a & m) prod ^= b;
        b = (b & 1) ? (b >> 1) ^ 0xEDB88320u : b >> 1;  // b * x
    }
    return prod;
}

// CRC(A || B) from CRC(A), CRC(B) and |B| bytes: CRC(A) times x^(8 |B|), plus
// CRC(B) (the initial and final inversions cancel in this form).
uint32_t crc32_combine(uint32_t crc_a, uint32_t crc_b, uint64_t len_b) {
    uint32_t xp = 1u << 31, base = 1u << 23;  // x^0 and x^8
    for (; len_b; len_b >>= 1) {
        if (len_b & 1) xp = crc_mulmod(xp, base);
        base = crc_mulmod(base, base);
    }
    return crc_mulmod(xp, crc_a) ^ crc_b;
}

struct CkptData {
    std::map<std::string, std::string> meta;
    std::map<std::string, std::pair<std::vector<uint64_t>, std::vector<float>>> tensors;
};

// ckpt.rs:299-383: every malformed / truncated / duplicate / trailing /
// inconsistent / non-finite case is rejected before anything is applied.
CkptData read_ckpt(const char *path) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) fail(NK_ERR_IO, std::string("cannot open checkpoint ") + path);
    const std::streamoff size = f.tellg();
    if (size < 0 || (uint64_t)size > MAX_CKPT_BYTES) fail(NK_ERR_IO, "checkpoint file exceeds the supported size limit");
    if (size < 24) fail(NK_ERR_IO, "checkpoint too small");
    std::vector<uint8_t> raw((size_t)size);
    f.seekg(0);
    f.read((char *)raw.data(), size);
    if (!f) fail(NK_ERR_IO, "checkpoint read failed");
    const size_t body = raw.size() - 4;
    const uint32_t want = raw[body] | (raw[body + 1] << 8) | (raw[body + 2] << 16) | ((uint32_t)raw[body + 3] << 24);
    if (crc32(raw.data(), body) != want) fail(NK_ERR_IO, "checkpoint CRC mismatch (corrupt file)");
    size_t off = 0;
    auto take = [&](size_t n) -> const uint8_t * {
        if (n > body - off) fail(NK_ERR_IO, "checkpoint truncated");
        const uint8_t *p = raw.data() + off;
        off += n;
        return p;
    };
    auto u32 = [&]() -> uint32_t {
        const uint8_t *p = take(4);
        return p[0] | (p[1] << 8) | (p[2] << 16) | ((uint32_t)p[3] << 24);
    };
    auto str = [&]() {
        const uint32_t n = u32();
        const uint8_t *p = take(n);
        return std::string((const char *)p, n);
    };
    if (std::memcmp(take(8), MAGIC, 8) != 0) fail(NK_ERR_IO, "not a noetic checkpoint");
    if (u32() != 1) fail(NK_ERR_IO, "unsupported checkpoint version");
    CkptData c;
    const uint32_t n_meta = u32();
    if (n_meta > 1000000) fail(NK_ERR_IO, "checkpoint contains too many metadata entries");
    for (uint32_t i = 0; i < n_meta; ++i) {
        std::string k = str(), v = str();
        if (k.empty() || c.meta.count(k)) fail(NK_ERR_IO, "checkpoint metadata contains an empty or duplicate key");
        c.meta[k] = v;
    }
    const uint32_t n_t = u32();
    if (n_t > 1000000) fail(NK_ERR_IO, "checkpoint contains too many tensors");
    for (uint32_t i = 0; i < n_t; ++i) {
        std::string name = str();
        if (name.empty() || c.tensors.count(name)) fail(NK_ERR_IO, "checkpoint contains an empty or duplicate tensor name");
        const uint32_t rank = u32();
        if (rank > 32 || rank > (body - off) / 4) fail(NK_ERR_IO, "checkpoint tensor rank is invalid");
        std::vector<uint64_t> shape(rank);
        uint64_t expect = 1;
        bool overflow = false;
        for (auto &d : shape) {
            d = u32();
            if (d != 0 && expect > UINT64_MAX / d) overflow = true;
            expect *= d;
        }
        const uint32_t numel = u32();
        if (numel > (body - off) / 4) fail(NK_ERR_IO, "checkpoint tensor payload is truncated");
        if (overflow || expect != numel) fail(NK_ERR_IO, "checkpoint tensor shape does not match its element count");
        std::vector<float> v(numel);
        std::memcpy(v.data(), take(4ull * numel), 4ull * numel);
        for (float x : v)
            if (!std::isfinite(x)) fail(NK_ERR_IO, "checkpoint tensor contains a non-finite value");
        c.tensors[name] = {std::move(shape), std::move(v)};
    }
    if (off != body) fail(NK_ERR_IO, "checkpoint has trailing data");
    return c;
}

uint64_t meta_usize(const CkptData &c, const char *key) {  // Ckpt::require_usize
    auto it = c.meta.find(key);
    if (it == c.meta.end()) fail(NK_ERR_IO, std::string("checkpoint metadata is missing '") + key + "'");
    const std::string &s = it->second;
    if (s.empty() || s.find_first_not_of("0123456789") != std::string::npos)
        fail(NK_ERR_IO, std::string("checkpoint metadata '") + key + "' is not a valid integer");
    try {
        return std::stoull(s);
    } catch (...) {
        fail(NK_ERR_IO, std::string("checkpoint metadata '") + key + "' is not a valid integer");
    }
}

float meta_f32(const CkptData &c, const char *key, bool required, float dflt) {
    auto it = c.meta.find(key);
    if (it == c.meta.end()) {
        if (required) fail(NK_ERR_IO, std::string("checkpoint metadata is missing '") + key + "'");
        return dflt;
    }
    char *end = nullptr;
    const float v = std::strtof(it->second.c_str(), &end);
    if (it->second.empty() || *end != 0) fail(NK_ERR_IO, std::string("checkpoint metadata '") + key + "' is not a valid number");
    if (!std::isfinite(v)) fail(NK_ERR_IO, std::string("checkpoint metadata '") + key + "' must be finite");
    return v;
}

void put_u32(std::vector<uint8_t> &b, uint32_t v) {
    for (int i = 0; i < 4; ++i) b.push_back((uint8_t)(v >> (8 * i)));
}
void put_str(std::vector<uint8_t> &b, const std::string &s) {
    put_u32(b, (uint32_t)s.size());
    b.insert(b.end(), s.begin(), s.end());
}

std::string fmt_f32(float v) {
    char buf[64];
    std::snprintf(buf, sizeof buf, "%.9g", (double)v);
    return buf;
}

}  // namespace

// ---------------------------------------------------------------- decoder
struct nk_decoder {
    nk_model *model = nullptr;
    uint32_t S = 0;
    cudaStream_t stream = nullptr;
    int engine = 0;
    uint64_t launches = 0;

    float *state = nullptr;  // [L][S][k+1][E]
    uint32_t *heads = nullptr;
    float *x = nullptr, *nrm = nullptr, *u = nullptr, *g = nullptr, *logits = nullptr;
    uint32_t *tok_a = nullptr, *tok_b = nullptr;
    int *err = nullptr;
    uint64_t *rng = nullptr;
    uint32_t *hist = nullptr, *hist_len = nullptr;
    uint32_t hist_cap = 0;
    // sampler scratch (lazy sort of large candidate sets), grown on demand
    void *samp_ws = nullptr;
    size_t samp_ws_bytes = 0;
    // Sampling epilogue of the logits projection (generate): when
    // fuse_sample is set, an eager step's tensor-core logits projection
    // writes pen(logit) / temperature with per-part maxima and +inf counts,
    // and records the part count in fused_parts (0: not fused).
    const nk::SampleParams *fuse_sample = nullptr;
    bool fuse_penalty = false;
    int fused_parts = 0;
    uint32_t *pen_bits = nullptr;
    float *prep_max = nullptr;
    uint32_t *prep_pinf = nullptr;
    size_t prep_cap = 0;
    // prefill scratch (grown on demand)
    float *p_x = nullptr, *p_n = nullptr, *p_u = nullptr, *p_y = nullptr, *p_last = nullptr,
          *p_scan = nullptr, *p_logits = nullptr;
    size_t p_rows = 0, p_scan_floats = 0;
    uint32_t *p_ids = nullptr, *p_lens = nullptr;
    size_t p_ids_cap = 0;
    // 3xTF32 activation operand pair (decode) and the fused argmax partials
    float *ahi = nullptr, *alo = nullptr;
    // RMSNorm folded into the projections: the normalised operand's pair
    // (split of x * gain, [S, d]) and the rows' partial sums of squares
    // ([S, ceil(d / 32)]) the producing epilogue writes
    float *nhi = nullptr, *nlo = nullptr, *nss = nullptr;
    float *best_val = nullptr;
    uint32_t *best_idx = nullptr;
    // prefill operand pair
    float *p_ahi = nullptr, *p_alo = nullptr;
    // small-batch engine: layer pointers and CUDA graphs of the greedy step,
    // one per (tokens in, tokens out) device buffer pair
    std::vector<nk::SmallLayer> small_layers;
    // stream-K workspace of the tensor-core projections (counters zeroed)
    float *ksplit_ws = nullptr;
    int *ksplit_flags = nullptr;
    static constexpr int KSPLIT_FLAGS = 4096;
    const float *layers_arena = nullptr;  // model arena the small-batch layer table points into
    // persistent step kernel: device layer table (keyed on the model's
    // transposed weights), accumulators and barrier words
    nk::PersistLayer *players_dev = nullptr;
    const float *players_key = nullptr;
    uint8_t *pws = nullptr;
    struct StepGraph {
        const uint32_t *in;
        uint32_t *out;
        cudaGraphExec_t exec;
        uint64_t launches;
    };
    std::vector<StepGraph> graphs;
    bool warm = false;  // an eager greedy step has run (buffers sized, attributes set)
    // projection profiling (CUDA events around each projection launch)
    bool profiling = false;
    std::vector<cudaEvent_t> ev_pool;
    size_t ev_used = 0;
    double prof_flops = 0, prof_bytes = 0;
    uint64_t prof_launch0 = 0, prof_proj = 0;
    bool prof_tc = false;
    // sampler launches while profiling (event pairs), reported beside the projections
    std::vector<cudaEvent_t> samp_ev;
    size_t samp_used = 0;
    uint64_t prof_samp = 0;

    uint64_t L() const { return model->cfg.n_layer; }
    size_t layer_state_floats() const { return (size_t)S * (model->k() + 1) * model->e(); }
    float *layer_state(uint64_t l) { return state + l * layer_state_floats(); }

    ~nk_decoder() {
        cudaSetDevice(model->device);
        if (stream) cudaStreamSynchronize(stream);
        for (void *p : {(void *)state, (void *)heads, (void *)x, (void *)nrm, (void *)u, (void *)g,
                        (void *)logits, (void *)tok_a, (void *)tok_b, (void *)err, (void *)rng,
                        (void *)hist, (void *)hist_len, (void *)p_x, (void *)p_n, (void *)p_u,
                        (void *)p_y, (void *)p_last, (void *)p_scan, (void *)p_logits, (void *)p_ids,
                        (void *)p_lens})
            if (p) cudaFree(p);
        for (void *p : {(void *)ahi, (void *)alo, (void *)best_val, (void *)best_idx, (void *)p_ahi, (void *)p_alo,
                        (void *)players_dev, (void *)pws, (void *)ksplit_ws, (void *)ksplit_flags, samp_ws,
                        (void *)pen_bits, (void *)prep_max, (void *)prep_pinf, (void *)nhi, (void *)nlo,
                        (void *)nss})
            if (p) cudaFree(p);
        for (cudaEvent_t e : ev_pool) cudaEventDestroy(e);
        for (cudaEvent_t e : samp_ev) cudaEventDestroy(e);
        for (auto &gph : graphs) cudaGraphExecDestroy(gph.exec);
        if (stream) cudaStreamDestroy(stream);
    }
};

namespace {

template <class T>
void dalloc(T **p, size_t n, const char *what) {
    cuda_check(cudaMalloc((void **)p, std::max<size_t>(n, 1) * sizeof(T)), what);
}

void launch_ok(nk_decoder *dec, cudaError_t e, const char *what, int count = 1) {
    cuda_check(e, what);
    dec->launches += (uint64_t)count;
}

// One projection: tensor-core 3xTF32 GEMM when eligible, else the f32
// CUDA-core kernels.
cudaEvent_t prof_event(nk_decoder *dec) {
    if (dec->ev_used == dec->ev_pool.size()) {
        cudaEvent_t e;
        cuda_check(cudaEventCreate(&e), "cudaEventCreate");
        dec->ev_pool.push_back(e);
    }
    return dec->ev_pool[dec->ev_used++];
}

// Which engine runs a projection of this shape: the tcgen05 3xTF32 kernel
// when eligible, else the f32 CUDA-core kernels.  The producer of the
// projection's input writes the operand form the chosen engine reads.
bool use_tc(const nk_decoder *dec, int M, int N, int K, const nk::TcOperand *Wtc) {
    return !(dec->engine & 1) && Wtc && nk::tc_eligible(M, N, K);
}

// An activation buffer in both forms: f32 for the CUDA-core engine, the hi/lo
// pair for the tensor-core engine.
struct Act {
    float *f32, *hi, *lo;
    nk::RowOut out(bool tc) const { return tc ? nk::RowOut{nullptr, hi, lo} : nk::RowOut{f32, nullptr, nullptr}; }
};

struct ProfScope {
    nk_decoder *dec;
    cudaEvent_t e1 = nullptr;
    ProfScope(nk_decoder *d, int M, int N, int K, bool residual, bool bias) : dec(d) {
        if (!dec->profiling) return;
        cudaEvent_t e0 = prof_event(dec);
        e1 = prof_event(dec);
        cuda_check(cudaEventRecord(e0, dec->stream), "cudaEventRecord");
        dec->prof_flops += 2.0 * M * (double)N * K;
        dec->prof_bytes += 4.0 * ((double)M * K + (double)N * K + (double)M * N * (residual ? 2 : 1) + (bias ? N : 0));
        dec->prof_proj += 1;
    }
    ~ProfScope() {
        if (e1) cudaEventRecord(e1, dec->stream);
    }
};

// CUDA events around a sampler launch while profiling.
struct SampScope {
    nk_decoder *dec;
    cudaEvent_t e1 = nullptr;
    explicit SampScope(nk_decoder *d) : dec(d) {
        if (!dec->profiling) return;
        auto next = [&]() {
            if (dec->samp_used == dec->samp_ev.size()) {
                cudaEvent_t e;
                cuda_check(cudaEventCreate(&e), "cudaEventCreate");
                dec->samp_ev.push_back(e);
            }
            return dec->samp_ev[dec->samp_used++];
        };
        cudaEvent_t e0 = next();
        e1 = next();
        cuda_check(cudaEventRecord(e0, dec->stream), "cudaEventRecord");
        dec->prof_samp += 1;
    }
    ~SampScope() {
        if (e1) cudaEventRecord(e1, dec->stream);
    }
};

// Test controls of the bounded waits (engine bits 12 / 13): the projections'
// stream-K partial tiles are not published, or the persistent step's CTA 0
// skips its first grid-barrier arrival, and the waits are bounded at 2 ms,
// so the failure path (an expired wait reported as an error code, then
// recovery) runs without a fault and without a hang.
constexpr int ENGINE_NO_TMA_STORE = 32768;  // epilogue stores from the threads instead of bulk stores
constexpr int ENGINE_WITHHOLD_PUBLISH = 4096;
constexpr int ENGINE_WITHHOLD_ARRIVAL = 8192;
// RMSNorm folded into the projection epilogues (forced at every batch; the
// default only below POST_NORM_MIN_ROWS streams): measured slower on B200 at
// large batches (77 vs 70 ms per step at 16384 streams, 12.7 vs 10.9 at
// 2048), since the 256-wide tile's epilogue is not overlapped with the next
// tile's main loop and the extra stores lengthen it by more than the norm
// kernels cost.
constexpr int ENGINE_FOLD = 16384;
// Engine bits 16 / 17: the split-K reductions of small projections do not
// take over the next RMSNorm / the recurrent branch (separate kernels, as
// above 512 streams).
constexpr int ENGINE_NO_POST_NORM = 65536;
constexpr int ENGINE_NO_POST_SSM = 131072;
constexpr int POST_NORM_MIN_ROWS = 384;  // streams from which the reductions take over RMSNorm
// Engine bit 18: no RMSNorm folding below POST_NORM_MIN_ROWS streams (the
// stand-alone norm kernels instead).
constexpr int ENGINE_NO_AUTO_FOLD = 262144;
// Engine bit 19: projection tiles in plain row-major order (no column groups).
constexpr int ENGINE_NO_TILE_GROUP = 524288;
constexpr uint64_t TEST_WAIT_NS = 2000000ull;
void test_controls(const nk_decoder *dec, nk::TcEpilogue &ep) {
    if (dec->engine & ENGINE_NO_TMA_STORE) ep.no_tma_store = true;
    if (dec->engine & ENGINE_NO_TILE_GROUP) ep.no_tile_group = true;
    if (dec->engine & ENGINE_WITHHOLD_PUBLISH) {
        ep.withhold_publish = true;
        ep.handoff_wait_ns = TEST_WAIT_NS;
    }
}

// Tile shape of a tensor-core projection; engine bits 4 / 5 / 7 force
// 128 / 256-wide single-SM tiles / the CTA-pair kernel; bit 8 keeps whole
// tiles (no stream-K).
int pick_bn(const nk_decoder *dec, int M, int N, bool argmax = false) {
    if (dec->engine & 16) return 128;
    if ((dec->engine & 32) && N >= 256) return 256;
    if ((dec->engine & 128) && N >= 256) return nk::TC_PAIR;
    return nk::tc_pick_bn(M, N, false, !argmax && !(dec->engine & 256));
}

// RMSNorm folded into a tensor-core projection: `rs` (the partial sums of
// squares of the rows whose gain-scaled split is the A operand) makes it a
// consumer; `nx_gain` makes a store-mode projection the producer of the
// next one's operand and sums.
struct Fold {
    const float *rs = nullptr;
    const float *nx_gain = nullptr;
};
void apply_fold(nk_decoder *dec, const Fold *f, nk::TcEpilogue &ep) {
    if (!f) return;
    const int d = (int)dec->model->d();
    if (f->rs) {
        ep.rs_parts = f->rs;
        ep.rs_nparts = (d + 31) / 32;
        ep.rs_d = d;
        ep.rs_eps = dec->model->cfg.eps;
    }
    if (f->nx_gain) {
        ep.nx_hi = dec->nhi;
        ep.nx_lo = dec->nlo;
        ep.nx_gain = f->nx_gain;
        ep.nx_ss = dec->nss;
    }
}

// Work that the split-K reduction of a small projection may take over (see
// TcEpilogue::post_*): the next RMSNorm after a residual projection, or the
// recurrent branch after the input projection.
struct Post {
    const float *norm_gain = nullptr;
    nk::RowOut norm_out{};
    float *state = nullptr;
    const float *conv_w = nullptr, *conv_b = nullptr;
    nk::RowOut g_out{};
};

// C = A.W^T (+bias) (R + ...), A read from `a` in the form `tc` selects.
// Returns whether the projection also did `post`'s work.
bool project(nk_decoder *dec, bool tc, const Act &a, int M, int K, const float *W, const nk::TcOperand *Wtc,
             int N, const float *bias, float *C, const float *R, const Fold *fold = nullptr,
             const Post *post = nullptr) {
    ProfScope prof(dec, M, N, K, R != nullptr, bias != nullptr);
    int done = 0;
    if (tc) {
        nk::TcEpilogue ep;
        ep.C = C;
        ep.ldc = N;
        ep.bias = bias;
        ep.R = R;
        ep.ldr = N;
        ep.ws = (dec->engine & 256) ? nullptr : dec->ksplit_ws;
        ep.l2hints = !(dec->engine & 512);
        ep.ws_floats = nk::tc_stream_k_ws_floats();
        ep.flags = dec->ksplit_flags;
        ep.n_flags = nk_decoder::KSPLIT_FLAGS;
        test_controls(dec, ep);
        apply_fold(dec, fold, ep);
        if (post && !(post->norm_gain ? (dec->engine & ENGINE_NO_POST_NORM) : (dec->engine & ENGINE_NO_POST_SSM))) {
            const nk_model *m = dec->model;
            if (post->norm_gain) {
                ep.post_norm_gain = post->norm_gain;
                ep.post_norm_eps = m->cfg.eps;
                ep.post_norm_hi = post->norm_out.hi;
                ep.post_norm_lo = post->norm_out.lo;
                ep.post_norm_f32 = post->norm_out.f32;
            } else if (post->state) {
                ep.post_state = post->state;
                ep.post_heads = dec->heads;
                ep.post_conv_w = post->conv_w;
                ep.post_conv_b = post->conv_b;
                ep.post_k = (int)m->k();
                ep.post_g_hi = post->g_out.hi;
                ep.post_g_lo = post->g_out.lo;
                ep.post_g_f32 = post->g_out.f32;
            }
            ep.post_done = &done;
        }
        ep.launches = &dec->launches;
        cuda_check(nk::tc_gemm(a.hi, a.lo, M, K, *Wtc, ep, pick_bn(dec, M, N), dec->stream, dec->err),
                   "tcgen05 projection");
        dec->prof_tc = dec->prof_tc || dec->profiling;
    } else {
        nk::GemmArgs p{a.f32, K, W, K, C, N, M, N, K, bias, R, N};
        launch_ok(dec, nk::gemm_nt_simt(p, dec->stream), "f32 projection");
    }
    return done != 0;
}

// s = SiLU(a) * b of up_proj (infer.rs:185-190) in the form the down
// projection reads (tensor-core operand pair when t_dn, else f32); returns
// where it is.  With the tensor-core operand stored gate/value-interleaved
// the SwiGLU runs in the projection's epilogue and the [M, 2H] product never
// reaches memory; the pair then goes to `scratch` ([M, 2H] floats), never to
// `gated`'s pair, which may be the A operand this projection is reading.
// Otherwise the product goes to `scratch` and a row kernel applies SwiGLU.
Act project_swiglu(nk_decoder *dec, bool tc, const Act &a, int M, int K, const float *W, const nk::TcOperand *Wtc,
                   int H, const float *bias, float *scratch, const Act &gated, bool t_dn, const Fold *fold = nullptr) {
    if (tc && Wtc->pair_half == H) {
        ProfScope prof(dec, M, 2 * H, K, false, true);
        nk::TcEpilogue ep;
        ep.swiglu = true;
        ep.bias = bias;
        ep.ldc = H;
        ep.ws = (dec->engine & 256) ? nullptr : dec->ksplit_ws;
        ep.l2hints = !(dec->engine & 512);
        ep.ws_floats = nk::tc_stream_k_ws_floats();
        ep.flags = dec->ksplit_flags;
        ep.n_flags = nk_decoder::KSPLIT_FLAGS;
        test_controls(dec, ep);
        apply_fold(dec, fold, ep);
        Act out = gated;
        if (t_dn) {
            out = Act{nullptr, scratch, scratch + (size_t)M * H};
            ep.C = out.hi;
            ep.C_lo = out.lo;
        } else {
            ep.C = gated.f32;
        }
        ep.launches = &dec->launches;
        cuda_check(nk::tc_gemm(a.hi, a.lo, M, K, *Wtc, ep, pick_bn(dec, M, 2 * H), dec->stream, dec->err),
                   "tcgen05 projection + SwiGLU");
        dec->prof_tc = dec->prof_tc || dec->profiling;
        return out;
    }
    if (tc && Wtc->pair_half) fail(NK_ERR_INVALID, "interleaved up_proj operand with a different hidden width");
    project(dec, tc, a, M, K, W, Wtc, 2 * H, bias, scratch, nullptr, fold);
    launch_ok(dec, nk::swiglu_rows(scratch, gated.out(t_dn), M, H, dec->stream), "swiglu");
    return gated;
}

// tokens[m] = argmax_n (A.W^T)[m, n] without storing the product when the
// tensor-core engine runs it (first strict maximum, tensor.rs:354-365).
void project_argmax(nk_decoder *dec, bool tc, const Act &a, int M, int K, const float *W,
                    const nk::TcOperand *Wtc, int N, uint32_t *tokens, const Fold *fold = nullptr) {
    if (tc) {
        const int bn = pick_bn(dec, M, N, true);
        int parts = 0;
        {
            ProfScope prof(dec, M, N, K, false, false);
            nk::TcEpilogue ep;
            ep.best_val = dec->best_val;
            ep.best_idx = dec->best_idx;
            ep.l2hints = false;  // the tied embedding (268 MB as hi + lo) does not fit L2
            ep.no_tile_group = (dec->engine & ENGINE_NO_TILE_GROUP) != 0;
            ep.launches = &dec->launches;
            ep.parts_out = &parts;
            if (!(dec->engine & 256)) {  // small projections split along K use the workspace
                ep.ws = dec->ksplit_ws;
                ep.ws_floats = nk::tc_stream_k_ws_floats();
            }
            apply_fold(dec, fold, ep);
            cuda_check(nk::tc_gemm(a.hi, a.lo, M, K, *Wtc, ep, bn, dec->stream, dec->err), "tcgen05 projection");
            dec->prof_tc = dec->prof_tc || dec->profiling;
        }
        launch_ok(dec, nk::argmax_partials(dec->best_val, dec->best_idx, parts, M, tokens, dec->stream),
                  "argmax partials");
    } else {
        project(dec, false, a, M, K, W, Wtc, N, nullptr, dec->logits, nullptr);
        launch_ok(dec, nk::argmax_rows(dec->logits, tokens, M, N, dec->stream), "argmax");
    }
}

// Logits projection with the sampling epilogue (pen(logit) / temperature
// into dec->logits, part maxima and +inf counts); returns the part count.
int project_sample_prep(nk_decoder *dec, const Act &a, int M, int K, const nk::TcOperand *Wtc, int N,
                        const Fold *fold = nullptr) {
    const nk::SampleParams &sp = *dec->fuse_sample;
    int bn = pick_bn(dec, M, N, true);
    if (bn == nk::TC_PAIR) bn = 256;
    int parts = 0;
    ProfScope prof(dec, M, N, K, false, false);
    nk::TcEpilogue ep;
    ep.C = dec->logits;
    ep.ldc = N;
    ep.l2hints = !(dec->engine & 512);
    ep.temperature = (std::isfinite(sp.temperature) && sp.temperature > 1e-4f) ? sp.temperature : 1e-4f;
    ep.rep_penalty = sp.rep_penalty;
    ep.pen_bits = dec->fuse_penalty ? dec->pen_bits : nullptr;
    ep.pen_words = (N + 31) / 32;
    ep.prep_max = dec->prep_max;
    ep.prep_pinf = dec->prep_pinf;
    ep.parts_out = &parts;
    if (!(dec->engine & 256)) {  // small projections split along K use the workspace
        ep.ws = dec->ksplit_ws;
        ep.ws_floats = nk::tc_stream_k_ws_floats();
    }
    apply_fold(dec, fold, ep);
    test_controls(dec, ep);
    ep.launches = &dec->launches;
    cuda_check(nk::tc_gemm(a.hi, a.lo, M, K, *Wtc, ep, bn, dec->stream, dec->err), "tcgen05 logits + sampling epilogue");
    dec->prof_tc = dec->prof_tc || dec->profiling;
    return parts;
}

bool use_persistent(const nk_decoder *dec);

void ensure_ready(nk_decoder *dec) {
    nk_model *m = dec->model;
    cuda_check(cudaSetDevice(m->device), "cudaSetDevice");
    if (m->dirty) {
        cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
        m->upload();
    }
    if (!(dec->engine & 1) && !m->tc.ready) {
        std::vector<nk::TcSource> srcs;
        for (const LayerIx &L : m->layers) {
            srcs.push_back({m->dp(L.in_w), (int)(3 * m->e()), (int)m->d()});
            srcs.push_back({m->dp(L.out_w), (int)m->d(), (int)m->e()});
            srcs.push_back({m->dp(L.up_w), (int)(2 * m->hidden()), (int)m->d(), (int)m->hidden()});
            srcs.push_back({m->dp(L.down_w), (int)m->d(), (int)m->hidden()});
        }
        srcs.push_back({m->dp(m->emb), (int)m->cfg.vocab, (int)m->d()});
        cuda_check(nk::tc_weights_build(m->tc, srcs), "tensor-core weight split");
    }
    if (dec->layers_arena != m->arena) {
        // Per-layer weight pointers for the small-batch engine; the arena
        // exists only after the first upload.
        dec->small_layers.clear();
        for (const LayerIx &L : m->layers)
            dec->small_layers.push_back({m->dp(L.n1), m->dp(L.in_w), m->dp(L.in_b), m->dp(L.conv_w), m->dp(L.conv_b),
                                         m->dp(L.out_w), m->dp(L.out_b), m->dp(L.n2), m->dp(L.up_w), m->dp(L.up_b),
                                         m->dp(L.down_w), m->dp(L.down_b)});
        dec->layers_arena = m->arena;
    }
    if (use_persistent(dec)) {
        // The persistent kernel reads out_w and down_w transposed: built once
        // per weight upload, shared by every decoder of the model.
        const size_t per = m->wT_layer_floats();
        const int d = (int)m->d(), E = (int)m->e(), H = (int)m->hidden();
        if (!m->wT) {
            cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
            cuda_check(cudaMalloc(&m->wT, std::max<size_t>(per * m->layers.size(), 1) * sizeof(float)),
                       "cudaMalloc(transposed weights)");
            for (size_t l = 0; l < m->layers.size(); ++l) {
                const LayerIx &L = m->layers[l];
                float *dst = m->wT + l * per;
                cuda_check(nk::transpose(m->dp(L.out_w), dst, d, E, dec->stream), "transpose out_w");
                cuda_check(nk::transpose(m->dp(L.down_w), dst + (size_t)E * d, d, H, dec->stream), "transpose down_w");
            }
            cuda_check(cudaStreamSynchronize(dec->stream), "cudaStreamSynchronize");
        }
        if (dec->players_key != m->wT) {
            std::vector<nk::PersistLayer> tab;
            for (size_t l = 0; l < m->layers.size(); ++l) {
                const LayerIx &L = m->layers[l];
                const float *t = m->wT + l * per;
                tab.push_back({m->dp(L.n1), m->dp(L.in_w), m->dp(L.in_b), m->dp(L.conv_w), m->dp(L.conv_b), t,
                               m->dp(L.out_b), m->dp(L.n2), m->dp(L.up_w), m->dp(L.up_b), t + (size_t)E * d,
                               m->dp(L.down_b)});
            }
            cuda_check(cudaMemcpyAsync(dec->players_dev, tab.data(), tab.size() * sizeof(nk::PersistLayer),
                                       cudaMemcpyHostToDevice, dec->stream),
                       "upload layer table");
            cuda_check(cudaStreamSynchronize(dec->stream), "cudaStreamSynchronize");
            dec->players_key = m->wT;
        }
    }
}

const nk::TcOperand *tc_op(nk_model *m, size_t i) { return m->tc.ready ? &m->tc.ops[i] : nullptr; }

void check_err_flag(nk_decoder *dec) {
    int h = 0;
    cuda_check(cudaMemcpyAsync(&h, dec->err, sizeof(int), cudaMemcpyDeviceToHost, dec->stream), "read error flag");
    cuda_check(cudaStreamSynchronize(dec->stream), "cudaStreamSynchronize");
    if (h) {
        cuda_check(cudaMemsetAsync(dec->err, 0, sizeof(int), dec->stream), "clear error flag");
        // A persistent step that stopped early may leave its accumulators
        // and barrier words set.
        if (dec->pws)
            cuda_check(cudaMemsetAsync(dec->pws, 0, nk::persistent_ws_bytes((int)dec->model->d()), dec->stream),
                       "clear persistent workspace");
        // A stream-K partial published after its finisher gave up would
        // leave a counter set for the next launch.
        if (dec->ksplit_flags)
            cuda_check(cudaMemsetAsync(dec->ksplit_flags, 0, nk_decoder::KSPLIT_FLAGS * sizeof(int), dec->stream),
                       "clear stream-K counters");
        cuda_check(cudaStreamSynchronize(dec->stream), "cudaStreamSynchronize");
        fail(NK_ERR_DEVICE, "a kernel reported an error (code " + std::to_string(h) +
                                ": 1 invalid token, 2 bounded draw, 101-104 tensor-core pipeline wait expired, 105-108 CTA-pair pipeline wait expired, 111-113 "
                                "persistent step wait expired, 121-123 stream-K hand-off wait expired, 131 prefill scan look-back wait "
                                "expired, 3 non-finite logit in "
                                "softmax_ce)");
    }
}

bool use_small(const nk_decoder *dec) {
    const nk_model *m = dec->model;
    return !(dec->engine & 8) &&
           nk::small_step_supported((int)dec->S, (int)m->d(), (int)m->e(), (int)m->hidden(), (int)m->k());
}

nk::SmallStepArgs small_args(nk_decoder *dec, const uint32_t *tokens, uint32_t *tokens_out, bool want_logits) {
    nk_model *m = dec->model;
    nk::SmallStepArgs a{};
    a.tokens = tokens;
    a.tokens_out = tokens_out;
    a.emb = m->dp(m->emb);
    a.norm_f = m->dp(m->norm_f);
    a.eps = m->cfg.eps;
    a.x = dec->x;
    a.g = dec->g;
    a.state = dec->state;
    a.heads = dec->heads;
    a.logits = want_logits ? dec->logits : nullptr;
    a.best_val = dec->best_val;
    a.best_idx = dec->best_idx;
    a.err = dec->err;
    a.M = (int)dec->S;
    a.d = (int)m->d();
    a.E = (int)m->e();
    a.H = (int)m->hidden();
    a.k = (int)m->k();
    a.V = (int)m->cfg.vocab;
    a.n_layer = (int)m->cfg.n_layer;
    a.layers = dec->small_layers.data();
    return a;
}

// The persistent step kernel for 1-4 streams when the weights are large
// (each of its 2L + 1 grid-wide phases costs a few microseconds of
// synchronisation, repaid when every phase streams megabytes of weights);
// models of under PERSISTENT_MIN_BYTES of weights (L2-resident, e.g. the
// d192 / 3-layer model: 33 us per token against 56 us) take the fused
// small-batch kernels.  Engine bit 6 forces the persistent kernel.
constexpr size_t PERSISTENT_MIN_BYTES = (size_t)96 << 20;
bool use_persistent(const nk_decoder *dec) {
    const nk_model *m = dec->model;
    const bool big = m->arena_floats * sizeof(float) >= PERSISTENT_MIN_BYTES;
    return !(dec->engine & 1024) && !(dec->engine & 8) && (big || (dec->engine & 64)) &&
           nk::persistent_step_supported((int)dec->S, (int)m->d(), (int)m->e(), (int)m->hidden(), (int)m->k(),
                                         (int)m->cfg.vocab, (int)m->cfg.n_layer);
}

void small_step_device(nk_decoder *dec, const uint32_t *tokens, bool want_logits, uint32_t *tokens_out) {
    const nk::SmallStepArgs a = small_args(dec, tokens, tokens_out, want_logits);
    if (use_persistent(dec)) {
        nk::PersistStepArgs pa{};
        pa.tokens = a.tokens;
        pa.tokens_out = a.tokens_out;
        pa.emb = a.emb;
        pa.norm_f = a.norm_f;
        pa.eps = a.eps;
        pa.state = a.state;
        pa.heads = a.heads;
        pa.logits = a.logits;
        pa.best_val = a.best_val;
        pa.best_idx = a.best_idx;
        pa.err = a.err;
        pa.ws = dec->pws;
        pa.layers = dec->players_dev;
        pa.M = a.M;
        pa.d = a.d;
        pa.E = a.E;
        pa.H = a.H;
        pa.k = a.k;
        pa.V = a.V;
        pa.n_layer = a.n_layer;
        if (dec->engine & ENGINE_WITHHOLD_ARRIVAL) {
            pa.withhold_arrival = 1;
            pa.barrier_wait_ns = TEST_WAIT_NS;
        }
        cuda_check(nk::persistent_step(pa, dec->stream), "persistent decode step");
        dec->launches += 1;
        return;
    }
    int n = 0;
    cuda_check(nk::small_step(a, dec->stream, &n), "small-batch step");
    dec->launches += (uint64_t)n;
}

void eager_step(nk_decoder *dec, const uint32_t *tokens, bool want_logits, uint32_t *tokens_out);

// Greedy steps replay a CUDA graph captured from the eager step (one per
// pair of token buffers, at most four) once an eager step has sized every
// buffer: the host cost of ~200 launches, tensor-map encodes included, is
// paid once.  Profiling and logit-producing steps run eagerly.
void step_device(nk_decoder *dec, const uint32_t *tokens, bool want_logits, uint32_t *tokens_out) {
    const bool graphable = tokens_out && !want_logits && !dec->profiling && dec->warm;
    if (graphable) {
        for (auto &gph : dec->graphs)
            if (gph.in == tokens && gph.out == tokens_out) {
                cuda_check(cudaGraphLaunch(gph.exec, dec->stream), "cudaGraphLaunch");
                dec->launches += gph.launches;
                return;
            }
        if (dec->graphs.size() < 4) {
            cudaGraph_t graph = nullptr;
            const uint64_t before = dec->launches;
            cuda_check(cudaStreamBeginCapture(dec->stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
            try {
                eager_step(dec, tokens, false, tokens_out);
            } catch (...) {
                cudaStreamEndCapture(dec->stream, &graph);
                if (graph) cudaGraphDestroy(graph);
                cudaGetLastError();
                throw;
            }
            cuda_check(cudaStreamEndCapture(dec->stream, &graph), "cudaStreamEndCapture");
            cudaGraphExec_t exec = nullptr;
            cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
            cudaGraphDestroy(graph);
            cuda_check(e, "cudaGraphInstantiate");
            dec->graphs.push_back({tokens, tokens_out, exec, dec->launches - before});
            cuda_check(cudaGraphLaunch(exec, dec->stream), "cudaGraphLaunch");
            return;
        }
    }
    eager_step(dec, tokens, want_logits, tokens_out);
    if (tokens_out && !want_logits) dec->warm = true;
}

// Decoder::step over every stream (infer.rs:106-200), tokens on the device.
// With tokens_out, the step ends in the greedy choice (sample_token with
// greedy and no penalty); the logits are then stored only if want_logits.
// Whether the step folds RMSNorm into the projections (engine bit 14):
// every projection on the tensor cores with the SwiGLU operand interleaved,
// widths on the 32-column grid.
bool fold_norms(const nk_decoder *dec) {
    const nk_model *m = dec->model;
    const int S = (int)dec->S, d = (int)m->d(), E = (int)m->e(), H = (int)m->hidden(), V = (int)m->cfg.vocab;
    // Folded by default below POST_NORM_MIN_ROWS streams at widths of 512 and
    // more, where every projection is split along K and its reduction applies
    // the row scale (measured, ms per step, folded / stand-alone norms: d768
    // 0.677 / 0.762 at 16 streams, 0.876 / 0.916 at 64, 1.335 / 1.377 at 256,
    // but 1.711 / 1.611 at 512 where the reductions take the norms over; the
    // headline widths 1.97 / 2.04 at 64 streams, 7.17 / 6.24 at 1024; d192 at
    // 256 streams 0.218 / 0.194).
    const bool want = (dec->engine & ENGINE_FOLD) ||
                      (S < POST_NORM_MIN_ROWS && d >= 512 && !(dec->engine & ENGINE_NO_AUTO_FOLD));
    if (!want || (dec->engine & 128)) return false;  // (no folded CTA-pair epilogue)
    if (d % 32 != 0 || m->cfg.n_layer == 0) return false;
    for (size_t i = 0; i < 4 * m->cfg.n_layer + 1; ++i)
        if (!tc_op(const_cast<nk_model *>(m), i)) return false;
    const nk::TcOperand *w_up = tc_op(const_cast<nk_model *>(m), 2);
    return w_up->pair_half == H && use_tc(dec, S, 3 * E, d, tc_op(const_cast<nk_model *>(m), 0)) &&
           use_tc(dec, S, d, E, tc_op(const_cast<nk_model *>(m), 1)) && use_tc(dec, S, 2 * H, d, w_up) &&
           use_tc(dec, S, d, H, tc_op(const_cast<nk_model *>(m), 3)) &&
           use_tc(dec, S, V, d, tc_op(const_cast<nk_model *>(m), 4 * m->cfg.n_layer));
}

void eager_step(nk_decoder *dec, const uint32_t *tokens, bool want_logits, uint32_t *tokens_out) {
    dec->fused_parts = 0;
    if (use_small(dec)) {
        small_step_device(dec, tokens, want_logits || !tokens_out, tokens_out);
        return;
    }
    nk_model *m = dec->model;
    const int S = (int)dec->S, d = (int)m->d(), E = (int)m->e(), H = (int)m->hidden(),
              k = (int)m->k(), V = (int)m->cfg.vocab;
    cudaStream_t st = dec->stream;
    const Act nrm{dec->nrm, dec->ahi, dec->alo}, gated{dec->g, dec->ahi, dec->alo};
    launch_ok(dec, nk::embed_rows(tokens, m->dp(m->emb), dec->x, S, d, V, dec->err, st), "embed");
    launch_ok(dec, nk::advance_heads(dec->heads, nullptr, S, k, st), "advance heads");
    if (fold_norms(dec)) {
        // RMSNorm folded into the projections: each residual projection's
        // epilogue writes the next normalisation's operand (split of x *
        // gain) and the rows' sums of squares, and the consuming projection
        // scales its rows by 1 / sqrt(ms / d + eps).  Only the first layer's
        // input norm runs as its own kernel.
        const Act nx{nullptr, dec->nhi, dec->nlo};
        const LayerIx &L0 = m->layers[0];
        launch_ok(dec, nk::rmsnorm_rows(dec->x, m->dp(L0.n1), m->cfg.eps, nx.out(true), S, d, st), "rmsnorm");
        for (uint64_t l = 0; l < m->cfg.n_layer; ++l) {
            const LayerIx &L = m->layers[l];
            const Fold f_in{l ? dec->nss : nullptr, nullptr}, f_out{nullptr, m->dp(L.n2)}, f_up{dec->nss, nullptr},
                f_dn{nullptr, l + 1 < m->cfg.n_layer ? m->dp(m->layers[l + 1].n1) : m->dp(m->norm_f)};
            Post p_ssm;
            p_ssm.state = dec->layer_state(l);
            p_ssm.conv_w = m->dp(L.conv_w);
            p_ssm.conv_b = m->dp(L.conv_b);
            p_ssm.g_out = gated.out(true);
            if (!project(dec, true, nx, S, d, m->dp(L.in_w), tc_op(m, 4 * l + 0), 3 * E, m->dp(L.in_b), dec->u,
                         nullptr, &f_in, &p_ssm))
                launch_ok(dec, nk::ssm_decode(dec->u, dec->layer_state(l), dec->heads, m->dp(L.conv_w),
                                              m->dp(L.conv_b), gated.out(true), S, E, k, st), "ssm step");
            project(dec, true, gated, S, E, m->dp(L.out_w), tc_op(m, 4 * l + 1), d, m->dp(L.out_b), dec->x, dec->x,
                    &f_out);
            const Act s_act = project_swiglu(dec, true, nx, S, d, m->dp(L.up_w), tc_op(m, 4 * l + 2), H,
                                             m->dp(L.up_b), dec->u, gated, true, &f_up);
            project(dec, true, s_act, S, H, m->dp(L.down_w), tc_op(m, 4 * l + 3), d, m->dp(L.down_b), dec->x, dec->x,
                    &f_dn);
        }
        const nk::TcOperand *w_lg = tc_op(m, 4 * m->cfg.n_layer);
        const Fold f_lg{dec->nss, nullptr};
        if (want_logits || !tokens_out) {
            if (dec->fuse_sample && !tokens_out) {
                dec->fused_parts = project_sample_prep(dec, nx, S, d, w_lg, V, &f_lg);
                return;
            }
            project(dec, true, nx, S, d, m->dp(m->emb), w_lg, V, nullptr, dec->logits, nullptr, &f_lg);
            if (tokens_out) launch_ok(dec, nk::argmax_rows(dec->logits, tokens_out, S, V, st), "argmax");
        } else {
            project_argmax(dec, true, nx, S, d, m->dp(m->emb), w_lg, V, tokens_out, &f_lg);
        }
        return;
    }
    const nk::TcOperand *w_lg = tc_op(m, 4 * m->cfg.n_layer);
    const bool t_lg = use_tc(dec, S, V, d, w_lg);
    // With few streams the projections are split along K, and their
    // reductions also run the recurrent branch (input projection) or the
    // next RMSNorm (residual projections); `normed` says that `nrm` holds the
    // next norm of x already.
    bool normed = false;
    for (uint64_t l = 0; l < m->cfg.n_layer; ++l) {
        const LayerIx &L = m->layers[l];
        const nk::TcOperand *w_in = tc_op(m, 4 * l + 0), *w_out = tc_op(m, 4 * l + 1), *w_up = tc_op(m, 4 * l + 2),
                            *w_dn = tc_op(m, 4 * l + 3);
        const bool t_in = use_tc(dec, S, 3 * E, d, w_in), t_out = use_tc(dec, S, d, E, w_out),
                   t_up = use_tc(dec, S, 2 * H, d, w_up), t_dn = use_tc(dec, S, d, H, w_dn);
        if (!normed)
            launch_ok(dec, nk::rmsnorm_rows(dec->x, m->dp(L.n1), m->cfg.eps, nrm.out(t_in), S, d, st), "rmsnorm");
        Post p_ssm;
        p_ssm.state = dec->layer_state(l);
        p_ssm.conv_w = m->dp(L.conv_w);
        p_ssm.conv_b = m->dp(L.conv_b);
        p_ssm.g_out = gated.out(t_out);
        if (!project(dec, t_in, nrm, S, d, m->dp(L.in_w), w_in, 3 * E, m->dp(L.in_b), dec->u, nullptr, nullptr,
                     &p_ssm))
            launch_ok(dec, nk::ssm_decode(dec->u, dec->layer_state(l), dec->heads, m->dp(L.conv_w), m->dp(L.conv_b),
                                          gated.out(t_out), S, E, k, st), "ssm step");
        // The norm-taking reduction runs one CTA per row: with few rows it is
        // slower than the separate kernels (measured, ms per step, with / without:
        // d768 1.070 / 1.019 at 64 streams and 1.657 / 1.763 at 512; d192 at 256
        // streams 0.214 / 0.194).
        const bool post_norm = S >= POST_NORM_MIN_ROWS;
        Post p_n2;
        p_n2.norm_gain = post_norm ? m->dp(L.n2) : nullptr;
        p_n2.norm_out = nrm.out(t_up);
        if (!project(dec, t_out, gated, S, E, m->dp(L.out_w), w_out, d, m->dp(L.out_b), dec->x, dec->x, nullptr,
                     &p_n2))
            launch_ok(dec, nk::rmsnorm_rows(dec->x, m->dp(L.n2), m->cfg.eps, nrm.out(t_up), S, d, st), "rmsnorm");
        const Act s_act = project_swiglu(dec, t_up, nrm, S, d, m->dp(L.up_w), w_up, H, m->dp(L.up_b), dec->u, gated,
                                         t_dn);
        Post p_next;
        const bool last = l + 1 == m->cfg.n_layer;
        p_next.norm_gain = !post_norm ? nullptr : last ? m->dp(m->norm_f) : m->dp(m->layers[l + 1].n1);
        p_next.norm_out = nrm.out(last ? t_lg : use_tc(dec, S, 3 * E, d, tc_op(m, 4 * (l + 1))));
        normed = project(dec, t_dn, s_act, S, H, m->dp(L.down_w), w_dn, d, m->dp(L.down_b), dec->x, dec->x, nullptr,
                         &p_next);
    }
    if (!normed)
        launch_ok(dec, nk::rmsnorm_rows(dec->x, m->dp(m->norm_f), m->cfg.eps, nrm.out(t_lg), S, d, st), "rmsnorm");
    if (want_logits || !tokens_out) {
        if (dec->fuse_sample && t_lg && !tokens_out) {
            dec->fused_parts = project_sample_prep(dec, nrm, S, d, w_lg, V);
            return;
        }
        project(dec, t_lg, nrm, S, d, m->dp(m->emb), w_lg, V, nullptr, dec->logits, nullptr);
        if (tokens_out) launch_ok(dec, nk::argmax_rows(dec->logits, tokens_out, S, V, st), "argmax");
    } else {
        project_argmax(dec, t_lg, nrm, S, d, m->dp(m->emb), w_lg, V, tokens_out);
    }
}

void validate_tokens(const nk_model *m, const uint32_t *t, size_t n) {
    for (size_t i = 0; i < n; ++i)
        if (t[i] >= m->cfg.vocab) fail(NK_ERR_INVALID, "streaming token is outside the vocabulary");
}

// The prompt loop as a chunked scan (model.rs:148-165 over each prompt,
// continuing from the current LmState).  ids/lens already on the device.
// per_chunk(t0, tcc), when set, runs after the layers of each prompt chunk,
// with the chunk's final hidden rows in p_x (row s * tcc + t is stream s,
// position t0 + t).
void prefill_device(nk_decoder *dec, const uint32_t *d_ids, const uint32_t *d_lens,
                    const std::vector<uint32_t> &lens, uint32_t max_t, float *last_logits_host,
                    const std::function<void(uint32_t, int)> &per_chunk = {}) {
    nk_model *m = dec->model;
    const int S = (int)dec->S, d = (int)m->d(), E = (int)m->e(), H = (int)m->hidden(),
              k = (int)m->k(), V = (int)m->cfg.vocab;
    cudaStream_t st = dec->stream;
    if (max_t == 0) return;
    // Rows per chunk: bounded scratch (about 3 GiB at most).
    const size_t row_bytes = 4 * (2 * (size_t)d + std::max(3 * (size_t)E, 2 * (size_t)H) + std::max((size_t)E, (size_t)H) +
                                  2 * std::max({(size_t)d, (size_t)E, (size_t)H}));
    size_t rows_budget = ((size_t)3 << 30) / row_bytes;
    rows_budget = std::min<size_t>(std::max<size_t>(rows_budget, (size_t)S), (size_t)1 << 20);
    int tc = (int)std::max<size_t>(1, std::min<size_t>(max_t, rows_budget / (size_t)S));
    const size_t rows = (size_t)S * tc;
    const size_t act_w = std::max({(size_t)d, (size_t)E, (size_t)H});
    if (rows > dec->p_rows) {
        for (float **p : {&dec->p_x, &dec->p_n, &dec->p_u, &dec->p_y, &dec->p_ahi, &dec->p_alo})
            if (*p) cudaFree(*p), *p = nullptr;
        dalloc(&dec->p_x, rows * d, "prefill x");
        dalloc(&dec->p_n, rows * d, "prefill norm");
        dalloc(&dec->p_u, rows * std::max(3 * E, 2 * H), "prefill projection");
        dalloc(&dec->p_y, rows * std::max(E, H), "prefill gated");
        dalloc(&dec->p_ahi, rows * act_w, "prefill operand hi");
        dalloc(&dec->p_alo, rows * act_w, "prefill operand lo");
        dec->p_rows = rows;
    }
    if (!dec->p_last) dalloc(&dec->p_last, (size_t)S * d, "prefill last rows");
    // Time-parallel scan when streams x channels cannot fill the GPU.
    bool chunked = (size_t)S * E < 148 * 512 && tc > 64;
    if (dec->engine & 2) chunked = true;
    if (dec->engine & 4) chunked = false;
    // The one-pass form when at least half of each warp's 32 lanes carry a
    // channel, else the three-pass form.
    const bool onepass = chunked && E >= 16;
    if (chunked) {
        const size_t need = onepass ? (nk::ssm_prefill_onepass_scratch_bytes(S, E, tc) + 3) / 4
                                    : nk::ssm_prefill_chunked_scratch_floats(S, E, tc);
        if (need > dec->p_scan_floats) {
            if (dec->p_scan) cudaFree(dec->p_scan), dec->p_scan = nullptr;
            dalloc(&dec->p_scan, need, "prefill scan scratch");
            dec->p_scan_floats = need;
        }
    }
    for (uint32_t t0 = 0; t0 < max_t; t0 += tc) {
        const int tcc = (int)std::min<uint32_t>(tc, max_t - t0);
        const int R = S * tcc;
        launch_ok(dec, nk::embed_prompt_chunk(d_ids, d_lens, (int)max_t, (int)t0, tcc, m->dp(m->emb),
                                              dec->p_x, S, d, V, dec->err, st), "prompt embed");
        const Act nrm{dec->p_n, dec->p_ahi, dec->p_alo}, gated{dec->p_y, dec->p_ahi, dec->p_alo};
        for (uint64_t l = 0; l < m->cfg.n_layer; ++l) {
            const LayerIx &L = m->layers[l];
            const nk::TcOperand *w_in = tc_op(m, 4 * l + 0), *w_out = tc_op(m, 4 * l + 1),
                                *w_up = tc_op(m, 4 * l + 2), *w_dn = tc_op(m, 4 * l + 3);
            const bool t_in = use_tc(dec, R, 3 * E, d, w_in), t_out = use_tc(dec, R, d, E, w_out),
                       t_up = use_tc(dec, R, 2 * H, d, w_up), t_dn = use_tc(dec, R, d, H, w_dn);
            launch_ok(dec, nk::rmsnorm_rows(dec->p_x, m->dp(L.n1), m->cfg.eps, nrm.out(t_in), R, d, st), "rmsnorm");
            project(dec, t_in, nrm, R, d, m->dp(L.in_w), w_in, 3 * E, m->dp(L.in_b), dec->p_u, nullptr);
            if (onepass)
                launch_ok(dec, nk::ssm_prefill_onepass(dec->p_u, dec->layer_state(l), dec->heads, d_lens, (int)t0, tcc,
                                                       m->dp(L.conv_w), m->dp(L.conv_b), gated.out(t_out), dec->p_scan,
                                                       S, E, k, dec->err, st),
                          "prefill scan");
            else if (chunked)
                launch_ok(dec, nk::ssm_prefill_chunked(dec->p_u, dec->layer_state(l), dec->heads, d_lens, (int)t0, tcc,
                                                       m->dp(L.conv_w), m->dp(L.conv_b), dec->p_y, gated.out(t_out),
                                                       dec->p_scan, S, E, k, st),
                          "prefill scan", 3);
            else
                launch_ok(dec, nk::ssm_prefill_seq(dec->p_u, dec->layer_state(l), dec->heads, d_lens, (int)t0, tcc,
                                                   m->dp(L.conv_w), m->dp(L.conv_b), gated.out(t_out), S, E, k, st),
                          "prefill scan");
            project(dec, t_out, gated, R, E, m->dp(L.out_w), w_out, d, m->dp(L.out_b), dec->p_x, dec->p_x);
            launch_ok(dec, nk::rmsnorm_rows(dec->p_x, m->dp(L.n2), m->cfg.eps, nrm.out(t_up), R, d, st), "rmsnorm");
            const Act s_act = project_swiglu(dec, t_up, nrm, R, d, m->dp(L.up_w), w_up, H, m->dp(L.up_b), dec->p_u,
                                             gated, t_dn);
            project(dec, t_dn, s_act, R, H, m->dp(L.down_w), w_dn, d, m->dp(L.down_b), dec->p_x, dec->p_x);
        }
        if (per_chunk) per_chunk(t0, tcc);
        launch_ok(dec, nk::gather_last_rows(dec->p_x, d_lens, (int)t0, tcc, dec->p_last, S, d, st), "gather last");
        launch_ok(dec, nk::advance_heads_prompt(dec->heads, d_lens, (int)t0, tcc, S, k, st), "advance heads");
    }
    // Final norm + tied logits at each stream's last prompt position.
    std::vector<uint32_t> live;
    for (int s = 0; s < S; ++s)
        if (lens[s] > 0) live.push_back((uint32_t)s);
    if (live.empty()) return;
    const nk::TcOperand *w_lg = tc_op(m, 4 * m->cfg.n_layer);
    const Act nrm{dec->nrm, dec->ahi, dec->alo};
    if ((int)live.size() == S) {
        const bool t_lg = use_tc(dec, S, V, d, w_lg);
        launch_ok(dec, nk::rmsnorm_rows(dec->p_last, m->dp(m->norm_f), m->cfg.eps, nrm.out(t_lg), S, d, st), "rmsnorm");
        project(dec, t_lg, nrm, S, d, m->dp(m->emb), w_lg, V, nullptr, dec->logits, nullptr);
    } else {
        const int n = (int)live.size();
        const bool t_lg = use_tc(dec, n, V, d, w_lg);
        uint32_t *d_idx = dec->tok_b;  // S u32 of scratch
        cuda_check(cudaMemcpyAsync(d_idx, live.data(), n * sizeof(uint32_t), cudaMemcpyHostToDevice, st), "upload index");
        launch_ok(dec, nk::gather_rows(dec->p_last, d_idx, dec->x, n, d, st), "gather");
        launch_ok(dec, nk::rmsnorm_rows(dec->x, m->dp(m->norm_f), m->cfg.eps, nrm.out(t_lg), n, d, st), "rmsnorm");
        if (!dec->p_logits) dalloc(&dec->p_logits, (size_t)S * V, "compacted logits");
        project(dec, t_lg, nrm, n, d, m->dp(m->emb), w_lg, V, nullptr, dec->p_logits, nullptr);
        launch_ok(dec, nk::scatter_rows(dec->p_logits, d_idx, dec->logits, n, V, st), "scatter");
        cuda_check(cudaStreamSynchronize(st), "cudaStreamSynchronize");
    }
    if (last_logits_host)
        cuda_check(cudaMemcpyAsync(last_logits_host, dec->logits, (size_t)S * V * sizeof(float),
                                   cudaMemcpyDeviceToHost, st), "download logits");
}

void upload_prompts(nk_decoder *dec, const uint32_t *ids, const uint32_t *lens, uint32_t max_t) {
    const size_t n = (size_t)dec->S * max_t;
    if (n > dec->p_ids_cap) {
        if (dec->p_ids) cudaFree(dec->p_ids), dec->p_ids = nullptr;
        dalloc(&dec->p_ids, n, "prompt ids");
        dec->p_ids_cap = n;
    }
    if (!dec->p_lens) dalloc(&dec->p_lens, dec->S, "prompt lengths");
    if (n) cuda_check(cudaMemcpyAsync(dec->p_ids, ids, n * sizeof(uint32_t), cudaMemcpyHostToDevice, dec->stream), "upload ids");
    cuda_check(cudaMemcpyAsync(dec->p_lens, lens, dec->S * sizeof(uint32_t), cudaMemcpyHostToDevice, dec->stream), "upload lens");
}

void ensure_history(nk_decoder *dec, uint32_t window) {
    if (window <= dec->hist_cap && dec->hist) return;
    if (dec->hist) cudaFree(dec->hist), dec->hist = nullptr;
    dalloc(&dec->hist, (size_t)dec->S * std::max<uint32_t>(window, 1), "history");
    if (!dec->hist_len) dalloc(&dec->hist_len, dec->S, "history lengths");
    dec->hist_cap = std::max<uint32_t>(window, 1);
}

nk::SampleParams to_params(const nk_sample_cfg &c) {
    return nk::SampleParams{c.temperature, c.top_k, c.top_p, c.rep_penalty, c.rep_window, c.greedy};
}

// Device scratch of the sampler for this configuration (none for most).
constexpr size_t SAMPLE_WS_BUDGET = (size_t)256 << 20;
void ensure_sample_ws(nk_decoder *dec, const nk::SampleParams &p) {
    const size_t need = nk::sample_ws_bytes((int)dec->S, (int)dec->model->cfg.vocab, p, SAMPLE_WS_BUDGET);
    if (need <= dec->samp_ws_bytes) return;
    cuda_check(cudaStreamSynchronize(dec->stream), "cudaStreamSynchronize");
    if (dec->samp_ws) cudaFree(dec->samp_ws), dec->samp_ws = nullptr, dec->samp_ws_bytes = 0;
    cuda_check(cudaMalloc(&dec->samp_ws, need), "cudaMalloc(sampler scratch)");
    dec->samp_ws_bytes = need;
}

}  // namespace

namespace nk {
void set_last_error(const std::string &msg) { g_err = msg; }
}  // namespace nk

// ================================================================ C ABI
extern "C" {

const char *nk_last_error(void) { return g_err.c_str(); }

nk_status nk_device_count(int *count) {
    return guard([&] {
        if (!count) fail(NK_ERR_INVALID, "null output");
        cuda_check(cudaGetDeviceCount(count), "cudaGetDeviceCount");
    });
}

nk_status nk_config_check(const nk_config *cfg) {
    return guard([&] {
        if (!cfg) fail(NK_ERR_INVALID, "null config");
        std::string e = config_error(*cfg);
        if (!e.empty()) fail(NK_ERR_INVALID, e);
    });
}

nk_status nk_model_create(const nk_config *cfg, int device, nk_model **out) {
    return guard([&] {
        if (!cfg || !out) fail(NK_ERR_INVALID, "null argument");
        *out = nullptr;
        std::string e = config_error(*cfg);
        if (!e.empty()) fail(NK_ERR_INVALID, e);
        e = device_limits_error(*cfg);
        if (!e.empty()) fail(NK_ERR_UNSUPPORTED, e);
        if (device != -1) {  // -1: host-only model (init, checkpoint I/O)
            int n = 0;
            cuda_check(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
            if (device < 0 || device >= n) fail(NK_ERR_INVALID, "device index out of range");
        }
        auto m = std::make_unique<nk_model>();
        m->cfg = *cfg;
        m->device = device;
        m->build_layout();
        *out = m.release();
    });
}

nk_status nk_model_destroy(nk_model *model) {
    return guard([&] { delete model; });
}

nk_status nk_model_config(const nk_model *model, nk_config *out) {
    return guard([&] {
        if (!model || !out) fail(NK_ERR_INVALID, "null argument");
        *out = model->cfg;
    });
}

nk_status nk_model_init_random(nk_model *model, uint64_t seed, uint64_t rng_after[4]) {
    return guard([&] {
        if (!model) fail(NK_ERR_INVALID, "null model");
        HostRng rng(seed);
        model->init_random(rng);
        if (rng_after)
            for (int i = 0; i < 4; ++i) rng_after[i] = rng.s[i];
    });
}

nk_status nk_model_tensor_count(const nk_model *model, uint64_t *count) {
    return guard([&] {
        if (!model || !count) fail(NK_ERR_INVALID, "null argument");
        *count = model->tensors.size();
    });
}

nk_status nk_model_tensor_info(const nk_model *model, uint64_t index, const char **name,
                               uint32_t *rank, uint64_t shape[4]) {
    return guard([&] {
        if (!model) fail(NK_ERR_INVALID, "null model");
        if (index >= model->tensors.size()) fail(NK_ERR_INVALID, "tensor index out of range");
        const Tensor &t = model->tensors[index];
        if (name) *name = t.name.c_str();
        if (rank) *rank = (uint32_t)t.shape.size();
        if (shape)
            for (size_t i = 0; i < 4; ++i) shape[i] = i < t.shape.size() ? t.shape[i] : 0;
    });
}

nk_status nk_model_set_tensor(nk_model *model, const char *name, const float *data,
                              const uint64_t *shape, uint32_t rank) {
    return guard([&] {
        if (!model || !name || (!data) || (!shape && rank)) fail(NK_ERR_INVALID, "null argument");
        auto it = model->by_name.find(name);
        if (it == model->by_name.end()) fail(NK_ERR_INVALID, std::string("unknown tensor '") + name + "'");
        Tensor &t = model->tensors[it->second];
        if (rank != t.shape.size() || !std::equal(t.shape.begin(), t.shape.end(), shape))
            fail(NK_ERR_INVALID, std::string("tensor '") + name + "' has the wrong shape");
        const uint64_t n = t.numel();
        for (uint64_t i = 0; i < n; ++i)
            if (!std::isfinite(data[i])) fail(NK_ERR_INVALID, std::string("tensor '") + name + "' contains a non-finite value");
        model->ensure_host();  // the next upload copies every tensor from the host
        std::memcpy(t.host.data(), data, n * sizeof(float));
        model->dirty = true;
    });
}

nk_status nk_model_get_tensor(const nk_model *model, const char *name, float *out, uint64_t numel) {
    return guard([&] {
        if (!model || !name || !out) fail(NK_ERR_INVALID, "null argument");
        auto it = model->by_name.find(name);
        if (it == model->by_name.end()) fail(NK_ERR_INVALID, std::string("unknown tensor '") + name + "'");
        const Tensor &t = model->tensors[it->second];
        if (numel != t.numel()) fail(NK_ERR_INVALID, "wrong element count");
        const_cast<nk_model *>(model)->ensure_host();
        std::memcpy(out, t.host.data(), numel * sizeof(float));
    });
}

namespace {

// Where one tensor's f32 payload sits in a checkpoint file.
struct CkptTensorRec {
    std::string name;
    std::vector<uint64_t> shape;
    uint64_t numel = 0, file_off = 0;
};

struct CkptIndex {
    CkptData meta;  // metadata only (no tensor payloads)
    std::vector<CkptTensorRec> tensors;  // file order
    uint64_t body = 0;                   // bytes covered by the CRC
    uint32_t want_crc = 0;
};

// ckpt.rs:299-383 without reading the payloads: the header, metadata and
// every tensor's name / shape / count are parsed with small reads, each
// payload is skipped; the same structural checks as read_ckpt.
CkptIndex scan_ckpt(int fd, uint64_t size) {
    if (size > MAX_CKPT_BYTES) fail(NK_ERR_IO, "checkpoint file exceeds the supported size limit");
    if (size < 24) fail(NK_ERR_IO, "checkpoint too small");
    CkptIndex ix;
    ix.body = size - 4;
    std::vector<uint8_t> buf(1 << 20);
    uint64_t buf_pos = 0, buf_len = 0, off = 0;
    auto fill = [&](uint64_t at, uint64_t want) {
        const uint64_t len = std::min<uint64_t>(std::max<uint64_t>(want, buf.size()), size - at);
        if (len > buf.size()) buf.resize(len);
        uint64_t got = 0;
        while (got < len) {
            const ssize_t r = pread(fd, buf.data() + got, len - got, (off_t)(at + got));
            if (r <= 0) fail(NK_ERR_IO, "checkpoint read failed");
            got += (uint64_t)r;
        }
        buf_pos = at;
        buf_len = len;
    };
    auto take = [&](uint64_t n) -> const uint8_t * {
        if (n > ix.body - off) fail(NK_ERR_IO, "checkpoint truncated");
        if (off < buf_pos || off + n > buf_pos + buf_len) fill(off, n);
        const uint8_t *p = buf.data() + (off - buf_pos);
        off += n;
        return p;
    };
    auto u32 = [&]() -> uint32_t {
        const uint8_t *p = take(4);
        return p[0] | (p[1] << 8) | (p[2] << 16) | ((uint32_t)p[3] << 24);
    };
    auto str = [&]() {
        const uint32_t n = u32();
        const uint8_t *p = take(n);
        return std::string((const char *)p, n);
    };
    {
        uint8_t t[4];
        if (pread(fd, t, 4, (off_t)ix.body) != 4) fail(NK_ERR_IO, "checkpoint read failed");
        ix.want_crc = t[0] | (t[1] << 8) | (t[2] << 16) | ((uint32_t)t[3] << 24);
    }
    if (std::memcmp(take(8), MAGIC, 8) != 0) fail(NK_ERR_IO, "not a noetic checkpoint");
    if (u32() != 1) fail(NK_ERR_IO, "unsupported checkpoint version");
    const uint32_t n_meta = u32();
    if (n_meta > 1000000) fail(NK_ERR_IO, "checkpoint contains too many metadata entries");
    for (uint32_t i = 0; i < n_meta; ++i) {
        std::string k = str(), v = str();
        if (k.empty() || ix.meta.meta.count(k)) fail(NK_ERR_IO, "checkpoint metadata contains an empty or duplicate key");
        ix.meta.meta[k] = v;
    }
    const uint32_t n_t = u32();
    if (n_t > 1000000) fail(NK_ERR_IO, "checkpoint contains too many tensors");
    std::map<std::string, int> seen;
    for (uint32_t i = 0; i < n_t; ++i) {
        CkptTensorRec r;
        r.name = str();
        if (r.name.empty() || seen.count(r.name)) fail(NK_ERR_IO, "checkpoint contains an empty or duplicate tensor name");
        seen[r.name] = 1;
        const uint32_t rank = u32();
        if (rank > 32 || rank > (ix.body - off) / 4) fail(NK_ERR_IO, "checkpoint tensor rank is invalid");
        r.shape.resize(rank);
        uint64_t expect = 1;
        bool overflow = false;
        for (auto &d : r.shape) {
            d = u32();
            if (d != 0 && expect > UINT64_MAX / d) overflow = true;
            expect *= d;
        }
        const uint32_t numel = u32();
        if (numel > (ix.body - off) / 4) fail(NK_ERR_IO, "checkpoint tensor payload is truncated");
        if (overflow || expect != numel) fail(NK_ERR_IO, "checkpoint tensor shape does not match its element count");
        r.numel = numel;
        r.file_off = off;
        off += 4ull * numel;  // the payload, read by the streaming pass
        ix.tensors.push_back(std::move(r));
    }
    if (off != ix.body) fail(NK_ERR_IO, "checkpoint has trailing data");
    return ix;
}

// The checkpoint body streamed from the file straight into device memory:
// worker threads take CKPT_CHUNK-byte chunks in turn, read each into one of
// two pinned buffers, CRC it, and copy the payload bytes it holds to their
// device destinations with cudaMemcpyAsync on the thread's own stream; the
// chunk CRCs are combined in file order at the end.  dest[i] is tensor i's
// device address (every tensor, aux.* included, has one).
constexpr uint64_t CKPT_CHUNK = 16ull << 20;
constexpr unsigned CKPT_THREADS = 16;

// Pinned staging buffers (two per loader thread), allocated on the first
// load and kept for later ones: pinning memory costs more than reading it.
struct PinnedPool {
    std::mutex mu;
    std::vector<uint8_t *> free;
    uint8_t *take() {
        std::lock_guard<std::mutex> g(mu);
        if (!free.empty()) {
            uint8_t *p = free.back();
            free.pop_back();
            return p;
        }
        uint8_t *p = nullptr;
        return cudaHostAlloc((void **)&p, CKPT_CHUNK, cudaHostAllocPortable) == cudaSuccess ? p : nullptr;
    }
    void give(uint8_t *p) {
        if (!p) return;
        std::lock_guard<std::mutex> g(mu);
        free.push_back(p);
    }
};
PinnedPool &pinned_pool() {
    static PinnedPool *pool = new PinnedPool();
    return *pool;
}

uint32_t stream_ckpt_to_device(int fd, int device, const CkptIndex &ix, const std::vector<char *> &dest) {
    const uint64_t n_chunks = (ix.body + CKPT_CHUNK - 1) / CKPT_CHUNK;
    std::vector<uint32_t> crc(n_chunks, 0);
    std::atomic<uint64_t> next{0};
    std::mutex err_mu;
    std::string err;
    auto worker = [&]() {
        cudaStream_t st = nullptr;
        uint8_t *pin[2] = {nullptr, nullptr};
        cudaEvent_t ev[2] = {nullptr, nullptr};
        auto set_err = [&](const std::string &m) {
            std::lock_guard<std::mutex> g(err_mu);
            if (err.empty()) err = m;
        };
        if (cudaSetDevice(device) != cudaSuccess || cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess ||
            !(pin[0] = pinned_pool().take()) || !(pin[1] = pinned_pool().take()) ||
            cudaEventCreateWithFlags(&ev[0], cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&ev[1], cudaEventDisableTiming) != cudaSuccess) {
            set_err("checkpoint staging buffers could not be allocated");
        } else {
            int b = 0;
            for (;;) {
                {
                    std::lock_guard<std::mutex> g(err_mu);
                    if (!err.empty()) break;
                }
                const uint64_t c = next.fetch_add(1);
                if (c >= n_chunks) break;
                const uint64_t c0 = c * CKPT_CHUNK, len = std::min(CKPT_CHUNK, ix.body - c0);
                if (cudaEventSynchronize(ev[b]) != cudaSuccess) {  // the buffer's previous copies are done
                    set_err("checkpoint upload failed");
                    break;
                }
                uint64_t got = 0;
                while (got < len) {
                    const ssize_t r = pread(fd, pin[b] + got, len - got, (off_t)(c0 + got));
                    if (r <= 0) break;
                    got += (uint64_t)r;
                }
                if (got != len) {
                    set_err("checkpoint read failed");
                    break;
                }
                crc[c] = crc32_fast(pin[b], len);
                // Payloads overlapping [c0, c0 + len): the first one ending after c0.
                size_t lo = 0, hi = ix.tensors.size();
                while (lo < hi) {
                    const size_t mid = (lo + hi) / 2;
                    const CkptTensorRec &t = ix.tensors[mid];
                    if (t.file_off + 4 * t.numel <= c0)
                        lo = mid + 1;
                    else
                        hi = mid;
                }
                bool ok = true;
                for (size_t i = lo; i < ix.tensors.size() && ix.tensors[i].file_off < c0 + len; ++i) {
                    const CkptTensorRec &t = ix.tensors[i];
                    const uint64_t s0 = std::max(t.file_off, c0), s1 = std::min(t.file_off + 4 * t.numel, c0 + len);
                    if (s1 <= s0) continue;
                    ok &= cudaMemcpyAsync(dest[i] + (s0 - t.file_off), pin[b] + (s0 - c0), s1 - s0,
                                          cudaMemcpyHostToDevice, st) == cudaSuccess;
                }
                ok &= cudaEventRecord(ev[b], st) == cudaSuccess;
                if (!ok) {
                    set_err("checkpoint upload failed");
                    break;
                }
                b ^= 1;
            }
        }
        if (st) cudaStreamSynchronize(st);
        for (int k = 0; k < 2; ++k) {
            if (ev[k]) cudaEventDestroy(ev[k]);
            pinned_pool().give(pin[k]);
        }
        if (st) cudaStreamDestroy(st);
    };
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const unsigned n_threads = (unsigned)std::min<uint64_t>({CKPT_THREADS, hw, std::max<uint64_t>(n_chunks, 1)});
    std::vector<std::thread> pool;
    for (unsigned i = 0; i < n_threads; ++i) pool.emplace_back(worker);
    for (auto &t : pool) t.join();
    if (!err.empty()) fail(NK_ERR_IO, err);
    uint32_t total = n_chunks ? crc[0] : crc32_fast(nullptr, 0);
    for (uint64_t c = 1; c < n_chunks; ++c)
        total = crc32_combine(total, crc[c], std::min(CKPT_CHUNK, ix.body - c * CKPT_CHUNK));
    return total;
}

nk_config ckpt_config(const CkptData &c) {
    nk_config cfg{};  // cmd_gen's metadata rules (cli.rs:909-920)
    cfg.vocab = meta_usize(c, "vocab");
    cfg.d_model = meta_usize(c, "d_model");
    cfg.n_layer = meta_usize(c, "n_layer");
    cfg.expand = meta_usize(c, "expand");
    cfg.conv_k = meta_usize(c, "conv_k");
    cfg.mlp_mult = meta_usize(c, "mlp_mult");
    cfg.eps = meta_f32(c, "eps", false, 1e-5f);
    cfg.tau_max = meta_f32(c, "tau_max", true, 0.0f);
    std::string e = config_error(cfg);
    if (!e.empty()) fail(NK_ERR_IO, "checkpoint model configuration is invalid: " + e);
    return cfg;
}

// The direct loader (device models): scan, create the model and its device
// arena, stream the payloads into it, then check the CRC and that every
// value is finite on the device.  Nothing of a rejected file is returned.
nk_model *load_ckpt_direct(const char *path, int device) {
    const int fd = open(path, O_RDONLY);
    if (fd < 0) fail(NK_ERR_IO, std::string("cannot open checkpoint ") + path);
    std::unique_ptr<int, void (*)(int *)> ofd(new int(fd), [](int *f) {
        close(*f);
        delete f;
    });
    const off_t size = lseek(fd, 0, SEEK_END);
    if (size < 0) fail(NK_ERR_IO, "cannot size the checkpoint file");
    const CkptIndex ix = scan_ckpt(fd, (uint64_t)size);
    nk_config cfg = ckpt_config(ix.meta);
    nk_model *m = nullptr;
    {
        std::string e = config_error(cfg);
        if (!e.empty()) fail(NK_ERR_IO, "checkpoint model configuration is invalid: " + e);
        e = device_limits_error(cfg);
        if (!e.empty()) fail(NK_ERR_UNSUPPORTED, e);
        int n = 0;
        cuda_check(cudaGetDeviceCount(&n), "cudaGetDeviceCount");
        if (device < 0 || device >= n) fail(NK_ERR_INVALID, "device index out of range");
        m = new nk_model();
        m->cfg = cfg;
        m->device = device;
        m->host_valid = false;  // no host copies: the arena is filled directly
        m->build_layout();
    }
    std::unique_ptr<nk_model> own(m);
    // apply_exact (ckpt.rs:410-436): the exact model tensor set; aux.* is
    // checked (CRC, finite) but not kept.
    size_t model_tensors = 0;
    uint64_t aux_bytes = 0;
    for (const auto &t : ix.tensors) {
        if (t.name.rfind("aux.", 0) == 0)
            aux_bytes += (4 * t.numel + 255) & ~uint64_t(255);
        else
            ++model_tensors;
    }
    if (model_tensors != own->tensors.size()) fail(NK_ERR_IO, "checkpoint tensor set does not exactly match the model");
    std::map<std::string, const CkptTensorRec *> by_name;
    for (const auto &t : ix.tensors) by_name[t.name] = &t;
    for (auto &t : own->tensors) {
        auto it = by_name.find(t.name);
        if (it == by_name.end()) fail(NK_ERR_IO, "checkpoint is missing tensor '" + t.name + "'");
        if (it->second->shape != t.shape) fail(NK_ERR_IO, "checkpoint tensor '" + t.name + "' has the wrong shape");
    }
    own->ensure_arena();
    cuda_check(cudaMemset(own->arena, 0, own->arena_floats * sizeof(float)), "memset");  // padding stays finite
    char *aux = nullptr;
    if (aux_bytes) cuda_check(cudaMalloc(&aux, aux_bytes), "cudaMalloc(aux tensors)");
    std::unique_ptr<char, void (*)(char *)> oaux(aux, [](char *q) {
        if (q) cudaFree(q);
    });
    if (aux) cuda_check(cudaMemset(aux, 0, aux_bytes), "memset");
    std::vector<char *> dest;
    uint64_t aux_off = 0;
    for (const auto &t : ix.tensors) {
        if (t.name.rfind("aux.", 0) == 0) {
            dest.push_back(aux + aux_off);
            aux_off += (4 * t.numel + 255) & ~uint64_t(255);
        } else {
            dest.push_back((char *)(own->arena + own->tensors[own->by_name.at(t.name)].dev_off));
        }
    }
    const uint32_t got = stream_ckpt_to_device(fd, device, ix, dest);
    if (got != ix.want_crc) fail(NK_ERR_IO, "checkpoint CRC mismatch (corrupt file)");
    int *flag = nullptr;
    dalloc(&flag, 1, "flag");
    std::unique_ptr<int, void (*)(int *)> oflag(flag, [](int *q) { cudaFree(q); });
    cuda_check(cudaMemset(flag, 0, sizeof(int)), "memset");
    cuda_check(nk::any_nonfinite(own->arena, own->arena_floats, flag, nullptr), "finite check");
    if (aux) cuda_check(nk::any_nonfinite((const float *)aux, aux_bytes / 4, flag, nullptr), "finite check");
    int h = 0;
    cuda_check(cudaMemcpy(&h, flag, sizeof(int), cudaMemcpyDeviceToHost), "finite check");
    if (h) fail(NK_ERR_IO, "checkpoint tensor contains a non-finite value");
    own->dirty = false;
    return own.release();
}

}  // namespace

nk_status nk_crc32(const uint8_t *data, uint64_t n, uint32_t *out) {
    return guard([&] {
        if (!out || (n && !data)) fail(NK_ERR_INVALID, "null argument");
        // The loader's form: CKPT_CHUNK pieces, CRC'd separately, combined.
        uint32_t total = crc32_fast(data, std::min(n, CKPT_CHUNK));
        for (uint64_t c0 = CKPT_CHUNK; c0 < n; c0 += CKPT_CHUNK) {
            const uint64_t len = std::min(CKPT_CHUNK, n - c0);
            total = crc32_combine(total, crc32_fast(data + c0, len), len);
        }
        *out = total;
    });
}

nk_status nk_model_load_ckpt(const char *path, int device, nk_model **out) {
    return guard([&] {
        if (!path || !out) fail(NK_ERR_INVALID, "null argument");
        *out = nullptr;
        if (device >= 0) {
            *out = load_ckpt_direct(path, device);
            return;
        }
        CkptData c = read_ckpt(path);
        nk_config cfg{};  // cmd_gen's metadata rules (cli.rs:909-920)
        cfg.vocab = meta_usize(c, "vocab");
        cfg.d_model = meta_usize(c, "d_model");
        cfg.n_layer = meta_usize(c, "n_layer");
        cfg.expand = meta_usize(c, "expand");
        cfg.conv_k = meta_usize(c, "conv_k");
        cfg.mlp_mult = meta_usize(c, "mlp_mult");
        cfg.eps = meta_f32(c, "eps", false, 1e-5f);
        cfg.tau_max = meta_f32(c, "tau_max", true, 0.0f);
        std::string e = config_error(cfg);
        if (!e.empty()) fail(NK_ERR_IO, "checkpoint model configuration is invalid: " + e);
        nk_model *m = nullptr;
        nk_status st = nk_model_create(&cfg, device, &m);
        if (st != NK_OK) fail(st, g_err);
        std::unique_ptr<nk_model> own(m);
        // apply_exact (ckpt.rs:410-436): exact model tensor set, aux.* ignored.
        size_t model_tensors = 0;
        for (auto &kv : c.tensors)
            if (kv.first.rfind("aux.", 0) != 0) ++model_tensors;
        if (model_tensors != own->tensors.size()) fail(NK_ERR_IO, "checkpoint tensor set does not exactly match the model");
        for (auto &t : own->tensors) {
            auto it = c.tensors.find(t.name);
            if (it == c.tensors.end()) fail(NK_ERR_IO, "checkpoint is missing tensor '" + t.name + "'");
            if (it->second.first != t.shape) fail(NK_ERR_IO, "checkpoint tensor '" + t.name + "' has the wrong shape");
        }
        for (auto &t : own->tensors) t.host = std::move(c.tensors[t.name].second);
        own->dirty = true;
        *out = own.release();
    });
}

nk_status nk_model_save_ckpt(const nk_model *model, const char *path) {
    return guard([&] {
        if (!model || !path) fail(NK_ERR_INVALID, "null argument");
        const_cast<nk_model *>(model)->ensure_host();
        const nk_config &c = model->cfg;
        std::vector<std::pair<std::string, std::string>> meta = {
            {"vocab", std::to_string(c.vocab)},       {"d_model", std::to_string(c.d_model)},
            {"n_layer", std::to_string(c.n_layer)},   {"expand", std::to_string(c.expand)},
            {"conv_k", std::to_string(c.conv_k)},     {"mlp_mult", std::to_string(c.mlp_mult)},
            {"eps", fmt_f32(c.eps)},                  {"tau_max", fmt_f32(c.tau_max)}};
        std::vector<uint8_t> b;
        b.insert(b.end(), MAGIC, MAGIC + 8);
        put_u32(b, 1);
        put_u32(b, (uint32_t)meta.size());
        for (auto &kv : meta) {
            put_str(b, kv.first);
            put_str(b, kv.second);
        }
        put_u32(b, (uint32_t)model->tensors.size());
        for (const Tensor &t : model->tensors) {
            put_str(b, t.name);
            put_u32(b, (uint32_t)t.shape.size());
            for (auto dmn : t.shape) put_u32(b, (uint32_t)dmn);
            put_u32(b, (uint32_t)t.numel());
            const size_t off = b.size();
            b.resize(off + 4 * t.numel());
            std::memcpy(b.data() + off, t.host.data(), 4 * t.numel());
        }
        put_u32(b, crc32(b.data(), b.size()));
        const std::string tmp = std::string(path) + ".tmp";
        {
            std::ofstream f(tmp, std::ios::binary);
            if (!f) fail(NK_ERR_IO, "cannot open checkpoint for writing");
            f.write((const char *)b.data(), (std::streamsize)b.size());
            if (!f) fail(NK_ERR_IO, "checkpoint write failed");
        }
        if (std::rename(tmp.c_str(), path) != 0) fail(NK_ERR_IO, "checkpoint rename failed");
    });
}

nk_status nk_decoder_create(nk_model *model, uint32_t n_streams, nk_decoder **out) {
    return guard([&] {
        if (!model || !out) fail(NK_ERR_INVALID, "null argument");
        if (n_streams == 0) fail(NK_ERR_INVALID, "n_streams must be positive");
        if (model->device < 0) fail(NK_ERR_INVALID, "a host-only model (device -1) cannot run a decoder");
        *out = nullptr;
        cuda_check(cudaSetDevice(model->device), "cudaSetDevice");
        auto dec = std::make_unique<nk_decoder>();
        dec->model = model;
        dec->S = n_streams;
        cuda_check(cudaStreamCreateWithFlags(&dec->stream, cudaStreamNonBlocking), "cudaStreamCreate");
        const size_t S = n_streams, d = model->d(), E = model->e(), H = model->hidden(), V = model->cfg.vocab;
        const size_t state_floats = model->cfg.n_layer * S * (model->k() + 1) * E;
        if ((double)S * V > 2.0e9 || (double)S * std::max(3 * E, 2 * H) > 2.0e9)
            fail(NK_ERR_UNSUPPORTED, "streams x vocabulary exceeds the decoder's logit buffer limit");
        dalloc(&dec->state, state_floats, "decoder state");
        dalloc(&dec->heads, S, "heads");
        dalloc(&dec->x, S * d, "x");
        dalloc(&dec->nrm, S * d, "norm");
        dalloc(&dec->u, S * std::max(3 * E, 2 * H), "projection");
        dalloc(&dec->g, S * std::max(E, H), "gated");
        dalloc(&dec->logits, S * V, "logits");
        const size_t act_w = std::max({d, E, H});
        dalloc(&dec->ahi, S * act_w, "operand hi");
        dalloc(&dec->alo, S * act_w, "operand lo");
        dalloc(&dec->nhi, S * d, "normalised operand hi");
        dalloc(&dec->nlo, S * d, "normalised operand lo");
        dalloc(&dec->nss, S * ((d + 31) / 32), "row sums of squares");
        const size_t tiles = std::max<size_t>({(size_t)nk::tc_argmax_parts((int)V, 128),
                                               (size_t)nk::small_logit_tiles((int)V),
                                               (size_t)nk::persistent_partials()});
        dalloc(&dec->best_val, S * tiles, "argmax partials");
        dalloc(&dec->best_idx, S * tiles, "argmax partials");
        dalloc(&dec->tok_a, S, "tokens");
        dalloc(&dec->tok_b, S, "tokens");
        dalloc(&dec->err, 1, "error flag");
        dalloc(&dec->pws, nk::persistent_ws_bytes((int)d), "persistent step workspace");
        cuda_check(cudaMemset(dec->pws, 0, nk::persistent_ws_bytes((int)d)), "memset");
        dalloc(&dec->ksplit_ws, nk::tc_stream_k_ws_floats(), "stream-K workspace");
        dalloc(&dec->ksplit_flags, nk_decoder::KSPLIT_FLAGS, "stream-K counters");
        cuda_check(cudaMemset(dec->ksplit_flags, 0, nk_decoder::KSPLIT_FLAGS * sizeof(int)), "memset");
        dalloc(&dec->players_dev, model->cfg.n_layer, "layer table");
        dalloc(&dec->rng, S * 4, "rng");
        cuda_check(cudaMemset(dec->err, 0, sizeof(int)), "memset");
        cuda_check(cudaMemset(dec->logits, 0, S * V * sizeof(float)), "memset");
        *out = dec.release();
        nk_status st = nk_decoder_reset(*out, 0, n_streams);
        if (st != NK_OK) {
            delete *out;
            *out = nullptr;
            fail(st, g_err);
        }
    });
}

nk_status nk_decoder_destroy(nk_decoder *dec) {
    return guard([&] { delete dec; });
}

nk_status nk_decoder_streams(const nk_decoder *dec, uint32_t *n) {
    return guard([&] {
        if (!dec || !n) fail(NK_ERR_INVALID, "null argument");
        *n = dec->S;
    });
}

nk_status nk_decoder_reset(nk_decoder *dec, uint32_t first, uint32_t count) {
    return guard([&] {
        if (!dec) fail(NK_ERR_INVALID, "null decoder");
        if ((uint64_t)first + count > dec->S) fail(NK_ERR_INVALID, "stream range out of bounds");
        cuda_check(cudaSetDevice(dec->model->device), "cudaSetDevice");
        const size_t per = (dec->model->k() + 1) * dec->model->e();
        for (uint64_t l = 0; l < dec->L(); ++l)
            cuda_check(cudaMemsetAsync(dec->layer_state(l) + (size_t)first * per, 0,
                                       (size_t)count * per * sizeof(float), dec->stream), "reset state");
        std::vector<uint32_t> h(count, (uint32_t)(dec->model->k() - 1));  // infer.rs:32, 42
        cuda_check(cudaMemcpyAsync(dec->heads + first, h.data(), count * sizeof(uint32_t),
                                   cudaMemcpyHostToDevice, dec->stream), "reset heads");
        cuda_check(cudaStreamSynchronize(dec->stream), "cudaStreamSynchronize");
    });
}

nk_status nk_decoder_step(nk_decoder *dec, const uint32_t *tokens, float *logits_out) {
    return guard([&] {
        if (!dec || !tokens) fail(NK_ERR_INVALID, "null argument");
        validate_tokens(dec->model, tokens, dec->S);
        ensure_ready(dec);
        cuda_check(cudaMemcpyAsync(dec->tok_a, tokens, dec->S * sizeof(uint32_t), cudaMemcpyHostToDevice,
                                   dec->stream), "upload tokens");
        step_device(dec, dec->tok_a, true, nullptr);
        if (logits_out)
            cuda_check(cudaMemcpyAsync(logits_out, dec->logits, (size_t)dec->S * dec->model->cfg.vocab * sizeof(float),
                                       cudaMemcpyDeviceToHost, dec->stream), "download logits");
        check_err_flag(dec);
    });
}

nk_status nk_decoder_step_greedy_device(nk_decoder *dec, const uint32_t *tokens_in, uint32_t *tokens_out) {
    return guard([&] {
        if (!dec || !tokens_in || !tokens_out) fail(NK_ERR_INVALID, "null argument");
        ensure_ready(dec);
        step_device(dec, tokens_in, false, tokens_out);
    });
}

nk_status nk_decoder_step_greedy(nk_decoder *dec, const uint32_t *tokens_in, uint32_t *tokens_out) {
    return guard([&] {
        if (!dec || !tokens_in || !tokens_out) fail(NK_ERR_INVALID, "null argument");
        validate_tokens(dec->model, tokens_in, dec->S);
        ensure_ready(dec);
        cuda_check(cudaMemcpyAsync(dec->tok_a, tokens_in, dec->S * sizeof(uint32_t), cudaMemcpyHostToDevice,
                                   dec->stream), "upload tokens");
        step_device(dec, dec->tok_a, false, dec->tok_b);
        cuda_check(cudaMemcpyAsync(tokens_out, dec->tok_b, dec->S * sizeof(uint32_t), cudaMemcpyDeviceToHost,
                                   dec->stream), "download tokens");
        check_err_flag(dec);
    });
}

nk_status nk_decoder_prefill(nk_decoder *dec, const uint32_t *ids, const uint32_t *lens, uint32_t max_t,
                             float *last_logits) {
    return guard([&] {
        if (!dec || !lens || (!ids && max_t)) fail(NK_ERR_INVALID, "null argument");
        std::vector<uint32_t> lv(lens, lens + dec->S);
        for (uint32_t s = 0; s < dec->S; ++s) {
            if (lv[s] > max_t) fail(NK_ERR_INVALID, "prompt length exceeds max_t");
            validate_tokens(dec->model, ids + (size_t)s * max_t, lv[s]);
        }
        ensure_ready(dec);
        upload_prompts(dec, ids, lens, max_t);
        prefill_device(dec, dec->p_ids, dec->p_lens, lv, max_t, last_logits);
        check_err_flag(dec);
    });
}

nk_status nk_model_loss(nk_model *model, const uint32_t *ids, const uint32_t *targets, uint32_t batch, uint32_t t,
                        float *loss_out, float *logits_out) {
    nk_decoder *tmp = nullptr;
    nk_status st = guard([&] {
        if (!model || !ids || !targets || !loss_out) fail(NK_ERR_INVALID, "null argument");
        if (batch == 0 || t == 0) fail(NK_ERR_INVALID, "batch and sequence length must be positive");
        const size_t n = (size_t)batch * t;
        validate_tokens(model, ids, n);
        const uint32_t V = (uint32_t)model->cfg.vocab;
        for (size_t i = 0; i < n; ++i)
            if (targets[i] != 0xFFFFFFFFu && targets[i] >= V) fail(NK_ERR_INVALID, "softmax_ce: target out of range");
    });
    if (st != NK_OK) return st;
    // A scratch decoder of `batch` streams from the zero state (Lm::logits
    // starts every sequence from zero padding and a zero scan carry).
    st = nk_decoder_create(model, batch, &tmp);
    if (st != NK_OK) return st;
    st = guard([&] {
        nk_decoder *dec = tmp;
        nk_model *m = model;
        const int S = (int)batch, d = (int)m->d();
        const size_t n = (size_t)batch * t, V = m->cfg.vocab;
        ensure_ready(dec);
        std::vector<uint32_t> lv(batch, t);
        upload_prompts(dec, ids, lv.data(), t);
        uint32_t *d_tg = nullptr;
        double *d_nll = nullptr;
        uint32_t *d_cnt = nullptr;
        float *d_lg = nullptr, *d_loss = nullptr;
        struct Free {
            std::vector<void *> p;
            ~Free() {
                for (void *q : p) cudaFree(q);
            }
        } fr;
        dalloc(&d_tg, n, "targets");
        fr.p.push_back(d_tg);
        dalloc(&d_nll, n, "nll");
        fr.p.push_back(d_nll);
        dalloc(&d_cnt, n, "nll counted");
        fr.p.push_back(d_cnt);
        dalloc(&d_loss, 1, "loss");
        fr.p.push_back(d_loss);
        // Logits in blocks of at most 512 MiB.
        const int block_rows = (int)std::max<size_t>(1, std::min<size_t>(((size_t)512 << 20) / (4 * V), 1u << 16));
        dalloc(&d_lg, (size_t)block_rows * V, "logits block");
        fr.p.push_back(d_lg);
        cuda_check(cudaMemcpyAsync(d_tg, targets, n * sizeof(uint32_t), cudaMemcpyHostToDevice, dec->stream),
                   "upload targets");
        const nk::TcOperand *w_lg = tc_op(m, 4 * m->cfg.n_layer);
        auto per_chunk = [&](uint32_t t0, int tcc) {
            const int R = S * tcc;
            for (int r0 = 0; r0 < R; r0 += block_rows) {
                const int rr = std::min(block_rows, R - r0);
                const bool t_lg = use_tc(dec, rr, (int)V, d, w_lg);
                const Act nrm{dec->p_n, dec->p_ahi, dec->p_alo};
                launch_ok(dec, nk::rmsnorm_rows(dec->p_x + (size_t)r0 * d, m->dp(m->norm_f), m->cfg.eps, nrm.out(t_lg),
                                                rr, d, dec->stream),
                          "rmsnorm");
                project(dec, t_lg, nrm, rr, d, m->dp(m->emb), w_lg, (int)V, nullptr, d_lg, nullptr);
                launch_ok(dec, nk::softmax_ce_rows(d_lg, rr, (int)V, r0, tcc, (int)t, (int)t0, d_tg, d_nll, d_cnt,
                                                   dec->err, dec->stream),
                          "softmax_ce");
                if (logits_out) {
                    // Rows of one stream are consecutive positions: one copy per run.
                    for (int r = 0; r < rr;) {
                        const int g = r0 + r, s = g / tcc, tt = g - s * tcc;
                        const int run = std::min(rr - r, tcc - tt);
                        cuda_check(cudaMemcpyAsync(logits_out + ((size_t)s * t + t0 + tt) * V, d_lg + (size_t)r * V,
                                                   (size_t)run * V * sizeof(float), cudaMemcpyDeviceToHost, dec->stream),
                                   "download logits");
                        r += run;
                    }
                }
            }
        };
        prefill_device(dec, dec->p_ids, dec->p_lens, lv, t, nullptr, per_chunk);
        launch_ok(dec, nk::ce_mean(d_nll, d_cnt, n, d_loss, dec->stream), "loss mean");
        cuda_check(cudaMemcpyAsync(loss_out, d_loss, sizeof(float), cudaMemcpyDeviceToHost, dec->stream), "download loss");
        check_err_flag(dec);
    });
    nk_decoder_destroy(tmp);
    return st;
}

nk_status nk_decoder_sample(nk_decoder *dec, const nk_sample_cfg *cfg, const uint32_t *history,
                            const uint32_t *history_len, uint32_t history_stride, uint64_t *rng_state,
                            uint32_t *out_tokens) {
    return guard([&] {
        if (!dec || !cfg || !rng_state || !out_tokens) fail(NK_ERR_INVALID, "null argument");
        ensure_ready(dec);
        ensure_sample_ws(dec, to_params(*cfg));
        const bool use_hist = history && history_len && history_stride > 0;
        if (use_hist) {
            for (uint32_t s = 0; s < dec->S; ++s)
                if (history_len[s] > history_stride) fail(NK_ERR_INVALID, "history length exceeds its stride");
            ensure_history(dec, history_stride);
            cuda_check(cudaMemcpyAsync(dec->hist, history, (size_t)dec->S * history_stride * sizeof(uint32_t),
                                       cudaMemcpyHostToDevice, dec->stream), "upload history");
            cuda_check(cudaMemcpyAsync(dec->hist_len, history_len, dec->S * sizeof(uint32_t),
                                       cudaMemcpyHostToDevice, dec->stream), "upload history lengths");
        }
        cuda_check(cudaMemcpyAsync(dec->rng, rng_state, (size_t)dec->S * 4 * sizeof(uint64_t),
                                   cudaMemcpyHostToDevice, dec->stream), "upload rng");
        SampScope prof(dec);
        launch_ok(dec, nk::sample_rows(dec->logits, (int)dec->S, (int)dec->model->cfg.vocab, to_params(*cfg),
                                       use_hist ? dec->hist : nullptr, use_hist ? dec->hist_len : nullptr,
                                       (int)history_stride, dec->rng, dec->tok_b, dec->err, dec->samp_ws,
                                       dec->samp_ws_bytes, dec->stream),
                  "sample");
        cuda_check(cudaMemcpyAsync(out_tokens, dec->tok_b, dec->S * sizeof(uint32_t), cudaMemcpyDeviceToHost,
                                   dec->stream), "download tokens");
        cuda_check(cudaMemcpyAsync(rng_state, dec->rng, (size_t)dec->S * 4 * sizeof(uint64_t),
                                   cudaMemcpyDeviceToHost, dec->stream), "download rng");
        check_err_flag(dec);
    });
}

nk_status nk_decoder_generate(nk_decoder *dec, const uint32_t *ids, const uint32_t *lens, uint32_t max_t,
                              uint32_t n_new, const nk_sample_cfg *cfg, uint64_t *rng_state,
                              uint32_t *out_tokens) {
    return guard([&] {
        if (!dec || !lens || !cfg || !rng_state || (n_new && !out_tokens) || (!ids && max_t))
            fail(NK_ERR_INVALID, "null argument");
        const uint32_t S = dec->S;
        // An empty prompt becomes the newline byte token (cli.rs:474-476).
        const uint32_t mt = std::max<uint32_t>(max_t, 1);
        std::vector<uint32_t> pid((size_t)S * mt, 0), plen(S);
        for (uint32_t s = 0; s < S; ++s) {
            if (lens[s] > max_t) fail(NK_ERR_INVALID, "prompt length exceeds max_t");
            if (lens[s] == 0) {
                if (10 >= dec->model->cfg.vocab) fail(NK_ERR_INVALID, "streaming token is outside the vocabulary");
                pid[(size_t)s * mt] = 10;
                plen[s] = 1;
            } else {
                std::memcpy(&pid[(size_t)s * mt], ids + (size_t)s * max_t, lens[s] * sizeof(uint32_t));
                plen[s] = lens[s];
            }
            validate_tokens(dec->model, &pid[(size_t)s * mt], plen[s]);
        }
        ensure_ready(dec);
        upload_prompts(dec, pid.data(), plen.data(), mt);
        prefill_device(dec, dec->p_ids, dec->p_lens, plen, mt, nullptr);
        // History = the last rep_window prompt ids (cli.rs:484-486).
        const uint32_t W = (uint32_t)std::min<uint64_t>(cfg->rep_window, 1u << 20);
        const bool use_hist = W > 0 && std::isfinite(cfg->rep_penalty) && cfg->rep_penalty > 1.0f;
        if (W > 0) {
            ensure_history(dec, W);
            std::vector<uint32_t> h((size_t)S * W, 0), hl(S);
            for (uint32_t s = 0; s < S; ++s) {
                const uint32_t n = plen[s], st = n > W ? n - W : 0;
                hl[s] = n - st;
                std::memcpy(&h[(size_t)s * W], &pid[(size_t)s * mt + st], hl[s] * sizeof(uint32_t));
            }
            cuda_check(cudaMemcpyAsync(dec->hist, h.data(), h.size() * sizeof(uint32_t), cudaMemcpyHostToDevice, dec->stream), "upload history");
            cuda_check(cudaMemcpyAsync(dec->hist_len, hl.data(), S * sizeof(uint32_t), cudaMemcpyHostToDevice, dec->stream), "upload history");
            cuda_check(cudaStreamSynchronize(dec->stream), "sync");
        }
        cuda_check(cudaMemcpyAsync(dec->rng, rng_state, (size_t)S * 4 * sizeof(uint64_t), cudaMemcpyHostToDevice,
                                   dec->stream), "upload rng");
        uint32_t *d_out = nullptr;
        dalloc(&d_out, (size_t)S * std::max<uint32_t>(n_new, 1), "generated tokens");
        std::unique_ptr<uint32_t, void (*)(uint32_t *)> own(d_out, [](uint32_t *p) { cudaFree(p); });
        const nk::SampleParams sp = to_params(*cfg);
        ensure_sample_ws(dec, sp);
        const int V = (int)dec->model->cfg.vocab;
        // Greedy without a penalty is the argmax of the logits: those steps
        // end in the projection's argmax epilogue (logits never stored) and
        // replay from a CUDA graph.  Sampled steps end in the projection's
        // sampling epilogue (penalty and temperature applied, row maxima and
        // +inf counts per part) whenever the tensor cores run the logits.
        // Engine bit 11 keeps the plain step + sampler for comparison.
        const bool unfused = (dec->engine & 2048) != 0;
        const bool greedy_fast = cfg->greedy && !use_hist && !unfused;
        if (!cfg->greedy && !unfused) {
            const size_t parts = (size_t)nk::tc_argmax_parts(V, 128);  // the most any tile width gives
            if (dec->prep_cap < (size_t)S * parts) {
                cuda_check(cudaStreamSynchronize(dec->stream), "cudaStreamSynchronize");
                for (void *q : {(void *)dec->prep_max, (void *)dec->prep_pinf})
                    if (q) cudaFree(q);
                dec->prep_max = nullptr;
                dec->prep_pinf = nullptr;
                dalloc(&dec->prep_max, (size_t)S * parts, "sampling epilogue maxima");
                dalloc(&dec->prep_pinf, (size_t)S * parts, "sampling epilogue +inf counts");
                dec->prep_cap = (size_t)S * parts;
            }
            if (use_hist && !dec->pen_bits) dalloc(&dec->pen_bits, (size_t)S * ((V + 31) / 32), "penalty bitmap");
        }
        int prep_parts = 0;  // parts of the last step's sampling epilogue (0: plain logits)
        uint32_t *tok = dec->tok_b, *spare = dec->tok_a;
        int *d_col = nullptr;  // the output column collect_tokens writes next
        dalloc(&d_col, 1, "token column");
        std::unique_ptr<int, void (*)(int *)> own_col(d_col, [](int *p) { cudaFree(p); });
        cuda_check(cudaMemsetAsync(d_col, 0, sizeof(int), dec->stream), "clear token column");
        // One token of every stream: draw (except on greedy argmax steps,
        // whose token the previous step's epilogue already chose), collect,
        // history, then the step that produces the next logits.  `direct`
        // launches the step's kernels without the decoder's own step graphs
        // (inside a capture).
        auto iteration = [&](bool draw, bool step, bool direct) {
            if (draw) {
                SampScope prof(dec);
                const nk::SamplePrepared prep{dec->prep_max, dec->prep_pinf, prep_parts};
                launch_ok(dec, nk::sample_rows(dec->logits, (int)S, V, sp, use_hist ? dec->hist : nullptr,
                                               use_hist ? dec->hist_len : nullptr, (int)W, dec->rng, tok, dec->err,
                                               dec->samp_ws, dec->samp_ws_bytes, dec->stream,
                                               prep_parts ? &prep : nullptr),
                          "sample");
            }
            launch_ok(dec, nk::collect_tokens(tok, d_out, (int)S, (int)n_new, d_col, dec->stream), "collect tokens", 2);
            if (W > 0) launch_ok(dec, nk::history_push(dec->hist, dec->hist_len, tok, (int)S, (int)W, dec->stream), "history");
            if (!step) return;
            if (greedy_fast) {
                if (direct) eager_step(dec, tok, false, spare);
                else step_device(dec, tok, false, spare);
                std::swap(tok, spare);
                return;
            }
            if (!cfg->greedy && !unfused) {
                dec->fuse_penalty = use_hist;
                if (use_hist)
                    launch_ok(dec, nk::sample_pen_bitmap(dec->hist, dec->hist_len, (int)W, sp, (int)S, V, dec->pen_bits,
                                                         (V + 31) / 32, dec->stream),
                              "penalty bitmap");
                dec->fuse_sample = &sp;
                try {
                    direct ? eager_step(dec, tok, true, nullptr) : step_device(dec, tok, true, nullptr);
                } catch (...) {
                    dec->fuse_sample = nullptr;
                    throw;
                }
                dec->fuse_sample = nullptr;
                prep_parts = dec->fused_parts;
            } else {
                direct ? eager_step(dec, tok, true, nullptr) : step_device(dec, tok, true, nullptr);
            }
        };
        // The middle iterations are identical launch sequences: from the
        // third on they replay a CUDA graph of one iteration (two for greedy
        // argmax steps, whose token buffers alternate), so the host launch
        // cost of the ~30 kernels of a step is paid once.  Profiled calls run
        // eagerly.
        struct BodyGraph {
            uint32_t *tok;
            cudaGraphExec_t exec;
            uint64_t launches;
        };
        struct Bodies {
            cudaStream_t st;
            std::vector<BodyGraph> v;
            ~Bodies() {
                if (v.empty()) return;
                cudaStreamSynchronize(st);
                for (auto &b : v) cudaGraphExecDestroy(b.exec);
            }
        } bodies_guard{dec->stream, {}};
        std::vector<BodyGraph> &bodies = bodies_guard.v;
        {
            for (uint32_t gi = 0; gi < n_new; ++gi) {
                const bool draw = gi == 0 || !greedy_fast, step = gi + 1 < n_new;
                if (gi < 2 || !step || dec->profiling) {
                    iteration(draw, step, false);
                    continue;
                }
                BodyGraph *bg = nullptr;
                for (auto &b : bodies)
                    if (b.tok == tok) bg = &b;
                if (!bg) {
                    uint32_t *tok0 = tok;
                    const uint64_t before = dec->launches;
                    cudaGraph_t graph = nullptr;
                    cuda_check(cudaStreamBeginCapture(dec->stream, cudaStreamCaptureModeThreadLocal),
                               "cudaStreamBeginCapture");
                    try {
                        iteration(draw, step, true);
                    } catch (...) {
                        cudaStreamEndCapture(dec->stream, &graph);
                        if (graph) cudaGraphDestroy(graph);
                        cudaGetLastError();
                        throw;
                    }
                    cuda_check(cudaStreamEndCapture(dec->stream, &graph), "cudaStreamEndCapture");
                    cudaGraphExec_t exec = nullptr;
                    cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
                    cudaGraphDestroy(graph);
                    cuda_check(e, "cudaGraphInstantiate");
                    bodies.push_back({tok0, exec, dec->launches - before});
                    cuda_check(cudaGraphLaunch(exec, dec->stream), "cudaGraphLaunch");
                    continue;
                }
                cuda_check(cudaGraphLaunch(bg->exec, dec->stream), "cudaGraphLaunch");
                dec->launches += bg->launches;
                if (greedy_fast) std::swap(tok, spare);
            }
        }
        if (n_new)
            cuda_check(cudaMemcpyAsync(out_tokens, d_out, (size_t)S * n_new * sizeof(uint32_t), cudaMemcpyDeviceToHost,
                                       dec->stream), "download tokens");
        cuda_check(cudaMemcpyAsync(rng_state, dec->rng, (size_t)S * 4 * sizeof(uint64_t), cudaMemcpyDeviceToHost,
                                   dec->stream), "download rng");
        check_err_flag(dec);
    });
}

nk_status nk_decoder_get_state(nk_decoder *dec, uint32_t first, uint32_t count, float *state, uint32_t *heads) {
    return guard([&] {
        if (!dec || !state) fail(NK_ERR_INVALID, "null argument");
        if ((uint64_t)first + count > dec->S) fail(NK_ERR_INVALID, "stream range out of bounds");
        cuda_check(cudaSetDevice(dec->model->device), "cudaSetDevice");
        const size_t per = (dec->model->k() + 1) * dec->model->e();
        for (uint64_t l = 0; l < dec->L(); ++l)
            cuda_check(cudaMemcpy2DAsync(state + l * per, dec->L() * per * sizeof(float),
                                         dec->layer_state(l) + (size_t)first * per, per * sizeof(float),
                                         per * sizeof(float), count, cudaMemcpyDeviceToHost, dec->stream),
                       "download state");
        if (heads)
            cuda_check(cudaMemcpyAsync(heads, dec->heads + first, count * sizeof(uint32_t), cudaMemcpyDeviceToHost,
                                       dec->stream), "download heads");
        cuda_check(cudaStreamSynchronize(dec->stream), "cudaStreamSynchronize");
    });
}

nk_status nk_decoder_set_state(nk_decoder *dec, uint32_t first, uint32_t count, const float *state,
                               const uint32_t *heads) {
    return guard([&] {
        if (!dec || !state || !heads) fail(NK_ERR_INVALID, "null argument");
        if ((uint64_t)first + count > dec->S) fail(NK_ERR_INVALID, "stream range out of bounds");
        const uint64_t k = dec->model->k();
        std::vector<uint32_t> hv(heads, heads + count);
        for (auto &h : hv)
            if (h >= k) fail(NK_ERR_INVALID, "conv head out of range");
        cuda_check(cudaSetDevice(dec->model->device), "cudaSetDevice");
        const size_t per = (k + 1) * dec->model->e();
        for (uint64_t l = 0; l < dec->L(); ++l)
            cuda_check(cudaMemcpy2DAsync(dec->layer_state(l) + (size_t)first * per, per * sizeof(float),
                                         state + l * per, dec->L() * per * sizeof(float), per * sizeof(float), count,
                                         cudaMemcpyHostToDevice, dec->stream),
                       "upload state");
        cuda_check(cudaMemcpyAsync(dec->heads + first, hv.data(), count * sizeof(uint32_t), cudaMemcpyHostToDevice,
                                   dec->stream), "upload heads");
        cuda_check(cudaStreamSynchronize(dec->stream), "cudaStreamSynchronize");
    });
}

nk_status nk_decoder_cuda_stream(nk_decoder *dec, void **stream) {
    return guard([&] {
        if (!dec || !stream) fail(NK_ERR_INVALID, "null argument");
        *stream = (void *)dec->stream;
    });
}

nk_status nk_decoder_sync(nk_decoder *dec) {
    return guard([&] {
        if (!dec) fail(NK_ERR_INVALID, "null decoder");
        cuda_check(cudaSetDevice(dec->model->device), "cudaSetDevice");
        check_err_flag(dec);
    });
}

nk_status nk_decoder_set_engine(nk_decoder *dec, int engine) {
    return guard([&] {
        if (!dec) fail(NK_ERR_INVALID, "null decoder");
        if (engine < 0 || engine > 1048575) fail(NK_ERR_INVALID, "unknown engine flags");
        dec->engine = engine;
        cudaSetDevice(dec->model->device);
        for (auto &gph : dec->graphs) cudaGraphExecDestroy(gph.exec);
        dec->graphs.clear();
    });
}

nk_status nk_decoder_launch_count(const nk_decoder *dec, uint64_t *count) {
    return guard([&] {
        if (!dec || !count) fail(NK_ERR_INVALID, "null argument");
        *count = dec->launches;
    });
}

nk_status nk_decoder_profile_begin(nk_decoder *dec) {
    return guard([&] {
        if (!dec) fail(NK_ERR_INVALID, "null decoder");
        dec->profiling = true;
        dec->ev_used = 0;
        dec->prof_flops = dec->prof_bytes = 0;
        dec->prof_proj = 0;
        dec->prof_tc = false;
        dec->prof_launch0 = dec->launches;
        dec->samp_used = 0;
        dec->prof_samp = 0;
    });
}

nk_status nk_decoder_profile_end(nk_decoder *dec, nk_profile *out) {
    return guard([&] {
        if (!dec || !out) fail(NK_ERR_INVALID, "null argument");
        cuda_check(cudaSetDevice(dec->model->device), "cudaSetDevice");
        cuda_check(cudaStreamSynchronize(dec->stream), "cudaStreamSynchronize");
        double ms = 0;
        for (size_t i = 0; i + 1 < dec->ev_used; i += 2) {
            float t = 0;
            cuda_check(cudaEventElapsedTime(&t, dec->ev_pool[i], dec->ev_pool[i + 1]), "cudaEventElapsedTime");
            ms += t;
        }
        double sms = 0;
        for (size_t i = 0; i + 1 < dec->samp_used; i += 2) {
            float t = 0;
            cuda_check(cudaEventElapsedTime(&t, dec->samp_ev[i], dec->samp_ev[i + 1]), "cudaEventElapsedTime");
            sms += t;
        }
        out->sample_ms = sms;
        out->sample_launches = dec->prof_samp;
        dec->samp_used = 0;
        out->proj_ms = ms;
        out->proj_launches = dec->prof_proj;
        out->proj_flops = dec->prof_flops;
        out->proj_bytes = dec->prof_bytes;
        out->launches = dec->launches - dec->prof_launch0;
        out->tensor_core = dec->prof_tc ? 1 : 0;
        dec->profiling = false;
        dec->ev_used = 0;
    });
}

namespace {
// Scratch for the synchronous stand-alone ops, kept per device between calls
// (grown on demand up to 8 GiB; larger requests allocate for the call).
// The lock is held from the request until the op has synchronised, so calls
// from several host threads take turns on it.
struct OpScratch {
    std::mutex mu;
    void *ptr = nullptr;
    size_t bytes = 0;
};
OpScratch &op_scratch(int device) {
    static std::mutex table_mu;
    static std::map<int, OpScratch *> table;
    std::lock_guard<std::mutex> g(table_mu);
    OpScratch *&e = table[device];
    if (!e) e = new OpScratch();
    return *e;
}
constexpr size_t OP_SCRATCH_CAP = size_t(8) << 30;

// Holds the device's scratch (or a private allocation) for one call.
struct ScratchLease {
    std::unique_lock<std::mutex> lock;
    void *own = nullptr;
    void *ptr = nullptr;
    ScratchLease(size_t bytes, const char *what) {
        int dev = 0;
        cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
        if (bytes > OP_SCRATCH_CAP) {
            cuda_check(cudaMalloc(&own, bytes), what);
            ptr = own;
            return;
        }
        OpScratch &sc = op_scratch(dev);
        lock = std::unique_lock<std::mutex>(sc.mu);
        if (sc.bytes < bytes) {
            if (sc.ptr) cudaFree(sc.ptr);
            sc.ptr = nullptr;
            sc.bytes = 0;
            cuda_check(cudaMalloc(&sc.ptr, bytes), what);
            sc.bytes = bytes;
        }
        ptr = sc.ptr;
    }
    ~ScratchLease() {
        if (own) cudaFree(own);
    }
};

// The time-chunked scan (or its adjoint) of nk_scan_device: the one-pass
// kernel where it suits the shape, else the three-pass form; synchronises
// the stream and reports an expired look-back wait as NK_ERR_DEVICE.
void chunked_scan(const float *a, const float *b, float *h, uint64_t batch, uint64_t t, uint64_t d, bool adjoint,
                  cudaStream_t st) {
    const int64_t B = (int64_t)batch, T = (int64_t)t, D = (int64_t)d;
    const char *what = adjoint ? "scan adjoint" : "scan";
    if (nk::scan_onepass_suits(B, T, D)) {
        ScratchLease lease(nk::scan_onepass_scratch_bytes(B, T, D), "scan scratch");
        cudaError_t e = nk::scan_onepass(a, b, h, B, T, D, adjoint, lease.ptr, st);
        cudaError_t e2 = cudaStreamSynchronize(st);
        cuda_check(e, what);
        cuda_check(e2, what);
        const int status = nk::scan_onepass_status(lease.ptr);
        if (status != 0)
            fail(NK_ERR_DEVICE, std::string(what) + ": device error code " + std::to_string(status) +
                                    " (131: a time block's look-back wait expired)");
        return;
    }
    ScratchLease lease(nk::scan_chunked_scratch_floats(B, T, D) * sizeof(float), "scan scratch");
    cudaError_t e = adjoint ? nk::scan_adjoint_chunked(a, b, h, B, T, D, (float *)lease.ptr, st)
                            : nk::scan_chunked(a, b, h, B, T, D, (float *)lease.ptr, st);
    cudaError_t e2 = cudaStreamSynchronize(st);
    cuda_check(e, what);
    cuda_check(e2, what);
}
}  // namespace

nk_status nk_scan_device(const float *a, const float *b, float *h, uint64_t batch, uint64_t t, uint64_t d,
                         int chunked, void *stream) {
    return guard([&] {
        uint64_t n = 0;
        if (!nk::scan_elements(batch, t, d, n)) fail(NK_ERR_INVALID, "scan shape too large: batch * t * d is limited to 2^37 elements");
        if (n == 0) return;
        if (!a || !b || !h) fail(NK_ERR_INVALID, "null argument");
        cudaStream_t st = (cudaStream_t)stream;
        if (!chunked) {
            cuda_check(nk::scan_sequential(a, b, h, (int64_t)batch, (int64_t)t, (int64_t)d, st), "scan");
            return;
        }
        chunked_scan(a, b, h, batch, t, d, false, st);
    });
}

nk_status nk_scan_adjoint_device(const float *a, const float *g, float *c, uint64_t batch, uint64_t t, uint64_t d,
                                 int chunked, void *stream) {
    return guard([&] {
        uint64_t n = 0;
        if (!nk::scan_elements(batch, t, d, n)) fail(NK_ERR_INVALID, "scan shape too large: batch * t * d is limited to 2^37 elements");
        if (n == 0) return;
        if (!a || !g || !c) fail(NK_ERR_INVALID, "null argument");
        cudaStream_t st = (cudaStream_t)stream;
        if (!chunked) {
            cuda_check(nk::scan_adjoint_sequential(a, g, c, (int64_t)batch, (int64_t)t, (int64_t)d, st), "scan adjoint");
            return;
        }
        chunked_scan(a, g, c, batch, t, d, true, st);
    });
}

// ---------------------------------------------------------------- training-side ops


nk_status nk_gemm_tn_device(const float *a, const float *b, float *c, uint64_t p, uint64_t m, uint64_t n,
                            void *stream) {
    return guard([&] {
        if (m == 0 || n == 0) return;
        if (!c || (p && (!a || !b))) fail(NK_ERR_INVALID, "null argument");
        uint64_t pm = 0, pn = 0, mn = 0;
        if (m >= (1ull << 22) || n >= (1ull << 31) || !nk::checked_mul(p, m, pm) || !nk::checked_mul(p, n, pn) ||
            !nk::checked_mul(m, n, mn))
            fail(NK_ERR_INVALID, "gemm_tn shape too large: m < 2^22, n < 2^31, p*m, p*n, m*n <= 2^37");
        cudaStream_t st = (cudaStream_t)stream;
        if (!nk::gemm_tn_tc_eligible((int64_t)p, (int)m, (int)n)) {
            cuda_check(nk::gemm_tn(a, b, c, (int64_t)p, (int)m, (int)n, st), "gemm_tn");
            return;
        }
        const int nflags = nk::gemm_tn_tc_flag_ints();
        const size_t fbytes = ((size_t)nflags * sizeof(int) + 255) & ~size_t(255);
        ScratchLease lease(fbytes + nk::gemm_tn_tc_scratch_floats((int64_t)p, (int)m, (int)n) * sizeof(float),
                           "gemm_tn operands");
        int *flags = (int *)lease.ptr;
        float *scratch = (float *)((char *)lease.ptr + fbytes);
        cuda_check(cudaMemsetAsync(flags, 0, nflags * sizeof(int), st), "memset");
        cuda_check(nk::gemm_tn_tc(a, b, c, (int64_t)p, (int)m, (int)n, scratch, flags, st), "gemm_tn (tensor cores)");
        int h[2] = {0, 0};
        cuda_check(cudaMemcpyAsync(h, flags, sizeof(h), cudaMemcpyDeviceToHost, st), "read gemm_tn flags");
        cuda_check(cudaStreamSynchronize(st), "gemm_tn sync");
        if (h[1]) fail(NK_ERR_DEVICE, "gemm_tn: a tensor-core pipeline wait expired (code " + std::to_string(h[1]) + ")");
    });
}

nk_status nk_gemm_tn(const float *a, const float *b, float *c, uint64_t p, uint64_t m, uint64_t n, int device) {
    return guard([&] {
        if (m == 0 || n == 0) return;
        if (!c || (p && (!a || !b))) fail(NK_ERR_INVALID, "null argument");
        uint64_t pm = 0, pn = 0, mn = 0;
        if (m >= (1ull << 22) || n >= (1ull << 31) || !nk::checked_mul(p, m, pm) || !nk::checked_mul(p, n, pn) ||
            !nk::checked_mul(m, n, mn))
            fail(NK_ERR_INVALID, "gemm_tn shape too large: m < 2^22, n < 2^31, p*m, p*n, m*n <= 2^37");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        float *da = nullptr, *db = nullptr, *dc = nullptr;
        dalloc(&da, p * m, "gemm_tn a");
        std::unique_ptr<float, void (*)(float *)> oa(da, [](float *q) { cudaFree(q); });
        dalloc(&db, p * n, "gemm_tn b");
        std::unique_ptr<float, void (*)(float *)> ob(db, [](float *q) { cudaFree(q); });
        dalloc(&dc, m * n, "gemm_tn c");
        std::unique_ptr<float, void (*)(float *)> oc(dc, [](float *q) { cudaFree(q); });
        if (p) {
            cuda_check(cudaMemcpy(da, a, p * m * 4, cudaMemcpyHostToDevice), "upload a");
            cuda_check(cudaMemcpy(db, b, p * n * 4, cudaMemcpyHostToDevice), "upload b");
        }
        nk_status st = nk_gemm_tn_device(da, db, dc, p, m, n, nullptr);
        if (st != NK_OK) fail(st, g_err);
        cuda_check(cudaMemcpy(c, dc, m * n * 4, cudaMemcpyDeviceToHost), "download c");
    });
}

nk_status nk_dwconv_backward_device(const float *x, const float *w, const float *go, float *gx, float *gw,
                                    float *gb, uint64_t batch, uint64_t t, uint64_t d, uint64_t k, void *stream) {
    return guard([&] {
        if (d == 0 || k == 0) fail(NK_ERR_INVALID, "dwconv: width and kernel width must be positive");
        if (k > (uint64_t)nk::dwconv_max_k()) fail(NK_ERR_INVALID, "dwconv backward: kernel width above 16");
        if (d >= (1ull << 21)) fail(NK_ERR_INVALID, "dwconv backward: width too large");
        uint64_t rows = 0, elems = 0;
        if (!nk::checked_mul(batch, t, rows) || !nk::checked_mul(rows, d, elems))
            fail(NK_ERR_INVALID, "dwconv backward: batch * t * d is limited to 2^37 elements");
        if (rows == 0 || (!gx && !gw && !gb)) return;
        if (!go || (gx && !w) || (gw && !x)) fail(NK_ERR_INVALID, "null argument");
        cudaStream_t st = (cudaStream_t)stream;
        std::unique_ptr<ScratchLease> lease;
        if (gw || gb)
            lease.reset(new ScratchLease(nk::dwconv_backward_scratch_floats((int64_t)rows, (int)d, (int)k) * sizeof(float),
                                         "dwconv scratch"));
        float *scratch = lease ? (float *)lease->ptr : nullptr;
        cudaError_t e = nk::dwconv_backward(x, w, go, gx, gw, gb, (int64_t)batch, (int64_t)t, (int)d, (int)k, scratch, st);
        cudaError_t e2 = scratch ? cudaStreamSynchronize(st) : cudaSuccess;
        cuda_check(e, "dwconv backward");
        cuda_check(e2, "dwconv backward sync");
    });
}

nk_status nk_dwconv_backward(const float *x, const float *w, const float *go, float *gx, float *gw, float *gb,
                             uint64_t batch, uint64_t t, uint64_t d, uint64_t k, int device) {
    return guard([&] {
        if (d == 0 || k == 0) fail(NK_ERR_INVALID, "dwconv: width and kernel width must be positive");
        if (k > (uint64_t)nk::dwconv_max_k()) fail(NK_ERR_INVALID, "dwconv backward: kernel width above 16");
        if (d >= (1ull << 21)) fail(NK_ERR_INVALID, "dwconv backward: width too large");
        uint64_t n = 0;
        if (!nk::scan_elements(batch, t, d, n))
            fail(NK_ERR_INVALID, "dwconv backward: batch * t * d is limited to 2^37 elements");
        if (n == 0 || (!gx && !gw && !gb)) return;
        if (!go || (gx && !w) || (gw && !x)) fail(NK_ERR_INVALID, "null argument");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        std::vector<std::unique_ptr<float, void (*)(float *)>> own;
        auto up = [&](const float *h, size_t cnt, const char *what) -> float * {
            if (!h) return nullptr;
            float *dp = nullptr;
            dalloc(&dp, cnt, what);
            own.emplace_back(dp, [](float *q) { cudaFree(q); });
            cuda_check(cudaMemcpy(dp, h, cnt * 4, cudaMemcpyHostToDevice), what);
            return dp;
        };
        float *dx = gw ? up(x, n, "dwconv x") : nullptr;
        float *dw = gx ? up(w, k * d, "dwconv w") : nullptr;
        float *dgo = up(go, n, "dwconv go");
        float *dgx = up(gx, n, "dwconv gx"), *dgw = up(gw, k * d, "dwconv gw"), *dgb = up(gb, d, "dwconv gb");
        nk_status st = nk_dwconv_backward_device(dx, dw, dgo, dgx, dgw, dgb, batch, t, d, k, nullptr);
        if (st != NK_OK) fail(st, g_err);
        if (gx) cuda_check(cudaMemcpy(gx, dgx, n * 4, cudaMemcpyDeviceToHost), "download gx");
        if (gw) cuda_check(cudaMemcpy(gw, dgw, k * d * 4, cudaMemcpyDeviceToHost), "download gw");
        if (gb) cuda_check(cudaMemcpy(gb, dgb, d * 4, cudaMemcpyDeviceToHost), "download gb");
    });
}

namespace {
// AdamW::step's checks and bias corrections (optim.rs:35-47), on the host.
nk::AdamwParams adamw_params(const nk_adamw_cfg *cfg) {
    if (!cfg) fail(NK_ERR_INVALID, "null AdamW configuration");
    const nk_adamw_cfg &c = *cfg;
    if (!(std::isfinite(c.lr) && c.lr >= 0.0f)) fail(NK_ERR_INVALID, "AdamW learning rate must be finite and non-negative");
    if (!(std::isfinite(c.b1) && c.b1 >= 0.0f && c.b1 < 1.0f)) fail(NK_ERR_INVALID, "AdamW beta1 must be in [0, 1)");
    if (!(std::isfinite(c.b2) && c.b2 >= 0.0f && c.b2 < 1.0f)) fail(NK_ERR_INVALID, "AdamW beta2 must be in [0, 1)");
    if (!(std::isfinite(c.eps) && c.eps > 0.0f)) fail(NK_ERR_INVALID, "AdamW epsilon must be finite and positive");
    if (!(std::isfinite(c.wd) && c.wd >= 0.0f)) fail(NK_ERR_INVALID, "AdamW weight decay must be finite and non-negative");
    if (c.t == 0) fail(NK_ERR_INVALID, "AdamW step counter must be at least 1");
    const float tf = (float)c.t;
    const float bc1 = 1.0f - powf(c.b1, tf), bc2 = 1.0f - powf(c.b2, tf);
    return nk::AdamwParams{c.lr, c.b1, c.b2, c.eps, c.wd, 1.0f / bc1, 1.0f / bc2, c.decay ? 1 : 0};
}
}  // namespace

nk_status nk_adamw_step_device(float *val, const float *grad, float *m, float *v, uint64_t n,
                               const nk_adamw_cfg *cfg, void *stream) {
    return guard([&] {
        const nk::AdamwParams a = adamw_params(cfg);
        if (n > nk::MAX_ELEMENTS) fail(NK_ERR_INVALID, "AdamW: n is limited to 2^37 parameters per call");
        if (n == 0) return;
        if (!val || !grad || !m || !v) fail(NK_ERR_INVALID, "null argument");
        cudaStream_t st = (cudaStream_t)stream;
        ScratchLease lease(sizeof(int), "error flag");
        int *de = (int *)lease.ptr;
        cuda_check(cudaMemsetAsync(de, 0, sizeof(int), st), "memset");
        cuda_check(nk::adamw_step(val, grad, m, v, (int64_t)n, a, de, st), "adamw");
        int e = 0;
        cuda_check(cudaMemcpyAsync(&e, de, sizeof(int), cudaMemcpyDeviceToHost, st), "download error flag");
        cuda_check(cudaStreamSynchronize(st), "adamw sync");
        if (e) fail(NK_ERR_INVALID, "AdamW received a non-finite gradient or parameter");
    });
}

nk_status nk_adamw_step(float *val, const float *grad, float *m, float *v, uint64_t n, const nk_adamw_cfg *cfg,
                        int device) {
    return guard([&] {
        adamw_params(cfg);
        if (n > nk::MAX_ELEMENTS) fail(NK_ERR_INVALID, "AdamW: n is limited to 2^37 parameters per call");
        if (n == 0) return;
        if (!val || !grad || !m || !v) fail(NK_ERR_INVALID, "null argument");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        float *dv = nullptr, *dg = nullptr, *dm = nullptr, *dvv = nullptr;
        dalloc(&dv, n, "adamw val");
        std::unique_ptr<float, void (*)(float *)> o1(dv, [](float *q) { cudaFree(q); });
        dalloc(&dg, n, "adamw grad");
        std::unique_ptr<float, void (*)(float *)> o2(dg, [](float *q) { cudaFree(q); });
        dalloc(&dm, n, "adamw m");
        std::unique_ptr<float, void (*)(float *)> o3(dm, [](float *q) { cudaFree(q); });
        dalloc(&dvv, n, "adamw v");
        std::unique_ptr<float, void (*)(float *)> o4(dvv, [](float *q) { cudaFree(q); });
        cuda_check(cudaMemcpy(dv, val, n * 4, cudaMemcpyHostToDevice), "upload val");
        cuda_check(cudaMemcpy(dg, grad, n * 4, cudaMemcpyHostToDevice), "upload grad");
        cuda_check(cudaMemcpy(dm, m, n * 4, cudaMemcpyHostToDevice), "upload m");
        cuda_check(cudaMemcpy(dvv, v, n * 4, cudaMemcpyHostToDevice), "upload v");
        const nk_status st = nk_adamw_step_device(dv, dg, dm, dvv, n, cfg, nullptr);
        // Copy back what the kernel wrote even after a non-finite element,
        // then report it.
        const std::string msg = st != NK_OK ? g_err : std::string();
        cuda_check(cudaMemcpy(val, dv, n * 4, cudaMemcpyDeviceToHost), "download val");
        cuda_check(cudaMemcpy(m, dm, n * 4, cudaMemcpyDeviceToHost), "download m");
        cuda_check(cudaMemcpy(v, dvv, n * 4, cudaMemcpyDeviceToHost), "download v");
        if (st != NK_OK) fail(st, msg);
    });
}

nk_status nk_scan_adjoint(const float *a, const float *g, float *c, uint64_t batch, uint64_t t, uint64_t d,
                          int chunked, int device) {
    return guard([&] {
        uint64_t n = 0;
        if (!nk::scan_elements(batch, t, d, n)) fail(NK_ERR_INVALID, "scan shape too large: batch * t * d is limited to 2^37 elements");
        if (n == 0) return;
        if (!a || !g || !c) fail(NK_ERR_INVALID, "null argument");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        float *da = nullptr, *dg = nullptr, *dc = nullptr;
        dalloc(&da, n, "adjoint a");
        std::unique_ptr<float, void (*)(float *)> oa(da, [](float *p) { cudaFree(p); });
        dalloc(&dg, n, "adjoint g");
        std::unique_ptr<float, void (*)(float *)> og(dg, [](float *p) { cudaFree(p); });
        dalloc(&dc, n, "adjoint c");
        std::unique_ptr<float, void (*)(float *)> oc(dc, [](float *p) { cudaFree(p); });
        cuda_check(cudaMemcpy(da, a, n * 4, cudaMemcpyHostToDevice), "upload a");
        cuda_check(cudaMemcpy(dg, g, n * 4, cudaMemcpyHostToDevice), "upload g");
        nk_status s = nk_scan_adjoint_device(da, dg, dc, batch, t, d, chunked, nullptr);
        if (s != NK_OK) fail(s, g_err);
        cuda_check(cudaMemcpy(c, dc, n * 4, cudaMemcpyDeviceToHost), "download c");
    });
}

nk_status nk_scan(const float *a, const float *b, float *h, uint64_t batch, uint64_t t, uint64_t d,
                  int chunked, int device) {
    return guard([&] {
        uint64_t n = 0;
        if (!nk::scan_elements(batch, t, d, n)) fail(NK_ERR_INVALID, "scan shape too large: batch * t * d is limited to 2^37 elements");
        if (n == 0) return;
        if (!a || !b || !h) fail(NK_ERR_INVALID, "null argument");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        float *da = nullptr, *db = nullptr, *dh = nullptr;
        dalloc(&da, n, "scan a");
        std::unique_ptr<float, void (*)(float *)> oa(da, [](float *p) { cudaFree(p); });
        dalloc(&db, n, "scan b");
        std::unique_ptr<float, void (*)(float *)> ob(db, [](float *p) { cudaFree(p); });
        dalloc(&dh, n, "scan h");
        std::unique_ptr<float, void (*)(float *)> oh(dh, [](float *p) { cudaFree(p); });
        cuda_check(cudaMemcpy(da, a, n * 4, cudaMemcpyHostToDevice), "upload a");
        cuda_check(cudaMemcpy(db, b, n * 4, cudaMemcpyHostToDevice), "upload b");
        nk_status s = nk_scan_device(da, db, dh, batch, t, d, chunked, nullptr);
        if (s != NK_OK) fail(s, g_err);
        cuda_check(cudaMemcpy(h, dh, n * 4, cudaMemcpyDeviceToHost), "download h");
    });
}

nk_status nk_sample_token(float *logits, uint64_t vocab, const nk_sample_cfg *cfg, const uint32_t *history,
                          uint64_t n_history, uint64_t *rng_state, uint32_t *out_token, int device) {
    return guard([&] {
        if (!logits || !cfg || !rng_state || !out_token || (n_history && !history)) fail(NK_ERR_INVALID, "null argument");
        if (vocab == 0) fail(NK_ERR_INVALID, "cannot sample from an empty vocabulary");
        if (vocab > (1u << 30)) fail(NK_ERR_UNSUPPORTED, "vocabulary too large");
        cuda_check(cudaSetDevice(device), "cudaSetDevice");
        const size_t ws_bytes = nk::sample_ws_bytes(1, (int)vocab, to_params(*cfg));
        void *dws = nullptr;
        if (ws_bytes) cuda_check(cudaMalloc(&dws, ws_bytes), "cudaMalloc(sampler scratch)");
        std::unique_ptr<void, void (*)(void *)> o0(dws, [](void *p) { if (p) cudaFree(p); });
        float *dl = nullptr;
        uint64_t *dr = nullptr;
        uint32_t *dh = nullptr, *dhl = nullptr, *dt = nullptr;
        int *de = nullptr;
        dalloc(&dl, vocab, "logits");
        std::unique_ptr<float, void (*)(float *)> o1(dl, [](float *p) { cudaFree(p); });
        dalloc(&dr, 4, "rng");
        std::unique_ptr<uint64_t, void (*)(uint64_t *)> o2(dr, [](uint64_t *p) { cudaFree(p); });
        dalloc(&dh, std::max<uint64_t>(n_history, 1), "history");
        std::unique_ptr<uint32_t, void (*)(uint32_t *)> o3(dh, [](uint32_t *p) { cudaFree(p); });
        dalloc(&dhl, 1, "history length");
        std::unique_ptr<uint32_t, void (*)(uint32_t *)> o4(dhl, [](uint32_t *p) { cudaFree(p); });
        dalloc(&dt, 1, "token");
        std::unique_ptr<uint32_t, void (*)(uint32_t *)> o5(dt, [](uint32_t *p) { cudaFree(p); });
        dalloc(&de, 1, "error flag");
        std::unique_ptr<int, void (*)(int *)> o6(de, [](int *p) { cudaFree(p); });
        const uint32_t hl = (uint32_t)n_history;
        cuda_check(cudaMemcpy(dl, logits, vocab * 4, cudaMemcpyHostToDevice), "upload logits");
        cuda_check(cudaMemcpy(dr, rng_state, 32, cudaMemcpyHostToDevice), "upload rng");
        if (n_history) cuda_check(cudaMemcpy(dh, history, n_history * 4, cudaMemcpyHostToDevice), "upload history");
        cuda_check(cudaMemcpy(dhl, &hl, 4, cudaMemcpyHostToDevice), "upload history length");
        cuda_check(cudaMemset(de, 0, 4), "memset");
        cuda_check(nk::sample_rows(dl, 1, (int)vocab, to_params(*cfg), n_history ? dh : nullptr, n_history ? dhl : nullptr,
                                   (int)std::max<uint64_t>(n_history, 1), dr, dt, de, dws, ws_bytes, nullptr),
                   "sample");
        int e = 0;
        cuda_check(cudaMemcpy(out_token, dt, 4, cudaMemcpyDeviceToHost), "download token");
        cuda_check(cudaMemcpy(rng_state, dr, 32, cudaMemcpyDeviceToHost), "download rng");
        cuda_check(cudaMemcpy(logits, dl, vocab * 4, cudaMemcpyDeviceToHost), "download logits");
        cuda_check(cudaMemcpy(&e, de, 4, cudaMemcpyDeviceToHost), "download error flag");
        if (e) fail(NK_ERR_DEVICE, "the bounded rejection draw failed");
    });
}

}  // extern "C"
