// bpe.cu -- byte-level BPE text I/O on the host (bpe.rs): the merges file
// (load / save), text and byte-buffer encoding, exact decoding.  This is the
// data format on either side of the token loop: prompts come in as ids,
// generated ids go out as bytes.  Host code only (no kernels).
//
// Encoding applies merges lowest rank first, leftmost first among equal
// ranks, exactly as Bpe::encode_raw (bpe.rs:222-246) does by rescanning the
// symbol list after every merge; here a heap of candidate pairs over a
// linked list gives the same merge sequence in O(n log n): a pair created by
// a merge contains the new token 256 + r, and every merge that uses that
// token has a rank above r, so no pending candidate is ever overtaken.

#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <memory>
#include <queue>
#include <sstream>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#include <unistd.h>

#include "noetic_gpu.h"
#include "nk_kernels.h"

namespace {

#include "unicode_alpha.inc"

constexpr uint64_t MAX_TOKENIZER_FILE_BYTES = 64ull << 20;  // bpe.rs:15-18
constexpr uint64_t MAX_SERIALIZED_MERGES = 1000000;
constexpr uint64_t MAX_EXPANDED_TOKEN_BYTES = 1ull << 20;
constexpr uint64_t MAX_TOTAL_EXPANDED_BYTES = 128ull << 20;

struct BpeError {
    nk_status code;
    std::string msg;
};
[[noreturn]] void bpe_fail(nk_status code, const std::string &msg) { throw BpeError{code, msg}; }

template <class F>
nk_status bpe_guard(F &&f) {
    try {
        f();
        return NK_OK;
    } catch (const BpeError &e) {
        nk::set_last_error(e.msg);
        return e.code;
    } catch (const std::bad_alloc &) {
        nk::set_last_error("host allocation failed");
        return NK_ERR_OOM;
    } catch (const std::exception &e) {
        nk::set_last_error(e.what());
        return NK_ERR_INVALID;
    }
}

// char::is_alphabetic: the Unicode Alphabetic property.
bool is_alphabetic(uint32_t c) {
    if (c < 0x80) return (c | 0x20) - 'a' < 26u;
    size_t lo = 0, hi = sizeof(kAlphabeticRanges) / sizeof(kAlphabeticRanges[0]);
    while (lo < hi) {
        const size_t mid = (lo + hi) / 2;
        if (c < kAlphabeticRanges[mid][0])
            hi = mid;
        else if (c > kAlphabeticRanges[mid][1])
            lo = mid + 1;
        else
            return true;
    }
    return false;
}

// char::is_whitespace: the Unicode White_Space property (str::trim and
// str::split_whitespace use it).
bool is_white_space(uint32_t c) {
    return (c >= 0x09 && c <= 0x0D) || c == 0x20 || c == 0x85 || c == 0xA0 || c == 0x1680 ||
           (c >= 0x2000 && c <= 0x200A) || c == 0x2028 || c == 0x2029 || c == 0x202F || c == 0x205F || c == 0x3000;
}

// Decodes one UTF-8 scalar value at s[i]; false on an invalid sequence
// (what std::str rejects: overlong forms, surrogates, values past U+10FFFF).
bool utf8_next(const uint8_t *s, size_t n, size_t &i, uint32_t &cp) {
    const uint8_t b0 = s[i];
    if (b0 < 0x80) {
        cp = b0;
        i += 1;
        return true;
    }
    int len;
    uint32_t min;
    if ((b0 & 0xE0) == 0xC0) {
        len = 2, cp = b0 & 0x1F, min = 0x80;
    } else if ((b0 & 0xF0) == 0xE0) {
        len = 3, cp = b0 & 0x0F, min = 0x800;
    } else if ((b0 & 0xF8) == 0xF0) {
        len = 4, cp = b0 & 0x07, min = 0x10000;
    } else {
        return false;
    }
    if (i + len > n) return false;
    for (int k = 1; k < len; ++k) {
        const uint8_t b = s[i + k];
        if ((b & 0xC0) != 0x80) return false;
        cp = (cp << 6) | (b & 0x3F);
    }
    if (cp < min || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF)) return false;
    i += len;
    return true;
}

}  // namespace

struct nk_bpe {
    std::vector<std::pair<uint32_t, uint32_t>> merges;  // merge i makes token 256 + i
    std::unordered_map<uint64_t, uint32_t> rank;          // (a << 32 | b) -> merge index
    std::vector<std::string> token_bytes;                 // byte expansion of every token
    uint64_t total_expanded = 256;

    nk_bpe() {
        token_bytes.reserve(256);
        for (int b = 0; b < 256; ++b) token_bytes.emplace_back(1, (char)b);
    }
    static uint64_t key(uint32_t a, uint32_t b) { return ((uint64_t)a << 32) | b; }

    // Bpe::push_merge (bpe.rs:59-75) with the loader's checks (bpe.rs:341-371).
    void push_merge(uint32_t a, uint32_t b) {
        const uint64_t next_id = token_bytes.size();
        if (a >= next_id || b >= next_id) bpe_fail(NK_ERR_IO, "tokenizer merge references an unknown token");
        if (rank.count(key(a, b))) bpe_fail(NK_ERR_IO, "tokenizer contains a duplicate merge pair");
        const uint64_t expanded = (uint64_t)token_bytes[a].size() + token_bytes[b].size();
        if (expanded > MAX_EXPANDED_TOKEN_BYTES)
            bpe_fail(NK_ERR_IO, "tokenizer contains an excessively large expanded token");
        total_expanded += expanded;
        if (total_expanded > MAX_TOTAL_EXPANDED_BYTES)
            bpe_fail(NK_ERR_IO, "tokenizer expanded vocabulary exceeds the supported size limit");
        rank.emplace(key(a, b), (uint32_t)merges.size());
        merges.emplace_back(a, b);
        token_bytes.push_back(token_bytes[a] + token_bytes[b]);
    }

    // Bpe::encode_raw (bpe.rs:222-246) on bytes [p, p + n), appended to out.
    void encode_raw(const uint8_t *p, size_t n, std::vector<uint32_t> &out) const {
        if (n == 0) return;
        if (merges.empty() || n == 1) {
            for (size_t i = 0; i < n; ++i) out.push_back(p[i]);
            return;
        }
        std::vector<uint32_t> sym(p, p + n);
        std::vector<int64_t> prev(n), next(n);
        std::vector<char> alive(n, 1);
        for (size_t i = 0; i < n; ++i) {
            prev[i] = (int64_t)i - 1;
            next[i] = i + 1 < n ? (int64_t)i + 1 : -1;
        }
        struct Cand {
            uint32_t r;
            int64_t pos;
            uint32_t a, b;
            bool operator>(const Cand &o) const { return r != o.r ? r > o.r : pos > o.pos; }
        };
        std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> heap;
        auto consider = [&](int64_t i) {
            if (i < 0) return;
            const int64_t j = next[i];
            if (j < 0) return;
            auto it = rank.find(key(sym[i], sym[j]));
            if (it != rank.end()) heap.push(Cand{it->second, i, sym[i], sym[j]});
        };
        for (size_t i = 0; i + 1 < n; ++i) consider((int64_t)i);
        while (!heap.empty()) {
            const Cand c = heap.top();
            heap.pop();
            const int64_t i = c.pos;
            if (!alive[i]) continue;
            const int64_t j = next[i];
            if (j < 0 || sym[i] != c.a || sym[j] != c.b) continue;  // stale
            sym[i] = 256u + c.r;
            alive[j] = 0;
            next[i] = next[j];
            if (next[j] >= 0) prev[next[j]] = i;
            consider(prev[i]);
            consider(i);
        }
        for (int64_t i = 0; i >= 0; i = next[i]) out.push_back(sym[i]);
    }
};

namespace {

// Bpe::pretokenize (bpe.rs:77-115) + encode_chunk over each chunk: a chunk
// is a run of one kind (alphabetic, ASCII digit; every other character its
// own chunk), and an ASCII space opens a chunk that the next character joins.
void encode_text(const nk_bpe &bpe, const uint8_t *s, size_t n, std::vector<uint32_t> &out) {
    size_t cur_begin = 0, cur_end = 0;  // current chunk [begin, end) in bytes
    int cur_kind = 0;                   // 0 none, 1 alpha, 2 digit, 3 other
    bool cur_is_space = false;          // the chunk is exactly " "
    auto flush = [&]() {
        if (cur_end > cur_begin) bpe.encode_raw(s + cur_begin, cur_end - cur_begin, out);
        cur_begin = cur_end;
    };
    size_t i = 0;
    while (i < n) {
        const size_t at = i;
        uint32_t cp;
        if (!utf8_next(s, n, i, cp)) bpe_fail(NK_ERR_INVALID, "text is not valid UTF-8");
        const int kind = is_alphabetic(cp) ? 1 : (cp >= '0' && cp <= '9') ? 2 : 3;
        if (cp == ' ') {
            flush();
            cur_begin = at;
            cur_end = i;
            cur_kind = 0;
            cur_is_space = true;
            continue;
        }
        if (cur_kind == 0 && cur_is_space) {
            cur_end = i;
            cur_kind = kind;
            cur_is_space = false;
            continue;
        }
        if (kind != cur_kind || kind == 3) {
            flush();
            cur_begin = at;
            cur_kind = kind;
        }
        cur_end = i;
        cur_is_space = false;
    }
    flush();
}

nk_status copy_ids(const std::vector<uint32_t> &ids, uint32_t *out, uint64_t cap, uint64_t *n_out) {
    *n_out = ids.size();
    if (ids.size() > cap) {
        nk::set_last_error("output buffer too small (" + std::to_string(ids.size()) + " ids needed)");
        return NK_ERR_INVALID;
    }
    if (!ids.empty()) std::memcpy(out, ids.data(), ids.size() * sizeof(uint32_t));
    return NK_OK;
}

// u32 / usize FromStr: optional '+', then decimal digits only.
bool parse_uint(const std::string &s, uint64_t max, uint64_t &v) {
    size_t i = 0;
    if (i < s.size() && s[i] == '+') ++i;
    if (i == s.size()) return false;
    v = 0;
    for (; i < s.size(); ++i) {
        if (s[i] < '0' || s[i] > '9') return false;
        const uint64_t d = (uint64_t)(s[i] - '0');
        if (v > (max - d) / 10) return false;
        v = v * 10 + d;
    }
    return true;
}

// str::split_whitespace over one line (valid UTF-8).
std::vector<std::string> split_ws(const std::string &line) {
    std::vector<std::string> out;
    const uint8_t *s = (const uint8_t *)line.data();
    size_t i = 0, start = 0;
    bool in = false;
    while (i < line.size()) {
        const size_t at = i;
        uint32_t cp;
        utf8_next(s, line.size(), i, cp);
        if (is_white_space(cp)) {
            if (in) out.push_back(line.substr(start, at - start));
            in = false;
        } else if (!in) {
            in = true;
            start = at;
        }
    }
    if (in) out.push_back(line.substr(start));
    return out;
}

}  // namespace

extern "C" {

nk_status nk_bpe_create_bytes_only(nk_bpe **out) {
    return bpe_guard([&] {
        if (!out) bpe_fail(NK_ERR_INVALID, "null argument");
        *out = new nk_bpe();
    });
}

nk_status nk_bpe_destroy(nk_bpe *bpe) {
    delete bpe;
    return NK_OK;
}

nk_status nk_bpe_vocab_size(const nk_bpe *bpe, uint64_t *out) {
    return bpe_guard([&] {
        if (!bpe || !out) bpe_fail(NK_ERR_INVALID, "null argument");
        *out = bpe->token_bytes.size();
    });
}

nk_status nk_bpe_merge(const nk_bpe *bpe, uint64_t i, uint32_t *a, uint32_t *b) {
    return bpe_guard([&] {
        if (!bpe || !a || !b) bpe_fail(NK_ERR_INVALID, "null argument");
        if (i >= bpe->merges.size()) bpe_fail(NK_ERR_INVALID, "merge index out of range");
        *a = bpe->merges[i].first;
        *b = bpe->merges[i].second;
    });
}

nk_status nk_bpe_load(const char *path, nk_bpe **out) {
    return bpe_guard([&] {
        if (!path || !out) bpe_fail(NK_ERR_INVALID, "null argument");
        *out = nullptr;
        std::ifstream f(path, std::ios::binary | std::ios::ate);
        if (!f) bpe_fail(NK_ERR_IO, std::string("cannot open ") + path + ": " + std::strerror(errno));
        const std::streamoff size = f.tellg();
        if (size < 0) bpe_fail(NK_ERR_IO, "cannot size the tokenizer file");
        if ((uint64_t)size > MAX_TOKENIZER_FILE_BYTES)
            bpe_fail(NK_ERR_IO, "tokenizer file exceeds the supported size limit");
        std::string text((size_t)size, '\0');
        f.seekg(0);
        if (size && !f.read(&text[0], size)) bpe_fail(NK_ERR_IO, "tokenizer file read failed");
        {  // read_to_string: the file must be UTF-8
            size_t i = 0;
            uint32_t cp;
            while (i < text.size())
                if (!utf8_next((const uint8_t *)text.data(), text.size(), i, cp))
                    bpe_fail(NK_ERR_IO, "stream did not contain valid UTF-8");
        }
        // str::lines: split on '\n', a '\r' before the '\n' dropped, no empty
        // last line after a trailing '\n'.
        std::vector<std::string> lines;
        size_t pos = 0;
        while (pos < text.size()) {
            size_t e = text.find('\n', pos);
            const bool nl = e != std::string::npos;
            if (!nl) e = text.size();
            std::string line = text.substr(pos, e - pos);
            if (nl && !line.empty() && line.back() == '\r') line.pop_back();
            lines.push_back(line);
            pos = nl ? e + 1 : e;
        }
        size_t li = 0;
        if (li >= lines.size() || lines[li++] != "noetic-bpe 1")
            bpe_fail(NK_ERR_IO, "unsupported tokenizer header or version");
        if (li >= lines.size()) bpe_fail(NK_ERR_IO, "tokenizer merge count is missing");
        uint64_t count = 0;
        if (!parse_uint(lines[li++], UINT64_MAX, count)) bpe_fail(NK_ERR_IO, "tokenizer merge count is invalid");
        if (count > MAX_SERIALIZED_MERGES || count > 0xFFFFFFFFull - 256)
            bpe_fail(NK_ERR_IO, "tokenizer declares too many merges");
        std::unique_ptr<nk_bpe> bpe(new nk_bpe());
        for (uint64_t m = 0; m < count; ++m) {
            if (li >= lines.size()) bpe_fail(NK_ERR_IO, "tokenizer merge list is truncated");
            const std::vector<std::string> fields = split_ws(lines[li++]);
            if (fields.size() < 1) bpe_fail(NK_ERR_IO, "tokenizer merge is missing its first token");
            uint64_t a = 0, b = 0;
            if (!parse_uint(fields[0], 0xFFFFFFFFull, a)) bpe_fail(NK_ERR_IO, "tokenizer merge token is invalid");
            if (fields.size() < 2) bpe_fail(NK_ERR_IO, "tokenizer merge is missing its second token");
            if (!parse_uint(fields[1], 0xFFFFFFFFull, b)) bpe_fail(NK_ERR_IO, "tokenizer merge token is invalid");
            if (fields.size() > 2) bpe_fail(NK_ERR_IO, "tokenizer merge has extra fields");
            bpe->push_merge((uint32_t)a, (uint32_t)b);
        }
        for (; li < lines.size(); ++li)
            if (!split_ws(lines[li]).empty()) bpe_fail(NK_ERR_IO, "tokenizer has trailing data");
        *out = bpe.release();
    });
}

// Bpe::save (bpe.rs:288-307): written to a unique temporary file, flushed,
// then renamed over the destination.
nk_status nk_bpe_save(const nk_bpe *bpe, const char *path) {
    return bpe_guard([&] {
        if (!bpe || !path) bpe_fail(NK_ERR_INVALID, "null argument");
        std::ostringstream os;
        os << "noetic-bpe 1\n" << bpe->merges.size() << "\n";
        for (const auto &m : bpe->merges) os << m.first << " " << m.second << "\n";
        const std::string body = os.str();
        const std::string tmp = std::string(path) + ".tmp." + std::to_string((long)getpid()) + "." +
                                std::to_string((unsigned long long)(uintptr_t)bpe);
        FILE *f = std::fopen(tmp.c_str(), "wbx");
        if (!f) bpe_fail(NK_ERR_IO, "cannot create " + tmp + ": " + std::strerror(errno));
        const bool ok = std::fwrite(body.data(), 1, body.size(), f) == body.size() && std::fflush(f) == 0 &&
                        fsync(fileno(f)) == 0;
        std::fclose(f);
        if (!ok || std::rename(tmp.c_str(), path) != 0) {
            std::remove(tmp.c_str());
            bpe_fail(NK_ERR_IO, std::string("cannot write ") + path);
        }
    });
}

nk_status nk_bpe_encode(const nk_bpe *bpe, const char *text, uint64_t len, uint32_t *ids, uint64_t cap,
                        uint64_t *n_out) {
    std::vector<uint32_t> out;
    const nk_status st = bpe_guard([&] {
        if (!bpe || !n_out || (len && !text) || (cap && !ids)) bpe_fail(NK_ERR_INVALID, "null argument");
        encode_text(*bpe, (const uint8_t *)text, len, out);
    });
    return st != NK_OK ? st : copy_ids(out, ids, cap, n_out);
}

nk_status nk_bpe_encode_bytes(const nk_bpe *bpe, const uint8_t *bytes, uint64_t len, uint32_t *ids, uint64_t cap,
                              uint64_t *n_out) {
    std::vector<uint32_t> out;
    const nk_status st = bpe_guard([&] {
        if (!bpe || !n_out || (len && !bytes) || (cap && !ids)) bpe_fail(NK_ERR_INVALID, "null argument");
        bpe->encode_raw(bytes, len, out);
    });
    return st != NK_OK ? st : copy_ids(out, ids, cap, n_out);
}

nk_status nk_bpe_decode_bytes(const nk_bpe *bpe, const uint32_t *ids, uint64_t n, uint8_t *out, uint64_t cap,
                              uint64_t *n_out) {
    return bpe_guard([&] {
        if (!bpe || !n_out || (n && !ids) || (cap && !out)) bpe_fail(NK_ERR_INVALID, "null argument");
        uint64_t total = 0;
        for (uint64_t i = 0; i < n; ++i) {
            if (ids[i] >= bpe->token_bytes.size()) bpe_fail(NK_ERR_INVALID, "token id out of range");
            total += bpe->token_bytes[ids[i]].size();
        }
        *n_out = total;
        if (total > cap) bpe_fail(NK_ERR_INVALID, "output buffer too small (" + std::to_string(total) + " bytes needed)");
        uint64_t o = 0;
        for (uint64_t i = 0; i < n; ++i) {
            const std::string &t = bpe->token_bytes[ids[i]];
            std::memcpy(out + o, t.data(), t.size());
            o += t.size();
        }
    });
}

}  // extern "C"
