// Reader of the reference's K50 expert pack (one directory per layer: codes.bin, scales.bf16,
// bias.bf16, index.json; mlx-qwen38/cpp/src/loader.cpp:1187-1470, record fields
// cpp/src/model.hpp:61-75). It materialises a record into the MLX affine layout the expert
// kernels and the pinned pools use: uint32 codes [rows][cols * bits / 32], bf16 scales and
// biases [rows][cols / group_size].
//
//   kind "tern"             5 base-3 digits per byte (least significant first), digit t -> 2-bit
//                           code t, 16 codes per uint32 word (lowest bits first); the bias of
//                           every group is -scale (the bf16 sign bit flipped), so the value is
//                           (t - 1) * scale. Rows of `row_bytes` (cols / 5) bytes.
//   kind "2t" "2" "3" "4"   the codes are already MLX words (code_nbytes / rows bytes per row)
//   "6" "8"                 and the biases come from bias.bf16, or are -scale when the record
//                           has no bias bytes.
//
// index.json: {"experts": {"<proj>": [record, ...], ...}, "dense": {"<name>": record, ...}, ...}
// with record = {"expert", "kind", "unit", "shape": [rows, cols], "row_bytes", "code_off",
// "code_nbytes", "scale_off", "scale_nbytes", "bias_off", "bias_nbytes", "group_size", ...};
// unknown keys and null values are skipped. The parser below is a small recursive-descent
// JSON reader for that document (no floats are needed from it).
#include <fcntl.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <exception>
#include <fstream>
#include <map>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "../../include/moe_b200.h"

int moe_set_error(int code, const char *fmt, ...);   // errors.cpp

namespace {

struct K50Rec {
    int expert = -1;
    std::string kind, unit;
    std::vector<int64_t> shape;
    int64_t row_bytes = 0, code_off = 0, code_nbytes = 0, scale_off = 0, scale_nbytes = 0, bias_off = 0,
            bias_nbytes = 0, group_size = 64;
};

// ------------------------------------------------------------------ JSON
struct Json {
    const std::string &s;
    size_t i = 0;
    bool bad = false;
    explicit Json(const std::string &t) : s(t) {}

    void ws() {
        while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
    }
    bool eat(char c) {
        ws();
        if (i < s.size() && s[i] == c) {
            ++i;
            return true;
        }
        return false;
    }
    bool peek(char c) {
        ws();
        return i < s.size() && s[i] == c;
    }
    std::string str() {
        std::string out;
        if (!eat('"')) {
            bad = true;
            return out;
        }
        while (i < s.size() && s[i] != '"') {
            if (s[i] == '\\' && i + 1 < s.size()) {
                const char e = s[i + 1];
                if (e == 'u') {              // keep \uXXXX escapes as text; keys here are ASCII
                    out += s.substr(i, 6);
                    i += 6;
                    continue;
                }
                out += (e == 'n') ? '\n' : (e == 't') ? '\t' : e;
                i += 2;
                continue;
            }
            out += s[i++];
        }
        if (i >= s.size()) bad = true;
        ++i;
        return out;
    }
    int64_t integer() {
        ws();
        size_t j = i;
        if (j < s.size() && (s[j] == '-' || s[j] == '+')) ++j;
        while (j < s.size() && s[j] >= '0' && s[j] <= '9') ++j;
        if (j == i) {
            bad = true;
            return 0;
        }
        const int64_t v = std::stoll(s.substr(i, j - i));
        i = j;
        // a value written as 12.0 or 1e3 is not an integer field of this format
        if (i < s.size() && (s[i] == '.' || s[i] == 'e' || s[i] == 'E')) bad = true;
        return v;
    }
    bool null() {
        ws();
        if (s.compare(i, 4, "null") == 0) {
            i += 4;
            return true;
        }
        return false;
    }
    void skip() {            // any value
        ws();
        if (i >= s.size()) {
            bad = true;
            return;
        }
        const char c = s[i];
        if (c == '"') {
            str();
        } else if (c == '{' || c == '[') {
            const char close = c == '{' ? '}' : ']';
            ++i;
            while (!bad && !eat(close)) {
                if (eat(',')) continue;
                if (c == '{') {
                    str();
                    if (!eat(':')) bad = true;
                }
                skip();
                if (i >= s.size()) bad = true;
            }
        } else {
            while (i < s.size() && s[i] != ',' && s[i] != '}' && s[i] != ']' && s[i] != ' ' && s[i] != '\n' &&
                   s[i] != '\r' && s[i] != '\t')
                ++i;
        }
    }
    template <class F>
    void object(F &&member) {           // member(key) consumes the value
        if (!eat('{')) {
            bad = true;
            return;
        }
        while (!bad && !eat('}')) {
            if (eat(',')) continue;
            const std::string k = str();
            if (!eat(':')) {
                bad = true;
                return;
            }
            member(k);
            if (i >= s.size()) bad = true;
        }
    }
    template <class F>
    void array(F &&elem) {
        if (!eat('[')) {
            bad = true;
            return;
        }
        while (!bad && !eat(']')) {
            if (eat(',')) continue;
            elem();
            if (i >= s.size()) bad = true;
        }
    }
    K50Rec record() {
        K50Rec r;
        object([&](const std::string &k) {
            if (null()) return;
            if (k == "expert") r.expert = (int)integer();
            else if (k == "kind") r.kind = str();
            else if (k == "unit") r.unit = str();
            else if (k == "shape") array([&] { r.shape.push_back(integer()); });
            else if (k == "row_bytes") r.row_bytes = integer();
            else if (k == "code_off") r.code_off = integer();
            else if (k == "code_nbytes") r.code_nbytes = integer();
            else if (k == "scale_off") r.scale_off = integer();
            else if (k == "scale_nbytes") r.scale_nbytes = integer();
            else if (k == "bias_off") r.bias_off = integer();
            else if (k == "bias_nbytes") r.bias_nbytes = integer();
            else if (k == "group_size") r.group_size = integer();
            else skip();
        });
        return r;
    }
};

// ------------------------------------------------------------------ pack
struct K50Pack {
    std::string dir;
    int fd[3] = {-1, -1, -1};        // codes, scales, biases
    std::map<std::string, K50Rec> recs;   // "<proj>:<expert>" and "dense:<name>"
    std::vector<std::string> dense_names;
    ~K50Pack() {
        for (int f : fd)
            if (f >= 0) ::close(f);
    }
};

int kind_bits(const std::string &k) {
    if (k == "tern" || k == "2t" || k == "2") return 2;
    if (k == "3") return 3;
    if (k == "4") return 4;
    if (k == "6") return 6;
    if (k == "8") return 8;
    return 0;
}

int kind_id(const std::string &k) {   // order of moe_k50_record's kind codes
    static const char *names[] = {"tern", "2t", "2", "3", "4", "6", "8"};
    for (int j = 0; j < 7; ++j)
        if (k == names[j]) return j;
    return -1;
}

int unit_id(const std::string &u) {
    static const char *names[] = {"hot", "warm", "mid", "cold", "dense"};
    for (int j = 0; j < 5; ++j)
        if (u == names[j]) return j;
    return -1;
}

bool pread_all(int fd, void *dst, size_t n, int64_t off) {
    auto *p = static_cast<unsigned char *>(dst);
    size_t done = 0;
    while (done < n) {
        const ssize_t r = ::pread(fd, p + done, n - done, (off_t)(off + (int64_t)done));
        if (r <= 0) return false;
        done += (size_t)r;
    }
    return true;
}

// geometry of a record's materialised form; 0 when the record is malformed
int geometry(const K50Rec &r, int64_t *rows, int64_t *cols, int64_t *words, int64_t *groups, int *bits) {
    const int b = kind_bits(r.kind);
    if (b == 0 || r.shape.size() != 2 || r.shape[0] <= 0 || r.shape[1] <= 0 || r.group_size <= 0 ||
        r.shape[1] % r.group_size)
        return 0;
    *rows = r.shape[0];
    *cols = r.shape[1];
    *bits = b;
    *groups = *cols / r.group_size;
    if (r.kind == "tern") {
        if (*cols % 80) return 0;            // 16 base-3 bytes -> 80 digits -> 5 words
        *words = *cols / 16;
    } else {
        if (r.code_nbytes % (*rows * 4)) return 0;
        *words = r.code_nbytes / (*rows * 4);
        if (*words * 32 != *cols * b) return 0;
    }
    if (r.scale_nbytes != *rows * *groups * 2) return 0;
    if (r.bias_nbytes != 0 && r.bias_nbytes != *rows * *groups * 2) return 0;
    return 1;
}

const K50Rec *find(K50Pack *p, const char *proj, int expert) {
    if (!p || !proj) return nullptr;
    const std::string key = expert >= 0 ? std::string(proj) + ":" + std::to_string(expert) : "dense:" + std::string(proj);
    auto it = p->recs.find(key);
    return it == p->recs.end() ? nullptr : &it->second;
}

}  // namespace

extern "C" {

void *moe_k50_open(const char *layer_dir) {
    if (!layer_dir) {
        moe_set_error(MOE_EINVAL, "k50_open: null directory");
        return nullptr;
    }
    auto p = std::make_unique<K50Pack>();
    p->dir = layer_dir;
    const char *files[3] = {"/codes.bin", "/scales.bf16", "/bias.bf16"};
    for (int j = 0; j < 3; ++j) {
        p->fd[j] = ::open((p->dir + files[j]).c_str(), O_RDONLY);
        if (p->fd[j] < 0) {
            moe_set_error(MOE_EIO, "k50_open: cannot open %s%s", layer_dir, files[j]);
            return nullptr;
        }
    }
    std::ifstream f(p->dir + "/index.json");
    if (!f) {
        moe_set_error(MOE_EIO, "k50_open: cannot open %s/index.json", layer_dir);
        return nullptr;
    }
    std::stringstream ss;
    ss << f.rdbuf();
    const std::string text = ss.str();
    Json js(text);
    try {    // no C++ exception may cross the C ABI (a number too large for int64, out of memory)
    js.object([&](const std::string &top) {
        if (top == "experts") {
            js.object([&](const std::string &proj) {
                js.array([&] {
                    K50Rec r = js.record();
                    if (r.expert >= 0) p->recs[proj + ":" + std::to_string(r.expert)] = r;
                    else js.bad = true;
                });
            });
        } else if (top == "dense") {
            js.object([&](const std::string &name) {
                p->recs["dense:" + name] = js.record();
                p->dense_names.push_back(name);
            });
        } else {
            js.skip();
        }
    });
    } catch (const std::exception &) {
        js.bad = true;
    }
    if (js.bad) {
        moe_set_error(MOE_EINVAL, "k50_open: %s/index.json is not a K50 index (parse error near byte %zu)",
                      layer_dir, js.i);
        return nullptr;
    }
    return p.release();
}

void moe_k50_close(void *h) { delete static_cast<K50Pack *>(h); }

int moe_k50_count(void *h, const char *proj) {
    auto *p = static_cast<K50Pack *>(h);
    if (!p || !proj) return moe_set_error(MOE_EINVAL, "k50_count: bad arguments");
    if (std::strcmp(proj, "dense") == 0) return (int)p->dense_names.size();
    const std::string pre = std::string(proj) + ":";
    int n = 0;
    for (auto &kv : p->recs)
        if (kv.first.compare(0, pre.size(), pre) == 0) ++n;
    return n;
}

int moe_k50_dense_name(void *h, int i, char *out, size_t out_bytes) {
    auto *p = static_cast<K50Pack *>(h);
    if (!p || !out || i < 0 || i >= (int)p->dense_names.size())
        return moe_set_error(MOE_EINVAL, "k50_dense_name: bad arguments");
    const std::string &n = p->dense_names[i];
    if (n.size() + 1 > out_bytes) return moe_set_error(MOE_EINVAL, "k50_dense_name: buffer too small");
    std::memcpy(out, n.c_str(), n.size() + 1);
    return MOE_OK;
}

int moe_k50_record(void *h, const char *proj, int expert, int64_t *out8) {
    auto *p = static_cast<K50Pack *>(h);
    const K50Rec *r = find(p, proj, expert);
    if (!r || !out8)
        return moe_set_error(MOE_EINVAL, "k50_record: no record %s:%d", proj ? proj : "(null)", expert);
    int64_t rows, cols, words, groups;
    int bits;
    if (!geometry(*r, &rows, &cols, &words, &groups, &bits))
        return moe_set_error(MOE_EINVAL, "k50_record: %s:%d (kind '%s') has inconsistent sizes", proj, expert,
                             r->kind.c_str());
    out8[0] = bits;
    out8[1] = r->group_size;
    out8[2] = rows;
    out8[3] = cols;
    out8[4] = words;
    out8[5] = groups;
    out8[6] = kind_id(r->kind);
    out8[7] = unit_id(r->unit);
    return MOE_OK;
}

int moe_k50_materialize(void *h, const char *proj, int expert, uint32_t *codes, uint16_t *scales,
                        uint16_t *biases) {
    auto *p = static_cast<K50Pack *>(h);
    const K50Rec *r = find(p, proj, expert);
    if (!r || !codes || !scales || !biases)
        return moe_set_error(MOE_EINVAL, "k50_materialize: no record %s:%d or null output", proj ? proj : "(null)",
                             expert);
    int64_t rows, cols, words, groups;
    int bits;
    if (!geometry(*r, &rows, &cols, &words, &groups, &bits))
        return moe_set_error(MOE_EINVAL, "k50_materialize: %s:%d has inconsistent sizes", proj, expert);
    if (!pread_all(p->fd[1], scales, (size_t)r->scale_nbytes, r->scale_off))
        return moe_set_error(MOE_EIO, "k50_materialize: short read of scales.bf16 (%s:%d)", proj, expert);
    if (r->kind == "tern") {
        const int64_t rb = r->row_bytes > 0 ? r->row_bytes : cols / 5;
        if (rb * 5 != cols || r->code_nbytes < rows * rb)
            return moe_set_error(MOE_EINVAL, "k50_materialize: ternary row of %lld bytes for %lld columns",
                                 (long long)rb, (long long)cols);
        std::vector<unsigned char> raw((size_t)(rows * rb));
        if (!pread_all(p->fd[0], raw.data(), raw.size(), r->code_off))
            return moe_set_error(MOE_EIO, "k50_materialize: short read of codes.bin (%s:%d)", proj, expert);
        for (int64_t row = 0; row < rows; ++row) {
            const unsigned char *src = raw.data() + row * rb;
            uint32_t *dst = codes + row * words;
            uint32_t word = 0;
            int64_t digit = 0;
            for (int64_t b = 0; b < rb; ++b) {
                unsigned v = src[b];
                for (int d = 0; d < 5; ++d, ++digit) {
                    word |= (uint32_t)(v % 3u) << (2 * (digit & 15));
                    v /= 3u;
                    if ((digit & 15) == 15) {
                        dst[digit >> 4] = word;
                        word = 0;
                    }
                }
            }
        }
        for (int64_t j = 0; j < rows * groups; ++j) biases[j] = (uint16_t)(scales[j] ^ 0x8000u);
        return MOE_OK;
    }
    if (!pread_all(p->fd[0], codes, (size_t)r->code_nbytes, r->code_off))
        return moe_set_error(MOE_EIO, "k50_materialize: short read of codes.bin (%s:%d)", proj, expert);
    if (r->bias_nbytes > 0) {
        if (!pread_all(p->fd[2], biases, (size_t)r->bias_nbytes, r->bias_off))
            return moe_set_error(MOE_EIO, "k50_materialize: short read of bias.bf16 (%s:%d)", proj, expert);
    } else {
        for (int64_t j = 0; j < rows * groups; ++j) biases[j] = (uint16_t)(scales[j] ^ 0x8000u);
    }
    return MOE_OK;
}

}  // extern "C"
