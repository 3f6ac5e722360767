// model_io.cu - host side of the model-level pipeline's file I/O (src/io.rs): a JSON subset parser, safetensors
// files read through mmap and written in the safetensors layout, and the calibration-Hessian store.
#include <errno.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>

#include "cdclq.h"
#include "common.cuh"
#include "model_io.h"

namespace cdclq {
namespace io {

// ---- JSON ------------------------------------------------------------------------------------------------
const Json* Json::get(const std::string& key) const {
    if (kind != Object) return nullptr;
    for (auto& kv : obj)
        if (kv.first == key) return &kv.second;
    return nullptr;
}

namespace {

struct Parser {
    const char* s;
    size_t n, i = 0;
    std::string err;

    void ws() {
        while (i < n && (s[i] == ' ' || s[i] == '\t' || s[i] == '\n' || s[i] == '\r')) i++;
    }
    bool fail(const std::string& m) {
        if (err.empty()) err = m + " at byte " + std::to_string(i);
        return false;
    }
    static void put_utf8(std::string& o, uint32_t c) {
        if (c < 0x80) {
            o += (char)c;
        } else if (c < 0x800) {
            o += (char)(0xC0 | (c >> 6));
            o += (char)(0x80 | (c & 0x3F));
        } else if (c < 0x10000) {
            o += (char)(0xE0 | (c >> 12));
            o += (char)(0x80 | ((c >> 6) & 0x3F));
            o += (char)(0x80 | (c & 0x3F));
        } else {
            o += (char)(0xF0 | (c >> 18));
            o += (char)(0x80 | ((c >> 12) & 0x3F));
            o += (char)(0x80 | ((c >> 6) & 0x3F));
            o += (char)(0x80 | (c & 0x3F));
        }
    }
    bool hex4(uint32_t* v) {
        if (i + 4 > n) return fail("truncated \\u escape");
        uint32_t r = 0;
        for (int k = 0; k < 4; k++) {
            char c = s[i++];
            r <<= 4;
            if (c >= '0' && c <= '9') r |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') r |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') r |= (uint32_t)(c - 'A' + 10);
            else return fail("bad \\u escape");
        }
        *v = r;
        return true;
    }
    bool string(std::string* o) {
        if (i >= n || s[i] != '"') return fail("expected a string");
        i++;
        while (i < n && s[i] != '"') {
            char c = s[i++];
            if (c != '\\') {
                *o += c;
                continue;
            }
            if (i >= n) return fail("truncated escape");
            char e = s[i++];
            switch (e) {
                case '"': *o += '"'; break;
                case '\\': *o += '\\'; break;
                case '/': *o += '/'; break;
                case 'b': *o += '\b'; break;
                case 'f': *o += '\f'; break;
                case 'n': *o += '\n'; break;
                case 'r': *o += '\r'; break;
                case 't': *o += '\t'; break;
                case 'u': {
                    uint32_t c1 = 0;
                    if (!hex4(&c1)) return false;
                    if (c1 >= 0xD800 && c1 < 0xDC00 && i + 6 <= n && s[i] == '\\' && s[i + 1] == 'u') {
                        i += 2;
                        uint32_t c2 = 0;
                        if (!hex4(&c2)) return false;
                        c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
                    }
                    put_utf8(*o, c1);
                    break;
                }
                default: return fail("bad escape");
            }
        }
        if (i >= n) return fail("unterminated string");
        i++;
        return true;
    }
    bool value(Json* v, int depth) {
        if (depth > 64) return fail("nesting too deep");
        ws();
        if (i >= n) return fail("unexpected end");
        char c = s[i];
        if (c == '{') {
            v->kind = Json::Object;
            i++;
            ws();
            if (i < n && s[i] == '}') {
                i++;
                return true;
            }
            for (;;) {
                ws();
                std::string k;
                if (!string(&k)) return false;
                ws();
                if (i >= n || s[i] != ':') return fail("expected ':'");
                i++;
                Json x;
                if (!value(&x, depth + 1)) return false;
                v->obj.emplace_back(std::move(k), std::move(x));
                ws();
                if (i < n && s[i] == ',') {
                    i++;
                    continue;
                }
                if (i < n && s[i] == '}') {
                    i++;
                    return true;
                }
                return fail("expected ',' or '}'");
            }
        }
        if (c == '[') {
            v->kind = Json::Array;
            i++;
            ws();
            if (i < n && s[i] == ']') {
                i++;
                return true;
            }
            for (;;) {
                Json x;
                if (!value(&x, depth + 1)) return false;
                v->arr.push_back(std::move(x));
                ws();
                if (i < n && s[i] == ',') {
                    i++;
                    continue;
                }
                if (i < n && s[i] == ']') {
                    i++;
                    return true;
                }
                return fail("expected ',' or ']'");
            }
        }
        if (c == '"') {
            v->kind = Json::String;
            return string(&v->str);
        }
        if (n - i >= 4 && !strncmp(s + i, "true", 4)) {
            v->kind = Json::Bool;
            v->b = true;
            i += 4;
            return true;
        }
        if (n - i >= 5 && !strncmp(s + i, "false", 5)) {
            v->kind = Json::Bool;
            i += 5;
            return true;
        }
        if (n - i >= 4 && !strncmp(s + i, "null", 4)) {
            v->kind = Json::Null;
            i += 4;
            return true;
        }
        size_t j = i;
        while (j < n && (s[j] == '-' || s[j] == '+' || s[j] == '.' || s[j] == 'e' || s[j] == 'E' ||
                         (s[j] >= '0' && s[j] <= '9')))
            j++;
        if (j == i) return fail("unexpected character");
        std::string num(s + i, j - i);
        char* end = nullptr;
        v->kind = Json::Number;
        v->num = strtod(num.c_str(), &end);
        if (!end || *end) return fail("bad number");
        i = j;
        return true;
    }
};

}  // namespace

bool parse_json(const char* s, size_t len, Json* out, std::string* err) {
    Parser p{s, len};
    if (!p.value(out, 0)) {
        if (err) *err = p.err;
        return false;
    }
    p.ws();
    if (p.i != len) {
        if (err) *err = "trailing data at byte " + std::to_string(p.i);
        return false;
    }
    return true;
}

std::string json_quote(const std::string& s) {
    std::string o = "\"";
    for (unsigned char c : s) {
        switch (c) {
            case '"': o += "\\\""; break;
            case '\\': o += "\\\\"; break;
            case '\n': o += "\\n"; break;
            case '\r': o += "\\r"; break;
            case '\t': o += "\\t"; break;
            default:
                if (c < 0x20) {
                    char b[8];
                    snprintf(b, sizeof b, "\\u%04x", c);
                    o += b;
                } else {
                    o += (char)c;
                }
        }
    }
    return o + "\"";
}

// ---- safetensors -----------------------------------------------------------------------------------------
size_t dtype_size(const std::string& d) {
    if (d == "F64" || d == "I64" || d == "U64") return 8;
    if (d == "F32" || d == "I32" || d == "U32") return 4;
    if (d == "F16" || d == "BF16" || d == "I16" || d == "U16") return 2;
    if (d == "U8" || d == "I8" || d == "BOOL" || d == "F8_E4M3" || d == "F8_E5M2") return 1;
    return 0;
}

// The safetensors crate's dtype order (its Dtype enum), used to lay tensors out: larger alignment first.
static int dtype_rank(const std::string& d) {
    static const char* order[] = {"BOOL", "U8", "I8", "F8_E5M2", "F8_E4M3", "I16", "U16", "F16",
                                  "BF16", "I32", "U32", "F32", "F64", "I64", "U64"};
    for (int k = 0; k < (int)(sizeof order / sizeof order[0]); k++)
        if (d == order[k]) return k;
    return -1;
}

SafeTensorsFile::~SafeTensorsFile() {
    if (map_) munmap(map_, size_);
}

int SafeTensorsFile::open(const std::string& path) {
    path_ = path;
    auto bad = [&](const std::string& m) { return set_error(CDCLQ_ERR_ARG, path + ": " + m); };
    int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) return set_error(CDCLQ_ERR_ARG, "cannot open " + path + ": " + strerror(errno));
    struct stat sb;
    if (fstat(fd, &sb) != 0) {
        ::close(fd);
        return bad(strerror(errno));
    }
    size_ = (size_t)sb.st_size;
    if (size_ < 8) {
        ::close(fd);
        return bad("not a safetensors file (shorter than its 8-byte header length)");
    }
    map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (map_ == MAP_FAILED) {
        map_ = nullptr;
        return set_error(CDCLQ_ERR_ARG, "cannot mmap " + path + ": " + strerror(errno));
    }
    const uint8_t* b = (const uint8_t*)map_;
    uint64_t hl = 0;
    for (int k = 7; k >= 0; k--) hl = (hl << 8) | b[k];
    if (hl > size_ - 8) return bad("header length " + std::to_string(hl) + " exceeds the file");
    Json h;
    std::string err;
    if (!parse_json((const char*)b + 8, (size_t)hl, &h, &err)) return bad("invalid header: " + err);
    if (h.kind != Json::Object) return bad("invalid header: not an object");
    const uint8_t* data = b + 8 + hl;
    const size_t dlen = size_ - 8 - (size_t)hl;
    for (auto& kv : h.obj) {
        if (kv.first == "__metadata__") {
            if (kv.second.kind != Json::Object) return bad("__metadata__ is not an object");
            for (auto& m : kv.second.obj) {
                if (m.second.kind != Json::String) return bad("metadata value of " + m.first + " is not a string");
                md_[m.first] = m.second.str;
            }
            continue;
        }
        const Json* dt = kv.second.get("dtype");
        const Json* sh = kv.second.get("shape");
        const Json* off = kv.second.get("data_offsets");
        if (!dt || dt->kind != Json::String || !sh || sh->kind != Json::Array || !off || off->kind != Json::Array ||
            off->arr.size() != 2)
            return bad("tensor " + kv.first + ": malformed entry");
        TensorView v;
        v.dtype = dt->str;
        for (auto& d : sh->arr) {
            if (d.kind != Json::Number || d.num < 0) return bad("tensor " + kv.first + ": bad shape");
            v.shape.push_back((size_t)d.num);
        }
        const double o0 = off->arr[0].num, o1 = off->arr[1].num;
        if (!(o0 >= 0 && o1 >= o0 && o1 <= (double)dlen)) return bad("tensor " + kv.first + ": offsets out of range");
        v.data = data + (size_t)o0;
        v.nbytes = (size_t)o1 - (size_t)o0;
        const size_t es = dtype_size(v.dtype);
        if (es && v.numel() * es != v.nbytes)
            return bad("tensor " + kv.first + ": " + std::to_string(v.nbytes) + " bytes for its shape and dtype " +
                       v.dtype);
        t_[kv.first] = std::move(v);
    }
    return 0;
}

std::vector<std::string> SafeTensorsFile::names() const {
    std::vector<std::string> v;
    for (auto& kv : t_) v.push_back(kv.first);
    return v;  // std::map keeps them sorted
}

const TensorView* SafeTensorsFile::tensor(const std::string& name) const {
    auto it = t_.find(name);
    return it == t_.end() ? nullptr : &it->second;
}

static int mkdirs(const std::string& dir) {
    if (dir.empty()) return 0;
    std::string cur;
    size_t p = 0;
    while (p != std::string::npos) {
        p = dir.find('/', p + 1);
        cur = dir.substr(0, p);
        if (cur.empty()) continue;
        if (mkdir(cur.c_str(), 0755) != 0 && errno != EEXIST)
            return set_error(CDCLQ_ERR_ARG, "cannot create " + cur + ": " + strerror(errno));
    }
    return 0;
}

int write_tensors(const std::string& path, const std::vector<OutTensor>& ts,
                  const std::map<std::string, std::string>& meta) {
    size_t slash = path.rfind('/');
    if (slash != std::string::npos) {
        int rc = mkdirs(path.substr(0, slash));
        if (rc) return rc;
    }
    std::vector<size_t> order(ts.size());
    for (size_t k = 0; k < ts.size(); k++) {
        order[k] = k;
        const size_t es = dtype_size(ts[k].dtype);
        size_t numel = 1;
        for (size_t d : ts[k].shape) numel *= d;
        if (!es || numel * es != ts[k].bytes.size())
            return set_error(CDCLQ_ERR_ARG, "tensor " + ts[k].name + ": " + std::to_string(ts[k].bytes.size()) +
                                                " bytes do not match its shape and dtype " + ts[k].dtype);
    }
    std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) {
        int ra = dtype_rank(ts[a].dtype), rb = dtype_rank(ts[b].dtype);
        if (ra != rb) return ra > rb;
        return ts[a].name < ts[b].name;
    });
    std::string hdr = "{";
    if (!meta.empty()) {
        hdr += "\"__metadata__\":{";
        bool first = true;
        for (auto& kv : meta) {
            if (!first) hdr += ",";
            first = false;
            hdr += json_quote(kv.first) + ":" + json_quote(kv.second);
        }
        hdr += "}";
    }
    size_t off = 0;
    for (size_t k : order) {
        const OutTensor& t = ts[k];
        if (hdr.size() > 1) hdr += ",";
        hdr += json_quote(t.name) + ":{\"dtype\":" + json_quote(t.dtype) + ",\"shape\":[";
        for (size_t d = 0; d < t.shape.size(); d++) hdr += (d ? "," : "") + std::to_string(t.shape[d]);
        hdr += "],\"data_offsets\":[" + std::to_string(off) + "," + std::to_string(off + t.bytes.size()) + "]}";
        off += t.bytes.size();
    }
    hdr += "}";
    while (hdr.size() % 8) hdr += ' ';
    FILE* f = fopen(path.c_str(), "wb");
    if (!f) return set_error(CDCLQ_ERR_ARG, "cannot write " + path + ": " + strerror(errno));
    uint8_t len[8];
    uint64_t hl = hdr.size();
    for (int k = 0; k < 8; k++) len[k] = (uint8_t)(hl >> (8 * k));
    bool ok = fwrite(len, 1, 8, f) == 8 && fwrite(hdr.data(), 1, hdr.size(), f) == hdr.size();
    for (size_t k : order)
        if (ok && !ts[k].bytes.empty()) ok = fwrite(ts[k].bytes.data(), 1, ts[k].bytes.size(), f) == ts[k].bytes.size();
    if (fclose(f) != 0) ok = false;
    if (!ok) return set_error(CDCLQ_ERR_ARG, "writing " + path + " failed: " + strerror(errno));
    return 0;
}

// ---- Hessian store --------------------------------------------------------------------------------------
int HessianStore::open(const std::vector<std::string>& paths) {
    for (size_t fi = 0; fi < paths.size(); fi++) {
        std::unique_ptr<SafeTensorsFile> f(new SafeTensorsFile());
        int rc = f->open(paths[fi]);
        if (rc) return rc;
        for (auto& name : f->names())
            if (name.size() > 2 && name.compare(name.size() - 2, 2, ".H") == 0) index_[name.substr(0, name.size() - 2)] = fi;
        auto it = f->metadata().find("aliases");
        if (it != f->metadata().end()) {
            Json a;
            std::string err;
            if (!parse_json(it->second.data(), it->second.size(), &a, &err) || a.kind != Json::Object)
                return set_error(CDCLQ_ERR_ARG, "invalid 'aliases' metadata in " + paths[fi] + ": " +
                                                    (err.empty() ? "not an object" : err));
            for (auto& kv : a.obj) {
                if (kv.second.kind != Json::String)
                    return set_error(CDCLQ_ERR_ARG, "invalid 'aliases' metadata in " + paths[fi] + ": " + kv.first +
                                                        " is not mapped to a layer name");
                aliases_[kv.first] = kv.second.str;
            }
        }
        files_.push_back(std::move(f));
    }
    return 0;
}

std::string HessianStore::resolve(const std::string& layer) const {
    if (index_.count(layer)) return layer;
    auto it = aliases_.find(layer);
    if (it != aliases_.end() && index_.count(it->second)) return it->second;
    return "";
}

const TensorView* HessianStore::tensor(const std::string& owner, const char* suffix, size_t* n, bool* missing) const {
    *missing = false;
    auto it = index_.find(owner);
    if (it == index_.end()) {
        set_error(CDCLQ_ERR_ARG, "no Hessian for " + owner);
        return nullptr;
    }
    const std::string key = owner + "." + suffix;
    const TensorView* t = files_[it->second]->tensor(key);
    if (!t) {
        *missing = true;
        return nullptr;
    }
    if (t->shape.size() != 2 || t->shape[0] != t->shape[1]) {
        std::string sh = "[";
        for (size_t d = 0; d < t->shape.size(); d++) sh += (d ? ", " : "") + std::to_string(t->shape[d]);
        set_error(CDCLQ_ERR_ARG, key + ": expected a square matrix, got " + sh + "]");
        return nullptr;
    }
    if (t->dtype != "F32" && t->dtype != "F16" && t->dtype != "BF16") {
        set_error(CDCLQ_ERR_ARG, "unsupported weight dtype " + t->dtype + " (need F32/F16/BF16)");
        return nullptr;
    }
    *n = t->shape[0];
    return t;
}

}  // namespace io
}  // namespace cdclq
