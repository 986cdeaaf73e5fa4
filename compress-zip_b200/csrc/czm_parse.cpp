// czm_parse.cpp -- a small recursive-descent JSON reader, enough for the
// safetensors header of a .czm file (rust/src/safetensors.rs:287-376).
#include "czm_parse.h"

#include <cstdlib>
#include <cstring>

namespace czg {
namespace {

struct JVal {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    bool b = false;
    double num = 0;
    int64_t inum = 0;
    bool is_int = false;
    std::string str;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
};

struct Reader {
    const char *p, *end;
    std::string err;
    int depth = 0;

    void ws() {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) p++;
    }
    bool fail(const char *m) {
        if (err.empty()) err = m;
        return false;
    }
    static void put_utf8(std::string &s, uint32_t cp) {
        if (cp < 0x80) s += (char)cp;
        else if (cp < 0x800) { s += (char)(0xC0 | (cp >> 6)); s += (char)(0x80 | (cp & 0x3F)); }
        else if (cp < 0x10000) {
            s += (char)(0xE0 | (cp >> 12)); s += (char)(0x80 | ((cp >> 6) & 0x3F));
            s += (char)(0x80 | (cp & 0x3F));
        } else {
            s += (char)(0xF0 | (cp >> 18)); s += (char)(0x80 | ((cp >> 12) & 0x3F));
            s += (char)(0x80 | ((cp >> 6) & 0x3F)); s += (char)(0x80 | (cp & 0x3F));
        }
    }
    bool hex4(uint32_t &v) {
        if (end - p < 4) return fail("bad \\u escape");
        v = 0;
        for (int i = 0; i < 4; i++) {
            char c = *p++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else return fail("bad \\u escape");
        }
        return true;
    }
    bool string(std::string &s) {
        if (p >= end || *p != '"') return fail("expected string");
        p++;
        while (p < end && *p != '"') {
            char c = *p++;
            if (c != '\\') { s += c; continue; }
            if (p >= end) return fail("bad escape");
            char e = *p++;
            switch (e) {
                case '"': s += '"'; break;
                case '\\': s += '\\'; break;
                case '/': s += '/'; break;
                case 'b': s += '\b'; break;
                case 'f': s += '\f'; break;
                case 'n': s += '\n'; break;
                case 'r': s += '\r'; break;
                case 't': s += '\t'; break;
                case 'u': {
                    uint32_t cp;
                    if (!hex4(cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00 && end - p >= 6 && p[0] == '\\' && p[1] == 'u') {
                        p += 2;
                        uint32_t lo;
                        if (!hex4(lo)) return false;
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    put_utf8(s, cp);
                    break;
                }
                default: return fail("bad escape");
            }
        }
        if (p >= end) return fail("unterminated string");
        p++;
        return true;
    }
    bool value(JVal &v) {
        if (++depth > 64) return fail("JSON nested too deeply");
        ws();
        if (p >= end) return fail("unexpected end of JSON");
        bool ok = true;
        if (*p == '{') {
            v.kind = JVal::Obj;
            p++;
            ws();
            if (p < end && *p == '}') { p++; }
            else {
                for (;;) {
                    ws();
                    std::pair<std::string, JVal> kv;
                    if (!string(kv.first)) { ok = false; break; }
                    ws();
                    if (p >= end || *p != ':') { ok = fail("expected ':'"); break; }
                    p++;
                    if (!value(kv.second)) { ok = false; break; }
                    v.obj.push_back(std::move(kv));
                    ws();
                    if (p < end && *p == ',') { p++; continue; }
                    if (p < end && *p == '}') { p++; break; }
                    ok = fail("expected ',' or '}'");
                    break;
                }
            }
        } else if (*p == '[') {
            v.kind = JVal::Arr;
            p++;
            ws();
            if (p < end && *p == ']') { p++; }
            else {
                for (;;) {
                    JVal e;
                    if (!value(e)) { ok = false; break; }
                    v.arr.push_back(std::move(e));
                    ws();
                    if (p < end && *p == ',') { p++; continue; }
                    if (p < end && *p == ']') { p++; break; }
                    ok = fail("expected ',' or ']'");
                    break;
                }
            }
        } else if (*p == '"') {
            v.kind = JVal::Str;
            ok = string(v.str);
        } else if (end - p >= 4 && !strncmp(p, "true", 4)) {
            v.kind = JVal::Bool; v.b = true; p += 4;
        } else if (end - p >= 5 && !strncmp(p, "false", 5)) {
            v.kind = JVal::Bool; v.b = false; p += 5;
        } else if (end - p >= 4 && !strncmp(p, "null", 4)) {
            v.kind = JVal::Null; p += 4;
        } else {
            const char *s = p;
            bool neg = false, frac = false;
            if (p < end && *p == '-') { neg = true; p++; }
            int64_t iv = 0;
            bool digits = false;
            while (p < end && *p >= '0' && *p <= '9') {
                iv = iv * 10 + (*p - '0');
                p++;
                digits = true;
            }
            while (p < end && (*p == '.' || *p == 'e' || *p == 'E' || *p == '+' || *p == '-' ||
                               (*p >= '0' && *p <= '9'))) { frac = true; p++; }
            if (!digits) ok = fail("bad JSON value");
            v.kind = JVal::Num;
            v.is_int = !frac;
            v.inum = neg ? -iv : iv;
            v.num = strtod(std::string(s, p).c_str(), nullptr);
        }
        depth--;
        return ok;
    }
};

}  // namespace

std::string parse_czm(const uint8_t *data, size_t len, CzmFile &out) {
    if (len < 8) return "Invalid header size";
    uint64_t hlen = 0;
    for (int i = 7; i >= 0; i--) hlen = (hlen << 8) | data[i];
    if (hlen > len - 8) return "Invalid header size";
    Reader r{reinterpret_cast<const char *>(data + 8), reinterpret_cast<const char *>(data + 8 + hlen)};
    JVal root;
    if (!r.value(root)) return "Header JSON error: " + r.err;
    if (root.kind != JVal::Obj) return "Header is not a JSON object";
    const uint8_t *base = data + 8 + hlen;
    size_t avail = len - 8 - hlen;
    for (auto &kv : root.obj) {
        if (kv.first == "__metadata__") {
            if (kv.second.kind == JVal::Obj)
                for (auto &m : kv.second.obj)
                    if (m.second.kind == JVal::Str) out.metadata[m.first] = m.second.str;
            continue;
        }
        const JVal &info = kv.second;
        if (info.kind != JVal::Obj) return "tensor entry is not an object: " + kv.first;
        TensorRef t;
        const JVal *offs = nullptr;
        bool have_dtype = false, have_shape = false;
        for (auto &f : info.obj) {
            if (f.first == "dtype" && f.second.kind == JVal::Str) { t.dtype = f.second.str; have_dtype = true; }
            else if (f.first == "shape" && f.second.kind == JVal::Arr) {
                have_shape = true;
                for (auto &s : f.second.arr) {
                    if (s.kind != JVal::Num || !s.is_int || s.inum < 0) return "bad shape: " + kv.first;
                    t.shape.push_back(s.inum);
                }
            } else if (f.first == "data_offsets" && f.second.kind == JVal::Arr) offs = &f.second;
        }
        if (!have_dtype || !have_shape || !offs || offs->arr.size() != 2) return "bad tensor entry: " + kv.first;
        if (t.shape.size() > 8) return "Tensor dimension exceeds maximum allowed";
        int64_t a = offs->arr[0].inum, b = offs->arr[1].inum;
        if (a < 0 || b < a || (uint64_t)b > avail) return "tensor data out of file bounds: " + kv.first;
        t.data = base + a;
        t.nbytes = (size_t)(b - a);
        out.tensors[kv.first] = std::move(t);
    }
    if (out.tensors.size() > 2048) return "Number of tensors exceeds maximum allowed";
    return "";
}

}  // namespace czg
