// json_lite.h -- a small validating JSON reader for host code (safetensors
// headers, the index's weight map, a model's config.json): recursive descent
// with a depth limit, strict literals and escapes, and non-negative integers
// kept exactly as uint64 (byte offsets past 2^53).
#pragma once

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

namespace tb_json {

struct JVal {
    enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
    bool b = false;
    bool is_uint = false;        // a non-negative integer literal, exactly in u
    uint64_t u = 0;
    double d = 0.0;
    std::string s;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;

    const JVal* get(const char* key) const {
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

class JsonParser {
public:
    JsonParser(const char* p, size_t n) : p_(p), e_(p + n) {}
    bool parse(JVal* out) {
        ws();
        if (!value(out, 0)) return false;
        ws();
        return p_ == e_;
    }

private:
    const char* p_;
    const char* e_;
    static constexpr int kMaxDepth = 64;

    void ws() {
        while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool lit(const char* w) {
        const size_t n = std::strlen(w);
        if (static_cast<size_t>(e_ - p_) < n || std::memcmp(p_, w, n) != 0) return false;
        p_ += n;
        return true;
    }
    static void put_utf8(std::string& s, uint32_t c) {
        if (c < 0x80) {
            s += static_cast<char>(c);
        } else if (c < 0x800) {
            s += static_cast<char>(0xC0 | (c >> 6));
            s += static_cast<char>(0x80 | (c & 0x3F));
        } else {
            s += static_cast<char>(0xE0 | (c >> 12));
            s += static_cast<char>(0x80 | ((c >> 6) & 0x3F));
            s += static_cast<char>(0x80 | (c & 0x3F));
        }
    }
    bool str(std::string* out) {
        if (p_ >= e_ || *p_ != '"') return false;
        ++p_;
        out->clear();
        while (p_ < e_ && *p_ != '"') {
            char c = *p_++;
            if (static_cast<unsigned char>(c) < 0x20) return false;
            if (c != '\\') {
                *out += c;
                continue;
            }
            if (p_ >= e_) return false;
            c = *p_++;
            switch (c) {
                case '"': *out += '"'; break;
                case '\\': *out += '\\'; break;
                case '/': *out += '/'; break;
                case 'b': *out += '\b'; break;
                case 'f': *out += '\f'; break;
                case 'n': *out += '\n'; break;
                case 'r': *out += '\r'; break;
                case 't': *out += '\t'; break;
                case 'u': {
                    if (e_ - p_ < 4) return false;
                    uint32_t cp = 0;
                    for (int i = 0; i < 4; ++i) {
                        const char h = *p_++;
                        cp <<= 4;
                        if (h >= '0' && h <= '9') cp |= h - '0';
                        else if (h >= 'a' && h <= 'f') cp |= h - 'a' + 10;
                        else if (h >= 'A' && h <= 'F') cp |= h - 'A' + 10;
                        else return false;
                    }
                    put_utf8(*out, cp);
                    break;
                }
                default: return false;
            }
        }
        if (p_ >= e_) return false;
        ++p_;
        return true;
    }
    bool num(JVal* v) {
        const char* s = p_;
        if (p_ < e_ && *p_ == '-') ++p_;
        if (p_ >= e_ || *p_ < '0' || *p_ > '9') return false;
        while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
        bool integer = true;
        if (p_ < e_ && *p_ == '.') {
            integer = false;
            ++p_;
            if (p_ >= e_ || *p_ < '0' || *p_ > '9') return false;
            while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        if (p_ < e_ && (*p_ == 'e' || *p_ == 'E')) {
            integer = false;
            ++p_;
            if (p_ < e_ && (*p_ == '+' || *p_ == '-')) ++p_;
            if (p_ >= e_ || *p_ < '0' || *p_ > '9') return false;
            while (p_ < e_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        v->kind = JVal::kNum;
        const std::string text(s, p_);
        v->d = std::strtod(text.c_str(), nullptr);
        if (integer && text[0] != '-') {
            uint64_t u = 0;
            for (char c : text) {
                const uint64_t dig = static_cast<uint64_t>(c - '0');
                if (u > (UINT64_MAX - dig) / 10) return false;   // overflow
                u = u * 10 + dig;
            }
            v->is_uint = true;
            v->u = u;
        }
        return true;
    }
    bool value(JVal* v, int depth) {
        if (depth > kMaxDepth || p_ >= e_) return false;
        const char c = *p_;
        if (c == '{') {
            ++p_;
            v->kind = JVal::kObj;
            ws();
            if (p_ < e_ && *p_ == '}') { ++p_; return true; }
            while (true) {
                ws();
                std::string key;
                if (!str(&key)) return false;
                ws();
                if (p_ >= e_ || *p_ != ':') return false;
                ++p_;
                ws();
                JVal child;
                if (!value(&child, depth + 1)) return false;
                v->obj.emplace_back(std::move(key), std::move(child));
                ws();
                if (p_ < e_ && *p_ == ',') { ++p_; continue; }
                if (p_ < e_ && *p_ == '}') { ++p_; return true; }
                return false;
            }
        }
        if (c == '[') {
            ++p_;
            v->kind = JVal::kArr;
            ws();
            if (p_ < e_ && *p_ == ']') { ++p_; return true; }
            while (true) {
                ws();
                JVal child;
                if (!value(&child, depth + 1)) return false;
                v->arr.push_back(std::move(child));
                ws();
                if (p_ < e_ && *p_ == ',') { ++p_; continue; }
                if (p_ < e_ && *p_ == ']') { ++p_; return true; }
                return false;
            }
        }
        if (c == '"') { v->kind = JVal::kStr; return str(&v->s); }
        if (c == 't') { v->kind = JVal::kBool; v->b = true; return lit("true"); }
        if (c == 'f') { v->kind = JVal::kBool; v->b = false; return lit("false"); }
        if (c == 'n') { v->kind = JVal::kNull; return lit("null"); }
        return num(v);
    }
};

}  // namespace tb_json
