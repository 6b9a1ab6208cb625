// json_lite.hpp -- small JSON reader for the CLI's config object.
//
// The reference CLIs parse stdin with nlohmann::json::parse(std::cin, nullptr,
// true, /*ignore_comments=*/true) (src/gpu_cli.cu:357); this reader accepts
// the same documents: objects, arrays, strings with escapes, numbers,
// true/false/null, and // or /* */ comments between tokens.
#pragma once

#include <cctype>
#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace bsb {
namespace json {

struct Value {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0.0;
    bool is_int = false;
    int64_t i = 0;
    std::string str;
    std::vector<Value> arr;
    std::map<std::string, Value> obj;

    bool contains(const std::string& k) const { return kind == Object && obj.count(k) != 0; }
    const Value* find(const std::string& k) const {
        if (kind != Object) return nullptr;
        auto it = obj.find(k);
        return it == obj.end() ? nullptr : &it->second;
    }
    // nlohmann-style value(key, default) for the scalar kinds the CLI uses
    std::string value(const std::string& k, const std::string& def) const {
        const Value* v = find(k);
        if (!v || v->kind == Null) return def;
        if (v->kind != String) throw std::runtime_error("type_error: \"" + k + "\" must be a string");
        return v->str;
    }
    int64_t value(const std::string& k, int64_t def) const {
        const Value* v = find(k);
        if (!v || v->kind == Null) return def;
        if (v->kind == Bool) return v->b ? 1 : 0;
        if (v->kind != Number) throw std::runtime_error("type_error: \"" + k + "\" must be a number");
        return v->is_int ? v->i : static_cast<int64_t>(v->num);
    }
};

class Parser {
public:
    explicit Parser(const std::string& s) : s_(s) {}
    Value parse() {
        Value v = value();
        ws();
        if (p_ != s_.size()) error("unexpected trailing characters");
        return v;
    }

private:
    const std::string& s_;
    size_t p_ = 0;

    [[noreturn]] void error(const std::string& what) const {
        throw std::runtime_error("parse error at byte " + std::to_string(p_) + ": " + what);
    }
    void ws() {
        for (;;) {
            while (p_ < s_.size() && std::isspace(static_cast<unsigned char>(s_[p_]))) ++p_;
            if (p_ + 1 < s_.size() && s_[p_] == '/' && s_[p_ + 1] == '/') {
                while (p_ < s_.size() && s_[p_] != '\n') ++p_;
                continue;
            }
            if (p_ + 1 < s_.size() && s_[p_] == '/' && s_[p_ + 1] == '*') {
                const size_t e = s_.find("*/", p_ + 2);
                if (e == std::string::npos) error("unterminated comment");
                p_ = e + 2;
                continue;
            }
            return;
        }
    }
    bool lit(const char* w) {
        size_t n = 0;
        while (w[n]) ++n;
        if (s_.compare(p_, n, w) == 0) { p_ += n; return true; }
        return false;
    }
    Value value() {
        ws();
        if (p_ >= s_.size()) error("unexpected end of input");
        const char c = s_[p_];
        Value v;
        if (c == '{') return object();
        if (c == '[') return array();
        if (c == '"') { v.kind = Value::String; v.str = string(); return v; }
        if (lit("true")) { v.kind = Value::Bool; v.b = true; return v; }
        if (lit("false")) { v.kind = Value::Bool; v.b = false; return v; }
        if (lit("null")) return v;
        if (c == '-' || std::isdigit(static_cast<unsigned char>(c))) return number();
        error(std::string("unexpected character '") + c + "'");
    }
    Value object() {
        Value v;
        v.kind = Value::Object;
        ++p_;
        ws();
        if (p_ < s_.size() && s_[p_] == '}') { ++p_; return v; }
        for (;;) {
            ws();
            if (p_ >= s_.size() || s_[p_] != '"') error("expected a key string");
            std::string k = string();
            ws();
            if (p_ >= s_.size() || s_[p_] != ':') error("expected ':'");
            ++p_;
            v.obj[k] = value();
            ws();
            if (p_ < s_.size() && s_[p_] == ',') { ++p_; continue; }
            if (p_ < s_.size() && s_[p_] == '}') { ++p_; return v; }
            error("expected ',' or '}'");
        }
    }
    Value array() {
        Value v;
        v.kind = Value::Array;
        ++p_;
        ws();
        if (p_ < s_.size() && s_[p_] == ']') { ++p_; return v; }
        for (;;) {
            v.arr.push_back(value());
            ws();
            if (p_ < s_.size() && s_[p_] == ',') { ++p_; continue; }
            if (p_ < s_.size() && s_[p_] == ']') { ++p_; return v; }
            error("expected ',' or ']'");
        }
    }
    static void utf8(std::string& out, uint32_t cp) {
        if (cp < 0x80) out += static_cast<char>(cp);
        else if (cp < 0x800) { out += static_cast<char>(0xC0 | (cp >> 6)); out += static_cast<char>(0x80 | (cp & 0x3F)); }
        else if (cp < 0x10000) {
            out += static_cast<char>(0xE0 | (cp >> 12));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        } else {
            out += static_cast<char>(0xF0 | (cp >> 18));
            out += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
            out += static_cast<char>(0x80 | (cp & 0x3F));
        }
    }
    uint32_t hex4() {
        if (p_ + 4 > s_.size()) error("short \\u escape");
        uint32_t v = 0;
        for (int i = 0; i < 4; ++i) {
            const char h = s_[p_++];
            v <<= 4;
            if (h >= '0' && h <= '9') v |= h - '0';
            else if (h >= 'a' && h <= 'f') v |= h - 'a' + 10;
            else if (h >= 'A' && h <= 'F') v |= h - 'A' + 10;
            else error("bad \\u escape");
        }
        return v;
    }
    std::string string() {
        ++p_;   // opening quote
        std::string out;
        while (p_ < s_.size()) {
            const char c = s_[p_++];
            if (c == '"') return out;
            if (c != '\\') { out += c; continue; }
            if (p_ >= s_.size()) break;
            const char e = s_[p_++];
            switch (e) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    uint32_t cp = hex4();
                    if (cp >= 0xD800 && cp < 0xDC00 && p_ + 6 <= s_.size() && s_[p_] == '\\' && s_[p_ + 1] == 'u') {
                        p_ += 2;
                        const uint32_t lo = hex4();
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(out, cp);
                    break;
                }
                default: error("bad escape");
            }
        }
        error("unterminated string");
    }
    Value number() {
        const size_t start = p_;
        if (s_[p_] == '-') ++p_;
        bool frac = false;
        while (p_ < s_.size()) {
            const char c = s_[p_];
            if (std::isdigit(static_cast<unsigned char>(c))) { ++p_; continue; }
            if (c == '.' || c == 'e' || c == 'E' || c == '+' || c == '-') { frac = true; ++p_; continue; }
            break;
        }
        const std::string t = s_.substr(start, p_ - start);
        Value v;
        v.kind = Value::Number;
        char* end = nullptr;
        v.num = std::strtod(t.c_str(), &end);
        if (!end || *end) error("bad number '" + t + "'");
        if (!frac) {
            v.is_int = true;
            v.i = std::strtoll(t.c_str(), nullptr, 10);
        }
        return v;
    }
};

inline Value parse(const std::string& text) { return Parser(text).parse(); }

}  // namespace json
}  // namespace bsb
