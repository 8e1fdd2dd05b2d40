// Minimal JSON reader for config.json and safetensors headers.
#pragma once

#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace msb {

struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0.0;
    bool is_int = false;
    std::string str;
    std::vector<Json> arr;
    std::map<std::string, Json> obj;

    bool has(const std::string& k) const { return kind == Object && obj.count(k) != 0; }
    const Json* get(const std::string& k) const {
        if (kind != Object) return nullptr;
        auto it = obj.find(k);
        return it == obj.end() ? nullptr : &it->second;
    }
    // Typed lookups with defaults (mirror Swift's `d[k] as? T ?? default`).
    long long int_or(const std::string& k, long long def) const {
        const Json* v = get(k);
        if (!v || v->kind != Number) return def;
        return (long long)v->num;
    }
    double num_or(const std::string& k, double def) const {
        const Json* v = get(k);
        return (v && v->kind == Number) ? v->num : def;
    }
    bool bool_or(const std::string& k, bool def) const {
        const Json* v = get(k);
        return (v && v->kind == Bool) ? v->b : def;
    }
    std::string str_or(const std::string& k, const std::string& def) const {
        const Json* v = get(k);
        return (v && v->kind == String) ? v->str : def;
    }

    static Json parse(const char* p, size_t n);
};

namespace detail {

struct Parser {
    const char* s;
    size_t n, i = 0;
    [[noreturn]] void fail(const char* what) const {
        throw std::runtime_error(std::string("json: ") + what + " at offset " + std::to_string(i));
    }
    void ws() {
        while (i < n && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
    }
    bool lit(const char* w) {
        size_t k = 0;
        while (w[k]) {
            if (i + k >= n || s[i + k] != w[k]) return false;
            ++k;
        }
        i += k;
        return true;
    }
    std::string string_() {
        if (s[i] != '"') fail("expected string");
        ++i;
        std::string out;
        while (i < n && s[i] != '"') {
            char c = s[i++];
            if (c == '\\') {
                if (i >= n) fail("bad escape");
                char e = s[i++];
                switch (e) {
                    case 'n': out += '\n'; break;
                    case 't': out += '\t'; break;
                    case 'r': out += '\r'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'u': {
                        if (i + 4 > n) fail("bad \\u");
                        unsigned cp = (unsigned)std::strtoul(std::string(s + i, 4).c_str(), nullptr, 16);
                        i += 4;
                        if (cp < 0x80) out += (char)cp;
                        else if (cp < 0x800) {
                            out += (char)(0xC0 | (cp >> 6));
                            out += (char)(0x80 | (cp & 0x3F));
                        } else {
                            out += (char)(0xE0 | (cp >> 12));
                            out += (char)(0x80 | ((cp >> 6) & 0x3F));
                            out += (char)(0x80 | (cp & 0x3F));
                        }
                        break;
                    }
                    default: out += e;
                }
            } else {
                out += c;
            }
        }
        if (i >= n) fail("unterminated string");
        ++i;
        return out;
    }
    Json value(int depth) {
        if (depth > 64) fail("nesting too deep");
        ws();
        if (i >= n) fail("unexpected end");
        Json v;
        char c = s[i];
        if (c == '{') {
            ++i;
            v.kind = Json::Object;
            ws();
            if (i < n && s[i] == '}') { ++i; return v; }
            while (true) {
                ws();
                std::string k = string_();
                ws();
                if (i >= n || s[i] != ':') fail("expected ':'");
                ++i;
                v.obj[k] = value(depth + 1);
                ws();
                if (i < n && s[i] == ',') { ++i; continue; }
                if (i < n && s[i] == '}') { ++i; break; }
                fail("expected ',' or '}'");
            }
        } else if (c == '[') {
            ++i;
            v.kind = Json::Array;
            ws();
            if (i < n && s[i] == ']') { ++i; return v; }
            while (true) {
                v.arr.push_back(value(depth + 1));
                ws();
                if (i < n && s[i] == ',') { ++i; continue; }
                if (i < n && s[i] == ']') { ++i; break; }
                fail("expected ',' or ']'");
            }
        } else if (c == '"') {
            v.kind = Json::String;
            v.str = string_();
        } else if (lit("true")) {
            v.kind = Json::Bool;
            v.b = true;
        } else if (lit("false")) {
            v.kind = Json::Bool;
        } else if (lit("null")) {
            v.kind = Json::Null;
        } else if (c == '-' || (c >= '0' && c <= '9')) {
            size_t st = i;
            bool integral = true;
            while (i < n && (s[i] == '-' || s[i] == '+' || s[i] == '.' || s[i] == 'e' || s[i] == 'E' ||
                             (s[i] >= '0' && s[i] <= '9'))) {
                if (s[i] == '.' || s[i] == 'e' || s[i] == 'E') integral = false;
                ++i;
            }
            v.kind = Json::Number;
            v.num = std::strtod(std::string(s + st, i - st).c_str(), nullptr);
            v.is_int = integral;
        } else {
            fail("unexpected character");
        }
        return v;
    }
};

}  // namespace detail

inline Json Json::parse(const char* p, size_t n) {
    detail::Parser ps{p, n};
    Json v = ps.value(0);
    return v;
}

}  // namespace msb
