// Minimal JSON reader for the .enargeia header (objects, arrays, strings, numbers, literals).
// Object members keep their file order.
#pragma once

#include <cstdlib>
#include <string>
#include <utility>
#include <vector>

namespace json {

struct Value {
    enum Type { Null, Bool, Num, Str, Arr, Obj } type = Null;
    double num = 0.0;
    bool b = false;
    std::string str;
    std::vector<Value> arr;
    std::vector<std::pair<std::string, Value>> obj;

    bool is_object() const { return type == Obj; }
    bool is_array() const { return type == Arr; }
    const Value* get(const std::string& key) const {
        for (auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};

namespace detail {

struct Parser {
    const std::string& s;
    size_t i = 0;
    std::string err;
    int depth = 0;

    explicit Parser(const std::string& src) : s(src) {}

    void ws() {
        while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
    }
    bool fail(const char* m) {
        if (err.empty()) err = std::string(m) + " at byte " + std::to_string(i);
        return false;
    }
    bool lit(const char* w) {
        size_t n = std::char_traits<char>::length(w);
        if (s.compare(i, n, w) != 0) return fail("bad literal");
        i += n;
        return true;
    }
    bool str(std::string& out) {
        if (i >= s.size() || s[i] != '"') return fail("expected string");
        ++i;
        out.clear();
        while (i < s.size() && s[i] != '"') {
            char c = s[i++];
            if (c == '\\') {
                if (i >= s.size()) return fail("bad escape");
                char e = s[i++];
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
                        if (i + 4 > s.size()) return fail("bad \\u escape");
                        unsigned cp = (unsigned)std::strtoul(s.substr(i, 4).c_str(), nullptr, 16);
                        i += 4;
                        if (cp < 0x80) out += (char)cp;
                        else if (cp < 0x800) { out += (char)(0xC0 | (cp >> 6)); out += (char)(0x80 | (cp & 0x3F)); }
                        else { out += (char)(0xE0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 0x3F)); out += (char)(0x80 | (cp & 0x3F)); }
                        break;
                    }
                    default: return fail("bad escape");
                }
            } else {
                out += c;
            }
        }
        if (i >= s.size()) return fail("unterminated string");
        ++i;
        return true;
    }
    bool value(Value& v) {
        if (++depth > 64) return fail("nesting too deep");
        ws();
        if (i >= s.size()) return fail("unexpected end");
        char c = s[i];
        bool ok = true;
        if (c == '{') {
            v.type = Value::Obj;
            ++i;
            ws();
            if (i < s.size() && s[i] == '}') { ++i; --depth; return true; }
            for (;;) {
                ws();
                std::string k;
                if (!str(k)) return false;
                ws();
                if (i >= s.size() || s[i] != ':') return fail("expected ':'");
                ++i;
                v.obj.emplace_back(std::move(k), Value());
                if (!value(v.obj.back().second)) return false;
                ws();
                if (i < s.size() && s[i] == ',') { ++i; continue; }
                if (i < s.size() && s[i] == '}') { ++i; break; }
                return fail("expected ',' or '}'");
            }
        } else if (c == '[') {
            v.type = Value::Arr;
            ++i;
            ws();
            if (i < s.size() && s[i] == ']') { ++i; --depth; return true; }
            for (;;) {
                v.arr.emplace_back();
                if (!value(v.arr.back())) return false;
                ws();
                if (i < s.size() && s[i] == ',') { ++i; continue; }
                if (i < s.size() && s[i] == ']') { ++i; break; }
                return fail("expected ',' or ']'");
            }
        } else if (c == '"') {
            v.type = Value::Str;
            ok = str(v.str);
        } else if (c == 't') {
            v.type = Value::Bool; v.b = true; ok = lit("true");
        } else if (c == 'f') {
            v.type = Value::Bool; v.b = false; ok = lit("false");
        } else if (c == 'n') {
            v.type = Value::Null; ok = lit("null");
        } else {
            const char* b = s.c_str() + i;
            char* e = nullptr;
            v.num = std::strtod(b, &e);
            if (e == b) return fail("bad number");
            v.type = Value::Num;
            i += (size_t)(e - b);
        }
        --depth;
        return ok;
    }
};

}  // namespace detail

inline bool parse(const std::string& src, Value& out, std::string& err) {
    detail::Parser p(src);
    out = Value();
    if (!p.value(out)) { err = p.err; return false; }
    p.ws();
    if (p.i != src.size()) { err = "trailing bytes after the header object"; return false; }
    return true;
}

}  // namespace json
