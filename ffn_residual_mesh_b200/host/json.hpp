// Minimal JSON reader for artifact manifests (objects, arrays, strings, numbers,
// true/false/null). Errors throw std::runtime_error, which the runners report as
// "error: ..." with exit status 1 like the reference runners.
#pragma once

#include <cctype>
#include <cstdint>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace ffnrm_host {

struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<Json> arr;
    std::map<std::string, Json> obj;

    bool has(const std::string &k) const { return kind == Object && obj.count(k) != 0; }
    const Json &at(const std::string &k) const {
        if (kind != Object) throw std::runtime_error("manifest: expected an object around \"" + k + "\"");
        auto it = obj.find(k);
        if (it == obj.end()) throw std::runtime_error("manifest missing \"" + k + "\"");
        return it->second;
    }
    int64_t integer() const {
        if (kind != Number || num != double(int64_t(num))) throw std::runtime_error("manifest value is not an integer");
        return int64_t(num);
    }
    const std::string &text() const {
        if (kind != String) throw std::runtime_error("manifest value is not a string");
        return str;
    }

    static Json parse(const std::string &s) {
        size_t i = 0;
        Json v = value(s, i);
        ws(s, i);
        if (i != s.size()) throw std::runtime_error("manifest: trailing characters");
        return v;
    }

private:
    static void ws(const std::string &s, size_t &i) {
        while (i < s.size() && (s[i] == ' ' || s[i] == '\t' || s[i] == '\n' || s[i] == '\r')) ++i;
    }
    static void expect(const std::string &s, size_t &i, char c) {
        ws(s, i);
        if (i >= s.size() || s[i] != c) throw std::runtime_error(std::string("manifest: expected '") + c + "'");
        ++i;
    }
    static std::string string_lit(const std::string &s, size_t &i) {
        expect(s, i, '"');
        std::string out;
        while (i < s.size() && s[i] != '"') {
            char c = s[i++];
            if (c != '\\') {
                out += c;
                continue;
            }
            if (i >= s.size()) break;
            const char e = s[i++];
            switch (e) {
                case 'n': out += '\n'; break;
                case 't': out += '\t'; break;
                case 'r': out += '\r'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'u': {
                    if (i + 4 > s.size()) throw std::runtime_error("manifest: bad \\u escape");
                    const unsigned cp = unsigned(std::stoul(s.substr(i, 4), nullptr, 16));
                    i += 4;
                    // UTF-8 encode (basic multilingual plane; surrogates kept as-is)
                    if (cp < 0x80) {
                        out += char(cp);
                    } else if (cp < 0x800) {
                        out += char(0xC0 | (cp >> 6));
                        out += char(0x80 | (cp & 0x3F));
                    } else {
                        out += char(0xE0 | (cp >> 12));
                        out += char(0x80 | ((cp >> 6) & 0x3F));
                        out += char(0x80 | (cp & 0x3F));
                    }
                    break;
                }
                default: out += e;
            }
        }
        if (i >= s.size()) throw std::runtime_error("manifest: unterminated string");
        ++i;
        return out;
    }
    static Json value(const std::string &s, size_t &i) {
        ws(s, i);
        if (i >= s.size()) throw std::runtime_error("manifest: unexpected end");
        Json v;
        const char c = s[i];
        if (c == '{') {
            v.kind = Object;
            ++i;
            ws(s, i);
            if (i < s.size() && s[i] == '}') {
                ++i;
                return v;
            }
            for (;;) {
                std::string k = string_lit(s, i);
                expect(s, i, ':');
                v.obj[k] = value(s, i);
                ws(s, i);
                if (i < s.size() && s[i] == ',') {
                    ++i;
                    continue;
                }
                expect(s, i, '}');
                return v;
            }
        }
        if (c == '[') {
            v.kind = Array;
            ++i;
            ws(s, i);
            if (i < s.size() && s[i] == ']') {
                ++i;
                return v;
            }
            for (;;) {
                v.arr.push_back(value(s, i));
                ws(s, i);
                if (i < s.size() && s[i] == ',') {
                    ++i;
                    continue;
                }
                expect(s, i, ']');
                return v;
            }
        }
        if (c == '"') {
            v.kind = String;
            v.str = string_lit(s, i);
            return v;
        }
        if (s.compare(i, 4, "true") == 0) {
            v.kind = Bool;
            v.b = true;
            i += 4;
            return v;
        }
        if (s.compare(i, 5, "false") == 0) {
            v.kind = Bool;
            i += 5;
            return v;
        }
        if (s.compare(i, 4, "null") == 0) {
            i += 4;
            return v;
        }
        size_t end = i;
        while (end < s.size() && (std::isdigit(static_cast<unsigned char>(s[end])) || s[end] == '-' || s[end] == '+' ||
                                  s[end] == '.' || s[end] == 'e' || s[end] == 'E'))
            ++end;
        if (end == i) throw std::runtime_error("manifest: unexpected character");
        v.kind = Number;
        v.num = std::stod(s.substr(i, end - i));
        i = end;
        return v;
    }
};

}  // namespace ffnrm_host
