#include "json.h"

#include <cstdlib>
#include <stdexcept>

namespace gb {
namespace {

struct Parser {
    const std::string& s;
    size_t i = 0;
    explicit Parser(const std::string& t) : s(t) {}

    void ws() {
        while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
    }
    char peek() {
        ws();
        if (i >= s.size()) throw std::runtime_error("json: unexpected end");
        return s[i];
    }
    void expect(char c) {
        if (peek() != c) throw std::runtime_error(std::string("json: expected '") + c + "'");
        ++i;
    }
    static void put_utf8(std::string& o, uint32_t cp) {
        if (cp < 0x80) o += (char)cp;
        else if (cp < 0x800) { o += (char)(0xC0 | (cp >> 6)); o += (char)(0x80 | (cp & 0x3F)); }
        else if (cp < 0x10000) {
            o += (char)(0xE0 | (cp >> 12)); o += (char)(0x80 | ((cp >> 6) & 0x3F));
            o += (char)(0x80 | (cp & 0x3F));
        } else {
            o += (char)(0xF0 | (cp >> 18)); o += (char)(0x80 | ((cp >> 12) & 0x3F));
            o += (char)(0x80 | ((cp >> 6) & 0x3F)); o += (char)(0x80 | (cp & 0x3F));
        }
    }
    std::string string() {
        expect('"');
        std::string o;
        while (i < s.size() && s[i] != '"') {
            char c = s[i++];
            if (c != '\\') { o += c; continue; }
            if (i >= s.size()) break;
            char e = s[i++];
            switch (e) {
                case 'n': o += '\n'; break;
                case 't': o += '\t'; break;
                case 'r': o += '\r'; break;
                case 'b': o += '\b'; break;
                case 'f': o += '\f'; break;
                case 'u': {
                    uint32_t cp = (uint32_t)std::strtoul(s.substr(i, 4).c_str(), nullptr, 16);
                    i += 4;
                    if (cp >= 0xD800 && cp < 0xDC00 && i + 6 <= s.size() && s[i] == '\\' &&
                        s[i + 1] == 'u') {
                        uint32_t lo = (uint32_t)std::strtoul(s.substr(i + 2, 4).c_str(), nullptr, 16);
                        i += 6;
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    put_utf8(o, cp);
                    break;
                }
                default: o += e;
            }
        }
        if (i >= s.size()) throw std::runtime_error("json: unterminated string");
        ++i;
        return o;
    }
    JValue value() {
        char c = peek();
        JValue v;
        if (c == '{') {
            ++i;
            v.kind = JValue::OBJ;
            if (peek() == '}') { ++i; return v; }
            while (true) {
                std::string k = string();
                expect(':');
                v.obj[k] = value();
                char n = peek();
                ++i;
                if (n == '}') break;
                if (n != ',') throw std::runtime_error("json: expected ',' or '}'");
            }
        } else if (c == '[') {
            ++i;
            v.kind = JValue::ARR;
            if (peek() == ']') { ++i; return v; }
            while (true) {
                v.arr.push_back(value());
                char n = peek();
                ++i;
                if (n == ']') break;
                if (n != ',') throw std::runtime_error("json: expected ',' or ']'");
            }
        } else if (c == '"') {
            v.kind = JValue::STR;
            v.str = string();
        } else if (s.compare(i, 4, "true") == 0) {
            v.kind = JValue::BOOL; v.b = true; i += 4;
        } else if (s.compare(i, 5, "false") == 0) {
            v.kind = JValue::BOOL; v.b = false; i += 5;
        } else if (s.compare(i, 4, "null") == 0) {
            v.kind = JValue::NUL; i += 4;
        } else if (s.compare(i, 3, "NaN") == 0) {
            v.kind = JValue::NUM; v.num = 0.0 / 0.0; i += 3;
        } else {
            size_t st = i;
            bool is_int = true;
            if (s[i] == '-' || s[i] == '+') ++i;
            if (s.compare(i, 8, "Infinity") == 0) {
                i += 8;
                v.kind = JValue::NUM;
                v.num = (s[st] == '-') ? -1.0 / 0.0 : 1.0 / 0.0;
                return v;
            }
            while (i < s.size() && ((s[i] >= '0' && s[i] <= '9') || s[i] == '.' || s[i] == 'e' ||
                                    s[i] == 'E' || s[i] == '-' || s[i] == '+')) {
                if (s[i] == '.' || s[i] == 'e' || s[i] == 'E') is_int = false;
                ++i;
            }
            if (i == st) throw std::runtime_error("json: bad token");
            std::string t = s.substr(st, i - st);
            v.kind = JValue::NUM;
            v.num = std::strtod(t.c_str(), nullptr);
            v.is_int = is_int;
            v.inum = is_int ? std::strtoll(t.c_str(), nullptr, 10) : (int64_t)v.num;
        }
        return v;
    }
};

}  // namespace

JValue json_parse(const std::string& text) {
    Parser p(text);
    return p.value();
}

}  // namespace gb
