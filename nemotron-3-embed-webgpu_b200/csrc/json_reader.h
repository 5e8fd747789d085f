// Minimal JSON reader shared by the .wgpack parser and the tokenizer loader.
#pragma once

#include <stdlib.h>
#include <string.h>

#include <string>
#include <utility>
#include <vector>

namespace nemo {
namespace json {

// Minimal JSON reader (the .wgpack header, tokenizer.json): objects, arrays,
// strings (with escapes, surrogate pairs joined), numbers, true/false/null.
struct Json {
  enum Kind { kNull, kBool, kNum, kStr, kArr, kObj } kind = kNull;
  bool b = false;
  double num = 0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;
  const Json* get(const char* key) const {
    for (const auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

inline void append_utf8(std::string* s, unsigned cp) {
  if (cp < 0x80) {
    s->push_back((char)cp);
  } else if (cp < 0x800) {
    s->push_back((char)(0xC0 | (cp >> 6)));
    s->push_back((char)(0x80 | (cp & 0x3F)));
  } else if (cp < 0x10000) {
    s->push_back((char)(0xE0 | (cp >> 12)));
    s->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
    s->push_back((char)(0x80 | (cp & 0x3F)));
  } else {
    s->push_back((char)(0xF0 | (cp >> 18)));
    s->push_back((char)(0x80 | ((cp >> 12) & 0x3F)));
    s->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
    s->push_back((char)(0x80 | (cp & 0x3F)));
  }
}

struct Reader {
  const char* p;
  const char* end;
  std::string err;
  int depth = 0;

  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool fail(const char* m) {
    if (err.empty()) err = m;
    return false;
  }
  bool parse_string(std::string* s) {
    if (p >= end || *p != '"') return fail("expected string");
    ++p;
    while (p < end && *p != '"') {
      char c = *p++;
      if (c == '\\') {
        if (p >= end) return fail("bad escape");
        char e = *p++;
        switch (e) {
          case '"': s->push_back('"'); break;
          case '\\': s->push_back('\\'); break;
          case '/': s->push_back('/'); break;
          case 'b': s->push_back('\b'); break;
          case 'f': s->push_back('\f'); break;
          case 'n': s->push_back('\n'); break;
          case 'r': s->push_back('\r'); break;
          case 't': s->push_back('\t'); break;
          case 'u': {
            if (end - p < 4) return fail("bad \\u escape");
            unsigned cp = 0;
            for (int i = 0; i < 4; ++i) {
              char h = *p++;
              cp <<= 4;
              if (h >= '0' && h <= '9') cp |= h - '0';
              else if (h >= 'a' && h <= 'f') cp |= h - 'a' + 10;
              else if (h >= 'A' && h <= 'F') cp |= h - 'A' + 10;
              else return fail("bad \\u escape");
            }
            // A high surrogate followed by \uDC00..\uDFFF is one code point.
            if (cp >= 0xD800 && cp < 0xDC00 && end - p >= 6 && p[0] == '\\' && p[1] == 'u') {
              unsigned lo = 0;
              bool ok = true;
              for (int i = 2; i < 6; ++i) {
                char h = p[i];
                lo <<= 4;
                if (h >= '0' && h <= '9') lo |= h - '0';
                else if (h >= 'a' && h <= 'f') lo |= h - 'a' + 10;
                else if (h >= 'A' && h <= 'F') lo |= h - 'A' + 10;
                else ok = false;
              }
              if (ok && lo >= 0xDC00 && lo < 0xE000) {
                cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                p += 6;
              }
            }
            append_utf8(s, cp);
            break;
          }
          default: return fail("bad escape");
        }
      } else {
        s->push_back(c);
      }
    }
    if (p >= end) return fail("unterminated string");
    ++p;
    return true;
  }
  bool parse(Json* v) {
    if (++depth > 128) return fail("JSON nested too deeply");
    ws();
    if (p >= end) return fail("unexpected end of JSON");
    bool ok = true;
    if (*p == '{') {
      ++p;
      v->kind = Json::kObj;
      ws();
      if (p < end && *p == '}') {
        ++p;
      } else {
        for (;;) {
          ws();
          std::string key;
          if (!parse_string(&key)) { ok = false; break; }
          ws();
          if (p >= end || *p != ':') { ok = fail("expected ':'"); break; }
          ++p;
          Json child;
          if (!parse(&child)) { ok = false; break; }
          v->obj.emplace_back(std::move(key), std::move(child));
          ws();
          if (p < end && *p == ',') { ++p; continue; }
          if (p < end && *p == '}') { ++p; break; }
          ok = fail("expected ',' or '}'");
          break;
        }
      }
    } else if (*p == '[') {
      ++p;
      v->kind = Json::kArr;
      ws();
      if (p < end && *p == ']') {
        ++p;
      } else {
        for (;;) {
          Json child;
          if (!parse(&child)) { ok = false; break; }
          v->arr.push_back(std::move(child));
          ws();
          if (p < end && *p == ',') { ++p; continue; }
          if (p < end && *p == ']') { ++p; break; }
          ok = fail("expected ',' or ']'");
          break;
        }
      }
    } else if (*p == '"') {
      v->kind = Json::kStr;
      ok = parse_string(&v->str);
    } else if (end - p >= 4 && !strncmp(p, "true", 4)) {
      v->kind = Json::kBool; v->b = true; p += 4;
    } else if (end - p >= 5 && !strncmp(p, "false", 5)) {
      v->kind = Json::kBool; v->b = false; p += 5;
    } else if (end - p >= 4 && !strncmp(p, "null", 4)) {
      v->kind = Json::kNull; p += 4;
    } else {
      const char* s = p;
      while (p < end && (strchr("+-0123456789.eE", *p) != nullptr)) ++p;
      if (p == s) return fail("unexpected character in JSON");
      v->kind = Json::kNum;
      v->num = strtod(std::string(s, p).c_str(), nullptr);
    }
    --depth;
    return ok;
  }
};

}  // namespace json
}  // namespace nemo
