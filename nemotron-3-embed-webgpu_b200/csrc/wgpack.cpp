#include "wgpack.h"

#include <string.h>

#include <memory>

namespace nemo {
namespace {

// Minimal JSON reader for the .wgpack header: objects, arrays, strings
// (with escapes), numbers, true/false/null.
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
            // Encode the code unit as UTF-8 (surrogates are kept as-is).
            if (cp < 0x80) s->push_back((char)cp);
            else if (cp < 0x800) {
              s->push_back((char)(0xC0 | (cp >> 6)));
              s->push_back((char)(0x80 | (cp & 0x3F)));
            } else {
              s->push_back((char)(0xE0 | (cp >> 12)));
              s->push_back((char)(0x80 | ((cp >> 6) & 0x3F)));
              s->push_back((char)(0x80 | (cp & 0x3F)));
            }
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
    if (++depth > 64) return fail("JSON nested too deeply");
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

bool num_is(const Json* v, double x) { return v && v->kind == Json::kNum && v->num == x; }

}  // namespace

bool parse_wgpack(const uint8_t* data, size_t bytes, Pack* out, std::string* err) {
  // format.ts:147-166
  if (bytes < 12) { *err = "prepacked model is shorter than its prelude"; return false; }
  if (memcmp(data, "WGPACK02", 8) != 0) {
    *err = "invalid prepacked model magic \"" + std::string((const char*)data, 8) + "\"";
    return false;
  }
  uint32_t hlen;
  memcpy(&hlen, data + 8, 4);
  if (12ull + hlen > bytes) { *err = "prepacked model header extends past end of file"; return false; }
  Reader r{(const char*)data + 12, (const char*)data + 12 + hlen, {}};
  Json header;
  if (!r.parse(&header) || header.kind != Json::kObj) {
    *err = "invalid prepacked header JSON: " + (r.err.empty() ? std::string("not an object") : r.err);
    return false;
  }
  const Json* layout = header.get("layout");
  if (!num_is(header.get("version"), 2) || !layout || layout->kind != Json::kStr ||
      layout->str != "q4_0-tile32-compact-v2" || !num_is(header.get("tileRows"), 32) ||
      !num_is(header.get("blockValues"), 32) || !num_is(header.get("blockBytes"), 20)) {
    *err = "unsupported prepacked layout " + (layout && layout->kind == Json::kStr ? layout->str : "undefined");
    return false;
  }
  out->version = 2;
  if (const Json* sha = header.get("sourceSha256"); sha && sha->kind == Json::kStr) out->source_sha256 = sha->str;
  out->data_offset = (12ull + hlen + 255) / 256 * 256;
  const Json* tensors = header.get("tensors");
  if (!tensors || tensors->kind != Json::kArr) { *err = "prepacked header has no tensor list"; return false; }
  for (const Json& t : tensors->arr) {
    PackTensor pt;
    const Json* name = t.get("name");
    const Json* dims = t.get("dimensions");
    const Json* type = t.get("type");
    const Json* storage = t.get("storage");
    const Json* offset = t.get("offset");
    const Json* blen = t.get("byteLength");
    if (!name || name->kind != Json::kStr || !dims || dims->kind != Json::kArr || !type ||
        type->kind != Json::kNum || !storage || storage->kind != Json::kStr || !offset ||
        offset->kind != Json::kNum || !blen || blen->kind != Json::kNum || offset->num < 0 || blen->num < 0) {
      *err = "malformed prepacked tensor entry";
      return false;
    }
    pt.name = name->str;
    for (const Json& d : dims->arr) {
      if (d.kind != Json::kNum || d.num < 0) { *err = pt.name + " has invalid dimensions"; return false; }
      pt.dims.push_back((int64_t)d.num);
    }
    pt.type = (int)type->num;
    pt.offset = (uint64_t)offset->num;
    pt.byte_length = (uint64_t)blen->num;
    pt.byte_offset = out->data_offset + pt.offset;
    if (pt.byte_offset + pt.byte_length > bytes) { *err = pt.name + " extends past end of prepacked file"; return false; }
    if (out->tensors.count(pt.name)) { *err = "duplicate prepacked tensor " + pt.name; return false; }
    if (storage->str == "q4_0-tile32-compact") {
      if (pt.type != kQ4_0 || pt.dims.size() != 2) { *err = pt.name + " has invalid compact Q4_0 metadata"; return false; }
      pt.compact = true;
    } else if (storage->str != "raw") {
      *err = pt.name + " has unsupported storage " + storage->str;
      return false;
    }
    out->tensors[pt.name] = pt;
  }
  return true;
}

}  // namespace nemo
