#include "wgpack.h"
#include "json_reader.h"

#include <string.h>

#include <memory>

namespace nemo {
namespace {

using json::Json;
using json::Reader;

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
