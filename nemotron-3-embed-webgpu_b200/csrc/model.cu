// Model load: parse the .wgpack, validate every tensor the forward needs,
// upload one replica per device and decode each projection once to its
// effective f16 weights (src/webgpu/model.ts:253-320 + the weight decode of
// every matmul pipeline). Each projection is kept twice: its tile-slab image
// (the quantised blocks re-tiled for the fused-dequant kernels) and the f16
// copy for the batched GEMM; the pack's own block layout is only a temporary
// decode source. Device memory per replica: ~0.53 GB tile-slab + 1.74 GB f16 +
// 0.22 GB token table, a small share of a B200's 180 GB. B200-tiled packs
// (nemo_pack_b200) already hold the tile-slab images, so their load skips the
// host re-tile and decodes the f16 copy from the images on the device.
#include <string.h>

#include <algorithm>

#include "runtime.h"

namespace nemo {
namespace {

struct PartSpec {
  const PackTensor* t;
  int fmt;
};

const char* kFused[4] = {"attn_qkv", "attn_output", "ffn_gate_up", "ffn_down"};
const std::vector<std::vector<const char*>> kParts = {
    {"attn_q", "attn_k", "attn_v"}, {"attn_output"}, {"ffn_gate", "ffn_up"}, {"ffn_down"}};

int fmt_of(const PackTensor& t, std::string* err) {
  if (t.compact) return kSegQ40Tile32;
  switch (t.type) {
    case kQ4_K: return kSegQ4K;
    case kQ6_K: return kSegQ6K;
    case kQ4_0: return kSegQ40;
    default:
      *err = "unsupported matrix type " + std::to_string(t.type) + " for " + t.name;  // model.ts:318
      return -1;
  }
}

size_t expected_bytes(int fmt, int64_t rows, int64_t k) {
  switch (fmt) {
    case kSegQ4K: return (size_t)(rows * (k / 256) * 144);
    case kSegQ6K: return (size_t)(rows * (k / 256) * 210);
    case kSegQ40: return (size_t)(rows * (k / 32) * 18);
    default: return (size_t)(((rows + 31) / 32) * (k / 32) * 32 * 20);
  }
}

// B200-tiled packs (written by nemo_pack_b200) carry each projection's
// tile-slab image as one raw tensor "blk.<l>.<fused name>.b200_tiles":
// [SkinnyTile table of n/128 entries, padded to 256 B][chunks], chunk
// (tile, slab) at chunks + offset + slab * chunk_bytes.
std::string b200_name(int l, int which) { return "blk." + std::to_string(l) + "." + kFused[which] + ".b200_tiles"; }

size_t b200_table_bytes(int n) { return ((size_t)(n / 128) * sizeof(SkinnyTile) + 255) / 256 * 256; }

// Checks one image against the projection's shape; on success *tiles holds its table.
int parse_b200_image(const uint8_t* bytes, uint64_t len, int which, std::vector<SkinnyTile>* tiles, int* chunk_max,
                     const std::string& name) {
  const int n = kProjN[which], slabs = kProjK[which] / 256, ntiles = n / 128;
  const size_t table = b200_table_bytes(n);
  if (len < table) {
    set_error(name + " is shorter than its tile table");
    return kErrFormat;
  }
  tiles->resize(ntiles);
  memcpy(tiles->data(), bytes, ntiles * sizeof(SkinnyTile));
  uint64_t expect = 0;
  *chunk_max = 0;
  for (int t = 0; t < ntiles; ++t) {
    const SkinnyTile& ti = (*tiles)[t];
    auto region = [](int f) { return f == kSegQ6K ? 64 * 210 : 64 * 144; };
    if (ti.fmt[0] > kSegQ40 || ti.fmt[1] > kSegQ40 || ti.offset != expect ||
        ti.chunk_bytes != (uint32_t)(region(ti.fmt[0]) + region(ti.fmt[1]))) {
      set_error(name + " has an inconsistent tile table (tile " + std::to_string(t) + ")");
      return kErrFormat;
    }
    expect += (uint64_t)ti.chunk_bytes * slabs;
    *chunk_max = std::max(*chunk_max, (int)ti.chunk_bytes);
  }
  if (table + expect != len) {
    set_error(name + " has " + std::to_string(len) + " bytes; its tile table describes " +
              std::to_string(table + expect));
    return kErrFormat;
  }
  return kOk;
}

template <typename T>
int dev_alloc(DeviceModel& dm, T** p, size_t bytes) {
  void* v = nullptr;
  NEMO_CUDA_TRY(cudaMalloc(&v, bytes));
  dm.allocations.push_back(v);
  dm.bytes += bytes;
  *p = reinterpret_cast<T*>(v);
  return kOk;
}

// Resolves the segments of projection `which` of layer l: one compact fused
// tensor, or the per-part raw tensors in output-column order.
int resolve(const Pack& pack, int l, int which, std::vector<PartSpec>* parts, std::string* err) {
  const std::string prefix = "blk." + std::to_string(l) + ".";
  auto it = pack.tensors.find(prefix + kFused[which] + ".weight");
  if (it != pack.tensors.end() && (it->second.compact || kParts[which].size() == 1)) {
    int fmt = fmt_of(it->second, err);
    if (fmt < 0) return kErrFormat;
    parts->push_back({&it->second, fmt});
    return kOk;
  }
  for (const char* pn : kParts[which]) {
    auto jt = pack.tensors.find(prefix + pn + ".weight");
    if (jt == pack.tensors.end()) {
      *err = "missing tensor " + prefix + (kParts[which].size() > 1 ? kFused[which] : pn) + ".weight";
      return kErrFormat;
    }
    int fmt = fmt_of(jt->second, err);
    if (fmt < 0) return kErrFormat;
    parts->push_back({&jt->second, fmt});
  }
  return kOk;
}

// Builds the tile-slab image of one projection from its pack segments (host
// bytes). Tile t holds matrix rows [128t, 128t+128), or for gate/up
// (interleave) gate rows [64t, 64t+64) then up rows [n/2 + 64t, +64), so the
// fused SwiGLU epilogue finds both halves of its outputs in one tile.
int build_tile_slab(const uint8_t* file, const std::vector<PartSpec>& parts, int n, int k, bool interleave,
                    TileSlabImage* img) {
  struct HostSeg {
    int fmt, row0, rows;
    const uint8_t* data;
  };
  std::vector<HostSeg> segs;
  int row0 = 0;
  for (const PartSpec& ps : parts) {
    segs.push_back({ps.fmt, row0, (int)ps.t->dims[1], file + ps.t->byte_offset});
    row0 += (int)ps.t->dims[1];
  }
  if (n % 128 || k % 256) {
    set_error("projection shape is not a multiple of the 128 x 256 tile");
    return kErrFormat;
  }
  const int ntiles = n / 128, slabs = k / 256;
  auto seg_of = [&](int row) -> const HostSeg* {
    for (const HostSeg& s : segs)
      if (row >= s.row0 && row < s.row0 + s.rows) return &s;
    return nullptr;
  };
  auto tile_fmt = [](int segfmt) { return segfmt == kSegQ4K ? kSegQ4K : segfmt == kSegQ6K ? kSegQ6K : kSegQ40; };
  auto region = [](int fmt) { return fmt == kSegQ6K ? 64 * 210 : 64 * 144; };
  std::vector<int> base(ntiles * 2);
  std::vector<const HostSeg*> tseg(ntiles * 2);
  img->tiles.resize(ntiles);
  uint64_t offset = 0;
  img->chunk_max = 0;
  for (int t = 0; t < ntiles; ++t) {
    for (int h = 0; h < 2; ++h) {
      const int r = interleave ? (h == 0 ? t * 64 : n / 2 + t * 64) : t * 128 + 64 * h;
      const HostSeg* s = seg_of(r);
      if (!s || seg_of(r + 63) != s) {
        set_error("projection segments must be aligned to 64-row groups");
        return kErrFormat;
      }
      base[t * 2 + h] = r;
      tseg[t * 2 + h] = s;
      img->tiles[t].fmt[h] = (uint8_t)tile_fmt(s->fmt);
    }
    img->tiles[t].chunk_bytes = region(img->tiles[t].fmt[0]) + region(img->tiles[t].fmt[1]);
    img->tiles[t].offset = (uint32_t)offset;
    offset += (uint64_t)img->tiles[t].chunk_bytes * slabs;
    img->chunk_max = std::max(img->chunk_max, (int)img->tiles[t].chunk_bytes);
  }
  if (offset >= (1ull << 32)) {
    set_error("projection too large for 32-bit tile offsets");
    return kErrFormat;
  }
  img->bytes.assign(offset, 0);
  const int kb32 = k / 32;
  for (int t = 0; t < ntiles; ++t)
    for (int s = 0; s < slabs; ++s)
      for (int h = 0; h < 2; ++h) {
        const HostSeg& sg = *tseg[t * 2 + h];
        const int fmt = img->tiles[t].fmt[h];
        uint8_t* reg = img->bytes.data() + img->tiles[t].offset + (size_t)s * img->tiles[t].chunk_bytes +
                       (h ? region(img->tiles[t].fmt[0]) : 0);
        for (int rr = 0; rr < 64; ++rr) {
          const int L = base[t * 2 + h] + rr - sg.row0;
          if (sg.fmt == kSegQ4K) {
            memcpy(reg + rr * 144, sg.data + ((size_t)L * slabs + s) * 144, 144);
          } else if (sg.fmt == kSegQ6K) {
            const uint8_t* src = sg.data + ((size_t)L * slabs + s) * 210;
            memcpy(reg + rr * 208, src, 208);
            memcpy(reg + 64 * 208 + rr * 2, src + 208, 2);
          } else {
            uint8_t* dst = reg + rr * 144;
            for (int b = 0; b < 8; ++b) {
              const uint8_t* blk;
              const uint8_t* qs;
              if (sg.fmt == kSegQ40) {
                blk = sg.data + ((size_t)L * kb32 + s * 8 + b) * 18;
                qs = blk + 2;
              } else {  // q4_0-tile32-compact (format.ts:84-97)
                blk = sg.data + ((((size_t)(L / 32)) * kb32 + s * 8 + b) * 32 + (L % 32)) * 20;
                qs = blk + 4;
              }
              dst[2 * b] = blk[0];
              dst[2 * b + 1] = blk[1];
              memcpy(dst + 16 + b * 16, qs, 16);
            }
          }
          (void)fmt;
        }
      }
  return kOk;
}

int upload_replica(const uint8_t* file, const Pack& pack, int n_layers, int vocab, DeviceModel& dm,
                   nemo_model* m, bool count, const std::vector<TileSlabImage>& images) {
  NEMO_CUDA_TRY(cudaSetDevice(dm.device));
  const PackTensor& te = pack.tensors.at("token_embd.weight");
  if (dev_alloc(dm, &dm.embd, te.byte_length)) return kErrCuda;
  NEMO_CUDA_TRY(cudaMemcpy(dm.embd, file + te.byte_offset, te.byte_length, cudaMemcpyHostToDevice));
  auto norm = [&](const std::string& name, float** dst) -> int {
    const PackTensor& t = pack.tensors.at(name);
    if (dev_alloc(dm, dst, t.byte_length)) return kErrCuda;
    NEMO_CUDA_TRY(cudaMemcpy(*dst, file + t.byte_offset, t.byte_length, cudaMemcpyHostToDevice));
    return kOk;
  };
  for (int l = 0; l < n_layers; ++l) {
    if (norm("blk." + std::to_string(l) + ".attn_norm.weight", &dm.attn_norm[l])) return kErrCuda;
    if (norm("blk." + std::to_string(l) + ".ffn_norm.weight", &dm.ffn_norm[l])) return kErrCuda;
  }
  if (norm("output_norm.weight", &dm.output_norm)) return kErrCuda;

  const bool b200 = pack.tensors.count(b200_name(0, 0)) != 0;
  for (int l = 0; l < n_layers; ++l) {
    for (int which = 0; which < 4; ++which) {
      Projection& pr = dm.proj[l][which];
      pr.n = kProjN[which];
      pr.k = kProjK[which];
      if (dev_alloc(dm, &pr.w16, (size_t)pr.n * pr.k * 2)) return kErrCuda;
      if (b200) {
        // the pack holds the device layout: upload it and decode the f16 weights from it
        const PackTensor& t = pack.tensors.at(b200_name(l, which));
        std::vector<SkinnyTile> tiles;
        int chunk_max = 0;
        if (int rc = parse_b200_image(file + t.byte_offset, t.byte_length, which, &tiles, &chunk_max, t.name)) return rc;
        const size_t table = b200_table_bytes(pr.n);
        pr.tiles = (int)tiles.size();
        pr.slabs = pr.k / 256;
        pr.chunk_max = chunk_max;
        pr.packed_bytes = t.byte_length - table;
        if (dev_alloc(dm, &pr.packed, pr.packed_bytes) || dev_alloc(dm, &pr.d_tiles, tiles.size() * sizeof(SkinnyTile)))
          return kErrCuda;
        NEMO_CUDA_TRY(cudaMemcpy(pr.packed, file + t.byte_offset + table, pr.packed_bytes, cudaMemcpyHostToDevice));
        NEMO_CUDA_TRY(cudaMemcpy(pr.d_tiles, tiles.data(), tiles.size() * sizeof(SkinnyTile), cudaMemcpyHostToDevice));
        NEMO_CUDA_TRY(launch_decode_image(pr.packed, pr.d_tiles, pr.tiles, pr.slabs, which == kProjGateUp, pr.n, pr.k,
                                          pr.w16, 0));
        if (count) {
          m->kquant++;
          m->packed_bytes += pr.packed_bytes;
        }
        for (int b = 0; b < kNumBn; ++b)
          if (int rc = make_tmap_f16(&pr.map[b], pr.w16, (uint64_t)pr.k, (uint64_t)pr.n, 64, kBnChoices[b])) return rc;
        continue;
      }
      std::vector<PartSpec> parts;
      std::string err;
      if (resolve(pack, l, which, &parts, &err)) {
        set_error(err);
        return kErrFormat;
      }
      int row0 = 0;
      for (const PartSpec& ps : parts) {
        Segment sg;
        sg.fmt = ps.fmt;
        sg.row0 = row0;
        sg.rows = (int)ps.t->dims[1];
        sg.bytes = ps.t->byte_length;
        // the pack's blocks only feed the decode: a temporary device copy
        uint8_t* raw = nullptr;
        NEMO_CUDA_TRY(cudaMalloc(&raw, sg.bytes));
        cudaError_t e = cudaMemcpy(raw, file + ps.t->byte_offset, sg.bytes, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) e = launch_decode(sg.fmt, raw, sg.rows, pr.k, pr.w16 + (size_t)row0 * pr.k, nullptr, 0);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        cudaFree(raw);
        if (e != cudaSuccess) {
          set_error(std::string("CUDA error: ") + cudaGetErrorString(e) + " decoding " + ps.t->name);
          return kErrCuda;
        }
        if (count) {
          if (sg.fmt == kSegQ40Tile32) m->compact++;
          else m->kquant++;
          m->packed_bytes += sg.bytes;
        }
        row0 += sg.rows;
        pr.segs.push_back(sg);
      }
      for (int b = 0; b < kNumBn; ++b)
        if (int rc = make_tmap_f16(&pr.map[b], pr.w16, (uint64_t)pr.k, (uint64_t)pr.n, 64, kBnChoices[b])) return rc;
      const TileSlabImage& img = images[l * 4 + which];
      pr.tiles = (int)img.tiles.size();
      pr.slabs = pr.k / 256;
      pr.chunk_max = img.chunk_max;
      pr.packed_bytes = img.bytes.size();
      if (dev_alloc(dm, &pr.packed, img.bytes.size())) return kErrCuda;
      NEMO_CUDA_TRY(cudaMemcpy(pr.packed, img.bytes.data(), img.bytes.size(), cudaMemcpyHostToDevice));
      if (dev_alloc(dm, &pr.d_tiles, img.tiles.size() * sizeof(SkinnyTile))) return kErrCuda;
      NEMO_CUDA_TRY(cudaMemcpy(pr.d_tiles, img.tiles.data(), img.tiles.size() * sizeof(SkinnyTile),
                               cudaMemcpyHostToDevice));
    }
  }
  NEMO_CUDA_TRY(cudaDeviceSynchronize());
  return kOk;
}

// Validation of everything the forward reads (format.ts checks are done by
// parse_wgpack; these mirror model.ts:278,309,315,318 for this build).
int validate(const Pack& pack, int* n_layers, int* vocab) {
  int layers = 0;
  while (layers < kMaxLayers && pack.tensors.count("blk." + std::to_string(layers) + ".attn_norm.weight")) ++layers;
  if (layers < kMergeAfterLayer + 1) {
    set_error("pack has " + std::to_string(layers) + " layers; expected 16 (at least 5 for reduced test packs)");
    return kErrFormat;
  }
  auto te = pack.tensors.find("token_embd.weight");
  if (te == pack.tensors.end()) {
    set_error("missing tensor token_embd.weight");
    return kErrFormat;
  }
  const PackTensor& t = te->second;
  if (t.type != kQ6_K || t.compact || t.dims.size() != 2 || t.dims[0] != kHidden || t.dims[1] < 1 ||
      t.byte_length != (uint64_t)t.dims[1] * (kHidden / 256) * 210) {
    set_error("token_embd.weight must be raw Q6_K [2048 x vocab]");
    return kErrFormat;
  }
  *vocab = (int)t.dims[1];
  auto check_norm = [&](const std::string& name) -> bool {
    auto it = pack.tensors.find(name);
    if (it == pack.tensors.end()) {
      set_error("missing tensor " + name);
      return false;
    }
    if (it->second.type != kF32 || it->second.compact || it->second.byte_length != kHidden * 4) {
      set_error(name + " must be raw F32 [2048]");
      return false;
    }
    return true;
  };
  const bool b200 = pack.tensors.count(b200_name(0, 0)) != 0;
  for (int l = 0; l < layers; ++l) {
    if (!check_norm("blk." + std::to_string(l) + ".attn_norm.weight")) return kErrFormat;
    if (!check_norm("blk." + std::to_string(l) + ".ffn_norm.weight")) return kErrFormat;
    for (int which = 0; which < 4 && b200; ++which) {
      auto it = pack.tensors.find(b200_name(l, which));
      if (it == pack.tensors.end()) {
        set_error("missing tensor " + b200_name(l, which));
        return kErrFormat;
      }
      if (it->second.compact || it->second.dims.size() != 1 || (uint64_t)it->second.dims[0] != it->second.byte_length) {
        set_error(it->first + " must be a raw byte tensor [bytes]");
        return kErrFormat;
      }
    }
    for (int which = 0; which < 4 && !b200; ++which) {
      std::vector<PartSpec> parts;
      std::string err;
      if (resolve(pack, l, which, &parts, &err)) {
        set_error(err);
        return kErrFormat;
      }
      int64_t rows = 0;
      for (const PartSpec& ps : parts) {
        const PackTensor& pt = *ps.t;
        if (pt.dims.size() != 2 || pt.dims[0] != kProjK[which]) {
          set_error("invalid matrix " + pt.name);  // model.ts:315
          return kErrFormat;
        }
        if ((ps.fmt == kSegQ4K || ps.fmt == kSegQ6K) && pt.dims[0] % 256 != 0) {
          set_error(pt.name + " K is not divisible by a K-quant block");
          return kErrFormat;
        }
        if (pt.byte_length != expected_bytes(ps.fmt, pt.dims[1], pt.dims[0])) {
          set_error(pt.name + " has " + std::to_string(pt.byte_length) + " bytes; expected " +
                    std::to_string(expected_bytes(ps.fmt, pt.dims[1], pt.dims[0])));
          return kErrFormat;
        }
        if (pt.dims[1] % 128 != 0 && parts.size() > 1) {
          set_error(pt.name + " rows must be a multiple of 128");
          return kErrFormat;
        }
        rows += pt.dims[1];
      }
      if (rows != kProjN[which]) {
        set_error("blk." + std::to_string(l) + "." + kFused[which] + " has " + std::to_string(rows) +
                  " output rows; expected " + std::to_string(kProjN[which]));
        return kErrFormat;
      }
    }
  }
  if (!check_norm("output_norm.weight")) return kErrFormat;
  *n_layers = layers;
  return kOk;
}

void free_replica(DeviceModel& dm) {
  cudaSetDevice(dm.device);
  for (void* p : dm.allocations) cudaFree(p);
  dm.allocations.clear();
}

}  // namespace

int model_load(const void* data, size_t bytes, const int* devices, int ndev, nemo_model** out) {
  if (!data || !out) {
    set_error("nemo_model_load: null argument");
    return kErrArgs;
  }
  *out = nullptr;
  Pack pack;
  std::string err;
  if (!parse_wgpack(reinterpret_cast<const uint8_t*>(data), bytes, &pack, &err)) {
    set_error(err);
    return kErrFormat;
  }
  int n_layers = 0, vocab = 0;
  if (int rc = validate(pack, &n_layers, &vocab)) return rc;
  int count = 0;
  NEMO_CUDA_TRY(cudaGetDeviceCount(&count));
  std::vector<int> devs;
  if (!devices || ndev <= 0) devs.push_back(0);
  else devs.assign(devices, devices + ndev);
  for (int d : devs)
    if (d < 0 || d >= count) {
      set_error("device " + std::to_string(d) + " is not present (" + std::to_string(count) + " devices)");
      return kErrArgs;
    }
  // Tile-slab images for the small-T kernel: built once on the host, uploaded
  // to every replica.
  const uint8_t* file = reinterpret_cast<const uint8_t*>(data);
  std::vector<TileSlabImage> images((size_t)n_layers * 4);
  const bool b200 = pack.tensors.count(b200_name(0, 0)) != 0;
  for (int l = 0; l < n_layers && !b200; ++l)
    for (int which = 0; which < 4; ++which) {
      std::vector<PartSpec> parts;
      std::string perr;
      if (resolve(pack, l, which, &parts, &perr)) {
        set_error(perr);
        return kErrFormat;
      }
      if (int rc = build_tile_slab(file, parts, kProjN[which], kProjK[which], which == kProjGateUp,
                                   &images[l * 4 + which]))
        return rc;
    }
  auto* m = new nemo_model();
  m->n_layers = n_layers;
  m->vocab = vocab;
  for (size_t i = 0; i < devs.size(); ++i) {
    auto dm = std::make_unique<DeviceModel>();
    dm->device = devs[i];
    dm->vocab = vocab;
    int rc = upload_replica(file, pack, n_layers, vocab, *dm, m, i == 0, images);
    m->devs.push_back(std::move(dm));
    if (rc) {
      for (auto& d : m->devs) free_replica(*d);
      delete m;
      return rc;
    }
  }
  *out = m;
  return kOk;
}

// Writes a B200-tiled pack: the input's token table and norms unchanged, and
// every projection as its tile-slab image in one raw tensor
// (blk.<l>.<fused name>.b200_tiles). The container stays WGPACK02 with the
// reference's header fields (src/prepacked/format.ts:105-144), so its parser
// still accepts the file (raw storage); metadata "nemo.layout" names the
// layout. With out == NULL only *out_bytes is set.
int pack_b200(const void* data, size_t bytes, void* out, size_t capacity, size_t* out_bytes) {
  if (!data || !out_bytes) {
    set_error("nemo_pack_b200: null argument");
    return kErrArgs;
  }
  Pack pack;
  std::string err;
  const uint8_t* file = reinterpret_cast<const uint8_t*>(data);
  if (!parse_wgpack(file, bytes, &pack, &err)) {
    set_error(err);
    return kErrFormat;
  }
  if (pack.tensors.count(b200_name(0, 0))) {
    set_error("the pack is already B200-tiled");
    return kErrArgs;
  }
  int n_layers = 0, vocab = 0;
  if (int rc = validate(pack, &n_layers, &vocab)) return rc;
  struct OutTensor {
    std::string name;
    std::vector<int64_t> dims;
    int type;
    const uint8_t* src;
    std::vector<uint8_t> own;
    uint64_t len;
  };
  std::vector<OutTensor> outs;
  auto keep = [&](const std::string& name) {
    const PackTensor& t = pack.tensors.at(name);
    outs.push_back({name, t.dims, t.type, file + t.byte_offset, {}, t.byte_length});
  };
  keep("token_embd.weight");
  for (int l = 0; l < n_layers; ++l) {
    keep("blk." + std::to_string(l) + ".attn_norm.weight");
    keep("blk." + std::to_string(l) + ".ffn_norm.weight");
  }
  keep("output_norm.weight");
  for (int l = 0; l < n_layers; ++l)
    for (int which = 0; which < 4; ++which) {
      std::vector<PartSpec> parts;
      if (resolve(pack, l, which, &parts, &err)) {
        set_error(err);
        return kErrFormat;
      }
      TileSlabImage img;
      if (int rc = build_tile_slab(file, parts, kProjN[which], kProjK[which], which == kProjGateUp, &img)) return rc;
      OutTensor o;
      o.name = b200_name(l, which);
      o.type = parts[0].t->type;
      o.src = nullptr;
      const size_t table = b200_table_bytes(kProjN[which]);
      o.own.assign(table + img.bytes.size(), 0);
      memcpy(o.own.data(), img.tiles.data(), img.tiles.size() * sizeof(SkinnyTile));
      memcpy(o.own.data() + table, img.bytes.data(), img.bytes.size());
      o.len = o.own.size();
      o.dims = {(int64_t)o.len};
      outs.push_back(std::move(o));
    }
  auto align = [](uint64_t v, uint64_t a) { return (v + a - 1) / a * a; };
  std::string hdr = "{\"version\":2,\"sourceSha256\":\"" + pack.source_sha256 + "\",\"sourceBytes\":" +
                    std::to_string(bytes) +
                    ",\"layout\":\"q4_0-tile32-compact-v2\",\"tileRows\":32,\"blockValues\":32,\"blockBytes\":20,"
                    "\"metadata\":{\"nemo.layout\":\"b200-tile-slab-v1\"},\"tensors\":[";
  std::vector<uint64_t> offs;
  uint64_t rel = 0;
  for (size_t i = 0; i < outs.size(); ++i) {
    rel = align(rel, 256);
    offs.push_back(rel);
    std::string dims;
    for (size_t d = 0; d < outs[i].dims.size(); ++d) dims += (d ? "," : "") + std::to_string(outs[i].dims[d]);
    hdr += std::string(i ? "," : "") + "{\"name\":\"" + outs[i].name + "\",\"dimensions\":[" + dims +
           "],\"type\":" + std::to_string(outs[i].type) + ",\"storage\":\"raw\",\"offset\":" + std::to_string(rel) +
           ",\"byteLength\":" + std::to_string(outs[i].len) + "}";
    rel += outs[i].len;
  }
  hdr += "]}";
  const uint64_t data_offset = align(12 + hdr.size(), 256);
  const uint64_t total = data_offset + rel;
  *out_bytes = (size_t)total;
  if (!out) return kOk;
  if (capacity < total) {
    set_error("nemo_pack_b200: output buffer holds " + std::to_string(capacity) + " bytes; " + std::to_string(total) +
              " needed");
    return kErrArgs;
  }
  uint8_t* o = reinterpret_cast<uint8_t*>(out);
  memset(o, 0, total);
  memcpy(o, "WGPACK02", 8);
  const uint32_t hl = (uint32_t)hdr.size();
  memcpy(o + 8, &hl, 4);  // little-endian host
  memcpy(o + 12, hdr.data(), hdr.size());
  for (size_t i = 0; i < outs.size(); ++i)
    memcpy(o + data_offset + offs[i], outs[i].own.empty() ? outs[i].src : outs[i].own.data(), outs[i].len);
  return kOk;
}

void model_destroy(nemo_model* m) {
  if (!m) return;
  for (auto& d : m->devs) free_replica(*d);
  delete m;
}

}  // namespace nemo
