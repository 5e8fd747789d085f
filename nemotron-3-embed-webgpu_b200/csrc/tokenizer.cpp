// Host tokenizer: text -> token ids for the encoder, from a Hugging Face
// tokenizer.json of the byte-level BPE family. The reference tokenizes in the
// browser with @huggingface/transformers (src/main.ts:164-165:
// AutoTokenizer.from_pretrained('nvidia/Nemotron-3-Embed-1B-BF16')) and the
// engine calls it as tokenizer(text).input_ids (src/webgpu/embedding-engine.ts:41).
// This restates the published tokenizer.json semantics (Hugging Face
// `tokenizers`) for the components such files use:
//   added tokens   split out of the raw text first (leftmost, longest content;
//                  lstrip / rstrip / single_word honoured), mapped to their ids
//   normalizer     none
//   pre-tokenizer  Split(regex, Isolated) then ByteLevel(use_regex = false), or
//                  ByteLevel(use_regex = true) alone; the regexes supported are
//                  the two used by this family (listed below), matched with
//                  leftmost-first alternation and greedy backtracking
//   model          BPE over the byte-to-unicode alphabet: merges applied by
//                  rank (lowest first, leftmost among equals); ignore_merges
//   post-processor TemplateProcessing (single), Bert/Roberta, ByteLevel, none
// Anything else in the file is rejected with a message naming it.
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/nemo.h"
#include "json_reader.h"
#include "unicode_classes.h"

namespace nemo {

void set_error(const std::string& msg);

namespace tokz {
namespace {

using json::Json;

// --- Unicode classes ----------------------------------------------------------
enum { kOther = 0, kLu = 1, kLl = 2, kLt = 3, kLm = 4, kLo = 5, kM = 6, kN = 7 };

int cls_of(uint32_t cp) {
  const uc::Range* r = uc::kClassRanges;
  size_t lo = 0, hi = sizeof(uc::kClassRanges) / sizeof(uc::kClassRanges[0]);
  while (lo < hi) {
    const size_t mid = (lo + hi) / 2;
    if (cp < r[mid].lo) hi = mid;
    else if (cp > r[mid].hi) lo = mid + 1;
    else return r[mid].cls;
  }
  return kOther;
}

bool is_space(uint32_t cp) {
  for (const auto& w : uc::kWhiteSpace)
    if (cp >= w[0] && cp <= w[1]) return true;
  return false;
}

bool is_letter(int c) { return c >= kLu && c <= kLo; }

// Character predicates of the supported patterns.
enum Pred {
  kPrefix,     // [^\r\n\p{L}\p{N}]
  kUpperish,   // [\p{Lu}\p{Lt}\p{Lm}\p{Lo}\p{M}]
  kLowerish,   // [\p{Ll}\p{Lm}\p{Lo}\p{M}]
  kNumber,     // \p{N}
  kLetter,     // \p{L}
  kSpaceChar,  // ' '
  kPunct,      // [^\s\p{L}\p{N}]
  kCrLfSlash,  // [\r\n/]
  kWhite,      // \s
  kCrLf,       // [\r\n]
};

bool test(Pred p, uint32_t cp) {
  const int c = cls_of(cp);
  switch (p) {
    case kPrefix: return cp != '\r' && cp != '\n' && !is_letter(c) && c != kN;
    case kUpperish: return c == kLu || c == kLt || c == kLm || c == kLo || c == kM;
    case kLowerish: return c == kLl || c == kLm || c == kLo || c == kM;
    case kNumber: return c == kN;
    case kLetter: return is_letter(c);
    case kSpaceChar: return cp == ' ';
    case kPunct: return !is_space(cp) && !is_letter(c) && c != kN;
    case kCrLfSlash: return cp == '\r' || cp == '\n' || cp == '/';
    case kWhite: return is_space(cp);
    case kCrLf: return cp == '\r' || cp == '\n';
  }
  return false;
}

// One element of an alternative: a class run with bounds, a literal, or the
// (?!\S) lookahead.
struct Item {
  enum Kind { kRun, kLiteral, kNotFollowedByNonSpace } kind;
  Pred pred;
  int min, max;
  std::vector<uint32_t> lit;
};

Item run(Pred p, int mn, int mx) { return Item{Item::kRun, p, mn, mx, {}}; }
Item lit(const char* s) {
  Item it{Item::kLiteral, kPrefix, 0, 0, {}};
  for (const char* c = s; *c; ++c) it.lit.push_back((uint8_t)*c);
  return it;
}
Item not_followed_by_nonspace() { return Item{Item::kNotFollowedByNonSpace, kPrefix, 0, 0, {}}; }

constexpr int kInf = 1 << 30;
using Alternative = std::vector<Item>;

// The Split pattern of Tekken-style tokenizers (Mistral-family vocabularies of
// 131,072 entries) and the GPT-2 byte-level pattern.
const char* kTekkenPattern =
    "[^\\r\\n\\p{L}\\p{N}]?[\\p{Lu}\\p{Lt}\\p{Lm}\\p{Lo}\\p{M}]*[\\p{Ll}\\p{Lm}\\p{Lo}\\p{M}]+|[^\\r\\n\\p{L}\\p{N}]?"
    "[\\p{Lu}\\p{Lt}\\p{Lm}\\p{Lo}\\p{M}]+[\\p{Ll}\\p{Lm}\\p{Lo}\\p{M}]*|\\p{N}| ?[^\\s\\p{L}\\p{N}]+[\\r\\n/]*|"
    "\\s*[\\r\\n]+|\\s+(?!\\S)|\\s+";
const char* kGpt2Pattern = "'s|'t|'re|'ve|'m|'ll|'d| ?\\p{L}+| ?\\p{N}+| ?[^\\s\\p{L}\\p{N}]+|\\s+(?!\\S)|\\s+";

std::vector<Alternative> tekken_alternatives() {
  return {{run(kPrefix, 0, 1), run(kUpperish, 0, kInf), run(kLowerish, 1, kInf)},
          {run(kPrefix, 0, 1), run(kUpperish, 1, kInf), run(kLowerish, 0, kInf)},
          {run(kNumber, 1, 1)},
          {run(kSpaceChar, 0, 1), run(kPunct, 1, kInf), run(kCrLfSlash, 0, kInf)},
          {run(kWhite, 0, kInf), run(kCrLf, 1, kInf)},
          {run(kWhite, 1, kInf), not_followed_by_nonspace()},
          {run(kWhite, 1, kInf)}};
}

std::vector<Alternative> gpt2_alternatives() {
  return {{lit("'s")},        {lit("'t")},         {lit("'re")}, {lit("'ve")}, {lit("'m")}, {lit("'ll")}, {lit("'d")},
          {run(kSpaceChar, 0, 1), run(kLetter, 1, kInf)},
          {run(kSpaceChar, 0, 1), run(kNumber, 1, kInf)},
          {run(kSpaceChar, 0, 1), run(kPunct, 1, kInf)},
          {run(kWhite, 1, kInf), not_followed_by_nonspace()},
          {run(kWhite, 1, kInf)}};
}

// Greedy match of items[k..] at cps[pos..]; backtracks run lengths.
bool match(const Alternative& a, size_t k, const std::vector<uint32_t>& cps, size_t pos, size_t* end) {
  if (k == a.size()) {
    *end = pos;
    return true;
  }
  const Item& it = a[k];
  if (it.kind == Item::kNotFollowedByNonSpace) {
    if (pos < cps.size() && !is_space(cps[pos])) return false;
    return match(a, k + 1, cps, pos, end);
  }
  if (it.kind == Item::kLiteral) {
    if (pos + it.lit.size() > cps.size()) return false;
    for (size_t i = 0; i < it.lit.size(); ++i)
      if (cps[pos + i] != it.lit[i]) return false;
    return match(a, k + 1, cps, pos + it.lit.size(), end);
  }
  size_t n = 0;
  while ((int)n < it.max && pos + n < cps.size() && test(it.pred, cps[pos + n])) ++n;
  for (size_t c = n + 1; c-- > (size_t)it.min;)
    if (match(a, k + 1, cps, pos + c, end)) return true;
  return false;
}

// Splits cps[b, e) into the pattern's matches and the gaps between them
// (Split behaviour "Isolated"); pieces as [begin, end) code point ranges.
void split(const std::vector<Alternative>& alts, const std::vector<uint32_t>& cps, size_t b, size_t e,
           std::vector<std::pair<size_t, size_t>>* pieces) {
  const std::vector<uint32_t> sub(cps.begin() + b, cps.begin() + e);
  size_t gap = 0, pos = 0;
  while (pos < sub.size()) {
    size_t end = 0;
    bool hit = false;
    for (const Alternative& a : alts)
      if (match(a, 0, sub, pos, &end) && end > pos) {
        hit = true;
        break;
      }
    if (!hit) {
      ++pos;
      continue;
    }
    if (gap < pos) pieces->push_back({b + gap, b + pos});
    pieces->push_back({b + pos, b + end});
    pos = gap = end;
  }
  if (gap < sub.size()) pieces->push_back({b + gap, e});
}

// --- UTF-8 ----------------------------------------------------------------------
bool decode_utf8(const char* s, size_t len, std::vector<uint32_t>* cps) {
  const uint8_t* p = reinterpret_cast<const uint8_t*>(s);
  size_t i = 0;
  while (i < len) {
    const uint8_t c = p[i];
    uint32_t cp;
    int n;
    if (c < 0x80) { cp = c; n = 1; }
    else if ((c & 0xE0) == 0xC0) { cp = c & 0x1F; n = 2; }
    else if ((c & 0xF0) == 0xE0) { cp = c & 0x0F; n = 3; }
    else if ((c & 0xF8) == 0xF0) { cp = c & 0x07; n = 4; }
    else return false;
    if (i + n > len) return false;
    for (int k = 1; k < n; ++k) {
      if ((p[i + k] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (p[i + k] & 0x3F);
    }
    const uint32_t min_cp[5] = {0, 0, 0x80, 0x800, 0x10000};
    if (cp < min_cp[n] || cp > 0x10FFFF || (cp >= 0xD800 && cp < 0xE000)) return false;
    cps->push_back(cp);
    i += n;
  }
  return true;
}

void utf8_of(uint32_t cp, std::string* out) { json::append_utf8(out, cp); }

}  // namespace

struct Added {
  std::string content;
  std::vector<uint32_t> cps;
  uint32_t id;
  bool lstrip, rstrip, single_word;
};

struct Tokenizer {
  std::vector<Added> added;
  std::vector<Alternative> alts;  // empty: no Split (ByteLevel without regex)
  bool own_regex = false;         // the alternatives are ByteLevel's own (GPT-2) regex
  bool add_prefix_space = false;
  std::unordered_map<std::string, uint32_t> vocab;
  std::unordered_map<uint64_t, std::pair<uint32_t, uint32_t>> merges;  // (left, right) -> (rank, merged id)
  bool ignore_merges = false;
  bool has_unk = false;
  uint32_t unk = 0;
  std::vector<std::vector<uint32_t>> before, after;  // post-processor ids around the sequence
  std::string byte_char[256];  // byte -> its character in the byte-level alphabet (UTF-8)
  mutable std::unordered_map<std::string, std::vector<uint32_t>> cache;
};

namespace {

void init_byte_alphabet(Tokenizer* t) {
  // bytes_to_unicode of the byte-level BPE family: printable bytes keep their
  // code point, the others map to 256, 257, ... in byte order.
  int next = 256;
  for (int b = 0; b < 256; ++b) {
    const bool printable = (b >= 0x21 && b <= 0x7E) || (b >= 0xA1 && b <= 0xAC) || (b >= 0xAE && b <= 0xFF);
    std::string s;
    utf8_of(printable ? (uint32_t)b : (uint32_t)next++, &s);
    t->byte_char[b] = s;
  }
}

uint64_t pair_key(uint32_t a, uint32_t b) { return ((uint64_t)a << 32) | b; }

int fail(const std::string& m) {
  set_error("tokenizer.json: " + m);
  return NEMO_ERR_FORMAT;
}

// Splits a UTF-8 string into its characters (byte-level vocab entries are
// sequences of alphabet characters).
std::vector<std::string> chars_of(const std::string& s) {
  std::vector<std::string> out;
  for (size_t i = 0; i < s.size();) {
    const uint8_t c = (uint8_t)s[i];
    const size_t n = c < 0x80 ? 1 : (c & 0xE0) == 0xC0 ? 2 : (c & 0xF0) == 0xE0 ? 3 : 4;
    out.push_back(s.substr(i, n));
    i += n;
  }
  return out;
}

int load_pre_tokenizer(const Json* pt, Tokenizer* t) {
  if (!pt || pt->kind == Json::kNull) return fail("a pre_tokenizer is required (ByteLevel)");
  const Json* type = pt->get("type");
  if (!type || type->kind != Json::kStr) return fail("pre_tokenizer without a type");
  auto byte_level = [&](const Json* bl, bool inner) -> int {
    const Json* ur = bl->get("use_regex");
    const bool use_regex = ur && ur->kind == Json::kBool ? ur->b : true;
    const Json* aps = bl->get("add_prefix_space");
    t->add_prefix_space = aps && aps->kind == Json::kBool && aps->b;
    if (use_regex) {
      if (inner) return fail("ByteLevel with use_regex after a Split is not supported");
      t->alts = gpt2_alternatives();
      t->own_regex = true;
    }
    return NEMO_OK;
  };
  if (type->str == "ByteLevel") return byte_level(pt, false);
  if (type->str != "Sequence") return fail("unsupported pre_tokenizer " + type->str);
  const Json* seq = pt->get("pretokenizers");
  if (!seq || seq->kind != Json::kArr || seq->arr.size() != 2) return fail("unsupported pre_tokenizer sequence");
  const Json& sp = seq->arr[0];
  const Json* st = sp.get("type");
  const Json* pat = sp.get("pattern");
  const Json* rx = pat ? pat->get("Regex") : nullptr;
  const Json* beh = sp.get("behavior");
  const Json* inv = sp.get("invert");
  if (!st || st->str != "Split" || !rx || rx->kind != Json::kStr || !beh || beh->str != "Isolated" ||
      (inv && inv->kind == Json::kBool && inv->b))
    return fail("the first pre_tokenizer must be Split(Regex, Isolated)");
  if (rx->str == kTekkenPattern) t->alts = tekken_alternatives();
  else if (rx->str == kGpt2Pattern) t->alts = gpt2_alternatives();
  else return fail("unsupported pre-tokenizer pattern " + rx->str);
  const Json& bl = seq->arr[1];
  const Json* bt = bl.get("type");
  if (!bt || bt->str != "ByteLevel") return fail("the second pre_tokenizer must be ByteLevel");
  return byte_level(&bl, true);
}

int load_post_processor(const Json* pp, Tokenizer* t) {
  if (!pp || pp->kind == Json::kNull) return NEMO_OK;
  const Json* type = pp->get("type");
  if (!type) return fail("post_processor without a type");
  if (type->str == "ByteLevel") return NEMO_OK;
  if (type->str == "BertProcessing" || type->str == "RobertaProcessing") {
    const Json* cls = pp->get("cls");
    const Json* sep = pp->get("sep");
    if (!cls || !sep || cls->arr.size() != 2 || sep->arr.size() != 2) return fail("bad Bert/Roberta post_processor");
    t->before.push_back({(uint32_t)cls->arr[1].num});
    t->after.push_back({(uint32_t)sep->arr[1].num});
    return NEMO_OK;
  }
  if (type->str != "TemplateProcessing") return fail("unsupported post_processor " + type->str);
  const Json* single = pp->get("single");
  const Json* specials = pp->get("special_tokens");
  if (!single || single->kind != Json::kArr || !specials) return fail("bad TemplateProcessing");
  bool seen_a = false;
  for (const Json& piece : single->arr) {
    if (const Json* sq = piece.get("Sequence")) {
      const Json* id = sq->get("id");
      if (!id || id->str != "A" || seen_a) return fail("TemplateProcessing single must hold sequence A once");
      seen_a = true;
      continue;
    }
    const Json* tok = piece.get("SpecialToken");
    const Json* name = tok ? tok->get("id") : nullptr;
    const Json* entry = name ? specials->get(name->str.c_str()) : nullptr;
    const Json* ids = entry ? entry->get("ids") : nullptr;
    if (!ids || ids->kind != Json::kArr) return fail("TemplateProcessing special token without ids");
    std::vector<uint32_t> v;
    for (const Json& x : ids->arr) v.push_back((uint32_t)x.num);
    (seen_a ? t->after : t->before).push_back(v);
  }
  if (!seen_a) return fail("TemplateProcessing single without sequence A");
  return NEMO_OK;
}

int load(const char* data, size_t bytes, Tokenizer* t) {
  json::Reader r{data, data + bytes, {}, 0};
  Json root;
  if (!r.parse(&root) || root.kind != Json::kObj) return fail("not a JSON object (" + r.err + ")");
  const Json* norm = root.get("normalizer");
  if (norm && norm->kind != Json::kNull) return fail("normalizers are not supported");
  const Json* model = root.get("model");
  const Json* mtype = model ? model->get("type") : nullptr;
  if (!mtype || mtype->str != "BPE") return fail("the model must be BPE");
  for (const char* key : {"continuing_subword_prefix", "end_of_word_suffix", "dropout"}) {
    const Json* v = model->get(key);
    if (v && v->kind != Json::kNull) return fail(std::string("BPE ") + key + " is not supported");
  }
  const Json* bf = model->get("byte_fallback");
  if (bf && bf->kind == Json::kBool && bf->b) return fail("BPE byte_fallback is not supported (byte-level vocabulary expected)");
  const Json* im = model->get("ignore_merges");
  t->ignore_merges = im && im->kind == Json::kBool && im->b;
  const Json* vocab = model->get("vocab");
  if (!vocab || vocab->kind != Json::kObj) return fail("BPE vocab missing");
  t->vocab.reserve(vocab->obj.size() * 2);
  for (const auto& kv : vocab->obj) t->vocab[kv.first] = (uint32_t)kv.second.num;
  const Json* unk = model->get("unk_token");
  if (unk && unk->kind == Json::kStr) {
    auto it = t->vocab.find(unk->str);
    if (it == t->vocab.end()) return fail("unk_token not in the vocab");
    t->has_unk = true;
    t->unk = it->second;
  }
  const Json* merges = model->get("merges");
  if (!merges || merges->kind != Json::kArr) return fail("BPE merges missing");
  uint32_t rank = 0;
  for (const Json& m : merges->arr) {
    std::string a, b;
    if (m.kind == Json::kArr && m.arr.size() == 2) {
      a = m.arr[0].str;
      b = m.arr[1].str;
    } else if (m.kind == Json::kStr) {
      const size_t sp = m.str.find(' ', 1);
      if (sp == std::string::npos) return fail("bad merge " + m.str);
      a = m.str.substr(0, sp);
      b = m.str.substr(sp + 1);
    } else {
      return fail("bad merge entry");
    }
    auto ia = t->vocab.find(a), ib = t->vocab.find(b), im2 = t->vocab.find(a + b);
    if (ia == t->vocab.end() || ib == t->vocab.end() || im2 == t->vocab.end())
      return fail("merge " + a + " " + b + " refers to tokens missing from the vocab");
    t->merges.emplace(pair_key(ia->second, ib->second), std::make_pair(rank++, im2->second));
  }
  const Json* added = root.get("added_tokens");
  if (added && added->kind == Json::kArr)
    for (const Json& a : added->arr) {
      Added x;
      const Json* c = a.get("content");
      const Json* id = a.get("id");
      if (!c || !id) return fail("added token without content or id");
      x.content = c->str;
      x.id = (uint32_t)id->num;
      auto flag = [&](const char* k) {
        const Json* v = a.get(k);
        return v && v->kind == Json::kBool && v->b;
      };
      x.lstrip = flag("lstrip");
      x.rstrip = flag("rstrip");
      x.single_word = flag("single_word");
      if (!decode_utf8(x.content.data(), x.content.size(), &x.cps) || x.cps.empty())
        return fail("added token with empty or invalid content");
      t->added.push_back(std::move(x));
    }
  if (int rc = load_pre_tokenizer(root.get("pre_tokenizer"), t)) return rc;
  if (int rc = load_post_processor(root.get("post_processor"), t)) return rc;
  init_byte_alphabet(t);
  return NEMO_OK;
}

bool is_word_char(uint32_t cp) {
  const int c = cls_of(cp);
  return is_letter(c) || c == kN || cp == '_';
}

// BPE of one pre-token (already mapped to the byte-level alphabet).
int bpe(const Tokenizer& t, const std::string& word, std::vector<uint32_t>* out) {
  auto hit = t.cache.find(word);
  if (hit != t.cache.end()) {
    out->insert(out->end(), hit->second.begin(), hit->second.end());
    return NEMO_OK;
  }
  std::vector<uint32_t> sym;
  if (t.ignore_merges) {
    auto it = t.vocab.find(word);
    if (it != t.vocab.end()) sym.push_back(it->second);
  }
  if (sym.empty()) {
    for (const std::string& ch : chars_of(word)) {
      auto it = t.vocab.find(ch);
      if (it != t.vocab.end()) sym.push_back(it->second);
      else if (t.has_unk) sym.push_back(t.unk);
      else {
        set_error("tokenizer: character missing from the vocabulary and no unk_token");
        return NEMO_ERR_ARGS;
      }
    }
    // merge the lowest-ranked adjacent pair (leftmost among equals) until none is left
    for (;;) {
      uint32_t best = UINT32_MAX, merged = 0;
      size_t at = 0;
      for (size_t i = 0; i + 1 < sym.size(); ++i) {
        auto m = t.merges.find(pair_key(sym[i], sym[i + 1]));
        if (m != t.merges.end() && m->second.first < best) {
          best = m->second.first;
          merged = m->second.second;
          at = i;
        }
      }
      if (best == UINT32_MAX) break;
      sym[at] = merged;
      sym.erase(sym.begin() + at + 1);
    }
  }
  if (t.cache.size() < (1u << 16)) t.cache.emplace(word, sym);
  out->insert(out->end(), sym.begin(), sym.end());
  return NEMO_OK;
}

// Normal (non-added) text cps[b, e): pre-tokenize, map bytes, BPE. ByteLevel's
// add_prefix_space prepends a space to every split it sees that does not
// start with one: the whole segment when ByteLevel splits with its own regex,
// each piece of a preceding Split otherwise.
int encode_plain(const Tokenizer& t, const std::vector<uint32_t>& cps, size_t b, size_t e, std::vector<uint32_t>* out) {
  if (b >= e) return NEMO_OK;
  std::vector<uint32_t> text(cps.begin() + b, cps.begin() + e);
  if (t.add_prefix_space && t.own_regex && text[0] != ' ') text.insert(text.begin(), ' ');
  std::vector<std::pair<size_t, size_t>> pieces;
  if (t.alts.empty()) pieces.push_back({0, text.size()});
  else split(t.alts, text, 0, text.size(), &pieces);
  for (const auto& pc : pieces) {
    std::string word;
    if (t.add_prefix_space && !t.own_regex && text[pc.first] != ' ') word += t.byte_char[' '];
    for (size_t i = pc.first; i < pc.second; ++i) {
      std::string u8;
      utf8_of(text[i], &u8);
      for (unsigned char byte : u8) word += t.byte_char[byte];
    }
    if (int rc = bpe(t, word, out)) return rc;
  }
  return NEMO_OK;
}

int encode(const Tokenizer& t, const char* s, size_t len, std::vector<uint32_t>* ids) {
  std::vector<uint32_t> cps;
  if (!decode_utf8(s, len, &cps)) {
    set_error("tokenizer: text is not valid UTF-8");
    return NEMO_ERR_ARGS;
  }
  for (const auto& v : t.before) ids->insert(ids->end(), v.begin(), v.end());
  // added tokens first: at each position the longest content that matches
  size_t pos = 0, plain = 0;
  while (pos < cps.size()) {
    const Added* best = nullptr;
    size_t mb = 0, me = 0;
    for (const Added& a : t.added) {
      if (pos + a.cps.size() > cps.size() || (best && a.cps.size() <= best->cps.size())) continue;
      if (!std::equal(a.cps.begin(), a.cps.end(), cps.begin() + pos)) continue;
      size_t e = pos + a.cps.size();
      if (a.single_word && ((pos > 0 && is_word_char(cps[pos - 1])) || (e < cps.size() && is_word_char(cps[e]))))
        continue;
      size_t b = pos;
      if (a.lstrip)
        while (b > plain && is_space(cps[b - 1])) --b;
      if (a.rstrip)
        while (e < cps.size() && is_space(cps[e])) ++e;
      best = &a;
      mb = b;
      me = e;
    }
    if (!best) {
      ++pos;
      continue;
    }
    if (int rc = encode_plain(t, cps, plain, mb, ids)) return rc;
    ids->push_back(best->id);
    pos = plain = me;
  }
  if (int rc = encode_plain(t, cps, plain, cps.size(), ids)) return rc;
  for (const auto& v : t.after) ids->insert(ids->end(), v.begin(), v.end());
  return NEMO_OK;
}

}  // namespace
}  // namespace tokz
}  // namespace nemo

struct nemo_tokenizer {
  nemo::tokz::Tokenizer t;
};

extern "C" int nemo_tokenizer_load(const void* json_bytes, size_t bytes, nemo_tokenizer** out) {
  if (!json_bytes || !out) {
    nemo::set_error("nemo_tokenizer_load: null argument");
    return NEMO_ERR_ARGS;
  }
  *out = nullptr;
  auto* tk = new nemo_tokenizer();
  if (int rc = nemo::tokz::load(static_cast<const char*>(json_bytes), bytes, &tk->t)) {
    delete tk;
    return rc;
  }
  *out = tk;
  return NEMO_OK;
}

extern "C" int nemo_tokenizer_encode(const nemo_tokenizer* tok, const char* text, size_t len, uint32_t* ids,
                                     size_t capacity, size_t* n_ids) {
  if (!tok || (!text && len) || !n_ids) {
    nemo::set_error("nemo_tokenizer_encode: null argument");
    return NEMO_ERR_ARGS;
  }
  std::vector<uint32_t> v;
  if (int rc = nemo::tokz::encode(tok->t, text ? text : "", len, &v)) return rc;
  *n_ids = v.size();
  if (!ids) return NEMO_OK;
  if (capacity < v.size()) {
    nemo::set_error("nemo_tokenizer_encode: " + std::to_string(v.size()) + " ids, capacity " + std::to_string(capacity));
    return NEMO_ERR_ARGS;
  }
  std::copy(v.begin(), v.end(), ids);
  return NEMO_OK;
}

extern "C" void nemo_tokenizer_destroy(nemo_tokenizer* tok) { delete tok; }
