// Host-side tokenizer behind the C ABI: ds::rt::Tokenizer
// (src/runtime/tokenizer.cpp:1-171, include/ds/runtime/tokenizer.h:19-38).
//
// tokenizer.json supplies model.vocab (piece -> id), model.unk_token_id, the
// added_tokens list (id, content, special) and optional root bos/eos ids, read
// as Tokenizer::load_from_file does (tokenizer.cpp:44-97).  Encoding is the
// reference's greedy longest match (tokenizer.cpp:116-155): at each byte
// offset the longest piece that is in the vocabulary as itself, as "▁" or
// "Ġ" + piece at a word start (offset 0 or after an isspace byte), or as
// piece + "</w>"; an unmatched whitespace run is skipped; any other unmatched
// byte is an error.  The candidate length is bounded by the longest
// vocabulary entry (the reference tries every remaining length, quadratic in
// the text; a piece longer than every entry matches no variant, so the ids
// are the same).  Decoding maps ids to pieces with the reference's trim
// (tokenizer.cpp:13-27: "##" dropped, "</w>" -> trailing space, a leading
// "▁" / "Ġ" -> space), skipping special ids on request.
//
// Differences from the reference, on purpose: an added token's
// "special": true counts (the reference's get_int_or skips JSON booleans,
// src/util/json.cpp:301-306, so it reads Hugging Face's booleans as false);
// ids must be non-negative and below 2^24 (the reference sizes its table from
// the largest id unchecked); a piece given twice in the vocabulary object is a
// JSON error; when several pieces share an id, decoding uses the last in file
// order (the reference's order is its hash map's).

#include <algorithm>
#include <cctype>
#include <cstdio>
#include <memory>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "dsb_internal.h"
#include "host_json.h"

struct dsb_tokenizer {
  std::string model_type;
  int32_t bos = -1, eos = -1, unk = -1;
  std::vector<std::string> id_to_token;
  std::unordered_map<std::string, int32_t> token_to_id;
  std::unordered_set<int32_t> special;
  size_t max_len = 0;  // longest vocabulary entry, bytes
};

namespace {

using dsb::Json;

constexpr int64_t kMaxTokenId = (1 << 24) - 1;

int tk_fail(int code, std::string msg) { return dsb::host_fail(code, std::move(msg), dsb::kHostTokenizer); }

bool read_file(const std::string& path, std::string* out) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (f == nullptr) return false;
  char buf[65536];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) out->append(buf, n);
  const bool ok = !std::ferror(f);
  std::fclose(f);
  return ok;
}

// maybe_get_token_id (tokenizer.cpp:36-40): -1 when absent or null.
bool token_id(const Json& j, const char* key, int32_t* id) {
  const Json* v = j.get(key);
  if (v == nullptr || v->kind == Json::Null) {
    *id = -1;
    return true;
  }
  if (v->kind != Json::Int || v->i < -1 || v->i > kMaxTokenId) return false;
  *id = (int32_t)v->i;
  return true;
}

const char kSpm[] = "\xE2\x96\x81";  // U+2581, SentencePiece word start
const char kGpt[] = "\xC4\xA0";      // U+0120, byte-level BPE space

bool starts_with(const std::string& s, const char* p) {
  const size_t n = std::char_traits<char>::length(p);
  return s.size() >= n && s.compare(0, n, p) == 0;
}

// trim_piece (tokenizer.cpp:13-27)
std::string trim_piece(std::string t) {
  if (starts_with(t, "##")) t.erase(0, 2);
  if (t.size() >= 4 && t.compare(t.size() - 4, 4, "</w>") == 0) {
    t.erase(t.size() - 4);
    t.push_back(' ');
  }
  if (starts_with(t, kSpm)) {
    t.erase(0, 3);
    t.insert(t.begin(), ' ');
  } else if (starts_with(t, kGpt)) {
    t.erase(0, 2);
    t.insert(t.begin(), ' ');
  }
  return t;
}

int load(const std::string& path, dsb_tokenizer* tk) {
  std::string text;
  if (!read_file(path, &text)) return tk_fail(DSB_EINVAL, "cannot read " + path);
  Json root;
  std::string err;
  if (!dsb::parse_json(text.data(), text.size(), &root, &err)) return tk_fail(DSB_EINVAL, path + ": " + err);
  if (root.kind != Json::Obj) return tk_fail(DSB_EINVAL, "tokenizer.json root is not an object");
  const Json* model = root.get("model");
  if (model == nullptr || model->kind != Json::Obj) return tk_fail(DSB_EINVAL, "tokenizer.json missing model object");
  if (const Json* t = model->get("type"); t != nullptr && t->kind == Json::Str) tk->model_type = t->s;
  const Json* vocab = model->get("vocab");
  if (vocab == nullptr || vocab->kind != Json::Obj) return tk_fail(DSB_EINVAL, "tokenizer.json missing model.vocab");
  int64_t max_id = -1;
  for (const auto& kv : vocab->o) {
    if (kv.second.kind != Json::Int || kv.second.i < 0 || kv.second.i > kMaxTokenId)
      return tk_fail(DSB_EINVAL, "tokenizer.json: bad id for piece " + kv.first);
    max_id = std::max(max_id, kv.second.i);
  }
  tk->id_to_token.assign((size_t)(max_id + 1), std::string());
  tk->token_to_id.reserve(vocab->o.size() * 2);
  for (const auto& kv : vocab->o) {
    tk->token_to_id.emplace(kv.first, (int32_t)kv.second.i);
    tk->id_to_token[(size_t)kv.second.i] = kv.first;
  }
  if (!token_id(*model, "unk_token_id", &tk->unk)) return tk_fail(DSB_EINVAL, "tokenizer.json: bad unk_token_id");
  if (const Json* added = root.get("added_tokens"); added != nullptr && added->kind == Json::Arr) {
    for (const Json& item : added->a) {
      int32_t id = -1;
      if (!token_id(item, "id", &id)) return tk_fail(DSB_EINVAL, "tokenizer.json: bad added token id");
      const Json* c = item.get("content");
      const std::string content = c != nullptr && c->kind == Json::Str ? c->s : std::string();
      const Json* sp = item.get("special");
      const bool special = sp != nullptr && ((sp->kind == Json::Bool && sp->b) || (sp->kind == Json::Int && sp->i != 0) ||
                                             (sp->kind == Json::Num && sp->d != 0.0));
      if (id >= 0 && (size_t)id < tk->id_to_token.size() && !content.empty()) {
        tk->id_to_token[(size_t)id] = content;
        tk->token_to_id[content] = id;
      }
      if (special && id >= 0) tk->special.insert(id);
    }
  }
  if (!token_id(root, "bos_token_id", &tk->bos) || !token_id(root, "eos_token_id", &tk->eos))
    return tk_fail(DSB_EINVAL, "tokenizer.json: bad bos/eos id");
  if (tk->bos >= 0) tk->special.insert(tk->bos);
  if (tk->eos >= 0) tk->special.insert(tk->eos);
  for (const auto& kv : tk->token_to_id) tk->max_len = std::max(tk->max_len, kv.first.size());
  return DSB_OK;
}

bool is_space(char c) { return std::isspace(static_cast<unsigned char>(c)) != 0; }

// lookup_piece_with_variants (tokenizer.cpp:106-114); `key` is scratch.
bool lookup(const dsb_tokenizer& tk, const char* p, size_t n, bool word_start, std::string& key, int32_t* id) {
  auto find = [&](const std::string& k) {
    auto it = tk.token_to_id.find(k);
    if (it == tk.token_to_id.end()) return false;
    *id = it->second;
    return true;
  };
  key.assign(p, n);
  if (find(key)) return true;
  if (word_start) {
    key.assign(kSpm).append(p, n);
    if (find(key)) return true;
    key.assign(kGpt).append(p, n);
    if (find(key)) return true;
  }
  key.assign(p, n).append("</w>");
  return find(key);
}

}  // namespace

extern "C" const char* dsb_tokenizer_error(void) { return dsb::host_error(dsb::kHostTokenizer); }

extern "C" int dsb_tokenizer_load(const char* path, dsb_tokenizer** out) {
  if (path == nullptr || out == nullptr) return tk_fail(DSB_EINVAL, "dsb_tokenizer_load: bad arguments");
  *out = nullptr;
  try {
    auto tk = std::make_unique<dsb_tokenizer>();
    const int rc = load(path, tk.get());
    if (rc != DSB_OK) return rc;
    *out = tk.release();
    return DSB_OK;
  } catch (const std::bad_alloc&) {
    return tk_fail(DSB_ENOMEM, "dsb_tokenizer_load: out of host memory");
  } catch (...) {
    return tk_fail(DSB_EINVAL, "dsb_tokenizer_load: unexpected error");
  }
}

extern "C" int dsb_tokenizer_destroy(dsb_tokenizer* tk) {
  delete tk;
  return DSB_OK;
}

extern "C" int dsb_tokenizer_info(const dsb_tokenizer* tk, int* n_ids, int32_t* bos_id, int32_t* eos_id,
                                  int32_t* unk_id) {
  if (tk == nullptr) return tk_fail(DSB_EINVAL, "dsb_tokenizer_info: bad arguments");
  if (n_ids) *n_ids = (int)tk->id_to_token.size();
  if (bos_id) *bos_id = tk->bos;
  if (eos_id) *eos_id = tk->eos;
  if (unk_id) *unk_id = tk->unk;
  return DSB_OK;
}

extern "C" int dsb_tokenizer_encode(const dsb_tokenizer* tk, const char* text, size_t len, int32_t* ids, size_t cap,
                                    size_t* n_ids) {
  if (tk == nullptr || n_ids == nullptr || (text == nullptr && len > 0) || (ids == nullptr && cap > 0))
    return tk_fail(DSB_EINVAL, "dsb_tokenizer_encode: bad arguments");
  *n_ids = 0;
  if (len == 0) return DSB_OK;
  if (tk->token_to_id.empty()) return tk_fail(DSB_EINVAL, "tokenizer has no vocabulary");
  try {
    std::string key;
    size_t n = 0, pos = 0;
    while (pos < len) {
      const bool word_start = pos == 0 || is_space(text[pos - 1]);
      int32_t best = -1;
      size_t best_len = 0;
      for (size_t l = std::min(len - pos, tk->max_len); l > 0; --l) {
        if (lookup(*tk, text + pos, l, word_start, key, &best)) {
          best_len = l;
          break;
        }
      }
      if (best_len == 0) {
        if (is_space(text[pos])) {  // an unencodable whitespace run is skipped
          do {
            ++pos;
          } while (pos < len && is_space(text[pos]));
          continue;
        }
        return tk_fail(DSB_EINVAL, "tokenizer could not encode input near byte offset " + std::to_string(pos));
      }
      if (n < cap) ids[n] = best;
      ++n;
      pos += best_len;
    }
    *n_ids = n;
    if (n > cap) return tk_fail(DSB_EINVAL, "dsb_tokenizer_encode: " + std::to_string(n) + " ids need a larger buffer");
    return DSB_OK;
  } catch (...) {
    return tk_fail(DSB_ENOMEM, "dsb_tokenizer_encode: out of host memory");
  }
}

extern "C" int dsb_tokenizer_decode(const dsb_tokenizer* tk, const int32_t* ids, size_t n, int skip_special, char* out,
                                    size_t cap, size_t* len) {
  if (tk == nullptr || len == nullptr || (ids == nullptr && n > 0) || (out == nullptr && cap > 0))
    return tk_fail(DSB_EINVAL, "dsb_tokenizer_decode: bad arguments");
  *len = 0;
  try {
    std::string s;
    for (size_t i = 0; i < n; ++i) {
      const int32_t id = ids[i];
      if (id < 0 || (size_t)id >= tk->id_to_token.size()) return tk_fail(DSB_EINVAL, "token id out of range");
      if (skip_special && tk->special.count(id) != 0) continue;
      s += trim_piece(tk->id_to_token[(size_t)id]);
    }
    *len = s.size();
    if (s.size() > cap)
      return tk_fail(DSB_EINVAL, "dsb_tokenizer_decode: " + std::to_string(s.size()) + " bytes need a larger buffer");
    if (!s.empty()) std::memcpy(out, s.data(), s.size());
    if (s.size() < cap) out[s.size()] = '\0';
    return DSB_OK;
  } catch (...) {
    return tk_fail(DSB_ENOMEM, "dsb_tokenizer_decode: out of host memory");
  }
}
