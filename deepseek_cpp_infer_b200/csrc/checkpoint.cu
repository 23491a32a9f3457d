// Host-side checkpoint ingest: a Hugging Face model directory (config.json,
// model.safetensors.index.json + shards, or one model.safetensors) read into
// a dsb_model_config and a name-ordered list of memory-mapped tensors, then
// uploaded through dsb_model_set_tensor.
//
// Stands in for the reference's loader chain:
//   load_model_dir           src/hf/model_loader.cpp:17-94
//   load_safetensors_index   src/hf/weights_index.cpp:10-59
//   load_safetensors_header  src/hf/safetensors.cpp:42-95
//   parse_deepseek_config    src/models/deepseek/config.cpp:9-52
// with DeepSeekWeightRegistry::from_model (src/models/deepseek/weights.cpp:54-113)
// played by dsb_model_set_tensor / dsb_model_finalize.
//
// The files are untrusted input: every length, offset and shard name is
// checked before use, the JSON parser bounds its nesting, and nothing throws
// across the C ABI.

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <charconv>
#include <cstring>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "dsb_internal.h"
#include "host_json.h"

namespace dsb {
namespace {
thread_local std::string g_host_error[2];
}  // namespace

int host_fail(int code, std::string msg, HostChannel channel) {
  g_host_error[channel] = std::move(msg);
  return code;
}

const char* host_error(HostChannel channel) { return g_host_error[channel].c_str(); }
}  // namespace dsb

namespace {

using dsb::Json;
using dsb::parse_json;

int ck_fail(int code, std::string msg) { return dsb::host_fail(code, std::move(msg)); }

// --------------------------------------------------------------- files

bool read_text(const std::string& path, std::string* out) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (f == nullptr) return false;
  char buf[65536];
  size_t n;
  while ((n = std::fread(buf, 1, sizeof buf, f)) > 0) out->append(buf, n);
  const bool ok = !std::ferror(f);
  std::fclose(f);
  return ok;
}

bool file_exists(const std::string& path) {
  struct stat st;
  return ::stat(path.c_str(), &st) == 0 && S_ISREG(st.st_mode);
}

std::string join(const std::string& dir, const std::string& name) {
  if (dir.empty()) return name;
  return dir.back() == '/' ? dir + name : dir + "/" + name;
}

// A read-only mapping of one shard.
struct Shard {
  std::string path;
  const uint8_t* base = nullptr;
  size_t size = 0;
  ~Shard() {
    if (base != nullptr) ::munmap(const_cast<uint8_t*>(base), size);
  }
};

int map_shard(const std::string& path, Shard* sh) {
  const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd < 0) return ck_fail(DSB_EINVAL, "cannot open shard " + path);
  struct stat st;
  if (::fstat(fd, &st) != 0 || !S_ISREG(st.st_mode)) {
    ::close(fd);
    return ck_fail(DSB_EINVAL, "not a regular file: " + path);
  }
  sh->path = path;
  sh->size = (size_t)st.st_size;
  if (sh->size < 8) {
    ::close(fd);
    return ck_fail(DSB_EINVAL, "safetensors file too small: " + path);
  }
  void* p = ::mmap(nullptr, sh->size, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (p == MAP_FAILED) return ck_fail(DSB_EINVAL, "cannot map shard " + path);
  sh->base = static_cast<const uint8_t*>(p);
  return DSB_OK;
}

// safetensors dtype string -> (DSB_DTYPE_* or DSB_DTYPE_OTHER, bytes per element; 0 = unknown)
std::pair<int, int> dtype_of(const std::string& s) {
  if (s == "F32") return {DSB_DTYPE_F32, 4};
  if (s == "BF16") return {DSB_DTYPE_BF16, 2};
  if (s == "F16") return {DSB_DTYPE_F16, 2};
  if (s == "F8_E4M3") return {DSB_DTYPE_F8E4M3, 1};
  if (s == "F64" || s == "I64" || s == "U64") return {DSB_DTYPE_OTHER, 8};
  if (s == "I32" || s == "U32") return {DSB_DTYPE_OTHER, 4};
  if (s == "I16" || s == "U16") return {DSB_DTYPE_OTHER, 2};
  if (s == "I8" || s == "U8" || s == "BOOL" || s == "F8_E5M2") return {DSB_DTYPE_OTHER, 1};
  return {DSB_DTYPE_OTHER, 0};
}

struct Tensor {
  std::string name, dtype_name;
  int dtype = DSB_DTYPE_OTHER;
  int ndim = 0;
  int64_t shape[DSB_CKPT_MAX_DIMS] = {};
  const uint8_t* data = nullptr;
  uint64_t nbytes = 0;
};

// The tensor table of one shard's header (safetensors layout: u64 LE header
// length, a JSON object name -> {dtype, shape, data_offsets}, then the data;
// offsets relative to the data).  The reference's load_safetensors_header
// checks only end >= start; here the range must also lie inside the file and
// hold exactly numel x element-size bytes.
int read_header(const Shard& sh, std::vector<Tensor>* out) {
  uint64_t hlen = 0;
  for (int k = 0; k < 8; ++k) hlen |= (uint64_t)sh.base[k] << (8 * k);
  if (hlen > sh.size - 8) return ck_fail(DSB_EINVAL, "safetensors header length beyond the file: " + sh.path);
  Json j;
  std::string err;
  if (!parse_json(reinterpret_cast<const char*>(sh.base + 8), (size_t)hlen, &j, &err))
    return ck_fail(DSB_EINVAL, "safetensors header of " + sh.path + ": " + err);
  if (j.kind != Json::Obj) return ck_fail(DSB_EINVAL, "safetensors header is not an object: " + sh.path);
  const uint64_t data_off = 8 + hlen, data_size = sh.size - data_off;
  for (const auto& kv : j.o) {
    if (kv.first == "__metadata__") continue;
    const Json& t = kv.second;
    const std::string where = kv.first + " in " + sh.path;
    const Json* dt = t.get("dtype");
    const Json* shp = t.get("shape");
    const Json* off = t.get("data_offsets");
    if (dt == nullptr || shp == nullptr || off == nullptr || dt->kind != Json::Str || shp->kind != Json::Arr ||
        off->kind != Json::Arr)
      return ck_fail(DSB_EINVAL, "safetensors: missing or malformed fields for " + where);
    Tensor x;
    x.name = kv.first;
    x.dtype_name = dt->s;
    const auto ds = dtype_of(dt->s);
    x.dtype = ds.first;
    if (shp->a.size() > DSB_CKPT_MAX_DIMS) return ck_fail(DSB_EINVAL, "safetensors: too many dimensions for " + where);
    x.ndim = (int)shp->a.size();
    uint64_t numel = 1;
    bool overflow = false;
    for (int d = 0; d < x.ndim; ++d) {
      const Json& v = shp->a[d];
      if (v.kind != Json::Int || v.i < 0) return ck_fail(DSB_EINVAL, "safetensors: bad shape for " + where);
      x.shape[d] = v.i;
      if (v.i != 0 && numel > UINT64_MAX / 64 / (uint64_t)v.i) overflow = true;
      numel *= (uint64_t)v.i;
    }
    if (off->a.size() != 2 || off->a[0].kind != Json::Int || off->a[1].kind != Json::Int || off->a[0].i < 0 ||
        off->a[1].i < off->a[0].i)
      return ck_fail(DSB_EINVAL, "safetensors: bad data_offsets for " + where);
    const uint64_t b0 = (uint64_t)off->a[0].i, b1 = (uint64_t)off->a[1].i;
    if (b1 > data_size) return ck_fail(DSB_EINVAL, "safetensors: tensor bytes beyond the file for " + where);
    if (ds.second == 0) return ck_fail(DSB_EINVAL, "safetensors: unknown dtype " + dt->s + " for " + where);
    if (overflow || numel * (uint64_t)ds.second != b1 - b0)
      return ck_fail(DSB_EINVAL, "safetensors: byte range does not match dtype and shape for " + where);
    x.data = sh.base + data_off + b0;
    x.nbytes = b1 - b0;
    out->push_back(std::move(x));
  }
  return DSB_OK;
}

// A shard file name from the index: a plain name inside the model directory.
bool plain_file_name(const std::string& s) {
  return !s.empty() && s != "." && s != ".." && s.find('/') == std::string::npos &&
         s.find('\\') == std::string::npos && s.find('\0') == std::string::npos;
}

// ------------------------------------------------------------- config

int64_t get_int(const Json& j, const char* key, int64_t def) {
  const Json* v = j.get(key);
  if (v == nullptr) return def;
  if (v->kind == Json::Int) return v->i;
  if (v->kind == Json::Num) return (int64_t)v->d;
  if (v->kind == Json::Bool) return v->b ? 1 : 0;
  return def;
}

double get_num(const Json& j, const char* key, double def) {
  const Json* v = j.get(key);
  return v != nullptr && v->is_number() ? v->d : def;
}

std::string get_str(const Json& j, const char* key, const std::string& def) {
  const Json* v = j.get(key);
  return v != nullptr && v->kind == Json::Str ? v->s : def;
}

bool fits_int(int64_t v) { return v >= -2147483647LL && v <= 2147483647LL; }

// parse_deepseek_config (src/models/deepseek/config.cpp:9-52): the same keys,
// aliases (later keys override earlier ones) and defaults, plus the router
// and quantisation fields the reference does not read.
int parse_config(const Json& j, dsb_model_config* c) {
  if (j.kind != Json::Obj) return ck_fail(DSB_EINVAL, "config.json: root is not an object");
  std::memset(c, 0, sizeof *c);
  int64_t v[32];
  int n = 0;
  auto take = [&](int64_t x) {
    v[n++] = x;
    return x;
  };
  c->hidden_size = (int)take(get_int(j, "hidden_size", 0));
  c->intermediate_size = (int)take(get_int(j, "intermediate_size", 0));
  c->num_hidden_layers = (int)take(get_int(j, "num_hidden_layers", 0));
  c->num_attention_heads = (int)take(get_int(j, "num_attention_heads", 0));
  c->vocab_size = (int)take(get_int(j, "vocab_size", 0));
  c->max_position_embeddings = (int)take(get_int(j, "max_position_embeddings", 0));
  c->rms_norm_eps = (float)get_num(j, "rms_norm_eps", 1e-5);
  c->rope_theta = (float)get_num(j, "rope_theta", 10000.0);
  int64_t E = get_int(j, "n_routed_experts", 0);
  E = get_int(j, "num_experts", E);
  E = get_int(j, "n_experts", E);
  c->n_routed_experts = (int)take(E);
  c->n_shared_experts = (int)take(get_int(j, "n_shared_experts", 0));
  int64_t k = get_int(j, "moe_top_k", 2);
  k = get_int(j, "num_experts_per_tok", k);
  c->num_experts_per_tok = (int)take(k);
  c->moe_intermediate_size =
      (int)take(j.get("moe_intermediate_size") != nullptr ? get_int(j, "moe_intermediate_size", 0) : c->intermediate_size);
  c->first_k_dense_replace = (int)take(get_int(j, "first_k_dense_replace", 0));
  c->routed_scaling_factor = (float)get_num(j, "routed_scaling_factor", 1.0);
  c->norm_topk_prob = get_int(j, "norm_topk_prob", 0) != 0 ? 1 : 0;
  const std::string scoring = get_str(j, "scoring_func", "softmax");
  if (scoring == "softmax") c->scoring_func = DSB_SCORE_SOFTMAX;
  else if (scoring == "sigmoid") c->scoring_func = DSB_SCORE_SIGMOID;
  else return ck_fail(DSB_EUNSUPPORTED, "config.json: scoring_func \"" + scoring + "\" is not supported");
  c->n_group = (int)take(get_int(j, "n_group", 1));
  c->topk_group = (int)take(get_int(j, "topk_group", 1));
  c->q_lora_rank = (int)take(get_int(j, "q_lora_rank", 0));  // null (q_proj) reads as 0
  c->kv_lora_rank = (int)take(get_int(j, "kv_lora_rank", 0));
  c->qk_nope_head_dim = (int)take(get_int(j, "qk_nope_head_dim", 0));
  c->qk_rope_head_dim = (int)take(get_int(j, "qk_rope_head_dim", 0));
  c->v_head_dim = (int)take(get_int(j, "v_head_dim", 0));
  for (int i = 0; i < n; ++i)
    if (!fits_int(v[i])) return ck_fail(DSB_EINVAL, "config.json: an integer field is out of range");
  if (const Json* q = j.get("quantization_config"); q != nullptr && q->kind == Json::Obj) {
    const std::string method = get_str(*q, "quant_method", "");
    if (method == "fp8") {
      c->weights_fp8 = 1;
      const std::string fmt = get_str(*q, "fmt", "e4m3");
      if (fmt != "e4m3") return ck_fail(DSB_EUNSUPPORTED, "config.json: FP8 format \"" + fmt + "\" is not supported");
      if (const Json* bs = q->get("weight_block_size"); bs != nullptr) {
        const bool ok = bs->kind == Json::Arr && bs->a.size() == 2 && bs->a[0].kind == Json::Int &&
                        bs->a[1].kind == Json::Int && bs->a[0].i == 128 && bs->a[1].i == 128;
        if (!ok) return ck_fail(DSB_EUNSUPPORTED, "config.json: FP8 weight_block_size must be [128, 128]");
      }
    } else if (!method.empty()) {
      return ck_fail(DSB_EUNSUPPORTED, "config.json: quant_method \"" + method + "\" is not supported");
    }
  }
  if (c->hidden_size <= 0 || c->num_hidden_layers <= 0 || c->vocab_size <= 0)
    return ck_fail(DSB_EINVAL, "config.json missing required fields (hidden_size/num_hidden_layers/vocab_size)");
  return DSB_OK;
}

// "model.layers.<i>." prefix -> i (false for other names or an index past 9 digits)
bool layer_index(const std::string& name, int* li) {
  static const char pre[] = "model.layers.";
  const size_t np = sizeof pre - 1;
  if (name.compare(0, np, pre) != 0) return false;
  size_t j = np;
  int v = 0;
  while (j < name.size() && name[j] >= '0' && name[j] <= '9') {
    if (j - np >= 9) return false;
    v = v * 10 + (name[j] - '0');
    ++j;
  }
  if (j == np || j >= name.size() || name[j] != '.') return false;
  *li = v;
  return true;
}

bool ends_with(const std::string& s, const char* suf) {
  const size_t n = std::strlen(suf);
  return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

}  // namespace

struct dsb_checkpoint {
  std::string dir;
  dsb_model_config cfg{};
  std::vector<std::unique_ptr<Shard>> shards;
  std::vector<Tensor> tensors;  // sorted by name
};

extern "C" const char* dsb_checkpoint_error(void) { return dsb::host_error(); }

namespace {

int open_checkpoint(const std::string& dir, dsb_checkpoint* ck) {
  ck->dir = dir;
  std::string text;
  const std::string cfg_path = join(dir, "config.json");
  if (!read_text(cfg_path, &text)) return ck_fail(DSB_EINVAL, "cannot read " + cfg_path);
  Json cj;
  std::string err;
  if (!parse_json(text.data(), text.size(), &cj, &err)) return ck_fail(DSB_EINVAL, cfg_path + ": " + err);
  int rc = parse_config(cj, &ck->cfg);
  if (rc != DSB_OK) return rc;

  const std::string idx_path = join(dir, "model.safetensors.index.json");
  if (file_exists(idx_path)) {
    // load_safetensors_index + load_model_dir: the index's weight_map names
    // each tensor's shard; every shard is opened once.
    text.clear();
    if (!read_text(idx_path, &text)) return ck_fail(DSB_EINVAL, "cannot read " + idx_path);
    Json ij;
    if (!parse_json(text.data(), text.size(), &ij, &err)) return ck_fail(DSB_EINVAL, idx_path + ": " + err);
    const Json* wm = ij.get("weight_map");
    if (wm == nullptr || wm->kind != Json::Obj)
      return ck_fail(DSB_EINVAL, "safetensors index: missing weight_map object");
    std::vector<std::pair<std::string, std::string>> want;  // (tensor, shard)
    std::vector<std::string> files;
    for (const auto& kv : wm->o) {
      if (kv.second.kind != Json::Str || !plain_file_name(kv.second.s))
        return ck_fail(DSB_EINVAL, "safetensors index: bad shard name for " + kv.first);
      want.emplace_back(kv.first, kv.second.s);
      files.push_back(kv.second.s);
    }
    if (want.empty()) return ck_fail(DSB_EINVAL, "index has no shards: " + idx_path);
    std::sort(files.begin(), files.end());
    files.erase(std::unique(files.begin(), files.end()), files.end());
    std::vector<std::vector<Tensor>> headers(files.size());
    for (size_t f = 0; f < files.size(); ++f) {
      const std::string path = join(dir, files[f]);
      if (!file_exists(path)) return ck_fail(DSB_EINVAL, "missing shard: " + path);
      ck->shards.push_back(std::make_unique<Shard>());
      rc = map_shard(path, ck->shards.back().get());
      if (rc == DSB_OK) rc = read_header(*ck->shards.back(), &headers[f]);
      if (rc != DSB_OK) return rc;
      std::sort(headers[f].begin(), headers[f].end(), [](const Tensor& a, const Tensor& b) { return a.name < b.name; });
    }
    for (const auto& w : want) {
      const size_t f = (size_t)(std::lower_bound(files.begin(), files.end(), w.second) - files.begin());
      const auto& h = headers[f];
      auto it = std::lower_bound(h.begin(), h.end(), w.first, [](const Tensor& t, const std::string& n) { return t.name < n; });
      if (it == h.end() || it->name != w.first)
        return ck_fail(DSB_EINVAL, "tensor not found in shard header: " + w.first + " shard=" + join(dir, w.second));
      ck->tensors.push_back(*it);
    }
  } else {
    const std::string path = join(dir, "model.safetensors");
    if (!file_exists(path))
      return ck_fail(DSB_EINVAL, "no model.safetensors.index.json or model.safetensors in " + dir);
    ck->shards.push_back(std::make_unique<Shard>());
    rc = map_shard(path, ck->shards.back().get());
    if (rc == DSB_OK) rc = read_header(*ck->shards.back(), &ck->tensors);
    if (rc != DSB_OK) return rc;
  }
  std::sort(ck->tensors.begin(), ck->tensors.end(), [](const Tensor& a, const Tensor& b) { return a.name < b.name; });
  return DSB_OK;
}

}  // namespace

extern "C" int dsb_checkpoint_open(const char* dir, dsb_checkpoint** out) {
  if (dir == nullptr || out == nullptr) return ck_fail(DSB_EINVAL, "dsb_checkpoint_open: bad arguments");
  *out = nullptr;
  try {
    auto ck = std::make_unique<dsb_checkpoint>();
    const int rc = open_checkpoint(dir, ck.get());
    if (rc != DSB_OK) return rc;
    *out = ck.release();
    return DSB_OK;
  } catch (const std::bad_alloc&) {
    return ck_fail(DSB_ENOMEM, "dsb_checkpoint_open: out of host memory");
  } catch (...) {
    return ck_fail(DSB_EINVAL, "dsb_checkpoint_open: unexpected error");
  }
}

extern "C" int dsb_checkpoint_close(dsb_checkpoint* ck) {
  delete ck;
  return DSB_OK;
}

extern "C" int dsb_checkpoint_config(const dsb_checkpoint* ck, dsb_model_config* out) {
  if (ck == nullptr || out == nullptr) return ck_fail(DSB_EINVAL, "dsb_checkpoint_config: bad arguments");
  *out = ck->cfg;
  return DSB_OK;
}

extern "C" int dsb_checkpoint_num_tensors(const dsb_checkpoint* ck, int* n) {
  if (ck == nullptr || n == nullptr) return ck_fail(DSB_EINVAL, "dsb_checkpoint_num_tensors: bad arguments");
  *n = (int)ck->tensors.size();
  return DSB_OK;
}

extern "C" int dsb_checkpoint_tensor(const dsb_checkpoint* ck, int i, dsb_tensor_info* out) {
  if (ck == nullptr || out == nullptr || i < 0 || (size_t)i >= ck->tensors.size())
    return ck_fail(DSB_EINVAL, "dsb_checkpoint_tensor: bad arguments");
  const Tensor& t = ck->tensors[(size_t)i];
  std::memset(out, 0, sizeof *out);
  out->name = t.name.c_str();
  out->dtype_name = t.dtype_name.c_str();
  out->dtype = t.dtype;
  out->ndim = t.ndim;
  for (int d = 0; d < t.ndim; ++d) out->shape[d] = t.shape[d];
  out->data = t.data;
  out->nbytes = t.nbytes;
  return DSB_OK;
}

extern "C" int dsb_checkpoint_find(const dsb_checkpoint* ck, const char* name, int* index) {
  if (ck == nullptr || name == nullptr || index == nullptr) return ck_fail(DSB_EINVAL, "dsb_checkpoint_find: bad arguments");
  const std::string n(name);
  auto it = std::lower_bound(ck->tensors.begin(), ck->tensors.end(), n,
                             [](const Tensor& t, const std::string& key) { return t.name < key; });
  *index = (it != ck->tensors.end() && it->name == n) ? (int)(it - ck->tensors.begin()) : -1;
  return DSB_OK;
}

extern "C" int dsb_model_upload_checkpoint(dsb_model* model, const dsb_checkpoint* ck, int* n_uploaded, int* n_skipped) {
  if (model == nullptr) return DSB_EINVAL;
  dsb_ctx* ctx = dsb::model_ctx(model);
  if (ck == nullptr) return dsb::fail(ctx, DSB_EINVAL, "dsb_model_upload_checkpoint: bad arguments");
  const int layers = dsb::model_config(model)->num_hidden_layers;
  int up = 0, skip = 0;
  for (const Tensor& t : ck->tensors) {
    int li = -1;
    if (ends_with(t.name, ".rotary_emb.inv_freq") || (layer_index(t.name, &li) && li >= layers)) {
      ++skip;
      continue;
    }
    if (t.dtype == DSB_DTYPE_OTHER)
      return dsb::fail(ctx, DSB_EUNSUPPORTED, "dsb_model_upload_checkpoint: %s has dtype %s, which the model does not take",
                       t.name.c_str(), t.dtype_name.c_str());
    if (t.ndim < 1 || t.ndim > 2)
      return dsb::fail(ctx, DSB_EINVAL, "dsb_model_upload_checkpoint: %s has %d dimensions", t.name.c_str(), t.ndim);
    int rc;
    try {
      rc = dsb_model_set_tensor(model, t.name.c_str(), t.dtype, t.shape, t.ndim, t.data);
    } catch (const std::exception& e) {  // host-side conversion buffers
      return dsb::fail(ctx, DSB_ENOMEM, "dsb_model_upload_checkpoint: %s: %s", t.name.c_str(), e.what());
    }
    if (rc != DSB_OK) return rc;
    ++up;
  }
  if (n_uploaded) *n_uploaded = up;
  if (n_skipped) *n_skipped = skip;
  return DSB_OK;
}
