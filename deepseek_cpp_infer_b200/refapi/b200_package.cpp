// ds::rt::Model / ModelSession over libdsb.so, for the reference engine's
// plug-in API (see b200_package.h).  Errors are thrown as std::runtime_error,
// as the reference's model and sessions do; no libdsb error is swallowed.

#include "b200_package.h"

#include "ds/models/deepseek/package.h"
#include "ds/runtime/model.h"
#include "dsb/dsb.h"

#include <algorithm>
#include <stdexcept>
#include <string>
#include <vector>

namespace ds::models::b200 {
namespace {

// The device context and model that a model and its sessions share.
struct Device {
  dsb_ctx* ctx = nullptr;
  dsb_model* model = nullptr;
  dsb_model_config cfg{};
  ~Device() {
    if (model != nullptr) dsb_model_destroy(model);
    if (ctx != nullptr) dsb_ctx_destroy(ctx);
  }
  void check(int rc, const char* what) const {
    if (rc != DSB_OK)
      throw std::runtime_error(std::string(what) + ": " + dsb_last_error(ctx) + " (dsb error " + std::to_string(rc) +
                               ")");
  }
};

// One sequence in a paged latent KV cache (DeepSeekSession, model.h:16-39).
class B200Session final : public ds::rt::ModelSession {
 public:
  B200Session(std::shared_ptr<Device> dev, std::size_t max_seq) : dev_(std::move(dev)), max_seq_(max_seq) {
    const int pages = static_cast<int>((max_seq_ + 63) / 64);
    dev_->check(dsb_kvcache_create(dev_->ctx, dev_->model, pages, 1, pages, &kv_), "dsb_kvcache_create");
    dev_->check(dsb_kvcache_alloc_seq(kv_, &seq_), "dsb_kvcache_alloc_seq");
  }
  ~B200Session() override {
    if (kv_ != nullptr) dsb_kvcache_destroy(kv_);
  }
  B200Session(const B200Session&) = delete;
  B200Session& operator=(const B200Session&) = delete;

  // DeepSeekSession::reset (model.cpp:57-69): position 0, an empty cache.
  void reset() override {
    dev_->check(dsb_kvcache_reset(kv_), "dsb_kvcache_reset");
    dev_->check(dsb_kvcache_alloc_seq(kv_, &seq_), "dsb_kvcache_alloc_seq");
    pos_ = 0;
  }
  std::size_t position() const override { return pos_; }

 private:
  friend class B200Model;
  std::shared_ptr<Device> dev_;
  dsb_kvcache* kv_ = nullptr;
  int seq_ = -1;
  std::size_t pos_ = 0, max_seq_ = 0;
};

class B200Model final : public ds::rt::Model {
 public:
  explicit B200Model(std::shared_ptr<Device> dev) : dev_(std::move(dev)) {
    info_.family_id = "deepseek";
    info_.model_type = "deepseek_b200";
    info_.vocab_size = dev_->cfg.vocab_size;
    info_.max_position_embeddings = dev_->cfg.max_position_embeddings;
    info_.supported_backends.push_back(ds::rt::BackendKind::CUDA);
  }

  const ds::rt::ModelInfo& info() const override { return info_; }

  // A session of run_cfg.max_seq positions (0: max_position_embeddings, as
  // DeepSeekSession does, model.cpp:34); the B200 path is a CUDA backend.
  std::unique_ptr<ds::rt::ModelSession> create_session(const ds::rt::RunConfig& run_cfg) const override {
    if (run_cfg.backend != ds::rt::BackendKind::CUDA)
      throw std::runtime_error("b200 package: the model runs on the CUDA backend only (RunConfig.backend = cuda)");
    const std::size_t max_seq =
        run_cfg.max_seq != 0 ? run_cfg.max_seq : static_cast<std::size_t>(std::max(1, info_.max_position_embeddings));
    return std::make_unique<B200Session>(dev_, max_seq);
  }

  // DeepSeekModel::forward (model.cpp:89-110): the input tokens in order
  // (more than one as a chunked batched prefill), the logits and greedy id
  // after the last; the same errors as the reference's forward / decode_next.
  ds::rt::ForwardOutput forward(ds::rt::ModelSession& session, const ds::rt::ForwardInput& input) const override {
    auto* s = dynamic_cast<B200Session*>(&session);
    if (s == nullptr || s->dev_ != dev_) throw std::runtime_error("b200 model requires a session it created");
    const std::vector<std::int32_t>& ids = input.token_ids;
    if (ids.empty()) throw std::runtime_error("forward: token_ids must not be empty");
    if (s->pos_ + ids.size() > s->max_seq_) throw std::runtime_error("executor: max sequence length reached");
    ds::rt::ForwardOutput out;
    out.logits.assign(static_cast<std::size_t>(info_.vocab_size), 0.0f);
    if (ids.size() == 1) {
      dev_->check(dsb_decode_step(dev_->ctx, dev_->model, s->kv_, &s->seq_, ids.data(), 1, out.logits.data(),
                                  &out.greedy_token_id),
                  "dsb_decode_step");
    } else {
      for (std::size_t c = 0; c < ids.size(); c += DSB_PREFILL_MAX_TOKENS) {
        const int n = static_cast<int>(std::min<std::size_t>(DSB_PREFILL_MAX_TOKENS, ids.size() - c));
        const std::vector<std::int32_t> seq_ids(static_cast<std::size_t>(n), s->seq_);
        int n_seq = 0;
        dev_->check(dsb_prefill(dev_->ctx, dev_->model, s->kv_, seq_ids.data(), ids.data() + c, n, out.logits.data(),
                                &out.greedy_token_id, &n_seq),
                    "dsb_prefill");
      }
    }
    s->pos_ += ids.size();
    out.position_after = s->pos_;
    return out;
  }

 private:
  std::shared_ptr<Device> dev_;
  ds::rt::ModelInfo info_;
};

std::shared_ptr<const ds::rt::Model> load_from_descriptor(const std::string& model_dir, const ds::hf::ModelConfig&) {
  return load_model(model_dir, 0);
}

}  // namespace

std::shared_ptr<const ds::rt::Model> load_model(const std::string& model_dir, int device) {
  dsb_checkpoint* ck = nullptr;
  int rc = dsb_checkpoint_open(model_dir.c_str(), &ck);
  if (rc != DSB_OK) throw std::runtime_error(std::string("b200 package: ") + dsb_checkpoint_error());
  struct Close {
    dsb_checkpoint* ck;
    ~Close() { dsb_checkpoint_close(ck); }
  } close{ck};
  auto dev = std::make_shared<Device>();
  dsb_checkpoint_config(ck, &dev->cfg);
  rc = dsb_ctx_create(device, &dev->ctx);
  if (rc != DSB_OK)
    throw std::runtime_error("b200 package: no usable CUDA device " + std::to_string(device) + " (dsb error " +
                             std::to_string(rc) + ")");
  dev->check(dsb_model_create(dev->ctx, &dev->cfg, &dev->model), "dsb_model_create");
  dev->check(dsb_model_upload_checkpoint(dev->model, ck, nullptr, nullptr), "dsb_model_upload_checkpoint");
  dev->check(dsb_model_finalize(dev->model), "dsb_model_finalize");
  return std::make_shared<const B200Model>(std::move(dev));
}

const ds::models::core::ModelPackageDescriptor& package_descriptor() {
  static const ds::models::core::ModelPackageDescriptor descriptor = [] {
    ds::models::core::ModelPackageDescriptor d = ds::models::deepseek::package_descriptor();
    d.package_id = "deepseek_b200";
    d.load = load_from_descriptor;
    return d;
  }();
  return descriptor;
}

}  // namespace ds::models::b200
