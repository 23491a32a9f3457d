// The B200 model package for the reference engine's own plug-in API.
//
// Built against the reference's headers (include/ds/...), this is the
// drop-in for its per-token decode path: ds::rt::Model and
// ds::rt::ModelSession (include/ds/runtime/model.h:37-51) implemented over
// libdsb.so, and a ModelPackageDescriptor
// (include/ds/models/core/registry.h:23-30) whose load() returns that model.
// The reference's ds::rt::generate (src/runtime/model.cpp:14-49),
// ModelExecutor (src/runtime/model_executor.cpp:18-50) and ds_chat then run
// the B200 path unchanged.  The package keeps the DeepSeek package's
// matches / print_config / inspect_index / inspect_loaded (host-only, off
// the hot path) and replaces only load
// (src/models/deepseek/package.cpp:140-150).
#pragma once

#include "ds/models/core/registry.h"

#include <memory>
#include <string>

namespace ds::models::b200 {

// The descriptor to list in the reference's builtin_packages()
// (src/models/core/registry.cpp:9-14) ahead of, or instead of, the DeepSeek one.
const ds::models::core::ModelPackageDescriptor& package_descriptor();

// load() of the descriptor: the checkpoint directory read by libdsb.so's
// reader and uploaded to CUDA device `device` (0 through the descriptor).
std::shared_ptr<const ds::rt::Model> load_model(const std::string& model_dir, int device = 0);

}  // namespace ds::models::b200
