// B200Engine: this engine behind the reference's engine boundary,
// wam::internal::gwp05::engine::Engine (src/models/gwp05/engine/engine.h:142-155).
//
// Compiled against the reference's own headers (engine.h and what it includes:
// artifact.h, scheduler.h, semantics.h, wam/types.h; none of them pulls in
// ggml), so the model registry can hold a B200Engine wherever it holds the
// ggml engine: Gwp05Model calls create_b200() instead of engine::create()
// (src/models/gwp05/model.cpp:134-161) and everything above the Engine
// interface (libwam_core, libwam_c_api, wam-bench, wam-compare) is unchanged.
#pragma once

#include <memory>
#include <string>

#include "models/gwp05/engine/engine.h"
#include "wam_b200.h"

namespace wam::internal::gwp05::engine {

class B200Engine final : public Engine {
 public:
  // Takes ownership of an engine created through the C ABI and fills the
  // public telemetry (cfg, resident_device_bytes, language_encoder_policy)
  // from its geometry; text_encoder: the engine was created with UMT5 (t5 = 1).
  explicit B200Engine(wam_b200_engine* handle, bool text_encoder = false);
  ~B200Engine() override;
  B200Engine(const B200Engine&) = delete;
  B200Engine& operator=(const B200Engine&) = delete;

  // Engine::predict (engine.cpp:230-449): de-normalised [action_chunk *
  // real_action_dim] actions, or {} on failure with the reason on stderr (the
  // model layer turns {} into inference_failed, model.cpp:240-245). Takes the
  // precomputed reference latent or the three camera views (vision front-end
  // on the device), and the precomputed prompt embedding or the prompt token
  // ids (UMT5 on the device, when the engine was created with it).
  std::vector<float> predict(const EngineInputsView& inputs) override;
  // Engine::reset: drops the projected-prompt cache.
  void reset() override;

 private:
  wam_b200_engine* h_ = nullptr;
  wam_b200_geometry g_{};
};

// engine::create for this engine (engine.h:202-203): loads the GGUF artifact
// at artifact_path onto options.device_index and checks it against the
// contract's geometry. nullptr on failure (the caller maps it to
// resource_exhausted, model.cpp:157-160).
std::unique_ptr<Engine> create_b200(const ArtifactContract& artifact, const EngineOptions& options,
                                    const std::string& artifact_path);

// The same over deterministic synthetic weights (no artifact), for tests and
// benchmarks.
std::unique_ptr<Engine> create_b200_synthetic(const wam_b200_options& options);

}  // namespace wam::internal::gwp05::engine
