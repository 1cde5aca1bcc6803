// Device model description: geometry, weight store, per-layer device views.
#pragma once
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/qwen_b200.h"
#include "checkpoint.h"
#include "common.cuh"

namespace qwen {

// Geometry derived from rs_qwen_config (native/mlx_bridge.h:50-53).
struct Dims {
  int H = 0, L = 0, V = 0, Hq = 0, Hkv = 0, D = 0, hk = 0, hv = 0, dk = 0, dv = 0, conv = 0,
      interval = 0, E = 0, top = 0, I = 0, S = 0, ctx = 0, chunk = 0, rope = 0;
  float eps = 1e-6f, theta = 1e7f;
  int kd = 0, vd = 0, cd = 0, n_gdn = 0, n_attn = 0;
  int gdn_in_rows = 0;   // cd + vd + 2*hv: [qkv | z | a | b]
  int attn_in_rows = 0;  // Hq*2D + 2*Hkv*D: [q+gate | k | v]
  static Dims from(const rs_qwen_config& c);
  bool is_attention(int layer) const { return (layer + 1) % interval == 0; }
  size_t state_count() const;  // native/qwen_model.inc:268-271
};

// One decoder layer's device view. The MoE expert arrays hold E+1 experts:
// index E is the shared expert (its gate scaled by sigmoid(shared_expert_gate)).
struct LayerDev {
  int mixer = 0;       // 0 = Gated-DeltaNet, 1 = gated attention
  int type_index = 0;  // index among layers of the same mixer
  const float* in_norm = nullptr;
  const float* post_norm = nullptr;
  QMat in_proj;   // DeltaNet [cd|vd|hv|hv] x H ; attention [Hq*2D|Hkv*D|Hkv*D] x H
  QMat out_proj;  // [H, vd] or [H, Hq*D]
  const float* conv_w = nullptr;  // [cd][conv]
  const float* a_log = nullptr;
  const float* dt_bias = nullptr;
  const float* gnorm = nullptr;  // [dv]
  const float* q_norm = nullptr;
  const float* k_norm = nullptr;  // [D]
  QMat router;     // [E+1, H]: router rows then shared_expert_gate
  QMat expert_gu;  // [(E+1)*2I, H]; tile rows: 64 gate rows then the 64 matching up rows
  QMat expert_dn;  // [(E+1)*H, I]
};

struct ModelDev {
  QMat embed, lm_head;
  const float* final_norm = nullptr;
  std::vector<LayerDev> layers;
  bool has_mtp = false;
  QMat mtp_fc;  // [H, 2H]
  const float* mtp_norm_emb = nullptr;
  const float* mtp_norm_hidden = nullptr;
  const float* mtp_norm = nullptr;
  LayerDev mtp_layer;  // attention + MoE
};

// Where a reference-named tensor lives on the device (for rs_mlx_weight_bytes).
struct TensorLoc {
  bool quantized = false;
  const QMat* mat = nullptr;
  int mode = 0;  // 0 plain rows, 1 expert gate rows, 2 expert up rows
  int row_offset = 0, rows = 0, cols = 0, experts = 1, per_expert = 0;
  const float* vec = nullptr;
  size_t len = 0;
};

struct WeightStore {
  int device = 0;
  bool ready = false;
  rs_qwen_config config{};
  Dims dims;
  ModelDev model;
  void* base = nullptr;  // one device allocation for every tensor
  size_t bytes = 0;
  std::map<std::string, TensorLoc> index;
  std::map<std::string, std::pair<int, int>> quant;  // rs_qwen_quant overrides
  // checkpoint tensors read by rs_mlx_weights_load (kept after the device
  // layout is built so rs_mlx_weight_bytes returns them byte for byte)
  std::map<std::string, HostTensor> host;
  bool shifted_norms = false;  // RMSNorm gains stored as offsets from 1
  // rs_qwen_forward's private device session for this store, with the
  // config bytes it was made for (rebuilt when they change; dies with the store)
  std::shared_ptr<void> forward_session;
  std::vector<uint8_t> forward_key;
  ~WeightStore();
  void synthesize(const rs_qwen_config& c, uint64_t seed, bool with_mtp);
  void load(const std::string& path);              // one safetensors shard
  void materialize(const rs_qwen_config& c);       // device layout of the loaded checkpoint
  void build(const rs_qwen_config& c, bool with_mtp, const uint64_t* seed);
  void export_bytes(const std::string& name, size_t offset, uint8_t* out, size_t count) const;
};

}  // namespace qwen
