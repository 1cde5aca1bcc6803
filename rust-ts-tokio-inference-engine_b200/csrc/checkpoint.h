// Host-side checkpoint tensors: safetensors shards read into memory before the
// device layout is built (src/serving/weights.rs:146-260 validates the same
// headers on the Rust side; native/mlx_bridge.cpp:108-119 loads them into the
// reference's store).
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace qwen {

// dtype codes of the reference's parameter interface (mlx_bridge.cpp:181):
// 0 float32, 1 int32, 2 uint32, 3 float16, 4 bfloat16.
enum HostDtype : int { kF32 = 0, kI32 = 1, kU32 = 2, kF16 = 3, kBF16 = 4 };

struct HostTensor {
  int dtype = kF32;
  std::vector<int64_t> shape;
  std::vector<uint8_t> bytes;
  size_t elements() const {
    size_t n = 1;
    for (int64_t s : shape) n *= size_t(s);
    return n;
  }
  // element i widened to double (float dtypes only)
  double at(size_t i) const;
};

// Reads every tensor of one safetensors shard into `out`. Throws on a
// malformed header, an unsupported dtype, overlapping or out-of-file data
// ranges, or a name already present. Returns true when a tensor name marks a
// checkpoint whose RMSNorm weights are stored as offsets from 1 (an MTP
// tensor, or a depthwise conv1d.weight in [channels, 1, taps] layout;
// native/mlx_bridge.cpp:115 applies the same rule).
bool load_safetensors(const std::string& path, std::map<std::string, HostTensor>& out);

}  // namespace qwen
