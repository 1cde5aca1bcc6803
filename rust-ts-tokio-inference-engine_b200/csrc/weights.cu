// Device weight store: layout planning, seeded synthetic generation, export.
//
// The generator is this library's own: every matrix element is an
// Irwin-Hall(4) approximation of N(0, 0.02) drawn from a counter-based hash of
// (seed, tensor name, element index), quantized per 64-column group to 4-bit
// affine with bf16 scale and bias (scale = (max-min)/15, bias = min). Only
// integer arithmetic and single correctly-rounded float operations are used,
// so a CPU restatement reproduces the bytes exactly (the test oracle does).
// The tiles hold each bf16 scale and bias as the fp16 of the same value (the
// GEMM's operand type); a value fp16 cannot hold exactly raises `inexact`.
#include <algorithm>
#include <cstring>
#include <exception>
#include <memory>
#include <stdexcept>
#include <thread>
#include <tuple>

#include "model.h"

namespace qwen {

Dims Dims::from(const rs_qwen_config& c) {
  Dims d;
  d.H = c.hidden; d.L = c.layers; d.V = c.vocab; d.Hq = c.q_heads; d.Hkv = c.kv_heads;
  d.D = c.head_dim; d.hk = c.key_heads; d.hv = c.value_heads; d.dk = c.key_dim;
  d.dv = c.value_dim; d.conv = c.conv; d.interval = c.interval; d.E = c.experts;
  d.top = c.top; d.I = c.intermediate; d.S = c.shared; d.ctx = c.context; d.chunk = c.chunk;
  d.rope = c.rope_dims; d.eps = c.epsilon; d.theta = c.theta;
  d.kd = d.hk * d.dk;
  d.vd = d.hv * d.dv;
  d.cd = 2 * d.kd + d.vd;
  d.n_attn = d.interval > 0 ? d.L / d.interval : 0;
  d.n_gdn = d.L - d.n_attn;
  d.gdn_in_rows = d.cd + d.vd + 2 * d.hv;
  d.attn_in_rows = d.Hq * 2 * d.D + 2 * d.Hkv * d.D;
  return d;
}

size_t Dims::state_count() const {
  return size_t(n_gdn) * (size_t(conv - 1) * cd + size_t(hv) * dv * dk) +
         size_t(n_attn) * 2 * size_t(Hkv) * size_t(ctx) * D;
}

namespace {

uint64_t name_hash(const std::string& name) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (unsigned char ch : name) { h ^= ch; h *= 0x100000001b3ull; }
  return h;
}

uint64_t key_of(uint64_t seed, const std::string& name) {
  return mix64(seed * 0x632BE59BD9B4E019ull ^ mix64(name_hash(name)));
}

// Maps a logical row of a tensor to its device row in the (possibly fused) matrix.
__device__ inline int device_row(int mode, int row, int row_offset, int per_expert) {
  if (mode == 0) return row_offset + row;
  int e = row / per_expert, n = row % per_expert;  // per_expert = I (gate/up)
  int base = e * 2 * per_expert + (n / 64) * 128 + (n % 64);
  return row_offset + base + (mode == 2 ? 64 : 0);
}

// One thread per (logical row, 64-column group).
__global__ void synth_qmat_kernel(uint8_t* tiles, int k_chunks, long long rows, int cols,
                                  uint64_t key, float k, int mode, int row_offset,
                                  int per_expert, uint32_t* inexact) {
  long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  int groups = cols / 64;
  if (idx >= rows * groups) return;
  int row = int(idx / groups), g = int(idx % groups);
  float w[64];
  float lo, hi;
#pragma unroll
  for (int i = 0; i < 64; ++i) w[i] = synth_normal(key, uint64_t(row) * cols + g * 64 + i, k);
  lo = hi = w[0];
#pragma unroll
  for (int i = 1; i < 64; ++i) { lo = fminf(lo, w[i]); hi = fmaxf(hi, w[i]); }
  float scale = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
  uint16_t sb = float_to_bf16_bits(scale), bb = float_to_bf16_bits(lo);
  float s = bf16_bits_to_float(sb), b = bf16_bits_to_float(bb);
  uint32_t words[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) words[j] = 0;
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    float v = s > 0.0f ? rintf(__fdiv_rn(__fsub_rn(w[i], b), s)) : 0.0f;
    v = fminf(fmaxf(v, 0.0f), 15.0f);
    words[i / 8] |= uint32_t(v) << (4 * nibble_of_col(i % 8));
  }
  int drow = device_row(mode, row, row_offset, per_expert);
  uint8_t* tile = tiles + (size_t(drow / kTileRows) * k_chunks + g) * kTileBytes;
  int r = drow % kTileRows;
  uint4* dst = reinterpret_cast<uint4*>(tile + r * 32);
  dst[0] = make_uint4(words[0], words[1], words[2], words[3]);
  dst[1] = make_uint4(words[4], words[5], words[6], words[7]);
  uint16_t sh = 0, bh = 0;
  // the scale times kTileScale (exact: a power of two, checked against overflow)
  const float s512 = s * kTileScale;
  sh = __half_as_ushort(__float2half_rn(s512));
  if (__half2float(__ushort_as_half(sh)) != s512 || !bf16_to_half_bits(bb, &bh)) atomicAdd(inexact, 1u);
  reinterpret_cast<uint16_t*>(tile + kTilePackedBytes)[r] = sh;
  reinterpret_cast<uint16_t*>(tile + kTilePackedBytes + kTileRows * 2)[r] = bh;
}

__global__ void synth_vector_kernel(float* out, size_t n, uint64_t key, float k, int gain) {
  size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x;
  if (i >= n) return;
  out[i] = gain ? 1.0f : synth_normal(key, i, k);
}

// Layout planner: assigns 256-byte aligned offsets inside one allocation.
struct Planner {
  size_t total = 0;
  size_t take(size_t bytes) {
    size_t off = total;
    total += (bytes + 255) & ~size_t(255);
    return off;
  }
};

struct PendingMat {
  QMat* mat;
  size_t offset;
};
struct PendingVec {
  const float** ptr;
  size_t offset, len;
  std::string name;
  int gain;
};
struct PendingGen {  // one logical tensor written into a fused matrix
  QMat* mat;
  std::string name;
  long long rows;
  int cols, mode, row_offset, per_expert;
};

}  // namespace

WeightStore::~WeightStore() {
  forward_session.reset();  // rs_qwen_forward's session reads this store's tensors
  if (base) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    cudaFree(base);
    cudaSetDevice(prev);
  }
}

namespace {

// --- checkpoint conversion (host) ------------------------------------------

// Per-module quantization of a checkpoint tensor: the store's override, else
// the config's default (native/qwen_model.inc:16).
std::pair<int, int> quant_of(const WeightStore& w, const std::string& name, const rs_qwen_config& c) {
  auto it = w.quant.find(name);
  return it == w.quant.end() ? std::pair<int, int>{c.group, c.bits} : it->second;
}

const HostTensor& need(const WeightStore& w, const std::string& name) {
  auto it = w.host.find(name);
  if (it == w.host.end()) throw std::invalid_argument("checkpoint tensor missing: " + name);
  return it->second;
}

// q of element `col` of a row's LSB-first bitstream of `bits`-bit values
// (native/projection_reference.h:16).
inline uint32_t bits_at(const uint32_t* row, size_t col, int bits) {
  const size_t bit = col * size_t(bits), word = bit / 32;
  const unsigned shift = unsigned(bit % 32);
  uint64_t v = row[word];
  if (shift + bits > 32) v |= uint64_t(row[word + 1]) << 32;
  return uint32_t(v >> shift) & ((1u << bits) - 1u);
}

// A quantized (or plain float) logical tensor of a checkpoint, row by row.
struct SourceRows {
  const HostTensor* w = nullptr;  // packed uint32 rows, or float rows when `dense`
  const HostTensor* s = nullptr;
  const HostTensor* b = nullptr;
  int group = 64, bits = 4;
  bool dense = false;
  size_t rows = 0, cols = 0, words = 0, groups = 0;
  SourceRows(const WeightStore& st, const std::string& name, const rs_qwen_config& c, size_t n_rows, size_t n_cols)
      : rows(n_rows), cols(n_cols) {
    w = &need(st, name + ".weight");
    if (w->dtype != kU32) {  // an unquantized projection (float rows)
      dense = true;
      if (w->elements() != rows * cols) throw std::invalid_argument("checkpoint tensor shape: " + name);
      return;
    }
    std::tie(group, bits) = quant_of(st, name, c);
    words = cols * size_t(bits) / 32;
    groups = cols / size_t(group);
    if ((cols * size_t(bits)) % 32 || cols % size_t(group) || w->elements() != rows * words)
      throw std::invalid_argument("checkpoint tensor shape for its quantization: " + name);
    s = &need(st, name + ".scales");
    b = &need(st, name + ".biases");
    if (s->elements() != rows * groups || b->elements() != rows * groups)
      throw std::invalid_argument("checkpoint scales / biases shape: " + name);
  }
  bool tile_format() const { return !dense && group == 64 && bits == 4; }
  // Exact value of element (r, col) as the reference computes it: scale * q + bias.
  double value(size_t r, size_t col) const {
    if (dense) return w->at(r * cols + col);
    const uint32_t* row = reinterpret_cast<const uint32_t*>(w->bytes.data()) + r * words;
    const size_t g = r * groups + col / size_t(group);
    return s->at(g) * double(bits_at(row, col, bits)) + b->at(g);
  }
};

uint16_t half_bits(double v) { return __half_as_ushort(__float2half_rn(float(v))); }
// factor times the bf16 / fp16 / fp32 scale or bias as exact fp16 bits (tile format)
uint16_t exact_half(const HostTensor& t, size_t i, const std::string& name, double factor) {
  const double v = t.at(i) * factor;
  const uint16_t h = half_bits(v);
  if (double(half_bits_to_float(h)) != v)
    throw std::invalid_argument("scale or bias not representable in the fp16 tile format: " + name);
  return h;
}

template <class F>
void parallel_rows(size_t n, F f) {
  const unsigned hw = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
  std::vector<std::thread> pool;
  const size_t chunk = (n + hw - 1) / hw;
  std::vector<std::exception_ptr> errs(hw);
  for (unsigned t = 0; t < hw; ++t)
    pool.emplace_back([&, t] {
      try {
        for (size_t r = t * chunk; r < std::min(n, (t + 1) * chunk); ++r) f(r);
      } catch (...) {
        errs[t] = std::current_exception();
      }
    });
  for (auto& th : pool) th.join();
  for (auto& e : errs)
    if (e) std::rethrow_exception(e);
}

int host_device_row(int mode, long long row, int row_offset, int per_expert) {
  if (mode == 0) return int(row_offset + row);
  const long long e = row / per_expert, n = row % per_expert;
  return int(row_offset + e * 2 * per_expert + (n / 64) * 128 + (n % 64) + (mode == 2 ? 64 : 0));
}

}  // namespace

// Device layout for configuration `c`. seed != nullptr: seeded synthetic
// weights generated on the device; nullptr: the checkpoint tensors in `host`.
void WeightStore::build(const rs_qwen_config& c, bool with_mtp, const uint64_t* seed) {
  if (ready) throw std::invalid_argument("weight store already populated");
  Dims d = Dims::from(c);
  if (d.H <= 0 || d.H % 128 || d.L <= 0 || d.interval <= 0 || d.L % d.interval || d.V <= 0 ||
      d.I % 64 || d.S != d.I || d.D % 64 || d.dk % 64 || d.dv % 64 || d.vd % 64 ||
      (d.Hq * d.D) % 64 || d.E <= 0 || d.top <= 0 || d.top > d.E || d.hv % d.hk || d.Hq % d.Hkv)
    throw std::invalid_argument(
        "architecture unsupported: hidden must be a multiple of 128, head/expert "
        "widths multiples of 64, shared expert width equal to expert width");
  if (d.E > kMaxExperts)
    throw std::invalid_argument("architecture unsupported: the routing kernels hold at most 1024 routed experts");
  config = c;
  dims = d;
  struct MatPlan {
    QMat* mat;
    bool grouped;  // expert matrices and the embedding: tile format only
  };
  std::vector<MatPlan> mats;
  std::vector<PendingVec> vecs;
  std::vector<PendingGen> gens;
  auto qmat = [&](QMat& m, int rows, int k, bool grouped = false) {
    m = QMat();
    m.rows = rows;
    m.k = k;
    m.row_tiles = (rows + kTileRows - 1) / kTileRows;
    mats.push_back({&m, grouped});
  };
  // gain: 0 = seeded normal (synthetic) / raw values, 1 = RMSNorm gain (1 when
  // synthetic; +1 for checkpoints that store offsets), 2 = the DeltaNet gated
  // norm gain (never offset, native/qwen_model.inc:203)
  auto vec = [&](const float*& p, const std::string& name, size_t len, int gain) {
    vecs.push_back({&p, 0, len, name, gain});
  };
  auto gen = [&](QMat& m, const std::string& name, long long rows, int cols, int mode, int off,
                 int per_expert) { gens.push_back({&m, name, rows, cols, mode, off, per_expert}); };
  auto moe = [&](LayerDev& ly, const std::string& p) {
    qmat(ly.router, d.E + 1, d.H);
    gen(ly.router, p + ".mlp.gate", d.E, d.H, 0, 0, 0);
    gen(ly.router, p + ".mlp.shared_expert_gate", 1, d.H, 0, d.E, 0);
    qmat(ly.expert_gu, (d.E + 1) * 2 * d.I, d.H, true);
    gen(ly.expert_gu, p + ".mlp.switch_mlp.gate_proj", (long long)d.E * d.I, d.H, 1, 0, d.I);
    gen(ly.expert_gu, p + ".mlp.switch_mlp.up_proj", (long long)d.E * d.I, d.H, 2, 0, d.I);
    gen(ly.expert_gu, p + ".mlp.shared_expert.gate_proj", d.I, d.H, 1, d.E * 2 * d.I, d.I);
    gen(ly.expert_gu, p + ".mlp.shared_expert.up_proj", d.I, d.H, 2, d.E * 2 * d.I, d.I);
    qmat(ly.expert_dn, (d.E + 1) * d.H, d.I, true);
    gen(ly.expert_dn, p + ".mlp.switch_mlp.down_proj", (long long)d.E * d.H, d.I, 0, 0, 0);
    gen(ly.expert_dn, p + ".mlp.shared_expert.down_proj", d.H, d.I, 0, d.E * d.H, 0);
  };
  auto attention = [&](LayerDev& ly, const std::string& p) {
    std::string a = p + ".self_attn";
    qmat(ly.in_proj, d.attn_in_rows, d.H);
    gen(ly.in_proj, a + ".q_proj", d.Hq * 2 * d.D, d.H, 0, 0, 0);
    gen(ly.in_proj, a + ".k_proj", d.Hkv * d.D, d.H, 0, d.Hq * 2 * d.D, 0);
    gen(ly.in_proj, a + ".v_proj", d.Hkv * d.D, d.H, 0, d.Hq * 2 * d.D + d.Hkv * d.D, 0);
    vec(ly.q_norm, a + ".q_norm.weight", d.D, 1);
    vec(ly.k_norm, a + ".k_norm.weight", d.D, 1);
    qmat(ly.out_proj, d.H, d.Hq * d.D);
    gen(ly.out_proj, a + ".o_proj", d.H, d.Hq * d.D, 0, 0, 0);
  };
  model = ModelDev();
  qmat(model.embed, d.V, d.H, true);
  gen(model.embed, "language_model.model.embed_tokens", d.V, d.H, 0, 0, 0);
  qmat(model.lm_head, d.V, d.H);
  gen(model.lm_head, "language_model.lm_head", d.V, d.H, 0, 0, 0);
  vec(model.final_norm, "language_model.model.norm.weight", d.H, 1);
  model.layers.resize(d.L);
  int n_gdn = 0, n_attn = 0;
  for (int i = 0; i < d.L; ++i) {
    LayerDev& ly = model.layers[i];
    std::string p = "language_model.model.layers." + std::to_string(i);
    vec(ly.in_norm, p + ".input_layernorm.weight", d.H, 1);
    vec(ly.post_norm, p + ".post_attention_layernorm.weight", d.H, 1);
    if (d.is_attention(i)) {
      ly.mixer = 1;
      ly.type_index = n_attn++;
      attention(ly, p);
    } else {
      ly.mixer = 0;
      ly.type_index = n_gdn++;
      std::string g = p + ".linear_attn";
      qmat(ly.in_proj, d.gdn_in_rows, d.H);
      gen(ly.in_proj, g + ".in_proj_qkv", d.cd, d.H, 0, 0, 0);
      gen(ly.in_proj, g + ".in_proj_z", d.vd, d.H, 0, d.cd, 0);
      gen(ly.in_proj, g + ".in_proj_a", d.hv, d.H, 0, d.cd + d.vd, 0);
      gen(ly.in_proj, g + ".in_proj_b", d.hv, d.H, 0, d.cd + d.vd + d.hv, 0);
      vec(ly.conv_w, g + ".conv1d.weight", size_t(d.cd) * d.conv, 0);
      vec(ly.a_log, g + ".A_log", d.hv, 0);
      vec(ly.dt_bias, g + ".dt_bias", d.hv, 0);
      vec(ly.gnorm, g + ".norm.weight", d.dv, 2);
      qmat(ly.out_proj, d.H, d.vd);
      gen(ly.out_proj, g + ".out_proj", d.H, d.vd, 0, 0, 0);
    }
    moe(ly, p);
  }
  model.has_mtp = with_mtp;
  if (with_mtp) {
    std::string m = "language_model.mtp";
    vec(model.mtp_norm_emb, m + ".pre_fc_norm_embedding.weight", d.H, 1);
    vec(model.mtp_norm_hidden, m + ".pre_fc_norm_hidden.weight", d.H, 1);
    qmat(model.mtp_fc, d.H, 2 * d.H);
    gen(model.mtp_fc, m + ".fc", d.H, 2 * d.H, 0, 0, 0);
    LayerDev& ly = model.mtp_layer;
    ly.mixer = 1;
    ly.type_index = 0;
    std::string p = m + ".layers.0";
    vec(ly.in_norm, p + ".input_layernorm.weight", d.H, 1);
    vec(ly.post_norm, p + ".post_attention_layernorm.weight", d.H, 1);
    attention(ly, p);
    moe(ly, p);
    vec(model.mtp_norm, m + ".norm.weight", d.H, 1);
  }

  // Checkpoint sources; a fused matrix holding any tensor outside 4-bit g64
  // (a quantization override, or float rows) is kept as dense fp16 rows
  // (dense projections only: the grouped MoE GEMM and the embedding read tiles).
  std::vector<std::unique_ptr<SourceRows>> src(gens.size());
  if (!seed) {
    for (size_t i = 0; i < gens.size(); ++i) {
      const auto& g = gens[i];
      src[i] = std::make_unique<SourceRows>(*this, g.name, c, size_t(g.rows), size_t(g.cols));
      if (!src[i]->tile_format()) const_cast<QMat*>(g.mat)->dense_f16 = true;
    }
    for (const auto& mp : mats)
      if (mp.mat->dense_f16 && mp.grouped)
        throw std::invalid_argument("expert and embedding tensors must be 4-bit affine, group 64 (the tensor-core "
                                    "MoE GEMM and the embedding kernel read that format only)");
  }
  Planner plan;
  std::vector<size_t> mat_off(mats.size());
  for (size_t i = 0; i < mats.size(); ++i) {
    const QMat& m = *mats[i].mat;
    mat_off[i] = plan.take(m.dense_f16 ? size_t(m.rows) * m.k * 2 : size_t(m.row_tiles) * (m.k / kTileK) * kTileBytes);
  }
  for (auto& pv : vecs) pv.offset = plan.take(pv.len * 4);

  QWEN_CUDA(cudaGetDevice(&device));
  QWEN_CUDA(cudaMalloc(&base, plan.total));
  bytes = plan.total;
  QWEN_CUDA(cudaMemset(base, 0, plan.total));  // zero padding rows and tiles
  uint8_t* b8 = static_cast<uint8_t*>(base);
  for (size_t i = 0; i < mats.size(); ++i) mats[i].mat->tiles = b8 + mat_off[i];
  const float k = 0.02f / 37837.2265f;
  for (auto& pv : vecs) {
    float* p = reinterpret_cast<float*>(b8 + pv.offset);
    *pv.ptr = p;
    if (seed) {
      synth_vector_kernel<<<unsigned((pv.len + 255) / 256), 256>>>(p, pv.len, key_of(*seed, pv.name), k,
                                                                   pv.gain != 0);
      QWEN_CUDA(cudaGetLastError());
    } else {
      const HostTensor& t = need(*this, pv.name);
      if (t.elements() != pv.len) throw std::invalid_argument("checkpoint vector length: " + pv.name);
      std::vector<float> v(pv.len);
      for (size_t i = 0; i < pv.len; ++i)
        v[i] = float(t.at(i)) + ((pv.gain == 1 && shifted_norms) ? 1.f : 0.f);
      QWEN_CUDA(cudaMemcpy(p, v.data(), pv.len * 4, cudaMemcpyHostToDevice));
    }
    TensorLoc loc;
    loc.vec = p;
    loc.len = pv.len;
    index[pv.name] = loc;
  }
  if (seed) {
    uint32_t* inexact = nullptr;
    QWEN_CUDA(cudaMalloc(&inexact, 4));
    QWEN_CUDA(cudaMemset(inexact, 0, 4));
    for (auto& g : gens) {
      long long threads = g.rows * (g.cols / 64);
      synth_qmat_kernel<<<unsigned((threads + 255) / 256), 256>>>(
          const_cast<uint8_t*>(g.mat->tiles), g.cols / 64, g.rows, g.cols, key_of(*seed, g.name), k,
          g.mode, g.row_offset, g.per_expert, inexact);
      QWEN_CUDA(cudaGetLastError());
    }
    QWEN_CUDA(cudaDeviceSynchronize());
    uint32_t n_inexact = 0;
    QWEN_CUDA(cudaMemcpy(&n_inexact, inexact, 4, cudaMemcpyDeviceToHost));
    QWEN_CUDA(cudaFree(inexact));
    if (n_inexact)
      throw std::runtime_error("quantized weights carry scales or biases outside the fp16 range (" +
                               std::to_string(n_inexact) + " groups)");
  } else {
    // one host image per fused matrix, filled in parallel, then one copy
    for (size_t mi = 0; mi < mats.size(); ++mi) {
      QMat& m = *mats[mi].mat;
      const size_t img_bytes = m.dense_f16 ? size_t(m.rows) * m.k * 2
                                           : size_t(m.row_tiles) * (m.k / kTileK) * kTileBytes;
      std::vector<uint8_t> img(img_bytes, 0);
      for (size_t gi = 0; gi < gens.size(); ++gi) {
        const PendingGen& g = gens[gi];
        if (g.mat != &m) continue;
        const SourceRows& sr = *src[gi];
        parallel_rows(size_t(g.rows), [&](size_t r) {
          const int drow = host_device_row(g.mode, (long long)r, g.row_offset, g.per_expert);
          if (m.dense_f16) {  // scale * q + bias rounded once to fp16, as the tile path's dequantisation does
            uint16_t* dst = reinterpret_cast<uint16_t*>(img.data()) + size_t(drow) * m.k;
            for (size_t col = 0; col < sr.cols; ++col) dst[col] = half_bits(sr.value(r, col));
            return;
          }
          const uint32_t* row = reinterpret_cast<const uint32_t*>(sr.w->bytes.data()) + r * sr.words;
          for (size_t gq = 0; gq < sr.groups; ++gq) {
            uint8_t* tile = img.data() + (size_t(drow / kTileRows) * (m.k / kTileK) + gq) * kTileBytes;
            const int tr = drow % kTileRows;
            uint32_t words[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int cc = 0; cc < 64; ++cc)  // canonical nibble cc%8 of word cc/8 -> pair-interleaved order
              words[cc / 8] |= ((row[gq * 8 + cc / 8] >> (4 * (cc % 8))) & 15u) << (4 * nibble_of_col(cc % 8));
            std::memcpy(tile + tr * 32, words, 32);
            const uint16_t sh = exact_half(*sr.s, r * sr.groups + gq, g.name, kTileScale);
            const uint16_t bh = exact_half(*sr.b, r * sr.groups + gq, g.name, 1.0);
            std::memcpy(tile + kTilePackedBytes + tr * 2, &sh, 2);
            std::memcpy(tile + kTilePackedBytes + kTileRows * 2 + tr * 2, &bh, 2);
          }
        });
      }
      QWEN_CUDA(cudaMemcpy(const_cast<uint8_t*>(m.tiles), img.data(), img_bytes, cudaMemcpyHostToDevice));
    }
  }
  for (auto& g : gens) {
    TensorLoc loc;
    loc.quantized = true;
    loc.mat = g.mat;
    loc.mode = g.mode;
    loc.row_offset = g.row_offset;
    loc.rows = int(g.rows);
    loc.cols = g.cols;
    loc.per_expert = g.per_expert;
    index[g.name] = loc;
  }
  ready = true;
}

void WeightStore::synthesize(const rs_qwen_config& c, uint64_t seed, bool with_mtp) {
  if (!host.empty()) throw std::invalid_argument("weight store holds checkpoint tensors");
  build(c, with_mtp, &seed);
}

void WeightStore::load(const std::string& path) {
  if (ready) throw std::invalid_argument("weight store already populated");
  shifted_norms = load_safetensors(path, host) || shifted_norms;
}

void WeightStore::materialize(const rs_qwen_config& c) {
  if (ready) return;
  if (host.empty()) throw std::invalid_argument("weight store is empty");
  build(c, host.count("language_model.mtp.fc.weight") > 0, nullptr);
}

// Reference canonical bytes of a named tensor (native/mlx_bridge.cpp:177-187
// semantics): "<name>.weight" packed uint32 rows, "<name>.scales"/".biases"
// float32 [rows, cols/64], vectors float32.
void WeightStore::export_bytes(const std::string& full, size_t offset, uint8_t* out,
                               size_t count) const {
  auto hit = host.find(full);
  if (hit != host.end()) {  // a checkpoint tensor: its bytes as loaded
    const HostTensor& t = hit->second;
    if (offset > t.bytes.size() || count > t.bytes.size() - offset) throw std::invalid_argument("tensor byte range");
    std::memcpy(out, t.bytes.data() + offset, count);
    return;
  }
  if (!ready) throw std::invalid_argument("unknown tensor: " + full);
  std::string name = full, part;
  for (const char* suffix : {".weight", ".scales", ".biases"}) {
    size_t n = std::strlen(suffix);
    if (full.size() > n && full.compare(full.size() - n, n, suffix) == 0 &&
        index.count(full.substr(0, full.size() - n)) &&
        index.at(full.substr(0, full.size() - n)).quantized) {
      name = full.substr(0, full.size() - n);
      part = suffix;
    }
  }
  auto it = index.find(name);
  if (it == index.end()) throw std::invalid_argument("unknown tensor: " + full);
  const TensorLoc& loc = it->second;
  if (!loc.quantized) {
    if (offset > loc.len * 4 || count > loc.len * 4 - offset)
      throw std::invalid_argument("tensor byte range");
    QWEN_CUDA(cudaMemcpy(out, reinterpret_cast<const uint8_t*>(loc.vec) + offset, count,
                         cudaMemcpyDeviceToHost));
    return;
  }
  const size_t cols = loc.cols, groups = cols / 64;
  const size_t row_bytes = part == ".weight" ? cols / 2 : groups * 4;
  if (offset > size_t(loc.rows) * row_bytes || count > size_t(loc.rows) * row_bytes - offset)
    throw std::invalid_argument("tensor byte range");
  if (!count) return;
  const size_t r0 = offset / row_bytes, r1 = (offset + count - 1) / row_bytes;
  std::vector<uint8_t> rowbuf(row_bytes), tile(kTileBytes);
  const QMat& m = *loc.mat;
  for (size_t r = r0; r <= r1; ++r) {
    int drow;
    if (loc.mode == 0) {
      drow = loc.row_offset + int(r);
    } else {
      int e = int(r) / loc.per_expert, n = int(r) % loc.per_expert;
      drow = loc.row_offset + e * 2 * loc.per_expert + (n / 64) * 128 + (n % 64) + (loc.mode == 2 ? 64 : 0);
    }
    for (size_t g = 0; g < groups; ++g) {
      const uint8_t* t = m.tile(drow / kTileRows, int(g));
      int lr = drow % kTileRows;
      if (part == ".weight") {
        uint32_t dev[8], canon[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        QWEN_CUDA(cudaMemcpy(dev, t + lr * 32, 32, cudaMemcpyDeviceToHost));
        for (int w = 0; w < 8; ++w)
          for (int i = 0; i < 8; ++i) canon[w] |= ((dev[w] >> (4 * i)) & 15u) << (4 * col_of_nibble(i));
        std::memcpy(rowbuf.data() + g * 32, canon, 32);
      } else {
        uint16_t bits;
        size_t off = kTilePackedBytes + (part == ".scales" ? 0 : kTileRows * 2) + lr * 2;
        QWEN_CUDA(cudaMemcpy(&bits, t + off, 2, cudaMemcpyDeviceToHost));
        // the checkpoint's bf16 value, widened exactly (scales are stored times kTileScale)
        const float v = half_bits_to_float(bits) / (part == ".scales" ? kTileScale : 1.f);
        std::memcpy(rowbuf.data() + g * 4, &v, 4);
      }
    }
    size_t row_begin = r * row_bytes;
    size_t lo = std::max(offset, row_begin), hi = std::min(offset + count, row_begin + row_bytes);
    std::memcpy(out + (lo - offset), rowbuf.data() + (lo - row_begin), hi - lo);
  }
}

}  // namespace qwen
