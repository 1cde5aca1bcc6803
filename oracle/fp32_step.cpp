// TEST INFRASTRUCTURE — the timed CPU baseline: an fp32, multi-threaded
// restatement of one batched decode step of the hybrid Qwen decoder.
//
// Only bench.py's CPU legs (cpu_baseline, --impl reference) and tests/ load
// this code; the product library never links or calls it.
//
// It computes what the FP64 oracle (qwen_oracle.cpp) computes, with the
// reference's per-layer order (native/qwen_model.inc:75-206 for MoE,
// attention and Gated-DeltaNet, :277-373 for the layer loop), in float, over a
// whole batch at once the way a CPU serving engine would run it:
//   - every projection reads each weight row once per step for all tokens: a
//     row's 4-bit groups are unpacked once and dotted with every token, using
//     the affine identity x.(s*q + b) = s*(x.q) + b*sum(x) per 64-column group
//     (native/projection_reference.h:8-22 element formula, factored);
//   - the MoE visits each routed expert once with the tokens routed to it;
//   - DeltaNet recurrences and attention heads run per (sequence, head);
//   - work is spread over a persistent pool of std::thread workers.
// Weights are the same seeded synthetic bytes as the device store and the
// oracle (synth.h); K/V caches are stored as bf16 like the device's.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <functional>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "../include/qwen_b200.h"
#include "synth.h"

namespace {

thread_local std::string f_error;

template <class F>
int guard(F f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    f_error = e.what();
  } catch (...) {
    f_error = "unknown fp32 step exception";
  }
  return -1;
}

// Persistent worker pool: run(n, fn) calls fn(i) for i in [0, n) on all
// workers (the caller included), handing out indices with an atomic counter.
class Pool {
 public:
  explicit Pool(int threads) : n_(std::max(1, threads)) {
    for (int i = 1; i < n_; ++i) workers_.emplace_back([this] { loop(); });
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> lock(mu_);
      stop_ = true;
      ++gen_;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  int size() const { return n_; }
  void run(size_t n, const std::function<void(size_t)>& fn) {
    if (n == 0) return;
    if (n == 1 || n_ == 1) {
      for (size_t i = 0; i < n; ++i) fn(i);
      return;
    }
    {
      std::lock_guard<std::mutex> lock(mu_);
      job_ = &fn;
      total_ = n;
      next_.store(0);
      busy_ = n_ - 1;
      ++gen_;
    }
    cv_.notify_all();
    work();
    std::unique_lock<std::mutex> lock(mu_);
    done_cv_.wait(lock, [this] { return busy_ == 0; });
    job_ = nullptr;
  }

 private:
  void work() {
    for (;;) {
      const size_t i = next_.fetch_add(1);
      if (i >= total_) break;
      (*job_)(i);
    }
  }
  void loop() {
    uint64_t seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lock(mu_);
        cv_.wait(lock, [&] { return gen_ != seen; });
        seen = gen_;
        if (stop_) return;
      }
      work();
      std::lock_guard<std::mutex> lock(mu_);
      if (--busy_ == 0) done_cv_.notify_one();
    }
  }
  int n_;
  std::vector<std::thread> workers_;
  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(size_t)>* job_ = nullptr;
  size_t total_ = 0;
  std::atomic<size_t> next_{0};
  int busy_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

float sigm(float x) { return 1.f / (1.f + std::exp(-x)); }
float silu(float x) { return x * sigm(x); }
uint16_t to_bf16(float f) { return synth::bf16_rne(f); }
float from_bf16(uint16_t b) { return synth::bf16_to_float(b); }

// 4-bit affine g64 matrix in the reference's canonical packing (nibble c%8 of
// word c/8), with the bf16 scales and biases widened to float.
struct QW {
  size_t rows = 0, cols = 0;
  std::vector<uint32_t> packed;
  std::vector<float> scale, bias;

  void generate(uint64_t seed, const std::string& name, size_t r, size_t c, Pool& pool) {
    if (c % 64) throw std::invalid_argument("fp32 step: width not a multiple of 64: " + name);
    rows = r;
    cols = c;
    packed.assign(r * c / 8, 0);
    scale.assign(r * c / 64, 0.f);
    bias.assign(r * c / 64, 0.f);
    const uint64_t key = synth::tensor_key(seed, synth::tensor_id(name));
    const size_t blocks = (r + 63) / 64;
    pool.run(blocks, [&](size_t b) {
      float w[64];
      uint8_t q[64];
      for (size_t row = b * 64; row < std::min(r, b * 64 + 64); ++row)
        for (size_t g = 0; g < c / 64; ++g) {
          for (int i = 0; i < 64; ++i) w[i] = synth::normal(key, row * c + g * 64 + i, 0.02f);
          uint16_t sb, bb;
          synth::quantize_group(w, q, &sb, &bb);
          scale[row * (c / 64) + g] = synth::bf16_to_float(sb);
          bias[row * (c / 64) + g] = synth::bf16_to_float(bb);
          uint32_t* words = &packed[row * (c / 8) + g * 8];
          for (int i = 0; i < 64; ++i) words[i / 8] |= uint32_t(q[i]) << (4 * (i % 8));
        }
    });
  }
};

// Built with AVX2 + FMA (oracle/Makefile); f32_create refuses hosts without them.
// The 64 nibbles of one group as floats (word w holds columns 8w..8w+7).
inline void unpack64(const uint32_t* words, float* q) {
  for (int w = 0; w < 8; ++w)
    for (int j = 0; j < 8; ++j) q[w * 8 + j] = float((words[w] >> (4 * j)) & 15u);
}

// Per-token group sums of x [T][cols] (the bias term of the factored dot).
std::vector<float> group_sums(const float* x, size_t T, size_t cols) {
  std::vector<float> s(T * (cols / 64));
  for (size_t t = 0; t < T; ++t)
    for (size_t g = 0; g < cols / 64; ++g) {
      float v = 0;
      for (int i = 0; i < 64; ++i) v += x[t * cols + g * 64 + i];
      s[t * (cols / 64) + g] = v;
    }
  return s;
}

// y[t][o] (row stride ldy) = x[tok[t]] . deq(W)[row0 + o] for o < n_out,
// t < T; tok == null means token t reads x row t. Rows are split over the pool.
void project(const QW& W, size_t row0, size_t n_out, const float* x, const float* xs, const int32_t* tok,
             size_t T, float* y, size_t ldy, Pool& pool, size_t rows_per_item = 16) {
  if (row0 + n_out > W.rows) throw std::invalid_argument("fp32 step: projection rows out of range");
  const size_t G = W.cols / 64;
  const size_t items = (n_out + rows_per_item - 1) / rows_per_item;
  auto body = [&](size_t it) {
    float q[64];
    // per token: 8 running lanes of s*q.x (reduced once per row) and the b*sum(x) term
    std::vector<float> acc(T * 8), bsum(T);
    for (size_t o = it * rows_per_item; o < std::min(n_out, (it + 1) * rows_per_item); ++o) {
      const size_t r = row0 + o;
      std::fill(acc.begin(), acc.end(), 0.f);
      std::fill(bsum.begin(), bsum.end(), 0.f);
      for (size_t g = 0; g < G; ++g) {
        unpack64(&W.packed[r * (W.cols / 8) + g * 8], q);
        const float s = W.scale[r * G + g], b = W.bias[r * G + g];
        for (int i = 0; i < 64; ++i) q[i] *= s;
        for (size_t t = 0; t < T; ++t) {
          const size_t xr = tok ? size_t(tok[t]) : t;
          const float* xp = x + xr * W.cols + g * 64;
          float av[8];
          for (int j = 0; j < 8; ++j) av[j] = acc[t * 8 + j];
          for (int k = 0; k < 8; ++k)
            for (int j = 0; j < 8; ++j) av[j] += q[k * 8 + j] * xp[k * 8 + j];
          for (int j = 0; j < 8; ++j) acc[t * 8 + j] = av[j];
          bsum[t] += b * xs[xr * G + g];
        }
      }
      for (size_t t = 0; t < T; ++t) {
        const float* a = &acc[t * 8];
        y[t * ldy + o] = (((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]))) + bsum[t];
      }
    }
  };
  if (items == 1)
    body(0);
  else
    pool.run(items, body);
}

void rms(const float* x, float* y, size_t width, const float* w, float eps) {
  double s = 0;
  for (size_t i = 0; i < width; ++i) s += double(x[i]) * x[i];
  const float inv = float(1.0 / std::sqrt(s / double(width) + eps));
  for (size_t i = 0; i < width; ++i) y[i] = x[i] * inv * (w ? w[i] : 1.f);
}

void rope(float* v, int rotary, double pos, double theta) {
  for (int j = 0; j < rotary / 2; ++j) {
    const double a = pos * std::pow(theta, -2.0 * j / rotary);
    const float c = float(std::cos(a)), s = float(std::sin(a));
    const float x0 = v[j], x1 = v[j + rotary / 2];
    v[j] = x0 * c - x1 * s;
    v[j + rotary / 2] = x0 * s + x1 * c;
  }
}

uint32_t total_key(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return (u & 0x80000000u) ? ~u : (u ^ 0x80000000u);
}

struct Layer {
  bool attention = false;
  std::vector<float> in_norm, post_norm;
  // DeltaNet
  QW qkv, z, a, b, out;
  std::vector<float> conv_w, a_log, dt_bias, gnorm;
  // attention
  QW qp, kp, vp, op;
  std::vector<float> q_norm, k_norm;
  // MoE
  QW router, sh_gate_row, gate, up, down, sh_gate, sh_up, sh_down;
};

struct Seq {
  size_t pos = 0, cap = 0;
  std::vector<std::vector<float>> conv, S;       // per DeltaNet layer
  std::vector<std::vector<uint16_t>> K, V;       // per attention layer: [kv][cap][d] bf16
};

struct Model {
  rs_qwen_config c{};
  std::unique_ptr<Pool> pool;
  QW embed, lm_head;
  std::vector<float> final_norm;
  std::vector<Layer> layers;
  std::vector<Seq> seqs;
  size_t H = 0, kd = 0, vd = 0, cd = 0, n_gdn = 0, n_attn = 0;
  double sec_deltanet = 0, sec_attention = 0, sec_moe = 0;  // last step, per mixer / MoE

  std::vector<float> normal_vec(uint64_t seed, const std::string& name, size_t n) {
    std::vector<float> v(n);
    const uint64_t key = synth::tensor_key(seed, synth::tensor_id(name));
    for (size_t i = 0; i < n; ++i) v[i] = synth::normal(key, i, 0.02f);
    return v;
  }

  void build(uint64_t seed) {
    Pool& P = *pool;
    H = c.hidden;
    kd = size_t(c.key_heads) * c.key_dim;
    vd = size_t(c.value_heads) * c.value_dim;
    cd = 2 * kd + vd;
    const size_t E = c.experts, I = c.intermediate, S = c.shared;
    embed.generate(seed, "language_model.model.embed_tokens", c.vocab, H, P);
    lm_head.generate(seed, "language_model.lm_head", c.vocab, H, P);
    final_norm.assign(H, 1.f);
    layers.resize(c.layers);
    for (int i = 0; i < c.layers; ++i) {
      Layer& L = layers[i];
      const std::string p = "language_model.model.layers." + std::to_string(i);
      L.in_norm.assign(H, 1.f);
      L.post_norm.assign(H, 1.f);
      L.attention = (i + 1) % c.interval == 0;
      if (L.attention) {
        ++n_attn;
        const size_t d = c.head_dim;
        L.qp.generate(seed, p + ".self_attn.q_proj", size_t(c.q_heads) * 2 * d, H, P);
        L.kp.generate(seed, p + ".self_attn.k_proj", size_t(c.kv_heads) * d, H, P);
        L.vp.generate(seed, p + ".self_attn.v_proj", size_t(c.kv_heads) * d, H, P);
        L.op.generate(seed, p + ".self_attn.o_proj", H, size_t(c.q_heads) * d, P);
        L.q_norm.assign(d, 1.f);
        L.k_norm.assign(d, 1.f);
      } else {
        ++n_gdn;
        const std::string g = p + ".linear_attn";
        L.qkv.generate(seed, g + ".in_proj_qkv", cd, H, P);
        L.z.generate(seed, g + ".in_proj_z", vd, H, P);
        L.a.generate(seed, g + ".in_proj_a", c.value_heads, H, P);
        L.b.generate(seed, g + ".in_proj_b", c.value_heads, H, P);
        L.out.generate(seed, g + ".out_proj", H, vd, P);
        L.conv_w = normal_vec(seed, g + ".conv1d.weight", cd * size_t(c.conv));
        L.a_log = normal_vec(seed, g + ".A_log", c.value_heads);
        L.dt_bias = normal_vec(seed, g + ".dt_bias", c.value_heads);
        L.gnorm.assign(c.value_dim, 1.f);
      }
      L.router.generate(seed, p + ".mlp.gate", E, H, P);
      L.sh_gate_row.generate(seed, p + ".mlp.shared_expert_gate", 1, H, P);
      L.gate.generate(seed, p + ".mlp.switch_mlp.gate_proj", E * I, H, P);
      L.up.generate(seed, p + ".mlp.switch_mlp.up_proj", E * I, H, P);
      L.down.generate(seed, p + ".mlp.switch_mlp.down_proj", E * H, I, P);
      L.sh_gate.generate(seed, p + ".mlp.shared_expert.gate_proj", S, H, P);
      L.sh_up.generate(seed, p + ".mlp.shared_expert.up_proj", S, H, P);
      L.sh_down.generate(seed, p + ".mlp.shared_expert.down_proj", H, S, P);
    }
  }

  size_t state_count() const {
    return n_gdn * (size_t(c.conv - 1) * cd + size_t(c.value_heads) * c.value_dim * c.key_dim) +
           n_attn * 2 * size_t(c.kv_heads) * size_t(c.context) * c.head_dim;
  }

  // ------------------------------------------------------------ layer math --
  void deltanet(Layer& L, int gi, const float* h, size_t T, float* y) {
    Pool& P = *pool;
    const size_t hv = c.value_heads, hk = c.key_heads, dk = c.key_dim, dv = c.value_dim, K = c.conv;
    const auto xs = group_sums(h, T, H);
    std::vector<float> qkv(T * cd), z(T * vd), a(T * hv), b(T * hv);
    project(L.qkv, 0, cd, h, xs.data(), nullptr, T, qkv.data(), cd, P);
    project(L.z, 0, vd, h, xs.data(), nullptr, T, z.data(), vd, P);
    project(L.a, 0, hv, h, xs.data(), nullptr, T, a.data(), hv, P);
    project(L.b, 0, hv, h, xs.data(), nullptr, T, b.data(), hv, P);
    std::vector<float> act(T * cd), o(T * vd), gated(T * vd);
    // causal conv over [history; this token] + SiLU, history shifted (one token per sequence)
    P.run(T, [&](size_t t) {
      float* hist = seqs[t].conv[gi].data();
      for (size_t ch = 0; ch < cd; ++ch) {
        float v = 0;
        for (size_t tap = 0; tap + 1 < K; ++tap) v += hist[tap * cd + ch] * L.conv_w[ch * K + tap];
        v += qkv[t * cd + ch] * L.conv_w[ch * K + K - 1];
        act[t * cd + ch] = silu(v);
      }
      for (size_t tap = 0; tap + 2 < K; ++tap) std::memcpy(hist + tap * cd, hist + (tap + 1) * cd, cd * 4);
      std::memcpy(hist + (K - 2) * cd, &qkv[t * cd], cd * 4);
    });
    // gated delta rule per (sequence, value head)
    P.run(T * hv, [&](size_t it) {
      const size_t t = it / hv, head = it % hv, kh = head / (hv / hk);
      std::vector<float> qh(dk), khv(dk);
      float qs = 0, ks = 0;
      for (size_t j = 0; j < dk; ++j) {
        qh[j] = act[t * cd + kh * dk + j];
        khv[j] = act[t * cd + kd + kh * dk + j];
        qs += qh[j] * qh[j];
        ks += khv[j] * khv[j];
      }
      const float qi = 1.f / (std::sqrt(qs / dk + 1e-6f) * dk), ki = 1.f / (std::sqrt(ks / dk + 1e-6f) * std::sqrt(float(dk)));
      for (size_t j = 0; j < dk; ++j) {
        qh[j] *= qi;
        khv[j] *= ki;
      }
      const float logit = a[t * hv + head] + L.dt_bias[head];
      const float sp = std::max(logit, 0.f) + std::log1p(std::exp(-std::abs(logit)));
      const float decay = std::exp(-std::exp(L.a_log[head]) * sp), beta = sigm(b[t * hv + head]);
      float* S = seqs[t].S[gi].data() + head * dv * dk;
      for (size_t r = 0; r < dv; ++r) {
        float* row = S + r * dk;
        float mem = 0;
        for (size_t j = 0; j < dk; ++j) {
          row[j] *= decay;
          mem += row[j] * khv[j];
        }
        const float delta = (act[t * cd + 2 * kd + head * dv + r] - mem) * beta;
        float rd = 0;
        for (size_t j = 0; j < dk; ++j) {
          row[j] += delta * khv[j];
          rd += row[j] * qh[j];
        }
        o[t * vd + head * dv + r] = rd;
      }
      rms(&o[t * vd + head * dv], &gated[t * vd + head * dv], dv, L.gnorm.data(), c.epsilon);
      for (size_t r = 0; r < dv; ++r) gated[t * vd + head * dv + r] *= silu(z[t * vd + head * dv + r]);
    });
    const auto gs = group_sums(gated.data(), T, vd);
    project(L.out, 0, H, gated.data(), gs.data(), nullptr, T, y, H, P);
  }

  void attention(Layer& L, int ai, const float* h, size_t T, float* y) {
    Pool& P = *pool;
    const size_t Hq = c.q_heads, Hk = c.kv_heads, d = c.head_dim, grp = Hq / Hk;
    const auto xs = group_sums(h, T, H);
    std::vector<float> qg(T * Hq * 2 * d), k(T * Hk * d), v(T * Hk * d);
    project(L.qp, 0, Hq * 2 * d, h, xs.data(), nullptr, T, qg.data(), Hq * 2 * d, P);
    project(L.kp, 0, Hk * d, h, xs.data(), nullptr, T, k.data(), Hk * d, P);
    project(L.vp, 0, Hk * d, h, xs.data(), nullptr, T, v.data(), Hk * d, P);
    std::vector<float> q(T * Hq * d), o(T * Hq * d);
    for (size_t t = 0; t < T; ++t)
      if (seqs[t].pos >= seqs[t].cap) throw std::runtime_error("fp32 step: KV capacity");
    P.run(T, [&](size_t t) {
      Seq& s = seqs[t];
      std::vector<float> tmp(d);
      for (size_t hh = 0; hh < Hq; ++hh) {
        rms(&qg[(t * Hq + hh) * 2 * d], &q[(t * Hq + hh) * d], d, L.q_norm.data(), c.epsilon);
        rope(&q[(t * Hq + hh) * d], c.rope_dims, double(s.pos), c.theta);
      }
      for (size_t g = 0; g < Hk; ++g) {
        rms(&k[(t * Hk + g) * d], tmp.data(), d, L.k_norm.data(), c.epsilon);
        rope(tmp.data(), c.rope_dims, double(s.pos), c.theta);
        for (size_t i = 0; i < d; ++i) {
          s.K[ai][(g * s.cap + s.pos) * d + i] = to_bf16(tmp[i]);
          s.V[ai][(g * s.cap + s.pos) * d + i] = to_bf16(v[(t * Hk + g) * d + i]);
        }
      }
    });
    const float scale = 1.f / std::sqrt(float(d));
    // one item per (sequence, kv head): each cached row is widened once for
    // the `grp` query heads that share it (attention_reference.h:15 mapping)
    P.run(T * Hk, [&](size_t it) {
      const size_t t = it / Hk, g = it % Hk;
      const Seq& s = seqs[t];
      const size_t n = s.pos + 1;
      std::vector<float> sc(grp * n), row(d), acc(grp * d, 0.f), peak(grp, -INFINITY), tot(grp, 0.f);
      for (size_t j = 0; j < n; ++j) {
        const uint16_t* kk = &s.K[ai][(g * s.cap + j) * d];
        for (size_t i = 0; i < d; ++i) row[i] = from_bf16(kk[i]);
        for (size_t h = 0; h < grp; ++h) {
          const float* qv = &q[(t * Hq + g * grp + h) * d];
          float dot = 0;
          for (size_t i = 0; i < d; ++i) dot += qv[i] * row[i];
          sc[h * n + j] = dot * scale;
          peak[h] = std::max(peak[h], sc[h * n + j]);
        }
      }
      for (size_t h = 0; h < grp; ++h)
        for (size_t j = 0; j < n; ++j) {
          sc[h * n + j] = std::exp(sc[h * n + j] - peak[h]);
          tot[h] += sc[h * n + j];
        }
      for (size_t j = 0; j < n; ++j) {
        const uint16_t* vv = &s.V[ai][(g * s.cap + j) * d];
        for (size_t i = 0; i < d; ++i) row[i] = from_bf16(vv[i]);
        for (size_t h = 0; h < grp; ++h) {
          const float p = sc[h * n + j] / tot[h];
          float* a = &acc[h * d];
          for (size_t i = 0; i < d; ++i) a[i] += p * row[i];
        }
      }
      for (size_t h = 0; h < grp; ++h) {
        const size_t hh = g * grp + h;
        const float* gate = &qg[(t * Hq + hh) * 2 * d + d];
        for (size_t i = 0; i < d; ++i) o[(t * Hq + hh) * d + i] = acc[h * d + i] * sigm(gate[i]);
      }
    });
    const auto os = group_sums(o.data(), T, Hq * d);
    project(L.op, 0, H, o.data(), os.data(), nullptr, T, y, H, P);
  }

  void moe(Layer& L, const float* h, size_t T, float* y) {
    Pool& P = *pool;
    const size_t E = c.experts, K = c.top, I = c.intermediate, S = c.shared;
    const auto xs = group_sums(h, T, H);
    std::vector<float> logits(T * E), sg(T);
    project(L.router, 0, E, h, xs.data(), nullptr, T, logits.data(), E, P);
    project(L.sh_gate_row, 0, 1, h, xs.data(), nullptr, T, sg.data(), 1, P);
    // top-k by (logit desc, expert id asc), weights renormalised over the selection
    std::vector<int32_t> sel(T * K);
    std::vector<float> wsel(T * K);
    for (size_t t = 0; t < T; ++t) {
      const float* lt = &logits[t * E];
      std::vector<int32_t> order(E);
      for (size_t e = 0; e < E; ++e) order[e] = int32_t(e);
      std::partial_sort(order.begin(), order.begin() + K, order.end(), [&](int32_t x, int32_t z) {
        const uint32_t kx = total_key(lt[x]), kz = total_key(lt[z]);
        return kx != kz ? kx > kz : x < z;
      });
      const float peak = lt[order[0]];
      float den = 0;
      for (size_t j = 0; j < K; ++j) den += std::exp(lt[order[j]] - peak);
      for (size_t j = 0; j < K; ++j) {
        sel[t * K + j] = order[j];
        wsel[t * K + j] = std::exp(lt[order[j]] - peak) / den;
      }
    }
    // tokens per expert (stable by token)
    std::vector<std::vector<int32_t>> by_expert(E);
    for (size_t t = 0; t < T; ++t)
      for (size_t j = 0; j < K; ++j) by_expert[sel[t * K + j]].push_back(int32_t(t * K + j));
    std::vector<int32_t> hit;
    for (size_t e = 0; e < E; ++e)
      if (!by_expert[e].empty()) hit.push_back(int32_t(e));
    // gate/up per (expert, 64-row block) -> act[slot][I]; down per (expert, 256-row block)
    std::vector<float> act(T * K * I), ys(T * K * H);
    const size_t gu_blocks = (I + 63) / 64, dn_blocks = (H + 255) / 256;
    P.run(hit.size() * gu_blocks, [&](size_t it) {
      const size_t e = size_t(hit[it / gu_blocks]), blk = it % gu_blocks;
      const auto& slots = by_expert[e];
      const size_t n = slots.size(), j0 = blk * 64, nj = std::min<size_t>(64, I - j0);
      std::vector<int32_t> toks(n);
      for (size_t i = 0; i < n; ++i) toks[i] = slots[i] / int32_t(K);
      std::vector<float> g(n * nj), u(n * nj);
      Pool serial(1);
      project(L.gate, e * I + j0, nj, h, xs.data(), toks.data(), n, g.data(), nj, serial, nj);
      project(L.up, e * I + j0, nj, h, xs.data(), toks.data(), n, u.data(), nj, serial, nj);
      for (size_t i = 0; i < n; ++i)
        for (size_t j = 0; j < nj; ++j) act[size_t(slots[i]) * I + j0 + j] = silu(g[i * nj + j]) * u[i * nj + j];
    });
    const auto as = group_sums(act.data(), T * K, I);
    P.run(hit.size() * dn_blocks, [&](size_t it) {
      const size_t e = size_t(hit[it / dn_blocks]), blk = it % dn_blocks;
      const auto& slots = by_expert[e];
      const size_t n = slots.size(), r0 = blk * 256, nr = std::min<size_t>(256, H - r0);
      std::vector<float> out(n * nr);
      Pool serial(1);
      project(L.down, e * H + r0, nr, act.data(), as.data(), slots.data(), n, out.data(), nr, serial, nr);
      for (size_t i = 0; i < n; ++i) std::memcpy(&ys[size_t(slots[i]) * H + r0], &out[i * nr], nr * 4);
    });
    // shared expert over every token
    std::vector<float> shg(T * S), shu(T * S), sha(T * S), sho(T * H);
    project(L.sh_gate, 0, S, h, xs.data(), nullptr, T, shg.data(), S, P);
    project(L.sh_up, 0, S, h, xs.data(), nullptr, T, shu.data(), S, P);
    for (size_t i = 0; i < T * S; ++i) sha[i] = silu(shg[i]) * shu[i];
    const auto ss = group_sums(sha.data(), T, S);
    project(L.sh_down, 0, H, sha.data(), ss.data(), nullptr, T, sho.data(), H, P);
    for (size_t t = 0; t < T; ++t) {
      const float gate = sigm(sg[t]);
      for (size_t i = 0; i < H; ++i) {
        float v = gate * sho[t * H + i];
        for (size_t j = 0; j < K; ++j) v += wsel[t * K + j] * ys[(t * K + j) * H + i];
        y[t * H + i] = v;
      }
    }
  }

  // One decode token per sequence. Returns seconds spent in the decoder
  // layers and in the final norm + vocabulary projection + argmax.
  void step(const uint32_t* tokens, uint32_t* sampled, float* logits_out, double* t_layers, double* t_head) {
    const size_t T = seqs.size();
    if (!T) throw std::invalid_argument("fp32 step: no sequences");
    auto now = [] { return std::chrono::steady_clock::now(); };
    const auto t0 = now();
    std::vector<float> x(T * H), hbuf(T * H), r(T * H);
    for (size_t t = 0; t < T; ++t) {
      if (tokens[t] >= uint32_t(c.vocab)) throw std::invalid_argument("token outside vocabulary");
      const size_t row = tokens[t], G = H / 64;
      for (size_t g = 0; g < G; ++g) {
        const uint32_t* words = &embed.packed[row * (H / 8) + g * 8];
        for (int i = 0; i < 64; ++i)
          x[t * H + g * 64 + i] = embed.scale[row * G + g] * float((words[i / 8] >> (4 * (i % 8))) & 15u) +
                                  embed.bias[row * G + g];
      }
    }
    int gi = 0, ai = 0;
    sec_deltanet = sec_attention = sec_moe = 0;
    auto secs = [](auto a, auto b) { return std::chrono::duration<double>(b - a).count(); };
    for (auto& L : layers) {
      for (size_t t = 0; t < T; ++t) rms(&x[t * H], &hbuf[t * H], H, L.in_norm.data(), c.epsilon);
      const auto a = now();
      if (L.attention)
        attention(L, ai++, hbuf.data(), T, r.data());
      else
        deltanet(L, gi++, hbuf.data(), T, r.data());
      const auto b = now();
      (L.attention ? sec_attention : sec_deltanet) += secs(a, b);
      for (size_t i = 0; i < T * H; ++i) x[i] += r[i];
      for (size_t t = 0; t < T; ++t) rms(&x[t * H], &hbuf[t * H], H, L.post_norm.data(), c.epsilon);
      moe(L, hbuf.data(), T, r.data());
      sec_moe += secs(b, now());
      for (size_t i = 0; i < T * H; ++i) x[i] += r[i];
    }
    const auto t1 = now();
    for (size_t t = 0; t < T; ++t) rms(&x[t * H], &hbuf[t * H], H, final_norm.data(), c.epsilon);
    const auto hs = group_sums(hbuf.data(), T, H);
    std::vector<float> lg(T * size_t(c.vocab));
    project(lm_head, 0, c.vocab, hbuf.data(), hs.data(), nullptr, T, lg.data(), c.vocab, *pool, 64);
    for (size_t t = 0; t < T; ++t) {
      const float* lt = &lg[t * c.vocab];
      size_t best = 0;
      for (size_t v = 1; v < size_t(c.vocab); ++v)
        if (total_key(lt[v]) > total_key(lt[best])) best = v;
      if (sampled) sampled[t] = uint32_t(best);
      seqs[t].pos += 1;
    }
    if (logits_out) std::memcpy(logits_out, lg.data(), lg.size() * 4);
    const auto t2 = now();
    if (t_layers) *t_layers = std::chrono::duration<double>(t1 - t0).count();
    if (t_head) *t_head = std::chrono::duration<double>(t2 - t1).count();
  }
};

}  // namespace

extern "C" {

const char* f32_last_error() { return f_error.c_str(); }

// Builds the model (same synthetic weights as rs_qwen_weights_synthetic) and
// a worker pool of `threads` (0: every hardware thread).
void* f32_create(const rs_qwen_config* config, uint64_t seed, int threads) {
  Model* out = nullptr;
  guard([&] {
    if (!config || config->interval <= 0 || config->layers % config->interval || config->hidden % 64)
      throw std::invalid_argument("fp32 step: model geometry");
    if (!__builtin_cpu_supports("avx2") || !__builtin_cpu_supports("fma"))
      throw std::runtime_error("fp32 step: this build needs a host CPU with AVX2 and FMA");
    auto m = std::make_unique<Model>();
    m->c = *config;
    const unsigned hw = std::thread::hardware_concurrency();
    m->pool = std::make_unique<Pool>(threads > 0 ? threads : int(hw ? hw : 1));
    m->build(seed);
    out = m.release();
  });
  return out;
}
void f32_destroy(void* m) { delete static_cast<Model*>(m); }
int f32_threads(void* m) { return static_cast<Model*>(m)->pool->size(); }

// Sets the batch: n sequences at positions[s], each with room for `extra`
// more tokens. states: n reference-layout states (rs_qwen_state_count floats
// each, layout of native/qwen_model.inc:268-271), or null for seeded
// synthetic prefix state (K/V bf16 N(0,1), conv N(0,1), recurrent N(0,0.02)).
int f32_set_batch(void* model, size_t n, const uint32_t* positions, const float* states, uint64_t seed,
                  size_t extra) {
  return guard([&] {
    Model& m = *static_cast<Model*>(model);
    const rs_qwen_config& c = m.c;
    m.seqs.assign(n, Seq());
    const size_t convn = size_t(c.conv - 1) * m.cd, sn = size_t(c.value_heads) * c.value_dim * c.key_dim;
    const size_t kvn = size_t(c.kv_heads) * c.head_dim, per = kvn * size_t(c.context);
    const size_t count = m.state_count();
    for (size_t s = 0; s < n; ++s)
      if (positions[s] >= size_t(c.context) || (states && positions[s] + extra > size_t(c.context)))
        throw std::invalid_argument("fp32 step: position beyond the context");
    m.pool->run(n, [&](size_t s) {
      Seq& q = m.seqs[s];
      q.pos = positions[s];
      q.cap = states ? size_t(c.context) : positions[s] + extra + 1;
      const float* src = states ? states + s * count : nullptr;
      uint64_t h = synth::mix64(seed ^ (s * 0x9E3779B97F4A7C15ull));
      auto rnd = [&](float sd) {
        h = synth::mix64(h);
        const int32_t v = int32_t(h & 0xFFFF) + int32_t((h >> 16) & 0xFFFF) + int32_t((h >> 32) & 0xFFFF) + int32_t(h >> 48);
        return float(v - 131070) * (sd / 37837.2265f);
      };
      size_t off = 0;
      for (const auto& L : m.layers) {
        if (L.attention) {
          q.K.emplace_back(kvn * q.cap, uint16_t(0));
          q.V.emplace_back(kvn * q.cap, uint16_t(0));
          auto& K = q.K.back();
          auto& V = q.V.back();
          for (size_t g = 0; g < size_t(c.kv_heads); ++g)
            for (size_t p = 0; p < q.pos; ++p)
              for (size_t i = 0; i < size_t(c.head_dim); ++i) {
                const size_t at = (g * q.cap + p) * c.head_dim + i;
                const size_t ref = (g * size_t(c.context) + p) * c.head_dim + i;
                K[at] = to_bf16(src ? src[off + ref] : rnd(1.f));
                V[at] = to_bf16(src ? src[off + per + ref] : rnd(1.f));
              }
          off += 2 * per;
        } else {
          q.conv.emplace_back(convn);
          q.S.emplace_back(sn);
          for (size_t i = 0; i < convn; ++i) q.conv.back()[i] = src ? src[off + i] : rnd(1.f);
          for (size_t i = 0; i < sn; ++i) q.S.back()[i] = src ? src[off + convn + i] : rnd(0.02f);
          off += convn + sn;
        }
      }
    });
  });
}

int f32_step(void* model, const uint32_t* tokens, uint32_t* sampled, float* logits, double* t_layers,
             double* t_head) {
  return guard([&] { static_cast<Model*>(model)->step(tokens, sampled, logits, t_layers, t_head); });
}

// Seconds of the last step spent in DeltaNet mixers, attention mixers and MoE blocks.
void f32_stage_seconds(void* model, double* out3) {
  const Model& m = *static_cast<Model*>(model);
  out3[0] = m.sec_deltanet;
  out3[1] = m.sec_attention;
  out3[2] = m.sec_moe;
}

}  // extern "C"
