// Decode-step kernels for sm_100a: packing, embedding + norms, attention
// prep and split merge, MoE routing / sort / combine and greedy selection.
// The DeltaNet kernels live in gdn.cu, the paged attention kernel in
// attention.cu and the 4-bit GEMMs in qgemm_tc.cu (qgemm.cu: CUDA-core
// reference engine).
#include <atomic>
#include <cfloat>

#include "kernels.h"

namespace qwen {

namespace {

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}

__device__ __forceinline__ int block_sum_int(int v, int* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  int t = lane < nw ? red[lane] : 0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}

// ------------------------------------------------------------------ packing --
// One block per sequence: prefix sum of new-token counts, child block-table
// row (parent prefix pages + new pages), per-token (sequence, position) and
// KV slot, and the token index of each output row.
__global__ void pack_kernel(const SeqDesc* __restrict__ descs, int n_seq,
                            const int32_t* __restrict__ new_pages, int32_t* block_table,
                            int stride, Packed p) {
  pdl_trigger();
  pdl_wait(descs, new_pages);
  __shared__ int red[32];
  const int s = blockIdx.x;
  int local = 0;
  for (int i = threadIdx.x; i < s; i += blockDim.x) local += descs[i].count;
  const int off = block_sum_int(local, red);
  const SeqDesc d = descs[s];
  if (threadIdx.x == 0) {
    p.cu_seqlens[s + 1] = off + d.count;
    if (s == 0) p.cu_seqlens[0] = 0;
  }
  int32_t* child = block_table + size_t(d.child) * stride;
  const int32_t* parent = d.parent >= 0 ? block_table + size_t(d.parent) * stride : nullptr;
  if (parent != child) {
    for (int j = threadIdx.x; j < d.n_shared; j += blockDim.x) child[j] = parent[j];
  }
  __syncthreads();
  for (int j = threadIdx.x; j < d.n_new; j += blockDim.x) child[d.n_shared + j] = new_pages[d.new_off + j];
  __syncthreads();
  const int n_pages = d.n_shared + d.n_new;
  for (int i = threadIdx.x; i < d.count; i += blockDim.x) {
    const int t = off + i, pos = d.position + i;
    p.token_seq[t] = s;
    p.token_pos[t] = pos;
    const int pi = pos / kPageTokens;
    const int page = pi < n_pages ? child[pi] : 0;  // host guarantees pi < n_pages
    p.slot_mapping[t] = int64_t(page) * kPageTokens + pos % kPageTokens;
  }
  for (int i = threadIdx.x; i < d.n_out; i += blockDim.x)
    p.out_token[d.out_row0 + i] = off + d.count - d.n_out + i;
}

// Copy-on-write of a shared partial page: tokens [0, cow_len) of cow_src into
// the sequence's first new page, for every attention layer, K and V.
__global__ void cow_kernel(KvPool kv, const SeqDesc* __restrict__ descs,
                           const int32_t* __restrict__ new_pages) {
  pdl_trigger();
  pdl_wait(descs, new_pages);
  const SeqDesc d = descs[blockIdx.x];
  if (d.cow_src < 0 || d.n_new <= 0) return;
  const int layer = blockIdx.y;
  const __nv_bfloat16* src = kv.page(layer, d.cow_src);
  __nv_bfloat16* dst = kv.page(layer, new_pages[d.new_off]);
  const int per_tok = kv.D;
  for (int kvh = 0; kvh < 2 * kv.Hkv; ++kvh)
    for (int i = threadIdx.x; i < d.cow_len * per_tok; i += blockDim.x) {
      size_t o = size_t(kvh) * kPageTokens * kv.D + i;
      dst[o] = src[o];
    }
}

// ---------------------------------------------------------- embed + norms --
// x[t] = dequant(embed[token[t]]) (fp32 residual), hb[t] = fp16(rms(x[t]) * w).
__global__ void embed_norm_kernel(QMat embed, const uint32_t* __restrict__ tokens,
                                  const float* __restrict__ norm_w, float eps, float* x,
                                  gemm_in_t* hb) {
  pdl_trigger();
  pdl_wait(tokens, norm_w);
  __shared__ float red[32];
  const int t = blockIdx.x, H = embed.k;
  const uint32_t tok = tokens[t];
  float* xr = x + size_t(t) * H;
  float ss = 0.f;
  for (int w = threadIdx.x; w < H / 8; w += blockDim.x) {
    const int c0 = w * 8;
    const uint8_t* tile = embed.tile(int(tok / kTileRows), c0 / kTileK);
    const int r = tok % kTileRows;
    const uint32_t word = *reinterpret_cast<const uint32_t*>(tile + r * 32 + (c0 % kTileK) / 2);
    const float sc = half_bits_to_float(reinterpret_cast<const uint16_t*>(tile + kTilePackedBytes)[r]) * (1.f / kTileScale);
    const float bi = half_bits_to_float(
        reinterpret_cast<const uint16_t*>(tile + kTilePackedBytes + kTileRows * 2)[r]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = fmaf(sc, float(nibble(word, j)), bi);
      xr[c0 + j] = v;
      ss += v * v;
    }
  }
  const float tot = block_sum(ss, red);
  const float inv = rsqrtf(tot / H + eps);
  for (int c = threadIdx.x; c < H; c += blockDim.x)
    hb[size_t(t) * H + c] = to_gemm_in(xr[c] * inv * norm_w[c]);
}

// Row r: t = out_token ? out_token[r] : r. x[t] += sum of split partials
// (only when partial != null); then hb[r] = fp16(rms(x[t]) * w) and optionally
// hidden[r] = fp32 normalized row.
__global__ void residual_norm_kernel(float* __restrict__ x, const float* __restrict__ partial, int splits,
                                     size_t split_stride, int H, const float* __restrict__ norm_w,
                                     float eps, gemm_in_t* __restrict__ hb,
                                     const int32_t* __restrict__ out_token, float* __restrict__ hidden) {
  pdl_trigger();
  pdl_wait(x, partial, norm_w, hb, out_token, hidden);
  // Thread i owns column pairs i, i + blockDim, ... (H <= 2 * kPer * blockDim);
  // every load of the row is issued before the first add.
  constexpr int kPer = 4, kSplits = 8;
  __shared__ float red[32];
  const int r = blockIdx.x;
  const int t = out_token ? out_token[r] : r;
  const int H2 = H >> 1;
  float2* xr = reinterpret_cast<float2*>(x + size_t(t) * H);
  float2 v[kPer];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    v[k] = c < H2 ? xr[c] : make_float2(0.f, 0.f);
  }
  if (partial) {
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int c = threadIdx.x + k * blockDim.x;
      if (c >= H2) continue;
      float2 p[kSplits];
#pragma unroll
      for (int sp = 0; sp < kSplits; ++sp)
        if (sp < splits) p[sp] = reinterpret_cast<const float2*>(partial + sp * split_stride + size_t(t) * H)[c];
#pragma unroll
      for (int sp = 0; sp < kSplits; ++sp)
        if (sp < splits) { v[k].x += p[sp].x; v[k].y += p[sp].y; }
      xr[c] = v[k];
    }
  }
#pragma unroll
  for (int k = 0; k < kPer; ++k) ss += v[k].x * v[k].x + v[k].y * v[k].y;
  const float tot = block_sum(ss, red);
  if (!norm_w) return;
  const float inv = rsqrtf(tot / H + eps);
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (c < H2) {
      const float2 w = reinterpret_cast<const float2*>(norm_w)[c];
      const float y0 = v[k].x * inv * w.x, y1 = v[k].y * inv * w.y;
      reinterpret_cast<__half2*>(hb + size_t(r) * H)[c] = to_gemm_in2(y0, y1);
      if (hidden) reinterpret_cast<float2*>(hidden + size_t(r) * H)[c] = make_float2(y0, y1);
    }
  }
}


// ----------------------------------------------------------------- attention --
// Per token: q/k RMSNorm (q_norm/k_norm), partial rotate-half RoPE on the
// first rope dims (angle in double precision), KV append into the paged cache.
template <int E>
__device__ __forceinline__ void load_lane(const float* p, float (&out)[E]) {
  if constexpr (E % 4 == 0) {
#pragma unroll
    for (int e = 0; e < E; e += 4) {
      const float4 v = *reinterpret_cast<const float4*>(p + e);
      out[e] = v.x; out[e + 1] = v.y; out[e + 2] = v.z; out[e + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      const float2 v = *reinterpret_cast<const float2*>(p + e);
      out[e] = v.x; out[e + 1] = v.y;
    }
  }
}
template <int E>
__device__ __forceinline__ void store_lane(float* p, const float (&in)[E]) {
  if constexpr (E % 4 == 0) {
#pragma unroll
    for (int e = 0; e < E; e += 4) *reinterpret_cast<float4*>(p + e) = make_float4(in[e], in[e + 1], in[e + 2], in[e + 3]);
  } else {
#pragma unroll
    for (int e = 0; e < E; e += 2) *reinterpret_cast<float2*>(p + e) = make_float2(in[e], in[e + 1]);
  }
}
// Sum of the split-K partials of E contiguous floats, in split order.
template <int E>
__device__ __forceinline__ void load_splits(const float* p, int splits, size_t split_stride, float (&out)[E]) {
  load_lane<E>(p, out);
#pragma unroll
  for (int sp = 1; sp < 8; ++sp) {
    if (sp < splits) {
      float part[E];
      load_lane<E>(p + sp * split_stride, part);
#pragma unroll
      for (int e = 0; e < E; ++e) out[e] += part[e];
    }
  }
}

// One warp per head vector (Hq query+gate heads, Hkv keys, Hkv values) of
// token blockIdx.x; lane l owns D/32 contiguous dims. The RoPE cos/sin of the
// token's position are computed once per CTA (double precision).
template <int D>
__global__ void __launch_bounds__(1024) attn_prep_kernel(const float* __restrict__ proj, int ld, int splits,
                                                         size_t split_stride, int Hq, int Hkv, int rope,
                                                         double theta, float eps, const float* __restrict__ qn,
                                                         const float* __restrict__ kn,
                                                         const int32_t* __restrict__ token_pos,
                                                         const int64_t* __restrict__ slots, KvPool kv, int layer,
                                                         float* q, float* gate) {
  pdl_trigger();
  pdl_wait(proj, qn, kn, token_pos, slots);
  constexpr int E = D / 32;
  __shared__ float sm[32][D];
  __shared__ double rot[2][D / 2];
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  const int half = rope / 2;
  {
    const double pos = token_pos[t];
    for (int j = threadIdx.x; j < half; j += blockDim.x) {
      double sn, cs;
      sincos(pos * pow(theta, -2.0 * j / rope), &sn, &cs);
      rot[0][j] = cs;
      rot[1][j] = sn;
    }
  }
  __syncthreads();
  float* buf = sm[warp];
  const float* pr = proj + size_t(t) * ld;
  const int64_t slot = slots[t];
  const int page = int(slot / kPageTokens), off = int(slot % kPageTokens);
  for (int v = warp; v < Hq + 2 * Hkv; v += nw) {
    const float* src;
    const float* w = nullptr;
    if (v < Hq) { src = pr + v * 2 * D; w = qn; }
    else if (v < Hq + Hkv) { src = pr + Hq * 2 * D + (v - Hq) * D; w = kn; }
    else src = pr + Hq * 2 * D + Hkv * D + (v - Hq - Hkv) * D;
    float val[E];
    load_splits<E>(src + lane * E, splits, split_stride, val);
    if (w) {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) ss += val[e] * val[e];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / D + eps);
      float wv[E];
      load_lane<E>(w + lane * E, wv);
#pragma unroll
      for (int e = 0; e < E; ++e) val[e] = val[e] * inv * wv[e];
      if (half > 0) {
        store_lane<E>(buf + lane * E, val);
        __syncwarp();
        for (int j = lane; j < half; j += 32) {
          const double c = rot[0][j], sn = rot[1][j];
          const float a = buf[j], b = buf[j + half];
          buf[j] = float(a * c - b * sn);
          buf[j + half] = float(a * sn + b * c);
        }
        __syncwarp();
        load_lane<E>(buf + lane * E, val);
        __syncwarp();
      }
    }
    if (v < Hq) {
      store_lane<E>(q + (size_t(t) * Hq + v) * D + lane * E, val);
      float gv[E];
      load_splits<E>(src + D + lane * E, splits, split_stride, gv);
      store_lane<E>(gate + (size_t(t) * Hq + v) * D + lane * E, gv);
    } else {
      const int g = v < Hq + Hkv ? v - Hq : v - Hq - Hkv;
      const int kvsel = v < Hq + Hkv ? 0 : 1;
      __nv_bfloat16* dst =
          kv.page(layer, page) + (size_t(kvsel) * Hkv + g) * kPageTokens * D + size_t(off) * D + lane * E;
#pragma unroll
      for (int e = 0; e < E; e += 2)
        *reinterpret_cast<__nv_bfloat162*>(dst + e) = __floats2bfloat162_rn(val[e], val[e + 1]);
    }
  }
}

// Merge split partials, apply the output gate sigmoid(gate), write fp16 (the o_proj input).
// The split weights exp(m_s - M) / sum_s l_s exp(m_s - M) are computed once
// per (token, head) into shared memory (dynamic: max_splits floats).
// tokens: the step's tokens that ran the split decode kernel (null: all of them).
__global__ void attention_merge_kernel(const float* __restrict__ ws, const float* __restrict__ gate,
                                       const int32_t* __restrict__ token_pos, const int32_t* __restrict__ tokens,
                                       int Hq, int D, int spl, int max_splits, gemm_in_t* out) {
  pdl_trigger();
  pdl_wait(ws, gate, token_pos, tokens);
  extern __shared__ float wsplit[];
  __shared__ float red[32];
  __shared__ float s_max, s_den;
  const int t = tokens ? tokens[blockIdx.x] : blockIdx.x, h = blockIdx.y;
  const int n = (token_pos[t] + 1 + spl - 1) / spl;
  const float* base = ws + (size_t(blockIdx.x) * Hq + h) * max_splits * (D + 2);
  float m = -FLT_MAX;
  for (int s = threadIdx.x; s < n; s += blockDim.x) m = fmaxf(m, base[s * (D + 2)]);
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = -FLT_MAX;
    for (int w = 0; w < int(blockDim.x >> 5); ++w) M = fmaxf(M, red[w]);
    s_max = M;
  }
  __syncthreads();
  const float M = s_max;
  float den = 0.f;
  for (int s = threadIdx.x; s < n; s += blockDim.x) {
    const float e = __expf(base[s * (D + 2)] - M);
    wsplit[s] = e;
    den += base[s * (D + 2) + 1] * e;
  }
  den = warp_sum(den);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = den;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < int(blockDim.x >> 5); ++w) tot += red[w];
    s_den = tot;
  }
  __syncthreads();
  const float inv = 1.f / s_den;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float num = 0.f;
    for (int s = 0; s < n; ++s) num += base[s * (D + 2) + 2 + i] * wsplit[s];
    const float y = num * inv * sigmoidf_(gate[(size_t(t) * Hq + h) * D + i]);
    out[size_t(t) * Hq * D + h * D + i] = to_gemm_in(y);
  }
}

// ------------------------------------------------------------------- routing --
// Top-k over the router logits by (logit desc, expert id asc) on the fp32
// total order; weights renormalised over the selection
// (native/qwen_model.inc:77-79: softmax then divide by the selected sum);
// slot `top` is the shared expert (id E) with weight sigmoid(shared gate).
// Both kernels below run the same rounds with the same arithmetic: the split-K
// partials summed in split order, one maximum of the packed (total-order key,
// ~id) per round, w_r = exp(l_r - l_0), then w_r / sum. The thread (lane) r
// keeps round r's id and weight in registers and writes them at the end.

// Decode of the total-order key back to the float.
__device__ __forceinline__ float from_total_key(uint32_t tk) {
  return __uint_as_float((tk & 0x80000000u) ? (tk ^ 0x80000000u) : ~tk);
}

// One CTA of 256 threads per token (thread i holds experts i, i + 256, ...;
// E <= 1024): used when the router GEMM split K, so each token's split
// partials (up to 8 x E values) are read by 256 threads at once.
__global__ void __launch_bounds__(256) route_block_kernel(const float* __restrict__ logits, int ld, int splits,
                                                          size_t split_stride, int E, int top, int32_t* ids,
                                                          float* weights, float* logits_out) {
  pdl_trigger();
  pdl_wait(logits);
  constexpr int kPer = 4, kSplits = 8;
  __shared__ uint64_t wbest[2][8];
  __shared__ float s_shared_logit;
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* lr = logits + size_t(t) * ld;
  // the shared expert's gate logit (column E): lane sp of warp 0 requests
  // split sp's partial together with the experts' logits
  const float sh_part = (threadIdx.x < kSplits && threadIdx.x < splits) ? lr[threadIdx.x * split_stride + E] : 0.f;
  float v[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int e = threadIdx.x + k * 256;
    float part[kSplits];
#pragma unroll
    for (int sp = 0; sp < kSplits; ++sp)  // independent loads, then the adds in split order
      part[sp] = (e < E && sp < splits) ? lr[sp * split_stride + e] : 0.f;
    float acc = part[0];
#pragma unroll
    for (int sp = 1; sp < kSplits; ++sp)
      if (sp < splits) acc += part[sp];
    v[k] = acc;
  }
  if (warp == 0) {
    float sl = __shfl_sync(0xffffffffu, sh_part, 0);
#pragma unroll
    for (int sp = 1; sp < kSplits; ++sp) {
      const float p = __shfl_sync(0xffffffffu, sh_part, sp);
      if (sp < splits) sl += p;
    }
    if (lane == 0) s_shared_logit = sl;
  }
  if (logits_out) {  // diagnostic capture of the summed router logits
    float* lo = logits_out + size_t(t) * (E + 1);
#pragma unroll
    for (int k = 0; k < kPer; ++k)
      if (threadIdx.x + k * 256 < E) lo[threadIdx.x + k * 256] = v[k];
  }
  uint32_t taken = 0;
  float top_val = 0.f, denom = 0.f, my_w = 0.f;
  int my_e = 0;
  for (int r = 0; r < top; ++r) {
    uint64_t best = 0;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int e = threadIdx.x + k * 256;
      if (e < E && !(taken >> k & 1u)) {
        const uint64_t key = (uint64_t(total_key(v[k])) << 32) | uint32_t(0xFFFFFFFFu - e);
        best = key > best ? key : best;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) wbest[r & 1][warp] = best;
    __syncthreads();
    best = wbest[r & 1][0];
#pragma unroll
    for (int w = 1; w < 8; ++w) best = wbest[r & 1][w] > best ? wbest[r & 1][w] : best;
    const int e = int(0xFFFFFFFFu - uint32_t(best & 0xFFFFFFFFu));
    if ((e & 255) == threadIdx.x) taken |= 1u << (e >> 8);
    const float sel_val = from_total_key(uint32_t(best >> 32));
    if (r == 0) top_val = sel_val;
    const float w = expf(sel_val - top_val);
    denom += w;
    if (threadIdx.x == r) { my_e = e; my_w = w; }
  }
  int32_t* out_ids = ids + size_t(t) * (top + 1);
  float* out_w = weights + size_t(t) * (top + 1);
  if (threadIdx.x < top) {
    out_ids[threadIdx.x] = my_e;
    out_w[threadIdx.x] = my_w / denom;
  } else if (threadIdx.x == top) {
    const float shared_logit = s_shared_logit;
    if (logits_out) logits_out[size_t(t) * (E + 1) + E] = shared_logit;
    out_ids[top] = E;
    out_w[top] = 1.f / (1.f + expf(-shared_logit));
  }
}

// One warp per token, 8 tokens per CTA, for unsplit router logits: lane l
// holds experts l, l + 32, ... (PL of them); each round is a lane-local
// maximum and five shuffles, with no block-wide barrier.
template <int PL>
__global__ void __launch_bounds__(256) route_warp_kernel(const float* __restrict__ logits, int ld, int E, int top,
                                                         int T, int32_t* ids, float* weights, float* logits_out) {
  pdl_trigger();
  pdl_wait(logits);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  const float* lr = logits + size_t(t) * ld;
  const float shared_logit = lr[E];
  float v[PL];
#pragma unroll
  for (int m = 0; m < PL; ++m) v[m] = lane + 32 * m < E ? lr[lane + 32 * m] : 0.f;
  if (logits_out) {  // diagnostic capture of the router logits
    float* lo = logits_out + size_t(t) * (E + 1);
#pragma unroll
    for (int m = 0; m < PL; ++m)
      if (lane + 32 * m < E) lo[lane + 32 * m] = v[m];
    if (lane == 0) lo[E] = shared_logit;
  }
  uint32_t taken = 0;
  float top_val = 0.f, denom = 0.f, my_w = 0.f;
  int my_e = 0;
  for (int r = 0; r < top; ++r) {
    uint64_t best = 0;
#pragma unroll
    for (int m = 0; m < PL; ++m) {
      const int e = lane + 32 * m;
      if (e < E && !(taken >> m & 1u)) {
        const uint64_t key = (uint64_t(total_key(v[m])) << 32) | uint32_t(0xFFFFFFFFu - e);
        best = key > best ? key : best;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    const int e = int(0xFFFFFFFFu - uint32_t(best & 0xFFFFFFFFu));
    if ((e & 31) == lane) taken |= 1u << (e >> 5);
    const float sel_val = from_total_key(uint32_t(best >> 32));
    if (r == 0) top_val = sel_val;
    const float w = expf(sel_val - top_val);
    denom += w;
    if (lane == r) { my_e = e; my_w = w; }
  }
  int32_t* out_ids = ids + size_t(t) * (top + 1);
  float* out_w = weights + size_t(t) * (top + 1);
  if (lane < top) {
    out_ids[lane] = my_e;
    out_w[lane] = my_w / denom;
  } else if (lane == top) {
    out_ids[top] = E;
    out_w[top] = 1.f / (1.f + expf(-shared_logit));
  }
}

// Stable counting sort of assignments by expert id (single CTA, 1024 threads):
// counts, exclusive offsets [n_experts + 1], perm (sorted -> flat) and inv
// (flat -> sorted). Ranks are stable by flat index: assignments are taken in
// rounds of 1024 in index order; inside a round a warp ranks equal keys with
// match_any, and a per-(warp, key) count table scanned over warps orders the
// warps.
__global__ void __launch_bounds__(1024) expert_sort_kernel(const int32_t* __restrict__ ids, int n,
                                                           int n_experts, int32_t* counts, int32_t* offsets,
                                                           int32_t* perm, int32_t* inv) {
  pdl_trigger();
  pdl_wait(ids);
  extern __shared__ int32_t smi[];
  int32_t* cnt = smi;                 // [n_experts]
  int32_t* cursor = cnt + n_experts;  // [n_experts]
  int32_t* tot = cursor + n_experts;  // [n_experts]
  uint16_t* table = reinterpret_cast<uint16_t*>(tot + n_experts);  // [32][n_experts]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < n_experts; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) atomicAdd(&cnt[ids[i]], 1);
  __syncthreads();
  if (warp == 0) {  // exclusive scan over experts (one warp, chunks of 32)
    int carry = 0;
    for (int base = 0; base < n_experts; base += 32) {
      const int e = base + lane;
      const int c = e < n_experts ? cnt[e] : 0;
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (e < n_experts) cursor[e] = carry + incl - c;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) offsets[n_experts] = carry;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < n_experts; e += blockDim.x) {
    offsets[e] = cursor[e];
    counts[e] = cnt[e];
  }
  const uint32_t lt = (1u << lane) - 1u;
  for (int base = 0; base < n; base += blockDim.x) {
    for (int k = threadIdx.x; k < 32 * n_experts; k += blockDim.x) table[k] = 0;
    __syncthreads();
    const int i = base + threadIdx.x;
    const int key = i < n ? ids[i] : -1;
    const uint32_t peers = __match_any_sync(0xffffffffu, key);
    const int rank = __popc(peers & lt);
    if (key >= 0 && rank == 0) table[warp * n_experts + key] = uint16_t(__popc(peers));
    __syncthreads();
    for (int e = threadIdx.x; e < n_experts; e += blockDim.x) {
      int acc = 0;
      for (int w = 0; w < 32; ++w) {
        const int c = table[w * n_experts + e];
        table[w * n_experts + e] = uint16_t(acc);
        acc += c;
      }
      tot[e] = acc;
    }
    __syncthreads();
    if (key >= 0) {
      const int pos = cursor[key] + table[warp * n_experts + key] + rank;
      perm[pos] = i;
      inv[i] = pos;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n_experts; e += blockDim.x) cursor[e] += tot[e];
    __syncthreads();
  }
}

// The same stable sort from one bit mask of tokens per expert (single CTA,
// 1024 threads; used when the masks fit in shared memory): a token picks an
// expert at most once, so an assignment's rank inside its expert, i.e. the
// number of assignments of that expert with a smaller flat index, is the
// number of earlier tokens that picked the expert: the popcount of the
// expert's mask below the token. Per expert the counts of every 8 mask words
// are prefix-summed, so a rank costs at most 8 popcounts. Same bytes as
// expert_sort_kernel (a stable sort has one result).
constexpr int kMaskWordsPerBlock = 8;

// Shared-memory state of the mask sort: per expert its token mask, the rank
// before each block of 8 mask words, and (after mask_sort_build) its offset.
struct MaskSort {
  uint32_t* mask;  // [n_exp][nw]
  int32_t* pre;    // [n_exp][nb]
  int32_t* off;    // [n_exp]
  int nw, nb;
};

// Builds the masks, block prefixes and expert offsets in shared memory (every
// CTA that runs it gets the same result); with `outputs`, writes counts and
// offsets. Ids outside [0, n_exp) raise kErrBounds and are left out.
__device__ __forceinline__ MaskSort mask_sort_build(const int32_t* ids, int T, int slots, int n_exp, uint32_t* smm,
                                                    int32_t* warp_tot, bool outputs, int32_t* counts,
                                                    int32_t* offsets, uint32_t* err) {
  MaskSort m;
  m.nw = (T + 31) >> 5;
  m.nb = (m.nw + kMaskWordsPerBlock - 1) / kMaskWordsPerBlock;
  const int nw = m.nw, nb = m.nb, A = T * slots;
  m.mask = smm;
  m.pre = reinterpret_cast<int32_t*>(m.mask + size_t(n_exp) * nw);
  m.off = m.pre + size_t(n_exp) * nb;
  for (int i = threadIdx.x; i < n_exp * nw; i += blockDim.x) m.mask[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < A; i += blockDim.x) {
    const int e = ids[i], t = i / slots;
    if (e >= 0 && e < n_exp) atomicOr(&m.mask[e * nw + (t >> 5)], 1u << (t & 31));
    else atomicOr(err, kErrBounds);
  }
  __syncthreads();
  // per expert: block prefixes and the count; then an exclusive scan over experts
  int cnt = 0;
  for (int e = threadIdx.x; e < n_exp; e += blockDim.x) {
    int run = 0;
    for (int b = 0; b < nb; ++b) {
      m.pre[e * nb + b] = run;
      const int w1 = min(nw, (b + 1) * kMaskWordsPerBlock);
      for (int w = b * kMaskWordsPerBlock; w < w1; ++w) run += __popc(m.mask[e * nw + w]);
    }
    m.off[e] = run;  // the count, until the scan below
  }
  __syncthreads();
  // exclusive scan of off[] (n_exp <= 1025): thread i owns experts [i * per, (i + 1) * per)
  const int per = (n_exp + blockDim.x - 1) / blockDim.x;
  const int e0 = threadIdx.x * per, e1 = min(n_exp, e0 + per);
  for (int e = e0; e < e1; ++e) cnt += m.off[e];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  int base = incl - cnt;
  for (int w = 0; w < warp; ++w) base += warp_tot[w];
  for (int e = e0; e < e1; ++e) {
    const int c = m.off[e];
    m.off[e] = base;
    if (outputs) {
      offsets[e] = base;
      counts[e] = c;
    }
    base += c;
  }
  if (outputs && threadIdx.x == blockDim.x - 1) offsets[n_exp] = base;
  __syncthreads();
  return m;
}

// Sorted position of assignment (token t, expert e): the expert's offset plus
// the number of earlier tokens that picked it.
__device__ __forceinline__ int mask_sort_pos(const MaskSort& m, int e, int t) {
  const uint32_t* w = m.mask + size_t(e) * m.nw;
  const int wt = t >> 5, b = wt / kMaskWordsPerBlock;
  int rank = m.pre[e * m.nb + b] + __popc(w[wt] & ((1u << (t & 31)) - 1u));
  for (int k = b * kMaskWordsPerBlock; k < wt; ++k) rank += __popc(w[k]);
  return m.off[e] + rank;
}

__global__ void __launch_bounds__(1024) expert_sort_mask_kernel(const int32_t* __restrict__ ids, int T, int slots,
                                                                int n_exp, int32_t* counts, int32_t* offsets,
                                                                int32_t* perm, int32_t* inv, uint32_t* err) {
  pdl_trigger();
  pdl_wait(ids);
  extern __shared__ uint32_t smm[];
  __shared__ int32_t warp_tot[32];
  const MaskSort m = mask_sort_build(ids, T, slots, n_exp, smm, warp_tot, true, counts, offsets, err);
  for (int i = threadIdx.x; i < T * slots; i += blockDim.x) {
    const int e = ids[i], t = i / slots;
    if (e < 0 || e >= n_exp) continue;
    const int pos = mask_sort_pos(m, e, t);
    perm[pos] = i;
    inv[i] = pos;
  }
}

// The mask sort fused with the gather of the MoE input rows: every CTA builds
// the (small) sort in its own shared memory; CTA 0 writes counts / offsets /
// perm / inv, and each CTA copies the rows of its slice of the assignments,
// dst[pos(i)] = src[i / slots] (16-byte copies, one warp per row). The same
// bytes as expert_sort_mask_kernel followed by gather_rows_kernel, one launch
// and one kernel-boundary wait fewer per MoE layer.
constexpr int kGatherVec = 8;  // 16-byte vectors in flight per lane
__global__ void __launch_bounds__(1024) expert_sort_gather_kernel(const int32_t* __restrict__ ids, int T, int slots,
                                                                  int n_exp, int32_t* counts, int32_t* offsets,
                                                                  int32_t* perm, int32_t* inv, uint32_t* err,
                                                                  const gemm_in_t* __restrict__ src, int ld, int H,
                                                                  gemm_in_t* __restrict__ dst) {
  pdl_trigger();
  pdl_wait(ids, src, dst);
  extern __shared__ uint32_t smm[];
  __shared__ int32_t warp_tot[32];
  const bool first = blockIdx.x == 0;
  const MaskSort m = mask_sort_build(ids, T, slots, n_exp, smm, warp_tot, first, counts, offsets, err);
  const int A = T * slots;
  if (first)
    for (int i = threadIdx.x; i < A; i += blockDim.x) {
      const int e = ids[i], t = i / slots;
      if (e < 0 || e >= n_exp) continue;
      const int pos = mask_sort_pos(m, e, t);
      perm[pos] = i;
      inv[i] = pos;
    }
  const int i0 = int(int64_t(A) * blockIdx.x / gridDim.x), i1 = int(int64_t(A) * (blockIdx.x + 1) / gridDim.x);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (int i = i0 + warp; i < i1; i += nwarps) {
    const int e = ids[i], t = i / slots;
    if (e < 0 || e >= n_exp) continue;
    const int pos = mask_sort_pos(m, e, t);
    const uint4* s4 = reinterpret_cast<const uint4*>(src + size_t(t) * ld);
    uint4* d4 = reinterpret_cast<uint4*>(dst + size_t(pos) * H);
    // all of a lane's loads of a 4 KB stretch are issued before its stores,
    // so a row costs one L2 round trip per 4 KB instead of one per 512 B
    for (int c0 = 0; c0 < H / 8; c0 += 32 * kGatherVec) {
      uint4 v[kGatherVec];
#pragma unroll
      for (int j = 0; j < kGatherVec; ++j) {
        const int c = c0 + j * 32 + lane;
        if (c < H / 8) v[j] = s4[c];
      }
#pragma unroll
      for (int j = 0; j < kGatherVec; ++j) {
        const int c = c0 + j * 32 + lane;
        if (c < H / 8) d4[c] = v[j];
      }
    }
  }
}

// x[t] += sum_j w[t][j] * y[inv[t*slots+j]] (fixed slot order, deterministic);
// then optional hb[t] = fp16(rms(x[t]) * norm_w). One CTA per token, thread i
// owns columns 4i..4i+3 (H <= 4096, H % 4 == 0): 512 threads for H = 2048,
// so two tokens share an SM and one token's dependent loads (its slot rows,
// then those rows' values) overlap the other's. The slot rows are requested
// in batches of 8 float4 before their ordered adds.
__global__ void __launch_bounds__(1024) moe_combine_kernel(float* __restrict__ x, const float* __restrict__ y,
                                   const int32_t* __restrict__ inv, const float* __restrict__ weights, int H,
                                   int slots, const float* __restrict__ norm_w, float eps,
                                   gemm_in_t* __restrict__ hb) {
  pdl_trigger();
  pdl_wait(x, y, inv, weights, norm_w, hb);
  constexpr int kBatch = 8;
  __shared__ float red[32];
  __shared__ float sw[64];
  __shared__ int32_t srow[64];
  const int t = blockIdx.x, c = threadIdx.x;
  if (c < slots) {
    sw[c] = weights[size_t(t) * slots + c];
    srow[c] = inv[size_t(t) * slots + c];
  }
  const bool live = c < (H >> 2);
  float4* xr = reinterpret_cast<float4*>(x + size_t(t) * H);
  const float4 xo = live ? xr[c] : make_float4(0.f, 0.f, 0.f, 0.f);
  __syncthreads();
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  float ss = 0.f;
  if (live) {
    for (int j0 = 0; j0 < slots; j0 += kBatch) {
      float4 yv[kBatch];
#pragma unroll
      for (int b = 0; b < kBatch; ++b)
        if (j0 + b < slots) yv[b] = reinterpret_cast<const float4*>(y + size_t(srow[j0 + b]) * H)[c];
#pragma unroll
      for (int b = 0; b < kBatch; ++b)
        if (j0 + b < slots) {
          const float w = sw[j0 + b];
          v.x += w * yv[b].x;
          v.y += w * yv[b].y;
          v.z += w * yv[b].z;
          v.w += w * yv[b].w;
        }
    }
    v.x += xo.x;
    v.y += xo.y;
    v.z += xo.z;
    v.w += xo.w;
    xr[c] = v;
    ss = v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  const float tot = block_sum(ss, red);
  if (!norm_w || !live) return;
  const float inv_r = rsqrtf(tot / H + eps);
  const float4 w = reinterpret_cast<const float4*>(norm_w)[c];
  __half2* o = reinterpret_cast<__half2*>(hb + size_t(t) * H) + 2 * c;
  o[0] = to_gemm_in2(v.x * inv_r * w.x, v.y * inv_r * w.y);
  o[1] = to_gemm_in2(v.z * inv_r * w.z, v.w * inv_r * w.w);
}

// X_perm[p] = X[perm[p] / slots]: expert-sorted copy of the MoE input rows
// (contiguous per expert, so the GEMM's TMA loads one box per expert).
__global__ void gather_rows_kernel(const gemm_in_t* __restrict__ src, int ld, const int32_t* __restrict__ perm,
                                   int div, int H, gemm_in_t* dst) {
  pdl_trigger();
  pdl_wait(src, perm);
  const int p = blockIdx.x;
  const int row = perm[p] / div;
  const uint4* s4 = reinterpret_cast<const uint4*>(src + size_t(row) * ld);
  uint4* d4 = reinterpret_cast<uint4*>(dst + size_t(p) * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) d4[i] = s4[i];
}

// Greedy selection per row: IEEE total order, lowest index on ties
// (native/selection.h:3-12); any non-finite logit raises kErrNonFinite.
// Grid (rows, kArgmaxSplit): each CTA scans a slice of the row with float4
// loads and four independent running maxima; the last CTA of a row (counted
// in done[row], which it resets) reduces the slice maxima. The packed key
// (total order << 32 | ~index) makes the result independent of the order.
constexpr int kArgmaxSplit = 8;
// Constrained greedy selection (src/serving/choices.rs:65-98): for listed
// output row rows[k], the id of ids[offsets[k], offsets[k+1]) with the largest
// logit on the fp32 total order, the lowest id on equal logits (repeats and
// order of the ids do not matter). One CTA per constrained row; it runs after
// argmax_kernel, which has checked every logit of the row for finiteness and
// written the unconstrained winner that this kernel replaces. Ids are checked
// against the vocabulary on the host.
__global__ void __launch_bounds__(256) choice_select_kernel(const float* __restrict__ logits, int V,
                                                           const int32_t* __restrict__ rows,
                                                           const uint32_t* __restrict__ offsets,
                                                           const uint32_t* __restrict__ ids, uint32_t* tokens) {
  pdl_trigger();
  pdl_wait(logits, rows, offsets, ids);
  __shared__ uint64_t red[8];
  const int k = blockIdx.x, r = rows[k];
  const float* lr = logits + size_t(r) * V;
  uint64_t best = 0;
  for (uint32_t i = offsets[k] + threadIdx.x; i < offsets[k + 1]; i += blockDim.x) {
    const uint32_t id = ids[i];
    const uint64_t key = (uint64_t(total_key(lr[id])) << 32) | uint32_t(0xFFFFFFFFu - id);
    best = key > best ? key : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t b = red[0];
    for (int w = 1; w < 8; ++w) b = red[w] > b ? red[w] : b;
    tokens[r] = 0xFFFFFFFFu - uint32_t(b & 0xFFFFFFFFu);
  }
}

__global__ void __launch_bounds__(512) argmax_kernel(const float* __restrict__ logits, int V, uint32_t* tokens,
                                                     uint32_t* err, uint64_t* part, uint32_t* done) {
  pdl_trigger();
  pdl_wait(logits);
  __shared__ uint64_t red[16];
  __shared__ bool last;
  const int r = blockIdx.x, sp = blockIdx.y;
  const float* lr = logits + size_t(r) * V;
  const int per = ((V + kArgmaxSplit - 1) / kArgmaxSplit + 3) & ~3;
  const int i0 = sp * per, i1 = min(V, i0 + per);
  uint64_t best[4] = {0, 0, 0, 0};
  bool finite = true;
  auto take = [&](int k, float f, int i) {
    finite &= isfinite(f);
    const uint64_t key = (uint64_t(total_key(f)) << 32) | uint32_t(0xFFFFFFFFu - i);
    best[k] = key > best[k] ? key : best[k];
  };
  if ((V & 3) == 0) {
    for (int i = i0 + 4 * threadIdx.x; i < i1; i += 4 * blockDim.x) {  // i1 - i0 is a multiple of 4
      const float4 f = *reinterpret_cast<const float4*>(lr + i);
      take(0, f.x, i);
      take(1, f.y, i + 1);
      take(2, f.z, i + 2);
      take(3, f.w, i + 3);
    }
  } else {
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) take(0, lr[i], i);
  }
  uint64_t b = best[0];
#pragma unroll
  for (int k = 1; k < 4; ++k) b = best[k] > b ? best[k] : b;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t other = __shfl_xor_sync(0xffffffffu, b, o);
    b = other > b ? other : b;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = b;
  if (!finite) atomicOr(err, kErrNonFinite);
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t m = 0;
    for (int w = 0; w < int(blockDim.x >> 5); ++w) m = red[w] > m ? red[w] : m;
    part[size_t(r) * kArgmaxSplit + sp] = m;
    __threadfence();
    last = atomicAdd(&done[r], 1u) == kArgmaxSplit - 1;
  }
  __syncthreads();
  if (last && threadIdx.x == 0) {
    __threadfence();
    uint64_t m = 0;
    for (int k = 0; k < kArgmaxSplit; ++k) {
      const uint64_t v = *reinterpret_cast<volatile uint64_t*>(&part[size_t(r) * kArgmaxSplit + k]);
      m = v > m ? v : m;
    }
    tokens[r] = 0xFFFFFFFFu - uint32_t(m & 0xFFFFFFFFu);
    done[r] = 0;
  }
}

// MTP draft input (native/qwen_mtp.inc:157-161): per token t,
// cat[t] = [fp16(rms(embed(token_t)) * w_e), fp16(rms(hidden_t) * w_h)]
// (the embedding dequantised from the 4-bit table as in embed_norm_kernel).
__global__ void mtp_input_kernel(QMat embed, const uint32_t* __restrict__ tokens, const float* __restrict__ hidden,
                                 const float* __restrict__ w_e, const float* __restrict__ w_h, float eps,
                                 gemm_in_t* __restrict__ cat) {
  pdl_trigger();
  pdl_wait(tokens, hidden, w_e, w_h, cat);
  __shared__ float red[32];
  extern __shared__ float erow[];  // [H]
  const int t = blockIdx.x, H = embed.k;
  const uint32_t tok = tokens[t];
  float se = 0.f, sh = 0.f;
  for (int w = threadIdx.x; w < H / 8; w += blockDim.x) {
    const int c0 = w * 8;
    const uint8_t* tile = embed.tile(int(tok / kTileRows), c0 / kTileK);
    const int r = tok % kTileRows;
    const uint32_t word = *reinterpret_cast<const uint32_t*>(tile + r * 32 + (c0 % kTileK) / 2);
    const float sc = half_bits_to_float(reinterpret_cast<const uint16_t*>(tile + kTilePackedBytes)[r]) * (1.f / kTileScale);
    const float bi = half_bits_to_float(reinterpret_cast<const uint16_t*>(tile + kTilePackedBytes + kTileRows * 2)[r]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = fmaf(sc, float(nibble(word, j)), bi);
      erow[c0 + j] = v;
      se += v * v;
    }
  }
  const float* hr = hidden + size_t(t) * H;
  for (int c = threadIdx.x; c < H; c += blockDim.x) sh += hr[c] * hr[c];
  const float tot_e = block_sum(se, red);
  const float tot_h = block_sum(sh, red);
  const float ie = rsqrtf(tot_e / H + eps), ih = rsqrtf(tot_h / H + eps);
  gemm_in_t* out = cat + size_t(t) * 2 * H;
  for (int c = threadIdx.x; c < H; c += blockDim.x) {
    out[c] = to_gemm_in(erow[c] * ie * w_e[c]);
    out[H + c] = to_gemm_in(hr[c] * ih * w_h[c]);
  }
}

// Speculative accept, one thread per sequence (the plan() rule of
// src/serving/native_speculative.rs:100-127). A verify step fed
// [seed, d_0 .. d_{k-1}] from the parent and sampled rows r_0 .. r_k (r_j =
// greedy token after fed token j). Emitted tokens are r_0, r_1, ... while
// d_i == r_i and r_i is not EOS; the first mismatch (or an EOS) is emitted and
// ends the plan; after k matches the bonus r_k is emitted if the context still
// has room (remaining = ctx - position - 1). accepted = matched drafts (an EOS
// that matched counts), so the new state is the state after token
// `accepted` of the fed sequence.
__global__ void accept_kernel(const SeqDesc* __restrict__ descs, int n, const int32_t* __restrict__ cu_seqlens,
                              const uint32_t* __restrict__ tokens, const uint32_t* __restrict__ sampled,
                              const uint32_t* __restrict__ eos, int n_eos, int ctx, int32_t* acc_out,
                              uint32_t* emitted, int emit_stride, uint32_t* n_emitted) {
  pdl_trigger();
  pdl_wait(descs, cu_seqlens, tokens, sampled, eos);
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= n) return;
  const SeqDesc d = descs[s];
  const int k = d.count - 1, t0 = cu_seqlens[s];
  const int remaining = ctx - d.position - 1;
  auto is_eos = [&](uint32_t t) {
    for (int e = 0; e < n_eos; ++e)
      if (eos[e] == t) return true;
    return false;
  };
  uint32_t* em = emitted + size_t(s) * emit_stride;
  int ne = 0, acc = 0;
  bool stopped = false;
  for (int i = 0; i < k; ++i) {
    const uint32_t target = sampled[d.out_row0 + i];
    em[ne++] = target;
    const bool term = is_eos(target);
    const uint32_t draft = tokens[t0 + 1 + i];
    if (draft != target || term) {
      acc += draft == target;
      stopped = true;
      break;
    }
    ++acc;
  }
  if (!stopped && ne < remaining) em[ne++] = sampled[d.out_row0 + k];
  acc_out[s] = acc;
  n_emitted[s] = uint32_t(ne);
}

// Verify compaction: the state after token `accepted` (candidate slot
// cand_slots[cand + accepted]) becomes the sequence's version. Its DeltaNet
// state and conv history were written there by the step; here its block-table
// row (the pages of positions < position + accepted + 1) is copied from the
// full-length candidate's row and, when kept, its hidden rows are written.
__global__ void verify_compact_kernel(const SeqDesc* __restrict__ descs, const int32_t* __restrict__ cand_slots,
                                      const int32_t* __restrict__ acc, int32_t* block_table, int stride,
                                      const float* __restrict__ hidden_stage, const int32_t* __restrict__ cu_seqlens,
                                      float* hidden_pool, int chunk, int H) {
  pdl_trigger();
  pdl_wait(descs, cand_slots, acc, hidden_stage, cu_seqlens);
  const int s = blockIdx.x;
  const SeqDesc d = descs[s];
  const int a = acc[s];
  const int chosen = cand_slots[d.cand + a];
  if (chosen != d.child) {
    const int n_keep = (d.position + a + 1 + kPageTokens - 1) / kPageTokens;
    for (int j = threadIdx.x; j < n_keep; j += blockDim.x)
      block_table[size_t(chosen) * stride + j] = block_table[size_t(d.child) * stride + j];
  }
  if (d.hidden) {
    const float* src = hidden_stage + size_t(cu_seqlens[s]) * H;
    float* dst = hidden_pool + size_t(chosen) * chunk * H;
    for (int i = threadIdx.x; i < (a + 1) * H; i += blockDim.x) dst[i] = src[i];
  }
}

// Seeded synthetic prefix state: KV bf16 N(0,1) for positions < position,
// DeltaNet S fp32 N(0, 0.02), conv history fp32 N(0, 1). Values depend on
// (seed, layer, element), never on the page or slot they land in.
__global__ void synth_kv_kernel(KvPool kv, const int32_t* __restrict__ pages, int position, int ctx,
                                uint64_t seed) {
  const int pi = blockIdx.x, layer = blockIdx.y;
  const int D = kv.D, Hkv = kv.Hkv;
  __nv_bfloat16* pg = kv.page(layer, pages[pi]);
  const uint64_t key = mix64(seed * 0x632BE59BD9B4E019ull ^ mix64(0x4B56000000000000ull + layer));
  const float k = 1.0f / 37837.2265f;
  const int per = 2 * Hkv * kPageTokens * D;
  for (int e = threadIdx.x; e < per; e += blockDim.x) {
    const int i = e % D, o = (e / D) % kPageTokens, g = (e / (D * kPageTokens)) % Hkv,
              kvsel = e / (D * kPageTokens * Hkv);
    const int pos = pi * kPageTokens + o;
    float v = 0.f;
    if (pos < position) v = synth_normal(key, ((uint64_t(kvsel) * Hkv + g) * ctx + pos) * D + i, k);
    pg[e] = __float2bfloat16_rn(v);
  }
}

__global__ void synth_fill_kernel(float* out, size_t n, uint64_t key, float k) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    out[i] = synth_normal(key, i, k);
}

}  // namespace

void launch_synth_state(KvPool kv, const int32_t* pages, int n_pages, int position, int ctx,
                        GdnPool pool, int slot, const Dims& d, uint64_t seed, cudaStream_t s) {
  if (n_pages > 0 && kv.layers > 0)
    synth_kv_kernel<<<dim3(n_pages, kv.layers), 256, 0, s>>>(kv, pages, position, ctx, seed);
  for (int li = 0; li < pool.n_gdn; ++li) {
    const uint64_t ks = mix64(seed * 0x632BE59BD9B4E019ull ^ mix64(0x5354000000000000ull + li));
    const uint64_t kc = mix64(seed * 0x632BE59BD9B4E019ull ^ mix64(0x434F000000000000ull + li));
    synth_fill_kernel<<<256, 256, 0, s>>>(pool.state + (size_t(slot) * pool.n_gdn + li) * pool.state_elems,
                                          pool.state_elems, ks, 0.02f / 37837.2265f);
    synth_fill_kernel<<<64, 256, 0, s>>>(pool.conv + (size_t(slot) * pool.n_gdn + li) * pool.conv_elems,
                                         pool.conv_elems, kc, 1.0f / 37837.2265f);
  }
  (void)d;
}

// ------------------------------------------------------------------ launchers --

// Number of kernels this library has launched (read by rs_qwen_device_stats).
std::atomic<uint64_t> g_kernel_launches{0};
uint64_t kernel_launches() { return g_kernel_launches.load(); }
// Threads for the per-row kernels: one float2 column pair each up to 1024
// threads (H <= 2048), then up to 4 pairs each.
static inline int row_threads(int H) { return std::min(1024, std::max(32, (H / 2 + 31) / 32 * 32)); }
static inline void count_launch(int n = 1) { g_kernel_launches.fetch_add(uint64_t(n), std::memory_order_relaxed); }

void launch_pack(const SeqDesc* descs, int n_seq, const int32_t* new_pages, int32_t* block_table,
                 int bt_stride, Packed p, cudaStream_t s) {
  launch_pdl(pack_kernel, n_seq, 256, 0, s, descs, n_seq, new_pages, block_table, bt_stride, p);
  count_launch();
}

void launch_cow(KvPool kv, const SeqDesc* descs, int n_seq, const int32_t* new_pages, cudaStream_t s) {
  if (kv.layers == 0) return;
  launch_pdl(cow_kernel, dim3(n_seq, kv.layers), 256, 0, s, kv, descs, new_pages);
  count_launch();
}

void launch_embed_norm(const QMat& embed, const uint32_t* tokens, int T, const float* norm_w,
                       float eps, float* x, gemm_in_t* hb, cudaStream_t s) {
  launch_pdl(embed_norm_kernel, T, 256, 0, s, embed, tokens, norm_w, eps, x, hb);
  count_launch();
}

void launch_residual_norm(float* x, const float* partial, int splits, size_t split_stride, int T,
                          int H, const float* norm_w, float eps, gemm_in_t* hb,
                          const int32_t* out_token, int rows, float* hidden_f32, cudaStream_t s) {
  const int n = out_token ? rows : T;
  if (n <= 0) return;
  if (H > 8 * 1024 || H % 2) throw std::invalid_argument("hidden width must be even and at most 8192");
  if (splits > 8) throw std::invalid_argument("residual split-K above 8");
  launch_pdl(residual_norm_kernel, n, row_threads(H), 0, s, x, partial, splits, split_stride, H, norm_w, eps, hb, out_token,
                                                    hidden_f32);
  count_launch();
}


void launch_attn_prep(const Dims& d, const LayerDev& ly, const float* proj, int ld_proj, int splits,
                      size_t split_stride, const int32_t* token_pos, const int64_t* slot_mapping, int T, KvPool kv,
                      int kv_layer, float* q, float* gate, cudaStream_t s) {
  if (T <= 0) return;
  if (splits > 8) throw std::invalid_argument("attention projection split-K above 8");
  if (d.rope > d.D || d.rope % 2) throw std::invalid_argument("rope dims must be even and at most head_dim");
  const int threads = 32 * std::min(32, d.Hq + 2 * d.Hkv);
#define QWEN_PREP(DD)                                                                                         \
  if (d.D == DD) {                                                                                          \
    launch_pdl(attn_prep_kernel<DD>, T, threads, 0, s, proj, ld_proj, splits, split_stride, d.Hq, d.Hkv, d.rope,     \
                                               double(d.theta), d.eps, ly.q_norm, ly.k_norm, token_pos,      \
                                               slot_mapping, kv, kv_layer, q, gate);                         \
    count_launch();                                                                                         \
    return;                                                                                                 \
  }
  QWEN_PREP(256)
  QWEN_PREP(128)
  QWEN_PREP(64)
#undef QWEN_PREP
  throw std::invalid_argument("head_dim must be 64, 128 or 256");
}

void launch_attention_merge(const Dims& d, const float* ws, const float* gate, const int32_t* token_pos,
                            const int32_t* tokens, int T, int split_pages, int max_splits, gemm_in_t* out,
                            cudaStream_t s) {
  if (T <= 0) return;
  launch_pdl(attention_merge_kernel, dim3(T, d.Hq), 128, size_t(max_splits) * sizeof(float), s, ws, gate, token_pos,
             tokens, d.Hq, d.D, split_pages * kPageTokens, max_splits, out);
  count_launch();
}

void launch_route(const float* logits, int ld, int splits, size_t split_stride, int T, int E, int top,
                  int32_t* ids, float* weights, float* logits_out, cudaStream_t s) {
  if (E > 1024) throw std::invalid_argument("more than 1024 experts");
  if (splits > 8) throw std::invalid_argument("router split-K above 8");
  if (top < 1 || top > E || top > 255) throw std::invalid_argument("router top-k outside 1..min(experts, 255)");
  if (T <= 0) return;
  if (splits > 1 || top > 31) {
    launch_pdl(route_block_kernel, T, 256, 0, s, logits, ld, splits, split_stride, E, top, ids, weights, logits_out);
  } else {
    const int grid = (T + 7) / 8;
    auto go = [&](auto kernel) { launch_pdl(kernel, grid, 256, 0, s, logits, ld, E, top, T, ids, weights, logits_out); };
    if (E <= 32) go(route_warp_kernel<1>);
    else if (E <= 64) go(route_warp_kernel<2>);
    else if (E <= 128) go(route_warp_kernel<4>);
    else if (E <= 256) go(route_warp_kernel<8>);
    else if (E <= 512) go(route_warp_kernel<16>);
    else go(route_warp_kernel<32>);
  }
  count_launch();
}

void launch_expert_sort(const int32_t* ids, int n_assign, int slots, int n_experts, int32_t* counts,
                        int32_t* offsets, int32_t* perm, int32_t* inv, uint32_t* err, cudaStream_t s) {
  if (n_assign <= 0) return;
  const int T = n_assign / slots, nw = (T + 31) / 32, nb = (nw + kMaskWordsPerBlock - 1) / kMaskWordsPerBlock;
  const size_t mask_smem = (size_t(n_experts) * (nw + nb) + n_experts) * 4;
  if (n_assign % slots == 0 && n_experts <= 1025 && mask_smem <= 200 * 1024) {
    static std::atomic<uint64_t> mask_configured{0};
    once_per_device(mask_configured, [] {
      QWEN_CUDA(cudaFuncSetAttribute(expert_sort_mask_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     200 * 1024));
    });
    launch_pdl(expert_sort_mask_kernel, 1, 1024, mask_smem, s, ids, T, slots, n_experts, counts, offsets, perm, inv,
               err);
    count_launch();
    return;
  }
  const size_t smem = size_t(3 * n_experts) * 4 + size_t(32) * n_experts * 2;
  if (smem > 200 * 1024) throw std::invalid_argument("expert sort exceeds shared memory");
  static std::atomic<uint64_t> configured{0};
  once_per_device(configured, [] {
    QWEN_CUDA(cudaFuncSetAttribute(expert_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   200 * 1024));
  });
  launch_pdl(expert_sort_kernel, 1, 1024, smem, s, ids, n_assign, n_experts, counts, offsets, perm, inv);
  count_launch();
}

void launch_expert_sort_gather(const int32_t* ids, int n_assign, int slots, int n_experts, int32_t* counts,
                               int32_t* offsets, int32_t* perm, int32_t* inv, uint32_t* err, const gemm_in_t* src,
                               int ld, int H, gemm_in_t* dst, int sm_count, cudaStream_t s) {
  if (n_assign <= 0) return;
  if (H % 8 || ld % 8) throw std::invalid_argument("sort + gather: rows must be whole 16-byte vectors");
  const int T = n_assign / slots, nw = (T + 31) / 32, nb = (nw + kMaskWordsPerBlock - 1) / kMaskWordsPerBlock;
  const size_t mask_smem = (size_t(n_experts) * (nw + nb) + n_experts) * 4;
  if (n_assign % slots == 0 && n_experts <= 1025 && mask_smem <= 200 * 1024) {
    static std::atomic<uint64_t> configured{0};
    once_per_device(configured, [] {
      QWEN_CUDA(cudaFuncSetAttribute(expert_sort_gather_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     200 * 1024));
    });
    // about 8 rows per CTA (a warp per row, 32 warps), at most one CTA per SM
    const int grid = std::max(1, std::min(sm_count, (n_assign + 7) / 8));
    launch_pdl(expert_sort_gather_kernel, grid, 1024, mask_smem, s, ids, T, slots, n_experts, counts, offsets, perm,
               inv, err, src, ld, H, dst);
    count_launch();
    return;
  }
  launch_expert_sort(ids, n_assign, slots, n_experts, counts, offsets, perm, inv, err, s);
  launch_gather_rows(src, ld, perm, slots, n_assign, H, dst, s);
}

void launch_moe_combine(float* x, const float* y_sorted, const int32_t* inv, const float* weights,
                        int T, int H, int slots, const float* norm_w, float eps, gemm_in_t* hb,
                        const int32_t* out_token, int rows, float* hidden_f32, cudaStream_t s) {
  (void)out_token; (void)rows; (void)hidden_f32;
  if (T <= 0) return;
  if (slots > 64 || H > 4096 || H % 4) throw std::invalid_argument("combine geometry");
  launch_pdl(moe_combine_kernel, T, std::max(64, (H / 4 + 31) / 32 * 32), 0, s, x, y_sorted, inv, weights, H, slots,
             norm_w, eps, hb);
  count_launch();
}

void launch_gather_rows(const gemm_in_t* src, int ld, const int32_t* perm, int div, int n, int H,
                        gemm_in_t* dst, cudaStream_t s) {
  if (n <= 0) return;
  launch_pdl(gather_rows_kernel, n, 128, 0, s, src, ld, perm, div, H, dst);
  count_launch();
}

void launch_mtp_input(const QMat& embed, const uint32_t* tokens, int T, const float* hidden, const float* w_e,
                      const float* w_h, float eps, gemm_in_t* cat, cudaStream_t s) {
  if (T <= 0) return;
  launch_pdl(mtp_input_kernel, T, 256, size_t(embed.k) * sizeof(float), s, embed, tokens, hidden, w_e, w_h, eps, cat);
  count_launch();
}

void launch_accept(const SeqDesc* descs, int n, const int32_t* cu_seqlens, const uint32_t* tokens,
                   const uint32_t* sampled, const uint32_t* eos, int n_eos, int ctx, int32_t* acc, uint32_t* emitted,
                   int emit_stride, uint32_t* n_emitted, cudaStream_t s) {
  if (n <= 0) return;
  launch_pdl(accept_kernel, (n + 127) / 128, 128, 0, s, descs, n, cu_seqlens, tokens, sampled, eos, n_eos, ctx, acc,
             emitted, emit_stride, n_emitted);
  count_launch();
}

void launch_verify_compact(const SeqDesc* descs, int n, const int32_t* cand_slots, const int32_t* acc,
                           int32_t* block_table, int stride, const float* hidden_stage, const int32_t* cu_seqlens,
                           float* hidden_pool, int chunk, int H, cudaStream_t s) {
  if (n <= 0) return;
  launch_pdl(verify_compact_kernel, n, 256, 0, s, descs, cand_slots, acc, block_table, stride, hidden_stage,
             cu_seqlens, hidden_pool, chunk, H);
  count_launch();
}

void launch_argmax(const float* logits, int rows, int V, uint32_t* tokens, uint32_t* err, uint64_t* part,
                   uint32_t* done, cudaStream_t s) {
  if (rows <= 0) return;
  launch_pdl(argmax_kernel, dim3(rows, kArgmaxSplit), 512, 0, s, logits, V, tokens, err, part, done);
  count_launch();
}

void launch_choice_select(const float* logits, int V, const int32_t* rows, const uint32_t* offsets,
                          const uint32_t* ids, int n_rows, uint32_t* tokens, cudaStream_t s) {
  if (n_rows <= 0) return;
  launch_pdl(choice_select_kernel, n_rows, 256, 0, s, logits, V, rows, offsets, ids, tokens);
  count_launch();
}

}  // namespace qwen
