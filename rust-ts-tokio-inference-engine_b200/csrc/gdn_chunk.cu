// Gated-DeltaNet over long token runs (prefill chunks): the chunked form of
// the recurrence of native/operator_reference.h:19-45 / qwen_model.inc:185-202.
//
// Per value head the state S[dv][dk] follows, token by token,
//   S_t = g_t S_{t-1} (I - b_t k_t k_t^T) + b_t v_t k_t^T,   o_t = S_t q_t.
// Over a chunk of C tokens with initial state S_0 and log-decay prefix sums
// lg_t = sum_{m<=t} log g_m (gamma_t = exp(lg_t)) it unrolls to
//   h_i  = u_i - S_0 w_i
//   o_t  = gamma_t S_0 q_t + sum_{i<=t} (gamma_t / gamma_i)(q_t . k_i) h_i
//   S_C  = gamma_C S_0 + sum_i (gamma_C / gamma_i) h_i k_i^T
// where U = T diag(b) V and W = T diag(b gamma) K with
//   T = (I + L)^-1,  L[t][i] = b_t (gamma_t / gamma_i)(k_t . k_i)  (i < t).
// (Induction on t: the S_0-free part satisfies u_t = b_t (v_t - sum_{i<t}
// (gamma_t/gamma_i)(k_i . k_t) u_i), the S_0 part is gamma_t S_0 prod(I - b k k^T),
// whose WY factors are w'_t = b_t (gamma_t k_t - sum_{i<t} (gamma_t/gamma_i)(k_i . k_t) w'_i).)
//
// Two kernels per layer for the sequences whose step feeds at least
// kChunkMin tokens (verify steps keep the per-token kernel, which writes
// every token's state):
//  gdn_chunk_prep: CTA = (chunk, value head). Everything that does not
//    depend on S_0: the decay prefix sums, L and the decayed masked q.k
//    products, and U and W by forward substitution (one thread per column,
//    the column in registers). Chunks of a sequence run in parallel.
//  gdn_chunk_scan: CTA = (sequence, value head, block of kScanRows rows).
//    The rows of S are independent given the chunk's U, W, q, k and decays,
//    so each CTA carries its rows through the sequence's chunks: h, the
//    outputs o and the next rows, all in fp32 on the CUDA cores.
// gdn_chunk_norm then applies the gated RMSNorm over dv (rows from different
// CTAs) and writes the fp16 out_proj input.
#include <atomic>

#include "kernels.h"

namespace qwen {

extern std::atomic<uint64_t> g_kernel_launches;

namespace {

constexpr int C = kGdnChunk;  // tokens per chunk
constexpr int kScanRows = 32;   // state rows per scan CTA
constexpr int kScanThreads = 256;

__device__ __forceinline__ float split_sum_c(const float* pr, int col, int splits, size_t split_stride) {
  float v = pr[col];
  for (int s = 1; s < splits; ++s) v += pr[size_t(s) * split_stride + col];
  return v;
}

template <int DK, int DV>
__global__ void __launch_bounds__(DK + DV)
    gdn_chunk_prep_kernel(const SeqDesc* __restrict__ descs, const int32_t* __restrict__ cu_seqlens,
                          const int32_t* __restrict__ items, int hk, int hv, const float* __restrict__ qk,
                          const float* __restrict__ vv, const float* __restrict__ gb, float* __restrict__ U,
                          float* __restrict__ W, float* __restrict__ A, float* __restrict__ LG) {
  pdl_trigger();
  pdl_wait();
  constexpr int P = DK + 1;  // padded row stride: lanes reading different rows hit different banks
  extern __shared__ float sm[];
  float* Ks = sm;               // [C][P]
  float* Qs = Ks + C * P;       // [C][P]
  float* L = Qs + C * P;        // [C][C+1]
  __shared__ float lg[C], beta[C];
  const int item = blockIdx.x, head = blockIdx.y;
  const int seq = items[2 * item], chunk = items[2 * item + 1];
  const SeqDesc d = descs[seq];
  const int t0 = cu_seqlens[seq] + chunk * C;
  const int n = min(C, d.count - chunk * C);
  const int kh = head / (hv / hk), vd = hv * DV;
  const int tid = threadIdx.x, nthr = DK + DV;
  for (int e = tid; e < C * DK; e += nthr) {
    const int t = e / DK, c = e % DK;
    const float* row = qk + ((size_t(t0 + t) * hk + kh) * 2) * DK;
    Qs[t * P + c] = t < n ? row[c] : 0.f;
    Ks[t * P + c] = t < n ? row[DK + c] : 0.f;
  }
  if (tid < C) {
    const float g = tid < n ? gb[(size_t(t0 + tid) * hv + head) * 2] : 1.f;
    lg[tid] = fmaxf(logf(g), -1e4f);  // a zero decay stays finite: later ratios underflow to 0
    beta[tid] = tid < n ? gb[(size_t(t0 + tid) * hv + head) * 2 + 1] : 0.f;
  }
  __syncthreads();
  if (tid == 0)
    for (int t = 1; t < C; ++t) lg[t] += lg[t - 1];
  __syncthreads();
  // decayed products: L (strictly lower, k.k) and A (lower with diagonal, q.k)
  const size_t sc = size_t(item) * hv + head;
  float* Ag = A + sc * C * C;
  for (int p = tid; p < C * C; p += nthr) {
    const int t = p / C, i = p % C;
    float kk = 0.f, qkv = 0.f;
    if (i <= t) {
#pragma unroll 8
      for (int c = 0; c < DK; ++c) {
        const float ki = Ks[i * P + c];
        kk = fmaf(Ks[t * P + c], ki, kk);
        qkv = fmaf(Qs[t * P + c], ki, qkv);
      }
    }
    const float ratio = i <= t ? expf(lg[t] - lg[i]) : 0.f;
    L[t * (C + 1) + i] = i < t ? beta[t] * ratio * kk : 0.f;
    Ag[p] = (i <= t && t < n) ? ratio * qkv : 0.f;
  }
  __syncthreads();
  // forward substitution, one column per thread: U columns (values), then W columns (keys)
  float x[C];
  const bool is_u = tid < DV;
  const int col = is_u ? tid : tid - DV;
#pragma unroll
  for (int t = 0; t < C; ++t) {
    float b;
    if (is_u) b = t < n ? beta[t] * vv[size_t(t0 + t) * vd + head * DV + col] : 0.f;
    else b = beta[t] * expf(lg[t]) * Ks[t * P + col];
    float acc = b;
#pragma unroll
    for (int i = 0; i < t; ++i) acc = fmaf(-L[t * (C + 1) + i], x[i], acc);
    x[t] = acc;
  }
  float* dst = is_u ? U + sc * C * DV : W + sc * C * DK;
  const int ld = is_u ? DV : DK;
#pragma unroll
  for (int t = 0; t < C; ++t) dst[t * ld + col] = x[t];
  if (tid < C) LG[sc * C + tid] = lg[tid];
}

template <int DK, int DV>
__global__ void __launch_bounds__(kScanThreads)
    gdn_chunk_scan_kernel(const SeqDesc* __restrict__ descs, const int32_t* __restrict__ cu_seqlens,
                          const int32_t* __restrict__ longs, GdnPool pool, int li, int hk, int hv,
                          const float* __restrict__ qk, const float* __restrict__ U, const float* __restrict__ W,
                          const float* __restrict__ A, const float* __restrict__ LG, float* __restrict__ obuf,
                          uint32_t* err) {
  pdl_trigger();
  pdl_wait();
  constexpr int P = DK + 1, RP = kScanRows + 1, BLOCKS = DV / kScanRows;
  extern __shared__ float sm[];
  float* Ws = sm;                    // [C][P]
  float* Qs = Ws + C * P;            // [C][P]
  float* Ks = Qs + C * P;            // [C][P]
  float* As = Ks + C * P;            // [C][C+1]
  float* S = As + C * (C + 1);       // [kScanRows][P]
  float* Us = S + kScanRows * P;     // [C][RP]
  float* Hs = Us + C * RP;           // [C][RP]
  __shared__ float lg[C];
  const int ls = blockIdx.x / (hv * BLOCKS), rem = blockIdx.x % (hv * BLOCKS);
  const int head = rem / BLOCKS, rb = rem % BLOCKS;
  const int seq = longs[3 * ls], item0 = longs[3 * ls + 1], n_chunks = longs[3 * ls + 2];
  const SeqDesc d = descs[seq];
  const int kh = head / (hv / hk), vd = hv * DV, r0 = rb * kScanRows;
  const int tid = threadIdx.x;
  const size_t sl = size_t(hv) * DV * DK;
  const float* src = d.parent >= 0 ? pool.state + (size_t(d.parent) * pool.n_gdn + li) * sl + size_t(head) * DV * DK
                                   : nullptr;
  float* dst = pool.state + (size_t(d.child) * pool.n_gdn + li) * sl + size_t(head) * DV * DK;
  for (int e = tid; e < kScanRows * DK; e += kScanThreads) {
    const int r = e / DK, c = e % DK;
    S[r * P + c] = src ? src[size_t(r0 + r) * DK + c] : 0.f;
  }
  // phase A / B: token t = tid / 4 (64 tokens), rows quarter*8 .. +8
  const int at = tid >> 2, aq = tid & 3;
  // phase C: row tid / 8, columns (tid % 8) + 8m
  const int cr = tid >> 3, cb = tid & 7;
  for (int j = 0; j < n_chunks; ++j) {
    const size_t sc = size_t(item0 + j) * hv + head;
    const int t0 = cu_seqlens[seq] + j * C;
    const int n = min(C, d.count - j * C);
    __syncthreads();  // the previous chunk's readers are done
    for (int e = tid; e < C * DK; e += kScanThreads) {
      const int t = e / DK, c = e % DK;
      const float* row = qk + ((size_t(t0 + t) * hk + kh) * 2) * DK;
      Ws[t * P + c] = W[sc * C * DK + e];
      Qs[t * P + c] = t < n ? row[c] : 0.f;
      Ks[t * P + c] = t < n ? row[DK + c] : 0.f;
    }
    for (int e = tid; e < C * C; e += kScanThreads) As[(e / C) * (C + 1) + e % C] = A[sc * C * C + e];
    for (int e = tid; e < C * kScanRows; e += kScanThreads) {
      const int t = e / kScanRows, r = e % kScanRows;
      Us[t * RP + r] = U[sc * C * DV + size_t(t) * DV + r0 + r];
    }
    if (tid < C) lg[tid] = LG[sc * C + tid];
    __syncthreads();
    float hacc[8], qacc[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) hacc[m] = qacc[m] = 0.f;
#pragma unroll 4
    for (int c = 0; c < DK; ++c) {
      const float w = Ws[at * P + c], q = Qs[at * P + c];
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const float s = S[(aq * 8 + m) * P + c];
        hacc[m] = fmaf(w, s, hacc[m]);
        qacc[m] = fmaf(q, s, qacc[m]);
      }
    }
#pragma unroll
    for (int m = 0; m < 8; ++m) Hs[at * RP + aq * 8 + m] = Us[at * RP + aq * 8 + m] - hacc[m];
    __syncthreads();
    const float gt = expf(lg[at]);
    float o[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) o[m] = gt * qacc[m];
    for (int i = 0; i <= at; ++i) {
      const float a = As[at * (C + 1) + i];
#pragma unroll
      for (int m = 0; m < 8; ++m) o[m] = fmaf(a, Hs[i * RP + aq * 8 + m], o[m]);
    }
    if (at < n) {
#pragma unroll
      for (int m = 0; m < 8; ++m) obuf[size_t(t0 + at) * vd + head * DV + r0 + aq * 8 + m] = o[m];
    }
    // next rows: S = gamma_C S + sum_t (gamma_C / gamma_t) h_t k_t^T
    const float lc = lg[C - 1];
    float acc[DK / 8];
#pragma unroll
    for (int m = 0; m < DK / 8; ++m) acc[m] = expf(lc) * S[cr * P + cb + 8 * m];
    for (int t = 0; t < C; ++t) {
      const float f = expf(lc - lg[t]) * Hs[t * RP + cr];
#pragma unroll
      for (int m = 0; m < DK / 8; ++m) acc[m] = fmaf(f, Ks[t * P + cb + 8 * m], acc[m]);
    }
    __syncthreads();  // phase A's readers of S are done before it is overwritten
#pragma unroll
    for (int m = 0; m < DK / 8; ++m) S[cr * P + cb + 8 * m] = acc[m];
  }
  __syncthreads();
  bool finite = true;
  for (int e = tid; e < kScanRows * DK; e += kScanThreads) {
    const int r = e / DK, c = e % DK;
    const float v = S[r * P + c];
    finite &= isfinite(v);
    dst[size_t(r0 + r) * DK + c] = v;
  }
  if (!finite) atomicOr(err, kErrNonFinite);
}

// Gated RMSNorm over dv of every head of the listed tokens
// (native/qwen_model.inc:203-204): y = rms(o) * w * silu(z), one warp per head.
template <int DV>
__global__ void __launch_bounds__(1024, 1)
    gdn_chunk_norm_kernel(const int32_t* __restrict__ tokens, int hv, const float* __restrict__ obuf,
                          const float* __restrict__ proj, int ld, int splits, size_t split_stride, int cd,
                          const float* __restrict__ gnorm, float eps, gemm_in_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  constexpr int PER = DV / 32;
  const int t = tokens[blockIdx.x];
  const int head = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (head >= hv) return;
  const int vd = hv * DV;
  float o[PER], ss = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    o[k] = obuf[size_t(t) * vd + head * DV + lane + 32 * k];
    ss += o[k] * o[k];
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / DV + eps);
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int c = lane + 32 * k;
    const float z = split_sum_c(proj + size_t(t) * ld, cd + head * DV + c, splits, split_stride);
    out[size_t(t) * vd + head * DV + c] = to_gemm_in(o[k] * inv * gnorm[c] * siluf_(z));
  }
}

// Token-parallel preparation of long runs: CTA = (64-token chunk, key head),
// one thread per channel of the key head (its q and k channels and its R
// value heads' v channels), gdn_prep's arithmetic per token: causal conv +
// SiLU, q / k RMS scaling (per-warp partials summed in a fixed order), decay
// and beta. A chunk starts from the K-1 inputs before it: earlier tokens of
// the run (their projection rows) or the parent's conv history. The child's
// history is written afterwards by gdn_conv_tail (a consumed parent's history
// is the child's, so it must not change while any chunk still reads it).
template <int DK, int DV, int R>
__global__ void __launch_bounds__(2 * DK + R * DV, 2)
    gdn_run_prep_kernel(const float* __restrict__ proj, int ld, int splits, size_t split_stride,
                        const SeqDesc* __restrict__ descs, const int32_t* __restrict__ cu_seqlens,
                        const int32_t* __restrict__ items, GdnPool pool, int li, int hk, int hv, int conv,
                        const float* __restrict__ conv_w, const float* __restrict__ a_log,
                        const float* __restrict__ dt_bias, float* __restrict__ qk_out, float* __restrict__ v_out,
                        float* __restrict__ gb_out) {
  pdl_trigger();
  pdl_wait();
  constexpr int QW = DK / 32;
  __shared__ float red[2][2 * QW];
  const int item = blockIdx.x, kh = blockIdx.y;
  const int seq = items[2 * item], chunk = items[2 * item + 1];
  const SeqDesc d = descs[seq];
  const int s0 = cu_seqlens[seq], c0 = chunk * C;
  const int n = min(C, d.count - c0);
  const int kd = hk * DK, vd = hv * DV, cd = 2 * kd + vd;
  const int c = threadIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gc = c < DK ? kh * DK + c : (c < 2 * DK ? kd + kh * DK + (c - DK) : 2 * kd + kh * R * DV + (c - 2 * DK));
  const size_t cl = size_t(conv - 1) * cd;
  const float* hist = d.parent >= 0 ? pool.conv + (size_t(d.parent) * pool.n_gdn + li) * cl : nullptr;
  auto P = [&](int pos) { return split_sum_c(proj + size_t(s0 + pos) * ld, gc, splits, split_stride); };
  float taps[7], cw[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) cw[j] = j < conv ? conv_w[size_t(gc) * conv + j] : 0.f;
#pragma unroll
  for (int j = 0; j < 7; ++j) {  // input at run position c0 - (conv-1) + j, oldest first
    const int pos = c0 - (conv - 1) + j;
    taps[j] = j < conv - 1 ? (pos >= 0 ? P(pos) : (hist ? hist[size_t(pos + conv - 1) * cd + gc] : 0.f)) : 0.f;
  }
  float cw_last = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (j == conv - 1) cw_last = cw[j];
  const int R_ = R;
  const int gh = kh * R_ + (c < R_ ? c : 0);
  const float gdt = c < R_ ? dt_bias[gh] : 0.f, galog = c < R_ ? a_log[gh] : 0.f;
  for (int i = 0; i < n; ++i) {
    const int t = s0 + c0 + i;
    const float* pr = proj + size_t(t) * ld;
    const float cur = split_sum_c(pr, gc, splits, split_stride);
    const float ga = c < R_ ? split_sum_c(pr, cd + vd + gh, splits, split_stride) : 0.f;
    const float gbeta = c < R_ ? split_sum_c(pr, cd + vd + hv + gh, splits, split_stride) : 0.f;
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 7; ++j)
      if (j < conv - 1) acc += taps[j] * cw[j];
    acc += cur * cw_last;
#pragma unroll
    for (int j = 0; j < 7; ++j)
      if (j < conv - 1) taps[j] = j + 1 < conv - 1 ? taps[j + 1] : cur;
    const float act = siluf_(acc);
    if (c >= 2 * DK) {
      v_out[size_t(t) * vd + kh * R_ * DV + (c - 2 * DK)] = act;
    } else {
      float ss = warp_sum(act * act);
      if (lane == 0) red[i & 1][warp] = ss;
      asm volatile("bar.sync 1, %0;" ::"r"(2 * DK) : "memory");
      const int g0 = c < DK ? 0 : QW;
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < QW; ++w) tot += red[i & 1][g0 + w];
      const float rinv = rsqrtf(tot / DK + 1e-6f);
      float* dstq = qk_out + ((size_t(t) * hk + kh) * 2) * DK;
      if (c < DK) dstq[c] = act * (rinv / DK);
      else dstq[DK + (c - DK)] = act * (rinv * rsqrtf(float(DK)));
    }
    if (c < R_) {
      const float av = ga + gdt;
      const float sp = fmaxf(av, 0.f) + log1pf(__expf(-fabsf(av)));
      gb_out[(size_t(t) * hv + gh) * 2 + 0] = expf(-expf(galog) * sp);
      gb_out[(size_t(t) * hv + gh) * 2 + 1] = sigmoidf_(gbeta);
    }
  }
}

// The child's conv history of each long run: its last conv-1 inputs.
__global__ void __launch_bounds__(256)
    gdn_conv_tail_kernel(const float* __restrict__ proj, int ld, int splits, size_t split_stride,
                         const SeqDesc* __restrict__ descs, const int32_t* __restrict__ cu_seqlens,
                         const int32_t* __restrict__ longs, GdnPool pool, int li, int conv, int cd) {
  pdl_trigger();
  pdl_wait();
  const int seq = longs[3 * blockIdx.y];
  const SeqDesc d = descs[seq];
  const int ch = blockIdx.x * blockDim.x + threadIdx.x;
  if (ch >= cd) return;
  const size_t cl = size_t(conv - 1) * cd;
  float* dst = pool.conv + (size_t(d.child) * pool.n_gdn + li) * cl;
  const int last = cu_seqlens[seq] + d.count - 1;  // runs are longer than conv - 1 tokens
  for (int j = 0; j < conv - 1; ++j)
    dst[size_t(j) * cd + ch] = split_sum_c(proj + size_t(last - (conv - 2) + j) * ld, ch, splits, split_stride);
}

template <int DK, int DV>
void launch_chunked(const GdnChunkPlan& cp, const Dims& d, const LayerDev& ly, const float* proj, int ld_proj,
                    int splits, size_t split_stride, const SeqDesc* descs, const int32_t* cu_seqlens, GdnPool pool,
                    int li, gemm_in_t* out, uint32_t* err, const float* qk_buf, float* v_buf, const float* gb_buf,
                    cudaStream_t s) {
  constexpr size_t prep_smem = (2 * C * (DK + 1) + C * (C + 1)) * sizeof(float);
  constexpr size_t scan_smem =
      (3 * C * (DK + 1) + C * (C + 1) + kScanRows * (DK + 1) + 2 * C * (kScanRows + 1)) * sizeof(float);
  static_assert(prep_smem <= 227 * 1024 && scan_smem <= 227 * 1024, "chunked DeltaNet shared memory");
  static std::atomic<uint64_t> set{0};
  once_per_device(set, [] {
    QWEN_CUDA(cudaFuncSetAttribute(gdn_chunk_prep_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   int(prep_smem)));
    QWEN_CUDA(cudaFuncSetAttribute(gdn_chunk_scan_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   int(scan_smem)));
  });
  launch_pdl(gdn_chunk_prep_kernel<DK, DV>, dim3(cp.n_items, d.hv), DK + DV, prep_smem, s, descs, cu_seqlens,
             cp.items, d.hk, d.hv, qk_buf, v_buf, gb_buf, cp.U, cp.W, cp.A, cp.LG);
  launch_pdl(gdn_chunk_scan_kernel<DK, DV>, cp.n_long * d.hv * (DV / kScanRows), kScanThreads, scan_smem, s, descs,
             cu_seqlens, cp.longs, pool, li, d.hk, d.hv, qk_buf, cp.U, cp.W, cp.A, cp.LG, v_buf, err);
  launch_pdl(gdn_chunk_norm_kernel<DV>, cp.n_tokens, 32 * d.hv, 0, s, cp.tokens, d.hv, v_buf, proj, ld_proj, splits,
             split_stride, d.cd, ly.gnorm, d.eps, out);
  QWEN_CUDA(cudaGetLastError());
  g_kernel_launches.fetch_add(3, std::memory_order_relaxed);
}

}  // namespace

void launch_gdn_run_prep(const GdnChunkPlan& cp, const Dims& d, const LayerDev& ly, const float* proj, int ld_proj,
                         int splits, size_t split_stride, const SeqDesc* descs, const int32_t* cu_seqlens,
                         GdnPool pool, int li, float* qk_buf, float* v_buf, float* gb_buf, cudaStream_t s) {
  if (cp.n_long <= 0) return;
  if (d.conv > 8 || d.conv < 2) throw std::invalid_argument("conv kernel width unsupported");
  const int R = d.hv / d.hk;
  auto go = [&](auto kernel, int threads) {
    launch_pdl(kernel, dim3(cp.n_items, d.hk), threads, 0, s, proj, ld_proj, splits, split_stride, descs, cu_seqlens,
               cp.items, pool, li, d.hk, d.hv, d.conv, ly.conv_w, ly.a_log, ly.dt_bias, qk_buf, v_buf, gb_buf);
  };
  if (d.dk == 128 && d.dv == 128 && R == 2) go(gdn_run_prep_kernel<128, 128, 2>, 2 * 128 + 2 * 128);
  else if (d.dk == 128 && d.dv == 128 && R == 1) go(gdn_run_prep_kernel<128, 128, 1>, 2 * 128 + 128);
  else if (d.dk == 64 && d.dv == 64 && R == 2) go(gdn_run_prep_kernel<64, 64, 2>, 2 * 64 + 2 * 64);
  else if (d.dk == 64 && d.dv == 64 && R == 1) go(gdn_run_prep_kernel<64, 64, 1>, 2 * 64 + 64);
  else throw std::invalid_argument("chunked DeltaNet geometry unsupported");
  launch_pdl(gdn_conv_tail_kernel, dim3((d.cd + 255) / 256, cp.n_long), 256, 0, s, proj, ld_proj, splits,
             split_stride, descs, cu_seqlens, cp.longs, pool, li, d.conv, d.cd);
  QWEN_CUDA(cudaGetLastError());
  g_kernel_launches.fetch_add(2, std::memory_order_relaxed);
}

void launch_gdn_chunked(const GdnChunkPlan& cp, const Dims& d, const LayerDev& ly, const float* proj, int ld_proj,
                        int splits, size_t split_stride, const SeqDesc* descs, const int32_t* cu_seqlens,
                        GdnPool pool, int li, gemm_in_t* out, uint32_t* err, const float* qk_buf, float* v_buf,
                        const float* gb_buf, cudaStream_t s) {
  if (cp.n_long <= 0) return;
  if (d.hv > 32) throw std::invalid_argument("chunked DeltaNet: at most 32 value heads");
  if (d.dk == 128 && d.dv == 128)
    launch_chunked<128, 128>(cp, d, ly, proj, ld_proj, splits, split_stride, descs, cu_seqlens, pool, li, out, err,
                             qk_buf, v_buf, gb_buf, s);
  else if (d.dk == 64 && d.dv == 64)
    launch_chunked<64, 64>(cp, d, ly, proj, ld_proj, splits, split_stride, descs, cu_seqlens, pool, li, out, err,
                           qk_buf, v_buf, gb_buf, s);
  else
    throw std::invalid_argument("chunked DeltaNet geometry unsupported (dk = dv in {64, 128})");
}

}  // namespace qwen
