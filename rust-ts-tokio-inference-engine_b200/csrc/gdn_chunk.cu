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
//    outputs o and the next rows as tensor-core products (3xTF32, fp32
//    accumulation, about fp32 accuracy), the state kept in fp32.
// gdn_chunk_norm then applies the gated RMSNorm over dv (rows from different
// CTAs) and writes the fp16 out_proj input.
#include <atomic>

#include "kernels.h"

namespace qwen {

extern std::atomic<uint64_t> g_kernel_launches;

namespace {

constexpr int C = kGdnChunk;  // tokens per chunk
constexpr int kScanRows = 32;   // state rows per scan CTA
constexpr int kScanThreads = 512;
constexpr int kRunBlock = 16;   // tokens per run-prep CTA

// Sum of the split-K partials of one column, in split order; the (at most
// 8) loads are issued together.
__device__ __forceinline__ float split_sum_c(const float* pr, int col, int splits, size_t split_stride) {
  float part[8];
#pragma unroll
  for (int s = 0; s < 8; ++s) part[s] = s < splits ? pr[size_t(s) * split_stride + col] : 0.f;
  float v = part[0];
#pragma unroll
  for (int s = 1; s < 8; ++s)
    if (s < splits) v += part[s];
  return v;
}

// 16-byte global -> shared copy without registers (zero-filled when !valid).
__device__ __forceinline__ void cp16(float* dst, const float* src, bool valid) {
  const uint32_t d = uint32_t(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(valid ? 16 : 0) : "memory");
}

template <int DK, int DV>
__global__ void __launch_bounds__(DK + DV)
    gdn_chunk_prep_kernel(const SeqDesc* __restrict__ descs, const int32_t* __restrict__ cu_seqlens,
                          const int32_t* __restrict__ items, int hk, int hv, const float* __restrict__ qk,
                          const float* __restrict__ vv, const float* __restrict__ proj, int ld, int splits,
                          size_t split_stride, int cd, const float* __restrict__ a_log,
                          const float* __restrict__ dt_bias, float* __restrict__ U, float* __restrict__ W,
                          float* __restrict__ A, float* __restrict__ LG) {
  pdl_trigger();
  pdl_wait(descs, cu_seqlens, items, qk, vv, proj, a_log, dt_bias, U, W, A, LG);
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
  {  // q and k rows of the chunk: all loads issued before the shared stores
    constexpr int PER = C * DK / 4 / (DK + DV);  // float4 per thread (8)
    float4 qv[PER], kv[PER];
#pragma unroll
    for (int m = 0; m < PER; ++m) {
      const int e = tid + m * nthr, t = e / (DK / 4), c4 = e % (DK / 4);
      const float4* row = reinterpret_cast<const float4*>(qk + ((size_t(t0 + t) * hk + kh) * 2) * DK);
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      qv[m] = t < n ? row[c4] : z;
      kv[m] = t < n ? row[DK / 4 + c4] : z;
    }
#pragma unroll
    for (int m = 0; m < PER; ++m) {
      const int e = tid + m * nthr, t = e / (DK / 4), c = 4 * (e % (DK / 4));
      Qs[t * P + c] = qv[m].x, Qs[t * P + c + 1] = qv[m].y, Qs[t * P + c + 2] = qv[m].z, Qs[t * P + c + 3] = qv[m].w;
      Ks[t * P + c] = kv[m].x, Ks[t * P + c + 1] = kv[m].y, Ks[t * P + c + 2] = kv[m].z, Ks[t * P + c + 3] = kv[m].w;
    }
  }
  if (tid < C) {  // decay and beta (gdn_prep's arithmetic), kept in log form for the products
    float lgv = 0.f, bt = 0.f;
    if (tid < n) {
      const float* pr = proj + size_t(t0 + tid) * ld;
      const float av = split_sum_c(pr, cd + vd + head, splits, split_stride) + dt_bias[head];
      const float bv = split_sum_c(pr, cd + vd + hv + head, splits, split_stride);
      const float sp = fmaxf(av, 0.f) + log1pf(__expf(-fabsf(av)));
      const float g = expf(-expf(a_log[head]) * sp);
      lgv = fmaxf(logf(g), -1e4f);  // a zero decay stays finite: later ratios underflow to 0
      bt = sigmoidf_(bv);
    }
    lg[tid] = lgv;
    beta[tid] = bt;
  }
  __syncthreads();
  if (tid == 0)
    for (int t = 1; t < C; ++t) lg[t] += lg[t - 1];
  __syncthreads();
  // decayed products: L (strictly lower, k.k) and A (lower with diagonal, q.k),
  // in 4x4 register tiles of (t, i); tiles above the diagonal are skipped
  const size_t sc = size_t(item) * hv + head;
  float* Ag = A + sc * C * C;
  for (int tile = tid; tile < (C / 4) * (C / 4); tile += nthr) {
    const int tb = tile / (C / 4), ib = tile % (C / 4);
    float kk[4][4], qq[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) kk[a][b] = qq[a][b] = 0.f;
    if (ib <= tb) {
#pragma unroll 4
      for (int c = 0; c < DK; ++c) {
        float kt[4], qt[4], ki[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          kt[a] = Ks[(4 * tb + a) * P + c];
          qt[a] = Qs[(4 * tb + a) * P + c];
          ki[a] = Ks[(4 * ib + a) * P + c];
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            kk[a][b] = fmaf(kt[a], ki[b], kk[a][b]);
            qq[a][b] = fmaf(qt[a], ki[b], qq[a][b]);
          }
      }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int t = 4 * tb + a, i = 4 * ib + b;
        const float ratio = i <= t ? expf(lg[t] - lg[i]) : 0.f;
        L[t * (C + 1) + i] = i < t ? beta[t] * ratio * kk[a][b] : 0.f;
        Ag[t * C + i] = (i <= t && t < n) ? ratio * qq[a][b] : 0.f;
      }
  }
  __syncthreads();
  // forward substitution, one column per thread: U columns (values), then W columns (keys)
  float x[C];
  const bool is_u = tid < DV;
  const int col = is_u ? tid : tid - DV;
  // right-hand sides: this thread's column of beta V (values, loaded up front)
  // or of beta gamma K (keys)
#pragma unroll
  for (int t = 0; t < C; ++t) x[t] = (is_u && t < n) ? vv[size_t(t0 + t) * vd + head * DV + col] : 0.f;
#pragma unroll
  for (int t = 0; t < C; ++t) {
    const float b = is_u ? beta[t] * x[t] : beta[t] * expf(lg[t]) * Ks[t * P + col];
    float part[4] = {b, 0.f, 0.f, 0.f};  // four independent chains
#pragma unroll
    for (int i = 0; i < t; ++i) part[i & 3] = fmaf(-L[t * (C + 1) + i], x[i], part[i & 3]);
    x[t] = (part[0] + part[1]) + (part[2] + part[3]);
  }
  float* dst = is_u ? U + sc * C * DV : W + sc * C * DK;
  const int ldx = is_u ? DV : DK;
#pragma unroll
  for (int t = 0; t < C; ++t) dst[t * ldx + col] = x[t];
  if (tid < C) LG[sc * C + tid] = lg[tid];
}

// 3xTF32 products on the tensor cores: x = big + small with big = tf32(x)
// and small = tf32(x - big); a.b ~ a_s.b_b + a_b.b_s + a_b.b_b (the small.small
// term is below fp32 rounding), accumulated in fp32 by mma.sync m16n8k8.
__device__ __forceinline__ void split_tf32(float x, uint32_t& big, uint32_t& small) {
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(big) : "f"(x));
  const float r = x - __uint_as_float(big);
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(small) : "f"(r));
}
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// d += A B for one m16n8k8 step from fp32 fragments (A: a[4], B: b0, b1).
__device__ __forceinline__ void mma3_tf32(float (&d)[4], const float (&a)[4], float b0, float b1) {
  uint32_t ab[4], as[4], bb0, bs0, bb1, bs1;
#pragma unroll
  for (int k = 0; k < 4; ++k) split_tf32(a[k], ab[k], as[k]);
  split_tf32(b0, bb0, bs0);
  split_tf32(b1, bb1, bs1);
  mma_tf32(d, as, bb0, bb1);
  mma_tf32(d, ab, bs0, bs1);
  mma_tf32(d, ab, bb0, bb1);
}
__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
// d += A B with single tf32 roundings (products that only reach the outputs).
__device__ __forceinline__ void mma1_tf32(float (&d)[4], const float (&a)[4], float b0, float b1) {
  const uint32_t ab[4] = {to_tf32(a[0]), to_tf32(a[1]), to_tf32(a[2]), to_tf32(a[3])};
  mma_tf32(d, ab, to_tf32(b0), to_tf32(b1));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_groups() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// One CTA carries kScanRows rows of one value head's state through the
// sequence's chunks. Per chunk, on the tensor cores (3xTF32, fp32
// accumulation; fragments of m16n8k8: lane (g, t) = (lane / 4, lane % 4)):
//   A: H = U - W S^T and QS = Q S^T (64 tokens x 32 rows, K = dk): warp w owns
//      the 16-token x 8-row tile (w / 4, w % 4) of both;
//   B: O = gamma_t QS + A H (the decayed masked q.k products times H, K = 64),
//      same tiles, written to obuf. QS and A H only reach the outputs, so they
//      take single tf32 roundings (relative error ~1e-3 of the output); the
//      products that carry the state (W S^T, phase C) take three;
//   C: S = gamma_C S + (f H)^T K with f_t = gamma_C / gamma_t (32 rows x dk,
//      K = 64), dk / 64 tiles per warp, read and written in place.
// The next chunk's W, q, U and decays are requested once phase A is done,
// its A block once phase B is done and its k rows once phase C is done, so
// the copies overlap the remaining phases. Shared-memory row strides put the
// 32 fragment elements a warp reads at once in distinct banks.
template <int DK, int DV>
__global__ void __launch_bounds__(kScanThreads, 1)
    gdn_chunk_scan_kernel(const SeqDesc* __restrict__ descs, const int32_t* __restrict__ cu_seqlens,
                          const int32_t* __restrict__ longs, GdnPool pool, int li, int hk, int hv,
                          const float* __restrict__ qk, const float* __restrict__ U, const float* __restrict__ W,
                          const float* __restrict__ A, const float* __restrict__ LG, float* __restrict__ obuf,
                          uint32_t* err) {
  pdl_trigger();
  pdl_wait(descs, cu_seqlens, longs, qk, U, W, A, LG, obuf);
  static_assert(kScanThreads == 512 && kScanRows == 32 && C == 64 && DK % 64 == 0, "scan tiling");
  constexpr int PQ = DK + 4;   // W, q rows (A operands: bank = 4g + t)
  constexpr int PK = DK + 8;   // k rows (B operand over tokens: bank = 8t + g)
  constexpr int PS = DK + 4;   // state rows (B operand of phase A: bank = 4g + t)
  constexpr int PA = C + 4;    // A block rows
  constexpr int PH = kScanRows + 8;  // H / U rows (bank = 8t + g)
  constexpr int BLOCKS = DV / kScanRows;
  constexpr int NTC = DK / 8, TPW = 2 * NTC / 16;  // phase C: n tiles, tiles per warp
  extern __shared__ __align__(16) float sm[];
  float* Ws = sm;                  // [C][PQ]
  float* Qs = Ws + C * PQ;         // [C][PQ]
  float* Ks = Qs + C * PQ;         // [C][PK]
  float* As = Ks + C * PK;         // [C][PA]
  float* S = As + C * PA;          // [kScanRows][PS]
  float* Us = S + kScanRows * PS;  // [C][PH]
  float* Hs = Us + C * PH;         // [C][PH]
  __shared__ __align__(16) float lgb[2][C];
  __shared__ float gs[C], fs[C];
  const int ls = blockIdx.x / (hv * BLOCKS), rem = blockIdx.x % (hv * BLOCKS);
  const int head = rem / BLOCKS, rb = rem % BLOCKS;
  const int seq = longs[3 * ls], item0 = longs[3 * ls + 1], n_chunks = longs[3 * ls + 2];
  const SeqDesc d = descs[seq];
  const int kh = head / (hv / hk), vd = hv * DV, r0 = rb * kScanRows;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, tq = lane & 3;
  const size_t sl = size_t(hv) * DV * DK;
  const float* src = d.parent >= 0 ? pool.state + (size_t(d.parent) * pool.n_gdn + li) * sl + size_t(head) * DV * DK
                                   : nullptr;
  float* dst = pool.state + (size_t(d.child) * pool.n_gdn + li) * sl + size_t(head) * DV * DK;
  const int cu0 = cu_seqlens[seq];

  // chunk j's inputs: group 1 = W, q, U, decays; group 2 = A; group 3 = k rows
  auto load_wqu = [&](int j) {
    const size_t sc = size_t(item0 + j) * hv + head;
    const int t0 = cu0 + j * C, n = min(C, d.count - j * C);
    for (int e = tid; e < C * DK / 4; e += kScanThreads) {
      const int t = e / (DK / 4), c = 4 * (e % (DK / 4));
      const float* row = qk + ((size_t(t0 + t) * hk + kh) * 2) * DK;
      cp16(Ws + t * PQ + c, W + sc * C * DK + size_t(t) * DK + c, true);
      cp16(Qs + t * PQ + c, t < n ? row + c : qk, t < n);
    }
    for (int e = tid; e < C * kScanRows / 4; e += kScanThreads) {
      const int t = e / (kScanRows / 4), r = 4 * (e % (kScanRows / 4));
      cp16(Us + t * PH + r, U + sc * C * DV + size_t(t) * DV + r0 + r, true);
    }
    if (tid < C / 4) cp16(lgb[j & 1] + 4 * tid, LG + sc * C + 4 * tid, true);
    cp_commit();
  };
  auto load_a = [&](int j) {
    const size_t sc = size_t(item0 + j) * hv + head;
    for (int e = tid; e < C * C / 4; e += kScanThreads) {
      const int t = e / (C / 4), i = 4 * (e % (C / 4));
      cp16(As + t * PA + i, A + sc * C * C + size_t(t) * C + i, true);
    }
    cp_commit();
  };
  auto load_k = [&](int j) {
    const int t0 = cu0 + j * C, n = min(C, d.count - j * C);
    for (int e = tid; e < C * DK / 4; e += kScanThreads) {
      const int t = e / (DK / 4), c = 4 * (e % (DK / 4));
      const float* row = qk + ((size_t(t0 + t) * hk + kh) * 2) * DK;
      cp16(Ks + t * PK + c, t < n ? row + DK + c : qk, t < n);
    }
    cp_commit();
  };
  load_wqu(0);
  load_a(0);
  load_k(0);
  for (int e = tid; e < kScanRows * DK; e += kScanThreads) {
    const int r = e / DK, c = e % DK;
    S[r * PS + c] = src ? src[size_t(r0 + r) * DK + c] : 0.f;
  }
  const int mt = warp >> 2, nt = warp & 3;          // phase A / B tile
  const int ta = 16 * mt + g, tb = ta + 8;          // this lane's two token rows
  const int rr = 8 * nt + 2 * tq;                   // and its two state rows (rr, rr + 1)
  for (int j = 0; j < n_chunks; ++j) {
    const int t0 = cu0 + j * C, n = min(C, d.count - j * C);
    const float* lg = lgb[j & 1];
    cp_wait_groups();
    __syncthreads();
    // phase A
    float hw[4] = {0.f, 0.f, 0.f, 0.f}, qs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int k0 = 0; k0 < DK; k0 += 8) {
      const float aw[4] = {Ws[ta * PQ + k0 + tq], Ws[tb * PQ + k0 + tq], Ws[ta * PQ + k0 + tq + 4],
                           Ws[tb * PQ + k0 + tq + 4]};
      const float aq[4] = {Qs[ta * PQ + k0 + tq], Qs[tb * PQ + k0 + tq], Qs[ta * PQ + k0 + tq + 4],
                           Qs[tb * PQ + k0 + tq + 4]};
      const float b0 = S[(8 * nt + g) * PS + k0 + tq], b1 = S[(8 * nt + g) * PS + k0 + tq + 4];
      uint32_t wb[4], ws[4], qb[4], bb0, bs0, bb1, bs1;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        split_tf32(aw[k], wb[k], ws[k]);
        qb[k] = to_tf32(aq[k]);
      }
      split_tf32(b0, bb0, bs0);
      split_tf32(b1, bb1, bs1);
      mma_tf32(hw, ws, bb0, bb1);
      mma_tf32(hw, wb, bs0, bs1);
      mma_tf32(hw, wb, bb0, bb1);
      mma_tf32(qs, qb, bb0, bb1);
    }
    Hs[ta * PH + rr] = Us[ta * PH + rr] - hw[0];
    Hs[ta * PH + rr + 1] = Us[ta * PH + rr + 1] - hw[1];
    Hs[tb * PH + rr] = Us[tb * PH + rr] - hw[2];
    Hs[tb * PH + rr + 1] = Us[tb * PH + rr + 1] - hw[3];
    if (tid < C) {
      gs[tid] = expf(lg[tid]);
      fs[tid] = expf(lg[C - 1] - lg[tid]);
    }
    __syncthreads();  // H, decays ready; W, q, U free
    if (j + 1 < n_chunks) load_wqu(j + 1);
    // phase B: o = gamma_t qs + A h (A is zero above the diagonal)
    float o[4] = {gs[ta] * qs[0], gs[ta] * qs[1], gs[tb] * qs[2], gs[tb] * qs[3]};
    for (int i0 = 0; i0 <= 16 * mt + 8; i0 += 8) {
      const float aa[4] = {As[ta * PA + i0 + tq], As[tb * PA + i0 + tq], As[ta * PA + i0 + tq + 4],
                           As[tb * PA + i0 + tq + 4]};
      mma1_tf32(o, aa, Hs[(i0 + tq) * PH + 8 * nt + g], Hs[(i0 + tq + 4) * PH + 8 * nt + g]);
    }
    if (ta < n)
      *reinterpret_cast<float2*>(obuf + size_t(t0 + ta) * vd + head * DV + r0 + rr) = make_float2(o[0], o[1]);
    if (tb < n)
      *reinterpret_cast<float2*>(obuf + size_t(t0 + tb) * vd + head * DV + r0 + rr) = make_float2(o[2], o[3]);
    __syncthreads();  // A free
    if (j + 1 < n_chunks) load_a(j + 1);
    // phase C: S = gamma_C S + (f h)^T k, in place (each warp owns its tiles)
    const float gc = gs[C - 1];
#pragma unroll
    for (int u = 0; u < TPW; ++u) {
      const int tile = warp * TPW + u, mc = tile / NTC, nc = tile % NTC;
      const int ra = 16 * mc + g, rb2 = ra + 8, cc = 8 * nc + 2 * tq;
      const float2 s0 = *reinterpret_cast<const float2*>(S + ra * PS + cc);
      const float2 s1 = *reinterpret_cast<const float2*>(S + rb2 * PS + cc);
      float acc[4] = {gc * s0.x, gc * s0.y, gc * s1.x, gc * s1.y};
#pragma unroll 2
      for (int k0 = 0; k0 < C; k0 += 8) {
        const float f0 = fs[k0 + tq], f1 = fs[k0 + tq + 4];
        const float ah[4] = {f0 * Hs[(k0 + tq) * PH + ra], f0 * Hs[(k0 + tq) * PH + rb2],
                             f1 * Hs[(k0 + tq + 4) * PH + ra], f1 * Hs[(k0 + tq + 4) * PH + rb2]};
        mma3_tf32(acc, ah, Ks[(k0 + tq) * PK + 8 * nc + g], Ks[(k0 + tq + 4) * PK + 8 * nc + g]);
      }
      *reinterpret_cast<float2*>(S + ra * PS + cc) = make_float2(acc[0], acc[1]);
      *reinterpret_cast<float2*>(S + rb2 * PS + cc) = make_float2(acc[2], acc[3]);
    }
    __syncthreads();  // k rows and H free; S complete
    if (j + 1 < n_chunks) load_k(j + 1);
  }
  bool finite = true;
  for (int e = tid; e < kScanRows * DK; e += kScanThreads) {
    const int r = e / DK, c = e % DK;
    const float v = S[r * PS + c];
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
  pdl_wait(tokens, obuf, proj, gnorm, out);
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

// Token-parallel preparation of long runs: CTA = (16 tokens of a 64-token
// chunk, key head), one thread per channel of the key head (its q and k
// channels and its R value heads' v channels), gdn_prep's arithmetic per
// token: causal conv + SiLU and q / k RMS scaling; the decay and beta come
// from gdn_chunk_prep. Each thread runs its channel's conv over the block's
// tokens with the taps in registers and leaves the q / k activations in
// shared memory; after one barrier, warp w scales token w's q and k rows
// (the sums of squares formed per 32 channels by the same butterfly, then
// added in channel-group order, as gdn_prep does). A chunk starts from the
// K-1 inputs before it: earlier tokens of the run (their projection rows) or
// the parent's conv history. The child's history is written afterwards by
// gdn_conv_tail (a consumed parent's history is the child's, so it must not
// change while any chunk still reads it).
template <int DK, int DV, int R>
__global__ void __launch_bounds__(2 * DK + R * DV, 1)
    gdn_run_prep_kernel(const float* __restrict__ proj, int ld, int splits, size_t split_stride,
                        const SeqDesc* __restrict__ descs, const int32_t* __restrict__ cu_seqlens,
                        const int32_t* __restrict__ items, GdnPool pool, int li, int hk, int hv, int conv,
                        const float* __restrict__ conv_w, const float* __restrict__ a_log,
                        const float* __restrict__ dt_bias, float* __restrict__ qk_out, float* __restrict__ v_out,
                        float* __restrict__ gb_out) {
  pdl_trigger();
  pdl_wait(proj, descs, cu_seqlens, items, conv_w, a_log, dt_bias, qk_out, v_out, gb_out);
  constexpr int QW = DK / 32;
  constexpr int SUB = C / kRunBlock;
  constexpr int kThreads = 2 * DK + R * DV;
  __shared__ float acts[kRunBlock][2 * DK];  // q and k activations of the block's tokens
  const int item = blockIdx.x / SUB, kh = blockIdx.y;
  const int seq = items[2 * item], chunk = items[2 * item + 1];
  const SeqDesc d = descs[seq];
  const int s0 = cu_seqlens[seq], c0 = chunk * C + (blockIdx.x % SUB) * kRunBlock;
  const int n = min(kRunBlock, d.count - c0);
  if (n <= 0) return;
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
  // the block's inputs: each split's 16 partials requested together, added
  // in split order (split_sum_c's order)
  float cur_g[kRunBlock];
  const float* base = proj + size_t(s0 + c0) * ld + gc;
#pragma unroll
  for (int k = 0; k < kRunBlock; ++k) cur_g[k] = base[size_t(min(k, n - 1)) * ld];
  for (int sp = 1; sp < splits; ++sp) {
    float part[kRunBlock];
#pragma unroll
    for (int k = 0; k < kRunBlock; ++k) part[k] = base[sp * split_stride + size_t(min(k, n - 1)) * ld];
#pragma unroll
    for (int k = 0; k < kRunBlock; ++k) cur_g[k] += part[k];
  }
#pragma unroll
  for (int i = 0; i < kRunBlock; ++i) {
    if (i < n) {
      const float cur = cur_g[i];
      float acc = 0.f;
#pragma unroll
      for (int j = 0; j < 7; ++j)
        if (j < conv - 1) acc += taps[j] * cw[j];
      acc += cur * cw_last;
#pragma unroll
      for (int j = 0; j < 7; ++j)
        if (j < conv - 1) taps[j] = j + 1 < conv - 1 ? taps[j + 1] : cur;
      const float act = siluf_(acc);
      if (c >= 2 * DK) v_out[size_t(s0 + c0 + i) * vd + kh * R * DV + (c - 2 * DK)] = act;
      else acts[i][c] = act;
    }
  }
  __syncthreads();
  for (int i = warp; i < n; i += kThreads / 32) {
    float* dstq = qk_out + ((size_t(s0 + c0 + i) * hk + kh) * 2) * DK;
#pragma unroll
    for (int h = 0; h < 2; ++h) {  // q, then k
      float a[QW], tot = 0.f;
#pragma unroll
      for (int j = 0; j < QW; ++j) {
        a[j] = acts[i][h * DK + 32 * j + lane];
        tot += warp_sum(a[j] * a[j]);
      }
      const float rinv = rsqrtf(tot / DK + 1e-6f);
      const float scale = h == 0 ? rinv / DK : rinv * rsqrtf(float(DK));
#pragma unroll
      for (int j = 0; j < QW; ++j) dstq[h * DK + 32 * j + lane] = a[j] * scale;
    }
  }
}

// The child's conv history of each long run: its last conv-1 inputs.
__global__ void __launch_bounds__(256)
    gdn_conv_tail_kernel(const float* __restrict__ proj, int ld, int splits, size_t split_stride,
                         const SeqDesc* __restrict__ descs, const int32_t* __restrict__ cu_seqlens,
                         const int32_t* __restrict__ longs, GdnPool pool, int li, int conv, int cd) {
  pdl_trigger();
  pdl_wait(proj, descs, cu_seqlens, longs);
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
  constexpr size_t scan_smem = (2 * C * (DK + 4) + C * (DK + 8) + C * (C + 4) + kScanRows * (DK + 4) +
                                2 * C * (kScanRows + 8)) * sizeof(float);
  static_assert(prep_smem <= 227 * 1024 && scan_smem <= 227 * 1024, "chunked DeltaNet shared memory");
  static std::atomic<uint64_t> set{0};
  once_per_device(set, [] {
    QWEN_CUDA(cudaFuncSetAttribute(gdn_chunk_prep_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   int(prep_smem)));
    QWEN_CUDA(cudaFuncSetAttribute(gdn_chunk_scan_kernel<DK, DV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   int(scan_smem)));
  });
  launch_pdl(gdn_chunk_prep_kernel<DK, DV>, dim3(cp.n_items, d.hv), DK + DV, prep_smem, s, descs, cu_seqlens,
             cp.items, d.hk, d.hv, qk_buf, v_buf, proj, ld_proj, splits, split_stride, d.cd, ly.a_log, ly.dt_bias,
             cp.U, cp.W, cp.A, cp.LG);
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
    launch_pdl(kernel, dim3(cp.n_items * (C / kRunBlock), d.hk), threads, 0, s, proj, ld_proj, splits, split_stride,
               descs, cu_seqlens,
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
