// Gated-DeltaNet mixer (native/qwen_model.inc:154-206, native/operator_reference.h:19-45).
// Decode steps (one token per sequence) run gdn_decode_kernel, one kernel per
// layer that streams the state through a shared-memory ring (gdn_stream_kernel
// after gdn_prep for conv widths other than 4, described below). Steps that
// feed several tokens to a sequence (prefill, speculative verify) run two
// kernels per layer:
//
//  gdn_prep:   CTA = (sequence, key head). Causal depthwise conv1d (K taps,
//              tap 0 oldest) over [conv history; new qkv rows] + SiLU for the key
//              head's q/k channels and its value heads' v channels; q and k
//              RMS-normalised and scaled (q/dk, k/sqrt(dk)); decay
//              g = exp(-exp(A_log) * softplus(a + dt_bias)) and beta = sigmoid(b).
//              Each channel is owned by one thread, which reads the parent's
//              conv history before writing the child's, so the update is safe
//              in place (consumed parents).
//  gdn_update: CTA = (sequence, value head), 8 warps. The head's fp32 state
//              S[dv][dk] is staged in shared memory by four bulk copies (one
//              per two warps' rows, each completing its own mbarrier), so a
//              CTA holds 64 KiB of state without registers and three CTAs fit
//              per SM; warp w owns rows [w*dv/8, (w+1)*dv/8), lane l columns
//              [l*dk/32, ...). Per token S *= g; m = S k; delta = beta (v - m);
//              S += delta k^T; o = S q; rows go back to shared memory, or
//              straight to the child's slot after the last token; then the
//              gated RMSNorm y = rms(o) * w * silu(z) is written as fp16 (the out_proj input).
// The state read + write (2 x 64 KiB per head for dk = dv = 128) is the
// HBM traffic that bounds the layer.
#include <atomic>

#include "kernels.h"
#include "tcgen05.cuh"

namespace qwen {

extern std::atomic<uint64_t> g_kernel_launches;

namespace {

constexpr int kGdnMaxSplits = 8;

// Sum of the split-K partials at column `col` of one token's projection row,
// in split order; the loads are issued in independent batches of four.
__device__ __forceinline__ float split_sum(const float* pr, int col, int splits, size_t split_stride) {
  float v = pr[col];
  for (int s0 = 1; s0 < splits; s0 += 4) {
    float part[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) part[k] = s0 + k < splits ? pr[(s0 + k) * split_stride + col] : 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (s0 + k < splits) v += part[k];
  }
  return v;
}

template <int DK, int DV, int R>
__global__ void __launch_bounds__(2 * DK + R * DV, 2)
    gdn_prep_kernel(const float* __restrict__ proj, int ld, int splits, size_t split_stride,
                    const SeqDesc* __restrict__ descs, const int32_t* __restrict__ cu_seqlens, GdnPool pool, int li,
                    int hk, int hv, int conv, const float* __restrict__ conv_w, const float* __restrict__ a_log,
                    const float* __restrict__ dt_bias, float* __restrict__ qk_out, float* __restrict__ v_out,
                    float* __restrict__ gb_out, const int32_t* __restrict__ cand_slots, int skip_count) {
  pdl_trigger();
  pdl_wait(proj, descs, cu_seqlens, conv_w, a_log, dt_bias, qk_out, v_out, gb_out, cand_slots);
  {
    const SeqDesc dd = descs[blockIdx.x];
    if (dd.cand < 0 && dd.count >= skip_count) return;  // a long run: gdn_run_prep owns it
  }
  // q / k sums of squares: one partial per warp (4 warps each for dk = 128),
  // double-buffered by token parity so one barrier per token suffices
  constexpr int QW = DK / 32;  // warps holding q (and as many holding k)
  __shared__ float red[2][2 * QW];
  const int seq = blockIdx.x, kh = blockIdx.y;
  const SeqDesc d = descs[seq];
  const int t0 = cu_seqlens[seq];
  const int kd = hk * DK, vd = hv * DV, cd = 2 * kd + vd;
  const int c = threadIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gc = c < DK ? kh * DK + c : (c < 2 * DK ? kd + kh * DK + (c - DK) : 2 * kd + kh * R * DV + (c - 2 * DK));
  const size_t cl = size_t(conv - 1) * cd;
  const float* src_conv = d.parent >= 0 ? pool.conv + (size_t(d.parent) * pool.n_gdn + li) * cl : nullptr;
  float* dst_conv = pool.conv + (size_t(d.child) * pool.n_gdn + li) * cl;
  // taps[j] = input j+1 steps before the newest tap; indices stay static so
  // both arrays live in registers (conv <= 8).
  float taps[7], cw[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) cw[j] = j < conv ? conv_w[size_t(gc) * conv + j] : 0.f;
#pragma unroll
  for (int j = 0; j < 7; ++j) taps[j] = (j < conv - 1 && src_conv) ? src_conv[size_t(j) * cd + gc] : 0.f;
  float cw_last = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (j == conv - 1) cw_last = cw[j];
  auto P = [&](const float* pr, int col) { return split_sum(pr, col, splits, split_stride); };
  // decay / beta inputs of value head kh*R + c (threads c < R), requested
  // with the token's conv input rather than after the q / k barrier
  const int gh = kh * R + (c < R ? c : 0);
  const float gdt = c < R ? dt_bias[gh] : 0.f, galog = c < R ? a_log[gh] : 0.f;
  for (int i = 0; i < d.count; ++i) {
    const int t = t0 + i;
    const float* pr = proj + size_t(t) * ld;
    const float cur = P(pr, gc);
    const float ga = c < R ? P(pr, cd + vd + gh) : 0.f, gbeta = c < R ? P(pr, cd + vd + hv + gh) : 0.f;
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 7; ++j)
      if (j < conv - 1) acc += taps[j] * cw[j];
    acc += cur * cw_last;
#pragma unroll
    for (int j = 0; j < 7; ++j)
      if (j < conv - 1) taps[j] = j + 1 < conv - 1 ? taps[j + 1] : cur;
    if (d.cand >= 0) {  // verify step: the history after token i is candidate i's conv state
      float* cc = pool.conv + (size_t(cand_slots[d.cand + i]) * pool.n_gdn + li) * cl;
#pragma unroll
      for (int j = 0; j < 7; ++j)
        if (j < conv - 1) cc[size_t(j) * cd + gc] = taps[j];
    }
    const float act = siluf_(acc);
    if (c >= 2 * DK) {
      v_out[size_t(t) * vd + kh * R * DV + (c - 2 * DK)] = act;
    } else {
      // q / k: inverse RMS over the head (warp partials, fixed order), folded
      // with the 1/dk and 1/sqrt(dk) scales; only these 2*dk threads meet
      float ss = warp_sum(act * act);
      if (lane == 0) red[i & 1][warp] = ss;
      asm volatile("bar.sync 1, %0;" ::"r"(2 * DK) : "memory");
      const int g0 = c < DK ? 0 : QW;
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < QW; ++w) tot += red[i & 1][g0 + w];
      const float rinv = rsqrtf(tot / DK + 1e-6f);
      float* dst = qk_out + ((size_t(t) * hk + kh) * 2) * DK;
      if (c < DK) dst[c] = act * (rinv / DK);
      else dst[DK + (c - DK)] = act * (rinv * rsqrtf(float(DK)));
    }
    if (c < R) {
      const float av = ga + gdt;
      const float sp = fmaxf(av, 0.f) + log1pf(__expf(-fabsf(av)));
      gb_out[(size_t(t) * hv + gh) * 2 + 0] = expf(-expf(galog) * sp);
      gb_out[(size_t(t) * hv + gh) * 2 + 1] = sigmoidf_(gbeta);
    }
  }
  if (d.cand < 0) {
#pragma unroll
    for (int j = 0; j < 7; ++j)
      if (j < conv - 1) dst_conv[size_t(j) * cd + gc] = taps[j];
  }
}

template <int DK, int DV>
__global__ void __launch_bounds__(256, 3)
    gdn_update_kernel(const SeqDesc* __restrict__ descs, const int32_t* __restrict__ cu_seqlens, GdnPool pool, int li,
                      int hk, int hv, const float* __restrict__ qk, const float* __restrict__ vv,
                      const float* __restrict__ gb, const float* __restrict__ proj, int ld, int splits,
                      size_t split_stride, int cd, const float* __restrict__ gnorm, float eps,
                      gemm_in_t* __restrict__ out, uint32_t* err, const int32_t* __restrict__ cand_slots,
                      int skip_count) {
  pdl_trigger();
  pdl_wait(descs, cu_seqlens, qk, vv, gb, proj, gnorm, out, cand_slots);
  constexpr int CPL = DK / 32;  // columns per lane (4 or 2)
  constexpr int RPW = DV / 8;   // rows per warp
  {
    const SeqDesc dd = descs[blockIdx.x];
    if (dd.cand < 0 && dd.count >= skip_count) return;  // a long run: the chunked kernels own it
  }
  constexpr int CROWS = 2 * RPW;  // rows per bulk copy: two warps' rows
  constexpr int CHUNKS = DV / CROWS;
  constexpr uint32_t CBYTES = CROWS * DK * 4;
  using Vec = typename std::conditional<CPL == 4, float4, float2>::type;
  extern __shared__ __align__(128) float st[];  // the head's state S[dv][dk]
  __shared__ uint64_t full[CHUNKS];
  __shared__ float os[DV];
  __shared__ float red[8];
  __shared__ int abort_flag;
  const int seq = blockIdx.x, head = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const SeqDesc d = descs[seq];
  const int t0 = cu_seqlens[seq];
  const int kh = head / (hv / hk);
  const int vd = hv * DV;
  const size_t sl = size_t(hv) * DV * DK;
  const float* src = d.parent >= 0 ? pool.state + (size_t(d.parent) * pool.n_gdn + li) * sl + size_t(head) * DV * DK
                                   : nullptr;
  float* dst = pool.state + (size_t(d.child) * pool.n_gdn + li) * sl + size_t(head) * DV * DK;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    if (src) {
#pragma unroll
      for (int c = 0; c < CHUNKS; ++c) mbar_init(&full[c], 1);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
#pragma unroll
      for (int c = 0; c < CHUNKS; ++c) {
        mbar_expect_tx(&full[c], CBYTES);
        bulk_load(st + c * CROWS * DK, src + c * CROWS * DK, CBYTES, &full[c]);
      }
    }
  }
  if (!src)
    for (int i = threadIdx.x; i < DV * DK / 4; i += blockDim.x) reinterpret_cast<float4*>(st)[i] = float4{0.f, 0.f, 0.f, 0.f};
  const float gw = threadIdx.x < DV ? gnorm[threadIdx.x] : 0.f;
  __syncthreads();
  bool ready = src == nullptr;  // this warp's rows are in shared memory
  bool finite = true;
  for (int it = 0; it < d.count; ++it) {
    const int t = t0 + it;
    // the gate input z of this thread's output channel, requested with the
    // token's other inputs instead of after the row barrier
    const float z = threadIdx.x < DV ? split_sum(proj + size_t(t) * ld, cd + head * DV + threadIdx.x, splits,
                                                 split_stride)
                                     : 0.f;
    const float* qkt = qk + ((size_t(t) * hk + kh) * 2) * DK;
    float qq[CPL], kq[CPL];
    {
      const Vec qv = *reinterpret_cast<const Vec*>(qkt + lane * CPL);
      const Vec kv = *reinterpret_cast<const Vec*>(qkt + DK + lane * CPL);
#pragma unroll
      for (int j = 0; j < CPL; ++j) {
        qq[j] = reinterpret_cast<const float*>(&qv)[j];
        kq[j] = reinterpret_cast<const float*>(&kv)[j];
      }
    }
    const float g = gb[(size_t(t) * hv + head) * 2], beta = gb[(size_t(t) * hv + head) * 2 + 1];
    const float* vt = vv + size_t(t) * vd + head * DV;
    if (!ready) {
      mbar_wait(&full[warp * RPW / CROWS], 0, &abort_flag, err);
      ready = true;
    }
    const bool last = it + 1 == d.count;
    float* cs = d.cand >= 0 ? pool.state + (size_t(cand_slots[d.cand + it]) * pool.n_gdn + li) * sl +
                                  size_t(head) * DV * DK
                            : nullptr;
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const int r = warp * RPW + i;
      Vec row = *reinterpret_cast<const Vec*>(st + r * DK + lane * CPL);
      float* S = reinterpret_cast<float*>(&row);
      float mem = 0.f;
#pragma unroll
      for (int j = 0; j < CPL; ++j) {
        S[j] *= g;
        mem += S[j] * kq[j];
      }
      mem = warp_sum(mem);
      const float delta = (vt[r] - mem) * beta;
      float rd = 0.f;
#pragma unroll
      for (int j = 0; j < CPL; ++j) {
        S[j] += delta * kq[j];
        rd += S[j] * qq[j];
      }
      rd = warp_sum(rd);
      if (lane == 0) os[r] = rd;
      // verify step: the state after this token is candidate `it`'s state
      if (cs) *reinterpret_cast<Vec*>(cs + size_t(r) * DK + lane * CPL) = row;
      if (last) {
#pragma unroll
        for (int j = 0; j < CPL; ++j) finite &= isfinite(S[j]);
        if (d.cand < 0) *reinterpret_cast<Vec*>(dst + size_t(r) * DK + lane * CPL) = row;
      } else {
        *reinterpret_cast<Vec*>(st + r * DK + lane * CPL) = row;
      }
    }
    __syncthreads();
    // gated RMSNorm over dv (native/qwen_model.inc:203-204)
    float o = threadIdx.x < DV ? os[threadIdx.x] : 0.f;
    float ss = warp_sum(o * o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    if (threadIdx.x < DV) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) tot += red[w];
      const float y = o * rsqrtf(tot / DV + eps) * gw * siluf_(z);
      out[size_t(t) * vd + head * DV + threadIdx.x] = to_gemm_in(y);
    }
  }
  if (d.count == 0) {  // no token: the child carries the parent's state
    if (!ready) mbar_wait(&full[warp * RPW / CROWS], 0, &abort_flag, err);
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      const int r = warp * RPW + i;
      const Vec row = *reinterpret_cast<const Vec*>(st + r * DK + lane * CPL);
      const float* S = reinterpret_cast<const float*>(&row);
#pragma unroll
      for (int j = 0; j < CPL; ++j) finite &= isfinite(S[j]);
      if (d.cand < 0) *reinterpret_cast<Vec*>(dst + size_t(r) * DK + lane * CPL) = row;
    }
  }
  if (!finite) atomicOr(err, kErrNonFinite);
  // after a timed-out wait, copies may still be landing: wait for them (bounded) before exiting
  __syncthreads();
  if (threadIdx.x == 0 && src && abort_flag) {
#pragma unroll 1
    for (int c = 0; c < CHUNKS; ++c) {
      const long long c0 = clock64();
      while (!mbar_try_sleep(&full[c], 0, kWaitSleepNs) && clock64() - c0 < kWaitCycles) {
      }
    }
  }
}


// Decode steps (every sequence feeds one token): the update streamed through a
// ring of shared-memory row chunks by persistent CTAs. The rows of a head's
// state are independent (the token's k, v, g, beta update a row from that row
// alone; only the gated RMSNorm spans rows), so a row is read once, updated,
// written straight to the child's slot, and its chunk slot refilled at once
// with the next rows, whichever head they belong to: HBM sees one continuous
// read stream per CTA instead of a load / compute / store wave per head.
//   warp 8 (producer): per item (sequence, value head) stages the token inputs
//     (q, k, v, the gate input z summed over the split-K partials, g, beta, the
//     output row and the destination) in one of two shared buffers, then
//     issues one bulk copy per 32-row chunk into the NS-slot ring;
//   warps 0-7 (consumers): 4 rows of every chunk each, then the gated RMSNorm
//     of the item over named barrier 1.
// Every wait is bounded; after a timeout (kErrTimeout) all warps run out their
// loops with no memory traffic and the same barrier count, and the producer's
// outstanding copies are waited for (bounded) before the CTA exits.
template <int DK, int DV>
__global__ void __launch_bounds__(288, 3)
    gdn_stream_kernel(const SeqDesc* __restrict__ descs, const int32_t* __restrict__ cu_seqlens, GdnPool pool, int li,
                      int hk, int hv, int n_items, const float* __restrict__ qk, const float* __restrict__ vv,
                      const float* __restrict__ gb, const float* __restrict__ proj, int ld, int splits,
                      size_t split_stride, int cd, const float* __restrict__ gnorm, float eps,
                      gemm_in_t* __restrict__ out, uint32_t* err, const int32_t* __restrict__ cand_slots) {
  pdl_trigger();
  pdl_wait(descs, cu_seqlens, qk, vv, gb, proj, gnorm, out, cand_slots);
  constexpr int CPL = DK / 32;   // state columns per lane
  constexpr int CR = 32;         // rows per chunk: 4 per consumer warp
  constexpr int CPI = DV / CR;   // chunks per item
  constexpr int NS = 4;          // ring slots
  constexpr uint32_t CBYTES = CR * DK * 4;
  using Vec = typename std::conditional<CPL == 4, float4, float2>::type;
  struct __align__(16) Stage {
    float qk[2 * DK];
    float v[DV];
    float z[DV];
    float* dst;
    float g, beta;
    int t;
  };
  extern __shared__ __align__(128) float ring[];  // [NS][CR][DK]
  __shared__ Stage stg[2];
  __shared__ uint64_t full[NS], empty[NS], in_full[2], in_empty[2];
  __shared__ float os[DV];
  __shared__ float red[8];
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    abort_flag = 0;
#pragma unroll
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 8);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(&in_full[i], 32);
      mbar_init(&in_empty[i], 8);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int vd = hv * DV;
  const size_t sl = size_t(hv) * DV * DK;
  int issued = 0;  // producer: chunks issued
  if (warp == 8) {
    int n = 0, j = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x, ++j) {
      const int seq = i / hv, head = i % hv, kh = head / (hv / hk);
      const SeqDesc d = descs[seq];
      const int t = cu_seqlens[seq];
      const int b = j & 1;
      if (!mbar_wait(&in_empty[b], ((j >> 1) & 1) ^ 1u, &abort_flag, err)) break;
      Stage& S = stg[b];
      const float* qkt = qk + ((size_t(t) * hk + kh) * 2) * DK;
      const float* vt = vv + size_t(t) * vd + size_t(head) * DV;
#pragma unroll
      for (int c = lane; c < 2 * DK; c += 32) S.qk[c] = qkt[c];
#pragma unroll
      for (int c = lane; c < DV; c += 32) {
        S.v[c] = vt[c];
        S.z[c] = split_sum(proj + size_t(t) * ld, cd + head * DV + c, splits, split_stride);
      }
      if (lane == 0) {
        S.g = gb[(size_t(t) * hv + head) * 2];
        S.beta = gb[(size_t(t) * hv + head) * 2 + 1];
        S.t = t;
        const int slot = d.cand >= 0 ? cand_slots[d.cand] : d.child;  // one token: its state is the result
        S.dst = pool.state + (size_t(slot) * pool.n_gdn + li) * sl + size_t(head) * DV * DK;
      }
      mbar_arrive(&in_full[b]);
      const float* src = d.parent >= 0 ? pool.state + (size_t(d.parent) * pool.n_gdn + li) * sl +
                                             size_t(head) * DV * DK
                                       : nullptr;
#pragma unroll 1
      for (int c = 0; c < CPI; ++c, ++n) {
        const int s = n % NS;
        if (!mbar_wait(&empty[s], ((n / NS) & 1) ^ 1u, &abort_flag, err)) {
          ok = false;
          break;
        }
        float* slot = ring + s * CR * DK;
        if (src) {
          if (lane == 0) {
            mbar_expect_tx(&full[s], CBYTES);
            bulk_load(slot, src + size_t(c) * CR * DK, CBYTES, &full[s]);
          }
          issued = n + 1;
        } else {  // no parent: zero state
          for (int k = lane; k < CR * DK / 4; k += 32) reinterpret_cast<float4*>(slot)[k] = float4{0.f, 0.f, 0.f, 0.f};
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[s]);
        }
      }
    }
  } else {
    const float gw = threadIdx.x < DV ? gnorm[threadIdx.x] : 0.f;
    bool finite = true;
    int n = 0, j = 0;
    for (int i = blockIdx.x; i < n_items; i += gridDim.x, ++j) {
      const int head = i % hv;
      const int b = j & 1;
      bool ok = mbar_wait(&in_full[b], (j >> 1) & 1u, &abort_flag, err);
      const Stage& S = stg[b];
      float qq[CPL], kq[CPL];
      {
        const Vec qv = *reinterpret_cast<const Vec*>(S.qk + lane * CPL);
        const Vec kv = *reinterpret_cast<const Vec*>(S.qk + DK + lane * CPL);
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
          qq[c] = reinterpret_cast<const float*>(&qv)[c];
          kq[c] = reinterpret_cast<const float*>(&kv)[c];
        }
      }
      const float g = S.g, beta = S.beta;
      float* dst = S.dst;
#pragma unroll 1
      for (int c = 0; c < CPI; ++c, ++n) {
        const int s = n % NS;
        ok = mbar_wait(&full[s], (n / NS) & 1u, &abort_flag, err) && ok;
        const float* chunk = ring + s * CR * DK;
#pragma unroll
        for (int k = 0; k < CR / 8; ++k) {
          const int rl = warp * (CR / 8) + k, r = c * CR + rl;
          Vec row = *reinterpret_cast<const Vec*>(chunk + rl * DK + lane * CPL);
          float* St = reinterpret_cast<float*>(&row);
          float mem = 0.f;
#pragma unroll
          for (int q = 0; q < CPL; ++q) {
            St[q] *= g;
            mem += St[q] * kq[q];
          }
          mem = warp_sum(mem);
          const float delta = (S.v[r] - mem) * beta;
          float rd = 0.f;
#pragma unroll
          for (int q = 0; q < CPL; ++q) {
            St[q] += delta * kq[q];
            rd += St[q] * qq[q];
          }
          rd = warp_sum(rd);
          if (lane == 0) os[r] = rd;
#pragma unroll
          for (int q = 0; q < CPL; ++q) finite &= isfinite(St[q]);
          if (ok) *reinterpret_cast<Vec*>(dst + size_t(r) * DK + lane * CPL) = row;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      // gated RMSNorm over dv (native/qwen_model.inc:203-204)
      asm volatile("bar.sync 1, 256;" ::: "memory");
      const float o = threadIdx.x < DV ? os[threadIdx.x] : 0.f;
      const float z = threadIdx.x < DV ? S.z[threadIdx.x] : 0.f;
      const int t = S.t;
      const float ss = warp_sum(o * o);
      if (lane == 0) red[warp] = ss;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (threadIdx.x < DV && ok) {
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) tot += red[w];
        const float y = o * rsqrtf(tot / DV + eps) * gw * siluf_(z);
        out[size_t(t) * vd + head * DV + threadIdx.x] = to_gemm_in(y);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&in_empty[b]);
    }
    if (!finite) atomicOr(err, kErrNonFinite);
  }
  __syncthreads();
  // after a timeout, copies may still be landing in the ring: wait for them (bounded)
  if (warp == 8 && lane == 0 && abort_flag) {
#pragma unroll 1
    for (int n = issued > NS ? issued - NS : 0; n < issued; ++n) {
      const long long c0 = clock64();
      while (!mbar_try_sleep(&full[n % NS], (n / NS) & 1u, kWaitSleepNs) && clock64() - c0 < kWaitCycles) {
      }
    }
  }
}


// Decode steps with the 4-tap conv: gdn_prep folded into the streamed update.
// Item = (sequence, key head): the conv of its q / k channels and of its R
// value heads' v channels, then the R heads' state rows. Persistent CTAs
// (kDecCtasPerSm per SM) with three warp roles:
//   consumers (the first kDecConsumerWarps warps): their share of the rows of
//     every chunk, then the R gated RMSNorms over named barrier 1;
//   issuer (the next warp): one bulk copy per 32-row chunk of the item's R
//     heads (contiguous in the slot) into a kDecRing-slot ring, running ahead
//     of the consumers by the ring's depth, across items;
//   stagers (the last kDecStagerWarps warps): for the next item, the causal
//     conv + SiLU of its 2*DK + R*DV channels with gdn_prep's arithmetic (the
//     new history written to the destination slot), q / k RMS scaling from the
//     same per-32-channel partials in the same order, g, beta and the
//     split-summed gate input z, into one of two stage buffers.
// The item's history and state are read and written by this CTA only, so a
// consumed parent is updated in place. Timeouts behave as in gdn_stream_kernel.
// Warp roles and ring depth of gdn_decode_kernel.
constexpr int kDecConsumerWarps = 8;
constexpr int kDecStagerWarps = 4;
constexpr int kDecRing = 6;          // 32-row chunks in the ring
constexpr int kDecCtasPerSm = 2;
constexpr int kDecThreads = (kDecConsumerWarps + 1 + kDecStagerWarps) * 32;

template <int DK, int DV, int R, int CONV>
__global__ void __launch_bounds__(kDecThreads, kDecCtasPerSm)
    gdn_decode_kernel(const float* __restrict__ proj, int ld, int splits, size_t split_stride,
                      const SeqDesc* __restrict__ descs, const int32_t* __restrict__ cu_seqlens, GdnPool pool, int li,
                      int hk, int hv, int n_items, const float* __restrict__ conv_w, const float* __restrict__ a_log,
                      const float* __restrict__ dt_bias, const float* __restrict__ gnorm, float eps,
                      gemm_in_t* __restrict__ out, uint32_t* err, const int32_t* __restrict__ cand_slots) {
  pdl_trigger();
  pdl_wait(proj, descs, cu_seqlens, conv_w, a_log, dt_bias, gnorm, out, cand_slots);
  constexpr int CPL = DK / 32;      // state columns per lane
  constexpr int NCW = kDecConsumerWarps, IW = NCW, SW0 = NCW + 1;  // consumer / issuer / first stager warp
  constexpr int CR = 32;            // rows per chunk
  constexpr int RPC = CR / NCW;     // rows of a chunk per consumer warp
  constexpr int HC = DV / CR;       // chunks per value head
  constexpr int IC = R * HC;        // chunks per item
  constexpr int NS = kDecRing;      // ring slots
  constexpr uint32_t CBYTES = CR * DK * 4;
  constexpr int NCH = 2 * DK + R * DV;  // conv channels per item: q | k | v
  constexpr int NP = kDecStagerWarps * 32;  // stager threads
  constexpr int NM = (NCH + NP - 1) / NP;
  constexpr int QW = DK / 32;
  using Vec = typename std::conditional<CPL == 4, float4, float2>::type;
  struct __align__(16) Stage {
    float qk[2 * DK];  // normalised and scaled q | k
    float v[R * DV];
    float z[R * DV];
    float g[R], beta[R];
    float* dst;        // the item's first value head in the destination slot
    int t;
  };
  extern __shared__ __align__(128) float ring[];  // [NS][CR][DK]
  __shared__ Stage stg[2];
  __shared__ uint64_t full[NS], empty[NS], in_full[2], in_empty[2];
  __shared__ float os[R * DV];
  __shared__ float red[R * DV / 32];
  __shared__ float pqk[2][2 * QW];
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    abort_flag = 0;
#pragma unroll
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NCW);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(&in_full[i], NP);
      mbar_init(&in_empty[i], NCW);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int kd = hk * DK, vd = hv * DV, cd = 2 * kd + vd;
  const size_t sl = size_t(hv) * DV * DK;
  const size_t cl = size_t(CONV - 1) * cd;
  int issued = 0;  // issuer: chunks issued
  if (warp == IW) {
    int n = 0;
    bool ok = true;
    for (int i = blockIdx.x; i < n_items && ok; i += gridDim.x) {
      const int seq = i / hk, kh = i % hk;
      const SeqDesc d = descs[seq];
      const float* src = d.parent >= 0 ? pool.state + (size_t(d.parent) * pool.n_gdn + li) * sl +
                                             size_t(kh) * R * DV * DK
                                       : nullptr;
#pragma unroll 1
      for (int c = 0; c < IC; ++c, ++n) {
        const int s = n % NS;
        if (!mbar_wait(&empty[s], ((n / NS) & 1) ^ 1u, &abort_flag, err)) {
          ok = false;
          break;
        }
        float* slot = ring + s * CR * DK;
        if (src) {
          if (lane == 0) {
            mbar_expect_tx(&full[s], CBYTES);
            bulk_load(slot, src + size_t(c) * CR * DK, CBYTES, &full[s]);
          }
          issued = n + 1;
        } else {  // no parent: zero state
          for (int k = lane; k < CR * DK / 4; k += 32) reinterpret_cast<float4*>(slot)[k] = float4{0.f, 0.f, 0.f, 0.f};
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[s]);
        }
      }
    }
  } else if (warp >= SW0) {
    const int p = threadIdx.x - SW0 * 32, pw = p >> 5;
    int j = 0;
    for (int i = blockIdx.x; i < n_items; i += gridDim.x, ++j) {
      const int seq = i / hk, kh = i % hk, b = j & 1;
      const bool ok = mbar_wait(&in_empty[b], ((j >> 1) & 1) ^ 1u, &abort_flag, err);
      const SeqDesc d = descs[seq];
      const int t = cu_seqlens[seq];
      const float* pr = proj + size_t(t) * ld;
      const float* src_conv = d.parent >= 0 ? pool.conv + (size_t(d.parent) * pool.n_gdn + li) * cl : nullptr;
      const int wslot = d.cand >= 0 ? cand_slots[d.cand] : d.child;  // one token: its state is the result
      float* dst_conv = pool.conv + (size_t(wslot) * pool.n_gdn + li) * cl;
      Stage& S = stg[b];
      // every input of the thread's channels is requested before the first
      // history store (the stores could alias later loads)
      int gc[NM];
      float cw[NM][CONV], taps[NM][CONV - 1], cur[NM];  // taps[m][0] oldest
#pragma unroll
      for (int m = 0; m < NM; ++m) {
        const int ch = p + NP * m;
        gc[m] = ch < DK ? kh * DK + ch
                        : (ch < 2 * DK ? kd + kh * DK + (ch - DK) : 2 * kd + kh * R * DV + (ch - 2 * DK));
        const bool v = ch < NCH;
#pragma unroll
        for (int q = 0; q < CONV; ++q) cw[m][q] = v ? conv_w[size_t(gc[m]) * CONV + q] : 0.f;
#pragma unroll
        for (int q = 0; q < CONV - 1; ++q) taps[m][q] = v && src_conv ? src_conv[size_t(q) * cd + gc[m]] : 0.f;
        cur[m] = v ? split_sum(pr, gc[m], splits, split_stride) : 0.f;
      }
      float act[NM];
#pragma unroll
      for (int m = 0; m < NM; ++m) {
        float acc = 0.f;
#pragma unroll
        for (int q = 0; q < CONV - 1; ++q) acc += taps[m][q] * cw[m][q];
        acc += cur[m] * cw[m][CONV - 1];
        if (ok && p + NP * m < NCH) {
#pragma unroll
          for (int q = 0; q < CONV - 1; ++q)
            dst_conv[size_t(q) * cd + gc[m]] = q + 1 < CONV - 1 ? taps[m][q + 1] : cur[m];
        }
        act[m] = siluf_(acc);
      }
      // q / k sums of squares: one partial per 32 channels, as gdn_prep's warps
#pragma unroll
      for (int m = 0; m < NM; ++m) {
        const int ch0 = NP * m + pw * 32;  // warp-uniform
        if (ch0 < 2 * DK) {
          const float ss = warp_sum(act[m] * act[m]);
          if (lane == 0) pqk[b][ch0 / 32] = ss;
        }
      }
#pragma unroll
      for (int m = 0; m < NM; ++m) {
        const int ch = p + NP * m;
        if (ch >= 2 * DK && ch < NCH) S.v[ch - 2 * DK] = act[m];
      }
      for (int c = p; c < R * DV; c += NP) S.z[c] = split_sum(pr, cd + kh * R * DV + c, splits, split_stride);
      if (p < R) {
        const int h = kh * R + p;
        const float av = split_sum(pr, cd + vd + h, splits, split_stride) + dt_bias[h];
        const float sp = fmaxf(av, 0.f) + log1pf(__expf(-fabsf(av)));
        S.g[p] = expf(-expf(a_log[h]) * sp);
        S.beta[p] = sigmoidf_(split_sum(pr, cd + vd + hv + h, splits, split_stride));
      }
      if (p == 0) {
        S.t = t;
        S.dst = pool.state + (size_t(wslot) * pool.n_gdn + li) * sl + size_t(kh) * R * DV * DK;
      }
      asm volatile("bar.sync 2, %0;" ::"n"(NP) : "memory");
      float tq = 0.f, tk = 0.f;
#pragma unroll
      for (int w = 0; w < QW; ++w) {
        tq += pqk[b][w];
        tk += pqk[b][QW + w];
      }
      const float rq = rsqrtf(tq / DK + 1e-6f), rk = rsqrtf(tk / DK + 1e-6f);
#pragma unroll
      for (int m = 0; m < NM; ++m) {
        const int ch = p + NP * m;
        if (ch < DK) S.qk[ch] = act[m] * (rq / DK);
        else if (ch < 2 * DK) S.qk[ch] = act[m] * (rk * rsqrtf(float(DK)));
      }
      mbar_arrive(&in_full[b]);
    }
  } else {
    const int tid = threadIdx.x;
    constexpr int NO = (R * DV + NCW * 32 - 1) / (NCW * 32);  // norm channels per consumer thread
    float gw[NO];
#pragma unroll
    for (int u = 0; u < NO; ++u) gw[u] = tid + u * NCW * 32 < R * DV ? gnorm[(tid + u * NCW * 32) % DV] : 0.f;
    bool finite = true;
    int n = 0, j = 0;
    for (int i = blockIdx.x; i < n_items; i += gridDim.x, ++j) {
      const int kh = i % hk, b = j & 1;
      bool ok = mbar_wait(&in_full[b], (j >> 1) & 1u, &abort_flag, err);
      const Stage& S = stg[b];
      float qq[CPL], kq[CPL];
      {
        const Vec qv = *reinterpret_cast<const Vec*>(S.qk + lane * CPL);
        const Vec kv = *reinterpret_cast<const Vec*>(S.qk + DK + lane * CPL);
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
          qq[c] = reinterpret_cast<const float*>(&qv)[c];
          kq[c] = reinterpret_cast<const float*>(&kv)[c];
        }
      }
      float* dst = S.dst;
#pragma unroll 1
      for (int c = 0; c < IC; ++c, ++n) {
        const int s = n % NS, hh = c / HC;
        ok = mbar_wait(&full[s], (n / NS) & 1u, &abort_flag, err) && ok;
        const float g = S.g[hh], beta = S.beta[hh];
        const float* chunk = ring + s * CR * DK;
#pragma unroll
        for (int k = 0; k < RPC; ++k) {
          const int rl = warp * RPC + k, r = (c % HC) * CR + rl;
          Vec row = *reinterpret_cast<const Vec*>(chunk + rl * DK + lane * CPL);
          float* St = reinterpret_cast<float*>(&row);
          float mem = 0.f;
#pragma unroll
          for (int q = 0; q < CPL; ++q) {
            St[q] *= g;
            mem += St[q] * kq[q];
          }
          mem = warp_sum(mem);
          const float delta = (S.v[hh * DV + r] - mem) * beta;
          float rd = 0.f;
#pragma unroll
          for (int q = 0; q < CPL; ++q) {
            St[q] += delta * kq[q];
            rd += St[q] * qq[q];
          }
          rd = warp_sum(rd);
          if (lane == 0) os[hh * DV + r] = rd;
#pragma unroll
          for (int q = 0; q < CPL; ++q) finite &= isfinite(St[q]);
          if (ok) *reinterpret_cast<Vec*>(dst + (size_t(hh) * DV + r) * DK + lane * CPL) = row;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      // the R gated RMSNorms over dv (native/qwen_model.inc:203-204); red[g]
      // holds the sum of squares of channels [32g, 32g + 32)
      asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
      float o[NO], z[NO];
#pragma unroll
      for (int u = 0; u < NO; ++u) {
        const int ch = tid + u * NCW * 32;
        o[u] = ch < R * DV ? os[ch] : 0.f;
        z[u] = ch < R * DV ? S.z[ch] : 0.f;
        const float ss = warp_sum(o[u] * o[u]);
        if (lane == 0 && ch < R * DV) red[ch / 32] = ss;
      }
      const int t = S.t;
      asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
#pragma unroll
      for (int u = 0; u < NO; ++u) {
        const int ch = tid + u * NCW * 32;
        if (ch < R * DV && ok) {
          const int hh = ch / DV;
          float tot = 0.f;
#pragma unroll
          for (int w = 0; w < DV / 32; ++w) tot += red[hh * (DV / 32) + w];
          const float y = o[u] * rsqrtf(tot / DV + eps) * gw[u] * siluf_(z[u]);
          out[size_t(t) * vd + size_t(kh) * R * DV + ch] = to_gemm_in(y);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&in_empty[b]);
    }
    if (!finite) atomicOr(err, kErrNonFinite);
  }
  __syncthreads();
  // after a timeout, copies may still be landing in the ring: wait for them (bounded)
  if (warp == IW && lane == 0 && abort_flag) {
#pragma unroll 1
    for (int n = issued > NS ? issued - NS : 0; n < issued; ++n) {
      const long long c0 = clock64();
      while (!mbar_try_sleep(&full[n % NS], (n / NS) & 1u, kWaitSleepNs) && clock64() - c0 < kWaitCycles) {
      }
    }
  }
}

}  // namespace

void launch_gdn(const Dims& d, const LayerDev& ly, const float* proj, int ld_proj, int splits, size_t split_stride,
                const SeqDesc* descs, const int32_t* cu_seqlens, int n_seq, int T, GdnPool pool, int gdn_index,
                gemm_in_t* out, uint32_t* err, float* qk_buf, float* v_buf, float* gb_buf, int sm_count,
                const int32_t* cand_slots, cudaStream_t s, const GdnChunkPlan* chunked) {
  const bool use_chunks = chunked && chunked->n_long > 0 && T != n_seq;
  const int skip_count = use_chunks ? kGdnChunkMin : 0x7fffffff;
  const int R = d.hv / d.hk;
  if (d.conv > 8) throw std::invalid_argument("conv kernel width > 8 unsupported");
  if (splits > kGdnMaxSplits) throw std::invalid_argument("DeltaNet input projection split more than 8 ways");
  bool done = false;
#define QWEN_GDN_DECODE(DK_, DV_, R_)                                                                             \
  if (!done && T == n_seq && d.conv == 4 && d.dk == DK_ && d.dv == DV_ && R == R_) {                             \
    constexpr int ring_bytes = kDecRing * 32 * DK_ * 4;                                                                 \
    static std::atomic<uint64_t> set_##DK_##_##R_{0};                                                            \
    once_per_device(set_##DK_##_##R_, [] {                                                                       \
      QWEN_CUDA(cudaFuncSetAttribute(gdn_decode_kernel<DK_, DV_, R_, 4>,                                         \
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, ring_bytes));                  \
      QWEN_CUDA(cudaFuncSetAttribute(gdn_decode_kernel<DK_, DV_, R_, 4>,                                         \
                                     cudaFuncAttributePreferredSharedMemoryCarveout,                             \
                                     int(cudaSharedmemCarveoutMaxShared)));                                     \
    });                                                                                                          \
    const int items = n_seq * d.hk;                                                                              \
    const int per_cta = (items + kDecCtasPerSm * sm_count - 1) / (kDecCtasPerSm * sm_count);                                             \
    launch_pdl(gdn_decode_kernel<DK_, DV_, R_, 4>, (items + per_cta - 1) / per_cta, kDecThreads, size_t(ring_bytes), s,   \
               proj, ld_proj, splits, split_stride, descs, cu_seqlens, pool, gdn_index, d.hk, d.hv, items,       \
               ly.conv_w, ly.a_log, ly.dt_bias, ly.gnorm, d.eps, out, err, cand_slots);                           \
    QWEN_CUDA(cudaGetLastError());                                                                               \
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);                                                   \
    return;                                                                                                      \
  }
  QWEN_GDN_DECODE(128, 128, 2)
  QWEN_GDN_DECODE(64, 64, 2)
  QWEN_GDN_DECODE(128, 128, 1)
  QWEN_GDN_DECODE(64, 64, 1)
#undef QWEN_GDN_DECODE
#define QWEN_GDN(DK_, DV_, R_)                                                                                    \
  if (!done && d.dk == DK_ && d.dv == DV_ && R == R_) {                                                          \
    launch_pdl(gdn_prep_kernel<DK_, DV_, R_>, dim3(n_seq, d.hk), 2 * DK_ + R_ * DV_, 0, s,                               \
        proj, ld_proj, splits, split_stride, descs, cu_seqlens, pool, gdn_index, d.hk, d.hv, d.conv, ly.conv_w,  \
        ly.a_log, ly.dt_bias, qk_buf, v_buf, gb_buf, cand_slots, use_chunks ? kGdnChunkMin : 0x7fffffff);        \
    if (use_chunks)                                                                                              \
      launch_gdn_run_prep(*chunked, d, ly, proj, ld_proj, splits, split_stride, descs, cu_seqlens, pool,         \
                          gdn_index, qk_buf, v_buf, gb_buf, s);                                                  \
    static std::atomic<uint64_t> smem_set_##DK_##_##R_{0};                                                       \
    once_per_device(smem_set_##DK_##_##R_, [] {                                                                  \
      const int bytes = DV_ * DK_ * 4;                                                                           \
      QWEN_CUDA(cudaFuncSetAttribute(gdn_update_kernel<DK_, DV_>, cudaFuncAttributeMaxDynamicSharedMemorySize,   \
                                     bytes));                                                                    \
      QWEN_CUDA(cudaFuncSetAttribute(gdn_update_kernel<DK_, DV_>,                                                \
                                     cudaFuncAttributePreferredSharedMemoryCarveout,                             \
                                     int(cudaSharedmemCarveoutMaxShared)));                                     \
    });                                                                                                          \
    if (T == n_seq) { /* one token per sequence: streamed update */                                             \
      static std::atomic<uint64_t> ring_set_##DK_##_##R_{0};                                                     \
      once_per_device(ring_set_##DK_##_##R_, [] {                                                                \
        QWEN_CUDA(cudaFuncSetAttribute(gdn_stream_kernel<DK_, DV_>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                       4 * 32 * DK_ * 4));                                                       \
        QWEN_CUDA(cudaFuncSetAttribute(gdn_stream_kernel<DK_, DV_>,                                              \
                                       cudaFuncAttributePreferredSharedMemoryCarveout,                           \
                                       int(cudaSharedmemCarveoutMaxShared)));                                   \
      });                                                                                                        \
      const int items = n_seq * d.hv;                                                                            \
      launch_pdl(gdn_stream_kernel<DK_, DV_>, std::min(items, 3 * sm_count), 288, size_t(4) * 32 * DK_ * 4, s,   \
                 descs, cu_seqlens, pool, gdn_index, d.hk, d.hv, items, qk_buf, v_buf, gb_buf, proj, ld_proj,     \
                 splits, split_stride, d.cd, ly.gnorm, d.eps, out, err, cand_slots);                             \
    } else {                                                                                                     \
      if (use_chunks)                                                                                            \
        launch_gdn_chunked(*chunked, d, ly, proj, ld_proj, splits, split_stride, descs, cu_seqlens, pool,        \
                           gdn_index, out, err, qk_buf, v_buf, gb_buf, s);                                       \
      launch_pdl(gdn_update_kernel<DK_, DV_>, dim3(n_seq, d.hv), 256, size_t(DV_) * DK_ * 4, s, descs,           \
                 cu_seqlens, pool, gdn_index, d.hk, d.hv, qk_buf, v_buf, gb_buf, proj, ld_proj, splits,           \
                 split_stride, d.cd, ly.gnorm, d.eps, out, err, cand_slots, skip_count);                         \
    }                                                                                                            \
    done = true;                                                                                                 \
  }
  QWEN_GDN(128, 128, 2)
  QWEN_GDN(64, 64, 2)
  QWEN_GDN(128, 128, 1)
  QWEN_GDN(64, 64, 1)
#undef QWEN_GDN
  if (!done) throw std::invalid_argument("DeltaNet geometry unsupported (dk = dv in {64,128}, hv/hk in {1,2})");
  QWEN_CUDA(cudaGetLastError());
  g_kernel_launches.fetch_add(2, std::memory_order_relaxed);
}

}  // namespace qwen
