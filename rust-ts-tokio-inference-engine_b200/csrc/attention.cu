// Paged GQA attention: the split decode kernel (flash-decoding) and the
// chunked-prefill kernel below.
//
// CTA = (work item, kv head g), kAttnWarps warps. A work item is one (query token t,
// KV split) pair from a host-built list holding only the splits that token
// attends, so no CTA is launched for keys beyond a token's position; a split
// covers `split_pages` consecutive 16-token pages (chosen per step). The
// split's pages are dealt round-robin to the warps; each warp streams its pages
// through a private 2-stage shared-memory ring filled by TMA (one 128B-swizzled
// 16x64 box per 64 head dims, K and V), computes S = Q K^T and O += P V with
// mma.sync (bf16 operands, fp32 accumulators; the G query heads of kv head g are
// the 16 MMA rows) and keeps an online softmax per head row in registers.
// The warps' (max, sum, O) are merged in shared memory and written as the
// split's partial; attention_merge_kernel combines splits and applies the
// output gate. Keys at positions >= pos(t)+1 are masked (causal, bottom-right).
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <cfloat>

#include "kernels.h"
#include "qgemm_tc.h"

namespace qwen {

extern std::atomic<uint64_t> g_kernel_launches;

namespace {

constexpr int kAttnWarps = 2;  // two warps per CTA: three CTAs fit an SM (shared memory, registers)
constexpr int kKvStages = 2;
constexpr long long kAttnWaitCycles = 2000000000ll;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t* err) {
  if (mbar_try(bar, parity)) return true;
  long long t0 = -1;
  for (uint32_t n = 1;; ++n) {
    if (mbar_try(bar, parity)) return true;
    if ((n & 255u) == 0) {
      const long long now = clock64();
      if (t0 < 0) t0 = now;
      else if (now - t0 > kAttnWaitCycles) {
        atomicOr(err, kErrTimeout);
        return false;
      }
    }
  }
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Byte offset of (row, 16-byte chunk) inside a 16-row x D tile stored as D/64
// 128B-swizzled boxes of 16 rows (the layout TMA SWIZZLE_128B writes).
__device__ __forceinline__ uint32_t sw_off(int row, int chunk) {
  const int box = chunk >> 3, c = chunk & 7;
  return uint32_t(box * 16 * 128 + row * 128 + ((c ^ (row & 7)) << 4));
}

template <int D>
__global__ void __launch_bounds__(kAttnWarps * 32)
    attn_decode_kernel(const __grid_constant__ CUtensorMap kvmap, const float* __restrict__ q,
                       const int32_t* __restrict__ token_seq, const int32_t* __restrict__ token_pos,
                       const int32_t* __restrict__ dec_tokens,
                       const SeqDesc* __restrict__ descs, const int32_t* __restrict__ block_table, int stride,
                       const int2* __restrict__ items, int split_pages, int Hq, int Hkv, int G, int max_splits,
                       float* __restrict__ ws, uint32_t* err) {
  pdl_trigger();
  pdl_wait(q, token_seq, token_pos, dec_tokens, descs, block_table, items, ws);
  constexpr int KS = D / 16;     // k-steps of Q K^T
  constexpr int NT = D / 8;      // n-tiles of O
  constexpr int TILE = 16 * D * 2;  // bytes of one 16-row tile
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = base;                                      // Q tile [16][D] bf16, swizzled
  uint8_t* kv = qs + TILE;                                 // [warps][stages][K tile, V tile]
  float* red = reinterpret_cast<float*>(kv + kAttnWarps * kKvStages * 2 * TILE);  // [warps][16][2]
  float* obuf = reinterpret_cast<float*>(kv);               // [16][D] merge buffer, on the drained ring
  uint64_t* bars = reinterpret_cast<uint64_t*>(red + kAttnWarps * 16 * 2);  // [warps][stages]

  // item.x indexes the step's split-decoded tokens (the workspace row);
  // dec_tokens maps it to the packed token (null: the same index)
  const int2 item = items[blockIdx.x];
  const int md = item.x, t = dec_tokens ? dec_tokens[md] : md, split = item.y, g = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = token_pos[t] + 1;
  const int n_pages = (len + kPageTokens - 1) / kPageTokens;
  const int p0 = split * split_pages;
  if (p0 >= n_pages || split >= max_splits) return;
  const int p1 = min(n_pages, p0 + split_pages);
  const int32_t* row = block_table + size_t(descs[token_seq[t]].child) * stride;

  // Q tile: rows 0..G-1 = heads g*G.., scaled by log2(e)/sqrt(D); rows >= G zero.
  const float qscale = 1.4426950408889634f * rsqrtf(float(D));
  for (int e = threadIdx.x; e < 16 * (D / 8); e += blockDim.x) {
    const int r = e / (D / 8), chunk = e % (D / 8);
    uint32_t w[4] = {0, 0, 0, 0};
    if (r < G) {
      const float* src = q + (size_t(t) * Hq + g * G + r) * D + chunk * 8;
#pragma unroll
      for (int j = 0; j < 4; ++j) w[j] = pack_bf16(src[2 * j] * qscale, src[2 * j + 1] * qscale);
    }
    *reinterpret_cast<uint4*>(qs + sw_off(r, chunk)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (threadIdx.x < kAttnWarps * kKvStages) mbar_init(&bars[threadIdx.x], 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  __syncthreads();

  uint64_t* mybars = bars + warp * kKvStages;
  uint8_t* mykv = kv + size_t(warp) * kKvStages * 2 * TILE;
  auto issue = [&](int page_local, int stage) {
    const int page = row[p0 + page_local];
    const int yk = ((page * 2 + 0) * Hkv + g) * kPageTokens;
    const int yv = ((page * 2 + 1) * Hkv + g) * kPageTokens;
    uint8_t* kt = mykv + stage * 2 * TILE;
    mbar_expect_tx(&mybars[stage], 2 * TILE);
#pragma unroll
    for (int b = 0; b < D / 64; ++b) {
      tma_load_2d(kt + b * 16 * 128, &kvmap, b * 64, yk, &mybars[stage]);
      tma_load_2d(kt + TILE + b * 16 * 128, &kvmap, b * 64, yv, &mybars[stage]);
    }
  };
  const int my_pages = (p1 - p0 - warp + kAttnWarps - 1) / kAttnWarps;  // pages warp, warp + kAttnWarps, ...
  if (lane == 0)
    for (int i = 0; i < kKvStages && i < my_pages; ++i) issue(warp + i * kAttnWarps, i);

  // Q fragments in registers (A operand, 16 rows x D)
  uint32_t qa[KS][4];
  {
    const int r = lane & 15, cadd = lane >> 4;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks)
      ldsm_x4(smem_u32(qs) + sw_off(r, ks * 2 + cadd), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
  }
  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -FLT_MAX, m1 = -FLT_MAX, l0 = 0.f, l1 = 0.f;  // rows lane/4 and lane/4+8
  bool ok = true;
  int stalled = 0;
  for (int i = 0; i < my_pages; ++i) {
    const int stage = i % kKvStages;
    if (!mbar_wait_bounded(&mybars[stage], (i / kKvStages) & 1, err)) { ok = false; stalled = i; break; }
    const uint32_t kt = smem_u32(mykv + stage * 2 * TILE), vt = kt + TILE;
    // S = Q K^T over 16 keys (two n-tiles of 8)
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const int krow = (lane & 7) + ((lane >> 4) << 3), cadd = (lane >> 3) & 1;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kt + sw_off(krow, ks * 2 + cadd), b0, b1, b2, b3);
        mma_bf16(s0, qa[ks], b0, b1);
        mma_bf16(s1, qa[ks], b2, b3);
      }
    }
    // causal mask on the last (partial) page
    const int key0 = (p0 + warp + i * kAttnWarps) * kPageTokens;
    const int c = (lane & 3) * 2;
    if (key0 + 16 > len) {
      if (key0 + c >= len) s0[0] = s0[2] = -FLT_MAX;
      if (key0 + c + 1 >= len) s0[1] = s0[3] = -FLT_MAX;
      if (key0 + 8 + c >= len) s1[0] = s1[2] = -FLT_MAX;
      if (key0 + 8 + c + 1 >= len) s1[1] = s1[3] = -FLT_MAX;
    }
    // online softmax (log2 domain), rows r0 = lane/4 (elements 0,1) and r1 = r0+8 (elements 2,3)
    float mx0 = fmaxf(fmaxf(s0[0], s0[1]), fmaxf(s1[0], s1[1]));
    float mx1 = fmaxf(fmaxf(s0[2], s0[3]), fmaxf(s1[2], s1[3]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float c0 = exp2f(m0 - mn0), c1 = exp2f(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    const float e00 = exp2f(s0[0] - mn0), e01 = exp2f(s0[1] - mn0), e02 = exp2f(s0[2] - mn1), e03 = exp2f(s0[3] - mn1);
    const float e10 = exp2f(s1[0] - mn0), e11 = exp2f(s1[1] - mn0), e12 = exp2f(s1[2] - mn1), e13 = exp2f(s1[3] - mn1);
    float rs0 = e00 + e01 + e10 + e11, rs1 = e02 + e03 + e12 + e13;
    rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1);
    rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
    rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1);
    rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
    l0 = l0 * c0 + rs0;
    l1 = l1 * c1 + rs1;
    const uint32_t pa[4] = {pack_bf16(e00, e01), pack_bf16(e02, e03), pack_bf16(e10, e11), pack_bf16(e12, e13)};
    // O = O*c + P V
    {
      const int vrow = (lane & 7) + (((lane >> 3) & 1) << 3), cadd = lane >> 4;
#pragma unroll
      for (int nt = 0; nt < NT; nt += 2) {
        o[nt][0] *= c0; o[nt][1] *= c0; o[nt][2] *= c1; o[nt][3] *= c1;
        o[nt + 1][0] *= c0; o[nt + 1][1] *= c0; o[nt + 1][2] *= c1; o[nt + 1][3] *= c1;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vt + sw_off(vrow, nt + cadd), b0, b1, b2, b3);
        mma_bf16(o[nt], pa, b0, b1);
        mma_bf16(o[nt + 1], pa, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0 && i + kKvStages < my_pages) issue(warp + (i + kKvStages) * kAttnWarps, stage);
  }
  if (!ok && lane == 0) {
    // timed out: wait (bounded) for this warp's page loads still in flight before
    // the ring is reused and the CTA leaves
    for (int j = stalled; j < min(my_pages, stalled + kKvStages); ++j)
      mbar_wait_bounded(&mybars[j % kKvStages], (j / kKvStages) & 1, err);
  }
  // merge the warps: row maxima and sums (the ring is drained: every page a
  // warp loaded it also consumed, so the ring now holds the merge buffer)
  __syncthreads();
  const int r0 = lane >> 2;
  if ((lane & 3) == 0) {
    red[(warp * 16 + r0) * 2 + 0] = m0;
    red[(warp * 16 + r0) * 2 + 1] = l0;
    red[(warp * 16 + r0 + 8) * 2 + 0] = m1;
    red[(warp * 16 + r0 + 8) * 2 + 1] = l1;
  }
  for (int e = threadIdx.x; e < 16 * D; e += blockDim.x) obuf[e] = 0.f;
  __syncthreads();
  float M0 = -FLT_MAX, M1 = -FLT_MAX;
  for (int w = 0; w < kAttnWarps; ++w) {
    M0 = fmaxf(M0, red[(w * 16 + r0) * 2]);
    M1 = fmaxf(M1, red[(w * 16 + r0 + 8) * 2]);
  }
  const float f0 = my_pages > 0 ? exp2f(m0 - M0) : 0.f, f1 = my_pages > 0 ? exp2f(m1 - M1) : 0.f;
  for (int w = 0; w < kAttnWarps; ++w) {
    if (w == warp) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int col = nt * 8 + (lane & 3) * 2;
        obuf[r0 * D + col] += o[nt][0] * f0;
        obuf[r0 * D + col + 1] += o[nt][1] * f0;
        obuf[(r0 + 8) * D + col] += o[nt][2] * f1;
        obuf[(r0 + 8) * D + col + 1] += o[nt][3] * f1;
      }
    }
    __syncthreads();
  }
  // write the split partial (m in natural-log units for the merge kernel)
  for (int hr = 0; hr < G; ++hr) {
    float Mh = -FLT_MAX, Lh = 0.f;
    for (int w = 0; w < kAttnWarps; ++w) Mh = fmaxf(Mh, red[(w * 16 + hr) * 2]);
    for (int w = 0; w < kAttnWarps; ++w) {
      const float mw = red[(w * 16 + hr) * 2];
      if (mw > -FLT_MAX) Lh += red[(w * 16 + hr) * 2 + 1] * exp2f(mw - Mh);
    }
    float* out = ws + ((size_t(md) * Hq + g * G + hr) * max_splits + split) * (D + 2);
    if (threadIdx.x == 0) {
      out[0] = Mh * 0.6931471805599453f;
      out[1] = Lh;
    }
    for (int i = threadIdx.x; i < D; i += blockDim.x) out[2 + i] = obuf[hr * D + i];
  }
}

// Chunked-prefill attention: CTA = (block of consecutive query tokens of one
// sequence, kv head g), kPfWarps warps. Warp w owns 16 query rows: tokens
// w*16/G .. of the block, each with the G query heads of kv head g (row r =
// token r / G, head r % G). Every K/V page of the block's prefix is loaded ONCE
// per CTA into a shared ring (one TMA per 64 head dims, K and V, 128B swizzle)
// and read by all warps, so a page crosses L2 once per (block, kv head)
// instead of once per query token. Per page a warp computes S = Q K^T (16 rows
// x 16 keys), the causal mask (key position <= the row token's position), the
// online softmax and O += P V with mma.sync (bf16 operands, fp32 accumulators),
// exactly like the decode kernel. Every warp releases a page it has read
// (empty barrier, one arrival per warp); lane 0 of warp 0 refills the slot.
// Pages are taken in increasing order and key 0 is visible to every token, so
// a row's running maximum is finite from the first page on. The epilogue
// divides by the row sum, applies the output gate sigmoid(gate) and writes the
// fp16 o_proj input; these tokens skip attention_merge_kernel.
constexpr int kPfWarps = kAttnPrefillWarps;
constexpr int kPfStages = 4;

template <int D>
__global__ void __launch_bounds__(kPfWarps * 32, 1)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap kvmap, const float* __restrict__ q,
                        const int32_t* __restrict__ token_pos, const SeqDesc* __restrict__ descs,
                        const int32_t* __restrict__ block_table, int stride, const int4* __restrict__ blocks,
                        int Hq, int Hkv, int G, const float* __restrict__ gate, gemm_in_t* __restrict__ out,
                        uint32_t* err) {
  pdl_trigger();
  pdl_wait(q, token_pos, descs, block_table, blocks, gate, out);
  constexpr int KS = D / 16;
  constexpr int NT = D / 8;
  constexpr int TILE = 16 * D * 2;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = base;  // [kPfStages][K tile, V tile]; first holds the warps' Q tiles
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + size_t(max(kPfStages * 2, kPfWarps)) * TILE);
  uint64_t* empty = full + kPfStages;

  const int4 blk = blocks[blockIdx.x];  // first packed token, tokens, sequence, pages
  const int t0 = blk.x, n_tok = blk.y, n_pages = blk.w, g = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tpw = 16 / G;  // tokens per warp
  const int32_t* row = block_table + size_t(descs[blk.z].child) * stride;

  // Q tiles (rows r: token w*tpw + r/G, head g*G + r%G), scaled by log2(e)/sqrt(D)
  const float qscale = 1.4426950408889634f * rsqrtf(float(D));
  for (int e = threadIdx.x; e < kPfWarps * 16 * (D / 8); e += blockDim.x) {
    const int w = e / (16 * (D / 8)), rem = e % (16 * (D / 8));
    const int r = rem / (D / 8), chunk = rem % (D / 8);
    const int tl = w * tpw + r / G;
    uint32_t v[4] = {0, 0, 0, 0};
    if (tl < n_tok) {
      const float* src = q + (size_t(t0 + tl) * Hq + g * G + r % G) * D + chunk * 8;
      const float4 x0 = *reinterpret_cast<const float4*>(src), x1 = *reinterpret_cast<const float4*>(src + 4);
      v[0] = pack_bf16(x0.x * qscale, x0.y * qscale);
      v[1] = pack_bf16(x0.z * qscale, x0.w * qscale);
      v[2] = pack_bf16(x1.x * qscale, x1.y * qscale);
      v[3] = pack_bf16(x1.z * qscale, x1.w * qscale);
    }
    *reinterpret_cast<uint4*>(ring + size_t(w) * TILE + sw_off(r, chunk)) = make_uint4(v[0], v[1], v[2], v[3]);
  }
  if (threadIdx.x < kPfStages) {
    mbar_init(&full[threadIdx.x], 1);
    mbar_init(&empty[threadIdx.x], kPfWarps);
  }
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  __syncthreads();
  uint32_t qa[KS][4];
  {
    const int r = lane & 15, cadd = lane >> 4;
    const uint32_t qt = smem_u32(ring + size_t(warp) * TILE);
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) ldsm_x4(qt + sw_off(r, ks * 2 + cadd), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
  }
  __syncthreads();  // the Q tiles are in registers: the ring is free
  auto issue = [&](int page_local, int stage) {
    const int page = row[page_local];
    const int yk = ((page * 2 + 0) * Hkv + g) * kPageTokens;
    const int yv = ((page * 2 + 1) * Hkv + g) * kPageTokens;
    uint8_t* kt = ring + size_t(stage) * 2 * TILE;
    mbar_expect_tx(&full[stage], 2 * TILE);
#pragma unroll
    for (int b = 0; b < D / 64; ++b) {
      tma_load_2d(kt + b * 16 * 128, &kvmap, b * 64, yk, &full[stage]);
      tma_load_2d(kt + TILE + b * 16 * 128, &kvmap, b * 64, yv, &full[stage]);
    }
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < kPfStages && i < n_pages; ++i) issue(i, i);

  // positions of this lane's two rows (-1: past the block's last token)
  const int r0 = lane >> 2, r1 = r0 + 8;
  const int tl0 = warp * tpw + r0 / G, tl1 = warp * tpw + r1 / G;
  const int pos0 = tl0 < n_tok ? token_pos[t0 + tl0] : -1;
  const int pos1 = tl1 < n_tok ? token_pos[t0 + tl1] : -1;
  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -FLT_MAX, m1 = -FLT_MAX, l0 = 0.f, l1 = 0.f;
  bool ok = true;
  int stalled = 0;
  for (int i = 0; i < n_pages; ++i) {
    const int stage = i % kPfStages;
    if (!mbar_wait_bounded(&full[stage], (i / kPfStages) & 1, err)) { ok = false; stalled = i; break; }
    const uint32_t kt = smem_u32(ring + size_t(stage) * 2 * TILE), vt = kt + TILE;
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const int krow = (lane & 7) + ((lane >> 4) << 3), cadd = (lane >> 3) & 1;
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kt + sw_off(krow, ks * 2 + cadd), b0, b1, b2, b3);
        mma_bf16(s0, qa[ks], b0, b1);
        mma_bf16(s1, qa[ks], b2, b3);
      }
    }
    const int key0 = i * kPageTokens + (lane & 3) * 2;
    if (key0 + 0 > pos0) s0[0] = -FLT_MAX;
    if (key0 + 1 > pos0) s0[1] = -FLT_MAX;
    if (key0 + 0 > pos1) s0[2] = -FLT_MAX;
    if (key0 + 1 > pos1) s0[3] = -FLT_MAX;
    if (key0 + 8 > pos0) s1[0] = -FLT_MAX;
    if (key0 + 9 > pos0) s1[1] = -FLT_MAX;
    if (key0 + 8 > pos1) s1[2] = -FLT_MAX;
    if (key0 + 9 > pos1) s1[3] = -FLT_MAX;
    float mx0 = fmaxf(fmaxf(s0[0], s0[1]), fmaxf(s1[0], s1[1]));
    float mx1 = fmaxf(fmaxf(s0[2], s0[3]), fmaxf(s1[2], s1[3]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float c0 = exp2f(m0 - mn0), c1 = exp2f(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    const float e00 = exp2f(s0[0] - mn0), e01 = exp2f(s0[1] - mn0), e02 = exp2f(s0[2] - mn1), e03 = exp2f(s0[3] - mn1);
    const float e10 = exp2f(s1[0] - mn0), e11 = exp2f(s1[1] - mn0), e12 = exp2f(s1[2] - mn1), e13 = exp2f(s1[3] - mn1);
    float rs0 = e00 + e01 + e10 + e11, rs1 = e02 + e03 + e12 + e13;
    rs0 += __shfl_xor_sync(0xffffffffu, rs0, 1);
    rs0 += __shfl_xor_sync(0xffffffffu, rs0, 2);
    rs1 += __shfl_xor_sync(0xffffffffu, rs1, 1);
    rs1 += __shfl_xor_sync(0xffffffffu, rs1, 2);
    l0 = l0 * c0 + rs0;
    l1 = l1 * c1 + rs1;
    const uint32_t pa[4] = {pack_bf16(e00, e01), pack_bf16(e02, e03), pack_bf16(e10, e11), pack_bf16(e12, e13)};
    {
      const int vrow = (lane & 7) + (((lane >> 3) & 1) << 3), cadd = lane >> 4;
#pragma unroll
      for (int nt = 0; nt < NT; nt += 2) {
        o[nt][0] *= c0; o[nt][1] *= c0; o[nt][2] *= c1; o[nt][3] *= c1;
        o[nt + 1][0] *= c0; o[nt + 1][1] *= c0; o[nt + 1][2] *= c1; o[nt + 1][3] *= c1;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vt + sw_off(vrow, nt + cadd), b0, b1, b2, b3);
        mma_bf16(o[nt], pa, b0, b1);
        mma_bf16(o[nt + 1], pa, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (warp == 0 && i + kPfStages < n_pages) {
      // refill this slot once every warp has left page i
      if (!mbar_wait_bounded(&empty[stage], (i / kPfStages) & 1, err)) { ok = false; stalled = i + 1; break; }
      if (lane == 0) issue(i + kPfStages, stage);
      __syncwarp();
    }
  }
  if (!ok) {
    // timed out: let the page loads in flight land before the CTA leaves
    __syncwarp();
    if (lane == 0)
      for (int j = stalled; j < min(n_pages, stalled + kPfStages); ++j)
        mbar_wait_bounded(&full[j % kPfStages], (j / kPfStages) & 1, err);
  }
  // epilogue: O / l * sigmoid(gate) -> fp16 rows of the o_proj input
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const int h0 = g * G + r0 % G, h1 = g * G + r1 % G;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int col = nt * 8 + (lane & 3) * 2;
    if (pos0 >= 0) {
      const size_t off = (size_t(t0 + tl0) * Hq + h0) * D + col;
      const float2 gt = *reinterpret_cast<const float2*>(gate + off);
      *reinterpret_cast<__half2*>(out + off) =
          to_gemm_in2(o[nt][0] * inv0 * sigmoidf_(gt.x), o[nt][1] * inv0 * sigmoidf_(gt.y));
    }
    if (pos1 >= 0) {
      const size_t off = (size_t(t0 + tl1) * Hq + h1) * D + col;
      const float2 gt = *reinterpret_cast<const float2*>(gate + off);
      *reinterpret_cast<__half2*>(out + off) =
          to_gemm_in2(o[nt][2] * inv1 * sigmoidf_(gt.x), o[nt][3] * inv1 * sigmoidf_(gt.y));
    }
  }
}

}  // namespace

size_t attn_prefill_smem(int D) {
  const size_t tile = 16 * size_t(D) * 2;
  return 1024 + size_t(std::max(kPfStages * 2, kPfWarps)) * tile + 2 * kPfStages * 8;
}

void launch_attn_prefill(const CUtensorMap& kvmap, const Dims& d, const float* q, const int32_t* token_pos,
                         const SeqDesc* descs, const int32_t* block_table, int bt_stride, const int4* blocks,
                         int n_blocks, const float* gate, gemm_in_t* out, uint32_t* err, cudaStream_t s) {
  const int G = d.Hq / d.Hkv;
  if (G < 1 || G > 16 || 16 % G) throw std::invalid_argument("prefill attention needs 16 % (query heads per KV head) == 0");
  if (n_blocks <= 0) return;
  dim3 grid(n_blocks, d.Hkv);
  const size_t smem = attn_prefill_smem(d.D);
#define QWEN_ATTN_PF(DD)                                                                                      \
  if (d.D == DD) {                                                                                          \
    static std::atomic<uint64_t> cfg_##DD{0};                                                               \
    once_per_device(cfg_##DD, [&] {                                                                         \
      QWEN_CUDA(cudaFuncSetAttribute(attn_prefill_kernel<DD>, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                                     int(smem)));                                                           \
    });                                                                                                     \
    launch_pdl(attn_prefill_kernel<DD>, grid, kPfWarps * 32, smem, s, kvmap, q, token_pos, descs, block_table, \
               bt_stride, blocks, d.Hq, d.Hkv, G, gate, out, err);                                            \
    QWEN_CUDA(cudaGetLastError());                                                                          \
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);                                              \
    return;                                                                                                 \
  }
  QWEN_ATTN_PF(256)
  QWEN_ATTN_PF(128)
  QWEN_ATTN_PF(64)
#undef QWEN_ATTN_PF
  throw std::invalid_argument("head_dim must be 64, 128 or 256");
}

size_t attn_decode_smem(int D) {
  const size_t tile = 16 * size_t(D) * 2;
  return 1024 + tile + kAttnWarps * kKvStages * 2 * tile + kAttnWarps * 16 * 2 * 4 + kAttnWarps * kKvStages * 8;
}

CUtensorMap make_kv_map(const KvPool& kv, int layer);

void launch_attn_decode(const CUtensorMap& kvmap, const Dims& d, const float* q, const int32_t* token_seq,
                        const int32_t* token_pos, const int32_t* dec_tokens, const SeqDesc* descs, const int32_t* block_table, int bt_stride,
                        const int2* items, int n_items, int split_pages, float* ws, int max_splits, uint32_t* err,
                        cudaStream_t s) {
  const int G = d.Hq / d.Hkv;
  if (G > 16) throw std::invalid_argument("attention kernel supports up to 16 query heads per KV head");
  if (n_items <= 0) return;
  if (split_pages < 1) throw std::invalid_argument("attention split must cover at least one page");
  dim3 grid(n_items, d.Hkv);
  const size_t smem = attn_decode_smem(d.D);
#define QWEN_ATTN(DD)                                                                                         \
  if (d.D == DD) {                                                                                          \
    static std::atomic<uint64_t> cfg_##DD{0};                                                               \
    once_per_device(cfg_##DD, [&] {                                                                         \
      QWEN_CUDA(cudaFuncSetAttribute(attn_decode_kernel<DD>, cudaFuncAttributeMaxDynamicSharedMemorySize,   \
                                     int(smem)));                                                           \
    });                                                                                                     \
    launch_pdl(attn_decode_kernel<DD>, grid, kAttnWarps * 32, smem, s, kvmap, q, token_seq, token_pos, dec_tokens, descs, \
                                                               block_table, bt_stride, items, split_pages,  \
                                                               d.Hq, d.Hkv, G, max_splits, ws, err);        \
    QWEN_CUDA(cudaGetLastError());                                                                          \
    g_kernel_launches.fetch_add(1, std::memory_order_relaxed);                                              \
    return;                                                                                                 \
  }
  QWEN_ATTN(256)
  QWEN_ATTN(128)
  QWEN_ATTN(64)
#undef QWEN_ATTN
  throw std::invalid_argument("head_dim must be 64, 128 or 256");
}

}  // namespace qwen
