// tcgen05 grouped GEMM over 4-bit affine (group 64 scale/bias) weights, IEEE
// half operands (dequantised weights in TMEM, activations in shared memory).
//
//   D[w_row, token] = sum_k deq(W)[w_row, k] * X[token, k]
//
// Weight rows are the MMA's M dimension (128 per tile), tokens are N (16..128),
// so the tiny token counts of decode (1-10 rows per expert) cost one N=16 MMA.
// Per CTA (persistent, one per SM), warp-specialised:
//   warp 0  weight producer: one cp.async.bulk per unit of U contiguous
//           4608-byte weight tiles into a deep ring (kWSlots units) that the
//           dequant warps release as soon as they have read it, so HBM reads
//           run far ahead of the tensor cores;
//   warp 2  activation producer: one 3-D TMA per unit (U 64-column tiles,
//           128B-swizzled) into its own ring of 96 KB (768 / box chunks, deeper
//           than the TMEM stages so L2 round trips overlap); a slot is
//           released by the dequant warpgroup that sees the MMAs reading it
//           complete (the TMEM slot wait of the unit NS units later);
//   warp 1  MMA issuer (converged warp, one elected lane issues): allocates
//           TMEM and works in units of U (= 4, 2 or 1) chunks: one mbarrier
//           wait, 4U tcgen05.mma (A from TMEM, B from shared memory) and one
//           tcgen05.commit per unit. Measured on B200, an MMA issue costs ~26
//           cycles, an mbarrier wait ~80 and a commit ~200 unless ~16 MMAs
//           separate commits, so units amortise the fixed costs;
//   warps 3-14 dequantise (three warpgroups taking whole units round-robin):
//           each thread owns one weight row, turns its 64 nibbles per chunk
//           into 32 f16x2 words (e4m3 conversion of nibble bytes, then
//           scale*q + bias with one fp16 rounding) and stores
//           them into TMEM with tcgen05.st (the A operand);
//   warps 15-18 epilogue: tcgen05.ld of the fp32 accumulator, then split-K
//           partial store / SwiGLU (fp16) / fp32 store.
// The dequantised weights never touch shared memory. A unit's TMEM A stages
// are released together by its commit. Units never straddle work items (split-K ranges are
// multiples of U). Every mbarrier wait is bounded (~1 s); on expiry the kernel
// raises kErrTimeout and drains out.
#include <cuda.h>

#include <algorithm>
#include <atomic>

#include "kernels.h"
#include "qgemm_tc.h"
#include "tcgen05.cuh"

namespace qwen {

extern std::atomic<uint64_t> g_kernel_launches;

namespace {

constexpr int kDequantGroups = 3;    // dequant warpgroups, round-robin over units
constexpr int kWSlots = 6;           // weight ring depth (units); a multiple of kDequantGroups
constexpr int kEpiWarp0 = 3 + 4 * kDequantGroups;  // first warp of the epilogue warpgroup
constexpr int kWarps = kEpiWarp0 + 4;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxStages = 12;       // shared-memory ring = TMEM A stages (32 columns each)
constexpr int kMaxGroups = 1040;     // shared-memory cache of group offsets
constexpr int kItemCache = 128;      // grouped: this CTA's first items, decoded once at kernel start
constexpr int kTmemCols = 512;
// One packed word (8 columns) into four f16x2 A-operand registers
// (columns 0-1, 2-3, 4-5, 6-7): the bytes of (w & 0x0F0F0F0F) and of
// ((w >> 4) & 0x0F0F0F0F) each hold one nibble q, which the e4m3 -> f16x2
// conversion turns into exactly q * 2^-9; fma.rn with the tile's scale (stored
// times 2^9) and bias then rounds scale * q + bias once to fp16. `m` =
// 0x0F0F0F0F lives in a register.
__device__ __forceinline__ void deq_word(uint32_t w, uint32_t m, uint32_t s2, uint32_t b2, uint32_t* out) {
  const uint32_t lo = w & m, hi = (w >> 4) & m;
  uint32_t c0, c1, c2, c3;
  asm("{\n\t.reg .b16 l, u;\n\t"
      "mov.b32 {l, u}, %4;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, l;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, u;\n\t"
      "mov.b32 {l, u}, %5;\n\t"
      "cvt.rn.f16x2.e4m3x2 %2, l;\n\t"
      "cvt.rn.f16x2.e4m3x2 %3, u;\n\t}"
      : "=r"(c0), "=r"(c1), "=r"(c2), "=r"(c3)
      : "r"(lo), "r"(hi));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(out[0]) : "r"(c0), "r"(s2), "r"(b2));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(out[1]) : "r"(c1), "r"(s2), "r"(b2));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(out[2]) : "r"(c2), "r"(s2), "r"(b2));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(out[3]) : "r"(c3), "r"(s2), "r"(b2));
}

// Token groups of a dense launch (1 when the tokens are not split).
__host__ __device__ __forceinline__ int dense_token_groups(const TcArgs& a) {
  return a.token_group > 0 ? (a.n_tokens + a.token_group - 1) / a.token_group : 1;
}

struct Work {
  int rt;       // global row tile of W
  int c0, c1;   // chunk range
  int p0, p1;   // token / sorted-position range
  int g;        // group (expert), or split index for dense
  int rt_local; // row tile within the group
  bool valid;
};

// Grouped items run over the non-empty groups only (`act`, built in shared
// memory at kernel start) and hold one token block each: item = (group, row
// tile, token block), token block fastest. `bpre[j]` counts the token blocks
// of the first j non-empty groups, so group j owns items
// [bpre[j] * expert_tiles, bpre[j + 1] * expert_tiles). A group far larger
// than the rest (the shared expert of a prefill step) is thereby spread over
// many CTAs instead of lengthening the few that draw its row tiles.
__device__ __forceinline__ int4 grouped_item(const TcArgs& a, int i, const int32_t* goff, const int32_t* act,
                                             const int32_t* bpre) {
  // the last non-empty group j with bpre[j] * expert_tiles <= i
  const int key = i / a.expert_tiles;
  int lo = 0, hi = act[kMaxGroups] - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (bpre[mid] <= key) lo = mid;
    else hi = mid - 1;
  }
  const int nb = bpre[lo + 1] - bpre[lo];
  const int local = i - bpre[lo] * a.expert_tiles;
  const int g = act[lo], rt_local = local / nb;
  const int p0 = goff[g] + (local - rt_local * nb) * a.box_rows;
  return make_int4(g, rt_local, p0, min(goff[g + 1], p0 + a.box_rows));
}

// Item i, the k-th of this CTA (i = blockIdx.x + k * gridDim.x).
__device__ __forceinline__ Work item_at(const TcArgs& a, int i, int k, const int32_t* goff, const int32_t* act,
                                        const int32_t* bpre, const int4* icache) {
  Work w;
  const int kc = a.W.k_chunks();
  if (a.mode == kGemmStoreF32) {
    // item = (row tile, split, token group), row tile fastest
    w.rt = i % a.W.row_tiles;
    const int rest = i / a.W.row_tiles;
    w.g = rest % a.splits;  // split
    w.rt_local = w.rt;
    const int per = (kc + a.splits - 1) / a.splits;
    w.c0 = w.g * per;
    w.c1 = min(kc, w.c0 + per);
    const int tg = rest / a.splits;
    w.p0 = a.token_group > 0 ? tg * a.token_group : 0;
    w.p1 = a.token_group > 0 ? min(a.n_tokens, w.p0 + a.token_group) : a.n_tokens;
  } else {
    const int4 it = k < kItemCache ? icache[k] : grouped_item(a, i, goff, act, bpre);
    w.g = it.x;
    w.rt_local = it.y;
    w.rt = w.g * a.expert_tiles + w.rt_local;
    w.c0 = 0;
    w.c1 = kc;
    w.p0 = it.z;
    w.p1 = it.w;
  }
  w.valid = w.p1 > w.p0 && w.c1 > w.c0;
  return w;
}


__global__ void __launch_bounds__(kThreads, 1)
    qgemm_tc_kernel(const __grid_constant__ CUtensorMap bmap, const TcArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // carve: [B ring (1024-aligned)] [W ring] [exchange] [barriers]
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;         // TMEM A stages = B ring depth in chunks (multiple of U)
  const int U = a.unit;           // chunks per unit (4, 2 or 1)
  const int ushift = U == 4 ? 2 : (U == 2 ? 1 : 0);
  const int NS = S / U;           // TMEM/B unit slots (multiple of kDequantGroups)
  const int box = a.box_rows;
  const int NSB = a.b_stages / U; // activation ring unit slots
  const int d_col0 = S * 32;      // accumulators after the A stages
  const int d_stride = box <= 64 ? 64 : 128;
  const uint32_t b_bytes = uint32_t(box) * 128;
  const uint32_t w_unit = uint32_t(U) * kTileBytes;
  uint8_t* ring_b = base;
  uint8_t* ring_w = ring_b + size_t(a.b_stages) * b_bytes;
  float* xchg = reinterpret_cast<float*>(ring_w + size_t(kWSlots) * w_unit);  // [64][9]
  uint64_t* bars = reinterpret_cast<uint64_t*>(xchg + 64 * 9);
  uint64_t* w_full = bars;              // [kWSlots] unit weights landed (tx)
  uint64_t* w_empty = w_full + kWSlots; // [kWSlots] unit weights read (4 dequant warps)
  uint64_t* b_full = w_empty + kWSlots; // [NSB] unit activations landed (tx)
  uint64_t* b_empty = b_full + NSB;     // [NSB] unit activations consumed (1 dequant lane)
  uint64_t* a_full = b_empty + NSB;     // [NS] unit A stages written (4 dequant warps)
  uint64_t* empty = a_full + NS;        // [NS] unit consumed by the MMAs (commit)
  uint64_t* acc_full = empty + NS;      // [2]  accumulator complete (commit)
  uint64_t* acc_empty = acc_full + 2;   // [2]  accumulator drained (4 epilogue warps)
  volatile int* abort_flag = reinterpret_cast<volatile int*>(acc_empty + 2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2) + 1;
  int32_t* goff = reinterpret_cast<int32_t*>(acc_empty + 3);  // [groups + 1]
  int32_t* act = goff + (kMaxGroups + 1);                      // [non-empty groups], then their count
  int32_t* bpre = act + (kMaxGroups + 1);                      // token blocks before each non-empty group
  int4* icache = reinterpret_cast<int4*>((reinterpret_cast<uintptr_t>(bpre + kMaxGroups + 1) + 15) & ~uintptr_t(15));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  // Dependencies on earlier kernels: the activations (warp 2), the outputs
  // (epilogue) and, grouped, the group offsets read below. In dense mode the
  // weight producer and the dequant/MMA warps start on the constant weights
  // while the previous kernel finishes.
  if (a.mode != kGemmStoreF32 || warp == 2 || warp >= kEpiWarp0) pdl_wait();
  if (threadIdx.x == 0) {
    for (int i = 0; i < kWSlots; ++i) { mbar_init(&w_full[i], 1); mbar_init(&w_empty[i], 4); }
    for (int i = 0; i < NSB; ++i) { mbar_init(&b_full[i], 1); mbar_init(&b_empty[i], 1); }
    for (int i = 0; i < NS; ++i) { mbar_init(&a_full[i], 4); mbar_init(&empty[i], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], 4); }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (a.mode != kGemmStoreF32)
    for (int g = threadIdx.x; g <= a.groups; g += blockDim.x) goff[g] = a.group_off[g];
  __syncthreads();
  if (a.mode != kGemmStoreF32 && warp == 2) {
    // stable compaction of the non-empty groups (ballot + popc per 32 groups)
    // and the prefix of their token block counts (warp scan)
    int n = 0, blocks = 0;
    for (int g0 = 0; g0 < a.groups; g0 += 32) {
      const int g = g0 + lane;
      const int cnt = g < a.groups ? goff[g + 1] - goff[g] : 0;
      const bool live = cnt > 0;
      const uint32_t m = __ballot_sync(0xffffffffu, live);
      int x = live ? (cnt + a.box_rows - 1) / a.box_rows : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (live) {
        const int j = n + __popc(m & ((1u << lane) - 1u));
        act[j] = g;
        bpre[j + 1] = blocks + x;
      }
      n += __popc(m);
      blocks += __shfl_sync(0xffffffffu, x, 31);
    }
    if (lane == 0) {
      act[kMaxGroups] = n;
      bpre[0] = 0;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int total = a.mode == kGemmStoreF32 ? a.W.row_tiles * a.splits * dense_token_groups(a)
                                             : bpre[act[kMaxGroups]] * a.expert_tiles;
  if (a.mode != kGemmStoreF32) {
    // decode this CTA's first items once (a binary search each), so the
    // roles' per-item lookups are one shared-memory load
    for (int k = threadIdx.x; k < kItemCache; k += blockDim.x) {
      const int i = blockIdx.x + k * gridDim.x;
      if (i < total) icache[k] = grouped_item(a, i, goff, act, bpre);
    }
    __syncthreads();
  }

  if (warp == 0) {
    // ---------------- weight producer ----------------
    int ws = 0;
    uint32_t wph = 0;
    bool ok = true;
    for (int i = blockIdx.x, k_item = 0; i < total && ok && !*abort_flag; i += gridDim.x, ++k_item) {
      const Work w = item_at(a, i, k_item, goff, act, bpre, icache);
      if (!w.valid) continue;
      for (int tb = w.p0; tb < w.p1 && ok; tb += box) {
        for (int c = w.c0; c < w.c1; c += U) {
          if (!mbar_wait(&w_empty[ws], wph ^ 1, abort_flag, a.err)) { ok = false; break; }
          if (elect_one()) {
            mbar_expect_tx(&w_full[ws], w_unit);
            bulk_load(ring_w + size_t(ws) * w_unit, a.W.tile(w.rt, c), w_unit, &w_full[ws]);
          }
          __syncwarp();
          if (++ws == kWSlots) { ws = 0; wph ^= 1; }
        }
      }
    }
  } else if (warp == 2) {
    // ---------------- activation producer ----------------
    int bs = 0;
    uint32_t bph = 0;
    bool ok = true;
    for (int i = blockIdx.x, k_item = 0; i < total && ok && !*abort_flag; i += gridDim.x, ++k_item) {
      const Work w = item_at(a, i, k_item, goff, act, bpre, icache);
      if (!w.valid) continue;
      for (int tb = w.p0; tb < w.p1 && ok; tb += box) {
        for (int c = w.c0; c < w.c1; c += U) {
          if (!mbar_wait(&b_empty[bs], bph ^ 1, abort_flag, a.err)) { ok = false; break; }
          if (elect_one()) {
            mbar_expect_tx(&b_full[bs], uint32_t(U) * b_bytes);
            tma_load_3d(ring_b + size_t(bs) * U * b_bytes, &bmap, 0, a.b_row0 + tb, c, &b_full[bs]);
          }
          __syncwarp();
          if (++bs == NSB) { bs = 0; bph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (converged warp, elected lane issues) ----------------
    int st = 0, bs = 0;
    uint32_t ph = 0, bph = 0, acc_it = 0;
    const uint32_t idesc = idesc_f16(box);
    bool ok = true;
    for (int i = blockIdx.x, k_item = 0; i < total && ok && !*abort_flag; i += gridDim.x, ++k_item) {
      const Work w = item_at(a, i, k_item, goff, act, bpre, icache);
      if (!w.valid) continue;
      for (int tb = w.p0; tb < w.p1 && ok; tb += box, ++acc_it) {
        const int d = acc_it & 1;
        if (!mbar_wait(&acc_empty[d], ((acc_it >> 1) & 1) ^ 1, abort_flag, a.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem + d_col0 + d * d_stride;
        for (int c = w.c0; c < w.c1; c += U) {
          const int slot = st >> ushift;
          if (!mbar_wait(&b_full[bs], bph, abort_flag, a.err)) { ok = false; break; }
          if (!mbar_wait(&a_full[slot], ph, abort_flag, a.err)) { ok = false; break; }
          tc_fence_after();
          if (elect_one()) {
            for (int u = 0; u < U; ++u) {
              const uint64_t bdesc = smem_desc_sw128(smem_u32(ring_b + size_t(bs * U + u) * b_bytes));
#pragma unroll
              for (int k = 0; k < kTileK / 16; ++k)
                mma_ts(d_tmem, tmem + (st + u) * 32 + k * 8, bdesc + uint64_t(k * 2), idesc,
                       (c + u > w.c0 || k > 0) ? 1u : 0u);
            }
            mma_commit(&empty[slot]);
          }
          __syncwarp();
          st += U;
          if (st == S) { st = 0; ph ^= 1; }
          if (++bs == NSB) { bs = 0; bph ^= 1; }
        }
        if (ok && elect_one()) mma_commit(&acc_full[d]);
        __syncwarp();
      }
    }
  } else if (warp < kEpiWarp0) {
    // ---------------- dequantise (warps 3..14), whole units round-robin ----------------
    const int wg = (warp - 3) >> 2;
    const int quad = warp & 3;             // TMEM lane quadrant this warp may access
    const int r = quad * 32 + lane;        // weight row within the tile
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    const uint32_t ring_w_s = smem_u32(ring_w);
    // nibble-byte mask in a register
    uint32_t k_mask = 0x0F0F0F0Fu;
    asm volatile("" : "+r"(k_mask));
    // This warpgroup takes units n = wg, wg + 3, ... of the CTA's unit
    // sequence. NS, kWSlots and NSB are multiples of 3, so its TMEM slot,
    // weight slot and released activation slot (of unit n - NS) each advance
    // by 3 per unit, and it never walks the other warpgroups' units.
    int st = wg * U, ws = wg, rel = wg, mine = 0, skip = wg;
    uint32_t ph = 0, wph = 0;
    bool ok = true;
    for (int i = blockIdx.x, k_item = 0; i < total && ok && !*abort_flag; i += gridDim.x, ++k_item) {
      const Work w = item_at(a, i, k_item, goff, act, bpre, icache);
      if (!w.valid) continue;
      const int nb = (w.c1 - w.c0) / U;  // units per token block (K ranges are multiples of U)
      for (int tb = w.p0; tb < w.p1 && ok; tb += box) {
        int k = skip;
        for (; k < nb; k += kDequantGroups) {
          const int slot = st >> ushift;
          if (!mbar_wait(&w_full[ws], wph, abort_flag, a.err)) { ok = false; break; }
          // the MMAs that read these TMEM stages last round must be done...
          if (!mbar_wait(&empty[slot], ph ^ 1, abort_flag, a.err)) { ok = false; break; }
          // ...which also ends their reads of unit (n - NS)'s activations
          if (mine >= NS / kDequantGroups && quad == 0 && lane == 0) mbar_arrive(&b_empty[rel]);
          tc_fence_after();
          for (int u = 0; u < U; ++u) {
            const uint32_t tile = ring_w_s + uint32_t(ws) * w_unit + uint32_t(u) * kTileBytes;
            const uint4 p0 = lds128(tile + r * 32);
            const uint4 p1 = lds128(tile + r * 32 + 16);
            const uint32_t sb = lds_u16(tile + kTilePackedBytes + r * 2);
            const uint32_t bb = lds_u16(tile + kTilePackedBytes + kTileRows * 2 + r * 2);
            const uint32_t s2 = __byte_perm(sb, 0, 0x1010), b2 = __byte_perm(bb, 0, 0x1010);
            uint32_t v[32];
#define QWEN_DEQ_WORD(WD, W) deq_word((W), k_mask, s2, b2, v + (WD) * 4);
            QWEN_DEQ_WORD(0, p0.x) QWEN_DEQ_WORD(1, p0.y) QWEN_DEQ_WORD(2, p0.z) QWEN_DEQ_WORD(3, p0.w)
            QWEN_DEQ_WORD(4, p1.x) QWEN_DEQ_WORD(5, p1.y) QWEN_DEQ_WORD(6, p1.z) QWEN_DEQ_WORD(7, p1.w)
#undef QWEN_DEQ_WORD
            tmem_st32(tmem + lane_addr + (st + u) * 32, v);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&w_empty[ws]);  // weights read: the producer may refill
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[slot]);
          st += kDequantGroups * U;
          if (st >= S) { st -= S; ph ^= 1; }
          ws += kDequantGroups;
          if (ws >= kWSlots) { ws -= kWSlots; wph ^= 1; }
          if (mine >= NS / kDequantGroups && (rel += kDequantGroups) >= NSB) rel -= NSB;
          ++mine;
        }
        skip = k - nb;
      }
    }
  } else {
    // ---------------- epilogue (warps 15..18) ----------------
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_addr = uint32_t(quad * 32) << 16;
    uint32_t acc_it = 0;
    bool ok = true;
    for (int i = blockIdx.x, k_item = 0; i < total && ok && !*abort_flag; i += gridDim.x, ++k_item) {
      const Work w = item_at(a, i, k_item, goff, act, bpre, icache);
      if (!w.valid) continue;
      for (int tb = w.p0; tb < w.p1 && ok; tb += box, ++acc_it) {
        const int d = acc_it & 1;
        if (!mbar_wait(&acc_full[d], (acc_it >> 1) & 1, abort_flag, a.err)) { ok = false; break; }
        tc_fence_after();
        const int nvalid = min(box, w.p1 - tb);
        const int n_glob = w.rt * kTileRows + r;
        for (int j0 = 0; j0 < box && j0 < nvalid; j0 += 8) {
          uint32_t v[8];
          tmem_ld8(tmem + lane_addr + d_col0 + d * d_stride + j0, v);
          tmem_wait_ld();
          if (a.mode == kGemmStoreF32) {
            if (n_glob < a.W.rows) {
              float* y = a.Y + size_t(w.g) * a.split_stride;
#pragma unroll
              for (int j = 0; j < 8; ++j)
                if (j0 + j < nvalid) y[size_t(tb + j0 + j) * a.ldy + n_glob] = __uint_as_float(v[j]);
            }
          } else if (a.mode == kGemmDown) {
            const int n = w.rt_local * kTileRows + r;
#pragma unroll
            for (int j = 0; j < 8; ++j)
              if (j0 + j < nvalid) a.Y[size_t(tb + j0 + j) * a.ldy + n] = __uint_as_float(v[j]);
          } else {
            if (r >= 64) {
#pragma unroll
              for (int j = 0; j < 8; ++j) xchg[(r - 64) * 9 + j] = __uint_as_float(v[j]);
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (r < 64) {
              const int jj = w.rt_local * 64 + r;
#pragma unroll
              for (int j = 0; j < 8; ++j)
                if (j0 + j < nvalid) {
                  const float gv = __uint_as_float(v[j]), uv = xchg[r * 9 + j];
                  a.Yb[size_t(tb + j0 + j) * a.ldyb + jj] = to_gemm_in(gv / (1.f + __expf(-gv)) * uv);
                }
            }
            asm volatile("bar.sync 1, 128;" ::: "memory");
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[d]);
      }
    }
  }
  // teardown: every warp reaches here (bounded waits); free TMEM
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

}  // namespace


size_t qgemm_tc_smem(int box_rows, int stages, int unit) {
  const int b_stages = qgemm_tc_bstages(box_rows);
  return 1024 + size_t(b_stages) * size_t(box_rows) * 128 + size_t(kWSlots) * unit * kTileBytes + 64 * 9 * 4 +
         (2 * size_t(kWSlots) + 2 * size_t(b_stages) + 3 * size_t(stages) + 4) * 8 + 16 +
         3 * (kMaxGroups + 1) * 4 + 16 + kItemCache * 16;  // group offsets, non-empty groups, token block
                                                            // prefix, item cache
}

// Activation ring depth (chunks): 96 KB of box-row tiles, at least the TMEM
// stages, a multiple of every unit size.
int qgemm_tc_bstages(int box_rows) { return std::max(qgemm_tc_stages(box_rows), 768 / box_rows); }

// Ring depth (chunks): A stages (32 TMEM columns each) plus two accumulators
// (64 or 128 columns) fit in 512 columns. The number of unit slots
// (stages / unit) must be a multiple of the dequant warpgroup count, so every
// round of a slot belongs to the same warpgroup: a warpgroup then can never
// wait on a slot more than one phase ahead (mbarrier parity would alias).
int qgemm_tc_stages(int box_rows) { return box_rows <= 64 ? 12 : 6; }

int qgemm_tc_unit(const TcArgs& a) {
  const int stages = qgemm_tc_stages(a.box_rows);
  const int kc = a.W.k_chunks();
  const int per = a.mode == kGemmStoreF32 ? (kc + a.splits - 1) / a.splits : kc;
  const bool even_split = a.mode != kGemmStoreF32 || per * a.splits == kc;
  for (int u : {4, 2})
    if (per % u == 0 && even_split && stages % u == 0 && (stages / u) % kDequantGroups == 0) return u;
  return 1;
}

// One wave at most: row tiles x splits <= SM count (rounded down, so a matrix
// with more row tiles than half the SMs runs unsplit). Every extra split adds
// a T x rows fp32 partial that the epilogue writes and the consumer re-reads,
// and a CTA with several short items pays an epilogue per item. On B200 at 64
// decode tokens (configs[1] shapes) the DeltaNet in_proj (97 row tiles) ran the
// 48-layer step in 14.66 ms unsplit, 14.80 with 2 splits and 14.91 with 4
// (two waves); out_proj and the router (16 and 5 row tiles) keep 8 splits,
// and capping them at 2 cost 0.13 ms per step.
int qgemm_tc_split_target(int row_tiles, int kc, int sm_count, int max_splits) {
  return std::max(1, std::min({std::max(1, sm_count / std::max(1, row_tiles)), max_splits, kc}));
}

void launch_qgemm_tc(const CUtensorMap& bmap, TcArgs a, int sm_count, cudaStream_t s) {
  if (a.box_rows != 16 && a.box_rows != 32 && a.box_rows != 64 && a.box_rows != 128)
    throw std::invalid_argument("tcgen05 GEMM box rows must be 16, 32, 64 or 128");
  if (a.mode == kGemmStoreF32 && a.n_tokens <= 0) return;
  if (a.mode != kGemmStoreF32 && a.groups > kMaxGroups) throw std::invalid_argument("too many GEMM groups");
  a.stages = qgemm_tc_stages(a.box_rows);
  a.b_stages = qgemm_tc_bstages(a.box_rows);
  a.unit = qgemm_tc_unit(a);  // largest of 4, 2, 1 dividing the items and the ring (slots % groups == 0)
  if ((a.stages / a.unit) % kDequantGroups) throw std::logic_error("GEMM unit slots not a multiple of warpgroups");
  if (a.b_stages % a.unit || a.b_stages < a.stages || (a.b_stages / a.unit) % kDequantGroups)
    throw std::logic_error("GEMM activation ring geometry");
  const size_t smem = qgemm_tc_smem(a.box_rows, a.stages, a.unit);
  static std::atomic<uint64_t> configured{0};
  once_per_device(configured, [] {
    QWEN_CUDA(cudaFuncSetAttribute(qgemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
  });
  if (a.mode == kGemmStoreF32 && a.token_group > 0 && (a.token_group % a.box_rows || a.splits != 1))
    throw std::invalid_argument("GEMM token groups must be whole boxes, without split-K");
  // grouped: the item count (token blocks x row tiles) is known on the device only
  const int items = a.mode == kGemmStoreF32 ? a.W.row_tiles * a.splits * dense_token_groups(a) : sm_count;
  const int grid = std::max(1, std::min(items, sm_count));
  if (smem > 227 * 1024) throw std::invalid_argument("tcgen05 GEMM shared memory above 227 KB");
  launch_pdl(qgemm_tc_kernel, grid, kThreads, smem, s, bmap, a);
  QWEN_CUDA(cudaGetLastError());
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
}

// ---------------------------------------------------------------- tensor maps --
namespace {
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    QWEN_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !p) throw std::runtime_error("cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}
}  // namespace

CUtensorMap make_act_map(const void* base, int rows, int k, int box_rows) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (k * 2) % 16)
    throw std::invalid_argument("activation tensor map alignment");
  CUtensorMap m;
  const cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(k) * 2};
  const cuuint32_t box[2] = {cuuint32_t(kTileK), cuuint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
  return m;
}

CUtensorMap make_act_map3d(const void* base, int rows, int k, int box_rows, int unit) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (k * 2) % 16 || k % kTileK)
    throw std::invalid_argument("activation tensor map alignment");
  CUtensorMap m;
  // X[rows][k] viewed as [k/64 chunks][rows][64]: one box = `unit` chunk tiles
  const cuuint64_t dims[3] = {cuuint64_t(kTileK), cuuint64_t(rows), cuuint64_t(k / kTileK)};
  const cuuint64_t strides[2] = {cuuint64_t(k) * 2, cuuint64_t(kTileK) * 2};
  const cuuint32_t box[3] = {cuuint32_t(kTileK), cuuint32_t(box_rows), cuuint32_t(unit)};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (3-D activations) failed: " + std::to_string(int(r)));
  return m;
}

CUtensorMap make_kv_map(const KvPool& kv, int layer) {
  CUtensorMap m;
  const void* base = kv.page(layer, 0);
  const cuuint64_t rows = cuuint64_t(kv.n_pages) * 2 * kv.Hkv * kPageTokens;
  const cuuint64_t dims[2] = {cuuint64_t(kv.D), rows};
  const cuuint64_t strides[1] = {cuuint64_t(kv.D) * 2};
  const cuuint32_t box[2] = {64, cuuint32_t(kPageTokens)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (KV) failed: " + std::to_string(int(r)));
  return m;
}

}  // namespace qwen
