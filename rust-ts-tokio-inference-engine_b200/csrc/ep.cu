// Expert parallelism for the MoE block (the survey's multi-GPU mode (b)):
// routed experts are split into `world` contiguous blocks, rank r owning
// experts [r*E/world, (r+1)*E/world); every rank keeps its own sequences and
// computes the shared expert (id E) for its own tokens.
//
// Per MoE layer, after the local routing and the stable sort (whose expert
// order already groups a rank's assignments by owner):
//   ep_pack          per peer p: a stage = [counts of p's experts][rows], the
//                    rows being the sorted gathered activations of the
//                    assignments p owns (contiguous in the sort);
//   transport        either direct NVLink stores of the valid rows into the
//                    owner's window (CUDA IPC mapping) followed by an epoch
//                    flag (release at system scope, set by the last CTA), or
//                    NCCL send/recv of fixed-size stages (cap rows each);
//   ep_plan          per local expert: rows from every source, in source
//                    order (then the source's sort order), and the shared
//                    expert's local rows last -> group offsets over E + 1
//                    experts for the grouped GEMM (non-local experts empty);
//   ep_gather        those rows into one fp16 matrix, with each row's origin;
//   grouped GEMMs    (unchanged) over the local rows;
//   ep_return_pack   each result row into its source's return stage (fp32);
//   transport        the same way back (flags / NCCL);
//   ep_return_unpack every local assignment's result row back to its sorted
//                    position, so the mixture runs unchanged.
// A token's expert rows see the same arithmetic as on one GPU (the GEMM's
// result does not depend on the other rows of its batch), so expert-parallel
// logits equal the single-GPU ones bit for bit.
#include <atomic>
#include <cstdint>

#include "kernels.h"

namespace qwen {

extern std::atomic<uint64_t> g_kernel_launches;

namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
constexpr long long kEpWaitCycles = 4000000000ll;  // ~2 s at 1.9 GHz

// Threads 0..world-1 wait (bounded) until flags[t] has reached `epoch`; on
// expiry kTimeout is raised and the CTA goes on (its results are then void).
__device__ __forceinline__ void ep_wait_flags(const uint32_t* flags, int world, uint32_t epoch, uint32_t* err) {
  if (flags && threadIdx.x < world) {
    const long long t0 = clock64();
    while (int32_t(ld_acquire_sys(flags + threadIdx.x) - epoch) < 0) {
      if (clock64() - t0 > kEpWaitCycles) {
        atomicOr(err, kErrTimeout);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
}

// After every CTA of the grid has written its rows: the last one (device
// counter, which it resets) publishes `epoch` to every peer's flag.
__device__ __forceinline__ void ep_signal_last(uint32_t* const* flag_dst, int world, uint32_t epoch, uint32_t* done) {
  if (!flag_dst) return;
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) {
    __threadfence_system();  // this CTA's stores (local and remote) before its arrival
    last = atomicAdd(done, 1u) == gridDim.x * gridDim.y - 1;
  }
  __syncthreads();
  if (!last) return;
  if (threadIdx.x == 0) {
    __threadfence_system();
    *done = 0;
  }
  if (threadIdx.x < world) st_release_sys(flag_dst[threadIdx.x], epoch);
}

// Stage layout: [hdr_ints int32 counts (padded to 16 B)] [cap rows x H fp16]
// Rows come straight from the MoE input: sorted position q is row perm[q] / div
// of `src` (stride ld), so no gathered copy is made first.
__global__ void ep_pack_kernel(const gemm_in_t* __restrict__ src, int ld, const int32_t* __restrict__ perm,
                               int div, const int32_t* __restrict__ counts,
                               const int32_t* __restrict__ offsets, uint8_t* const* __restrict__ dst,
                               int per_rank, int hdr_ints, int cap, int H, uint32_t* const* flag_dst, uint32_t epoch,
                               uint32_t* done) {
  pdl_trigger();
  pdl_wait(src, perm, counts, offsets, dst);
  const int p = blockIdx.y;
  uint8_t* st = dst[p];
  const int e0 = p * per_rank;
  if (blockIdx.x == 0)
    for (int j = threadIdx.x; j < hdr_ints; j += blockDim.x)
      reinterpret_cast<int32_t*>(st)[j] = j < per_rank ? counts[e0 + j] : 0;
  const int r0 = offsets[e0], n = offsets[e0 + per_rank] - r0;
  gemm_in_t* rows = reinterpret_cast<gemm_in_t*>(st + size_t(hdr_ints) * 4);
  const int h8 = H / 8;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < n * h8; idx += gridDim.x * blockDim.x) {
    if (idx / h8 >= cap) break;  // cannot happen: n <= cap is checked by the planner of the step
    const int row = idx / h8, c = idx - row * h8;
    reinterpret_cast<uint4*>(rows + size_t(row) * H)[c] =
        reinterpret_cast<const uint4*>(src + size_t(perm[r0 + row] / div) * ld)[c];
  }
  ep_signal_last(flag_dst, gridDim.y, epoch, done);
}

// Exclusive scan of v[0..n) by one warp (each lane a consecutive run of
// ceil(n/32) entries, then a shuffle scan of the run totals); returns the total.
__device__ int warp_exclusive_scan(const int32_t* v, int32_t* out, int n, int lane) {
  const int per = (n + 31) / 32, b = lane * per, e = min(n, b + per);
  int run = 0;
  for (int i = b; i < e; ++i) run += v[i];
  int incl = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  int acc = incl - run;
  for (int i = b; i < e; ++i) {
    const int c = v[i];
    out[i] = acc;
    acc += c;
  }
  return __shfl_sync(0xffffffffu, incl, 31);
}

// One CTA: group offsets over E + 1 experts of the local rows and, for every
// (local expert e, source p) segment, its first row in p's stage and in the
// local matrix: seg[(e * world + p) * 2 + {0, 1}]. goff[E + 1] ends the shared
// expert's rows; a source sending more than `cap` rows raises kErrBounds.
__global__ void ep_plan_kernel(const uint8_t* const* __restrict__ srcs, int world, int rank, int per_rank, int E,
                               const int32_t* __restrict__ counts, int32_t* __restrict__ goff,
                               int32_t* __restrict__ seg, int32_t* __restrict__ n_rows, uint32_t* err, int cap,
                               const uint32_t* wait_flags, uint32_t epoch) {
  pdl_trigger();
  pdl_wait(srcs, counts, goff, seg, n_rows);
  ep_wait_flags(wait_flags, world, epoch, err);
  extern __shared__ int32_t sm[];
  const int n = world * per_rank;
  int32_t* cnt_pe = sm;           // [world][per_rank]  (stage order)
  int32_t* cnt_ep = sm + n;       // [per_rank][world]  (local order)
  int32_t* sc_pe = sm + 2 * n;    // exclusive scans of the two orders
  int32_t* sc_ep = sm + 3 * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int p = i / per_rank, e = i - p * per_rank;
    const int c = reinterpret_cast<const int32_t*>(srcs[p])[e];
    cnt_pe[i] = c;
    cnt_ep[e * world + p] = c;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int total = 0;
  if (warp == 0) total = warp_exclusive_scan(cnt_ep, sc_ep, n, lane);
  if (warp == 1) warp_exclusive_scan(cnt_pe, sc_pe, n, lane);  // restarts per source below
  __syncthreads();
  const int e_lo = rank * per_rank;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int e = i / world, p = i - e * world;
    // first row of (e, p) in p's stage = scan in stage order minus p's start
    seg[i * 2] = sc_pe[p * per_rank + e] - sc_pe[p * per_rank];
    seg[i * 2 + 1] = sc_ep[i];
  }
  for (int g = threadIdx.x; g < e_lo; g += blockDim.x) goff[g] = 0;
  for (int e = threadIdx.x; e < per_rank; e += blockDim.x) goff[e_lo + e] = sc_ep[e * world];
  __syncthreads();
  if (warp == 0) {
    const int routed = __shfl_sync(0xffffffffu, total, 0);
    for (int g = e_lo + per_rank + lane; g <= E; g += 32) goff[g] = routed;  // later routed experts empty; shared starts
    for (int p = lane; p < world; p += 32) {
      const int sent = (p + 1 < world ? sc_pe[(p + 1) * per_rank] : routed) - sc_pe[p * per_rank];
      if (sent > cap) atomicOr(err, kErrBounds);
    }
    if (lane == 0) {
      goff[E + 1] = routed + counts[E];
      *n_rows = routed + counts[E];
    }
  }
}

// Copy the routed rows of every (local expert, source) segment and the
// shared expert's local rows into the local matrix; origin[row] = p * cap +
// stage row for routed rows, -1 - sorted position for shared rows.
__global__ void ep_gather_kernel(const uint8_t* const* __restrict__ srcs, int world, int per_rank, int hdr_ints,
                                 int E, const int32_t* __restrict__ goff, const int32_t* __restrict__ seg,
                                 const int32_t* __restrict__ offsets, const gemm_in_t* __restrict__ xsrc, int ld,
                                 const int32_t* __restrict__ perm, int div,
                                 gemm_in_t* __restrict__ xloc, int32_t* __restrict__ origin, int cap, int H,
                                 int rank) {
  pdl_trigger();
  pdl_wait(srcs, goff, seg, offsets, xsrc, perm, xloc, origin);
  extern __shared__ int32_t sseg[];  // [per_rank * world][2]
  const int nseg = per_rank * world;
  for (int i = threadIdx.x; i < 2 * nseg; i += blockDim.x) sseg[i] = seg[i];
  __syncthreads();
  const int e_lo = rank * per_rank;
  const int n_routed = goff[e_lo + per_rank] - goff[e_lo];
  const int n_total = goff[E + 1] - goff[e_lo];
  const int h8 = H / 8;
  for (int row = blockIdx.x; row < n_total; row += gridDim.x) {
    const uint4* src;
    if (row < n_routed) {
      // the last (e, p) segment whose local start <= row (starts increase with
      // the index; empty segments share the next one's start and are skipped)
      int lo = 0, hi = nseg - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (sseg[mid * 2 + 1] <= row) lo = mid; else hi = mid - 1;
      }
      const int p = lo % world;
      const int srow = sseg[lo * 2] + (row - sseg[lo * 2 + 1]);
      src = reinterpret_cast<const uint4*>(srcs[p] + size_t(hdr_ints) * 4 + size_t(srow) * H * 2);
      if (threadIdx.x == 0) origin[row] = p * cap + srow;
    } else {
      const int q = offsets[E] + (row - n_routed);
      src = reinterpret_cast<const uint4*>(xsrc + size_t(perm[q] / div) * ld);
      if (threadIdx.x == 0) origin[row] = -1 - q;
    }
    uint4* dst = reinterpret_cast<uint4*>(xloc + size_t(row) * H);
    for (int c = threadIdx.x; c < h8; c += blockDim.x) dst[c] = src[c];
  }
}

// Result rows back: routed rows into their source's return stage (fp32,
// cap rows per source), shared rows straight into the sorted result matrix.
__global__ void ep_return_pack_kernel(const float* __restrict__ yloc, const int32_t* __restrict__ origin,
                                      const int32_t* __restrict__ n_rows, float* const* __restrict__ rdst,
                                      float* __restrict__ y_sorted, int cap, int H, int world,
                                      uint32_t* const* flag_dst, uint32_t epoch, uint32_t* done) {
  pdl_trigger();
  pdl_wait(yloc, origin, n_rows, rdst, y_sorted);
  const int n = *n_rows;
  const int h4 = H / 4;
  for (int row = blockIdx.x; row < n; row += gridDim.x) {
    const int o = origin[row];  // p * cap + stage row, or -1 - sorted position (shared expert)
    float* dst = o >= 0 ? rdst[o / cap] + size_t(o % cap) * H : y_sorted + size_t(-1 - o) * H;
    const float4* src = reinterpret_cast<const float4*>(yloc + size_t(row) * H);
    for (int c = threadIdx.x; c < h4; c += blockDim.x) reinterpret_cast<float4*>(dst)[c] = src[c];
  }
  ep_signal_last(flag_dst, world, epoch, done);
}

// Every local routed assignment's result from its owner's return stage.
__global__ void ep_return_unpack_kernel(const float* const* __restrict__ rsrcs, const int32_t* __restrict__ offsets,
                                        float* __restrict__ y_sorted, int world, int per_rank, int H,
                                        const uint32_t* wait_flags, uint32_t epoch, uint32_t* err) {
  pdl_trigger();
  pdl_wait(rsrcs, offsets, y_sorted);
  ep_wait_flags(wait_flags, world, epoch, err);
  const int n_routed = offsets[world * per_rank];
  const int h4 = H / 4;
  for (int q = blockIdx.x; q < n_routed; q += gridDim.x) {
    int p = 0;
    while (p + 1 < world && offsets[(p + 1) * per_rank] <= q) ++p;
    const int srow = q - offsets[p * per_rank];
    const float4* src = reinterpret_cast<const float4*>(rsrcs[p] + size_t(srow) * H);
    for (int c = threadIdx.x; c < h4; c += blockDim.x) reinterpret_cast<float4*>(y_sorted + size_t(q) * H)[c] = src[c];
  }
}

}  // namespace

void launch_ep_pack(const gemm_in_t* src, int ld, const int32_t* perm, int div, const int32_t* counts,
                    const int32_t* offsets, uint8_t* const* dst,
                    int world, int per_rank, int hdr_ints, int cap, int H, uint32_t* const* flag_dst, uint32_t epoch,
                    uint32_t* done, cudaStream_t s) {
  launch_pdl(ep_pack_kernel, dim3(64, world), 256, 0, s, src, ld, perm, div, counts, offsets, dst, per_rank, hdr_ints,
             cap, H,
             flag_dst, epoch, done);
  QWEN_CUDA(cudaGetLastError());
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
}

void launch_ep_plan_gather(const uint8_t* const* srcs, int world, int rank, int per_rank, int hdr_ints, int E,
                           const int32_t* counts, const int32_t* offsets, const gemm_in_t* xsrc, int ld,
                           const int32_t* perm, int div, int32_t* goff,
                           int32_t* seg, int32_t* n_rows, gemm_in_t* xloc, int32_t* origin, int cap, int H,
                           int max_rows, uint32_t* err, const uint32_t* wait_flags, uint32_t epoch, int sm_count,
                           cudaStream_t s) {
  const size_t n = size_t(world) * per_rank;
  if (4 * n * 4 > 48 * 1024) throw std::invalid_argument("expert-parallel plan: too many (expert, rank) segments");
  launch_pdl(ep_plan_kernel, 1, 256, 4 * n * 4, s, srcs, world, rank, per_rank, E, counts, goff, seg, n_rows, err, cap,
             wait_flags, epoch);
  launch_pdl(ep_gather_kernel, std::max(1, std::min(max_rows, 4 * sm_count)), 256, 2 * n * 4, s, srcs, world, per_rank,
             hdr_ints, E, goff, seg, offsets, xsrc, ld, perm, div, xloc, origin, cap, H, rank);
  QWEN_CUDA(cudaGetLastError());
  g_kernel_launches.fetch_add(2, std::memory_order_relaxed);
}

void launch_ep_return(const float* yloc, const int32_t* origin, const int32_t* n_rows, float* const* rdst,
                      float* y_sorted, int cap, int H, int world, int max_rows, uint32_t* const* flag_dst,
                      uint32_t epoch, uint32_t* done, int sm_count, cudaStream_t s) {
  launch_pdl(ep_return_pack_kernel, std::max(1, std::min(max_rows, 4 * sm_count)), 256, 0, s, yloc, origin, n_rows,
             rdst, y_sorted, cap, H, world, flag_dst, epoch, done);
  QWEN_CUDA(cudaGetLastError());
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
}

void launch_ep_return_unpack(const float* const* rsrcs, const int32_t* offsets, float* y_sorted, int world,
                             int per_rank, int H, int max_rows, const uint32_t* wait_flags, uint32_t epoch,
                             uint32_t* err, int sm_count, cudaStream_t s) {
  launch_pdl(ep_return_unpack_kernel, std::max(1, std::min(max_rows, 4 * sm_count)), 256, 0, s, rsrcs, offsets,
             y_sorted, world, per_rank, H, wait_flags, epoch, err);
  QWEN_CUDA(cudaGetLastError());
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
}

}  // namespace qwen
