// 4-bit affine (group 64 scale/bias) grouped GEMM on CUDA cores: Y = X * deq(W)^T.
//
// CUDA-core implementation: one CTA per 128-row weight tile; each thread owns
// one weight row, dequantizes its 64-column slice of each tile in registers
// and accumulates up to 32 token rows staged in shared memory. Modes:
//  - dense (kGemmStoreF32): split-K slices write separate fp32 partials;
//  - grouped experts (kGemmGateUp / kGemmDown): blockIdx.z = expert, tokens of
//    the expert are the sorted assignment rows [off[e], off[e+1]).
#include <atomic>

#include "kernels.h"

namespace qwen {

extern std::atomic<uint64_t> g_kernel_launches;
static inline void count_launch_external() { g_kernel_launches.fetch_add(1, std::memory_order_relaxed); }

namespace {

constexpr int kTok = 32;

__global__ void __launch_bounds__(128) qgemm_simple_kernel(GemmArgs a) {
  __shared__ float xs[kTok][kTileK + 1];
  __shared__ float ex[kTileRows][kTok + 1];
  const int r = threadIdx.x;
  const int g = blockIdx.z;
  int row_tile, p0, p1;
  if (a.mode == kGemmStoreF32) {
    row_tile = blockIdx.x;
    p0 = 0;
    p1 = a.n_tokens;
  } else {
    p0 = a.group_off[g];
    p1 = a.group_off[g + 1];
    if (p0 == p1) return;
    row_tile = g * a.expert_tiles + blockIdx.x;
  }
  const int kc = a.W.k_chunks();
  const int split = blockIdx.y;
  const int c_per = (kc + a.splits - 1) / a.splits;
  const int c0 = split * c_per, c1 = min(kc, c0 + c_per);
  for (int tb = p0; tb < p1; tb += kTok) {
    const int nt = min(kTok, p1 - tb);
    float acc[kTok];
#pragma unroll
    for (int i = 0; i < kTok; ++i) acc[i] = 0.f;
    for (int c = c0; c < c1; ++c) {
      __syncthreads();
      for (int e = threadIdx.x; e < kTok * kTileK; e += blockDim.x) {
        const int i = e / kTileK, k = e % kTileK;
        float v = 0.f;
        if (i < nt) {
          const int p = tb + i;
          const int xr = a.x_row ? a.x_row[p] / a.x_div : p;
          v = __half2float(a.X[size_t(xr) * a.ldx + c * kTileK + k]);
        }
        xs[i][k] = v;
      }
      __syncthreads();
      const uint8_t* tile = a.W.tile(row_tile, c);
      const uint4* pk = reinterpret_cast<const uint4*>(tile + r * 32);
      const uint4 w0 = pk[0], w1 = pk[1];
      const float sc = half_bits_to_float(reinterpret_cast<const uint16_t*>(tile + kTilePackedBytes)[r]) * (1.f / kTileScale);
      const float bi = half_bits_to_float(
          reinterpret_cast<const uint16_t*>(tile + kTilePackedBytes + kTileRows * 2)[r]);
      const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
      float w[kTileK];
#pragma unroll
      for (int j = 0; j < kTileK; ++j) w[j] = fmaf(sc, float(nibble(words[j / 8], j % 8)), bi);
#pragma unroll
      for (int i = 0; i < kTok; ++i) {
        if (i < nt) {
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < kTileK; ++j) s += w[j] * xs[i][j];
          acc[i] += s;
        }
      }
    }
    if (a.mode == kGemmStoreF32) {
      const int n = row_tile * kTileRows + r;
      if (n < a.W.rows) {
        float* y = a.Y + size_t(split) * a.split_stride;
        for (int i = 0; i < nt; ++i) y[size_t(tb + i) * a.ldy + n] = acc[i];
      }
    } else if (a.mode == kGemmDown) {
      const int n = blockIdx.x * kTileRows + r;
      for (int i = 0; i < nt; ++i) a.Y[size_t(tb + i) * a.ldy + n] = acc[i];
    } else {  // gate/up: rows [0,64) gate, [64,128) up of intermediate j = blockIdx.x*64 + r
      __syncthreads();
      for (int i = 0; i < kTok; ++i) ex[r][i] = acc[i];
      __syncthreads();
      if (r < 64) {
        const int j = blockIdx.x * 64 + r;
        for (int i = 0; i < nt; ++i) {
          const float gv = ex[r][i], uv = ex[r + 64][i];
          a.Yb[size_t(tb + i) * a.ldyb + j] = to_gemm_in(gv / (1.f + __expf(-gv)) * uv);
        }
      }
    }
  }
}

// Dense fp16 weight rows (checkpoint modules outside 4-bit g64):
// Y[t][n] = sum_k X[t][k] * W[n][k], fp32 accumulation. One warp per output
// row and block of 8 tokens; each lane reads 8 consecutive halves (16 bytes) of
// the row and of each token per step.
__global__ void __launch_bounds__(256) dense_f16_kernel(const __half* __restrict__ W, int rows, int K,
                                                        const __half* __restrict__ X, int T, float* __restrict__ Y,
                                                        int ldy) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + warp, t0 = blockIdx.y * 8;
  if (n >= rows) return;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  const __half* w = W + size_t(n) * K;
  for (int k = lane * 8; k < K; k += 256) {
    const uint4 wv = *reinterpret_cast<const uint4*>(w + k);
    const __half2* wh = reinterpret_cast<const __half2*>(&wv);
    float2 wf[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) wf[j] = __half22float2(wh[j]);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      if (t0 + t >= T) break;
      const uint4 xv = *reinterpret_cast<const uint4*>(X + size_t(t0 + t) * K + k);
      const __half2* xh = reinterpret_cast<const __half2*>(&xv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 xf = __half22float2(xh[j]);
        acc[t] = fmaf(wf[j].x, xf.x, acc[t]);
        acc[t] = fmaf(wf[j].y, xf.y, acc[t]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const float v = warp_sum(acc[t]);
    if (lane == 0 && t0 + t < T) Y[size_t(t0 + t) * ldy + n] = v;
  }
}

}  // namespace

void launch_dense_f16(const QMat& W, const gemm_in_t* X, int T, float* Y, int ldy, cudaStream_t s) {
  if (!W.dense_f16) throw std::logic_error("dense fp16 kernel on a tiled matrix");
  if (T <= 0) return;
  if (W.k % 64 || (reinterpret_cast<uintptr_t>(X) & 15) || (reinterpret_cast<uintptr_t>(W.tiles) & 15))
    throw std::invalid_argument("dense fp16 projection alignment");
  dim3 grid((W.rows + 7) / 8, (T + 7) / 8);
  dense_f16_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const __half*>(W.tiles), W.rows, W.k, X, T, Y, ldy);
  QWEN_CUDA(cudaGetLastError());
  count_launch_external();
}

void launch_qgemm(const GemmArgs& a, cudaStream_t s) {
  dim3 grid;
  if (a.mode == kGemmStoreF32) {
    if (a.n_tokens <= 0) return;
    grid = dim3(a.W.row_tiles, a.splits, 1);
  } else {
    grid = dim3(a.expert_tiles, 1, a.groups);
  }
  qgemm_simple_kernel<<<grid, 128, 0, s>>>(a);
  count_launch_external();
}

}  // namespace qwen
