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
      const float sc = half_bits_to_float(reinterpret_cast<const uint16_t*>(tile + kTilePackedBytes)[r]);
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

}  // namespace

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
