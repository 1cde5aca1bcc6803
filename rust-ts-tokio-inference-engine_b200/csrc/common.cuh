// Shared definitions for the B200 ragged hybrid-Qwen decode step.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <stdexcept>
#include <string>
#include <utility>

#define QWEN_CUDA(call)                                                                    \
  do {                                                                                     \
    cudaError_t qwen_err_ = (call);                                                        \
    if (qwen_err_ != cudaSuccess)                                                          \
      throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(qwen_err_) + \
                               " at " + __FILE__ + ":" + std::to_string(__LINE__));        \
  } while (0)

namespace qwen {

// Runs `setup` the first time it is reached on the calling thread's current
// CUDA device, once per device: kernel attributes such as the dynamic
// shared-memory limit are per-device state, so a process that drives several
// GPUs must set them on each. `seen` holds one bit per device (devices past
// 63 simply repeat the cheap setup on every call).
template <class F>
inline void once_per_device(std::atomic<uint64_t>& seen, F setup) {
  int dev = 0;
  QWEN_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = dev >= 0 && dev < 64 ? uint64_t(1) << dev : 0;
  if (bit && (seen.load(std::memory_order_acquire) & bit)) return;
  setup();
  if (bit) seen.fetch_or(bit, std::memory_order_release);
}

// 4-bit affine g64 weight tile: 128 rows x 64 columns (one quant group per row).
// Layout: packed nibbles [128 rows][8 uint32 words], then 128 scales, then 128
// biases, IEEE half. The bias is the checkpoint's bf16 value and the scale is
// that value times kTileScale (512), both exact (every bf16 value of magnitude
// >= 2^-17, and zero, is an fp16 value, and so is 512 s for s < 128; the
// loaders reject others). Word w of a row holds columns 8w..8w+7 with column
// c in nibble nibble_of_col(c) = {0,2,4,6,1,3,5,7}[c]: the bytes of
// (word & 0x0F0F0F0F) then hold columns (0,1 | 2,3) and those of
// ((word >> 4) & 0x0F0F0F0F) columns (4,5 | 6,7), each byte a nibble that an
// e4m3 conversion reads as exactly q * 2^-9. A matrix [rows, K] is stored as
// [ceil(rows/128) row tiles][K/64 column chunks] tiles, each 4608 bytes, so one
// tile is one contiguous bulk copy.
constexpr int kTileRows = 128;
constexpr int kTileK = 64;
constexpr int kTilePackedBytes = kTileRows * kTileK / 2;  // 4096
constexpr int kTileBytes = kTilePackedBytes + kTileRows * 2 * 2;  // 4608
constexpr int kPageTokens = 16;  // paged-KV page size (tokens)
// Routed experts per MoE layer the routing kernels hold (route_kernel keeps
// four experts per thread of a 256-thread CTA; the sort's shared tables scale
// with the expert count).
constexpr int kMaxExperts = 1024;

// Nibble index holding column c (0..7) of a packed word, and its inverse.
__host__ __device__ __forceinline__ int nibble_of_col(int c) { return c < 4 ? 2 * c : 2 * (c - 4) + 1; }
__host__ __device__ __forceinline__ int col_of_nibble(int i) { return (i & 1) ? 4 + (i >> 1) : (i >> 1); }
// Tile scales are stored times this power of two (see above).
constexpr float kTileScale = 512.f;
__device__ __forceinline__ uint32_t nibble(uint32_t word, int col) { return (word >> (4 * nibble_of_col(col))) & 15u; }

struct QMat {
  const uint8_t* tiles = nullptr;
  int rows = 0;       // logical output rows
  int row_tiles = 0;  // ceil(rows / 128)
  int k = 0;          // input width (multiple of 64)
  // true: `tiles` holds dense fp16 rows [rows][k] (checkpoint modules outside
  // 4-bit g64: quantization overrides or float weights), run by the CUDA-core
  // dense kernel instead of the tcgen05 GEMM
  bool dense_f16 = false;
  __host__ __device__ int k_chunks() const { return k / kTileK; }
  __host__ __device__ const uint8_t* tile(int row_tile, int chunk) const {
    return tiles + (size_t(row_tile) * (k / kTileK) + chunk) * kTileBytes;
  }
};

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(uint32_t(b) << 16);
}

// Element type of every projection input (the activations the tcgen05 GEMM
// reads as its B operand) and of the dequantised weights (its A operand):
// IEEE half. Its 11-bit significand rounds scale*q + bias and each activation
// 8x more finely than bfloat16 (the end-to-end logits error of a decode step
// drops by about that factor), and the values that enter a projection
// (RMS-normalised rows, gated attention / DeltaNet outputs, SwiGLU products)
// stay far inside its range.
using gemm_in_t = __half;
__device__ __forceinline__ gemm_in_t to_gemm_in(float v) { return __float2half_rn(v); }
__device__ __forceinline__ __half2 to_gemm_in2(float a, float b) { return __floats2half2_rn(a, b); }
__host__ __device__ __forceinline__ float half_bits_to_float(uint16_t b) {
#ifdef __CUDA_ARCH__
  return __half2float(__ushort_as_half(b));
#else
  // host: widen IEEE binary16 exactly
  const uint32_t sign = uint32_t(b & 0x8000u) << 16, ex = (b >> 10) & 0x1Fu, man = b & 0x3FFu;
  uint32_t u;
  if (ex == 0x1F) {
    u = sign | 0x7F800000u | (man << 13);
  } else if (ex) {
    u = sign | ((ex + 112u) << 23) | (man << 13);
  } else if (!man) {
    u = sign;
  } else {  // subnormal: normalise
    int e = -1;
    uint32_t m = man;
    do { m <<= 1; ++e; } while (!(m & 0x400u));
    u = sign | (uint32_t(112 - e) << 23) | ((m & 0x3FFu) << 13);
  }
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}
// bf16 bits -> the fp16 bits of the same value; false when fp16 cannot hold it exactly.
__host__ __device__ __forceinline__ bool bf16_to_half_bits(uint16_t b, uint16_t* out) {
  const uint32_t sign = (b & 0x8000u) ? 0x8000u : 0u;
  const int ex = (b >> 7) & 0xFF, man = b & 0x7F;
  if (ex == 0 && man == 0) { *out = uint16_t(sign); return true; }
  if (ex == 0xFF) return false;
  const int e = ex - 127;  // value = 1.man * 2^e (bf16 subnormals are below fp16's range)
  if (ex == 0) return false;
  if (e > 15) return false;
  if (e >= -14) { *out = uint16_t(sign | uint32_t(e + 15) << 10 | uint32_t(man) << 3); return true; }
  // fp16 subnormal: value = m * 2^-24 with m = (128 + man) * 2^(e + 24 - 7)
  const int shift = e + 17;  // left shift of (128+man) if >= 0
  if (shift < 0) {
    const uint32_t full = 128u + uint32_t(man);
    if (full & ((1u << -shift) - 1u)) return false;
    *out = uint16_t(sign | (full >> -shift));
    return true;
  }
  *out = uint16_t(sign | ((128u + uint32_t(man)) << shift));
  return true;
}

// Round-to-nearest-even narrowing to bf16 bits (matches the host generator).
__host__ __device__ __forceinline__ uint16_t float_to_bf16_bits(float f) {
#ifdef __CUDA_ARCH__
  uint32_t u = __float_as_uint(f);
#else
  uint32_t u;
  memcpy(&u, &f, 4);
#endif
  if ((u & 0x7F800000u) == 0x7F800000u) return uint16_t((u >> 16) | ((u & 0xFFFF) ? 0x40 : 0));
  u += 0x7FFFu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }
__device__ __forceinline__ float siluf_(float x) { return x / (1.0f + __expf(-x)); }

// IEEE total-order key: -0 < +0, matches Rust f32::total_cmp for finite values.
__device__ __forceinline__ uint32_t total_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u ^ 0x80000000u);
}

// Counter-based hash (splitmix64 finalizer) and the Irwin-Hall(4) normal
// approximation used by the seeded synthetic generators.
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ float synth_normal(uint64_t key, uint64_t index, float k) {
  uint64_t h = mix64(key ^ (index * 0xD1B54A32D192ED03ull));
  int32_t s = int32_t(h & 0xFFFF) + int32_t((h >> 16) & 0xFFFF) + int32_t((h >> 32) & 0xFFFF) +
              int32_t(h >> 48);
  return __fmul_rn(float(s - 131070), k);
}

// Error flags raised by kernels and read back by the host after a step.
enum ErrorBits : uint32_t {
  kErrNonFinite = 1u,
  kErrBounds = 2u,
  kErrTimeout = 4u,
};

// Programmatic dependent launch. Every step kernel is launched with
// programmatic stream serialisation: it calls pdl_trigger() on entry so the
// next kernel may start launching, and pdl_wait() before it touches memory
// that earlier kernels of the stream write (pdl_wait returns once they have
// completed and their writes are visible; without a programmatic predecessor
// it returns at once).
//
// pdl_wait(p, q, ...) takes the kernel's __restrict__ pointer parameters.
// The wait's memory clobber does not order accesses through a __restrict__
// pointer (restrict promises the compiler that nothing else touches that
// data), so the compiler may schedule such loads before the wait, where they
// can read what the still-running predecessor has not written yet. Each
// pointer is therefore passed through an empty asm after the wait: every
// access through it then depends on an instruction that follows the wait.
template <typename P>
__device__ __forceinline__ void pdl_reseat(P& p) {
  uint64_t v = reinterpret_cast<uint64_t>(p);
  asm volatile("" : "+l"(v));
  p = reinterpret_cast<P>(v);
}
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
template <typename... P>
__device__ __forceinline__ void pdl_wait(P&... ptrs) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  (pdl_reseat(ptrs), ...);
}

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QWEN_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

}  // namespace qwen
