// Allocation-free dense projection: the split-K tcgen05 4-bit GEMM with its
// split partials in a fixed, file-scope device array instead of session or
// caller buffers, followed by a fixed-order reduction into the caller's output.
//
// Scratch: kScratchBytes (16 MiB) of static device memory per device, shared
// by every call on that device. The first 256 bytes hold the call's device
// status word (the GEMM's error bits), which must start at zero and is cleared
// on the stream at the start of each call; the split partials that follow need
// no initial value (every element the reduction reads is written by the GEMM
// of the same call). Calls that overlap in time on one device race on the
// array and corrupt each other's results, so callers serialise them.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "noalloc.h"
#include "qgemm_tc.h"

namespace {
constexpr size_t kScratchBytes = size_t(16) << 20;
}  // namespace

// The scratch array: one copy per device, in the library's device image.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

namespace qwen {

extern std::atomic<uint64_t> g_kernel_launches;

namespace {

constexpr size_t kStatusBytes = 256;
constexpr size_t kPartialFloats = (kScratchBytes - kStatusBytes) / sizeof(float);
constexpr int kMaxDevices = 64;

std::mutex g_setup_mu;

// Formats into the caller's buffer (nothing when it is null or empty).
void fail(char* error, size_t capacity, const char* fmt, ...) {
  if (!error || !capacity) return;
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(error, capacity, fmt, ap);
  va_end(ap);
}

void* g_scratch_ptr[kMaxDevices] = {};

// Resolves this device's copy of the array once (the device must be current).
void* scratch_for_current_device(char* error, size_t capacity, bool* ok) {
  int dev = -1;
  cudaError_t rc = cudaGetDevice(&dev);
  if (rc != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    fail(error, capacity, "no-alloc projection: cudaGetDevice failed (%s)", cudaGetErrorString(rc));
    *ok = false;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    rc = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (rc != cudaSuccess || !p) {
      fail(error, capacity, "no-alloc projection: cudaGetSymbolAddress failed on device %d (%s)", dev,
                    cudaGetErrorString(rc));
      *ok = false;
      return nullptr;
    }
    g_scratch_ptr[dev] = p;
  }
  *ok = true;
  return g_scratch_ptr[dev];
}

// y[i] = ((0 + p_0[i]) + p_1[i]) + ... : the split order every other caller of
// the split-K GEMM sums in.
__global__ void reduce_partials_kernel(const float* __restrict__ part, int splits, size_t n, float* __restrict__ y) {
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    float v = 0.f;
    for (int s = 0; s < splits; ++s) v += part[s * n + i];
    y[i] = v;
  }
}

}  // namespace

size_t noalloc_scratch_bytes() { return kScratchBytes; }

int project_noalloc(const QMat& W, int max_splits, const gemm_in_t* x, int T, float* y, int sm_count,
                    cudaStream_t s, char* error, size_t capacity) {
  if (W.dense_f16) {
    fail(error, capacity, "no-alloc projection: the matrix is held as dense fp16 rows (a checkpoint module "
                          "outside 4-bit g64); this entry point runs the 4-bit tensor-core GEMM only");
    return -1;
  }
  if (!x || !y || T <= 0 || size_t(T) > kPartialFloats) {
    fail(error, capacity, "no-alloc projection: null buffer or token count outside [1, %zu]", kPartialFloats);
    return -1;
  }
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 3)) {
    fail(error, capacity, "no-alloc projection: x must be 16-byte and y 4-byte aligned");
    return -1;
  }
  const size_t n = size_t(T) * size_t(W.rows);
  if (n > kPartialFloats) {
    fail(error, capacity,
                  "no-alloc projection: %d tokens x %d rows = %zu floats exceeds the %zu-float scratch (16 MiB); "
                  "split the tokens into smaller calls",
                  T, W.rows, n, kPartialFloats);
    return -1;
  }
  bool ok = false;
  unsigned char* base = static_cast<unsigned char*>(scratch_for_current_device(error, capacity, &ok));
  if (!ok) return -1;
  uint32_t* status = reinterpret_cast<uint32_t*>(base);
  float* part = reinterpret_cast<float*>(base + kStatusBytes);

  // split-K choice of the session's dense projection, then capped so all
  // partials fit the scratch
  TcArgs a;
  a.W = W;
  a.mode = kGemmStoreF32;
  a.n_tokens = T;
  const int tb = std::min(T, 128);
  a.box_rows = tb <= 16 ? 16 : tb <= 32 ? 32 : tb <= 64 ? 64 : 128;
  const int kc = W.k_chunks();
  const int want = qgemm_tc_split_target(W.row_tiles, kc, sm_count, max_splits);
  int splits = 1;
  for (int sp = want; sp >= 1; --sp)
    if (kc % sp == 0 && (kc / sp) % 4 == 0 && size_t(sp) * n <= kPartialFloats) {
      splits = sp;
      break;
    }
  a.splits = splits;
  a.split_stride = n;
  a.Y = part;
  a.ldy = W.rows;
  a.err = status;

  cudaError_t rc = cudaMemsetAsync(status, 0, sizeof(uint32_t), s);
  if (rc != cudaSuccess) {
    fail(error, capacity, "no-alloc projection: status clear failed (%s)", cudaGetErrorString(rc));
    return -1;
  }
  try {
    launch_qgemm_tc(make_act_map3d(x, T, W.k, a.box_rows, qgemm_tc_unit(a)), a, sm_count, s);
  } catch (const std::exception& e) {
    fail(error, capacity, "no-alloc projection: %s", e.what());
    return -1;
  }
  const int threads = 256;
  const int blocks = int(std::min<size_t>((n + threads - 1) / threads, size_t(sm_count) * 8));
  reduce_partials_kernel<<<blocks, threads, 0, s>>>(part, splits, n, y);
  rc = cudaGetLastError();
  if (rc != cudaSuccess) {
    fail(error, capacity, "no-alloc projection: reduction launch failed (%s)", cudaGetErrorString(rc));
    return -1;
  }
  g_kernel_launches.fetch_add(1, std::memory_order_relaxed);
  uint32_t h_status = 0;
  rc = cudaMemcpyAsync(&h_status, status, sizeof(h_status), cudaMemcpyDeviceToHost, s);
  if (rc == cudaSuccess) rc = cudaStreamSynchronize(s);
  if (rc != cudaSuccess) {
    fail(error, capacity, "no-alloc projection: %s", cudaGetErrorString(rc));
    return -1;
  }
  if (h_status) {
    fail(error, capacity, "no-alloc projection: device error flag %u", h_status);
    return -1;
  }
  return 0;
}

}  // namespace qwen
