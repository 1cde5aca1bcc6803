// Device session: state versions, paged-KV and DeltaNet pools, the ragged
// step executor and the rs_qwen_* C ABI (include/qwen_b200.h).
//
// Replaces the reference's MLX device session (native/qwen_device.inc,
// native/qwen_batch.inc). A state version (StateId) is one DeltaNet slot
// (recurrent state + conv history, fp32) plus a list of 16-token KV pages
// shared copy-on-write with its ancestors; parents are never mutated unless a
// step is asked to consume them.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstring>
#include <memory>
#include <numeric>
#include <string>
#include <vector>

#include <map>
#include <tuple>

#include <nccl.h>

#include "kernels.h"
#include "noalloc.h"
#include "qgemm_tc.h"
#include "state_table.h"

using namespace qwen;

namespace {

void report(char* error, size_t capacity, const char* message) noexcept {
  if (error && capacity) {
    const size_t n = std::min(std::strlen(message), capacity - 1);
    std::memcpy(error, message, n);
    error[n] = 0;
  }
}

// Error convention of native/mlx_bridge.cpp:19-31: 0 ok, -1 + message.
template <class F>
int checked(char* error, size_t capacity, F f) noexcept {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    report(error, capacity, e.what());
  } catch (...) {
    report(error, capacity, "unknown native CUDA exception");
  }
  return -1;
}

uint64_t allocate_owner() {
  static std::atomic<uint64_t> next{1};
  uint64_t owner = next.load();
  for (;;) {
    if (!owner || owner >= UINT64_MAX - 1) throw std::overflow_error("session owner exhausted");
    if (next.compare_exchange_weak(owner, owner + 2)) return owner;
  }
}

uint64_t now_ns() {
  return uint64_t(std::chrono::duration_cast<std::chrono::nanoseconds>(
                      std::chrono::steady_clock::now().time_since_epoch())
                      .count());
}

template <class T>
struct DevBuf {
  T* p = nullptr;
  size_t n = 0;
  cudaStream_t pool_stream = nullptr;  // set while p comes from the stream-ordered pool
  bool pooled = false;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  ~DevBuf() {  // the owner has synchronised its stream
    if (p) {
      if (pooled) cudaFreeAsync(p, nullptr);
      else cudaFree(p);
    }
  }
  void release() {
    if (!p) return;
    if (pooled) {
      QWEN_CUDA(cudaFreeAsync(p, pool_stream));
      QWEN_CUDA(cudaStreamSynchronize(pool_stream));
    } else {
      QWEN_CUDA(cudaFree(p));
    }
    p = nullptr;
    n = 0;
    pooled = false;
  }
  void ensure(size_t count) {
    if (count <= n) return;
    release();
    QWEN_CUDA(cudaMalloc(&p, std::max<size_t>(count, 1) * sizeof(T)));
    n = count;
  }
  // Per-step buffers whose size varies from step to step: grow with headroom
  // by stream-ordered free and allocation on the stream that uses them, so a
  // step that needs more does not synchronise the device.
  void ensure_grow(size_t count, cudaStream_t s) {
    if (count <= n) return;
    const size_t want = count + count / 2;
    if (p) {
      if (pooled) QWEN_CUDA(cudaFreeAsync(p, s));
      else QWEN_CUDA(cudaFree(p));
    }
    p = nullptr;
    n = 0;
    QWEN_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&p), want * sizeof(T), s));
    n = want;
    pooled = true;
    pool_stream = s;
  }
};

template <class T>
struct PinBuf {
  T* p = nullptr;
  size_t n = 0;
  ~PinBuf() {
    if (p) cudaFreeHost(p);
    for (T* r : retired) cudaFreeHost(r);
  }
  void ensure(size_t count) {
    if (count <= n) return;
    if (p) cudaFreeHost(p);
    p = nullptr;
    QWEN_CUDA(cudaMallocHost(&p, std::max<size_t>(count, 1) * sizeof(T)));
    n = count;
  }
  // Growth keeps the old buffer (an async copy of the previous step may
  // still read it) until the owner goes away, instead of freeing it, which
  // would synchronise the device.
  void ensure_grow(size_t count) {
    if (count <= n) return;
    if (p) retired.push_back(p);
    p = nullptr;
    n = 0;
    ensure(count + count / 2);
  }
  std::vector<T*> retired;
};

struct Version {
  std::vector<int32_t> pages;  // KV pages covering [0, position)
  uint32_t hidden_rows = 0;    // post-norm hidden rows kept (hidden_* calls)
};

// MTP draft version (native/qwen_mtp.inc): KV of the MTP attention layer for
// [0, position) in the draft page pool, and the MTP head's post-norm hidden
// rows of the step that made it.
struct DraftVersion {
  std::vector<int32_t> pages;
  uint32_t hidden_rows = 0;
};

constexpr size_t kStatsCount = 17 + 19 * 3;
constexpr int kMaxSplits = 8;
constexpr int kMaxDraft = 8;  // drafts per verified sequence (native_speculative.rs: at most 8)
constexpr int kMaxEos = 64;

struct Session {
  WeightStore* store = nullptr;
  int device = 0;
  rs_qwen_config config{};
  Dims d;
  std::vector<rs_qwen_layer> program;
  size_t slots = 0;
  uint64_t limit = 0;
  std::unique_ptr<StateTable<Version>> table;
  cudaStream_t stream = nullptr;

  // pools
  KvPool kv;
  GdnPool gdn;
  DevBuf<__nv_bfloat16> kv_mem;
  DevBuf<float> gdn_state, gdn_conv, hidden_pool;
  DevBuf<int32_t> block_table;
  int bt_stride = 0;
  size_t gdn_slot_bytes = 0, page_bytes = 0;
  std::vector<int32_t> free_pages;
  std::vector<int32_t> page_ref;
  std::vector<uint8_t> page_filled;

  // step scratch
  int max_tokens = 0, max_rows = 0, max_seqs = 0;
  DevBuf<SeqDesc> descs;
  DevBuf<int32_t> new_pages, cu_seqlens, token_seq, token_pos, out_token, ids, counts, offsets,
      perm, inv, capture;
  DevBuf<int64_t> slot_mapping;
  DevBuf<uint32_t> tokens, sampled, err;
  DevBuf<float> x, proj, partial, q, gate, attn_ws, weights, moe_y, logits, hidden_stage;
  DevBuf<float> gdn_qk, gdn_v, gdn_gb;  // DeltaNet prepared q/k, v, (decay, beta) per token
  DevBuf<int2> attn_items;              // attention work list: (token, KV split) pairs
  DevBuf<int4> pf_dev;                  // chunked-prefill attention blocks
  DevBuf<int32_t> merge_dev;            // tokens of the split decode attention (when some run the prefill kernel)
  DevBuf<uint64_t> argmax_part;         // per-row slice maxima of the split argmax
  DevBuf<uint32_t> argmax_done;         // per-row slice counters (kept at zero between launches)
  // speculative verify: per-token candidate state slots, EOS list, accept results
  DevBuf<int32_t> cand_dev, acc_dev;
  DevBuf<uint32_t> eos_dev, emitted_dev, nemit_dev;
  // MTP draft head: its own version table (sharing the slot and byte budget),
  // a one-layer KV page pool with block-table rows per draft slot, and the
  // draft hidden rows (at most kMaxDraft per version)
  bool mtp_on = false;
  std::unique_ptr<StateTable<DraftVersion>> drafts;
  KvPool mkv;
  DevBuf<__nv_bfloat16> mkv_mem;
  DevBuf<gemm_in_t> mcat;
  CUtensorMap mkv_map;
  DevBuf<int32_t> mbt;
  DevBuf<float> mhidden;
  std::vector<int32_t> mfree, mref;
  std::vector<uint8_t> mfilled;
  size_t mpage_bytes = 0;
  size_t draft_residents() const { return drafts ? drafts->residents() : 0; }
  uint64_t draft_bytes() const { return drafts ? drafts->bytes() : 0; }
  int attn_split_pages = 16, attn_n_items = 0, attn_splits = 1, pf_n_blocks = 0, n_merge = 0;
  DevBuf<gemm_in_t> hb, hb2, act, xperm, hb_out;  // projection inputs (fp16)
  int sm_count = 148;
  int cur_layer = 0;
  bool simple_gemm = false;  // debugging aid: CUDA-core GEMM instead of tcgen05
  std::map<std::tuple<const void*, int, int, int, int>, CUtensorMap> maps;
  std::vector<CUtensorMap> kv_maps;  // one per attention layer

  const CUtensorMap& act_map(const void* p, int rows, int k, int box, int unit) {
    auto key = std::make_tuple(p, rows, k, box, unit);
    auto it = maps.find(key);
    if (it == maps.end()) it = maps.emplace(key, make_act_map3d(p, rows, k, box, unit)).first;
    return it->second;
  }
  void launch_tc(const void* X, int rows_cap, TcArgs& a, cudaStream_t s) {
    launch_qgemm_tc(act_map(X, rows_cap, a.W.k, a.box_rows, qgemm_tc_unit(a)), a, sm_count, s);
  }
  static int box_for(int n) { return n <= 16 ? 16 : n <= 32 ? 32 : n <= 64 ? 64 : 128; }

  // Dense Y[t][n] (+ split partials) = X[t] . deq(W)[n]; returns the split count.
  int dense(const QMat& W, const gemm_in_t* X, int rows_cap, int T, float* Y, int ldy,
            size_t split_stride, int max_splits, cudaStream_t s) {
    if (W.dense_f16) {  // a checkpoint module kept as fp16 rows: one partial
      launch_dense_f16(W, X, T, Y, ldy, s);
      return 1;
    }
    if (simple_gemm) {
      GemmArgs g;
      g.W = W;
      g.X = X;
      g.ldx = W.k;
      g.n_tokens = T;
      g.Y = Y;
      g.ldy = ldy;
      launch_qgemm(g, s);
      return 1;
    }
    TcArgs a;
    a.W = W;
    a.mode = kGemmStoreF32;
    a.n_tokens = T;
    a.box_rows = box_for(std::min(T, 128));
    const int kc = W.k_chunks();
    int splits = 1;
    if (T > 128) {
      // many tokens: one 128-token block per work item, no split-K (the
      // weights of a row tile are re-read from L2 by each block)
      a.token_group = 128;
    } else {
      // split-K: at most one wave of items, slices of whole 4-chunk units when possible
      const int want = qgemm_tc_split_target(W.row_tiles, kc, sm_count, max_splits);
      for (int sp = want; sp >= 1; --sp)
        if (kc % sp == 0 && (kc / sp) % 4 == 0) { splits = sp; break; }
    }
    a.splits = splits;
    a.split_stride = split_stride;
    a.Y = Y;
    a.ldy = ldy;
    a.err = err.p;
    launch_tc(X, rows_cap, a, s);
    return splits;
  }
  PinBuf<uint8_t> staging;
  bool capture_routing = false;
  int captured_tokens = 0;
  DevBuf<float> cap_logits;
  DevBuf<int32_t> cap_offsets, cap_perm;
  std::vector<SeqDesc> last_descs;
  std::vector<int32_t> last_new_pages;
  int last_n = 0, last_T = 0, last_R = 0;

  // device timing (CUDA events on `stream`)
  cudaEvent_t ev_begin = nullptr, ev_end = nullptr;
  bool profile = false;
  std::vector<cudaEvent_t> ev_pool;
  std::vector<std::pair<int, std::pair<int, int>>> ev_marks;  // stage, (begin event, end event)
  int ev_used = 0, open_stage = -1, open_event = -1;
  double last_ms = 0, total_ms = 0, stage_ms[19] = {};
  uint64_t timed_steps = 0, stage_calls[19] = {};

  cudaEvent_t next_event() {
    if (ev_used == int(ev_pool.size())) {
      cudaEvent_t e;
      QWEN_CUDA(cudaEventCreate(&e));
      ev_pool.push_back(e);
    }
    return ev_pool[ev_used++];
  }
  // Stage boundaries (native/operator_timing.h:5-9 ids); no-op unless profiling.
  void stage(int id) {
    if (!profile) return;
    const int e = ev_used;
    QWEN_CUDA(cudaEventRecord(next_event(), stream));
    if (open_stage >= 0) ev_marks.push_back({open_stage, {open_event, e}});
    open_stage = id;
    open_event = e;
  }
  void stage_close() {
    if (!profile || open_stage < 0) return;
    const int e = ev_used;
    QWEN_CUDA(cudaEventRecord(next_event(), stream));
    ev_marks.push_back({open_stage, {open_event, e}});
    open_stage = -1;
  }

  // stats (rs_qwen_device_stats layout, native/qwen_device.inc:62)
  uint64_t exports = 0, uploads = 0, steps = 0, calls = 0, completed = 0, graph_ns = 0,
           wait_ns = 0, export_ns = 0, wall_ns = 0, groups = 0, launches = 0;

  // Expert parallelism (survey multi-GPU mode b): routed experts split over
  // `world` ranks, rank r owning [r*E/world, (r+1)*E/world); rows travel in
  // fixed-size NCCL stages of `cap` = cap_tokens * top rows per peer, so a step
  // needs no host synchronisation. All ranks must step in lockstep (the same
  // number of target steps, each with at most cap_tokens tokens).
  // Two transports: direct NVLink stores into every rank's window (a CUDA IPC
  // mapped allocation holding the stages addressed to that rank and epoch
  // flags; `p2p`), or NCCL send/recv of fixed-size stages.
  struct EpState {
    bool on = false, p2p = false;
    int world = 1, rank = 0, per_rank = 0, cap_tokens = 0, cap = 0, hdr_ints = 0, max_rows = 0;
    size_t stage_bytes = 0, disp_bytes = 0, ret_bytes = 0, win_bytes = 0;
    uint32_t epoch = 0;
    ncclComm_t comm = nullptr;
    uint8_t* window = nullptr;            // p2p: [world][stage] dispatch | [world][cap*H] f32 return | flags
    std::vector<void*> peer_windows;      // p2p: opened peer mappings (nullptr for this rank)
    DevBuf<uint8_t> send, recv;           // nccl: per-peer stages
    DevBuf<float> rsend, rrecv, yloc;
    DevBuf<gemm_in_t> xloc, actloc;
    DevBuf<int32_t> goff, seg, origin, n_rows;
    DevBuf<uint32_t> done;                // last-CTA counters (pack, return)
    // device pointer tables, world entries each: where this rank writes for
    // peer p (dispatch / return), flags it raises at p, where it reads
    // source p's stages (dispatch / return)
    DevBuf<uint64_t> disp_dst, ret_dst, disp_flag, ret_flag, srcs, rsrcs;
    const uint32_t* wait_disp = nullptr;  // p2p: this rank's flag arrays
    const uint32_t* wait_ret = nullptr;
  } ep;
  bool in_mtp = false;  // the MTP head's MoE computes every expert locally

  ~Session() {
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);  // pooled step buffers are freed after this
    if (ep.comm) ncclCommDestroy(ep.comm);
    for (void* w : ep.peer_windows)
      if (w) cudaIpcCloseMemHandle(w);
    if (ep.window) cudaFree(ep.window);
    for (auto e : ev_pool) cudaEventDestroy(e);
    if (ev_begin) cudaEventDestroy(ev_begin);
    if (ev_end) cudaEventDestroy(ev_end);
    if (stream) cudaStreamDestroy(stream);
  }

  void set_device() const { QWEN_CUDA(cudaSetDevice(device)); }

  uint64_t version_bytes(size_t n_pages, size_t hidden_rows) const {
    return gdn_slot_bytes + n_pages * page_bytes + hidden_rows * size_t(d.H) * 4;
  }

  void unref_pages(const std::vector<int32_t>& pages) {
    for (int32_t p : pages) {
      if (--page_ref[p] == 0) {
        page_filled[p] = 0;
        free_pages.push_back(p);
      }
    }
  }

  // step_tokens: per-step token budget that sizes the scratch (0: the
  // QWEN_STEP_TOKENS environment variable, else 4096).
  void init(WeightStore* w, int gpu, const rs_qwen_config& c, const rs_qwen_layer* layers,
            size_t count, size_t n_slots, uint64_t bytes, int step_tokens = 0) {
    if (gpu != 1) throw std::invalid_argument("device session requires gpu=1: this backend has no CPU path");
    if (!w || !w->ready) throw std::invalid_argument("weight store is empty");
    store = w;
    device = w->device;
    set_device();
    cudaDeviceProp prop;
    QWEN_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) throw std::runtime_error("device is not sm_100 (B200): kernels are built for sm_100a only");
    config = c;
    d = Dims::from(c);
    const Dims& wd = w->dims;
    if (d.H != wd.H || d.L != wd.L || d.V != wd.V || d.Hq != wd.Hq || d.Hkv != wd.Hkv ||
        d.D != wd.D || d.hk != wd.hk || d.hv != wd.hv || d.dk != wd.dk || d.dv != wd.dv ||
        d.conv != wd.conv || d.interval != wd.interval || d.E != wd.E || d.top != wd.top ||
        d.I != wd.I || d.S != wd.S)
      throw std::invalid_argument("device session architecture does not match the weight store");
    if (c.context <= 0 || c.chunk <= 0 || c.rope_dims <= 0 || c.rope_dims > c.head_dim ||
        c.rope_dims % 2 || !(c.epsilon > 0) || !(c.theta > 1))
      throw std::invalid_argument("device session architecture/profile");
    if (c.layer_group < 0 || c.fused_recurrent < 0 || c.fused_recurrent > 1 ||
        c.execution_timing < 0 || c.execution_timing > 1 || c.compiled_decode < 0 ||
        c.compiled_decode > 1 || c.operator_profile < 0 || c.operator_profile > 1 ||
        c.fused_attention < 0 || c.fused_attention > 2 || c.validation_mode < 0 ||
        c.validation_mode > 2 || c.expert_kernel < 0 || c.expert_kernel > 2)
      throw std::invalid_argument("device session execution knobs out of range");
    if (count != size_t(c.layers)) throw std::invalid_argument("device session program");
    for (size_t i = 0; i < count; ++i)
      if (layers[i].index != i || layers[i].mixer != uint32_t((i + 1) % c.interval == 0))
        throw std::invalid_argument("device session program");
    program.assign(layers, layers + count);
    if (!n_slots || n_slots > (size_t(1) << 20) || !bytes) throw std::invalid_argument("state table bounds");
    slots = n_slots;
    limit = bytes;
    table = std::make_unique<StateTable<Version>>(allocate_owner(), n_slots, bytes);
    QWEN_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    QWEN_CUDA(cudaEventCreate(&ev_begin));
    QWEN_CUDA(cudaEventCreate(&ev_end));

    // DeltaNet pool: one slot per version
    gdn.slots = int(n_slots);
    gdn.n_gdn = d.n_gdn;
    gdn.state_elems = size_t(d.hv) * d.dv * d.dk;
    gdn.conv_elems = size_t(d.conv - 1) * d.cd;
    gdn_slot_bytes = size_t(d.n_gdn) * (gdn.state_elems + gdn.conv_elems) * 4;
    gdn_state.ensure(std::max<size_t>(1, n_slots * d.n_gdn * gdn.state_elems));
    gdn_conv.ensure(std::max<size_t>(1, n_slots * d.n_gdn * gdn.conv_elems));
    gdn.state = gdn_state.p;
    gdn.conv = gdn_conv.p;

    // scratch sizing
    const char* env = std::getenv("QWEN_STEP_TOKENS");
    max_tokens = step_tokens > 0 ? step_tokens : env ? std::max(1, atoi(env)) : 4096;
    max_rows = std::min(max_tokens, 1024);
    max_seqs = max_tokens;
    bt_stride = (d.ctx + kPageTokens - 1) / kPageTokens;
    block_table.ensure(n_slots * size_t(bt_stride));
    QWEN_CUDA(cudaMemset(block_table.p, 0, n_slots * size_t(bt_stride) * 4));
    hidden_pool.ensure(n_slots * size_t(std::max(1, d.chunk)) * d.H);
    const int T = max_tokens, A = T * (d.top + 1);
    descs.ensure(max_seqs);
    new_pages.ensure(size_t(max_seqs) + T / kPageTokens + 16);
    cu_seqlens.ensure(max_seqs + 1);
    token_seq.ensure(T);
    token_pos.ensure(T);
    slot_mapping.ensure(T);
    out_token.ensure(T);
    tokens.ensure(T);
    sampled.ensure(max_rows);
    argmax_part.ensure(size_t(max_rows) * 8);
    argmax_done.ensure(max_rows);
    QWEN_CUDA(cudaMemset(argmax_done.p, 0, size_t(max_rows) * 4));
    cand_dev.ensure(T);
    acc_dev.ensure(max_seqs);
    eos_dev.ensure(kMaxEos);
    emitted_dev.ensure(size_t(max_seqs) * (kMaxDraft + 1));
    nemit_dev.ensure(max_seqs);
    err.ensure(1);
    x.ensure(size_t(T) * d.H);
    const int proj_w = std::max({d.gdn_in_rows, d.attn_in_rows, d.E + 1});
    proj.ensure(size_t(T) * proj_w);
    const int hbw = std::max({d.H, d.vd, d.Hq * d.D});
    hb.ensure(size_t(T) * hbw);
    hb2.ensure(size_t(T) * hbw);
    gdn_qk.ensure(size_t(T) * std::max(1, d.hk * 2 * d.dk));
    gdn_v.ensure(size_t(T) * std::max(1, d.vd));
    gdn_gb.ensure(size_t(T) * std::max(1, d.hv * 2));
    q.ensure(size_t(T) * d.Hq * d.D);
    gate.ensure(size_t(T) * d.Hq * d.D);
    ids.ensure(A);
    weights.ensure(A);
    counts.ensure(d.E + 1);
    offsets.ensure(d.E + 2);
    perm.ensure(A);
    inv.ensure(A);
    act.ensure(size_t(A) * d.I);
    moe_y.ensure(size_t(A) * d.H);
    hidden_stage.ensure(size_t(T) * d.H);
    xperm.ensure(size_t(A) * d.H);
    hb_out.ensure(size_t(max_rows) * d.H);
    QWEN_CUDA(cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, device));
    simple_gemm = std::getenv("QWEN_GEMM") && std::string(std::getenv("QWEN_GEMM")) == "simple";
    const int max_split_w = std::max({d.gdn_in_rows, d.attn_in_rows, d.E + 1, d.H});
    partial.ensure(size_t(kMaxSplits) * T * max_split_w);

    // KV page pool: what the byte budget leaves after the DeltaNet pool,
    // capped by free device memory (keep 2 GiB of headroom).
    page_bytes = size_t(d.n_attn) * 2 * d.Hkv * kPageTokens * d.D * 2;
    size_t budget_pages = 0;
    const uint64_t fixed = uint64_t(n_slots) * gdn_slot_bytes;
    if (d.n_attn > 0) {
      if (bytes <= fixed) throw std::invalid_argument("state byte budget smaller than the DeltaNet pool");
      budget_pages = (bytes - fixed) / page_bytes;
      size_t free_b = 0, total_b = 0;
      QWEN_CUDA(cudaMemGetInfo(&free_b, &total_b));
      const size_t headroom = size_t(2) << 30;
      size_t mem_pages = free_b > headroom ? (free_b - headroom) / page_bytes : 0;
      budget_pages = std::min({budget_pages, mem_pages, size_t(INT32_MAX / kPageTokens)});
      if (budget_pages == 0) throw std::runtime_error("no device memory left for KV pages");
      kv_mem.ensure(budget_pages * (page_bytes / 2));
    }
    kv.base = kv_mem.p;
    kv.n_pages = int(budget_pages);
    kv.layers = d.n_attn;
    kv.Hkv = d.Hkv;
    kv.D = d.D;
    for (int l = 0; l < d.n_attn && budget_pages > 0; ++l) kv_maps.push_back(make_kv_map(kv, l));
    free_pages.resize(budget_pages);
    for (size_t i = 0; i < budget_pages; ++i) free_pages[i] = int32_t(budget_pages - 1 - i);
    page_ref.assign(budget_pages, 0);
    page_filled.assign(budget_pages, 0);
  }

  // ------------------------------------------------------------ the step --
  struct SeqIn {
    const StateId* parent;  // null iff position == 0
    uint32_t position, count;
    const uint32_t* tokens;
  };
  // Speculative verify (rs_qwen_device_mtp_verify_accept): each sequence's
  // tokens are [seed, drafts...]; results per sequence.
  struct VerifyIn {
    const uint32_t* eos;
    size_t n_eos;
    uint32_t* accepted;
    uint32_t* emitted;  // [n][emit_stride]
    size_t emit_stride;
    uint32_t* n_emitted;
  };
  // Constrained greedy selection (rs_qwen_device_step_ragged_choices): output
  // row r chooses among ids[offsets[r], offsets[r+1]); an empty range leaves
  // the row unconstrained.
  struct ChoiceIn {
    const uint32_t* offsets;  // output rows + 1
    const uint32_t* ids;
    size_t n_ids;
  };
  int n_choice_rows = 0;  // constrained rows of the step being enqueued
  PinBuf<uint32_t> choice_stage;
  DevBuf<uint32_t> choice_dev;  // [rows list][offsets][ids]
  // chunked DeltaNet for long token runs: work lists and per-(chunk, head) scratch
  GdnChunkPlan gplan;
  PinBuf<int32_t> gplan_stage;
  DevBuf<int32_t> gplan_dev;
  DevBuf<float> gplan_u, gplan_w, gplan_a, gplan_lg;

  // Runs one ragged step. Outputs: outs[s], then per output row a sampled
  // token and/or fp32 logits. Throws on any error after rolling back.
  void step(const std::vector<SeqIn>& seqs, uint32_t flags, StateId* outs, uint32_t* sampled_out,
            float* logits_out, const VerifyIn* vin = nullptr, const ChoiceIn* choice = nullptr) {
    set_device();
    const uint64_t t_start = now_ns();
    ++calls;
    n_choice_rows = 0;
    const int n = int(seqs.size());
    if (n <= 0) throw std::invalid_argument("ragged step needs at least one sequence");
    if (n > max_seqs) throw std::invalid_argument("too many sequences in one step");
    if (vin) {
      if (flags & (RS_QWEN_RAGGED_CONSUME | RS_QWEN_RAGGED_LOGITS))
        throw std::invalid_argument("verify steps keep their parents and return no logits");
      if (vin->n_eos > size_t(kMaxEos)) throw std::invalid_argument("too many EOS tokens");
      flags |= RS_QWEN_RAGGED_ALL_ROWS;
      size_t cand_total = 0;
      for (const auto& s : seqs) {
        if (!s.parent) throw std::invalid_argument("verify needs a parent version per sequence");
        if (s.count < 1 || s.count > uint32_t(kMaxDraft + 1)) throw std::invalid_argument("draft count above 8");
        cand_total += s.count;
      }
      if (table->residents() + draft_residents() + cand_total > slots)
        throw std::runtime_error("combined resident budget exhausted");
    }
    const bool consume = flags & RS_QWEN_RAGGED_CONSUME;
    const bool all_rows = flags & RS_QWEN_RAGGED_ALL_ROWS;
    const bool keep_hidden = flags & RS_QWEN_RAGGED_HIDDEN;
    int T = 0, R = 0, max_len = 0;
    for (const auto& s : seqs) {
      if (!s.count) throw std::invalid_argument("sequence with no tokens");
      if ((s.position == 0) != (s.parent == nullptr)) throw std::invalid_argument("device previous state presence");
      if (size_t(s.position) + s.count > size_t(d.ctx)) throw std::invalid_argument("device step capacity");
      if (keep_hidden && s.count > uint32_t(d.chunk)) throw std::invalid_argument("hidden capture exceeds chunk rows");
      for (uint32_t i = 0; i < s.count; ++i)
        if (s.tokens[i] >= uint32_t(d.V)) throw std::invalid_argument("token outside vocabulary");
      T += int(s.count);
      R += all_rows ? int(s.count) : 1;
      max_len = std::max<int>(max_len, int(s.position + s.count));
    }
    if (T > max_tokens) throw std::invalid_argument("ragged step exceeds the token budget");
    // Attention work list. A split spans enough pages to amortise its CTA's
    // query load and warp merge (16..64 pages) while leaving at least four
    // CTAs per SM; each token gets one item per split its keys reach.
    // Sequences that feed at least kAttnPrefillMin tokens run the chunked-prefill
    // kernel (blocks of consecutive tokens sharing each K/V page load, longest
    // prefixes first); the decode kernel and the split merge take the rest.
    std::vector<int2> items;
    std::vector<int4> pf_blocks;
    std::vector<int32_t> merge_tokens;
    attn_n_items = pf_n_blocks = 0;
    if (d.n_attn > 0) {
      const int G = d.Hq / d.Hkv;
      const bool pf_ok = G >= 1 && G <= 16 && 16 % G == 0;
      const int QB = pf_ok ? kAttnPrefillWarps * (16 / G) : 0;
      auto prefill = [&](const SeqIn& s) { return pf_ok && s.count >= uint32_t(kAttnPrefillMin); };
      int64_t page_heads = 0;
      int dec_len = 1;  // longest context of a split-decoded token
      for (const auto& s : seqs)
        if (!prefill(s)) {
          for (uint32_t j = 0; j < s.count; ++j) page_heads += (int64_t(s.position) + j + kPageTokens) / kPageTokens;
          dec_len = std::max<int>(dec_len, int(s.position + s.count));
        }
      page_heads *= d.Hkv;
      int sp = 16;
      while (sp < 64 && page_heads / (2 * sp) >= int64_t(sm_count) * 4) sp *= 2;
      attn_split_pages = sp;
      attn_splits = std::max(1, (dec_len + sp * kPageTokens - 1) / (sp * kPageTokens));
      int t = 0;
      for (int i = 0; i < n; ++i) {
        const SeqIn& s = seqs[i];
        if (prefill(s)) {
          for (int j0 = 0; j0 < int(s.count); j0 += QB) {
            const int nb = std::min(QB, int(s.count) - j0);
            const int last = int(s.position) + j0 + nb - 1;
            pf_blocks.push_back(make_int4(t + j0, nb, i, last / kPageTokens + 1));
          }
          t += int(s.count);
          continue;
        }
        for (uint32_t j = 0; j < s.count; ++j, ++t) {
          const int pages = int((int64_t(s.position) + j + kPageTokens) / kPageTokens);
          const int md = int(merge_tokens.size());  // workspace row (= t when nothing runs the prefill kernel)
          for (int k = 0; k * sp < pages; ++k) items.push_back(make_int2(md, k));
          merge_tokens.push_back(t);
        }
      }
      std::stable_sort(pf_blocks.begin(), pf_blocks.end(), [](const int4& x, const int4& y) { return x.w > y.w; });
      attn_n_items = int(items.size());
      pf_n_blocks = int(pf_blocks.size());
      n_merge = int(merge_tokens.size());
      if (pf_blocks.empty()) merge_tokens.clear();  // every token merges: no list needed
    }
    if (R > max_rows) throw std::invalid_argument("ragged step exceeds the output-row budget");
    // DeltaNet runs of at least kGdnChunkMin tokens (not verify steps) take the chunked kernels
    gplan = GdnChunkPlan();
    std::vector<int32_t> gl_longs, gl_items, gl_tokens;
    if (d.n_gdn > 0 && !vin && T != n) {
      int off = 0;
      for (int i = 0; i < n; ++i) {
        const int cnt = int(seqs[i].count);
        if (cnt >= kGdnChunkMin) {
          const int chunks = (cnt + kGdnChunk - 1) / kGdnChunk;
          gl_longs.insert(gl_longs.end(), {i, int(gl_items.size() / 2), chunks});
          for (int j = 0; j < chunks; ++j) gl_items.insert(gl_items.end(), {i, j});
          for (int j = 0; j < cnt; ++j) gl_tokens.push_back(off + j);
        }
        off += cnt;
      }
    }
    // constrained rows: validated and compacted on the host (choices.rs:83-86 checks)
    std::vector<uint32_t> ch_host;
    if (choice) {
      if (!sampled_out || vin) throw std::invalid_argument("constrained selection needs sampled tokens");
      const uint32_t* off = choice->offsets;
      if (!off || off[0] != 0 || off[R] != choice->n_ids || (choice->n_ids && !choice->ids))
        throw std::invalid_argument("allowed-token offsets");
      std::vector<uint32_t> rows_l, offs{0};
      for (int r = 0; r < R; ++r) {
        if (off[r + 1] < off[r]) throw std::invalid_argument("allowed-token offsets");
        if (off[r + 1] == off[r]) continue;
        rows_l.push_back(uint32_t(r));
        offs.push_back(offs.back() + (off[r + 1] - off[r]));
      }
      for (size_t i = 0; i < choice->n_ids; ++i)
        if (choice->ids[i] >= uint32_t(d.V)) throw std::invalid_argument("invalid legal token");
      n_choice_rows = int(rows_l.size());
      if (n_choice_rows) {
        ch_host = rows_l;
        ch_host.insert(ch_host.end(), offs.begin(), offs.end());
        for (int k = 0; k < n_choice_rows; ++k)  // the ids of the constrained rows, in row order
          ch_host.insert(ch_host.end(), choice->ids + off[rows_l[k]], choice->ids + off[rows_l[k] + 1]);
      }
    }
    // parents must be distinct when consumed
    std::vector<const Version*> par(n, nullptr);
    for (int i = 0; i < n; ++i) {
      if (!seqs[i].parent) continue;
      if (seqs[i].parent->position != seqs[i].position) throw std::invalid_argument("device position mismatch");
      par[i] = &table->get(*seqs[i].parent);
      if (consume)
        for (int j = 0; j < i; ++j)
          if (seqs[j].parent && seqs[j].parent->slot == seqs[i].parent->slot)
            throw std::invalid_argument("consumed parent used twice");
    }
    if (!consume && table->residents() + draft_residents() + size_t(n) > slots)
      throw std::runtime_error("combined resident budget exhausted");

    // page planning (host), descriptors
    staging.ensure_grow(sizeof(SeqDesc) * n + 4 * (size_t(T) + n + T / kPageTokens + 16) + 64 + items.size() * 8 +
                        16 + pf_blocks.size() * 16 + merge_tokens.size() * 4);
    SeqDesc* hd = reinterpret_cast<SeqDesc*>(staging.p);
    std::vector<int32_t> npages;
    std::vector<std::vector<int32_t>> child_pages(n);
    std::vector<StateId> reserved;
    std::vector<int32_t> deferred_free;
    std::vector<int> tok_off(n + 1, 0);
    std::vector<std::vector<StateId>> cands(vin ? n : 0);  // verify: per token's candidate version
    std::vector<int32_t> cand_host;
    // On failure every page reference taken for a child is dropped (shared
    // pages were either ref'd or inherited from a consumed parent), and
    // consumed parents' dropped pages are released too.
    auto fail_cleanup = [&]() {
      for (auto& cp : child_pages) unref_pages(cp);
      unref_pages(deferred_free);
      for (auto& id : reserved) {
        try {
          table->rollback(id);
        } catch (...) {
        }
      }
    };
    try {
      int row = 0;
      for (int i = 0; i < n; ++i) {
        const auto& s = seqs[i];
        tok_off[i + 1] = tok_off[i] + int(s.count);
        SeqDesc& sd = hd[i];
        std::memset(&sd, 0, sizeof(sd));
        sd.position = int32_t(s.position);
        sd.count = int32_t(s.count);
        sd.parent = s.parent ? int32_t(s.parent->slot) : -1;
        sd.cow_src = -1;
        const int pos = int(s.position), cnt = int(s.count);
        const int n_prefix = (pos + kPageTokens - 1) / kPageTokens;
        const int n_total = (pos + cnt + kPageTokens - 1) / kPageTokens;
        if (par[i] && int(par[i]->pages.size()) != n_prefix) throw std::runtime_error("parent page list inconsistent");
        int n_shared = n_prefix;
        if (d.n_attn > 0 && pos % kPageTokens) {
          const int32_t lp = par[i]->pages[n_prefix - 1];
          if (page_filled[lp] > pos % kPageTokens) {  // a sibling extended it: copy on write
            n_shared = n_prefix - 1;
            sd.cow_src = lp;
            sd.cow_len = pos % kPageTokens;
          } else {
            page_filled[lp] = uint8_t(std::min(kPageTokens, pos + cnt - (n_prefix - 1) * kPageTokens));
          }
        }
        if (d.n_attn == 0) n_shared = 0;
        const int n_new = d.n_attn > 0 ? n_total - n_shared : 0;
        if (n_new > int(free_pages.size())) throw std::runtime_error("KV page pool exhausted");
        sd.n_shared = n_shared;
        sd.new_off = int32_t(npages.size());
        sd.n_new = n_new;
        auto& cp = child_pages[i];
        if (d.n_attn > 0) {
          cp.assign(par[i] ? par[i]->pages.begin() : cp.end(), par[i] ? par[i]->pages.begin() + n_shared : cp.end());
          if (!consume)
            for (int32_t p : cp) ++page_ref[p];
          for (int j = 0; j < n_new; ++j) {
            const int32_t p = free_pages.back();
            free_pages.pop_back();
            page_ref[p] = 1;
            const int first = (n_shared + j) * kPageTokens;
            page_filled[p] = uint8_t(std::min(kPageTokens, pos + cnt - first));
            npages.push_back(p);
            cp.push_back(p);
          }
        }
        if (int(cp.size()) > bt_stride) throw std::invalid_argument("context exceeds block table");
        sd.n_out = all_rows ? cnt : 1;
        sd.out_row0 = row;
        row += sd.n_out;
        sd.hidden = keep_hidden ? 1 : 0;
        const uint64_t charge = version_bytes(cp.size(), keep_hidden ? cnt : 0);
        StateId id;
        sd.cand = -1;
        if (vin) {
          // one candidate version per fed token, charged for its own length
          sd.cand = int32_t(cand_host.size());
          for (int j = 0; j < cnt; ++j) {
            const size_t pj = d.n_attn > 0 ? size_t(pos + j + 1 + kPageTokens - 1) / kPageTokens : 0;
            const StateId cj = table->reserve(s.position + j + 1, version_bytes(pj, keep_hidden ? j + 1 : 0));
            reserved.push_back(cj);
            cands[i].push_back(cj);
            cand_host.push_back(int32_t(cj.slot));
          }
          sd.child = cand_host.back();
          continue;
        }
        if (consume && s.parent) {
          // consume: the parent's pages move to the child; a dropped COW page is freed after the step
          std::vector<int32_t> parent_pages = par[i]->pages;
          for (size_t j = n_shared; j < parent_pages.size(); ++j) deferred_free.push_back(parent_pages[j]);
          table->release(*s.parent);
          par[i] = nullptr;
          id = table->reserve_at(s.parent->slot, s.position + s.count, charge);
        } else {
          id = table->reserve(s.position + s.count, charge);
        }
        reserved.push_back(id);
        sd.child = int32_t(id.slot);
      }
    } catch (...) {
      fail_cleanup();
      throw;
    }

    // upload: descriptors, new page ids, tokens (one pinned staging buffer)
    uint8_t* sp = staging.p + sizeof(SeqDesc) * n;
    int32_t* hp = reinterpret_cast<int32_t*>(sp);
    std::memcpy(hp, npages.data(), npages.size() * 4);
    uint32_t* ht = reinterpret_cast<uint32_t*>(hp + npages.size());
    for (int i = 0; i < n; ++i) std::memcpy(ht + tok_off[i], seqs[i].tokens, seqs[i].count * 4);
    int2* hi = reinterpret_cast<int2*>((reinterpret_cast<uintptr_t>(ht + T) + 7) & ~uintptr_t(7));
    if (!items.empty()) std::memcpy(hi, items.data(), items.size() * 8);
    int4* hpf = reinterpret_cast<int4*>((reinterpret_cast<uintptr_t>(hi + items.size()) + 15) & ~uintptr_t(15));
    if (!pf_blocks.empty()) std::memcpy(hpf, pf_blocks.data(), pf_blocks.size() * 16);
    int32_t* hmt = reinterpret_cast<int32_t*>(hpf + pf_blocks.size());
    if (!merge_tokens.empty()) std::memcpy(hmt, merge_tokens.data(), merge_tokens.size() * 4);
    try {
      QWEN_CUDA(cudaMemcpyAsync(descs.p, hd, sizeof(SeqDesc) * n, cudaMemcpyHostToDevice, stream));
      if (!npages.empty())
        QWEN_CUDA(cudaMemcpyAsync(new_pages.p, hp, npages.size() * 4, cudaMemcpyHostToDevice, stream));
      QWEN_CUDA(cudaMemcpyAsync(tokens.p, ht, size_t(T) * 4, cudaMemcpyHostToDevice, stream));
      if (vin) {
        QWEN_CUDA(cudaMemcpyAsync(cand_dev.p, cand_host.data(), cand_host.size() * 4, cudaMemcpyHostToDevice,
                                  stream));
        if (vin->n_eos)
          QWEN_CUDA(cudaMemcpyAsync(eos_dev.p, vin->eos, vin->n_eos * 4, cudaMemcpyHostToDevice, stream));
      }
      QWEN_CUDA(cudaMemsetAsync(err.p, 0, 4, stream));
      if (!items.empty()) {
        attn_items.ensure_grow(items.size(), stream);
        QWEN_CUDA(cudaMemcpyAsync(attn_items.p, hi, items.size() * 8, cudaMemcpyHostToDevice, stream));
      }
      if (!pf_blocks.empty()) {
        pf_dev.ensure_grow(pf_blocks.size(), stream);
        QWEN_CUDA(cudaMemcpyAsync(pf_dev.p, hpf, pf_blocks.size() * 16, cudaMemcpyHostToDevice, stream));
      }
      if (!merge_tokens.empty()) {
        merge_dev.ensure_grow(merge_tokens.size(), stream);
        QWEN_CUDA(cudaMemcpyAsync(merge_dev.p, hmt, merge_tokens.size() * 4, cudaMemcpyHostToDevice, stream));
      }
      if (!gl_longs.empty()) {
        const size_t nl = gl_longs.size(), ni = gl_items.size(), nt = gl_tokens.size();
        gplan_stage.ensure_grow(nl + ni + nt);
        gplan_dev.ensure_grow(nl + ni + nt, stream);
        std::memcpy(gplan_stage.p, gl_longs.data(), nl * 4);
        std::memcpy(gplan_stage.p + nl, gl_items.data(), ni * 4);
        std::memcpy(gplan_stage.p + nl + ni, gl_tokens.data(), nt * 4);
        QWEN_CUDA(cudaMemcpyAsync(gplan_dev.p, gplan_stage.p, (nl + ni + nt) * 4, cudaMemcpyHostToDevice, stream));
        uploads += (nl + ni + nt) * 4;
        const size_t units = ni / 2 * size_t(d.hv) * kGdnChunk;  // (chunk, head) pairs x chunk tokens
        gplan_u.ensure_grow(units * d.dv, stream);
        gplan_w.ensure_grow(units * d.dk, stream);
        gplan_a.ensure_grow(units * kGdnChunk, stream);
        gplan_lg.ensure_grow(units, stream);
        gplan.n_long = int(nl / 3);
        gplan.n_items = int(ni / 2);
        gplan.n_tokens = int(nt);
        gplan.longs = gplan_dev.p;
        gplan.items = gplan_dev.p + nl;
        gplan.tokens = gplan_dev.p + nl + ni;
        gplan.U = gplan_u.p;
        gplan.W = gplan_w.p;
        gplan.A = gplan_a.p;
        gplan.LG = gplan_lg.p;
      }
      if (!ch_host.empty()) {
        QWEN_CUDA(cudaStreamSynchronize(stream));  // the pinned stage may still feed the previous step's copy
        choice_stage.ensure_grow(ch_host.size());
        choice_dev.ensure_grow(ch_host.size(), stream);
        std::memcpy(choice_stage.p, ch_host.data(), ch_host.size() * 4);
        QWEN_CUDA(cudaMemcpyAsync(choice_dev.p, choice_stage.p, ch_host.size() * 4, cudaMemcpyHostToDevice, stream));
        uploads += ch_host.size() * 4;
      }
      uploads += sizeof(SeqDesc) * n + npages.size() * 4 + size_t(T) * 4 + items.size() * 8 +
                 pf_blocks.size() * 16 + merge_tokens.size() * 4 +
                 (vin ? cand_host.size() * 4 + vin->n_eos * 4 : 0);
      const uint64_t t_graph = now_ns();
      ev_used = 0;
      ev_marks.clear();
      open_stage = -1;
      QWEN_CUDA(cudaEventRecord(ev_begin, stream));
      if (capture_routing) {
        last_descs.assign(hd, hd + n);
        last_new_pages = npages;
        last_n = n;
        last_T = T;
        last_R = R;
      }
      forward(n, T, R, max_len, keep_hidden, logits_out != nullptr);
      std::vector<int32_t> acc_h(vin ? n : 0);
      std::vector<uint32_t> emit_h(vin ? size_t(n) * (kMaxDraft + 1) : 0), nemit_h(vin ? n : 0);
      if (vin) {
        launch_accept(descs.p, n, cu_seqlens.p, tokens.p, sampled.p, eos_dev.p, int(vin->n_eos), d.ctx, acc_dev.p,
                      emitted_dev.p, kMaxDraft + 1, nemit_dev.p, stream);
        launch_verify_compact(descs.p, n, cand_dev.p, acc_dev.p, block_table.p, bt_stride, hidden_stage.p,
                              cu_seqlens.p, hidden_pool.p, d.chunk, d.H, stream);
      }
      stage_close();
      QWEN_CUDA(cudaEventRecord(ev_end, stream));
      if (vin) {
        QWEN_CUDA(cudaMemcpyAsync(acc_h.data(), acc_dev.p, size_t(n) * 4, cudaMemcpyDeviceToHost, stream));
        QWEN_CUDA(cudaMemcpyAsync(emit_h.data(), emitted_dev.p, emit_h.size() * 4, cudaMemcpyDeviceToHost, stream));
        QWEN_CUDA(cudaMemcpyAsync(nemit_h.data(), nemit_dev.p, size_t(n) * 4, cudaMemcpyDeviceToHost, stream));
      }
      if (keep_hidden && !vin)
        for (int i = 0; i < n; ++i)
          QWEN_CUDA(cudaMemcpyAsync(hidden_pool.p + size_t(hd[i].child) * d.chunk * d.H,
                                    hidden_stage.p + size_t(tok_off[i]) * d.H, size_t(seqs[i].count) * d.H * 4,
                                    cudaMemcpyDeviceToDevice, stream));
      uint32_t h_err = 0;
      if (sampled_out) QWEN_CUDA(cudaMemcpyAsync(sampled_out, sampled.p, size_t(R) * 4, cudaMemcpyDeviceToHost, stream));
      if (logits_out)
        QWEN_CUDA(cudaMemcpyAsync(logits_out, logits.p, size_t(R) * d.V * 4, cudaMemcpyDeviceToHost, stream));
      QWEN_CUDA(cudaMemcpyAsync(&h_err, err.p, 4, cudaMemcpyDeviceToHost, stream));
      const uint64_t t_wait = now_ns();
      graph_ns += t_wait - t_graph;
      QWEN_CUDA(cudaStreamSynchronize(stream));
      const uint64_t t_done = now_ns();
      wait_ns += t_done - t_wait;
      ++groups;
      float ms = 0.f;
      QWEN_CUDA(cudaEventElapsedTime(&ms, ev_begin, ev_end));
      last_ms = ms;
      total_ms += ms;
      ++timed_steps;
      for (auto& m : ev_marks) {
        float sm = 0.f;
        QWEN_CUDA(cudaEventElapsedTime(&sm, ev_pool[m.second.first], ev_pool[m.second.second]));
        stage_ms[m.first] += sm;
        ++stage_calls[m.first];
      }
      if (h_err & kErrNonFinite) throw std::runtime_error("nonfinite device state");
      if (h_err) throw std::runtime_error("device step error flag " + std::to_string(h_err));
      if (vin) {
        // publish the candidate after `accepted` drafts; roll the others back
        for (int i = 0; i < n; ++i) {
          const int a = acc_h[i], pos = int(seqs[i].position);
          if (a < 0 || a >= int(seqs[i].count) || nemit_h[i] > uint32_t(kMaxDraft + 1))
            throw std::runtime_error("verify accept result out of range");
          Version v;
          v.pages = child_pages[i];
          const int len = pos + a + 1;
          const size_t keep = d.n_attn > 0 ? size_t(len + kPageTokens - 1) / kPageTokens : 0;
          std::vector<int32_t> dropped(v.pages.begin() + keep, v.pages.end());
          v.pages.resize(keep);
          if (keep) page_filled[v.pages.back()] = uint8_t(len - int(keep - 1) * kPageTokens);
          v.hidden_rows = keep_hidden ? uint32_t(a + 1) : 0;
          table->publish(cands[i][a], std::move(v));
          for (int j = 0; j < int(cands[i].size()); ++j)
            if (j != a) table->rollback(cands[i][j]);
          unref_pages(dropped);
          outs[i] = cands[i][a];
          vin->accepted[i] = uint32_t(a);
          vin->n_emitted[i] = nemit_h[i];
          for (size_t e = 0; e < vin->emit_stride; ++e)
            vin->emitted[i * vin->emit_stride + e] = e < nemit_h[i] ? emit_h[size_t(i) * (kMaxDraft + 1) + e] : 0u;
        }
        steps += uint64_t(n);
        ++completed;
        wall_ns += now_ns() - t_start;
        return;
      }
    } catch (...) {
      cudaStreamSynchronize(stream);
      fail_cleanup();
      throw;
    }
    // publish
    for (int i = 0; i < n; ++i) {
      Version v;
      v.pages = std::move(child_pages[i]);
      v.hidden_rows = keep_hidden ? seqs[i].count : 0;
      table->publish(reserved[i], std::move(v));
      outs[i] = reserved[i];
    }
    unref_pages(deferred_free);
    steps += uint64_t(n);
    ++completed;
    const uint64_t t_end = now_ns();
    export_ns += 0;
    wall_ns += t_end - t_start;
  }

  // Enqueue the whole decoder on `stream` (no host synchronisation).
  void forward(int n, int T, int R, int max_len, bool keep_hidden, bool want_logits) {
    (void)want_logits;
    cudaStream_t s = stream;
    const ModelDev& m = store->model;
    Packed pk{cu_seqlens.p, token_seq.p, token_pos.p, slot_mapping.p, out_token.p};
    stage(0);  // Embedding (packing + embedding)
    launch_pack(descs.p, n, new_pages.p, block_table.p, bt_stride, pk, s);
    if (d.n_attn > 0) launch_cow(kv, descs.p, n, new_pages.p, s);
    launch_embed_norm(m.embed, tokens.p, T, m.layers[0].in_norm, d.eps, x.p, hb.p, s);
    const int slots_per_tok = d.top + 1, A = T * slots_per_tok;
    if (d.n_attn > 0) attn_ws.ensure_grow(size_t(pf_n_blocks ? n_merge : T) * d.Hq * attn_splits * (d.D + 2), s);
    if (capture_routing) {
      capture.ensure(size_t(d.L) * A);
      cap_logits.ensure(size_t(d.L) * T * (d.E + 1));
      cap_offsets.ensure(size_t(d.L) * (d.E + 2));
      cap_perm.ensure(size_t(d.L) * A);
    }
    captured_tokens = T;
    cur_layer = 0;
    const int proj_w = std::max({d.gdn_in_rows, d.attn_in_rows, d.E + 1});
    const size_t proj_stride = size_t(T) * proj_w;
    for (int li = 0; li < d.L; ++li) {
      const LayerDev& ly = m.layers[li];
      stage(ly.mixer == 0 ? 2 : 6);  // RecurrentProjection / AttentionProjection
      const int ps = dense(ly.in_proj, hb.p, max_tokens, T, partial.p, proj_w, proj_stride, kMaxSplits, s);
      const int k_out = ly.mixer == 0 ? d.vd : d.Hq * d.D;
      if (ly.mixer == 0) {
        stage(4);  // RecurrentUpdate (conv + prepare + recurrence + gated norm)
        launch_gdn(d, ly, partial.p, proj_w, ps, proj_stride, descs.p, cu_seqlens.p, n, T, gdn, ly.type_index,
                   hb2.p, err.p, gdn_qk.p, gdn_v.p, gdn_gb.p, sm_count, cand_dev.p, s, &gplan);
        stage(5);  // RecurrentOutput
      } else {
        stage(7);  // AttentionReduction (q/k norm, RoPE, KV append, paged attention)
        launch_attn_prep(d, ly, partial.p, proj_w, ps, proj_stride, token_pos.p, slot_mapping.p, T, kv,
                         ly.type_index, q.p, gate.p, s);
        launch_attn_decode(kv_maps[ly.type_index], d, q.p, token_seq.p, token_pos.p,
                           pf_n_blocks ? merge_dev.p : nullptr, descs.p, block_table.p,
                           bt_stride, attn_items.p, attn_n_items, attn_split_pages, attn_ws.p, attn_splits, err.p,
                           s);
        launch_attn_prefill(kv_maps[ly.type_index], d, q.p, token_pos.p, descs.p, block_table.p, bt_stride,
                            pf_dev.p, pf_n_blocks, gate.p, hb2.p, err.p, s);
        launch_attention_merge(d, attn_ws.p, gate.p, token_pos.p, pf_n_blocks ? merge_dev.p : nullptr,
                               pf_n_blocks ? n_merge : T, attn_split_pages, attn_splits, hb2.p, s);
        stage(8);  // AttentionOutput
      }
      const size_t out_stride = size_t(T) * d.H;
      const int os = dense(ly.out_proj, hb2.p, max_tokens, T, partial.p, d.H, out_stride, kMaxSplits, s);
      (void)k_out;
      stage(9);  // ResidualNorm
      launch_residual_norm(x.p, partial.p, os, out_stride, T, d.H, ly.post_norm, d.eps, hb.p, nullptr, 0,
                           nullptr, s);
      cur_layer = li;
      moe(ly, T, A, s);
      if (capture_routing) {
        QWEN_CUDA(cudaMemcpyAsync(capture.p + size_t(li) * A, ids.p, size_t(A) * 4, cudaMemcpyDeviceToDevice, s));
        QWEN_CUDA(cudaMemcpyAsync(cap_offsets.p + size_t(li) * (d.E + 2), offsets.p, size_t(d.E + 2) * 4,
                                  cudaMemcpyDeviceToDevice, s));
        QWEN_CUDA(cudaMemcpyAsync(cap_perm.p + size_t(li) * A, perm.p, size_t(A) * 4, cudaMemcpyDeviceToDevice, s));
      }
      const float* next_norm = li + 1 < d.L ? m.layers[li + 1].in_norm : nullptr;
      stage(13);  // MoeMixture (+ shared merge, residual, next input norm)
      launch_moe_combine(x.p, moe_y.p, inv.p, weights.p, T, d.H, slots_per_tok, next_norm, d.eps, hb.p,
                         nullptr, 0, nullptr, s);
    }
    stage(17);  // FinalProjection
    if (keep_hidden)  // post-norm hidden rows of every token (fp32)
      launch_residual_norm(x.p, nullptr, 0, 0, T, d.H, m.final_norm, d.eps, hb.p, nullptr, 0, hidden_stage.p, s);
    // compact fp16 rows of the output tokens for the vocabulary projection
    launch_residual_norm(x.p, nullptr, 0, 0, T, d.H, m.final_norm, d.eps, hb_out.p, out_token.p, R, nullptr, s);
    logits.ensure(size_t(R) * d.V);
    dense(m.lm_head, hb_out.p, max_rows, R, logits.p, d.V, size_t(R) * d.V, 1, s);
    stage(18);  // StateValidation (finite check + greedy selection)
    launch_argmax(logits.p, R, d.V, sampled.p, err.p, argmax_part.p, argmax_done.p, s);
    if (n_choice_rows) {
      const int32_t* rows_l = reinterpret_cast<const int32_t*>(choice_dev.p);
      const uint32_t* offs = choice_dev.p + n_choice_rows;
      launch_choice_select(logits.p, d.V, rows_l, offs, offs + n_choice_rows + 1, n_choice_rows, sampled.p, s);
    }
    launches += 1;
  }

  // ------------------------------------------------- reference-layout state
  // Writes version `id` in the layout of native/qwen_model.inc:268-271 (per
  // layer: DeltaNet conv history then recurrent state; attention K then V as
  // [kv][context][d]; all fp32, positions past the version's length zero).
  void export_snapshot(const StateId& id, float* output, size_t count) {
    const Version& v = table->get(id);
    if (count != d.state_count()) throw std::invalid_argument("snapshot capacity");
    set_device();
    QWEN_CUDA(cudaStreamSynchronize(stream));
    size_t off = 0;
    const size_t slot = id.slot, pos = id.position;
    std::vector<__nv_bfloat16> page(kv.page_elems());
    for (int li = 0; li < d.L; ++li) {
      const LayerDev& ly = store->model.layers[li];
      if (ly.mixer == 0) {
        const size_t cl = gdn.conv_elems, sl = gdn.state_elems;
        QWEN_CUDA(cudaMemcpy(output + off, gdn.conv + (slot * d.n_gdn + ly.type_index) * cl, cl * 4,
                             cudaMemcpyDeviceToHost));
        off += cl;
        QWEN_CUDA(cudaMemcpy(output + off, gdn.state + (slot * d.n_gdn + ly.type_index) * sl, sl * 4,
                             cudaMemcpyDeviceToHost));
        off += sl;
      } else {
        const size_t per = size_t(d.Hkv) * d.ctx * d.D;
        std::fill(output + off, output + off + 2 * per, 0.f);
        for (size_t pi = 0; pi < v.pages.size(); ++pi) {
          QWEN_CUDA(cudaMemcpy(page.data(), kv.page(ly.type_index, v.pages[pi]), page.size() * 2,
                               cudaMemcpyDeviceToHost));
          for (int kvsel = 0; kvsel < 2; ++kvsel)
            for (int g = 0; g < d.Hkv; ++g)
              for (int o = 0; o < kPageTokens; ++o) {
                const size_t p = pi * kPageTokens + o;
                if (p >= pos) continue;
                const __nv_bfloat16* src = page.data() + ((size_t(kvsel) * d.Hkv + g) * kPageTokens + o) * d.D;
                float* dst = output + off + kvsel * per + (size_t(g) * d.ctx + p) * d.D;
                for (int i = 0; i < d.D; ++i) dst[i] = __bfloat162float(src[i]);
              }
        }
        off += 2 * per;
      }
    }
    if (off != count) throw std::runtime_error("snapshot accounting");
    exports += count * 4;
  }

  // The inverse: a new version at `position` holding a reference-layout state
  // (rs_qwen_forward's old_state). K/V rows are stored in the bf16 cache.
  StateId import_snapshot(const float* flat, size_t position) {
    if (!position || position > size_t(d.ctx)) throw std::invalid_argument("imported state position");
    set_device();
    const int n_pages = d.n_attn > 0 ? int((position + kPageTokens - 1) / kPageTokens) : 0;
    if (n_pages > int(free_pages.size())) throw std::runtime_error("KV page pool exhausted");
    if (table->residents() + draft_residents() + 1 > slots) throw std::runtime_error("combined resident budget exhausted");
    StateId id = table->reserve(position, version_bytes(n_pages, 0));
    Version v;
    for (int j = 0; j < n_pages; ++j) {
      const int32_t p = free_pages.back();
      free_pages.pop_back();
      page_ref[p] = 1;
      page_filled[p] = uint8_t(std::min<size_t>(kPageTokens, position - size_t(j) * kPageTokens));
      v.pages.push_back(p);
    }
    try {
      QWEN_CUDA(cudaStreamSynchronize(stream));
      if (n_pages)
        QWEN_CUDA(cudaMemcpy(block_table.p + id.slot * size_t(bt_stride), v.pages.data(), size_t(n_pages) * 4,
                             cudaMemcpyHostToDevice));
      std::vector<uint16_t> page(kv.page_elems());
      size_t off = 0;
      for (int li = 0; li < d.L; ++li) {
        const LayerDev& ly = store->model.layers[li];
        if (ly.mixer == 0) {
          const size_t cl = gdn.conv_elems, sl = gdn.state_elems;
          QWEN_CUDA(cudaMemcpy(gdn.conv + (id.slot * d.n_gdn + ly.type_index) * cl, flat + off, cl * 4,
                               cudaMemcpyHostToDevice));
          off += cl;
          QWEN_CUDA(cudaMemcpy(gdn.state + (id.slot * d.n_gdn + ly.type_index) * sl, flat + off, sl * 4,
                               cudaMemcpyHostToDevice));
          off += sl;
        } else {
          const size_t per = size_t(d.Hkv) * d.ctx * d.D;
          for (int pi = 0; pi < n_pages; ++pi) {
            std::fill(page.begin(), page.end(), uint16_t(0));
            for (int kvsel = 0; kvsel < 2; ++kvsel)
              for (int g = 0; g < d.Hkv; ++g)
                for (int o = 0; o < kPageTokens; ++o) {
                  const size_t p = size_t(pi) * kPageTokens + o;
                  if (p >= position) continue;
                  const float* src = flat + off + kvsel * per + (size_t(g) * d.ctx + p) * d.D;
                  uint16_t* dst = page.data() + ((size_t(kvsel) * d.Hkv + g) * kPageTokens + o) * d.D;
                  for (int i = 0; i < d.D; ++i) dst[i] = float_to_bf16_bits(src[i]);
                }
            QWEN_CUDA(cudaMemcpy(kv.page(ly.type_index, v.pages[pi]), page.data(), page.size() * 2,
                                 cudaMemcpyHostToDevice));
          }
          off += 2 * per;
        }
      }
      if (off != d.state_count()) throw std::runtime_error("imported state accounting");
    } catch (...) {
      unref_pages(v.pages);
      table->rollback(id);
      throw;
    }
    table->publish(id, std::move(v));
    return id;
  }

  // ------------------------------------------------------------ MTP draft head
  // rs_qwen_device_mtp_attach (native/qwen_mtp.inc:2-6): must precede any admission.
  void mtp_attach(WeightStore* w) {
    set_device();
    if (!w || !w->ready || !w->model.has_mtp) throw std::invalid_argument("MTP weights missing (language_model.mtp.*)");
    if (w != store) throw std::invalid_argument("the MTP head must live in the session's weight store");
    if (mtp_on) throw std::invalid_argument("MTP already attached");
    if (table->residents()) throw std::invalid_argument("MTP attach must precede admission");
    mpage_bytes = size_t(2) * d.Hkv * kPageTokens * d.D * 2;
    // as many pages as the target pool (one attention layer each), at least a
    // full context for every slot when the target has no attention layers
    size_t pages = d.n_attn > 0 ? size_t(kv.n_pages) : slots * size_t(bt_stride);
    size_t free_b = 0, total_b = 0;
    QWEN_CUDA(cudaMemGetInfo(&free_b, &total_b));
    const size_t headroom = size_t(2) << 30;
    pages = std::min({pages, free_b > headroom ? (free_b - headroom) / mpage_bytes : size_t(0),
                      size_t(INT32_MAX / kPageTokens)});
    if (pages == 0) throw std::runtime_error("no device memory left for MTP KV pages");
    mkv_mem.ensure(pages * (mpage_bytes / 2));
    mkv.base = mkv_mem.p;
    mkv.n_pages = int(pages);
    mkv.layers = 1;
    mkv.Hkv = d.Hkv;
    mkv.D = d.D;
    mkv_map = make_kv_map(mkv, 0);
    mbt.ensure(slots * size_t(bt_stride));
    QWEN_CUDA(cudaMemset(mbt.p, 0, slots * size_t(bt_stride) * 4));
    mhidden.ensure(slots * size_t(kMaxDraft) * d.H);
    mcat.ensure(size_t(kMaxDraft) * 2 * d.H);
    mref.assign(pages, 0);
    mfilled.assign(pages, 0);
    mfree.resize(pages);
    for (size_t i = 0; i < pages; ++i) mfree[i] = int32_t(pages - 1 - i);
    drafts = std::make_unique<StateTable<DraftVersion>>(allocate_owner(), slots, limit);
    mtp_on = true;
  }

  void mtp_unref(const std::vector<int32_t>& pages) {
    for (int32_t p : pages)
      if (--mref[p] == 0) {
        mfilled[p] = 0;
        mfree.push_back(p);
      }
  }

  // rs_qwen_device_mtp_step (native/qwen_mtp.inc:8-56 and 133-181): `count`
  // draft tokens at positions [p, p + count), p = previous ? previous.position
  // : 0, each paired with a hidden row of `source` (a target version's kept
  // rows, or with draft_source the previous draft's last row). Writes the
  // vocabulary logits of the last token.
  void mtp_step(const StateId* previous, const StateId* source, int draft_source, size_t row,
                const uint32_t* toks, size_t count, StateId* output, float* logits_out) {
    set_device();
    if (!mtp_on) throw std::invalid_argument("MTP unavailable: attach a head first");
    if (!source || !toks || !output || !logits_out || draft_source < 0 || draft_source > 1 || !count ||
        count > size_t(kMaxDraft))
      throw std::invalid_argument("MTP descriptor");
    const size_t position = previous ? previous->position : 0;
    if (position > size_t(d.ctx) || count > size_t(d.ctx) - position) throw std::invalid_argument("MTP context capacity");
    for (size_t i = 0; i < count; ++i)
      if (toks[i] >= uint32_t(d.V)) throw std::invalid_argument("MTP token vocabulary");
    const DraftVersion* old = previous ? &drafts->get(*previous) : nullptr;
    const float* hidden_src = nullptr;
    if (draft_source) {
      const auto& src = drafts->get(*source);
      if (!previous || source->owner != previous->owner || source->slot != previous->slot ||
          source->generation != previous->generation || source->position != previous->position ||
          source->bytes != previous->bytes || count != 1 || row + 1 != src.hidden_rows)
        throw std::invalid_argument("MTP autoregressive parent identity");
      hidden_src = mhidden.p + (size_t(source->slot) * kMaxDraft + row) * d.H;
    } else {
      const auto& src = table->get(*source);
      const size_t rows = src.hidden_rows;
      if (!rows || row > rows || count > rows - row) throw std::invalid_argument("MTP hidden row capacity");
      if (source->position < rows || source->position - rows + row != position)
        throw std::invalid_argument("MTP target hidden alignment");
      hidden_src = hidden_pool.p + (size_t(source->slot) * d.chunk + row) * d.H;
    }
    const int pos = int(position), cnt = int(count);
    const int n_prefix = (pos + kPageTokens - 1) / kPageTokens;
    const int n_total = (pos + cnt + kPageTokens - 1) / kPageTokens;
    if (old && int(old->pages.size()) != n_prefix) throw std::runtime_error("MTP parent page list inconsistent");
    if (n_total > bt_stride) throw std::invalid_argument("context exceeds block table");
    const uint64_t charge = uint64_t(n_total) * mpage_bytes + uint64_t(count) * d.H * 4;
    if (table->residents() + draft_residents() >= slots || charge > limit - table->bytes() - draft_bytes())
      throw std::runtime_error("combined resident budget exhausted");
    // page planning (the target's rules on the draft pool)
    SeqDesc sd;
    std::memset(&sd, 0, sizeof(sd));
    sd.position = pos;
    sd.count = cnt;
    sd.parent = previous ? int32_t(previous->slot) : -1;
    sd.cow_src = -1;
    sd.cand = -1;
    int n_shared = n_prefix;
    if (pos % kPageTokens) {
      const int32_t lp = old->pages[n_prefix - 1];
      if (mfilled[lp] > pos % kPageTokens) {
        n_shared = n_prefix - 1;
        sd.cow_src = lp;
        sd.cow_len = pos % kPageTokens;
      } else {
        mfilled[lp] = uint8_t(std::min(kPageTokens, pos + cnt - (n_prefix - 1) * kPageTokens));
      }
    }
    const int n_new = n_total - n_shared;
    if (n_new > int(mfree.size())) throw std::runtime_error("MTP KV page pool exhausted");
    std::vector<int32_t> cp(old ? old->pages.begin() : cp.end(), old ? old->pages.begin() + n_shared : cp.end());
    for (int32_t p : cp) ++mref[p];
    std::vector<int32_t> fresh;
    for (int j = 0; j < n_new; ++j) {
      const int32_t p = mfree.back();
      mfree.pop_back();
      mref[p] = 1;
      mfilled[p] = uint8_t(std::min(kPageTokens, pos + cnt - (n_shared + j) * kPageTokens));
      fresh.push_back(p);
      cp.push_back(p);
    }
    sd.n_shared = n_shared;
    sd.new_off = 0;
    sd.n_new = n_new;
    sd.out_row0 = 0;
    sd.n_out = 1;
    StateId id{};
    bool reserved = false;
    try {
      id = drafts->reserve(position + count, charge);
      reserved = true;
      sd.child = int32_t(id.slot);
      // attention work list (16-page splits)
      std::vector<int2> items;
      for (int j = 0; j < cnt; ++j)
        for (int k = 0; k * 16 < (pos + j + kPageTokens) / kPageTokens; ++k) items.push_back(make_int2(j, k));
      const int splits = std::max(1, (pos + cnt + 16 * kPageTokens - 1) / (16 * kPageTokens));
      attn_ws.ensure(size_t(cnt) * d.Hq * splits * (d.D + 2));
      attn_items.ensure_grow(items.size(), stream);
      cudaStream_t s = stream;
      QWEN_CUDA(cudaMemcpyAsync(descs.p, &sd, sizeof(sd), cudaMemcpyHostToDevice, s));
      if (n_new) QWEN_CUDA(cudaMemcpyAsync(new_pages.p, fresh.data(), size_t(n_new) * 4, cudaMemcpyHostToDevice, s));
      QWEN_CUDA(cudaMemcpyAsync(tokens.p, toks, count * 4, cudaMemcpyHostToDevice, s));
      QWEN_CUDA(cudaMemcpyAsync(attn_items.p, items.data(), items.size() * 8, cudaMemcpyHostToDevice, s));
      QWEN_CUDA(cudaMemsetAsync(err.p, 0, 4, s));
      mtp_forward(cnt, hidden_src, int(items.size()), splits, sd.cow_src >= 0);
      QWEN_CUDA(cudaMemcpyAsync(mhidden.p + size_t(id.slot) * kMaxDraft * d.H, hidden_stage.p, count * d.H * 4,
                                cudaMemcpyDeviceToDevice, s));
      uint32_t h_err = 0;
      QWEN_CUDA(cudaMemcpyAsync(logits_out, logits.p, size_t(d.V) * 4, cudaMemcpyDeviceToHost, s));
      QWEN_CUDA(cudaMemcpyAsync(&h_err, err.p, 4, cudaMemcpyDeviceToHost, s));
      QWEN_CUDA(cudaStreamSynchronize(s));
      if (h_err & kErrNonFinite) throw std::runtime_error("nonfinite MTP result");
      if (h_err) throw std::runtime_error("MTP device error flag " + std::to_string(h_err));
    } catch (...) {
      cudaStreamSynchronize(stream);
      mtp_unref(cp);
      if (reserved) drafts->rollback(id);
      throw;
    }
    DraftVersion v;
    v.pages = std::move(cp);
    v.hidden_rows = uint32_t(count);
    drafts->publish(id, std::move(v));
    *output = id;
    ++calls;
  }

  // The MTP head over T tokens (native/qwen_mtp.inc:157-171): fc of the
  // normalised [embedding, target hidden], one gated-attention layer on the
  // draft pool, the MoE, the MTP norm; the target's lm_head on the last row.
  void mtp_forward(int T, const float* hidden_src, int n_items, int splits, bool cow) {
    cudaStream_t s = stream;
    const ModelDev& m = store->model;
    const LayerDev& ly = m.mtp_layer;
    Packed pk{cu_seqlens.p, token_seq.p, token_pos.p, slot_mapping.p, out_token.p};
    launch_pack(descs.p, 1, new_pages.p, mbt.p, bt_stride, pk, s);
    if (cow) launch_cow(mkv, descs.p, 1, new_pages.p, s);
    launch_mtp_input(m.embed, tokens.p, T, hidden_src, m.mtp_norm_emb, m.mtp_norm_hidden, d.eps, mcat.p, s);
    QWEN_CUDA(cudaMemsetAsync(x.p, 0, size_t(T) * d.H * 4, s));
    const size_t hstride = size_t(T) * d.H;
    const int fs = dense(m.mtp_fc, mcat.p, kMaxDraft, T, partial.p, d.H, hstride, kMaxSplits, s);
    launch_residual_norm(x.p, partial.p, fs, hstride, T, d.H, ly.in_norm, d.eps, hb.p, nullptr, 0, nullptr, s);
    const int aw = d.attn_in_rows;
    const size_t astride = size_t(T) * aw;
    const int ps = dense(ly.in_proj, hb.p, max_tokens, T, partial.p, aw, astride, kMaxSplits, s);
    launch_attn_prep(d, ly, partial.p, aw, ps, astride, token_pos.p, slot_mapping.p, T, mkv, 0, q.p, gate.p, s);
    launch_attn_decode(mkv_map, d, q.p, token_seq.p, token_pos.p, nullptr, descs.p, mbt.p, bt_stride, attn_items.p, n_items,
                       16, attn_ws.p, splits, err.p, s);
    launch_attention_merge(d, attn_ws.p, gate.p, token_pos.p, nullptr, T, 16, splits, hb2.p, s);
    const int os = dense(ly.out_proj, hb2.p, max_tokens, T, partial.p, d.H, hstride, kMaxSplits, s);
    launch_residual_norm(x.p, partial.p, os, hstride, T, d.H, ly.post_norm, d.eps, hb.p, nullptr, 0, nullptr, s);
    const int A = T * (d.top + 1);
    cur_layer = 0;
    in_mtp = true;
    try {
      moe(ly, T, A, s);
    } catch (...) {
      in_mtp = false;
      throw;
    }
    in_mtp = false;
    if (capture_routing) {  // the MTP layer's routing, reported as layer 0
      capture.ensure(size_t(std::max(1, d.L)) * A);
      QWEN_CUDA(cudaMemcpyAsync(capture.p, ids.p, size_t(A) * 4, cudaMemcpyDeviceToDevice, s));
      captured_tokens = T;
    }
    launch_moe_combine(x.p, moe_y.p, inv.p, weights.p, T, d.H, d.top + 1, nullptr, d.eps, hb.p, nullptr, 0, nullptr,
                       s);
    launch_residual_norm(x.p, nullptr, 0, 0, T, d.H, m.mtp_norm, d.eps, hb.p, nullptr, 0, hidden_stage.p, s);
    launch_residual_norm(x.p, nullptr, 0, 0, T, d.H, m.mtp_norm, d.eps, hb_out.p, out_token.p, 1, nullptr, s);
    logits.ensure(size_t(d.V));
    dense(m.lm_head, hb_out.p, max_rows, 1, logits.p, d.V, size_t(d.V), 1, s);
    launch_argmax(logits.p, 1, d.V, sampled.p, err.p, argmax_part.p, argmax_done.p, s);  // finite check
  }

  void mtp_release(const StateId& id) {
    set_device();
    if (!mtp_on) throw std::invalid_argument("MTP unavailable");
    std::vector<int32_t> pages = drafts->get(id).pages;
    drafts->release(id);
    mtp_unref(pages);
  }

  void ep_alloc(int world, int rank, int cap_tokens) {
    if (ep.on || ep.world > 1 || ep.window || ep.comm) throw std::invalid_argument("expert parallelism already initialised");
    if (world < 1 || rank < 0 || rank >= world || d.E % world) throw std::invalid_argument("expert-parallel geometry");
    if (cap_tokens < 1 || cap_tokens > max_tokens) throw std::invalid_argument("expert-parallel token capacity");
    set_device();
    ep.world = world;
    ep.rank = rank;
    ep.per_rank = d.E / world;
    ep.cap_tokens = cap_tokens;
    ep.cap = cap_tokens * d.top;
    ep.hdr_ints = (ep.per_rank + 3) & ~3;
    ep.stage_bytes = size_t(ep.hdr_ints) * 4 + size_t(ep.cap) * d.H * 2;
    ep.max_rows = world * ep.cap + cap_tokens;  // routed rows from every source + this rank's shared rows
    ep.xloc.ensure(size_t(ep.max_rows) * d.H);
    ep.actloc.ensure(size_t(ep.max_rows) * d.I);
    ep.yloc.ensure(size_t(ep.max_rows) * d.H);
    ep.goff.ensure(d.E + 2);
    ep.seg.ensure(size_t(2) * world * ep.per_rank);
    ep.origin.ensure(ep.max_rows);
    ep.n_rows.ensure(1);
    ep.done.ensure(2);
    QWEN_CUDA(cudaMemset(ep.done.p, 0, 8));
    for (auto* t : {&ep.disp_dst, &ep.ret_dst, &ep.disp_flag, &ep.ret_flag, &ep.srcs, &ep.rsrcs}) t->ensure(world);
  }
  void ep_tables(const std::vector<uint64_t>& disp_dst, const std::vector<uint64_t>& ret_dst,
                 const std::vector<uint64_t>& disp_flag, const std::vector<uint64_t>& ret_flag,
                 const std::vector<uint64_t>& srcs, const std::vector<uint64_t>& rsrcs) {
    const size_t b = size_t(ep.world) * 8;
    QWEN_CUDA(cudaMemcpy(ep.disp_dst.p, disp_dst.data(), b, cudaMemcpyHostToDevice));
    QWEN_CUDA(cudaMemcpy(ep.ret_dst.p, ret_dst.data(), b, cudaMemcpyHostToDevice));
    QWEN_CUDA(cudaMemcpy(ep.disp_flag.p, disp_flag.data(), b, cudaMemcpyHostToDevice));
    QWEN_CUDA(cudaMemcpy(ep.ret_flag.p, ret_flag.data(), b, cudaMemcpyHostToDevice));
    QWEN_CUDA(cudaMemcpy(ep.srcs.p, srcs.data(), b, cudaMemcpyHostToDevice));
    QWEN_CUDA(cudaMemcpy(ep.rsrcs.p, rsrcs.data(), b, cudaMemcpyHostToDevice));
  }

  // NCCL transport.
  void ep_init(int world, int rank, const ncclUniqueId& uid, int cap_tokens) {
    ep_alloc(world, rank, cap_tokens);
    ep.send.ensure(size_t(world) * ep.stage_bytes);
    ep.recv.ensure(size_t(world) * ep.stage_bytes);
    ep.rsend.ensure(size_t(world) * ep.cap * d.H);
    ep.rrecv.ensure(size_t(world) * ep.cap * d.H);
    std::vector<uint64_t> dd(world), rd(world), z(world, 0), sr(world), rs(world);
    for (int p = 0; p < world; ++p) {
      dd[p] = reinterpret_cast<uint64_t>(ep.send.p + size_t(p) * ep.stage_bytes);
      rd[p] = reinterpret_cast<uint64_t>(ep.rsend.p + size_t(p) * ep.cap * d.H);
      sr[p] = reinterpret_cast<uint64_t>((p == rank ? ep.send.p : ep.recv.p) + size_t(p) * ep.stage_bytes);
      rs[p] = reinterpret_cast<uint64_t>((p == rank ? ep.rsend.p : ep.rrecv.p) + size_t(p) * ep.cap * d.H);
    }
    ep_tables(dd, rd, z, z, sr, rs);
    const ncclResult_t r = ncclCommInitRank(&ep.comm, world, uid, rank);
    if (r != ncclSuccess) throw std::runtime_error(std::string("ncclCommInitRank: ") + ncclGetErrorString(r));
    ep.on = true;
  }

  // Direct NVLink transport, step 1: this rank's window (stages addressed to
  // it and its flags), exported as a CUDA IPC handle.
  void ep_window(int world, int rank, int cap_tokens, cudaIpcMemHandle_t* handle) {
    ep_alloc(world, rank, cap_tokens);
    ep.disp_bytes = size_t(world) * ep.stage_bytes;
    ep.ret_bytes = size_t(world) * ep.cap * d.H * 4;
    ep.win_bytes = ep.disp_bytes + ep.ret_bytes + 256;
    QWEN_CUDA(cudaMalloc(&ep.window, ep.win_bytes));
    QWEN_CUDA(cudaMemset(ep.window + ep.disp_bytes + ep.ret_bytes, 0, 256));  // epoch flags start at 0
    QWEN_CUDA(cudaIpcGetMemHandle(handle, ep.window));
  }
  // Step 2: open every peer's window and build the tables.
  void ep_connect(const cudaIpcMemHandle_t* handles) {
    if (!ep.window || ep.on) throw std::invalid_argument("expert-parallel window missing or already connected");
    set_device();
    const int world = ep.world, me = ep.rank;
    ep.peer_windows.assign(world, nullptr);
    std::vector<uint8_t*> win(world);
    for (int p = 0; p < world; ++p) {
      if (p == me) {
        win[p] = ep.window;
        continue;
      }
      void* ptr = nullptr;
      QWEN_CUDA(cudaIpcOpenMemHandle(&ptr, handles[p], cudaIpcMemLazyEnablePeerAccess));
      ep.peer_windows[p] = ptr;
      win[p] = static_cast<uint8_t*>(ptr);
    }
    const size_t flags_off = ep.disp_bytes + ep.ret_bytes;
    std::vector<uint64_t> dd(world), rd(world), df(world), rf(world), sr(world), rs(world);
    for (int p = 0; p < world; ++p) {
      dd[p] = reinterpret_cast<uint64_t>(win[p] + size_t(me) * ep.stage_bytes);
      rd[p] = reinterpret_cast<uint64_t>(win[p] + ep.disp_bytes + size_t(me) * ep.cap * d.H * 4);
      df[p] = reinterpret_cast<uint64_t>(win[p] + flags_off + size_t(me) * 4);
      rf[p] = reinterpret_cast<uint64_t>(win[p] + flags_off + size_t(world + me) * 4);
      sr[p] = reinterpret_cast<uint64_t>(ep.window + size_t(p) * ep.stage_bytes);
      rs[p] = reinterpret_cast<uint64_t>(ep.window + ep.disp_bytes + size_t(p) * ep.cap * d.H * 4);
    }
    ep_tables(dd, rd, df, rf, sr, rs);
    ep.wait_disp = reinterpret_cast<const uint32_t*>(ep.window + flags_off);
    ep.wait_ret = ep.wait_disp + world;
    ep.p2p = true;
    ep.on = true;
  }

  // One grouped exchange of equal-size buffers with every other rank.
  void ep_exchange(const void* send, void* recv, size_t bytes, cudaStream_t s) {
    ncclResult_t r = ncclGroupStart();
    for (int p = 0; p < ep.world && r == ncclSuccess; ++p) {
      if (p == ep.rank) continue;
      r = ncclSend(static_cast<const uint8_t*>(send) + size_t(p) * bytes, bytes, ncclUint8, p, ep.comm, s);
      if (r == ncclSuccess) r = ncclRecv(static_cast<uint8_t*>(recv) + size_t(p) * bytes, bytes, ncclUint8, p, ep.comm, s);
    }
    const ncclResult_t r2 = ncclGroupEnd();
    if (r != ncclSuccess || r2 != ncclSuccess)
      throw std::runtime_error(std::string("expert-parallel exchange: ") + ncclGetErrorString(r != ncclSuccess ? r : r2));
  }

  // The MoE block with the routed experts split over the ranks (see EpState).
  void moe_ep(const LayerDev& ly, int T, int A, cudaStream_t s) {
    if (T > ep.cap_tokens) throw std::logic_error("expert-parallel step above its token capacity");
    const int world = ep.world;
    const uint32_t epoch = ++ep.epoch;  // the same on every rank (lockstep)
    uint32_t* const* dflag = ep.p2p ? reinterpret_cast<uint32_t* const*>(ep.disp_flag.p) : nullptr;
    uint32_t* const* rflag = ep.p2p ? reinterpret_cast<uint32_t* const*>(ep.ret_flag.p) : nullptr;
    launch_ep_pack(hb.p, d.H, perm.p, d.top + 1, counts.p, offsets.p, reinterpret_cast<uint8_t* const*>(ep.disp_dst.p),
                   world, ep.per_rank, ep.hdr_ints, ep.cap, d.H, dflag, epoch, ep.done.p, s);
    if (!ep.p2p) {
      stage(15);  // MoeMerge: the expert-parallel exchanges
      ep_exchange(ep.send.p, ep.recv.p, ep.stage_bytes, s);
      stage(11);  // MoeUpGate
    }
    launch_ep_plan_gather(reinterpret_cast<const uint8_t* const*>(ep.srcs.p), world, ep.rank, ep.per_rank, ep.hdr_ints,
                          d.E, counts.p, offsets.p, hb.p, d.H, perm.p, d.top + 1, ep.goff.p, ep.seg.p, ep.n_rows.p,
                          ep.xloc.p, ep.origin.p,
                          ep.cap, d.H, ep.max_rows, err.p, ep.p2p ? ep.wait_disp : nullptr, epoch, sm_count, s);
    const int per_expert = (world * T * d.top + T + d.E) / (d.E + 1);
    const int box = box_for(std::max(1, 2 * per_expert));
    TcArgs gu;
    gu.W = ly.expert_gu;
    gu.mode = kGemmGateUp;
    gu.expert_tiles = 2 * d.I / kTileRows;
    gu.groups = d.E + 1;
    gu.group_off = ep.goff.p;
    gu.box_rows = box;
    gu.Yb = ep.actloc.p;
    gu.ldyb = d.I;
    gu.err = err.p;
    launch_tc(ep.xloc.p, ep.max_rows, gu, s);
    stage(12);  // MoeDown
    TcArgs dn;
    dn.W = ly.expert_dn;
    dn.mode = kGemmDown;
    dn.expert_tiles = d.H / kTileRows;
    dn.groups = d.E + 1;
    dn.group_off = ep.goff.p;
    dn.box_rows = box;
    dn.Y = ep.yloc.p;
    dn.ldy = d.H;
    dn.err = err.p;
    launch_tc(ep.actloc.p, ep.max_rows, dn, s);
    launch_ep_return(ep.yloc.p, ep.origin.p, ep.n_rows.p, reinterpret_cast<float* const*>(ep.ret_dst.p), moe_y.p,
                     ep.cap, d.H, world, ep.max_rows, rflag, epoch, ep.done.p + 1, sm_count, s);
    if (!ep.p2p) {
      stage(15);  // MoeMerge
      ep_exchange(ep.rsend.p, ep.rrecv.p, size_t(ep.cap) * d.H * 4, s);
      stage(12);  // MoeDown
    }
    launch_ep_return_unpack(reinterpret_cast<const float* const*>(ep.rsrcs.p), offsets.p, moe_y.p, world, ep.per_rank,
                            d.H, A, ep.p2p ? ep.wait_ret : nullptr, epoch, err.p, sm_count, s);
  }

  void moe(const LayerDev& ly, int T, int A, cudaStream_t s) {
    stage(10);  // MoeRouting
    const int rw = d.E + 1;
    const size_t rstride = size_t(T) * rw;
    const int rs = dense(ly.router, hb.p, max_tokens, T, partial.p, rw, rstride, kMaxSplits, s);
    launch_route(partial.p, rw, rs, rstride, T, d.E, d.top, ids.p, weights.p,
                 capture_routing ? cap_logits.p + size_t(cur_layer) * T * (d.E + 1) : nullptr, s);
    const bool ep_layer = ep.on && !in_mtp && !simple_gemm;
    if (ep_layer || simple_gemm)  // these read the input rows through the permutation themselves
      launch_expert_sort(ids.p, A, d.top + 1, d.E + 1, counts.p, offsets.p, perm.p, inv.p, err.p, s);
    else  // the grouped tcgen05 GEMM reads its input rows in expert order
      launch_expert_sort_gather(ids.p, A, d.top + 1, d.E + 1, counts.p, offsets.p, perm.p, inv.p, err.p, hb.p, d.H,
                                d.H, xperm.p, sm_count, s);
    stage(11);  // MoeUpGate
    if (ep_layer) {
      moe_ep(ly, T, A, s);
      return;
    }
    if (simple_gemm) {
      GemmArgs gu;
      gu.W = ly.expert_gu;
      gu.mode = kGemmGateUp;
      gu.expert_tiles = 2 * d.I / kTileRows;
      gu.X = hb.p;
      gu.ldx = d.H;
      gu.x_row = perm.p;
      gu.x_div = d.top + 1;
      gu.group_off = offsets.p;
      gu.groups = d.E + 1;
      gu.Yb = act.p;
      gu.ldyb = d.I;
      launch_qgemm(gu, s);
      stage(12);  // MoeDown
      GemmArgs dn;
      dn.W = ly.expert_dn;
      dn.mode = kGemmDown;
      dn.expert_tiles = d.H / kTileRows;
      dn.X = act.p;
      dn.ldx = d.I;
      dn.group_off = offsets.p;
      dn.groups = d.E + 1;
      dn.Y = moe_y.p;
      dn.ldy = d.H;
      launch_qgemm(dn, s);
      return;
    }
    // Token block of the grouped GEMMs: the mean rows per expert plus two
    // standard deviations of a binomial count, so nearly every expert fits one
    // block (a larger block re-reads more activation rows per weight tile and
    // runs wider MMAs on padding; an expert over the block takes a second one)
    const int per_expert = (A + d.E) / (d.E + 1);
    const int box = box_for(std::max(1, per_expert + int(2.0 * std::sqrt(double(per_expert)) + 0.5)));
    TcArgs gu;
    gu.W = ly.expert_gu;
    gu.mode = kGemmGateUp;
    gu.expert_tiles = 2 * d.I / kTileRows;
    gu.groups = d.E + 1;
    gu.group_off = offsets.p;
    gu.box_rows = box;
    gu.Yb = act.p;
    gu.ldyb = d.I;
    gu.err = err.p;
    const int a_cap = max_tokens * (d.top + 1);
    launch_tc(xperm.p, a_cap, gu, s);
    stage(12);  // MoeDown
    TcArgs dn;
    dn.W = ly.expert_dn;
    dn.mode = kGemmDown;
    dn.expert_tiles = d.H / kTileRows;
    dn.groups = d.E + 1;
    dn.group_off = offsets.p;
    dn.box_rows = box;
    dn.Y = moe_y.p;
    dn.ldy = d.H;
    dn.err = err.p;
    launch_tc(act.p, a_cap, dn, s);
  }
};

Session* S(void* h) {
  if (!h) throw std::invalid_argument("null session");
  return static_cast<Session*>(h);
}

// rs_qwen_forward's session: two state slots (the imported parent, then the
// child that consumes it in place), KV pages for one full context, scratch
// for one chunk. Kept in the weight store and remade when the config changes.
Session& forward_session(WeightStore* w, const rs_qwen_config& c, const rs_qwen_layer* layers, size_t count) {
  const uint8_t* key = reinterpret_cast<const uint8_t*>(&c);
  if (w->forward_session && w->forward_key.size() == sizeof(c) &&
      std::memcmp(w->forward_key.data(), key, sizeof(c)) == 0)
    return *static_cast<Session*>(w->forward_session.get());
  w->forward_session.reset();
  w->forward_key.clear();
  const Dims d = Dims::from(c);
  const uint64_t gdn_slot = uint64_t(d.n_gdn) * (size_t(d.hv) * d.dv * d.dk + size_t(d.conv - 1) * d.cd) * 4;
  const uint64_t page = uint64_t(d.n_attn) * 2 * d.Hkv * kPageTokens * d.D * 2;
  const uint64_t pages = d.ctx > 0 ? uint64_t(d.ctx + kPageTokens - 1) / kPageTokens + 2 : 0;
  auto sess = std::make_unique<Session>();
  sess->init(w, 1, c, layers, count, 2, 2 * gdn_slot + pages * page + 1, std::max(1, c.chunk));
  w->forward_session = std::shared_ptr<void>(sess.release(), [](void* p) {
    auto* ss = static_cast<Session*>(p);
    cudaSetDevice(ss->device);
    cudaStreamSynchronize(ss->stream);
    delete ss;
  });
  w->forward_key.assign(key, key + sizeof(c));
  return *static_cast<Session*>(w->forward_session.get());
}

}  // namespace

// ----------------------------------------------------------------- C ABI --
extern "C" {

const char* rs_mlx_version(void) { return "qwen-b200-cuda sm_100a"; }

size_t rs_qwen_state_count(const rs_qwen_config* c) { return c ? Dims::from(*c).state_count() : 0; }

void* rs_mlx_weights_create(char* error, size_t capacity) {
  void* out = nullptr;
  checked(error, capacity, [&] {
    auto* w = new WeightStore();
    // the store binds to the calling thread's current device when its device
    // layout is built; reading checkpoint shards needs no device
    if (cudaGetDevice(&w->device) != cudaSuccess) {
      w->device = -1;
      cudaGetLastError();
    }
    out = w;
  });
  return out;
}

void rs_mlx_weights_destroy(void* store) { delete static_cast<WeightStore*>(store); }

int rs_mlx_weights_load(void* store, const char* file, char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    if (!store || !file) throw std::invalid_argument("invalid weight load descriptor");
    static_cast<WeightStore*>(store)->load(file);
  });
}

int rs_qwen_quant(void* store, const char* module, int group, int bits, char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    if (!store || !module || !(group == 32 || group == 64 || group == 128) ||
        !(bits == 2 || bits == 3 || bits == 4 || bits == 5 || bits == 6 || bits == 8))
      throw std::invalid_argument("invalid model quantization");
    auto* w = static_cast<WeightStore*>(store);
    if (w->ready) throw std::invalid_argument("quantization overrides must precede the device layout");
    w->quant[module] = {group, bits};
  });
}

// One-shot forward of `count` tokens at `offset` from a reference-layout state
// (native/qwen_model.inc:278-373 semantics): old_state in, new_state and the
// last row's logits out. Runs the same ragged CUDA step as the device session.
int rs_qwen_forward(void* store, int gpu, const rs_qwen_config* config, const rs_qwen_layer* layers,
                    size_t layer_count, const uint32_t* tokens, size_t count, size_t offset, const float* old_state,
                    size_t old_count, float* new_state, size_t new_count, float* logits, size_t logits_count,
                    int projection_checks, const uint32_t* projection_outputs, size_t projection_output_count,
                    float* trace, size_t trace_count, char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    if (!store || !config || !layers || !tokens || !new_state || !logits)
      throw std::invalid_argument("invalid model descriptor");
    const rs_qwen_config& c = *config;
    if (c.chunk <= 0 || c.chunk > 8 || c.context <= 0 || count == 0 || count > size_t(c.chunk) ||
        offset + count > size_t(c.context) || logits_count != size_t(c.vocab))
      throw std::invalid_argument("model geometry/capacity");
    if (gpu != 1) throw std::invalid_argument("rs_qwen_forward: the CUDA backend has no CPU path (gpu must be 1)");
    if (projection_checks || projection_outputs || projection_output_count || trace || trace_count)
      throw std::invalid_argument("rs_qwen_forward: projection checks and layer traces are MLX diagnostics the "
                                  "CUDA backend does not provide");
    const Dims d = Dims::from(c);
    if (new_count != d.state_count() || (offset ? (old_count != d.state_count() || !old_state) : old_count != 0))
      throw std::invalid_argument("model state length");
    for (size_t i = 0; i < count; ++i)
      if (tokens[i] >= uint32_t(c.vocab)) throw std::invalid_argument("token outside vocabulary");
    auto* w = static_cast<WeightStore*>(store);
    if (!w->ready) throw std::invalid_argument("weight store is empty");
    int caller_device = 0;
    QWEN_CUDA(cudaGetDevice(&caller_device));
    try {
      Session& s = forward_session(w, c, layers, layer_count);
      StateId parent{};
      const bool have = offset > 0;
      if (have) parent = s.import_snapshot(old_state, offset);
      Session::SeqIn in{have ? &parent : nullptr, uint32_t(offset), uint32_t(count), tokens};
      StateId out{};
      s.step({in}, RS_QWEN_RAGGED_LOGITS | (have ? RS_QWEN_RAGGED_CONSUME : 0u), &out, nullptr, logits);
      try {
        s.export_snapshot(out, new_state, new_count);
      } catch (...) {
        std::vector<int32_t> pages = s.table->get(out).pages;
        s.table->release(out);
        s.unref_pages(pages);
        throw;
      }
      std::vector<int32_t> pages = s.table->get(out).pages;
      s.table->release(out);
      s.unref_pages(pages);
    } catch (...) {
      w->forward_session.reset();  // a failed call leaves no half-imported state behind
      w->forward_key.clear();
      cudaSetDevice(caller_device);
      throw;
    }
    QWEN_CUDA(cudaSetDevice(caller_device));
  });
}

// The reference's generic MLX graph builder (native/mlx_bridge.h:8-43), used by
// its in-process MLX executor (src/serving/native_mlx.rs). This backend runs
// no MLX graphs: each entry point reports that with the ABI's error
// convention, so a caller built against the full surface links and fails
// cleanly at run time.
static const char kNoGraph[] = "the MLX graph interface is not provided by the CUDA backend (no MLX graphs run here)";

void* rs_mlx_create(int gpu, char* error, size_t capacity) {
  (void)gpu;
  report(error, capacity, kNoGraph);
  return nullptr;
}
void rs_mlx_destroy(void* graph) { (void)graph; }
int rs_mlx_input(void* graph, int dtype, const void* data, const int32_t* shape, size_t rank, char* error,
                 size_t capacity) {
  (void)graph, (void)dtype, (void)data, (void)shape, (void)rank;
  report(error, capacity, kNoGraph);
  return -1;
}
int rs_mlx_op(void* graph, int op, const uint32_t* inputs, size_t count, int group, float epsilon, char* error,
              size_t capacity) {
  (void)graph, (void)op, (void)inputs, (void)count, (void)group, (void)epsilon;
  report(error, capacity, kNoGraph);
  return -1;
}
int rs_mlx_finish(void* graph, uint32_t output, void* data, size_t elements, char* error, size_t capacity) {
  (void)graph, (void)output, (void)data, (void)elements;
  report(error, capacity, kNoGraph);
  return -1;
}
int rs_mlx_kernel(void* graph, int op, const uint32_t* inputs, size_t count, const int32_t* ints, size_t ni,
                  const float* floats, size_t nf, char* error, size_t capacity) {
  (void)graph, (void)op, (void)inputs, (void)count, (void)ints, (void)ni, (void)floats, (void)nf;
  report(error, capacity, kNoGraph);
  return -1;
}
int rs_mlx_parameter(void* graph, void* store, const char* name, const int32_t* shape, size_t rank, int dtype,
                     char* error, size_t capacity) {
  (void)graph, (void)store, (void)name, (void)shape, (void)rank, (void)dtype;
  report(error, capacity, kNoGraph);
  return -1;
}
// The reference clears MLX's per-thread streams when an executor thread exits
// (native/mlx_bridge.cpp:96); sessions here own their CUDA streams, so there is
// nothing per-thread to release.
void rs_mlx_cleanup(void) {}

int rs_mlx_weight_bytes(void* store, const char* name, const int32_t* shape, size_t rank, int dtype,
                        size_t offset, uint8_t* output, size_t count, char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    if (!store || !name || !output) throw std::invalid_argument("invalid weight bytes descriptor");
    auto* w = static_cast<WeightStore*>(store);
    auto hit = w->host.find(name);
    if (hit != w->host.end()) {  // a checkpoint tensor (native/mlx_bridge.cpp:179-185 checks)
      const HostTensor& t = hit->second;
      if (dtype != t.dtype || (shape && (rank != t.shape.size() ||
                                         !std::equal(t.shape.begin(), t.shape.end(), shape,
                                                     [](int64_t a, int32_t b) { return a == int64_t(b); }))))
        throw std::invalid_argument("weight byte export bounds/type");
      w->export_bytes(name, offset, output, count);
      return;
    }
    if (dtype != 0 && dtype != 2) throw std::invalid_argument("weight bytes dtype");
    QWEN_CUDA(cudaSetDevice(w->device));
    w->export_bytes(name, offset, output, count);
  });
}

int rs_qwen_weights_synthetic(void* store, const rs_qwen_config* config, uint64_t seed, int with_mtp,
                              char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    if (!store || !config) throw std::invalid_argument("invalid synthetic weight descriptor");
    auto* w = static_cast<WeightStore*>(store);
    if (w->device < 0) QWEN_CUDA(cudaGetDevice(&w->device));
    QWEN_CUDA(cudaSetDevice(w->device));
    w->synthesize(*config, seed, with_mtp != 0);
  });
}

void* rs_qwen_device_create(void* weights, int gpu, const rs_qwen_config* config, const rs_qwen_layer* layers,
                            size_t count, size_t slots, uint64_t bytes, char* error, size_t capacity) {
  void* out = nullptr;
  checked(error, capacity, [&] {
    if (!weights || !config || !layers) throw std::invalid_argument("device session descriptor");
    auto* w = static_cast<WeightStore*>(weights);
    if (!w->ready && !w->host.empty()) {  // a loaded checkpoint: build its device layout on this device
      QWEN_CUDA(cudaGetDevice(&w->device));
      w->materialize(*config);
    }
    auto s = std::make_unique<Session>();
    s->init(static_cast<WeightStore*>(weights), gpu, *config, layers, count, slots, bytes);
    out = s.release();
  });
  return out;
}

void rs_qwen_device_destroy(void* session) {
  if (!session) return;
  auto* s = static_cast<Session*>(session);
  cudaSetDevice(s->device);
  cudaStreamSynchronize(s->stream);
  delete s;
}

int rs_qwen_device_step_ragged(void* session, size_t n_seq, const StateId* parents, const uint32_t* positions,
                               const uint32_t* counts, const uint32_t* tokens_flat, uint32_t flags,
                               StateId* outs, uint32_t* sampled, size_t sampled_count, float* logits,
                               size_t logits_count, char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!n_seq || !positions || !counts || !tokens_flat || !outs) throw std::invalid_argument("ragged step descriptor");
    if (flags & ~uint32_t(31)) throw std::invalid_argument("unknown ragged step flags");
    std::vector<Session::SeqIn> seqs(n_seq);
    size_t off = 0, rows = 0;
    for (size_t i = 0; i < n_seq; ++i) {
      const bool has_parent = parents && positions[i] != 0;
      seqs[i] = {has_parent ? &parents[i] : nullptr, positions[i], counts[i], tokens_flat + off};
      off += counts[i];
      rows += (flags & RS_QWEN_RAGGED_ALL_ROWS) ? counts[i] : 1;
    }
    if ((flags & RS_QWEN_RAGGED_SAMPLED) && (!sampled || sampled_count != rows))
      throw std::invalid_argument("sampled output capacity");
    if ((flags & RS_QWEN_RAGGED_LOGITS) && (!logits || logits_count != rows * size_t(s->d.V)))
      throw std::invalid_argument("logits output capacity");
    s->step(seqs, flags, outs, (flags & RS_QWEN_RAGGED_SAMPLED) ? sampled : nullptr,
            (flags & RS_QWEN_RAGGED_LOGITS) ? logits : nullptr);
  });
}

int rs_qwen_device_step_ragged_choices(void* session, size_t n_seq, const StateId* parents,
                                       const uint32_t* positions, const uint32_t* counts, const uint32_t* tokens_flat,
                                       uint32_t flags, const uint32_t* allowed_offsets, const uint32_t* allowed_ids,
                                       size_t allowed_count, StateId* outs, uint32_t* sampled, size_t sampled_count,
                                       float* logits, size_t logits_count, char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!n_seq || !positions || !counts || !tokens_flat || !outs || !allowed_offsets)
      throw std::invalid_argument("ragged step descriptor");
    if (flags & ~uint32_t(31)) throw std::invalid_argument("unknown ragged step flags");
    if (!(flags & RS_QWEN_RAGGED_SAMPLED)) throw std::invalid_argument("constrained selection needs sampled tokens");
    std::vector<Session::SeqIn> seqs(n_seq);
    size_t off = 0, rows = 0;
    for (size_t i = 0; i < n_seq; ++i) {
      const bool has_parent = parents && positions[i] != 0;
      seqs[i] = {has_parent ? &parents[i] : nullptr, positions[i], counts[i], tokens_flat + off};
      off += counts[i];
      rows += (flags & RS_QWEN_RAGGED_ALL_ROWS) ? counts[i] : 1;
    }
    if (!sampled || sampled_count != rows) throw std::invalid_argument("sampled output capacity");
    if ((flags & RS_QWEN_RAGGED_LOGITS) && (!logits || logits_count != rows * size_t(s->d.V)))
      throw std::invalid_argument("logits output capacity");
    const Session::ChoiceIn ch{allowed_offsets, allowed_ids, allowed_count};
    s->step(seqs, flags, outs, sampled, (flags & RS_QWEN_RAGGED_LOGITS) ? logits : nullptr, nullptr, &ch);
  });
}

int rs_qwen_device_decode_batch(void* session, const StateId* parents, const uint32_t* tokens, size_t batch,
                                StateId* outputs, float* logits, size_t logits_count, char* error,
                                size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!parents || !tokens || !outputs || !logits || batch < 1) throw std::invalid_argument("batch descriptor");
    if (logits_count != batch * size_t(s->d.V)) throw std::invalid_argument("batch geometry");
    std::vector<Session::SeqIn> seqs(batch);
    for (size_t i = 0; i < batch; ++i) {
      if (!parents[i].position) throw std::invalid_argument("batch parent/token geometry");
      seqs[i] = {&parents[i], uint32_t(parents[i].position), 1, tokens + i};
    }
    s->step(seqs, RS_QWEN_RAGGED_LOGITS, outputs, nullptr, logits);
  });
}

static int device_step(void* session, const StateId* previous, size_t position, const uint32_t* tokens,
                       size_t count, StateId* output, float* logits, size_t logits_count, char* error,
                       size_t capacity, bool all_logits, bool hidden, uint32_t* sampled) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!output || !tokens || (!logits && !sampled)) throw std::invalid_argument("device step descriptor");
    if (!count || count > size_t(s->d.chunk) || position > size_t(s->d.ctx) ||
        count > size_t(s->d.ctx) - position ||
        (sampled ? logits_count != 0 : logits_count != size_t(s->d.V) * (all_logits ? count : 1)))
      throw std::invalid_argument("device step capacity");
    if ((position == 0) != (previous == nullptr)) throw std::invalid_argument("device previous state presence");
    std::vector<Session::SeqIn> seqs{{previous, uint32_t(position), uint32_t(count), tokens}};
    uint32_t flags = (sampled ? RS_QWEN_RAGGED_SAMPLED : RS_QWEN_RAGGED_LOGITS) |
                     (all_logits ? RS_QWEN_RAGGED_ALL_ROWS : 0) | (hidden ? RS_QWEN_RAGGED_HIDDEN : 0);
    s->step(seqs, flags, output, sampled, logits);
  });
}

int rs_qwen_device_step(void* h, const StateId* p, size_t position, const uint32_t* t, size_t n, StateId* out,
                        float* logits, size_t lc, float* trace, size_t tc, char* e, size_t ec) {
  if (trace || tc) {
    report(e, ec, "trace capture is an MLX-baseline diagnostic not offered by the CUDA backend");
    return -1;
  }
  return device_step(h, p, position, t, n, out, logits, lc, e, ec, false, false, nullptr);
}
int rs_qwen_device_step_sampled(void* h, const StateId* p, size_t position, const uint32_t* t, size_t n,
                                StateId* out, uint32_t* token, char* e, size_t ec) {
  if (!token) {
    report(e, ec, "device step descriptor");
    return -1;
  }
  return device_step(h, p, position, t, n, out, nullptr, 0, e, ec, false, false, token);
}
int rs_qwen_device_block(void* h, const StateId* p, size_t position, const uint32_t* t, size_t n, StateId* out,
                         float* logits, size_t lc, char* e, size_t ec) {
  return device_step(h, p, position, t, n, out, logits, lc, e, ec, true, false, nullptr);
}
int rs_qwen_device_hidden_step(void* h, const StateId* p, size_t position, const uint32_t* t, size_t n,
                               StateId* out, float* logits, size_t lc, char* e, size_t ec) {
  return device_step(h, p, position, t, n, out, logits, lc, e, ec, false, true, nullptr);
}
int rs_qwen_device_hidden_block(void* h, const StateId* p, size_t position, const uint32_t* t, size_t n,
                                StateId* out, float* logits, size_t lc, char* e, size_t ec) {
  return device_step(h, p, position, t, n, out, logits, lc, e, ec, true, true, nullptr);
}

int rs_qwen_device_release(void* session, const StateId* id, char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!id) throw std::invalid_argument("release descriptor");
    std::vector<int32_t> pages = s->table->get(*id).pages;
    s->table->release(*id);
    s->unref_pages(pages);
  });
}

int rs_qwen_device_snapshot(void* session, const StateId* id, float* output, size_t count, char* error,
                            size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!id || !output) throw std::invalid_argument("snapshot descriptor");
    s->export_snapshot(*id, output, count);
  });
}

int rs_qwen_device_hidden_snapshot(void* session, const StateId* id, float* output, size_t count, char* error,
                                   size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!id || !output) throw std::invalid_argument("hidden snapshot descriptor");
    const Version& v = s->table->get(*id);
    if (!v.hidden_rows || count != size_t(v.hidden_rows) * s->d.H)
      throw std::invalid_argument("missing hidden or snapshot capacity");
    s->set_device();
    QWEN_CUDA(cudaStreamSynchronize(s->stream));
    QWEN_CUDA(cudaMemcpy(output, s->hidden_pool.p + id->slot * size_t(s->d.chunk) * s->d.H, count * 4,
                         cudaMemcpyDeviceToHost));
    s->exports += count * 4;
  });
}

int rs_qwen_device_stats(void* session, uint64_t* output, size_t count, char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!output || count != kStatsCount) throw std::invalid_argument("stats capacity");
    std::fill(output, output + count, 0);
    output[0] = s->table->residents();
    output[1] = s->table->bytes();
    output[2] = s->exports;
    output[3] = s->uploads;
    output[4] = s->steps;
    size_t free_b = 0, total_b = 0;
    s->set_device();
    if (cudaMemGetInfo(&free_b, &total_b) == cudaSuccess) output[5] = total_b - free_b;
    output[6] = output[5];
    output[7] = s->calls;
    output[8] = s->completed;
    output[9] = s->graph_ns;
    output[10] = s->wait_ns;
    output[11] = s->export_ns;
    output[12] = s->wall_ns;
    output[13] = s->groups;
    output[16] = kernel_launches();
    for (int i = 0; i < 19; ++i) {
      output[17 + i * 3] = s->stage_calls[i];
      output[19 + i * 3] = uint64_t(s->stage_ms[i] * 1e6);
    }
  });
}

int rs_qwen_device_drain(void* session, uint64_t* invalidated, char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!invalidated) throw std::invalid_argument("drain descriptor");
    *invalidated = s->table->residents();
    s->set_device();
    QWEN_CUDA(cudaStreamSynchronize(s->stream));
    s->table->clear();
    const size_t np = s->page_ref.size();
    s->free_pages.resize(np);
    for (size_t i = 0; i < np; ++i) s->free_pages[i] = int32_t(np - 1 - i);
    std::fill(s->page_ref.begin(), s->page_ref.end(), 0);
    std::fill(s->page_filled.begin(), s->page_filled.end(), 0);
    if (s->table->residents() || s->table->bytes()) throw std::runtime_error("device drain residual");
    if (s->mtp_on) {  // draft versions too (native/qwen_device.inc:65 drains both tables)
      *invalidated += s->drafts->residents();
      s->drafts->clear();
      const size_t mp = s->mref.size();
      s->mfree.resize(mp);
      for (size_t i = 0; i < mp; ++i) s->mfree[i] = int32_t(mp - 1 - i);
      std::fill(s->mref.begin(), s->mref.end(), 0);
      std::fill(s->mfilled.begin(), s->mfilled.end(), 0);
    }
  });
}

int rs_qwen_device_set_capture(void* session, int routing, char* error, size_t capacity) {
  return checked(error, capacity, [&] { S(session)->capture_routing = routing != 0; });
}

int rs_qwen_device_debug_routing(void* session, int32_t* out, size_t count, char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!s->capture_routing || !out) throw std::invalid_argument("routing capture disabled");
    const int T = s->captured_tokens, K = s->d.top, A = T * (K + 1);
    if (count != size_t(s->d.L) * T * K) throw std::invalid_argument("routing capture capacity");
    s->set_device();
    QWEN_CUDA(cudaStreamSynchronize(s->stream));
    std::vector<int32_t> all(size_t(s->d.L) * A);
    QWEN_CUDA(cudaMemcpy(all.data(), s->capture.p, all.size() * 4, cudaMemcpyDeviceToHost));
    for (int l = 0; l < s->d.L; ++l)
      for (int t = 0; t < T; ++t)
        for (int j = 0; j < K; ++j) out[(size_t(l) * T + t) * K + j] = all[size_t(l) * A + t * (K + 1) + j];
  });
}

int rs_qwen_device_debug_capture(void* session, int what, void* out, size_t count, size_t* written, char* error,
                                 size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!s->capture_routing || !out || !written) throw std::invalid_argument("capture disabled or no output");
    s->set_device();
    QWEN_CUDA(cudaStreamSynchronize(s->stream));
    const int T = s->captured_tokens, A = T * (s->d.top + 1), L = s->d.L, E = s->d.E;
    auto copy = [&](const void* src, size_t bytes) {
      if (bytes > count) throw std::invalid_argument("capture capacity");
      QWEN_CUDA(cudaMemcpy(out, src, bytes, cudaMemcpyDeviceToHost));
      *written = bytes;
    };
    if (what == 0) return copy(s->cap_logits.p, size_t(L) * T * (E + 1) * 4);
    if (what == 1) return copy(s->cap_offsets.p, size_t(L) * (E + 2) * 4);
    if (what == 2) return copy(s->cap_perm.p, size_t(L) * A * 4);
    if (what == 3) {
      const int n = s->last_n, TT = s->last_T, R = s->last_R, nn = int(s->last_new_pages.size());
      std::vector<int32_t> blob;
      blob.insert(blob.end(), {n, TT, R, nn});
      for (const auto& sd : s->last_descs) {
        const int32_t* f = reinterpret_cast<const int32_t*>(&sd);
        blob.insert(blob.end(), f, f + sizeof(SeqDesc) / 4);
      }
      blob.insert(blob.end(), s->last_new_pages.begin(), s->last_new_pages.end());
      std::vector<int32_t> tmp(std::max(n + 1, TT));
      auto pull = [&](const int32_t* src, int cnt) {
        QWEN_CUDA(cudaMemcpy(tmp.data(), src, size_t(cnt) * 4, cudaMemcpyDeviceToHost));
        blob.insert(blob.end(), tmp.begin(), tmp.begin() + cnt);
      };
      pull(s->cu_seqlens.p, n + 1);
      pull(s->token_seq.p, TT);
      pull(s->token_pos.p, TT);
      std::vector<int64_t> sm(TT);
      QWEN_CUDA(cudaMemcpy(sm.data(), s->slot_mapping.p, size_t(TT) * 8, cudaMemcpyDeviceToHost));
      for (auto v : sm) blob.push_back(int32_t(v));
      pull(s->out_token.p, R);
      if (blob.size() * 4 > count) throw std::invalid_argument("capture capacity");
      std::memcpy(out, blob.data(), blob.size() * 4);
      *written = blob.size() * 4;
      return;
    }
    if (what == 4) {
      int maxp = 0;
      for (const auto& sd : s->last_descs) maxp = std::max(maxp, sd.n_shared + sd.n_new);
      std::vector<int32_t> rows(size_t(s->last_n) * maxp, -1);
      for (int i = 0; i < s->last_n; ++i) {
        const auto& sd = s->last_descs[i];
        const int np = sd.n_shared + sd.n_new;
        if (np)
          QWEN_CUDA(cudaMemcpy(rows.data() + size_t(i) * maxp, s->block_table.p + size_t(sd.child) * s->bt_stride,
                               size_t(np) * 4, cudaMemcpyDeviceToHost));
      }
      if (rows.size() * 4 > count) throw std::invalid_argument("capture capacity");
      std::memcpy(out, rows.data(), rows.size() * 4);
      *written = rows.size() * 4;
      return;
    }
    throw std::invalid_argument("unknown capture selector");
  });
}

int rs_qwen_device_mtp_attach(void* session, void* weights, char* error, size_t capacity) {
  return checked(error, capacity, [&] { S(session)->mtp_attach(static_cast<WeightStore*>(weights)); });
}
int rs_qwen_device_mtp_step(void* session, const StateId* previous, const StateId* source, int draft_source,
                            size_t row, const uint32_t* tokens, size_t count, StateId* output, float* logits,
                            size_t logits_count, int diagnostics, char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (diagnostics < 0 || diagnostics > 1) throw std::invalid_argument("MTP descriptor");
    if (diagnostics) throw std::invalid_argument("MTP diagnostics are an MLX-baseline feature not offered here");
    if (logits_count != size_t(s->d.V)) throw std::invalid_argument("MTP unavailable or vocabulary capacity");
    s->mtp_step(previous, source, draft_source, row, tokens, count, output, logits);
  });
}
int rs_qwen_device_mtp_release(void* session, const StateId* id, char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    if (!id) throw std::invalid_argument("MTP release descriptor");
    S(session)->mtp_release(*id);
  });
}
int rs_qwen_device_mtp_snapshot(void* session, const StateId* id, float* output, size_t count, char* error,
                                size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!id || !output) throw std::invalid_argument("MTP snapshot capacity");
    if (!s->mtp_on) throw std::invalid_argument("MTP unavailable");
    s->set_device();
    const Dims& d = s->d;
    const auto& v = s->drafts->get(*id);
    const size_t per = size_t(d.Hkv) * d.ctx * d.D;
    if (count != 2 * per + size_t(v.hidden_rows) * d.H) throw std::invalid_argument("MTP snapshot capacity");
    std::fill(output, output + 2 * per, 0.f);
    std::vector<__nv_bfloat16> page(size_t(2) * d.Hkv * kPageTokens * d.D);
    for (size_t pi = 0; pi < v.pages.size(); ++pi) {
      QWEN_CUDA(cudaMemcpy(page.data(), s->mkv.page(0, v.pages[pi]), page.size() * 2, cudaMemcpyDeviceToHost));
      for (int kvsel = 0; kvsel < 2; ++kvsel)
        for (int g = 0; g < d.Hkv; ++g)
          for (int o = 0; o < kPageTokens; ++o) {
            const size_t p = pi * kPageTokens + o;
            if (p >= id->position) continue;
            const __nv_bfloat16* src = page.data() + ((size_t(kvsel) * d.Hkv + g) * kPageTokens + o) * d.D;
            float* dst = output + kvsel * per + (size_t(g) * d.ctx + p) * d.D;
            for (int i = 0; i < d.D; ++i) dst[i] = __bfloat162float(src[i]);
          }
    }
    QWEN_CUDA(cudaMemcpy(output + 2 * per, s->mhidden.p + size_t(id->slot) * kMaxDraft * d.H,
                         size_t(v.hidden_rows) * d.H * 4, cudaMemcpyDeviceToHost));
    s->exports += count * 4;
  });
}
int rs_qwen_device_mtp_verify_accept(void* session, size_t n_seq, const StateId* parents, const uint32_t* seeds,
                                     const uint32_t* drafts, const uint32_t* ndraft, size_t width,
                                     const uint32_t* eos, size_t n_eos, uint32_t flags, StateId* outs,
                                     uint32_t* accepted, uint32_t* emitted, uint32_t* n_emitted, char* error,
                                     size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!n_seq || !parents || !seeds || !ndraft || !outs || !accepted || !emitted || !n_emitted ||
        (width && !drafts) || (n_eos && !eos))
      throw std::invalid_argument("verify descriptor");
    if (width > size_t(kMaxDraft)) throw std::invalid_argument("draft width above 8");
    if (flags & ~RS_QWEN_RAGGED_HIDDEN) throw std::invalid_argument("verify flags: only RS_QWEN_RAGGED_HIDDEN");
    std::vector<uint32_t> fed;
    std::vector<size_t> off(n_seq);
    for (size_t i = 0; i < n_seq; ++i) {
      if (ndraft[i] > width) throw std::invalid_argument("draft count above the width");
      off[i] = fed.size();
      fed.push_back(seeds[i]);
      for (uint32_t j = 0; j < ndraft[i]; ++j) fed.push_back(drafts[i * width + j]);
    }
    std::vector<Session::SeqIn> seqs(n_seq);
    for (size_t i = 0; i < n_seq; ++i)
      seqs[i] = {&parents[i], uint32_t(parents[i].position), 1 + ndraft[i], fed.data() + off[i]};
    Session::VerifyIn vin{eos, n_eos, accepted, emitted, width + 1, n_emitted};
    s->step(seqs, flags, outs, nullptr, nullptr, &vin);
  });
}

int rs_qwen_debug_gemm(void* session, int which, int layer, const uint16_t* x, size_t T, float* y, size_t y_count,
                       int engine, double* ms, char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!x || !y || !T || T > size_t(s->max_tokens)) throw std::invalid_argument("debug gemm descriptor");
    if (layer < 0 || layer >= s->d.L) throw std::invalid_argument("debug gemm layer");
    const LayerDev& ly = s->store->model.layers[layer];
    const QMat& W = which == 0 ? ly.in_proj : which == 1 ? ly.out_proj : which == 2 ? ly.router : s->store->model.lm_head;
    if (which < 0 || which > 3) throw std::invalid_argument("debug gemm matrix");
    if (y_count != T * size_t(W.rows)) throw std::invalid_argument("debug gemm output capacity");
    s->set_device();
    gemm_in_t* xin = which == 1 ? s->hb2.p : which == 3 ? s->hb_out.p : s->hb.p;
    if (which == 3 && T > size_t(s->max_rows)) throw std::invalid_argument("debug gemm rows");
    QWEN_CUDA(cudaMemcpyAsync(xin, x, T * W.k * 2, cudaMemcpyHostToDevice, s->stream));
    QWEN_CUDA(cudaMemsetAsync(s->err.p, 0, 4, s->stream));
    const bool prev = s->simple_gemm;
    s->simple_gemm = engine == 1;
    const size_t stride = T * size_t(W.rows);
    float* out = which == 3 ? s->logits.p : s->partial.p;
    if (which == 3) s->logits.ensure(stride);
    out = which == 3 ? s->logits.p : s->partial.p;
    QWEN_CUDA(cudaEventRecord(s->ev_begin, s->stream));
    int splits = 1;
    try {
      splits = s->dense(W, xin, which == 3 ? s->max_rows : s->max_tokens, int(T), out, W.rows, stride,
                        which == 3 ? 1 : kMaxSplits, s->stream);
    } catch (...) {
      s->simple_gemm = prev;
      throw;
    }
    s->simple_gemm = prev;
    QWEN_CUDA(cudaEventRecord(s->ev_end, s->stream));
    std::vector<float> part(stride * splits);
    uint32_t h_err = 0;
    QWEN_CUDA(cudaMemcpyAsync(part.data(), out, part.size() * 4, cudaMemcpyDeviceToHost, s->stream));
    QWEN_CUDA(cudaMemcpyAsync(&h_err, s->err.p, 4, cudaMemcpyDeviceToHost, s->stream));
    QWEN_CUDA(cudaStreamSynchronize(s->stream));
    float fms = 0.f;
    QWEN_CUDA(cudaEventElapsedTime(&fms, s->ev_begin, s->ev_end));
    if (ms) *ms = fms;
    if (h_err) throw std::runtime_error("debug gemm device error flag " + std::to_string(h_err));
    for (size_t i = 0; i < stride; ++i) {
      float v = 0.f;
      for (int sp = 0; sp < splits; ++sp) v += part[sp * stride + i];
      y[i] = v;
    }
  });
}

int rs_qwen_project_noalloc(void* session, int which, int layer, const void* x_device, size_t T, float* y_device,
                            size_t y_count, void* stream, char* error, size_t capacity) {
  if (!session) {
    report(error, capacity, "no-alloc projection: null session");
    return -1;
  }
  Session* s = static_cast<Session*>(session);
  if (which < 0 || which > 3 || layer < 0 || layer >= s->d.L) {
    report(error, capacity, "no-alloc projection: matrix selector or layer out of range");
    return -1;
  }
  const LayerDev& ly = s->store->model.layers[layer];
  const QMat& W = which == 0 ? ly.in_proj : which == 1 ? ly.out_proj : which == 2 ? ly.router : s->store->model.lm_head;
  if (T == 0 || T > size_t(INT32_MAX) / size_t(W.rows) || y_count != T * size_t(W.rows)) {
    report(error, capacity, "no-alloc projection: output capacity must be T x rows of the selected matrix");
    return -1;
  }
  // run on the session's device and give the caller back its own current device
  int caller_device = -1;
  cudaError_t rc = cudaGetDevice(&caller_device);
  if (rc == cudaSuccess) rc = cudaSetDevice(s->device);
  if (rc != cudaSuccess) {
    report(error, capacity, cudaGetErrorString(rc));
    return -1;
  }
  const int status = project_noalloc(W, which == 3 ? 1 : kMaxSplits, static_cast<const gemm_in_t*>(x_device),
                                     int(T), y_device, s->sm_count,
                                     stream ? static_cast<cudaStream_t>(stream) : s->stream, error, capacity);
  if (caller_device != s->device) {
    rc = cudaSetDevice(caller_device);
    if (rc != cudaSuccess && status == 0) {
      report(error, capacity, cudaGetErrorString(rc));
      return -1;
    }
  }
  return status;
}

int rs_qwen_ep_unique_id(uint8_t* out, size_t out_bytes, char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    if (!out || out_bytes != sizeof(ncclUniqueId)) throw std::invalid_argument("expert-parallel id capacity");
    ncclUniqueId id;
    const ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) throw std::runtime_error(std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
    std::memcpy(out, &id, sizeof(id));
  });
}

int rs_qwen_device_ep_init(void* session, int world, int rank, const uint8_t* id, size_t id_bytes, size_t cap_tokens,
                           char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    if (!id || id_bytes != sizeof(ncclUniqueId) || cap_tokens > size_t(1) << 30)
      throw std::invalid_argument("expert-parallel init arguments");
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    S(session)->ep_init(world, rank, uid, int(cap_tokens));
  });
}

int rs_qwen_device_ep_window(void* session, int world, int rank, size_t cap_tokens, uint8_t* handle,
                             size_t handle_bytes, char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    if (!handle || handle_bytes != sizeof(cudaIpcMemHandle_t) || cap_tokens > size_t(1) << 30)
      throw std::invalid_argument("expert-parallel window arguments");
    cudaIpcMemHandle_t h;
    S(session)->ep_window(world, rank, int(cap_tokens), &h);
    std::memcpy(handle, &h, sizeof(h));
  });
}

int rs_qwen_device_ep_connect(void* session, const uint8_t* handles, size_t handles_bytes, char* error,
                              size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!handles || handles_bytes != size_t(s->ep.world) * sizeof(cudaIpcMemHandle_t))
      throw std::invalid_argument("expert-parallel handles");
    std::vector<cudaIpcMemHandle_t> hs(s->ep.world);
    std::memcpy(hs.data(), handles, handles_bytes);
    s->ep_connect(hs.data());
  });
}

int rs_qwen_device_set_profile(void* session, int profile, char* error, size_t capacity) {
  return checked(error, capacity, [&] { S(session)->profile = profile != 0; });
}

int rs_qwen_device_timing(void* session, double* out, size_t count, char* error, size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!out || count != 3 + 19) throw std::invalid_argument("timing capacity");
    out[0] = s->last_ms;
    out[1] = s->total_ms;
    out[2] = double(s->timed_steps);
    for (int i = 0; i < 19; ++i) out[3 + i] = s->stage_ms[i];
  });
}

int rs_qwen_device_synthetic_state(void* session, size_t position, uint64_t seed, StateId* out, char* error,
                                   size_t capacity) {
  return checked(error, capacity, [&] {
    Session* s = S(session);
    if (!out || !position || position > size_t(s->d.ctx)) throw std::invalid_argument("synthetic state geometry");
    s->set_device();
    const int n_pages = s->d.n_attn > 0 ? int((position + kPageTokens - 1) / kPageTokens) : 0;
    if (n_pages > int(s->free_pages.size())) throw std::runtime_error("KV page pool exhausted");
    if (s->table->residents() + 1 > s->slots) throw std::runtime_error("combined resident budget exhausted");
    StateId id = s->table->reserve(position, s->version_bytes(n_pages, 0));
    Version v;
    for (int j = 0; j < n_pages; ++j) {
      const int32_t p = s->free_pages.back();
      s->free_pages.pop_back();
      s->page_ref[p] = 1;
      s->page_filled[p] = uint8_t(std::min<size_t>(kPageTokens, position - size_t(j) * kPageTokens));
      v.pages.push_back(p);
    }
    try {
      s->new_pages.ensure(std::max(1, n_pages));
      if (n_pages) {
        QWEN_CUDA(cudaMemcpyAsync(s->block_table.p + id.slot * size_t(s->bt_stride), v.pages.data(),
                                  size_t(n_pages) * 4, cudaMemcpyHostToDevice, s->stream));
        QWEN_CUDA(cudaMemcpyAsync(s->new_pages.p, v.pages.data(), size_t(n_pages) * 4, cudaMemcpyHostToDevice,
                                  s->stream));
      }
      launch_synth_state(s->kv, s->new_pages.p, n_pages, int(position), s->d.ctx, s->gdn, int(id.slot), s->d,
                         seed, s->stream);
      QWEN_CUDA(cudaGetLastError());
      QWEN_CUDA(cudaStreamSynchronize(s->stream));
    } catch (...) {
      s->unref_pages(v.pages);
      s->table->rollback(id);
      throw;
    }
    s->table->publish(id, std::move(v));
    *out = id;
  });
}

}  // extern "C"
