// Launch interface of the decode-step kernels (all sm_100a).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "model.h"

namespace qwen {

// Per-sequence packing descriptor, uploaded once per step (host -> device).
struct SeqDesc {
  int32_t position;   // first new position
  int32_t count;      // new tokens
  int32_t parent;     // parent state slot (= block-table row), -1 = empty prefix
  int32_t child;      // child state slot
  int32_t n_shared;   // parent pages kept in the child's block table
  int32_t new_off;    // offset of this sequence's new pages in the page list
  int32_t n_new;      // freshly allocated pages
  int32_t out_row0;   // first output row (logits / sampled)
  int32_t n_out;      // output rows (1 = last token, count = every token)
  int32_t cow_src;    // page copied into the first new page (copy-on-write), -1 none
  int32_t cow_len;    // tokens copied by the copy-on-write
  int32_t hidden;     // keep post-norm hidden rows in the child slot
  int32_t cand;       // verify steps: offset of this sequence's per-token state slots in the
                      // candidate list (slot of the state after token j = cand_slots[cand + j]), -1 none
};

// Device-built packing results.
struct Packed {
  int32_t* cu_seqlens;    // [n+1]
  int32_t* token_seq;     // [T]
  int32_t* token_pos;     // [T]
  int64_t* slot_mapping;  // [T] page*16 + pos%16
  int32_t* out_token;     // [R] token index of each output row
};

struct KvPool {
  __nv_bfloat16* base = nullptr;  // [layers][pages][2][Hkv][16][D]
  int n_pages = 0, layers = 0, Hkv = 0, D = 0;
  __host__ __device__ size_t page_elems() const { return size_t(2) * Hkv * kPageTokens * D; }
  __host__ __device__ __nv_bfloat16* page(int layer, int p) const {
    return base + (size_t(layer) * n_pages + p) * page_elems();
  }
};

struct GdnPool {
  float* state = nullptr;  // [slots][n_gdn][hv][dv][dk]
  float* conv = nullptr;   // [slots][n_gdn][conv-1][cd]
  int slots = 0, n_gdn = 0;
  size_t state_elems = 0;  // per layer per slot
  size_t conv_elems = 0;
};

// GEMM descriptor for the 4-bit affine g64 grouped GEMM.
enum GemmMode : int {
  kGemmStoreF32 = 0,  // Y[t][n] = acc (split s writes Y + s*split_stride)
  kGemmGateUp = 1,    // grouped experts: act[p][j] = silu(gate)*up as fp16
  kGemmDown = 2,      // grouped experts: Y[p][n] = acc (fp32)
};

struct GemmArgs {
  QMat W;
  int mode = kGemmStoreF32;
  int expert_tiles = 0;  // row tiles per expert (grouped modes)
  const gemm_in_t* X = nullptr;
  int ldx = 0;
  const int32_t* x_row = nullptr;  // grouped: X row of sorted position p = x_row[p] / x_div
  int x_div = 1;
  const int32_t* group_off = nullptr;  // grouped: positions of expert g = [off[g], off[g+1])
  int groups = 1;
  int n_tokens = 0;  // dense: number of token rows
  int splits = 1;    // dense split-K
  size_t split_stride = 0;
  float* Y = nullptr;
  int ldy = 0;
  gemm_in_t* Yb = nullptr;
  int ldyb = 0;
};

uint64_t kernel_launches();

void launch_pack(const SeqDesc* descs, int n_seq, const int32_t* new_pages, int32_t* block_table,
                 int bt_stride, Packed p, cudaStream_t s);
void launch_cow(KvPool kv, const SeqDesc* descs, int n_seq, const int32_t* new_pages,
                cudaStream_t s);
void launch_embed_norm(const QMat& embed, const uint32_t* tokens, int T, const float* norm_w,
                       float eps, float* x, gemm_in_t* hb, cudaStream_t s);
void launch_residual_norm(float* x, const float* partial, int splits, size_t split_stride, int T,
                          int H, const float* norm_w, float eps, gemm_in_t* hb,
                          const int32_t* out_token, int rows, float* hidden_f32,
                          cudaStream_t s);
void launch_qgemm(const GemmArgs& a, cudaStream_t s);
// Long token runs of the DeltaNet layers (prefill chunks), gdn_chunk.cu: the
// sequences of a step that feed at least kGdnChunkMin tokens (and are not
// verify steps) run the chunked form; gdn_update skips them.
constexpr int kGdnChunk = 64;      // tokens per chunk
constexpr int kGdnChunkMin = 64;   // tokens a sequence feeds before it takes the chunked path
struct GdnChunkPlan {
  int n_long = 0, n_items = 0, n_tokens = 0;
  const int32_t* longs = nullptr;   // [n_long][3]: sequence, first chunk item, chunks
  const int32_t* items = nullptr;   // [n_items][2]: sequence, chunk index
  const int32_t* tokens = nullptr;  // [n_tokens]: packed indices of those sequences' tokens
  float* U = nullptr;               // [item][hv][chunk][dv]
  float* W = nullptr;               // [item][hv][chunk][dk]
  float* A = nullptr;               // [item][hv][chunk][chunk]
  float* LG = nullptr;              // [item][hv][chunk] log-decay prefix sums
};
// conv + SiLU, q / k scaling, decay and beta of the long runs, chunk-parallel,
// then the children's conv histories
void launch_gdn_run_prep(const GdnChunkPlan& cp, const Dims& d, const LayerDev& ly, const float* proj, int ld_proj,
                         int splits, size_t split_stride, const SeqDesc* descs, const int32_t* cu_seqlens,
                         GdnPool pool, int li, float* qk_buf, float* v_buf, float* gb_buf, cudaStream_t s);
void launch_gdn_chunked(const GdnChunkPlan& cp, const Dims& d, const LayerDev& ly, const float* proj, int ld_proj,
                        int splits, size_t split_stride, const SeqDesc* descs, const int32_t* cu_seqlens,
                        GdnPool pool, int li, gemm_in_t* out, uint32_t* err, const float* qk_buf, float* v_buf,
                        const float* gb_buf, cudaStream_t s);
void launch_gdn(const Dims& d, const LayerDev& ly, const float* proj, int ld_proj, int splits,
                size_t split_stride, const SeqDesc* descs, const int32_t* cu_seqlens, int n_seq, int T, GdnPool pool,
                int gdn_index, gemm_in_t* out, uint32_t* err, float* qk_buf, float* v_buf, float* gb_buf,
                int sm_count, const int32_t* cand_slots, cudaStream_t s, const GdnChunkPlan* chunked = nullptr);
void launch_attn_prep(const Dims& d, const LayerDev& ly, const float* proj, int ld_proj, int splits,
                      size_t split_stride, const int32_t* token_pos, const int64_t* slot_mapping, int T, KvPool kv,
                      int kv_layer, float* q, float* gate, cudaStream_t s);
void launch_route(const float* logits, int ld, int splits, size_t split_stride, int T, int E, int top,
                  int32_t* ids, float* weights, float* logits_out, cudaStream_t s);
// Stable sort of the assignments (n_assign = tokens * slots, each token's
// slots distinct experts) by expert: token bit masks when they fit in shared
// memory, else per-round counting.
void launch_expert_sort(const int32_t* ids, int n_assign, int slots, int n_experts, int32_t* counts,
                        int32_t* offsets, int32_t* perm, int32_t* inv, uint32_t* err, cudaStream_t s);
// The same sort fused with the gather of the MoE input rows:
// dst[sorted position] = src[token] (H fp16 columns, row stride ld).
void launch_expert_sort_gather(const int32_t* ids, int n_assign, int slots, int n_experts, int32_t* counts,
                               int32_t* offsets, int32_t* perm, int32_t* inv, uint32_t* err, const gemm_in_t* src,
                               int ld, int H, gemm_in_t* dst, int sm_count, cudaStream_t s);
void launch_moe_combine(float* x, const float* y_sorted, const int32_t* inv,
                        const float* weights, int T, int H, int slots, const float* norm_w,
                        float eps, gemm_in_t* hb, const int32_t* out_token, int rows,
                        float* hidden_f32, cudaStream_t s);
void launch_mtp_input(const QMat& embed, const uint32_t* tokens, int T, const float* hidden, const float* w_e,
                      const float* w_h, float eps, gemm_in_t* cat, cudaStream_t s);
void launch_accept(const SeqDesc* descs, int n, const int32_t* cu_seqlens, const uint32_t* tokens,
                   const uint32_t* sampled, const uint32_t* eos, int n_eos, int ctx, int32_t* acc, uint32_t* emitted,
                   int emit_stride, uint32_t* n_emitted, cudaStream_t s);
void launch_verify_compact(const SeqDesc* descs, int n, const int32_t* cand_slots, const int32_t* acc,
                           int32_t* block_table, int stride, const float* hidden_stage, const int32_t* cu_seqlens,
                           float* hidden_pool, int chunk, int H, cudaStream_t s);
// Y[t][n] = X[t] . W[n] for a matrix stored as dense fp16 rows (QMat::dense_f16).
void launch_dense_f16(const QMat& W, const gemm_in_t* X, int T, float* Y, int ldy, cudaStream_t s);
void launch_argmax(const float* logits, int rows, int V, uint32_t* tokens, uint32_t* err, uint64_t* part,
                   uint32_t* done, cudaStream_t s);
// Constrained greedy selection for the listed output rows (choices.rs:65-98);
// runs after launch_argmax on the same logits.
void launch_choice_select(const float* logits, int V, const int32_t* rows, const uint32_t* offsets,
                          const uint32_t* ids, int n_rows, uint32_t* tokens, cudaStream_t s);
void launch_synth_state(KvPool kv, const int32_t* pages, int n_pages, int position, int ctx,
                        GdnPool pool, int slot, const Dims& d, uint64_t seed, cudaStream_t s);
// Expert parallelism (ep.cu): stage packing, local row plan / gather, result
// return. Per-peer destination tables; flag tables / wait flags non-null for
// the direct NVLink transport (null with NCCL).
void launch_ep_pack(const gemm_in_t* src, int ld, const int32_t* perm, int div, const int32_t* counts,
                    const int32_t* offsets, uint8_t* const* dst,
                    int world, int per_rank, int hdr_ints, int cap, int H, uint32_t* const* flag_dst, uint32_t epoch,
                    uint32_t* done, cudaStream_t s);
void launch_ep_plan_gather(const uint8_t* const* srcs, int world, int rank, int per_rank, int hdr_ints, int E,
                           const int32_t* counts, const int32_t* offsets, const gemm_in_t* xsrc, int ld,
                           const int32_t* perm, int div, int32_t* goff,
                           int32_t* seg, int32_t* n_rows, gemm_in_t* xloc, int32_t* origin, int cap, int H,
                           int max_rows, uint32_t* err, const uint32_t* wait_flags, uint32_t epoch, int sm_count,
                           cudaStream_t s);
void launch_ep_return(const float* yloc, const int32_t* origin, const int32_t* n_rows, float* const* rdst,
                      float* y_sorted, int cap, int H, int world, int max_rows, uint32_t* const* flag_dst,
                      uint32_t epoch, uint32_t* done, int sm_count, cudaStream_t s);
void launch_ep_return_unpack(const float* const* rsrcs, const int32_t* offsets, float* y_sorted, int world,
                             int per_rank, int H, int max_rows, const uint32_t* wait_flags, uint32_t epoch,
                             uint32_t* err, int sm_count, cudaStream_t s);
void launch_gather_rows(const gemm_in_t* src, int ld, const int32_t* perm, int div, int n, int H,
                        gemm_in_t* dst, cudaStream_t s);

}  // namespace qwen
