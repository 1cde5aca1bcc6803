// tcgen05 4-bit grouped GEMM: launch interface.
#pragma once
#include <cuda.h>

#include "kernels.h"

namespace qwen {

struct TcArgs {
  QMat W;
  int mode = kGemmStoreF32;  // kGemmStoreF32 / kGemmGateUp / kGemmDown
  int expert_tiles = 0;      // grouped: row tiles per expert
  int groups = 1;
  const int32_t* group_off = nullptr;  // grouped: sorted positions of expert g = [off[g], off[g+1])
  int n_tokens = 0;                    // dense: token rows
  int splits = 1;                      // dense: split-K slices (partials at Y + split*split_stride)
  size_t split_stride = 0;
  int token_group = 0;                 // dense: tokens per work item (0 = all; many-token steps
                                       // split the tokens instead of K)
  int b_row0 = 0;      // first activation row of the B tensor map
  int box_rows = 16;   // N tile: 16, 32, 64 or 128 (the tensor map's box height)
  int stages = 0;      // TMEM A stages in chunks (set by the launcher)
  int b_stages = 0;    // activation ring depth in chunks (set by the launcher)
  int unit = 1;        // chunks per MMA unit (set by the launcher)
  float* Y = nullptr;
  int ldy = 0;
  gemm_in_t* Yb = nullptr;  // kGemmGateUp output (the down GEMM input)
  int ldyb = 0;
  uint32_t* err = nullptr;
};

// Tensor map over a row-major fp16 activation matrix [rows, k] with a
// (64 columns x box_rows) box and 128-byte swizzle (the UMMA K-major layout).
CUtensorMap make_act_map(const void* base, int rows, int k, int box_rows);
// The same matrix viewed as [k/64 chunks][rows][64]: one box brings `unit`
// consecutive 64-column tiles (the B operand of one MMA unit).
CUtensorMap make_act_map3d(const void* base, int rows, int k, int box_rows, int unit);
// Chunks per MMA unit the launcher will use for these arguments (4, 2 or 1).
int qgemm_tc_unit(const TcArgs& a);
// Largest split-K count worth trying for a dense launch of at most 128 tokens
// over `row_tiles` row tiles and `kc` 64-column chunks (callers then take the
// largest count <= this that divides kc into whole 4-chunk units).
int qgemm_tc_split_target(int row_tiles, int kc, int sm_count, int max_splits);
// Tensor map over one attention layer's KV page pool: rows
// ((page*2 + k_or_v)*Hkv + head)*16 + token, D columns, 16x64 128B-swizzled box.
CUtensorMap make_kv_map(const KvPool& kv, int layer);
// items[i] = (index into dec_tokens, KV split); dec_tokens maps that index to
// the packed token (null: identity); the split partials are stored per index.
void launch_attn_decode(const CUtensorMap& kvmap, const Dims& d, const float* q, const int32_t* token_seq,
                        const int32_t* token_pos, const int32_t* dec_tokens, const SeqDesc* descs, const int32_t* block_table, int bt_stride,
                        const int2* items, int n_items, int split_pages, float* ws, int max_splits, uint32_t* err,
                        cudaStream_t s);
// Merges the split partials of `T` split-decoded tokens (partials stored per
// index; `tokens` maps an index to the packed token, null: identity) and
// applies the output gate.
void launch_attention_merge(const Dims& d, const float* ws, const float* gate, const int32_t* token_pos,
                            const int32_t* tokens, int T, int split_pages, int max_splits, gemm_in_t* out,
                            cudaStream_t s);
// Chunked-prefill attention (attention.cu): blocks[i] = (first packed token,
// tokens, sequence, pages) of kAttnPrefillWarps * 16 / G consecutive tokens of
// one sequence; writes the gated fp16 o_proj input of those tokens.
constexpr int kAttnPrefillWarps = 8;
constexpr int kAttnPrefillMin = 16;  // tokens a sequence feeds before its attention takes the prefill kernel
void launch_attn_prefill(const CUtensorMap& kvmap, const Dims& d, const float* q, const int32_t* token_pos,
                         const SeqDesc* descs, const int32_t* block_table, int bt_stride, const int4* blocks,
                         int n_blocks, const float* gate, gemm_in_t* out, uint32_t* err, cudaStream_t s);
void launch_qgemm_tc(const CUtensorMap& bmap, TcArgs a, int sm_count, cudaStream_t s);
size_t qgemm_tc_smem(int box_rows, int stages, int unit);
int qgemm_tc_stages(int box_rows);
int qgemm_tc_bstages(int box_rows);

}  // namespace qwen
