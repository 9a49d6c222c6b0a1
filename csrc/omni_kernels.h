// Host-side launchers of the sm_100a kernels.  The .cu files implement them
// against raw device pointers (no torch headers, so they compile fast); the
// torch bindings in bindings.cpp validate tensors and forward here.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace omni {

// ---------------------------------------------------------------- GEMM (tcgen05)
// out[r, m] = act( sum_k B[r, k] * A[g * a_rows + m, k] ) (+ bias[g, m]) (+ residual[r, m])
// for every row r of group g (rows offsets[g] .. offsets[g+1]) and m < m_out.
// A holds the weights ([groups * a_rows, k] bf16, K contiguous); B holds the
// activations ([rows, k] bf16).  With gated=1 a_rows = 2 * m_out: the first
// m_out rows of each group are the gate projection, the next m_out the up
// projection, and the epilogue emits silu(gate) * up.
enum GemmAct : int { kActNone = 0, kActGeluTanh = 1, kActGeluErf = 2, kActSilu = 3 };

struct GemmArgs {
  const void* a;          // weights, bf16
  const void* b;          // activations, bf16
  void* out;              // bf16 or fp32
  int64_t ldo;            // out row stride in elements
  int out_f32;
  const void* bias;       // bf16 [groups, m_out] or nullptr
  const void* residual;   // bf16, row stride ldr, or nullptr
  int64_t ldr;
  int m_out;
  int a_rows;             // weight rows per group
  int k;
  int groups;
  const int* offsets;     // device int32 [groups + 1], or nullptr for one dense group
  int rows;               // total rows of B (for the tensor map and dense mode)
  int expected_rows_per_group;  // host hint used to pick the token tile
  int gated;
  int act;
  int* status;            // device int32 status word (may be nullptr)
  int max_ctas;           // 0 = one CTA per SM
  // Optional split-K scratch for dense, non-gated GEMMs with few output tiles:
  // one fp32 plane [tiles][128][token tile] that the splits add into and the
  // last split of each tile (per-tile arrival counters) reads back, re-zeroes
  // and finalises.  Calls that share it must not overlap on the GPU.
  float* splitk_ws;
  long long splitk_ws_floats;
  int* splitk_counters;
  int splitk_counter_slots;
  // Split-K over a thread-block cluster instead (one cluster of splits per output tile, the
  // partial tiles reduced through distributed shared memory): needs no scratch at all.
  int splitk_cluster;
  // Optional owner scatter (tensor parallel): bf16 output row r is stored at
  // peer_out[r / rows_per] + r * ldo, i.e. straight into the memory of the
  // rank that owns token r (over NVLink for the other ranks).
  const unsigned long long* peer_out;   // device [world]
  int rows_per;
  // Optional wait before the first TMA load: flags[i] == *wait_seq for i < wait_count
  // (the all-gather of this GEMM's activations has landed).  Bounded by wait_timeout_ns.
  const unsigned int* wait_flags;
  const unsigned int* wait_seq;
  int wait_count;
  long long wait_timeout_ns;
  // The weights (A) are not written by any kernel still in flight on the stream (model
  // parameters): with programmatic dependent launch the GEMM may fetch its first weight
  // tiles before the previous kernel has finished.
  int static_a;
  // ---- expert-parallel fused modes (the grouped GEMMs of an EP MoE layer, csrc/ep_moe.cu)
  // Segment layout instead of offsets: group g's rows are B rows [g * seg_cap, g * seg_cap +
  // min(seg_counts[g], seg_cap)) and the output rows with the same indices.  CTA 0 copies the
  // counts it used into seg_counts_copy (when set) for a later kernel of the layer.
  int seg_cap;
  const int* seg_counts;
  int* seg_counts_copy;
  // wait_flags are awaited before the group counts are read (they are final only then), not
  // just before the first operand load.
  int setup_wait;
  // Combine epilogue: bf16 output row r is stored at peer_rows[row_tag[2r]] + row_tag[2r + 1] * ldo,
  // i.e. into the slot of the routed row on its source rank; tags outside [0, tag_ranks) x
  // [0, tag_slots) drop the row.
  const int* row_tag;
  const unsigned long long* peer_rows;
  int tag_ranks, tag_slots;
  // Completion signal: when every CTA has stored its outputs, the last CTA to finish
  // release-stores *signal_seq into signal_flags[d] for d < signal_count (one address per
  // rank).  CTA 0 first clears zero_ptr[0 .. zero_n).  arrive_counter is zero between calls.
  const unsigned long long* signal_flags;
  const unsigned int* signal_seq;
  int signal_count;
  int* arrive_counter;
  int* zero_ptr;
  int zero_n;
};
cudaError_t gemm_bf16(const GemmArgs& args, cudaStream_t stream);

// ---------------------------------------------------------------- normalisation
// y = rmsnorm(x (+ residual)) * w ; when residual != nullptr the sum is also
// written back into residual (fused residual add).
cudaError_t rmsnorm_bf16(const void* x, const void* w, void* y, void* residual, int rows, int hidden,
                         int64_t ld_x, int64_t ld_y, float eps, cudaStream_t stream);
// Per-head RMSNorm over the last dim (head_dim) of a [rows, heads, head_dim] view.
cudaError_t layernorm_bf16(const void* x, const void* w, const void* b, void* y, int rows, int hidden, float eps,
                           cudaStream_t stream);


// ---------------------------------------------------------------- attention
// Paged KV cache of one layer: [pages, hkv, 64, head_dim] bf16 (page size 64).
struct AttnPrefillArgs {
  const void* q;          // [tokens, hq, D] rows of stride q_stride
  int64_t q_stride;
  const void* k;          // paged cache, or contiguous [kv_tokens, hkv, D] rows of stride kv_stride
  const void* v;
  int64_t kv_stride;
  const int* block_table; // [B, bt_stride] page ids, nullptr => contiguous K/V
  int bt_stride;
  const int* cu_q;        // [B + 1]
  const int* kv_lens;     // [B] keys visible to each request (including this chunk)
  const int* cu_kv;       // contiguous mode: [B + 1] first key row of each request
  const int* tile_req;    // [num_tiles] request of each 64-row query tile
  const int* tile_tok0;   // [num_tiles] first query token (within the request) of the tile
  int num_tiles;
  int hq, hkv, head_dim;
  float scale;
  int causal;
  void* out;              // [tokens, hq, D] rows of stride out_stride
  int64_t out_stride;
  int window;             // > 0: causal sliding window (a query sees its last `window` keys)
  int num_pages;          // paged mode: pages in the cache; block-table entries outside [0, num_pages)
                          // read page 0 (the reserved padding page). 0 = unchecked
  int tile_rows;          // packed query rows per tile: 64 (mma.sync kernel), 128 (tcgen05 kernel,
                          // csrc/attention_sm100.cu: paged, head_dim 128, no window) or 256 (its
                          // two-tile ping-pong variant)
  int q_rows;             // rows of q (tokens of the batch)
  int* status;            // bounded-wait status word (tcgen05 kernel), may be nullptr
  int kv_rows;            // contiguous mode: rows of k / v
};
cudaError_t attention_prefill(const AttnPrefillArgs& a, cudaStream_t stream);
bool attention_prefill_sm100_supported(const AttnPrefillArgs& a);
cudaError_t attention_prefill_sm100(const AttnPrefillArgs& a, cudaStream_t stream);

struct AttnDecodeArgs {
  const void* q;          // [B, hq, D] rows of stride q_stride
  int64_t q_stride;
  const void* k;
  const void* v;
  const int* block_table;
  int bt_stride;
  const int* kv_lens;
  int batch, hq, hkv, head_dim;
  float scale;
  int keys_per_split;     // multiple of 64
  int max_splits;         // grid.x; splits beyond a request's length exit at once
  void* out;
  int64_t out_stride;
  float* part_o;          // scratch [B, hq, max_splits, D] fp32
  float* part_lse;        // scratch [B, hq, max_splits] fp32
  int num_pages;          // as in AttnPrefillArgs (0 = unchecked)
  int* counters;          // [B, hkv] int32 zeros: the last split merges (nullptr: separate combine launch)
};
cudaError_t attention_decode(const AttnDecodeArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- fused decoder-step ops
struct RopeStoreArgs {
  void* qkv;               // [tokens, (hq + 2 hkv) * D], q and k rotated in place
  int64_t qkv_stride;
  int tokens, hq, hkv, head_dim;
  const void* q_norm;      // [D] bf16 or nullptr
  const void* k_norm;
  float eps;
  const int* positions;    // [pos_rows, tokens]
  int pos_rows;            // 1 (plain RoPE) or 3 (M-RoPE t/h/w)
  int section[3];          // M-RoPE frequency sections (pairs)
  int interleaved;         // M-RoPE interleaved (THWTHW...) layout
  const float* cos_tab;    // [max_pos, rot_dim / 2]
  const float* sin_tab;
  int rot_dim;             // rotated dims (<= D); 0 disables RoPE
  int neox;                // 1: rotate halves, 0: rotate adjacent pairs
  const int* slot_mapping; // [tokens] page * 64 + offset, -1 skips; nullptr => no cache write
  void* k_cache;
  void* v_cache;
  int64_t num_slots;       // cache slots (pages * 64); stores at slots >= num_slots are skipped. 0 = unchecked
};
cudaError_t qkv_rope_store(const RopeStoreArgs& a, cudaStream_t stream);

struct MoeRouteArgs {
  const float* logits;     // [tokens, experts] router logits (fp32)
  int64_t logits_stride;
  int tokens, experts, topk;
  int mode;                // 0 softmax top-k; 1 sigmoid + bias, group-limited
  const float* bias;       // [experts] selection bias (mode 1) or nullptr
  int n_group, topk_group;
  int renormalize;
  float scaling;
  int* topk_ids;           // [tokens, topk]
  float* topk_w;           // [tokens, topk]
  int* counts;             // scratch [experts]; nullptr => routing only
  int* cursor;             // scratch [experts]
  int* offsets;            // [experts + 1]
  int* inv_perm;           // [tokens, topk] row of each (token, k) in the permuted layout
  const void* x;           // [tokens, hidden] bf16 rows to gather (or nullptr)
  void* x_perm;            // [tokens * topk, hidden]
  int hidden;
  int self_clean;          // cursor has experts + 1 entries: the last scatter CTA re-zeroes counts / cursor
  int local_e0, local_el;  // local_el > 0: copy x rows only for experts [e0, e0 + El) (tensor-parallel MoE)
};
cudaError_t moe_route(const MoeRouteArgs& a, cudaStream_t stream);

struct MoeCombineArgs {
  const void* y_perm;      // [tokens * topk, hidden]
  const int* inv_perm;
  const float* topk_w;
  int tokens, topk, hidden;
  const void* shared;      // [tokens, hidden] shared-expert output or nullptr
  const float* shared_gate;// [tokens] gate logits (sigmoid applied) or nullptr (=1)
  int shared_gate_stride;
  void* out;               // [tokens, hidden] (may be nullptr when the residual / norm outputs are used)
  // optional fused "add + RMSNorm" of the next block: residual += out (bf16), normed = w * rmsnorm(residual)
  void* residual;          // [tokens, hidden] or nullptr
  const void* norm_w;      // [hidden]
  void* normed;            // [tokens, hidden]
  float eps;
  // tensor-parallel MoE: only positions of this rank's experts count (offsets of
  // experts e0 .. e0 + El, pointer already advanced to e0), and row t is stored at
  // peer_out[t / rows_per] + t * hidden (the owner's partial-sum slot)
  const int* local_offsets;
  int local_experts;
  const unsigned long long* peer_out;
  int rows_per;
  // expert-parallel: wait (bounded) until wait_flags[i] reaches *wait_seq for i < wait_count
  // (every expert owner has stored this rank's routed rows) before reading y_perm
  const unsigned int* wait_flags;
  const unsigned int* wait_seq;
  int wait_count;
  int* status;
  long long wait_timeout_ns;
};
cudaError_t moe_combine(const MoeCombineArgs& a, cudaStream_t stream);

struct EmbedArgs {
  const int* ids;
  const void* table;       // [vocab, hidden]
  const int* mm_index;     // [tokens] row of mm_embeds or -1 (nullptr => none)
  const void* mm_embeds;
  void* out;
  int tokens, hidden;
  int vocab;               // rows of table; ids are clamped into [0, vocab) (0 = unchecked)
};
cudaError_t embed(const EmbedArgs& a, cudaStream_t stream);

// In-place rotate-half RoPE over the first `rot` dims of `heads` heads per row (head h at
// column h * head_stride), angles given per row: cos / sin fp32 [rows, rot] (row stride cs_stride).
// The vision tower's 2-D rotary embedding on the q and k heads of its fused QKV rows.
cudaError_t rope_half_inplace(void* x, int64_t row_stride, int rows, int heads, int head_stride, int rot,
                              const float* cos, const float* sin, int64_t cs_stride, cudaStream_t stream);

// Dual-AR (S2-Pro) input embedding: token embedding plus, at VQ positions, the
// sum of one codebook embedding per codebook, scaled:
//   out[t] = vq(t) ? bf16(bf16(E[id] + bf16(sum_c CB[c * cb_size + code_c])) * scale) : E[id]
// Token id: slot_tokens[slot[t]] when slot != nullptr, else ids[t].
// Code row r: code_row[t] when code_row != nullptr (r < 0: no VQ), else slot[t] or t;
// without code_row, vq(t) holds for ids in [sem_lo, sem_hi].
struct VqEmbedArgs {
  const int* ids;
  const int* slot;
  const int* slot_tokens;
  const void* table;       // [vocab, hidden] bf16
  const void* codebooks;   // [ncb * cb_size, hidden] bf16
  const int* codes;        // [rows, codes_stride] int32
  int codes_stride;
  const int* code_row;
  int sem_lo, sem_hi, ncb, cb_size;
  float scale;
  void* out;
  int tokens, hidden;
  int vocab;               // rows of table (ids clamped into range; 0 = unchecked)
};
cudaError_t vq_embed(const VqEmbedArgs& a, cudaStream_t stream);

struct SampleArgs {
  float* logits;           // [rows, vocab] fp32, processed in place
  int64_t logits_stride;
  int rows, vocab;
  const float* temperature;  // [rows] (0 => greedy) or nullptr (all greedy)
  const int* top_k;          // [rows] (<= 0 disables)
  const float* top_p;        // [rows]
  const float* min_p;        // [rows]
  const float* rep_penalty;  // [rows]
  uint8_t* seen;             // [rows, seen_stride] token-seen mask (penalty + update)
  int64_t seen_stride;
  int suppress_lo, suppress_hi, suppress_keep;  // [lo, hi) masked except keep; lo < 0 disables
  const int64_t* seeds;      // [rows]
  int* step;                 // [rows] decode step (RNG counter), incremented after the draw
  int* out_tokens;           // [rows]
  const int* row_slot;       // optional [rows]: per-row state lives at index row_slot[row]
                             // of temperature / top_k / top_p / min_p / rep_penalty / seen /
                             // seeds / step, and the token is also written to slot_tokens[slot]
  int* slot_tokens;
};
cudaError_t sample(const SampleArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- vocab-parallel sampling
// The LM head split over the vocabulary: rank r holds logits columns
// [vocab0, vocab0 + vocab_local) of the full vocabulary.  ``vocab_sample_local``
// processes this rank's slice (same rules as ``sample``) and publishes one record
// per row into every rank's exchange region: its max, sum of exp, the greedy /
// Gumbel-max winner of the slice and its top-``cand`` (value, token) pairs.
// ``vocab_sample_merge`` waits (bounded) for every rank's records and draws the
// token from them; every rank draws the same token.
constexpr int kVpMaxCand = 256;
constexpr int kVpMaxWorld = 8;
constexpr int kVpHeaderBytes = 32;
struct VocabSampleArgs {
  float* logits;              // [rows, logits_stride] fp32 slice of this rank (processed in place)
  int64_t logits_stride;
  int rows, vocab_local, vocab0, vocab;
  int rank, world, cand, max_rows;
  const int64_t* peer_xchg;   // [world] base of every rank's exchange region
  const int64_t* peer_flags;  // [world] base of every rank's u32 flags[world]
  int* seq;                   // device sequence number of the exchange
  int* counter;               // CTA arrival counter of the local phase
  int* status;
  int64_t timeout_ns;
  int* inexact;               // rows drawn from an incomplete candidate set (counter)
  const float* temperature;
  const int* top_k;
  const float* top_p;
  const float* min_p;
  const float* rep_penalty;
  uint8_t* seen;              // full-vocabulary seen mask [slots, seen_stride]
  int64_t seen_stride;
  int suppress_lo, suppress_hi, suppress_keep;  // full-vocabulary ids
  const int64_t* seeds;
  int* step;
  int* out_tokens;
  const int* row_slot;
  int* slot_tokens;
};
cudaError_t vocab_sample_local(const VocabSampleArgs& a, cudaStream_t stream);
cudaError_t vocab_sample_merge(const VocabSampleArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- audio / vocoder ops (channels-last)
cudaError_t snake(const void* x, const float* alpha, const float* beta, void* y, int64_t n, int C, int log_scale,
                  cudaStream_t stream);
cudaError_t conv1d_im2col(const void* x, void* out, int B, int T_in, int T_out, int C, int K, int dil, int stride,
                          int pad_left, int out_row_stride, cudaStream_t stream);
cudaError_t conv_transpose_ola(const void* y, const void* bias, void* out, int B, int T, int s, int C, int T_out,
                               int shift, cudaStream_t stream);
cudaError_t dwconv1d_causal(const void* x, const float* w, const float* bias, void* out, int B, int T, int C, int K,
                            cudaStream_t stream);
cudaError_t conv2d_im2col(const void* x, void* out, int N, int H, int W, int C, int Ho, int Wo, int kh, int kw,
                          int stride, int pad, int K_stride, cudaStream_t stream);

// Expert-parallel MoE dispatch over peer memory (csrc/ep_moe.cu).  Every rank's
// symmetric buffer holds, at the same offsets:
//   flags   u32 [2][world]        [0][s]: source s has dispatched this layer's rows here,
//                                 [1][s]: owner s has stored this rank's expert outputs
//   cursor  i32 [El]              rows received per local expert (peers add with system atomics)
//   recv_x  bf16 [El * seg_cap, H]   segment g = rows routed to local expert g
//   recv_tag i32 [El * seg_cap, 2]   (source rank, source slot = token * topk + k) of every row
//   comb    bf16 [max_slots, H]   expert outputs of this rank's routed rows, by slot
struct EpDispatchArgs {
  int rank, world, experts, local_experts, topk, hidden;
  int tokens;                  // this rank's tokens
  const int* topk_ids;         // [tokens, topk]
  const void* x;               // [tokens, hidden] bf16
  const int64_t* peer_base;    // [world] base address of every rank's symmetric buffer
  int64_t off_flags, off_cursor, off_recv_x, off_recv_tag;
  int seg_cap;
  uint32_t* seq;               // [1] layer sequence number, bumped by the last CTA
  int* arrive;                 // [1] CTA arrival counter, zero between calls
  int* status;
};
cudaError_t ep_dispatch(const EpDispatchArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- tensor parallel
struct TpReduceArgs {
  const unsigned long long* peer_part;   // [world] each rank's part region bf16 [world][max_tokens][H]
  const unsigned long long* peer_gath;   // [world] each rank's gath region bf16 [max_tokens][H]
  const unsigned long long* peer_gres;   // [world] each rank's gres region, or nullptr (no residual gather)
  const unsigned long long* peer_flags;  // [world] each rank's flags u32 [2][world]
  int rank, world, tokens, hidden, rows_per, max_tokens;
  void* residual;          // local bf16 [tokens, H]: owned rows read and updated
  const void* norm_w;      // bf16 [H]
  float eps;
  unsigned int* seq;       // local sequence counter (device)
  int* counter;            // local CTA arrival counter, zero between calls
  int* status;
  long long timeout_ns;
  int single_src;          // 1: the owned rows are already reduced in part[rank] (sum that slot only)
  int gather_local;        // 1: store the normalised rows into this rank's gath only (no all-gather)
};
cudaError_t tp_reduce_norm(const TpReduceArgs& a, cudaStream_t stream);
cudaError_t tp_wait(const TpReduceArgs& a, cudaStream_t stream);

}  // namespace omni
