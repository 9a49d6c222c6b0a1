// torch bindings of the sm_100a kernels (module sglang_omni_b200._C).
// Every entry validates device, dtype, contiguity and shape, then forwards raw
// pointers and the current CUDA stream to the launchers in omni_kernels.h.
#include <cstring>
#include <string>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "omni_kernels.h"

namespace {

#define OMNI_CHECK_CUDA(t) TORCH_CHECK((t).is_cuda(), #t " must be a CUDA tensor")
#define OMNI_CHECK_BF16(t) TORCH_CHECK((t).scalar_type() == at::kBFloat16, #t " must be bfloat16")
#define OMNI_CHECK_CONTIG(t) TORCH_CHECK((t).is_contiguous(), #t " must be contiguous")

void check_launch(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, what, " failed: ", cudaGetErrorString(e));
}

int* status_ptr(const c10::optional<torch::Tensor>& status) {
  if (!status.has_value()) return nullptr;
  TORCH_CHECK(status->scalar_type() == at::kInt && status->is_cuda(), "status must be a CUDA int32 tensor");
  return status->data_ptr<int>();
}

// out[r, m] = act(b[r] . a[g*a_rows + m]) (+ bias) (+ residual)
void gemm(const torch::Tensor& a, const torch::Tensor& b, torch::Tensor& out, const c10::optional<torch::Tensor>& offsets,
          int64_t m_out, bool gated, const c10::optional<torch::Tensor>& bias,
          const c10::optional<torch::Tensor>& residual, int64_t act, int64_t expected_rows,
          const c10::optional<torch::Tensor>& status, int64_t max_ctas,
          const c10::optional<torch::Tensor>& splitk_ws, const c10::optional<torch::Tensor>& splitk_counters,
          const c10::optional<torch::Tensor>& peer_out, int64_t rows_per, const c10::optional<torch::Tensor>& wait_flags,
          const c10::optional<torch::Tensor>& wait_seq, double wait_timeout_s, bool static_a, bool splitk_cluster) {
  OMNI_CHECK_CUDA(a);
  OMNI_CHECK_CUDA(b);
  OMNI_CHECK_CUDA(out);
  OMNI_CHECK_BF16(a);
  OMNI_CHECK_BF16(b);
  OMNI_CHECK_CONTIG(a);
  OMNI_CHECK_CONTIG(b);
  TORCH_CHECK(out.stride(-1) == 1, "out must have a contiguous last dim");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 || out.scalar_type() == at::kFloat, "out must be bf16 or fp32");
  const int64_t k = b.size(-1);
  TORCH_CHECK(a.size(-1) == k, "K mismatch: a ", a.sizes(), " b ", b.sizes());
  const int64_t rows = b.numel() / k;
  int groups = 1;
  int64_t a_rows;
  const int* off = nullptr;
  if (a.dim() == 3) {
    groups = static_cast<int>(a.size(0));
    a_rows = a.size(1);
  } else {
    TORCH_CHECK(a.dim() == 2, "a must be 2-D or 3-D");
    a_rows = a.size(0);
  }
  if (offsets.has_value()) {
    TORCH_CHECK(offsets->scalar_type() == at::kInt && offsets->is_cuda() && offsets->numel() == groups + 1,
                "offsets must be CUDA int32 [groups+1]");
    off = offsets->data_ptr<int>();
  } else {
    TORCH_CHECK(groups == 1, "grouped GEMM needs offsets");
  }
  TORCH_CHECK(gated ? a_rows == 2 * m_out : a_rows >= m_out, "weight rows do not match m_out");
  TORCH_CHECK(out.numel() / out.size(-1) == rows && out.size(-1) >= m_out, "out shape mismatch");
  const at::cuda::CUDAGuard guard(b.device());
  omni::GemmArgs args{};
  args.a = a.data_ptr();
  args.b = b.data_ptr();
  args.out = out.data_ptr();
  args.ldo = out.dim() >= 2 ? out.stride(-2) : out.size(-1);
  args.out_f32 = out.scalar_type() == at::kFloat;
  if (bias.has_value()) {
    OMNI_CHECK_BF16(*bias);
    TORCH_CHECK(bias->numel() == static_cast<int64_t>(groups) * m_out, "bias size mismatch");
    args.bias = bias->data_ptr();
  }
  if (residual.has_value()) {
    OMNI_CHECK_BF16(*residual);
    TORCH_CHECK(residual->stride(-1) == 1 && residual->numel() / residual->size(-1) == rows, "residual shape");
    args.residual = residual->data_ptr();
    args.ldr = residual->dim() >= 2 ? residual->stride(-2) : residual->size(-1);
  }
  args.m_out = static_cast<int>(m_out);
  args.a_rows = static_cast<int>(a_rows);
  args.k = static_cast<int>(k);
  args.groups = groups;
  args.offsets = off;
  args.rows = static_cast<int>(rows);
  args.expected_rows_per_group = static_cast<int>(expected_rows);
  args.gated = gated ? 1 : 0;
  args.act = static_cast<int>(act);
  args.status = status_ptr(status);
  args.max_ctas = static_cast<int>(max_ctas);
  if (splitk_ws.has_value()) {
    TORCH_CHECK(splitk_ws->scalar_type() == at::kFloat, "split-K scratch must be fp32");
    args.splitk_ws = splitk_ws->data_ptr<float>();
    args.splitk_ws_floats = splitk_ws->numel();
    if (splitk_counters.has_value()) {  // without counters a second kernel finalises the splits
      TORCH_CHECK(splitk_counters->scalar_type() == at::kInt, "split-K counters must be int32");
      args.splitk_counters = splitk_counters->data_ptr<int>();
      args.splitk_counter_slots = static_cast<int>(splitk_counters->numel());
    }
  }
  if (peer_out.has_value()) {
    TORCH_CHECK(peer_out->scalar_type() == at::kLong && peer_out->is_cuda() && !args.out_f32 && rows_per > 0,
                "owner scatter: int64 device pointer table, bf16 output, rows_per > 0");
    TORCH_CHECK((rows + rows_per - 1) / rows_per <= peer_out->numel(), "owner scatter: more owners than pointers");
    args.peer_out = reinterpret_cast<const unsigned long long*>(peer_out->data_ptr<int64_t>());
    args.rows_per = static_cast<int>(rows_per);
  }
  if (wait_flags.has_value()) {
    TORCH_CHECK(wait_seq.has_value() && wait_flags->scalar_type() == at::kInt && wait_seq->scalar_type() == at::kInt,
                "wait flags / sequence must be int32");
    args.wait_flags = reinterpret_cast<const unsigned int*>(wait_flags->data_ptr<int>());
    args.wait_seq = reinterpret_cast<const unsigned int*>(wait_seq->data_ptr<int>());
    args.wait_count = static_cast<int>(wait_flags->numel());
    args.wait_timeout_ns = static_cast<long long>(wait_timeout_s * 1e9);
  }
  args.static_a = static_a ? 1 : 0;
  args.splitk_cluster = splitk_cluster ? 1 : 0;
  check_launch(omni::gemm_bf16(args, at::cuda::getCurrentCUDAStream()), "gemm_bf16");
}

void rmsnorm(const torch::Tensor& x, const torch::Tensor& w, torch::Tensor& y,
             const c10::optional<torch::Tensor>& residual, double eps) {
  OMNI_CHECK_CUDA(x);
  OMNI_CHECK_BF16(x);
  OMNI_CHECK_BF16(w);
  OMNI_CHECK_BF16(y);
  const int64_t hidden = x.size(-1);
  TORCH_CHECK(w.numel() == hidden && x.stride(-1) == 1 && y.stride(-1) == 1, "rmsnorm shapes");
  const int64_t rows = x.numel() / hidden;
  const int64_t ld_x = x.dim() >= 2 ? x.stride(-2) : hidden;
  const int64_t ld_y = y.dim() >= 2 ? y.stride(-2) : hidden;
  void* res = nullptr;
  if (residual.has_value()) {
    OMNI_CHECK_BF16(*residual);
    OMNI_CHECK_CONTIG(*residual);
    TORCH_CHECK(residual->numel() == rows * hidden, "residual shape");
    res = residual->data_ptr();
  }
  const at::cuda::CUDAGuard guard(x.device());
  check_launch(omni::rmsnorm_bf16(x.data_ptr(), w.data_ptr(), y.data_ptr(), res, static_cast<int>(rows),
                                  static_cast<int>(hidden), ld_x, ld_y, static_cast<float>(eps),
                                  at::cuda::getCurrentCUDAStream()),
               "rmsnorm_bf16");
}

void layernorm(const torch::Tensor& x, const torch::Tensor& w, const c10::optional<torch::Tensor>& b, torch::Tensor& y,
               double eps) {
  OMNI_CHECK_CUDA(x);
  OMNI_CHECK_BF16(x);
  OMNI_CHECK_CONTIG(x);
  OMNI_CHECK_CONTIG(y);
  const int64_t hidden = x.size(-1);
  const at::cuda::CUDAGuard guard(x.device());
  check_launch(omni::layernorm_bf16(x.data_ptr(), w.data_ptr(), b.has_value() ? b->data_ptr() : nullptr,
                                    y.data_ptr(), static_cast<int>(x.numel() / hidden), static_cast<int>(hidden),
                                    static_cast<float>(eps), at::cuda::getCurrentCUDAStream()),
               "layernorm_bf16");
}


template <class T>
const T* opt_ptr(const c10::optional<torch::Tensor>& t) {
  return t.has_value() ? static_cast<const T*>(t->data_ptr()) : nullptr;
}
template <class T>
T* opt_mut(const c10::optional<torch::Tensor>& t) {
  return t.has_value() ? static_cast<T*>(t->data_ptr()) : nullptr;
}

void attention_prefill(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, torch::Tensor& out,
                       const c10::optional<torch::Tensor>& block_table, const torch::Tensor& cu_q,
                       const torch::Tensor& kv_lens, const c10::optional<torch::Tensor>& cu_kv,
                       const torch::Tensor& tile_req, const torch::Tensor& tile_tok0, int64_t hq, int64_t hkv,
                       int64_t head_dim, double scale, bool causal, int64_t window, int64_t tile_rows,
                       const c10::optional<torch::Tensor>& status) {
  OMNI_CHECK_CUDA(q);
  OMNI_CHECK_BF16(q);
  OMNI_CHECK_BF16(k);
  OMNI_CHECK_BF16(v);
  OMNI_CHECK_BF16(out);
  TORCH_CHECK(q.stride(-1) == 1 && out.stride(-1) == 1, "rows must be contiguous");
  const at::cuda::CUDAGuard guard(q.device());
  omni::AttnPrefillArgs a{};
  a.q = q.data_ptr();
  a.q_stride = q.stride(0);
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.kv_stride = block_table.has_value() ? 0 : k.stride(0);
  if (block_table.has_value()) {
    a.block_table = block_table->data_ptr<int>();
    a.bt_stride = static_cast<int>(block_table->stride(0));
  }
  a.cu_q = cu_q.data_ptr<int>();
  a.kv_lens = kv_lens.data_ptr<int>();
  a.cu_kv = cu_kv.has_value() ? cu_kv->data_ptr<int>() : nullptr;
  TORCH_CHECK(block_table.has_value() || cu_kv.has_value(), "contiguous K/V needs cu_kv");
  a.tile_req = tile_req.data_ptr<int>();
  a.tile_tok0 = tile_tok0.data_ptr<int>();
  a.num_tiles = static_cast<int>(tile_req.numel());
  a.hq = static_cast<int>(hq);
  a.hkv = static_cast<int>(hkv);
  a.head_dim = static_cast<int>(head_dim);
  a.scale = static_cast<float>(scale);
  a.causal = causal ? 1 : 0;
  a.out = out.data_ptr();
  a.out_stride = out.stride(0);
  a.window = static_cast<int>(window);
  a.num_pages = block_table.has_value() ? static_cast<int>(k.size(0)) : 0;
  a.tile_rows = static_cast<int>(tile_rows);
  a.q_rows = static_cast<int>(q.size(0));
  a.status = status_ptr(status);
  a.kv_rows = block_table.has_value() ? 0 : static_cast<int>(k.size(0));
  TORCH_CHECK(tile_rows == 64 || tile_rows == 128 || tile_rows == 256, "tile_rows must be 64, 128 or 256");
  TORCH_CHECK(tile_rows == 64 || omni::attention_prefill_sm100_supported(a),
              "128 / 256-row tiles need the tcgen05 kernel (paged: head_dim 128; contiguous: head_dim 64..128 "
              "in steps of 16; no window; aligned rows)");
  check_launch(omni::attention_prefill(a, at::cuda::getCurrentCUDAStream()), "attention_prefill");
}

void attention_decode(const torch::Tensor& q, const torch::Tensor& k, const torch::Tensor& v, torch::Tensor& out,
                      const torch::Tensor& block_table, const torch::Tensor& kv_lens, int64_t hq, int64_t hkv,
                      int64_t head_dim, double scale, int64_t keys_per_split, int64_t max_splits,
                      torch::Tensor& part_o, torch::Tensor& part_lse,
                      const c10::optional<torch::Tensor>& counters) {
  OMNI_CHECK_CUDA(q);
  OMNI_CHECK_BF16(q);
  TORCH_CHECK(q.stride(-1) == 1 && out.stride(-1) == 1, "rows must be contiguous");
  const int64_t batch = kv_lens.numel();
  TORCH_CHECK(part_o.numel() >= batch * hq * max_splits * head_dim && part_lse.numel() >= batch * hq * max_splits,
              "decode scratch too small");
  const at::cuda::CUDAGuard guard(q.device());
  omni::AttnDecodeArgs a{};
  a.q = q.data_ptr();
  a.q_stride = q.stride(0);
  a.k = k.data_ptr();
  a.v = v.data_ptr();
  a.block_table = block_table.data_ptr<int>();
  a.bt_stride = static_cast<int>(block_table.stride(0));
  a.kv_lens = kv_lens.data_ptr<int>();
  a.batch = static_cast<int>(batch);
  a.hq = static_cast<int>(hq);
  a.hkv = static_cast<int>(hkv);
  a.head_dim = static_cast<int>(head_dim);
  a.scale = static_cast<float>(scale);
  a.keys_per_split = static_cast<int>(keys_per_split);
  a.max_splits = static_cast<int>(max_splits);
  a.out = out.data_ptr();
  a.out_stride = out.stride(0);
  a.part_o = part_o.data_ptr<float>();
  a.part_lse = part_lse.data_ptr<float>();
  a.num_pages = static_cast<int>(k.size(0));
  if (counters.has_value()) {
    TORCH_CHECK(counters->scalar_type() == at::kInt && counters->numel() >= batch * hkv, "split counters int32 [B, hkv]");
    a.counters = counters->data_ptr<int>();
  }
  check_launch(omni::attention_decode(a, at::cuda::getCurrentCUDAStream()), "attention_decode");
}

void qkv_rope_store(torch::Tensor& qkv, int64_t hq, int64_t hkv, int64_t head_dim,
                    const c10::optional<torch::Tensor>& q_norm, const c10::optional<torch::Tensor>& k_norm, double eps,
                    const torch::Tensor& positions, const std::vector<int64_t>& section, bool interleaved,
                    const torch::Tensor& cos_tab, const torch::Tensor& sin_tab, int64_t rot_dim, bool neox,
                    const c10::optional<torch::Tensor>& slot_mapping, const c10::optional<torch::Tensor>& k_cache,
                    const c10::optional<torch::Tensor>& v_cache) {
  OMNI_CHECK_CUDA(qkv);
  OMNI_CHECK_BF16(qkv);
  TORCH_CHECK(qkv.stride(-1) == 1, "qkv rows must be contiguous");
  TORCH_CHECK(positions.scalar_type() == at::kInt && positions.is_contiguous(), "positions int32");
  TORCH_CHECK(cos_tab.scalar_type() == at::kFloat && sin_tab.scalar_type() == at::kFloat, "fp32 rope tables");
  TORCH_CHECK(rot_dim % 2 == 0 && rot_dim <= head_dim, "rot_dim must be even and <= head_dim");
  const at::cuda::CUDAGuard guard(qkv.device());
  omni::RopeStoreArgs a{};
  a.qkv = qkv.data_ptr();
  a.qkv_stride = qkv.stride(0);
  a.tokens = static_cast<int>(qkv.size(0));
  a.hq = static_cast<int>(hq);
  a.hkv = static_cast<int>(hkv);
  a.head_dim = static_cast<int>(head_dim);
  a.q_norm = q_norm.has_value() ? q_norm->data_ptr() : nullptr;
  a.k_norm = k_norm.has_value() ? k_norm->data_ptr() : nullptr;
  a.eps = static_cast<float>(eps);
  a.positions = positions.data_ptr<int>();
  a.pos_rows = positions.dim() == 2 ? static_cast<int>(positions.size(0)) : 1;
  for (int i = 0; i < 3; ++i) a.section[i] = i < static_cast<int>(section.size()) ? static_cast<int>(section[i]) : 0;
  a.interleaved = interleaved ? 1 : 0;
  a.cos_tab = cos_tab.data_ptr<float>();
  a.sin_tab = sin_tab.data_ptr<float>();
  a.rot_dim = static_cast<int>(rot_dim);
  a.neox = neox ? 1 : 0;
  a.slot_mapping = slot_mapping.has_value() ? slot_mapping->data_ptr<int>() : nullptr;
  a.k_cache = k_cache.has_value() ? k_cache->data_ptr() : nullptr;
  a.v_cache = v_cache.has_value() ? v_cache->data_ptr() : nullptr;
  a.num_slots = k_cache.has_value() ? k_cache->size(0) * 64 : 0;
  check_launch(omni::qkv_rope_store(a, at::cuda::getCurrentCUDAStream()), "qkv_rope_store");
}

void moe_route(const torch::Tensor& logits, int64_t topk, int64_t mode, const c10::optional<torch::Tensor>& bias,
               int64_t n_group, int64_t topk_group, bool renormalize, double scaling, torch::Tensor& topk_ids,
               torch::Tensor& topk_w, const c10::optional<torch::Tensor>& counts,
               const c10::optional<torch::Tensor>& cursor, const c10::optional<torch::Tensor>& offsets,
               const c10::optional<torch::Tensor>& inv_perm, const c10::optional<torch::Tensor>& x,
               const c10::optional<torch::Tensor>& x_perm, int64_t local_e0, int64_t local_el) {
  OMNI_CHECK_CUDA(logits);
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(-1) == 1, "router logits must be fp32");
  const at::cuda::CUDAGuard guard(logits.device());
  omni::MoeRouteArgs a{};
  a.logits = logits.data_ptr<float>();
  a.logits_stride = logits.stride(0);
  a.tokens = static_cast<int>(logits.size(0));
  a.experts = static_cast<int>(logits.size(1));
  a.topk = static_cast<int>(topk);
  a.mode = static_cast<int>(mode);
  a.bias = opt_ptr<float>(bias);
  a.n_group = static_cast<int>(n_group);
  a.topk_group = static_cast<int>(topk_group);
  a.renormalize = renormalize ? 1 : 0;
  a.scaling = static_cast<float>(scaling);
  a.topk_ids = topk_ids.data_ptr<int>();
  a.topk_w = topk_w.data_ptr<float>();
  a.counts = opt_mut<int>(counts);
  a.cursor = opt_mut<int>(cursor);
  a.offsets = opt_mut<int>(offsets);
  a.inv_perm = opt_mut<int>(inv_perm);
  if (a.counts) TORCH_CHECK(a.cursor && a.offsets && a.inv_perm, "permutation outputs required");
  // a cursor with one extra slot (a done counter) makes the scatter leave counts / cursor zeroed itself
  a.self_clean = a.counts && cursor->numel() > a.experts ? 1 : 0;
  if (x.has_value()) {
    OMNI_CHECK_BF16(*x);
    TORCH_CHECK(x_perm.has_value() && x->is_contiguous() && x->size(-1) % 8 == 0, "x / x_perm");
    a.x = x->data_ptr();
    a.x_perm = x_perm->data_ptr();
    a.hidden = static_cast<int>(x->size(-1));
  }
  TORCH_CHECK(local_el >= 0 && local_e0 >= 0 && local_e0 + local_el <= a.experts, "local expert range");
  a.local_e0 = static_cast<int>(local_e0);
  a.local_el = static_cast<int>(local_el);
  check_launch(omni::moe_route(a, at::cuda::getCurrentCUDAStream()), "moe_route");
}

void moe_combine(const torch::Tensor& y_perm, const torch::Tensor& inv_perm, const torch::Tensor& topk_w,
                 const c10::optional<torch::Tensor>& out, const c10::optional<torch::Tensor>& shared,
                 const c10::optional<torch::Tensor>& shared_gate, const c10::optional<torch::Tensor>& residual,
                 const c10::optional<torch::Tensor>& norm_w, const c10::optional<torch::Tensor>& normed, double eps,
                 const c10::optional<torch::Tensor>& local_offsets, const c10::optional<torch::Tensor>& peer_out,
                 int64_t rows_per, const c10::optional<torch::Tensor>& wait_flags,
                 const c10::optional<torch::Tensor>& wait_seq, const c10::optional<torch::Tensor>& status,
                 double timeout_s) {
  OMNI_CHECK_CUDA(y_perm);
  OMNI_CHECK_BF16(y_perm);
  OMNI_CHECK_CONTIG(y_perm);
  TORCH_CHECK(topk_w.dim() == 2 && topk_w.is_contiguous() && inv_perm.is_contiguous(), "topk weights / inverse permutation");
  TORCH_CHECK(out.has_value() || residual.has_value() || peer_out.has_value(), "moe_combine needs an output");
  const at::cuda::CUDAGuard guard(y_perm.device());
  omni::MoeCombineArgs a{};
  a.y_perm = y_perm.data_ptr();
  a.inv_perm = inv_perm.data_ptr<int>();
  a.topk_w = topk_w.data_ptr<float>();
  a.tokens = static_cast<int>(topk_w.size(0));
  a.topk = static_cast<int>(topk_w.size(1));
  a.hidden = static_cast<int>(y_perm.size(1));
  TORCH_CHECK(inv_perm.numel() == static_cast<int64_t>(a.tokens) * a.topk, "inverse permutation size");
  auto rows_of = [&](const torch::Tensor& t, const char* what) {
    OMNI_CHECK_BF16(t);
    TORCH_CHECK(t.is_contiguous() && t.dim() == 2 && t.size(0) == a.tokens && t.size(1) == a.hidden, what,
                " must be a contiguous [tokens, hidden] tensor");
    return t.data_ptr();
  };
  if (shared.has_value()) a.shared = rows_of(*shared, "shared expert output");
  if (shared_gate.has_value()) {
    TORCH_CHECK(shared_gate->scalar_type() == at::kFloat, "shared gate fp32");
    a.shared_gate = shared_gate->data_ptr<float>();
    a.shared_gate_stride = static_cast<int>(shared_gate->dim() >= 2 ? shared_gate->stride(0) : 1);
  }
  if (out.has_value()) a.out = rows_of(*out, "out");
  if (residual.has_value()) {
    TORCH_CHECK(norm_w.has_value() && normed.has_value(), "fused norm needs its weight and output");
    a.residual = rows_of(*residual, "residual");
    a.normed = rows_of(*normed, "normed");
    OMNI_CHECK_BF16(*norm_w);
    TORCH_CHECK(norm_w->numel() == a.hidden && norm_w->is_contiguous(), "norm weight");
    a.norm_w = norm_w->data_ptr();
    a.eps = static_cast<float>(eps);
  }
  if (local_offsets.has_value()) {
    TORCH_CHECK(local_offsets->scalar_type() == at::kInt && local_offsets->is_contiguous() && local_offsets->numel() >= 2,
                "local expert offsets");
    a.local_offsets = local_offsets->data_ptr<int>();
    a.local_experts = static_cast<int>(local_offsets->numel() - 1);
  }
  if (peer_out.has_value()) {
    TORCH_CHECK(peer_out->scalar_type() == at::kLong && rows_per > 0 && !residual.has_value(),
                "owner scatter: int64 pointer table, rows_per > 0, no fused norm");
    TORCH_CHECK((a.tokens + rows_per - 1) / rows_per <= peer_out->numel(), "owner scatter: more owners than pointers");
    a.peer_out = reinterpret_cast<const unsigned long long*>(peer_out->data_ptr<int64_t>());
    a.rows_per = static_cast<int>(rows_per);
    a.out = nullptr;
  }
  if (wait_flags.has_value()) {
    TORCH_CHECK(wait_seq.has_value() && wait_flags->scalar_type() == at::kInt && wait_seq->scalar_type() == at::kInt,
                "wait flags / sequence int32");
    a.wait_flags = reinterpret_cast<const unsigned int*>(wait_flags->data_ptr<int>());
    a.wait_seq = reinterpret_cast<const unsigned int*>(wait_seq->data_ptr<int>());
    a.wait_count = static_cast<int>(wait_flags->numel());
    a.wait_timeout_ns = static_cast<long long>(timeout_s * 1e9);
  }
  a.status = status_ptr(status);
  check_launch(omni::moe_combine(a, at::cuda::getCurrentCUDAStream()), "moe_combine");
}

void rope_half_inplace(torch::Tensor& x, int64_t heads, int64_t head_stride, int64_t rot, const torch::Tensor& cos,
                       const torch::Tensor& sin) {
  OMNI_CHECK_CUDA(x);
  OMNI_CHECK_BF16(x);
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1, "x: [rows, cols] with unit column stride");
  TORCH_CHECK(heads * head_stride <= x.size(1), "heads exceed the row");
  TORCH_CHECK(cos.scalar_type() == at::kFloat && sin.scalar_type() == at::kFloat && cos.dim() == 2 &&
                  cos.sizes() == sin.sizes() && cos.stride(1) == 1 && sin.stride(1) == 1 &&
                  cos.stride(0) == sin.stride(0) && cos.size(0) >= x.size(0) && cos.size(1) >= rot,
              "cos / sin: fp32 [rows, >= rot]");
  const at::cuda::CUDAGuard guard(x.device());
  check_launch(omni::rope_half_inplace(x.data_ptr(), x.stride(0), static_cast<int>(x.size(0)),
                                       static_cast<int>(heads), static_cast<int>(head_stride),
                                       static_cast<int>(rot), cos.data_ptr<float>(), sin.data_ptr<float>(),
                                       cos.stride(0), at::cuda::getCurrentCUDAStream()),
               "rope_half_inplace");
}

void embed(const torch::Tensor& ids, const torch::Tensor& table, torch::Tensor& out,
           const c10::optional<torch::Tensor>& mm_index, const c10::optional<torch::Tensor>& mm_embeds) {
  OMNI_CHECK_CUDA(ids);
  TORCH_CHECK(ids.scalar_type() == at::kInt, "ids int32");
  OMNI_CHECK_BF16(table);
  OMNI_CHECK_CONTIG(table);
  OMNI_CHECK_CONTIG(out);
  const at::cuda::CUDAGuard guard(ids.device());
  omni::EmbedArgs a{};
  a.ids = ids.data_ptr<int>();
  a.table = table.data_ptr();
  a.mm_index = mm_index.has_value() ? mm_index->data_ptr<int>() : nullptr;
  a.mm_embeds = mm_embeds.has_value() ? mm_embeds->data_ptr() : nullptr;
  a.out = out.data_ptr();
  a.tokens = static_cast<int>(ids.numel());
  a.hidden = static_cast<int>(table.size(1));
  a.vocab = static_cast<int>(table.size(0));
  check_launch(omni::embed(a, at::cuda::getCurrentCUDAStream()), "embed");
}

void vq_embed(const c10::optional<torch::Tensor>& ids, const c10::optional<torch::Tensor>& slot,
              const c10::optional<torch::Tensor>& slot_tokens, const torch::Tensor& table,
              const torch::Tensor& codebooks, const torch::Tensor& codes, const c10::optional<torch::Tensor>& code_row,
              int64_t sem_lo, int64_t sem_hi, int64_t cb_size, double scale, torch::Tensor& out) {
  OMNI_CHECK_BF16(table);
  OMNI_CHECK_BF16(codebooks);
  OMNI_CHECK_BF16(out);
  OMNI_CHECK_CONTIG(table);
  OMNI_CHECK_CONTIG(codebooks);
  OMNI_CHECK_CONTIG(out);
  TORCH_CHECK(codes.scalar_type() == at::kInt && codes.dim() == 2 && codes.stride(1) == 1, "codes int32 [rows, ncb]");
  TORCH_CHECK(ids.has_value() != slot.has_value(), "give ids or slot");
  TORCH_CHECK(!slot.has_value() || slot_tokens.has_value(), "slot needs slot_tokens");
  const int64_t tokens = ids.has_value() ? ids->numel() : slot->numel();
  TORCH_CHECK(out.size(0) >= tokens && out.size(1) == table.size(1) && codebooks.size(1) == table.size(1),
              "vq_embed shapes");
  TORCH_CHECK(codebooks.size(0) >= codes.size(1) * cb_size, "codebook table too small");
  const at::cuda::CUDAGuard guard(table.device());
  omni::VqEmbedArgs a{};
  a.ids = ids.has_value() ? ids->data_ptr<int>() : nullptr;
  a.slot = slot.has_value() ? slot->data_ptr<int>() : nullptr;
  a.slot_tokens = slot_tokens.has_value() ? slot_tokens->data_ptr<int>() : nullptr;
  a.table = table.data_ptr();
  a.codebooks = codebooks.data_ptr();
  a.codes = codes.data_ptr<int>();
  a.codes_stride = static_cast<int>(codes.stride(0));
  a.code_row = code_row.has_value() ? code_row->data_ptr<int>() : nullptr;
  a.sem_lo = static_cast<int>(sem_lo);
  a.sem_hi = static_cast<int>(sem_hi);
  a.ncb = static_cast<int>(codes.size(1));
  a.cb_size = static_cast<int>(cb_size);
  a.scale = static_cast<float>(scale);
  a.out = out.data_ptr();
  a.tokens = static_cast<int>(tokens);
  a.hidden = static_cast<int>(table.size(1));
  a.vocab = static_cast<int>(table.size(0));
  check_launch(omni::vq_embed(a, at::cuda::getCurrentCUDAStream()), "vq_embed");
}

// ---- symmetric memory through CUDA IPC (one cudaMalloc per rank, mapped by peers)
int64_t ipc_alloc(int64_t bytes) {
  void* p = nullptr;
  check_launch(cudaMalloc(&p, static_cast<size_t>(bytes)), "cudaMalloc");
  check_launch(cudaMemset(p, 0, static_cast<size_t>(bytes)), "cudaMemset");
  return reinterpret_cast<int64_t>(p);
}
void ipc_free(int64_t ptr) { check_launch(cudaFree(reinterpret_cast<void*>(ptr)), "cudaFree"); }
py::bytes ipc_handle(int64_t ptr) {
  cudaIpcMemHandle_t h;
  check_launch(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)), "cudaIpcGetMemHandle");
  return py::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
}
int64_t ipc_open(const py::bytes& handle) {
  std::string s = handle;
  TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, s.data(), sizeof(h));
  void* p = nullptr;
  check_launch(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return reinterpret_cast<int64_t>(p);
}
void ipc_close(int64_t ptr) { check_launch(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)), "cudaIpcCloseMemHandle"); }
torch::Tensor tensor_at(int64_t ptr, const std::vector<int64_t>& shape, c10::ScalarType dtype, int64_t device) {
  return at::from_blob(reinterpret_cast<void*>(ptr), shape,
                       at::TensorOptions().dtype(dtype).device(at::kCUDA, static_cast<c10::DeviceIndex>(device)));
}

// ---- expert-parallel MoE layer (csrc/ep_moe.cu + the EP modes of the grouped GEMM)
// peer_base: int64 [world] symmetric-buffer bases; offs = {flags, cursor, recv_x, recv_tag, comb}.
void ep_dispatch(const torch::Tensor& x, const torch::Tensor& topk_ids, const torch::Tensor& peer_base,
                 const std::vector<int64_t>& offs, int64_t rank, int64_t world, int64_t experts, int64_t seg_cap,
                 torch::Tensor& seq, torch::Tensor& arrive, const c10::optional<torch::Tensor>& status) {
  OMNI_CHECK_CUDA(x);
  OMNI_CHECK_BF16(x);
  OMNI_CHECK_CONTIG(x);
  TORCH_CHECK(topk_ids.scalar_type() == at::kInt && topk_ids.dim() == 2 && topk_ids.is_contiguous() &&
                  topk_ids.size(0) == x.size(0), "topk_ids int32 [tokens, topk]");
  TORCH_CHECK(peer_base.scalar_type() == at::kLong && peer_base.is_cuda() && peer_base.numel() == world,
              "peer_base int64 [world] on the device");
  TORCH_CHECK(offs.size() == 5 && world >= 1 && rank >= 0 && rank < world && experts % world == 0, "EP geometry");
  TORCH_CHECK(seq.scalar_type() == at::kInt && arrive.scalar_type() == at::kInt, "seq / arrive int32");
  const at::cuda::CUDAGuard guard(x.device());
  omni::EpDispatchArgs a{};
  a.rank = static_cast<int>(rank);
  a.world = static_cast<int>(world);
  a.experts = static_cast<int>(experts);
  a.local_experts = static_cast<int>(experts / world);
  a.topk = static_cast<int>(topk_ids.size(1));
  a.hidden = static_cast<int>(x.size(1));
  a.tokens = static_cast<int>(x.size(0));
  a.topk_ids = topk_ids.data_ptr<int>();
  a.x = x.data_ptr();
  a.peer_base = peer_base.data_ptr<int64_t>();
  a.off_flags = offs[0];
  a.off_cursor = offs[1];
  a.off_recv_x = offs[2];
  a.off_recv_tag = offs[3];
  a.seg_cap = static_cast<int>(seg_cap);
  a.seq = reinterpret_cast<uint32_t*>(seq.data_ptr<int>());
  a.arrive = arrive.data_ptr<int>();
  a.status = status_ptr(status);
  check_launch(omni::ep_dispatch(a, at::cuda::getCurrentCUDAStream()), "ep_dispatch");
}

// Grouped GEMM of an EP layer over the receive segments: group g = rows [g * seg_cap, + counts[g]).
// w13 (gated): waits for the dispatch flags before reading counts, copies them to counts_copy.
// w2: row_tag / peer_rows route every output row to its source rank's slot, then the completion
// flags are raised (signal_flags: int64 [world] peer addresses) and the counters zero_ptr cleared.
void gemm_ep(const torch::Tensor& a, const torch::Tensor& b, torch::Tensor& out, int64_t m_out, bool gated,
             int64_t seg_cap, const torch::Tensor& counts, const c10::optional<torch::Tensor>& counts_copy,
             const c10::optional<torch::Tensor>& wait_flags, const c10::optional<torch::Tensor>& wait_seq,
             double timeout_s, const c10::optional<torch::Tensor>& row_tag,
             const c10::optional<torch::Tensor>& peer_rows, int64_t tag_slots,
             const c10::optional<torch::Tensor>& signal_flags, const c10::optional<torch::Tensor>& signal_seq,
             const c10::optional<torch::Tensor>& arrive, const c10::optional<torch::Tensor>& zero,
             int64_t expected_rows, const c10::optional<torch::Tensor>& status) {
  OMNI_CHECK_CUDA(a);
  OMNI_CHECK_CUDA(b);
  OMNI_CHECK_BF16(a);
  OMNI_CHECK_BF16(b);
  OMNI_CHECK_CONTIG(a);
  OMNI_CHECK_CONTIG(b);
  TORCH_CHECK(a.dim() == 3, "expert weights [groups, rows, K]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.stride(-1) == 1, "bf16 output rows");
  const int64_t k = b.size(-1);
  const int groups = static_cast<int>(a.size(0));
  TORCH_CHECK(a.size(2) == k && (gated ? a.size(1) == 2 * m_out : a.size(1) >= m_out), "weight shape");
  TORCH_CHECK(b.size(0) >= seg_cap * groups && seg_cap > 0, "B holds groups x seg_cap rows");
  TORCH_CHECK(counts.scalar_type() == at::kInt && counts.is_cuda() && counts.numel() >= groups, "counts int32");
  const at::cuda::CUDAGuard guard(b.device());
  omni::GemmArgs args{};
  args.a = a.data_ptr();
  args.b = b.data_ptr();
  args.out = out.data_ptr();
  args.ldo = out.stride(0);
  args.m_out = static_cast<int>(m_out);
  args.a_rows = static_cast<int>(a.size(1));
  args.k = static_cast<int>(k);
  args.groups = groups;
  args.rows = static_cast<int>(b.size(0));
  args.expected_rows_per_group = static_cast<int>(expected_rows);
  args.gated = gated ? 1 : 0;
  args.status = status_ptr(status);
  args.seg_cap = static_cast<int>(seg_cap);
  args.seg_counts = counts.data_ptr<int>();
  if (counts_copy.has_value()) args.seg_counts_copy = counts_copy->data_ptr<int>();
  if (wait_flags.has_value()) {
    TORCH_CHECK(wait_seq.has_value(), "wait needs the sequence word");
    args.wait_flags = reinterpret_cast<const unsigned int*>(wait_flags->data_ptr<int>());
    args.wait_seq = reinterpret_cast<const unsigned int*>(wait_seq->data_ptr<int>());
    args.wait_count = static_cast<int>(wait_flags->numel());
    args.wait_timeout_ns = static_cast<long long>(timeout_s * 1e9);
    args.setup_wait = 1;
  }
  if (row_tag.has_value()) {
    TORCH_CHECK(peer_rows.has_value() && peer_rows->scalar_type() == at::kLong && row_tag->scalar_type() == at::kInt &&
                    row_tag->numel() >= 2 * b.size(0), "combine epilogue: int32 tags [rows, 2], int64 row bases");
    args.row_tag = row_tag->data_ptr<int>();
    args.peer_rows = reinterpret_cast<const unsigned long long*>(peer_rows->data_ptr<int64_t>());
    args.tag_ranks = static_cast<int>(peer_rows->numel());
    args.tag_slots = static_cast<int>(tag_slots);
  } else {
    TORCH_CHECK(out.size(0) >= b.size(0), "out rows");
  }
  if (signal_flags.has_value()) {
    TORCH_CHECK(signal_seq.has_value() && arrive.has_value() && signal_flags->scalar_type() == at::kLong,
                "completion signal: int64 flag addresses, sequence word, arrival counter");
    args.signal_flags = reinterpret_cast<const unsigned long long*>(signal_flags->data_ptr<int64_t>());
    args.signal_seq = reinterpret_cast<const unsigned int*>(signal_seq->data_ptr<int>());
    args.signal_count = static_cast<int>(signal_flags->numel());
    args.arrive_counter = arrive->data_ptr<int>();
  }
  if (zero.has_value()) {
    args.zero_ptr = zero->data_ptr<int>();
    args.zero_n = static_cast<int>(zero->numel());
  }
  check_launch(omni::gemm_bf16(args, at::cuda::getCurrentCUDAStream()), "gemm_ep");
}

// Tensor-parallel reduce point: ptrs = int64 [4, world] device table of the
// part / gath / gres / flags region bases of every rank (gres row 0 = none).
omni::TpReduceArgs tp_args(const torch::Tensor& ptrs, int64_t rank, int64_t world, int64_t tokens, int64_t hidden,
                           int64_t rows_per, int64_t max_tokens, bool gather_residual, torch::Tensor& seq,
                           torch::Tensor& counter, const c10::optional<torch::Tensor>& status, double timeout_s) {
  TORCH_CHECK(ptrs.scalar_type() == at::kLong && ptrs.is_cuda() && ptrs.is_contiguous() && ptrs.dim() == 2 &&
                  ptrs.size(0) == 4 && ptrs.size(1) == world,
              "pointer table must be int64 [4, world] on the device");
  TORCH_CHECK(seq.scalar_type() == at::kInt && counter.scalar_type() == at::kInt, "seq / counter int32");
  TORCH_CHECK(rank >= 0 && rank < world && tokens <= max_tokens && rows_per > 0, "tp reduce geometry");
  omni::TpReduceArgs a{};
  const auto* p = reinterpret_cast<const unsigned long long*>(ptrs.data_ptr<int64_t>());
  a.peer_part = p;
  a.peer_gath = p + world;
  a.peer_gres = gather_residual ? p + 2 * world : nullptr;
  a.peer_flags = p + 3 * world;
  a.rank = static_cast<int>(rank);
  a.world = static_cast<int>(world);
  a.tokens = static_cast<int>(tokens);
  a.hidden = static_cast<int>(hidden);
  a.rows_per = static_cast<int>(rows_per);
  a.max_tokens = static_cast<int>(max_tokens);
  a.seq = reinterpret_cast<unsigned int*>(seq.data_ptr<int>());
  a.counter = counter.data_ptr<int>();
  a.status = status_ptr(status);
  a.timeout_ns = static_cast<long long>(timeout_s * 1e9);
  return a;
}

void tp_reduce_norm(const torch::Tensor& ptrs, int64_t rank, int64_t world, int64_t tokens, int64_t rows_per,
                    int64_t max_tokens, torch::Tensor& residual, const torch::Tensor& norm_w, double eps,
                    bool gather_residual, torch::Tensor& seq, torch::Tensor& counter,
                    const c10::optional<torch::Tensor>& status, double timeout_s, bool single_src,
                    bool gather_local) {
  OMNI_CHECK_CUDA(residual);
  OMNI_CHECK_BF16(residual);
  OMNI_CHECK_CONTIG(residual);
  OMNI_CHECK_BF16(norm_w);
  TORCH_CHECK(residual.dim() == 2 && residual.size(0) >= tokens && norm_w.numel() == residual.size(1),
              "residual [tokens, H] / norm weight [H]");
  const at::cuda::CUDAGuard guard(residual.device());
  auto a = tp_args(ptrs, rank, world, tokens, residual.size(1), rows_per, max_tokens, gather_residual, seq, counter,
                   status, timeout_s);
  a.residual = residual.data_ptr();
  a.norm_w = norm_w.data_ptr();
  a.eps = static_cast<float>(eps);
  a.single_src = single_src ? 1 : 0;
  a.gather_local = gather_local ? 1 : 0;
  TORCH_CHECK(!(gather_local && gather_residual), "gather_local with gather_residual");
  check_launch(omni::tp_reduce_norm(a, at::cuda::getCurrentCUDAStream()), "tp_reduce_norm");
}

void tp_wait(const torch::Tensor& ptrs, int64_t rank, int64_t world, torch::Tensor& seq, torch::Tensor& counter,
             const c10::optional<torch::Tensor>& status, double timeout_s) {
  const at::cuda::CUDAGuard guard(ptrs.device());
  auto a = tp_args(ptrs, rank, world, 0, 8, 1, 0, false, seq, counter, status, timeout_s);
  check_launch(omni::tp_wait(a, at::cuda::getCurrentCUDAStream()), "tp_wait");
}

void sample(torch::Tensor& logits, torch::Tensor& out_tokens, const c10::optional<torch::Tensor>& temperature,
            const c10::optional<torch::Tensor>& top_k, const c10::optional<torch::Tensor>& top_p,
            const c10::optional<torch::Tensor>& min_p, const c10::optional<torch::Tensor>& rep_penalty,
            const c10::optional<torch::Tensor>& seen, int64_t suppress_lo, int64_t suppress_hi,
            int64_t suppress_keep, const c10::optional<torch::Tensor>& seeds,
            const c10::optional<torch::Tensor>& step, const c10::optional<torch::Tensor>& row_slot,
            const c10::optional<torch::Tensor>& slot_tokens) {
  OMNI_CHECK_CUDA(logits);
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(-1) == 1, "logits fp32");
  const at::cuda::CUDAGuard guard(logits.device());
  omni::SampleArgs a{};
  a.logits = logits.data_ptr<float>();
  a.logits_stride = logits.stride(0);
  a.rows = static_cast<int>(logits.size(0));
  a.vocab = static_cast<int>(logits.size(1));
  a.temperature = opt_ptr<float>(temperature);
  a.top_k = opt_ptr<int>(top_k);
  a.top_p = opt_ptr<float>(top_p);
  a.min_p = opt_ptr<float>(min_p);
  a.rep_penalty = opt_ptr<float>(rep_penalty);
  if (seen.has_value()) {
    TORCH_CHECK(seen->scalar_type() == at::kByte, "seen must be uint8");
    a.seen = seen->data_ptr<uint8_t>();
    a.seen_stride = seen->stride(0);
  }
  a.suppress_lo = static_cast<int>(suppress_lo);
  a.suppress_hi = static_cast<int>(suppress_hi);
  a.suppress_keep = static_cast<int>(suppress_keep);
  a.seeds = seeds.has_value() ? seeds->data_ptr<int64_t>() : nullptr;
  a.step = opt_mut<int>(step);
  a.out_tokens = out_tokens.data_ptr<int>();
  a.row_slot = opt_ptr<int>(row_slot);
  a.slot_tokens = opt_mut<int>(slot_tokens);
  check_launch(omni::sample(a, at::cuda::getCurrentCUDAStream()), "sample");
}

void vocab_sample(torch::Tensor& logits, torch::Tensor& out_tokens, const torch::Tensor& peer_xchg,
                  const torch::Tensor& peer_flags, int64_t rank, int64_t world, int64_t cand, int64_t max_rows,
                  int64_t vocab0, int64_t vocab_local, int64_t vocab, torch::Tensor& seq, torch::Tensor& counter,
                  const c10::optional<torch::Tensor>& inexact, const c10::optional<torch::Tensor>& status,
                  double timeout_s, const c10::optional<torch::Tensor>& temperature,
                  const c10::optional<torch::Tensor>& top_k, const c10::optional<torch::Tensor>& top_p,
                  const c10::optional<torch::Tensor>& min_p, const c10::optional<torch::Tensor>& rep_penalty,
                  const c10::optional<torch::Tensor>& seen, int64_t suppress_lo, int64_t suppress_hi,
                  int64_t suppress_keep, const c10::optional<torch::Tensor>& seeds,
                  const c10::optional<torch::Tensor>& step, const c10::optional<torch::Tensor>& row_slot,
                  const c10::optional<torch::Tensor>& slot_tokens, int64_t phases) {
  OMNI_CHECK_CUDA(logits);
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.stride(-1) == 1, "logits fp32 with unit column stride");
  TORCH_CHECK(logits.size(1) >= vocab_local, "logits narrower than the vocabulary slice");
  TORCH_CHECK(peer_xchg.scalar_type() == at::kLong && peer_xchg.numel() == world, "peer_xchg: int64 [world]");
  TORCH_CHECK(peer_flags.scalar_type() == at::kLong && peer_flags.numel() == world, "peer_flags: int64 [world]");
  TORCH_CHECK(seq.scalar_type() == at::kInt && counter.scalar_type() == at::kInt, "seq / counter int32");
  const at::cuda::CUDAGuard guard(logits.device());
  omni::VocabSampleArgs a{};
  a.logits = logits.data_ptr<float>();
  a.logits_stride = logits.stride(0);
  a.rows = static_cast<int>(logits.size(0));
  a.vocab_local = static_cast<int>(vocab_local);
  a.vocab0 = static_cast<int>(vocab0);
  a.vocab = static_cast<int>(vocab);
  a.rank = static_cast<int>(rank);
  a.world = static_cast<int>(world);
  a.cand = static_cast<int>(cand);
  a.max_rows = static_cast<int>(max_rows);
  a.peer_xchg = peer_xchg.data_ptr<int64_t>();
  a.peer_flags = peer_flags.data_ptr<int64_t>();
  a.seq = seq.data_ptr<int>();
  a.counter = counter.data_ptr<int>();
  a.inexact = opt_mut<int>(inexact);
  a.status = status_ptr(status);
  a.timeout_ns = static_cast<int64_t>(timeout_s * 1e9);
  a.temperature = opt_ptr<float>(temperature);
  a.top_k = opt_ptr<int>(top_k);
  a.top_p = opt_ptr<float>(top_p);
  a.min_p = opt_ptr<float>(min_p);
  a.rep_penalty = opt_ptr<float>(rep_penalty);
  if (seen.has_value()) {
    TORCH_CHECK(seen->scalar_type() == at::kByte && seen->size(1) >= vocab, "seen: uint8 [slots, >= vocab]");
    a.seen = seen->data_ptr<uint8_t>();
    a.seen_stride = seen->stride(0);
  }
  a.suppress_lo = static_cast<int>(suppress_lo);
  a.suppress_hi = static_cast<int>(suppress_hi);
  a.suppress_keep = static_cast<int>(suppress_keep);
  a.seeds = seeds.has_value() ? seeds->data_ptr<int64_t>() : nullptr;
  a.step = opt_mut<int>(step);
  a.out_tokens = out_tokens.data_ptr<int>();
  a.row_slot = opt_ptr<int>(row_slot);
  a.slot_tokens = opt_mut<int>(slot_tokens);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (phases & 1) check_launch(omni::vocab_sample_local(a, stream), "vocab_sample_local");
  if (phases & 2) check_launch(omni::vocab_sample_merge(a, stream), "vocab_sample_merge");
}

void snake(const torch::Tensor& x, const torch::Tensor& alpha, const c10::optional<torch::Tensor>& beta,
           torch::Tensor& y, bool log_scale) {
  OMNI_CHECK_CUDA(x);
  OMNI_CHECK_BF16(x);
  OMNI_CHECK_CONTIG(x);
  OMNI_CHECK_CONTIG(y);
  TORCH_CHECK(alpha.scalar_type() == at::kFloat, "alpha fp32");
  const at::cuda::CUDAGuard guard(x.device());
  check_launch(omni::snake(x.data_ptr(), alpha.data_ptr<float>(), opt_ptr<float>(beta), y.data_ptr(), x.numel(),
                           static_cast<int>(x.size(-1)), log_scale ? 1 : 0, at::cuda::getCurrentCUDAStream()),
               "snake");
}

void conv1d_im2col(const torch::Tensor& x, torch::Tensor& out, int64_t K, int64_t dil, int64_t stride,
                   int64_t pad_left) {
  OMNI_CHECK_CUDA(x);
  OMNI_CHECK_BF16(x);
  OMNI_CHECK_CONTIG(x);
  TORCH_CHECK(x.dim() == 3 && out.dim() == 3 && out.stride(-1) == 1, "x [B, T, C], out [B, T_out, >= K*C]");
  const at::cuda::CUDAGuard guard(x.device());
  check_launch(omni::conv1d_im2col(x.data_ptr(), out.data_ptr(), static_cast<int>(x.size(0)),
                                   static_cast<int>(x.size(1)), static_cast<int>(out.size(1)),
                                   static_cast<int>(x.size(2)), static_cast<int>(K), static_cast<int>(dil),
                                   static_cast<int>(stride), static_cast<int>(pad_left),
                                   static_cast<int>(out.stride(1)), at::cuda::getCurrentCUDAStream()),
               "conv1d_im2col");
}

void conv_transpose_ola(const torch::Tensor& y, const c10::optional<torch::Tensor>& bias, torch::Tensor& out,
                        int64_t s, int64_t shift) {
  OMNI_CHECK_CUDA(y);
  OMNI_CHECK_BF16(y);
  OMNI_CHECK_CONTIG(y);
  OMNI_CHECK_CONTIG(out);
  TORCH_CHECK(y.dim() == 3, "y [B, T, 2s*C]");
  const int64_t C = out.size(-1);
  TORCH_CHECK(y.size(2) == 2 * s * C, "y width must be 2*s*C");
  const at::cuda::CUDAGuard guard(y.device());
  check_launch(omni::conv_transpose_ola(y.data_ptr(), bias.has_value() ? bias->data_ptr() : nullptr,
                                        out.data_ptr(), static_cast<int>(y.size(0)), static_cast<int>(y.size(1)),
                                        static_cast<int>(s), static_cast<int>(C), static_cast<int>(out.size(1)),
                                        static_cast<int>(shift), at::cuda::getCurrentCUDAStream()),
               "conv_transpose_ola");
}

void dwconv1d_causal(const torch::Tensor& x, const torch::Tensor& w, const c10::optional<torch::Tensor>& bias,
                     torch::Tensor& out) {
  OMNI_CHECK_CUDA(x);
  OMNI_CHECK_BF16(x);
  OMNI_CHECK_CONTIG(x);
  TORCH_CHECK(w.scalar_type() == at::kFloat && w.is_contiguous(), "w fp32 [C, K]");
  const at::cuda::CUDAGuard guard(x.device());
  check_launch(omni::dwconv1d_causal(x.data_ptr(), w.data_ptr<float>(), opt_ptr<float>(bias), out.data_ptr(),
                                     static_cast<int>(x.size(0)), static_cast<int>(x.size(1)),
                                     static_cast<int>(x.size(2)), static_cast<int>(w.size(1)),
                                     at::cuda::getCurrentCUDAStream()),
               "dwconv1d_causal");
}

void conv2d_im2col(const torch::Tensor& x, torch::Tensor& out, int64_t kh, int64_t kw, int64_t stride, int64_t pad) {
  OMNI_CHECK_CUDA(x);
  OMNI_CHECK_BF16(x);
  OMNI_CHECK_CONTIG(x);
  TORCH_CHECK(x.dim() == 4 && out.dim() == 4, "x [N, H, W, C], out [N, Ho, Wo, >= kh*kw*C]");
  const at::cuda::CUDAGuard guard(x.device());
  check_launch(omni::conv2d_im2col(x.data_ptr(), out.data_ptr(), static_cast<int>(x.size(0)),
                                   static_cast<int>(x.size(1)), static_cast<int>(x.size(2)),
                                   static_cast<int>(x.size(3)), static_cast<int>(out.size(1)),
                                   static_cast<int>(out.size(2)), static_cast<int>(kh), static_cast<int>(kw),
                                   static_cast<int>(stride), static_cast<int>(pad), static_cast<int>(out.stride(2)),
                                   at::cuda::getCurrentCUDAStream()),
               "conv2d_im2col");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "sm_100a kernels of sglang_omni_b200";
  m.def("gemm", &gemm, "tcgen05 GEMM (dense / grouped / gated)", py::arg("a"), py::arg("b"), py::arg("out"),
        py::arg("offsets"), py::arg("m_out"), py::arg("gated"), py::arg("bias"), py::arg("residual"), py::arg("act"),
        py::arg("expected_rows"), py::arg("status"), py::arg("max_ctas") = 0, py::arg("splitk_ws") = py::none(),
        py::arg("splitk_counters") = py::none(), py::arg("peer_out") = py::none(), py::arg("rows_per") = 0,
        py::arg("wait_flags") = py::none(), py::arg("wait_seq") = py::none(), py::arg("wait_timeout_s") = 2.0,
        py::arg("static_a") = false, py::arg("splitk_cluster") = false);
  m.def("rmsnorm", &rmsnorm, "RMSNorm (+ fused residual add)");
  m.def("layernorm", &layernorm, "LayerNorm");
  m.def("attention_prefill", &attention_prefill, "paged / varlen GQA prefill attention", py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("out"), py::arg("block_table"), py::arg("cu_q"), py::arg("kv_lens"), py::arg("cu_kv"),
        py::arg("tile_req"), py::arg("tile_tok0"), py::arg("hq"), py::arg("hkv"), py::arg("head_dim"),
        py::arg("scale"), py::arg("causal"), py::arg("window"), py::arg("tile_rows") = 64,
        py::arg("status") = py::none());
  m.def("attention_decode", &attention_decode, "paged split-KV GQA decode attention");
  m.def("qkv_rope_store", &qkv_rope_store, "QK RMSNorm + (M-)RoPE + paged KV store");
  m.def("moe_route", &moe_route, "MoE top-k routing + permutation + gather", py::arg("logits"), py::arg("topk"),
        py::arg("mode"), py::arg("bias"), py::arg("n_group"), py::arg("topk_group"), py::arg("renormalize"),
        py::arg("scaling"), py::arg("topk_ids"), py::arg("topk_w"), py::arg("counts"), py::arg("cursor"),
        py::arg("offsets"), py::arg("inv_perm"), py::arg("x"), py::arg("x_perm"), py::arg("local_e0") = 0,
        py::arg("local_el") = 0);
  m.def("moe_combine", &moe_combine, "MoE top-k weighted combine (+ shared expert), optionally fused with the "
        "next block's residual add + RMSNorm", py::arg("y_perm"), py::arg("inv_perm"), py::arg("topk_w"),
        py::arg("out"), py::arg("shared") = py::none(), py::arg("shared_gate") = py::none(),
        py::arg("residual") = py::none(), py::arg("norm_w") = py::none(), py::arg("normed") = py::none(),
        py::arg("eps") = 1e-6, py::arg("local_offsets") = py::none(), py::arg("peer_out") = py::none(),
        py::arg("rows_per") = 0, py::arg("wait_flags") = py::none(), py::arg("wait_seq") = py::none(),
        py::arg("status") = py::none(), py::arg("timeout_s") = 2.0);
  m.def("embed", &embed, "embedding gather with multimodal overwrite");
  m.def("rope_half_inplace", &rope_half_inplace, "in-place rotate-half RoPE with per-row angles");
  m.def("vq_embed", &vq_embed, "dual-AR input embedding with the scaled VQ codebook sum");
  m.def("ipc_alloc", &ipc_alloc, "cudaMalloc + zero, returns the device address");
  m.def("ipc_free", &ipc_free, "cudaFree");
  m.def("ipc_handle", &ipc_handle, "CUDA IPC handle of an ipc_alloc buffer");
  m.def("ipc_open", &ipc_open, "maps a peer's IPC handle, returns its address in this process");
  m.def("ipc_close", &ipc_close, "unmaps a peer buffer");
  m.def("tensor_at", &tensor_at, "non-owning CUDA tensor over a device address");
  m.def("tp_reduce_norm", &tp_reduce_norm, "tensor-parallel reduce-scatter + residual + RMSNorm + all-gather "
        "over peer memory", py::arg("ptrs"), py::arg("rank"), py::arg("world"), py::arg("tokens"), py::arg("rows_per"),
        py::arg("max_tokens"), py::arg("residual"), py::arg("norm_w"), py::arg("eps"), py::arg("gather_residual"),
        py::arg("seq"), py::arg("counter"), py::arg("status"), py::arg("timeout_s"), py::arg("single_src") = false,
        py::arg("gather_local") = false);
  m.def("tp_wait", &tp_wait, "tensor-parallel: wait until every rank's gathered rows have landed");
  m.def("ep_dispatch", &ep_dispatch, "expert-parallel: every routed row into its expert owner's receive segment "
                                      "(system-atomic reservations), then the dispatch flags");
  m.def("gemm_ep", &gemm_ep, "expert-parallel grouped GEMM over receive segments (flag wait / combine epilogue / "
                             "completion flags)");
  m.def("sample", &sample, "fused logits processing + sampling");
  m.def("vocab_sample", &vocab_sample, "vocab-parallel sampling: per-rank candidate records over peer memory "
                                       "(phase 1) and the merged draw (phase 2)");
  m.def("snake", &snake, "Snake / SnakeBeta activation (channels-last)");
  m.def("conv1d_im2col", &conv1d_im2col, "causal dilated conv1d im2col rows");
  m.def("conv_transpose_ola", &conv_transpose_ola, "transposed-conv overlap-add + bias + causal trim");
  m.def("dwconv1d_causal", &dwconv1d_causal, "depthwise causal conv1d");
  m.def("conv2d_im2col", &conv2d_im2col, "2-D conv im2col rows (kh, kw, c)");
}
