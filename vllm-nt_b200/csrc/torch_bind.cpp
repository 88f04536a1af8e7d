// torch.ops.ntb200.* -- a thin binding from torch tensors to the libntb200 C ABI.
//
// Every op writes into caller-allocated outputs (schemas mark them mutable), runs on the
// current CUDA stream of the tensors' device, and turns a non-zero C-ABI status into a
// c10::Error carrying the status string and detail.  There is no CPU implementation: a
// CPU tensor reaching these ops is an error, never a silent fallback.
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "ntb200.h"

namespace {

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return NTB200_DTYPE_F32;
    case at::kBFloat16: return NTB200_DTYPE_BF16;
    case at::kHalf: return NTB200_DTYPE_F16;
    case at::kInt: return NTB200_DTYPE_I32;
    case at::kLong: return NTB200_DTYPE_I64;
    default: TORCH_CHECK(false, "ntb200: unsupported dtype ", t.scalar_type());
  }
}

void check(int status, const char* op) {
  TORCH_CHECK(status == NTB200_OK, "ntb200.", op, " failed: ", ntb200_status_string(status),
              ": ", ntb200_last_error());
}

void* stream_of(const at::Tensor& t) {
  return static_cast<void*>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

void require_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "ntb200: ", name, " must be a CUDA tensor (no CPU path exists)");
}

void require_rows(const at::Tensor& t, const char* name) {
  require_cuda(t, name);
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, "ntb200: ", name,
              " must be 2-D with unit stride in the last dim");
}

// A tensor seen as rows of its last dimension: the last dimension has unit stride and the
// leading dimensions collapse into one row index with a single stride (any contiguous
// tensor, a row-strided 2-D view, ...).  vLLM hands the hooks [tokens, hidden] or
// [batch, tokens, hidden] activations; viewing them here saves the Python reshapes.
struct Rows {
  int64_t rows = 0, stride = 0, cols = 0;
};

Rows rows_of(const at::Tensor& t, const char* name) {
  require_cuda(t, name);
  const int64_t d = t.dim();
  TORCH_CHECK(d >= 1 && t.stride(d - 1) == 1, "ntb200: ", name, " needs unit stride in the last dim");
  Rows r;
  r.cols = t.size(d - 1);
  if (d == 1) {
    r.rows = 1;
    r.stride = r.cols;
    return r;
  }
  r.rows = t.size(d - 2);
  r.stride = t.stride(d - 2);
  int64_t expect = r.stride * t.size(d - 2);
  for (int64_t i = d - 3; i >= 0; --i) {
    if (t.size(i) == 1) continue;
    TORCH_CHECK(t.stride(i) == expect, "ntb200: ", name, "'s leading dims do not collapse into rows");
    r.rows *= t.size(i);
    expect = t.stride(i) * t.size(i);
  }
  if (r.rows <= 1) r.stride = r.cols > r.stride ? r.cols : r.stride;
  return r;
}

void same_leading(const at::Tensor& a, const at::Tensor& b, const char* what) {
  TORCH_CHECK(a.dim() == b.dim(), "ntb200.", what, ": rank mismatch");
  for (int64_t i = 0; i + 1 < a.dim(); ++i)
    TORCH_CHECK(a.size(i) == b.size(i), "ntb200.", what, ": leading shape mismatch");
}

const void* norm_weight(const std::optional<at::Tensor>& weight, const at::Tensor& x, int64_t hidden,
                        const char* what) {
  if (!weight.has_value()) return nullptr;
  TORCH_CHECK(weight->is_contiguous() && weight->numel() == hidden && weight->scalar_type() == x.scalar_type(),
              "ntb200.", what, ": weight must be contiguous [hidden] of x's dtype");
  return weight->data_ptr();
}

void rms_norm(at::Tensor out, const at::Tensor& x, const std::optional<at::Tensor>& weight,
              double eps) {
  const Rows xr = rows_of(x, "x"), orr = rows_of(out, "out");
  TORCH_CHECK(out.sizes() == x.sizes() && out.scalar_type() == x.scalar_type(), "ntb200.rms_norm: out mismatch");
  const void* w = norm_weight(weight, x, xr.cols, "rms_norm");
  c10::cuda::CUDAGuard guard(x.device());
  check(ntb200_rms_norm(out.data_ptr(), x.data_ptr(), w, xr.rows, xr.cols, xr.stride, orr.stride,
                        static_cast<float>(eps), dtype_code(x), stream_of(x)),
        "rms_norm");
}

void fused_add_rms_norm(at::Tensor out, at::Tensor residual, const at::Tensor& x,
                        const std::optional<at::Tensor>& weight, double eps) {
  const Rows xr = rows_of(x, "x"), orr = rows_of(out, "out"), rr = rows_of(residual, "residual");
  TORCH_CHECK(out.sizes() == x.sizes() && residual.sizes() == x.sizes() &&
                  out.scalar_type() == x.scalar_type() &&
                  residual.scalar_type() == x.scalar_type(),
              "ntb200.fused_add_rms_norm: shape/dtype mismatch");
  const void* w = norm_weight(weight, x, xr.cols, "fused_add_rms_norm");
  c10::cuda::CUDAGuard guard(x.device());
  check(ntb200_fused_add_rms_norm(out.data_ptr(), residual.data_ptr(), x.data_ptr(), w, xr.rows,
                                  xr.cols, xr.stride, rr.stride, orr.stride,
                                  static_cast<float>(eps), dtype_code(x), stream_of(x)),
        "fused_add_rms_norm");
}

void gemma_rms_norm(at::Tensor out, const at::Tensor& x, const at::Tensor& weight, double eps) {
  const Rows xr = rows_of(x, "x"), orr = rows_of(out, "out");
  TORCH_CHECK(out.sizes() == x.sizes() && out.scalar_type() == x.scalar_type(), "ntb200.gemma_rms_norm: out mismatch");
  const void* w = norm_weight(weight, x, xr.cols, "gemma_rms_norm");
  c10::cuda::CUDAGuard guard(x.device());
  check(ntb200_gemma_rms_norm(out.data_ptr(), x.data_ptr(), w, xr.rows, xr.cols, xr.stride, orr.stride,
                              static_cast<float>(eps), dtype_code(x), stream_of(x)),
        "gemma_rms_norm");
}

void gemma_fused_add_rms_norm(at::Tensor out, at::Tensor residual, const at::Tensor& x, const at::Tensor& weight,
                              double eps) {
  const Rows xr = rows_of(x, "x"), orr = rows_of(out, "out"), rr = rows_of(residual, "residual");
  TORCH_CHECK(out.sizes() == x.sizes() && residual.sizes() == x.sizes() && out.scalar_type() == x.scalar_type() &&
                  residual.scalar_type() == x.scalar_type(),
              "ntb200.gemma_fused_add_rms_norm: shape/dtype mismatch");
  const void* w = norm_weight(weight, x, xr.cols, "gemma_fused_add_rms_norm");
  c10::cuda::CUDAGuard guard(x.device());
  check(ntb200_gemma_fused_add_rms_norm(out.data_ptr(), residual.data_ptr(), x.data_ptr(), w, xr.rows, xr.cols,
                                        xr.stride, rr.stride, orr.stride, static_cast<float>(eps), dtype_code(x),
                                        stream_of(x)),
        "gemma_fused_add_rms_norm");
}

void silu_and_mul(at::Tensor out, const at::Tensor& x) {
  const Rows xr = rows_of(x, "x"), orr = rows_of(out, "out");
  same_leading(x, out, "silu_and_mul");
  TORCH_CHECK(xr.cols % 2 == 0 && orr.cols == xr.cols / 2 && out.scalar_type() == x.scalar_type(),
              "ntb200.silu_and_mul: out must be [..., d] for x [..., 2d]");
  c10::cuda::CUDAGuard guard(x.device());
  check(ntb200_silu_and_mul(out.data_ptr(), x.data_ptr(), xr.rows, orr.cols, xr.stride, orr.stride,
                            dtype_code(x), stream_of(x)),
        "silu_and_mul");
}

// query/key as vLLM passes them ([tokens, heads * head_size], a column slice of the qkv
// projection) or as [tokens, heads, head_size]; returns heads, token and head strides.
void head_geometry(const at::Tensor& t, int64_t tokens, int64_t head_size, const char* name,
                   int64_t& heads, int64_t& ts, int64_t& hs) {
  require_cuda(t, name);
  if (t.dim() == 2) {
    TORCH_CHECK(t.stride(1) == 1 && t.size(0) == tokens && t.size(1) % head_size == 0,
                "ntb200.rope: ", name, " [tokens, heads * head_size] with unit inner stride");
    heads = t.size(1) / head_size;
    ts = t.stride(0);
    hs = head_size;
    return;
  }
  TORCH_CHECK(t.dim() == 3 && t.size(2) == head_size && t.stride(2) == 1 && t.size(0) == tokens,
              "ntb200.rope: ", name, " must be [tokens, heads, head_size] with unit inner stride");
  heads = t.size(1);
  ts = t.stride(0);
  hs = t.stride(1);
}

void rotary_embedding_neox(const at::Tensor& positions, at::Tensor query,
                           const std::optional<at::Tensor>& key, const at::Tensor& cache,
                           int64_t head_size, int64_t rotary_dim) {
  require_cuda(positions, "positions");
  require_rows(cache, "cos_sin_cache");
  TORCH_CHECK(positions.is_contiguous(), "ntb200.rope: positions must be contiguous");
  TORCH_CHECK(cache.scalar_type() == query.scalar_type(), "ntb200.rope: cos_sin_cache dtype must match query");
  const int64_t tokens = positions.numel();
  int64_t hq = 0, qts = 0, qhs = 0, hk = 0, kts = 0, khs = 0;
  head_geometry(query, tokens, head_size, "query", hq, qts, qhs);
  void* kptr = nullptr;
  if (key.has_value()) {
    TORCH_CHECK(key->scalar_type() == query.scalar_type(), "ntb200.rope: key dtype must match query");
    head_geometry(*key, tokens, head_size, "key", hk, kts, khs);
    kptr = key->data_ptr();
  }
  c10::cuda::CUDAGuard guard(query.device());
  check(ntb200_rotary_embedding_neox(positions.data_ptr(), dtype_code(positions), query.data_ptr(),
                                     kptr, cache.data_ptr(), tokens, hq, hk, head_size, rotary_dim,
                                     qts, qhs, kts, khs, cache.stride(0), cache.size(0),
                                     dtype_code(query), stream_of(query)),
        "rotary_embedding_neox");
}

void reshape_and_cache(const at::Tensor& key, const at::Tensor& value, at::Tensor key_cache,
                       at::Tensor value_cache, const at::Tensor& slot_mapping) {
  require_cuda(key, "key");
  require_cuda(value, "value");
  require_cuda(key_cache, "key_cache");
  require_cuda(value_cache, "value_cache");
  require_cuda(slot_mapping, "slot_mapping");
  TORCH_CHECK(key.dim() == 3 && value.sizes() == key.sizes() && key.stride(2) == 1 &&
                  value.stride(2) == 1,
              "ntb200.reshape_and_cache: key/value must be [tokens, heads, head_size]");
  TORCH_CHECK(key_cache.dim() == 4 && value_cache.sizes() == key_cache.sizes() &&
                  key_cache.strides() == value_cache.strides() && key_cache.stride(3) == 1,
              "ntb200.reshape_and_cache: caches must be [blocks, block_size, heads, head_size] with equal strides");
  TORCH_CHECK(key_cache.size(2) == key.size(1) && key_cache.size(3) == key.size(2),
              "ntb200.reshape_and_cache: head geometry mismatch");
  TORCH_CHECK(key_cache.scalar_type() == key.scalar_type() && value.scalar_type() == key.scalar_type() &&
                  value_cache.scalar_type() == key.scalar_type(),
              "ntb200.reshape_and_cache: dtype mismatch");
  TORCH_CHECK(slot_mapping.dim() == 1 && slot_mapping.is_contiguous() &&
                  slot_mapping.size(0) <= key.size(0),
              "ntb200.reshape_and_cache: slot_mapping must be 1-D contiguous, <= tokens");
  c10::cuda::CUDAGuard guard(key.device());
  check(ntb200_reshape_and_cache(
            key.data_ptr(), value.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
            slot_mapping.data_ptr(), dtype_code(slot_mapping), slot_mapping.size(0), key.size(1),
            key.size(2), key_cache.size(1), key_cache.size(0) * key_cache.size(1), key.stride(0),
            key.stride(1), value.stride(0), value.stride(1), key_cache.stride(0),
            key_cache.stride(1), key_cache.stride(2), static_cast<int>(key.element_size()),
            stream_of(key)),
        "reshape_and_cache");
}

// RoPE of query/key fused with the store of the rotated key and the value into the paged
// caches.  query/key/value as the rotary op takes them ([tokens, heads * head_size] rows or
// [tokens, heads, head_size]); caches [blocks, block_size, kv_heads, head_size] with equal
// strides.
void rope_and_cache(const at::Tensor& positions, at::Tensor query, at::Tensor key, const at::Tensor& value,
                    const at::Tensor& cos_sin_cache, at::Tensor key_cache, at::Tensor value_cache,
                    const at::Tensor& slot_mapping, int64_t head_size, int64_t rotary_dim) {
  require_cuda(positions, "positions");
  require_cuda(slot_mapping, "slot_mapping");
  require_cuda(key_cache, "key_cache");
  require_cuda(value_cache, "value_cache");
  require_rows(cos_sin_cache, "cos_sin_cache");
  TORCH_CHECK(positions.is_contiguous(), "ntb200.rope_and_cache: positions must be contiguous");
  const int64_t tokens = positions.numel();
  TORCH_CHECK(slot_mapping.dim() == 1 && slot_mapping.is_contiguous() && slot_mapping.size(0) <= tokens,
              "ntb200.rope_and_cache: slot_mapping must be 1-D contiguous, <= tokens");
  const auto dt = query.scalar_type();
  TORCH_CHECK(key.scalar_type() == dt && value.scalar_type() == dt && cos_sin_cache.scalar_type() == dt &&
                  key_cache.scalar_type() == dt && value_cache.scalar_type() == dt,
              "ntb200.rope_and_cache: query, key, value, cos_sin_cache and the caches must share a dtype");
  int64_t hq = 0, qts = 0, qhs = 0, hk = 0, kts = 0, khs = 0, hv = 0, vts = 0, vhs = 0;
  head_geometry(query, tokens, head_size, "query", hq, qts, qhs);
  head_geometry(key, tokens, head_size, "key", hk, kts, khs);
  head_geometry(value, tokens, head_size, "value", hv, vts, vhs);
  TORCH_CHECK(key_cache.dim() == 4 && value_cache.sizes() == key_cache.sizes() &&
                  key_cache.strides() == value_cache.strides() && key_cache.stride(3) == 1,
              "ntb200.rope_and_cache: caches must be [blocks, block_size, heads, head_size] with equal strides");
  TORCH_CHECK(hv == hk && key_cache.size(2) == hk && key_cache.size(3) == head_size,
              "ntb200.rope_and_cache: kv head geometry mismatch");
  c10::cuda::CUDAGuard guard(query.device());
  check(ntb200_rope_and_cache(positions.data_ptr(), dtype_code(positions), query.data_ptr(), key.data_ptr(),
                              value.data_ptr(), cos_sin_cache.data_ptr(), key_cache.data_ptr(),
                              value_cache.data_ptr(), slot_mapping.data_ptr(), dtype_code(slot_mapping), tokens,
                              slot_mapping.size(0), hq, hk, head_size, rotary_dim, qts, qhs, kts, khs, vts, vhs,
                              cos_sin_cache.stride(0), cos_sin_cache.size(0), key_cache.size(1),
                              key_cache.size(0) * key_cache.size(1), key_cache.stride(0), key_cache.stride(1),
                              key_cache.stride(2), dtype_code(query), stream_of(query)),
        "rope_and_cache");
}

// rope_and_cache on vLLM's combined cache: [2, blocks, block_size, kv_heads, head_size]
// (kv_dim 0, FlashAttention) or [blocks, 2, block_size, kv_heads, head_size] (kv_dim 1,
// FlashInfer).
void rope_and_cache_flash_layout(const at::Tensor& positions, at::Tensor query, at::Tensor key,
                                 const at::Tensor& value, const at::Tensor& cos_sin_cache, at::Tensor kv_cache,
                                 const at::Tensor& slot_mapping, int64_t head_size, int64_t rotary_dim,
                                 int64_t kv_dim) {
  require_cuda(kv_cache, "kv_cache");
  TORCH_CHECK((kv_dim == 0 || kv_dim == 1) && kv_cache.dim() == 5 && kv_cache.size(kv_dim) == 2,
              "ntb200.rope_and_cache_flash_layout: kv_cache must be [2, blocks, block_size, kv_heads, head_size] "
              "(kv_dim 0) or [blocks, 2, block_size, kv_heads, head_size] (kv_dim 1)");
  rope_and_cache(positions, query, key, value, cos_sin_cache, kv_cache.select(kv_dim, 0), kv_cache.select(kv_dim, 1),
                 slot_mapping.dim() == 1 ? slot_mapping : slot_mapping.reshape({-1}), head_size, rotary_dim);
}

void embedding(at::Tensor out, const at::Tensor& ids, const at::Tensor& weight) {
  require_rows(weight, "weight");
  require_rows(out, "out");
  require_cuda(ids, "ids");
  TORCH_CHECK(ids.dim() == 1 && ids.is_contiguous() && out.size(0) == ids.size(0) &&
                  out.size(1) == weight.size(1) && out.scalar_type() == weight.scalar_type(),
              "ntb200.embedding: ids [T], weight [V, H], out [T, H]");
  c10::cuda::CUDAGuard guard(weight.device());
  check(ntb200_embedding(out.data_ptr(), ids.data_ptr(), dtype_code(ids), weight.data_ptr(),
                         ids.size(0), weight.size(0), weight.size(1), weight.stride(0),
                         out.stride(0), static_cast<int>(weight.element_size()),
                         stream_of(weight)),
        "embedding");
}

void paged_attention_decode(at::Tensor out, const at::Tensor& query, const at::Tensor& key_cache,
                            const at::Tensor& value_cache, const at::Tensor& seq_lens,
                            const at::Tensor& block_table, double scale, int64_t max_seq_len,
                            at::Tensor workspace) {
  require_cuda(query, "query");
  require_cuda(out, "out");
  require_cuda(key_cache, "key_cache");
  require_cuda(value_cache, "value_cache");
  require_cuda(seq_lens, "seq_lens");
  require_cuda(block_table, "block_table");
  require_cuda(workspace, "workspace");
  TORCH_CHECK(query.dim() == 3 && query.stride(2) == 1 && out.sizes() == query.sizes() &&
                  out.stride(2) == 1 && out.scalar_type() == query.scalar_type(),
              "ntb200.paged_attention_decode: query/out must be [seqs, q_heads, head_size]");
  TORCH_CHECK(key_cache.dim() == 4 && value_cache.sizes() == key_cache.sizes() &&
                  key_cache.strides() == value_cache.strides() && key_cache.stride(3) == 1 &&
                  key_cache.scalar_type() == query.scalar_type() &&
                  value_cache.scalar_type() == query.scalar_type(),
              "ntb200.paged_attention_decode: caches must be [blocks, block_size, kv_heads, head_size] like query");
  TORCH_CHECK(seq_lens.scalar_type() == at::kInt && seq_lens.is_contiguous() &&
                  seq_lens.numel() >= query.size(0),
              "ntb200.paged_attention_decode: seq_lens must be int32 contiguous [seqs]");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && block_table.dim() == 2 &&
                  block_table.stride(1) == 1 && block_table.size(0) >= query.size(0),
              "ntb200.paged_attention_decode: block_table must be int32 [seqs, max_blocks]");
  c10::cuda::CUDAGuard guard(query.device());
  check(ntb200_paged_attention_decode(
            out.data_ptr(), query.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
            seq_lens.data_ptr<int32_t>(), block_table.data_ptr<int32_t>(), query.size(0),
            query.size(1), key_cache.size(2), query.size(2), key_cache.size(1), key_cache.size(0),
            block_table.size(1), block_table.stride(0), max_seq_len, static_cast<float>(scale),
            query.stride(0), query.stride(1), out.stride(0), out.stride(1), key_cache.stride(0),
            key_cache.stride(1), key_cache.stride(2), workspace.data_ptr(),
            static_cast<size_t>(workspace.numel() * workspace.element_size()), dtype_code(query),
            stream_of(query)),
        "paged_attention_decode");
}

int64_t decode_workspace_size(int64_t num_seqs, int64_t num_q_heads, int64_t num_kv_heads,
                              int64_t head_size, int64_t block_size, int64_t max_seq_len) {
  return static_cast<int64_t>(ntb200_paged_attention_decode_workspace_size(
      num_seqs, num_q_heads, num_kv_heads, head_size, block_size, max_seq_len));
}

// vLLM FlashAttention layout entry points: the KV cache is one [2, blocks, block_size,
// kv_heads, head_size] tensor and activations are padded to the batch's token capacity;
// only the first num_tokens rows are real.  Views, slicing and the split-K workspace (from
// the caching allocator, on the current stream) are made here, so that a hook makes one
// call per layer.
void decode_flash_layout(at::Tensor output, const at::Tensor& query, const at::Tensor& kv_cache,
                         const at::Tensor& seq_lens, const at::Tensor& block_table, int64_t num_tokens,
                         double scale, int64_t max_seq_len, int64_t kv_dim) {
  require_cuda(kv_cache, "kv_cache");
  TORCH_CHECK((kv_dim == 0 || kv_dim == 1) && kv_cache.dim() == 5 && kv_cache.size(kv_dim) == 2,
              "ntb200.decode_flash_layout: kv_cache must be [2, blocks, block_size, kv_heads, head_size] "
              "(kv_dim 0) or [blocks, 2, block_size, kv_heads, head_size] (kv_dim 1)");
  const at::Tensor kc = kv_cache.select(kv_dim, 0), vc = kv_cache.select(kv_dim, 1);
  const int64_t head = kc.size(3);
  at::Tensor q = query.dim() == 2 ? query.view({query.size(0), -1, head}) : query;
  at::Tensor o = output.dim() == 2 ? output.view({output.size(0), -1, head}) : output;
  TORCH_CHECK(num_tokens >= 0 && num_tokens <= q.size(0) && num_tokens <= o.size(0),
              "ntb200.decode_flash_layout: num_tokens exceeds the activations");
  q = q.narrow(0, 0, num_tokens);
  o = o.narrow(0, 0, num_tokens);
  const int64_t cap = block_table.size(1) * kc.size(1);
  const int64_t msl = max_seq_len <= 0 || max_seq_len > cap ? cap : max_seq_len;
  const size_t need = ntb200_paged_attention_decode_workspace_size(num_tokens, q.size(1), kc.size(2), head,
                                                                   kc.size(1), msl);
  at::Tensor ws = at::empty({static_cast<int64_t>(need > 256 ? need : 256)}, query.options().dtype(at::kByte));
  paged_attention_decode(o, q, kc, vc, seq_lens, block_table, scale, msl, ws);
}

// varlen prefill: query/out [tokens, q_heads, head_size] (the queries of sequence b are rows
// query_start_loc[b] .. query_start_loc[b + 1]); caches as for decode
void paged_attention_prefill(at::Tensor out, const at::Tensor& query, const at::Tensor& key_cache,
                             const at::Tensor& value_cache, const at::Tensor& query_start_loc,
                             const at::Tensor& seq_lens, const at::Tensor& block_table, int64_t max_query_len,
                             double scale, bool causal) {
  require_cuda(query, "query");
  require_cuda(out, "out");
  require_cuda(key_cache, "key_cache");
  require_cuda(value_cache, "value_cache");
  require_cuda(query_start_loc, "query_start_loc");
  require_cuda(seq_lens, "seq_lens");
  require_cuda(block_table, "block_table");
  TORCH_CHECK(query.dim() == 3 && query.stride(2) == 1 && out.sizes() == query.sizes() && out.stride(2) == 1 &&
                  out.scalar_type() == query.scalar_type(),
              "ntb200.paged_attention_prefill: query/out must be [tokens, q_heads, head_size]");
  TORCH_CHECK(key_cache.dim() == 4 && value_cache.sizes() == key_cache.sizes() &&
                  key_cache.strides() == value_cache.strides() && key_cache.stride(3) == 1 &&
                  key_cache.scalar_type() == query.scalar_type() && value_cache.scalar_type() == query.scalar_type(),
              "ntb200.paged_attention_prefill: caches must be [blocks, block_size, kv_heads, head_size] like query");
  TORCH_CHECK(query_start_loc.scalar_type() == at::kInt && query_start_loc.is_contiguous() &&
                  query_start_loc.dim() == 1 && query_start_loc.numel() >= 1,
              "ntb200.paged_attention_prefill: query_start_loc must be int32 contiguous [seqs + 1]");
  const int64_t seqs = query_start_loc.numel() - 1;
  TORCH_CHECK(seq_lens.scalar_type() == at::kInt && seq_lens.is_contiguous() && seq_lens.numel() >= seqs,
              "ntb200.paged_attention_prefill: seq_lens must be int32 contiguous [seqs]");
  TORCH_CHECK(block_table.scalar_type() == at::kInt && block_table.dim() == 2 && block_table.stride(1) == 1 &&
                  block_table.size(0) >= seqs,
              "ntb200.paged_attention_prefill: block_table must be int32 [seqs, max_blocks]");
  c10::cuda::CUDAGuard guard(query.device());
  check(ntb200_paged_attention_prefill(
            out.data_ptr(), query.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
            query_start_loc.data_ptr<int32_t>(), seq_lens.data_ptr<int32_t>(), block_table.data_ptr<int32_t>(), seqs,
            query.size(0), query.size(1), key_cache.size(2), query.size(2), key_cache.size(1), key_cache.size(0),
            block_table.size(1), block_table.stride(0), max_query_len, static_cast<float>(scale), causal ? 1 : 0,
            query.stride(0), query.stride(1), out.stride(0), out.stride(1), key_cache.stride(0), key_cache.stride(1),
            key_cache.stride(2), dtype_code(query), stream_of(query)),
        "paged_attention_prefill");
}

// contiguous varlen: query/out [q_tokens, q_heads, 128], key/value [k_tokens, kv_heads, 128]
void flash_attn_varlen(at::Tensor out, const at::Tensor& query, const at::Tensor& key, const at::Tensor& value,
                       const at::Tensor& cu_seqlens_q, const at::Tensor& cu_seqlens_k, int64_t max_query_len,
                       double scale, bool causal) {
  require_cuda(query, "query");
  require_cuda(out, "out");
  require_cuda(key, "key");
  require_cuda(value, "value");
  require_cuda(cu_seqlens_q, "cu_seqlens_q");
  require_cuda(cu_seqlens_k, "cu_seqlens_k");
  TORCH_CHECK(query.dim() == 3 && query.stride(2) == 1 && out.sizes() == query.sizes() && out.stride(2) == 1 &&
                  out.scalar_type() == query.scalar_type(),
              "ntb200.flash_attn_varlen: query/out must be [tokens, q_heads, head_size]");
  TORCH_CHECK(key.dim() == 3 && value.sizes() == key.sizes() && key.stride(2) == 1 && value.stride(2) == 1 &&
                  key.size(2) == query.size(2) && key.scalar_type() == query.scalar_type() &&
                  value.scalar_type() == query.scalar_type(),
              "ntb200.flash_attn_varlen: key/value must be [tokens, kv_heads, head_size] like query");
  TORCH_CHECK(cu_seqlens_q.scalar_type() == at::kInt && cu_seqlens_k.scalar_type() == at::kInt &&
                  cu_seqlens_q.is_contiguous() && cu_seqlens_k.is_contiguous() && cu_seqlens_q.dim() == 1 &&
                  cu_seqlens_q.numel() >= 1 && cu_seqlens_k.numel() == cu_seqlens_q.numel(),
              "ntb200.flash_attn_varlen: cu_seqlens_q/k must be int32 contiguous [seqs + 1]");
  c10::cuda::CUDAGuard guard(query.device());
  check(ntb200_flash_attn_varlen(out.data_ptr(), query.data_ptr(), key.data_ptr(), value.data_ptr(),
                                 cu_seqlens_q.data_ptr<int32_t>(), cu_seqlens_k.data_ptr<int32_t>(),
                                 cu_seqlens_q.numel() - 1, query.size(0), key.size(0), query.size(1), key.size(1),
                                 query.size(2), max_query_len, static_cast<float>(scale), causal ? 1 : 0,
                                 query.stride(0), query.stride(1), key.stride(0), key.stride(1), value.stride(0),
                                 value.stride(1), out.stride(0), out.stride(1), dtype_code(query), stream_of(query)),
        "flash_attn_varlen");
}

void prefill_flash_layout(at::Tensor output, const at::Tensor& query, const at::Tensor& kv_cache,
                          const at::Tensor& query_start_loc, const at::Tensor& seq_lens,
                          const at::Tensor& block_table, int64_t num_tokens, int64_t max_query_len, double scale,
                          bool causal, int64_t kv_dim) {
  require_cuda(kv_cache, "kv_cache");
  TORCH_CHECK((kv_dim == 0 || kv_dim == 1) && kv_cache.dim() == 5 && kv_cache.size(kv_dim) == 2,
              "ntb200.prefill_flash_layout: kv_cache must be [2, blocks, block_size, kv_heads, head_size] "
              "(kv_dim 0) or [blocks, 2, block_size, kv_heads, head_size] (kv_dim 1)");
  const at::Tensor kc = kv_cache.select(kv_dim, 0), vc = kv_cache.select(kv_dim, 1);
  const int64_t head = kc.size(3);
  at::Tensor q = query.dim() == 2 ? query.view({query.size(0), -1, head}) : query;
  at::Tensor o = output.dim() == 2 ? output.view({output.size(0), -1, head}) : output;
  TORCH_CHECK(num_tokens >= 0 && num_tokens <= q.size(0) && num_tokens <= o.size(0),
              "ntb200.prefill_flash_layout: num_tokens exceeds the activations");
  paged_attention_prefill(o.narrow(0, 0, num_tokens), q.narrow(0, 0, num_tokens), kc, vc, query_start_loc, seq_lens,
                          block_table, max_query_len, scale, causal);
}

// Any vLLM batch (decodes, prefills, chunked prefills, mixed) on its combined cache: the
// single-query sequences through the decode kernel, the rest through the prefill kernel.
void attention_flash_layout(at::Tensor output, const at::Tensor& query, const at::Tensor& kv_cache,
                            const at::Tensor& query_start_loc, const at::Tensor& seq_lens,
                            const at::Tensor& block_table, int64_t num_tokens, int64_t max_query_len,
                            int64_t max_seq_len, double scale, int64_t kv_dim) {
  require_cuda(kv_cache, "kv_cache");
  require_cuda(query, "query");
  require_cuda(output, "output");
  require_cuda(query_start_loc, "query_start_loc");
  require_cuda(seq_lens, "seq_lens");
  require_cuda(block_table, "block_table");
  TORCH_CHECK((kv_dim == 0 || kv_dim == 1) && kv_cache.dim() == 5 && kv_cache.size(kv_dim) == 2,
              "ntb200.attention_flash_layout: kv_cache must be [2, blocks, block_size, kv_heads, head_size] "
              "(kv_dim 0) or [blocks, 2, block_size, kv_heads, head_size] (kv_dim 1)");
  const at::Tensor kc = kv_cache.select(kv_dim, 0), vc = kv_cache.select(kv_dim, 1);
  const int64_t head = kc.size(3);
  at::Tensor q = query.dim() == 2 ? query.view({query.size(0), -1, head}) : query;
  at::Tensor o = output.dim() == 2 ? output.view({output.size(0), -1, head}) : output;
  TORCH_CHECK(num_tokens >= 0 && num_tokens <= q.size(0) && num_tokens <= o.size(0) && q.stride(2) == 1 &&
                  o.stride(2) == 1 && o.size(1) == q.size(1) && o.scalar_type() == q.scalar_type() &&
                  kc.scalar_type() == q.scalar_type() && kc.stride(3) == 1,
              "ntb200.attention_flash_layout: query/output [tokens, heads, head_size] like the cache");
  TORCH_CHECK(query_start_loc.scalar_type() == at::kInt && query_start_loc.is_contiguous() &&
                  query_start_loc.dim() == 1 && query_start_loc.numel() >= 1 &&
                  seq_lens.scalar_type() == at::kInt && seq_lens.is_contiguous() &&
                  seq_lens.numel() >= query_start_loc.numel() - 1 && block_table.scalar_type() == at::kInt &&
                  block_table.dim() == 2 && block_table.stride(1) == 1 &&
                  block_table.size(0) >= query_start_loc.numel() - 1,
              "ntb200.attention_flash_layout: int32 query_start_loc [seqs + 1], seq_lens [seqs], "
              "block_table [seqs, max_blocks]");
  const int64_t seqs = query_start_loc.numel() - 1;
  const int64_t cap = block_table.size(1) * kc.size(1);
  const int64_t msl = max_seq_len <= 0 || max_seq_len > cap ? cap : max_seq_len;
  const size_t need = ntb200_paged_attention_decode_workspace_size(seqs, q.size(1), kc.size(2), head, kc.size(1), msl);
  at::Tensor ws = at::empty({static_cast<int64_t>(need > 256 ? need : 256)}, query.options().dtype(at::kByte));
  c10::cuda::CUDAGuard guard(query.device());
  check(ntb200_paged_attention_varlen(
            o.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), query_start_loc.data_ptr<int32_t>(),
            seq_lens.data_ptr<int32_t>(), block_table.data_ptr<int32_t>(), seqs, num_tokens, q.size(1), kc.size(2),
            head, kc.size(1), kc.size(0), block_table.size(1), block_table.stride(0), max_query_len, msl,
            static_cast<float>(scale), q.stride(0), q.stride(1), o.stride(0), o.stride(1), kc.stride(0),
            kc.stride(1), kc.stride(2), ws.data_ptr(), static_cast<size_t>(ws.numel()), dtype_code(query),
            stream_of(query)),
        "attention_flash_layout");
}

void store_flash_layout(const at::Tensor& key, const at::Tensor& value, at::Tensor kv_cache,
                        const at::Tensor& slot_mapping, int64_t kv_dim) {
  require_cuda(kv_cache, "kv_cache");
  TORCH_CHECK((kv_dim == 0 || kv_dim == 1) && kv_cache.dim() == 5 && kv_cache.size(kv_dim) == 2,
              "ntb200.store_flash_layout: kv_cache must be [2, blocks, block_size, kv_heads, head_size] "
              "(kv_dim 0) or [blocks, 2, block_size, kv_heads, head_size] (kv_dim 1)");
  at::Tensor kc = kv_cache.select(kv_dim, 0), vc = kv_cache.select(kv_dim, 1);
  const int64_t heads = kc.size(2), head = kc.size(3);
  const at::Tensor k = key.dim() == 2 ? key.view({key.size(0), heads, head}) : key;
  const at::Tensor v = value.dim() == 2 ? value.view({value.size(0), heads, head}) : value;
  reshape_and_cache(k, v, kc, vc, slot_mapping.dim() == 1 ? slot_mapping : slot_mapping.reshape({-1}));
}

// x [..., K] (rows must collapse; a TMA operand needs a 16-byte aligned base and a row
// stride that is a multiple of 8 elements, otherwise x is copied once into a fresh tensor)
void linear(at::Tensor out, const at::Tensor& x_in, const at::Tensor& weight,
            const std::optional<at::Tensor>& bias, const std::optional<at::Tensor>& workspace) {
  require_rows(weight, "weight");
  at::Tensor x = x_in;
  Rows xr = rows_of(x, "x");
  if ((reinterpret_cast<uintptr_t>(x.data_ptr()) & 15u) != 0 || xr.stride % 8 != 0) {
    x = at::empty(x_in.sizes(), x_in.options());
    x.copy_(x_in);
    xr = rows_of(x, "x");
  }
  const Rows orr = rows_of(out, "out");
  same_leading(x, out, "linear");
  TORCH_CHECK(weight.size(1) == xr.cols && orr.cols == weight.size(0) &&
                  weight.scalar_type() == x.scalar_type() && out.scalar_type() == x.scalar_type(),
              "ntb200.linear: x [..., K], weight [N, K], out [..., N] of one dtype");
  const void* b = nullptr;
  if (bias.has_value()) {
    TORCH_CHECK(bias->is_contiguous() && bias->numel() == weight.size(0) &&
                    bias->scalar_type() == x.scalar_type(),
                "ntb200.linear: bias must be contiguous [N]");
    b = bias->data_ptr();
  }
  void* ws = nullptr;
  size_t ws_bytes = 0;
  if (workspace.has_value()) {
    require_cuda(*workspace, "workspace");
    ws = workspace->data_ptr();
    ws_bytes = static_cast<size_t>(workspace->numel() * workspace->element_size());
  }
  c10::cuda::CUDAGuard guard(x.device());
  check(ntb200_linear(out.data_ptr(), x.data_ptr(), weight.data_ptr(), b, xr.rows, weight.size(0),
                      xr.cols, xr.stride, weight.stride(0), orr.stride, ws, ws_bytes, dtype_code(x),
                      stream_of(x)),
        "linear");
}

// out [..., I] = silu(x W[:I]^T) * (x W[I:]^T) for the merged gate_up weight [2I, K]
void linear_silu_and_mul(at::Tensor out, const at::Tensor& x_in, const at::Tensor& weight) {
  require_rows(weight, "weight");
  at::Tensor x = x_in;
  Rows xr = rows_of(x, "x");
  if ((reinterpret_cast<uintptr_t>(x.data_ptr()) & 15u) != 0 || xr.stride % 8 != 0) {
    x = at::empty(x_in.sizes(), x_in.options());
    x.copy_(x_in);
    xr = rows_of(x, "x");
  }
  const Rows orr = rows_of(out, "out");
  same_leading(x, out, "linear_silu_and_mul");
  TORCH_CHECK(weight.size(1) == xr.cols && weight.size(0) % 2 == 0 && orr.cols == weight.size(0) / 2 &&
                  weight.scalar_type() == x.scalar_type() && out.scalar_type() == x.scalar_type(),
              "ntb200.linear_silu_and_mul: x [..., K], weight [2I, K], out [..., I] of one dtype");
  c10::cuda::CUDAGuard guard(x.device());
  check(ntb200_linear_silu_and_mul(out.data_ptr(), x.data_ptr(), weight.data_ptr(), xr.rows, orr.cols, xr.cols,
                                   xr.stride, weight.stride(0), orr.stride, dtype_code(x), stream_of(x)),
        "linear_silu_and_mul");
}

// out [M, N] = rms_norm(x (+ residual)) * norm_weight . weight^T for M <= 16 rows; with a
// residual, residual_out [M, K] receives x + residual
void rms_norm_linear(at::Tensor out, const std::optional<at::Tensor>& residual_out, const at::Tensor& x,
                     const std::optional<at::Tensor>& residual, const at::Tensor& norm_weight, double eps,
                     const at::Tensor& weight) {
  require_rows(weight, "weight");
  const Rows xr = rows_of(x, "x");
  const Rows orr = rows_of(out, "out");
  same_leading(x, out, "rms_norm_linear");
  TORCH_CHECK(weight.size(1) == xr.cols && orr.cols == weight.size(0) && weight.scalar_type() == x.scalar_type() &&
                  out.scalar_type() == x.scalar_type() && norm_weight.is_contiguous() &&
                  norm_weight.numel() == xr.cols && norm_weight.scalar_type() == x.scalar_type(),
              "ntb200.rms_norm_linear: x [M, K], norm_weight [K], weight [N, K], out [M, N] of one dtype");
  TORCH_CHECK(residual.has_value() == residual_out.has_value(),
              "ntb200.rms_norm_linear: residual and residual_out go together");
  const void* r = nullptr;
  void* ro = nullptr;
  int64_t rs = 0, ros = 0;
  if (residual.has_value()) {
    const Rows rr = rows_of(*residual, "residual");
    const Rows ror = rows_of(*residual_out, "residual_out");
    TORCH_CHECK(rr.rows == xr.rows && rr.cols == xr.cols && ror.rows == xr.rows && ror.cols == xr.cols &&
                    residual->scalar_type() == x.scalar_type() && residual_out->scalar_type() == x.scalar_type(),
                "ntb200.rms_norm_linear: residual / residual_out must match x");
    r = residual->data_ptr();
    ro = residual_out->data_ptr();
    rs = rr.stride;
    ros = ror.stride;
  }
  c10::cuda::CUDAGuard guard(x.device());
  check(ntb200_rms_norm_linear(out.data_ptr(), ro, x.data_ptr(), r, norm_weight.data_ptr(), static_cast<float>(eps),
                               weight.data_ptr(), xr.rows, weight.size(0), xr.cols, xr.stride, rs, ros,
                               weight.stride(0), orr.stride, dtype_code(x), stream_of(x)),
        "rms_norm_linear");
}

// out_index [M] (int64) = greedy argmax over the vocabulary of x [M, K] . weight [V, K]^T
void linear_argmax(at::Tensor out_index, const at::Tensor& x_in, const at::Tensor& weight) {
  require_rows(weight, "weight");
  require_cuda(out_index, "out_index");
  at::Tensor x = x_in;
  Rows xr = rows_of(x, "x");
  if ((reinterpret_cast<uintptr_t>(x.data_ptr()) & 15u) != 0 || xr.stride % 8 != 0) {
    x = at::empty(x_in.sizes(), x_in.options());
    x.copy_(x_in);
    xr = rows_of(x, "x");
  }
  TORCH_CHECK(weight.size(1) == xr.cols && weight.scalar_type() == x.scalar_type() &&
                  out_index.scalar_type() == at::kLong && out_index.is_contiguous() && out_index.numel() == xr.rows,
              "ntb200.linear_argmax: x [..., K], weight [V, K] of one dtype, out_index int64 [rows]");
  c10::cuda::CUDAGuard guard(x.device());
  const size_t need = ntb200_linear_argmax_workspace_size(xr.rows, weight.size(0), xr.cols);
  at::Tensor ws = at::empty({static_cast<int64_t>(need > 256 ? need : 256)}, x.options().dtype(at::kByte));
  check(ntb200_linear_argmax(out_index.data_ptr<int64_t>(), x.data_ptr(), weight.data_ptr(), xr.rows,
                             weight.size(0), xr.cols, xr.stride, weight.stride(0), ws.data_ptr(),
                             static_cast<size_t>(ws.numel()), dtype_code(x), stream_of(x)),
        "linear_argmax");
}

// out = sum over ranks of their partials (see ntb200_allreduce_oneshot / _twoshot);
// peer_buffers is an int64 CUDA tensor of the world's buffer addresses.
using AllreduceFn = int (*)(void*, const void*, const uint64_t*, int64_t, int64_t, int, int, int, void*);

void allreduce_call(AllreduceFn fn, const char* name, at::Tensor& out, const at::Tensor& partial,
                    const at::Tensor& peer_buffers, int64_t capacity, int64_t rank, int64_t world_size) {
  require_cuda(out, "out");
  require_cuda(partial, "partial");
  require_cuda(peer_buffers, "peer_buffers");
  TORCH_CHECK(out.is_contiguous() && partial.is_contiguous() && out.numel() == partial.numel() &&
                  out.scalar_type() == partial.scalar_type(),
              "ntb200.", name, ": out and partial must be contiguous, of one size and dtype");
  TORCH_CHECK(peer_buffers.scalar_type() == at::kLong && peer_buffers.is_contiguous() &&
                  peer_buffers.numel() == world_size,
              "ntb200.", name, ": peer_buffers must be int64 [world_size]");
  c10::cuda::CUDAGuard guard(out.device());
  check(fn(out.data_ptr(), partial.data_ptr(), reinterpret_cast<const uint64_t*>(peer_buffers.data_ptr()),
           out.numel(), capacity, static_cast<int>(rank), static_cast<int>(world_size), dtype_code(out),
           stream_of(out)),
        name);
}

void allreduce_oneshot(at::Tensor out, const at::Tensor& partial, const at::Tensor& peer_buffers, int64_t capacity,
                       int64_t rank, int64_t world_size) {
  allreduce_call(&ntb200_allreduce_oneshot, "allreduce_oneshot", out, partial, peer_buffers, capacity, rank,
                 world_size);
}

void allreduce_twoshot(at::Tensor out, const at::Tensor& partial, const at::Tensor& peer_buffers, int64_t capacity,
                       int64_t rank, int64_t world_size) {
  allreduce_call(&ntb200_allreduce_twoshot, "allreduce_twoshot", out, partial, peer_buffers, capacity, rank,
                 world_size);
}

int64_t allreduce_buffer_size(int64_t capacity, int64_t elem_bytes, int64_t world_size) {
  return static_cast<int64_t>(
      ntb200_allreduce_buffer_size(capacity, static_cast<int>(elem_bytes), static_cast<int>(world_size)));
}

int64_t linear_workspace_size(int64_t m, int64_t n, int64_t k) {
  return static_cast<int64_t>(ntb200_linear_workspace_size(m, n, k));
}


// Top-k / top-p mask of fp32 logits [rows, vocab] in place; k (int32/int64 [rows]) or p
// (fp32 [rows]) may be absent.
void top_k_top_p(at::Tensor logits, const std::optional<at::Tensor>& k, const std::optional<at::Tensor>& p) {
  require_rows(logits, "logits");
  TORCH_CHECK(logits.scalar_type() == at::kFloat, "ntb200.top_k_top_p: logits must be float32");
  const int64_t rows = logits.size(0);
  const void* kp = nullptr;
  int kdt = NTB200_DTYPE_I64;
  if (k.has_value()) {
    require_cuda(*k, "k");
    TORCH_CHECK(k->dim() == 1 && k->is_contiguous() && k->size(0) == rows &&
                    (k->scalar_type() == at::kInt || k->scalar_type() == at::kLong),
                "ntb200.top_k_top_p: k must be contiguous int32/int64 [rows]");
    kp = k->data_ptr();
    kdt = dtype_code(*k);
  }
  const float* pp = nullptr;
  if (p.has_value()) {
    require_cuda(*p, "p");
    TORCH_CHECK(p->dim() == 1 && p->is_contiguous() && p->size(0) == rows && p->scalar_type() == at::kFloat,
                "ntb200.top_k_top_p: p must be contiguous float32 [rows]");
    pp = p->data_ptr<float>();
  }
  c10::cuda::CUDAGuard guard(logits.device());
  check(ntb200_top_k_top_p(logits.data_ptr<float>(), rows, logits.size(1), logits.stride(0), kp, kdt, pp,
                           stream_of(logits)),
        "top_k_top_p");
}

// out[b] = argmax_i probs[b, i] / q[b, i] (int64 [rows]); probs and q fp32 [rows, vocab]
void random_sample(at::Tensor out, const at::Tensor& probs, const at::Tensor& q) {
  require_rows(probs, "probs");
  require_rows(q, "q");
  require_cuda(out, "out");
  TORCH_CHECK(probs.scalar_type() == at::kFloat && q.scalar_type() == at::kFloat && q.sizes() == probs.sizes(),
              "ntb200.random_sample: probs and q must be float32 of one shape");
  TORCH_CHECK(out.scalar_type() == at::kLong && out.is_contiguous() && out.numel() == probs.size(0),
              "ntb200.random_sample: out must be contiguous int64 [rows]");
  c10::cuda::CUDAGuard guard(probs.device());
  check(ntb200_random_sample(out.data_ptr<int64_t>(), probs.data_ptr<float>(), q.data_ptr<float>(), probs.size(0),
                             probs.size(1), probs.stride(0), q.stride(0), stream_of(probs)),
        "random_sample");
}
}  // namespace

TORCH_LIBRARY(ntb200, m) {
  m.def("rms_norm(Tensor(a!) out, Tensor x, Tensor? weight, float eps) -> ()");
  m.def(
      "fused_add_rms_norm(Tensor(a!) out, Tensor(b!) residual, Tensor x, Tensor? weight, "
      "float eps) -> ()");
  m.def("gemma_rms_norm(Tensor(a!) out, Tensor x, Tensor weight, float eps) -> ()");
  m.def(
      "gemma_fused_add_rms_norm(Tensor(a!) out, Tensor(b!) residual, Tensor x, Tensor weight, "
      "float eps) -> ()");
  m.def("silu_and_mul(Tensor(a!) out, Tensor x) -> ()");
  m.def(
      "rotary_embedding_neox(Tensor positions, Tensor(a!) query, Tensor(b!)? key, "
      "Tensor cos_sin_cache, int head_size, int rotary_dim) -> ()");
  m.def(
      "reshape_and_cache(Tensor key, Tensor value, Tensor(a!) key_cache, "
      "Tensor(b!) value_cache, Tensor slot_mapping) -> ()");
  m.def(
      "rope_and_cache(Tensor positions, Tensor(a!) query, Tensor(b!) key, Tensor value, "
      "Tensor cos_sin_cache, Tensor(c!) key_cache, Tensor(d!) value_cache, Tensor slot_mapping, "
      "int head_size, int rotary_dim) -> ()");
  m.def(
      "rope_and_cache_flash_layout(Tensor positions, Tensor(a!) query, Tensor(b!) key, Tensor value, "
      "Tensor cos_sin_cache, Tensor(c!) kv_cache, Tensor slot_mapping, int head_size, int rotary_dim, "
      "int kv_dim=0) -> ()");
  m.def("embedding(Tensor(a!) out, Tensor ids, Tensor weight) -> ()");
  m.def(
      "paged_attention_decode(Tensor(a!) out, Tensor query, Tensor key_cache, "
      "Tensor value_cache, Tensor seq_lens, Tensor block_table, float scale, int max_seq_len, "
      "Tensor(b!) workspace) -> ()");
  m.def(
      "decode_workspace_size(int num_seqs, int num_q_heads, int num_kv_heads, int head_size, "
      "int block_size, int max_seq_len) -> int",
      &decode_workspace_size);
  m.def(
      "decode_flash_layout(Tensor(a!) output, Tensor query, Tensor kv_cache, Tensor seq_lens, "
      "Tensor block_table, int num_tokens, float scale, int max_seq_len, int kv_dim=0) -> ()");
  m.def(
      "store_flash_layout(Tensor key, Tensor value, Tensor(a!) kv_cache, Tensor slot_mapping, "
      "int kv_dim=0) -> ()");
  m.def("linear(Tensor(a!) out, Tensor x, Tensor weight, Tensor? bias, Tensor(b!)? workspace) -> ()");
  m.def("linear_workspace_size(int m, int n, int k) -> int", &linear_workspace_size);
  m.def("linear_silu_and_mul(Tensor(a!) out, Tensor x, Tensor weight) -> ()");
  m.def("rms_norm_linear(Tensor(a!) out, Tensor(b!)? residual_out, Tensor x, Tensor? residual, Tensor norm_weight, float eps, Tensor weight) -> ()");
  m.def("linear_argmax(Tensor(a!) out_index, Tensor x, Tensor weight) -> ()");
  m.def(
      "paged_attention_prefill(Tensor(a!) out, Tensor query, Tensor key_cache, Tensor value_cache, "
      "Tensor query_start_loc, Tensor seq_lens, Tensor block_table, int max_query_len, float scale, "
      "bool causal) -> ()");
  m.def(
      "attention_flash_layout(Tensor(a!) output, Tensor query, Tensor kv_cache, Tensor query_start_loc, "
      "Tensor seq_lens, Tensor block_table, int num_tokens, int max_query_len, int max_seq_len, float scale, "
      "int kv_dim=0) -> ()");
  m.def(
      "flash_attn_varlen(Tensor(a!) out, Tensor query, Tensor key, Tensor value, Tensor cu_seqlens_q, "
      "Tensor cu_seqlens_k, int max_query_len, float scale, bool causal) -> ()");
  m.def(
      "prefill_flash_layout(Tensor(a!) output, Tensor query, Tensor kv_cache, Tensor query_start_loc, "
      "Tensor seq_lens, Tensor block_table, int num_tokens, int max_query_len, float scale, bool causal, "
      "int kv_dim=0) -> ()");
  m.def(
      "allreduce_oneshot(Tensor(a!) out, Tensor partial, Tensor peer_buffers, int capacity, int rank, "
      "int world_size) -> ()");
  m.def(
      "allreduce_twoshot(Tensor(a!) out, Tensor partial, Tensor peer_buffers, int capacity, int rank, "
      "int world_size) -> ()");
  m.def("allreduce_buffer_size(int capacity, int elem_bytes, int world_size) -> int", &allreduce_buffer_size);
  m.def("top_k_top_p(Tensor(a!) logits, Tensor? k, Tensor? p) -> ()");
  m.def("random_sample(Tensor(a!) out, Tensor probs, Tensor q) -> ()");
}

TORCH_LIBRARY_IMPL(ntb200, CUDA, m) {
  m.impl("rms_norm", &rms_norm);
  m.impl("fused_add_rms_norm", &fused_add_rms_norm);
  m.impl("gemma_rms_norm", &gemma_rms_norm);
  m.impl("gemma_fused_add_rms_norm", &gemma_fused_add_rms_norm);
  m.impl("silu_and_mul", &silu_and_mul);
  m.impl("rotary_embedding_neox", &rotary_embedding_neox);
  m.impl("reshape_and_cache", &reshape_and_cache);
  m.impl("rope_and_cache", &rope_and_cache);
  m.impl("rope_and_cache_flash_layout", &rope_and_cache_flash_layout);
  m.impl("embedding", &embedding);
  m.impl("paged_attention_decode", &paged_attention_decode);
  m.impl("decode_flash_layout", &decode_flash_layout);
  m.impl("store_flash_layout", &store_flash_layout);
  m.impl("linear", &linear);
  m.impl("allreduce_oneshot", &allreduce_oneshot);
  m.impl("allreduce_twoshot", &allreduce_twoshot);
  m.impl("linear_silu_and_mul", &linear_silu_and_mul);
  m.impl("rms_norm_linear", &rms_norm_linear);
  m.impl("linear_argmax", &linear_argmax);
  m.impl("paged_attention_prefill", &paged_attention_prefill);
  m.impl("prefill_flash_layout", &prefill_flash_layout);
  m.impl("flash_attn_varlen", &flash_attn_varlen);
  m.impl("attention_flash_layout", &attention_flash_layout);
  m.impl("top_k_top_p", &top_k_top_p);
  m.impl("random_sample", &random_sample);
}
