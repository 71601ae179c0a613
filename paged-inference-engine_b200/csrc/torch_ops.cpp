// torch.library registration of the paged-attention C ABI (libpaged_attn_b200.so):
// the thin torch extension the Python drop-in calls.
//
//   pie_b200::paged_attention(_out)         flash_attention_forward
//                                           (kernels/flash_attention.py:139-172)
//   pie_b200::paged_attention_varlen(_out)  the same over packed query rows
//   pie_b200::write_kv                      the quantise-on-write / copy of new
//                                           K/V rows (transformer/model.py:85-122)
//   pie_b200::project_write_kv              the K/V projection with that write in
//                                           its epilogue (transformer/model.py:75-122)
//
// Each op reads pointers, sizes and element strides from its tensors, fills the
// C structs of include/paged_attn_b200.h and calls the library on the current
// CUDA stream of the tensors' device; a nonzero return code becomes a
// TORCH_CHECK failure (RuntimeError) carrying paged_attn_error_string().  The
// split-K workspace is one cached uint8 tensor per device from torch's
// allocator, grown on demand.  Meta kernels give shapes for fake tensors.
// Malformed arguments raise ValueError (TORCH_CHECK_VALUE), as the Python
// front end does; a failing library call raises RuntimeError.
//
// Pools arrive as [num_blocks, block_size, num_kv_heads, head_dim] views (the
// launcher's [block, slot, head, d] reading, kernels/flash_attention.py:158-159);
// scales as [num_blocks, num_kv_heads] (per block) or
// [num_blocks, block_size, num_kv_heads] (per token).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <mutex>
#include <optional>
#include <vector>

#include "paged_attn_b200.h"

namespace {

int pa_dtype(at::ScalarType t) {
  switch (t) {
    case at::kHalf:
      return PA_DTYPE_F16;
    case at::kBFloat16:
      return PA_DTYPE_BF16;
    case at::kChar:
      return PA_DTYPE_I8;
    case at::kFloat:
      return PA_DTYPE_F32;
    default:
      TORCH_CHECK_VALUE(false, "pie_b200: unsupported dtype ", t);
  }
  return -1;
}

void check_rc(int rc, const char* fn) {
  TORCH_CHECK(rc == PA_OK, fn, " failed (code ", rc, "): ", paged_attn_error_string());
}

void* ptr(const at::Tensor& t) { return t.data_ptr(); }
template <typename T>
T* opt_ptr(const std::optional<at::Tensor>& t) {
  return t.has_value() ? static_cast<T*>(t->data_ptr()) : nullptr;
}

void check_device(const at::Tensor& ref, const at::Tensor& t, const char* name) {
  TORCH_CHECK_VALUE(t.is_cuda() && t.device() == ref.device(), "pie_b200: ", name, " must be on ", ref.device());
}
void check_i32(const at::Tensor& ref, const at::Tensor& t, const char* name, int64_t n) {
  check_device(ref, t, name);
  TORCH_CHECK_VALUE(t.scalar_type() == at::kInt && t.dim() == 1 && t.is_contiguous(), "pie_b200: ", name,
              " must be a contiguous int32 vector");
  TORCH_CHECK_VALUE(t.numel() == n, "pie_b200: ", name, " has ", t.numel(), " entries, expected ", n);
}

pa_kv_cache_t kv_desc(const at::Tensor& K, const at::Tensor& V, const std::optional<at::Tensor>& ks,
                      const std::optional<at::Tensor>& vs) {
  TORCH_CHECK_VALUE(K.dim() == 4 && V.dim() == 4 && K.sizes() == V.sizes() && K.scalar_type() == V.scalar_type(),
              "pie_b200: K and V pools must be 4-D [num_blocks, block_size, num_kv_heads, head_dim] and alike");
  check_device(K, V, "V");
  pa_kv_cache_t kv{};
  kv.k = ptr(K);
  kv.v = ptr(V);
  kv.dtype = pa_dtype(K.scalar_type());
  kv.num_blocks = static_cast<int32_t>(K.size(0));
  kv.block_size = static_cast<int32_t>(K.size(1));
  kv.num_kv_heads = static_cast<int32_t>(K.size(2));
  kv.head_dim = static_cast<int32_t>(K.size(3));
  TORCH_CHECK_VALUE(K.stride(3) == 1 && V.stride(3) == 1, "pie_b200: K/V pools need a contiguous head_dim");
  kv.k_stride_block = K.stride(0);
  kv.k_stride_slot = K.stride(1);
  kv.k_stride_head = K.stride(2);
  kv.v_stride_block = V.stride(0);
  kv.v_stride_slot = V.stride(1);
  kv.v_stride_head = V.stride(2);
  kv.scale_dtype = PA_DTYPE_F16;
  if (kv.dtype == PA_DTYPE_I8) {
    TORCH_CHECK_VALUE(ks.has_value() && vs.has_value(), "pie_b200: an int8 KV pool needs k_scale and v_scale");
    const at::Tensor* sc[2] = {&*ks, &*vs};
    int64_t st[2][3];
    for (int i = 0; i < 2; ++i) {
      const at::Tensor& s = *sc[i];
      check_device(K, s, i ? "v_scale" : "k_scale");
      if (s.dim() == 2) {
        TORCH_CHECK_VALUE(s.size(0) == K.size(0) && s.size(1) == K.size(2), "pie_b200: per-block scales must be [",
                    K.size(0), ", ", K.size(2), "]");
        st[i][0] = s.stride(0);
        st[i][1] = 0;
        st[i][2] = s.stride(1);
      } else {
        TORCH_CHECK_VALUE(s.dim() == 3 && s.size(0) == K.size(0) && s.size(1) == K.size(1) && s.size(2) == K.size(2),
                    "pie_b200: per-token scales must be [", K.size(0), ", ", K.size(1), ", ", K.size(2), "]");
        st[i][0] = s.stride(0);
        st[i][1] = s.stride(1);
        st[i][2] = s.stride(2);
      }
    }
    TORCH_CHECK_VALUE(ks->scalar_type() == vs->scalar_type() &&
                    (ks->scalar_type() == at::kHalf || ks->scalar_type() == at::kFloat),
                "pie_b200: k_scale / v_scale must share a float16 or float32 dtype");
    kv.scale_dtype = pa_dtype(ks->scalar_type());
    kv.k_scale = ptr(*ks);
    kv.v_scale = ptr(*vs);
    kv.ks_stride_block = st[0][0];
    kv.ks_stride_slot = st[0][1];
    kv.ks_stride_head = st[0][2];
    kv.vs_stride_block = st[1][0];
    kv.vs_stride_slot = st[1][1];
    kv.vs_stride_head = st[1][2];
  }
  return kv;
}

pa_paging_t paging(const at::Tensor& ref, const at::Tensor& block_table, const at::Tensor& num_blocks,
                   const at::Tensor& q_len, const at::Tensor& kv_len) {
  check_device(ref, block_table, "block_table");
  TORCH_CHECK_VALUE(block_table.scalar_type() == at::kInt && block_table.dim() == 2,
              "pie_b200: block_table must be int32 [num_seqs, max_blocks]");
  const int64_t B = block_table.size(0);
  check_i32(ref, num_blocks, "num_blocks_per_seq", B);
  check_i32(ref, q_len, "q_len_per_seq", B);
  check_i32(ref, kv_len, "kv_len_per_seq", B);
  pa_paging_t pg{};
  pg.block_table = static_cast<const int32_t*>(block_table.data_ptr());
  pg.bt_stride_seq = block_table.stride(0);
  pg.bt_stride_col = block_table.stride(1);
  pg.bt_cols = static_cast<int32_t>(block_table.size(1));
  pg.num_seqs = static_cast<int32_t>(B);
  pg.num_blocks_per_seq = static_cast<const int32_t*>(num_blocks.data_ptr());
  pg.q_len_per_seq = static_cast<const int32_t*>(q_len.data_ptr());
  pg.kv_len_per_seq = static_cast<const int32_t*>(kv_len.data_ptr());
  return pg;
}

// One cached workspace per device (256-byte aligned by torch's allocator).
at::Tensor workspace(const at::Device& dev, size_t bytes) {
  static std::mutex mu;
  static std::vector<at::Tensor> cache;
  std::lock_guard<std::mutex> lk(mu);
  const size_t i = static_cast<size_t>(dev.index());
  if (cache.size() <= i) cache.resize(i + 1);
  at::Tensor& ws = cache[i];
  if (!ws.defined() || static_cast<size_t>(ws.numel()) < bytes) {
    const int64_t n = static_cast<int64_t>(bytes > (1u << 20) ? bytes : (1u << 20));
    ws = at::empty({n}, at::TensorOptions().dtype(at::kByte).device(dev));
  }
  return ws;
}

pa_attn_io_t io_desc(const at::Tensor& Q, const at::Tensor& O, const at::Tensor& L, bool ragged, int64_t max_q_len,
                     bool causal_top_left, double softmax_scale) {
  pa_attn_io_t io{};
  io.q = ptr(Q);
  io.q_dtype = pa_dtype(Q.scalar_type());
  io.num_q_heads = static_cast<int32_t>(Q.size(1));
  io.max_q_len = static_cast<int32_t>(max_q_len);
  io.causal_top_left = causal_top_left ? 1 : 0;
  if (ragged) {  // [T, Hq, D] / [T, Hq]
    io.q_stride_seq = 0;
    io.q_stride_head = Q.stride(1);
    io.q_stride_row = Q.stride(0);
    io.o_stride_seq = 0;
    io.o_stride_head = O.stride(1);
    io.o_stride_row = O.stride(0);
    io.l_stride_seq = 0;
    io.l_stride_head = L.stride(1);
    io.l_stride_row = L.stride(0);
  } else {  // [B, Hq, maxq, D] / [B, Hq, maxq]
    io.q_stride_seq = Q.stride(0);
    io.q_stride_head = Q.stride(1);
    io.q_stride_row = Q.stride(2);
    io.o_stride_seq = O.stride(0);
    io.o_stride_head = O.stride(1);
    io.o_stride_row = O.stride(2);
    io.l_stride_seq = L.stride(0);
    io.l_stride_head = L.stride(1);
    io.l_stride_row = L.stride(2);
  }
  io.o = ptr(O);
  io.lse = ptr(L);
  io.softmax_scale = static_cast<float>(softmax_scale);
  return io;
}

void check_q(const at::Tensor& Q, int64_t dims) {
  TORCH_CHECK_VALUE(Q.is_cuda() && Q.dim() == dims, "pie_b200: Q must be a ", dims, "-D CUDA tensor");
  TORCH_CHECK_VALUE(Q.scalar_type() == at::kHalf || Q.scalar_type() == at::kBFloat16, "pie_b200: Q must be fp16 or bf16");
  TORCH_CHECK_VALUE(Q.stride(dims - 1) == 1, "pie_b200: Q needs a contiguous head_dim");
}

void check_out(const at::Tensor& Q, const at::Tensor& O, const at::Tensor& L) {
  check_device(Q, O, "out");
  check_device(Q, L, "lse");
  TORCH_CHECK_VALUE(O.scalar_type() == at::kHalf && O.sizes() == Q.sizes(), "pie_b200: out must be float16 shaped like Q");
  TORCH_CHECK_VALUE(L.scalar_type() == at::kHalf && L.sizes() == Q.sizes().slice(0, Q.dim() - 1),
              "pie_b200: lse must be float16 shaped like Q without head_dim");
}

// mode: 0 = choose (paged_attn_forward), 1 = split-K decode, 2 = prefill kernel
void paged_attention_out(const at::Tensor& Q, const at::Tensor& K, const at::Tensor& V, const at::Tensor& q_len,
                         const at::Tensor& block_table, const at::Tensor& num_blocks, const at::Tensor& kv_len,
                         const std::optional<at::Tensor>& k_scale, const std::optional<at::Tensor>& v_scale,
                         bool causal_top_left, double softmax_scale, int64_t mode,
                         const std::optional<at::Tensor>& status, at::Tensor& out, at::Tensor& lse) {
  check_q(Q, 4);
  check_out(Q, out, lse);
  check_device(Q, K, "K");
  TORCH_CHECK_VALUE(block_table.size(0) == Q.size(0), "pie_b200: block_table has ", block_table.size(0), " rows for ",
              Q.size(0), " sequences");
  const c10::cuda::CUDAGuard guard(Q.device());
  pa_kv_cache_t kv = kv_desc(K, V, k_scale, v_scale);
  pa_paging_t pg = paging(Q, block_table, num_blocks, q_len, kv_len);
  pa_attn_io_t io = io_desc(Q, out, lse, false, Q.size(2), causal_top_left, softmax_scale);
  void* stream = c10::cuda::getCurrentCUDAStream(Q.device().index()).stream();
  int32_t* st = opt_ptr<int32_t>(status);
  if (mode == 2) {
    check_rc(paged_attn_prefill(&io, &kv, &pg, st, stream), "paged_attn_prefill");
    return;
  }
  size_t bytes = 0;
  check_rc(paged_attn_workspace_size(&io, &kv, &pg, &bytes), "paged_attn_workspace_size");
  at::Tensor ws;
  if (bytes) ws = workspace(Q.device(), bytes);
  void* wp = bytes ? ws.data_ptr() : nullptr;
  const size_t wb = bytes ? static_cast<size_t>(ws.numel()) : 0;
  if (mode == 1) check_rc(paged_attn_decode(&io, &kv, &pg, wp, wb, st, stream), "paged_attn_decode");
  else check_rc(paged_attn_forward(&io, &kv, &pg, wp, wb, st, stream), "paged_attn_forward");
}

std::tuple<at::Tensor, at::Tensor> paged_attention(const at::Tensor& Q, const at::Tensor& K, const at::Tensor& V,
                                                   const at::Tensor& q_len, const at::Tensor& block_table,
                                                   const at::Tensor& num_blocks, const at::Tensor& kv_len,
                                                   const std::optional<at::Tensor>& k_scale,
                                                   const std::optional<at::Tensor>& v_scale, bool causal_top_left,
                                                   double softmax_scale, int64_t mode,
                                                   const std::optional<at::Tensor>& status) {
  at::Tensor out = at::empty(Q.sizes(), Q.options().dtype(at::kHalf));
  at::Tensor lse = at::empty(Q.sizes().slice(0, 3), Q.options().dtype(at::kHalf));
  paged_attention_out(Q, K, V, q_len, block_table, num_blocks, kv_len, k_scale, v_scale, causal_top_left,
                      softmax_scale, mode, status, out, lse);
  return {out, lse};
}

void paged_attention_varlen_out(const at::Tensor& Q, const at::Tensor& q_start, const at::Tensor& q_len,
                                int64_t max_q_len, const at::Tensor& K, const at::Tensor& V,
                                const at::Tensor& block_table, const at::Tensor& num_blocks, const at::Tensor& kv_len,
                                const std::optional<at::Tensor>& k_scale, const std::optional<at::Tensor>& v_scale,
                                bool causal_top_left, double softmax_scale, const std::optional<at::Tensor>& status,
                                at::Tensor& out, at::Tensor& lse) {
  check_q(Q, 3);
  check_out(Q, out, lse);
  check_device(Q, K, "K");
  const c10::cuda::CUDAGuard guard(Q.device());
  pa_kv_cache_t kv = kv_desc(K, V, k_scale, v_scale);
  pa_paging_t pg = paging(Q, block_table, num_blocks, q_len, kv_len);
  check_i32(Q, q_start, "q_start", block_table.size(0));
  pa_attn_io_t io = io_desc(Q, out, lse, true, max_q_len, causal_top_left, softmax_scale);
  void* stream = c10::cuda::getCurrentCUDAStream(Q.device().index()).stream();
  size_t bytes = 0;
  check_rc(paged_attn_workspace_size(&io, &kv, &pg, &bytes), "paged_attn_workspace_size");
  at::Tensor ws;
  if (bytes) ws = workspace(Q.device(), bytes);
  check_rc(paged_attn_varlen(&io, &kv, &pg, static_cast<const int32_t*>(q_start.data_ptr()),
                             static_cast<int32_t>(Q.size(0)), bytes ? ws.data_ptr() : nullptr,
                             bytes ? static_cast<size_t>(ws.numel()) : 0, opt_ptr<int32_t>(status), stream),
           "paged_attn_varlen");
}

std::tuple<at::Tensor, at::Tensor> paged_attention_varlen(
    const at::Tensor& Q, const at::Tensor& q_start, const at::Tensor& q_len, int64_t max_q_len, const at::Tensor& K,
    const at::Tensor& V, const at::Tensor& block_table, const at::Tensor& num_blocks, const at::Tensor& kv_len,
    const std::optional<at::Tensor>& k_scale, const std::optional<at::Tensor>& v_scale, bool causal_top_left,
    double softmax_scale, const std::optional<at::Tensor>& status) {
  at::Tensor out = at::empty(Q.sizes(), Q.options().dtype(at::kHalf));
  at::Tensor lse = at::empty(Q.sizes().slice(0, 2), Q.options().dtype(at::kHalf));
  paged_attention_varlen_out(Q, q_start, q_len, max_q_len, K, V, block_table, num_blocks, kv_len, k_scale, v_scale,
                             causal_top_left, softmax_scale, status, out, lse);
  return {out, lse};
}

void write_kv(const at::Tensor& k_new, const at::Tensor& v_new, const at::Tensor& block_table,
              const at::Tensor& seq_index, const at::Tensor& positions, at::Tensor& k_cache, at::Tensor& v_cache,
              const std::optional<at::Tensor>& k_scale, const std::optional<at::Tensor>& v_scale,
              const std::optional<at::Tensor>& status) {
  TORCH_CHECK_VALUE(k_new.dim() == 3 && v_new.sizes() == k_new.sizes() && v_new.scalar_type() == k_new.scalar_type(),
              "pie_b200: k_new / v_new must be [num_tokens, num_kv_heads, head_dim] of equal shape and dtype");
  TORCH_CHECK_VALUE(k_new.stride(2) == 1 && v_new.stride(2) == 1, "pie_b200: new rows need a contiguous head_dim");
  check_device(k_cache, k_new, "k_new");
  check_device(k_cache, v_new, "v_new");
  check_device(k_cache, block_table, "block_table");
  TORCH_CHECK_VALUE(block_table.scalar_type() == at::kInt && block_table.dim() == 2, "pie_b200: block_table must be int32 2-D");
  const int64_t T = k_new.size(0);
  check_i32(k_cache, seq_index, "seq_index", T);
  check_i32(k_cache, positions, "positions", T);
  const c10::cuda::CUDAGuard guard(k_cache.device());
  pa_kv_cache_t kv = kv_desc(k_cache, v_cache, k_scale, v_scale);
  pa_paging_t pg{};
  pg.block_table = static_cast<const int32_t*>(block_table.data_ptr());
  pg.bt_stride_seq = block_table.stride(0);
  pg.bt_stride_col = block_table.stride(1);
  pg.bt_cols = static_cast<int32_t>(block_table.size(1));
  pg.num_seqs = static_cast<int32_t>(block_table.size(0));
  pa_kv_new_t nw{};
  nw.k_new = ptr(k_new);
  nw.v_new = ptr(v_new);
  nw.dtype = pa_dtype(k_new.scalar_type());
  nw.num_tokens = static_cast<int32_t>(T);
  nw.k_stride_token = k_new.stride(0);
  nw.k_stride_head = k_new.stride(1);
  nw.v_stride_token = v_new.stride(0);
  nw.v_stride_head = v_new.stride(1);
  nw.seq_index = static_cast<const int32_t*>(seq_index.data_ptr());
  nw.positions = static_cast<const int32_t*>(positions.data_ptr());
  void* stream = c10::cuda::getCurrentCUDAStream(k_cache.device().index()).stream();
  int32_t* st = opt_ptr<int32_t>(status);
  if (kv.dtype == PA_DTYPE_I8) check_rc(kv_write_quant(&nw, &kv, &pg, st, stream), "kv_write_quant");
  else check_rc(kv_write_copy(&nw, &kv, &pg, st, stream), "kv_write_copy");
}

void project_write_kv(const at::Tensor& x, const at::Tensor& w, const std::optional<at::Tensor>& bias,
                      const at::Tensor& block_table, const at::Tensor& seq_index, const at::Tensor& positions,
                      at::Tensor& k_cache, at::Tensor& v_cache, const std::optional<at::Tensor>& k_scale,
                      const std::optional<at::Tensor>& v_scale, const std::optional<at::Tensor>& status) {
  TORCH_CHECK_VALUE(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1) && x.scalar_type() == w.scalar_type(),
                    "pie_b200: x [T, d_model] and w [2 * Hkv * D, d_model] must share d_model and dtype");
  TORCH_CHECK_VALUE(x.stride(1) == 1 && w.stride(1) == 1, "pie_b200: x / w need contiguous rows");
  TORCH_CHECK_VALUE(w.size(0) == 2 * k_cache.size(2) * k_cache.size(3),
                    "pie_b200: w must hold 2 * num_kv_heads * head_dim rows (W_k then W_v)");
  check_device(k_cache, x, "x");
  check_device(k_cache, w, "w");
  check_device(k_cache, block_table, "block_table");
  TORCH_CHECK_VALUE(block_table.scalar_type() == at::kInt && block_table.dim() == 2,
                    "pie_b200: block_table must be int32 2-D");
  const int64_t T = x.size(0);
  check_i32(k_cache, seq_index, "seq_index", T);
  check_i32(k_cache, positions, "positions", T);
  if (bias.has_value()) {
    check_device(k_cache, *bias, "bias");
    TORCH_CHECK_VALUE(bias->scalar_type() == at::kFloat && bias->is_contiguous() && bias->numel() == w.size(0),
                      "pie_b200: bias must be a contiguous float32 vector of w's rows");
  }
  const c10::cuda::CUDAGuard guard(k_cache.device());
  pa_kv_cache_t kv = kv_desc(k_cache, v_cache, k_scale, v_scale);
  pa_paging_t pg{};
  pg.block_table = static_cast<const int32_t*>(block_table.data_ptr());
  pg.bt_stride_seq = block_table.stride(0);
  pg.bt_stride_col = block_table.stride(1);
  pg.bt_cols = static_cast<int32_t>(block_table.size(1));
  pg.num_seqs = static_cast<int32_t>(block_table.size(0));
  pa_kv_proj_t pj{};
  pj.x = ptr(x);
  pj.w = ptr(w);
  pj.bias = bias.has_value() ? static_cast<const float*>(bias->data_ptr()) : nullptr;
  pj.x_stride = x.stride(0);
  pj.w_stride = w.stride(0);
  pj.dtype = pa_dtype(x.scalar_type());
  pj.num_tokens = static_cast<int32_t>(T);
  pj.d_model = static_cast<int32_t>(x.size(1));
  pj.seq_index = static_cast<const int32_t*>(seq_index.data_ptr());
  pj.positions = static_cast<const int32_t*>(positions.data_ptr());
  void* stream = c10::cuda::getCurrentCUDAStream(k_cache.device().index()).stream();
  check_rc(kv_project_write(&pj, &kv, &pg, opt_ptr<int32_t>(status), stream), "kv_project_write");
}

// ---- shapes only (fake / meta tensors) ------------------------------------
std::tuple<at::Tensor, at::Tensor> paged_attention_meta(const at::Tensor& Q, const at::Tensor&, const at::Tensor&,
                                                        const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                                        const at::Tensor&, const std::optional<at::Tensor>&,
                                                        const std::optional<at::Tensor>&, bool, double, int64_t,
                                                        const std::optional<at::Tensor>&) {
  return {at::empty(Q.sizes(), Q.options().dtype(at::kHalf)),
          at::empty(Q.sizes().slice(0, 3), Q.options().dtype(at::kHalf))};
}

std::tuple<at::Tensor, at::Tensor> paged_attention_varlen_meta(
    const at::Tensor& Q, const at::Tensor&, const at::Tensor&, int64_t, const at::Tensor&, const at::Tensor&,
    const at::Tensor&, const at::Tensor&, const at::Tensor&, const std::optional<at::Tensor>&,
    const std::optional<at::Tensor>&, bool, double, const std::optional<at::Tensor>&) {
  return {at::empty(Q.sizes(), Q.options().dtype(at::kHalf)),
          at::empty(Q.sizes().slice(0, 2), Q.options().dtype(at::kHalf))};
}

}  // namespace

TORCH_LIBRARY(pie_b200, m) {
  m.def("paged_attention(Tensor Q, Tensor K, Tensor V, Tensor q_len, Tensor block_table, Tensor num_blocks, "
        "Tensor kv_len, Tensor? k_scale, Tensor? v_scale, bool causal_top_left, float softmax_scale, int mode, "
        "Tensor(s!)? status) -> (Tensor, Tensor)");
  m.def("paged_attention_out(Tensor Q, Tensor K, Tensor V, Tensor q_len, Tensor block_table, Tensor num_blocks, "
        "Tensor kv_len, Tensor? k_scale, Tensor? v_scale, bool causal_top_left, float softmax_scale, int mode, "
        "Tensor(s!)? status, Tensor(a!) out, Tensor(b!) lse) -> ()");
  m.def("paged_attention_varlen(Tensor Q, Tensor q_start, Tensor q_len, int max_q_len, Tensor K, Tensor V, "
        "Tensor block_table, Tensor num_blocks, Tensor kv_len, Tensor? k_scale, Tensor? v_scale, "
        "bool causal_top_left, float softmax_scale, Tensor(s!)? status) -> (Tensor, Tensor)");
  m.def("paged_attention_varlen_out(Tensor Q, Tensor q_start, Tensor q_len, int max_q_len, Tensor K, Tensor V, "
        "Tensor block_table, Tensor num_blocks, Tensor kv_len, Tensor? k_scale, Tensor? v_scale, "
        "bool causal_top_left, float softmax_scale, Tensor(s!)? status, Tensor(a!) out, Tensor(b!) lse) -> ()");
  m.def("write_kv(Tensor k_new, Tensor v_new, Tensor block_table, Tensor seq_index, Tensor positions, "
        "Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor(c!)? k_scale, Tensor(d!)? v_scale, Tensor(s!)? status) -> ()");
  m.def("project_write_kv(Tensor x, Tensor w, Tensor? bias, Tensor block_table, Tensor seq_index, Tensor positions, "
        "Tensor(a!) k_cache, Tensor(b!) v_cache, Tensor(c!)? k_scale, Tensor(d!)? v_scale, Tensor(s!)? status) -> ()");
}

TORCH_LIBRARY_IMPL(pie_b200, CUDA, m) {
  m.impl("paged_attention", &paged_attention);
  m.impl("paged_attention_out", &paged_attention_out);
  m.impl("paged_attention_varlen", &paged_attention_varlen);
  m.impl("paged_attention_varlen_out", &paged_attention_varlen_out);
  m.impl("write_kv", &write_kv);
  m.impl("project_write_kv", &project_write_kv);
}

TORCH_LIBRARY_IMPL(pie_b200, Meta, m) {
  m.impl("paged_attention", &paged_attention_meta);
  m.impl("paged_attention_varlen", &paged_attention_varlen_meta);
}
