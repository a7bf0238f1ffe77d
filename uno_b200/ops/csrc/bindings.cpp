// Python bindings of the uno_b200 sm_100a kernels (module ``uno_b200._C``).
#include <torch/extension.h>

#include "uno_ops.h"

namespace uno {

// Forward declarations (defined in the .cu files).
void rmsnorm_launch(const at::Tensor& x, const c10::optional<at::Tensor>& residual, const at::Tensor& w,
                    at::Tensor& y, double eps, int groups);
void embedding_launch(const at::Tensor& ids, const at::Tensor& table, at::Tensor& out, int64_t start);
void silu_mul_launch(const at::Tensor& x, at::Tensor& out);
void qk_norm_rope_store_launch(const at::Tensor& qkv, at::Tensor& q_out, at::Tensor& k_cache, at::Tensor& v_cache,
                               const at::Tensor& slots, const at::Tensor& positions, const at::Tensor& cos_sin,
                               const c10::optional<at::Tensor>& qw, const c10::optional<at::Tensor>& kw, double eps,
                               int hq, int hkv, int D, int page);
void copy_tree_kv_launch(at::Tensor& cache, const at::Tensor& tables, const at::Tensor& src, const at::Tensor& dst,
                         int page);
void argmax_launch(const at::Tensor& x, at::Tensor& out);
void gumbel_sample_launch(const at::Tensor& x, at::Tensor& out, double inv_temp, int64_t seed, int64_t offset);
void fused_verify_launch(const at::Tensor& clean, const at::Tensor& draft, const at::Tensor& spec, double inv_temp,
                         int64_t seed, int64_t offset, at::Tensor& accepted, at::Tensor& corr);
void topk_lse_launch(const at::Tensor& x, int K, double inv_temp, at::Tensor& ids, at::Tensor& lp);
void filtered_sample_launch(const at::Tensor& x, double inv_temp, int64_t k, double top_p, int64_t seed,
                            int64_t offset, at::Tensor& tokens, at::Tensor& params);
void filtered_verify_launch(const at::Tensor& clean, const at::Tensor& draft, const at::Tensor& dparams,
                            const at::Tensor& spec, double inv_temp, int64_t k, double top_p, int64_t seed,
                            int64_t offset, at::Tensor& accepted, at::Tensor& corr);
void build_tree_launch(const at::Tensor& roots, const at::Tensor& ids, const at::Tensor& lp, int Qn, at::Tensor& tok,
                       at::Tensor& par, at::Tensor& dep, at::Tensor& mass, at::Tensor& count);
void reduce_norm_gather_launch(const std::vector<int64_t>& peers, int64_t rank, int64_t T, int64_t H,
                               int64_t recv_off, int64_t gather_off, at::Tensor& residual, bool add_residual,
                               const at::Tensor& weight, int64_t groups, double eps, bool wait_all);
void embedding_scatter_launch(const std::vector<int64_t>& peers, int64_t rank, const at::Tensor& ids,
                              const at::Tensor& table, int64_t start, int64_t recv_off, int64_t gather_off);
void vp_sample_launch(const at::Tensor& x, at::Tensor& out, double inv_temp, bool greedy, int64_t seed,
                      int64_t offset, const std::vector<int64_t>& regions, int64_t rank, int64_t max_rows,
                      int64_t vstart);
void vp_verify_launch(const at::Tensor& clean, const at::Tensor& draft, const at::Tensor& spec, double inv_temp,
                      int64_t seed, int64_t offset, at::Tensor& accepted, at::Tensor& corr,
                      const std::vector<int64_t>& regions, int64_t rank, int64_t max_rows, int64_t vstart);
int64_t vp_region_bytes(int64_t max_rows);
void fused_adamw_launch(const std::vector<int64_t>& ws, int64_t rank, int64_t params_off, int64_t grads_off,
                        int64_t ctl_off, int64_t n, at::Tensor& m, at::Tensor& v, at::Tensor& scratch,
                        at::Tensor& norm_out, double lr, double beta1, double beta2, double eps, double weight_decay,
                        double max_norm, int64_t step);
int64_t opt_ctl_bytes();
void rmsnorm_fwd_train(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, at::Tensor& rstd, double eps,
                       int64_t groups);
void rmsnorm_bwd_train(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w, const at::Tensor& rstd,
                       at::Tensor& dx, int64_t groups);
void silu_mul_fwd(const at::Tensor& gu, at::Tensor& a);
void silu_mul_bwd(const at::Tensor& da, const at::Tensor& gu, at::Tensor& dgu);
void qk_norm_rope_fwd(const at::Tensor& x, c10::optional<at::Tensor> w, double eps, const at::Tensor& pos,
                      const at::Tensor& cos_sin, at::Tensor& out, at::Tensor& rstd);
void qk_norm_rope_bwd(const at::Tensor& dy, const at::Tensor& x, c10::optional<at::Tensor> w, const at::Tensor& pos,
                      const at::Tensor& cos_sin, const at::Tensor& rstd, at::Tensor& dx);
void train_attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& seg,
                    const at::Tensor& pos, const at::Tensor& noisy, const at::Tensor& tiles, int64_t block,
                    double scale, at::Tensor& out, at::Tensor& lse);
void train_attn_bwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& seg,
                    const at::Tensor& pos, const at::Tensor& noisy, const at::Tensor& tiles, int64_t block,
                    double scale, const at::Tensor& out, const at::Tensor& dout, const at::Tensor& lse,
                    at::Tensor& delta, at::Tensor& dq, at::Tensor& dk, at::Tensor& dv);
void uno_loss_launch(const at::Tensor& s, const at::Tensor& t, const at::Tensor& target, bool teacher_ce,
                     const at::Tensor& ce_w, const at::Tensor& dist_w, double tv_w, double kl_w, double ce_weight,
                     at::Tensor& row_loss, at::Tensor& grad);
std::vector<int64_t> symm_alloc(int64_t nbytes);
int64_t symm_open(const std::vector<int64_t>& handle_bytes);
void symm_close(int64_t ptr, bool owned);
void walk_tree_launch(const at::Tensor& tok, const at::Tensor& par, const at::Tensor& tgt, int max_depth, int64_t pad,
                      at::Tensor& committed, at::Tensor& accepted, at::Tensor& lengths);

static DeviceScratch g_scratch[64];

DeviceScratch& device_scratch() {
  int dev;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  DeviceScratch& s = g_scratch[dev];
  if (s.err == nullptr) {
    s.max_counters = 16384;
    s.ws_floats = (size_t)16 << 20;  // 64 MB of fp32 split-K partials
    C10_CUDA_CHECK(cudaMalloc(&s.err, sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(s.err, 0, sizeof(int)));
    C10_CUDA_CHECK(cudaMalloc(&s.counters, s.max_counters * sizeof(int)));
    C10_CUDA_CHECK(cudaMemset(s.counters, 0, s.max_counters * sizeof(int)));
    C10_CUDA_CHECK(cudaMalloc(&s.ws, s.ws_floats * sizeof(float)));
  }
  return s;
}

static int64_t read_error_flag(bool reset) {
  int* f = device_error_flag();
  int h = 0;
  C10_CUDA_CHECK(cudaMemcpy(&h, f, sizeof(int), cudaMemcpyDeviceToHost));
  if (reset) C10_CUDA_CHECK(cudaMemset(f, 0, sizeof(int)));
  return h;
}

// Every pointer handed to a kernel must live on the current CUDA device: a
// host or foreign-device tensor is rejected here instead of faulting on the GPU.

template <typename T>
static T* ptr_or_null(const c10::optional<at::Tensor>& t, const char* what = "tensor argument") {
  if (!(t.has_value() && t->defined())) return nullptr;
  check_dev(*t, what);
  return reinterpret_cast<T*>(t->data_ptr());
}

// Generic GEMM entry: out = epilogue(a[M,K] . b[N,K]^T [+ a2[M,K2] . b2[N,K2]^T]).
static void gemm(const at::Tensor& a, const at::Tensor& b, int64_t epi, int64_t bn, c10::optional<at::Tensor> c,
                 c10::optional<at::Tensor> r, c10::optional<at::Tensor> a2, c10::optional<at::Tensor> b2,
                 double lora_scale, c10::optional<at::Tensor> row_mask, c10::optional<at::Tensor> q_out,
                 c10::optional<at::Tensor> k_cache, c10::optional<at::Tensor> v_cache,
                 c10::optional<at::Tensor> slots, c10::optional<at::Tensor> positions,
                 c10::optional<at::Tensor> cos_sin, c10::optional<at::Tensor> q_norm_w,
                 c10::optional<at::Tensor> k_norm_w, double eps, int64_t hq, int64_t hkv, int64_t page,
                 int64_t max_ctas, int64_t splits, std::vector<int64_t> rs_peers, int64_t rs_rank,
                 int64_t rs_recv_off, int64_t ag_base, int64_t ag_R) {
  check_dev(a, "gemm A");
  check_dev(b, "gemm B");
  UNO_CHECK_BF16(a);
  UNO_CHECK_BF16(b);
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(1), "gemm: shape mismatch");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1, "gemm operands must be K-contiguous");
  GemmParams p{};
  p.M = a.size(0);
  p.N = b.size(0);
  p.K = a.size(1);
  if (p.M == 0) return;
  const bool ext = a2.has_value() && a2->defined();
  if (ext) {
    check_dev(*a2, "gemm A2");
    TORCH_CHECK(b2.has_value() && b2->defined(), "K extension needs both A2 and B2");
    check_dev(*b2, "gemm B2");
    UNO_CHECK_BF16(*a2);
    UNO_CHECK_BF16(*b2);
    TORCH_CHECK(a2->dim() == 2 && b2->dim() == 2 && a2->size(0) == p.M && b2->size(0) == p.N &&
                    a2->size(1) == b2->size(1) && a2->stride(1) == 1 && b2->stride(1) == 1,
                "gemm: K-extension shape mismatch");
    p.K2 = a2->size(1);
  }
  p.C = ptr_or_null<__nv_bfloat16>(c);
  p.ldc = c.has_value() ? c->stride(0) : 0;
  p.R = ptr_or_null<const __nv_bfloat16>(r);
  p.ldr = r.has_value() ? r->stride(0) : 0;
  TORCH_CHECK(p.ldc % 8 == 0 && p.ldr % 8 == 0, "output strides must be multiples of 8");
  p.lora_scale = lora_scale;
  p.row_mask = ptr_or_null<const float>(row_mask);
  p.q_out = ptr_or_null<__nv_bfloat16>(q_out);
  p.k_cache = ptr_or_null<__nv_bfloat16>(k_cache);
  p.v_cache = ptr_or_null<__nv_bfloat16>(v_cache);
  p.slots = ptr_or_null<const int64_t>(slots);
  p.positions = ptr_or_null<const int64_t>(positions);
  p.cos_sin = ptr_or_null<const float>(cos_sin);
  p.q_norm_w = ptr_or_null<const __nv_bfloat16>(q_norm_w);
  p.k_norm_w = ptr_or_null<const __nv_bfloat16>(k_norm_w);
  p.eps = eps;
  p.num_q_heads = hq;
  p.num_kv_heads = hkv;
  p.page_size = page;
  if (epi == 5) TORCH_CHECK(p.q_out && p.slots && p.positions && p.cos_sin, "QK-RoPE epilogue arguments missing");
  if (epi == 2) TORCH_CHECK(p.row_mask != nullptr, "ROWSCALE needs row_mask");
  if (epi == 3) TORCH_CHECK(p.R != nullptr, "ADD needs a residual");
  if (!rs_peers.empty()) {
    TORCH_CHECK(epi == 0 && rs_peers.size() <= 8, "reduce-scatter send needs the STORE epilogue and <= 8 ranks");
    const int tp = (int)rs_peers.size();
    for (int j = 0; j < tp; ++j) p.rs_peers[j] = reinterpret_cast<uint8_t*>(rs_peers[j]);
    p.rs_enable = 1;
    p.rs_rank = (int)rs_rank;
    p.rs_R = (p.M + tp - 1) / tp;
    p.rs_recv_off = (int)rs_recv_off;
    TORCH_CHECK((p.N * 2) % 16 == 0, "row width must be 16-byte aligned");
  } else if (epi != 5) {
    TORCH_CHECK(p.C != nullptr, "output tensor missing");
  }
  if (ag_base) {
    TORCH_CHECK(ag_R > 0, "all-gathered operand needs rows per rank");
    p.ag_base = reinterpret_cast<const uint8_t*>(ag_base);
    p.ag_R = (int)ag_R;
  }
  DeviceScratch& scratch = device_scratch();
  p.err = scratch.err;
  int tile = 0;
  pick_tile(p.M, p.N, p.K + p.K2, (int)epi, (int)bn, (int)splits, &tile, &p.splits);
  const int64_t tiles = splitk_tiles(p.M, p.N, tile);
  if (p.splits > 1 &&
      (tiles > scratch.max_counters || (size_t)tiles * p.splits * 128 * tile > scratch.ws_floats))
    p.splits = 1;
  p.ws = scratch.ws;
  p.counters = scratch.counters;
  gemm_dispatch((int)epi, tile, a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0),
                ext ? a2->data_ptr() : nullptr, ext ? a2->stride(0) : 0, ext ? b2->data_ptr() : nullptr,
                ext ? b2->stride(0) : 0, p, cur_stream(), (int)max_ctas);
}

// c32[M, N] += a^T b with a [K, M], b [K, N] bf16 (row-major, reduced over rows) and c32 fp32.
static void gemm_wgrad(const at::Tensor& a, const at::Tensor& b, at::Tensor& c32, int64_t splits) {
  check_dev(a, "wgrad A");
  check_dev(b, "wgrad B");
  check_dev(c32, "wgrad C");
  UNO_CHECK_BF16(a);
  UNO_CHECK_BF16(b);
  TORCH_CHECK(c32.scalar_type() == at::kFloat && c32.dim() == 2 && c32.stride(1) == 1, "wgrad C must be fp32 rows");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(0) == b.size(0), "wgrad: operands must share their rows");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1, "wgrad operands must be contiguous along their columns");
  TORCH_CHECK(c32.size(0) == a.size(1) && c32.size(1) == b.size(1), "wgrad: C must be [a.cols, b.cols]");
  TORCH_CHECK(c32.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(c32.data_ptr()) % 16 == 0,
              "wgrad C rows must be 16-byte aligned");
  GemmParams p{};
  p.M = a.size(1);
  p.N = b.size(1);
  p.K = a.size(0);
  if (p.M == 0 || p.N == 0 || p.K == 0) return;
  p.C32 = c32.data_ptr<float>();
  p.ldc32 = (int)c32.stride(0);
  DeviceScratch& scratch = device_scratch();
  p.err = scratch.err;
  const int bn = p.N <= 64 ? 64 : 128;
  p.splits = pick_splits(p.M, p.N, p.K, bn, (int)splits);
  const int tiles = ((p.M + 127) / 128) * ((p.N + bn - 1) / bn);
  if (p.splits > 1 && (tiles > scratch.max_counters || (size_t)tiles * p.splits * 128 * bn > scratch.ws_floats))
    p.splits = 1;
  p.ws = scratch.ws;
  p.counters = scratch.counters;
  gemm_wgrad_dispatch(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), p, bn, cur_stream());
}

static void rms_norm(const at::Tensor& x, c10::optional<at::Tensor> residual, const at::Tensor& w, at::Tensor& y,
                     double eps, int64_t groups) {
  rmsnorm_launch(x, residual, w, y, eps, (int)groups);
}

static void attention(const at::Tensor& q, at::Tensor& o, const at::Tensor& k_cache, const at::Tensor& v_cache,
                      const at::Tensor& block_tables, c10::optional<at::Tensor> prefix_lens,
                      c10::optional<at::Tensor> suffix_mask, c10::optional<at::Tensor> cu_q,
                      c10::optional<at::Tensor> cu_k, int64_t mode, int64_t B, int64_t Q, int64_t max_q,
                      double scale, int64_t num_splits, int64_t keys_per_split, c10::optional<at::Tensor> o_part,
                      c10::optional<at::Tensor> lse_part) {
  check_dev(q, "q");
  check_dev(o, "attention output");
  check_dev(k_cache, "k_cache");
  check_dev(v_cache, "v_cache");
  check_dev(block_tables, "block_tables");
  UNO_CHECK_BF16(q);
  UNO_CHECK_CONTIG(q);
  TORCH_CHECK(block_tables.scalar_type() == at::kInt, "block_tables must be int32");
  TORCH_CHECK(o.is_contiguous() && o.numel() == q.numel(), "attention output must match q");
  AttnLaunch a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.o_part = ptr_or_null<float>(o_part);
  a.lse_part = ptr_or_null<float>(lse_part);
  a.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  a.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  a.num_pages = k_cache.size(0);
  a.hkv = k_cache.size(1);
  a.page = k_cache.size(2);
  a.head_dim = k_cache.size(3);
  a.block_tables = block_tables.data_ptr<int>();
  a.bt_stride = block_tables.stride(0);
  a.prefix_lens = ptr_or_null<const int>(prefix_lens);
  a.suffix_mask = ptr_or_null<const int64_t>(suffix_mask);
  a.cu_q = ptr_or_null<const int>(cu_q);
  a.cu_k = ptr_or_null<const int>(cu_k);
  a.B = B;
  a.Q = Q;
  a.T = q.size(0);
  a.max_q = max_q;
  a.hq = q.size(1);
  a.scale = scale;
  a.mode = mode;
  a.num_splits = num_splits;
  a.keys_per_split = keys_per_split;
  a.err = device_error_flag();
  if (a.T == 0 || B == 0) return;
  paged_attention_launch(a, cur_stream());
}

static void attention_tc(const at::Tensor& q, at::Tensor& o, const at::Tensor& k_cache, const at::Tensor& v_cache,
                         const at::Tensor& block_tables, c10::optional<at::Tensor> prefix_lens,
                         c10::optional<at::Tensor> suffix_mask, c10::optional<at::Tensor> cu_q,
                         c10::optional<at::Tensor> cu_k, int64_t mode, int64_t B, int64_t Q, double scale,
                         at::Tensor& o_part, at::Tensor& lse_part, at::Tensor& counters,
                         c10::optional<at::Tensor> trace) {
  check_dev(q, "q");
  check_dev(o, "attention output");
  check_dev(k_cache, "k_cache");
  check_dev(v_cache, "v_cache");
  check_dev(block_tables, "block_tables");
  check_dev(o_part, "attention o_part");
  check_dev(lse_part, "attention lse_part");
  check_dev(counters, "attention counters");
  UNO_CHECK_BF16(q);
  UNO_CHECK_CONTIG(q);
  TORCH_CHECK(k_cache.is_contiguous() && v_cache.is_contiguous(), "KV cache must be contiguous");
  TORCH_CHECK(block_tables.scalar_type() == at::kInt, "block_tables must be int32");
  TORCH_CHECK(o.is_contiguous() && o.numel() == q.numel(), "attention output must match q");
  TORCH_CHECK(counters.scalar_type() == at::kInt, "attention counters must be int32");
  const int rows = attention_tc_rows();
  const int64_t slots = 2LL * num_sms();
  TORCH_CHECK(o_part.scalar_type() == at::kFloat && o_part.numel() >= slots * rows * 128,
              "attention o_part needs ", slots * rows * 128, " floats");
  TORCH_CHECK(lse_part.scalar_type() == at::kFloat && lse_part.numel() >= slots * rows,
              "attention lse_part needs ", slots * rows, " floats");
  TORCH_CHECK(counters.numel() >= q.size(0) * k_cache.size(1), "attention counters need T * kv_heads ints");
  if (mode == 0) {
    TORCH_CHECK(prefix_lens.has_value() && suffix_mask.has_value(), "decode attention needs prefix_lens and masks");
    TORCH_CHECK(prefix_lens->scalar_type() == at::kInt && suffix_mask->scalar_type() == at::kLong,
                "prefix_lens int32, suffix_mask int64");
    TORCH_CHECK(prefix_lens->numel() >= B && suffix_mask->numel() >= B * Q && q.size(0) >= B * Q,
                "decode attention metadata too short");
    check_dev(*prefix_lens, "prefix_lens");
    check_dev(*suffix_mask, "suffix_mask");
  } else {
    TORCH_CHECK(cu_q.has_value() && cu_k.has_value(), "prefill attention needs cu_seqlens");
    TORCH_CHECK(cu_q->scalar_type() == at::kInt && cu_k->scalar_type() == at::kInt, "cu_seqlens must be int32");
    TORCH_CHECK(cu_q->numel() >= B + 1 && cu_k->numel() >= B + 1, "cu_seqlens too short");
    check_dev(*cu_q, "cu_seqlens_q");
    check_dev(*cu_k, "cu_seqlens_k");
  }
  AttnLaunch a{};
  a.q = reinterpret_cast<const __nv_bfloat16*>(q.data_ptr());
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.o_part = o_part.data_ptr<float>();
  a.lse_part = lse_part.data_ptr<float>();
  a.k_cache = reinterpret_cast<const __nv_bfloat16*>(k_cache.data_ptr());
  a.v_cache = reinterpret_cast<const __nv_bfloat16*>(v_cache.data_ptr());
  a.num_pages = k_cache.size(0);
  a.hkv = k_cache.size(1);
  a.page = k_cache.size(2);
  a.head_dim = k_cache.size(3);
  a.block_tables = block_tables.data_ptr<int>();
  a.bt_stride = block_tables.stride(0);
  a.prefix_lens = ptr_or_null<const int>(prefix_lens);
  a.suffix_mask = ptr_or_null<const int64_t>(suffix_mask);
  a.cu_q = ptr_or_null<const int>(cu_q);
  a.cu_k = ptr_or_null<const int>(cu_k);
  a.B = B;
  a.Q = Q;
  a.T = q.size(0);
  a.max_q = Q;
  a.hq = q.size(1);
  a.scale = scale;
  a.mode = mode;
  a.num_splits = 1;
  a.keys_per_split = 0;
  a.err = device_error_flag();
  if (a.T == 0 || B == 0) return;
  unsigned long long* tr = nullptr;
  if (trace.has_value()) {
    check_dev(*trace, "attention trace");
    TORCH_CHECK(trace->scalar_type() == at::kLong && trace->numel() >= 1024 + 4 * num_sms(),
                "trace needs 1024 + 4 * SMs int64");
    tr = reinterpret_cast<unsigned long long*>(trace->data_ptr<int64_t>());
  }
  attention_tc_launch(a, counters.data_ptr<int>(), cur_stream(), tr);
}

void cycle_payload_launch(const at::Tensor& proposal, c10::optional<at::Tensor> accepted,
                          c10::optional<at::Tensor> target, c10::optional<at::Tensor> corr, const at::Tensor& lookahead,
                          const at::Tensor& stops, at::Tensor& payload);
void tree_meta_launch(const at::Tensor& parents, const at::Tensor& depths, const at::Tensor& prefix, at::Tensor& masks,
                      at::Tensor& positions);

}  // namespace uno

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("gemm", &uno::gemm, "tcgen05 GEMM with fused epilogues");
  m.def("rms_norm", &uno::rms_norm);
  m.def("attention_tc", &uno::attention_tc, "tcgen05 paged attention (persistent, balanced tile ranges)",
        py::arg("q"), py::arg("o"), py::arg("k_cache"), py::arg("v_cache"), py::arg("block_tables"),
        py::arg("prefix_lens"), py::arg("suffix_mask"), py::arg("cu_q"), py::arg("cu_k"), py::arg("mode"),
        py::arg("B"), py::arg("Q"), py::arg("scale"), py::arg("o_part"), py::arg("lse_part"), py::arg("counters"),
        py::arg("trace") = py::none());
  m.def("attention_tc_rows", &uno::attention_tc_rows);
  m.def("cycle_payload", &uno::cycle_payload_launch, "committed tokens + count of a linear Psi-Spec cycle");
  m.def("tree_meta", &uno::tree_meta_launch, "draft-tree ancestor masks and node positions");
  m.def("embedding", &uno::embedding_launch);
  m.def("silu_mul", &uno::silu_mul_launch);
  m.def("qk_norm_rope_store", &uno::qk_norm_rope_store_launch);
  m.def("copy_tree_kv", &uno::copy_tree_kv_launch);
  m.def("attention", &uno::attention);
  m.def("argmax", &uno::argmax_launch);
  m.def("gumbel_sample", &uno::gumbel_sample_launch);
  m.def("fused_verify", &uno::fused_verify_launch);
  m.def("topk_lse", &uno::topk_lse_launch);
  m.def("filtered_sample", &uno::filtered_sample_launch);
  m.def("filtered_verify", &uno::filtered_verify_launch);
  m.def("build_tree", &uno::build_tree_launch);
  m.def("walk_tree", &uno::walk_tree_launch);
  m.def("reduce_norm_gather", &uno::reduce_norm_gather_launch);
  m.def("embedding_scatter", &uno::embedding_scatter_launch);
  m.def("gemm_wgrad", &uno::gemm_wgrad);
  m.def("vp_sample", &uno::vp_sample_launch);
  m.def("vp_verify", &uno::vp_verify_launch);
  m.def("vp_region_bytes", &uno::vp_region_bytes);
  m.def("fused_adamw", &uno::fused_adamw_launch);
  m.def("opt_ctl_bytes", &uno::opt_ctl_bytes);
  m.def("uno_loss", &uno::uno_loss_launch);
  m.def("train_attn_fwd", &uno::train_attn_fwd);
  m.def("rmsnorm_fwd_train", &uno::rmsnorm_fwd_train);
  m.def("rmsnorm_bwd_train", &uno::rmsnorm_bwd_train);
  m.def("silu_mul_fwd", &uno::silu_mul_fwd);
  m.def("silu_mul_bwd", &uno::silu_mul_bwd);
  m.def("qk_norm_rope_fwd", &uno::qk_norm_rope_fwd);
  m.def("qk_norm_rope_bwd", &uno::qk_norm_rope_bwd);
  m.def("train_attn_bwd", &uno::train_attn_bwd);
  m.def("symm_alloc", &uno::symm_alloc);
  m.def("symm_open", &uno::symm_open);
  m.def("symm_close", &uno::symm_close);
  m.def("error_flag", &uno::read_error_flag, py::arg("reset") = false);
}
