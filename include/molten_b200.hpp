// molten_b200.hpp -- C++17 host mirror of Molten's op interface over the C ABI
// (molten_cuda.h).
//
// The reference's host side is Rust: src/kernels/{lfm,quant,elementwise}.rs
// expose functions of the form
//   fn op(ctx: &MetalContext, pass: &ComputePass, <tensors>, <dims>) -> Result<()>
// that check shapes and dtypes with `ensure!` and then encode a dispatch. This
// header keeps those names, argument meanings and checks for a C++ host:
// `Context` stands for MetalContext + ComputePass (one device and stream,
// metal.rs:91-400), `Tensor` for a device buffer view with shape and dtype
// (tensor.rs:30-96; caller-owned, never allocated here), `QuantWeights` for
// weights.rs:11-30, and a failed `ensure!` or a failed ABI call throws
// molten::Error (the ABI code and its message) before anything is enqueued.
// Calls are asynchronous on the context's stream; Context::commit_wait() is
// `commit_wait` (metal.rs:385-399).
#pragma once

#include <cstddef>
#include <cstdint>
#include <initializer_list>
#include <stdexcept>
#include <string>
#include <vector>

#include "molten_cuda.h"

namespace molten {

class Error : public std::runtime_error {
 public:
  Error(int code, const std::string& msg) : std::runtime_error(msg), code_(code) {}
  int code() const { return code_; }

 private:
  int code_;
};

inline void ensure(bool cond, const std::string& msg) {
  if (!cond) throw Error(MC_EINVAL, msg);
}

inline void check(int rc) {
  if (rc != MC_OK) {
    const char* m = mc_last_error();
    throw Error(rc, std::string("molten_cuda error ") + std::to_string(rc) + ": " + (m ? m : ""));
  }
}

// DType (tensor.rs); U64 holds the argmax keys of the head.
enum class DType { BF16, F32, U32, U64 };

inline size_t dtype_size(DType d) {
  return d == DType::BF16 ? 2 : (d == DType::U64 ? 8 : 4);
}

// A device buffer view: pointer (buffer + offset), shape, dtype.
struct Tensor {
  void* data = nullptr;
  std::vector<int64_t> shape;
  DType dtype = DType::BF16;

  Tensor() = default;
  Tensor(void* p, std::initializer_list<int64_t> s, DType d) : data(p), shape(s), dtype(d) {}
  Tensor(void* p, std::vector<int64_t> s, DType d) : data(p), shape(std::move(s)), dtype(d) {}

  int64_t numel() const {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    return n;
  }
  int64_t dim(int i) const { return shape.at(i < 0 ? shape.size() + i : i); }
  size_t nbytes() const { return (size_t)numel() * dtype_size(dtype); }
  template <typename T>
  T* as() const { return static_cast<T*>(data); }
};

// QuantWeights (weights.rs:11-30): codes U32 [out][in*bits/32], scales and
// biases BF16 [out][in/group_size].
struct QuantWeights {
  Tensor codes, scales, biases;
  int group_size = 64;
  int bits = 4;

  int out_features() const { return (int)codes.dim(0); }
  int in_features() const { return (int)(codes.dim(-1) * 32 / bits); }
  mc_qweights abi() const {
    return mc_qweights{codes.as<const uint32_t>(), scales.as<const uint16_t>(),
                       biases.as<const uint16_t>(), out_features(), in_features(), group_size,
                       bits};
  }
};

// check_quant (quant.rs:42-66) on the host-visible shape; the ABI re-checks
// the pointers' alignment.
inline void check_quant(const QuantWeights& w) {
  ensure(w.codes.shape.size() == 2 && w.codes.dtype == DType::U32, "codes must be U32 [out][words]");
  ensure(w.scales.dtype == DType::BF16 && w.biases.dtype == DType::BF16,
         "scales/biases must be BF16");
  ensure(w.group_size > 0 && w.in_features() % w.group_size == 0, "K must be a multiple of group");
  const int64_t n = w.out_features(), g = w.in_features() / w.group_size;
  ensure(w.scales.numel() == n * g && w.biases.numel() == n * g,
         "scales/biases shape mismatch");
}

class Context {
 public:
  explicit Context(int device = 0, void* stream = nullptr) : owned_(true) {
    check(mc_create(device, stream, &h_));
  }
  ~Context() {
    if (owned_ && h_) mc_destroy(h_);
  }
  Context(const Context&) = delete;
  Context& operator=(const Context&) = delete;

  // A non-owning view of an existing handle (the handle stays the caller's).
  static Context wrap(mc_ctx* h) { return Context(h); }
  Context(Context&& o) noexcept : h_(o.h_), owned_(o.owned_) { o.h_ = nullptr; }

  mc_ctx* handle() const { return h_; }
  void set_stream(void* stream) { check(mc_set_stream(h_, stream)); }
  void commit_wait() { check(mc_sync(h_)); }

 private:
  explicit Context(mc_ctx* h) : h_(h), owned_(false) {}
  mc_ctx* h_ = nullptr;
  bool owned_ = false;
};

namespace kernels {

inline int rows_of(const Tensor& t, int64_t row_len) { return (int)(t.numel() / row_len); }

// gemv_quant (kernels/lfm.rs:112-149): y[b] = W x[b] for the batch rows of x.
inline void gemv_quant(Context& ctx, const QuantWeights& w, const Tensor& x, const Tensor& y) {
  check_quant(w);
  const int64_t n = w.out_features(), k = w.in_features();
  ensure(x.numel() % k == 0 && y.numel() == x.numel() / k * n, "gemv shape mismatch");
  ensure(x.dtype == DType::BF16 && y.dtype == DType::BF16, "gemv BF16 only");
  const mc_qweights q = w.abi();
  check(mc_gemv_quant(ctx.handle(), &q, x.as<const uint16_t>(), y.as<uint16_t>(),
                      rows_of(x, k)));
}

// gemv_head_argmax (kernels/lfm.rs:826-844): argmax keys folded into best
// (U64 [batch], zero on entry).
inline void gemv_head_argmax(Context& ctx, const QuantWeights& w, const Tensor& x,
                             const Tensor& best) {
  check_quant(w);
  const int64_t k = w.in_features();
  ensure(x.numel() % k == 0 && x.dtype == DType::BF16, "head input shape");
  ensure(best.dtype == DType::U64 && best.numel() == x.numel() / k, "head keys shape");
  const mc_qweights q = w.abi();
  check(mc_gemv_head_argmax(ctx.handle(), &q, x.as<const uint16_t>(),
                            best.as<unsigned long long>(), rows_of(x, k)));
}

// token_tail (kernels/lfm.rs:850-888): key -> token (clearing the key), the
// next input row from a bf16 embedding table (optional) and its RMSNorm.
inline void token_tail(Context& ctx, const Tensor& best, const Tensor& out_tok,
                       const Tensor* embed, const Tensor* norm_w, const Tensor* x_next,
                       const Tensor* normed_next, float eps = 1e-5f) {
  const int batch = (int)best.numel();
  ensure(best.dtype == DType::U64 && out_tok.dtype == DType::U32 && out_tok.numel() == batch,
         "token tail shapes");
  int vocab = 0, hidden = 0;
  if (embed) {
    ensure(embed->dtype == DType::BF16 && embed->shape.size() == 2, "embedding table shape");
    ensure(norm_w && x_next && normed_next, "embedding gather needs norm_w, x_next, normed_next");
    vocab = (int)embed->dim(0);
    hidden = (int)embed->dim(1);
    ensure(norm_w->numel() == hidden && x_next->numel() == (int64_t)batch * hidden &&
               normed_next->numel() == (int64_t)batch * hidden,
           "token tail row shapes");
  }
  check(mc_token_tail(ctx.handle(), best.as<unsigned long long>(), out_tok.as<uint32_t>(),
                      embed ? embed->as<const uint16_t>() : nullptr, vocab,
                      norm_w ? norm_w->as<const uint16_t>() : nullptr,
                      x_next ? x_next->as<uint16_t>() : nullptr,
                      normed_next ? normed_next->as<uint16_t>() : nullptr, hidden, eps, batch));
}

// argmax_bf16 (kernels/lfm.rs:794-820): per row of logits [batch][n].
inline void argmax_bf16(Context& ctx, const Tensor& logits, const Tensor& out) {
  ensure(logits.dtype == DType::BF16 && logits.shape.size() == 2, "argmax logits shape");
  ensure(out.dtype == DType::U32 && out.numel() == logits.dim(0), "argmax out shape");
  check(mc_argmax_bf16(ctx.handle(), logits.as<const uint16_t>(), (int)logits.dim(1),
                       out.as<uint32_t>(), (int)logits.dim(0)));
}

// router_addnorm_route (kernels/lfm.rs:266-311): h' = h + b, RMSNorm, router
// logits, top-4 ids and weights. w: router [E][H], F32 (reference) or BF16
// (BASELINE); bias: expert_bias [E] F32 (route_mode SIGMOID_BIAS) or null;
// counter: U32 [batch], zero on entry and left zero.
inline void router_addnorm_route(Context& ctx, const Tensor& h, const Tensor* b, const Tensor& nw,
                                 const Tensor& hout, const Tensor& normed, const Tensor& w,
                                 const Tensor& logits, const Tensor* bias, const Tensor& ids,
                                 const Tensor& weights, const Tensor& counter, float eps = 1e-5f,
                                 int route_mode = MC_ROUTE_SOFTMAX_RENORM) {
  ensure(w.shape.size() == 2, "router weight must be [E][H]");
  const int e = (int)w.dim(0), k = (int)w.dim(1);
  ensure(w.dtype == DType::F32 || w.dtype == DType::BF16, "router weight dtype");
  ensure(h.numel() % k == 0, "router norm shapes");
  const int batch = (int)(h.numel() / k);
  ensure(logits.dtype == DType::F32 && logits.numel() == (int64_t)batch * e, "router logits shape");
  ensure(!bias || (bias->dtype == DType::F32 && bias->numel() == e), "router bias shape");
  ensure((!b || b->numel() == h.numel()) && hout.numel() == h.numel() &&
             normed.numel() == h.numel() && nw.numel() == k,
         "router norm shapes");
  ensure(ids.dtype == DType::U32 && ids.numel() == 4 * batch, "route ids shape");
  ensure(weights.dtype == DType::BF16 && weights.numel() == 4 * batch, "route weights shape");
  ensure(counter.dtype == DType::U32 && counter.numel() == batch, "route counter shape");
  check(mc_router_addnorm_route(
      ctx.handle(), h.as<const uint16_t>(), b ? b->as<const uint16_t>() : nullptr,
      nw.as<const uint16_t>(), hout.as<uint16_t>(), normed.as<uint16_t>(), w.data,
      w.dtype == DType::F32 ? MC_DTYPE_F32 : MC_DTYPE_BF16, bias ? bias->as<const float>() : nullptr,
      route_mode, logits.as<float>(), ids.as<uint32_t>(), weights.as<uint16_t>(),
      counter.as<uint32_t>(), e, k, eps, 1e-6f, batch));
}

// gemv_gather_act (kernels/lfm.rs:421-460): act[b][slot] = SwiGLU of the
// selected expert's gate/up rows against x[b].
inline void gemv_gather_act(Context& ctx, const QuantWeights& gate, const QuantWeights& up,
                            const Tensor& x, const Tensor& ids, const Tensor& act,
                            int n_experts = 64) {
  check_quant(gate);
  check_quant(up);
  const int64_t k = gate.in_features(), inter = gate.out_features() / n_experts;
  ensure(x.numel() % k == 0, "gather act input shape");
  const int batch = rows_of(x, k);
  ensure(ids.dtype == DType::U32 && ids.numel() == 4 * batch, "gather act ids shape");
  ensure(act.dtype == DType::BF16 && act.numel() == 4 * batch * inter, "gather act output shape");
  const mc_qweights g = gate.abi(), u = up.abi();
  check(mc_gemv_gather_act(ctx.handle(), &g, &u, x.as<const uint16_t>(), ids.as<const uint32_t>(),
                           act.as<uint16_t>(), n_experts, batch));
}

// gemv_gather_down_combine4 (kernels/lfm.rs:499-533).
inline void gemv_gather_down_combine4(Context& ctx, const QuantWeights& down, const Tensor& act,
                                      const Tensor& ids, const Tensor& weights, const Tensor& out,
                                      int n_experts = 64) {
  check_quant(down);
  const int64_t hidden = down.out_features() / n_experts, inter = down.in_features();
  ensure(act.numel() % (4 * inter) == 0, "down act shape");
  const int batch = (int)(act.numel() / (4 * inter));
  ensure(ids.numel() == 4 * batch && weights.numel() == 4 * batch, "down ids/weights shape");
  ensure(out.dtype == DType::BF16 && out.numel() == batch * hidden, "down output shape");
  const mc_qweights d = down.abi();
  check(mc_gemv_gather_down_combine4(ctx.handle(), &d, act.as<const uint16_t>(),
                                     ids.as<const uint32_t>(), weights.as<const uint16_t>(),
                                     out.as<uint16_t>(), n_experts, batch));
}

// moe_decode (lfm.rs:967-1011) as one launch: router + gate/up + down +
// combine for batch 1..; workspace: U32 [mc_moe_decode_workspace_words(I)],
// zeroed once.
inline void moe_decode_layer(Context& ctx, const Tensor& h, const Tensor* b, const Tensor& nw,
                             const Tensor& hout, const Tensor& normed, const Tensor& router,
                             const Tensor& logits, const Tensor* bias, const Tensor& ids,
                             const Tensor& weights, const QuantWeights& gate,
                             const QuantWeights& up, const QuantWeights& down, const Tensor& out,
                             const Tensor& workspace, int n_experts = 64, float eps = 1e-5f,
                             int route_mode = MC_ROUTE_SOFTMAX_RENORM) {
  check_quant(gate);
  check_quant(up);
  check_quant(down);
  ensure(router.dtype == DType::F32 || router.dtype == DType::BF16, "router weight dtype");
  ensure(workspace.dtype == DType::U32 &&
             (size_t)workspace.numel() >=
                 mc_moe_decode_workspace_words(gate.out_features() / n_experts),
         "decode workspace too small");
  ensure(out.numel() == h.numel() && hout.numel() == h.numel(), "decode row shapes");
  const mc_qweights g = gate.abi(), u = up.abi(), d = down.abi();
  check(mc_moe_decode_layer(
      ctx.handle(), h.as<const uint16_t>(), b ? b->as<const uint16_t>() : nullptr,
      nw.as<const uint16_t>(), hout.as<uint16_t>(), normed.as<uint16_t>(), router.data,
      router.dtype == DType::F32 ? MC_DTYPE_F32 : MC_DTYPE_BF16,
      bias ? bias->as<const float>() : nullptr, route_mode, logits.as<float>(), ids.as<uint32_t>(),
      weights.as<uint16_t>(), &g, &u, &d, n_experts, out.as<uint16_t>(), workspace.as<uint32_t>(),
      (size_t)workspace.numel(), eps, 1e-6f));
}

// gemv_quant(proj, h) -> b (kernels/lfm.rs:112-149) and moe_decode_layer(h, b,
// ...) in one launch, bit-identical to the two calls; proj Q4 2048 x 2048;
// workspace: U32 [mc_moe_decode_proj_workspace_words(I)], zeroed once;
// p_out (optional) receives b.
inline void moe_decode_layer_proj(Context& ctx, const Tensor& h, const QuantWeights& proj,
                                  const Tensor* p_out, const Tensor& nw, const Tensor& hout,
                                  const Tensor& normed, const Tensor& router,
                                  const Tensor& logits, const Tensor* bias, const Tensor& ids,
                                  const Tensor& weights, const QuantWeights& gate,
                                  const QuantWeights& up, const QuantWeights& down,
                                  const Tensor& out, const Tensor& workspace, int n_experts = 64,
                                  float eps = 1e-5f, int route_mode = MC_ROUTE_SOFTMAX_RENORM) {
  check_quant(proj);
  check_quant(gate);
  check_quant(up);
  check_quant(down);
  ensure(proj.bits == 4 && proj.in_features() == 2048 && proj.out_features() == 2048,
         "projection must be Q4 2048 x 2048");
  ensure(router.dtype == DType::F32 || router.dtype == DType::BF16, "router weight dtype");
  ensure(workspace.dtype == DType::U32 &&
             (size_t)workspace.numel() >=
                 mc_moe_decode_proj_workspace_words(gate.out_features() / n_experts),
         "decode workspace too small");
  ensure(out.numel() == h.numel() && hout.numel() == h.numel(), "decode row shapes");
  ensure(!p_out || p_out->numel() == h.numel(), "projection output shape");
  const mc_qweights pj = proj.abi(), g = gate.abi(), u = up.abi(), d = down.abi();
  check(mc_moe_decode_layer_proj(
      ctx.handle(), h.as<const uint16_t>(), &pj, p_out ? p_out->as<uint16_t>() : nullptr,
      nw.as<const uint16_t>(), hout.as<uint16_t>(), normed.as<uint16_t>(), router.data,
      router.dtype == DType::F32 ? MC_DTYPE_F32 : MC_DTYPE_BF16,
      bias ? bias->as<const float>() : nullptr, route_mode, logits.as<float>(), ids.as<uint32_t>(),
      weights.as<uint16_t>(), &g, &u, &d, n_experts, out.as<uint16_t>(), workspace.as<uint32_t>(),
      (size_t)workspace.numel(), eps, 1e-6f));
}

// gemm_q4_grouped_mlx (quant.rs:223-266): c rows of each row tile of `tiles`
// (uint4 {m0, m_end, expert, 0}, n_tiles entries) against that expert.
inline void gemm_q4_grouped_mlx(Context& ctx, const Tensor& a, const QuantWeights& w,
                                const Tensor& c, const Tensor& tiles, const Tensor& n_tiles,
                                int n_experts, const Tensor* status = nullptr) {
  check_quant(w);
  ensure(a.shape.size() == 2 && a.dim(1) == w.in_features() && a.dtype == DType::BF16,
         "grouped GEMM input shape");
  ensure(c.dtype == DType::BF16 && c.numel() == a.dim(0) * (w.out_features() / n_experts),
         "grouped GEMM output shape");
  ensure(tiles.dtype == DType::U32 && tiles.numel() % 4 == 0 && n_tiles.dtype == DType::U32,
         "grouped GEMM tile list");
  const mc_qweights q = w.abi();
  check(mc_gemm_q4_grouped(ctx.handle(), a.as<const uint16_t>(), (int)a.dim(0), &q, n_experts,
                           c.as<uint16_t>(), tiles.as<const uint32_t>(),
                           n_tiles.as<const uint32_t>(), (int)(tiles.numel() / 4),
                           status ? status->as<uint32_t>() : nullptr));
}

// gemm_q4_grouped_mlx_gu + silu_mul_bf16 (quant.rs:146-199,
// elementwise.rs:48-56): act = SwiGLU(gate, up) of each row tile.
inline void gemm_q4_grouped_mlx_gu(Context& ctx, const Tensor& a, const QuantWeights& gate,
                                   const QuantWeights& up, const Tensor& act, const Tensor& tiles,
                                   const Tensor& n_tiles, int n_experts,
                                   const Tensor* status = nullptr) {
  check_quant(gate);
  check_quant(up);
  ensure(a.shape.size() == 2 && a.dim(1) == gate.in_features() && a.dtype == DType::BF16,
         "grouped gate/up input shape");
  ensure(act.dtype == DType::BF16 && act.numel() == a.dim(0) * (gate.out_features() / n_experts),
         "grouped gate/up output shape");
  const mc_qweights g = gate.abi(), u = up.abi();
  check(mc_gemm_q4_grouped_gu(ctx.handle(), a.as<const uint16_t>(), (int)a.dim(0), &g, &u,
                              n_experts, act.as<uint16_t>(), tiles.as<const uint32_t>(),
                              n_tiles.as<const uint32_t>(), (int)(tiles.numel() / 4),
                              status ? status->as<uint32_t>() : nullptr));
}

// dequant_q4_bf16_bulk + gemm_bf16_nt (quant.metal:69-114, gemm.rs:33-60):
// c = a . bf16(W)^T; workspace U32 [mc_gemm_q4_workspace_words(m)].
inline void gemm_q4(Context& ctx, const Tensor& a, const QuantWeights& w, const Tensor& c,
                    const Tensor& workspace, const Tensor* status = nullptr) {
  check_quant(w);
  ensure(a.shape.size() == 2 && a.dim(1) == w.in_features() && a.dtype == DType::BF16,
         "gemm input shape");
  ensure(c.dtype == DType::BF16 && c.numel() == a.dim(0) * w.out_features(), "gemm output shape");
  ensure(workspace.dtype == DType::U32, "gemm workspace dtype");
  const mc_qweights q = w.abi();
  check(mc_gemm_q4(ctx.handle(), a.as<const uint16_t>(), (int)a.dim(0), &q, c.as<uint16_t>(),
                   workspace.as<uint32_t>(), (size_t)workspace.numel(),
                   status ? status->as<uint32_t>() : nullptr));
}

// gather_rows_bf16 (elementwise.rs:59-104): out[i] = table[ids[i]].
inline void gather_rows_bf16(Context& ctx, const Tensor& table, const Tensor& ids,
                             const Tensor& out) {
  ensure(table.dtype == DType::BF16 && table.shape.size() == 2, "gather table shape");
  ensure(ids.dtype == DType::U32 && out.numel() == ids.numel() * table.dim(1), "gather shapes");
  check(mc_gather_rows_bf16(ctx.handle(), table.as<const uint16_t>(), ids.as<const uint32_t>(),
                            (int)ids.numel(), (int)table.dim(1), out.as<uint16_t>()));
}

// silu_mul_bf16 (elementwise.rs:48-56).
inline void silu_mul_bf16(Context& ctx, const Tensor& gate, const Tensor& up, const Tensor& out) {
  ensure(gate.numel() == up.numel() && up.numel() == out.numel(), "silu_mul shapes");
  ensure(gate.dtype == DType::BF16 && up.dtype == DType::BF16 && out.dtype == DType::BF16,
         "silu_mul BF16 only");
  check(mc_silu_mul_bf16(ctx.handle(), gate.as<const uint16_t>(), up.as<const uint16_t>(),
                         out.as<uint16_t>(), (size_t)out.numel()));
}

// moe_combine_rows (kernels/lfm.rs:701-756): out[t] = sum_r gw[t][r] ed[slotpos[t][r]].
inline void moe_combine_rows(Context& ctx, const Tensor& ed, const Tensor& slotpos,
                             const Tensor& gw, const Tensor& out, int topk = 4) {
  ensure(out.shape.size() == 2 && ed.dtype == DType::BF16 && out.dtype == DType::BF16,
         "combine shapes");
  const int m = (int)out.dim(0), hidden = (int)out.dim(1);
  ensure(slotpos.numel() == (int64_t)m * topk && gw.numel() == (int64_t)m * topk,
         "combine slot shapes");
  check(mc_moe_combine_rows(ctx.handle(), ed.as<const uint16_t>(), slotpos.as<const uint32_t>(),
                            gw.as<const uint16_t>(), out.as<uint16_t>(), m, topk, hidden));
}

// moe_prefill (lfm.rs:847-965, the MoE FFN): route, sort, gather, grouped
// GEMMs, combine in one call over one workspace of
// mc_moe_prefill_workspace_size(m, E, H, I) bytes.
inline void moe_prefill(Context& ctx, const Tensor& x, const Tensor& logits,
                        const QuantWeights& gate, const QuantWeights& up,
                        const QuantWeights& down, const Tensor& workspace, const Tensor& out,
                        int n_experts = 64, int route_mode = MC_ROUTE_SOFTMAX_RENORM,
                        const Tensor* bias = nullptr) {
  check_quant(gate);
  check_quant(up);
  check_quant(down);
  ensure(x.shape.size() == 2 && x.dtype == DType::BF16, "prefill input shape");
  const int m = (int)x.dim(0);
  ensure(logits.dtype == DType::F32 && logits.numel() == (int64_t)m * n_experts,
         "prefill logits shape");
  ensure(out.numel() == x.numel() && out.dtype == DType::BF16, "prefill output shape");
  const mc_qweights g = gate.abi(), u = up.abi(), d = down.abi();
  check(mc_moe_prefill(ctx.handle(), x.as<const uint16_t>(), logits.as<const float>(), m, &g, &u,
                       &d, n_experts, route_mode, bias ? bias->as<const float>() : nullptr,
                       workspace.data, workspace.nbytes(), out.as<uint16_t>()));
}

// proj3_gemv_scatter (kernels/lfm.rs:150-205): Q, K, V projections of one
// row in one launch, V written into the KV cache [nv/64][max_seq][64] at pos.
inline void proj3_gemv_scatter(Context& ctx, const QuantWeights& q, const QuantWeights& k,
                               const QuantWeights& v, const Tensor& x, const Tensor& q_out,
                               const Tensor& k_out, const Tensor& v_cache, int pos) {
  const int64_t kdim = x.numel();
  const int64_t nq = q.out_features(), nk = k.out_features(), nv = v.out_features();
  ensure(q.in_features() == kdim && k.in_features() == kdim && v.in_features() == kdim,
         "proj3 input width");
  ensure(q.bits == 4 && k.bits == 4 && v.bits == 4 && q.group_size == 64 &&
             k.group_size == 64 && v.group_size == 64,
         "proj3 is affine 4-bit/64");
  ensure(kdim == 2048, "proj3 input width is the compile-time hidden size");
  ensure(q_out.numel() == nq && k_out.numel() == nk && nv % 64 == 0, "proj3 output shape");
  ensure(x.dtype == DType::BF16 && q_out.dtype == DType::BF16 && k_out.dtype == DType::BF16,
         "proj3 BF16");
  ensure(v_cache.shape.size() == 3 && v_cache.dim(0) * 64 == nv && v_cache.dim(2) == 64 &&
             pos >= 0 && pos < v_cache.dim(1),
         "proj3 KV cache shape");
  check_quant(q);
  check_quant(k);
  check_quant(v);
  const mc_qweights a = q.abi(), b = k.abi(), c = v.abi();
  check(mc_proj3_gemv_scatter(ctx.handle(), &a, &b, &c, x.as<const uint16_t>(),
                              q_out.as<uint16_t>(), k_out.as<uint16_t>(), v_cache.as<uint16_t>(),
                              (int)v_cache.dim(1), pos));
}

// conv3_gemv (kernels/lfm.rs:207-246): short-conv B/C/X projection and the
// conv; w taps [H][3], state and new_state [2][H].
inline void conv3_gemv(Context& ctx, const QuantWeights& wproj, const Tensor& x, const Tensor& w,
                       const Tensor& state, const Tensor& out, const Tensor& new_state) {
  const int64_t kdim = x.numel(), h = out.numel();
  ensure(wproj.out_features() == 3 * h && wproj.in_features() == kdim, "conv3 projection shape");
  ensure(wproj.bits == 4 && wproj.group_size == 64, "conv3 projection 4-bit/64");
  ensure(kdim == 2048, "conv3 input width is the compile-time hidden size");
  ensure(w.numel() == 3 * h, "conv3 tap shape");
  ensure(state.shape == std::vector<int64_t>{2, h} && new_state.shape == std::vector<int64_t>{2, h},
         "conv3 state shape");
  check_quant(wproj);
  const mc_qweights q = wproj.abi();
  check(mc_conv3_gemv(ctx.handle(), &q, x.as<const uint16_t>(), w.as<const uint16_t>(),
                      state.as<const uint16_t>(), out.as<uint16_t>(), new_state.as<uint16_t>(),
                      (int)h));
}

// gemv_gu_act (kernels/lfm.rs:462-495): dense FFN front half.
inline void gemv_gu_act(Context& ctx, const QuantWeights& gate, const QuantWeights& up,
                        const Tensor& x, const Tensor& act) {
  const int64_t n = gate.out_features(), k = gate.in_features();
  ensure(gate.bits == 4 && up.bits == 4, "dense gate/up must be 4-bit");
  ensure(up.out_features() == n && up.in_features() == k && up.group_size == gate.group_size,
         "dense gate/up shapes");
  ensure(x.numel() % k == 0 && act.numel() == x.numel() / k * n, "dense gate/up rows");
  ensure(x.dtype == DType::BF16 && act.dtype == DType::BF16, "dense gate/up BF16");
  check_quant(gate);
  check_quant(up);
  const mc_qweights g = gate.abi(), u = up.abi();
  check(mc_gemv_gu_act(ctx.handle(), &g, &u, x.as<const uint16_t>(), act.as<uint16_t>(),
                       (int)(x.numel() / k)));
}

// SampleScratch::encode_draw / encode_mark (lfm/sample.rs:248-353): the
// sampled token of position pos into the zeroed argmax key `best`, read and
// cleared by token_tail; the workspace of mc_sample_workspace_bytes(vocab)
// bytes is zeroed once by the caller.
inline void sample_draw(Context& ctx, const Tensor& logits, const Tensor* seen,
                        const mc_sampling& s, uint32_t pos, const Tensor& best,
                        const Tensor& workspace) {
  ensure(logits.dtype == DType::BF16, "sampling logits row");
  ensure(best.dtype == DType::U64 && best.numel() >= 1, "sampling key");
  ensure(s.repetition_penalty == 1.0f || seen, "a repetition penalty needs the seen set");
  check(mc_sample_draw(ctx.handle(), logits.as<const uint16_t>(), (int)logits.numel(),
                       seen ? seen->as<const uint32_t>() : nullptr, &s, pos, nullptr,
                       best.as<unsigned long long>(), workspace.data, workspace.nbytes()));
}

inline void sample_mark(Context& ctx, const Tensor& tok, const Tensor& seen, int vocab) {
  ensure(tok.numel() == 1 && tok.dtype == DType::U32, "sampled token slot");
  check(mc_sample_mark(ctx.handle(), tok.as<const uint32_t>(), seen.as<uint32_t>(), vocab,
                       nullptr));
}

// Tensor::write_bytes / contents (tensor.rs:127-146, 165-200): stream-ordered
// copy between device memory and page-locked host memory.
inline void copy_async(Context& ctx, void* dst, const void* src, size_t bytes) {
  check(mc_copy_async(ctx.handle(), dst, src, bytes));
}

}  // namespace kernels
}  // namespace molten
