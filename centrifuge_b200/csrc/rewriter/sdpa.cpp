// Filtered ("restore-Q") attention backward node that replaces the SDPA backward nodes.
//
// Reference: ScaledDotProductFlashAttentionFilterRestoreQ (grad_filter/token_filter/csrc/
// backward_filters.cpp:420-505) and its efficient / cuDNN siblings (:547-839).  Given the kept
// query rows, the node returns
//   dQ  of kept queries, summed over every key at or before the query's position,
//   dK, dV of kept keys, summed over kept queries only,
// i.e. the exact gradient with K/V of dropped positions held constant.  Outputs are compact
// ([B, h, S_keep, d]); the rest of the graph has been shrunk to match.
//
// On CUDA bf16 causal attention without bias the node calls the fused sm_100a backward
// (op cfb::attn_bwd_rows, registered by centrifuge_b200._kernels); otherwise it evaluates the
// same formula with ATen in fp32 (CPU graphs, or attention with an explicit bias/mask).
#include <ATen/core/dispatch/Dispatcher.h>

#include <cmath>

#include "rewriter.h"

namespace cfb_filter {

using torch::autograd::variable_list;
using namespace torch::autograd::generated;

namespace {

struct FilteredAttentionBackward : public Node {
  SavedVariable query_, key_, value_, bias_, output_, lse_;
  bool causal = true;
  double dropout = 0.0;
  std::optional<double> scale;
  bool lse_is_rowwise = false;  // lse_ holds the [B, h, S] log-sum-exp of scale * q k^T
  Tensor pos_;                  // [B, S_keep] kept positions
  int64_t S = 0;
  std::string source;

  std::string name() const override { return "FilteredAttentionBackward"; }
  void release_variables() override {
    query_.reset_data();
    key_.reset_data();
    value_.reset_data();
    bias_.reset_data();
    output_.reset_data();
    lse_.reset_data();
  }
  variable_list apply(variable_list&& grads) override;

  variable_list math(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& bias,
                     const Tensor& dO) const;
  bool kernel_ok(const Tensor& q) const;
  variable_list kernel(const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& dO);
};

Tensor gather_rows3(const Tensor& t, const Tensor& pos) {
  // t [B, h, S, ...] -> [B, h, Sk, ...] at positions pos [B, Sk]
  auto idx = pos.to(t.device()).view({pos.size(0), 1, pos.size(1)});
  std::vector<int64_t> shape = {t.size(0), t.size(1), pos.size(1)};
  for (int64_t i = 3; i < t.dim(); ++i) {
    idx = idx.unsqueeze(-1);
    shape.push_back(t.size(i));
  }
  return at::gather(t, 2, idx.expand(shape));
}

variable_list FilteredAttentionBackward::math(const Tensor& q, const Tensor& k, const Tensor& v,
                                              const Tensor& bias, const Tensor& dO) const {
  const int64_t B = q.size(0), h = q.size(1), d = q.size(3), hk = k.size(1);
  const int64_t Sk = pos_.size(1);
  const int64_t rep = h / hk;
  const double sc = scale.has_value() ? *scale : 1.0 / std::sqrt(static_cast<double>(d));
  const Tensor qf = q.to(at::kFloat), kf0 = k.to(at::kFloat), vf0 = v.to(at::kFloat);
  const Tensor kf = rep > 1 ? kf0.repeat_interleave(rep, 1) : kf0;
  const Tensor vf = rep > 1 ? vf0.repeat_interleave(rep, 1) : vf0;
  const Tensor pos = pos_.to(q.device());
  const Tensor qk = gather_rows3(qf, pos);                            // [B,h,Sk,d]
  Tensor s = at::matmul(qk, kf.transpose(-1, -2)) * sc;               // [B,h,Sk,S]
  if (causal) {
    const Tensor keys = at::arange(S, pos.options()).view({1, 1, 1, S});
    const Tensor allowed = keys.le(pos.view({B, 1, Sk, 1}));
    s = s.masked_fill(allowed.logical_not(), -std::numeric_limits<float>::infinity());
  }
  if (bias.defined()) {
    Tensor b = bias.to(at::kFloat);
    if (b.dim() == 2) b = b.view({1, 1, b.size(0), b.size(1)});
    b = b.expand({B, h, S, S});
    if (b.scalar_type() == at::kBool)
      s = s.masked_fill(gather_rows3(b, pos).logical_not(), -std::numeric_limits<float>::infinity());
    else
      s = s + gather_rows3(b.contiguous(), pos);
  }
  const Tensor p = at::softmax(s, -1);
  const Tensor dOf = dO.to(at::kFloat);
  const Tensor ok = at::matmul(p, vf);
  const Tensor dp = at::matmul(dOf, vf.transpose(-1, -2));
  const Tensor delta = (dOf * ok).sum(-1, true);
  const Tensor ds = p * (dp - delta);
  Tensor dq = at::matmul(ds, kf) * sc;
  const Tensor kidx = pos.view({B, 1, 1, Sk}).expand({B, h, Sk, Sk});
  const Tensor ds_kk = at::gather(ds, 3, kidx);
  const Tensor p_kk = at::gather(p, 3, kidx);
  Tensor dk = at::matmul(ds_kk.transpose(-1, -2), qk) * sc;  // [B,h,Sk,d]
  Tensor dv = at::matmul(p_kk.transpose(-1, -2), dOf);
  if (rep > 1) {
    dk = dk.view({B, hk, rep, Sk, d}).sum(2);
    dv = dv.view({B, hk, rep, Sk, d}).sum(2);
  }
  return {dq.to(q.scalar_type()), dk.to(k.scalar_type()), dv.to(v.scalar_type())};
}

bool FilteredAttentionBackward::kernel_ok(const Tensor& q) const {
  if (!q.is_cuda() || q.scalar_type() != at::kBFloat16 || !causal || dropout != 0.0) return false;
  if (bias_.unpack().defined()) return false;
  const int64_t d = q.size(3);
  if (d != 64 && d != 128) return false;
  return c10::Dispatcher::singleton().findSchema({"cfb::attn_bwd_rows", ""}).has_value();
}

// [B, h, S, d] -> token-major rows [B*S, h*d]
Tensor to_rows(const Tensor& t) {
  return t.transpose(1, 2).contiguous().view({t.size(0) * t.size(2), t.size(1) * t.size(3)});
}

variable_list FilteredAttentionBackward::kernel(const Tensor& q, const Tensor& k, const Tensor& v,
                                                const Tensor& dO) {
  const int64_t B = q.size(0), h = q.size(1), d = q.size(3), hk = k.size(1);
  const int64_t Sk = pos_.size(1);
  const double sc = scale.has_value() ? *scale : 1.0 / std::sqrt(static_cast<double>(d));
  const Tensor qkv = at::cat({to_rows(q), to_rows(k), to_rows(v)}, 1).contiguous();
  const Tensor pos = pos_.to(q.device());
  const Tensor rows =
      (pos + at::arange(B, pos.options()).unsqueeze(1) * S).reshape({-1});
  const Tensor qkv_k = qkv.index_select(0, rows);
  Tensor o_k, lse_k;
  Tensor o = output_.unpack();
  Tensor lse = lse_.unpack();
  if (o.defined() && lse.defined() && lse_is_rowwise) {
    o_k = to_rows(o).index_select(0, rows);
    lse_k = lse.narrow(2, 0, S).transpose(1, 2).contiguous().view({B * S, h}).index_select(0, rows)
                .to(at::kFloat)
                .contiguous();
  } else {
    static auto fwd = c10::Dispatcher::singleton()
                          .findSchemaOrThrow("cfb::attn_fwd_rows", "")
                          .typed<std::tuple<Tensor, Tensor>(const Tensor&, int64_t, int64_t,
                                                            int64_t, int64_t, int64_t, double)>();
    auto ol = fwd.call(qkv, B, S, h, hk, d, sc);
    o_k = std::get<0>(ol).index_select(0, rows);
    lse_k = std::get<1>(ol).index_select(0, rows).contiguous();
  }
  const Tensor do_k = to_rows(dO.to(q.scalar_type()));
  static auto bwd = c10::Dispatcher::singleton()
                        .findSchemaOrThrow("cfb::attn_bwd_rows", "")
                        .typed<Tensor(const Tensor&, const Tensor&, const Tensor&, const Tensor&,
                                      const Tensor&, const Tensor&, int64_t, int64_t, int64_t,
                                      int64_t, int64_t, int64_t, double)>();
  const Tensor pos32 = pos.to(at::kInt).contiguous();
  const Tensor dqkv = bwd.call(qkv_k, qkv, o_k.contiguous(), do_k, lse_k, pos32, B, S, Sk, h, hk,
                               d, sc);
  auto split = [&](int64_t c0, int64_t heads) {
    return dqkv.narrow(1, c0, heads * d).view({B, Sk, heads, d}).transpose(1, 2);
  };
  return {split(0, h), split(h * d, hk), split((h + hk) * d, hk)};
}

variable_list FilteredAttentionBackward::apply(variable_list&& grads) {
  Tensor dO = grads[0];
  const size_t n_out = next_edges().size();
  variable_list out(n_out);
  if (!dO.defined()) return out;
  Tensor q = query_.unpack(), k = key_.unpack(), v = value_.unpack(), bias = bias_.unpack();
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4, "filtered attention expects [B, h, S, d] inputs");
  if (dO.size(2) == S && pos_.size(1) != S) dO = gather_rows3(dO, pos_);
  variable_list r = kernel_ok(q) ? kernel(q, k, v, dO) : math(q, k, v, bias, dO);
  for (size_t i = 0; i < n_out && i < 3; ++i) out[i] = r[i];
  return out;
}

}  // namespace

bool is_attention_node(const std::string& name) {
  return name == "ScaledDotProductFlashAttentionBackward0" ||
         name == "ScaledDotProductEfficientAttentionBackward0" ||
         name == "ScaledDotProductCudnnAttentionBackward0" ||
         name == "ScaledDotProductFlashAttentionForCpuBackward0";
}

void replace_attention_edge(Edge& edge, Shrinker& s) {
  Node* old = edge.function.get();
  const std::string name = old->name();
  s.shrink_input_metadata(old);
  auto node = std::shared_ptr<FilteredAttentionBackward>(new FilteredAttentionBackward(),
                                                         torch::autograd::deleteNode);
  for (uint32_t i = 0; i < old->num_inputs(); ++i) {
    const auto& m = old->input_metadata(i);
    node->add_input_metadata(m.options(), m.shape_as_dim_vector(), m.is_tensor_subclass(),
                             m.is_nested_tensor(), m.grad_dtype());
  }
  for (const Edge& e : old->next_edges()) node->add_next_edge(e);
  auto own = old->getptr();
  auto keep = [&](SavedVariable& dst, SavedVariable& src, bool is_out) {
    Tensor t = is_out ? src.unpack(own) : src.unpack();
    if (t.defined()) dst = SavedVariable(t.detach(), false);
  };
  if (name == "ScaledDotProductFlashAttentionBackward0") {
    auto* n = static_cast<ScaledDotProductFlashAttentionBackward0*>(old);
    keep(node->query_, n->query_, false);
    keep(node->key_, n->key_, false);
    keep(node->value_, n->value_, false);
    keep(node->output_, n->output_, true);
    keep(node->lse_, n->logsumexp_, true);
    node->lse_is_rowwise = true;
    node->causal = n->is_causal;
    node->dropout = n->dropout_p;
    node->scale = n->scale;
  } else if (name == "ScaledDotProductEfficientAttentionBackward0") {
    auto* n = static_cast<ScaledDotProductEfficientAttentionBackward0*>(old);
    keep(node->query_, n->query_, false);
    keep(node->key_, n->key_, false);
    keep(node->value_, n->value_, false);
    keep(node->bias_, n->attn_bias_, false);
    keep(node->output_, n->output_, true);
    keep(node->lse_, n->log_sumexp_, true);
    node->lse_is_rowwise = true;
    node->causal = n->is_causal;
    node->dropout = n->dropout_p;
    node->scale = n->scale;
  } else if (name == "ScaledDotProductCudnnAttentionBackward0") {
    auto* n = static_cast<ScaledDotProductCudnnAttentionBackward0*>(old);
    keep(node->query_, n->query_, false);
    keep(node->key_, n->key_, false);
    keep(node->value_, n->value_, false);
    keep(node->bias_, n->attn_bias_, false);
    node->causal = n->is_causal;
    node->dropout = n->dropout_p;
    node->scale = n->scale;
  } else {
    auto* n = static_cast<ScaledDotProductFlashAttentionForCpuBackward0*>(old);
    keep(node->query_, n->query_, false);
    keep(node->key_, n->key_, false);
    keep(node->value_, n->value_, false);
    keep(node->bias_, n->attn_mask_, false);
    node->causal = n->is_causal;
    node->dropout = n->dropout_p;
    node->scale = n->scale;
  }
  TORCH_CHECK(node->dropout == 0.0, "backward_filter: attention dropout is not supported");
  Tensor q = node->query_.unpack();
  TORCH_CHECK(q.defined() && q.size(2) == s.S(), "backward_filter: attention query length ",
              q.defined() ? q.size(2) : -1, " differs from the mask length ", s.S());
  node->S = s.S();
  node->pos_ = s.pos();
  node->source = name;
  edge.function = node;
}

}  // namespace cfb_filter
