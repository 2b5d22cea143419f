// Shrinker: kept-row index state, sequence-dimension classification (record or replay) and
// the shrinking of saved tensors, size vectors and input metadata.
//
// Behaviour follows GraphFilter (grad_filter/token_filter/csrc/graph_filter.cpp:45-329):
// a dimension is a sequence dimension when its extent equals S, B*S, S-1 or B*(S-1); with
// several candidates the first of B*S / S-1 / B*(S-1) wins, while extents equal to S are
// collected (up to two, encoded a + 10*b).  Unlike the reference, a batch-dependent gather is
// one index_select over a flattened [B*S, ...] view instead of a per-row loop, and two
// sequence dimensions are supported for any batch size.
#include "rewriter.h"

#include <cstdlib>

namespace cfb_filter {

Shrinker::Shrinker(const Tensor& mask_in) {
  TORCH_CHECK(mask_in.dim() == 2, "backward_filter: mask must be [batch, seq], got ",
              mask_in.sizes());
  torch::NoGradGuard ng;
  mask_ = mask_in;
  B_ = mask_in.size(0);
  S_ = mask_in.size(1);
  const Tensor keep = mask_in.ne(0);
  const int64_t total = keep.sum().item<int64_t>();
  TORCH_CHECK(B_ > 0 && total % B_ == 0,
              "backward_filter: every row of the mask must keep the same number of tokens");
  Sk_ = total / B_;
  const auto opts = mask_in.options().dtype(at::kLong);
  pos_ = keep.nonzero().select(1, 1).reshape({B_, Sk_});
  const Tensor keep_m1 = keep.narrow(1, 0, S_ - 1);
  const int64_t total_m1 = keep_m1.sum().item<int64_t>();
  TORCH_CHECK(total_m1 % B_ == 0, "backward_filter: rows keep different loss positions");
  pos_m1_ = keep_m1.nonzero().select(1, 1).reshape({B_, total_m1 / B_});
  const Tensor base = at::arange(B_, opts).unsqueeze(1);
  flat_ = (pos_ + base * S_).reshape({-1});
  flat_m1_ = (pos_m1_ + base * (S_ - 1)).reshape({-1});
}

// ------------------------------------------------------------------ dims text
// Plain string handling (no iostreams: the extension's stream instantiations crashed when mixed
// with the host process's libstdc++ locale state).
std::vector<std::string> split_lines(const std::string& text) {
  std::vector<std::string> lines;
  size_t start = 0;
  while (start < text.size()) {
    size_t end = text.find('\n', start);
    if (end == std::string::npos) end = text.size();
    std::string line = text.substr(start, end - start);
    if (!line.empty() && line.back() == '\r') line.pop_back();
    lines.push_back(std::move(line));
    start = end + 1;
  }
  return lines;
}

static bool parse_ints(const std::string& line, int* out, int n) {
  const char* p = line.c_str();
  for (int i = 0; i < n; ++i) {
    char* end = nullptr;
    const long v = std::strtol(p, &end, 10);
    if (end == p) return false;
    out[i] = static_cast<int>(v);
    p = end;
  }
  return true;
}

void Shrinker::load_dims(const std::string& text) {
  records_.clear();
  const auto lines = split_lines(text);
  size_t i = 0;
  while (i < lines.size()) {
    const std::string& name = lines[i++];
    if (name == "---" || name.empty()) continue;
    NodeRecord rec;
    rec.name = name;
    while (i < lines.size() && lines[i] != "---") {
      int v[3];
      TORCH_CHECK(parse_ints(lines[i], v, 3), "backward_filter: malformed dims line '", lines[i],
                  "'");
      TORCH_CHECK(v[2] >= 0 && v[2] <= 4, "backward_filter: bad dims mode ", v[2]);
      rec.dims.push_back(DimRecord{v[0], v[1], static_cast<SeqMode>(v[2])});
      ++i;
    }
    ++i;  // separator
    records_.push_back(std::move(rec));
  }
  replay_ = true;
  cursor_ = 0;
}

std::string Shrinker::dims_text() const {
  std::string out;
  for (const auto& r : records_) {
    out += r.name + "\n";
    for (const auto& d : r.dims)
      out += std::to_string(d.index) + " " + std::to_string(d.bsz_index) + " " +
             std::to_string(static_cast<int>(d.mode)) + "\n";
    out += "---\n";
  }
  return out;
}

void Shrinker::begin_node(const std::string& name) {
  ++processed_nodes;
  if (replay_) {
    TORCH_CHECK(cursor_ < records_.size(), "backward_filter: the replayed dims describe ",
                records_.size(), " nodes but the graph has more (at '", name, "')");
    TORCH_CHECK(records_[cursor_].name == name, "backward_filter: replayed dims expect node '",
                records_[cursor_].name, "' but the graph has '", name, "'");
    current_ = &records_[cursor_];
  } else {
    records_.push_back(NodeRecord{name, {}});
    current_ = &records_.back();
  }
}

void Shrinker::end_node() {
  if (replay_) ++cursor_;
  current_ = nullptr;
}

// ------------------------------------------------------------------ classification
DimRecord Shrinker::classify(c10::ArrayRef<c10::SymInt> sizes) {
  TORCH_CHECK(current_ != nullptr, "backward_filter: classify outside a node");
  if (replay_) {
    TORCH_CHECK(!current_->dims.empty(), "backward_filter: replayed dims of '", current_->name,
                "' are exhausted");
    DimRecord d = current_->dims.front();
    current_->dims.pop_front();
    return d;
  }
  DimRecord d;
  for (size_t i = 0; i < sizes.size(); ++i) {
    const c10::SymInt& s = sizes[i];
    if (s == S_) {
      d.index = d.index == -1 ? static_cast<int>(i) : d.index + static_cast<int>(i) * 10;
      d.mode = SeqMode::kSeq;
    } else if (s == S_ * B_) {
      d.index = static_cast<int>(i);
      d.mode = SeqMode::kBatchSeq;
      break;
    } else if (s == S_ - 1) {
      d.index = static_cast<int>(i);
      d.mode = SeqMode::kSeqMinus1;
      break;
    } else if (s == (S_ - 1) * B_) {
      d.index = static_cast<int>(i);
      d.mode = SeqMode::kBatchSeqMinus1;
      break;
    }
  }
  for (size_t i = 0; i < sizes.size(); ++i) {
    if (sizes[i] == B_) {
      d.bsz_index = static_cast<int>(i);
      break;
    }
  }
  current_->dims.push_back(d);
  return d;
}

int64_t Shrinker::new_extent(SeqMode mode) const {
  switch (mode) {
    case SeqMode::kSeq: return Sk_;
    case SeqMode::kBatchSeq: return Sk_ * B_;
    case SeqMode::kSeqMinus1: return pos_m1_.size(1);
    case SeqMode::kBatchSeqMinus1: return pos_m1_.size(1) * B_;
    default: return -1;
  }
}

// ------------------------------------------------------------------ gathers
Tensor Shrinker::gather_flat(const Tensor& t, int dim, bool minus1) {
  const Tensor& idx = minus1 ? flat_m1_ : flat_;
  return t.index_select(dim, idx.to(t.device()));
}

// Per-batch gather of sequence dim `dim` with batch dim `bdim` in one index_select.
Tensor Shrinker::gather_seq(const Tensor& t, int dim, int bdim, bool minus1) {
  const Tensor& pos = minus1 ? pos_m1_ : pos_;
  if (B_ > 1 && bdim < 0 && dim != 0 && t.dim() >= 2 && t.size(0) == 1) {
    // a tensor broadcast over the batch (e.g. RoPE cos/sin [1, S, d]): rows keep different
    // positions, so materialise one row per batch entry before gathering
    std::vector<int64_t> shape = t.sizes().vec();
    shape[0] = B_;
    return gather_seq(t.expand(shape), dim, 0, minus1);
  }
  if (B_ > 1 && bdim < 0 && dim != 0 && t.dim() >= 2 && t.size(0) > B_ &&
      t.size(0) % B_ == 0) {
    // batch folded into dim 0, batch-major (the [B*heads, S, *] operands of a batched matmul
    // over [B, heads, S, *]): unfold it so that every sequence keeps its own positions (the
    // reference uses sequence 0's positions here, graph_filter.cpp:216-221), then fold back
    std::vector<int64_t> shape = t.sizes().vec();
    shape[0] = t.size(0) / B_;
    shape.insert(shape.begin(), B_);
    const Tensor r = gather_seq(t.reshape(shape), dim + 1, 0, minus1);
    std::vector<int64_t> out = r.sizes().vec();
    out[1] *= out[0];
    out.erase(out.begin());
    return r.reshape(out);
  }
  if (B_ == 1 || bdim < 0) {
    // no batch dimension: every row must share the kept positions; use row 0
    return t.index_select(dim, pos.select(0, 0).to(t.device()));
  }
  const int64_t nd = t.dim();
  std::vector<int64_t> perm;
  perm.push_back(bdim);
  perm.push_back(dim);
  for (int64_t i = 0; i < nd; ++i)
    if (i != bdim && i != dim) perm.push_back(i);
  std::vector<int64_t> inv(nd);
  for (int64_t i = 0; i < nd; ++i) inv[perm[i]] = i;
  const Tensor p = t.permute(perm);
  const int64_t L = t.size(dim);
  std::vector<int64_t> flat_shape = {B_ * L};
  for (int64_t i = 2; i < nd; ++i) flat_shape.push_back(p.size(i));
  const Tensor base = at::arange(B_, pos.options()).unsqueeze(1) * L;
  const Tensor rows = (pos + base).reshape({-1}).to(t.device());
  Tensor g = p.reshape(flat_shape).index_select(0, rows);
  std::vector<int64_t> out_shape = {B_, pos.size(1)};
  for (int64_t i = 2; i < nd; ++i) out_shape.push_back(p.size(i));
  Tensor r = g.view(out_shape).permute(inv);
  return t.is_contiguous() ? r.contiguous() : r;
}

Tensor Shrinker::shrink_tensor(const Tensor& t) {
  const DimRecord d = classify(t.sym_sizes());
  if (d.mode == SeqMode::kNone || d.index < 0) return t;
  auto key = std::make_tuple(t.const_data_ptr(), t.sizes().vec(), t.strides().vec());
  auto it = cache_.find(key);
  if (it != cache_.end()) return it->second;
  torch::NoGradGuard ng;
  Tensor r;
  switch (d.mode) {
    case SeqMode::kBatchSeq: r = gather_flat(t, d.index, false); break;
    case SeqMode::kBatchSeqMinus1: r = gather_flat(t, d.index, true); break;
    case SeqMode::kSeq:
    case SeqMode::kSeqMinus1: {
      const bool m1 = d.mode == SeqMode::kSeqMinus1;
      if (d.index < 10) {
        TORCH_CHECK(d.index < t.dim(), "backward_filter: replayed dim ", d.index,
                    " out of range for a ", t.dim(), "-d tensor");
        r = gather_seq(t, d.index, d.bsz_index, m1);
      } else {
        r = gather_seq(t, d.index % 10, d.bsz_index, m1);
        r = gather_seq(r, d.index / 10, d.bsz_index, m1);
      }
      break;
    }
    default: r = t;
  }
  cache_[key] = r;
  return r;
}

void Shrinker::shrink_saved(SavedVariable& sv, bool is_output, Node* owner) {
  Variable v;
  try {
    v = is_output ? sv.unpack(owner->getptr()) : sv.unpack();
  } catch (const c10::Error&) {
    return;  // saved data already released
  }
  if (!v.defined()) return;
  Tensor r = shrink_tensor(v);
  if (r.unsafeGetTensorImpl() == v.unsafeGetTensorImpl()) return;
  sv = SavedVariable(r, is_output);
}

void Shrinker::shrink_sizes(std::vector<c10::SymInt>& sizes) {
  const DimRecord d = classify(sizes);
  if (d.mode == SeqMode::kNone || d.index < 0) return;
  const int64_t n = new_extent(d.mode);
  if (d.index < 10) {
    if (d.index < static_cast<int>(sizes.size())) sizes[d.index] = n;
  } else {
    sizes[d.index % 10] = n;
    sizes[d.index / 10] = n;
  }
}

void Shrinker::shrink_sizes_list(std::vector<std::vector<c10::SymInt>>& list) {
  for (auto& sizes : list)
    if (sizes.size() > 1) shrink_sizes(sizes);
}

// Slice along the sequence dimension: an absolute end equal to the old extent (or extent - 1)
// is moved to the new extent (or new extent - 1); relative ends (-1, open) need nothing.
void Shrinker::shrink_slice(std::vector<c10::SymInt>& sizes, int64_t dim,
                            std::optional<c10::SymInt>& end) {
  const std::vector<c10::SymInt> before = sizes;
  shrink_sizes(sizes);
  const int64_t nd = static_cast<int64_t>(sizes.size());
  const int64_t d = dim < 0 ? dim + nd : dim;
  if (d < 0 || d >= nd || !end.has_value()) return;
  if (before[d] == sizes[d]) return;
  if (*end == before[d]) {
    end = sizes[d];
  } else if (*end == before[d] - 1) {
    end = sizes[d] - 1;
  }
}

void Shrinker::shrink_numel(c10::SymInt& n) {
  if (n % S_ == 0) n = Sk_ * (n / S_);
}

void Shrinker::shrink_input_metadata(Node* fn) {
  for (uint32_t i = 0; i < fn->num_inputs(); ++i) {
    const auto& meta = fn->input_metadata(i);
    if (meta.is_nested_tensor()) continue;
    std::vector<c10::SymInt> shape(meta.shape_as_dim_vector().begin(),
                                   meta.shape_as_dim_vector().end());
    const DimRecord d = classify(shape);
    if (d.mode == SeqMode::kNone || d.index < 0) continue;
    auto& dims = fn->mutable_input_metadata(i).mutable_shape_as_dim_vector();
    const int64_t n = new_extent(d.mode);
    if (d.index < 10) {
      if (d.index < static_cast<int>(dims.size())) dims[d.index] = n;
    } else {
      dims[d.index % 10] = n;
      dims[d.index / 10] = n;
    }
  }
}

}  // namespace cfb_filter
