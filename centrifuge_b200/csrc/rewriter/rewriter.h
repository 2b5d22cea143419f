// Autograd-graph rewriter behind token_filter::backward_filter (module centrifuge_b200._filter_C).
//
// Before loss.backward(), the rewriter walks the autograd graph of `loss` and makes every
// backward node work on the kept token rows only:
//   * saved tensors with a sequence dimension are replaced by their kept rows,
//   * saved size vectors / numels and the nodes' input metadata are shrunk from S to S_keep,
//   * attention backward nodes are replaced by a filtered ("restore-Q") attention node,
//   * native B200 model nodes (Python autograd Functions named "_Cf...") get the keep mask
//     attached and filter themselves.
// Behavioural reference: grad_filter/token_filter/csrc/{backward_filter_api,graph_filter,
// node_processing,edge_processing,backward_filters}.cpp.  The sequence-dimension detection
// modes and the per-node dims text format are kept so that recorded dims can be replayed.
#pragma once

#include <torch/csrc/autograd/function.h>
#include <torch/csrc/autograd/generated/Functions.h>
#include <torch/csrc/autograd/saved_variable.h>
#include <torch/extension.h>

#include <deque>
#include <functional>
#include <map>
#include <string>
#include <unordered_map>
#include <vector>

namespace cfb_filter {

using torch::autograd::Edge;
using torch::autograd::Node;
using torch::autograd::SavedVariable;
using torch::autograd::Variable;
using at::Tensor;

// How a sequence dimension was recognised (integer values are the dims-text encoding).
enum class SeqMode : int {
  kBatchSeq = 0,         // dim == B * S           (flattened tokens)
  kBatchSeqMinus1 = 1,   // dim == B * (S - 1)     (flattened loss positions)
  kSeq = 2,              // dim == S (two such dims: index = a + 10 * b)
  kSeqMinus1 = 3,        // dim == S - 1           (per-token loss)
  kNone = 4,
};

struct DimRecord {
  int index = -1;      // dim, or a + 10*b for two sequence dims
  int bsz_index = -1;  // batch dim, -1 if none
  SeqMode mode = SeqMode::kNone;
};

struct NodeRecord {
  std::string name;
  std::deque<DimRecord> dims;
};

// Mask state + the per-call record/replay of sequence-dimension decisions.
class Shrinker {
 public:
  explicit Shrinker(const Tensor& mask);

  // Recording (probe) vs replay of a dims text.
  void load_dims(const std::string& text);
  std::string dims_text() const;
  bool replay() const { return replay_; }
  void begin_node(const std::string& name);
  void end_node();

  // Decide (or replay) which dimension of `sizes` is the sequence dimension.
  DimRecord classify(c10::ArrayRef<c10::SymInt> sizes);

  // Saved tensors / metadata.
  Tensor shrink_tensor(const Tensor& t);
  void shrink_saved(SavedVariable& sv, bool is_output, Node* owner);
  void shrink_sizes(std::vector<c10::SymInt>& sizes);
  void shrink_numel(c10::SymInt& n);
  void shrink_sizes_list(std::vector<std::vector<c10::SymInt>>& list);
  void shrink_slice(std::vector<c10::SymInt>& sizes, int64_t dim,
                    std::optional<c10::SymInt>& end);
  void shrink_input_metadata(Node* fn);

  // Index tensors (on the mask's device).
  int64_t B() const { return B_; }
  int64_t S() const { return S_; }
  int64_t S_keep() const { return Sk_; }
  const Tensor& mask() const { return mask_; }
  const Tensor& pos() const { return pos_; }             // [B, Sk] int64
  const Tensor& pos_m1() const { return pos_m1_; }       // [B, Sk-1] int64 (< S-1)
  const Tensor& flat_rows() const { return flat_; }      // [B*Sk] b*S + pos
  const Tensor& flat_rows_m1() const { return flat_m1_; }  // [B*(Sk-1)] b*(S-1) + pos

  int processed_nodes = 0;

 private:
  Tensor gather_seq(const Tensor& t, int dim, int bdim, bool minus1);
  Tensor gather_flat(const Tensor& t, int dim, bool minus1);
  int64_t new_extent(SeqMode mode) const;

  Tensor mask_, pos_, pos_m1_, flat_, flat_m1_;
  int64_t B_ = 0, S_ = 0, Sk_ = 0;
  bool replay_ = false;
  std::vector<NodeRecord> records_;
  size_t cursor_ = 0;       // replay: index of the current node record
  NodeRecord* current_ = nullptr;
  std::map<std::tuple<const void*, std::vector<int64_t>, std::vector<int64_t>>, Tensor> cache_;
};

using Handler = void (*)(Node*, Shrinker&);
using HandlerTable = std::unordered_map<std::string, Handler>;

// Generated from target_node_names.yaml and the installed torch's derivatives.yaml.
void register_generated_handlers(HandlerTable& table);

// Line splitter shared by the dims-text readers.
std::vector<std::string> split_lines(const std::string& text);
std::vector<std::string> generated_handler_names();

// Attention nodes: shrink + replace the incoming edge's function with a filtered node.
bool is_attention_node(const std::string& name);
void replace_attention_edge(Edge& edge, Shrinker& s);

// Python autograd Function nodes (PyNode): native "_Cf" nodes get the mask; listed Megatron
// style nodes get their saved variables / input-output info shrunk.
bool process_pynode(Node* fn, Shrinker& s, const Tensor& mask);

}  // namespace cfb_filter
