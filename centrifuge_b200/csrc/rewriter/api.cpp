// token_filter operators: backward_filter, backward_filter_with_dims, collect_node_names.
//
// Schemas and the dims text format are those of the reference (grad_filter/token_filter/csrc/
// backward_filter_api.cpp:291-307, ops.py:9-55).  The walk is a breadth-first pass over the
// nodes reachable from loss.grad_fn; each node is processed once, attention nodes are replaced
// on the edge that reaches them (every edge that points at a replaced node is redirected).
#include <pybind11/stl.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <deque>
#include <unordered_set>

#include "rewriter.h"

namespace cfb_filter {

void add_pynode_targets(const std::vector<std::string>& names);

namespace {

HandlerTable& handlers() {
  static HandlerTable t = [] {
    HandlerTable h;
    register_generated_handlers(h);
    return h;
  }();
  return t;
}

bool verbose() {
  static const bool v = std::getenv("CFB_FILTER_VERBOSE") != nullptr;
  return v;
}

void process_node(Node* fn, Shrinker& s, const Tensor& mask) {
  if (verbose()) std::fprintf(stderr, "[backward_filter] node %s\n", fn->name().c_str());
  s.begin_node(fn->name());
  if (!process_pynode(fn, s, mask)) {
    s.shrink_input_metadata(fn);
    auto it = handlers().find(fn->name());
    if (it != handlers().end()) it->second(fn, s);
  }
  s.end_node();
  if (verbose()) std::fprintf(stderr, "[backward_filter] done %s\n", fn->name().c_str());
}

// Names of nodes in the order the rewrite visits them (attention replacements included).
std::vector<std::string> visit_order(Node* root) {
  std::vector<std::string> names;
  std::unordered_set<Node*> seen;
  std::deque<Node*> q{root};
  while (!q.empty()) {
    Node* fn = q.front();
    q.pop_front();
    if (!seen.insert(fn).second) continue;
    names.push_back(fn->name());
    for (auto& e : fn->next_edges()) {
      if (!e.function) continue;
      if (is_attention_node(e.function->name()) && !seen.count(e.function.get())) {
        names.push_back(e.function->name());
        seen.insert(e.function.get());
        for (auto& ce : e.function->next_edges())
          if (ce.function) q.push_back(ce.function.get());
        continue;
      }
      q.push_back(e.function.get());
    }
  }
  return names;
}

std::vector<std::string> record_names(const std::string& dims) {
  std::vector<std::string> out;
  bool expect_name = true;
  for (const auto& line : split_lines(dims)) {
    if (line == "---") {
      expect_name = true;
      continue;
    }
    if (expect_name && !line.empty()) {
      out.push_back(line);
      expect_name = false;
    }
  }
  return out;
}

std::string rewrite(const Tensor& loss, const Tensor& mask, const std::string& dims_in) {
  TORCH_CHECK(loss.grad_fn() != nullptr, "backward_filter: loss has no autograd graph");
  torch::NoGradGuard ng;
  Shrinker s(mask);
  if (!dims_in.empty()) s.load_dims(dims_in);
  std::unordered_set<Node*> seen;
  std::unordered_map<Node*, std::shared_ptr<Node>> replaced;
  std::deque<Node*> q{loss.grad_fn().get()};
  while (!q.empty()) {
    Node* fn = q.front();
    q.pop_front();
    if (!seen.insert(fn).second) continue;
    process_node(fn, s, mask);
    for (auto& e : fn->next_edges()) {
      if (!e.function) continue;
      Node* nf = e.function.get();
      auto r = replaced.find(nf);
      if (r != replaced.end()) {
        e.function = r->second;
        continue;
      }
      if (is_attention_node(nf->name()) && !seen.count(nf)) {
        auto old = e.function;  // keep the original alive while it is being replaced
        seen.insert(nf);
        if (verbose()) std::fprintf(stderr, "[backward_filter] replace %s\n", nf->name().c_str());
        s.begin_node(nf->name());
        replace_attention_edge(e, s);
        s.end_node();
        replaced[nf] = e.function;
        seen.insert(e.function.get());
        for (auto& ce : e.function->next_edges())
          if (ce.function) q.push_back(ce.function.get());
        continue;
      }
      q.push_back(nf);
    }
  }
  if (verbose()) std::fprintf(stderr, "[backward_filter] walk finished\n");
  return s.dims_text();
}

std::string dims_file() {
  const char* p = std::getenv("CFB_NODE_TRACING_FILE");
  return p ? std::string(p) : std::string("/tmp/node_tracing.txt");
}

}  // namespace

// backward_filter(loss, mask): rewrite using the cached dims file when it describes this
// graph (same node sequence), otherwise record and (re)write the cache.
at::Tensor backward_filter(at::Tensor loss, at::Tensor mask) {
  const std::string path = dims_file();
  std::string cached;
  if (FILE* f = std::fopen(path.c_str(), "rb")) {
    char buf[1 << 16];
    size_t n;
    while ((n = std::fread(buf, 1, sizeof(buf), f)) > 0) cached.append(buf, n);
    std::fclose(f);
  }
  if (!cached.empty() && record_names(cached) != visit_order(loss.grad_fn().get()))
    cached.clear();
  const std::string dims = rewrite(loss, mask, cached);
  if (cached.empty()) {
    if (FILE* f = std::fopen(path.c_str(), "wb")) {
      std::fwrite(dims.data(), 1, dims.size(), f);
      std::fclose(f);
    }
  }
  return loss;
}

std::string backward_filter_with_dims(at::Tensor loss, at::Tensor mask, std::string dims) {
  const std::string in = dims;
  const std::string out = rewrite(loss, mask, dims);
  return in.empty() ? out : in;
}

std::vector<std::string> collect_node_names(at::Tensor loss) {
  TORCH_CHECK(loss.grad_fn() != nullptr, "collect_node_names: loss has no autograd graph");
  std::unordered_set<std::string> names;
  std::unordered_set<Node*> seen;
  std::deque<Node*> q{loss.grad_fn().get()};
  while (!q.empty()) {
    Node* fn = q.front();
    q.pop_front();
    if (!seen.insert(fn).second) continue;
    names.insert(fn->name());
    for (auto& e : fn->next_edges())
      if (e.function) q.push_back(e.function.get());
  }
  std::vector<std::string> out(names.begin(), names.end());
  std::sort(out.begin(), out.end());
  return out;
}

}  // namespace cfb_filter

TORCH_LIBRARY(token_filter, m) {
  m.def("backward_filter(Tensor loss, Tensor mask) -> Tensor");
  m.def("backward_filter_with_dims(Tensor loss, Tensor mask, str input_node_filter_dims) -> str");
  m.def("collect_node_names(Tensor loss) -> str[]");
}

namespace cfb_filter {
namespace {

// Tensors of a tracer (FakeTensor and other Python-dispatched tensors, meta tensors) have no
// autograd graph to rewrite: their calls go below autograd to the fake kernels registered from
// Python (centrifuge_b200.filter), which is what torch.compile's tracing sees.
bool traced(const at::Tensor& t) {
  return t.defined() && (t.is_meta() || t.key_set().has(c10::DispatchKey::Python));
}

c10::OperatorHandle op_handle(const char* name) {
  return c10::Dispatcher::singleton().findSchemaOrThrow(name, "");
}

// The rewrite runs at the autograd key: it reads and edits the graph behind loss.grad_fn and
// returns the loss itself, so nothing below autograd is involved for real tensors.
at::Tensor backward_filter_ad(at::Tensor loss, at::Tensor mask) {
  if (traced(loss) || traced(mask)) {
    at::AutoDispatchBelowADInplaceOrView guard;
    static auto op = op_handle("token_filter::backward_filter")
                         .typed<at::Tensor(at::Tensor, at::Tensor)>();
    return op.call(loss, mask);
  }
  return backward_filter(loss, mask);
}

std::string backward_filter_with_dims_ad(at::Tensor loss, at::Tensor mask, std::string dims) {
  if (traced(loss) || traced(mask)) {
    at::AutoDispatchBelowADInplaceOrView guard;
    static auto op = op_handle("token_filter::backward_filter_with_dims")
                         .typed<std::string(at::Tensor, at::Tensor, std::string)>();
    return op.call(loss, mask, dims);
  }
  return backward_filter_with_dims(loss, mask, dims);
}

std::vector<std::string> collect_node_names_ad(at::Tensor loss) {
  if (traced(loss)) {
    at::AutoDispatchBelowADInplaceOrView guard;
    static auto op = op_handle("token_filter::collect_node_names")
                         .typed<std::vector<std::string>(at::Tensor)>();
    return op.call(loss);
  }
  return collect_node_names(loss);
}

}  // namespace
}  // namespace cfb_filter

TORCH_LIBRARY_IMPL(token_filter, Autograd, m) {
  m.impl("backward_filter", &cfb_filter::backward_filter_ad);
  m.impl("backward_filter_with_dims", &cfb_filter::backward_filter_with_dims_ad);
  m.impl("collect_node_names", &cfb_filter::collect_node_names_ad);
}

// Tensors without autograd keys (inference mode) reach the backend kernels directly.
TORCH_LIBRARY_IMPL(token_filter, CPU, m) {
  m.impl("backward_filter", &cfb_filter::backward_filter);
  m.impl("backward_filter_with_dims", &cfb_filter::backward_filter_with_dims);
  m.impl("collect_node_names", &cfb_filter::collect_node_names);
}

TORCH_LIBRARY_IMPL(token_filter, CUDA, m) {
  m.impl("backward_filter", &cfb_filter::backward_filter);
  m.impl("backward_filter_with_dims", &cfb_filter::backward_filter_with_dims);
  m.impl("collect_node_names", &cfb_filter::collect_node_names);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "autograd-graph rewriter of centrifuge_b200 (token_filter operators)";
  m.def("generated_handler_names", &cfb_filter::generated_handler_names);
  m.def("add_pynode_targets", &cfb_filter::add_pynode_targets);
}
