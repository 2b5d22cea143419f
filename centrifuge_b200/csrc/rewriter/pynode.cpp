// Python autograd Function nodes (PyNode).
//
// * Native B200 nodes (class name prefix "_Cf", e.g. _CfLlamaFnBackward): their input metadata
//   is shrunk like any node's, then the Function's `cf_attach(ctx, mask)` is called so that
//   its backward runs on the kept rows with the fused kernels.
// * Megatron-style nodes (reference list, node_processing.cpp:369-427) and every PyNode named
//   in the target list: saved variables are shrunk, and the sizes in input_info / output_info.
#include <torch/csrc/autograd/python_cpp_function.h>
#include <torch/csrc/autograd/python_function.h>
#include <torch/csrc/autograd/python_variable.h>
#include <pybind11/pybind11.h>

#include <cstring>
#include <typeinfo>
#include <unordered_set>

#include "rewriter.h"

namespace cfb_filter {

static std::unordered_set<std::string>& pynode_targets() {
  static std::unordered_set<std::string> names = {
      "LinearWithGradAccumulationAndAsyncCommunicationBackward",
      "_ReduceFromModelParallelRegionBackward",
      "_GatherFromModelParallelRegionBackward",
      "_AllToAllBackward",
      "_LinearBackward",
      "_LayerNormLinearBackward",
      "_SplitAlongDimBackward",
      "FusedRoPEFuncBackward",
      "_ReduceScatterToSequenceParallelRegionBackward",
      "_VocabParallelCrossEntropyBackward",
      "MakeViewlessTensorBackward",
      "_LayerNormBackward",
      "CompiledFunctionBackward",
      "SwiGLUFunctionBackward",
      "FastLayerNormFNBackward",
      "ScaledUpperTriangMaskedSoftmaxBackward",
  };
  return names;
}

void add_pynode_targets(const std::vector<std::string>& names) {
  for (const auto& n : names) pynode_targets().insert(n);
}

// PyNode's type_info is not exported by libtorch_python, so the node type is recognised by
// the runtime type name and then cast statically (the layout comes from torch's header).
static bool is_pynode(Node* fn) {
  return std::strcmp(typeid(*fn).name(), "N5torch8autograd6PyNodeE") == 0;
}

bool process_pynode(Node* fn, Shrinker& s, const Tensor& mask) {
  if (!is_pynode(fn)) return false;
  auto* py = static_cast<torch::autograd::PyNode*>(fn);
  const std::string name = fn->name();
  if (name.rfind("_Cf", 0) == 0) {
    s.shrink_input_metadata(fn);
    pybind11::gil_scoped_acquire gil;
    PyObject* ctx = py->obj;
    PyObject* cls = PyObject_GetAttrString(ctx, "_forward_cls");
    if (cls == nullptr) throw pybind11::error_already_set();
    PyObject* m = THPVariable_Wrap(mask);
    PyObject* r = PyObject_CallMethod(cls, "cf_attach", "OO", ctx, m);
    Py_XDECREF(m);
    Py_DECREF(cls);
    if (r == nullptr) throw pybind11::error_already_set();
    Py_DECREF(r);
    return true;
  }
  s.shrink_input_metadata(fn);
  if (!pynode_targets().count(name)) return true;  // unknown PyNode: metadata only
  THPFunction* f = reinterpret_cast<THPFunction*>(py->obj);
  for (auto& sv : f->saved_variables) s.shrink_saved(sv, false, fn);
  for (auto& info : f->input_info) s.shrink_sizes(info.size);
  for (auto& info : f->output_info) s.shrink_sizes(info.size);
  return true;
}

}  // namespace cfb_filter
