// Build shim for compiling the reference's grad_filter extension against torch 2.11 without
// editing its sources.  Force-included (`-include`) ahead of every translation unit.
//
// torch 2.11 added a fifth parameter to Node::add_input_metadata (the gradient dtype the
// engine checks incoming gradients against).  The reference (written for torch 2.8) calls the
// 4-argument form once, in grad_filter/token_filter/csrc/node_processing.cpp:13, to copy input
// metadata between nodes.  The torch headers are included here first, so their own calls are
// already parsed; the macro below then rewrites only the reference's 4-argument call to pass
// the dtype of the copied options, which is the dtype torch 2.8 validated against.
#pragma once
#include <torch/extension.h>
#include <torch/csrc/autograd/function.h>
#include <torch/csrc/autograd/generated/Functions.h>
#include <torch/csrc/autograd/python_function.h>
#include <ATen/ATen.h>

#define add_input_metadata(opts, shape, is_subclass, is_nested) \
  add_input_metadata(opts, shape, is_subclass, is_nested,       \
                     c10::typeMetaToScalarType((opts).dtype()))
