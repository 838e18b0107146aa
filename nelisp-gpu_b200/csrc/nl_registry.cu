// nl_registry.cu -- the kernel registry: the reference's DSL kernel names
// (lisp/nelisp-gpu-kernels.el) mapped to their CUDA implementations.
//
// vkserver looks a kernel up by name and loads <dir>/<name>.spv on first use
// (host/vkserver.c:247-272); here every kernel is compiled into the library
// and the name selects it.
#include <string.h>

#include "nl_internal.h"

namespace nl {
namespace {

struct Table {
  const OpSpec *ops;
  const int *count;
};

const Table kTables[] = {
    {kTernaryOps, &kTernaryOpsCount}, {kInt8Ops, &kInt8OpsCount},
    {kDenseOps, &kDenseOpsCount},     {kRowOps, &kRowOpsCount},
    {kAttnOps, &kAttnOpsCount},       {kKvOps, &kKvOpsCount},
    {kMiscOps, &kMiscOpsCount},       {kQuantOps, &kQuantOpsCount},
    {kTrainOps, &kTrainOpsCount},
};

}  // namespace

int op_count() {
  int n = 0;
  for (const Table &t : kTables) n += *t.count;
  return n;
}

const OpSpec *op_at(int index) {
  if (index < 0) return nullptr;
  for (const Table &t : kTables) {
    if (index < *t.count) return &t.ops[index];
    index -= *t.count;
  }
  return nullptr;
}

const OpSpec *find_op(const char *name) {
  if (!name) return nullptr;
  for (const Table &t : kTables)
    for (int i = 0; i < *t.count; i++)
      if (strcmp(t.ops[i].name, name) == 0) return &t.ops[i];
  return nullptr;
}

}  // namespace nl
