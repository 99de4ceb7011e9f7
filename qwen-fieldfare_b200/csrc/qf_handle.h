// qf_handle.h -- the qf_moe handle and the argument helpers shared by the
// C-ABI translation units (qf_api.cu, qf_cache.cu).
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "../../include/qf_moe.h"
#include "qf_internal.h"

struct qf_moe {
  int device;
  qf_moe_dims dims;
  cudaStream_t stream;
  int* d_status;
  std::string err;
  qf::Prof prof;
};

namespace qf {
// Sets the handle's error text (printf-style with one string argument).
qf_status fail(qf_moe* h, qf_status s, const char* fmt, const char* a = "");
qf_status cuda_fail(qf_moe* h, cudaError_t e, const char* where);
// Checks one layer descriptor (pointers, alignment, stride, bank size) and
// converts it for the kernels; on failure *why names the broken rule.  Needs
// no handle: the allocation-free entry applies the same rules.
qf_status check_layer(const qf_moe_layer* l, LayerW* w, const char** why);
// check_layer with the failure text stored in the handle.
qf_status layer_to_w(qf_moe* h, const qf_moe_layer* l, LayerW* w);
}  // namespace qf
