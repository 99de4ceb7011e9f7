// qf_api.cu -- the C ABI declared in include/qf_moe.h: argument checks, device
// selection, error text, and dispatch to the kernels.
#include <stdio.h>
#include <string.h>

#include <string>
#include <vector>

#include "../../include/qf_moe.h"
#include "qf_handle.h"
#include "qf_internal.h"

namespace qf {
void prof_release(Prof* p);
}
using qf::prof_release;

namespace {

struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) {
      ok = false;
      return;
    }
    if (prev != dev && cudaSetDevice(dev) != cudaSuccess) ok = false;
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace

qf_status qf::fail(qf_moe* h, qf_status s, const char* fmt, const char* a) {
  if (h) {
    char buf[512];
    snprintf(buf, sizeof(buf), fmt, a);
    h->err = buf;
  }
  return s;
}

qf_status qf::cuda_fail(qf_moe* h, cudaError_t e, const char* where) {
  if (h) h->err = std::string(where) + ": " + cudaGetErrorString(e);
  return QF_ERR_CUDA;
}

namespace {
using qf::cuda_fail;
using qf::fail;

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

cudaStream_t stream_of(const qf_moe* h) { return h->stream; }

}  // namespace

qf_status qf::check_layer(const qf_moe_layer* l, qf::LayerW* w, const char** why) {
  auto bad = [&](const char* m) {
    if (why) *why = m;
    return QF_ERR_ARG;
  };
  if (!l) return bad("layer descriptor is NULL");
  if (!l->router_w || !l->router_s || !l->router_b || !l->coef_w || !l->coef_s || !l->coef_b ||
      !l->shared_record || !l->expert_bank)
    return bad("layer descriptor has a NULL weight pointer");
  if (l->record_stride < qf::kRecordBytes || (l->record_stride % 32) != 0)
    return bad("record_stride must be >= 1769472 and a multiple of 32");
  // the router and coefficient codes are read as uint4, their scales/biases as
  // 16-bit words (router rows 16 bytes at a time)
  if (!aligned(l->router_w, 16) || !aligned(l->coef_w, 16) || !aligned(l->router_s, 16) ||
      !aligned(l->router_b, 16) || !aligned(l->coef_s, 2) || !aligned(l->coef_b, 2))
    return bad("router/coefficient codes and router scales/biases must be 16-byte aligned, "
               "coefficient scales/biases 2-byte aligned");
  // expert codes are read 32 bytes at a time
  if (!aligned(l->shared_record, 32) || !aligned(l->expert_bank, 32))
    return bad("shared record and bank must be 32-byte aligned");
  if (l->bank_records == 0 || l->bank_records >= (1u << 23))
    return bad("bank_records must be in [1, 2^23)");
  if (l->reserved != 0) return bad("reserved field must be 0");
  w->rw = l->router_w;
  w->rs = l->router_s;
  w->rb = l->router_b;
  w->cw = l->coef_w;
  w->cs = l->coef_s;
  w->cb = l->coef_b;
  w->shared = l->shared_record;
  w->bank = l->expert_bank;
  w->stride = l->record_stride;
  w->bank_records = l->bank_records;
  return QF_OK;
}

qf_status qf::layer_to_w(qf_moe* h, const qf_moe_layer* l, qf::LayerW* w) {
  const char* why = "";
  qf_status s = check_layer(l, w, &why);
  return s == QF_OK ? QF_OK : fail(h, s, "%s", why);
}

namespace {
using qf::layer_to_w;

qf_status routing_args(qf_moe* h, const qf_routing* r, qf::RoutingArgs* a) {
  a->bias = nullptr;
  a->idx_in = nullptr;
  a->w_in = nullptr;
  a->rec_of_pos = nullptr;
  if (!r) return QF_OK;
  if ((r->topk_idx == nullptr) != (r->topk_w == nullptr))
    return fail(h, QF_ERR_ARG, "routing: topk_idx and topk_w must be given together");
  a->bias = r->logit_bias;
  a->idx_in = r->topk_idx;
  a->w_in = r->topk_w;
  a->rec_of_pos = r->record_of_pos;
  return QF_OK;
}

}  // namespace

extern "C" {

int qf_moe_abi_version(void) { return QF_MOE_ABI_VERSION; }

qf_status qf_moe_create(const qf_moe_dims* dims, int device, qf_moe** out) {
  if (!out) return QF_ERR_ARG;
  *out = nullptr;
  if (!dims) return QF_ERR_ARG;
  if (dims->hidden != qf::kHidden || dims->experts != qf::kExperts || dims->top_k != qf::kTopK ||
      dims->intermediate != qf::kInter || dims->group != qf::kGroup ||
      (dims->scale_dtype != QF_SCALE_F16 && dims->scale_dtype != QF_SCALE_BF16))
    return QF_ERR_ARG;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return QF_ERR_CUDA;
  DeviceGuard g(device);
  if (!g.ok) return QF_ERR_CUDA;
  qf_moe* h = new qf_moe();
  h->device = device;
  h->dims = *dims;
  h->stream = nullptr;
  if (cudaMalloc(&h->d_status, 256) != cudaSuccess) {
    delete h;
    return QF_ERR_OOM;
  }
  if (cudaMemset(h->d_status, 0, 256) != cudaSuccess || qf::decode_init_attributes() != cudaSuccess ||
      qf::fused_init_attributes() != cudaSuccess || qf::prefill_init_attributes() != cudaSuccess) {
    cudaFree(h->d_status);
    delete h;
    return QF_ERR_CUDA;
  }
  *out = h;
  return QF_OK;
}

void qf_moe_destroy(qf_moe* h) {
  if (!h) return;
  DeviceGuard g(h->device);
  prof_release(&h->prof);
  cudaFree(h->d_status);
  delete h;
}

qf_status qf_moe_set_stream(qf_moe* h, void* stream) {
  if (!h) return QF_ERR_ARG;
  h->stream = static_cast<cudaStream_t>(stream);
  return QF_OK;
}

const char* qf_last_error(const qf_moe* h) {
  if (!h) return "null handle";
  return h->err.c_str();
}

qf_status qf_moe_check(qf_moe* h) {
  if (!h) return QF_ERR_ARG;
  DeviceGuard g(h->device);
  cudaError_t e = cudaStreamSynchronize(stream_of(h));
  if (e != cudaSuccess) return cuda_fail(h, e, "qf_moe_check: stream");
  int st = 0;
  e = cudaMemcpy(&st, h->d_status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(h, e, "qf_moe_check: status");
  if (st != 0) {
    cudaMemset(h->d_status, 0, sizeof(int));
    if (st == QF_ERR_TIMEOUT) return fail(h, QF_ERR_TIMEOUT, "a bounded device wait expired");
    return fail(h, QF_ERR_DEVICE,
                "device status: an index or record id was out of range (the access was skipped)");
  }
  return QF_OK;
}

qf_status qf_router_logits_q8(qf_moe* h, const qf_moe_layer* layer, int32_t T, const uint16_t* x,
                              float* logits, float* coef) {
  if (!h) return QF_ERR_ARG;
  qf::LayerW w;
  qf_status s = layer_to_w(h, layer, &w);
  if (s != QF_OK) return s;
  if (T < 1 || T > 65536) return fail(h, QF_ERR_ARG, "T must be in [1, 65536]");
  if (!x || !logits || !aligned(x, 16)) return fail(h, QF_ERR_ARG, "x (16-B aligned) and logits are required");
  DeviceGuard g(h->device);
  const bool bf16 = h->dims.scale_dtype == QF_SCALE_BF16;
  cudaError_t e = T > qf::kDecodeMaxTokens
                      ? qf::router_logits_prefill(stream_of(h), w, bf16, T, x, logits, coef)
                      : qf::router_logits(stream_of(h), w, bf16, T, x, logits, coef, h->d_status);
  return e == cudaSuccess ? QF_OK : cuda_fail(h, e, "qf_router_logits_q8");
}

qf_status qf_moe_block_forward_prenorm(qf_moe* h, const qf_moe_layer* layer, int32_t T, const float* hidden,
                                       const float* norm_w, float eps, float* out, const qf_routing* routing,
                                       int32_t* idx_out, float* w_out, void* workspace, size_t workspace_bytes) {
  if (!h) return QF_ERR_ARG;
  if (T < 1 || T > qf::kPrefillMaxTokens) return fail(h, QF_ERR_ARG, "T must be in [1, 32768]");
  if (!hidden || !norm_w || !out) return fail(h, QF_ERR_ARG, "hidden, norm_w and out are required");
  size_t need = 0;
  qf_moe_workspace_size(h, T, &need);
  need = (need + 255) & ~size_t(255);
  const size_t x_bytes = (size_t)T * 2048 * 2;
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < need + x_bytes)
    return fail(h, QF_ERR_ARG, "workspace below qf_moe_workspace_size (rounded to 256) + T * 4096 bytes");
  uint16_t* x16 = reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(workspace) + need);
  if (T == 1 && h->prof.kernel < 0) {
    // one token: the norm runs in the one-token kernel's prologue
    qf::LayerW w;
    qf_status s = layer_to_w(h, layer, &w);
    if (s != QF_OK) return s;
    qf::RoutingArgs r;
    s = routing_args(h, routing, &r);
    if (s != QF_OK) return s;
    DeviceGuard g(h->device);
    const cudaError_t e = qf::fused1_stack(stream_of(h), &w, 1, h->dims.scale_dtype == QF_SCALE_BF16, nullptr,
                                           hidden, out, 1e-6f, r, idx_out, w_out, workspace, h->d_status,
                                           &h->prof, hidden, norm_w, eps);
    if (e != cudaErrorNotSupported) return e == cudaSuccess ? QF_OK : cuda_fail(h, e, "qf_moe_block_forward_prenorm");
  }
  {
    DeviceGuard g(h->device);
    const cudaError_t e = qf::prenorm_f16(stream_of(h), T, hidden, norm_w, eps, x16);
    if (e != cudaSuccess) return cuda_fail(h, e, "qf_moe_block_forward_prenorm");
  }
  return qf_moe_block_forward(h, layer, T, x16, hidden, out, routing, idx_out, w_out, workspace, need);
}

qf_status qf_lm_head_q4(qf_moe* h, const void* w, const void* scales, const void* biases, int32_t rows,
                        int32_t T, const float* x, float* logits) {
  if (!h) return QF_ERR_ARG;
  if (rows < 1 || T < 1 || T > 64) return fail(h, QF_ERR_ARG, "rows must be >= 1 and T in [1, 64]");
  if (!w || !scales || !biases || !x || !logits || !aligned(w, 16) || !aligned(scales, 16) ||
      !aligned(biases, 16) || !aligned(x, 16))
    return fail(h, QF_ERR_ARG, "w, scales, biases and x (16-B aligned) and logits are required");
  DeviceGuard g(h->device);
  int sms = 0;
  cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, h->device);
  const bool bf16 = h->dims.scale_dtype == QF_SCALE_BF16;
  // one token row per launch: the weights stream once per token
  for (int t = 0; t < T && e == cudaSuccess; t++)
    e = qf::lm_head_q4(stream_of(h), bf16, w, scales, biases, rows, x + (size_t)t * 2048,
                       logits + (size_t)t * rows, sms);
  return e == cudaSuccess ? QF_OK : cuda_fail(h, e, "qf_lm_head_q4");
}

qf_status qf_router_topk(qf_moe* h, const float* logits, const float* bias, int32_t T, int32_t* idx,
                         float* w) {
  if (!h) return QF_ERR_ARG;
  if (T < 1 || T > 65536) return fail(h, QF_ERR_ARG, "T must be in [1, 65536]");
  if (!logits || !idx || !w) return fail(h, QF_ERR_ARG, "logits, idx and w are required");
  DeviceGuard g(h->device);
  cudaError_t e = qf::router_topk(stream_of(h), T, logits, bias, idx, w, h->d_status);
  return e == cudaSuccess ? QF_OK : cuda_fail(h, e, "qf_router_topk");
}

qf_status qf_moe_routed_subset(qf_moe* h, const qf_moe_layer* layer, const uint16_t* x,
                               const int32_t* slot_of_pos, const float* w, const int32_t* positions,
                               int32_t n, float* routed_out, void* workspace, size_t workspace_bytes) {
  if (!h) return QF_ERR_ARG;
  qf::LayerW L;
  qf_status s = layer_to_w(h, layer, &L);
  if (s != QF_OK) return s;
  if (n < 0 || n > qf::kTopK) return fail(h, QF_ERR_ARG, "subset size n must be in [0, 8]");
  if (!x || !aligned(x, 16) || !routed_out || (n > 0 && (!slot_of_pos || !w || !positions)))
    return fail(h, QF_ERR_ARG, "x (16-B aligned), slot_of_pos, w, positions and routed_out are required");
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < qf::decode_workspace_bytes(1))
    return fail(h, QF_ERR_ARG, "workspace too small (qf_moe_workspace_size at T = 1) or not 256-byte aligned");
  DeviceGuard g(h->device);
  qf::DecodeWs ws;
  qf::decode_carve(workspace, 1, &ws);
  cudaError_t e = qf::routed_subset(stream_of(h), L, h->dims.scale_dtype == QF_SCALE_BF16, x, slot_of_pos, w,
                                    positions, n, routed_out, ws, h->d_status);
  return e == cudaSuccess ? QF_OK : cuda_fail(h, e, "qf_moe_routed_subset");
}

qf_status qf_shared_expert(qf_moe* h, const qf_moe_layer* layer, int32_t T, const uint16_t* x,
                           const float* coef, float* out, void* workspace, size_t workspace_bytes) {
  if (!h) return QF_ERR_ARG;
  qf::LayerW L;
  qf_status s = layer_to_w(h, layer, &L);
  if (s != QF_OK) return s;
  if (T < 1 || T > qf::kDecodeMaxTokens) return fail(h, QF_ERR_ARG, "T must be in [1, 64]");
  if (!x || !aligned(x, 16) || !coef || !out)
    return fail(h, QF_ERR_ARG, "x (16-B aligned), coef and out are required");
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < qf::decode_workspace_bytes(T))
    return fail(h, QF_ERR_ARG, "workspace too small (qf_moe_workspace_size at T) or not 256-byte aligned");
  DeviceGuard g(h->device);
  qf::DecodeWs ws;
  qf::decode_carve(workspace, T, &ws);
  cudaError_t e = qf::shared_expert(stream_of(h), L, h->dims.scale_dtype == QF_SCALE_BF16, T, x, coef, out, ws);
  return e == cudaSuccess ? QF_OK : cuda_fail(h, e, "qf_shared_expert");
}

qf_status qf_moe_combine(qf_moe* h, int32_t T, const float* residual, const float* shared_out,
                         const float* hit_out, const float* miss_out, float* out) {
  if (!h) return QF_ERR_ARG;
  if (T < 1 || T > 65536) return fail(h, QF_ERR_ARG, "T must be in [1, 65536]");
  if (!shared_out || !out) return fail(h, QF_ERR_ARG, "shared_out and out are required");
  DeviceGuard g(h->device);
  cudaError_t e = qf::combine_subsets(stream_of(h), T, residual, shared_out, hit_out, miss_out, out);
  return e == cudaSuccess ? QF_OK : cuda_fail(h, e, "qf_moe_combine");
}

qf_status qf_moe_grouped_ffn(qf_moe* h, const qf_moe_layer* layer, int32_t T, const uint16_t* x,
                             const int32_t* idx, float* y, void* workspace, size_t workspace_bytes) {
  if (!h) return QF_ERR_ARG;
  qf::LayerW L;
  qf_status s = layer_to_w(h, layer, &L);
  if (s != QF_OK) return s;
  if (T < 1 || T > qf::kPrefillMaxTokens) return fail(h, QF_ERR_ARG, "T must be in [1, 32768]");
  if (L.bank_records < static_cast<uint32_t>(qf::kExperts))
    return fail(h, QF_ERR_ARG, "the grouped FFN needs a resident bank of 256 experts");
  if (!x || !aligned(x, 16) || !idx || !y || !aligned(y, 16))
    return fail(h, QF_ERR_ARG, "x and y (16-B aligned) and idx are required");
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < qf::prefill_workspace_bytes(T))
    return fail(h, QF_ERR_ARG, "workspace too small (qf_moe_grouped_ffn_workspace_size) or not 256-byte aligned");
  DeviceGuard g(h->device);
  cudaError_t e = qf::grouped_ffn_routed(stream_of(h), L, h->dims.scale_dtype == QF_SCALE_BF16, T, x, idx, y,
                                         workspace, h->d_status, &h->prof);
  return e == cudaSuccess ? QF_OK : cuda_fail(h, e, "qf_moe_grouped_ffn");
}

qf_status qf_moe_grouped_ffn_workspace_size(qf_moe* h, int32_t T, size_t* bytes) {
  if (!h || !bytes) return QF_ERR_ARG;
  if (T < 1 || T > qf::kPrefillMaxTokens) return fail(h, QF_ERR_ARG, "T must be in [1, 32768]");
  *bytes = qf::prefill_workspace_bytes(T);
  return QF_OK;
}

qf_status qf_moe_dispatch_workspace_size(qf_moe* h, int32_t T, size_t* bytes) {
  if (!h || !bytes) return QF_ERR_ARG;
  if (T < 1 || T > 32768) return fail(h, QF_ERR_ARG, "T must be in [1, 32768]");
  *bytes = qf::dispatch_workspace_bytes(T);
  return QF_OK;
}

qf_status qf_moe_dispatch_plan(qf_moe* h, const int32_t* idx, int32_t T, int32_t* counts,
                               int32_t* offsets, int32_t* perm, void* workspace,
                               size_t workspace_bytes) {
  if (!h) return QF_ERR_ARG;
  if (T < 1 || T > 32768) return fail(h, QF_ERR_ARG, "T must be in [1, 32768]");
  if (!idx || !counts || !offsets || !perm) return fail(h, QF_ERR_ARG, "idx/counts/offsets/perm required");
  if (!workspace || workspace_bytes < qf::dispatch_workspace_bytes(T) || !aligned(workspace, 16))
    return fail(h, QF_ERR_ARG, "workspace too small or misaligned");
  DeviceGuard g(h->device);
  cudaError_t e = qf::dispatch_plan_ws(stream_of(h), idx, T, counts, offsets, perm,
                                       static_cast<int*>(workspace), h->d_status);
  return e == cudaSuccess ? QF_OK : cuda_fail(h, e, "qf_moe_dispatch_plan");
}

namespace {
size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }
// grouped path for a stack of T = 9..64 tokens: fp32 h and fp16 x ping-pong
// buffers, then one block's grouped-path workspace
size_t grouped_stack_bytes(int T) {
  const size_t th = static_cast<size_t>(T) * qf::kHidden;
  return 2 * al256(4 * th) + 2 * al256(2 * th) + qf::prefill_workspace_bytes(T);
}
}  // namespace

qf_status qf_moe_workspace_size(qf_moe* h, int32_t T, size_t* bytes) {
  if (!h || !bytes) return QF_ERR_ARG;
  if (T < 1 || T > qf::kPrefillMaxTokens) return fail(h, QF_ERR_ARG, "T must be in [1, 32768]");
  if (T > qf::kDecodeMaxTokens) {
    *bytes = qf::prefill_workspace_bytes(T);
    return QF_OK;
  }
  const size_t a = qf::decode_workspace_bytes(T);
  const size_t b = T <= qf::kFusedMaxTokens ? qf::fused_workspace_bytes(T) : grouped_stack_bytes(T);
  *bytes = a > b ? a : b;
  return QF_OK;
}

qf_status qf_moe_block_forward(qf_moe* h, const qf_moe_layer* layer, int32_t T, const uint16_t* x,
                               const float* residual, float* out, const qf_routing* routing,
                               int32_t* idx_out, float* w_out, void* workspace,
                               size_t workspace_bytes) {
  if (!h) return QF_ERR_ARG;
  qf::LayerW w;
  qf_status s = layer_to_w(h, layer, &w);
  if (s != QF_OK) return s;
  if (T < 1 || T > qf::kPrefillMaxTokens) return fail(h, QF_ERR_ARG, "T must be in [1, 32768]");
  if (!x || !out || !aligned(x, 16)) return fail(h, QF_ERR_ARG, "x (16-B aligned) and out are required");
  size_t need = 0;
  qf_moe_workspace_size(h, T, &need);
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < need)
    return fail(h, QF_ERR_ARG, "workspace too small or not 256-byte aligned");
  qf::RoutingArgs r;
  s = routing_args(h, routing, &r);
  if (s != QF_OK) return s;
  DeviceGuard g(h->device);
  const bool bf16 = h->dims.scale_dtype == QF_SCALE_BF16;
  cudaError_t e;
  if (T > qf::kDecodeMaxTokens) {
    if (w.bank_records < (uint32_t)qf::kExperts || r.rec_of_pos)
      return fail(h, QF_ERR_ARG, "the prefill path needs a resident bank of 256 experts");
    e = qf::prefill_block(stream_of(h), w, bf16, T, x, residual, out, r, idx_out, w_out, workspace,
                          h->d_status, &h->prof);
  } else if (T <= qf::kFusedMaxTokens && (h->prof.kernel < 0 || h->prof.kernel == qf::kKFused)) {
    if (workspace_bytes < qf::fused_workspace_bytes(T))
      return fail(h, QF_ERR_ARG, "workspace too small");
    e = qf::fused_stack(stream_of(h), &w, 1, bf16, T, x, residual, out, 1e-6f, r, idx_out, w_out,
                        workspace, h->d_status, &h->prof);
  } else if (T >= qf::kGroupedMinTokens && w.bank_records >= (uint32_t)qf::kExperts && !r.rec_of_pos) {
    e = qf::prefill_block(stream_of(h), w, bf16, T, x, residual, out, r, idx_out, w_out, workspace,
                          h->d_status, &h->prof);
  } else {
    qf::DecodeWs ws;
    qf::decode_carve(workspace, T, &ws);
    e = qf::decode_block(stream_of(h), w, bf16, T, x, residual, out, r, idx_out, w_out, ws,
                         nullptr, 0.f, h->d_status, &h->prof);
  }
  return e == cudaSuccess ? QF_OK : cuda_fail(h, e, "qf_moe_block_forward");
}

qf_status qf_moe_stack_forward(qf_moe* h, const qf_moe_layer* layers, int32_t n_layers, int32_t T,
                               const uint16_t* x, const float* residual, float* out, float eps,
                               int32_t* idx_out, float* w_out, void* workspace,
                               size_t workspace_bytes) {
  if (!h) return QF_ERR_ARG;
  if (!layers || n_layers < 1) return fail(h, QF_ERR_ARG, "layers array and n_layers >= 1 required");
  if (T < 1 || T > qf::kDecodeMaxTokens)
    return fail(h, QF_ERR_ARG, "T must be in [1, 64] (decode path)");
  if (!x || !out || !aligned(x, 16)) return fail(h, QF_ERR_ARG, "x (16-B aligned) and out are required");
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < qf::decode_workspace_bytes(T))
    return fail(h, QF_ERR_ARG, "workspace too small or not 256-byte aligned");
  if (!(eps > 0.f)) return fail(h, QF_ERR_ARG, "eps must be > 0");
  size_t need = 0;
  qf_moe_workspace_size(h, T, &need);
  if (workspace_bytes < need) return fail(h, QF_ERR_ARG, "workspace too small");
  std::vector<qf::LayerW> lw(n_layers);
  for (int l = 0; l < n_layers; l++) {
    qf_status s = layer_to_w(h, &layers[l], &lw[l]);
    if (s != QF_OK) return s;
  }
  qf::RoutingArgs r = {nullptr, nullptr, nullptr, nullptr};
  DeviceGuard g(h->device);
  const bool bf16 = h->dims.scale_dtype == QF_SCALE_BF16;
  if (T <= qf::kFusedMaxTokens && (h->prof.kernel < 0 || h->prof.kernel == qf::kKFused)) {
    cudaError_t e = qf::fused_stack(stream_of(h), lw.data(), n_layers, bf16, T, x, residual, out,
                                    eps, r, idx_out, w_out, workspace, h->d_status, &h->prof);
    return e == cudaSuccess ? QF_OK : cuda_fail(h, e, "qf_moe_stack_forward");
  }
  const size_t PT = static_cast<size_t>(T) * qf::kTopK;
  bool resident = T >= qf::kGroupedMinTokens;
  for (int l = 0; l < n_layers && resident; l++) resident = lw[l].bank_records >= (uint32_t)qf::kExperts;
  if (resident) {
    // grouped path per block; its combine also writes the next block's RMSNorm
    // input (same order as the decode kernels)
    const size_t th = static_cast<size_t>(T) * qf::kHidden;
    char* p = static_cast<char*>(workspace);
    float* hb[2] = {reinterpret_cast<float*>(p), reinterpret_cast<float*>(p + al256(4 * th))};
    p += 2 * al256(4 * th);
    uint16_t* xb[2] = {reinterpret_cast<uint16_t*>(p), reinterpret_cast<uint16_t*>(p + al256(2 * th))};
    p += 2 * al256(2 * th);
    for (int l = 0; l < n_layers; l++) {
      const int cur = l & 1;
      const uint16_t* xin = (l == 0) ? x : xb[cur];
      const float* res = (l == 0) ? residual : hb[cur];
      float* o = (l == n_layers - 1) ? out : hb[cur ^ 1];
      cudaError_t e = qf::prefill_block(stream_of(h), lw[l], bf16, T, xin, res, o, r,
                                        idx_out ? idx_out + l * PT : nullptr,
                                        w_out ? w_out + l * PT : nullptr, p, h->d_status, &h->prof,
                                        l + 1 < n_layers ? xb[cur ^ 1] : nullptr, eps);
      if (e != cudaSuccess) return cuda_fail(h, e, "qf_moe_stack_forward");
    }
    return QF_OK;
  }
  qf::DecodeWs ws;
  qf::decode_carve(workspace, T, &ws);
  for (int l = 0; l < n_layers; l++) {
    const int cur = l & 1;
    const uint16_t* xin = (l == 0) ? x : ws.x16[cur];
    const float* res = (l == 0) ? residual : ws.h[cur];
    float* o = (l == n_layers - 1) ? out : ws.h[cur ^ 1];
    uint16_t* xn = (l == n_layers - 1) ? nullptr : ws.x16[cur ^ 1];
    cudaError_t e = qf::decode_block(stream_of(h), lw[l], bf16, T, xin, res, o, r,
                                     idx_out ? idx_out + l * PT : nullptr,
                                     w_out ? w_out + l * PT : nullptr, ws, xn, eps, h->d_status,
                                     &h->prof);
    if (e != cudaSuccess) return cuda_fail(h, e, "qf_moe_stack_forward");
  }
  return QF_OK;
}

qf_status qf_synth_records(qf_moe* h, uint64_t seed, uint32_t layer, uint32_t expert0,
                           uint32_t count, uint8_t* bank, uint64_t stride) {
  if (!h) return QF_ERR_ARG;
  if (!bank || count == 0 || stride < qf::kRecordBytes || stride % 16 || !aligned(bank, 16) ||
      expert0 + count > 257u)
    return fail(h, QF_ERR_ARG, "bad synth_records arguments");
  DeviceGuard g(h->device);
  cudaError_t e = qf::synth_records(stream_of(h), seed, layer, expert0, count, bank, stride,
                                    h->dims.scale_dtype == QF_SCALE_BF16);
  return e == cudaSuccess ? QF_OK : cuda_fail(h, e, "qf_synth_records");
}

qf_status qf_synth_router(qf_moe* h, uint64_t seed, uint32_t layer, uint8_t* w, uint16_t* s,
                          uint16_t* b) {
  if (!h) return QF_ERR_ARG;
  if (!w || !s || !b || !aligned(w, 8) || !aligned(s, 2) || !aligned(b, 2))
    return fail(h, QF_ERR_ARG, "bad synth_router arguments");
  DeviceGuard g(h->device);
  cudaError_t e = qf::synth_q8(stream_of(h), seed, layer, true, w, s, b,
                               h->dims.scale_dtype == QF_SCALE_BF16);
  return e == cudaSuccess ? QF_OK : cuda_fail(h, e, "qf_synth_router");
}

qf_status qf_synth_coef(qf_moe* h, uint64_t seed, uint32_t layer, uint8_t* w, uint16_t* s,
                        uint16_t* b) {
  if (!h) return QF_ERR_ARG;
  if (!w || !s || !b || !aligned(w, 8) || !aligned(s, 2) || !aligned(b, 2))
    return fail(h, QF_ERR_ARG, "bad synth_coef arguments");
  DeviceGuard g(h->device);
  cudaError_t e = qf::synth_q8(stream_of(h), seed, layer, false, w, s, b,
                               h->dims.scale_dtype == QF_SCALE_BF16);
  return e == cudaSuccess ? QF_OK : cuda_fail(h, e, "qf_synth_coef");
}

}  // extern "C"

void qf::prof_release(qf::Prof* p) {
  for (int i = 0; i < p->cap; i++) {
    cudaEventDestroy(p->ev0[i]);
    cudaEventDestroy(p->ev1[i]);
  }
  delete[] p->ev0;
  delete[] p->ev1;
  *p = qf::Prof();
}

extern "C" {

qf_status qf_moe_profile_begin(qf_moe* h, int32_t kernel_id, int32_t max_launches) {
  if (!h) return QF_ERR_ARG;
  if (kernel_id < 0 || kernel_id > 6 || max_launches < 1 || max_launches > 65536)
    return fail(h, QF_ERR_ARG, "kernel_id in [0,6], max_launches in [1,65536]");
  DeviceGuard g(h->device);
  prof_release(&h->prof);
  h->prof.ev0 = new cudaEvent_t[max_launches];
  h->prof.ev1 = new cudaEvent_t[max_launches];
  for (int i = 0; i < max_launches; i++) {
    if (cudaEventCreate(&h->prof.ev0[i]) != cudaSuccess ||
        cudaEventCreate(&h->prof.ev1[i]) != cudaSuccess) {
      h->prof.cap = i;
      prof_release(&h->prof);
      return fail(h, QF_ERR_CUDA, "cudaEventCreate failed");
    }
  }
  h->prof.cap = max_launches;
  h->prof.n = 0;
  h->prof.kernel = kernel_id;
  return QF_OK;
}

qf_status qf_moe_profile_end(qf_moe* h, float* total_ms, int32_t* launches) {
  if (!h || !total_ms || !launches) return QF_ERR_ARG;
  DeviceGuard g(h->device);
  float tot = 0.f;
  const int n = h->prof.n;
  for (int i = 0; i < n; i++) {
    cudaError_t e = cudaEventSynchronize(h->prof.ev1[i]);
    float ms = 0.f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, h->prof.ev0[i], h->prof.ev1[i]);
    if (e != cudaSuccess) {
      prof_release(&h->prof);
      return cuda_fail(h, e, "qf_moe_profile_end");
    }
    tot += ms;
  }
  prof_release(&h->prof);
  *total_ms = tot;
  *launches = n;
  return QF_OK;
}

void qf_synth_hidden_host(uint64_t seed, uint64_t tok0, int32_t T, uint16_t* x) {
  if (!x || T < 1) return;
  qf::synth_hidden_host(seed, tok0, T, x);
}

}  // extern "C"
