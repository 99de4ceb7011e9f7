// qf_static.cu -- MoE block forward that allocates nothing.
//
// Some callers cannot call cudaMalloc at the point where they run the MoE
// block: an engine whose device memory is handed out by its own arena and
// forbids the CUDA allocator after start-up, a host runtime (a Swift or Go
// binding, a plugin) that owns no device allocator of its own, or code that
// must not touch the allocator inside a latency-critical step.  For them this
// file keeps the block's scratch in a file-scope device array that exists for
// as long as the library is loaded, so the call needs no handle, no workspace
// argument and no allocation of any kind.
//
// Limits and rules:
//   - at most kStaticMaxTokens (8) tokens per call; larger T returns QF_ERR_ARG;
//   - the array (kStaticScratchBytes = 1 MiB) is held on every GPU that loads
//     the library until the process exits;
//   - every call on a device shares the array: calls whose GPU work overlaps
//     (two streams, two threads) race and give undefined results;
//   - the array keeps the previous call's contents; the only field that must
//     start at zero (the device status word) is cleared by each call;
//   - the first call on a device does the set-up (the array's device address
//     via cudaGetSymbolAddress, kernel attributes); make that first call before
//     any stream capture.
#include <mutex>

#include "../../include/qf_moe.h"
#include "qf_handle.h"
#include "qf_internal.h"

namespace qf {

constexpr int kStaticMaxTokens = 8;
constexpr size_t kStaticStatusBytes = 256;
constexpr size_t kStaticScratchBytes = 1u << 20;  // 1 MiB: status word + block workspace(8)

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void* g_scratch_addr[kMaxDevices] = {};  // device address of g_static_scratch per device

// Once per device, with that device current: resolve the array's device
// address (the host-side symbol is only a stand-in) and set kernel attributes.
cudaError_t setup_device(int dev, void** addr) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_scratch_addr[dev] != nullptr) {
    *addr = g_scratch_addr[dev];
    return cudaSuccess;
  }
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
  if (e != cudaSuccess) return e;
  e = decode_init_attributes();
  if (e != cudaSuccess) return e;
  g_scratch_addr[dev] = p;
  *addr = p;
  return cudaSuccess;
}
}  // namespace

}  // namespace qf

extern "C" qf_status qf_moe_block_forward_static(int32_t scale_dtype, const qf_moe_layer* layer,
                                                 int32_t T, const uint16_t* x,
                                                 const float* residual, float* out,
                                                 int32_t* idx_out, float* w_out, void* stream) {
  if (T < 1 || T > qf::kStaticMaxTokens) return QF_ERR_ARG;
  if (scale_dtype != QF_SCALE_F16 && scale_dtype != QF_SCALE_BF16) return QF_ERR_ARG;
  if (!x || !out || (reinterpret_cast<uintptr_t>(x) % 16) != 0) return QF_ERR_ARG;
  // the same descriptor rules as qf_moe_block_forward: a descriptor rejected
  // there is rejected here, before anything is launched
  qf::LayerW w;
  if (qf::check_layer(layer, &w, nullptr) != QF_OK) return QF_ERR_ARG;
  if (qf::decode_workspace_bytes(T) + qf::kStaticStatusBytes > qf::kStaticScratchBytes)
    return QF_ERR_ARG;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= qf::kMaxDevices) return QF_ERR_CUDA;
  void* base = nullptr;
  if (qf::setup_device(dev, &base) != cudaSuccess) return QF_ERR_CUDA;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* status = static_cast<int*>(base);
  if (cudaMemsetAsync(status, 0, qf::kStaticStatusBytes, st) != cudaSuccess) return QF_ERR_CUDA;
  qf::DecodeWs ws;
  qf::decode_carve(static_cast<unsigned char*>(base) + qf::kStaticStatusBytes, T, &ws);
  qf::RoutingArgs r = {nullptr, nullptr, nullptr, nullptr};
  cudaError_t e = qf::decode_block(st, w, scale_dtype == QF_SCALE_BF16, T, x, residual, out, r,
                                   idx_out, w_out, ws, nullptr, 0.f, status, nullptr);
  return e == cudaSuccess ? QF_OK : QF_ERR_CUDA;
}
