// qf_internal.h -- host-side declarations shared by the library's translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "qf_common.cuh"

namespace qf {

// ---- synthetic data (qf_synth.cu)
cudaError_t synth_records(cudaStream_t st, uint64_t seed, uint32_t layer, uint32_t expert0,
                          uint32_t count, uint8_t* bank, uint64_t stride, bool bf16);
cudaError_t synth_q8(cudaStream_t st, uint64_t seed, uint32_t layer, bool router, uint8_t* w,
                     uint16_t* s, uint16_t* b, bool bf16);
void synth_hidden_host(uint64_t seed, uint64_t tok0, int T, uint16_t* x);

// ---- decode path (qf_decode.cu)
struct DecodeWs {
  float* logits;      // [T, 256]
  float* coef;        // [T]
  int* idx;           // [T, 8]
  float* w;           // [T, 8]
  int* meta;          // [0] = n_groups
  int* group_rec;     // [512]
  int* group_start;   // [512]
  int* group_cnt;     // [512]
  int* sorted_pos;    // [512]
  float* act;         // [T*8, 512]
  float* act_sh;      // [T, 512]
  float* y_part;      // [T*8, 2048]
  float* y_sh;        // [T, 2048]
  float* h[2];        // stack residual ping-pong [T, 2048]
  uint16_t* x16[2];   // stack input ping-pong [T, 2048]
};

size_t decode_workspace_bytes(int T);
// Subset pieces of the streaming runner (T = 1 for routed_subset).
cudaError_t routed_subset(cudaStream_t st, const LayerW& L, bool bf16, const uint16_t* x,
                          const int* slot_of_pos, const float* w, const int* positions, int n,
                          float* routed_out, const DecodeWs& ws, int* status);
cudaError_t shared_expert(cudaStream_t st, const LayerW& L, bool bf16, int T, const uint16_t* x,
                          const float* coef, float* out, const DecodeWs& ws);
cudaError_t combine_subsets(cudaStream_t st, int T, const float* residual, const float* shared_out,
                            const float* hit, const float* miss, float* out);
void decode_carve(void* base, int T, DecodeWs* ws);
cudaError_t decode_init_attributes();

// Event pairs recorded around launches of one kernel (bench timing).
struct Prof {
  int kernel = -1;  // -1: off
  int cap = 0;
  int n = 0;
  cudaEvent_t* ev0 = nullptr;
  cudaEvent_t* ev1 = nullptr;
};
enum KernelId { kKRouter = 0, kKTopk = 1, kKGateUp = 2, kKDown = 3, kKCombine = 4, kKFused = 5, kKDispatch = 6 };

// Records the event pair of one launch of `kernel` when it is being profiled.
struct ProfScope {
  Prof* p;
  cudaStream_t st;
  int slot = -1;
  unsigned flags = cudaEventRecordDefault;
  ProfScope(Prof* prof, int kernel, cudaStream_t s) : p(prof), st(s) {
    if (p && p->kernel == kernel && p->n < p->cap) {
      // inside stream capture a plain record only orders streams; an external
      // record becomes a timing node of the graph
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      cudaStreamIsCapturing(st, &cs);
      if (cs == cudaStreamCaptureStatusActive) flags = cudaEventRecordExternal;
      slot = p->n++;
      cudaEventRecordWithFlags(p->ev0[slot], st, flags);
    }
  }
  ~ProfScope() {
    if (slot >= 0) cudaEventRecordWithFlags(p->ev1[slot], st, flags);
  }
};

struct RoutingArgs {
  const float* bias;
  const int* idx_in;
  const float* w_in;
  const int* rec_of_pos;
};

// One block: launches router, top-k/grouping, gate/up, down, combine.
// x16_next (optional): fp16 RMSNorm of the output for a following block.
cudaError_t decode_block(cudaStream_t st, const LayerW& L, bool bf16, int T, const uint16_t* x,
                         const float* residual, float* out, const RoutingArgs& r, int* idx_out,
                         float* w_out, const DecodeWs& ws, uint16_t* x16_next, float eps,
                         int* status, Prof* prof);

// ---- post-attention RMSNorm (qwen_rmsnorm_f32 order) into fp16 block input
cudaError_t prenorm_f16(cudaStream_t st, int T, const float* h, const float* w, float eps, uint16_t* x16);

// ---- Q4 LM head (qf_lmhead.cu): logits of one fp32 row, rows x 2048 Q4 g64
cudaError_t lm_head_q4(cudaStream_t st, bool bf16, const void* w, const void* s, const void* b, int rows,
                       const float* x, float* out, int sms);

cudaError_t router_logits(cudaStream_t st, const LayerW& L, bool bf16, int T, const uint16_t* x,
                          float* logits, float* coef, int* status);
cudaError_t router_topk(cudaStream_t st, int T, const float* logits, const float* bias,
                        int* idx, float* w, int* status);

// ---- persistent fused decode for T <= 8 (qf_fused.cu)
constexpr int kFusedMaxTokens = 8;
size_t fused_workspace_bytes(int T);
cudaError_t fused_init_attributes();
// layers: host array of n_layers descriptors (passed by value to the kernel).
// Supplied routing (r.idx_in / w_in / rec_of_pos) holds n_layers * T * 8
// entries, layer-major.
cudaError_t fused_stack(cudaStream_t st, const LayerW* layers, int n_layers, bool bf16, int T,
                        const uint16_t* x, const float* residual, float* out, float eps,
                        const RoutingArgs& r, int* idx_out, float* w_out, void* workspace,
                        int* status, Prof* prof);

// ---- persistent fused decode for one token (qf_fused1.cu); fused_stack calls
// it for T == 1.  Returns cudaErrorNotSupported (having done nothing) when the
// device has fewer than 128 SMs or a weight pointer is not 16-byte aligned.
cudaError_t fused1_init_attributes();
size_t fused1_workspace_bytes();
// pre_h / pre_w (optional): layer 0's input is the post-attention RMSNorm of
// pre_h with weight pre_w, computed in the kernel's prologue (x unused)
cudaError_t fused1_stack(cudaStream_t st, const LayerW* layers, int n_layers, bool bf16,
                         const uint16_t* x, const float* residual, float* out, float eps,
                         const RoutingArgs& r, int* idx_out, float* w_out, void* workspace,
                         int* status, Prof* prof, const float* pre_h = nullptr,
                         const float* pre_w = nullptr, float pre_eps = 0.f);

// ---- prefill path, T > 64 (qf_prefill.cu)
constexpr int kPrefillMaxTokens = 32768;
size_t prefill_workspace_bytes(int T);
cudaError_t grouped_ffn_routed(cudaStream_t st, const LayerW& L, bool bf16, int T, const uint16_t* x,
                               const int* idx, float* y, void* workspace, int* status, Prof* prof);
cudaError_t prefill_init_attributes();
cudaError_t router_logits_prefill(cudaStream_t st, const LayerW& L, bool bf16, int T,
                                  const uint16_t* x, float* logits, float* coef);
// T = 9..64 with a resident bank also takes the grouped path (its tcgen05
// GEMMs stream the routed weights faster than the per-kernel decode path).
constexpr int kGroupedMinTokens = 9;
// x16_next (optional): fp16 RMSNorm(out) with `eps` for a following block
cudaError_t prefill_block(cudaStream_t st, const LayerW& L, bool bf16, int T, const uint16_t* x,
                          const float* residual, float* out, const RoutingArgs& r, int* idx_out,
                          float* w_out, void* workspace, int* status, Prof* prof,
                          uint16_t* x16_next = nullptr, float eps = 0.f);

// grouped expert FFN over a row space (qf_prefill.cu): tiles of <= 128 rows per
// expert from counts/offsets (expert 256 = the shared expert over T_shared rows
// starting at *shared_base, or T_shared * 8), then gate/up -> act and down -> y.
// rows: fp16 [R][2048] in the MMA K order; y row of routed row i = perm[i]
// (perm NULL: i).
size_t grouped_max_tiles(int T);
// Expert-parallel output of the down GEMM: ret[row] = (rank << 24) | r sends
// result row `row` to row r of rank's result area (peer[rank] + y_off).
// Expert-parallel epilogue routing: the result rows (down, MODE 1) or the
// activation rows (gate/up, MODE 0, down-at-home mode) of received row r go to
// rank ret[r] >> 24, row ret[r] & 0xFFFFFF of that rank's region (y_off /
// act_off); rows_cap bounds the row.
struct EpOut {
  uint8_t* peer[8];
  int n_peers;
  int rows_cap;
  size_t y_off;
  size_t act_off;
  const int* ret;
};
cudaError_t tile_list(cudaStream_t st, const int* counts, const int* offsets, int T_shared,
                      const int* shared_base, int4* tiles, int* n_tiles);
cudaError_t grouped_ffn(cudaStream_t st, const LayerW& L, bool bf16, const uint16_t* rows, size_t R,
                        __half* act, float* y, const int* perm, const int4* tiles, const int* n_tiles,
                        size_t max_tiles, int sms, int* status, Prof* prof, const EpOut* ep);
// The same GEMMs, stage by stage (bit 0: gate/up over `rows`, bit 1: down over
// `act`; the maps of a stage that does not run are not built), with separate
// epilogue routing per stage (ep0: activation rows, ep1: result rows).
cudaError_t grouped_ffn_stages(cudaStream_t st, const LayerW& L, bool bf16, const uint16_t* rows, size_t R,
                               __half* act, float* y, const int* perm, const int4* tiles, const int* n_tiles,
                               size_t max_tiles, int sms, int* status, Prof* prof, int stages,
                               const EpOut* ep0, const EpOut* ep1);

// ---- dispatch plan (qf_route.cu)
size_t dispatch_workspace_bytes(int T);
cudaError_t dispatch_plan_ws(cudaStream_t st, const int* idx, int T, int* counts, int* offsets,
                             int* perm, int* scratch, int* status);

}  // namespace qf
