// qf_route.cu -- dispatch plan: histogram, exclusive scan and a stable
// permutation of the T*top_k routed positions by expert.
//
// The reference is decode-only and has no counterpart (its prefill calls the
// single-token path per prompt token).  Order is deterministic and stable:
// positions of one expert appear in increasing (token, k) order, which is the
// order the grouped expert GEMM reads rows in.
//   k_plan_hist     one CTA per 1024-position chunk: per-chunk expert counts
//   k_plan_scan     one CTA: chunk offsets (expert-major, chunk-minor), counts,
//                   offsets
//   k_plan_scatter  one CTA per chunk: rank inside the chunk from warp
//                   __match_any_sync peers plus per-warp prefix counts
#include "qf_internal.h"

namespace qf {

constexpr int kPlanChunk = 1024;
constexpr int kPlanMaxChunks = 256;  // 262,144 positions = 32,768 tokens x 8

__global__ void __launch_bounds__(kPlanChunk) k_plan_hist(const int* __restrict__ idx, int n,
                                                           int* __restrict__ chunk_counts,
                                                           int* status) {
  __shared__ int h[kExperts];
  for (int i = threadIdx.x; i < kExperts; i += blockDim.x) h[i] = 0;
  __syncthreads();
  const int i = blockIdx.x * kPlanChunk + threadIdx.x;
  if (i < n) {
    const int e = idx[i];
    if (e >= 0 && e < kExperts)
      atomicAdd(&h[e], 1);
    else
      set_status(status, kStatusDevice);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < kExperts; e += blockDim.x)
    chunk_counts[blockIdx.x * kExperts + e] = h[e];
}

// chunk_counts [C][E] -> chunk_offsets [C][E] (start of chunk c's run of expert e)
__global__ void __launch_bounds__(kExperts) k_plan_scan(int n_chunks, const int* __restrict__ chunk_counts,
                                                         int* __restrict__ chunk_offsets,
                                                         int* __restrict__ counts,
                                                         int* __restrict__ offsets) {
  __shared__ int s_warp[kExperts / 32];
  const int e = threadIdx.x;
  int s = 0;
  for (int c = 0; c < n_chunks; c++) s += chunk_counts[c * kExperts + e];
  int total = 0;
  const int ex = block_scan256(s, s_warp, &total);
  counts[e] = s;
  offsets[e] = ex;
  if (e == 0) offsets[kExperts] = total;
  int run = ex;
  for (int c = 0; c < n_chunks; c++) {
    chunk_offsets[c * kExperts + e] = run;
    run += chunk_counts[c * kExperts + e];
  }
}

__global__ void __launch_bounds__(kPlanChunk) k_plan_scatter(const int* __restrict__ idx, int n,
                                                              const int* __restrict__ chunk_offsets,
                                                              int* __restrict__ perm) {
  __shared__ int wh[kPlanChunk / 32][kExperts];  // per-warp counts, then exclusive prefix
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < (kPlanChunk / 32) * kExperts; i += blockDim.x) (&wh[0][0])[i] = 0;
  __syncthreads();
  const int i = blockIdx.x * kPlanChunk + threadIdx.x;
  const bool valid = i < n;
  int e = valid ? idx[i] : -1;
  if (valid && (e < 0 || e >= kExperts)) e = -1;
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  const bool leader = (peers & ((1u << lane) - 1u)) == 0;
  if (e >= 0 && leader) wh[warp][e] = __popc(peers);
  __syncthreads();
  for (int x = threadIdx.x; x < kExperts; x += blockDim.x) {
    int acc = 0;
    for (int w = 0; w < kPlanChunk / 32; w++) {
      const int c = wh[w][x];
      wh[w][x] = acc;
      acc += c;
    }
  }
  __syncthreads();
  if (e >= 0) perm[chunk_offsets[blockIdx.x * kExperts + e] + wh[warp][e] + rank] = i;
}

size_t dispatch_workspace_bytes(int T) {
  const int n = T * kTopK;
  const int chunks = (n + kPlanChunk - 1) / kPlanChunk;
  return static_cast<size_t>(2) * chunks * kExperts * sizeof(int);
}

cudaError_t dispatch_plan_ws(cudaStream_t st, const int* idx, int T, int* counts, int* offsets,
                             int* perm, int* scratch, int* status) {
  const int n = T * kTopK;
  const int chunks = (n + kPlanChunk - 1) / kPlanChunk;
  if (chunks > kPlanMaxChunks) return cudaErrorInvalidValue;
  int* chunk_counts = scratch;
  int* chunk_offsets = scratch + chunks * kExperts;
  k_plan_hist<<<chunks, kPlanChunk, 0, st>>>(idx, n, chunk_counts, status);
  k_plan_scan<<<1, kExperts, 0, st>>>(chunks, chunk_counts, chunk_offsets, counts, offsets);
  k_plan_scatter<<<chunks, kPlanChunk, 0, st>>>(idx, n, chunk_offsets, perm);
  return cudaGetLastError();
}

}  // namespace qf
