// qf_ep.cu -- expert-parallel MoE block over NVLink peer memory.
//
// The 256 routed experts are split across `world` GPUs (rank r owns experts
// [r*256/world, (r+1)*256/world)); router, shared-gate coefficient and the
// shared expert are replicated and run on each rank's own tokens.  No
// collective library is on the data path: every rank exports one device
// region (CUDA IPC), and
//   dispatch  one kernel publishes this rank's per-expert counts into every
//             rank's count board, waits until all ranks have published (which
//             also means every rank has finished reading the previous call's
//             buffers), and stores each token row (fp16, already in the grouped
//             GEMM's K order) over NVLink ONCE per owner rank that holds any of
//             its 8 experts: into the receive row of the token's first position
//             (lowest k) with an expert there, recording that row in the
//             owner's first-row map (source rank x max_tokens + token); the
//             token's other positions on that owner send only the 4-byte map
//             index; receive rows land expert-major, then by source rank, then
//             in the source's (token, k) order;
//   expand    the owner copies each such duplicate from its first row (local
//             HBM), so its grouped GEMM reads contiguous rows of its own memory;
//   GEMMs     the owner runs the grouped tcgen05 gate/up and down GEMMs over
//             its received rows plus its own tokens' shared-expert rows; the
//             down GEMM's epilogue stores each fp32 result row straight into the
//             sending rank's result area (at the row's send index, from the
//             return address dispatch left beside it), so the transfer back
//             overlaps the remaining tiles; then it signals every rank;
//   combine   each rank reads its tokens' eight result rows from its own region
//             and forms residual + c*shared + sum_k w_k y_k in router order --
//             the same arithmetic as the single-GPU block, so the outputs are
//             bit-identical to it.
// Down-at-home mode (qf_ep_set_down_at_home; every rank holds all 256
// experts): the owner runs only the gate/up GEMM and its epilogue stores each
// fp16 activation row (1 KB) into the sending rank's activation area at the
// row's send index; after every owner has signalled, each rank runs the down
// GEMM over its own tokens' activation rows with all 256 experts (the
// single-GPU block's down stage, same rows and tiles per expert), then the
// same combine.  The NVLink return shrinks from 8 KB of fp32 results to 1 KB
// of activations per routed row, at the cost of replicating the down
// projections; the outputs stay bit-identical.
// Counters are monotonically increasing (never reset) and every wait is bounded
// (globaltimer deadline); an expired wait sets QF_ERR_TIMEOUT in the status word
// and the kernel returns.
//
// Reference: the reference runs one GPU and has no expert parallelism; the
// per-token math is the MoE step of QwenQ4ActiveExpertStreamingRunner.forwardToken
// (QwenQ4ActiveExpertStreamingRunner.swift:1169-1381).
#include <algorithm>
#include <cstring>
#include <new>
#include <vector>

#include "../../include/qf_moe.h"
#include "qf_handle.h"
#include "qf_internal.h"

namespace qf {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kDispBlocks = 256;  // identical on every rank: the delivery count expects it
constexpr int kDispThreads = 256;  // one thread per expert in the count phase
static_assert(kDispThreads == kExperts, "count phase maps threads to experts");
constexpr size_t kSigBytes = 65536;
// u32 counters of the signal area (each on its own 128-byte line)
constexpr int kSigArrive = 0;      // +1 per rank entering a call
constexpr int kSigDelivered = 32;  // +kDispBlocks per rank whose rows have landed
constexpr int kSigDone = 64;       // +1 per owner whose result rows are written
constexpr size_t kBoardOff = 4096;  // int board[2][kMaxRanks][256]
constexpr size_t kHeaderOff = 1024;  // RegionHeader, written at creation
struct RegionHeader {
  uint64_t region_bytes;
  uint64_t rows_cap;
  uint32_t world;
  uint32_t magic;
};
constexpr uint32_t kRegionMagic = 0x51464550u;
constexpr uint64_t kWaitNs = 2000000000ull;  // default deadline of every wait: 2 s

__device__ __forceinline__ uint64_t gtime() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Bounded wait until *c has reached target (wrap-safe); false once wait_ns of
// globaltimer time have passed.
__device__ bool wait_counter(const unsigned* c, unsigned target, uint64_t wait_ns) {
  const uint64_t t0 = gtime();
  for (unsigned i = 0;; i++) {
    if (static_cast<int>(ld_acquire_sys(c) - target) >= 0) return true;
    if ((i & 15) == 15) {
      if (gtime() - t0 > wait_ns) return false;
      __nanosleep(100);
    }
  }
}

struct EpArgs {
  int rank, world, epr;  // experts per rank
  unsigned epoch;        // 1, 2, ... (calls so far, this one included)
  int T, P;              // this rank's tokens and routed positions
  int rows_cap;          // receive rows of every rank's region
  const int* idx;        // [P] expert of each position (t*8+k)
  const int* offsets;    // [257] first send row of each expert
  const int* perm;       // [P] send row -> position, sorted by (expert, token, k)
  const int* counts;     // [256] routed positions per expert
  const uint4* x;        // [T][256] this rank's fp16 token rows
  uint8_t* peer[kMaxRanks];  // exported region of each rank (this rank's own included)
  size_t x_off, y_off;   // receive rows / result rows inside a region
  size_t ret_off;        // int [rows_cap]: return address of each received row
  size_t tok_off;        // first-row map: int [world][t_max], the receive row of each (source rank, token)
  size_t src_off;        // int [rows_cap]: map index of a duplicate received row, -1 for a first row
  int t_max;             // tokens per rank of the token area
  int pmax;              // result rows [0, pmax) are send rows, [pmax, pmax + T) shared rows
  int* loc_of_pos;       // [P] send row of each position (its result row here)
  int* counts_local;     // [256] received rows per local expert (zero past epr)
  int* offsets_local;    // [256] first received row of each local expert
  int* q_rows;           // received routed rows (the shared rows follow them)
  int* status;
  uint64_t wait_ns;      // deadline of each bounded wait
};

__device__ __forceinline__ unsigned* sig(uint8_t* region, int word) {
  return reinterpret_cast<unsigned*>(region) + word;
}

// Publishes this rank's per-expert counts on every rank's board, then arrives.
__global__ void __launch_bounds__(kDispThreads) k_ep_publish(const __grid_constant__ EpArgs a) {
  const int tid = threadIdx.x;
  const unsigned par = a.epoch & 1u;
  const int c = a.counts[tid];
  for (int d = 0; d < a.world; d++)
    reinterpret_cast<int*>(a.peer[d] + kBoardOff)[(par * kMaxRanks + a.rank) * kExperts + tid] = c;
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    for (int d = 0; d < a.world; d++) red_release_sys(sig(a.peer[d], kSigArrive), 1u);
  }
}

__global__ void __launch_bounds__(kDispThreads) k_ep_dispatch(const __grid_constant__ EpArgs a) {
  __shared__ int s_scan[kExperts];
  __shared__ int s_base[kExperts];
  __shared__ int s_warp[kDispThreads / 32];
  __shared__ int s_q;
  __shared__ int s_ok;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const unsigned par = a.epoch & 1u;
  uint8_t* mine = a.peer[a.rank];

  // 1. every rank's counts are on this rank's board once all have arrived
  if (tid == 0) s_ok = wait_counter(sig(mine, kSigArrive), a.epoch * (unsigned)a.world, a.wait_ns);
  __syncthreads();
  if (!s_ok) {
    if (tid == 0) set_status(a.status, kStatusTimeout);
    // a rank is missing: leave the GEMMs nothing to do (no routed rows, no
    // shared rows: q_rows < 0 drops the shared tiles from the tile list)
    if (blockIdx.x == 0) {
      a.counts_local[tid] = 0;
      a.offsets_local[tid] = 0;
      if (tid == 0) *a.q_rows = -1;
    }
    return;
  }
  const int* board = reinterpret_cast<const int*>(mine + kBoardOff) + par * kMaxRanks * kExperts;
  int tot = 0, before = 0;
  for (int s = 0; s < a.world; s++) {
    const int v = __ldcg(board + s * kExperts + tid);
    tot += v;
    if (s < a.rank) before += v;
  }
  // exclusive scan of the per-expert totals
  int v = tot;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += o;
  }
  if (lane == 31) s_warp[warp] = v;
  __syncthreads();
  int wbefore = 0;
  for (int w = 0; w < warp; w++) wbefore += s_warp[w];
  const int excl = wbefore + v - tot;
  s_scan[tid] = excl;
  __syncthreads();
  const int owner_first = (tid / a.epr) * a.epr;
  s_base[tid] = excl - s_scan[owner_first] + before;  // first row of my expert-tid rows at the owner
  const int my_first = a.rank * a.epr;
  if (tid == my_first + a.epr - 1) s_q = excl + tot - s_scan[my_first];
  if (blockIdx.x == 0) {
    const bool local = tid >= my_first && tid < my_first + a.epr;
    const int le = tid - my_first;
    if (local) {
      a.counts_local[le] = tot;
      a.offsets_local[le] = excl - s_scan[my_first];
    }
    if (tid >= a.epr) {  // entries past the local experts: empty
      a.counts_local[tid] = 0;
      a.offsets_local[tid] = 0;
    }
  }
  __syncthreads();
  if (blockIdx.x == 0 && tid == 0) *a.q_rows = s_q;

  // 2. rows: routed positions to their owners, then this rank's shared rows
  const int n_rows = a.P + a.T;
  for (int j = blockIdx.x * (kDispThreads / 32) + warp; j < n_rows; j += gridDim.x * (kDispThreads / 32)) {
    int src_t, d, row;
    uint4* dst;
    if (j < a.P) {
      const int pos = a.perm[j];
      const int e = a.idx[pos];
      src_t = pos >> 3;
      if (e < 0 || e >= kExperts) {  // a bad supplied expert id: skipped, reported
        if (lane == 0) {
          a.loc_of_pos[pos] = j;
          set_status(a.status, kStatusDevice);
        }
        continue;
      }
      d = e / a.epr;
      row = s_base[e] + (j - a.offsets[e]);
      if (lane == 0) a.loc_of_pos[pos] = j;
      if (row < 0 || row >= a.rows_cap || src_t >= a.t_max) {
        if (lane == 0) set_status(a.status, kStatusDevice);
        continue;
      }
      const int trow = a.rank * a.t_max + src_t;
      // the token row crosses once per owner: the token's first position
      // (lowest k) with an expert on that owner carries it (its 8 expert ids
      // in two 16-byte loads)
      const int4 i0 = __ldg(reinterpret_cast<const int4*>(a.idx) + 2 * src_t);
      const int4 i1 = __ldg(reinterpret_cast<const int4*>(a.idx) + 2 * src_t + 1);
      const int es[8] = {i0.x, i0.y, i0.z, i0.w, i1.x, i1.y, i1.z, i1.w};
      bool first = true;
      const int k = pos & 7;
#pragma unroll
      for (int kk = 0; kk < 7; kk++)
        first &= !(kk < k && es[kk] >= 0 && es[kk] < kExperts && es[kk] / a.epr == d);
      if (lane == 0) {
        // where the owner's down GEMM sends this row's result; a duplicate
        // names the map entry of the row its bytes are copied from
        reinterpret_cast<int*>(a.peer[d] + a.ret_off)[row] = (a.rank << 24) | j;
        reinterpret_cast<int*>(a.peer[d] + a.src_off)[row] = first ? -1 : trow;
        if (first) reinterpret_cast<int*>(a.peer[d] + a.tok_off)[trow] = row;
      }
      if (!first) continue;
      dst = reinterpret_cast<uint4*>(a.peer[d] + a.x_off) + static_cast<size_t>(row) * (kHidden / 8);
    } else {
      d = a.rank;
      src_t = j - a.P;
      row = s_q + src_t;
      if (row < 0 || row >= a.rows_cap) {
        if (lane == 0) set_status(a.status, kStatusDevice);
        continue;
      }
      if (lane == 0) reinterpret_cast<int*>(a.peer[d] + a.ret_off)[row] = (a.rank << 24) | (a.pmax + src_t);
      dst = reinterpret_cast<uint4*>(a.peer[d] + a.x_off) + static_cast<size_t>(row) * (kHidden / 8);
    }
    const uint4* s = a.x + static_cast<size_t>(src_t) * (kHidden / 8);
    uint4 vv[kHidden / 8 / 32];
#pragma unroll
    for (int q = 0; q < kHidden / 8 / 32; q++) vv[q] = __ldg(s + lane + 32 * q);
#pragma unroll
    for (int q = 0; q < kHidden / 8 / 32; q++) dst[lane + 32 * q] = permute8(vv[q]);
  }
  // 3. this block's rows are out: count it on every rank
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    for (int dd = 0; dd < a.world; dd++) red_release_sys(sig(a.peer[dd], kSigDelivered), 1u);
  }
}

// Waits until every rank's dispatch blocks have delivered (one thread).  After
// an expired wait earlier in this call (q_rows < 0) there is nothing to wait for.
__global__ void k_ep_wait_rows(uint8_t* mine, unsigned target, const int* q_rows, int* status,
                               uint64_t wait_ns) {
  if (threadIdx.x == 0 && *(volatile const int*)q_rows >= 0 &&
      !wait_counter(sig(mine, kSigDelivered), target, wait_ns))
    set_status(status, kStatusTimeout);
}

// Owner: each duplicate receive row r < q_rows (routed) <- the first row of
// its (source rank, token), named by the first-row map (local copy, one warp
// per row).  Nothing after an expired wait (q_rows < 0).
__global__ void __launch_bounds__(256) k_ep_expand(uint8_t* mine, size_t x_off, size_t tok_off, size_t src_off,
                                                   int tok_rows, const int* q_rows, int* status) {
  const int q = *q_rows;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  const int* src = reinterpret_cast<const int*>(mine + src_off);
  const int* first_row = reinterpret_cast<const int*>(mine + tok_off);
  uint4* rows = reinterpret_cast<uint4*>(mine + x_off);
  for (int r = warp; r < q; r += nw) {
    const int t = __ldcg(src + r);
    if (t < 0) continue;  // a first row: its bytes came over NVLink
    const int f = t < tok_rows ? __ldcg(first_row + t) : -1;
    if (f < 0 || f >= q) {
      if (lane == 0) set_status(status, kStatusDevice);
      continue;
    }
    uint4 v[kHidden / 8 / 32];
#pragma unroll
    for (int i = 0; i < kHidden / 8 / 32; i++) v[i] = __ldcg(rows + static_cast<size_t>(f) * (kHidden / 8) + lane + 32 * i);
#pragma unroll
    for (int i = 0; i < kHidden / 8 / 32; i++) rows[static_cast<size_t>(r) * (kHidden / 8) + lane + 32 * i] = v[i];
  }
}

// Down-at-home mode: wait (one thread) until every owner's activation rows
// have landed here.  After an expired wait earlier in this call (q_rows < 0)
// there is nothing to wait for.
__global__ void k_ep_wait_done(uint8_t* mine, unsigned target, const int* q_rows, int* status, uint64_t wait_ns) {
  if (threadIdx.x == 0 && *(volatile const int*)q_rows >= 0 &&
      !wait_counter(sig(mine, kSigDone), target, wait_ns))
    set_status(status, kStatusTimeout);
}

// Down-at-home mode, before the home tile list: the shared rows start at
// `pmax`, and after an expired wait (q_rows < 0) the list is empty (no routed
// counts, a negative shared base), so the home down GEMM does no work.
__global__ void k_ep_home_guard(const int* q_rows, int* counts, int* home_base, int pmax) {
  const bool abort = *(volatile const int*)q_rows < 0;
  if (abort) counts[threadIdx.x] = 0;
  if (threadIdx.x == 0) *home_base = abort ? -1 : pmax;
}

// The owner's result rows are written: tell every rank.
__global__ void k_ep_signal_done(EpArgs a) {
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int d = 0; d < a.world; d++) red_release_sys(sig(a.peer[d], kSigDone), 1u);
  }
}

// out = (residual + sigmoid(c) * shared) + sum_k w_k * y_k in router order; the
// owners have stored y_k into this rank's result area at the send row.
__global__ void __launch_bounds__(256) k_ep_combine(const __grid_constant__ EpArgs a, const float* __restrict__ residual,
                                                    const float* __restrict__ w, const float* __restrict__ coef,
                                                    float* __restrict__ out) {
  __shared__ int s_ok;
  const int t = blockIdx.x;
  if (threadIdx.x == 0)
    s_ok = *(volatile const int*)a.q_rows >= 0 &&
           wait_counter(sig(a.peer[a.rank], kSigDone), a.epoch * (unsigned)a.world, a.wait_ns);
  __syncthreads();
  if (!s_ok) {
    if (threadIdx.x == 0) set_status(a.status, kStatusTimeout);
    return;
  }
  const float c = coef[t];
  const float coeff = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-c)));
  float wk[kTopK];
  const float4* yk[kTopK];
#pragma unroll
  for (int k = 0; k < kTopK; k++) {
    wk[k] = w[t * kTopK + k];
    int row = a.loc_of_pos[t * kTopK + k];
    if (row < 0 || row >= a.pmax) {
      if (threadIdx.x == 0) set_status(a.status, kStatusDevice);
      row = 0;
    }
    yk[k] = reinterpret_cast<const float4*>(a.peer[a.rank] + a.y_off) + static_cast<size_t>(row) * (kHidden / 4);
  }
  const float4* s4 = reinterpret_cast<const float4*>(a.peer[a.rank] + a.y_off) + static_cast<size_t>(a.pmax + t) * (kHidden / 4);
  const float4* r4 = residual ? reinterpret_cast<const float4*>(residual + static_cast<size_t>(t) * kHidden) : nullptr;
  float4* o4 = reinterpret_cast<float4*>(out + static_cast<size_t>(t) * kHidden);
  for (int i = threadIdx.x; i < kHidden / 4; i += 256) {
    float4 y[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; k++) y[k] = __ldcg(yk[k] + i);
    float4 acc = make_float4(__fmul_rn(y[0].x, wk[0]), __fmul_rn(y[0].y, wk[0]), __fmul_rn(y[0].z, wk[0]),
                             __fmul_rn(y[0].w, wk[0]));
#pragma unroll
    for (int k = 1; k < kTopK; k++) {
      acc.x = __fadd_rn(acc.x, __fmul_rn(y[k].x, wk[k]));
      acc.y = __fadd_rn(acc.y, __fmul_rn(y[k].y, wk[k]));
      acc.z = __fadd_rn(acc.z, __fmul_rn(y[k].z, wk[k]));
      acc.w = __fadd_rn(acc.w, __fmul_rn(y[k].w, wk[k]));
    }
    const float4 sh = __ldcg(s4 + i);
    const float4 base = r4 ? r4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    o4[i] = make_float4(__fadd_rn(__fadd_rn(base.x, __fmul_rn(sh.x, coeff)), acc.x),
                        __fadd_rn(__fadd_rn(base.y, __fmul_rn(sh.y, coeff)), acc.y),
                        __fadd_rn(__fadd_rn(base.z, __fmul_rn(sh.z, coeff)), acc.z),
                        __fadd_rn(__fadd_rn(base.w, __fmul_rn(sh.w, coeff)), acc.w));
  }
}

size_t al256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

}  // namespace
}  // namespace qf

struct qf_ep {
  qf_moe* h = nullptr;
  int device = 0, rank = 0, world = 1, epr = 256, t_max = 0, sms = 0;
  size_t rows_cap = 0, region_bytes = 0, x_off = 0, y_off = 0, ret_off = 0, tok_off = 0, src_off = 0, act_off = 0;
  size_t max_tiles = 0, home_max_tiles = 0;
  bool down_at_home = false;
  int4* home_tiles = nullptr;
  int* home_n_tiles = nullptr;
  int* pmax_dev = nullptr;
  uint8_t* region = nullptr;
  uint8_t* peer[qf::kMaxRanks] = {};
  bool opened[qf::kMaxRanks] = {};
  bool connected = false;
  unsigned epoch = 0;
  uint8_t* ws = nullptr;
  float* logits = nullptr;
  float* coef = nullptr;
  int* idx = nullptr;
  float* w = nullptr;
  int* counts = nullptr;
  int* offsets = nullptr;
  int* perm = nullptr;
  int* plan_ws = nullptr;
  int4* tiles = nullptr;
  int* n_tiles = nullptr;
  int* loc_of_pos = nullptr;
  int* counts_local = nullptr;
  int* offsets_local = nullptr;
  int* q_rows = nullptr;
  __half* act = nullptr;
  uint64_t wait_ns = qf::kWaitNs;
};

namespace {

struct EpDevice {
  int prev = -1;
  explicit EpDevice(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~EpDevice() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" {

qf_status qf_ep_create(qf_moe* h, int32_t rank, int32_t world, int32_t max_tokens, qf_ep** out) {
  using qf::al256;
  if (!h || !out) return QF_ERR_ARG;
  *out = nullptr;
  if (world < 1 || world > qf::kMaxRanks || qf::kExperts % world != 0 || rank < 0 || rank >= world)
    return qf::fail(h, QF_ERR_ARG, "EP: world must be 1, 2, 4 or 8 and rank in [0, world)");
  if (max_tokens < 1 || max_tokens > 32768)
    return qf::fail(h, QF_ERR_ARG, "EP: max_tokens must be in [1, 32768]");
  EpDevice g(h->device);
  qf_ep* ep = new (std::nothrow) qf_ep();
  if (!ep) return QF_ERR_OOM;
  ep->h = h;
  ep->device = h->device;
  ep->rank = rank;
  ep->world = world;
  ep->epr = qf::kExperts / world;
  ep->t_max = max_tokens;
  const size_t P = static_cast<size_t>(max_tokens) * qf::kTopK;
  // rows an owner can receive: eight per token of every rank, plus its own shared rows
  ep->rows_cap = static_cast<size_t>(world) * P + max_tokens;
  ep->x_off = qf::kSigBytes;
  ep->y_off = ep->x_off + al256(ep->rows_cap * qf::kHidden * 2);
  ep->ret_off = ep->y_off + al256(ep->rows_cap * qf::kHidden * 4);
  ep->src_off = ep->ret_off + al256(ep->rows_cap * 4);
  ep->tok_off = ep->src_off + al256(ep->rows_cap * 4);
  // down-at-home activation rows: [0, 8 max_tokens) routed by send row, then
  // [8 max_tokens, +max_tokens) this rank's shared rows
  ep->act_off = ep->tok_off + al256(static_cast<size_t>(world) * max_tokens * 4);
  ep->region_bytes = ep->act_off + al256((P + max_tokens) * qf::kInter * 2);
  ep->home_max_tiles = qf::grouped_max_tiles(max_tokens);
  ep->max_tiles = qf::grouped_max_tiles(max_tokens * world);
  size_t wsb = 0;
  wsb += al256(4 * (size_t)max_tokens * qf::kExperts) + al256(4 * (size_t)max_tokens);
  wsb += al256(4 * P) * 3 + al256(4 * (qf::kExperts + 1)) * 4 + al256(qf::dispatch_workspace_bytes(max_tokens));
  wsb += al256(16 * ep->max_tiles) + al256(16) + al256(4 * P) + al256(16);
  wsb += al256(ep->rows_cap * qf::kInter * 2);
  wsb += al256(16 * ep->home_max_tiles) + al256(16) + al256(16);
  cudaError_t e = cudaDeviceGetAttribute(&ep->sms, cudaDevAttrMultiProcessorCount, h->device);
  if (e == cudaSuccess) e = cudaMalloc(&ep->region, ep->region_bytes);
  if (e == cudaSuccess) e = cudaMemset(ep->region, 0, qf::kSigBytes);
  if (e == cudaSuccess) {
    const qf::RegionHeader hd = {ep->region_bytes, ep->rows_cap, static_cast<uint32_t>(world), qf::kRegionMagic};
    e = cudaMemcpy(ep->region + qf::kHeaderOff, &hd, sizeof(hd), cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess) e = cudaMalloc(&ep->ws, wsb);
  if (e != cudaSuccess) {
    cudaFree(ep->region);
    delete ep;
    return qf::cuda_fail(h, e, "EP: allocation");
  }
  uint8_t* p = ep->ws;
  auto take = [&](size_t n) {
    uint8_t* q = p;
    p += al256(n);
    return q;
  };
  ep->logits = reinterpret_cast<float*>(take(4 * (size_t)max_tokens * qf::kExperts));
  ep->coef = reinterpret_cast<float*>(take(4 * (size_t)max_tokens));
  ep->idx = reinterpret_cast<int*>(take(4 * P));
  ep->w = reinterpret_cast<float*>(take(4 * P));
  ep->perm = reinterpret_cast<int*>(take(4 * P));
  ep->counts = reinterpret_cast<int*>(take(4 * (qf::kExperts + 1)));
  ep->offsets = reinterpret_cast<int*>(take(4 * (qf::kExperts + 1)));
  ep->counts_local = reinterpret_cast<int*>(take(4 * (qf::kExperts + 1)));
  ep->offsets_local = reinterpret_cast<int*>(take(4 * (qf::kExperts + 1)));
  ep->plan_ws = reinterpret_cast<int*>(take(qf::dispatch_workspace_bytes(max_tokens)));
  ep->tiles = reinterpret_cast<int4*>(take(16 * ep->max_tiles));
  ep->n_tiles = reinterpret_cast<int*>(take(16));
  ep->loc_of_pos = reinterpret_cast<int*>(take(4 * P));
  ep->q_rows = reinterpret_cast<int*>(take(16));
  ep->act = reinterpret_cast<__half*>(take(ep->rows_cap * qf::kInter * 2));
  ep->home_tiles = reinterpret_cast<int4*>(take(16 * ep->home_max_tiles));
  ep->home_n_tiles = reinterpret_cast<int*>(take(16));
  ep->pmax_dev = reinterpret_cast<int*>(take(16));
  // (pmax_dev: the home tile list's shared base, set per call by k_ep_home_guard)
  ep->peer[rank] = ep->region;
  if (world == 1) ep->connected = true;
  *out = ep;
  return QF_OK;
}

qf_status qf_ep_ipc_handle(const qf_ep* ep, void* handle) {
  if (!ep || !handle) return QF_ERR_ARG;
  EpDevice g(ep->device);
  cudaIpcMemHandle_t hd;
  cudaError_t e = cudaIpcGetMemHandle(&hd, ep->region);
  if (e != cudaSuccess) return qf::cuda_fail(ep->h, e, "EP: cudaIpcGetMemHandle");
  static_assert(sizeof(cudaIpcMemHandle_t) == QF_EP_HANDLE_BYTES, "handle size");
  std::memcpy(handle, &hd, sizeof(hd));
  return QF_OK;
}

qf_status qf_ep_connect(qf_ep* ep, const void* handles) {
  if (!ep || !handles) return QF_ERR_ARG;
  EpDevice g(ep->device);
  const uint8_t* hb = static_cast<const uint8_t*>(handles);
  for (int d = 0; d < ep->world; d++) {
    if (d == ep->rank || ep->opened[d]) continue;
    cudaIpcMemHandle_t hd;
    std::memcpy(&hd, hb + static_cast<size_t>(d) * QF_EP_HANDLE_BYTES, sizeof(hd));
    void* ptr = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&ptr, hd, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return qf::cuda_fail(ep->h, e, "EP: cudaIpcOpenMemHandle");
    ep->peer[d] = static_cast<uint8_t*>(ptr);
    ep->opened[d] = true;
    // every rank must have been created with the same world and max_tokens
    qf::RegionHeader rh;
    e = cudaMemcpy(&rh, ep->peer[d] + qf::kHeaderOff, sizeof(rh), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return qf::cuda_fail(ep->h, e, "EP: reading a peer region header");
    if (rh.magic != qf::kRegionMagic || rh.world != static_cast<uint32_t>(ep->world) ||
        rh.rows_cap != ep->rows_cap || rh.region_bytes != ep->region_bytes)
      return qf::fail(ep->h, QF_ERR_ARG, "EP: ranks were created with different world or max_tokens");
  }
  ep->connected = true;
  return QF_OK;
}

void qf_ep_destroy(qf_ep* ep) {
  if (!ep) return;
  EpDevice g(ep->device);
  cudaDeviceSynchronize();
  for (int d = 0; d < qf::kMaxRanks; d++)
    if (ep->opened[d]) cudaIpcCloseMemHandle(ep->peer[d]);
  cudaFree(ep->ws);
  cudaFree(ep->region);
  delete ep;
}

qf_status qf_moe_block_forward_ep(qf_ep* ep, const qf_moe_layer* layer, int32_t T, const uint16_t* x,
                                  const float* residual, float* out, const qf_routing* routing,
                                  int32_t* idx_out, float* w_out) {
  if (!ep) return QF_ERR_ARG;
  qf_moe* h = ep->h;
  if (!ep->connected) return qf::fail(h, QF_ERR_ARG, "EP: qf_ep_connect has not been called");
  qf::LayerW L;
  qf_status s = qf::layer_to_w(h, layer, &L);
  if (s != QF_OK) return s;
  if (L.bank_records < static_cast<uint32_t>(ep->down_at_home ? qf::kExperts : ep->epr))
    return qf::fail(h, QF_ERR_ARG,
                    ep->down_at_home ? "EP: down-at-home mode needs all 256 experts in the bank"
                                     : "EP: the bank must hold this rank's 256/world experts");
  if (T < 1 || T > ep->t_max) return qf::fail(h, QF_ERR_ARG, "EP: T must be in [1, max_tokens]");
  if (!x || !out || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (residual && (reinterpret_cast<uintptr_t>(residual) & 15)))
    return qf::fail(h, QF_ERR_ARG, "EP: x, out (and residual) must be 16-byte aligned device pointers");
  const float* bias = routing ? routing->logit_bias : nullptr;
  if (routing && (routing->record_of_pos || (routing->topk_idx == nullptr) != (routing->topk_w == nullptr)))
    return qf::fail(h, QF_ERR_ARG, "EP: routing supports logit_bias or a supplied top-k");
  EpDevice g(ep->device);
  cudaStream_t st = h->stream;
  const bool bf16 = h->dims.scale_dtype == QF_SCALE_BF16;
  const size_t P = static_cast<size_t>(T) * qf::kTopK;
  cudaError_t e;
  {
    qf::ProfScope ps(&h->prof, qf::kKRouter, st);
    e = qf::router_logits_prefill(st, L, bf16, T, x, ep->logits, ep->coef);
  }
  if (e != cudaSuccess) return qf::cuda_fail(h, e, "EP: router");
  if (routing && routing->topk_idx) {
    e = cudaMemcpyAsync(ep->idx, routing->topk_idx, 4 * P, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(ep->w, routing->topk_w, 4 * P, cudaMemcpyDeviceToDevice, st);
  } else {
    qf::ProfScope ps(&h->prof, qf::kKTopk, st);
    e = qf::router_topk(st, T, ep->logits, bias, ep->idx, ep->w, h->d_status);
  }
  if (e == cudaSuccess && idx_out) e = cudaMemcpyAsync(idx_out, ep->idx, 4 * P, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess && w_out) e = cudaMemcpyAsync(w_out, ep->w, 4 * P, cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess) e = qf::dispatch_plan_ws(st, ep->idx, T, ep->counts, ep->offsets, ep->perm, ep->plan_ws, h->d_status);
  if (e != cudaSuccess) return qf::cuda_fail(h, e, "EP: routing");

  qf::EpArgs a;
  a.rank = ep->rank;
  a.world = ep->world;
  a.epr = ep->epr;
  a.epoch = ep->epoch + 1;
  a.T = T;
  a.P = static_cast<int>(P);
  a.rows_cap = static_cast<int>(ep->rows_cap);
  a.idx = ep->idx;
  a.offsets = ep->offsets;
  a.perm = ep->perm;
  a.counts = ep->counts;
  a.x = reinterpret_cast<const uint4*>(x);
  for (int d = 0; d < qf::kMaxRanks; d++) a.peer[d] = ep->peer[d];
  a.x_off = ep->x_off;
  a.y_off = ep->y_off;
  a.ret_off = ep->ret_off;
  a.tok_off = ep->tok_off;
  a.src_off = ep->src_off;
  a.t_max = ep->t_max;
  a.pmax = ep->t_max * qf::kTopK;
  a.loc_of_pos = ep->loc_of_pos;
  a.counts_local = ep->counts_local;
  a.offsets_local = ep->offsets_local;
  a.q_rows = ep->q_rows;
  a.status = h->d_status;
  a.wait_ns = ep->wait_ns;
  {
    qf::ProfScope ps(&h->prof, qf::kKDispatch, st);
    qf::k_ep_publish<<<1, qf::kDispThreads, 0, st>>>(a);
    qf::k_ep_dispatch<<<qf::kDispBlocks, qf::kDispThreads, 0, st>>>(a);
    qf::k_ep_wait_rows<<<1, 32, 0, st>>>(ep->region, a.epoch * (unsigned)ep->world * qf::kDispBlocks, ep->q_rows,
                                         h->d_status, ep->wait_ns);
    qf::k_ep_expand<<<2 * ep->sms, 256, 0, st>>>(ep->region, ep->x_off, ep->tok_off, ep->src_off,
                                                 ep->world * ep->t_max, ep->q_rows, h->d_status);
  }
  e = cudaGetLastError();
  if (e == cudaSuccess) e = qf::tile_list(st, ep->counts_local, ep->offsets_local, T, ep->q_rows, ep->tiles, ep->n_tiles);
  qf::EpOut out_route{};
  for (int d = 0; d < qf::kMaxRanks; d++) out_route.peer[d] = ep->peer[d];
  out_route.n_peers = ep->world;
  out_route.rows_cap = static_cast<int>(ep->rows_cap);
  out_route.y_off = ep->y_off;
  out_route.ret = reinterpret_cast<const int*>(ep->region + ep->ret_off);
  if (!ep->down_at_home) {
    if (e == cudaSuccess)
      e = qf::grouped_ffn(st, L, bf16, reinterpret_cast<const uint16_t*>(ep->region + ep->x_off), ep->rows_cap,
                          ep->act, reinterpret_cast<float*>(ep->region + ep->y_off), nullptr, ep->tiles,
                          ep->n_tiles, ep->max_tiles, ep->sms, h->d_status, &h->prof, &out_route);
    if (e != cudaSuccess) return qf::cuda_fail(h, e, "EP: grouped experts");
    qf::k_ep_signal_done<<<1, 32, 0, st>>>(a);
  } else {
    // the owner: gate/up of its experts (records rank * epr ... of the full
    // bank), activation rows to their senders
    qf::LayerW Lo = L;
    Lo.bank = L.bank + static_cast<uint64_t>(ep->rank) * ep->epr * L.stride;
    Lo.bank_records = static_cast<uint32_t>(ep->epr);
    qf::EpOut act_route = out_route;
    act_route.act_off = ep->act_off;
    act_route.rows_cap = ep->t_max * (qf::kTopK + 1);
    if (e == cudaSuccess)
      e = qf::grouped_ffn_stages(st, Lo, bf16, reinterpret_cast<const uint16_t*>(ep->region + ep->x_off),
                                 ep->rows_cap, ep->act, nullptr, nullptr, ep->tiles, ep->n_tiles, ep->max_tiles,
                                 ep->sms, h->d_status, &h->prof, 1, &act_route, nullptr);
    if (e != cudaSuccess) return qf::cuda_fail(h, e, "EP: grouped gate/up");
    qf::k_ep_signal_done<<<1, 32, 0, st>>>(a);
    // home: every owner's activation rows have landed; the down GEMM of this
    // rank's own rows with all 256 experts, results at the send rows
    qf::k_ep_wait_done<<<1, 32, 0, st>>>(ep->region, a.epoch * (unsigned)ep->world, ep->q_rows, h->d_status,
                                         ep->wait_ns);
    qf::k_ep_home_guard<<<1, qf::kExperts, 0, st>>>(ep->q_rows, ep->counts, ep->pmax_dev, ep->t_max * qf::kTopK);
    e = qf::tile_list(st, ep->counts, ep->offsets, T, ep->pmax_dev, ep->home_tiles, ep->home_n_tiles);
    if (e == cudaSuccess)
      e = qf::grouped_ffn_stages(st, L, bf16, nullptr, static_cast<size_t>(ep->t_max) * (qf::kTopK + 1),
                                 reinterpret_cast<__half*>(ep->region + ep->act_off),
                                 reinterpret_cast<float*>(ep->region + ep->y_off), nullptr, ep->home_tiles,
                                 ep->home_n_tiles, ep->home_max_tiles, ep->sms, h->d_status, &h->prof, 2, nullptr,
                                 nullptr);
    if (e != cudaSuccess) return qf::cuda_fail(h, e, "EP: grouped down");
  }
  {
    qf::ProfScope ps(&h->prof, qf::kKCombine, st);
    qf::k_ep_combine<<<T, 256, 0, st>>>(a, residual, ep->w, ep->coef, out);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return qf::cuda_fail(h, e, "EP: combine");
  ep->epoch++;
  return QF_OK;
}

qf_status qf_ep_set_down_at_home(qf_ep* ep, int32_t enable) {
  if (!ep || (enable != 0 && enable != 1)) return QF_ERR_ARG;
  ep->down_at_home = enable != 0;
  return QF_OK;
}

qf_status qf_ep_set_timeout_ms(qf_ep* ep, uint32_t ms) {
  if (!ep || ms < 1 || ms > 60000) return QF_ERR_ARG;
  ep->wait_ns = static_cast<uint64_t>(ms) * 1000000ull;
  return QF_OK;
}

qf_status qf_ep_info(const qf_ep* ep, int32_t* experts_per_rank, int64_t* receive_rows,
                     uint64_t* region_bytes) {
  if (!ep) return QF_ERR_ARG;
  if (experts_per_rank) *experts_per_rank = ep->epr;
  if (receive_rows) *receive_rows = static_cast<int64_t>(ep->rows_cap);
  if (region_bytes) *region_bytes = ep->region_bytes;
  return QF_OK;
}

}  // extern "C"
