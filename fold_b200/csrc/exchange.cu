// Peer-to-peer exchange of per-rank far-memory partials, fused with the split combine before it and
// the merge after it, for a side cache sharded by position across the GPUs of one node.
//
// Each rank owns one device region, mapped into every other rank's address space with CUDA IPC:
//   recv  float32 [2 parities][world][part_floats]   partials pushed by every rank
//   flags uint32  [world][max_items]                  epoch at which rank r pushed item i
//   ctr   uint32  [4]: last completed epoch, blocks done in this launch, poisoned
// One launch of exchange_merge_kernel on every rank (all ranks make the same sequence of calls):
//   1. per item (row t, query head h, 128-column slice): combine this rank's split partials
//      (log-sum-exp), store the result into the recv slot [parity][rank] of EVERY rank (NVLink
//      stores into the peers' memory), fence, and raise flag [rank][item] on every rank;
//   2. per item: wait until every rank's flag for the item reaches this epoch (bounded wait), then
//      merge the world partials with the window read and write the bf16 output.
// The epoch is a device counter: every launch uses ctr[0] + 1, and its last block to finish
// stores it, so graph replays need no host input. Data slots alternate between two parities: a
// rank can be at most one epoch ahead of a peer that is still reading (its own epoch-e+1 wait
// needs the peer's epoch-e+1 push, which the peer issues only after its epoch-e launch is done).
//
// No counterpart in the reference (one GPU); it replaces an all-gather of the partials (NCCL)
// followed by the merge kernel. No TMA and no bulk copies are used: plain vector stores to peer
// memory, release/acquire flags at system scope.
#include <cuda_bf16.h>

#include <cstring>
#include <new>

#include "common.cuh"
#include "host_common.h"
#include "merge.cuh"

namespace fold {

constexpr int kMaxRanks = 8;
// A wait for a peer's partial gives up after this long: the kernel records FOLD_DEVERR_TIMEOUT,
// marks the exchange poisoned (later launches do not wait at all) and merges what it has.
constexpr uint64_t kPeerWaitTimeoutNs = 2000000000ull;

struct Exchange {
  int world = 0, rank = 0, device = -1;
  int64_t part_floats = 0;  // floats of one rank's partial: n*hq*hd + hq*n at the largest shape
  int max_items = 0;        // items (row, q head, 128-column slice) at the largest shape
  size_t bytes = 0, off_flags = 0, off_ctr = 0;
  char* base = nullptr;           // this rank's region
  char* peer[kMaxRanks] = {};     // every rank's region in this process's address space
  bool opened[kMaxRanks] = {};    // mapped with cudaIpcOpenMemHandle (to be closed)
  bool ready = false;
};

struct ExParams {
  MergeParams m;  // split partials (o_f/lse_f, float32 contiguous) and the window read / output
  float* recv[kMaxRanks];
  uint32_t* flags[kMaxRanks];
  const float* my_recv;
  const uint32_t* my_flags;
  uint32_t* ctr;
  int64_t part_floats;
  int max_items, items, slices, hd;
  int world, rank;
  int* err;
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits until *flag has reached `epoch` (wrap-safe). False when the exchange is poisoned or the
// wait ran out of time (kPeerWaitTimeoutNs on the global timer; independently of the timer, after
// kPeerWaitMaxPolls polls, which take far longer than that).
constexpr uint32_t kPeerWaitMaxPolls = 1u << 26;
__device__ bool wait_epoch(const uint32_t* flag, uint32_t epoch, const uint32_t* poisoned) {
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 0; it < kPeerWaitMaxPolls; ++it) {
    if (static_cast<int32_t>(ld_acquire_sys(flag) - epoch) >= 0) return true;
    if ((it & 31u) == 31u) {
      if (ld_relaxed_gpu(poisoned)) return false;
      if (globaltimer() - t0 > kPeerWaitTimeoutNs) return false;
    }
    if (it >= 256) __nanosleep(64);
  }
  return false;
}

__global__ void __launch_bounds__(kMergeWarps * 32) exchange_merge_kernel(const ExParams p) {
  __shared__ SliceSums sums;
  __shared__ uint32_t s_epoch;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const MergeParams& m = p.m;
  if (threadIdx.x == 0) s_epoch = ld_relaxed_gpu(p.ctr) + 1;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  const int64_t slot = (static_cast<int64_t>(epoch & 1u) * p.world + p.rank) * p.part_floats;
  const bool active = lane * 4 < min(p.hd, kSlice);
  const int64_t lse_base = static_cast<int64_t>(m.n) * m.hq * p.hd;

  // 1. combine this rank's splits of each item and push the result to every rank
  for (int item = blockIdx.x; item < p.items; item += gridDim.x) {
    const int slice = item % p.slices, th = item / p.slices;
    const int t = th / m.hq, h = th - (th / m.hq) * m.hq;
    const int col = slice * kSlice + lane * 4;
    float of[4], lse_far;
    combine_slice(m, t, h, col, active, true, sums, of, lse_far);
    if (warp == 0) {
      const int64_t o_off = slot + (static_cast<int64_t>(t) * m.hq + h) * p.hd + col;
      const int64_t l_off = slot + lse_base + static_cast<int64_t>(h) * m.n + t;
      // every slice of (t, h) stores the same LSE, so that each item's flag covers what its
      // reader loads
      for (int r = 0; r < p.world; ++r) {
        if (active) *reinterpret_cast<float4*>(p.recv[r] + o_off) = make_float4(of[0], of[1], of[2], of[3]);
        if (lane == 0) p.recv[r][l_off] = lse_far;
      }
      __threadfence_system();
      __syncwarp();
      if (lane < p.world) st_release_sys(p.flags[lane] + static_cast<int64_t>(p.rank) * p.max_items + item, epoch);
    }
    __syncthreads();  // `sums` is reused by the next item
  }

  // 2. per item (one warp each): wait for every rank's partial, merge with the window read
  const uint32_t* poisoned = p.ctr + 2;
  for (int item = blockIdx.x * kMergeWarps + warp; item < p.items; item += gridDim.x * kMergeWarps) {
    const int slice = item % p.slices, th = item / p.slices;
    const int t = th / m.hq, h = th - (th / m.hq) * m.hq;
    const int col = slice * kSlice + lane * 4;
    bool ok = true;
    if (lane < p.world) ok = wait_epoch(p.my_flags + static_cast<int64_t>(lane) * p.max_items + item, epoch, poisoned);
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0) {
        set_error(p.err, FOLD_DEVERR_TIMEOUT);
        atomicExch(p.ctr + 2, 1u);
      }
    }
    __syncwarp();
    const int64_t base = static_cast<int64_t>(epoch & 1u) * p.world * p.part_floats;
    const float l = lane < p.world
                        ? __ldcg(p.my_recv + base + lane * p.part_floats + lse_base + static_cast<int64_t>(h) * m.n + t)
                        : -INFINITY;
    const float mx = warp_max(l);
    const float w = l == -INFINITY ? 0.f : expf(l - mx);
    const float W = warp_sum(w);
    float of[4] = {0.f, 0.f, 0.f, 0.f};
    const int64_t o_off = base + (static_cast<int64_t>(t) * m.hq + h) * p.hd + col;
    for (int r = 0; r < p.world; ++r) {
      const float wr = __shfl_sync(0xffffffffu, w, r);
      if (active && wr > 0.f) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(p.my_recv + o_off + r * p.part_floats));
        of[0] = fmaf(wr, v.x, of[0]), of[1] = fmaf(wr, v.y, of[1]);
        of[2] = fmaf(wr, v.z, of[2]), of[3] = fmaf(wr, v.w, of[3]);
      }
    }
    const bool any = mx != -INFINITY && W > 0.f && row_has_far(m, t);
    const float inv = any ? 1.f / W : 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) of[i] *= inv;
    if (active) merge_store(m, t, h, col, of, any ? mx + logf(W) : -INFINITY);
  }

  // the last block of the launch publishes the epoch for the next launch
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(p.ctr + 1, 1u) == gridDim.x - 1) {
      atomicExch(p.ctr + 1, 0u);
      __threadfence();
      atomicExch(p.ctr, epoch);
    }
  }
}

static size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

static int current_device(int* dev) { return check_cuda(cudaGetDevice(dev), "exchange: cudaGetDevice"); }

}  // namespace fold

extern "C" {

int fold_exchange_create(int world, int rank, int64_t part_floats, int max_items, void** exchange, void* handle) {
  using namespace fold;
  static_assert(sizeof(cudaIpcMemHandle_t) == FOLD_EXCHANGE_HANDLE_BYTES, "IPC handle size");
  if (!exchange || !handle) return fail(FOLD_ERR_INVALID_ARGUMENT, "exchange: null pointer");
  *exchange = nullptr;
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "exchange: world must be 1..8 and 0 <= rank < world");
  if (part_floats < 1 || part_floats % 4 || max_items < 1)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "exchange: partial size must be a positive multiple of 4 floats");
  Exchange* ex = new (std::nothrow) Exchange();
  if (!ex) return fail(FOLD_ERR_INVALID_ARGUMENT, "exchange: out of host memory");
  ex->world = world, ex->rank = rank, ex->part_floats = part_floats, ex->max_items = max_items;
  ex->off_flags = round_up(sizeof(float) * 2 * static_cast<size_t>(world) * part_floats, 256);
  ex->off_ctr = ex->off_flags + round_up(sizeof(uint32_t) * static_cast<size_t>(world) * max_items, 256);
  ex->bytes = ex->off_ctr + 256;
  int st = current_device(&ex->device);
  if (!st) st = check_cuda(cudaMalloc(&ex->base, ex->bytes), "exchange: cudaMalloc");
  if (!st) st = check_cuda(cudaMemset(ex->base, 0, ex->bytes), "exchange: cudaMemset");
  if (!st) st = check_cuda(cudaDeviceSynchronize(), "exchange: cudaDeviceSynchronize");
  cudaIpcMemHandle_t h;
  if (!st) st = check_cuda(cudaIpcGetMemHandle(&h, ex->base), "exchange: cudaIpcGetMemHandle");
  if (st) {
    if (ex->base) cudaFree(ex->base);
    delete ex;
    return st;
  }
  std::memcpy(handle, &h, sizeof(h));
  ex->peer[rank] = ex->base;
  *exchange = ex;
  return FOLD_OK;
}

int fold_exchange_open(void* exchange, const void* handles) {
  using namespace fold;
  Exchange* ex = static_cast<Exchange*>(exchange);
  if (!ex || !handles) return fail(FOLD_ERR_INVALID_ARGUMENT, "exchange: null pointer");
  if (ex->ready) return fail(FOLD_ERR_INVALID_ARGUMENT, "exchange: already open");
  int dev;
  int st = current_device(&dev);
  if (st) return st;
  if (dev != ex->device) return fail(FOLD_ERR_INVALID_ARGUMENT, "exchange: opened on another device than created");
  for (int r = 0; r < ex->world; ++r) {
    if (r == ex->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const char*>(handles) + static_cast<size_t>(r) * sizeof(h), sizeof(h));
    void* p = nullptr;
    st = check_cuda(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "exchange: cudaIpcOpenMemHandle");
    if (st) return st;
    ex->peer[r] = static_cast<char*>(p);
    ex->opened[r] = true;
  }
  ex->ready = true;
  return FOLD_OK;
}

int fold_exchange_destroy(void* exchange) {
  using namespace fold;
  Exchange* ex = static_cast<Exchange*>(exchange);
  if (!ex) return FOLD_OK;
  int st = FOLD_OK;
  for (int r = 0; r < ex->world; ++r) {
    if (ex->opened[r]) {
      const int s = check_cuda(cudaIpcCloseMemHandle(ex->peer[r]), "exchange: cudaIpcCloseMemHandle");
      if (!st) st = s;
    }
  }
  if (ex->base) {
    const int s = check_cuda(cudaFree(ex->base), "exchange: cudaFree");
    if (!st) st = s;
  }
  delete ex;
  return st;
}

int fold_exchange_merge(void* exchange, const float* o_part, const float* lse_part, int splits, const void* o_l,
                        int64_t ol_stride_tok, int64_t ol_stride_head, const float* lse_l, int64_t ll_stride_head,
                        int64_t ll_stride_tok, void* out, int64_t out_stride_tok, int64_t out_stride_head,
                        const int* qsl, const int* seq_lens, int n, int hq, int hd, int window, int block,
                        float inv_alpha, int* err, void* stream) {
  using namespace fold;
  Exchange* ex = static_cast<Exchange*>(exchange);
  if (!ex || !o_part || !lse_part || !o_l || !lse_l || !out || !qsl || !seq_lens)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "exchange merge: null pointer");
  if (!ex->ready) return fail(FOLD_ERR_INVALID_ARGUMENT, "exchange merge: the exchange is not open");
  if (n < 1 || hq < 1 || splits < 1) return fail(FOLD_ERR_INVALID_ARGUMENT, "exchange merge: bad sizes");
  if (hd < 4 || (hd > kSlice && hd % kSlice) || (hd <= kSlice && hd % 4))
    return fail(FOLD_ERR_UNSUPPORTED, "exchange merge: head size must be a multiple of 128, or of 4 up to 128");
  const int slices = hd > kSlice ? hd / kSlice : 1;
  const int64_t items = static_cast<int64_t>(n) * hq * slices;
  const int64_t part = static_cast<int64_t>(n) * hq * hd + static_cast<int64_t>(hq) * n;
  if (part > ex->part_floats || items > ex->max_items)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "exchange merge: the step is larger than the exchange was created for");
  if (ol_stride_tok % 2 || ol_stride_head % 2 || out_stride_tok % 2 || out_stride_head % 2 ||
      (reinterpret_cast<uintptr_t>(o_l) & 3) || (reinterpret_cast<uintptr_t>(out) & 3) ||
      (reinterpret_cast<uintptr_t>(o_part) & 7))
    return fail(FOLD_ERR_ALIGNMENT, "exchange merge: rows must start on element pairs");
  int dev;
  int st = current_device(&dev);
  if (st) return st;
  if (dev != ex->device) return fail(FOLD_ERR_INVALID_ARGUMENT, "exchange merge: called on another device");

  ExParams p{};
  MergeParams& m = p.m;
  m.o_l = static_cast<const __nv_bfloat16*>(o_l), m.ol_st = ol_stride_tok, m.ol_sh = ol_stride_head;
  m.lse_l = lse_l, m.ll_sh = ll_stride_head, m.ll_st = ll_stride_tok;
  m.o_f = o_part, m.of_bf16 = 0;
  m.of_ss = static_cast<int64_t>(n) * hq * hd, m.of_st = static_cast<int64_t>(hq) * hd, m.of_sh = hd;
  m.lse_f = lse_part, m.lf_ss = static_cast<int64_t>(hq) * n, m.lf_sh = n, m.lf_st = 1;
  m.splits = splits;
  m.out = static_cast<__nv_bfloat16*>(out), m.out_st = out_stride_tok, m.out_sh = out_stride_head;
  m.qsl = qsl, m.seq = seq_lens, m.n = n, m.hq = hq, m.window = window, m.block = block, m.inv_alpha = inv_alpha;
  for (int r = 0; r < ex->world; ++r) {
    p.recv[r] = reinterpret_cast<float*>(ex->peer[r]);
    p.flags[r] = reinterpret_cast<uint32_t*>(ex->peer[r] + ex->off_flags);
  }
  p.my_recv = reinterpret_cast<const float*>(ex->base);
  p.my_flags = reinterpret_cast<const uint32_t*>(ex->base + ex->off_flags);
  p.ctr = reinterpret_cast<uint32_t*>(ex->base + ex->off_ctr);
  p.part_floats = ex->part_floats, p.max_items = ex->max_items;
  p.items = static_cast<int>(items), p.slices = slices, p.hd = hd;
  p.world = ex->world, p.rank = ex->rank, p.err = err;

  // Every block pushes all of its items before it waits for any, and all blocks must be resident
  // together (a block that waits must not keep a pushing block of another rank from running):
  // the grid is at most what the device holds at once, and the launch is cooperative.
  int per_sm = 0;
  st = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, exchange_merge_kernel, kMergeWarps * 32, 0),
                  "exchange merge: occupancy");
  if (st) return st;
  int sms = device_sm_count();
  if (sms <= 0) sms = 148;
  const int64_t cap = static_cast<int64_t>(per_sm) * sms;
  if (cap < 1) return fail(FOLD_ERR_CUDA, "exchange merge: kernel does not fit on an SM");
  const int grid = static_cast<int>(items < cap ? items : cap);

  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid), cfg.blockDim = dim3(kMergeWarps * 32), cfg.dynamicSmemBytes = 0;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr, cfg.numAttrs = 1;
  st = check_cuda(cudaLaunchKernelEx(&cfg, exchange_merge_kernel, p), "exchange merge: launch");
  if (st) return st;
  return check_launch("exchange_merge_kernel");
}

}  // extern "C"
