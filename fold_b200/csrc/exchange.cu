// Peer-to-peer exchange of per-rank far-memory partials, fused with the split combine before it and
// the merge after it, for a side cache sharded by position across the GPUs of one node.
//
// Each rank owns one device region, mapped into every other rank's address space with CUDA IPC:
//   recv  [2 parities][world source ranks][max_items] records of kRecordBytes
//   ctr   uint32 [4]: last completed epoch, blocks done in this launch, poisoned
// A record holds one item (row t, query head h, 128-column slice) of one rank's combined partial
// in 16-byte lines {x, epoch, y, epoch}: 64 lines of o (lane l owns lines 2l and 2l+1, i.e.
// columns 4l..4l+3) and one line with the LSE. Every 8-byte half of a line pairs a value with
// the epoch that wrote it, and aligned 8-byte stores and loads are single-copy atomic, so a reader
// that sees the current epoch in both halves of every line it needs has the current data: no
// fence and no separate flag (the low-latency line format that NCCL's LL protocol also uses).
//
// One launch of exchange_merge_kernel on every rank (all ranks make the same sequence of calls);
// block b handles items b, b + grid, ...; per item:
//   1. the block combines this rank's split partials (log-sum-exp) into registers of warp 0;
//   2. warp 0 stores the item's record into slot [parity][this rank] of every other rank (NVLink
//      stores into the peers' memory);
//   3. warp 0 polls its own slots [parity][r] for the item until every line carries this epoch
//      (bounded wait), and merges the world partials (rank order, so that every rank computes the
//      same output) with the window read.
// The epoch is a device counter: every launch uses ctr[0] + 1, and its last block to finish
// stores it, so graph replays need no host input. Records alternate between two parities: a rank
// writes epoch e + 2 into a peer's slot only after its epoch-e+1 launch read the peer's epoch-e+1
// records, which the peer wrote after its epoch-e launch (the last reader of that slot) ended.
//
// No counterpart in the reference (one GPU); it replaces an all-gather of the partials (NCCL)
// followed by the merge kernel. No TMA and no bulk copies are used: plain vector stores to peer
// memory and volatile polling loads of local memory.
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

constexpr int kLinesPerItem = 2 * 32 + 1;  // 64 lines of o + 1 line of LSE
constexpr int kRecordBytes = kLinesPerItem * 16;

struct Exchange {
  int world = 0, rank = 0, device = -1;
  int64_t part_floats = 0;  // floats of one rank's partial at the largest step: n*hq*hd + hq*n
  int max_items = 0;        // items (row, q head, 128-column slice) at the largest step
  size_t bytes = 0, off_ctr = 0;
  char* base = nullptr;           // this rank's region
  char* peer[kMaxRanks] = {};     // every rank's region in this process's address space
  bool opened[kMaxRanks] = {};    // mapped with cudaIpcOpenMemHandle (to be closed)
  bool ready = false;
};

struct ExParams {
  MergeParams m;  // split partials (o_f/lse_f, float32 contiguous) and the window read / output
  char* recv[kMaxRanks];  // every rank's record area
  const char* my_recv;
  uint32_t* ctr;
  int max_items, items, slices, hd;
  int world, rank;
  int* err;
};

__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_line(void* p, float x, float y, uint32_t flag) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(__float_as_uint(x)), "r"(flag),
               "r"(__float_as_uint(y)), "r"(flag)
               : "memory");
}
__device__ __forceinline__ uint4 ld_line(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ bool line_is(const uint4& v, uint32_t flag) { return v.y == flag && v.w == flag; }

// A wait for a peer's record gives up after kPeerWaitTimeoutNs on the global timer, or
// independently of the timer after kPeerWaitMaxPolls polls (which take far longer than that).
constexpr uint32_t kPeerWaitMaxPolls = 1u << 26;

// Polls this lane's lines of one record until they carry `epoch`. False when the exchange is
// poisoned or the wait ran out.
__device__ __forceinline__ bool read_record(const char* rec, int lane, bool active, uint32_t epoch, const uint32_t* poisoned,
                            float (&o)[4], float& lse) {
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 0; it < kPeerWaitMaxPolls; ++it) {
    const uint4 c = ld_line(rec + 64 * 16);
    uint4 a = c, b = c;
    if (active) {
      a = ld_line(rec + (2 * lane) * 16);
      b = ld_line(rec + (2 * lane + 1) * 16);
    }
    if (line_is(a, epoch) && line_is(b, epoch) && line_is(c, epoch)) {
      o[0] = __uint_as_float(a.x), o[1] = __uint_as_float(a.z);
      o[2] = __uint_as_float(b.x), o[3] = __uint_as_float(b.z);
      lse = __uint_as_float(c.x);
      return true;
    }
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
  // the epoch load is in flight while the first combine loads the partials; combine_slice's
  // barrier publishes s_epoch
  if (threadIdx.x == 0) s_epoch = ld_relaxed_gpu(p.ctr) + 1;
  const bool active = lane * 4 < min(p.hd, kSlice);
  const uint32_t* poisoned = p.ctr + 2;
  uint32_t epoch = 0;

  for (int item = blockIdx.x; item < p.items; item += gridDim.x) {
    const int slice = item % p.slices, th = item / p.slices;
    const int t = th / m.hq, h = th - (th / m.hq) * m.hq;
    const int col = slice * kSlice + lane * 4;
    float of[4], lse_far;
    combine_slice(m, t, h, col, active, true, sums, of, lse_far);
    epoch = s_epoch;
    if (warp == 0) {
      const int par = static_cast<int>(epoch & 1u);
      // window read first: its loads overlap the pushes and the wait
      float ol[4] = {0.f, 0.f, 0.f, 0.f};
      if (active) load_row<4>(m.o_l, 1, static_cast<int64_t>(t) * m.ol_st + static_cast<int64_t>(h) * m.ol_sh + col, ol);
      const float ll = m.lse_l[static_cast<int64_t>(h) * m.ll_sh + static_cast<int64_t>(t) * m.ll_st];
      // push this rank's record of the item to every other rank
      const int64_t mine = ((static_cast<int64_t>(par) * p.world + p.rank) * p.max_items + item) * kRecordBytes;
      for (int r = 0; r < p.world; ++r) {
        if (r == p.rank) continue;
        char* rec = p.recv[r] + mine;
        if (active) {
          st_line(rec + (2 * lane) * 16, of[0], of[1], epoch);
          st_line(rec + (2 * lane + 1) * 16, of[2], of[3], epoch);
        }
        if (lane == 0) st_line(rec + 64 * 16, lse_far, lse_far, epoch);
      }
      // every rank's partial of the item, in rank order
      float o_r[kMaxRanks][4], lse_r[kMaxRanks];
      bool ok = true;
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r) {
        lse_r[r] = -INFINITY;
#pragma unroll
        for (int i = 0; i < 4; ++i) o_r[r][i] = of[i];
        if (r < p.world && r != p.rank) {
          const char* rec = p.my_recv + ((static_cast<int64_t>(par) * p.world + r) * p.max_items + item) * kRecordBytes;
          if (!read_record(rec, lane, active, epoch, poisoned, o_r[r], lse_r[r])) {
            ok = false;
            lse_r[r] = -INFINITY;
          }
        } else if (r == p.rank) {
          lse_r[r] = lse_far;
        }
      }
      if (!__all_sync(0xffffffffu, ok) && lane == 0) {
        set_error(p.err, FOLD_DEVERR_TIMEOUT);
        atomicExch(p.ctr + 2, 1u);
      }
      // log-sum-exp over the ranks (lse_r is the same in every lane)
      float mx = -INFINITY;
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r) mx = fmaxf(mx, lse_r[r]);  // ranks >= world hold -inf
      float W = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
      if (mx != -INFINITY) {
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r) {
          const float w = lse_r[r] == -INFINITY ? 0.f : expf(lse_r[r] - mx);
          W += w;
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[i] = fmaf(w, o_r[r][i], acc[i]);
        }
      }
      const bool any = mx != -INFINITY && W > 0.f && row_has_far(m, t);
      const float inv = any ? 1.f / W : 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] *= inv;
      if (active) merge_store_loaded(m, t, h, col, acc, any ? mx + logf(W) : -INFINITY, ol, ll);
    }
    __syncthreads();  // `sums` is reused by the next item
  }

  // the last block of the launch publishes the epoch for the next launch
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
  ex->off_ctr = round_up(static_cast<size_t>(2) * world * max_items * kRecordBytes, 256);
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
  for (int r = 0; r < ex->world; ++r) p.recv[r] = ex->peer[r];
  p.my_recv = ex->base;
  p.ctr = reinterpret_cast<uint32_t*>(ex->base + ex->off_ctr);
  p.max_items = ex->max_items;
  p.items = static_cast<int>(items), p.slices = slices, p.hd = hd;
  p.world = ex->world, p.rank = ex->rank, p.err = err;

  // Block b of every rank handles the same items in the same order and pushes each item before it
  // waits for the peers' records of it, so all blocks must be resident together (a block that
  // waits must not keep the block of another rank that it waits for from running on that rank):
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
