// Peer-to-peer exchange of per-rank far-memory partials, fused with the split combine before it and
// the merge after it, for a side cache sharded by position across the GPUs of one node (the
// region, record format and epochs are described in exchange.cuh).
//
// One launch of exchange_merge_kernel on every rank (all ranks make the same sequence of calls);
// block b handles items b, b + grid, ...; per item:
//   1. the block combines this rank's split partials (log-sum-exp) into registers of warp 0;
//   2. warp 0 stores the item's record into slot [parity][this rank] of every other rank (NVLink
//      stores into the peers' memory);
//   3. warp 0 polls its own slots [parity][r] for the item until every line carries this epoch
//      (bounded wait), and merges the world partials (rank order, so that every rank computes the
//      same output) with the window read.
//
// No counterpart in the reference (one GPU); it replaces an all-gather of the partials (NCCL)
// followed by the merge kernel. far_exchange.cu does the same work at the end of the far read.
#include <cuda_bf16.h>

#include <cstring>
#include <new>

#include "exchange.cuh"
#include "host_common.h"

namespace fold {

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
  ExchangeView ex;
  int items, slices, hd;
  int* err;
};

// Block b of every rank handles items b, b + grid, ...; per item the block combines this rank's
// split partials (log-sum-exp) into registers of warp 0, and warp 0 exchanges and merges the item.
__global__ void __launch_bounds__(kMergeWarps * 32) exchange_merge_kernel(const ExParams p) {
  __shared__ SliceSums sums;
  __shared__ uint32_t s_epoch;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const MergeParams& m = p.m;
  // the epoch load is in flight while the first combine loads the partials; combine_slice's
  // barrier publishes s_epoch. The counter is written only by the previous exchange launch, which
  // completed before this one's producer (the far read) started.
  if (threadIdx.x == 0) s_epoch = ld_relaxed_gpu(p.ex.ctr) + 1;
  // Launched behind the far read: its partials (and every write of the kernels before it, which
  // had completed when the far read released its dependents) are visible from here on.
  wait_for_producer();
  const bool active = lane * 4 < min(p.hd, kSlice);
  uint32_t epoch = 0;

  for (int item = blockIdx.x; item < p.items; item += gridDim.x) {
    const int slice = item % p.slices, th = item / p.slices;
    const int t = th / m.hq, h = th - (th / m.hq) * m.hq;
    const int col = slice * kSlice + lane * 4;
    float of[4], lse_far;
    combine_slice(m, t, h, col, active, true, sums, of, lse_far, m.splits);
    epoch = s_epoch;
    if (warp == 0) {
      // window read first: its loads overlap the pushes and the wait
      float ol[4] = {0.f, 0.f, 0.f, 0.f};
      if (active) load_row<4>(m.o_l, 1, static_cast<int64_t>(t) * m.ol_st + static_cast<int64_t>(h) * m.ol_sh + col, ol);
      const float ll = m.lse_l[static_cast<int64_t>(h) * m.ll_sh + static_cast<int64_t>(t) * m.ll_st];
      exchange_item(p.ex, m, item, t, h, col, active, of, lse_far, ol, ll, epoch, p.err);
    }
    __syncthreads();  // `sums` is reused by the next item
  }
  exchange_publish_epoch(p.ex, epoch, gridDim.x);
}

static size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

static int current_device(int* dev) { return check_cuda(cudaGetDevice(dev), "exchange: cudaGetDevice"); }

int exchange_view(void* exchange, int n, int hq, int hd, ExchangeView* view) {
  Exchange* ex = static_cast<Exchange*>(exchange);
  if (!ex) return fail(FOLD_ERR_INVALID_ARGUMENT, "exchange: null pointer");
  if (!ex->ready) return fail(FOLD_ERR_INVALID_ARGUMENT, "exchange: the exchange is not open");
  const int slices = hd > kSlice ? hd / kSlice : 1;
  const int64_t items = static_cast<int64_t>(n) * hq * slices;
  const int64_t part = static_cast<int64_t>(n) * hq * hd + static_cast<int64_t>(hq) * n;
  if (part > ex->part_floats || items > ex->max_items)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "exchange: the step is larger than the exchange was created for");
  int dev;
  if (int st = current_device(&dev)) return st;
  if (dev != ex->device) return fail(FOLD_ERR_INVALID_ARGUMENT, "exchange: called on another device");
  ExchangeView v{};
  for (int r = 0; r < ex->world; ++r) v.recv[r] = ex->peer[r];
  v.my_recv = ex->base;
  v.ctr = reinterpret_cast<uint32_t*>(ex->base + ex->off_ctr);
  v.done = reinterpret_cast<uint32_t*>(ex->base + ex->off_ctr + kCtrBytes);
  v.max_items = ex->max_items, v.world = ex->world, v.rank = ex->rank;
  *view = v;
  return FOLD_OK;
}

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
  ex->bytes = ex->off_ctr + kCtrBytes + kMaxKvHeads * sizeof(uint32_t);
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
  if (ol_stride_tok % 2 || ol_stride_head % 2 || out_stride_tok % 2 || out_stride_head % 2 ||
      (reinterpret_cast<uintptr_t>(o_l) & 3) || (reinterpret_cast<uintptr_t>(out) & 3) ||
      (reinterpret_cast<uintptr_t>(o_part) & 7))
    return fail(FOLD_ERR_ALIGNMENT, "exchange merge: rows must start on element pairs");
  ExParams p{};
  if (int st = exchange_view(ex, n, hq, hd, &p.ex)) return st;
  MergeParams& m = p.m;
  m.o_l = static_cast<const __nv_bfloat16*>(o_l), m.ol_st = ol_stride_tok, m.ol_sh = ol_stride_head;
  m.lse_l = lse_l, m.ll_sh = ll_stride_head, m.ll_st = ll_stride_tok;
  m.o_f = o_part, m.of_bf16 = 0;
  m.of_ss = static_cast<int64_t>(n) * hq * hd, m.of_st = static_cast<int64_t>(hq) * hd, m.of_sh = hd;
  m.lse_f = lse_part, m.lf_ss = static_cast<int64_t>(hq) * n, m.lf_sh = n, m.lf_st = 1;
  m.splits = splits;
  m.out = static_cast<__nv_bfloat16*>(out), m.out_st = out_stride_tok, m.out_sh = out_stride_head;
  m.qsl = qsl, m.seq = seq_lens, m.n = n, m.hq = hq, m.window = window, m.block = block, m.inv_alpha = inv_alpha;
  p.items = static_cast<int>(items), p.slices = slices, p.hd = hd;
  p.err = err;

  // Block b of every rank handles the same items in the same order and pushes each item before it
  // waits for the peers' records of it, so all blocks must be resident together (a block that
  // waits must not keep the block of another rank that it waits for from running on that rank):
  // the grid is at most what the device holds at once, and the launch is cooperative.
  int per_sm = 0;
  int st = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, exchange_merge_kernel, kMergeWarps * 32, 0),
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
  // Cooperative, and behind the far read (programmatic stream serialisation): the blocks are
  // scheduled as the far read's CTAs finish instead of after the whole grid has retired, and wait
  // for it in wait_for_producer.
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr, cfg.numAttrs = 2;
  st = check_cuda(cudaLaunchKernelEx(&cfg, exchange_merge_kernel, p), "exchange merge: launch");
  if (st) return st;
  return check_launch("exchange_merge_kernel");
}

}  // extern "C"
