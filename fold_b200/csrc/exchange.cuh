// The peer exchange of per-rank far-memory partials, as device pieces shared by the standalone
// exchange kernel (exchange.cu) and the far read that ends with the exchange (far_exchange.cu).
//
// Each rank owns one device region, mapped into every other rank's address space with CUDA IPC:
//   recv  [2 parities][world source ranks][max_items] records of kRecordBytes
//   ctr   uint32 [4]: last completed epoch, blocks done in this launch, poisoned
//   done  uint32 [kMaxKvHeads]: far-read splits finished per KV head in the current launch (the
//         fused read; its last block zeroes them)
// A record holds one item (row t, query head h, 128-column slice) of one rank's combined partial
// in 16-byte lines {x, epoch, y, epoch}: 64 lines of o (lane l owns lines l and 32 + l, i.e.
// columns 4l, 4l+1 and 4l+2, 4l+3, so that each warp-wide store covers 512 contiguous bytes: whole
// 128-byte requests over NVLink) and one line with the LSE. Every 8-byte half of a line pairs a value with
// the epoch that wrote it, and aligned 8-byte stores and loads are single-copy atomic, so a reader
// that sees the current epoch in both halves of every line it needs has the current data: no
// fence and no separate flag (the low-latency line format that NCCL's LL protocol also uses).
//
// The epoch is a device counter: every launch uses ctr[0] + 1, and its last block to finish
// stores it, so graph replays need no host input. Records alternate between two parities: a rank
// writes epoch e + 2 into a peer's slot only after its epoch-e+1 launch read the peer's epoch-e+1
// records, which the peer wrote after its epoch-e launch (the last reader of that slot) ended.
// No TMA and no bulk copies: plain vector stores to peer memory and volatile loads of local
// memory.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"
#include "merge.cuh"

namespace fold {

constexpr int kMaxRanks = 8;
constexpr int kMaxKvHeads = 256;
// A wait for a peer's partial (or, in the fused read, for this rank's splits) gives up after this
// long: the kernel records FOLD_DEVERR_TIMEOUT, marks the exchange poisoned (later launches do not
// wait at all) and merges what it has.
constexpr uint64_t kPeerWaitTimeoutNs = 2000000000ull;
// ... or, independently of the timer, after this many polls (which take far longer than that).
constexpr uint32_t kPeerWaitMaxPolls = 1u << 26;

constexpr int kLinesPerItem = 2 * 32 + 1;  // 64 lines of o + 1 line of LSE
constexpr int kRecordBytes = kLinesPerItem * 16;
constexpr int kCtrBytes = 256;  // ctr area; the done counters follow it

// The device view of one rank's exchange.
struct ExchangeView {
  char* recv[kMaxRanks];  // every rank's record area, in this process's address space
  const char* my_recv;
  uint32_t* ctr;
  uint32_t* done;
  int max_items, world, rank;
};

// Host side (exchange.cu): the view of `exchange` for a step of n rows, hq query heads and head
// size hd, after checking that the step fits the exchange and runs on its device.
int exchange_view(void* exchange, int n, int hq, int hd, ExchangeView* view);

__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
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

// Polls this lane's lines of one record until they carry `epoch`. False when the exchange is
// poisoned or the wait ran out.
__device__ __forceinline__ bool read_record(const char* rec, int lane, bool active, uint32_t epoch,
                                            const uint32_t* poisoned, float (&o)[4], float& lse) {
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 0; it < kPeerWaitMaxPolls; ++it) {
    const uint4 c = ld_line(rec + 64 * 16);
    uint4 a = c, b = c;
    if (active) {
      a = ld_line(rec + lane * 16);
      b = ld_line(rec + (32 + lane) * 16);
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

// Exchange and merge of one item by one warp, given this rank's combined partial of it (of, the
// LSE lse_far) on the columns [col, col + 4) of each lane: stores the item's record into every
// other rank's slot, waits (bounded) for every other rank's record, combines the world partials
// in rank order (so that every rank computes the same output) and merges them with the window
// read into the bf16 output. ol/ll are the window read's values of the lane.
__device__ __forceinline__ void exchange_item(const ExchangeView& ex, const MergeParams& m, int item, int t, int h,
                                              int col, bool active, const float (&of)[4], float lse_far,
                                              const float (&ol)[4], float ll, uint32_t epoch, int* err) {
  const int lane = threadIdx.x & 31;
  const int par = static_cast<int>(epoch & 1u);
  const uint32_t* poisoned = ex.ctr + 2;
  const int64_t mine = ((static_cast<int64_t>(par) * ex.world + ex.rank) * ex.max_items + item) * kRecordBytes;
  for (int r = 0; r < ex.world; ++r) {
    if (r == ex.rank) continue;
    char* rec = ex.recv[r] + mine;
    if (active) {
      st_line(rec + lane * 16, of[0], of[1], epoch);
      st_line(rec + (32 + lane) * 16, of[2], of[3], epoch);
    }
    if (lane == 0) st_line(rec + 64 * 16, lse_far, lse_far, epoch);
  }
  float o_r[kMaxRanks][4], lse_r[kMaxRanks];
  bool ok = true;
#pragma unroll
  for (int r = 0; r < kMaxRanks; ++r) {
    lse_r[r] = -INFINITY;
#pragma unroll
    for (int i = 0; i < 4; ++i) o_r[r][i] = of[i];
    if (r < ex.world && r != ex.rank) {
      const char* rec = ex.my_recv + ((static_cast<int64_t>(par) * ex.world + r) * ex.max_items + item) * kRecordBytes;
      if (!read_record(rec, lane, active, epoch, poisoned, o_r[r], lse_r[r])) {
        ok = false;
        lse_r[r] = -INFINITY;
      }
    } else if (r == ex.rank) {
      lse_r[r] = lse_far;
    }
  }
  if (!__all_sync(0xffffffffu, ok) && lane == 0) {
    set_error(err, FOLD_DEVERR_TIMEOUT);
    atomicExch(ex.ctr + 2, 1u);
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

// Counts this launch's block as done; the last block zeroes `reset[0, nreset)` (counters that
// every block of the launch has finished with) and publishes the launch's epoch for the next.
__device__ __forceinline__ void exchange_publish_epoch(const ExchangeView& ex, uint32_t epoch, unsigned blocks,
                                                       uint32_t* reset = nullptr, int nreset = 0) {
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(ex.ctr + 1, 1u) == blocks - 1) {
      for (int i = 0; i < nreset; ++i) reset[i] = 0u;
      atomicExch(ex.ctr + 1, 0u);
      __threadfence();
      atomicExch(ex.ctr, epoch);
    }
  }
}

}  // namespace fold
