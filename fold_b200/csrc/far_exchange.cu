// The far read that ends with the exchange of the ranks' partials and the merge, in one
// cooperative launch per rank: the compute step (the split-KV read of this rank's chunk of the
// side cache) and the collective (the NVLink exchange of the combined partials) in one kernel.
//
// Every CTA first runs the far read of its split (split_read.cuh) and writes its partial. It then
// counts the split as finished in a per-KV-head counter of the exchange region and waits (bounded)
// until every split of its KV head has finished. The head's items (row, query head of the group,
// 128-column slice) are shared out over the head's CTAs, one warp per item. For each item the warp:
//   1. combines the head's split partials by log-sum-exp (from L2);
//   2. stores the item's record into every other rank's slot over NVLink;
//   3. waits for the other ranks' records of the item;
//   4. merges the world partials with the window read into the output (exchange.cuh).
// With one rank (an exchange without peers) it is the far read and the merge in one launch.
//
// All CTAs wait for one another, so the launch is cooperative: the grid (splits x KV heads, one
// CTA per SM) is resident at once. Every rank makes the same sequence of calls with the same
// split count, so that an item is pushed and awaited by the same warp on every rank, and every
// warp pushes an item before it waits for it.
#include <cuda_bf16.h>

#include "exchange.cuh"
#include "far_launch.h"
#include "host_common.h"

namespace fold {

struct TailParams {
  ExchangeView ex;
  MergeParams m;  // this rank's far partials (o_f/lse_f, float32 contiguous), the window read, the output
  int slices, hd;
};

// Log-sum-exp combine of the split partials of (row t, query head h) on the columns
// [col, col + 4) of this lane, by one warp. The partials were written by other CTAs of this
// launch: they are read from L2 (ld.global.cg), never from this SM's L1.
__device__ __forceinline__ void warp_combine(const MergeParams& m, int t, int h, int col, bool active,
                                             float (&of)[4], float& lse) {
  constexpr int BATCH = 8;
  const int lane = threadIdx.x & 31;
  const float* lf = m.lse_f + static_cast<int64_t>(h) * m.lf_sh + static_cast<int64_t>(t) * m.lf_st;
  float mx = -INFINITY;
  for (int s = lane; s < m.splits; s += 32) mx = fmaxf(mx, __ldcg(lf + s * m.lf_ss));
  mx = warp_max(mx);
  float acc[4] = {0.f, 0.f, 0.f, 0.f}, wsum = 0.f;
  if (mx != -INFINITY) {
    const float* o = static_cast<const float*>(m.o_f) + static_cast<int64_t>(t) * m.of_st +
                     static_cast<int64_t>(h) * m.of_sh + col;
    for (int sb = 0; sb < m.splits; sb += 32) {
      const int cnt = min(32, m.splits - sb);
      const float l = lane < cnt ? __ldcg(lf + (sb + lane) * m.lf_ss) : -INFINITY;
      const float w = l == -INFINITY ? 0.f : expf(l - mx);  // an empty split carries no mass
      wsum += w;
      for (int j = 0; j < cnt; j += BATCH) {
        float4 v[BATCH];
#pragma unroll
        for (int u = 0; u < BATCH; ++u)
          v[u] = (active && j + u < cnt) ? __ldcg(reinterpret_cast<const float4*>(o + (sb + j + u) * m.of_ss))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < BATCH; ++u) {
          const float wu = __shfl_sync(0xffffffffu, w, (j + u) & 31);
          if (j + u < cnt) {
            acc[0] = fmaf(wu, v[u].x, acc[0]), acc[1] = fmaf(wu, v[u].y, acc[1]);
            acc[2] = fmaf(wu, v[u].z, acc[2]), acc[3] = fmaf(wu, v[u].w, acc[3]);
          }
        }
      }
    }
    wsum = warp_sum(wsum);
  }
  const bool any = mx != -INFINITY && wsum > 0.f;
  const float inv = any ? 1.f / wsum : 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) of[i] = acc[i] * inv;
  lse = any ? mx + logf(wsum) : -INFINITY;
}

// Everything after a CTA's far read: count its split, wait for the KV head's other splits, then
// combine, exchange and merge this CTA's share of the head's items. Not inlined: compiled into the
// kernel body, this code changes the code generation of the far read's loop (which uses all 255
// registers) and slowed the whole read by about 20 %; as a call it costs the loop about 5 %.
template <int NW>
__device__ __noinline__ void exchange_tail(const FarParams& p, const TailParams& t, int split, int h) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint32_t* done = t.ex.done;  // zero at the start of every launch: its last CTA resets it
  // the previous launch's last block stored ctr[0] (read here, not before the far read, so that
  // the far read's loop keeps all its registers)
  const uint32_t epoch = ld_relaxed_gpu(t.ex.ctr) + 1;
  __threadfence();  // this thread's partial stores, before the split is counted
  __syncthreads();
  if (tid == 0) {
    atomicAdd(done + h, 1u);
    bool ok = true;
    const uint64_t t0 = globaltimer();
    // This rank's own splits: the cooperative launch keeps every CTA resident, so they finish.
    // Only the timer and the poll bound end this wait; a poisoned exchange (a peer that stopped
    // answering) must not cut it short, or the combine below would read partials still in flight.
    for (uint32_t it = 0; ld_acquire_gpu(done + h) < static_cast<uint32_t>(p.splits); ++it) {
      if (it >= kPeerWaitMaxPolls || ((it & 31u) == 31u && globaltimer() - t0 > kPeerWaitTimeoutNs)) {
        ok = false;
        break;
      }
      __nanosleep(32);
    }
    if (!ok) {
      set_error(p.err, FOLD_DEVERR_TIMEOUT);
      atomicExch(t.ex.ctr + 2, 1u);
    }
  }
  __syncthreads();

  const MergeParams& m = t.m;
  const int G = p.group, slices = t.slices;
  const int items_h = p.n * G * slices;
  const bool active = lane * 4 < min(t.hd, kSlice);
  for (int k = split + p.splits * warp; k < items_h; k += p.splits * NW) {
    const int slice = k % slices, tg = k / slices;
    const int r = tg / G, hq = h * G + (tg - (tg / G) * G);
    const int item = (r * m.hq + hq) * slices + slice;  // the exchange's item numbering
    const int col = slice * kSlice + lane * 4;
    float ol[4] = {0.f, 0.f, 0.f, 0.f};
    if (active) load_row<4>(m.o_l, 1, static_cast<int64_t>(r) * m.ol_st + static_cast<int64_t>(hq) * m.ol_sh + col, ol);
    const float ll = m.lse_l[static_cast<int64_t>(hq) * m.ll_sh + static_cast<int64_t>(r) * m.ll_st];
    float of[4], lse_far;
    warp_combine(m, r, hq, col, active, of, lse_far);
    exchange_item(t.ex, m, item, r, hq, col, active, of, lse_far, ol, ll, epoch, p.err);
  }
  __syncthreads();
  exchange_publish_epoch(t.ex, epoch, gridDim.x * gridDim.y, done, p.hkv);
}

template <class C>
__global__ void __launch_bounds__(C::NTHREADS, 1)
    far_exchange_kernel(const __grid_constant__ CUtensorMap map, const __grid_constant__ FarParams p,
                        const __grid_constant__ TailParams t) {
  split_read<C, false>(&map, nullptr, p, blockIdx.x, blockIdx.y, p.splits);
  exchange_tail<C::NW>(p, t, blockIdx.x, blockIdx.y);
}

struct FarExchangeLaunch {
  const FarParams& prm;
  const TailParams& tail;
  const void* side;
  int pages;
  cudaStream_t stream;
  template <class C>
  int run() const {
    CUtensorMap map;
    if (int s = side_tensor_map(side, pages, prm.hkv, C::HD, C::TK, &map)) return s;
    auto kern = far_exchange_kernel<C>;
    static std::atomic<uint64_t> configured{0};  // per instantiation, one bit per device
    if (int e = allow_smem(kern, C::SMEM, configured, "cudaFuncSetAttribute(far_exchange)")) return e;
    static int resident = 0;  // CTAs of this instantiation the device holds at once (per process, one device type)
    if (!resident) {
      int per_sm = 0;
      if (int e = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, C::NTHREADS, C::SMEM),
                             "far read + exchange: occupancy"))
        return e;
      resident = per_sm * device_sm_count();
    }
    if (static_cast<int64_t>(prm.splits) * prm.hkv > resident)
      return fail(FOLD_ERR_INVALID_ARGUMENT, "far read + exchange: splits * hkv CTAs do not fit the device at once");
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(prm.splits, prm.hkv), cfg.blockDim = dim3(C::NTHREADS), cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr, cfg.numAttrs = 1;
    if (int e = check_cuda(cudaLaunchKernelEx(&cfg, kern, map, prm, tail), "far read + exchange: launch")) return e;
    return check_launch("far_exchange_kernel");
  }
};

}  // namespace fold

extern "C" {

int fold_far_read_exchange(void* exchange, const void* q, int64_t q_stride_tok, int64_t q_stride_head, const int* qsl,
                           const int* seq_lens, const float* rope_table, int table_rows, int rot_dim, const void* side,
                           int pages, int64_t pos_lo, int64_t capacity, int* far_len, float* o_part, float* lse_part,
                           int splits, const void* o_l, int64_t ol_stride_tok, int64_t ol_stride_head,
                           const float* lse_l, int64_t ll_stride_head, int64_t ll_stride_tok, void* out,
                           int64_t out_stride_tok, int64_t out_stride_head, int n, int hq, int hkv, int hd, int window,
                           int block, int far_distance, float softmax_scale, float inv_alpha, int* err, void* stream) {
  using namespace fold;
  if (!exchange || !o_l || !lse_l || !out) return fail(FOLD_ERR_INVALID_ARGUMENT, "far read + exchange: null pointer");
  FarParams prm;
  if (int s = make_far_params(q, q_stride_tok, q_stride_head, qsl, seq_lens, rope_table, table_rows, rot_dim, side,
                              pages, pos_lo, capacity, far_len, nullptr, 0, 0, o_part, lse_part, splits, n, hq, hkv,
                              hd, window, block, far_distance, softmax_scale, err, &prm))
    return s;
  const int rows = n * (hq / hkv);
  if (far_read_variant(hd, rows) == 1) {  // the tcgen05 far read has no exchange tail: two launches
    if (int s = far_read_tc_launch(prm, side, pages, hd, ((rows + 15) / 16) * 16, true,
                                   static_cast<cudaStream_t>(stream)))
      return s;
    return fold_exchange_merge(exchange, o_part, lse_part, splits, o_l, ol_stride_tok, ol_stride_head, lse_l,
                               ll_stride_head, ll_stride_tok, out, out_stride_tok, out_stride_head, qsl, seq_lens, n,
                               hq, hd, window, block, inv_alpha, err, stream);
  }
  if (hkv > kMaxKvHeads) return fail(FOLD_ERR_UNSUPPORTED, "far read + exchange: at most 256 KV heads");
  if (ol_stride_tok % 2 || ol_stride_head % 2 || out_stride_tok % 2 || out_stride_head % 2 ||
      (reinterpret_cast<uintptr_t>(o_l) & 3) || (reinterpret_cast<uintptr_t>(out) & 3) || !aligned16(o_part))
    return fail(FOLD_ERR_ALIGNMENT, "far read + exchange: rows must start on element pairs, o_part 16-byte aligned");
  TailParams tail{};
  if (int s = exchange_view(exchange, n, hq, hd, &tail.ex)) return s;
  MergeParams& m = tail.m;
  m.o_l = static_cast<const __nv_bfloat16*>(o_l), m.ol_st = ol_stride_tok, m.ol_sh = ol_stride_head;
  m.lse_l = lse_l, m.ll_sh = ll_stride_head, m.ll_st = ll_stride_tok;
  m.o_f = o_part, m.of_bf16 = 0;
  m.of_ss = static_cast<int64_t>(n) * hq * hd, m.of_st = static_cast<int64_t>(hq) * hd, m.of_sh = hd;
  m.lse_f = lse_part, m.lf_ss = static_cast<int64_t>(hq) * n, m.lf_sh = n, m.lf_st = 1;
  m.splits = splits;
  m.out = static_cast<__nv_bfloat16*>(out), m.out_st = out_stride_tok, m.out_sh = out_stride_head;
  m.qsl = qsl, m.seq = seq_lens, m.n = n, m.hq = hq, m.window = window, m.block = block, m.inv_alpha = inv_alpha;
  tail.slices = hd > kSlice ? hd / kSlice : 1;
  tail.hd = hd;
  return with_mma_config(hd, rows, FarExchangeLaunch{prm, tail, side, pages, static_cast<cudaStream_t>(stream)});
}

}  // extern "C"
