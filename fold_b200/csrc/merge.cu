// LSE merge of the local window and the far memory (fold/kernels.py:86-108 of the reference),
// fused with the log-sum-exp combine of the far read's split partials.
#include <cuda_bf16.h>

#include "common.cuh"
#include "host_common.h"
#include "merge.cuh"

namespace fold {

// One block per (row t, query head h, 128-wide slice of the head dims). Lane l holds columns
// [4l, 4l+4) of the slice. The far partials are log-sum-exp combined by the whole block
// (combine_slice). FINAL merges the result with the window read (fold/kernels.py:94-107) into the
// bf16 output; otherwise the combined partial itself is written (float32 o and lse).
template <bool FINAL>
__global__ void __launch_bounds__(kMergeWarps * 32) merge_kernel(const MergeParams p, int slices, int hd) {
  __shared__ SliceSums sums;
  wait_for_producer();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slice = blockIdx.x % slices, th = blockIdx.x / slices;
  const int t = th / p.hq, h = th - (th / p.hq) * p.hq;
  const bool active = lane * 4 < min(hd, kSlice);
  const int col = slice * kSlice + lane * 4;
  const bool has_far = FINAL ? row_has_far(p, t) : true;
  float of[4], lse_far;
  combine_slice(p, t, h, col, active, has_far, sums, of, lse_far, p.splits);
  if (warp != 0) return;
  if constexpr (FINAL) {
    if (active) merge_store(p, t, h, col, of, lse_far);
  } else {
    if (active) {
      float* o = p.o_out + (static_cast<int64_t>(t) * p.hq + h) * hd + col;
      *reinterpret_cast<float4*>(o) = make_float4(of[0], of[1], of[2], of[3]);
    }
    if (lane == 0 && slice == 0) p.lse_out[static_cast<int64_t>(h) * p.n + t] = lse_far;
  }
}

// Both sides as split partials: the window read's splits (pw) are combined by log-sum-exp, then
// the far read's (pf, which also carries the output and the step geometry), and the two are merged
// with the alpha weighting. Without far splits the output is the combined window read. With
// `plan` (the step read's device word), the window set uses its first plan[0] slots and the far
// set all of its slots (a block that drew no far tile left an empty partial).
__global__ void __launch_bounds__(kMergeWarps * 32)
    merge_partials_kernel(const MergeParams pw, const MergeParams pf, const int* plan, int slices, int hd) {
  __shared__ SliceSums sums;
  wait_for_producer();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slice = blockIdx.x % slices, th = blockIdx.x / slices;
  const int t = th / pf.hq, h = th - (th / pf.hq) * pf.hq;
  const bool active = lane * 4 < min(hd, kSlice);
  const int col = slice * kSlice + lane * 4;
  const int wsplits = plan ? min(max(*plan, 0), pw.splits) : pw.splits;
  const int fsplits = pf.splits;
  float ol[4], ll;
  combine_slice(pw, t, h, col, active, true, sums, ol, ll, wsplits);
  float of[4] = {0.f, 0.f, 0.f, 0.f}, lf = -INFINITY;
  if (pf.splits > 0) {
    __syncthreads();  // warp 0 has read the window sums
    combine_slice(pf, t, h, col, active, row_has_far(pf, t), sums, of, lf, fsplits);
  }
  if (warp != 0 || !active) return;
  merge_store_loaded(pf, t, h, col, of, lf, ol, ll);
}

static int merge_launch(const MergeParams& p, int hd, bool combine, cudaStream_t stream) {
  if (hd < 8 || (hd > kSlice && hd % kSlice) || (hd <= kSlice && hd % 4))
    return fail(FOLD_ERR_UNSUPPORTED, "merge: head size must be a multiple of 128, or of 4 up to 128");
  const int slices = hd > kSlice ? hd / kSlice : 1;
  const int64_t blocks = static_cast<int64_t>(p.n) * p.hq * slices;
  if (blocks > 2147483647) return fail(FOLD_ERR_INVALID_ARGUMENT, "merge: too many rows");
  const dim3 grid(static_cast<unsigned>(blocks));
  if (combine)
    return launch_behind(merge_kernel<false>, grid, kMergeWarps * 32, 0, stream, "combine_kernel", p, slices, hd);
  return launch_behind(merge_kernel<true>, grid, kMergeWarps * 32, 0, stream, "merge_kernel", p, slices, hd);
}

int merge_contiguous_partials(const void* o_l, int64_t ol_stride_tok, int64_t ol_stride_head, const float* lse_l,
                              int64_t ll_stride_head, int64_t ll_stride_tok, const float* o_part,
                              const float* lse_part, int splits, void* out, int64_t out_stride_tok,
                              int64_t out_stride_head, const int* qsl, const int* seq_lens, int n, int hq, int hd,
                              int window, int block, float inv_alpha, cudaStream_t stream) {
  if (!o_l || !lse_l || !o_part || !lse_part || !out || !qsl || !seq_lens)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "merge: null pointer");
  if (n < 1 || hq < 1 || splits < 1) return fail(FOLD_ERR_INVALID_ARGUMENT, "merge: bad sizes");
  if (ol_stride_tok % 2 || ol_stride_head % 2 || out_stride_tok % 2 || out_stride_head % 2 ||
      (reinterpret_cast<uintptr_t>(o_l) & 3) || (reinterpret_cast<uintptr_t>(out) & 3) ||
      (reinterpret_cast<uintptr_t>(o_part) & 7))
    return fail(FOLD_ERR_ALIGNMENT, "merge: rows must start on element pairs");
  MergeParams p{};
  p.o_l = static_cast<const __nv_bfloat16*>(o_l), p.ol_st = ol_stride_tok, p.ol_sh = ol_stride_head;
  p.lse_l = lse_l, p.ll_sh = ll_stride_head, p.ll_st = ll_stride_tok;
  p.o_f = o_part, p.of_bf16 = 0;
  p.of_ss = static_cast<int64_t>(n) * hq * hd, p.of_st = static_cast<int64_t>(hq) * hd, p.of_sh = hd;
  p.lse_f = lse_part, p.lf_ss = static_cast<int64_t>(hq) * n, p.lf_sh = n, p.lf_st = 1;
  p.splits = splits;
  p.out = static_cast<__nv_bfloat16*>(out), p.out_st = out_stride_tok, p.out_sh = out_stride_head;
  p.qsl = qsl, p.seq = seq_lens, p.n = n, p.hq = hq, p.window = window, p.block = block, p.inv_alpha = inv_alpha;
  return merge_launch(p, hd, false, stream);
}

}  // namespace fold

extern "C" {

int fold_merge(const void* o_l, int64_t ol_stride_tok, int64_t ol_stride_head, const float* lse_l,
               int64_t ll_stride_head, int64_t ll_stride_tok, const void* o_f, int of_bf16, int64_t of_stride_split,
               int64_t of_stride_tok, int64_t of_stride_head, const float* lse_f, int64_t lf_stride_split,
               int64_t lf_stride_head, int64_t lf_stride_tok, int splits, void* out, int64_t out_stride_tok,
               int64_t out_stride_head, const int* qsl, const int* seq_lens, int n, int hq, int hd, int window,
               int block, float inv_alpha, void* stream) {
  using namespace fold;
  if (!o_l || !lse_l || !o_f || !lse_f || !out || !qsl || !seq_lens)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "merge: null pointer");
  if (n < 1 || hq < 1 || splits < 1) return fail(FOLD_ERR_INVALID_ARGUMENT, "merge: bad sizes");
  const int epl = hd / 32;
  const int64_t vec = epl;  // elements per lane must start on an aligned pair
  if (ol_stride_tok % 2 || ol_stride_head % 2 || out_stride_tok % 2 || out_stride_head % 2 || of_stride_split % 2 ||
      of_stride_tok % 2 || of_stride_head % 2 || (reinterpret_cast<uintptr_t>(o_l) & 3) ||
      (reinterpret_cast<uintptr_t>(out) & 3) || (reinterpret_cast<uintptr_t>(o_f) & (of_bf16 ? 3 : 7)) || vec < 2)
    return fail(FOLD_ERR_ALIGNMENT, "merge: rows must start on element pairs");
  MergeParams p{};
  p.o_l = static_cast<const __nv_bfloat16*>(o_l), p.ol_st = ol_stride_tok, p.ol_sh = ol_stride_head;
  p.lse_l = lse_l, p.ll_sh = ll_stride_head, p.ll_st = ll_stride_tok;
  p.o_f = o_f, p.of_bf16 = of_bf16, p.of_ss = of_stride_split, p.of_st = of_stride_tok, p.of_sh = of_stride_head;
  p.lse_f = lse_f, p.lf_ss = lf_stride_split, p.lf_sh = lf_stride_head, p.lf_st = lf_stride_tok;
  p.splits = splits;
  p.out = static_cast<__nv_bfloat16*>(out), p.out_st = out_stride_tok, p.out_sh = out_stride_head;
  p.qsl = qsl, p.seq = seq_lens, p.n = n, p.hq = hq, p.window = window, p.block = block, p.inv_alpha = inv_alpha;
  return merge_launch(p, hd, false, static_cast<cudaStream_t>(stream));
}

int fold_merge_partials(const float* o_wpart, const float* lse_wpart, int wsplits, const float* o_fpart,
                        const float* lse_fpart, int fsplits, const int* plan, void* out, int64_t out_stride_tok,
                        int64_t out_stride_head, const int* qsl, const int* seq_lens, int n, int hq, int hd,
                        int window, int block, float inv_alpha, void* stream) {
  using namespace fold;
  if (!o_wpart || !lse_wpart || !out || !qsl || !seq_lens || (fsplits > 0 && (!o_fpart || !lse_fpart)))
    return fail(FOLD_ERR_INVALID_ARGUMENT, "merge partials: null pointer");
  if (n < 1 || hq < 1 || wsplits < 1 || fsplits < 0) return fail(FOLD_ERR_INVALID_ARGUMENT, "merge partials: bad sizes");
  if (plan && fsplits != wsplits)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "merge partials: with a step plan both sets have the same slot count");
  if (hd < 8 || (hd > kSlice && hd % kSlice) || (hd <= kSlice && hd % 4))
    return fail(FOLD_ERR_UNSUPPORTED, "merge partials: head size must be a multiple of 128, or of 4 up to 128");
  if (out_stride_tok % 2 || out_stride_head % 2 || (reinterpret_cast<uintptr_t>(out) & 3) ||
      (reinterpret_cast<uintptr_t>(o_wpart) & 7) || (reinterpret_cast<uintptr_t>(o_fpart) & 7))
    return fail(FOLD_ERR_ALIGNMENT, "merge partials: rows must start on element pairs");
  MergeParams pw{}, pf{};
  for (MergeParams* p : {&pw, &pf}) {
    p->of_bf16 = 0;
    p->of_ss = static_cast<int64_t>(n) * hq * hd, p->of_st = static_cast<int64_t>(hq) * hd, p->of_sh = hd;
    p->lf_ss = static_cast<int64_t>(hq) * n, p->lf_sh = n, p->lf_st = 1;
    p->qsl = qsl, p->seq = seq_lens, p->n = n, p->hq = hq;
  }
  pw.o_f = o_wpart, pw.lse_f = lse_wpart, pw.splits = wsplits;
  pf.o_f = o_fpart, pf.lse_f = lse_fpart, pf.splits = fsplits;
  pf.out = static_cast<__nv_bfloat16*>(out), pf.out_st = out_stride_tok, pf.out_sh = out_stride_head;
  pf.window = window, pf.block = block, pf.inv_alpha = inv_alpha;
  const int slices = hd > kSlice ? hd / kSlice : 1;
  const int64_t blocks = static_cast<int64_t>(n) * hq * slices;
  if (blocks > 2147483647) return fail(FOLD_ERR_INVALID_ARGUMENT, "merge partials: too many rows");
  return launch_behind(merge_partials_kernel, dim3(static_cast<unsigned>(blocks)), kMergeWarps * 32, 0,
                       static_cast<cudaStream_t>(stream), "merge_partials_kernel", pw, pf, plan, slices, hd);
}

int fold_combine(const float* o_part, const float* lse_part, int splits, float* o_out, float* lse_out, int n, int hq,
                 int hd, void* stream) {
  using namespace fold;
  if (!o_part || !lse_part || !o_out || !lse_out) return fail(FOLD_ERR_INVALID_ARGUMENT, "combine: null pointer");
  if (n < 1 || hq < 1 || splits < 1) return fail(FOLD_ERR_INVALID_ARGUMENT, "combine: bad sizes");
  if ((reinterpret_cast<uintptr_t>(o_part) & 7) || (reinterpret_cast<uintptr_t>(o_out) & 15) || hd % 4)
    return fail(FOLD_ERR_ALIGNMENT, "combine: o_part 8-byte and o_out 16-byte aligned, head size a multiple of 4");
  MergeParams p{};
  p.o_f = o_part, p.of_bf16 = 0;
  p.of_ss = static_cast<int64_t>(n) * hq * hd, p.of_st = static_cast<int64_t>(hq) * hd, p.of_sh = hd;
  p.lse_f = lse_part, p.lf_ss = static_cast<int64_t>(hq) * n, p.lf_sh = n, p.lf_st = 1;
  p.splits = splits, p.o_out = o_out, p.lse_out = lse_out, p.n = n, p.hq = hq;
  return merge_launch(p, hd, true, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
