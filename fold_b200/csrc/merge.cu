// LSE merge of the local window and the far memory (fold/kernels.py:86-108 of the reference),
// fused with the log-sum-exp combine of the far read's split partials.
//
// One warp per (row, query head): lanes hold hd/32 consecutive output elements; the split LSEs
// are reduced with warp shuffles, then every lane accumulates its slice of the partials.
#include <cuda_bf16.h>

#include "common.cuh"
#include "host_common.h"

namespace fold {

struct MergeParams {
  const __nv_bfloat16* o_l;
  int64_t ol_st, ol_sh;
  const float* lse_l;
  int64_t ll_sh, ll_st;
  const void* o_f;
  int of_bf16;
  int64_t of_ss, of_st, of_sh;
  const float* lse_f;
  int64_t lf_ss, lf_sh, lf_st;
  int splits;
  __nv_bfloat16* out;
  int64_t out_st, out_sh;
  float* o_out;  // combine mode: float32 [n, hq, hd]
  float* lse_out;  // combine mode: float32 [hq, n]
  const int* qsl;
  const int* seq;
  int n, hq, window, block;
  float inv_alpha;
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int EPL>
__device__ __forceinline__ void load_row(const void* base, int bf16, int64_t off, float (&v)[EPL]) {
  if (bf16) {
    const __nv_bfloat16* b = static_cast<const __nv_bfloat16*>(base) + off;
#pragma unroll
    for (int i = 0; i < EPL; i += 2) {
      const __nv_bfloat162 x = *reinterpret_cast<const __nv_bfloat162*>(b + i);
      v[i] = __low2float(x), v[i + 1] = __high2float(x);
    }
  } else {
    const float* f = static_cast<const float*>(base) + off;
#pragma unroll
    for (int i = 0; i < EPL; i += 2) {
      const float2 x = *reinterpret_cast<const float2*>(f + i);
      v[i] = x.x, v[i + 1] = x.y;
    }
  }
}

constexpr int kMergeWarps = 4;  // warps of one block; they split the far partials between them
constexpr int kSlice = 128;     // head dims per block: 32 lanes x 4 consecutive values

// One block per (row t, query head h, 128-wide slice of the head dims). Lane l holds columns
// [4l, 4l+4) of the slice. The far partials are log-sum-exp combined: every warp takes a quarter
// of the splits, loads its partial rows in batches of independent loads (they sit in L2 after
// the far read) and the four weighted sums meet in shared memory. FINAL merges the result with
// the window read (fold/kernels.py:94-107) into the bf16 output; otherwise the combined partial
// itself is written (float32 o and lse).
template <bool FINAL>
__global__ void __launch_bounds__(kMergeWarps * 32) merge_kernel(const MergeParams p, int slices, int hd) {
  __shared__ float s_acc[kMergeWarps][kSlice];
  __shared__ float s_w[kMergeWarps];
  constexpr int BATCH = 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slice = blockIdx.x % slices, th = blockIdx.x / slices;
  const int t = th / p.hq, h = th - (th / p.hq) * p.hq;
  const int width = min(hd, kSlice);
  const bool active = lane * 4 < width;
  const int col = slice * kSlice + lane * 4;

  bool has_far = true;
  if constexpr (FINAL) {
    const int qlen = p.qsl[1] - p.qsl[0];
    const int hist = max(p.seq[0] - qlen, 0);
    has_far = hist - p.window - p.block + 1 + t > 0;  // fold/kernels.py:94-95
  }
  const float* lf = p.lse_f + static_cast<int64_t>(h) * p.lf_sh + static_cast<int64_t>(t) * p.lf_st;
  float mx = -INFINITY;
  if (has_far) {
    for (int s = lane; s < p.splits; s += 32) mx = fmaxf(mx, lf[s * p.lf_ss]);
    mx = warp_max(mx);
  }
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float wsum = 0.f;
  if (mx != -INFINITY) {
    const int per = (p.splits + kMergeWarps - 1) / kMergeWarps;
    const int s0 = warp * per, s1 = min(p.splits, s0 + per);
    const int64_t base = static_cast<int64_t>(t) * p.of_st + static_cast<int64_t>(h) * p.of_sh + col;
    for (int sb = s0; sb < s1; sb += 32) {
      const int cnt = min(32, s1 - sb);
      const float l = lane < cnt ? lf[(sb + lane) * p.lf_ss] : -INFINITY;
      const float w = l == -INFINITY ? 0.f : expf(l - mx);  // an empty split carries no mass
      wsum += w;
      for (int j = 0; j < cnt; j += BATCH) {
        float v[BATCH][4];
#pragma unroll
        for (int u = 0; u < BATCH; ++u) {
          if (active && j + u < cnt) {
            load_row<4>(p.o_f, p.of_bf16, base + (sb + j + u) * p.of_ss, v[u]);
          } else {
            v[u][0] = v[u][1] = v[u][2] = v[u][3] = 0.f;
          }
        }
#pragma unroll
        for (int u = 0; u < BATCH; ++u) {
          const float wu = __shfl_sync(0xffffffffu, w, (j + u) & 31);
          if (j + u < cnt) {
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] = fmaf(wu, v[u][i], acc[i]);
          }
        }
      }
    }
    wsum = warp_sum(wsum);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) s_acc[warp][lane * 4 + i] = acc[i];
  if (lane == 0) s_w[warp] = wsum;
  __syncthreads();
  if (warp != 0) return;
  float W = 0.f, of[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int w = 0; w < kMergeWarps; ++w) {
    W += s_w[w];
#pragma unroll
    for (int i = 0; i < 4; ++i) of[i] += s_acc[w][lane * 4 + i];
  }
  const bool any = mx != -INFINITY && W > 0.f;
  const float inv = any ? 1.f / W : 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) of[i] *= inv;
  const float lse_far = any ? mx + logf(W) : -INFINITY;
  if constexpr (FINAL) {
    if (!active) return;
    float ol[4];
    load_row<4>(p.o_l, 1, static_cast<int64_t>(t) * p.ol_st + static_cast<int64_t>(h) * p.ol_sh + col, ol);
    float y[4] = {ol[0], ol[1], ol[2], ol[3]};
    if (any) {
      const float ll = p.lse_l[static_cast<int64_t>(h) * p.ll_sh + static_cast<int64_t>(t) * p.ll_st];
      const float lfa = lse_far * p.inv_alpha;  // memory log-mass (Eq. 3)
      const float m = fmaxf(ll, lfa);
      const float wl = expf(ll - m), wf = expf(lfa - m);
      const float r = 1.f / (wl + wf);
#pragma unroll
      for (int i = 0; i < 4; ++i) y[i] = (wl * ol[i] + wf * of[i]) * r;
    }
    __nv_bfloat16* o = p.out + static_cast<int64_t>(t) * p.out_st + static_cast<int64_t>(h) * p.out_sh + col;
    *reinterpret_cast<__nv_bfloat162*>(o) = __floats2bfloat162_rn(y[0], y[1]);
    *reinterpret_cast<__nv_bfloat162*>(o + 2) = __floats2bfloat162_rn(y[2], y[3]);
  } else {
    if (active) {
      float* o = p.o_out + (static_cast<int64_t>(t) * p.hq + h) * hd + col;
      *reinterpret_cast<float4*>(o) = make_float4(of[0], of[1], of[2], of[3]);
    }
    if (lane == 0 && slice == 0) p.lse_out[static_cast<int64_t>(h) * p.n + t] = lse_far;
  }
}

static int merge_launch(const MergeParams& p, int hd, bool combine, cudaStream_t stream) {
  if (hd < 8 || (hd > kSlice && hd % kSlice) || (hd <= kSlice && hd % 4))
    return fail(FOLD_ERR_UNSUPPORTED, "merge: head size must be a multiple of 128, or of 4 up to 128");
  const int slices = hd > kSlice ? hd / kSlice : 1;
  const int64_t blocks = static_cast<int64_t>(p.n) * p.hq * slices;
  if (blocks > 2147483647) return fail(FOLD_ERR_INVALID_ARGUMENT, "merge: too many rows");
  if (combine)
    merge_kernel<false><<<static_cast<unsigned>(blocks), kMergeWarps * 32, 0, stream>>>(p, slices, hd);
  else
    merge_kernel<true><<<static_cast<unsigned>(blocks), kMergeWarps * 32, 0, stream>>>(p, slices, hd);
  return check_launch(combine ? "combine_kernel" : "merge_kernel");
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
