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

// Combines the far partials of (t, h) into acc (normalised) and returns their LSE (-inf if none).
// Lane s holds split s's weight; the partial rows are loaded in batches of independent loads (the
// partials sit in L2 right after the far read, so latency, not bandwidth, bounds this).
template <int EPL>
__device__ __forceinline__ float combine_far(const MergeParams& p, int t, int h, int lane, float (&acc)[EPL]) {
  constexpr int BATCH = EPL <= 4 ? 16 : 8;
  const float* lf = p.lse_f + static_cast<int64_t>(h) * p.lf_sh + static_cast<int64_t>(t) * p.lf_st;
  float mx = -INFINITY;
  for (int s = lane; s < p.splits; s += 32) mx = fmaxf(mx, lf[s * p.lf_ss]);
  mx = warp_max(mx);
#pragma unroll
  for (int i = 0; i < EPL; ++i) acc[i] = 0.f;
  if (mx == -INFINITY) return -INFINITY;
  float wsum = 0.f;
  const int64_t base = static_cast<int64_t>(t) * p.of_st + static_cast<int64_t>(h) * p.of_sh + lane * EPL;
  for (int s0 = 0; s0 < p.splits; s0 += 32) {
    const int cnt = min(32, p.splits - s0);
    const float l = lane < cnt ? lf[(s0 + lane) * p.lf_ss] : -INFINITY;
    const float w = l == -INFINITY ? 0.f : expf(l - mx);  // an empty split carries no mass
    wsum += w;
    for (int j = 0; j < cnt; j += BATCH) {
      float v[BATCH][EPL];
#pragma unroll
      for (int u = 0; u < BATCH; ++u) {
        if (j + u < cnt) {
          load_row<EPL>(p.o_f, p.of_bf16, base + (s0 + j + u) * p.of_ss, v[u]);
        } else {
#pragma unroll
          for (int i = 0; i < EPL; ++i) v[u][i] = 0.f;
        }
      }
#pragma unroll
      for (int u = 0; u < BATCH; ++u) {
        const float wu = __shfl_sync(0xffffffffu, w, (j + u) & 31);
        if (j + u < cnt) {
#pragma unroll
          for (int i = 0; i < EPL; ++i) acc[i] = fmaf(wu, v[u][i], acc[i]);
        }
      }
    }
  }
  wsum = warp_sum(wsum);
  const float inv = 1.f / wsum;
#pragma unroll
  for (int i = 0; i < EPL; ++i) acc[i] *= inv;
  return mx + logf(wsum);
}

template <int EPL>
__global__ void merge_kernel(const MergeParams p) {
  const int lane = threadIdx.x & 31;
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= p.n * p.hq) return;
  const int t = w / p.hq, h = w - (w / p.hq) * p.hq;
  const int qlen = p.qsl[1] - p.qsl[0];
  const int hist = max(p.seq[0] - qlen, 0);
  const bool has_far = hist - p.window - p.block + 1 + t > 0;  // fold/kernels.py:94-95
  float ol[EPL];
  load_row<EPL>(p.o_l, 1, static_cast<int64_t>(t) * p.ol_st + static_cast<int64_t>(h) * p.ol_sh + lane * EPL, ol);
  float y[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) y[i] = ol[i];
  if (has_far) {
    float of[EPL];
    const float lse_far = combine_far<EPL>(p, t, h, lane, of);
    if (lse_far != -INFINITY) {
      const float ll = p.lse_l[static_cast<int64_t>(h) * p.ll_sh + static_cast<int64_t>(t) * p.ll_st];
      const float lf = lse_far * p.inv_alpha;  // memory log-mass (Eq. 3)
      const float m = fmaxf(ll, lf);
      const float wl = expf(ll - m), wf = expf(lf - m);
      const float inv = 1.f / (wl + wf);
#pragma unroll
      for (int i = 0; i < EPL; ++i) y[i] = (wl * ol[i] + wf * of[i]) * inv;
    }
  }
  __nv_bfloat16* o = p.out + static_cast<int64_t>(t) * p.out_st + static_cast<int64_t>(h) * p.out_sh + lane * EPL;
#pragma unroll
  for (int i = 0; i < EPL; i += 2) *reinterpret_cast<__nv_bfloat162*>(o + i) = __floats2bfloat162_rn(y[i], y[i + 1]);
}

template <int EPL>
__global__ void combine_kernel(const MergeParams p) {
  const int lane = threadIdx.x & 31;
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= p.n * p.hq) return;
  const int t = w / p.hq, h = w - (w / p.hq) * p.hq;
  float acc[EPL];
  const float lse = combine_far<EPL>(p, t, h, lane, acc);
  float* o = p.o_out + (static_cast<int64_t>(t) * p.hq + h) * (EPL * 32) + lane * EPL;
#pragma unroll
  for (int i = 0; i < EPL; i += 2) *reinterpret_cast<float2*>(o + i) = make_float2(acc[i], acc[i + 1]);
  if (lane == 0) p.lse_out[static_cast<int64_t>(h) * p.n + t] = lse;
}

static int merge_launch(const MergeParams& p, int hd, bool combine, cudaStream_t stream) {
  const int warps = p.n * p.hq;
  const int threads = 128;
  const int blocks = (warps + 3) / 4;
  switch (hd) {
    case 64:
      combine ? combine_kernel<2><<<blocks, threads, 0, stream>>>(p) : merge_kernel<2><<<blocks, threads, 0, stream>>>(p);
      break;
    case 128:
      combine ? combine_kernel<4><<<blocks, threads, 0, stream>>>(p) : merge_kernel<4><<<blocks, threads, 0, stream>>>(p);
      break;
    case 256:
      combine ? combine_kernel<8><<<blocks, threads, 0, stream>>>(p) : merge_kernel<8><<<blocks, threads, 0, stream>>>(p);
      break;
    case 512:
      combine ? combine_kernel<16><<<blocks, threads, 0, stream>>>(p)
              : merge_kernel<16><<<blocks, threads, 0, stream>>>(p);
      break;
    default:
      return fail(FOLD_ERR_UNSUPPORTED, "merge: head size must be 64, 128, 256 or 512");
  }
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
  if ((reinterpret_cast<uintptr_t>(o_part) & 7) || (reinterpret_cast<uintptr_t>(o_out) & 7))
    return fail(FOLD_ERR_ALIGNMENT, "combine: buffers must be 8-byte aligned");
  MergeParams p{};
  p.o_f = o_part, p.of_bf16 = 0;
  p.of_ss = static_cast<int64_t>(n) * hq * hd, p.of_st = static_cast<int64_t>(hq) * hd, p.of_sh = hd;
  p.lse_f = lse_part, p.lf_ss = static_cast<int64_t>(hq) * n, p.lf_sh = n, p.lf_st = 1;
  p.splits = splits, p.o_out = o_out, p.lse_out = lse_out, p.n = n, p.hq = hq;
  return merge_launch(p, hd, true, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
