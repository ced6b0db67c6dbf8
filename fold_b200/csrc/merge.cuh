// Device pieces shared by the LSE merge (merge.cu) and the peer exchange (exchange.cu): the
// parameter block, warp reductions, and the block-wide log-sum-exp combine of far partials on one
// 128-column slice of one (row, query head).
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

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
  float* o_out;    // combine mode: float32 [n, hq, hd]
  float* lse_out;  // combine mode: float32 [hq, n]
  const int* qsl;
  const int* seq;
  int n, hq, window, block;
  float inv_alpha;
};

constexpr int kMergeWarps = 4;  // warps of one block; they split the far partials between them
constexpr int kSlice = 128;     // head dims per block: 32 lanes x 4 consecutive values

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

// Whether row t of the step has far memory (fold/kernels.py:94-95).
__device__ __forceinline__ bool row_has_far(const MergeParams& p, int t) {
  const int qlen = p.qsl[1] - p.qsl[0];
  const int hist = max(p.seq[0] - qlen, 0);
  return hist - p.window - p.block + 1 + t > 0;
}

struct SliceSums {
  float acc[kMergeWarps][kSlice];
  float w[kMergeWarps];
};

// Log-sum-exp combine of the first `splits` far partials of (row t, head h) on the columns
// [col, col + 4) of each lane, by all kMergeWarps warps of the block: every warp takes a share of the splits, loads
// its partial rows in batches of independent loads (they sit in L2 after the far read), and the
// weighted sums meet in shared memory. Warp 0 returns the normalised combined values `of` and the
// combined LSE (-inf when no split holds a key); the other warps' outputs are meaningless. Ends
// with the block barrier after which warp 0 has read the shared sums: the caller needs another
// barrier before `sums` is written again.
__device__ __forceinline__ void combine_slice(const MergeParams& p, int t, int h, int col, bool active,
                                              bool has_far, SliceSums& sums, float (&of)[4], float& lse_far,
                                              int splits) {
  constexpr int BATCH = 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* lf = p.lse_f + static_cast<int64_t>(h) * p.lf_sh + static_cast<int64_t>(t) * p.lf_st;
  float mx = -INFINITY;
  if (has_far) {
    for (int s = lane; s < splits; s += 32) mx = fmaxf(mx, lf[s * p.lf_ss]);
    mx = warp_max(mx);
  }
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float wsum = 0.f;
  if (mx != -INFINITY) {
    const int per = (splits + kMergeWarps - 1) / kMergeWarps;
    const int s0 = warp * per, s1 = min(splits, s0 + per);
    const int64_t base = static_cast<int64_t>(t) * p.of_st + static_cast<int64_t>(h) * p.of_sh + col;
    for (int sb = s0; sb < s1; sb += 32) {
      const int cnt = min(32, s1 - sb);
      const float l = lane < cnt ? lf[(sb + lane) * p.lf_ss] : -INFINITY;
      const float w = l == -INFINITY ? 0.f : expf(l - mx);  // an empty split carries no mass
      wsum += w;
      for (int j = 0; j < cnt; j += BATCH) {
        float v[BATCH][4], wu[BATCH];
#pragma unroll
        for (int u = 0; u < BATCH; ++u) {
          wu[u] = __shfl_sync(0xffffffffu, w, (j + u) & 31);
          if (active && j + u < cnt && wu[u] > 0.f) {  // an empty split's o is not read
            load_row<4>(p.o_f, p.of_bf16, base + (sb + j + u) * p.of_ss, v[u]);
          } else {
            v[u][0] = v[u][1] = v[u][2] = v[u][3] = 0.f;
          }
        }
#pragma unroll
        for (int u = 0; u < BATCH; ++u) {
          if (j + u < cnt && wu[u] > 0.f) {
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[i] = fmaf(wu[u], v[u][i], acc[i]);
          }
        }
      }
    }
    wsum = warp_sum(wsum);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) sums.acc[warp][lane * 4 + i] = acc[i];
  if (lane == 0) sums.w[warp] = wsum;
  __syncthreads();
  float W = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) of[i] = 0.f;
  if (warp == 0) {
#pragma unroll
    for (int w = 0; w < kMergeWarps; ++w) {
      W += sums.w[w];
#pragma unroll
      for (int i = 0; i < 4; ++i) of[i] += sums.acc[w][lane * 4 + i];
    }
  }
  const bool any = mx != -INFINITY && W > 0.f;
  const float inv = any ? 1.f / W : 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) of[i] *= inv;
  lse_far = any ? mx + logf(W) : -INFINITY;
}

// The alpha-weighted merge (fold/kernels.py:94-107) of the window read (ol, its LSE ll) with a
// combined far partial for the 4 columns of one lane, written as bf16.
__device__ __forceinline__ void merge_store_loaded(const MergeParams& p, int t, int h, int col, const float (&of)[4],
                                                   float lse_far, const float (&ol)[4], float ll) {
  float y[4] = {ol[0], ol[1], ol[2], ol[3]};
  if (lse_far != -INFINITY) {
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
}

// The same, loading the window read itself.
__device__ __forceinline__ void merge_store(const MergeParams& p, int t, int h, int col, const float (&of)[4],
                                            float lse_far) {
  float ol[4];
  load_row<4>(p.o_l, 1, static_cast<int64_t>(t) * p.ol_st + static_cast<int64_t>(h) * p.ol_sh + col, ol);
  const float ll = lse_far != -INFINITY ? p.lse_l[static_cast<int64_t>(h) * p.ll_sh + static_cast<int64_t>(t) * p.ll_st]
                                        : 0.f;
  merge_store_loaded(p, t, h, col, of, lse_far, ol, ll);
}

}  // namespace fold
