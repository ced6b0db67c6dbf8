// Parameters and helpers shared by the two far-read kernels (mma.sync in far_read.cu, tcgen05 in
// far_read_tc.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fold {

// Lazy row-maximum threshold (log2 units): the running maximum of a row only moves when a logit
// passes it by more than this, so P = 2^(logit - maximum) stays below 2^15 and fits f16 (whose
// largest finite value is 65504).
constexpr float kRaise = 15.0f;

struct FarParams {
  const __nv_bfloat16* q;
  int64_t q_st, q_sh;
  const int* qsl;
  const int* seq;
  const float* table;
  int table_rows, rot_dim;
  int64_t pos_lo, capacity, local_cap;
  int* far_len;
  __nv_bfloat16* qf;
  int64_t qf_st, qf_sh;
  float* o_part;
  float* lse_part;
  int splits, n, hq, hkv, group;
  int window, block, far_distance;
  float scale_log2;
  int* err;
  int vec_rot;  // q, qf and the table rows allow the 16-byte vector path of the rotation
  // Window read only (window_read_kernel): the paged cache's K and V planes (strides in elements),
  // its block table and the window.
  const __nv_bfloat16* kc;
  const __nv_bfloat16* vc;
  int64_t s_block, s_head, s_slot;
  const int* block_table;
  int bt_len, num_blocks, block_size;
  int win_left, win_right, causal;
  // Far read of an fp8 side cache only: per-KV-head dequantisation scales of K and V (float [hkv]).
  const float* k_scale;
  const float* v_scale;
};

constexpr int kSmemLimit = 232448;  // 227 KB of dynamic shared memory per CTA on sm_100

__device__ __forceinline__ float bf2f(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
__device__ __forceinline__ int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

// Launches the tcgen05 far read for n*G rows padded to np (16, 32, 48 or 64) with hd 128 or 256.
int far_read_tc_launch(const FarParams& prm, const void* side, int pages, int hd, int np, bool cached_map,
                       cudaStream_t stream);

// Which far-read kernel serves (hd, n*G): 0 = mma.sync, 1 = tcgen05. FOLD_FAR_READ_KERNEL=mma|tc
// in the environment forces one (read once per process).
int far_read_variant(int hd, int rows);

}  // namespace fold
