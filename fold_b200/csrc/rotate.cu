// Far-query rotation and the ReRoPE query pair (fold/kernels.py:21-83 of the reference), and the
// ReRoPE query scale alone (fold/attention.py:76-83, logn_scale_rows): fold_rerope_query without
// a far query and table writes only the scaled query.
//
// One CTA per (row, head); thread d computes output element d from q[d] and its neox partner.
// cos/sin come from a float32 table formed in float64 (rows = |offset|, vLLM cos_sin_cache
// layout), which keeps the rotation accurate at offsets near 1e5 where a float32 angle is not.
#include <cuda_bf16.h>

#include "common.cuh"
#include "host_common.h"

namespace fold {

struct RotParams {
  const __nv_bfloat16* q;
  int64_t q_st, q_sh;
  __nv_bfloat16* qs;  // ReRoPE scaled query (may be null)
  int64_t qs_st, qs_sh;
  __nv_bfloat16* qf;
  int64_t qf_st, qf_sh;
  const int* qsl;
  const int* seq;
  const float* table;
  int table_rows, rot_dim;
  int* far_len;
  int hq, hd, window, block, far_distance, constant;
  float inv_log_ref;
  int* err;
};

__global__ void rotate_kernel(const RotParams p) {
  const int t = blockIdx.x / p.hq, h = blockIdx.x - (blockIdx.x / p.hq) * p.hq;
  const int qlen = p.qsl[1] - p.qsl[0];
  const int hist = max(p.seq[0] - qlen, 0);
  if (blockIdx.x == 0 && threadIdx.x == 0 && p.far_len) *p.far_len = max(hist - p.window - p.block + qlen, 0);
  int off = p.far_distance - hist - (p.constant ? t : 0);
  const float sgn = off < 0 ? -1.f : 1.f;
  int ad = off < 0 ? -off : off;
  if (p.qf && ad >= p.table_rows) {
    if (threadIdx.x == 0) set_error(p.err, FOLD_DEVERR_ROPE_RANGE);
    ad = p.table_rows - 1;
  }
  float sc = 1.f;
  if (p.inv_log_ref > 0.f) sc = fmaxf(logf(static_cast<float>(hist + t + 1)) * p.inv_log_ref, 1.f);
  const int RH = p.rot_dim >> 1;
  const __nv_bfloat16* qr = p.q + t * p.q_st + h * p.q_sh;
  const float* trow = p.qf ? p.table + static_cast<int64_t>(ad) * p.rot_dim : nullptr;
  for (int d = threadIdx.x; d < p.hd; d += blockDim.x) {
    const float x = __bfloat162float(qr[d]) * sc;
    if (p.qs) p.qs[t * p.qs_st + h * p.qs_sh + d] = __float2bfloat16_rn(x);
    if (!p.qf) continue;  // the query scale alone
    float y = x;
    if (d < 2 * RH) {
      const bool lo = d < RH;
      const int i = lo ? d : d - RH;
      const float xp = __bfloat162float(qr[lo ? d + RH : d - RH]) * sc;
      const float c = trow[i], s = sgn * trow[RH + i];
      y = lo ? x * c - xp * s : x * c + xp * s;
    }
    p.qf[t * p.qf_st + h * p.qf_sh + d] = __float2bfloat16_rn(y);
  }
}

static int launch_rotate(const RotParams& p, int n, cudaStream_t stream) {
  const int threads = p.hd >= 128 ? 128 : 64;
  rotate_kernel<<<n * p.hq, threads, 0, stream>>>(p);
  return check_launch("rotate_kernel");
}

static int check_rot_args(const void* q, const void* qf, const int* qsl, const int* seq, const float* table,
                          int table_rows, int rot_dim, int n, int hq, int hd) {
  if (!q || !qf || !qsl || !seq || !table) return fail(FOLD_ERR_INVALID_ARGUMENT, "query rotation: null pointer");
  if (n < 1 || hq < 1 || hd < 2 || rot_dim < 2 || rot_dim % 2 || rot_dim > hd || table_rows < 1)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "query rotation: bad sizes");
  if (static_cast<int64_t>(n) * hq > 2147483647) return fail(FOLD_ERR_INVALID_ARGUMENT, "query rotation: too many rows");
  return FOLD_OK;
}

}  // namespace fold

extern "C" {

int fold_far_query(const void* q, int64_t q_stride_tok, int64_t q_stride_head, void* qf, int64_t qf_stride_tok,
                   int64_t qf_stride_head, const int* qsl, const int* seq_lens, const float* rope_table,
                   int table_rows, int rot_dim, int* far_len, int n, int hq, int hd, int window, int block,
                   int far_distance, int* err, void* stream) {
  using namespace fold;
  if (int s = check_rot_args(q, qf, qsl, seq_lens, rope_table, table_rows, rot_dim, n, hq, hd)) return s;
  RotParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q), p.q_st = q_stride_tok, p.q_sh = q_stride_head;
  p.qf = static_cast<__nv_bfloat16*>(qf), p.qf_st = qf_stride_tok, p.qf_sh = qf_stride_head;
  p.qsl = qsl, p.seq = seq_lens, p.table = rope_table, p.table_rows = table_rows, p.rot_dim = rot_dim;
  p.far_len = far_len, p.hq = hq, p.hd = hd, p.window = window, p.block = block, p.far_distance = far_distance;
  p.err = err;
  return launch_rotate(p, n, static_cast<cudaStream_t>(stream));
}

int fold_rerope_query(const void* q, int64_t q_stride_tok, int64_t q_stride_head, void* qs, int64_t qs_stride_tok,
                      int64_t qs_stride_head, void* qf, int64_t qf_stride_tok, int64_t qf_stride_head,
                      const int* qsl, const int* seq_lens, const float* rope_table, int table_rows, int rot_dim,
                      int* far_len, int n, int hq, int hd, int window, int block, int far_distance, int constant,
                      float inv_log_ref, int* err, void* stream) {
  using namespace fold;
  if (!qs) return fail(FOLD_ERR_INVALID_ARGUMENT, "rerope: null qs");
  if (!qf && !rope_table) {  // the query scale alone: qs only
    if (!q || !qsl || !seq_lens) return fail(FOLD_ERR_INVALID_ARGUMENT, "rerope: null pointer");
    if (n < 1 || hq < 1 || hd < 1 || static_cast<int64_t>(n) * hq > 2147483647)
      return fail(FOLD_ERR_INVALID_ARGUMENT, "rerope: bad sizes");
    rot_dim = 2, table_rows = 1;
  } else if (int s = check_rot_args(q, qf, qsl, seq_lens, rope_table, table_rows, rot_dim, n, hq, hd)) {
    return s;
  }
  RotParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q), p.q_st = q_stride_tok, p.q_sh = q_stride_head;
  p.qs = static_cast<__nv_bfloat16*>(qs), p.qs_st = qs_stride_tok, p.qs_sh = qs_stride_head;
  p.qf = static_cast<__nv_bfloat16*>(qf), p.qf_st = qf_stride_tok, p.qf_sh = qf_stride_head;
  p.qsl = qsl, p.seq = seq_lens, p.table = rope_table, p.table_rows = table_rows, p.rot_dim = rot_dim;
  p.far_len = far_len, p.hq = hq, p.hd = hd, p.window = window, p.block = block, p.far_distance = far_distance;
  p.constant = constant, p.inv_log_ref = inv_log_ref, p.err = err;
  return launch_rotate(p, n, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
