// Far read + merge for callers that cannot allocate device memory.
//
// Some callers of the draft step cannot call cudaMalloc (or any allocator) at the point where
// they run it: an inference engine that plans every device buffer ahead of time and hands the
// attention plugin only the tensors of the step, a C runtime without PyTorch's caching allocator,
// or code that must not grow the process's device footprint between steps. The regular far read
// needs float32 split partials as scratch, which the caller allocates. This entry point keeps
// that scratch in a static device array of the library instead, so the caller passes only the
// step's inputs and its output.
#include <mutex>

#include "common.cuh"
#include "host_common.h"

namespace fold {

// 16 MiB of float32 scratch per GPU: split partials o [splits, n, hq, hd] followed by their
// LSEs [splits, hq, n]. A GPU holds it from the library's first use on that device (with lazy
// module loading, the first kernel call or symbol lookup there) until the process exits.
constexpr int64_t kStaticScratchFloats = int64_t(4) << 20;

static __device__ __align__(256) float g_far_scratch[kStaticScratchFloats];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
float* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once per device). In
// host code the array's name is only a host-side stand-in, so kernels get this address instead.
int scratch_on_current_device(float** out) {
  int dev = 0;
  if (int s = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return s;
  if (dev < 0 || dev >= kMaxDevices) return fail(FOLD_ERR_UNSUPPORTED, "static far read: device ordinal >= 64");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    if (int s = check_cuda(cudaGetSymbolAddress(&p, g_far_scratch), "cudaGetSymbolAddress(far scratch)")) return s;
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return FOLD_OK;
}
}  // namespace

}  // namespace fold

extern "C" {

int fold_far_read_merge_static(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const int* qsl,
                               const int* seq_lens, const float* rope_table, int table_rows, int rot_dim,
                               const void* side, int pages, int64_t pos_lo, int64_t capacity, int* far_len,
                               const void* o_l, int64_t ol_stride_tok, int64_t ol_stride_head, const float* lse_l,
                               int64_t ll_stride_head, int64_t ll_stride_tok, void* out, int64_t out_stride_tok,
                               int64_t out_stride_head, int splits, int n, int hq, int hkv, int hd, int window,
                               int block, int far_distance, float softmax_scale, float inv_alpha, int* err,
                               void* stream) {
  using namespace fold;
  if (splits < 1 || n < 1 || hq < 1 || hd < 1) return fail(FOLD_ERR_INVALID_ARGUMENT, "static far read: bad sizes");
  const int64_t o_floats = static_cast<int64_t>(splits) * n * hq * hd;
  const int64_t need = o_floats + static_cast<int64_t>(splits) * hq * n;
  if (need > kStaticScratchFloats)
    return fail(FOLD_ERR_INVALID_ARGUMENT,
                "static far read: splits * n * hq * (hd + 1) = " + std::to_string(need) +
                    " floats exceeds the static scratch of " + std::to_string(kStaticScratchFloats) +
                    " floats (16 MiB); use fewer splits");
  float* scratch = nullptr;
  if (int s = scratch_on_current_device(&scratch)) return s;
  float* o_part = scratch;
  float* lse_part = scratch + o_floats;  // o_floats is a multiple of 4 (hd is 128 or 256)
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Every split writes its whole partial (an empty split writes o = 0, lse = -inf), so nothing in
  // the scratch has to be cleared between calls.
  if (int s = far_read_uncached(q, q_stride_tok, q_stride_head, qsl, seq_lens, rope_table, table_rows, rot_dim, side,
                                pages, pos_lo, capacity, far_len, o_part, lse_part, splits, n, hq, hkv, hd, window,
                                block, far_distance, softmax_scale, err, st))
    return s;
  return merge_contiguous_partials(o_l, ol_stride_tok, ol_stride_head, lse_l, ll_stride_head, ll_stride_tok, o_part,
                                   lse_part, splits, out, out_stride_tok, out_stride_head, qsl, seq_lens, n, hq, hd,
                                   window, block, inv_alpha, st);
}

}  // extern "C"
