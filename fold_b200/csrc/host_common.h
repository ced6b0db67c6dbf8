// Host-side helpers shared by the entry points: error reporting, argument checks, the TMA
// descriptor of a side cache.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "../../include/fold_b200.h"

namespace fold {

// Records `msg` as the calling thread's last error and returns `status`.
int fail(int status, const std::string& msg);
// Returns FOLD_OK, or FOLD_ERR_CUDA with the runtime's message for `e`.
int check_cuda(cudaError_t e, const char* what);
// Checks the launch just made on the current thread.
int check_launch(const char* what);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 3-D TMA descriptor of a side cache side[pages, hkv, 256, 2*hd] bf16 seen as
// (cols = 2*hd, offset in page = 256, page*hkv + head), box (64 cols, box_rows, 1), 128-byte
// swizzle. Descriptors are cached per (pointer, shape, box).
int side_tensor_map(const void* side, int pages, int hkv, int hd, int box_rows, CUtensorMap* out);

// The same descriptor, encoded into *out on every call without touching the cache (no heap use).
int side_tensor_map_uncached(const void* side, int pages, int hkv, int hd, int box_rows, CUtensorMap* out);

// 2-D TMA descriptor of an fp8 side cache uint8 [pages][hkv][2][2][128][128] seen as rows of
// 128 bytes, box 128 x 128, 128-byte swizzle (cached like side_tensor_map).
int fp8_side_tensor_map(const void* side8, int pages, int hkv, CUtensorMap* out);

int device_sm_count();

// Raises a kernel's dynamic shared-memory limit to `bytes` on the current device. The attribute
// belongs to the device's context, so `configured` keeps one bit per device ordinal (< 64; any
// higher ordinal sets the attribute on every call). Safe to call from several host threads: a
// race only repeats the idempotent attribute call.
template <class K>
int allow_smem(K kern, int bytes, std::atomic<uint64_t>& configured, const char* what) {
  int dev = 0;
  if (int s = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return s;
  const uint64_t bit = dev >= 0 && dev < 64 ? (uint64_t(1) << dev) : 0;
  if (bit && (configured.load(std::memory_order_acquire) & bit)) return FOLD_OK;
  if (int s = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), what))
    return s;
  if (bit) configured.fetch_or(bit, std::memory_order_release);
  return FOLD_OK;
}

// Launches `kern` with programmatic stream serialisation: its blocks may be scheduled while the
// previous kernel on the stream is still running, once every block of that kernel has executed
// release_dependents (or exited). Only kernels that call wait_for_producer before their first
// global write, and before reading what such a producer writes, are launched this way.
template <class... KArgs, class... Args>
int launch_behind(void (*kern)(KArgs...), dim3 grid, int threads, int smem, cudaStream_t stream, const char* what,
                  Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid, cfg.blockDim = dim3(threads), cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream, cfg.attrs = attr, cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...), what);
}

// Far read into caller-given partial buffers with the descriptor built on the stack; the
// arguments and checks are those of fold_far_read.
int far_read_uncached(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const int* qsl,
                      const int* seq_lens, const float* rope_table, int table_rows, int rot_dim, const void* side,
                      int pages, int64_t pos_lo, int64_t capacity, int* far_len, float* o_part, float* lse_part,
                      int splits, int n, int hq, int hkv, int hd, int window, int block, int far_distance,
                      float softmax_scale, int* err, cudaStream_t stream);

// Merge of contiguous float32 split partials [splits, n, hq, hd] / [splits, hq, n] with the window
// read; the arguments of fold_merge for that partial layout.
int merge_contiguous_partials(const void* o_l, int64_t ol_stride_tok, int64_t ol_stride_head, const float* lse_l,
                              int64_t ll_stride_head, int64_t ll_stride_tok, const float* o_part,
                              const float* lse_part, int splits, void* out, int64_t out_stride_tok,
                              int64_t out_stride_head, const int* qsl, const int* seq_lens, int n, int hq, int hd,
                              int window, int block, float inv_alpha, cudaStream_t stream);

}  // namespace fold
