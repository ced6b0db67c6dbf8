// Host-side helpers shared by the entry points: error reporting, argument checks, the TMA
// descriptor of a side cache.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

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

int device_sm_count();

}  // namespace fold
