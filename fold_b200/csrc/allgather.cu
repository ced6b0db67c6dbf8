// The NCCL data plane of the sequence-sharded far read: every rank folds its split partials into
// one (o, lse) record and the ranks' records are all-gathered with ncclAllGather over NVLink;
// fold_merge then merges the gathered records with the window read.
//
// NCCL is not linked: the first call looks ncclAllGather up in the libnccl.so.2 the process has
// already loaded (the one PyTorch's ProcessGroupNCCL uses, so the communicator and the call come
// from the same library), else in the system's libnccl.so.2. Only the types come from nccl.h.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <string>

#include "host_common.h"

namespace fold {
namespace {

using AllGatherFn = ncclResult_t (*)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
using ErrorStringFn = const char* (*)(ncclResult_t);

std::once_flag g_nccl_once;
AllGatherFn g_all_gather = nullptr;
ErrorStringFn g_error_string = nullptr;
std::string g_nccl_missing;

void resolve_nccl() {
  void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
  if (!lib) {
    const char* e = dlerror();
    g_nccl_missing = std::string("libnccl.so.2 not found: ") + (e ? e : "");
    return;
  }
  g_all_gather = reinterpret_cast<AllGatherFn>(dlsym(lib, "ncclAllGather"));
  g_error_string = reinterpret_cast<ErrorStringFn>(dlsym(lib, "ncclGetErrorString"));
  if (!g_all_gather) g_nccl_missing = "libnccl.so.2 has no ncclAllGather";
}

}  // namespace
}  // namespace fold

extern "C" {

int fold_allgather_partials(void* comm, const float* o_part, const float* lse_part, int splits, float* send,
                            float* recv, int n, int hq, int hd, void* stream) {
  using namespace fold;
  if (!comm || !send || !recv) return fail(FOLD_ERR_INVALID_ARGUMENT, "all-gather of partials: null pointer");
  if (n < 1 || hq < 1 || hd < 4 || splits < 1)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "all-gather of partials: bad sizes");
  std::call_once(g_nccl_once, resolve_nccl);
  if (!g_all_gather) return fail(FOLD_ERR_UNSUPPORTED, "all-gather of partials: " + g_nccl_missing);
  const int64_t o_floats = static_cast<int64_t>(n) * hq * hd;
  // this rank's record: o [n, hq, hd] then lse [hq, n] (o_floats is a multiple of 4, so the LSE
  // part keeps the 16-byte alignment of `send`)
  if (int s = fold_combine(o_part, lse_part, splits, send, send + o_floats, n, hq, hd, stream)) return s;
  const size_t per = static_cast<size_t>(o_floats + static_cast<int64_t>(hq) * n);
  const ncclResult_t r = g_all_gather(send, recv, per, ncclFloat32, static_cast<ncclComm_t>(comm),
                                      static_cast<cudaStream_t>(stream));
  if (r != ncclSuccess)
    return fail(FOLD_ERR_CUDA, std::string("ncclAllGather: ") +
                                   (g_error_string ? g_error_string(r) : std::to_string(static_cast<int>(r))));
  return FOLD_OK;
}

}  // extern "C"
