// Far-memory read, window read and one-launch step read of FOLD (fold/attention.py:148-170 of the
// reference): the kernels over the split-read template (split_read.cuh) and their C entry points.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <string>

#include "far_launch.h"
#include "host_common.h"

namespace fold {

template <class C>
__global__ void __launch_bounds__(C::NTHREADS, 1)
    far_read_kernel(const __grid_constant__ CUtensorMap map, const FarParams p) {
  split_read<C, false>(&map, nullptr, p, blockIdx.x, blockIdx.y, p.splits);
}

template <class C>
__global__ void __launch_bounds__(C::NTHREADS, 1) window_read_kernel(const FarParams p) {
  split_read<C, true>(nullptr, nullptr, p, blockIdx.x, blockIdx.y, p.splits);
}

// Cost model of the step read, in tenths of a far tile: a window tile (the window read copies
// 16-byte chunks with cp.async, which one SM issues at a lower rate than TMA moves the far read's
// boxes), and the second prologue and epilogue of a block that reads both.
constexpr int kWindowTileCost10 = 24;
constexpr int kPhaseCost10 = 30;

// How a step's S blocks per KV head share the two reads, from the device-side lengths (every
// block computes the same): w window blocks, the fewest whose window share (with a second
// prologue) fits a block's average work, and `fw` far tiles for each of them after the window.
struct StepSplit {
  int w, fw, far_tiles;
};

template <class C>
__device__ __forceinline__ StepSplit step_split(const FarParams& far, const FarParams& win, int S) {
  const int qlen = far.qsl[1] - far.qsl[0];
  const int seq = far.seq[0];
  const int hist = max(seq - qlen, 0);
  int64_t pos0, end;
  const int F = far_tiles<C::TK>(far, hist, &pos0, &end);
  const int Wt = window_tiles<C::TK>(win, hist, seq, &pos0, &end);
  StepSplit sp{max(S - 1, 1), 0, F};
  for (int w = 1; w < S; ++w) {
    const int64_t avg = (10ll * F + static_cast<int64_t>(kWindowTileCost10) * Wt + kPhaseCost10 * w) / S;
    const int64_t mine = static_cast<int64_t>(kWindowTileCost10) * ((Wt + w - 1) / w) + kPhaseCost10;
    if (mine <= avg || w == S - 1) {
      sp.w = w;
      sp.fw = static_cast<int>(max64(avg - mine, 0) / 10);
      if (static_cast<int64_t>(sp.fw) * w > F) sp.fw = F / w;
      break;
    }
  }
  return sp;
}

// The far read and the window read of one draft step in one launch. Of the S = gridDim.x blocks of
// KV head blockIdx.y, the first w read their share of the window into window slots [0, w) and
// then far tiles [x * fw, (x + 1) * fw); the other S - w blocks share the remaining far tiles
// evenly. Every block writes far slot blockIdx.x (a block without far tiles writes an empty
// partial). So the window read (a few MB) runs beside the far read, and its blocks take a smaller
// share of the far tiles. Block (0, 0) stores w in plan[0] for the merge.
template <class C>
__global__ void __launch_bounds__(C::NTHREADS, 1)
    step_read_kernel(const __grid_constant__ CUtensorMap far_map, const FarParams far, const FarParams win,
                     int* plan) {
  const int S = static_cast<int>(gridDim.x), x = static_cast<int>(blockIdx.x), h = static_cast<int>(blockIdx.y);
  const StepSplit sp = step_split<C>(far, win, S);  // lengths only: before the producer wait
  wait_for_producer();
  if (x == 0 && h == 0 && threadIdx.x == 0) *plan = sp.w;
  int b0, b1;  // this block's far tiles
  if (x < sp.w) {
    split_read<C, true>(nullptr, nullptr, win, x, h, sp.w);
    // The window read is done: its stage barriers are re-initialised for the far read (every
    // phase is complete), and its generic shared-memory accesses are ordered before the far
    // read's TMA writes into the same stages.
    fence_proxy_async_smem();
    __syncthreads();
    if (threadIdx.x == 0)
      for (int i = 0; i < C::NSTAGE; ++i) mbar_inval(stage_barriers<C>() + i);
    __syncthreads();
    b0 = x * sp.fw, b1 = b0 + sp.fw;
  } else {
    const int base = min(sp.w * sp.fw, sp.far_tiles), rest = sp.far_tiles - base, j = x - sp.w, n = S - sp.w;
    b0 = base + static_cast<int>(static_cast<int64_t>(rest) * j / n);
    b1 = base + static_cast<int>(static_cast<int64_t>(rest) * (j + 1) / n);
  }
  split_read<C, false>(&far_map, nullptr, far, x, h, S, b0, b1 - b0);
}

// ------------------------------------------------------------------ host side
namespace {
// -2: not read yet; -1: choose per shape; 0: mma.sync; 1: tcgen05.
std::atomic<int> g_far_variant{-2};
}  // namespace

int far_read_variant(int hd, int rows) {
  int v = g_far_variant.load(std::memory_order_relaxed);
  if (v == -2) {
    const char* e = getenv("FOLD_FAR_READ_KERNEL");
    v = (e && !strcmp(e, "mma")) ? 0 : (e && !strcmp(e, "tc")) ? 1 : -1;
    int expected = -2;
    g_far_variant.compare_exchange_strong(expected, v);
    v = g_far_variant.load(std::memory_order_relaxed);
  }
  if (v >= 0) return v;
  // The mma.sync kernel streams at HBM speed while its tensor work fits; past 48 query rows per
  // KV head it becomes tensor-bound and the tcgen05 kernel is faster.
  (void)hd;
  return rows > 48 ? 1 : 0;
}


// Whether the 16-byte vector rotation applies: 16-byte aligned rows of q (and qf), rotary halves
// in whole 8-element chunks, unrotated tail in whole 16-element pairs.
static int vec_rotation_ok(const void* q, int64_t q_st, int64_t q_sh, const void* qf, int64_t qf_st, int64_t qf_sh,
                           const float* table, int rot_dim, int hd) {
  if (!aligned16(q) || q_st % 8 || q_sh % 8) return 0;
  if (qf && (!aligned16(qf) || qf_st % 8 || qf_sh % 8)) return 0;
  if (table) {
    if (!aligned16(table) || rot_dim % 16 || (hd - rot_dim) % 16) return 0;
  }
  return 1;
}

// Checks the arguments of a far read (those of fold_far_read) and fills its parameter block.
int make_far_params(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const int* qsl,
                           const int* seq_lens, const float* rope_table, int table_rows, int rot_dim, const void* side,
                           int pages, int64_t pos_lo, int64_t capacity, int* far_len, void* qf, int64_t qf_stride_tok,
                           int64_t qf_stride_head, float* o_part, float* lse_part, int splits, int n, int hq, int hkv,
                           int hd, int window, int block, int far_distance, float softmax_scale, int* err,
                           FarParams* out) {
  if (!q || !qsl || !seq_lens || !side || !o_part || !lse_part)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "far read: null pointer");
  if (n < 1 || hq < 1 || hkv < 1 || hq % hkv || splits < 1 || pages < 2 || window < 1 || block < 1)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "far read: bad sizes (n, hq, hkv, splits, pages, window, block)");
  if (splits > 65535) return fail(FOLD_ERR_INVALID_ARGUMENT, "far read: too many splits");
  if (hd != 128 && hd != 256) return fail(FOLD_ERR_UNSUPPORTED, "far read: head size must be 128 or 256");
  if (rope_table && (rot_dim < 2 || rot_dim % 2 || rot_dim > hd || table_rows < 1))
    return fail(FOLD_ERR_INVALID_ARGUMENT, "far read: bad rotary size or table");
  if (pos_lo < 0 || pos_lo % 256) return fail(FOLD_ERR_INVALID_ARGUMENT, "far read: pos_lo must be a multiple of 256");
  if (static_cast<int64_t>(pages) * hkv > (1ll << 31) - 1)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "far read: side cache too large for one descriptor");
  if (n * (hq / hkv) > 64) return fail(FOLD_ERR_UNSUPPORTED, "far read: n * (hq / hkv) must be at most 64");
  FarParams prm{};
  prm.q = static_cast<const __nv_bfloat16*>(q);
  prm.q_st = q_stride_tok, prm.q_sh = q_stride_head;
  prm.qsl = qsl, prm.seq = seq_lens;
  prm.table = rope_table, prm.table_rows = table_rows, prm.rot_dim = rot_dim;
  prm.pos_lo = pos_lo, prm.capacity = capacity, prm.local_cap = static_cast<int64_t>(pages - 1) * 256;
  prm.far_len = far_len;
  prm.qf = static_cast<__nv_bfloat16*>(qf), prm.qf_st = qf_stride_tok, prm.qf_sh = qf_stride_head;
  prm.o_part = o_part, prm.lse_part = lse_part;
  prm.splits = splits, prm.n = n, prm.hq = hq, prm.hkv = hkv, prm.group = hq / hkv;
  prm.window = window, prm.block = block, prm.far_distance = far_distance;
  prm.scale_log2 = softmax_scale * kLog2e;
  prm.err = err;
  prm.vec_rot = vec_rotation_ok(q, q_stride_tok, q_stride_head, qf, qf_stride_tok, qf_stride_head, rope_table,
                                rot_dim, hd);
  *out = prm;
  return FOLD_OK;
}

// Checks the arguments of a window read (those of fold_window_read) and fills its parameter block.
int make_window_params(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const int* qsl, const int* seq_lens,
                       const void* k_cache, const void* v_cache, int64_t num_blocks, int block_size,
                       int64_t cache_stride_block, int64_t cache_stride_head, int64_t cache_stride_slot,
                       const int* block_table, int block_table_len, int window_left, int window_right, int causal,
                       float softmax_scale, float* o_part, float* lse_part, int splits, int n, int hq, int hkv, int hd,
                       int* err, FarParams* out) {
  if (!q || !qsl || !seq_lens || !k_cache || !v_cache || !block_table || !o_part || !lse_part)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "window read: null pointer");
  if (n < 1 || hq < 1 || hkv < 1 || hq % hkv || splits < 1 || splits > 65535 || block_table_len < 1)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "window read: bad sizes (n, hq, hkv, splits, block table)");
  if (hd != 128 && hd != 256) return fail(FOLD_ERR_UNSUPPORTED, "window read: head size must be 128 or 256");
  if (block_size < 16 || block_size % 16)
    return fail(FOLD_ERR_UNSUPPORTED, "window read: block size must be a positive multiple of 16");
  if (num_blocks < 1 || num_blocks > (1ll << 31) - 1)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "window read: number of blocks out of range");
  if (cache_stride_block <= 0 || cache_stride_head <= 0 || cache_stride_slot <= 0 || cache_stride_block % 8 ||
      cache_stride_head % 8 || cache_stride_slot % 8 || !aligned16(k_cache) || !aligned16(v_cache))
    return fail(FOLD_ERR_ALIGNMENT, "window read: cache planes must be 16-byte aligned with strides of 8 elements");
  if (n * (hq / hkv) > 64) return fail(FOLD_ERR_UNSUPPORTED, "window read: n * (hq / hkv) must be at most 64");
  FarParams prm{};
  prm.q = static_cast<const __nv_bfloat16*>(q);
  prm.q_st = q_stride_tok, prm.q_sh = q_stride_head;
  prm.qsl = qsl, prm.seq = seq_lens;
  prm.o_part = o_part, prm.lse_part = lse_part;
  prm.splits = splits, prm.n = n, prm.hq = hq, prm.hkv = hkv, prm.group = hq / hkv;
  prm.scale_log2 = softmax_scale * kLog2e;
  prm.err = err;
  prm.vec_rot = vec_rotation_ok(q, q_stride_tok, q_stride_head, nullptr, 0, 0, nullptr, 0, hd);
  prm.kc = static_cast<const __nv_bfloat16*>(k_cache), prm.vc = static_cast<const __nv_bfloat16*>(v_cache);
  prm.s_block = cache_stride_block, prm.s_head = cache_stride_head, prm.s_slot = cache_stride_slot;
  prm.block_table = block_table, prm.bt_len = block_table_len;
  prm.num_blocks = static_cast<int>(num_blocks), prm.block_size = block_size;
  prm.win_left = window_left, prm.win_right = window_right, prm.causal = causal ? 1 : 0;
  *out = prm;
  return FOLD_OK;
}

struct FarLaunch {
  const FarParams& prm;
  const void* side;
  int pages;
  bool cached_map;  // false: the descriptor is encoded on the stack (no heap use)
  cudaStream_t stream;
  template <class C>
  int run() const {
    CUtensorMap map;
    int s;
    if constexpr (C::FP8)
      s = fp8_side_tensor_map(side, pages, prm.hkv, &map);
    else
      s = cached_map ? side_tensor_map(side, pages, prm.hkv, C::HD, C::TK, &map)
                     : side_tensor_map_uncached(side, pages, prm.hkv, C::HD, C::TK, &map);
    if (s) return s;
    static std::atomic<uint64_t> configured{0};  // per instantiation, one bit per device
    if (int e = allow_smem(far_read_kernel<C>, C::SMEM, configured, "cudaFuncSetAttribute(far_read)")) return e;
    return launch_behind(far_read_kernel<C>, dim3(prm.splits, prm.hkv), C::NTHREADS, C::SMEM, stream,
                         "far_read_kernel", map, prm);
  }
};

struct WindowLaunch {
  const FarParams& prm;
  cudaStream_t stream;
  template <class C>
  int run() const {
    static std::atomic<uint64_t> configured{0};  // per instantiation, one bit per device
    if (int e = allow_smem(window_read_kernel<C>, C::SMEM, configured, "cudaFuncSetAttribute(window_read)")) return e;
    return launch_behind(window_read_kernel<C>, dim3(prm.splits, prm.hkv), C::NTHREADS, C::SMEM, stream,
                         "window_read_kernel", prm);
  }
};

struct StepLaunch {
  const FarParams& far;
  const FarParams& win;
  const void* side;
  int pages;
  int* plan;
  cudaStream_t stream;
  template <class C>
  int run() const {
    CUtensorMap map;
    if (int s = side_tensor_map(side, pages, far.hkv, C::HD, C::TK, &map)) return s;
    static std::atomic<uint64_t> configured{0};  // per instantiation, one bit per device
    if (int e = allow_smem(step_read_kernel<C>, C::SMEM, configured, "cudaFuncSetAttribute(step_read)")) return e;
    return launch_behind(step_read_kernel<C>, dim3(far.splits, far.hkv), C::NTHREADS, C::SMEM, stream,
                         "step_read_kernel", map, far, win, plan);
  }
};

int far_read_uncached(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const int* qsl,
                      const int* seq_lens, const float* rope_table, int table_rows, int rot_dim, const void* side,
                      int pages, int64_t pos_lo, int64_t capacity, int* far_len, float* o_part, float* lse_part,
                      int splits, int n, int hq, int hkv, int hd, int window, int block, int far_distance,
                      float softmax_scale, int* err, cudaStream_t stream) {
  FarParams prm;
  if (int s = make_far_params(q, q_stride_tok, q_stride_head, qsl, seq_lens, rope_table, table_rows, rot_dim, side,
                              pages, pos_lo, capacity, far_len, nullptr, 0, 0, o_part, lse_part, splits, n, hq, hkv,
                              hd, window, block, far_distance, softmax_scale, err, &prm))
    return s;
  const int rows = n * (hq / hkv);
  if (far_read_variant(hd, rows) == 1)
    return far_read_tc_launch(prm, side, pages, hd, ((rows + 15) / 16) * 16, false, stream);
  return with_mma_config(hd, rows, FarLaunch{prm, side, pages, false, stream});
}

}  // namespace fold

extern "C" {

int fold_far_read_select_kernel(int kernel) {
  if (kernel < -1 || kernel > 1) return fold::fail(FOLD_ERR_INVALID_ARGUMENT, "far read kernel: -1, 0 or 1");
  fold::g_far_variant.store(kernel);
  return FOLD_OK;
}

int fold_far_read_kernel_for(int hd, int n, int hq, int hkv) {
  if (hd < 1 || n < 1 || hq < 1 || hkv < 1 || hq % hkv) return -1;
  return fold::far_read_variant(hd, n * (hq / hkv));
}

int fold_far_read_default_splits(int hkv, int hd, int n, int hq) {
  (void)hd, (void)n, (void)hq;
  int sms = fold::device_sm_count();
  if (sms <= 0) sms = 148;
  if (hkv <= 0) return 1;
  return std::max(1, sms / hkv);
}

int fold_far_read(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const int* qsl, const int* seq_lens,
                  const float* rope_table, int table_rows, int rot_dim, const void* side, int pages, int64_t pos_lo,
                  int64_t capacity, int* far_len, void* qf, int64_t qf_stride_tok, int64_t qf_stride_head,
                  float* o_part, float* lse_part, int splits, int n, int hq, int hkv, int hd, int window, int block,
                  int far_distance, float softmax_scale, int* err, void* stream) {
  using namespace fold;
  FarParams prm;
  if (int s = make_far_params(q, q_stride_tok, q_stride_head, qsl, seq_lens, rope_table, table_rows, rot_dim, side,
                              pages, pos_lo, capacity, far_len, qf, qf_stride_tok, qf_stride_head, o_part, lse_part,
                              splits, n, hq, hkv, hd, window, block, far_distance, softmax_scale, err, &prm))
    return s;
  const int rows = n * (hq / hkv);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (far_read_variant(hd, rows) == 1) return far_read_tc_launch(prm, side, pages, hd, ((rows + 15) / 16) * 16, true, st);
  return with_mma_config(hd, rows, FarLaunch{prm, side, pages, true, st});
}

int fold_far_read_fp8(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const int* qsl,
                      const int* seq_lens, const float* rope_table, int table_rows, int rot_dim, const void* side8,
                      int pages, int64_t pos_lo, int64_t capacity, int* far_len, const float* k_scale,
                      const float* v_scale, float* o_part, float* lse_part, int splits, int n, int hq, int hkv, int hd,
                      int window, int block, int far_distance, float softmax_scale, int* err, void* stream) {
  using namespace fold;
  if (!k_scale || !v_scale) return fail(FOLD_ERR_INVALID_ARGUMENT, "fp8 far read: null scales");
  if (hd != 128) return fail(FOLD_ERR_UNSUPPORTED, "fp8 far read: head size must be 128");
  FarParams prm;
  if (int s = make_far_params(q, q_stride_tok, q_stride_head, qsl, seq_lens, rope_table, table_rows, rot_dim, side8,
                              pages, pos_lo, capacity, far_len, nullptr, 0, 0, o_part, lse_part, splits, n, hq, hkv,
                              hd, window, block, far_distance, softmax_scale, err, &prm))
    return s;
  if (static_cast<int64_t>(pages) * hkv * 512 > (1ll << 31) - 1)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "fp8 far read: side cache too large for one descriptor");
  prm.k_scale = k_scale, prm.v_scale = v_scale;
  const FarLaunch f{prm, side8, pages, true, static_cast<cudaStream_t>(stream)};
  return with_row_tiles<128, 128, 4, FarLaunch, true>((n * (hq / hkv) + 7) / 8, f);
}

int fold_window_read(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const int* qsl, const int* seq_lens,
                     const void* k_cache, const void* v_cache, int64_t num_blocks, int block_size,
                     int64_t cache_stride_block, int64_t cache_stride_head, int64_t cache_stride_slot,
                     const int* block_table, int block_table_len, int window_left, int window_right, int causal,
                     float softmax_scale, float* o_part, float* lse_part, int splits, int n, int hq, int hkv, int hd,
                     int* err, void* stream) {
  using namespace fold;
  FarParams prm;
  if (int s = make_window_params(q, q_stride_tok, q_stride_head, qsl, seq_lens, k_cache, v_cache, num_blocks,
                                 block_size, cache_stride_block, cache_stride_head, cache_stride_slot, block_table,
                                 block_table_len, window_left, window_right, causal, softmax_scale, o_part, lse_part,
                                 splits, n, hq, hkv, hd, err, &prm))
    return s;
  return with_mma_config(hd, n * (hq / hkv), WindowLaunch{prm, static_cast<cudaStream_t>(stream)});
}

int fold_step_read(const void* q_far, int64_t qf_stride_tok, int64_t qf_stride_head, const void* q_win,
                   int64_t qw_stride_tok, int64_t qw_stride_head, const int* qsl, const int* seq_lens,
                   const float* rope_table, int table_rows, int rot_dim, const void* side, int pages, int64_t pos_lo,
                   int64_t capacity, int* far_len, float* o_fpart, float* lse_fpart, const void* k_cache,
                   const void* v_cache, int64_t num_blocks, int block_size, int64_t cache_stride_block,
                   int64_t cache_stride_head, int64_t cache_stride_slot, const int* block_table, int block_table_len,
                   int window_left, int window_right, int causal, float* o_wpart, float* lse_wpart, int splits,
                   int* plan, int n, int hq, int hkv, int hd, int window, int block, int far_distance, float far_scale,
                   float win_scale, int* err, void* stream) {
  using namespace fold;
  if (!plan) return fail(FOLD_ERR_INVALID_ARGUMENT, "step read: null plan");
  FarParams far, win;
  if (int s = make_far_params(q_far, qf_stride_tok, qf_stride_head, qsl, seq_lens, rope_table, table_rows, rot_dim,
                              side, pages, pos_lo, capacity, far_len, nullptr, 0, 0, o_fpart, lse_fpart, splits, n,
                              hq, hkv, hd, window, block, far_distance, far_scale, err, &far))
    return s;
  if (int s = make_window_params(q_win, qw_stride_tok, qw_stride_head, qsl, seq_lens, k_cache, v_cache, num_blocks,
                                 block_size, cache_stride_block, cache_stride_head, cache_stride_slot, block_table,
                                 block_table_len, window_left, window_right, causal, win_scale, o_wpart, lse_wpart,
                                 splits, n, hq, hkv, hd, err, &win))
    return s;
  const int rows = n * (hq / hkv);
  if (far_read_variant(hd, rows) == 1)
    return fail(FOLD_ERR_UNSUPPORTED,
                "step read: this shape's far read takes the tcgen05 kernel (fold_far_read_kernel_for); issue "
                "fold_far_read and fold_window_read");
  if (splits < 2) return fail(FOLD_ERR_INVALID_ARGUMENT, "step read: at least 2 blocks per KV head");
  return with_mma_config(hd, rows, StepLaunch{far, win, side, pages, plan, static_cast<cudaStream_t>(stream)});
}

}  // extern "C"
