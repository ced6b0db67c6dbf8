// Side-cache append and gather (fold/attention.py:260-265 of the reference).
//
// One thread moves one 16-byte chunk of one (token, head) row: consecutive threads walk the 2*hd
// bf16 columns of a side-cache row, so every warp stores whole contiguous rows (512 B at hd 128).
#include <cuda_bf16.h>

#include "common.cuh"
#include "host_common.h"
#include "split_read.cuh"

namespace fold {

struct AppendParams {
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t ks_tok, ks_head, vs_tok, vs_head;
  const int64_t* positions;
  const int64_t* slots;
  __nv_bfloat16* side;
  int64_t total;  // ctx * hkv * chunks
  int64_t pos_lo, held;  // positions [pos_lo, pos_lo + held) live in this cache
  int pages, hkv, hd, chunks, skip_foreign;
  int* err;
};

__global__ void append_kernel(const AppendParams p) {
  release_dependents();  // the far read behind it may be scheduled; it waits for this grid to complete
  const int kc = p.hd >> 3;  // 16-byte chunks per K (and per V) row
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < p.total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % p.chunks);
    const int64_t rest = idx / p.chunks;
    const int h = static_cast<int>(rest % p.hkv);
    const int64_t i = rest / p.hkv;
    int64_t lp;
    if (__ldg(p.slots + i) >= 0) {
      lp = __ldg(p.positions + i) - p.pos_lo;
      if (lp < 0 || lp >= p.held) {
        const int64_t pos = lp + p.pos_lo;
        if (!p.skip_foreign || pos < 0) set_error(p.err, FOLD_DEVERR_APPEND_RANGE);
        continue;
      }
    } else {
      lp = static_cast<int64_t>(p.pages) * 256 - 1;  // dummy slot (fold/attention.py:262)
    }
    const uint4* src = c < kc ? reinterpret_cast<const uint4*>(p.k + i * p.ks_tok + h * p.ks_head) + c
                              : reinterpret_cast<const uint4*>(p.v + i * p.vs_tok + h * p.vs_head) + (c - kc);
    const int64_t row = ((lp >> 8) * p.hkv + h) * 256 + (lp & 255);
    reinterpret_cast<uint4*>(p.side + row * 2 * p.hd)[c] = __ldg(src);
  }
}

// fp8 side cache (layout in split_read.cuh, fp8_side_row): one thread quantises 16 head dims of
// one (token, head) row of K or V. A K chunk is 16 consecutive bytes of the key's row; a V chunk
// goes to 16 V^T rows, one byte each (neighbouring threads hold neighbouring tokens, so a warp's
// bytes of one V^T row land together).
struct AppendFp8Params {
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t ks_tok, ks_head, vs_tok, vs_head;
  const int64_t* positions;
  const int64_t* slots;
  uint8_t* side8;
  const float* k_scale;
  const float* v_scale;
  int64_t ctx, pos_lo, held;
  int pages, hkv, skip_foreign;
  int* err;
};

__device__ __forceinline__ uint32_t pack_e4m3x4(float a, float b, float c, float d) {
  uint32_t lo, hi;
  asm("{\n\t.reg .b16 t;\n\tcvt.rn.satfinite.e4m3x2.f32 t, %2, %1;\n\tcvt.u32.u16 %0, t;\n\t}"
      : "=r"(lo) : "f"(a), "f"(b));
  asm("{\n\t.reg .b16 t;\n\tcvt.rn.satfinite.e4m3x2.f32 t, %2, %1;\n\tcvt.u32.u16 %0, t;\n\t}"
      : "=r"(hi) : "f"(c), "f"(d));
  return lo | (hi << 16);
}

// Index layout: idx = ((chunk * hkv + h) * 2 + plane) * ctx + token, so consecutive threads walk
// consecutive tokens of one (chunk, head, plane).
__global__ void append_fp8_kernel(const AppendFp8Params p) {
  release_dependents();
  const int64_t total = p.ctx * p.hkv * 2 * 8;  // 8 chunks of 16 head dims (hd 128)
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = idx % p.ctx;
    int64_t rest = idx / p.ctx;
    const int plane = static_cast<int>(rest & 1);
    rest >>= 1;
    const int h = static_cast<int>(rest % p.hkv);
    const int c = static_cast<int>(rest / p.hkv);
    int64_t lp;
    if (__ldg(p.slots + i) >= 0) {
      lp = __ldg(p.positions + i) - p.pos_lo;
      if (lp < 0 || lp >= p.held) {
        const int64_t pos = lp + p.pos_lo;
        if (!p.skip_foreign || pos < 0) set_error(p.err, FOLD_DEVERR_APPEND_RANGE);
        continue;
      }
    } else {
      lp = static_cast<int64_t>(p.pages) * 256 - 1;  // dummy slot (fold/attention.py:262)
    }
    const __nv_bfloat16* src = plane ? p.v + i * p.vs_tok + h * p.vs_head : p.k + i * p.ks_tok + h * p.ks_head;
    const float inv = 1.f / __ldg((plane ? p.v_scale : p.k_scale) + h);
    const uint4 raw0 = __ldg(reinterpret_cast<const uint4*>(src + 16 * c));
    const uint4 raw1 = __ldg(reinterpret_cast<const uint4*>(src + 16 * c + 8));
    const __nv_bfloat162* x0 = reinterpret_cast<const __nv_bfloat162*>(&raw0);
    const __nv_bfloat162* x1 = reinterpret_cast<const __nv_bfloat162*>(&raw1);
    float f[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 a = __bfloat1622float2(x0[j]), b = __bfloat1622float2(x1[j]);
      f[2 * j] = a.x * inv, f[2 * j + 1] = a.y * inv, f[8 + 2 * j] = b.x * inv, f[9 + 2 * j] = b.y * inv;
    }
    const int page = static_cast<int>(lp >> 8), r = static_cast<int>(lp & 255), half = r >> 7, rr = r & 127;
    uint8_t* block = p.side8 + static_cast<int64_t>(fp8_side_row(page, p.hkv, h, plane, half)) * 128;
    if (plane == 0) {  // 16 consecutive bytes of the key's row
      *reinterpret_cast<uint4*>(block + rr * 128 + 16 * c) =
          make_uint4(pack_e4m3x4(f[0], f[1], f[2], f[3]), pack_e4m3x4(f[4], f[5], f[6], f[7]),
                     pack_e4m3x4(f[8], f[9], f[10], f[11]), pack_e4m3x4(f[12], f[13], f[14], f[15]));
    } else {  // one byte in each of 16 V^T rows
#pragma unroll
      for (int j = 0; j < 16; j += 4) {
        const uint32_t w = pack_e4m3x4(f[j], f[j + 1], f[j + 2], f[j + 3]);
#pragma unroll
        for (int b = 0; b < 4; ++b) block[(16 * c + j + b) * 128 + rr] = static_cast<uint8_t>(w >> (8 * b));
      }
    }
  }
}

struct GatherParams {
  const __nv_bfloat16* side;
  const int64_t* positions;
  __nv_bfloat16* k_out;
  __nv_bfloat16* v_out;
  int64_t total, pos_lo, held;
  int hkv, hd, chunks;
  int* err;
};

__global__ void gather_kernel(const GatherParams p) {
  const int kc = p.hd >> 3;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < p.total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(idx % p.chunks);
    const int64_t rest = idx / p.chunks;
    const int h = static_cast<int>(rest % p.hkv);
    const int64_t j = rest / p.hkv;
    const int64_t lp = __ldg(p.positions + j) - p.pos_lo;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (lp < 0 || lp >= p.held) {
      set_error(p.err, FOLD_DEVERR_APPEND_RANGE);
    } else {
      const int64_t row = ((lp >> 8) * p.hkv + h) * 256 + (lp & 255);
      val = reinterpret_cast<const uint4*>(p.side + row * 2 * p.hd)[c];
    }
    __nv_bfloat16* dst = c < kc ? p.k_out : p.v_out;
    reinterpret_cast<uint4*>(dst + (j * p.hkv + h) * p.hd)[c < kc ? c : c - kc] = val;
  }
}

static int grid_for(int64_t total, int threads) {
  const int64_t want = (total + threads - 1) / threads;
  int sms = device_sm_count();
  if (sms <= 0) sms = 148;
  const int64_t cap = static_cast<int64_t>(sms) * 16;
  return static_cast<int>(want < 1 ? 1 : (want > cap ? cap : want));
}

}  // namespace fold

extern "C" {

int fold_append(const void* k, int64_t k_stride_tok, int64_t k_stride_head, const void* v, int64_t v_stride_tok,
                int64_t v_stride_head, const int64_t* positions, const int64_t* slots, int ctx, void* side,
                int pages, int hkv, int hd, int64_t pos_lo, int skip_foreign, int* err, void* stream) {
  using namespace fold;
  if (ctx == 0) return FOLD_OK;
  if (!k || !v || !positions || !slots || !side) return fail(FOLD_ERR_INVALID_ARGUMENT, "append: null pointer");
  if (ctx < 0 || pages < 2 || hkv < 1 || hd < 8 || hd % 8)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "append: bad sizes (ctx, pages, hkv, hd % 8)");
  if (!aligned16(k) || !aligned16(v) || !aligned16(side) || k_stride_tok % 8 || k_stride_head % 8 ||
      v_stride_tok % 8 || v_stride_head % 8)
    return fail(FOLD_ERR_ALIGNMENT, "append: K/V rows must start on 16-byte boundaries");
  AppendParams p{};
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.ks_tok = k_stride_tok, p.ks_head = k_stride_head, p.vs_tok = v_stride_tok, p.vs_head = v_stride_head;
  p.positions = positions, p.slots = slots;
  p.side = static_cast<__nv_bfloat16*>(side);
  p.chunks = 2 * hd / 8;
  p.total = static_cast<int64_t>(ctx) * hkv * p.chunks;
  p.pos_lo = pos_lo, p.held = static_cast<int64_t>(pages - 1) * 256;
  p.pages = pages, p.hkv = hkv, p.hd = hd, p.skip_foreign = skip_foreign;
  p.err = err;
  append_kernel<<<grid_for(p.total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("append_kernel");
}

int fold_append_fp8(const void* k, int64_t k_stride_tok, int64_t k_stride_head, const void* v,
                    int64_t v_stride_tok, int64_t v_stride_head, const int64_t* positions, const int64_t* slots,
                    int ctx, void* side8, int pages, int hkv, int hd, const float* k_scale, const float* v_scale,
                    int64_t pos_lo, int skip_foreign, int* err, void* stream) {
  using namespace fold;
  if (ctx == 0) return FOLD_OK;
  if (!k || !v || !positions || !slots || !side8 || !k_scale || !v_scale)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "fp8 append: null pointer");
  if (hd != 128) return fail(FOLD_ERR_UNSUPPORTED, "fp8 append: head size must be 128");
  if (ctx < 0 || pages < 2 || hkv < 1) return fail(FOLD_ERR_INVALID_ARGUMENT, "fp8 append: bad sizes");
  if (!aligned16(k) || !aligned16(v) || !aligned16(side8) || k_stride_tok % 8 || k_stride_head % 8 ||
      v_stride_tok % 8 || v_stride_head % 8)
    return fail(FOLD_ERR_ALIGNMENT, "fp8 append: K/V rows must start on 16-byte boundaries");
  AppendFp8Params p{};
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.ks_tok = k_stride_tok, p.ks_head = k_stride_head, p.vs_tok = v_stride_tok, p.vs_head = v_stride_head;
  p.positions = positions, p.slots = slots;
  p.side8 = static_cast<uint8_t*>(side8);
  p.k_scale = k_scale, p.v_scale = v_scale;
  p.ctx = ctx, p.pos_lo = pos_lo, p.held = static_cast<int64_t>(pages - 1) * 256;
  p.pages = pages, p.hkv = hkv, p.skip_foreign = skip_foreign;
  p.err = err;
  append_fp8_kernel<<<grid_for(static_cast<int64_t>(ctx) * hkv * 16, 256), 256, 0,
                      static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("append_fp8_kernel");
}

int fold_gather(const void* side, int pages, int hkv, int hd, int64_t pos_lo, const int64_t* positions, int m,
                void* k_out, void* v_out, int* err, void* stream) {
  using namespace fold;
  if (m == 0) return FOLD_OK;
  if (!side || !positions || !k_out || !v_out) return fail(FOLD_ERR_INVALID_ARGUMENT, "gather: null pointer");
  if (m < 0 || pages < 2 || hkv < 1 || hd < 8 || hd % 8)
    return fail(FOLD_ERR_INVALID_ARGUMENT, "gather: bad sizes");
  if (!aligned16(side) || !aligned16(k_out) || !aligned16(v_out))
    return fail(FOLD_ERR_ALIGNMENT, "gather: buffers must be 16-byte aligned");
  GatherParams p{};
  p.side = static_cast<const __nv_bfloat16*>(side);
  p.positions = positions;
  p.k_out = static_cast<__nv_bfloat16*>(k_out);
  p.v_out = static_cast<__nv_bfloat16*>(v_out);
  p.chunks = 2 * hd / 8;
  p.total = static_cast<int64_t>(m) * hkv * p.chunks;
  p.pos_lo = pos_lo, p.held = static_cast<int64_t>(pages - 1) * 256;
  p.hkv = hkv, p.hd = hd, p.err = err;
  gather_kernel<<<grid_for(p.total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("gather_kernel");
}

}  // extern "C"
