#pragma once

// The split-KV read of FOLD (fold/attention.py:162-170 of the reference) as a device template:
// one CTA per (split, KV head) streams tiles of keys with TMA and computes the split's partial
// (o, lse) on mma.sync tiles. far_read.cu instantiates it as the far-memory read (side cache,
// query rotated to the shared far position) and as the window read (paged drafter cache, exact
// positions); far_exchange.cu adds the exchange of the partials after it.
//
// Per CTA: thread 0 keeps a ring of shared-memory stages filled with tiles of TK keys of this
// head's K and V rows (TMA, 128-byte swizzle, completion on mbarriers), and all eight warps
// compute, per tile,
//   S^T = K . Qf^T     (keys on the MMA M dimension, the n*G query rows on N: no row padding)
//   P^T = exp2(S^T * scale * log2e - m)      (online softmax with a lazily raised row maximum)
//   O^T += V^T . P^T
// on mma.sync tiles (bf16 for S^T, f16 for O^T), and finally write the split's normalised partial
// (o, lse).
//
// The running row maximum m only moves when a new logit exceeds it by more than kRaise (log2
// units), which is decided for the whole CTA by one OR-barrier per tile. So the common tile needs
// no cross-warp max exchange and no rescaling. P stays below 2^kRaise, inside the f16 range, and
// the fp32 sums of at most 2^15 * (keys per split) stay far from overflow, so a high threshold
// costs no accuracy and makes raises rare after the first tile.
//
// P is rounded to f16 (11 significant bits) for the PV product. With bf16 P (8 bits), a row whose
// mass sits on a few keys carried the rounding of those weights straight into the output:
// 0.03-0.05 on the x8 outlier channels of the 128K Llama workload, against 0.002 with f16. V tiles are bf16 in
// memory; their MMA fragments are re-encoded as f16 in registers (exact in the f16 range; the
// conversion saturates at +-65504), since an MMA takes both operands in one type. Q and K stay
// bf16 for S^T = K . Q^T.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "far_read.cuh"

namespace fold {

// FP8: the side cache holds e4m3 K rows and V^T (fp8_side layout below); head size 128 only, so
// one 128-byte row of K (or of V^T over 128 keys) is one TMA box row.
template <int HD_, int NT_, int TK_, int HG_, bool FP8_ = false, int NW_ = 8>
struct FarCfg {
  static constexpr int HD = HD_, NT = NT_, TK = TK_, HG = HG_;
  static constexpr bool FP8 = FP8_;
  static constexpr int ROWS = 8 * NT;
  static constexpr int NW = NW_;  // warps; thread 0 also issues the TMA copies
  static constexpr int NTHREADS = NW * 32;
  static constexpr int KBOX = HD / 64;  // 64-column boxes per K (and per V) row block
  static constexpr int BOX_BYTES = TK * 128;
  static constexpr int STAGE_BYTES = FP8 ? 2 * BOX_BYTES : 2 * KBOX * BOX_BYTES;
  static constexpr int MT = TK / 16;  // key m-tiles per tile (one per QK warp column)
  static constexpr int NG = NW / MT;  // QK warps sharing one m-tile split the n-tiles
  static constexpr int QNT = (NT + NG - 1) / NG;
  static constexpr int KG = NW / HG;  // PV: HG hd groups x KG key groups
  static constexpr int PV_MT = HD / 16 / HG;
  static constexpr int PV_KS = TK / 16 / KG;
  static constexpr int QSTRIDE = HD + 8;                        // elements; 16-byte units odd
  static constexpr int PSTRIDE = 8 * ((NT & 1) ? NT : NT + 1);  // elements; 16-byte units odd
  static constexpr bool Q_REGS = QNT * (HD / 16) * 2 <= 80;
  static constexpr int Q_BYTES = ROWS * QSTRIDE * 2;
  static constexpr int P_BYTES = 2 * TK * PSTRIDE * 2;
  static constexpr int RED_BYTES = MT * ROWS * 4;
  static constexpr int ROW_BYTES = 2 * 64 * 4;
  static constexpr int FIXED = Q_BYTES + P_BYTES + RED_BYTES + ROW_BYTES + 8 * 8 + 1024;
  static constexpr int NSTAGE_FIT = (kSmemLimit - FIXED) / STAGE_BYTES;
  static constexpr int NSTAGE_MAX = FP8 ? 6 : 4;  // at most 8: the barriers share 64 bytes
  static constexpr int NSTAGE = NSTAGE_FIT > NSTAGE_MAX ? NSTAGE_MAX : NSTAGE_FIT;
  static constexpr int OFF_Q = NSTAGE * STAGE_BYTES;
  static constexpr int OFF_P = OFF_Q + Q_BYTES;
  static constexpr int OFF_RED = OFF_P + P_BYTES;
  static constexpr int OFF_ROW = OFF_RED + RED_BYTES;
  static constexpr int OFF_BAR = OFF_ROW + ROW_BYTES;
  static constexpr int SMEM = OFF_BAR + 8 * 8 + 1024;
  static_assert(NSTAGE >= 2, "shared memory too small for two stages");
  static_assert(SMEM <= kSmemLimit, "shared memory budget");
  static_assert(MT * NG == NW && HG * KG == NW, "warp split");
  static_assert(PV_MT >= 1 && PV_KS >= 1, "warp split");
  static_assert(ROWS * HD * 4 <= NSTAGE * STAGE_BYTES, "epilogue staging");
  static_assert(TK <= 256 && 256 % TK == 0, "tiles stay inside one 256-entry page");
  static_assert(!FP8 || (HD == 128 && TK == 128), "fp8 side cache: head size 128, tiles of 128 keys");
};

// The fp8 side cache: uint8 [pages][hkv][2 planes][2 halves][128 rows][128 bytes]. Plane 0 holds
// K: row r of half kh is key kh * 128 + r of the page, its 128 bytes the e4m3 head dims. Plane 1
// holds V^T: row d of half kh is head dim d, byte c the e4m3 value of key kh * 128 + c. So a tile
// of 128 keys is one 16 KB box of K and one of V^T, and a V^T row gives the keys of one head dim
// in consecutive bytes (the order an MMA fragment of V^T takes them in). Row of a (page, head,
// plane, half) block in the 2-D view [rows][128 bytes]:
__device__ __forceinline__ int fp8_side_row(int page, int hkv, int h, int plane, int half) {
  return (((page * hkv + h) * 2 + plane) * 2 + half) * 128;
}

// FP8 fragment order: an ldmatrix of byte pairs gives a thread the bytes [4 t4, 4 t4 + 4) of a
// 16-byte chunk, while an f16 MMA fragment takes k = (2 t4, 2 t4 + 1) and (2 t4 + 8, 2 t4 + 9).
// So within each group of 16, element p of the chunk (a head dim of K, a key of V^T) is used as k
// slot fp8_slot(p): Q is stored with its head dims at these slots, and P^T with its keys.
__host__ __device__ constexpr int fp8_slot(int p) {
  return (p >> 1) + 7 * ((p >> 1) & 1) + (p & 1);
}


// Issues the TMA copies of tile `tile` (index in this cache) of head h into stage `st`.
template <class C>
__device__ __forceinline__ void issue_tile(unsigned char* smem, uint64_t* full, const CUtensorMap* map, int st,
                                           int tile, int hkv, int h, uint64_t pol) {
  mbar_arrive_expect_tx(&full[st], C::STAGE_BYTES);
  const int64_t lp = static_cast<int64_t>(tile) * C::TK;
  const int page = static_cast<int>(lp >> 8), off = static_cast<int>(lp & 255);
  unsigned char* dst = smem + st * C::STAGE_BYTES;
  if constexpr (C::FP8) {  // the K box, then the V^T box, of the tile's half of its page
    const int half = off >> 7;
    tma_load_2d(dst, map, &full[st], 0, fp8_side_row(page, hkv, h, 0, half), pol);
    tma_load_2d(dst + C::BOX_BYTES, map, &full[st], 0, fp8_side_row(page, hkv, h, 1, half), pol);
  } else {
    const int c2 = page * hkv + h;
#pragma unroll
    for (int b = 0; b < 2 * C::KBOX; ++b) tma_load_3d(dst + b * C::BOX_BYTES, map, &full[st], b * 64, off, c2, pol);
  }
}

// Window read: the cache block that holds a warp's rows of the tile at tpos (the warp's TK / 8
// rows lie in one 16-position chunk of one block: every block size is a multiple of 16), or -1
// past the context. An entry outside the cache records FOLD_DEVERR_BLOCK_TABLE and reads as -1.
template <class C>
__device__ __forceinline__ int window_block(const FarParams& p, int64_t tpos, int seq) {
  const int64_t pos = tpos + (threadIdx.x >> 5) * (C::TK / C::NW);
  if (pos >= seq) return -1;
  const int64_t lb = pos / p.block_size;
  const int blk = lb < p.bt_len ? __ldg(p.block_table + lb) : -1;
  if (blk < 0 || blk >= p.num_blocks) {
    set_error(p.err, FOLD_DEVERR_BLOCK_TABLE);
    return -1;
  }
  return blk;
}

// Window read: all threads copy the tile of positions [tpos, tpos + TK) of head h from the paged
// cache into stage `st` with 16-byte cp.async, each warp its TK / 8 consecutive rows from block
// `blk` (window_block). A half-warp copies one row's K or V plane (contiguous), and each 16-byte
// chunk lands at its 128-byte-swizzled place in the stage, the layout a TMA box of the far read
// gives. Rows at or past seq, and all rows when blk is -1, are zero-filled, so no slot that holds
// no context entry reaches the MMAs. Every thread then arrives on the stage's mbarrier when its
// copies have landed.
template <class C>
__device__ __forceinline__ void issue_window_tile(unsigned char* smem, uint64_t* full, int st, int64_t tpos, int seq,
                                                  int h, int blk, const FarParams& p) {
  constexpr int RPW = C::TK / C::NW;  // rows per warp
  constexpr int CPR = C::HD / 8;      // 16-byte chunks per K (or V) row
  constexpr int LPP = CPR >= 32 ? 32 : CPR;  // lanes per (row, plane): 16 at hd 128, 32 at hd 256
  constexpr int STEPS = RPW * 2 * CPR / 32;
  static_assert(RPW <= 16 && 16 % RPW == 0 && CPR % LPP == 0 && (RPW * 2 * CPR) % 32 == 0, "window tile split");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = warp * RPW;
  const int64_t pos0 = tpos + row0;
  // lane -> 16-byte chunk cc of a row; at hd 128 lanes 0-15 copy K and 16-31 copy V of one row per
  // step, at hd 256 every lane copies one chunk of K, then of V
  const int cc = lane % LPP;
  const int lane_plane = LPP == 16 ? lane / 16 : 0;
  const int64_t slot0 = pos0 - (pos0 / p.block_size) * p.block_size;
  const int64_t off = blk >= 0 ? static_cast<int64_t>(blk) * p.s_block + h * p.s_head + slot0 * p.s_slot + cc * 8 : 0;
  const int rows_valid = blk >= 0 ? static_cast<int>(max64(0, min64(RPW, seq - pos0))) : 0;
  const uint32_t stage = smem_u32(smem + st * C::STAGE_BYTES);
#pragma unroll 1
  for (int k = 0; k < STEPS; ++k) {
    const int plane = LPP == 16 ? lane_plane : (k & 1);
    const int r = LPP == 16 ? k : (k >> 1);
    const int row = row0 + r;
    const bool valid = r < rows_valid;
    const __nv_bfloat16* src = (plane ? p.vc : p.kc) + (valid ? off + r * p.s_slot : 0);
    const uint32_t dst = stage + (plane * C::KBOX + (cc >> 3)) * C::BOX_BYTES + row * 128 + (((cc & 7) ^ (row & 7)) << 4);
    cp_async_16(dst, src, valid ? 16u : 0u);
  }
  cp_async_mbar_arrive(&full[st]);
}

// One thread's share of a CTA's query rows for the vectorised rotation: each work item is one
// row's pair of 8-element chunks ([8c, 8c+8) with its neox partner [RH+8c, ...), or 16 unrotated
// elements), held as 16-byte vectors. The loads are issued first thing in the kernel (they depend
// on nothing the kernel reads), so their latency overlaps the step-length and table reads.
template <class C>
struct QueryLoad {
  static constexpr int PAIRS = C::HD / 16;
  static constexpr int ITEMS = C::ROWS * PAIRS;
  static constexpr int MAXI = (ITEMS + C::NTHREADS - 1) / C::NTHREADS;
  uint4 a[MAXI], b[MAXI];
  float4 c0[MAXI], c1[MAXI], s0[MAXI], s1[MAXI];  // the rows' cos and sin (load_table_vec)
};

// rh8 = rotated 8-element chunks per half (0: no rotation).
template <class C>
__device__ __forceinline__ void load_query_vec(const FarParams& p, int rh8, int RH, int h, int nrows, int G,
                                               QueryLoad<C>& ql) {
  constexpr int PAIRS = QueryLoad<C>::PAIRS, ITEMS = QueryLoad<C>::ITEMS;
#pragma unroll
  for (int k = 0; k < QueryLoad<C>::MAXI; ++k) {
    const int e = threadIdx.x + k * C::NTHREADS;
    ql.a[k] = ql.b[k] = make_uint4(0, 0, 0, 0);
    if (e < ITEMS) {
      const int rho = e / PAIRS, c = e - (e / PAIRS) * PAIRS;
      if (rho < nrows) {
        const int r = rho / G, hq = h * G + (rho - r * G);
        const __nv_bfloat16* qr = p.q + r * p.q_st + hq * p.q_sh;
        const int off_a = c < rh8 ? 8 * c : 2 * RH * (rh8 > 0) + 16 * (c - rh8);
        const int off_b = c < rh8 ? RH + 8 * c : off_a + 8;
        ql.a[k] = __ldg(reinterpret_cast<const uint4*>(qr + off_a));
        ql.b[k] = __ldg(reinterpret_cast<const uint4*>(qr + off_b));
      }
    }
  }
}

// Issues the loads of the cos/sin values of the table row `trow` (cos then sin; read only when
// rh8 > 0) that this thread's rotation items take. Called before the producer wait: no kernel that
// releases its dependents early writes the table.
template <class C>
__device__ __forceinline__ void load_table_vec(const float* trow, int rh8, int RH, int nrows, QueryLoad<C>& ql) {
  constexpr int PAIRS = QueryLoad<C>::PAIRS, ITEMS = QueryLoad<C>::ITEMS;
#pragma unroll
  for (int k = 0; k < QueryLoad<C>::MAXI; ++k) {
    const int e = threadIdx.x + k * C::NTHREADS;
    ql.c0[k] = ql.c1[k] = ql.s0[k] = ql.s1[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (e < ITEMS) {
      const int rho = e / PAIRS, c = e - (e / PAIRS) * PAIRS;
      if (rho < nrows && c < rh8) {
        const float4* tc = reinterpret_cast<const float4*>(trow + 8 * c);
        const float4* ts = reinterpret_cast<const float4*>(trow + RH + 8 * c);
        ql.c0[k] = __ldg(tc), ql.c1[k] = __ldg(tc + 1), ql.s0[k] = __ldg(ts), ql.s1[k] = __ldg(ts + 1);
      }
    }
  }
}

// Vectorised far-query rotation of the loaded rows with the loaded table values (load_query_vec,
// load_table_vec), written to the query tile Qs (and to qf by split 0).
template <class C>
__device__ __forceinline__ void rotate_query_vec(const FarParams& p, const QueryLoad<C>& ql, int rh8, int RH,
                                                 float sgn, int h, int split, int nrows, int G, __nv_bfloat16* Qs) {
  constexpr int PAIRS = QueryLoad<C>::PAIRS, ITEMS = QueryLoad<C>::ITEMS, MAXI = QueryLoad<C>::MAXI;
  const int tid = threadIdx.x;
  const float4 *c0 = ql.c0, *c1 = ql.c1, *s0 = ql.s0, *s1 = ql.s1;
#pragma unroll
  for (int k = 0; k < MAXI; ++k) {
    const int e = tid + k * C::NTHREADS;
    if (e >= ITEMS) continue;
    const int rho = e / PAIRS, c = e - (e / PAIRS) * PAIRS;
    int off_a, off_b;
    uint4 ya = ql.a[k], yb = ql.b[k];
    if (c < rh8) {
      off_a = 8 * c, off_b = RH + 8 * c;
      const float cs[8] = {c0[k].x, c0[k].y, c0[k].z, c0[k].w, c1[k].x, c1[k].y, c1[k].z, c1[k].w};
      const float sn[8] = {s0[k].x, s0[k].y, s0[k].z, s0[k].w, s1[k].x, s1[k].y, s1[k].z, s1[k].w};
      const __nv_bfloat162* xa = reinterpret_cast<const __nv_bfloat162*>(&ql.a[k]);
      const __nv_bfloat162* xb = reinterpret_cast<const __nv_bfloat162*>(&ql.b[k]);
      uint32_t* oa = reinterpret_cast<uint32_t*>(&ya);
      uint32_t* ob = reinterpret_cast<uint32_t*>(&yb);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 x = __bfloat1622float2(xa[j]), xp = __bfloat1622float2(xb[j]);
        const float c_0 = cs[2 * j], c_1 = cs[2 * j + 1];
        const float s_0 = sgn * sn[2 * j], s_1 = sgn * sn[2 * j + 1];
        const float a0 = x.x * c_0 - xp.x * s_0, a1 = x.y * c_1 - xp.y * s_1;
        const float b0 = xp.x * c_0 + x.x * s_0, b1 = xp.y * c_1 + x.y * s_1;
        oa[j] = C::FP8 ? pack_f16_sat(a0, a1) : pack_bf16(a0, a1);
        ob[j] = C::FP8 ? pack_f16_sat(b0, b1) : pack_bf16(b0, b1);
      }
    } else {
      off_a = 2 * RH * (rh8 > 0) + 16 * (c - rh8), off_b = off_a + 8;
      if constexpr (C::FP8) {
        uint32_t* oa = reinterpret_cast<uint32_t*>(&ya);
        uint32_t* ob = reinterpret_cast<uint32_t*>(&yb);
#pragma unroll
        for (int j = 0; j < 4; ++j) oa[j] = bf16x2_to_f16x2(oa[j]), ob[j] = bf16x2_to_f16x2(ob[j]);
      }
    }
    if constexpr (C::FP8) {  // f16, each pair of head dims at its fp8 fragment slot
      const uint32_t* wa = reinterpret_cast<const uint32_t*>(&ya);
      const uint32_t* wb = reinterpret_cast<const uint32_t*>(&yb);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int da = off_a + 2 * j, db = off_b + 2 * j;
        *reinterpret_cast<uint32_t*>(Qs + rho * C::QSTRIDE + (da & ~15) + fp8_slot(da & 15)) = wa[j];
        *reinterpret_cast<uint32_t*>(Qs + rho * C::QSTRIDE + (db & ~15) + fp8_slot(db & 15)) = wb[j];
      }
      continue;  // no far-query output for the fp8 read
    }
    *reinterpret_cast<uint4*>(Qs + rho * C::QSTRIDE + off_a) = ya;
    *reinterpret_cast<uint4*>(Qs + rho * C::QSTRIDE + off_b) = yb;
    if (p.qf && split == 0 && rho < nrows) {
      const int r = rho / G, hq = h * G + (rho - r * G);
      __nv_bfloat16* o = p.qf + r * p.qf_st + hq * p.qf_sh;
      *reinterpret_cast<uint4*>(o + off_a) = ya;
      *reinterpret_cast<uint4*>(o + off_b) = yb;
    }
  }
}

// Element-wise far-query rotation for the layouts the vector path does not take (unaligned rows of
// q or qf, or a rotary size that is not whole 8-element chunks); trow as for rotate_query_vec.
template <class C>
__device__ __forceinline__ void rotate_query_scalar(const FarParams& p, const float* trow, int RH, float sgn, int h,
                                                    int split, int nrows, int G, __nv_bfloat16* Qs) {
  for (int e = threadIdx.x; e < C::ROWS * C::HD; e += C::NTHREADS) {
    const int rho = e / C::HD, d = e - (e / C::HD) * C::HD;
    float y = 0.f;
    if (rho < nrows) {
      const int r = rho / G, hq = h * G + (rho - r * G);
      const __nv_bfloat16* qr = p.q + r * p.q_st + hq * p.q_sh;
      const float x = bf2f(qr[d]);
      if (trow && d < 2 * RH) {
        const bool lo = d < RH;
        const int i = lo ? d : d - RH;
        const float xp = bf2f(qr[lo ? d + RH : d - RH]);
        const float c = trow[i], s = sgn * trow[RH + i];
        y = lo ? x * c - xp * s : x * c + xp * s;
      } else {
        y = x;
      }
      if constexpr (C::FP8) {
        const __half yh = __float2half_rn(y);
        *reinterpret_cast<__half*>(Qs + rho * C::QSTRIDE + (d & ~15) + fp8_slot(d & 15)) = yh;
      } else {
        const __nv_bfloat16 yb = __float2bfloat16_rn(y);
        if (p.qf && split == 0) p.qf[r * p.qf_st + hq * p.qf_sh + d] = yb;
        Qs[rho * C::QSTRIDE + d] = yb;
      }
    } else {
      Qs[rho * C::QSTRIDE + d] = __float2bfloat16_rn(0.f);  // zero bits: 0 in f16 as well
    }
  }
}

// Window read: first and one-past-last visible position of row r (at position hist + r) under the
// FlashAttention window [p - left, p + right] (a negative side is unbounded), causal or not,
// within the seq context entries. Both grow with r.
__device__ __forceinline__ int64_t window_lo(const FarParams& p, int hist, int r) {
  return p.win_left < 0 ? 0 : max64(0, static_cast<int64_t>(hist) + r - p.win_left);
}
__device__ __forceinline__ int64_t window_hi(const FarParams& p, int hist, int seq, int r) {
  const int64_t pos = static_cast<int64_t>(hist) + r;
  int64_t hi = seq;
  if (p.win_right >= 0) hi = min64(hi, pos + p.win_right + 1);
  if (p.causal) hi = min64(hi, pos + 1);
  return max64(hi, 0);
}

// Far read: the tiles of TK keys this cache holds for the step, the position of tile 0 and the end
// of the last row's far keys in this cache (row r reads [0, H - W - B + 1 + r)).
template <int TK>
__device__ __forceinline__ int far_tiles(const FarParams& p, int hist, int64_t* pos0, int64_t* end) {
  const int lim_base = hist - p.window - p.block + 1;
  *end = min64(max(lim_base + p.n - 1, 0), p.pos_lo + p.local_cap);
  *pos0 = p.pos_lo;
  const int64_t len = max64(*end - p.pos_lo, 0);
  return static_cast<int>((len + TK - 1) / TK);
}

// Window read: the tiles of TK positions (aligned to TK) covering the union of the rows' windows,
// the position of tile 0 and the union's end.
template <int TK>
__device__ __forceinline__ int window_tiles(const FarParams& p, int hist, int seq, int64_t* pos0, int64_t* end) {
  const int64_t u_lo = window_lo(p, hist, 0), u_hi = window_hi(p, hist, seq, p.n - 1);
  const int64_t t0 = u_lo / TK;
  *pos0 = t0 * TK;
  *end = u_hi;
  return u_hi > u_lo ? static_cast<int>((u_hi + TK - 1) / TK - t0) : 0;
}

// The mbarriers of a CTA's stage ring (in the dynamic shared memory of a split read).
template <class C>
__device__ __forceinline__ uint64_t* stage_barriers() {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  return reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
}

// The split-KV read of one (split of nsplits, KV head h), in two modes.
//   WIN = false, far memory: K|V rows of the side cache through `map`, the query rotated to the
//     shared far position, row r reads positions [0, H - W - B + 1 + r) (fold/attention.py:164).
//   WIN = true, window read: K and V rows of the paged cache (p.kc, p.vc, cp.async by every
//     thread), the query as given, row r reads its exact-position window
//     (fold/attention.py:148-151,163).
// The CTA reads tiles [t_begin, t_begin + ntiles) of the cache's tiles for the step: the share of
// split `split` of `nsplits`, or, with range_begin >= 0, the range [range_begin, range_begin +
// range_tiles) clipped to the step's tiles (`split` is then only the slot of its partial).
template <class C, bool WIN>
__device__ __forceinline__ void split_read(const CUtensorMap* map, const CUtensorMap* vmap, const FarParams& p,
                                           int split, int h, int nsplits, int range_begin = -1,
                                           int range_tiles = 0) {
  static_assert(!(WIN && C::FP8), "the window read takes the drafter's bf16 cache");
  constexpr int HD = C::HD, NT = C::NT, TK = C::TK, ROWS = C::ROWS, NTH = C::NTHREADS;
  constexpr int NSTAGE = C::NSTAGE, QNT = C::QNT, PV_MT = C::PV_MT, MT = C::MT, NG = C::NG;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(smem + C::OFF_Q);
  float* red = reinterpret_cast<float*>(smem + C::OFF_RED);
  float* row_m = reinterpret_cast<float*>(smem + C::OFF_ROW);
  float* row_inv = row_m + 64;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = p.group;
  const int nrows = p.n * G;
  const int RH = p.rot_dim >> 1;
  const int rh8 = (!WIN && p.table) ? RH / 8 : 0;  // the far read rotates when it has a table
  QueryLoad<C> ql;
  if (p.vec_rot) load_query_vec<C>(p, rh8, RH, h, nrows, G, ql);

  // Step geometry, from the device-side lengths (fold/kernels.py:24-30).
  const int qlen = p.qsl[1] - p.qsl[0];
  const int seq = p.seq[0];
  const int hist = max(seq - qlen, 0);
  const int lim_base = hist - p.window - p.block + 1;  // far: row r reads positions [0, lim_base + r)
  int64_t end;   // far: end of this cache's keys for the last row
  int64_t pos0;  // position of tile 0
  const int tiles = WIN ? window_tiles<TK>(p, hist, seq, &pos0, &end) : far_tiles<TK>(p, hist, &pos0, &end);
  const int t_begin = range_begin >= 0 ? min(range_begin, tiles)
                                       : static_cast<int>(static_cast<int64_t>(tiles) * split / nsplits);
  const int ntiles = range_begin >= 0
                         ? max(min(range_begin + range_tiles, tiles) - t_begin, 0)
                         : static_cast<int>(static_cast<int64_t>(tiles) * (split + 1) / nsplits) - t_begin;

  // Far query (fold/kernels.py:31-46): rotate by (D - H) * inv_freq with cos/sin from the table
  // row of |D - H|; the row's loads are issued here. The window read takes the query as it is.
  const float* trow = nullptr;
  float sgn = 1.f;
  bool rope_range = false;  // |D - H| past the table: recorded once the outputs may be written
  if constexpr (!WIN) {
    const int delta = p.far_distance - hist;
    int ad = delta < 0 ? -delta : delta;
    sgn = delta < 0 ? -1.f : 1.f;
    if (p.table && ad >= p.table_rows) {
      rope_range = true;
      ad = p.table_rows - 1;
    }
    trow = p.table ? p.table + static_cast<int64_t>(ad) * p.rot_dim : nullptr;
    if (p.vec_rot) load_table_vec<C>(trow, rh8, RH, nrows, ql);
  }

  // Everything above read only the query, the lengths and the rope table, which no kernel that
  // releases its dependents early writes; the side cache and every output wait for the producer.
  wait_for_producer();

  uint64_t pol = 0;
  // Window read: lane 0 of each warp holds the block of the warp's rows in the next tile to be
  // issued (looked up one tile ahead, so that the lookup's latency is off the refill's path).
  int next_blk = -1;
  // Tile t of this cache into stage st: far read by thread 0 (TMA), window read by every thread.
  auto issue = [&](int st, int t) {
    if constexpr (WIN) {
      const int blk = __shfl_sync(0xffffffffu, next_blk, 0);
      if (lane == 0 && t + 1 < t_begin + ntiles)
        next_blk = window_block<C>(p, pos0 + static_cast<int64_t>(t + 1) * TK, seq);
      issue_window_tile<C>(smem, full, st, pos0 + static_cast<int64_t>(t) * TK, seq, h, blk, p);
    } else {
      issue_tile<C>(smem, full, map, st, t, p.hkv, h, pol);
    }
  };
  if (tid == 0) {
    if constexpr (!WIN) {
      if (split == 0 && h == 0) {
        const int far_len = max(hist - p.window - p.block + qlen, 0);
        if (p.far_len) *p.far_len = far_len;
        if (far_len > p.capacity) set_error(p.err, FOLD_DEVERR_CAPACITY);
      }
    }
#pragma unroll
    for (int i = 0; i < NSTAGE; ++i) mbar_init(&full[i], WIN ? NTH : 1);
    fence_mbar_init();
    if constexpr (!WIN) {
      // Fill the ring right away, so the first copies overlap the query rotation below.
      pol = l2_evict_first_policy();
      prefetch_tensormap(map);
      for (int i = 0; i < NSTAGE && i < ntiles; ++i) issue(i, t_begin + i);
    }
  }

  if (rope_range && tid == 0 && split == 0 && h == 0) set_error(p.err, FOLD_DEVERR_ROPE_RANGE);
  if (p.vec_rot) {
    rotate_query_vec<C>(p, ql, rh8, RH, sgn, h, split, nrows, G, Qs);
  } else {
    rotate_query_scalar<C>(p, trow, RH, sgn, h, split, nrows, G, Qs);
  }
  __syncthreads();  // barrier inits and the query tile are visible to every warp
  if constexpr (WIN) {
    if (ntiles > 0) {
      // the first tiles' blocks in one round of loads: lane i looks up tile t_begin + i
      int first = -1;
      if (lane < NSTAGE + 1 && lane < ntiles)
        first = window_block<C>(p, pos0 + static_cast<int64_t>(t_begin + lane) * TK, seq);
      for (int i = 0; i < NSTAGE && i < ntiles; ++i) {
        const int blk = __shfl_sync(0xffffffffu, first, i);
        issue_window_tile<C>(smem, full, i, pos0 + static_cast<int64_t>(t_begin + i) * TK, seq, h, blk, p);
      }
      next_blk = __shfl_sync(0xffffffffu, first, NSTAGE < 31 ? NSTAGE : 31);
    }
  }

  // Warp roles.
  const int mt = warp % MT, ng = warp / MT, nt_lo = ng * QNT;  // QK: key m-tile, n-tile group
  const int hg = warp % C::HG, kg = warp / C::HG;                 // PV: hd group, key group
  const int g4 = lane >> 2, t4 = lane & 3;

  // Query fragments (B operand of S^T = K . Q^T) for this warp's n-tiles.
  uint32_t qfr[C::Q_REGS ? QNT : 1][C::Q_REGS ? HD / 16 : 1][2];
  const uint32_t qs_base = smem_u32(Qs);
  if constexpr (C::Q_REGS) {
#pragma unroll
    for (int j = 0; j < QNT; ++j) {
      const int nt = min(nt_lo + j, NT - 1);
#pragma unroll
      for (int kp = 0; kp < HD / 32; ++kp) {
        const uint32_t a = qs_base + ((nt * 8 + (lane & 7)) * C::QSTRIDE + kp * 32 + (lane >> 3) * 8) * 2;
        ldsm_x4(a, qfr[j][2 * kp][0], qfr[j][2 * kp][1], qfr[j][2 * kp + 1][0], qfr[j][2 * kp + 1][1]);
      }
    }
  }

  // Row limits of this thread's QK rows (global positions; 0 for padding rows): keys
  // [llo, lim) are visible, llo being 0 for the far read.
  int lim[QNT][2];
  int llo[WIN ? QNT : 1][2];
#pragma unroll
  for (int j = 0; j < QNT; ++j)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int rho = (nt_lo + j) * 8 + t4 * 2 + c;
      const bool valid = rho < nrows && nt_lo + j < NT;
      if constexpr (WIN) {
        lim[j][c] = valid ? static_cast<int>(window_hi(p, hist, seq, rho / G)) : 0;
        llo[j][c] = valid ? static_cast<int>(window_lo(p, hist, rho / G)) : 0;
      } else {
        lim[j][c] = valid ? static_cast<int>(min64(lim_base + rho / G, end)) : 0;
      }
    }
  // Far read: the row limits grow with the row, so a tile that ends at or below row 0's limit is
  // visible to every query row. Its logits skip the per-key test; the padding rows of the last
  // n-tile (limit 0) still get -inf (their Q rows are zero, so their products are 0).
  const int64_t open_end = WIN ? 0 : min64(lim_base, end);

  float oacc[PV_MT][NT][4];
#pragma unroll
  for (int a = 0; a < PV_MT; ++a)
#pragma unroll
    for (int b = 0; b < NT; ++b) oacc[a][b][0] = oacc[a][b][1] = oacc[a][b][2] = oacc[a][b][3] = 0.f;
  // Row maxima (log2 domain) of all rows this thread touches in PV; with NG > 1 the QK rows are a
  // subset kept separately (same values, computed from the same shared data).
  // The far read starts them at 0 and its first tile always sets them (below), so they stay
  // finite; the window read starts them at -inf (no maximum yet).
  constexpr float kNoMax = WIN ? -INFINITY : 0.f;
  float mrow[NT][2], mq_own[NG == 1 ? 1 : QNT][2], lq[QNT][2];
#pragma unroll
  for (int b = 0; b < NT; ++b) mrow[b][0] = mrow[b][1] = kNoMax;
#pragma unroll
  for (int j = 0; j < (NG == 1 ? 1 : QNT); ++j) mq_own[j][0] = mq_own[j][1] = kNoMax;
#pragma unroll
  for (int j = 0; j < QNT; ++j) lq[j][0] = lq[j][1] = 0.f;
  auto MQ = [&](int j, int c) -> float& {
    if constexpr (NG == 1) return mrow[j][c];
    else return mq_own[j][c];
  };
  // Logits are kept relative to the row maximum m (0 while a row has none): x * scale_log2 - m in
  // one FFMA, and P = 2^that. The CTA raises a maximum when some relative logit exceeds THR(j, c):
  // kRaise, or -inf while the row has no maximum, so that its first finite logit sets one. The
  // far read needs no per-row threshold: its first tile, which always sets the maxima, holds a
  // visible key of every row that sees any key of the split (a row sees a prefix of the
  // positions). A row without a key in that tile never sees one in the split; its maximum is kept
  // at 0, so every far-read maximum is finite and the bias is -m itself. Padding rows of the far
  // read have zero queries, so logit 0 and P = 1 in open tiles: their columns of P^T and O are
  // never written out.
  float thr[WIN ? QNT : 1][2];
#pragma unroll
  for (int j = 0; j < (WIN ? QNT : 1); ++j) thr[j][0] = thr[j][1] = -INFINITY;
  auto THR = [&](int j, int c) -> float {
    if constexpr (WIN) return thr[j][c];
    else return kRaise;
  };
  auto neg_max = [&](int j, int c) -> float {
    if constexpr (WIN) return MQ(j, c) == -INFINITY ? 0.f : -MQ(j, c);
    else return -MQ(j, c);
  };
  // P of QK n-tile j (keys g4 and g4 + 8, rows t4 * 2 and t4 * 2 + 1) into P^T and the row sums.
  auto write_p = [&](int j, float p0, float p1, float p2, float p3, float (&lsum)[QNT][2], uint32_t pt) {
    const uint32_t pa = pack_f16_sat(p0, p1), pb = pack_f16_sat(p2, p3);
    fadd2(lsum[j][0], lsum[j][1], p0, p1, p2, p3);
    if (nt_lo + j < NT) {
      const int r0 = (nt_lo + j) * 8 + t4 * 2;
      // P^T row of keys g4 and g4 + 8 (fp8: their fragment slots, the order V^T gives keys in)
      const int ka = mt * 16 + (C::FP8 ? fp8_slot(g4) : g4), kb = mt * 16 + (C::FP8 ? fp8_slot(g4 + 8) : g4 + 8);
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(pt + (ka * C::PSTRIDE + r0) * 2), "r"(pa));
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(pt + (kb * C::PSTRIDE + r0) * 2), "r"(pb));
    }
  };
  // P from the relative logits moved by sh[c] (after a raise of the row maxima).
  auto store_p = [&](int j, const float (&sh)[2], float (&xs)[QNT][4], float (&lsum)[QNT][2], uint32_t pt) {
    write_p(j, fast_exp2(xs[j][0] + sh[0]), fast_exp2(xs[j][1] + sh[1]), fast_exp2(xs[j][2] + sh[0]),
            fast_exp2(xs[j][3] + sh[1]), lsum, pt);
  };

  bool timed_out = false;
  int consumed = 0;
  const uint32_t p_base = smem_u32(smem + C::OFF_P);
  // fp8: the K scale of this head multiplies every logit, the V scale the output
  float scale_log2 = p.scale_log2, out_scale = 1.f;
  if constexpr (C::FP8) scale_log2 *= __ldg(p.k_scale + h), out_scale = __ldg(p.v_scale + h);

  // Ring position of the current tile and of the previous one, the current stage's mbarrier
  // phase and the tile's first position, advanced per tile (no division in the loop).
  int st = 0, st_prev = NSTAGE - 1;
  uint32_t phase = 0;
  int64_t tpos = pos0 + static_cast<int64_t>(t_begin) * TK;
  for (int it = 0; it < ntiles; ++it) {
    const bool ok = mbar_wait(&full[st], phase);
    const uint32_t kv_base = smem_u32(smem + st * C::STAGE_BYTES);
    const uint32_t pt = p_base + (it & 1) * (TK * C::PSTRIDE * 2);
    const int64_t key0 = tpos + mt * 16 + g4;

    float x[QNT][4];
    float ls[QNT][2];
    bool exceed = false;
#pragma unroll
    for (int j = 0; j < QNT; ++j) x[j][0] = x[j][1] = x[j][2] = x[j][3] = 0.f, ls[j][0] = ls[j][1] = 0.f;
    if (ok) {
      // ---- S^T = K . Q^T for keys [mt*16, mt*16+16) of the tile
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        uint32_t a0, a1, a2, a3;
        if constexpr (C::FP8) {
          // e4m3 K: byte pairs of keys g4 and g4 + 8, head dims [16 kk + 4 t4, +4) -> f16 pairs
          const int row = mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          uint32_t r0, r1;
          ldsm_x2(kv_base + row * 128 + ((kk ^ (row & 7)) << 4), r0, r1);
          e4m3x4_to_f16(r0, a0, a2);
          e4m3x4_to_f16(r1, a1, a3);
        } else {
          const int row = mt * 16 + (lane & 15);
          const int chunk = (kk & 3) * 2 + (lane >> 4);
          ldsm_x4(kv_base + (kk >> 2) * C::BOX_BYTES + row * 128 + ((chunk ^ (row & 7)) << 4), a0, a1, a2, a3);
        }
#pragma unroll
        for (int j = 0; j < QNT; ++j) {
          if (nt_lo + j < NT) {
            uint32_t b0, b1;
            if constexpr (C::Q_REGS) {
              b0 = qfr[j][kk][0];
              b1 = qfr[j][kk][1];
            } else {
              const uint32_t qa =
                  qs_base + (((nt_lo + j) * 8 + (lane & 7)) * C::QSTRIDE + kk * 16 + ((lane >> 3) & 1) * 8) * 2;
              ldsm_x2(qa, b0, b1);
            }
            if constexpr (C::FP8)
              mma_f16(x[j], a0, a1, a2, a3, b0, b1);
            else
              mma_bf16(x[j], a0, a1, a2, a3, b0, b1);
          }
        }
      }
      // ---- scale, mask, and exponentiate relative to the current row maximum
      if (!WIN && tpos + TK <= open_end) {
        // every key of the tile is visible to every row: one comparison of the thread's largest
        // relative logit against kRaise decides
        float mx = -INFINITY;
#pragma unroll
        for (int j = 0; j < QNT; ++j) {
          // keys g4 and g4 + 8 of the row pair (t4 * 2, t4 * 2 + 1): packed FMAs with the rows' biases
          const float b0 = neg_max(j, 0), b1 = neg_max(j, 1);
          ffma2(x[j][0], x[j][1], scale_log2, b0, b1);
          ffma2(x[j][2], x[j][3], scale_log2, b0, b1);
          mx = fmax3(mx, x[j][0], x[j][1]);
          mx = fmax3(mx, x[j][2], x[j][3]);
        }
        exceed = mx > kRaise;
      } else {
#pragma unroll
        for (int j = 0; j < QNT; ++j) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int c = e & 1;
            const int64_t key = key0 + (e >> 1) * 8;
            bool vis = key < lim[j][c];
            if constexpr (WIN) vis = vis && key >= llo[j][c];
            const float v = vis ? fmaf(x[j][e], scale_log2, neg_max(j, c)) : -INFINITY;
            x[j][e] = v;
            exceed |= v > THR(j, c);
          }
        }
      }
      if (it == 0) {
        exceed = true;  // the first tile always sets the row maxima: skip the provisional P
      } else {
#pragma unroll
        for (int j = 0; j < QNT; ++j)
          write_p(j, fast_exp2(x[j][0]), fast_exp2(x[j][1]), fast_exp2(x[j][2]), fast_exp2(x[j][3]), ls, pt);
      }
    }

    // One barrier per tile: P^T of every warp is written, every warp is done with the previous
    // tile (so its stage may be refilled), and the CTA learns whether any row maximum must move.
    const bool attention = named_bar_or(exceed || !ok, 1, NTH);
    if ((WIN || tid == 0) && it >= 1 && it - 1 + NSTAGE < ntiles) issue(st_prev, t_begin + it - 1 + NSTAGE);
    if (attention) {
      if (named_bar_or(!ok, 2, NTH)) {
        timed_out = true;
        if (lane == 0) set_error(p.err, FOLD_DEVERR_TIMEOUT);
        break;
      }
      // ---- raise the row maximum where a logit passed it by more than 2^kRaise (the shared
      // row maxima are of the logits relative to the old maximum, the same in every warp); the far
      // read's first tile sets every maximum (its accumulators are still zero: factor 1)
      const bool first = !WIN && it == 0;
#pragma unroll
      for (int j = 0; j < QNT; ++j) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float v = fmaxf(x[j][c], x[j][c + 2]);
          v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
          v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
          v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
          if (lane < 4 && nt_lo + j < NT) red[mt * ROWS + (nt_lo + j) * 8 + lane * 2 + c] = v;
        }
      }
      named_bar_sync(2, NTH);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float sh[2];  // old maximum - new maximum (0 while a row has none)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int row = nt * 8 + t4 * 2 + c;
          float tm = red[row];
#pragma unroll
          for (int q = 1; q < MT; ++q) tm = fmaxf(tm, red[q * ROWS + row]);
          const float mo = mrow[nt][c];
          const float meo = mo == -INFINITY ? 0.f : mo;
          tm += meo;
          float mn = tm > mo + kRaise || first ? tm : mo;
          if (!WIN && mn == -INFINITY) mn = 0.f;  // far read: no key of the split for this row
          const float f = mn == -INFINITY || first ? 1.f : fast_exp2(mo - mn);
          mrow[nt][c] = mn;
          sh[c] = meo - (mn == -INFINITY ? 0.f : mn);
#pragma unroll
          for (int a = 0; a < PV_MT; ++a) {
            oacc[a][nt][c] *= f;
            oacc[a][nt][c + 2] *= f;
          }
          if constexpr (NG == 1) {
            lq[nt][c] *= f;
            if constexpr (WIN) thr[nt][c] = mn == -INFINITY ? -INFINITY : kRaise;
          }
        }
        if constexpr (NG == 1) store_p(nt, sh, x, ls, pt);
      }
      if constexpr (NG > 1) {
#pragma unroll
        for (int j = 0; j < QNT; ++j) {
          float sh[2];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int row = min(nt_lo + j, NT - 1) * 8 + t4 * 2 + c;
            float tm = red[row];
#pragma unroll
            for (int q = 1; q < MT; ++q) tm = fmaxf(tm, red[q * ROWS + row]);
            const float mo = mq_own[j][c];
            const float meo = mo == -INFINITY ? 0.f : mo;
            tm += meo;
            float mn = tm > mo + kRaise || first ? tm : mo;
            if (!WIN && mn == -INFINITY) mn = 0.f;
            lq[j][c] *= mn == -INFINITY || first ? 1.f : fast_exp2(mo - mn);
            mq_own[j][c] = mn;
            sh[c] = meo - (mn == -INFINITY ? 0.f : mn);
            if constexpr (WIN) thr[j][c] = mn == -INFINITY ? -INFINITY : kRaise;
          }
          store_p(j, sh, x, ls, pt);
        }
      }
      named_bar_sync(2, NTH);
    }
#pragma unroll
    for (int j = 0; j < QNT; ++j) fadd2(lq[j][0], lq[j][1], lq[j][0], lq[j][1], ls[j][0], ls[j][1]);

    // ---- O^T += V^T . P^T over this warp's hd group and key group
#pragma unroll
    for (int ks = 0; ks < C::PV_KS; ++ks) {
      const int kk = kg * C::PV_KS + ks;
      uint32_t bfr[NT][2];
#pragma unroll
      for (int nt = 0; nt + 1 < NT; nt += 2) {
        const int key = kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
        const int col = (nt + (lane >> 4)) * 8;
        ldsm_x4_t(pt + (key * C::PSTRIDE + col) * 2, bfr[nt][0], bfr[nt][1], bfr[nt + 1][0], bfr[nt + 1][1]);
      }
      if constexpr (NT & 1) {
        const int key = kk * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
        ldsm_x2_t(pt + (key * C::PSTRIDE + (NT - 1) * 8) * 2, bfr[NT - 1][0], bfr[NT - 1][1]);
      }
#pragma unroll
      for (int a = 0; a < PV_MT; ++a) {
        const int ht = hg * PV_MT + a;
        uint32_t a0, a1, a2, a3;
        if constexpr (C::FP8) {
          // e4m3 V^T: byte pairs of head dims g4 and g4 + 8, keys [16 kk + 4 t4, +4) -> f16 pairs
          const int row = ht * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          uint32_t r0, r1;
          ldsm_x2(kv_base + C::BOX_BYTES + row * 128 + ((kk ^ (row & 7)) << 4), r0, r1);
          e4m3x4_to_f16(r0, a0, a2);
          e4m3x4_to_f16(r1, a1, a3);
        } else {
          const int q = lane >> 3;
          const int key_row = kk * 16 + (q >> 1) * 8 + (lane & 7);
          const int chunk = (ht & 3) * 2 + (q & 1);
          ldsm_x4_t(kv_base + (C::KBOX + (ht >> 2)) * C::BOX_BYTES + key_row * 128 + ((chunk ^ (key_row & 7)) << 4),
                    a0, a1, a2, a3);
          a0 = bf16x2_to_f16x2(a0), a1 = bf16x2_to_f16x2(a1), a2 = bf16x2_to_f16x2(a2), a3 = bf16x2_to_f16x2(a3);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma_f16(oacc[a][nt], a0, a1, a2, a3, bfr[nt][0], bfr[nt][1]);
      }
    }
    consumed = it + 1;
    st_prev = st;
    if (++st == NSTAGE) st = 0, phase ^= 1u;
    tpos += TK;
  }

  // -------------------------------------------------------------- epilogue
  // The merge may be scheduled; it waits for this grid to complete. A read that writes the rotated
  // query (qf) releases nothing early: a far read behind it could read qf as its query before its
  // wait.
  if (!p.qf) release_dependents();
  const int64_t o_split = static_cast<int64_t>(split) * p.n * p.hq * HD;
  const int64_t l_split = static_cast<int64_t>(split) * p.hq * p.n;
  if (timed_out) {
    // Copies still in flight must land before this CTA's shared memory is released.
    if constexpr (WIN) {
      cp_async_wait_all();
    } else if (tid == 0) {
      const int issued = min(ntiles, max(consumed, 1) - 1 + NSTAGE);
      for (int i = consumed; i < issued; ++i)
        if (!mbar_wait(&full[i % NSTAGE], (i / NSTAGE) & 1)) break;
    }
    for (int e = tid; e < nrows * HD; e += NTH) {
      const int rho = e / HD, d = e - rho * HD;
      const int r = rho / G, hq = h * G + (rho - r * G);
      p.o_part[o_split + (static_cast<int64_t>(r) * p.hq + hq) * HD + d] = 0.f;
      if (d == 0) p.lse_part[l_split + static_cast<int64_t>(hq) * p.n + r] = -INFINITY;
    }
    return;
  }
  // row sums: lanes sharing t4 hold the same rows
#pragma unroll
  for (int j = 0; j < QNT; ++j)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float v = lq[j][c];
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      if (lane < 4 && nt_lo + j < NT) red[mt * ROWS + (nt_lo + j) * 8 + lane * 2 + c] = v;
    }
  if (warp == 0 && lane < 4) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) row_m[nt * 8 + lane * 2] = mrow[nt][0], row_m[nt * 8 + lane * 2 + 1] = mrow[nt][1];
  }
  // every copy has landed and been consumed: the stage memory holds the O reduction
  float* ored = reinterpret_cast<float*>(smem);
#pragma unroll
  for (int kgi = 0; kgi < C::KG; ++kgi) {
    __syncthreads();
    if (kg == kgi) {
#pragma unroll
      for (int a = 0; a < PV_MT; ++a)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int d = (hg * PV_MT + a) * 16 + g4 + (e >> 1) * 8;
            const int row = nt * 8 + t4 * 2 + (e & 1);
            float* o = ored + row * HD + d;
            *o = kgi == 0 ? oacc[a][nt][e] : *o + oacc[a][nt][e];
          }
    }
  }
  __syncthreads();
  if (tid < ROWS) {
    float L = 0.f;
#pragma unroll
    for (int q = 0; q < MT; ++q) L += red[q * ROWS + tid];
    const float m = row_m[tid];
    row_inv[tid] = L > 0.f ? out_scale / L : 0.f;
    if (tid < nrows) {
      const int r = tid / G, hq = h * G + (tid - r * G);
      p.lse_part[l_split + static_cast<int64_t>(hq) * p.n + r] = L > 0.f ? (m + __log2f(L)) * kLn2 : -INFINITY;
    }
  }
  __syncthreads();
  for (int e = tid; e < nrows * (HD / 4); e += NTH) {
    const int rho = e / (HD / 4), d4 = e - rho * (HD / 4);
    const int r = rho / G, hq = h * G + (rho - r * G);
    const float s = row_inv[rho];
    float4 v = reinterpret_cast<const float4*>(ored + rho * HD)[d4];
    v.x *= s, v.y *= s, v.z *= s, v.w *= s;
    reinterpret_cast<float4*>(p.o_part + o_split + (static_cast<int64_t>(r) * p.hq + hq) * HD)[d4] = v;
  }
}

}  // namespace fold
