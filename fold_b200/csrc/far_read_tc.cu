// Far read on the fifth-generation tensor cores: tcgen05 MMAs with accumulators in tensor memory
// (TMEM), operands staged in shared memory by TMA.
//
// One CTA per (split, KV head), 10 warps with fixed roles:
//   warp 8 lane 0  TMA producer: streams 32 KB units (128 keys x 128 columns of K or of V) of this
//                  head's side-cache rows into a ring of shared-memory slots;
//   warp 9 lane 0  MMA issuer:   S^T(i) = K(i) . Q^T  into one of two TMEM buffers (M = 128 keys,
//                  N = the n*G query rows padded to 16..64), and O^T += V^T(i-1) . P^T(i-1)
//                  (M = 128 head dims per block, accumulated in TMEM across the whole split);
//   warps 0-7      softmax: warp w reads TMEM lane quarter w % 4 (a thread owns one key of the
//                  tile) and column half w / 4 of S^T, masks, raises the row maxima lazily (as in
//                  the mma.sync kernel), writes its part of P^T to shared memory and keeps
//                  per-thread row sums; at the end they read O^T and write the split's
//                  normalised partial. With four softmax warps (all columns per thread, one warp
//                  per SM sub-partition) the softmax bounded the kernel: 112.7 us at the 128K
//                  Llama shape against 97.8 us for the mma.sync kernel (ncu, same box).
// Shared-memory operand layouts (sm_100 matrix descriptors):
//   K tile   K-major, 128-byte swizzle: exactly what TMA writes (64-column boxes of 128 B rows);
//   Q        K-major, 128-byte swizzle, written by the rotation prologue;
//   V^T      MN-major, 128-byte swizzle: the same TMA boxes read with hd as the M dimension;
//   P^T      MN-major, no swizzle: [row group of 8][key][8 rows] bf16, so each softmax thread
//            stores 16-byte vectors. P is split into a bf16 high part and the bf16 rounding of
//            the rest (two buffers of that layout), and O^T += V^T . P^T takes one MMA for each:
//            P then carries 16 significant bits. A bf16 P alone (8 bits) put its rounding of the
//            weights of a few dominant keys straight into the output, 0.03-0.05 on the x8
//            outlier channels of the 128K Llama workload. The row sums add the same two parts.
// Every mbarrier wait is bounded (FOLD_DEVERR_TIMEOUT); TMEM is freed on every exit path.
#include <cuda_bf16.h>

#include "common.cuh"
#include "far_read.cuh"
#include "host_common.h"
#include "tcgen05.cuh"

namespace fold {
namespace {
using namespace tc;

// Position in the TMA load sequence of unit j (j < KU: K unit, else V unit j-KU) of tile t. The
// sequence is K(0), then per tile b: K(b+1) (when it exists) and V(b), i.e. the order in which the
// MMAs consume them, so a V unit does not sit landed while the softmax of its tile runs.
__device__ __forceinline__ int unit_seq(int t, int j, int ntiles, int KU) {
  const int UPT = 2 * KU;
  if (j < KU) return t == 0 ? j : KU + (t - 1) * UPT + j;
  const int r = j - KU;
  return t + 1 < ntiles ? KU + t * UPT + KU + r : KU + t * UPT + r;
}
// Inverse: tile and unit index of sequence position q.
__device__ __forceinline__ void unit_of(int q, int ntiles, int KU, int& t, int& j) {
  const int UPT = 2 * KU;
  if (q < KU) {
    t = 0, j = q;
    return;
  }
  const int qq = q - KU, b = qq / UPT, r = qq - (qq / UPT) * UPT;
  if (b + 1 < ntiles) {
    if (r < KU) t = b + 1, j = r;
    else t = b, j = r;  // V unit r - KU of tile b
  } else {
    t = b, j = KU + r;
  }
}

template <int HD_, int NP_>
struct TcCfg {
  static constexpr int HD = HD_, NP = NP_, TK = 128;
  static constexpr int KU = HD / 128;  // K units (and V units) per tile
  static constexpr int UPT = 2 * KU;   // units per tile
  static constexpr int BOX_BYTES = TK * 128;
  static constexpr int UNIT_BYTES = 2 * BOX_BYTES;
  // Softmax warps: warp w serves TMEM lane quarter w % 4 (keys of the tile; head dims of O^T)
  // and column half w / 4 (query rows [HALF * (w / 4), HALF * (w / 4 + 1))), so two warps share
  // every quarter of the lanes and each thread handles half of a key's columns.
  static constexpr int NSW = 8;
  static constexpr int NSM = NSW * 32;
  static constexpr int NTHREADS = NSM + 64;
  static constexpr int HALF = NP / 2;
  static constexpr int Q_CHUNK = NP * 128;  // 64 columns of Q, swizzled
  static constexpr int Q_BYTES = (HD / 64) * Q_CHUNK;
  static constexpr int P_HALF = NP * TK * 2;  // one bf16 part of P^T
  static constexpr int P_BYTES = 2 * P_HALF;   // high and low parts
  static constexpr int RED_BYTES = 4 * NP * 4;  // [lane quarter][column]
  static constexpr int ROW_BYTES = 3 * NP * 4;  // row limits, row maxima, rescale factors
  static constexpr int NBAR = 26;
  static constexpr int BASE_FIXED = Q_BYTES + RED_BYTES + ROW_BYTES + NBAR * 8 + 16 + 1024;
  static constexpr int fit(int pbufs) { return (kSmemLimit - BASE_FIXED - pbufs * P_BYTES) / UNIT_BYTES; }
  // Two P^T buffers let the softmax of tile i+1 write while the PV MMAs of tile i read; one buffer
  // is used when it buys another ring slot (more K/V bytes in flight matter more).
  static constexpr int P_BUFS = fit(1) > fit(2) ? 1 : 2;
  static constexpr int NSLOT_FIT = fit(P_BUFS);
  static constexpr int NSLOT = NSLOT_FIT > 8 ? 8 : NSLOT_FIT;
  static constexpr int OFF_Q = NSLOT * UNIT_BYTES;
  static constexpr int OFF_P = OFF_Q + Q_BYTES;
  static constexpr int OFF_RED = OFF_P + P_BUFS * P_BYTES;
  static constexpr int OFF_ROW = OFF_RED + RED_BYTES;
  static constexpr int OFF_BAR = OFF_ROW + ROW_BYTES;
  static constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
  static constexpr int SMEM = OFF_TMEM + 16 + 1024;
  static constexpr int TMEM_O = 0;        // O^T: KU blocks of NP columns
  static constexpr int TMEM_S = KU * NP;  // S^T: 2 buffers of NP columns
  static constexpr int TMEM_NEED = KU * NP + 2 * NP;
  static constexpr int TMEM_COLS = TMEM_NEED <= 32 ? 32 : TMEM_NEED <= 64 ? 64 : TMEM_NEED <= 128 ? 128 : 256;
  static_assert(NP % 16 == 0 && NP >= 16 && NP <= 64, "N of an M=128 MMA: multiple of 16");
  static_assert(HALF % 8 == 0, "a column half is whole groups of 8 rows");
  static_assert(NSLOT >= UPT, "a tile's units must fit the ring");
  static_assert(SMEM <= kSmemLimit, "shared memory budget");
  static_assert(TMEM_NEED <= 256, "TMEM columns");
  static_assert(OFF_BAR % 8 == 0, "mbarrier alignment");
};

// Rotation of the query rows of KV head h into Q (K-major, 128-byte swizzle). Same arithmetic as
// the mma.sync kernel: 16-byte vector loads of each row's neox chunk pairs, all loads of a round
// issued before any arithmetic.
template <class C>
__device__ __forceinline__ void rotate_query_tc(const FarParams& p, const float* trow, int RH, float sgn, int h,
                                                int split, int nrows, int G, unsigned char* qbuf) {
  constexpr int PAIRS = C::HD / 16;
  constexpr int ITEMS = C::NP * PAIRS;
  constexpr int ROUND = 4;
  const int tid = threadIdx.x;
  const int rh8 = trow ? RH / 8 : 0;
  auto chunk_addr = [&](int rho, int c8) {  // 16-byte chunk c8 (8 elements) of row rho
    return qbuf + (c8 >> 3) * C::Q_CHUNK + rho * 128 + (((c8 & 7) ^ (rho & 7)) << 4);
  };
  for (int base = 0; base < ITEMS; base += ROUND * C::NSM) {
    uint4 qa[ROUND], qb[ROUND];
    float4 c0[ROUND], c1[ROUND], s0[ROUND], s1[ROUND];
#pragma unroll
    for (int k = 0; k < ROUND; ++k) {
      const int e = base + tid + k * C::NSM;
      qa[k] = qb[k] = make_uint4(0, 0, 0, 0);
      c0[k] = c1[k] = s0[k] = s1[k] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e < ITEMS) {
        const int rho = e / PAIRS, c = e - (e / PAIRS) * PAIRS;
        if (rho < nrows) {
          const int r = rho / G, hq = h * G + (rho - r * G);
          const __nv_bfloat16* qr = p.q + r * p.q_st + hq * p.q_sh;
          if (c < rh8) {
            qa[k] = __ldg(reinterpret_cast<const uint4*>(qr + 8 * c));
            qb[k] = __ldg(reinterpret_cast<const uint4*>(qr + RH + 8 * c));
            const float4* tc = reinterpret_cast<const float4*>(trow + 8 * c);
            const float4* ts = reinterpret_cast<const float4*>(trow + RH + 8 * c);
            c0[k] = __ldg(tc), c1[k] = __ldg(tc + 1), s0[k] = __ldg(ts), s1[k] = __ldg(ts + 1);
          } else {
            const int off = 2 * RH * (rh8 > 0) + 16 * (c - rh8);
            qa[k] = __ldg(reinterpret_cast<const uint4*>(qr + off));
            qb[k] = __ldg(reinterpret_cast<const uint4*>(qr + off + 8));
          }
        }
      }
    }
#pragma unroll
    for (int k = 0; k < ROUND; ++k) {
      const int e = base + tid + k * C::NSM;
      if (e >= ITEMS) continue;
      const int rho = e / PAIRS, c = e - (e / PAIRS) * PAIRS;
      int off_a, off_b;
      uint4 ya = qa[k], yb = qb[k];
      if (c < rh8) {
        off_a = 8 * c, off_b = RH + 8 * c;
        const float cs[8] = {c0[k].x, c0[k].y, c0[k].z, c0[k].w, c1[k].x, c1[k].y, c1[k].z, c1[k].w};
        const float sn[8] = {s0[k].x, s0[k].y, s0[k].z, s0[k].w, s1[k].x, s1[k].y, s1[k].z, s1[k].w};
        const __nv_bfloat162* xa = reinterpret_cast<const __nv_bfloat162*>(&qa[k]);
        const __nv_bfloat162* xb = reinterpret_cast<const __nv_bfloat162*>(&qb[k]);
        uint32_t* oa = reinterpret_cast<uint32_t*>(&ya);
        uint32_t* ob = reinterpret_cast<uint32_t*>(&yb);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 x = __bfloat1622float2(xa[j]), xp = __bfloat1622float2(xb[j]);
          const float c_0 = cs[2 * j], c_1 = cs[2 * j + 1];
          const float s_0 = sgn * sn[2 * j], s_1 = sgn * sn[2 * j + 1];
          oa[j] = pack_bf16(x.x * c_0 - xp.x * s_0, x.y * c_1 - xp.y * s_1);
          ob[j] = pack_bf16(xp.x * c_0 + x.x * s_0, xp.y * c_1 + x.y * s_1);
        }
      } else {
        off_a = 2 * RH * (rh8 > 0) + 16 * (c - rh8), off_b = off_a + 8;
      }
      *reinterpret_cast<uint4*>(chunk_addr(rho, off_a >> 3)) = ya;
      *reinterpret_cast<uint4*>(chunk_addr(rho, off_b >> 3)) = yb;
      if (p.qf && split == 0 && rho < nrows) {
        const int r = rho / G, hq = h * G + (rho - r * G);
        __nv_bfloat16* o = p.qf + r * p.qf_st + hq * p.qf_sh;
        *reinterpret_cast<uint4*>(o + off_a) = ya;
        *reinterpret_cast<uint4*>(o + off_b) = yb;
      }
    }
  }
}

// Scalar rotation for layouts the vector path does not take.
template <class C>
__device__ __forceinline__ void rotate_query_tc_scalar(const FarParams& p, const float* trow, int RH, float sgn,
                                                       int h, int split, int nrows, int G, unsigned char* qbuf) {
  for (int e = threadIdx.x; e < C::NP * C::HD; e += C::NSM) {
    const int rho = e / C::HD, d = e - (e / C::HD) * C::HD;
    float y = 0.f;
    if (rho < nrows) {
      const int r = rho / G, hq = h * G + (rho - r * G);
      const __nv_bfloat16* qr = p.q + r * p.q_st + hq * p.q_sh;
      const float x = bf2f(qr[d]);
      y = x;
      if (trow && d < 2 * RH) {
        const bool lo = d < RH;
        const int i = lo ? d : d - RH;
        const float xp = bf2f(qr[lo ? d + RH : d - RH]);
        const float c = trow[i], s = sgn * trow[RH + i];
        y = lo ? x * c - xp * s : x * c + xp * s;
      }
      if (p.qf && split == 0) p.qf[r * p.qf_st + hq * p.qf_sh + d] = __float2bfloat16_rn(y);
    }
    const int c8 = d >> 3;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(qbuf + (c8 >> 3) * C::Q_CHUNK + rho * 128 +
                                                          (((c8 & 7) ^ (rho & 7)) << 4)) + (d & 7);
    *dst = __float2bfloat16_rn(y);
  }
}

template <class C>
__global__ void __launch_bounds__(C::NTHREADS, 1)
    far_read_tc_kernel(const __grid_constant__ CUtensorMap map, const FarParams p) {
  constexpr int HD = C::HD, NP = C::NP, TK = C::TK, KU = C::KU, UPT = C::UPT, NSLOT = C::NSLOT, NSM = C::NSM;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
  uint64_t* full = bars;         // [8] unit landed (TMA bytes)
  uint64_t* empty = bars + 8;    // [8] unit consumed by its MMAs
  uint64_t* s_full = bars + 16;  // [2] S^T buffer written
  uint64_t* s_free = bars + 18;  // [2] S^T buffer read by the softmax warps
  uint64_t* p_full = bars + 20;  // [2] P^T written (and O^T rescaled) for the tile
  uint64_t* pv_done = bars + 22; // [2] the PV MMAs of the tile completed
  uint64_t* o_final = bars + 25;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_TMEM);
  float* red = reinterpret_cast<float*>(smem + C::OFF_RED);
  int* lims = reinterpret_cast<int*>(smem + C::OFF_ROW);
  float* rowm = reinterpret_cast<float*>(smem + C::OFF_ROW) + NP;  // running row maxima (log2 units)
  float* rowf = rowm + NP;                                         // factors of the last raise

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int split = blockIdx.x, h = blockIdx.y;
  const int G = p.group, nrows = p.n * G;
  wait_for_producer();

  // Step geometry, from the device-side lengths (fold/kernels.py:24-30).
  const int qlen = p.qsl[1] - p.qsl[0];
  const int hist = max(p.seq[0] - qlen, 0);
  const int far_len = max(hist - p.window - p.block + qlen, 0);
  const int lim_base = hist - p.window - p.block + 1;  // row r reads positions [0, lim_base + r)
  const int64_t end = min64(max(lim_base + p.n - 1, 0), p.pos_lo + p.local_cap);
  const int64_t len = max64(end - p.pos_lo, 0);
  const int tiles = static_cast<int>((len + TK - 1) / TK);
  const int t_begin = static_cast<int>(static_cast<int64_t>(tiles) * split / p.splits);
  const int ntiles = static_cast<int>(static_cast<int64_t>(tiles) * (split + 1) / p.splits) - t_begin;

  // Prologue. The producer warp initialises the mbarriers and starts streaming at once (named
  // barrier 3 releases the other warps once the barriers exist); warp 0 allocates TMEM; the
  // softmax warps rotate the query meanwhile. Named barrier 4 (softmax + MMA warps) then publishes
  // the TMEM address and the finished query tile.
  if (warp == C::NSW) {
    if (lane == 0) {
      if (split == 0 && h == 0) {
        if (p.far_len) *p.far_len = far_len;
        if (far_len > p.capacity) set_error(p.err, FOLD_DEVERR_CAPACITY);
      }
      for (int i = 0; i < NSLOT; ++i) mbar_init(&full[i], 1), mbar_init(&empty[i], 1);
      for (int b = 0; b < 2; ++b) {
        mbar_init(&s_full[b], 1);
        mbar_init(&s_free[b], C::NSW);
        mbar_init(&p_full[b], C::NSW);
        mbar_init(&pv_done[b], 1);
      }
      mbar_init(o_final, 1);
      fence_mbar_init();
    }
    __syncwarp();
    named_bar_arrive(3, C::NTHREADS);
  } else {
    if (warp == 0) {
      tmem_alloc(tmem_slot, C::TMEM_COLS);
      tmem_relinquish();
    }
    if (warp < C::NSW) {
      if (tid < NP) {
        lims[tid] = tid < nrows ? static_cast<int>(min64(lim_base + tid / G, end)) : 0;
        rowm[tid] = -INFINITY;
      }
      const int delta = p.far_distance - hist;
      int ad = delta < 0 ? -delta : delta;
      const float sgn = delta < 0 ? -1.f : 1.f;
      if (p.table && ad >= p.table_rows) {
        if (tid == 0 && split == 0 && h == 0) set_error(p.err, FOLD_DEVERR_ROPE_RANGE);
        ad = p.table_rows - 1;
      }
      const int RH = p.rot_dim >> 1;
      const float* trow = p.table ? p.table + static_cast<int64_t>(ad) * p.rot_dim : nullptr;
      if (p.vec_rot)
        rotate_query_tc<C>(p, trow, RH, sgn, h, split, nrows, G, smem + C::OFF_Q);
      else
        rotate_query_tc_scalar<C>(p, trow, RH, sgn, h, split, nrows, G, smem + C::OFF_Q);
      fence_proxy_async();  // Q is read by the tensor cores
    }
    named_bar_sync(3, C::NTHREADS);  // the mbarriers exist
    tc_fence_before();
    named_bar_sync(4, C::NSM + 32);  // TMEM address, row limits and Q are ready
    tc_fence_after();
  }
  const uint32_t tmem = warp == C::NSW ? 0u : *tmem_slot;  // the producer never touches TMEM

  if (warp == C::NSW) {
    // -------------------------------------------------------------- TMA producer
    if (lane == 0 && ntiles > 0) {
      prefetch_tensormap(&map);
      const uint64_t pol = l2_evict_first_policy();
      const int units = ntiles * UPT;
      int issued = 0;
      for (int u = 0; u < units; ++u) {
        const int slot = u % NSLOT;
        if (u >= NSLOT && !mbar_wait(&empty[slot], ((u / NSLOT) - 1) & 1)) {
          set_error(p.err, FOLD_DEVERR_TIMEOUT);
          break;
        }
        mbar_arrive_expect_tx(&full[slot], C::UNIT_BYTES);
        int ut, uj;
        unit_of(u, ntiles, KU, ut, uj);
        const int64_t lp = static_cast<int64_t>(t_begin + ut) * TK;  // key index in this cache
        const int page = static_cast<int>(lp >> 8), off = static_cast<int>(lp & 255);
        const int c2 = page * p.hkv + h, col = uj * 128;
        unsigned char* dst = smem + slot * C::UNIT_BYTES;
        tma_load_3d(dst, &map, &full[slot], col, off, c2, pol);
        tma_load_3d(dst + C::BOX_BYTES, &map, &full[slot], col + 64, off, c2, pol);
        issued = u + 1;
      }
      for (int u = max(issued - NSLOT, 0); u < issued; ++u)  // copies in flight land before exit
        if (!mbar_wait(&full[u % NSLOT], (u / NSLOT) & 1)) set_error(p.err, FOLD_DEVERR_TIMEOUT);
    }
    __syncwarp();
  } else if (warp == C::NSW + 1) {
    // -------------------------------------------------------------- MMA issuer
    if (lane == 0 && ntiles > 0) {
      bool ok = true;
      constexpr uint32_t idesc_s = idesc_bf16(128, NP, 0, 0);
      constexpr uint32_t idesc_o = idesc_bf16(128, NP, 1, 1);
      const uint32_t q_base = smem_u32(smem + C::OFF_Q);
      const uint32_t p_base = smem_u32(smem + C::OFF_P);
      const uint32_t slot_base = smem_u32(smem);
      for (int i = 0; ok && i <= ntiles; ++i) {
        if (i < ntiles) {
          const int b = i & 1;
          if (i >= 2) ok = mbar_wait(&s_free[b], ((i >> 1) - 1) & 1);
          for (int j = 0; ok && j < KU; ++j) {
            const int u = unit_seq(i, j, ntiles, KU);
            ok = mbar_wait(&full[u % NSLOT], (u / NSLOT) & 1);
          }
          if (!ok) break;
          tc_fence_after();
          const uint32_t d = tmem + C::TMEM_S + b * NP;
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const int u = unit_seq(i, kk >> 3, ntiles, KU);
            const uint32_t a = slot_base + (u % NSLOT) * C::UNIT_BYTES + ((kk & 7) >> 2) * C::BOX_BYTES + (kk & 3) * 32;
            const uint32_t bq = q_base + (kk >> 2) * C::Q_CHUNK + (kk & 3) * 32;
            tc_mma(d, smem_desc(a, 16, 1024, kSwizzle128), smem_desc(bq, 16, 1024, kSwizzle128), idesc_s, kk > 0);
          }
          tc_commit(&s_full[b]);
          for (int j = 0; j < KU; ++j) tc_commit(&empty[unit_seq(i, j, ntiles, KU) % NSLOT]);
        }
        if (i >= 1) {
          const int t = i - 1, b = t & 1;
          ok = mbar_wait(&p_full[b], (t >> 1) & 1);
          for (int j = KU; ok && j < UPT; ++j) {
            const int u = unit_seq(t, j, ntiles, KU);
            ok = mbar_wait(&full[u % NSLOT], (u / NSLOT) & 1);
          }
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int hh = 0; hh < KU; ++hh) {
            const int u = unit_seq(t, KU + hh, ntiles, KU);
            const uint32_t v = slot_base + (u % NSLOT) * C::UNIT_BYTES;
#pragma unroll
            for (int ks = 0; ks < TK / 16; ++ks) {
              const uint64_t vd = smem_desc(v + ks * 2048, C::BOX_BYTES, 1024, kSwizzle128);
              const uint32_t pp = p_base + (t % C::P_BUFS) * C::P_BYTES + ks * 256;
              tc_mma(tmem + C::TMEM_O + hh * NP, vd, smem_desc(pp, 128, TK * 16, kSwizzleNone), idesc_o,
                     (t > 0 || ks > 0));
              tc_mma(tmem + C::TMEM_O + hh * NP, vd, smem_desc(pp + C::P_HALF, 128, TK * 16, kSwizzleNone), idesc_o,
                     1u);
            }
          }
          tc_commit(&pv_done[b]);
          for (int hh = 0; hh < KU; ++hh) tc_commit(&empty[unit_seq(t, KU + hh, ntiles, KU) % NSLOT]);
        }
      }
      if (!ok) set_error(p.err, FOLD_DEVERR_TIMEOUT);
      tc_commit(o_final);  // arrives once every MMA above has completed
    }
    __syncwarp();
  } else {
    // -------------------------------------------------------------- softmax warps
    constexpr int HALF = C::HALF;
    const int q4 = warp & 3, c_lo = (warp >> 2) * HALF;  // lane quarter and first column of this warp
    const int lrow = q4 * 32 + lane;                      // this thread's TMEM lane
    float l[HALF];  // this thread's share of the row sums of its columns
#pragma unroll
    for (int c = 0; c < HALF; ++c) l[c] = 0.f;
    const uint32_t lane_addr = static_cast<uint32_t>(q4 * 32) << 16;
    const uint32_t p_base_gen = C::OFF_P;
    bool timed_out = false;
    bool bad = false;  // a wait of this thread gave up; acted on uniformly at the next barrier
    const int lim_lo = static_cast<int>(min64(lim_base, end));  // smallest row limit

    for (int i = 0; i < ntiles; ++i) {
      const int b = i & 1;
      // tcgen05.ld is warp-collective: the warp takes the tile only if every lane saw it land
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&s_full[b], (i >> 1) & 1));
      float x[HALF];
      if (ok) {
        tc_fence_after();
        tmem_ld_cols<HALF>(tmem + C::TMEM_S + b * NP + c_lo + lane_addr, x);
      } else {
#pragma unroll
        for (int c = 0; c < HALF; ++c) x[c] = -INFINITY;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[b]);

      const int64_t key0 = p.pos_lo + static_cast<int64_t>(t_begin + i) * TK;
      const int64_t key = key0 + lrow;
      const bool clean = key0 + TK <= lim_lo;  // every key of the tile is valid for every row
      bool exceed = i == 0;  // the first tile always sets the row maxima
#pragma unroll
      for (int c = 0; c < HALF; ++c) {
        float v = x[c] * p.scale_log2;
        if (!clean && key >= lims[c_lo + c]) v = -INFINITY;
        x[c] = v;
        exceed |= v > rowm[c_lo + c] + kRaise;
      }
      if (named_bar_or(exceed || !ok || bad, 1, NSM)) {
        if (named_bar_or(!ok || bad, 2, NSM)) {
          timed_out = true;
          if (tid == 0) set_error(p.err, FOLD_DEVERR_TIMEOUT);
          break;
        }
        // ---- raise the row maxima that a logit passed by more than kRaise
#pragma unroll
        for (int c = 0; c < HALF; ++c) {
          float v = x[c];
#pragma unroll
          for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
          if (lane == 0) red[q4 * NP + c_lo + c] = v;
        }
        named_bar_sync(2, NSM);
        if (tid < NP) {  // thread c owns row maximum c
          const float tm = fmaxf(fmaxf(red[tid], red[NP + tid]), fmaxf(red[2 * NP + tid], red[3 * NP + tid]));
          const float mo = rowm[tid];
          const float mn = tm > mo + kRaise ? tm : mo;
          rowf[tid] = mn == -INFINITY ? 1.f : fast_exp2(mo - mn);
          rowm[tid] = mn;
        }
        named_bar_sync(2, NSM);  // new maxima and factors visible; red free again
#pragma unroll
        for (int c = 0; c < HALF; ++c) l[c] *= rowf[c_lo + c];
        if (i >= 1) {
          // O^T holds the PV products up to tile i-1: let them finish, then scale its columns
          if (!mbar_wait(&pv_done[(i - 1) & 1], ((i - 1) >> 1) & 1)) bad = true;
          tc_fence_after();
#pragma unroll
          for (int hh = 0; hh < KU; ++hh) {
#pragma unroll
            for (int c0 = 0; c0 < HALF; c0 += 8) {
              float v[8];
              const uint32_t a = tmem + C::TMEM_O + hh * NP + c_lo + c0 + lane_addr;
              tmem_ld8(a, v);
#pragma unroll
              for (int j = 0; j < 8; ++j) v[j] *= rowf[c_lo + c0 + j];
              tmem_st8(a, v);
            }
          }
        }
      }
      // ---- P^T of this thread's key and columns: 16-byte stores into [row group][key][8 rows],
      // the high bf16 part and the rest in the buffer's two halves
      if (i >= C::P_BUFS) {  // the PV MMAs of tile i - P_BUFS read this buffer
        const int t = i - C::P_BUFS;
        if (!mbar_wait(&pv_done[t & 1], (t >> 1) & 1)) bad = true;
      }
      unsigned char* pb = smem + p_base_gen + (i % C::P_BUFS) * C::P_BYTES + (c_lo / 8) * TK * 16 + lrow * 16;
#pragma unroll
      for (int g = 0; g < HALF / 8; ++g) {
        uint32_t w[4], wl[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = g * 8 + 2 * j;
          const float m0 = rowm[c_lo + c] == -INFINITY ? 0.f : rowm[c_lo + c];
          const float m1 = rowm[c_lo + c + 1] == -INFINITY ? 0.f : rowm[c_lo + c + 1];
          const float p0 = fast_exp2(x[c] - m0), p1 = fast_exp2(x[c + 1] - m1);
          w[j] = pack_bf16(p0, p1);  // high parts
          const float h0 = __uint_as_float(w[j] << 16), h1 = __uint_as_float(w[j] & 0xffff0000u);
          wl[j] = pack_bf16(p0 - h0, p1 - h1);  // the rest, rounded (exact differences)
          l[c] += h0 + __uint_as_float(wl[j] << 16);
          l[c + 1] += h1 + __uint_as_float(wl[j] & 0xffff0000u);
        }
        *reinterpret_cast<uint4*>(pb + g * TK * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(pb + C::P_HALF + g * TK * 16) = make_uint4(wl[0], wl[1], wl[2], wl[3]);
      }
      fence_proxy_async();  // P^T is read by the tensor cores
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
    }
    if (named_bar_or(bad, 2, NSM) && !timed_out) {
      timed_out = true;
      if (tid == 0) set_error(p.err, FOLD_DEVERR_TIMEOUT);
    }

    // -------------------------------------------------------------- epilogue
    if (!p.qf) release_dependents();  // as in split_read: the merge may be scheduled
    // row sums over the 128 keys of each tile position
#pragma unroll
    for (int c = 0; c < HALF; ++c) {
      float v = l[c];
#pragma unroll
      for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[q4 * NP + c_lo + c] = v;
    }
    named_bar_sync(2, NSM);
    const bool landed = ntiles == 0 || mbar_wait(o_final, 0);
    const bool fin = !named_bar_or(!landed || timed_out, 1, NSM);  // uniform: TMEM reads are collective
    if (!landed && tid == 0) set_error(p.err, FOLD_DEVERR_TIMEOUT);
    // thread c turns row c into its reciprocal sum and output offset (lims/rowf are free now)
    int* row_off = lims;
    float* row_inv = rowf;
    if (tid < NP) {
      const float L = red[tid] + red[NP + tid] + red[2 * NP + tid] + red[3 * NP + tid];
      const bool live = fin && L > 0.f && tid < nrows;
      row_inv[tid] = live ? 1.f / L : 0.f;
      const int r = tid / G, hq = h * G + (tid - r * G);
      row_off[tid] = tid < nrows ? (r * p.hq + hq) * HD : -1;
      if (tid < nrows)
        p.lse_part[static_cast<int64_t>(split) * p.hq * p.n + static_cast<int64_t>(hq) * p.n + r] =
            live ? (rowm[tid] + __log2f(L)) * kLn2 : -INFINITY;
    }
    named_bar_sync(2, NSM);
    float inv[HALF];
    int off[HALF];
#pragma unroll
    for (int c = 0; c < HALF; ++c) inv[c] = row_inv[c_lo + c], off[c] = row_off[c_lo + c];
    tc_fence_after();
    // O^T lane = head dim: this thread writes head dim lrow of its rows
    float* __restrict__ out = p.o_part + static_cast<int64_t>(split) * p.n * p.hq * HD + lrow;
#pragma unroll
    for (int hh = 0; hh < KU; ++hh) {
#pragma unroll
      for (int c0 = 0; c0 < HALF; c0 += 8) {
        float v[8];
        if (fin && ntiles > 0) {
          tmem_ld8(tmem + C::TMEM_O + hh * NP + c_lo + c0 + lane_addr, v);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) v[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (off[c0 + j] >= 0) out[off[c0 + j] + hh * 128] = v[j] * inv[c0 + j];
      }
    }
  }

  // -------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <class C>
int launch_tc(const FarParams& prm, const void* side, int pages, bool cached, cudaStream_t stream) {
  CUtensorMap map;
  const int s = cached ? side_tensor_map(side, pages, prm.hkv, C::HD, C::TK, &map)
                       : side_tensor_map_uncached(side, pages, prm.hkv, C::HD, C::TK, &map);
  if (s) return s;
  auto kern = far_read_tc_kernel<C>;
  static std::atomic<uint64_t> configured{0};  // per instantiation, one bit per device
  if (int e = allow_smem(kern, C::SMEM, configured, "cudaFuncSetAttribute(far_read_tc)")) return e;
  return launch_behind(kern, dim3(prm.splits, prm.hkv), C::NTHREADS, C::SMEM, stream, "far_read_tc_kernel", map,
                       prm);
}

template <int HD>
int dispatch_np(int np, const FarParams& prm, const void* side, int pages, bool cached, cudaStream_t stream) {
  switch (np) {
    case 16: return launch_tc<TcCfg<HD, 16>>(prm, side, pages, cached, stream);
    case 32: return launch_tc<TcCfg<HD, 32>>(prm, side, pages, cached, stream);
    case 48: return launch_tc<TcCfg<HD, 48>>(prm, side, pages, cached, stream);
    case 64: return launch_tc<TcCfg<HD, 64>>(prm, side, pages, cached, stream);
    default: return fail(FOLD_ERR_UNSUPPORTED, "far read (tcgen05): n * (hq / hkv) must be at most 64");
  }
}

}  // namespace

int far_read_tc_launch(const FarParams& prm, const void* side, int pages, int hd, int np, bool cached_map,
                       cudaStream_t stream) {
  if (hd == 128) return dispatch_np<128>(np, prm, side, pages, cached_map, stream);
  if (hd == 256) return dispatch_np<256>(np, prm, side, pages, cached_map, stream);
  return fail(FOLD_ERR_UNSUPPORTED, "far read (tcgen05): head size must be 128 or 256");
}

}  // namespace fold
