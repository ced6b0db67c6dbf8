// Host-side pieces of the split-read launches shared by far_read.cu and far_exchange.cu: the
// argument checks that fill a parameter block, and the dispatch over the compiled row counts.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "far_read.cuh"
#include "host_common.h"
#include "split_read.cuh"

namespace fold {

// Checks the arguments of a far read (those of fold_far_read) and fills its parameter block.
int make_far_params(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const int* qsl, const int* seq_lens,
                    const float* rope_table, int table_rows, int rot_dim, const void* side, int pages, int64_t pos_lo,
                    int64_t capacity, int* far_len, void* qf, int64_t qf_stride_tok, int64_t qf_stride_head,
                    float* o_part, float* lse_part, int splits, int n, int hq, int hkv, int hd, int window, int block,
                    int far_distance, float softmax_scale, int* err, FarParams* out);

// Checks the arguments of a window read (those of fold_window_read) and fills its parameter block.
int make_window_params(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const int* qsl, const int* seq_lens,
                       const void* k_cache, const void* v_cache, int64_t num_blocks, int block_size,
                       int64_t cache_stride_block, int64_t cache_stride_head, int64_t cache_stride_slot,
                       const int* block_table, int block_table_len, int window_left, int window_right, int causal,
                       float softmax_scale, float* o_part, float* lse_part, int splits, int n, int hq, int hkv, int hd,
                       int* err, FarParams* out);

// Calls f.run<FarCfg<HD, nt, TK, HG, FP8, NW>>() for nt in 1..8 (n * G query rows in n8 tiles).
template <int HD, int TK, int HG, class F, bool FP8 = false, int NW = 8>
int with_row_tiles(int nt, const F& f) {
  switch (nt) {
    case 1: return f.template run<FarCfg<HD, 1, TK, HG, FP8, NW>>();
    case 2: return f.template run<FarCfg<HD, 2, TK, HG, FP8, NW>>();
    case 3: return f.template run<FarCfg<HD, 3, TK, HG, FP8, NW>>();
    case 4: return f.template run<FarCfg<HD, 4, TK, HG, FP8, NW>>();
    case 5: return f.template run<FarCfg<HD, 5, TK, HG, FP8, NW>>();
    case 6: return f.template run<FarCfg<HD, 6, TK, HG, FP8, NW>>();
    case 7: return f.template run<FarCfg<HD, 7, TK, HG, FP8, NW>>();
    case 8: return f.template run<FarCfg<HD, 8, TK, HG, FP8, NW>>();
    default: return fail(FOLD_ERR_UNSUPPORTED, "n * (hq / hkv) must be at most 64");
  }
}

// Runs f.run<C>() with the mma.sync configuration of head size hd and n*G rows.
template <class F>
int with_mma_config(int hd, int rows, const F& f) {
  const int nt = (rows + 7) / 8;
  if (hd == 128) return with_row_tiles<128, 128, 4>(nt, f);
  return with_row_tiles<256, 64, 8>(nt, f);
}

}  // namespace fold
