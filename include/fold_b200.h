/* C-ABI of the FOLD drafter-attention hot path on B200 (sm_100a).
 *
 * Every entry point takes plain device pointers (owned by the caller), sizes and strides in
 * elements, and a CUDA stream (`stream`, a cudaStream_t passed as void*). None of the step entry
 * points allocates device memory, synchronises the host or reads a device value on the host: the
 * lengths of a draft step (query_start_loc, seq_lens) are read on the device, so every call can be
 * captured in a CUDA graph (the setup calls fold_exchange_create/open/destroy do allocate and
 * synchronise). Each returns FOLD_OK (0) or a fold_status; fold_last_error() gives the detail
 * of the last failure on the calling thread.
 *
 * Conventions (fold/kernels.py:1-13 of the reference): batch 1; qlen = qsl[1] - qsl[0];
 * H = max(seq_lens[0] - qlen, 0) committed entries; W = window; B = block; D = far distance
 * (W + B by default); far_len = max(0, H - W - B + qlen); row r reads the far keys
 * [0, H - W - B + 1 + r). LSE arrays are natural logs laid out [Hq, n] like FlashAttention's;
 * an empty row has lse = -inf and output 0.
 *
 * The side cache keeps the reference's layout side[pages, Hkv, 256, 2*hd] bf16, contiguous, keys
 * before RoPE in [..., :hd] and values in [..., hd:] (fold/attention.py:48,64-66). The last page
 * holds the dummy slot pages*256 - 1 that rows with an invalid slot are written to.
 *
 * Device error word: kernels OR FOLD_DEVERR_* bits into `err` (an int32 in device memory, may be
 * NULL) instead of faulting; the caller reads it when convenient.
 */
#ifndef FOLD_B200_H_
#define FOLD_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum fold_status {
  FOLD_OK = 0,
  FOLD_ERR_INVALID_ARGUMENT = 1, /* a size, stride or option the kernels do not take */
  FOLD_ERR_UNSUPPORTED = 2,      /* a head size / row count without a compiled kernel */
  FOLD_ERR_ALIGNMENT = 3,        /* a pointer or stride breaks the 16-byte vector rule */
  FOLD_ERR_CUDA = 4,             /* a CUDA runtime call failed */
  FOLD_ERR_TENSOR_MAP = 5        /* the TMA descriptor of the side cache could not be built */
};

#define FOLD_DEVERR_APPEND_RANGE 1 /* an append/gather position lies outside the cache */
#define FOLD_DEVERR_ROPE_RANGE 2   /* |rotation offset| beyond the rope table (offset clamped) */
#define FOLD_DEVERR_TIMEOUT 4      /* a pipeline wait of the far read, or a wait for a peer, gave up */
#define FOLD_DEVERR_CAPACITY 8     /* far_len exceeds the side cache's capacity */
#define FOLD_DEVERR_BLOCK_TABLE 16 /* a window-read block-table entry lies outside the paged cache */

const char* fold_status_string(int status);
const char* fold_last_error(void);
int fold_version(void);
/* Number of streaming multiprocessors of the current device (0 if unknown). */
int fold_num_sms(void);

/* Side-cache append. Replaces the scatter of fold/attention.py:260-265
 * (ws.side[pg, :, off, :hd] = raw; ws.side[pg, :, off, hd:] = v).
 * k, v: [ctx, hkv, hd] bf16, innermost dim contiguous, strides (tok, head) in elements.
 * positions, slots: int64[ctx]; a row with slot < 0 goes to the dummy slot pages*256 - 1.
 * pos_lo: first absolute position this cache holds (0 unless the cache is a shard). A row whose
 * position lies outside [pos_lo, pos_lo + (pages-1)*256) is skipped; it sets
 * FOLD_DEVERR_APPEND_RANGE unless `skip_foreign` (a shard skips other ranks' positions). */
int fold_append(const void* k, int64_t k_stride_tok, int64_t k_stride_head, const void* v, int64_t v_stride_tok,
                int64_t v_stride_head, const int64_t* positions, const int64_t* slots, int ctx, void* side,
                int pages, int hkv, int hd, int64_t pos_lo, int skip_foreign, int* err, void* stream);

/* Side-cache append into the fp8 side cache (the storage-format option of the far memory; no
 * reference counterpart: the reference stores the side cache in the KV-cache dtype,
 * fold/attention.py:66). K/V rows as fold_append (bf16, before RoPE), quantised to e4m3 (round to
 * nearest even, saturating at +-448) after division by the per-KV-head scales k_scale, v_scale
 * (float [hkv], device). side8: uint8 [pages][hkv][2][2][128][128]: per (page, head), plane 0
 * holds the K rows of keys [0, 128) and [128, 256) of the page (128 bytes each), plane 1 their V
 * transposed (row = head dim, byte = key). Head size 128 only. Rows with slot < 0 go to the
 * dummy slot (the last position of the last page), as fold_append. */
int fold_append_fp8(const void* k, int64_t k_stride_tok, int64_t k_stride_head, const void* v,
                    int64_t v_stride_tok, int64_t v_stride_head, const int64_t* positions, const int64_t* slots,
                    int ctx, void* side8, int pages, int hkv, int hd, const float* k_scale, const float* v_scale,
                    int64_t pos_lo, int skip_foreign, int* err, void* stream);

/* Read back K and V of absolute positions into k_out, v_out [m, hkv, hd] bf16 (contiguous).
 * The inverse of fold_append for checks and shard moves; no reference counterpart beyond the
 * FlashAttention page read of fold/attention.py:165. */
int fold_gather(const void* side, int pages, int hkv, int hd, int64_t pos_lo, const int64_t* positions, int m,
                void* k_out, void* v_out, int* err, void* stream);

/* Far query. Replaces far_query / _far_query_kernel (fold/kernels.py:21-46,111-119): rotates the
 * RoPE'd block queries q [n, hq, hd] by the angle (D - H) * inv_freq on the first rot_dim dims
 * (neox halves), writes qf [n, hq, hd] bf16 and far_len[0] (may be NULL).
 * rope_table: float32 [table_rows, rot_dim] holding cos(p f_i) then sin(p f_i) for p = 0.. (the
 * layout of vLLM's cos_sin_cache), indexed by |D - H|. */
int fold_far_query(const void* q, int64_t q_stride_tok, int64_t q_stride_head, void* qf, int64_t qf_stride_tok,
                   int64_t qf_stride_head, const int* qsl, const int* seq_lens, const float* rope_table,
                   int table_rows, int rot_dim, int* far_len, int n, int hq, int hd, int window, int block,
                   int far_distance, int* err, void* stream);

/* ReRoPE query pair. Replaces rerope_queries / _rerope_query_kernel (fold/kernels.py:49-83,
 * 122-132): qs = q * max(1, log(H + t + 1) * inv_log_ref) when inv_log_ref > 0, else q;
 * qf = qs rotated by (D - H) (minus t when `constant`). Writes far_len[0] (may be NULL).
 * With qf and rope_table both NULL only qs is written: the ReRoPE query scale of the sliding and
 * native-window layers, replacing logn_scale_rows (fold/attention.py:76-83). */
int fold_rerope_query(const void* q, int64_t q_stride_tok, int64_t q_stride_head, void* qs, int64_t qs_stride_tok,
                      int64_t qs_stride_head, void* qf, int64_t qf_stride_tok, int64_t qf_stride_head,
                      const int* qsl, const int* seq_lens, const float* rope_table, int table_rows, int rot_dim,
                      int* far_len, int n, int hq, int hd, int window, int block, int far_distance, int constant,
                      float inv_log_ref, int* err, void* stream);

/* Far-memory read with the far-query rotation fused in. Replaces the FlashAttention read of the
 * side cache (fold/attention.py:164-170; causal bottom-right, seqused_k = far_len,
 * softmax_scale = alpha * scale, num_splits) together with far_query (fold/attention.py:162).
 * q: RoPE'd queries [n, hq, hd] bf16. With rope_table == NULL, q is used unrotated (it already
 * is the far query, e.g. from fold_rerope_query). The cache holds positions
 * [pos_lo, pos_lo + (pages-1)*256); `capacity` is the total number of positions all shards hold
 * (FOLD_DEVERR_CAPACITY if far_len exceeds it). Each of `splits` CTAs per KV head reads a
 * contiguous range of this cache's far keys and writes a partial (o, lse):
 * o_part [splits, n, hq, hd] float32, lse_part [splits, hq, n] float32 (natural log of the sum of
 * exp(softmax_scale * q.k)). far_len (may be NULL) and qf (may be NULL; [n, hq, hd] bf16 with the
 * given strides) are also written. Supports hd in {128, 256}, rot_dim even <= hd,
 * n * (hq / hkv) <= 64. */
int fold_far_read(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const int* qsl, const int* seq_lens,
                  const float* rope_table, int table_rows, int rot_dim, const void* side, int pages, int64_t pos_lo,
                  int64_t capacity, int* far_len, void* qf, int64_t qf_stride_tok, int64_t qf_stride_head,
                  float* o_part, float* lse_part, int splits, int n, int hq, int hkv, int hd, int window, int block,
                  int far_distance, float softmax_scale, int* err, void* stream);

/* Window (exact-position) read of the paged drafter cache. Replaces the FlashAttention window
 * read of fold/attention.py:148-151,163 (window_size = [W + B - 1, B - 1], causal = False) and of
 * the sliding layers, :211-215 (the native window, causal), with split partials instead of one
 * output. q: RoPE'd queries [n, hq, hd] bf16; row r sits at position p = H + r
 * (FlashAttention's bottom-right alignment, H = seq_lens[0] - qlen) and reads the cached
 * positions j with p - window_left <= j <= p + window_right (a negative bound is unbounded),
 * j <= p when `causal`, and j < seq_lens[0]. k_cache and v_cache are the K and V planes of the
 * paged cache, [num_blocks, hkv, block_size, hd] bf16 with the given strides (elements, multiples
 * of 8; innermost dim contiguous; both planes share them): for vLLM's FlashAttention cache
 * kv[num_blocks, hkv, block_size, 2*hd], k_cache = kv, v_cache = kv + hd. block_table[i] is the
 * cache block of positions [i*block_size, (i+1)*block_size) (block_table_len entries; an entry
 * outside [0, num_blocks) sets FOLD_DEVERR_BLOCK_TABLE). block_size is a multiple of 16. Each of
 * `splits` CTAs per KV head reads a contiguous range of the window and writes a normalised
 * partial: o_part [splits, n, hq, hd], lse_part [splits, hq, n] float32 (natural log of the sum of
 * exp(softmax_scale * q.k); -inf for a split without keys). hd in {128, 256},
 * n * (hq / hkv) <= 64. */
int fold_window_read(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const int* qsl, const int* seq_lens,
                     const void* k_cache, const void* v_cache, int64_t num_blocks, int block_size,
                     int64_t cache_stride_block, int64_t cache_stride_head, int64_t cache_stride_slot,
                     const int* block_table, int block_table_len, int window_left, int window_right, int causal,
                     float softmax_scale, float* o_part, float* lse_part, int splits, int n, int hq, int hkv, int hd,
                     int* err, void* stream);

/* Far-memory read of an fp8 side cache (fold_append_fp8): the work of fold_far_read with the keys
 * and values dequantised by k_scale, v_scale (float [hkv], device): K and V of the side cache are
 * e4m3 (exact in f16), the tiles f16 MMAs with f32 accumulation, the query rotated in float32 and
 * rounded to f16. Half the bytes of the bf16 side cache per key. Head size 128, at most 64 query
 * rows per KV head; no qf output. No reference counterpart (a storage-format option of the far
 * memory, beside fold_far_read). */
int fold_far_read_fp8(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const int* qsl,
                      const int* seq_lens, const float* rope_table, int table_rows, int rot_dim, const void* side8,
                      int pages, int64_t pos_lo, int64_t capacity, int* far_len, const float* k_scale,
                      const float* v_scale, float* o_part, float* lse_part, int splits, int n, int hq, int hkv, int hd,
                      int window, int block, int far_distance, float softmax_scale, int* err, void* stream);

/* The far read and the window read of one draft step in one launch. Replaces, for a full-attention
 * FOLD layer, far_query + both FlashAttention reads of fold/attention.py:162-170. Arguments as
 * fold_far_read (q_far, the rope table, the side cache, far_len, the far partials o_fpart/lse_fpart,
 * far_scale = alpha * scale) and as fold_window_read (q_win, the paged cache, its block table, the
 * window, the window partials o_wpart/lse_wpart, win_scale = scale). `splits` blocks per KV head
 * (at least 2; fold_far_read_default_splits, one block per SM in all, keeps the launch one wave)
 * share the two reads: from the device-side lengths each step picks w, the number that read the
 * window, so that the window read (a few MB) runs beside the far read instead of after it. The
 * window read fills window slots [0, w); the window blocks then read a smaller share of the far
 * tiles than the others (a cost model of the two reads), and every block writes far slot [its
 * index] of partial sets of `splits` slots each. The step stores w in plan[0] (a device int),
 * which fold_merge_partials reads. Shapes whose far read takes the tcgen05 kernel
 * (fold_far_read_kernel_for) fail with FOLD_ERR_UNSUPPORTED: issue fold_far_read and
 * fold_window_read for them. */
int fold_step_read(const void* q_far, int64_t qf_stride_tok, int64_t qf_stride_head, const void* q_win,
                   int64_t qw_stride_tok, int64_t qw_stride_head, const int* qsl, const int* seq_lens,
                   const float* rope_table, int table_rows, int rot_dim, const void* side, int pages, int64_t pos_lo,
                   int64_t capacity, int* far_len, float* o_fpart, float* lse_fpart, const void* k_cache,
                   const void* v_cache, int64_t num_blocks, int block_size, int64_t cache_stride_block,
                   int64_t cache_stride_head, int64_t cache_stride_slot, const int* block_table, int block_table_len,
                   int window_left, int window_right, int causal, float* o_wpart, float* lse_wpart, int splits,
                   int* plan, int n, int hq, int hkv, int hd, int window, int block, int far_distance, float far_scale,
                   float win_scale, int* err, void* stream);

/* Chooses the far-read kernel for later calls: 0 = mma.sync tiles, 1 = tcgen05 tiles with TMEM
 * accumulators, -1 = per shape (the default: tcgen05 above 48 query rows per KV head). Both give
 * the same results within rounding. The environment variable FOLD_FAR_READ_KERNEL=mma|tc sets
 * the initial choice. No reference counterpart (a tuning switch of this implementation). */
int fold_far_read_select_kernel(int kernel);

/* The far-read kernel later calls take for this shape: 0 = mma.sync tiles, 1 = tcgen05 tiles,
 * -1 = invalid sizes. No reference counterpart. */
int fold_far_read_kernel_for(int hd, int n, int hq, int hkv);

/* Split count that fills the device for `hkv` KV heads (one CTA per SM). */
int fold_far_read_default_splits(int hkv, int hd, int n, int hq);

/* LSE merge. Replaces merge / _merge_kernel (fold/kernels.py:86-108,135-142) and absorbs the
 * split-KV combine: o_f holds `splits` far partials (float32 when of_bf16 == 0, else bf16) with
 * strides (split, tok, head), lse_f their LSEs with strides (split, head, tok). Per row t and head:
 * the far partials are combined by log-sum-exp, lf = lse_far * inv_alpha, and when
 * H - W - B + 1 + t > 0 the output is (e^{ll-m} o_l + e^{lf-m} o_f) / (e^{ll-m} + e^{lf-m}),
 * m = max(ll, lf); otherwise it is o_l. o_l [n, hq, hd] bf16, lse_l [hq, n] float32 with the
 * given strides; out bf16 with strides (tok, head). */
int fold_merge(const void* o_l, int64_t ol_stride_tok, int64_t ol_stride_head, const float* lse_l,
               int64_t ll_stride_head, int64_t ll_stride_tok, const void* o_f, int of_bf16, int64_t of_stride_split,
               int64_t of_stride_tok, int64_t of_stride_head, const float* lse_f, int64_t lf_stride_split,
               int64_t lf_stride_head, int64_t lf_stride_tok, int splits, void* out, int64_t out_stride_tok,
               int64_t out_stride_head, const int* qsl, const int* seq_lens, int n, int hq, int hd, int window,
               int block, float inv_alpha, void* stream);

/* LSE merge of two sets of split partials. Replaces merge / _merge_kernel
 * (fold/kernels.py:86-108,135-142) together with both FlashAttention split combines: the window
 * read's wsplits partials (o_wpart [wsplits, n, hq, hd], lse_wpart [wsplits, hq, n], as written
 * by fold_window_read) and the far read's fsplits partials (as written by fold_far_read) are each
 * combined by log-sum-exp, then merged with the alpha weighting of fold_merge. fsplits = 0 (far
 * pointers may then be NULL) writes the combined window read alone (the window ablation and plain
 * sliding layers). `plan` (may be NULL) is fold_step_read's device word: then wsplits == fsplits
 * and the window set uses its first plan[0] slots, the far set all fsplits. All
 * partials float32 and contiguous; out bf16 with strides (tok, head). */
int fold_merge_partials(const float* o_wpart, const float* lse_wpart, int wsplits, const float* o_fpart,
                        const float* lse_fpart, int fsplits, const int* plan, void* out, int64_t out_stride_tok,
                        int64_t out_stride_head, const int* qsl, const int* seq_lens, int n, int hq, int hd,
                        int window, int block, float inv_alpha, void* stream);

/* Log-sum-exp combine of `splits` partials o_part [splits, n, hq, hd], lse_part [splits, hq, n]
 * (float32, contiguous) into one partial o_out [n, hq, hd], lse_out [hq, n]. Used on each rank
 * of a sharded far read before the partials are exchanged; no reference counterpart (the
 * reference runs on one GPU; FlashAttention combines its splits internally). */
int fold_combine(const float* o_part, const float* lse_part, int splits, float* o_out, float* lse_out, int n, int hq,
                 int hd, void* stream);

/* The NCCL data plane of the sequence-sharded far read: each rank's partial, an all-gather over
 * NVLink, then fold_merge. No reference counterpart (the reference runs on one GPU); it replaces
 * the survey's fold_allgather_partials(comm, ...). Combines this rank's split partials o_part
 * [splits, n, hq, hd] / lse_part [splits, hq, n] (as fold_combine) into one record {o [n, hq, hd],
 * lse [hq, n]} in `send` (n*hq*hd + hq*n floats, 16-byte aligned) and all-gathers every rank's
 * record into recv [world][n*hq*hd + hq*n] with ncclAllGather on `comm` (an ncclComm_t of the
 * group, e.g. the communicator of PyTorch's ProcessGroupNCCL) on `stream`. fold_merge then merges
 * the world records with the window read: out_f = recv with split stride n*hq*hd + hq*n, token
 * stride hq*hd, head stride hd; lse_f = recv + n*hq*hd with the same split stride, head stride n,
 * token stride 1. NCCL is looked up at the first call (the libnccl.so.2 already loaded in the
 * process, else the system's); graph-capturable like any NCCL call. */
int fold_allgather_partials(void* comm, const float* o_part, const float* lse_part, int splits, float* send,
                            float* recv, int n, int hq, int hd, void* stream);

/* Far read + merge that allocates nothing, for callers that cannot allocate device memory when
 * they run the draft step (an engine that plans every device buffer ahead of time and passes the
 * attention plugin only the step's tensors, a C runtime without a caching allocator). No
 * counterpart in the reference. The same work as fold_far_read followed by fold_merge, with the
 * split partials kept in a 16 MiB static device array of the library (4 Mi floats per GPU, held
 * on each device from the library's first use there, typically the first kernel call, until
 * process exit; CUDA_MODULE_LOADING=EAGER moves it to context creation) instead of caller
 * memory: requests needing more than
 * splits * n * hq * (hd + 1) = 4194304 floats fail with FOLD_ERR_INVALID_ARGUMENT. The first call
 * on each device looks the array up (cudaGetSymbolAddress); make it before any stream capture.
 * The array is shared by every call on a device and keeps the last call's partials (each call
 * overwrites all it reads), so calls that overlap on the GPU race: issue them on one stream.
 * Arguments as fold_far_read (without qf and the partial buffers) and fold_merge (the window
 * read o_l/lse_l and out). */
int fold_far_read_merge_static(const void* q, int64_t q_stride_tok, int64_t q_stride_head, const int* qsl,
                               const int* seq_lens, const float* rope_table, int table_rows, int rot_dim,
                               const void* side, int pages, int64_t pos_lo, int64_t capacity, int* far_len,
                               const void* o_l, int64_t ol_stride_tok, int64_t ol_stride_head, const float* lse_l,
                               int64_t ll_stride_head, int64_t ll_stride_tok, void* out, int64_t out_stride_tok,
                               int64_t out_stride_head, int splits, int n, int hq, int hkv, int hd, int window,
                               int block, int far_distance, float softmax_scale, float inv_alpha, int* err,
                               void* stream);

/* ---- Sequence-sharded far memory: peer-to-peer exchange of the per-rank partials ----
 *
 * With the side cache partitioned by position across the GPUs of one node (one process per GPU),
 * every rank reads its chunk with fold_far_read and the ranks' partials must be combined. The
 * reference runs on one GPU and has no counterpart; these entry points replace an all-gather of
 * the partials (ncclAllGather) followed by fold_merge with one kernel that combines this rank's
 * splits, stores the result into every rank's receive buffer over NVLink, raises a flag per item,
 * waits for the peers' flags (at most 2 s; then FOLD_DEVERR_TIMEOUT, and later calls on this
 * exchange stop waiting) and merges. Setup is collective: every rank calls fold_exchange_create,
 * the ranks share their handles (any host transport, e.g. an all-gather of the 64-byte handles),
 * and every rank calls fold_exchange_open with all handles in rank order. The exchange allocates
 * its device region at creation; the step itself allocates nothing and is graph-capturable.
 * Every rank must make the same sequence of fold_exchange_merge calls with the same n, hq and hd
 * (one call per layer per draft step); calls on one exchange must be issued in one stream order. */
#define FOLD_EXCHANGE_HANDLE_BYTES 64

/* Creates this rank's exchange on the current device for partials of up to part_floats floats
 * (n*hq*hd + hq*n at the largest step; a multiple of 4) and max_items items (n*hq*ceil(hd/128)).
 * Writes the opaque exchange to *exchange and this rank's FOLD_EXCHANGE_HANDLE_BYTES-byte IPC
 * handle to `handle`. world <= 8. */
int fold_exchange_create(int world, int rank, int64_t part_floats, int max_items, void** exchange, void* handle);

/* Maps the other ranks' regions: `handles` holds world handles of FOLD_EXCHANGE_HANDLE_BYTES
 * bytes, in rank order (this rank's own entry is ignored). */
int fold_exchange_open(void* exchange, const void* handles);

/* Unmaps the peers and frees this rank's region. Call after the last merge has completed on every
 * rank (e.g. after a device synchronisation and a host barrier). */
int fold_exchange_destroy(void* exchange);

/* The step: o_part [splits, n, hq, hd] / lse_part [splits, hq, n] are this rank's far-read
 * partials (float32, contiguous, as written by fold_far_read over this rank's chunk); the window
 * read o_l, lse_l and the output `out` are as in fold_merge. Every rank writes the same merged
 * output. Replaces, on each rank, fold_combine + the all-gather + fold_merge of the partials. */
int fold_exchange_merge(void* exchange, const float* o_part, const float* lse_part, int splits, const void* o_l,
                        int64_t ol_stride_tok, int64_t ol_stride_head, const float* lse_l, int64_t ll_stride_head,
                        int64_t ll_stride_tok, void* out, int64_t out_stride_tok, int64_t out_stride_head,
                        const int* qsl, const int* seq_lens, int n, int hq, int hd, int window, int block,
                        float inv_alpha, int* err, void* stream);

/* The far read and the exchange in one kernel: on every rank, fold_far_read of this rank's chunk
 * followed, in the same cooperative launch, by the work of fold_exchange_merge. Each CTA writes
 * its split partial into o_part/lse_part (as fold_far_read; they stay scratch in L2) and counts it
 * in the exchange's per-KV-head counter. Once every split of its KV head has finished (bounded
 * wait), the head's CTAs share out the head's items: combine the splits, store the item into every
 * peer over NVLink, wait for the peers' records and merge with the window read (o_l, lse_l) into
 * `out`. This saves the separate exchange launch and its ramp. With an exchange of one rank it is
 * the far read and the merge in one launch. Arguments as fold_far_read (without qf) and
 * fold_exchange_merge; every rank passes the same `splits`, and splits * hkv CTAs must fit the
 * device at once (one per SM). When the far read takes the tcgen05 kernel it issues fold_far_read
 * and fold_exchange_merge as two launches. No reference counterpart (the reference runs on one
 * GPU). */
int fold_far_read_exchange(void* exchange, const void* q, int64_t q_stride_tok, int64_t q_stride_head, const int* qsl,
                           const int* seq_lens, const float* rope_table, int table_rows, int rot_dim, const void* side,
                           int pages, int64_t pos_lo, int64_t capacity, int* far_len, float* o_part, float* lse_part,
                           int splits, const void* o_l, int64_t ol_stride_tok, int64_t ol_stride_head,
                           const float* lse_l, int64_t ll_stride_head, int64_t ll_stride_tok, void* out,
                           int64_t out_stride_tok, int64_t out_stride_head, int n, int hq, int hkv, int hd, int window,
                           int block, int far_distance, float softmax_scale, float inv_alpha, int* err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FOLD_B200_H_ */
