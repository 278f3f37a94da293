/*
 * veda_b200.h -- C ABI of the B200 (sm_100a) Veda sparse-attention library.
 *
 * Every entry point takes plain device pointers, sizes and strides (in
 * elements), plus the CUDA stream to launch on (cudaStream_t passed as
 * void*). Inputs are borrowed, outputs are preallocated by the caller; no
 * entry point allocates memory. Each returns VEDA_OK or an error code whose
 * message is available from veda_last_error() (thread-local).
 *
 * Tensor conventions (the reference's own, miowtion/kernels/fa4.py:38-39):
 *   packed tokens   x[S, H, D]      bf16, D == 128, last dim contiguous
 *   tile-ordered    t[N, H', D]     bf16, N = n_tiles * 128
 *   block mask      m[H', R, n]     uint8 (0/1)
 *   index lists     cnt[H', R] int32, idx[H', R, n] int32 (BlockSparseTensors)
 *
 * Kernels that wait on barriers give up after a bounded time; they then
 * record VEDA_ERR_TIMEOUT in a device status word (veda_device_status) and
 * return early instead of hanging.
 */
#ifndef VEDA_B200_H_
#define VEDA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  VEDA_OK = 0,
  VEDA_ERR_INVALID = 1,      /* argument or shape misuse  -> ValueError */
  VEDA_ERR_UNSUPPORTED = 2,  /* arch / dtype / head_dim   -> NotImplementedError */
  VEDA_ERR_CUDA = 3,         /* CUDA runtime/driver error -> RuntimeError */
  VEDA_ERR_TIMEOUT = 4       /* a device-side wait gave up -> RuntimeError */
};

/* A tiled span of packed rows [start, start + t*h*w) cut into (st,sh,sw)
 * boxes of 128 tokens (miowtion/veda/tiling.py:108-119, TiledSpan). */
typedef struct {
  int64_t start;
  int32_t grid[3];   /* t, h, w */
  int32_t shape[3];  /* tile extents, product 128 */
} veda_span_t;

/* A sparse column block of the video quadrant with its resolved budget
 * (miowtion/veda/mask.py:96-103 ColumnBlock, :68-76 split_budget). */
typedef struct {
  int32_t start;
  int32_t stop;
  int32_t k_lo;
  int32_t k_hi;
  double frac;        /* Bresenham fraction, already rounded to 12 decimals */
  int32_t keeps_all;  /* Budget.keeps_all: every non-empty column is kept */
  int32_t pad_;
} veda_column_block_t;

/* ---- library state ---------------------------------------------------- */

/* Copies the calling thread's last error message into buf (NUL-terminated);
 * returns the last error code. */
int veda_last_error(char* buf, size_t size);

/* Reads (and with reset != 0 clears) the device status word that kernels
 * set when a bounded wait times out. Synchronizes the current device. */
int veda_device_status(int32_t* status, int32_t reset);

/* No counterpart in the reference (it overlaps no communication). Leaves n
 * SMs free of the persistent attention forward (veda_bsa_fwd,
 * veda_bsa_fwd_packed, veda_dense_fwd, veda_bsa_fwd_heat launch at most
 * SMs - n CTAs), so that kernels running beside it, such as NCCL
 * collectives on another stream, find an SM. Process-wide; 0 by default;
 * n in [0, 128]. */
int veda_set_sm_reserve(int32_t n);

/* No counterpart in the reference (a property of this library's forward
 * kernel). How the attention forward's softmax is organised: 2 (default),
 * two groups of warps on alternate key blocks of a query tile, feeding one
 * accumulator with a running reference handed from block to block, and,
 * where every query tile walks the same key tiles (veda_dense_fwd,
 * veda_bsa_fwd_heat), query tiles in pairs that share each key and value
 * tile, one group per tile; 1, one group of warps on every block of one
 * query tile. Both compute the same attention (fp32 summation order
 * differs). Process-wide; returns VEDA_ERR_INVALID for other values. */
int veda_set_fwd_groups(int32_t groups);

/* ---- head-parallel exchange on the copy engines ------------------------- */
/* No counterpart in the reference (it runs one clip per GPU). Plumbing that
 * lets the head-parallel wrapper move its shards between GPUs with the copy
 * engines instead of kernels: the persistent attention holds every SM. */

/* Bytes of a CUDA IPC memory handle. */
#define VEDA_IPC_HANDLE_BYTES 64

/* The IPC handle of the device allocation that holds ptr (which may point
 * inside it, as tensors of a caching allocator do) and ptr's byte offset in
 * it. The peer adds the offset to the base veda_ipc_open returns. */
int veda_ipc_handle(const void* ptr, void* handle, int64_t* offset);

/* Maps another process's allocation (its veda_ipc_handle) into this one,
 * enabling peer access; *base receives its address here. */
int veda_ipc_open(const void* handle, void** base);

/* Unmaps an allocation opened with veda_ipc_open. */
int veda_ipc_close(void* base);

/* Strided device-to-device copy (height rows of width bytes) on the copy
 * engines, asynchronous on `stream`; either side may be another GPU's
 * memory mapped with veda_ipc_open. */
int veda_copy_2d(void* dst, int64_t dst_pitch, const void* src,
                 int64_t src_pitch, int64_t width, int64_t height,
                 void* stream);

/* 1 when the current device is sm_100 (B200) and the library can run. */
int veda_supported_device(void);

/* ---- a1: tile layout -------------------------------------------------- */

/* Replaces miowtion/veda/tiling.py:214-275 (build_tile_layout) for the
 * permutation itself: writes perm[n_tiles*128] (int64, -1 on padding) and
 * valid_count[n_tiles] (int32). n_tiles must equal the sum of the spans'
 * tile counts plus ceil(global rows / 128). */
int veda_build_layout(const veda_span_t* spans, int32_t n_spans,
                      int64_t used, int64_t seq_len, int64_t n_tiles,
                      int64_t* perm, int32_t* valid_count, void* stream);

/* The same permutation in box order, for attention that reads the packed
 * tensors in place (veda_bsa_fwd_packed). Replaces the gather index of
 * miowtion/veda/tiling.py:214-275 on that path: box_perm[n_tiles*128]
 * (int64) holds, for slot `pos` of a video tile, the packed row at position
 * (pos / (sh*sw), (pos / sw) % sh, pos % sw) of the tile's (st, sh, sw) box
 * (-1 outside the grid); global tiles keep perm's prefix order.
 * key_mask[n_tiles*4] (uint32) has bit (slot % 32) of word slot / 32 set
 * for every real row. */
int veda_build_box_layout(const veda_span_t* spans, int32_t n_spans,
                          int64_t used, int64_t seq_len, int64_t n_tiles,
                          int64_t* box_perm, uint32_t* key_mask,
                          void* stream);

/* ---- a2/a3/a12/a14: permutation, pooling, inverse ---------------------- */

/* Replaces miowtion/kernels/tile_gather_triton.py:156-209 (gather_tiles /
 * gather_and_pool) and miowtion/veda/predictor.py:82-168 (pool_tiles):
 *   out[slot, h, :] = x[perm[slot], heads[h], :] (0 where perm < 0)
 *   feats[h, tile, 0:3D] = masked mean | max | min over the tile's prefix
 *   sq[h, tile, :] = E[x^2], var[h, tile, :] = centred Var(x)
 * perm == NULL pools already tile-ordered rows (x is then [N, H', D] and
 * heads == NULL). feats / sq / var may be NULL. */
int veda_gather_pool(const void* x, int64_t x_stride_s, int64_t x_stride_h,
                     const int64_t* perm, const int32_t* valid_count,
                     int64_t n_tiles, const int64_t* heads, int32_t n_heads,
                     void* out, int64_t out_stride_n, int64_t out_stride_h,
                     float* feats, float* sq, float* var, void* stream);

/* veda_gather_pool with the tile-ordered rows written as shared-memory
 * images, the key / value input of veda_bsa_fwd_packed (kv_tile_order 2):
 * image [H', n_tiles, 2, 128, 64] bf16, tile (h, t) a contiguous 32 KB
 * block of two 64-column halves, each 128 rows x 128 bytes whose 16-byte
 * chunk c of row r sits at position c ^ (r % 8) (the 128-byte swizzle a
 * TMA load writes to shared memory). Padding rows are zero. feats as for
 * veda_gather_pool (NULL to skip). */
int veda_gather_pool_images(const void* x, int64_t x_stride_s,
                            int64_t x_stride_h, const int64_t* perm,
                            const int32_t* valid_count, int64_t n_tiles,
                            const int64_t* heads, int32_t n_heads,
                            void* image, float* feats, void* stream);

/* Replaces miowtion/kernels/tile_gather_triton.py:212-224 (scatter_tiles_):
 *   out[perm[slot], heads[h], :] = tiled[slot, h, :] for perm[slot] >= 0. */
int veda_scatter(const void* tiled, int64_t t_stride_n, int64_t t_stride_h,
                 const int64_t* perm, int64_t n_tiles, const int64_t* heads,
                 int32_t n_heads, void* out, int64_t out_stride_s,
                 int64_t out_stride_h, void* stream);

/* No counterpart in the reference (it has no head parallelism). The send /
 * receive layout of the head-parallel all-to-all. The strided side holds,
 * per row, `blocks` segments of seg_bytes at row * row_bytes + b *
 * block_bytes + offset_bytes (one per rank's heads, or a piece of them);
 * the packed side holds them as [block][row][seg_bytes]. pack != 0 copies
 * strided (src) -> packed (dst), pack == 0 packed (src) -> strided (dst).
 * All sizes and offsets multiples of 16 bytes, buffers 16-byte aligned. */
int veda_head_blocks(const void* src, void* dst, int64_t rows,
                     int32_t blocks, int64_t seg_bytes, int64_t row_bytes,
                     int64_t block_bytes, int64_t offset_bytes, int32_t pack,
                     void* stream);

/* Replaces miowtion/veda/attention.py:299-305 (_gather_lse):
 *   out[slot, h] = lse[perm[slot], heads[h]] (0 where perm < 0). */
int veda_gather_lse(const float* lse, int64_t l_stride_s, int64_t l_stride_h,
                    const int64_t* perm, int64_t n_tiles,
                    const int64_t* heads, int32_t n_heads, float* out,
                    void* stream);

/* ---- a4: predictor logits ---------------------------------------------- */

/* Bytes of workspace veda_predict_logits needs; -1 for sizes it rejects
 * (n_heads outside [1, 65535], tile counts negative or above 2^31). */
int64_t veda_predict_workspace(int32_t n_heads, int64_t n_q, int64_t n_k);

/* Replaces miowtion/veda/predictor.py:251-255 + :299-338 (LayerPredictor
 * embed / forward without optional terms), all fp32:
 *   q_hat = feats_q @ proj_q[heads[h]] + mean_q,  k_hat likewise,
 *   logits[h] = q_hat . k_hat^T / sqrt(D).
 * feats_*: [H', n, 3D]; proj_*: [num_heads, 3D, D]; logits: [H', n_q, n_k]. */
int veda_predict_logits(const float* feats_q, const float* feats_k,
                        const float* proj_q, const float* proj_k,
                        const int64_t* heads, int32_t n_heads, int64_t n_q,
                        int64_t n_k, float* logits, void* workspace,
                        int64_t workspace_bytes, void* stream);

/* No counterpart in the reference. veda_predict_logits without a workspace
 * argument, for callers that cannot allocate device memory themselves: a
 * host framework that owns the GPU's memory through its own pool (PyTorch's
 * caching allocator can hold most of HBM, so a plain cudaMalloc fails even
 * though the pool has room), or a plugin interface that hands a kernel only
 * its inputs and outputs. The caller still passes inputs and outputs.
 * Its scratch is a fixed array inside the library of
 * VEDA_PREDICT_NOALLOC_MAX_FLOATS floats (32 MiB), which every GPU that loads
 * the library holds until exit; calls needing more (n_heads * (n_q + n_k) *
 * 128 floats) are rejected with VEDA_ERR_INVALID. The first call on a device
 * looks the array's device address up (cudaGetSymbolAddress) and caches it
 * for the life of the process; make that first call before any stream
 * capture, and do not use the entry point across a cudaDeviceReset (the
 * library's module is then loaded again and the cached address is stale).
 * Every call shares the one array, so
 * calls that overlap on the GPU (e.g. on two streams) race; serialise them.
 * Nothing carries over between calls: every scratch element read is first
 * written by the same call. Calls no cudaMalloc, cudaFree or allocating
 * library routine. */
#define VEDA_PREDICT_NOALLOC_MAX_FLOATS 8388608
int veda_predict_logits_noalloc(const float* feats_q, const float* feats_k,
                                const float* proj_q, const float* proj_k,
                                const int64_t* heads, int32_t n_heads,
                                int64_t n_q, int64_t n_k, float* logits,
                                void* stream);

/* ---- a5-a8: top-k selection, block mask, index lists ------------------- */

/* Replaces miowtion/veda/mask.py:200-285 (select_video_blocks, rule topk),
 * :288-317 (dense_block_mask) and miowtion/kernels/fa4.py:266-296
 * (index_lists, forward direction) in one pass.
 * scores: [H', R, ld_scores] fp32, row i is video query tile rows[i]
 *   (rows == NULL: i itself). Columns [0, n_video) are ranked.
 * global_rows != 0 appends the n - n_video global query rows (R must then be
 *   n_video); they keep every non-empty tile.
 * Outputs (each may be NULL):
 *   mask [H', R_out, n] uint8; lists part/full cnt [H', R_out] and idx
 *   [H', R_out, n] int32 (fill_tails != 0 writes the non-members after the
 *   members, ascending, exactly as the reference's stable argsort does);
 *   sel_index [H', R, K] int64 / sel_keep [H', R, K] uint8 with K = sum of
 *   the blocks' k_hi (keeps_all blocks contribute their width), in the
 *   reference's rank order. Ties rank the lower column first. */
int veda_block_select(const float* scores, int64_t ld_scores,
                      int32_t n_heads, int64_t n_rows, const int64_t* rows,
                      const int32_t* valid_count, int64_t n_tiles,
                      int64_t n_video, const veda_column_block_t* blocks,
                      int32_t n_blocks, int32_t global_rows, uint8_t* mask,
                      int32_t* part_cnt, int32_t* part_idx,
                      int32_t* full_cnt, int32_t* full_idx,
                      int32_t fill_tails, int64_t* sel_index,
                      uint8_t* sel_keep, void* stream);

/* Replaces miowtion/kernels/fa4.py:275-296 (index_lists) for an arbitrary
 * mask [H', R, n] uint8: transpose == 0 gives per-query-tile lists
 * ([H', R, n]); transpose != 0 gives per-key-tile query lists ([H', n, R]),
 * partial iff the key tile is partial. */
int veda_index_lists(const uint8_t* mask, int32_t n_heads, int64_t n_rows,
                     int64_t n_cols, const int32_t* valid_count,
                     int32_t transpose, int32_t* part_cnt, int32_t* part_idx,
                     int32_t* full_cnt, int32_t* full_idx, int32_t fill_tails,
                     void* stream);

/* ---- a9/a11: block-sparse and dense attention forward (tcgen05) --------- */

/* Replaces miowtion/kernels/fa4.py:299-377 (block_sparse_attention,
 * forward) with semantics miowtion/kernels/reference.py:1-10, :23-56:
 *   q [R*128, H', D], k/v [N, H', D] bf16 (head dim contiguous, row stride
 *   multiple of 8 elements, 16-byte aligned), lists as veda_block_select
 *   writes them (idx row stride ld_idx), out [R*128, H', D] bf16,
 *   lse [H', R*128] fp32 (NULL to skip). Query tiles with an empty list
 *   output 0 and lse -inf. */
int veda_bsa_fwd(const void* q, int64_t q_stride_n, int64_t q_stride_h,
                 const void* k, int64_t k_stride_n, int64_t k_stride_h,
                 const void* v, int64_t v_stride_n, int64_t v_stride_h,
                 int32_t n_heads, int64_t n_q_tiles, int64_t n_kv_tiles,
                 const int32_t* valid_count, const int32_t* part_cnt,
                 const int32_t* part_idx, const int32_t* full_cnt,
                 const int32_t* full_idx, int64_t ld_idx, void* out,
                 int64_t out_stride_n, int64_t out_stride_h, float* lse,
                 float softmax_scale, void* stream);

/* The same forward reading the packed tensors in place, for one head group
 * of miowtion/veda/attention.py:724-743: one launch replaces the gather of
 * q (miowtion/veda/tiling.py:278-297), the forward
 * (miowtion/kernels/fa4.py:299-377) and the scatter of the output
 * (miowtion/veda/tiling.py:300-312).
 *   q [S, H, D] bf16 (row stride stride_s, head stride stride_h,
 *   total_heads heads): the video tiles of the spans (at most 2, as given
 *   to veda_build_layout) are read as 5D TMA boxes (t, h, w, head, d), the
 *   layout's global tiles from q_glob [n_global*128, H', D] (tile order,
 *   strides glob_stride_n / glob_stride_h; NULL when n_tiles == n_video);
 *   k, v: with kv_tile_order == 1, tile-ordered [n_tiles*128, H', D]
 *   (strides kv_stride_n / kv_stride_h, as veda_gather_pool writes them);
 *   with kv_tile_order == 2, tile images [H', n_tiles, 32 KB] as
 *   veda_gather_pool_images writes them, each loaded with one bulk copy
 *   (the fastest form; partial tiles in both masked by valid_count); with
 *   kv_tile_order == 0, packed like q and read in place too (global tiles
 *   from k_glob / v_glob, partial tiles masked by key_mask; no copies, but
 *   the 5D loads make the kernel about a third slower);
 *   heads[H'] (device int64): the packed head of each head of the group,
 *   in [0, total_heads) (a head outside reads zeros and writes nothing);
 *   box_perm, key_mask: veda_build_box_layout of the same spans;
 *   lists as for veda_bsa_fwd with rows = all n_tiles query tiles (tile ids
 *   are those of the tile order);
 *   out [S, H, D] (strides out_stride_s, out_stride_h): the rows
 *   box_perm >= 0 of heads[] are written, nothing else.
 * item_order (device int32, NULL for the default order): a work order of
 * order_slots = rounds x order_ctas slots, each h * n_tiles + qt or -1;
 * the kernel then runs order_ctas CTAs, CTA c taking slots c,
 * c + order_ctas, ... (every item exactly once; the order only balances
 * the CTAs' work, the results do not depend on it).
 * Rows of a partial video tile sit in box order rather than as a prefix;
 * the masked softmax is the same, so only the fp32 summation order differs
 * from veda_bsa_fwd. */
int veda_bsa_fwd_packed(const void* q, const void* k, const void* v,
                        int64_t stride_s, int64_t stride_h, int64_t seq_len,
                        int32_t total_heads, int32_t kv_tile_order,
                        int64_t kv_stride_n, int64_t kv_stride_h,
                        const void* q_glob, const void* k_glob,
                        const void* v_glob, int64_t glob_stride_n,
                        int64_t glob_stride_h, const veda_span_t* spans,
                        int32_t n_spans, int64_t n_tiles, int64_t n_video,
                        const int64_t* heads, int32_t n_heads,
                        const int64_t* box_perm, const uint32_t* key_mask,
                        const int32_t* valid_count, const int32_t* part_cnt,
                        const int32_t* part_idx, const int32_t* full_cnt,
                        const int32_t* full_idx, int64_t ld_idx, void* out,
                        int64_t out_stride_s, int64_t out_stride_h,
                        float softmax_scale, const int32_t* item_order,
                        int32_t order_ctas, int64_t order_slots,
                        void* stream);

/* Replaces miowtion/kernels/fa4.py:185-205 (dense_attention) and the
 * row-subset contract of miowtion/h3/attention.py:28-102: full attention of
 * rows [0, used) of q/k/v [S, H, D]; out [S, H, D] (rows >= used are 0),
 * lse [S, H] fp32 natural log (rows >= used are 0; NULL to skip). */
int veda_dense_fwd(const void* q, const void* k, const void* v,
                   int64_t stride_s, int64_t stride_h, int64_t seq_len,
                   int64_t used, int32_t n_heads, void* out,
                   int64_t out_stride_s, int64_t out_stride_h, float* lse,
                   int64_t lse_stride_s, int64_t lse_stride_h,
                   float softmax_scale, void* stream);

/* ---- a10: block-sparse attention backward (tcgen05) ---------------------- */

/* Bytes of device workspace veda_bsa_bwd needs (the per-row D = rowsum(dO*O)
 * and LSE*log2(e), fp32 [2][H'][R*128], then two work-item counters that
 * veda_bsa_bwd zeroes on the stream); -1 for a bad shape. Concurrent calls
 * need separate workspaces. */
int64_t veda_bsa_bwd_workspace(int32_t n_heads, int64_t n_q_tiles);

/* Replaces the backward of miowtion/kernels/fa4.py:299-377 (FA4 through
 * autograd, fa4.py:337-359; reference gradients
 * tests/gpu/test_kernels_gpu.py:200-250): dq, dk, dv of the forward above.
 *   q/k/v/out/dout as in veda_bsa_fwd (out, dout [R*128, H', D]);
 *   lse fp32 natural log as veda_bsa_fwd wrote it, element (row, head) at
 *   lse[row * lse_stride_row + head * lse_stride_h];
 *   the forward lists (per query tile, ld_idx >= n_kv_tiles) and the
 *   transposed lists (per key tile, ld_t_idx >= n_q_tiles) as
 *   veda_index_lists writes them;
 *   dq [R*128, H', D], dk/dv [N, H', D] bf16 outputs (every row written:
 *   rows of tiles without any block get 0);
 *   workspace: veda_bsa_bwd_workspace bytes, 16-byte aligned.
 * Deterministic (no atomics): dq query-major, dk/dv key-major. */
int veda_bsa_bwd(const void* q, int64_t q_stride_n, int64_t q_stride_h,
                 const void* k, int64_t k_stride_n, int64_t k_stride_h,
                 const void* v, int64_t v_stride_n, int64_t v_stride_h,
                 const void* out, int64_t out_stride_n, int64_t out_stride_h,
                 const void* dout, int64_t dout_stride_n,
                 int64_t dout_stride_h, const float* lse,
                 int64_t lse_stride_row, int64_t lse_stride_h,
                 int32_t n_heads, int64_t n_q_tiles, int64_t n_kv_tiles,
                 const int32_t* valid_count, const int32_t* part_cnt,
                 const int32_t* part_idx, const int32_t* full_cnt,
                 const int32_t* full_idx, int64_t ld_idx,
                 const int32_t* t_part_cnt, const int32_t* t_part_idx,
                 const int32_t* t_full_cnt, const int32_t* t_full_idx,
                 int64_t ld_t_idx, void* dq, int64_t dq_stride_n,
                 int64_t dq_stride_h, void* dk, int64_t dk_stride_n,
                 int64_t dk_stride_h, void* dv, int64_t dv_stride_n,
                 int64_t dv_stride_h, float softmax_scale, void* workspace,
                 size_t workspace_bytes, void* stream);

/* ---- a13: teacher block heat (tcgen05) ------------------------------------ */

/* Replaces miowtion/veda/heatmap.py:36-110 (teacher_heat_reference and the
 * Triton kernel it dispatches to, miowtion/kernels/block_heat_triton.py:
 * 140-173): heat [H', n_q, n_tiles] fp32 for query tiles q_tiles[0..n_q)
 * against every key tile. q, k [n_tiles*128, H', D] bf16 tile-ordered; lse
 * the dense teacher's natural-log LSE in tile order, element (slot, head) at
 * lse[slot * lse_stride_row + head * lse_stride_h]. reduce_sum == 0: the
 * block's peak probability exp(max s*scale - L); != 0: its mass
 * sum exp(s*scale - L); s is q.k rounded to bf16; 0 where a tile has no
 * valid row or key. */
int veda_teacher_heat(const void* q, int64_t q_stride_n, int64_t q_stride_h,
                      const void* k, int64_t k_stride_n, int64_t k_stride_h,
                      const float* lse, int64_t lse_stride_row,
                      int64_t lse_stride_h, int32_t n_heads, int64_t n_tiles,
                      const int32_t* valid_count, const int64_t* q_tiles,
                      int64_t n_q, int32_t reduce_sum, float* heat,
                      float softmax_scale, void* stream);

/* ---- (f) fused dense forward + LSE + teacher heat -------------------------- */

/* Workspace bytes veda_bsa_fwd_heat needs (two [n_tiles][128] fp32
 * scratches per SM of the current device). */
int64_t veda_bsa_fwd_heat_workspace(int64_t n_tiles);

/* The fused teacher pass the reference plans in
 * docs/features/veda_kernel.md:285-288: dense attention of one head group in
 * tile order (every query tile against the key tiles of the given lists,
 * normally all non-empty tiles), writing out, the natural-log LSE
 * [H', n_tiles*128] (row stride 1) and the teacher heat [H', n_tiles,
 * n_tiles] of every (query tile, key tile) block in the same pass
 * (miowtion/veda/heatmap.py:36-99 semantics): reduce_sum == 0 gives
 * max_r exp(bf16(max_k q.k) * scale - L_r) (the reference's rounding of the
 * scores, applied to the row maximum, which is the same by monotonicity);
 * reduce_sum != 0 gives sum_r sum_k exp(q.k * scale - L_r) from the fp32
 * scores the softmax already has. Padding query rows contribute nothing;
 * blocks not walked keep whatever heat holds (the caller zeroes it). The
 * lists are those of veda_bsa_fwd with R = n_tiles. With two softmax groups
 * (veda_set_fwd_groups, the default) the pass runs query tiles in pairs
 * (2i, 2i + 1) over the key tiles of tile 2i's lists, so every query tile
 * must have the same lists (all non-empty key tiles, as the teacher passes);
 * with one group each tile walks its own. */
int veda_bsa_fwd_heat(const void* q, int64_t q_stride_n, int64_t q_stride_h,
                      const void* k, int64_t k_stride_n, int64_t k_stride_h,
                      const void* v, int64_t v_stride_n, int64_t v_stride_h,
                      int32_t n_heads, int64_t n_tiles,
                      const int32_t* valid_count, const int32_t* part_cnt,
                      const int32_t* part_idx, const int32_t* full_cnt,
                      const int32_t* full_idx, int64_t ld_idx, void* out,
                      int64_t out_stride_n, int64_t out_stride_h, float* lse,
                      int32_t reduce_sum, float* heat, float softmax_scale,
                      void* workspace, int64_t workspace_bytes, void* stream);

/* ---- (f) tile search: oracle relative error ------------------------------- */

/* Workspace bytes veda_rel_mse needs for n_rows sampled tiles and n_heads. */
int64_t veda_rel_mse_workspace(int64_t n_rows, int32_t n_heads);

/* The error step of the tile-search oracle, miowtion/veda/search.py:117-126
 * (`_oracle_rel_mse_kernels`): per head h,
 *   rel_mse[h] = sum ||o_sparse - o_dense||^2 / max(sum ||o_dense||^2, tiny)
 * over the real rows of the sampled tiles. o_sparse [n_rows*128, H', 128]
 * bf16 is the sparse output of the sampled query tiles (slot r*128 + i);
 * seq_row[slot] is that slot's row in o_dense [S, H, 128] bf16, or -1 for a
 * padding slot (skipped); head h of o_sparse is head heads[h] of o_dense.
 * Deterministic (fixed reduction order). */
int veda_rel_mse(const void* o_sparse, int64_t s_stride_n, int64_t s_stride_h,
                 const void* o_dense, int64_t d_stride_s, int64_t d_stride_h,
                 const int64_t* seq_row, const int64_t* heads, int64_t n_rows,
                 int32_t n_heads, float* rel_mse, void* workspace,
                 int64_t workspace_bytes, void* stream);

/* ---- (f) zero-order compensation ----------------------------------------- */

/* Workspace bytes veda_compensate needs: the bf16 key centroids and value
 * sums of every key tile, [n_pad, H', 128] each, n_pad = n_kv_tiles rounded
 * up to a multiple of 128. */
int64_t veda_compensate_workspace(int32_t n_heads, int64_t n_kv_tiles);

/* Replaces miowtion/kernels/compensation_triton.py:139-226 (`summaries`
 * and `compensate`) and the torch form miowtion/veda/attention.py:591-689
 * (`zero_order_compensation`): every key tile a query tile did not keep
 * (and that has a real row) becomes one virtual key at its centroid mean k
 * with value sum v and weight B_t (its real row count):
 *   out = (o_kept + sum_t p_t vsum_t) / (1 + sum_t p_t B_t),
 *   p_t = exp(q . kmean_t * softmax_scale - L), L = lse_kept of the row
 *   (0 where not finite).
 * o_kept [n_q_tiles*128, H', 128] bf16 and lse_kept [H', n_q_tiles*128]
 * fp32 (row stride 1) are the sparse forward's outputs over the kept tiles,
 * which are given as that forward's index lists (rows = query tiles of q).
 * q [n_q_tiles*128, H', 128], k, v [n_kv_tiles*128, H', 128] bf16 tile
 * ordered, padding slots zero. out may be o_kept (in place). */
int veda_compensate(const void* o_kept, int64_t ok_stride_n,
                    int64_t ok_stride_h, const float* lse_kept, const void* q,
                    int64_t q_stride_n, int64_t q_stride_h, const void* k,
                    int64_t k_stride_n, int64_t k_stride_h, const void* v,
                    int64_t v_stride_n, int64_t v_stride_h, int32_t n_heads,
                    int64_t n_q_tiles, int64_t n_kv_tiles,
                    const int32_t* valid_count, const int32_t* part_cnt,
                    const int32_t* part_idx, const int32_t* full_cnt,
                    const int32_t* full_idx, int64_t ld_idx, void* out,
                    int64_t out_stride_n, int64_t out_stride_h,
                    float softmax_scale, void* workspace,
                    int64_t workspace_bytes, void* stream);

/* ---- diagnostics --------------------------------------------------------- */

/* One 128x128x128 bf16 tcgen05 MMA per mode, for checking operand and
 * accumulator layouts on a new device: mode 0 computes d = a . b^T with a,b
 * K-major in shared memory; mode 1 computes d = a . b with a staged through
 * tensor memory and b MN-major. a, b: [128,128] bf16 row-major; d: [128,128]
 * fp32 row-major. */
int veda_probe_umma(const void* a, const void* b, float* d, int32_t mode,
                    void* stream);

/* Failure-detection check; the reference has no device-side waits and so no
 * counterpart. Launches one CTA of two warps that wait on mbarriers nothing
 * ever completes, through the same bounded wait every kernel here uses:
 * warp 0 with a limit of limit_ns (1 ms .. 4 s), warp 1 with the library's
 * 4 s limit, which it leaves as soon as warp 0 raises the CTA's abort flag.
 * The kernel records VEDA_ERR_TIMEOUT in the device status word and returns;
 * completed[2] (device int32) receives 1 for each warp whose wait completed
 * (0 expected). No fault and no hang: the context stays usable. */
int veda_expire_wait(int64_t limit_ns, int32_t* completed, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VEDA_B200_H_ */
