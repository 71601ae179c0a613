/*
 * paged_attn_b200.h -- C ABI of the B200 (sm_100a) paged-attention library
 * (libpaged_attn_b200.so).
 *
 * The library replaces the paged-attention hot path of
 * VrajPatel105/paged-inference-engine:
 *   - kernels/flash_attention.py:19-136   flash_attention_kernel (Triton)
 *   - kernels/flash_attention.py:139-172  flash_attention_forward (launcher)
 *   - transformer/model.py:85-122         quantise-on-write of new K/V into the
 *                                          paged INT8 block cache
 *
 * Conventions (all entry points):
 *   - Every pointer is a device pointer unless stated otherwise; strides are in
 *     ELEMENTS; the innermost (head_dim) stride of every tensor must be 1 and
 *     every row must start on a 16-byte boundary.
 *   - The KV pool is addressed as logical [block, slot, head, d] through the
 *     three strides given, exactly as the reference launcher passes
 *     K.stride(0), K.stride(2), K.stride(1) to its kernel
 *     (kernels/flash_attention.py:158-159): for a tensor of shape
 *     [num_blocks, block_size, num_kv_heads, head_dim] that is
 *     (stride(0), stride(1), stride(2)).
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default).
 *   - Nothing allocates.  Outputs and the split-K workspace are owned by the
 *     caller.  Work is enqueued asynchronously on `stream`; the return value
 *     only reports argument / launch errors.  Device-side range problems
 *     (block ids outside the pool, positions beyond the block table) are
 *     skipped by the kernels and OR-ed into *status (PA_STATUS_*) when a
 *     status word is supplied.
 *   - Return value: PA_OK (0) or a negative PA_ERR_* code;
 *     paged_attn_error_string() gives the message of the last failing call on
 *     the calling thread.
 */
#ifndef PAGED_ATTN_B200_H
#define PAGED_ATTN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types. */
enum {
  PA_DTYPE_F16 = 0,
  PA_DTYPE_BF16 = 1,
  PA_DTYPE_I8 = 2,
  PA_DTYPE_F32 = 3
};

/* Return codes. */
enum {
  PA_OK = 0,
  PA_ERR_INVALID = -1,     /* bad argument (shape, stride, alignment, dtype) */
  PA_ERR_UNSUPPORTED = -2, /* valid but not compiled (e.g. head_dim 96)      */
  PA_ERR_WORKSPACE = -3,   /* workspace missing or too small                 */
  PA_ERR_CUDA = -4         /* a CUDA runtime call or launch failed           */
};

/* Device status bits written through the optional status pointer. */
enum {
  PA_STATUS_BAD_BLOCK_ID = 1,
  PA_STATUS_BAD_POSITION = 2,
  PA_STATUS_BAD_NUM_BLOCKS = 4,
  PA_STATUS_BAD_SEQ_INDEX = 8,
  PA_STATUS_PEER_TIMEOUT = 32
};

/*
 * Paged KV pool.  Replaces the cache buffers of transformer/model.py:62-67
 * and the K/V/scale arguments of kernels/flash_attention.py:21-33.
 *   k, v            logical [num_blocks, block_size, num_kv_heads, head_dim]
 *   dtype           PA_DTYPE_F16, PA_DTYPE_BF16, PA_DTYPE_I8 or PA_DTYPE_F32.
 *                   fp32 pools (the reference kernel accepts any float pool,
 *                   kernels/flash_attention.py:79-84) are read by the tiled
 *                   kernel only, rounded to fp16 operands in shared memory
 *                   (TF32's 11-bit significand, the precision of the
 *                   reference's tl.dot); |values| must stay below 65520.
 *                   The split-K decode entry points reject them.
 *   k_scale/v_scale dequantisation scales, required for PA_DTYPE_I8 and
 *                   ignored otherwise.  Per-(token, head) scales use all three
 *                   strides; the reference's per-(block, head) scales
 *                   ([num_blocks, num_kv_heads], kernels/flash_attention.py:73-77)
 *                   use stride_slot = 0.
 *   scale_dtype     PA_DTYPE_F16 or PA_DTYPE_F32
 *   block_size      any power of two
 */
typedef struct {
  void* k;
  void* v;
  int32_t dtype;
  int32_t num_blocks;
  int32_t block_size;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t scale_dtype;
  int64_t k_stride_block, k_stride_slot, k_stride_head;
  int64_t v_stride_block, v_stride_slot, v_stride_head;
  void* k_scale;
  void* v_scale;
  int64_t ks_stride_block, ks_stride_slot, ks_stride_head;
  int64_t vs_stride_block, vs_stride_slot, vs_stride_head;
} pa_kv_cache_t;

/*
 * Per-step paging metadata (kernels/flash_attention.py:27-30, 56-67):
 *   block_table         int32 [num_seqs, bt_cols], physical block ids
 *   num_blocks_per_seq  int32 [num_seqs]
 *   q_len_per_seq       int32 [num_seqs]  query rows of each sequence
 *   kv_len_per_seq      int32 [num_seqs]  keys of each sequence (incl. the new ones)
 */
typedef struct {
  const int32_t* block_table;
  int64_t bt_stride_seq, bt_stride_col;
  int32_t bt_cols;
  int32_t num_seqs;
  const int32_t* num_blocks_per_seq;
  const int32_t* q_len_per_seq;
  const int32_t* kv_len_per_seq;
} pa_paging_t;

/*
 * Attention inputs / outputs (kernels/flash_attention.py:139-150):
 *   q    [num_seqs, num_q_heads, max_q_len, head_dim], PA_DTYPE_F16 or BF16;
 *        num_q_heads must be a multiple of num_kv_heads (grouped-query).
 *   o    fp16, same logical shape as q.  Rows >= q_len_per_seq are not written.
 *   lse  fp16 [num_seqs, num_q_heads, max_q_len] natural-log log-sum-exp of
 *        the scaled logits, or NULL.
 *   softmax_scale   <= 0 selects 1/sqrt(head_dim) (kernels/flash_attention.py:90)
 *   causal_top_left 0: query row m of a sequence sits at absolute position
 *        kv_len - q_len + m (correct for decode and chunked prefill);
 *        1: row m sees keys 0..m, the reference kernel's own mask
 *        (kernels/flash_attention.py:97), kept for bit-for-bit comparisons.
 */
typedef struct {
  const void* q;
  int32_t q_dtype;
  int32_t num_q_heads;
  int32_t max_q_len;
  int32_t causal_top_left;
  int64_t q_stride_seq, q_stride_head, q_stride_row;
  void* o;
  int64_t o_stride_seq, o_stride_head, o_stride_row;
  void* lse;
  int64_t l_stride_seq, l_stride_head, l_stride_row;
  float softmax_scale;
  int32_t _reserved;
} pa_attn_io_t;

/*
 * New K/V rows to append (transformer/model.py:76-92):
 *   k_new, v_new  [num_tokens, num_kv_heads, head_dim], F16 / BF16 / F32
 *   seq_index     int32 [num_tokens]: block-table row of each token
 *                 (pos_seq_id in the reference)
 *   positions     int32 [num_tokens]: absolute position of each token
 *                 (position_ids in the reference)
 */
typedef struct {
  const void* k_new;
  const void* v_new;
  int32_t dtype;
  int32_t num_tokens;
  int64_t k_stride_token, k_stride_head;
  int64_t v_stride_token, v_stride_head;
  const int32_t* seq_index;
  const int32_t* positions;
} pa_kv_new_t;

/*
 * Bytes of split-K workspace paged_attn_forward / paged_attn_decode need for
 * this problem on the current device (0 when the prefill kernel is used).
 */
int paged_attn_workspace_size(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg,
                              size_t* bytes);

/*
 * Paged causal attention forward: replaces flash_attention_forward
 * (kernels/flash_attention.py:139-172).  Chooses the split-K decode kernel
 * when max_q_len * (num_q_heads / num_kv_heads) <= 16, else the prefill
 * kernel.  workspace: >= paged_attn_workspace_size() bytes, 256-byte aligned.
 */
int paged_attn_forward(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg, void* workspace,
                       size_t workspace_bytes, int32_t* status, void* stream);

/*
 * Split-K (flash-decoding) paged attention for short query blocks: the q_len=1
 * grid of kernels/flash_attention.py:38-40,153 with grouped-query packing.
 * Launches the split kernel and its merge kernel on `stream`.
 */
int paged_attn_decode(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg, void* workspace,
                      size_t workspace_bytes, int32_t* status, void* stream);

/*
 * The two launches of paged_attn_decode as separate calls, for a caller that
 * schedules them itself (other work between them, or its own stream order):
 * paged_attn_decode_split runs the split-K kernel, which writes the final
 * output of every (sequence, kv head) segment that one worker covered and
 * leaves fp32 partials (running max, sum, unnormalised O) in `workspace` for
 * the others; paged_attn_reduce then combines those partials into O and LSE
 * (the paged_attn_reduce step of the flash-decoding split; the reference's
 * single kernel, kernels/flash_attention.py:19-136, has no separate reduce).
 * Both calls take the same arguments and the same workspace, and the reduce
 * must run after the split on the same stream (or after an event of it).
 */
int paged_attn_decode_split(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg, void* workspace,
                            size_t workspace_bytes, int32_t* status, void* stream);
int paged_attn_reduce(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg, void* workspace,
                      size_t workspace_bytes, int32_t* status, void* stream);

/*
 * paged_attn_decode without a caller-supplied workspace.  It has no
 * counterpart in the reference.  It is meant for callers that cannot allocate
 * device memory per call: a serving engine that has pre-reserved all of HBM for
 * its KV pool and owns the only allocator, or a host binding (JNI, cgo, a
 * plugin ABI) that has pointers to tensors but no allocator of its own.
 * The split-K partials live in one 24 MiB static device array inside this
 * library, which every GPU that loads the library keeps until the process
 * exits.  Limits: num_seqs <= 8192 and max_q_len * (num_q_heads / num_kv_heads)
 * <= 16 (PA_ERR_UNSUPPORTED otherwise); when the partials of the full
 * persistent grid would not fit, fewer warps per CTA are launched.
 * The first call on each device looks up the array's device address (and may
 * load the library's GPU module), so make that first call before any stream
 * capture.  All calls share the one array: calls that overlap on the GPU (other
 * streams, other threads) race and must be serialised by the caller.  The array
 * keeps the last call's contents; nothing in it needs to start at zero because
 * every call writes each partial before it reads it.
 */
int paged_attn_decode_noalloc(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg,
                              int32_t* status, void* stream);

/*
 * paged_attn_forward over ragged query rows, for callers that keep the rows of
 * all sequences packed instead of padding them to max_q_len (the pad / unpad
 * loops of transformer/model.py:133-141,162-167 and the padded Q of
 * kernels/flash_attention.py:139-150):
 *   q_start       int32 [num_seqs] on the device, first row of each sequence
 *                 (cu_seqlens[:-1]); sequence b owns rows q_start[b] ..
 *                 q_start[b] + q_len_per_seq[b] - 1
 *   total_q_rows  T, the rows of Q / O / L
 * io->q is [T, num_q_heads, head_dim] (io->q_stride_row between rows,
 * io->q_stride_head between heads; q_stride_seq is unused), O likewise and
 * LSE [T, num_q_heads]; io->max_q_len >= every q_len_per_seq[b] sizes the
 * grid.  Rows outside [0, T) are never read or written: a sequence's rows
 * are clamped to T - q_start[b].  Picks the decode or prefill kernel as
 * paged_attn_forward does; the workspace rule is the same.
 */
int paged_attn_varlen(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg, const int32_t* q_start,
                      int32_t total_q_rows, void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/*
 * Head-sharded decode with the output exchange fused into the attention
 * kernels (the NCCL all-gather of head outputs that follows per-GPU decode in
 * a KV-head-sharded engine; the reference runs on one GPU and has none).
 * Each GPU of one box computes its KV heads and stores every finished O row
 * straight into the output buffer of every GPU over NVLink, while its other
 * heads are still being computed; paged_attn_peer_barrier then ends the step.
 *
 * Set-up, once per buffer and GPU (these allocate and map; the attention
 * calls below never do):
 *   paged_attn_peer_alloc   cudaMalloc + zero fill + a 64-byte IPC handle
 *   paged_attn_peer_open    map another process's buffer from its handle
 *   paged_attn_peer_close / paged_attn_peer_free
 * Per step:
 *   paged_attn_decode_peers  as paged_attn_decode, but O goes to o_peers[0..n)
 *       (n <= 8): o_peers[r] points at the same logical position in GPU r's
 *       buffer that io->o gives the layout for (the caller adds its own
 *       head offset); LSE stays local.  Decode shapes only.
 *   paged_attn_peer_barrier  posts `epoch` into slot `rank` of every peer's
 *       int32 flag array and waits until every slot of local_flags holds
 *       `epoch`: after it, this GPU's buffer holds every GPU's rows.  Each
 *       wait gives up after about 0.4 s and sets PA_STATUS_PEER_TIMEOUT.
 * Every GPU must make the same calls with the same epoch (increasing per
 * step), and a buffer must not be written again while a peer still reads the
 * previous step's rows (alternate two buffers).
 */
int paged_attn_peer_alloc(size_t bytes, void** ptr, void* ipc_handle);
int paged_attn_peer_free(void* ptr);
int paged_attn_peer_open(const void* ipc_handle, void** ptr);
int paged_attn_peer_close(void* ptr);
int paged_attn_decode_peers(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg, void* workspace,
                            size_t workspace_bytes, void* const* o_peers, int32_t n_peers, int32_t* status,
                            void* stream);
int paged_attn_peer_barrier(int32_t* local_flags, int32_t* const* peer_flags, int32_t n_peers, int32_t rank,
                            int32_t epoch, int32_t* status, void* stream);

/*
 * Tiled causal paged attention for long query blocks (prefill / chunked
 * prefill): the q_len > 1 grid of kernels/flash_attention.py:19-136.
 */
int paged_attn_prefill(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg, int32_t* status,
                       void* stream);

/*
 * Quantise-on-write of new K/V rows into an INT8 pool: replaces the per-token
 * loop of transformer/model.py:85-122 with one scale per (token, kv head):
 *   absmax = max |x| (fp32), scale = absmax / 127 (fp32; 1.0 when absmax == 0,
 *   tests/pre_quantize_test.py:6-10), q = clamp(round_half_even(x / scale),
 *   -127, 127); the scale is stored in the pool's scale dtype.
 * kv->dtype must be PA_DTYPE_I8 and kv->k_scale / v_scale per-token.
 */
int kv_write_quant(const pa_kv_new_t* nw, const pa_kv_cache_t* kv, const pa_paging_t* pg, int32_t* status,
                   void* stream);

/*
 * K/V projection with the cache write in its epilogue: replaces
 * transformer/model.py:75-82 (k = W_k(x), v = W_v(x), split into heads)
 * followed by the cache write of :85-122.  For every token t and output n of
 * W = [W_k; W_v] (nn.Linear's [out, in] layout, W_k's 2-D rows first):
 *   out[t, n] = sum_c x[t, c] * W[n, c] + bias[n]   (fp32 accumulation)
 * and output n = (kv, head h, d) goes to row (h, d) of token t's slot in the
 * K (kv = 0) or V (kv = 1) pool, through block_table[seq_index[t]]
 * [positions[t] / block_size] -- quantised with one scale per (token, head)
 * exactly as kv_write_quant quantises its input rows for an INT8 pool, or
 * rounded for an F16 / BF16 pool.  The projected rows never exist unpaged in
 * device memory.  One launch on the tensor cores (tcgen05).
 *   x         [num_tokens, d_model], PA_DTYPE_F16 or BF16, row stride x_stride
 *   w         [2 * num_kv_heads * head_dim, d_model], same dtype, row stride w_stride
 *   bias      fp32 [2 * num_kv_heads * head_dim], or NULL
 * Limits: head_dim 128, d_model a positive multiple of 128, rows 16-byte
 * aligned; an INT8 pool needs per-token scales.
 */
typedef struct {
  const void* x;
  const void* w;
  const float* bias;
  int64_t x_stride, w_stride;
  int32_t dtype;
  int32_t num_tokens;
  int32_t d_model;
  int32_t _reserved;
  const int32_t* seq_index;
  const int32_t* positions;
} pa_kv_proj_t;

int kv_project_write(const pa_kv_proj_t* pj, const pa_kv_cache_t* kv, const pa_paging_t* pg, int32_t* status,
                     void* stream);

/*
 * Write of new K/V rows into an F16 / BF16 pool (round-to-nearest-even
 * conversion from the input dtype).  The pool fill of
 * tests/test_flash_attention.py:33-49 as a scatter through the block table.
 */
int kv_write_copy(const pa_kv_new_t* nw, const pa_kv_cache_t* kv, const pa_paging_t* pg, int32_t* status,
                  void* stream);

/*
 * Device-resident block pool: the free list and every sequence's block list
 * kept in device memory and updated in place, replacing the host allocator
 * and the per-step block-table rebuild of the reference:
 *   core/block_manager.py:19-68    BlockManager (allocate / release_blocks)
 *   transformer/model.py:126-152   num_blocks_per_seq + padded int32 table
 *   core/model_runner.py:66-107    per-token positions / sequence rows
 * All arrays are int32 device memory owned by the caller:
 *   free_stack  [num_blocks]   free ids in [0, *free_top); the top is the end
 *   free_top    [1]
 *   table       [max_seqs, table_stride]  block ids of each sequence slot
 *               (row width max_blocks_per_seq <= table_stride)
 *   count       [max_seqs]     blocks of each slot, -1 = no entry
 * A "slot" is the caller's small integer name for a live sequence (the
 * reference keys its dict by seq_id; the host side maps seq_id -> slot).
 */
typedef struct {
  int32_t* free_stack;
  int32_t* free_top;
  int32_t* table;
  int32_t* count;
  int64_t table_stride;
  int32_t num_blocks;
  int32_t max_seqs;
  int32_t max_blocks_per_seq;
  int32_t _reserved;
} pa_block_pool_t;

/* Operation kinds and per-operation results of block_pool_apply
 * (results 0-2 are the values of the reference's AllocStatus,
 * core/block_manager.py:9-12). */
enum { PA_POOL_ALLOCATE = 0, PA_POOL_RELEASE = 1 };
enum {
  PA_POOL_SUCCESS = 0,
  PA_POOL_INSUFFICIENT_SPACE = 1,
  PA_POOL_FAILURE = 2,           /* release of a slot without an entry      */
  PA_POOL_ROW_FULL = 3,          /* allocation past max_blocks_per_seq      */
  PA_POOL_INVALID = 4            /* bad slot, negative count, unknown kind  */
};

/* Fill the free list with 0..num_blocks-1 (list(range(num_blocks)),
 * core/block_manager.py:27) and mark every slot empty. */
int block_pool_init(const pa_block_pool_t* pool, void* stream);

/*
 * Apply n_ops operations in order, ops int32 [n_ops][3] = (kind, slot, n):
 *   PA_POOL_ALLOCATE  pop n ids off the end of the free list and append them
 *                     to the slot's list (creating it), or leave everything
 *                     unchanged with INSUFFICIENT_SPACE when fewer than n are
 *                     free (BlockManager.allocate, core/block_manager.py:29-44)
 *   PA_POOL_RELEASE   push the slot's ids back in list order and remove the
 *                     entry, or FAILURE when the slot has none
 *                     (BlockManager.release_blocks, :47-57)
 * results (int32 [n_ops], device, may be NULL) receives each status.  One
 * launch; ops and results are device pointers.
 */
int block_pool_apply(const pa_block_pool_t* pool, const int32_t* ops, int32_t n_ops, int32_t* results, void* stream);

/*
 * Per-step attention inputs of num_seqs sequences (device arrays):
 *   seq_slot, q_len, kv_len  int32 [num_seqs]; cu_seqlens int32 [num_seqs + 1]
 * writes
 *   block_table  int32 [num_seqs, bt_cols] (row stride bt_stride): each row
 *                the slot's block ids, zero-padded (transformer/model.py:145-152)
 *   num_blocks   int32 [num_seqs]
 *   positions    int32 [total_tokens]: token i of sequence k, at row
 *                cu_seqlens[k] + i, sits at kv_len[k] - q_len[k] + i
 *                (core/model_runner.py:84-85, 96-97); may be NULL
 *   token_seq    int32 [total_tokens]: its row k of block_table (the
 *                seq_index of kv_write_quant); may be NULL
 * A slot without an entry gives an all-zero row and PA_STATUS_BAD_SEQ_INDEX;
 * a slot with more than bt_cols blocks is truncated with
 * PA_STATUS_BAD_NUM_BLOCKS.
 */
int block_pool_step(const pa_block_pool_t* pool, const int32_t* seq_slot, const int32_t* q_len, const int32_t* kv_len,
                    const int32_t* cu_seqlens, int32_t num_seqs, int32_t* block_table, int64_t bt_stride,
                    int32_t bt_cols, int32_t* num_blocks, int32_t* positions, int32_t* token_seq,
                    int32_t total_tokens, int32_t* status, void* stream);

/* Message for the last failing call on this thread ("" if none). */
const char* paged_attn_error_string(void);

/* Library version, e.g. "0.1.0". */
const char* paged_attn_version(void);

#ifdef __cplusplus
}
#endif

#endif /* PAGED_ATTN_B200_H */
