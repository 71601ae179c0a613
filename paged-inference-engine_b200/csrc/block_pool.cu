// Device-resident block pool: the paged cache's free list and per-sequence
// block lists kept in HBM and updated in place each step, so no host copy of
// the block table exists and nothing is rebuilt from host lists.
//
// Replaces:
//   core/block_manager.py:19-68      BlockManager (LIFO free list, allocate /
//                                    release_blocks), as one ordered batch of
//                                    operations per launch
//   transformer/model.py:126-152     num_blocks_per_seq + the zero-padded
//                                    int32 block table of the step's sequences
//   core/model_runner.py:66-107      per-token positions and sequence rows of
//                                    the step (per-sequence q_len / kv_len /
//                                    row offsets come from the host scheduler)
//
// Integer work, tiny and latency-bound: the operations are applied in order
// by one CTA (each allocation or release moves its ids with all threads
// between two barriers); the step gather runs one CTA per sequence.
#include "pa_common.cuh"

namespace pa {
namespace {

constexpr int kApplyThreads = 256;
constexpr int kStepThreads = 128;

// Free list initialised as list(range(num_blocks)) (core/block_manager.py:27):
// the top of the stack is the end, so the first id handed out is num_blocks - 1.
__global__ void block_pool_init_kernel(int* free_stack, int* free_top, int* count, int num_blocks, int max_seqs) {
  pdl_enter();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < num_blocks) free_stack[i] = i;
  if (i < max_seqs) count[i] = -1;
  if (i == 0) *free_top = num_blocks;
}

// ops[3 i + {0,1,2}] = (kind, slot, n).  Statuses follow AllocStatus
// (core/block_manager.py:9-12): allocate pops n ids off the end of the free
// list (:36-37) and appends them to the slot's list (:39-42), or reports
// INSUFFICIENT_SPACE and changes nothing (:32-33); release pushes the slot's
// ids back in list order (:52-55) and removes the entry, or reports FAILURE
// for a slot without an entry (:49-50).
__global__ void __launch_bounds__(kApplyThreads) block_pool_apply_kernel(const PoolParams p, const int* ops, int n_ops,
                                                                         int* results) {
  pdl_enter();
  __shared__ int s_top;
  if (threadIdx.x == 0) s_top = *p.free_top;
  __syncthreads();
  for (int i = 0; i < n_ops; ++i) {
    const int kind = ops[3 * i];
    const int slot = ops[3 * i + 1];
    const int n = ops[3 * i + 2];
    const int top = s_top;
    int res;
    if (slot < 0 || slot >= p.max_seqs || n < 0 || (kind != POOL_ALLOC && kind != POOL_RELEASE)) {
      res = POOL_INVALID;
    } else {
      int* row = p.table + static_cast<long long>(slot) * p.table_stride;
      const int c = p.count[slot];
      if (kind == POOL_ALLOC) {
        const int base = c < 0 ? 0 : c;
        if (top < n) {
          res = POOL_INSUFFICIENT_SPACE;
        } else if (base + n > p.max_blocks_per_seq) {
          res = POOL_ROW_FULL;
        } else {
          for (int j = threadIdx.x; j < n; j += blockDim.x) row[base + j] = p.free_stack[top - 1 - j];
          res = POOL_SUCCESS;
        }
        __syncthreads();  // every thread has read count / the stack before they change
        if (res == POOL_SUCCESS && threadIdx.x == 0) {
          p.count[slot] = base + n;
          s_top = top - n;
        }
      } else {
        if (c < 0) {
          res = POOL_FAILURE;
        } else if (top + c > p.num_blocks || c > p.max_blocks_per_seq) {
          res = POOL_INVALID;  // inconsistent state: never written past the arrays
        } else {
          for (int j = threadIdx.x; j < c; j += blockDim.x) p.free_stack[top + j] = row[j];
          res = POOL_SUCCESS;
        }
        __syncthreads();
        if (res == POOL_SUCCESS && threadIdx.x == 0) {
          p.count[slot] = -1;
          s_top = top + c;
        }
      }
    }
    if (threadIdx.x == 0 && results) results[i] = res;
    __syncthreads();  // the next operation sees this one's stack, counts and rows
  }
  if (threadIdx.x == 0) *p.free_top = s_top;
}

// One CTA per step sequence k: the padded block-table row (zeros past the
// sequence's blocks, transformer/model.py:145-152), its block count and the
// position / row index of each of its query tokens.  Token i of sequence k
// sits at row cu_seqlens[k] + i and absolute position kv_len[k] - q_len[k] + i
// (core/model_runner.py:84-85 for prefill, :96-97 for decode).
__global__ void __launch_bounds__(kStepThreads) block_pool_step_kernel(const PoolParams p, const StepParams s) {
  pdl_enter();
  for (int k = blockIdx.x; k < s.num_seqs; k += gridDim.x) {
    const int slot = s.seq_slot[k];
    const bool ok = slot >= 0 && slot < p.max_seqs;
    int c = ok ? p.count[slot] : -1;
    if (!ok || c < 0) {
      if (threadIdx.x == 0) set_status(s.status, ST_BAD_SEQ_INDEX);
      c = 0;
    }
    if (c > s.bt_cols) {
      if (threadIdx.x == 0) set_status(s.status, ST_BAD_NUM_BLOCKS);
      c = s.bt_cols;
    }
    const int* src = ok ? p.table + static_cast<long long>(slot) * p.table_stride : nullptr;
    int* dst = s.block_table + static_cast<long long>(k) * s.bt_stride;
    for (int j = threadIdx.x; j < s.bt_cols; j += blockDim.x) dst[j] = j < c ? src[j] : 0;
    if (threadIdx.x == 0) s.num_blocks[k] = c;
    const int q0 = s.cu_seqlens[k];
    const int ql = s.q_len[k];
    const int first = s.kv_len[k] - ql;
    for (int i = threadIdx.x; i < ql; i += blockDim.x) {
      const int t = q0 + i;
      if (t < 0 || t >= s.total_tokens) {
        set_status(s.status, ST_BAD_POSITION);
        continue;
      }
      if (s.positions) s.positions[t] = first + i;
      if (s.token_seq) s.token_seq[t] = k;
    }
  }
}

}  // namespace

cudaError_t launch_block_pool_init(const PoolParams& p, cudaStream_t stream) {
  const int n = p.num_blocks > p.max_seqs ? p.num_blocks : p.max_seqs;
  const int blocks = (n + 255) / 256 > 0 ? (n + 255) / 256 : 1;
  cudaError_t e = launch_pdl(block_pool_init_kernel, dim3(blocks), dim3(256), 0, stream, p.free_stack, p.free_top,
                             p.count, p.num_blocks, p.max_seqs);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_block_pool_apply(const PoolParams& p, const int* ops, int n_ops, int* results,
                                    cudaStream_t stream) {
  if (n_ops <= 0) return cudaSuccess;
  cudaError_t e = launch_pdl(block_pool_apply_kernel, dim3(1), dim3(kApplyThreads), 0, stream, p, ops, n_ops, results);
  return e != cudaSuccess ? e : cudaGetLastError();
}

cudaError_t launch_block_pool_step(const PoolParams& p, const StepParams& s, cudaStream_t stream) {
  if (s.num_seqs <= 0) return cudaSuccess;
  const int grid = s.num_seqs < 4 * 148 ? s.num_seqs : 4 * 148;
  cudaError_t e = launch_pdl(block_pool_step_kernel, dim3(grid), dim3(kStepThreads), 0, stream, p, s);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace pa
