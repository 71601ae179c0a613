// Internal parameter blocks shared by the C-ABI layer (capi.cu) and the
// kernels.  Plain C structs: pointers, element strides and sizes only.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "paged_attn_b200.h"

namespace pa {

// Element types of the KV pool / Q operand (kernel template tags).
enum : int { KV_F16 = 0, KV_BF16 = 1, KV_I8 = 2, KV_F32 = 3 };
enum : int { Q_F16 = 0, Q_BF16 = 1 };

// Device-side status bits (OR-ed into the optional status word).
enum : int {
  ST_BAD_BLOCK_ID = 1,     // block table entry outside [0, num_pool_blocks)
  ST_BAD_POSITION = 2,     // write position beyond the block table row
  ST_BAD_NUM_BLOCKS = 4,   // num_blocks_per_seq larger than the block table width
  ST_BAD_SEQ_INDEX = 8,    // token -> sequence index outside [0, num_seqs)
  ST_WAIT_TIMEOUT = 16,    // a bounded wait on an asynchronous copy gave up
  ST_PEER_TIMEOUT = 32,    // the cross-GPU barrier gave up waiting for a peer's flag
};
constexpr int kMaxPeers = 8;  // GPUs of one box taking part in a peer output exchange

// TMA descriptors of the K and V pools (4-D maps over [block, slot, head, d]).
struct alignas(64) KvMaps {
  CUtensorMap k;
  CUtensorMap v;
};

struct AttnParams {
  // Q [B, Hq, maxq, D] (head_dim contiguous)
  const void* q;
  long long q_sb, q_sh, q_sm;
  int q_bf16;
  // Ragged rows: when q_start is set, sequence b's rows start at row
  // q_start[b] of Q, O and L, which are packed as [T, Hq, D] / [T, Hq]
  // (q_total = T rows; the per-sequence strides are unused).
  const int* q_start;
  int q_total;
  // KV pool, logical [block, slot, head, d]
  const void* k;
  const void* v;
  long long k_sblk, k_sslot, k_shead;
  long long v_sblk, v_sslot, v_shead;
  // Dequantisation scales (int8 pools); slot stride 0 => one scale per (block, head)
  const void* ks;
  const void* vs;
  long long ks_sblk, ks_sslot, ks_shead;
  long long vs_sblk, vs_sslot, vs_shead;
  int scale_f32;
  // Paging metadata
  const int* bt;
  long long bt_ss, bt_sc;
  int bt_cols;
  const int* nblk;
  const int* qlen;
  const int* kvlen;
  // Outputs: O [B, Hq, maxq, D] fp16, L [B, Hq, maxq] fp16.  With n_peers > 0
  // every O element goes to o_peer[0..n_peers) at its offset from o instead
  // (the same position in each GPU's output buffer, mapped into this process).
  void* o_peer[kMaxPeers];
  int n_peers;
  void* o;
  long long o_sb, o_sh, o_sm;
  void* lse;
  long long l_sb, l_sh, l_sm;
  // Split-K workspace
  float* part_o;
  float* part_ml;
  int* tstart;
  int num_warps_total;  // decode: warps of the persistent grid
  // Shapes
  int B, Hq, Hkv, G, BS, log2BS, NB, maxq;
  float scale_log2;  // softmax scale * log2(e)
  float sm_scale;
  int top_left;
  int* status;
  unsigned int abort_gen;  // launch generation used by bounded waits to stop together
};

struct WriteParams {
  const void* k_new;
  const void* v_new;
  long long kn_st, kn_sh, vn_st, vn_sh;  // [T, Hkv, D] strides (d contiguous)
  int in_dtype;                          // PA_DTYPE_*
  const int* seq_idx;                    // [T] row of the block table
  const int* pos;                        // [T] absolute position in the sequence
  int T;
  const int* bt;
  long long bt_ss, bt_sc;
  int bt_cols, num_seqs;
  void* k;
  void* v;
  long long k_sblk, k_sslot, k_shead;
  long long v_sblk, v_sslot, v_shead;
  int cache_dtype;  // PA_DTYPE_*
  void* ks;
  void* vs;
  long long ks_sblk, ks_sslot, ks_shead;
  long long vs_sblk, vs_sslot, vs_shead;
  int scale_f32;
  int Hkv, D, BS, log2BS, NB;
  int* status;
};

// Device-resident block pool (csrc/block_pool.cu).
enum : int { POOL_ALLOC = 0, POOL_RELEASE = 1 };
enum : int {
  POOL_SUCCESS = PA_POOL_SUCCESS,
  POOL_INSUFFICIENT_SPACE = PA_POOL_INSUFFICIENT_SPACE,
  POOL_FAILURE = PA_POOL_FAILURE,
  POOL_ROW_FULL = PA_POOL_ROW_FULL,
  POOL_INVALID = PA_POOL_INVALID,
};
struct PoolParams {
  int* free_stack;  // [num_blocks]; free ids at [0, *free_top), the top is the end
  int* free_top;
  int* table;       // [max_seqs, table_stride]: block ids of each sequence slot
  int* count;       // [max_seqs]: blocks of each slot, -1 = no entry
  long long table_stride;
  int num_blocks, max_seqs, max_blocks_per_seq;
};
struct StepParams {
  const int* seq_slot;   // [num_seqs] pool slot of each step sequence
  const int* q_len;      // [num_seqs]
  const int* kv_len;     // [num_seqs]
  const int* cu_seqlens; // [num_seqs + 1] first query row of each sequence
  int num_seqs;
  int* block_table;      // [num_seqs, bt_cols] out (row stride bt_stride)
  long long bt_stride;
  int bt_cols;
  int* num_blocks;       // [num_seqs] out
  int* positions;        // [total_tokens] out (may be NULL)
  int* token_seq;        // [total_tokens] out (may be NULL)
  int total_tokens;
  int* status;
};
cudaError_t launch_block_pool_init(const PoolParams& p, cudaStream_t stream);
cudaError_t launch_block_pool_apply(const PoolParams& p, const int* ops, int n_ops, int* results,
                                    cudaStream_t stream);
cudaError_t launch_block_pool_step(const PoolParams& p, const StepParams& s, cudaStream_t stream);

// K/V projection with the cache write in its epilogue (kv_project.cu): the
// destination fields of WriteParams plus the projection's inner dimension and bias.
struct ProjParams : WriteParams {
  int d_model;
  const float* bias;  // [2 * Hkv * D] or NULL
};
cudaError_t launch_kv_project(const ProjParams& p, const CUtensorMap& xmap, const CUtensorMap& wmap, int bf16,
                              cudaStream_t stream);

// Streaming multiprocessors of the current device (cached per device).
int device_sm_count();

// Launchers implemented in the kernel translation units.
cudaError_t launch_kv_write(const WriteParams& p, cudaStream_t stream);
// Decode: persistent grid size (CTAs) for a configuration on the current
// device, warps per CTA, and the launch of the split kernel + merge kernel.
struct DecodeLaunch {
  int ctas;           // persistent CTAs
  int warps_per_cta;  // worker warps per CTA
  size_t smem;        // dynamic shared memory per CTA
};
// use_tma: the pool can be read with TMA boxes (block_size >= 8, maps built).
int decode_plan(int kv_kind, int q_bf16, int D, int nt, int B, int use_tma, DecodeLaunch* out);
// phase: DECODE_BOTH launches the split kernel and the merge kernel,
// DECODE_SPLIT only the split kernel, DECODE_MERGE only the merge kernel (over
// the workspace a DECODE_SPLIT launch with the same problem filled).
enum : int { DECODE_BOTH = 0, DECODE_SPLIT = 1, DECODE_MERGE = 2 };
// Cross-GPU barrier of a peer output exchange: post `epoch` into slot `rank`
// of every peer's flag array, then wait (bounded) until every slot of this
// GPU's array holds `epoch`.
struct PeerFlags {
  int* flag[kMaxPeers];
};
cudaError_t launch_peer_barrier(int* local_flags, const PeerFlags& peers, int n, int rank, int epoch, int* status,
                                cudaStream_t stream);
cudaError_t launch_decode(const AttnParams& p, const KvMaps* maps, int kv_kind, int q_bf16, int D, int nt,
                          const DecodeLaunch& plan, cudaStream_t stream, int phase = DECODE_BOTH);
cudaError_t launch_prefill(const AttnParams& p, int kv_kind, int D, int mma_bf16, cudaStream_t stream);
// INT8 blocks of a prefill call -> fp16 scratch pool (gather: block (b, j) to b * bt_cols + j with the
// matching table written to dbt; mirror: block x to x).
cudaError_t launch_kv_dequant(const AttnParams& p, __half* dk, __half* dv, int* dbt, int gather, int D,
                              cudaStream_t stream);
// tcgen05/TMEM prefill (16-bit pools, head_dim 128, block_size >= 8).
bool prefill_tc_supported(int kv_kind, int D, int BS);
cudaError_t launch_prefill_tc(const AttnParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                              const CUtensorMap& qmap, int kv_kind, cudaStream_t stream);

}  // namespace pa
