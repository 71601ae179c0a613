// Dequantisation of the INT8 blocks a prefill call reads into an fp16 scratch
// pool, so that the tcgen05 prefill kernel streams fp16 tiles through TMA.
//
// The reference dequantises inside its attention loop
// (kernels/flash_attention.py:73-84): every program converts every block it
// reads.  A prefill CTA pair of the tcgen05 kernel reads each K/V tile of its
// sequence once per 128 query rows and head pair, so converting in the
// attention kernel would repeat the conversion of a tile tens of times and put
// integer work on the softmax warps' issue slots.  Here each value is
// converted once, HBM-bound: int8 * scale in fp32 (exact: an 8-bit integer
// times a scale of at most 24 significant bits), rounded once to fp16 -- the
// 11-bit significand of the TF32 operands the reference's dot uses.
//
// Two layouts of the scratch pool:
//   gather  block (b, j) of the call (j < num_blocks_per_seq[b]) goes to
//           scratch block b * bt_cols + j, and a scratch block table holding
//           exactly those ids is written alongside (used when the call's
//           table covers fewer blocks than the pool holds);
//   mirror  block x goes to scratch block x, the call's own table is kept
//           (when the table's capacity is larger than the pool).
#include "pa_common.cuh"

namespace pa {
namespace {

constexpr int DQ_THREADS = 256;

__device__ __forceinline__ float scale_at(const void* s, long long off, int f32) {
  return f32 ? static_cast<const float*>(s)[off] : __half2float(static_cast<const __half*>(s)[off]);
}

// 16 int8 values times a scale -> 16 fp16 values (two 16-byte stores).
__device__ __forceinline__ void dequant16(const int8_t* src, float sc, __half* dst) {
  const uint4 w = *reinterpret_cast<const uint4*>(src);
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  uint32_t o[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int8_t* b = reinterpret_cast<const int8_t*>(&ws[k]);
    o[2 * k] = pack_f16(static_cast<float>(b[0]) * sc, static_cast<float>(b[1]) * sc);
    o[2 * k + 1] = pack_f16(static_cast<float>(b[2]) * sc, static_cast<float>(b[3]) * sc);
  }
  uint4* d = reinterpret_cast<uint4*>(dst);
  d[0] = make_uint4(o[0], o[1], o[2], o[3]);
  d[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

// One CTA per scratch block.  gather: blockIdx = (j, b); mirror: blockIdx.x = x.
__global__ void __launch_bounds__(DQ_THREADS) kv_dequant_kernel(const AttnParams p, __half* dk, __half* dv, int* dbt,
                                                                int gather, int D) {
  pdl_enter();
  int x, out;
  if (gather) {
    const int j = blockIdx.x;
    const int b = blockIdx.y;
    out = b * p.bt_cols + j;
    if (threadIdx.x == 0) dbt[out] = out;
    int nb = p.nblk[b];
    if (nb > p.bt_cols) nb = p.bt_cols;
    if (j >= nb) return;  // never read by the attention kernel
    x = p.bt[static_cast<long long>(b) * p.bt_ss + static_cast<long long>(j) * p.bt_sc];
    if (x < 0 || x >= p.NB) {
      if (threadIdx.x == 0) set_status(p.status, ST_BAD_BLOCK_ID);
      x = -1;  // an out-of-pool id reads as zeros
    }
  } else {
    x = blockIdx.x;
    out = x;
  }
  const int chunks = D / 16;
  const int rows = p.BS * p.Hkv;
  const long long obase = static_cast<long long>(out) * rows * D;
  for (int idx = threadIdx.x; idx < 2 * rows * chunks; idx += DQ_THREADS) {
    const int isv = idx >= rows * chunks;
    const int rc = isv ? idx - rows * chunks : idx;
    const int row = rc / chunks;
    const int ch = rc - row * chunks;
    const int slot = row / p.Hkv;
    const int h = row - slot * p.Hkv;
    __half* dst = (isv ? dv : dk) + obase + static_cast<long long>(row) * D + 16 * ch;
    if (x < 0) {
      uint4* d = reinterpret_cast<uint4*>(dst);
      d[0] = d[1] = make_uint4(0, 0, 0, 0);
      continue;
    }
    const long long xo = x;
    const int8_t* src = static_cast<const int8_t*>(isv ? p.v : p.k) +
                        (isv ? xo * p.v_sblk + slot * p.v_sslot + h * p.v_shead
                             : xo * p.k_sblk + slot * p.k_sslot + h * p.k_shead) + 16 * ch;
    const long long so = isv ? xo * p.vs_sblk + slot * p.vs_sslot + h * p.vs_shead
                             : xo * p.ks_sblk + slot * p.ks_sslot + h * p.ks_shead;
    dequant16(src, scale_at(isv ? p.vs : p.ks, so, p.scale_f32), dst);
  }
}

}  // namespace

cudaError_t launch_kv_dequant(const AttnParams& p, __half* dk, __half* dv, int* dbt, int gather, int D,
                              cudaStream_t stream) {
  const dim3 grid = gather ? dim3(p.bt_cols, p.B) : dim3(p.NB);
  if (grid.x == 0 || grid.y == 0) return cudaSuccess;
  cudaError_t e = launch_pdl(kv_dequant_kernel, grid, dim3(DQ_THREADS), 0, stream, p, dk, dv, dbt, gather, D);
  return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace pa
