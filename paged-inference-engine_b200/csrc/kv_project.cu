// K/V projection with the cache write in its epilogue: the new tokens' K and
// V rows are computed on the tensor cores and written straight into the paged
// pool (quantised for INT8 pools), never stored unpaged in HBM.
//
// Replaces transformer/model.py:75-82 (k = W_k(x), v = W_v(x), head split)
// followed by the cache write of :85-122: there the projected K/V go to HBM
// and are read back by the write; here one kernel does both.
//
// Out[t, n] = sum_c X[t, c] * W[n, c] + bias[n] for the rows n of W = [W_k;
// W_v] ([2 * Hkv * D, d_model], nn.Linear's [out, in] layout) and the tokens t
// of X ([T, d_model]).  A CTA computes 128 tokens x 128 outputs -- one head of
// K or of V -- on tcgen05:
//   warp 4 (one lane)  TMA: X and W tiles of 128 rows x 128 columns (two
//                      64-column SW128 boxes each) into a 3-stage ring;
//   warp 5 (one lane)  8 x K16 MMAs per stage into a 128-column TMEM
//                      accumulator (fp32), committing each stage free;
//   warps 0-3          the epilogue: thread r owns token m0 + r (TMEM lane r):
//                      bias, then for INT8 pools the row's absmax and the
//                      reference's quantisation rule (quant.cuh), else a
//                      rounded copy; the row goes to the token's slot of its
//                      block (block_table[seq_index[t]][pos >> log2 BS]).
#include "pa_common.cuh"
#include "quant.cuh"

namespace pa {
namespace {

constexpr int KP_BM = 128;             // tokens per CTA
constexpr int KP_BN = 128;             // outputs per CTA (= head_dim)
constexpr int KP_BK = 128;             // d_model columns per stage
constexpr int KP_STAGES = 3;
constexpr int KP_HALF = KP_BM * 128;   // one 64-column half of a 128-row tile: 16 KB
constexpr int KP_TILE = 2 * KP_HALF;   // 32 KB
constexpr int KP_A = 0;
constexpr int KP_B = KP_STAGES * KP_TILE;
constexpr int KP_BAR = 2 * KP_STAGES * KP_TILE;  // 192 KB
constexpr int KP_BIAS = KP_BAR + 256;            // float[128]
constexpr int KP_SMEM = KP_BIAS + 512 + 1024;    // + alignment slack
constexpr int KP_THREADS = 192;
static_assert(KP_SMEM <= 227 * 1024, "shared memory per CTA");
enum : int { P_FULL = 0, P_EMPTY = 3, P_DONE = 6, P_TMEMSLOT = 7 };

// Bounded mbarrier wait; false (and a status bit) when it gives up.
__device__ __forceinline__ bool kp_wait(int* status, uint32_t bar, uint32_t parity) {
  for (int i = 0; i < (1 << 22); ++i)
    if (mbar_try_wait(bar, parity)) return true;
  set_status(status, ST_WAIT_TIMEOUT);
  return false;
}

template <bool BF16>
__global__ void __launch_bounds__(KP_THREADS, 1)
    kv_project_kernel(const ProjParams p, const __grid_constant__ CUtensorMap xmap,
                      const __grid_constant__ CUtensorMap wmap) {
  pdl_enter();
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* sm = smem_raw + (base - raw);
  const uint32_t bars = base + KP_BAR;
  auto bar = [&](int i) { return bars + 8u * i; };
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int m0 = blockIdx.x * KP_BM;
  const int n0 = blockIdx.y * KP_BN;  // rows of W: head blockIdx.y of K (< Hkv) or V
  const int nk = p.d_model / KP_BK;

  if (tid == 0) {
    for (int s = 0; s < KP_STAGES; ++s) {
      mbar_init(bar(P_FULL + s), 1);
      mbar_init(bar(P_EMPTY + s), 1);
    }
    mbar_init(bar(P_DONE), 1);
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(bar(P_TMEMSLOT), 128);
    tmem_relinquish();
  }
  float* sbias = reinterpret_cast<float*>(sm + KP_BIAS);
  if (tid < KP_BN) sbias[tid] = p.bias ? p.bias[n0 + tid] : 0.f;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + KP_BAR + 8 * P_TMEMSLOT);

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % KP_STAGES;
        if (kb >= KP_STAGES) kp_wait(p.status, bar(P_EMPTY + s), ((kb / KP_STAGES) - 1) & 1);
        mbar_arrive_expect_tx(bar(P_FULL + s), 2 * KP_TILE);
        const uint32_t a = base + KP_A + s * KP_TILE;
        const uint32_t b = base + KP_B + s * KP_TILE;
        tma_load_2d(a, &xmap, bar(P_FULL + s), kb * KP_BK, m0);
        tma_load_2d(a + KP_HALF, &xmap, bar(P_FULL + s), kb * KP_BK + 64, m0);
        tma_load_2d(b, &wmap, bar(P_FULL + s), kb * KP_BK, n0);
        tma_load_2d(b + KP_HALF, &wmap, bar(P_FULL + s), kb * KP_BK + 64, n0);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = instr_desc_f16(BF16, false, false, KP_BM, KP_BN);
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % KP_STAGES;
        kp_wait(p.status, bar(P_FULL + s), (kb / KP_STAGES) & 1);
        tc_fence_after();
        tc_mma_ss_k128_acc<KP_HALF / 16, KP_HALF / 16>(tmem, smem_desc(base + KP_A + s * KP_TILE, 16, 1024),
                                                       smem_desc(base + KP_B + s * KP_TILE, 16, 1024), IDESC,
                                                       kb > 0 ? 1u : 0u);
        tc_commit(bar(P_EMPTY + s));
      }
      tc_commit(bar(P_DONE));
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 0-3)
    const int r = tid;  // TMEM lane = token row
    const int t = m0 + r;
    const uint32_t trow = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    kp_wait(p.status, bar(P_DONE), 0);
    tc_fence_after();
    // destination row of token t (range checks as the quantise-on-write kernel)
    bool ok = t < p.T;
    long long dst_k = 0, dst_s = 0;
    if (ok) {
      const int sq = p.seq_idx[t];
      const int pos = p.pos[t];
      if (sq < 0 || sq >= p.num_seqs) {
        set_status(p.status, ST_BAD_SEQ_INDEX);
        ok = false;
      } else if (pos < 0 || (pos >> p.log2BS) >= p.bt_cols) {
        set_status(p.status, ST_BAD_POSITION);
        ok = false;
      } else {
        const int blk = p.bt[static_cast<long long>(sq) * p.bt_ss + static_cast<long long>(pos >> p.log2BS) * p.bt_sc];
        if (blk < 0 || blk >= p.NB) {
          set_status(p.status, ST_BAD_BLOCK_ID);
          ok = false;
        } else {
          const int slot = pos & (p.BS - 1);
          const int isv = blockIdx.y >= p.Hkv;
          const int h = isv ? blockIdx.y - p.Hkv : blockIdx.y;
          const long long b64 = blk;
          dst_k = isv ? b64 * p.v_sblk + slot * p.v_sslot + h * p.v_shead : b64 * p.k_sblk + slot * p.k_sslot + h * p.k_shead;
          dst_s = isv ? b64 * p.vs_sblk + slot * p.vs_sslot + h * p.vs_shead
                      : b64 * p.ks_sblk + slot * p.ks_sslot + h * p.ks_shead;
        }
      }
    }
    const bool isv = blockIdx.y >= p.Hkv;
    if (p.cache_dtype == PA_DTYPE_I8) {
      // pass 1: the row's absmax (bias included); pass 2: quantise 32 values at a time
      float amax = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(trow + 32 * c, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(__uint_as_float(v[i]) + sbias[32 * c + i]));
      }
      const float sc = amax == 0.f ? 1.0f : div127_rn(amax);
      const float inv = rcp_approx(sc);
      int8_t* row = static_cast<int8_t*>(isv ? p.v : p.k) + dst_k;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(trow + 32 * c, v);
        tmem_wait_ld();
        float f[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]) + sbias[32 * c + i];
        uint32_t w[8];
        if (quant_row_fast<32>(f, inv, w)) quant_row_exact<32>(f, sc, w);
        if (ok) {
          uint4* d = reinterpret_cast<uint4*>(row + 32 * c);
          d[0] = make_uint4(w[0], w[1], w[2], w[3]);
          d[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
      }
      if (ok) {
        void* sp = isv ? p.vs : p.ks;
        if (p.scale_f32) static_cast<float*>(sp)[dst_s] = sc;
        else static_cast<__half*>(sp)[dst_s] = __float2half_rn(sc);
      }
    } else {
      const bool bf = p.cache_dtype == PA_DTYPE_BF16;
      uint16_t* row = static_cast<uint16_t*>(isv ? p.v : p.k) + dst_k;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(trow + 32 * c, v);
        tmem_wait_ld();
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float a = __uint_as_float(v[2 * i]) + sbias[32 * c + 2 * i];
          const float b = __uint_as_float(v[2 * i + 1]) + sbias[32 * c + 2 * i + 1];
          w[i] = bf ? pack2<true>(a, b) : pack2<false>(a, b);
        }
        if (ok) {
          uint4* d = reinterpret_cast<uint4*>(row + 32 * c);
#pragma unroll
          for (int q = 0; q < 4; ++q) d[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

}  // namespace

int kv_project_smem() { return KP_SMEM; }

cudaError_t launch_kv_project(const ProjParams& p, const CUtensorMap& xmap, const CUtensorMap& wmap, int bf16,
                              cudaStream_t stream) {
  if (p.T == 0) return cudaSuccess;
  const dim3 grid((p.T + KP_BM - 1) / KP_BM, 2 * p.Hkv);
  auto go = [&](auto kern) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, KP_SMEM);
    if (e != cudaSuccess) return e;
    e = launch_pdl(kern, grid, dim3(KP_THREADS), KP_SMEM, stream, p, xmap, wmap);
    return e != cudaSuccess ? e : cudaGetLastError();
  };
  return bf16 ? go(kv_project_kernel<true>) : go(kv_project_kernel<false>);
}

}  // namespace pa
