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
// of X ([T, d_model]).  A tile is 128 tokens x 256 outputs -- two heads of K
// and/or V (2 * Hkv heads in all, so Hkv tiles per 128 tokens).  The kernel is
// persistent: one CTA per SM walks the tiles (outputs fastest, so the CTAs
// resident at one time share their X rows in L2 and W stays L2-resident), with
//   warp 8 (one lane)   TMA: X (128 x 64) and W (256 x 64) SW128 boxes into a
//                       4-stage ring of 48 KB stages;
//   warp 9 (one lane)   4 x (M128 N256 K16) MMAs per stage into one of two
//                       256-column TMEM accumulators (fp32), committing each
//                       stage free and each finished tile to the epilogue;
//   warps 0-7           the epilogue of the previous tile while the next one
//                       accumulates: warp w reads TMEM lanes 32 (w % 4).. of
//                       head w / 4 of the tile, thread = one token: bias, then
//                       for INT8 pools the row's absmax and the reference's
//                       quantisation rule (quant.cuh), else a rounded copy;
//                       the row goes to the token's slot of its block
//                       (block_table[seq_index[t]][pos >> log2 BS]).
// Roofline: tensor-bound, 2 * T * d_model * (2 * Hkv * D) FLOPs per launch;
// the operand traffic per stage (48 KB for 128 x 256 x 64) is 96 B per MMA
// cycle, inside the 128 B/clk shared-memory budget of the tensor core.
#include "pa_common.cuh"
#include "quant.cuh"

namespace pa {
namespace {

constexpr int KP_BM = 128;                        // tokens per tile
constexpr int KP_BN = 256;                        // outputs per tile (two heads)
constexpr int KP_BK = 64;                         // d_model columns per stage (one SW128 atom row)
constexpr int KP_STAGES = 4;
constexpr int KP_A_BYTES = KP_BM * 128;           // 16 KB
constexpr int KP_B_BYTES = KP_BN * 128;           // 32 KB
constexpr int KP_STAGE = KP_A_BYTES + KP_B_BYTES;  // 48 KB
constexpr int KP_BAR = KP_STAGES * KP_STAGE;      // 192 KB
constexpr int KP_SMEM = KP_BAR + 256 + 1024;      // barriers + alignment slack
constexpr int KP_EPI_WARPS = 8;
constexpr int KP_PRODUCER = 8;
constexpr int KP_MMA = 9;
constexpr int KP_THREADS = 320;
constexpr int KP_TMEM_COLS = 2 * KP_BN;           // two accumulators
static_assert(KP_SMEM <= 227 * 1024, "shared memory per CTA");
enum : int { P_FULL = 0, P_EMPTY = 4, P_TFULL = 8, P_TEMPTY = 10, P_TMEMSLOT = 12 };

// Bounded mbarrier wait; false (and a status bit) when it gives up.
__device__ __forceinline__ bool kp_wait(int* status, uint32_t bar, uint32_t parity) {
  for (int i = 0; i < (1 << 22); ++i)
    if (mbar_try_wait(bar, parity)) return true;
  set_status(status, ST_WAIT_TIMEOUT);
  return false;
}

// Destination of token t's row of head hh (0..2 Hkv-1: K heads, then V
// heads) in the pool and in the scale array, with the quantise-on-write
// kernel's range checks; false (and, when `report`, a status bit) for a token
// whose row is skipped.
__device__ __forceinline__ bool kp_dest(const ProjParams& p, int t, int hh, bool report, long long& dst_k,
                                        long long& dst_s) {
  if (t >= p.T) return false;
  const int sq = p.seq_idx[t];
  const int pos = p.pos[t];
  if (sq < 0 || sq >= p.num_seqs) {
    if (report) set_status(p.status, ST_BAD_SEQ_INDEX);
    return false;
  }
  if (pos < 0 || (pos >> p.log2BS) >= p.bt_cols) {
    if (report) set_status(p.status, ST_BAD_POSITION);
    return false;
  }
  const int blk = p.bt[static_cast<long long>(sq) * p.bt_ss + static_cast<long long>(pos >> p.log2BS) * p.bt_sc];
  if (blk < 0 || blk >= p.NB) {
    if (report) set_status(p.status, ST_BAD_BLOCK_ID);
    return false;
  }
  const bool isv = hh >= p.Hkv;
  const int h = isv ? hh - p.Hkv : hh;
  const int slot = pos & (p.BS - 1);
  const long long b64 = blk;
  dst_k = isv ? b64 * p.v_sblk + slot * p.v_sslot + h * p.v_shead : b64 * p.k_sblk + slot * p.k_sslot + h * p.k_shead;
  dst_s = isv ? b64 * p.vs_sblk + slot * p.vs_sslot + h * p.vs_shead
              : b64 * p.ks_sblk + slot * p.ks_sslot + h * p.ks_shead;
  return true;
}

// The four K16 steps of one 64-column stage: descriptors advance 32 bytes
// (2 in 16-byte units) per step inside the 128-byte swizzle atom.
__device__ __forceinline__ void kp_mma_stage(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  tc_mma_ss(d, a, b, idesc, acc);
  tc_mma_ss(d, a + 2, b + 2, idesc, 1u);
  tc_mma_ss(d, a + 4, b + 4, idesc, 1u);
  tc_mma_ss(d, a + 6, b + 6, idesc, 1u);
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
  const int n_tiles = p.Hkv;  // 2 * Hkv heads, two per tile
  const int tiles = n_tiles * ((p.T + KP_BM - 1) / KP_BM);
  const int nk = p.d_model / KP_BK;

  if (tid == 0) {
    for (int s = 0; s < KP_STAGES; ++s) {
      mbar_init(bar(P_FULL + s), 1);
      mbar_init(bar(P_EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(P_TFULL + b), 1);
      mbar_init(bar(P_TEMPTY + b), KP_EPI_WARPS);
    }
    fence_mbar_init();
  }
  if (warp == KP_MMA) {
    tmem_alloc(bar(P_TMEMSLOT), KP_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + KP_BAR + 8 * P_TMEMSLOT);

  if (warp == KP_PRODUCER) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const int m0 = (tile / n_tiles) * KP_BM;
        const int n0 = (tile % n_tiles) * KP_BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % KP_STAGES;
          if (it >= KP_STAGES) kp_wait(p.status, bar(P_EMPTY + s), ((it / KP_STAGES) - 1) & 1);
          mbar_arrive_expect_tx(bar(P_FULL + s), KP_STAGE);
          const uint32_t a = base + s * KP_STAGE;
          tma_load_2d(a, &xmap, bar(P_FULL + s), kb * KP_BK, m0);
          tma_load_2d(a + KP_A_BYTES, &wmap, bar(P_FULL + s), kb * KP_BK, n0);
        }
      }
      // every copy has landed before the CTA can exit (the MMA warp waits for
      // them too; this covers a consumer that gave up on a bounded wait)
      for (int s = 0; s < KP_STAGES && s < it; ++s) {
        const int last = it - 1 - ((it - 1 - s) % KP_STAGES);
        kp_wait(p.status, bar(P_FULL + s), (last / KP_STAGES) & 1);
      }
    }
  } else if (warp == KP_MMA) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = instr_desc_f16(BF16, false, false, KP_BM, KP_BN);
      int it = 0, lt = 0;
      for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++lt) {
        const int b = lt & 1;
        if (lt >= 2) kp_wait(p.status, bar(P_TEMPTY + b), ((lt >> 1) - 1) & 1);
        tc_fence_after();
        const uint32_t d = tmem + b * KP_BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % KP_STAGES;
          kp_wait(p.status, bar(P_FULL + s), (it / KP_STAGES) & 1);
          tc_fence_after();
          const uint32_t a = base + s * KP_STAGE;
          kp_mma_stage(d, smem_desc(a, 16, 1024), smem_desc(a + KP_A_BYTES, 16, 1024), IDESC, kb > 0 ? 1u : 0u);
          tc_commit(bar(P_EMPTY + s));
        }
        tc_commit(bar(P_TFULL + b));
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 0-7)
    const int q = warp & 3;   // TMEM lane quarter
    const int hf = warp >> 2; // head of the tile
    const int r = q * 32 + lane;
    int lt = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++lt) {
      const int b = lt & 1;
      const int m0 = (tile / n_tiles) * KP_BM;
      const int hh = 2 * (tile % n_tiles) + hf;  // head among [K heads | V heads]
      const bool isv = hh >= p.Hkv;
      const int t = m0 + r;
      // destination row of token t, resolved while the tile accumulates; one
      // of the two threads of a token reports
      long long dst_k = 0, dst_s = 0;
      const bool ok = kp_dest(p, t, hh, hf == 0, dst_k, dst_s);
      const float* bias = p.bias ? p.bias + hh * 128 : nullptr;  // head_dim 128 outputs per head
      const uint32_t trow = tmem + b * KP_BN + hf * 128 + (static_cast<uint32_t>(q * 32) << 16);
      kp_wait(p.status, bar(P_TFULL + b), (lt >> 1) & 1);
      tc_fence_after();
      if (p.cache_dtype == PA_DTYPE_I8) {
        // pass 1: the row's absmax (bias included); pass 2: quantise 32 values at a time
        float amax = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t v[32];
          tmem_ld32(trow + 32 * c, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            amax = fmaxf(amax, fabsf(__uint_as_float(v[i]) + (bias ? __ldg(bias + 32 * c + i) : 0.f)));
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
          for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]) + (bias ? __ldg(bias + 32 * c + i) : 0.f);
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
            const float a = __uint_as_float(v[2 * i]) + (bias ? __ldg(bias + 32 * c + 2 * i) : 0.f);
            const float e = __uint_as_float(v[2 * i + 1]) + (bias ? __ldg(bias + 32 * c + 2 * i + 1) : 0.f);
            w[i] = bf ? pack2<true>(a, e) : pack2<false>(a, e);
          }
          if (ok) {
            uint4* d = reinterpret_cast<uint4*>(row + 32 * c);
#pragma unroll
            for (int k = 0; k < 4; ++k) d[k] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
          }
        }
      }
      // this warp's reads of the accumulator are done: hand it back to the MMA warp
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(P_TEMPTY + b));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == KP_MMA) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, KP_TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Small batches (a decode step's tokens): Hkv * ceil(T / 128) tiles cannot
// fill the SMs, and each CTA would stream a 256-row slice of W on its own.
// kv_project_split_kernel splits every tile's d_model across the S CTAs of a
// thread-block cluster (S = gridDim.x <= 8): CTA c accumulates k-blocks
// [c nk / S, (c + 1) nk / S) in TMEM, parks the partial tile's rows of real
// tokens (fp32) in its own shared memory (the operand ring is free by then),
// and after a cluster barrier sums rows [c R, c R + R), R = ceil(rows / S),
// of all S partials through
// distributed shared memory (peers in rank order, so the sum is
// deterministic) and runs the epilogue for them: one warp per (token, head)
// row, four values a lane, the same bias / absmax / quantisation rule.  A
// second cluster barrier keeps every CTA's partial alive until its peers have
// read it.  Every CTA loads its own x and W slices (single-CTA TMA destinations).
constexpr int KS_STRIDE = 1040;  // bytes per staged row: 256 fp32 + 16 bytes of padding (no bank conflicts)
static_assert(KP_BM * KS_STRIDE <= KP_BAR, "the staged partial tile fits in the operand ring");
constexpr int KS_MAX = 8;        // CTAs per cluster (portable cluster size)
#ifndef PA_KVP_SPLIT
#define PA_KVP_SPLIT 1             // 0: every batch size takes the persistent kernel
#endif

__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];\n"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}

template <bool BF16>
__global__ void __launch_bounds__(KP_THREADS, 1)
    kv_project_split_kernel(const ProjParams p, const __grid_constant__ CUtensorMap xmap,
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
  const int S = gridDim.x;  // the cluster spans x
  const int rank = static_cast<int>(cluster_ctarank());
  const int n0 = blockIdx.y * KP_BN;
  const int m0 = blockIdx.z * KP_BM;
  const int nk = p.d_model / KP_BK;
  const int kb0 = rank * nk / S;
  const int kb1 = (rank + 1) * nk / S;  // non-empty: the host keeps S <= nk
  const int rows = min(KP_BM, p.T - m0);  // rows of real tokens in this tile

  if (tid == 0) {
    for (int st = 0; st < KP_STAGES; ++st) {
      mbar_init(bar(P_FULL + st), 1);
      mbar_init(bar(P_EMPTY + st), 1);
    }
    mbar_init(bar(P_TFULL), 1);
    fence_mbar_init();
  }
  if (warp == KP_MMA) {
    tmem_alloc(bar(P_TMEMSLOT), KP_BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + KP_BAR + 8 * P_TMEMSLOT);

  if (warp == KP_PRODUCER) {
    if (lane == 0) {
      int it = 0;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int st = it % KP_STAGES;
        if (it >= KP_STAGES) kp_wait(p.status, bar(P_EMPTY + st), ((it / KP_STAGES) - 1) & 1);
        mbar_arrive_expect_tx(bar(P_FULL + st), KP_STAGE);
        const uint32_t a = base + st * KP_STAGE;
        tma_load_2d(a, &xmap, bar(P_FULL + st), kb * KP_BK, m0);
        tma_load_2d(a + KP_A_BYTES, &wmap, bar(P_FULL + st), kb * KP_BK, n0);
      }
      for (int st = 0; st < KP_STAGES && st < it; ++st) {  // every copy has landed
        const int last = it - 1 - ((it - 1 - st) % KP_STAGES);
        kp_wait(p.status, bar(P_FULL + st), (last / KP_STAGES) & 1);
      }
    }
  } else if (warp == KP_MMA) {
    if (lane == 0) {
      constexpr uint32_t IDESC = instr_desc_f16(BF16, false, false, KP_BM, KP_BN);
      int it = 0;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int st = it % KP_STAGES;
        kp_wait(p.status, bar(P_FULL + st), (it / KP_STAGES) & 1);
        tc_fence_after();
        const uint32_t a = base + st * KP_STAGE;
        kp_mma_stage(tmem, smem_desc(a, 16, 1024), smem_desc(a + KP_A_BYTES, 16, 1024), IDESC, it > 0 ? 1u : 0u);
        tc_commit(bar(P_EMPTY + st));
      }
      tc_commit(bar(P_TFULL));
    }
  } else {
    // park the partial tile's rows of real tokens: thread = row r, warp w / 4 = head (128 columns)
    const int hf = warp >> 2;
    const int r = (warp & 3) * 32 + lane;
    kp_wait(p.status, bar(P_TFULL), 0);
    tc_fence_after();
    unsigned char* dst = sm + r * KS_STRIDE + hf * 512;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t v[32];
      tmem_ld32(tmem + hf * 128 + 32 * c + (static_cast<uint32_t>((warp & 3) * 32) << 16), v);
      tmem_wait_ld();
      if (r < rows)
#pragma unroll
        for (int i = 0; i < 8; ++i)
          *reinterpret_cast<uint4*>(dst + 128 * c + 16 * i) =
              make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // every CTA's partial is in its shared memory
  tc_fence_after();

  if (warp < KP_EPI_WARPS) {
    // CTA `rank` reduces and writes rows [rank R, rank R + R) of the tile's real rows
    const int R = (rows + S - 1) / S;
    const int nu = 2 * max(0, min(R, rows - rank * R));  // (row, head) units of this CTA
    for (int u = warp; u < nu; u += KP_EPI_WARPS) {
      const int row = rank * R + (u >> 1);
      const int hh = 2 * blockIdx.y + (u & 1);  // head among [K heads | V heads]
      const uint32_t src = base + row * KS_STRIDE + (u & 1) * 512 + 16 * lane;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int c = 0; c < S; ++c) {
        const float4 v = ld_cluster_f4(mapa_shared(src, c));
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
      }
      if (p.bias) {  // 4-byte aligned only: scalar loads
        const float* bv = p.bias + hh * 128 + 4 * lane;
        acc.x += __ldg(bv);
        acc.y += __ldg(bv + 1);
        acc.z += __ldg(bv + 2);
        acc.w += __ldg(bv + 3);
      }
      long long dst_k = 0, dst_s = 0;
      const bool ok = kp_dest(p, m0 + row, hh, lane == 0 && (u & 1) == 0, dst_k, dst_s);
      const bool isv = hh >= p.Hkv;
      const float f[4] = {acc.x, acc.y, acc.z, acc.w};
      if (p.cache_dtype == PA_DTYPE_I8) {
        float amax = fmaxf(fmaxf(fabsf(f[0]), fabsf(f[1])), fmaxf(fabsf(f[2]), fabsf(f[3])));
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float sc = amax == 0.f ? 1.0f : div127_rn(amax);
        uint32_t w[1];
        const bool near = quant_row_fast<4>(f, rcp_approx(sc), w);
        if (__any_sync(0xffffffffu, near)) quant_row_exact<4>(f, sc, w);
        if (ok) {
          *reinterpret_cast<uint32_t*>(static_cast<int8_t*>(isv ? p.v : p.k) + dst_k + 4 * lane) = w[0];
          if (lane == 0) {
            void* sp = isv ? p.vs : p.ks;
            if (p.scale_f32) static_cast<float*>(sp)[dst_s] = sc;
            else static_cast<__half*>(sp)[dst_s] = __float2half_rn(sc);
          }
        }
      } else if (ok) {
        const bool bf = p.cache_dtype == PA_DTYPE_BF16;
        const uint2 w = bf ? make_uint2(pack2<true>(f[0], f[1]), pack2<true>(f[2], f[3]))
                           : make_uint2(pack2<false>(f[0], f[1]), pack2<false>(f[2], f[3]));
        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(isv ? p.v : p.k) + dst_k + 4 * lane) = w;
      }
    }
  }
  __syncwarp();
  cluster_sync_all();  // no CTA leaves while a peer may still read its partial
  if (warp == KP_MMA) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, KP_BN);
  }
}

}  // namespace

int device_sm_count() {
  static int n[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (n[dev] == 0) {
    int v = 0;
    n[dev] = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0 ? v : 148;
  }
  return n[dev];
}

cudaError_t launch_kv_project(const ProjParams& p, const CUtensorMap& xmap, const CUtensorMap& wmap, int bf16,
                              cudaStream_t stream) {
  if (p.T == 0) return cudaSuccess;
  const int m_tiles = (p.T + KP_BM - 1) / KP_BM;
  const long long tiles = static_cast<long long>(p.Hkv) * m_tiles;
  const int sms = device_sm_count();
  const int nk = p.d_model / KP_BK;
  if (PA_KVP_SPLIT && tiles * 2 <= sms && nk >= 2 && m_tiles <= 65535) {
    // too few tiles for the SMs: split each tile's d_model across a cluster, with
    // the largest cluster size whose clusters (one per tile) are all resident at
    // once -- one wave; a second wave would double the time
    auto split_cfg = [&](int S, cudaLaunchAttribute* attr) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(S, p.Hkv, m_tiles);
      cfg.blockDim = dim3(KP_THREADS);
      cfg.dynamicSmemBytes = KP_SMEM;
      cfg.stream = stream;
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = S;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      return cfg;
    };
    auto go_split = [&](auto kern) -> cudaError_t {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, KP_SMEM);
      if (e != cudaSuccess) return e;
      // resident clusters per cluster size, cached per device (a property of the kernel and the GPU)
      static int resident_cache[64][KS_MAX + 1] = {};
      int dev = 0;
      if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
      int S = 0;
      for (int c = KS_MAX; c >= 2 && S == 0; c >>= 1) {
        if (c > nk) continue;
        int& resident = resident_cache[dev][c];
        if (resident == 0) {
          cudaLaunchAttribute attr[1];
          const cudaLaunchConfig_t cfg = split_cfg(c, attr);
          if (cudaOccupancyMaxActiveClusters(&resident, kern, &cfg) != cudaSuccess || resident <= 0) {
            (void)cudaGetLastError();
            resident = -1;  // cannot launch clusters of this size
          }
        }
        if (tiles <= resident) S = c;
      }
      if (S == 0) return cudaErrorNotReady;  // no cluster size fits in one wave: the persistent kernel
      cudaLaunchAttribute attr[1];
      const cudaLaunchConfig_t cfg = split_cfg(S, attr);
      e = cudaLaunchKernelEx(&cfg, kern, p, xmap, wmap);
      return e != cudaSuccess ? e : cudaGetLastError();
    };
    const cudaError_t e = bf16 ? go_split(kv_project_split_kernel<true>) : go_split(kv_project_split_kernel<false>);
    if (e != cudaErrorNotReady) return e;
  }
  const int grid = static_cast<int>(tiles < sms ? tiles : sms);
  auto go = [&](auto kern) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, KP_SMEM);
    if (e != cudaSuccess) return e;
    e = launch_pdl(kern, dim3(grid), dim3(KP_THREADS), KP_SMEM, stream, p, xmap, wmap);
    return e != cudaSuccess ? e : cudaGetLastError();
  };
  return bf16 ? go(kv_project_kernel<true>) : go(kv_project_kernel<false>);
}

}  // namespace pa
