// Causal paged prefill on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Replaces the q_len > 1 use of flash_attention_kernel
// (kernels/flash_attention.py:19-136) for 16-bit pools with head_dim 128.
// A CTA computes 128 query rows (FlashAttention-2 recurrence,
// kernels/flash_attention.py:102-123) with warp-specialised roles:
//
//   producer    TMA: the Q tile once, then K and V tiles of 128 keys gathered
//               through the block table (one 4-D TMA box per block and per 64
//               columns of head_dim) into separate K and V rings; the block ids
//               of a tile are fetched by 8-16 lanes at once, one tile ahead.
//               Boxes past the sequence or of an out-of-pool block id are
//               fetched at an out-of-range block coordinate (zero fill).
//   MMA issuer  one lane: S = Q K^T (M=128, N=128, K=128 as 8 x K16 steps, both
//               operands K-major SW128 in shared memory) and O += P V with P read
//               from TMEM and V an MN-major SW128 operand; each 8-step product
//               is one asm sequence.  tcgen05.commit signals S ready, ring
//               stages free and O done.
//   softmax     the threads of query row t (TMEM lane t) mask it (bottom-right
//               causal, sequence end), keep its running max in base 2, write P
//               (fp16/bf16) over S in TMEM, and rescale its O row only when the
//               max grows by more than 2^8 (a stale max leaves the result
//               exact).  The epilogue normalises O and writes O and LSE.
//
// pa_prefill_tc2_kernel (GQA groups of even size, the default): two query
// heads of one KV head share every K/V tile; TMEM holds S_a, S_b, O_a, O_b;
// each row of each head is split between two softmax warps (64 keys each).
// pa_prefill_tc_kernel (one head): TMEM holds S0, S1 (double-buffered) and O;
// each row's 128 columns are split between two softmax warpgroups.
#include <atomic>
#include <cstdlib>

#include "pa_common.cuh"

namespace pa {
namespace {

constexpr int TC_BM = 128;        // query rows per CTA
constexpr int TC_BN = 128;        // keys per tile
constexpr int TC_D = 128;         // head_dim
constexpr int TC_THREADS = 320;   // 8 softmax warps (two per row) + producer + MMA
constexpr int HALF_B = TC_BM * 128;               // one 64-column half of a 128-row tile: 16 KB
constexpr int TILE_B = 2 * HALF_B;                // 32 KB
constexpr uint32_t TMEM_COLS = 512;
__device__ __forceinline__ constexpr uint32_t s_col(int s) { return s ? 128u : 0u; }
constexpr uint32_t O_COL = 256;
constexpr float RESCALE_THRESHOLD = 8.0f;         // log2 units
// With PA_EMU_EVERY_MASK = M >= 0, pairs of probabilities whose index i
// satisfies (i & M) == M compute 2^x with the FMA-pipe polynomial instead of
// MUFU.EX2 (MUFU throughput per SM matches the tensor core's rate per score
// element for head_dim 128).  Off by default: measured on B200, every kernel
// here is faster with all exponentials on MUFU (paired heads 674 against 642
// TFLOP/s with a quarter on the FMA pipe); the polynomial's instructions cost
// more issue slots than the MUFU queue wait they save.
#ifndef PA_EMU_EVERY_MASK
#define PA_EMU_EVERY_MASK -1
#endif
constexpr int EMU_EVERY_MASK = PA_EMU_EVERY_MASK;
__device__ __forceinline__ constexpr bool emu_pair(int i) {
  return EMU_EVERY_MASK >= 0 && (i & EMU_EVERY_MASK) == EMU_EVERY_MASK;
}

struct alignas(64) TcMaps {
  CUtensorMap k;
  CUtensorMap v;
  CUtensorMap q;
};

__device__ __forceinline__ int tc_seq_qlen(const AttnParams& p, int b) { return seq_rows(p, b); }

__device__ __forceinline__ int tc_seq_keys(const AttnParams& p, int b, int q) {
  if (q <= 0) return 0;
  int nb = p.nblk[b];
  if (nb > p.bt_cols) nb = p.bt_cols;
  if (nb < 0) nb = 0;
  long long nk = p.kvlen[b];
  const long long cap = static_cast<long long>(nb) << p.log2BS;
  if (nk > cap) nk = cap;
  if (nk < 0) nk = 0;
  if (p.top_left && nk > q) nk = q;
  return static_cast<int>(nk);
}

// Named barrier `id` over `n` threads (the softmax warpgroups of a CTA).
__device__ __forceinline__ void named_barrier_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(n) : "memory");
}

// Launch generation of the last launch in which a wait gave up: once one CTA
// times out, every other wait of that launch stops within ~1k polls instead of
// running into its own limit.
__device__ unsigned int g_tc_abort_gen = 0;

// Work counters of the persistent paired-head prefill grid.  Slot
// (launch generation & 255) holds [next item, CTAs finished]; the last CTA of
// a launch zeroes its slot, so a slot is ready for the next launch (also for
// a replay of a captured graph, which reuses its generation).  Two launches
// in flight at the same time use different slots unless their generations
// are 256 apart.
__device__ unsigned int g_pf_sched[256][2];

// 8 x 8 transpose of 16-byte pieces across the eight lanes of a group (lane
// index i = lane & 7): on return lane i holds piece i of lanes 0..7's rows.
// Three butterfly stages; in stage m a lane swaps, with lane i ^ m, the four
// pieces whose index differs from i in bit m (selects on compile-time
// indices, 16 shuffles a stage).
__device__ __forceinline__ void transpose8_u4(uint4 (&v)[8], int i) {
#pragma unroll
  for (int m = 1; m < 8; m <<= 1) {
    const bool hi = (i & m) != 0;
#pragma unroll
    for (int j0 = 0; j0 < 8; ++j0) {
      if (j0 & m) continue;
      const int j1 = j0 | m;
      const uint4 t = hi ? v[j0] : v[j1];
      uint4 u;
      u.x = __shfl_xor_sync(0xffffffffu, t.x, m);
      u.y = __shfl_xor_sync(0xffffffffu, t.y, m);
      u.z = __shfl_xor_sync(0xffffffffu, t.z, m);
      u.w = __shfl_xor_sync(0xffffffffu, t.w, m);
      if (hi) v[j0] = u;
      else v[j1] = u;
    }
  }
}

// Bounded mbarrier wait; false (and a status bit) on time-out or abort.  The
// first poll is inlined: a wait on a phase that has already completed costs
// ~55 cycles this way against ~240 through the out-of-line loop.
__device__ __noinline__ bool wait_or_flag_slow(const AttnParams& p, uint32_t bar, uint32_t parity) {
  constexpr int kLimit = 1 << 20;
  for (int i = 0; i < kLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023) == 1023 && *reinterpret_cast<volatile unsigned int*>(&g_tc_abort_gen) == p.abort_gen) return false;
  }
  atomicExch(&g_tc_abort_gen, p.abort_gen);
  set_status(p.status, ST_WAIT_TIMEOUT);
  return false;
}
__device__ __forceinline__ bool wait_or_flag(const AttnParams& p, uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  return wait_or_flag_slow(p, bar, parity);
}

// Single-head kernel: K and V in separate 3-stage rings of 128-key tiles.
constexpr int T1_KS = 3;
constexpr int T1_VS = 3;
constexpr int T1_K = TILE_B;                          // after Q
constexpr int T1_V = T1_K + T1_KS * TILE_B;
constexpr int T1_BAR = T1_V + T1_VS * TILE_B;         // 224 KB
constexpr int T1_SMEM = T1_BAR + 256 + 1024 + 1024;  // barriers, row-max / row-sum exchange, alignment
static_assert(T1_SMEM <= 227 * 1024, "shared memory per CTA");
enum : int { E_QFULL = 0, E_QREADY = 1, E_KFULL = 2, E_KEMPTY = 5, E_VFULL = 8, E_VEMPTY = 11, E_SFULL = 14,
             E_PFULL = 16, E_ODONE = 18, E_TMEMSLOT = 19 };

template <bool MMA_BF16, bool Q_CONVERT>
__global__ void __launch_bounds__(TC_THREADS, 1)
    pa_prefill_tc_kernel(const AttnParams p, const __grid_constant__ TcMaps maps) {
  pdl_enter();
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // grid (head, sequence, query tile), the query tile slowest and counted down:
  // CTAs are dispatched in x, y, z order, so every sequence's and head's last
  // (longest causal) tiles start first and the short ones fill the tail
  const int mtile = gridDim.z - 1 - blockIdx.z;
  const int hq = blockIdx.x;
  const int b = blockIdx.y;
  const int qlen = tc_seq_qlen(p, b);
  const int m0 = mtile * TC_BM;
  if (m0 >= qlen) return;

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* sm = smem_raw + (base - raw);
  const uint32_t bars = base + T1_BAR;
  auto bar = [&](int i) { return bars + 8u * i; };
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  const int kvh = hq / p.G;
  const int nkeys = tc_seq_keys(p, b, qlen);
  const int off = p.top_left ? 0 : p.kvlen[b] - qlen;
  const int kend = min(nkeys, off + m0 + TC_BM);
  const int nt = kend > 0 ? (kend + TC_BN - 1) / TC_BN : 0;

  if (tid == 0) {
    mbar_init(bar(E_QFULL), 1);
    mbar_init(bar(E_QREADY), 256);
    for (int s = 0; s < T1_KS; ++s) {
      mbar_init(bar(E_KFULL + s), 1);
      mbar_init(bar(E_KEMPTY + s), 1);
    }
    for (int s = 0; s < T1_VS; ++s) {
      mbar_init(bar(E_VFULL + s), 1);
      mbar_init(bar(E_VEMPTY + s), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(E_SFULL + s), 1);
      mbar_init(bar(E_PFULL + s), 256);
    }
    mbar_init(bar(E_ODONE), 1);
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(bar(E_TMEMSLOT), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + T1_BAR + 8 * E_TMEMSLOT);

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && nt > 0) {
      mbar_arrive_expect_tx(bar(E_QFULL), TILE_B);
      // Q tile: rows m0.. of sequence b (ragged rows: rows q_start[b] + m0.. of the packed Q; rows past
      // its end read as zeros and rows of the next sequence are computed but never stored)
      const int q_row0 = p.q_start ? p.q_start[b] + m0 : m0;
      const int q_seq = p.q_start ? 0 : b;
      tma_load_4d(base, &maps.q, bar(E_QFULL), 0, q_row0, hq, q_seq);
      tma_load_4d(base + HALF_B, &maps.q, bar(E_QFULL), 64, q_row0, hq, q_seq);
    }
    if (nt > 0) {
      // Lane i owns box i of every tile: the block ids of a tile are fetched in
      // one round trip (and one tile ahead), and each lane issues its own boxes.
      const int boxs = p.BS < 16 ? p.BS : 16;
      const int nbox = TC_BN / boxs;  // <= 16 (block_size >= 8)
      const int* bt_row = p.bt + static_cast<long long>(b) * p.bt_ss;
      auto fetch = [&](int j) {
        const int key = j * TC_BN + lane * boxs;
        int blk = p.NB;  // out of range: TMA fills the box with zeros
        if (lane < nbox && key < nkeys) {
          const int x = __ldg(bt_row + static_cast<long long>(key >> p.log2BS) * p.bt_sc);
          if (x >= 0 && x < p.NB) blk = x;
          else set_status(p.status, ST_BAD_BLOCK_ID);
        }
        return blk;
      };
      int blk = fetch(0);
      for (int j = 0; j < nt; ++j) {
        const int blk_next = (j + 1 < nt) ? fetch(j + 1) : p.NB;
        const int slot = (j * TC_BN + lane * boxs) & (p.BS - 1);
        const uint32_t roff = static_cast<uint32_t>(lane * boxs * 128);
        const int ks = j % T1_KS;
        const int vs = j % T1_VS;
        if (lane == 0) {
          if (j >= T1_KS) wait_or_flag(p, bar(E_KEMPTY + ks), ((j / T1_KS) - 1) & 1);
          mbar_arrive_expect_tx(bar(E_KFULL + ks), TILE_B);
        }
        __syncwarp();
        if (lane < nbox) {
          const uint32_t dst = base + T1_K + ks * TILE_B + roff;
          tma_load_4d(dst, &maps.k, bar(E_KFULL + ks), 0, kvh, blk < p.NB ? slot : 0, blk);
          tma_load_4d(dst + HALF_B, &maps.k, bar(E_KFULL + ks), 64, kvh, blk < p.NB ? slot : 0, blk);
        }
        if (lane == 0) {
          if (j >= T1_VS) wait_or_flag(p, bar(E_VEMPTY + vs), ((j / T1_VS) - 1) & 1);
          mbar_arrive_expect_tx(bar(E_VFULL + vs), TILE_B);
        }
        __syncwarp();
        if (lane < nbox) {
          const uint32_t dst = base + T1_V + vs * TILE_B + roff;
          tma_load_4d(dst, &maps.v, bar(E_VFULL + vs), 0, kvh, blk < p.NB ? slot : 0, blk);
          tma_load_4d(dst + HALF_B, &maps.v, bar(E_VFULL + vs), 64, kvh, blk < p.NB ? slot : 0, blk);
        }
        blk = blk_next;
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && nt > 0) {
      constexpr uint32_t IDESC_QK = instr_desc_f16(MMA_BF16, false, false, TC_BM, TC_BN);
      constexpr uint32_t IDESC_PV = instr_desc_f16(MMA_BF16, false, true, TC_BM, TC_D);
      auto pv = [&](int jj) {
        wait_or_flag(p, bar(E_PFULL + (jj & 1)), (jj >> 1) & 1);
        wait_or_flag(p, bar(E_VFULL + jj % T1_VS), (jj / T1_VS) & 1);
        tc_fence_after();
        tc_mma_ts_seq<TC_BN / 16>(tmem + O_COL, tmem + s_col(jj & 1),
                                  smem_desc(base + T1_V + (jj % T1_VS) * TILE_B, HALF_B, 1024), IDESC_PV,
                                  jj > 0 ? 1u : 0u);
        tc_commit(bar(E_VEMPTY + jj % T1_VS));
        tc_commit(bar(E_ODONE));
      };
      wait_or_flag(p, bar(E_QREADY), 0);
      for (int j = 0; j < nt; ++j) {
        // S_j into buffer j % 2 (its previous P was consumed by a P*V issued earlier)
        wait_or_flag(p, bar(E_KFULL + j % T1_KS), (j / T1_KS) & 1);
        tc_fence_after();
        tc_mma_ss_k128<HALF_B / 16, HALF_B / 16>(tmem + s_col(j & 1), smem_desc(base, 16, 1024),
                                                 smem_desc(base + T1_K + (j % T1_KS) * TILE_B, 16, 1024), IDESC_QK);
        tc_commit(bar(E_SFULL + (j & 1)));
        tc_commit(bar(E_KEMPTY + j % T1_KS));
        if (j > 0) pv(j - 1);
      }
      pv(nt - 1);
    }
  } else {
    // ------------------------------------------------------------ softmax (warps 0..7)
    // Two warpgroups share every row: warp w serves TMEM lanes 32 (w % 4) ..,
    // warpgroup 0 the keys [0, 64) of each tile, warpgroup 1 the keys [64, 128).
    // Row maxima are combined through shared memory at a named barrier of the
    // 256 softmax threads, which also orders both halves' S loads before either
    // overwrites S with P.  Each half keeps its own row sum and rescales and
    // stores its own 64 columns of O.
    const int hf = warp >> 2;           // column half
    const int r = tid & 127;            // query row within the tile = TMEM lane
    const int row = m0 + r;
    const uint32_t trow = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    float* mxs = reinterpret_cast<float*>(sm + T1_BAR + 256);  // [2 halves][128 rows]
    if (nt > 0) {
      wait_or_flag(p, bar(E_QFULL), 0);
      if constexpr (Q_CONVERT) {
        // Q arrives in its own 16-bit type; convert in place to the pool's type
        uint4* q4 = reinterpret_cast<uint4*>(sm);
#pragma unroll 4
        for (int i = tid; i < TILE_B / 16; i += 256) {
          uint4 v = q4[i];
          v.x = cvt_pair<!MMA_BF16, MMA_BF16>(v.x);
          v.y = cvt_pair<!MMA_BF16, MMA_BF16>(v.y);
          v.z = cvt_pair<!MMA_BF16, MMA_BF16>(v.z);
          v.w = cvt_pair<!MMA_BF16, MMA_BF16>(v.w);
          q4[i] = v;
        }
        fence_proxy_async_smem();
      }
      mbar_arrive(bar(E_QREADY));
    }
    const int lim = min(nkeys, off + row + 1);
    float m_ref = -INFINITY;
    float l = 0.f;
    // O-done phases are consumed one by one and never more than one phase
    // away from the barrier: a parity wait on a phase two ahead succeeds at
    // once, one on a phase two behind never does.
    int od = 0;
    auto wait_o_done = [&](int k) {
      for (; od <= k; ++od) wait_or_flag(p, bar(E_ODONE), od & 1);
    };
    for (int j = 0; j < nt; ++j) {
      const int s = j & 1;
      wait_or_flag(p, bar(E_SFULL + s), (j >> 1) & 1);
      tc_fence_after();
      const uint32_t scol = s_col(s);
      const int k0 = j * TC_BN + 64 * hf;  // first key of this half
      const bool need_mask = (k0 + 64 > off + m0 + 1) || (k0 + 64 > nkeys);
      // this half's 64 logits of the row (masked entries -inf) and their max
      uint32_t r0[32], r1[32];
      tmem_ld32(trow + scol + 64 * hf, r0);
      tmem_ld32(trow + scol + 64 * hf + 32, r1);
      tmem_wait_ld();
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      if (need_mask) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float v0 = (k0 + i < lim) ? __uint_as_float(r0[i]) : -INFINITY;
          const float v1 = (k0 + 32 + i < lim) ? __uint_as_float(r1[i]) : -INFINITY;
          r0[i] = __float_as_uint(v0);
          r1[i] = __float_as_uint(v1);
          mx4[i & 3] = fmax3f(mx4[i & 3], v0, v1);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) mx4[i & 3] = fmax3f(mx4[i & 3], __uint_as_float(r0[i]), __uint_as_float(r1[i]));
      }
      const float mhalf = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      mxs[hf * 128 + r] = mhalf;
      named_barrier_sync(2, 256);
      const float mx = fmaxf(mhalf, mxs[(hf ^ 1) * 128 + r]) * p.scale_log2;
      named_barrier_sync(2, 256);  // both halves have read before the next write
      float alpha = 1.f;
      bool resc = false;
      if (mx > m_ref + RESCALE_THRESHOLD) {  // also the first finite max (m_ref = -inf)
        alpha = ex2(m_ref - mx);
        // O holds P*V of earlier tiles once j > 0, whatever this half's own sum
        // is (every probability of a half can underflow): both halves decide
        // alike from the shared maximum.
        resc = j > 0;
        m_ref = mx;
      }
      if (__any_sync(0xffffffffu, resc)) {
        // O holds P_0..P_{j-1} V: wait for the last of them, then rescale this half of the row
        wait_o_done(j - 1);
        tc_fence_after();
        const float a = resc ? alpha : 1.f;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t rr[32];
          tmem_ld32(trow + O_COL + 64 * hf + 32 * c, rr);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) rr[i] = __float_as_uint(__uint_as_float(rr[i]) * a);
          tmem_st32(trow + O_COL + 64 * hf + 32 * c, rr);
        }
        tmem_wait_st();
      }
      l *= alpha;
      const float neg_m = (m_ref == -INFINITY) ? 0.f : -m_ref;
      const float c2 = p.scale_log2;
      // P = 2^(s*c - m) packed in pairs from the registers; P of keys
      // [64 hf, 64 hf + 64) goes to TMEM columns [32 hf, 32 hf + 32) of the S buffer
      uint64_t lsum2[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
      uint32_t pk[32];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t* rr = h ? r1 : r0;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float p0, p1;
          f2_unpack(f2_fma(f2_pack(__uint_as_float(rr[2 * i]), __uint_as_float(rr[2 * i + 1])), f2_pack(c2, c2),
                           f2_pack(neg_m, neg_m)),
                    p0, p1);
          if (emu_pair(i)) {
            exp2_fma_x2(p0, p1);  // optionally a share of the exponentials on the FMA pipe
          } else {
            p0 = ex2(p0);
            p1 = ex2(p1);
          }
          if (need_mask) {
            const int kk = k0 + 32 * h + 2 * i;
            if (kk >= lim) p0 = 0.f;
            if (kk + 1 >= lim) p1 = 0.f;
          }
          lsum2[h] = f2_add(lsum2[h], f2_pack(p0, p1));
          pk[16 * h + i] = pack2<MMA_BF16>(p0, p1);
        }
      }
      tmem_st32(trow + scol + 32 * hf, pk);
      {
        float a0, a1, b0, b1;
        f2_unpack(lsum2[0], a0, a1);
        f2_unpack(lsum2[1], b0, b1);
        l += (a0 + a1) + (b0 + b1);
      }
      tmem_wait_st();
      const int kt = j * TC_BN;
      if (nkeys - kt < TC_BN) {
        // keys past the sequence: zero their V rows (each half zeroes its
        // 64-column half of the row) so that P = 0 contributes exactly nothing
        wait_or_flag(p, bar(E_VFULL + j % T1_VS), (j / T1_VS) & 1);
        if (kt + r >= nkeys) {
          unsigned char* vrow = sm + T1_V + (j % T1_VS) * TILE_B + hf * HALF_B + r * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(vrow + 16 * c) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
      }
      // stay within one phase of the O-done barrier (P*V(j-1) finished long ago)
      if (j >= 1) wait_o_done(j - 1);
      tc_fence_before();
      mbar_arrive(bar(E_PFULL + s));
    }
    // ---- epilogue: O / l, LSE ---------------------------------------------
    // the row sum is the sum of the two halves' sums
    mxs[hf * 128 + r] = l;
    named_barrier_sync(2, 256);
    const float lt = l + mxs[(hf ^ 1) * 128 + r];
    const bool valid = row < qlen;
    uint4 ov[8];  // this thread's 64 output columns, eight 16-byte pieces
    if (nt > 0) {
      wait_o_done(nt - 1);
      tc_fence_after();
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t rr[32];
        tmem_ld32(trow + O_COL + 64 * hf + 32 * c, rr);
        tmem_wait_ld();
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          ov[4 * c + v].x = pack_f16(__uint_as_float(rr[8 * v + 0]) * inv, __uint_as_float(rr[8 * v + 1]) * inv);
          ov[4 * c + v].y = pack_f16(__uint_as_float(rr[8 * v + 2]) * inv, __uint_as_float(rr[8 * v + 3]) * inv);
          ov[4 * c + v].z = pack_f16(__uint_as_float(rr[8 * v + 4]) * inv, __uint_as_float(rr[8 * v + 5]) * inv);
          ov[4 * c + v].w = pack_f16(__uint_as_float(rr[8 * v + 6]) * inv, __uint_as_float(rr[8 * v + 7]) * inv);
        }
      }
    } else {
#pragma unroll
      for (int v = 0; v < 8; ++v) ov[v] = make_uint4(0, 0, 0, 0);
    }
    // coalesced stores, as in the paired kernel: store k of a lane group writes row 8 g + k
    transpose8_u4(ov, lane & 7);
    {
      const int r0 = (warp & 3) * 32 + (lane & ~7);
      __half* obase = static_cast<__half*>(p.o) + o_seq_base(p, b) + hq * p.o_sh + 64 * hf + 8 * (lane & 7);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int rw = m0 + r0 + kk;
        if (rw < qlen) *reinterpret_cast<uint4*>(obase + static_cast<long long>(rw) * p.o_sm) = ov[kk];
      }
    }
    if (valid && p.lse && hf == 0) {
      const float L = lt > 0.f ? (m_ref + lg2(lt)) * 0.6931471805599453f : -INFINITY;
      static_cast<__half*>(p.lse)[l_seq_base(p, b) + hq * p.l_sh + static_cast<long long>(row) * p.l_sm] =
          __float2half_rn(L);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Paired-head kernel (grouped-query attention with an even group): one CTA
// computes the same 128 query rows for two query heads of one KV group, so each
// K/V tile is fetched once for both.  The softmax warps of the two heads
// alternate with the tensor core: while one head turns S into P, the MMA warp
// runs the other head's P*V and next Q*K^T ("ping-pong").  K and V have
// separate rings (3 and 2 stages) so a K stage is recycled as soon as both
// Q*K^T products have consumed it.  TMEM: S_a [0,128), S_b [128,256),
// O_a [256,384), O_b [384,512).
//
// Warp w < 16 serves TMEM lanes 32 (w % 4) .. of head (w >> 2) & 1 and the
// keys [64 h, 64 h + 64) of every tile, h = w >> 3: each sub-partition runs
// two warps per head, so one warp's independent work issues while the other
// waits on MUFU, and each warp reads its 64 logits from TMEM once.  Row maxima
// are combined through shared memory at a named barrier of the head's 256
// threads (half 1 posts its maximum, half 0 posts the row's), which also
// orders both halves' S loads before either overwrites S with P.
// ---------------------------------------------------------------------------
constexpr int P2_KS = 3;          // K stages
constexpr int P2_VS = 2;          // V stages
constexpr int P2_QA = 0;
constexpr int P2_QB = TILE_B;
constexpr int P2_K = 2 * TILE_B;
constexpr int P2_V = P2_K + P2_KS * TILE_B;
constexpr int P2_BAR = P2_V + P2_VS * TILE_B;     // 224 KB
enum : int { C_QFULL = 0, C_QREADY = 1, C_KFULL = 2, C_KEMPTY = 5, C_VFULL = 8, C_VEMPTY = 10, C_SFULL = 12,
             C_PFULL = 14, C_ODONE = 16, C_TMEMSLOT = 18, C_QEMPTY = 19, C_IFULL = 20, C_IEMPTY = 22,
             C_RING = 24,  // two 16-byte work-item slots, bytes 192..223 of the barrier area
             C_QFULL_B = 28, C_QREADY_B = 29, C_QEMPTY_B = 30 };
// Q barriers per head: head a uses C_QFULL / C_QREADY / C_QEMPTY, head b the _B slots, so head a's
// next Q tile loads as soon as head a's last Q*K^T has read its buffer.
__device__ __forceinline__ constexpr int q_full(int x) { return x ? C_QFULL_B : C_QFULL; }
__device__ __forceinline__ constexpr int q_ready(int x) { return x ? C_QREADY_B : C_QREADY; }
__device__ __forceinline__ constexpr int q_empty(int x) { return x ? C_QEMPTY_B : C_QEMPTY; }

// PA_PF_ROW1 = 0 (default): two softmax threads per query row, each taking
// 64 keys of every tile (16 softmax warps, 96 registers a thread), the row
// maxima and sums combined through shared memory.  1: one thread per row (8
// softmax warps, 168 registers a thread).  Measured on B200 (bf16, 32/8
// heads): 773 against 750 TFLOP/s on the 8-prompt L ~ U[1024, 4096] batch and
// 1107 against 1034 on one 16K prompt, but 363 against 391 on 64 prompts of
// 512 tokens, where one row per thread's shorter epilogue pays off.
#ifndef PA_PF_ROW1
#define PA_PF_ROW1 0
#endif
constexpr int P2_SOFTMAX_WARPS = PA_PF_ROW1 ? 8 : 16;
constexpr int P2_THREADS = 32 * (P2_SOFTMAX_WARPS + 2);  // softmax warps + producer + MMA
constexpr int P2_PRODUCER = P2_SOFTMAX_WARPS;
constexpr int P2_MMA = P2_SOFTMAX_WARPS + 1;
constexpr int P2_XCH = P2_BAR + 256;              // float [2 heads][128 rows]
constexpr int P2_SMEM = P2_XCH + 1024 + 1024;      // + alignment slack
static_assert(P2_SMEM <= 227 * 1024, "shared memory per CTA");

template <bool MMA_BF16, bool Q_CONVERT>
__global__ void __launch_bounds__(P2_THREADS, 1)
    pa_prefill_tc2_kernel(const AttnParams p, const __grid_constant__ TcMaps maps) {
  pdl_enter();
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* sm = smem_raw + (base - raw);
  const uint32_t bars = base + P2_BAR;
  auto bar = [&](int i) { return bars + 8u * i; };
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  // Persistent: a CTA runs work items (head pair, sequence, 128-row query
  // tile) until none is left.  Item i = (z * B + b) * pairs_total + pair, with
  // query tile MT - 1 - z: every sequence's longest (causal) tiles are handed
  // out first; tiles past a sequence's rows are skipped by the producer.  The
  // producer takes items from a launch-wide counter and passes each, with its
  // sequence's lengths, through a two-slot ring (IFULL / IEMPTY); it loads
  // the next item's Q as soon as the last Q*K^T of the current one has read Q
  // (QEMPTY) and its K/V tiles as ring stages free up, and the MMA warp starts
  // the next item's Q*K^T behind the current item's last P*V, so consecutive
  // items overlap.  Every barrier counts phases across items: tile gt + j of
  // the CTA uses ring stage (gt + j) % stages and phase (gt + j) / stages, and
  // the Q barriers count items with keys (qi).
  const int pairs = p.G >> 1;
  const int P = p.Hkv * pairs;
  const int MT = (p.maxq + TC_BM - 1) / TC_BM;
  const int PB = P * p.B;
  const unsigned total = static_cast<unsigned>(PB) * static_cast<unsigned>(MT);
  unsigned int* sched = g_pf_sched[p.abort_gen & 255u];
  volatile int* ring = reinterpret_cast<volatile int*>(sm + P2_BAR + 8 * C_RING);  // [2][item, qlen, nkeys, off]

  if (tid == 0) {
    for (int x = 0; x < 2; ++x) {
      mbar_init(bar(q_full(x)), 1);
      mbar_init(bar(q_ready(x)), 16 * P2_SOFTMAX_WARPS);  // the head's softmax threads
      mbar_init(bar(q_empty(x)), 1);
    }
    for (int s = 0; s < P2_KS; ++s) {
      mbar_init(bar(C_KFULL + s), 1);
      mbar_init(bar(C_KEMPTY + s), 1);
    }
    for (int s = 0; s < P2_VS; ++s) {
      mbar_init(bar(C_VFULL + s), 1);
      mbar_init(bar(C_VEMPTY + s), 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(bar(C_SFULL + x), 1);
      mbar_init(bar(C_PFULL + x), 16 * P2_SOFTMAX_WARPS);  // the head's softmax threads
      mbar_init(bar(C_ODONE + x), 1);
      mbar_init(bar(C_IFULL + x), 1);
      mbar_init(bar(C_IEMPTY + x), 1 + P2_SOFTMAX_WARPS);  // the MMA lane and one lane of each softmax warp
    }
    fence_mbar_init();
  }
  if (warp == P2_MMA) {
    tmem_alloc(bar(C_TMEMSLOT), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + P2_BAR + 8 * C_TMEMSLOT);

  // the item of ring slot `slot`, for the MMA and softmax roles
  auto take_item = [&](int it, int& item, int& qlen, int& nkeys, int& off) {
    const int slot = it & 1;
    wait_or_flag(p, bar(C_IFULL + slot), (it >> 1) & 1);
    item = ring[4 * slot];
    qlen = ring[4 * slot + 1];
    nkeys = ring[4 * slot + 2];
    off = ring[4 * slot + 3];
  };

  if (warp == P2_PRODUCER) {
    // ------------------------------------------------------------ producer
    int gt = 0, qi = 0;
    for (int it = 0;; ++it) {
      int item = -1, qlen = 0, nkeys = 0, off = 0;
      if (lane == 0) {
        for (;;) {
          const unsigned i = atomicAdd(&sched[0], 1u);
          if (i >= total) break;
          const int zz = static_cast<int>(i / static_cast<unsigned>(PB));
          const int bb = (static_cast<int>(i) - zz * PB) / P;
          const int ql = tc_seq_qlen(p, bb);
          if ((MT - 1 - zz) * TC_BM < ql) {
            item = static_cast<int>(i);
            qlen = ql;
            nkeys = tc_seq_keys(p, bb, ql);
            off = p.top_left ? 0 : p.kvlen[bb] - ql;
            break;
          }
        }
        const int slot = it & 1;
        if (it >= 2) wait_or_flag(p, bar(C_IEMPTY + slot), ((it >> 1) - 1) & 1);
        ring[4 * slot] = item;
        ring[4 * slot + 1] = qlen;
        ring[4 * slot + 2] = nkeys;
        ring[4 * slot + 3] = off;
        mbar_arrive(bar(C_IFULL + slot));  // release: the slot's words are visible to its waiters
      }
      item = __shfl_sync(0xffffffffu, item, 0);
      if (item < 0) break;
      qlen = __shfl_sync(0xffffffffu, qlen, 0);
      nkeys = __shfl_sync(0xffffffffu, nkeys, 0);
      off = __shfl_sync(0xffffffffu, off, 0);
      const int zi = item / PB;
      const int b = (item - zi * PB) / P;
      const int hp = item - zi * PB - b * P;
      const int m0 = (MT - 1 - zi) * TC_BM;
      const int kvh = hp / pairs;
      const int hq0 = kvh * p.G + 2 * (hp - kvh * pairs);
      const int kend = min(nkeys, off + m0 + TC_BM);
      const int nt = kend > 0 ? (kend + TC_BN - 1) / TC_BN : 0;
      if (nt > 0) {
        if (lane == 0) {
          // Q tile: rows m0.. of sequence b (ragged rows: rows q_start[b] + m0.. of the packed Q; rows past
          // its end read as zeros and rows of the next sequence are computed but never stored)
          const int q_row0 = p.q_start ? p.q_start[b] + m0 : m0;
          const int q_seq = p.q_start ? 0 : b;
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            // head x's buffer is free once the last item's Q*K^T of head x have read it
            if (qi > 0) wait_or_flag(p, bar(q_empty(x)), (qi - 1) & 1);
            mbar_arrive_expect_tx(bar(q_full(x)), TILE_B);
            tma_load_4d(base + (x ? P2_QB : P2_QA), &maps.q, bar(q_full(x)), 0, q_row0, hq0 + x, q_seq);
            tma_load_4d(base + (x ? P2_QB : P2_QA) + HALF_B, &maps.q, bar(q_full(x)), 64, q_row0, hq0 + x, q_seq);
          }
        }
        const int boxs = p.BS < 16 ? p.BS : 16;
        const int nbox = TC_BN / boxs;  // <= 16 (block_size >= 8)
        const int* bt_row = p.bt + static_cast<long long>(b) * p.bt_ss;
        auto fetch = [&](int j) {
          const int key = j * TC_BN + lane * boxs;
          int blk = p.NB;  // out of range: TMA fills the box with zeros
          if (lane < nbox && key < nkeys) {
            const int x = __ldg(bt_row + static_cast<long long>(key >> p.log2BS) * p.bt_sc);
            if (x >= 0 && x < p.NB) blk = x;
            else set_status(p.status, ST_BAD_BLOCK_ID);
          }
          return blk;
        };
        int blk = fetch(0);
        for (int j = 0; j < nt; ++j) {
          const int blk_next = (j + 1 < nt) ? fetch(j + 1) : p.NB;
          const int slot = (j * TC_BN + lane * boxs) & (p.BS - 1);
          const uint32_t roff = static_cast<uint32_t>(lane * boxs * 128);
          const int g = gt + j;
          const int ks = g % P2_KS;
          const int vs = g % P2_VS;
          if (lane == 0) {
            if (g >= P2_KS) wait_or_flag(p, bar(C_KEMPTY + ks), ((g / P2_KS) - 1) & 1);
            mbar_arrive_expect_tx(bar(C_KFULL + ks), TILE_B);
          }
          __syncwarp();
          if (lane < nbox) {
            const uint32_t dst = base + P2_K + ks * TILE_B + roff;
            tma_load_4d(dst, &maps.k, bar(C_KFULL + ks), 0, kvh, blk < p.NB ? slot : 0, blk);
            tma_load_4d(dst + HALF_B, &maps.k, bar(C_KFULL + ks), 64, kvh, blk < p.NB ? slot : 0, blk);
          }
          if (lane == 0) {
            if (g >= P2_VS) wait_or_flag(p, bar(C_VEMPTY + vs), ((g / P2_VS) - 1) & 1);
            mbar_arrive_expect_tx(bar(C_VFULL + vs), TILE_B);
          }
          __syncwarp();
          if (lane < nbox) {
            const uint32_t dst = base + P2_V + vs * TILE_B + roff;
            tma_load_4d(dst, &maps.v, bar(C_VFULL + vs), 0, kvh, blk < p.NB ? slot : 0, blk);
            tma_load_4d(dst + HALF_B, &maps.v, bar(C_VFULL + vs), 64, kvh, blk < p.NB ? slot : 0, blk);
          }
          blk = blk_next;
        }
      }
      gt += nt;
      qi += nt > 0;
    }
  } else if (warp == P2_MMA) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC_QK = instr_desc_f16(MMA_BF16, false, false, TC_BM, TC_BN);
      constexpr uint32_t IDESC_PV = instr_desc_f16(MMA_BF16, false, true, TC_BM, TC_D);
      int gt = 0, qi = 0;
      // j: tile of the current item; stages and phases run on gt + j
      auto qk = [&](int x, int j) {
        const uint32_t kb = base + P2_K + ((gt + j) % P2_KS) * TILE_B;
        const uint32_t qb = base + (x ? P2_QB : P2_QA);
        tc_mma_ss_k128<HALF_B / 16, HALF_B / 16>(tmem + s_col(x), smem_desc(qb, 16, 1024), smem_desc(kb, 16, 1024),
                                                 IDESC_QK);
        tc_commit(bar(C_SFULL + x));
      };
      auto pv = [&](int x, int j) {
        wait_or_flag(p, bar(C_PFULL + x), (gt + j) & 1);
        tc_fence_after();
        const uint32_t vb = base + P2_V + ((gt + j) % P2_VS) * TILE_B;
        tc_mma_ts_seq<TC_BN / 16>(tmem + O_COL + 128 * x, tmem + s_col(x), smem_desc(vb, HALF_B, 1024), IDESC_PV,
                                  j > 0 ? 1u : 0u);
        tc_commit(bar(C_ODONE + x));
      };
      for (int it = 0; it <= static_cast<int>(total); ++it) {
        int item, qlen, nkeys, off;
        take_item(it, item, qlen, nkeys, off);
        mbar_arrive(bar(C_IEMPTY + (it & 1)));
        if (item < 0) break;
        const int zi = item / PB;
        const int m0 = (MT - 1 - zi) * TC_BM;
        const int kend = min(nkeys, off + m0 + TC_BM);
        const int nt = kend > 0 ? (kend + TC_BN - 1) / TC_BN : 0;
        if (nt == 0) continue;
        wait_or_flag(p, bar(C_KFULL + gt % P2_KS), (gt / P2_KS) & 1);
#pragma unroll
        for (int x = 0; x < 2; ++x) {  // each head as soon as its own Q tile is ready
          wait_or_flag(p, bar(Q_CONVERT ? q_ready(x) : q_full(x)), qi & 1);
          tc_fence_after();
          qk(x, 0);
          if (nt == 1) tc_commit(bar(q_empty(x)));  // head x's Q is free once this product is done
        }
        tc_commit(bar(C_KEMPTY + gt % P2_KS));
        for (int j = 0; j < nt; ++j) {
          const int g = gt + j;
          wait_or_flag(p, bar(C_VFULL + g % P2_VS), (g / P2_VS) & 1);
          pv(0, j);
          const bool more = j + 1 < nt;
          if (more) {
            wait_or_flag(p, bar(C_KFULL + (g + 1) % P2_KS), ((g + 1) / P2_KS) & 1);
            tc_fence_after();
            qk(0, j + 1);
            if (j + 2 == nt) tc_commit(bar(q_empty(0)));
          }
          pv(1, j);
          tc_commit(bar(C_VEMPTY + g % P2_VS));
          if (more) {
            qk(1, j + 1);
            tc_commit(bar(C_KEMPTY + (g + 1) % P2_KS));
            if (j + 2 == nt) tc_commit(bar(q_empty(1)));
          }
        }
        gt += nt;
        ++qi;
      }
    }
#if PA_PF_ROW1
  } else {
    // ------------------------------------------------------------ softmax (warps 0-7), one row per thread
    // Warp w serves TMEM lanes 32 (w % 4) .. of head w / 4: thread r owns query row r of its head and
    // all 128 keys of every tile, so the row's maximum and sum never leave the thread.
    const int x = warp >> 2;  // 0: head a, 1: head b
    const int r = tid & 127;  // query row within the tile = TMEM lane
    const uint32_t trow = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t scol = s_col(x);
    const uint32_t ocol = O_COL + 128 * x;
    // tiles of an item (0 for none or the end marker)
    auto item_tiles = [&](int itm, int nk, int of) {
      if (itm < 0) return 0;
      const int ke = min(nk, of + (MT - 1 - itm / PB) * TC_BM + TC_BM);
      return ke > 0 ? (ke + TC_BN - 1) / TC_BN : 0;
    };
    // Q arrives in the other 16-bit type: the item's Q tile is converted in
    // place, then released to the MMA warp (without conversion the MMA warp
    // waits for the Q tile itself).  A next item's Q is converted before the
    // current item's epilogue, so its first Q*K^T overlaps that epilogue.
    auto convert_q = [&](int q_phase) {
      wait_or_flag(p, bar(q_full(x)), q_phase & 1);
      uint4* q4 = reinterpret_cast<uint4*>(sm + (x ? P2_QB : P2_QA));
#pragma unroll 4
      for (int i = r; i < TILE_B / 16; i += 128) {
        uint4 v = q4[i];
        v.x = cvt_pair<!MMA_BF16, MMA_BF16>(v.x);
        v.y = cvt_pair<!MMA_BF16, MMA_BF16>(v.y);
        v.z = cvt_pair<!MMA_BF16, MMA_BF16>(v.z);
        v.w = cvt_pair<!MMA_BF16, MMA_BF16>(v.w);
        q4[i] = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(bar(q_ready(x)));
    };
    int gt = 0, qi = 0;
    int item, qlen, nkeys, off;
    take_item(0, item, qlen, nkeys, off);
    __syncwarp();
    if (lane == 0) mbar_arrive(bar(C_IEMPTY));
    if (Q_CONVERT && item_tiles(item, nkeys, off) > 0) convert_q(0);
    for (int it = 0; it <= static_cast<int>(total); ++it) {
      if (item < 0) break;
      const int zi = item / PB;
      const int b = (item - zi * PB) / P;
      const int hp = item - zi * PB - b * P;
      const int m0 = (MT - 1 - zi) * TC_BM;
      const int kvh = hp / pairs;
      const int hq0 = kvh * p.G + 2 * (hp - kvh * pairs);
      const int nt = item_tiles(item, nkeys, off);
      const int row = m0 + r;
      const int lim = min(nkeys, off + row + 1);
      float m_ref = -INFINITY;
      float l = 0.f;
      // The MMA warp issues Q*K^T(x, j+1) after P*V(x, j), and a tcgen05.commit
      // arrives only once every earlier tcgen05 operation of its thread has
      // completed: S(x, j) ready implies P*V(x, j-1) done.  O-done is therefore
      // waited on once, for the last P*V, in the epilogue.
      for (int j = 0; j < nt; ++j) {
        wait_or_flag(p, bar(C_SFULL + x), (gt + j) & 1);
        tc_fence_after();
        const int k0 = j * TC_BN;
        const bool need_mask = (k0 + TC_BN > off + m0 + 1) || (k0 + TC_BN > nkeys);
        uint32_t s0[32], s1[32], s2[32], s3[32];
        tmem_ld32(trow + scol, s0);
        tmem_ld32(trow + scol + 32, s1);
        tmem_ld32(trow + scol + 64, s2);
        tmem_ld32(trow + scol + 96, s3);
        tmem_wait_ld();
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float v0 = (k0 + i < lim) ? __uint_as_float(s0[i]) : -INFINITY;
            const float v1 = (k0 + 32 + i < lim) ? __uint_as_float(s1[i]) : -INFINITY;
            const float v2 = (k0 + 64 + i < lim) ? __uint_as_float(s2[i]) : -INFINITY;
            const float v3 = (k0 + 96 + i < lim) ? __uint_as_float(s3[i]) : -INFINITY;
            s0[i] = __float_as_uint(v0);
            s1[i] = __float_as_uint(v1);
            s2[i] = __float_as_uint(v2);
            s3[i] = __float_as_uint(v3);
            mx4[i & 3] = fmax3f(mx4[i & 3], fmax3f(v0, v1, v2), v3);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            mx4[i & 3] = fmax3f(mx4[i & 3], fmax3f(__uint_as_float(s0[i]), __uint_as_float(s1[i]), __uint_as_float(s2[i])),
                                __uint_as_float(s3[i]));
        }
        const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * p.scale_log2;
        float alpha = 1.f;
        bool resc = false;
        if (mx > m_ref + RESCALE_THRESHOLD) {  // also the first finite max (m_ref = -inf)
          alpha = ex2(m_ref - mx);
          resc = j > 0;  // O holds P*V of earlier tiles once j > 0
          m_ref = mx;
        }
        const float neg_m = (m_ref == -INFINITY) ? 0.f : -m_ref;
        const float c2 = p.scale_log2;
        // P of keys [16 q, 16 q + 16) goes to TMEM columns [8 q, 8 q + 8) of S
        uint64_t lsum2[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
        auto exp_chunk = [&](const uint32_t (&rv)[32], int kc) {
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            uint32_t pk[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              float p0, p1;
              f2_unpack(f2_fma(f2_pack(__uint_as_float(rv[16 * q + 2 * i]), __uint_as_float(rv[16 * q + 2 * i + 1])),
                               f2_pack(c2, c2), f2_pack(neg_m, neg_m)),
                        p0, p1);
              if (emu_pair(i)) {
                exp2_fma_x2(p0, p1);
              } else {
                p0 = ex2(p0);
                p1 = ex2(p1);
              }
              if (need_mask) {
                const int kk = k0 + kc + 16 * q + 2 * i;
                if (kk >= lim) p0 = 0.f;
                if (kk + 1 >= lim) p1 = 0.f;
              }
              lsum2[q] = f2_add(lsum2[q], f2_pack(p0, p1));
              pk[i] = pack2<MMA_BF16>(p0, p1);
            }
            tmem_st8(trow + scol + (kc >> 1) + 8 * q, pk);
          }
        };
        exp_chunk(s0, 0);
        exp_chunk(s1, 32);
        exp_chunk(s2, 64);
        exp_chunk(s3, 96);
        {
          float a0, a1, b0, b1;
          f2_unpack(lsum2[0], a0, a1);
          f2_unpack(lsum2[1], b0, b1);
          l = l * alpha + ((a0 + a1) + (b0 + b1));
        }
        // Rescale the O row after the logits are dead (fewer live registers);
        // P*V(j) is issued only after PFULL, so O is still P*V(<j).
        if (__any_sync(0xffffffffu, resc)) {
          const float a = resc ? alpha : 1.f;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t rr[32];
            tmem_ld32(trow + ocol + 32 * c, rr);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) rr[i] = __float_as_uint(__uint_as_float(rr[i]) * a);
            tmem_st32(trow + ocol + 32 * c, rr);
          }
        }
        tmem_wait_st();
        const int kt = j * TC_BN;
        if (x == 0 && nkeys - kt < TC_BN) {
          // keys past the sequence: zero their V rows (head a's P*V runs first)
          wait_or_flag(p, bar(C_VFULL + (gt + j) % P2_VS), ((gt + j) / P2_VS) & 1);
          if (kt + r >= nkeys) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              unsigned char* vrow = sm + P2_V + ((gt + j) % P2_VS) * TILE_B + h * HALF_B + r * 128;
#pragma unroll
              for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(vrow + 16 * c) = make_uint4(0, 0, 0, 0);
            }
          }
          fence_proxy_async_smem();
        }
        tc_fence_before();
        mbar_arrive(bar(C_PFULL + x));
      }
      // ---- the next item (its Q converted now), then this item's epilogue
      int n_item, n_qlen, n_nkeys, n_off;
      take_item(it + 1, n_item, n_qlen, n_nkeys, n_off);
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(C_IEMPTY + ((it + 1) & 1)));
      if (Q_CONVERT && item_tiles(n_item, n_nkeys, n_off) > 0) convert_q(qi + (nt > 0));
      // ---- epilogue: O / l, LSE ---------------------------------------------
      const int hq = hq0 + x;
      const bool valid = row < qlen;
      __half* orow = static_cast<__half*>(p.o) + o_seq_base(p, b) + hq * p.o_sh + static_cast<long long>(row) * p.o_sm;
      if (nt > 0) {
        wait_or_flag(p, bar(C_ODONE + x), (gt + nt - 1) & 1);  // the item's last P*V
        tc_fence_after();
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t rr[32];
          tmem_ld32(trow + ocol + 32 * c, rr);
          tmem_wait_ld();
          if (valid) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 w;
              w.x = pack_f16(__uint_as_float(rr[8 * v + 0]) * inv, __uint_as_float(rr[8 * v + 1]) * inv);
              w.y = pack_f16(__uint_as_float(rr[8 * v + 2]) * inv, __uint_as_float(rr[8 * v + 3]) * inv);
              w.z = pack_f16(__uint_as_float(rr[8 * v + 4]) * inv, __uint_as_float(rr[8 * v + 5]) * inv);
              w.w = pack_f16(__uint_as_float(rr[8 * v + 6]) * inv, __uint_as_float(rr[8 * v + 7]) * inv);
              *reinterpret_cast<uint4*>(orow + 32 * c + 8 * v) = w;
            }
          }
        }
      } else if (valid) {
        for (int d = 0; d < 128; d += 8) *reinterpret_cast<uint4*>(orow + d) = make_uint4(0, 0, 0, 0);
      }
      if (valid && p.lse) {
        const float L = l > 0.f ? (m_ref + lg2(l)) * 0.6931471805599453f : -INFINITY;
        static_cast<__half*>(p.lse)[l_seq_base(p, b) + hq * p.l_sh + static_cast<long long>(row) * p.l_sm] =
            __float2half_rn(L);
      }
      gt += nt;
      qi += nt > 0;
      item = n_item;
      qlen = n_qlen;
      nkeys = n_nkeys;
      off = n_off;
    }
#else
  } else {
    // ------------------------------------------------------------ softmax (warps 0-15)
    const int x = (warp >> 2) & 1;  // 0: head a, 1: head b
    const int hf = warp >> 3;       // key half of every tile
    const int r = tid & 127;        // query row within the tile = TMEM lane
    const int bar_id = 1 + x;       // named barrier of this head's 256 threads
    const uint32_t trow = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t scol = s_col(x);
    const uint32_t ocol = O_COL + 128 * x + 64 * hf;
    float* xch = reinterpret_cast<float*>(sm + P2_XCH) + x * 128 + r;
    // tiles of an item (0 for none or the end marker)
    auto item_tiles = [&](int itm, int nk, int of) {
      if (itm < 0) return 0;
      const int ke = min(nk, of + (MT - 1 - itm / PB) * TC_BM + TC_BM);
      return ke > 0 ? (ke + TC_BN - 1) / TC_BN : 0;
    };
    // Q arrives in the other 16-bit type: the item's Q tile is converted in
    // place, then released to the MMA warp (without conversion the MMA warp
    // waits for the Q tile itself).  A next item's Q is converted before the
    // current item's epilogue, so its first Q*K^T overlaps that epilogue
    // (measured: 721-737 TFLOP/s against 695-704 converting after it).
    auto convert_q = [&](int q_phase) {
      wait_or_flag(p, bar(q_full(x)), q_phase & 1);
      uint4* q4 = reinterpret_cast<uint4*>(sm + (x ? P2_QB : P2_QA));
#pragma unroll 4
      for (int i = hf * 128 + r; i < TILE_B / 16; i += 256) {
        uint4 v = q4[i];
        v.x = cvt_pair<!MMA_BF16, MMA_BF16>(v.x);
        v.y = cvt_pair<!MMA_BF16, MMA_BF16>(v.y);
        v.z = cvt_pair<!MMA_BF16, MMA_BF16>(v.z);
        v.w = cvt_pair<!MMA_BF16, MMA_BF16>(v.w);
        q4[i] = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(bar(q_ready(x)));
    };
    int gt = 0, qi = 0;
    int item, qlen, nkeys, off;
    take_item(0, item, qlen, nkeys, off);
    __syncwarp();
    if (lane == 0) mbar_arrive(bar(C_IEMPTY));
    if (Q_CONVERT && item_tiles(item, nkeys, off) > 0) convert_q(0);
    for (int it = 0; it <= static_cast<int>(total); ++it) {
      if (item < 0) break;
      const int zi = item / PB;
      const int b = (item - zi * PB) / P;
      const int hp = item - zi * PB - b * P;
      const int m0 = (MT - 1 - zi) * TC_BM;
      const int kvh = hp / pairs;
      const int hq0 = kvh * p.G + 2 * (hp - kvh * pairs);
      const int nt = item_tiles(item, nkeys, off);
      const int row = m0 + r;
      // Half 1 posts a value, half 0 combines it with its own and posts the
      // result, half 1 reads it back: two barriers, one float per row and head.
      auto combine = [&](float v, bool is_max) {
        if (hf) {
          *xch = v;
          named_barrier_sync(bar_id, 256);
          named_barrier_sync(bar_id, 256);
          return *xch;
        }
        named_barrier_sync(bar_id, 256);
        const float o = *xch;
        const float t = is_max ? fmaxf(v, o) : v + o;
        *xch = t;
        named_barrier_sync(bar_id, 256);
        return t;
      };
      const int lim = min(nkeys, off + row + 1);
      float m_ref = -INFINITY;
      float l = 0.f;
      // The MMA warp issues Q*K^T(x, j+1) after P*V(x, j), and a tcgen05.commit
      // arrives only once every earlier tcgen05 operation of its thread has
      // completed: S(x, j) ready implies P*V(x, j-1) done.  O-done is therefore
      // waited on once, for the last P*V, in the epilogue.
      for (int j = 0; j < nt; ++j) {
        wait_or_flag(p, bar(C_SFULL + x), (gt + j) & 1);
        tc_fence_after();
        const int k0 = j * TC_BN + 64 * hf;  // first key of this half
        const bool need_mask = (k0 + 64 > off + m0 + 1) || (k0 + 64 > nkeys);
        uint32_t r0[32], r1[32];
        tmem_ld32(trow + scol + 64 * hf, r0);
        tmem_ld32(trow + scol + 64 * hf + 32, r1);
        tmem_wait_ld();
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float v0 = (k0 + i < lim) ? __uint_as_float(r0[i]) : -INFINITY;
            const float v1 = (k0 + 32 + i < lim) ? __uint_as_float(r1[i]) : -INFINITY;
            r0[i] = __float_as_uint(v0);
            r1[i] = __float_as_uint(v1);
            mx4[i & 3] = fmax3f(mx4[i & 3], v0, v1);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) mx4[i & 3] = fmax3f(mx4[i & 3], __uint_as_float(r0[i]), __uint_as_float(r1[i]));
        }
        const float mx = combine(fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])), true) * p.scale_log2;
        float alpha = 1.f;
        bool resc = false;
        if (mx > m_ref + RESCALE_THRESHOLD) {  // also the first finite max (m_ref = -inf)
          alpha = ex2(m_ref - mx);
          // O holds P*V of earlier tiles once j > 0, whatever this half's own sum
          // is: both halves decide alike from the shared maximum.
          resc = j > 0;
          m_ref = mx;
        }
        const float neg_m = (m_ref == -INFINITY) ? 0.f : -m_ref;
        const float c2 = p.scale_log2;
        // P of keys [64 hf + 16 q, +16) goes to TMEM columns [32 hf + 8 q, +8) of S
        uint64_t lsum2[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int h = q >> 1;
          const uint32_t* rr = (h ? r1 : r0) + 16 * (q & 1);
          uint32_t pk[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float p0, p1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(rr[2 * i]), __uint_as_float(rr[2 * i + 1])), f2_pack(c2, c2),
                             f2_pack(neg_m, neg_m)),
                      p0, p1);
            if (emu_pair(i)) {
              exp2_fma_x2(p0, p1);
            } else {
              p0 = ex2(p0);
              p1 = ex2(p1);
            }
            if (need_mask) {
              const int kk = k0 + 16 * q + 2 * i;
              if (kk >= lim) p0 = 0.f;
              if (kk + 1 >= lim) p1 = 0.f;
            }
            lsum2[h] = f2_add(lsum2[h], f2_pack(p0, p1));
            pk[i] = pack2<MMA_BF16>(p0, p1);
          }
          tmem_st8(trow + scol + 32 * hf + 8 * q, pk);
        }
        {
          float a0, a1, b0, b1;
          f2_unpack(lsum2[0], a0, a1);
          f2_unpack(lsum2[1], b0, b1);
          l = l * alpha + ((a0 + a1) + (b0 + b1));
        }
        // Rescale this half's O columns after the logits are dead (fewer live
        // registers); P*V(j) is issued only after PFULL, so O is still P*V(<j).
        if (__any_sync(0xffffffffu, resc)) {  // O holds P*V(<j), complete (see above)
          const float a = resc ? alpha : 1.f;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t rr[32];
            tmem_ld32(trow + ocol + 32 * c, rr);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) rr[i] = __float_as_uint(__uint_as_float(rr[i]) * a);
            tmem_st32(trow + ocol + 32 * c, rr);
          }
        }
        tmem_wait_st();
        const int kt = j * TC_BN;
        if (x == 0 && nkeys - kt < TC_BN) {
          // keys past the sequence: zero their V rows (head a's P*V runs first;
          // each half zeroes its 64-column half of the row)
          wait_or_flag(p, bar(C_VFULL + (gt + j) % P2_VS), ((gt + j) / P2_VS) & 1);
          if (kt + r >= nkeys) {
            unsigned char* vrow = sm + P2_V + ((gt + j) % P2_VS) * TILE_B + hf * HALF_B + r * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(vrow + 16 * c) = make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();
        }
        tc_fence_before();
        mbar_arrive(bar(C_PFULL + x));
      }
      // ---- the next item (its Q converted now), then this item's epilogue
      int n_item, n_qlen, n_nkeys, n_off;
      take_item(it + 1, n_item, n_qlen, n_nkeys, n_off);
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(C_IEMPTY + ((it + 1) & 1)));
      if (Q_CONVERT && item_tiles(n_item, n_nkeys, n_off) > 0) convert_q(qi + (nt > 0));
      // ---- epilogue: O / l, LSE ---------------------------------------------
      const float lt = combine(l, false);
      const int hq = hq0 + x;
      const bool valid = row < qlen;
      // this thread's 64 output columns of its row, as eight 16-byte pieces
      uint4 ov[8];
      if (nt > 0) {
        wait_or_flag(p, bar(C_ODONE + x), (gt + nt - 1) & 1);  // the item's last P*V
        tc_fence_after();
        const float inv = lt > 0.f ? 1.f / lt : 0.f;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t rr[32];
          tmem_ld32(trow + ocol + 32 * c, rr);
          tmem_wait_ld();
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            ov[4 * c + v].x = pack_f16(__uint_as_float(rr[8 * v + 0]) * inv, __uint_as_float(rr[8 * v + 1]) * inv);
            ov[4 * c + v].y = pack_f16(__uint_as_float(rr[8 * v + 2]) * inv, __uint_as_float(rr[8 * v + 3]) * inv);
            ov[4 * c + v].z = pack_f16(__uint_as_float(rr[8 * v + 4]) * inv, __uint_as_float(rr[8 * v + 5]) * inv);
            ov[4 * c + v].w = pack_f16(__uint_as_float(rr[8 * v + 6]) * inv, __uint_as_float(rr[8 * v + 7]) * inv);
          }
        }
      } else {
#pragma unroll
        for (int v = 0; v < 8; ++v) ov[v] = make_uint4(0, 0, 0, 0);
      }
      // Coalesced stores: the eight lanes of a group (rows 8 g .. 8 g + 7 of
      // the warp) transpose their 8 x 8 pieces, so that store k writes row
      // 8 g + k as 128 contiguous bytes, four rows per warp instruction
      // instead of 32 scattered 16-byte pieces.
      transpose8_u4(ov, lane & 7);
      {
        const int gi = lane & 7;
        const int r0 = (warp & 3) * 32 + (lane & ~7);  // first row of this lane's group
        __half* obase = static_cast<__half*>(p.o) + o_seq_base(p, b) + hq * p.o_sh + 64 * hf + 8 * gi;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const int rw = m0 + r0 + kk;
          if (rw < qlen) *reinterpret_cast<uint4*>(obase + static_cast<long long>(rw) * p.o_sm) = ov[kk];
        }
      }
      if (valid && p.lse && hf == 0) {
        const float L = lt > 0.f ? (m_ref + lg2(lt)) * 0.6931471805599453f : -INFINITY;
        static_cast<__half*>(p.lse)[l_seq_base(p, b) + hq * p.l_sh + static_cast<long long>(row) * p.l_sm] =
            __float2half_rn(L);
      }
      gt += nt;
      qi += nt > 0;
      item = n_item;
      qlen = n_qlen;
      nkeys = n_nkeys;
      off = n_off;
    }
#endif
  }
  tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(&sched[1], 1u) == gridDim.x - 1) {  // the launch's last CTA: ready the slot for the next
      atomicExch(&sched[0], 0u);
      atomicExch(&sched[1], 0u);
    }
  }
  if (warp == P2_MMA) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

bool prefill_tc_supported(int kv_kind, int D, int BS) {
  return (kv_kind == KV_F16 || kv_kind == KV_BF16) && D == TC_D && BS >= 8;
}

cudaError_t launch_prefill_tc(const AttnParams& p_in, const CUtensorMap& kmap, const CUtensorMap& vmap,
                              const CUtensorMap& qmap, int kv_kind, cudaStream_t stream) {
  if (p_in.B == 0 || p_in.maxq == 0) return cudaSuccess;
  static std::atomic<unsigned int> generation{0};
  AttnParams p = p_in;
  p.abort_gen = ++generation;
  if (p.abort_gen == 0) p.abort_gen = ++generation;
  TcMaps maps;
  maps.k = kmap;
  maps.v = vmap;
  maps.q = qmap;
  const bool mma_bf16 = kv_kind == KV_BF16;
  const bool convert = (p.q_bf16 != 0) != mma_bf16;
  if ((p.G & 1) == 0 && !std::getenv("PIE_B200_TC_SINGLE")) {
    const long long items = static_cast<long long>(p.Hkv) * (p.G / 2) * p.B * ((p.maxq + TC_BM - 1) / TC_BM);
    if (items >= (1LL << 31)) return cudaErrorInvalidValue;
    const dim3 grid2(static_cast<unsigned>(items < device_sm_count() ? items : device_sm_count()));
    auto launch2 = [&](auto kern) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, P2_SMEM);
      if (e != cudaSuccess) return e;
      e = launch_pdl(kern, grid2, dim3(P2_THREADS), P2_SMEM, stream, p, maps);
      if (e != cudaSuccess) return e;
      return cudaGetLastError();
    };
    if (mma_bf16)
      return convert ? launch2(pa_prefill_tc2_kernel<true, true>) : launch2(pa_prefill_tc2_kernel<true, false>);
    return convert ? launch2(pa_prefill_tc2_kernel<false, true>) : launch2(pa_prefill_tc2_kernel<false, false>);
  }
  const dim3 grid(p.Hq, p.B, (p.maxq + TC_BM - 1) / TC_BM);
  auto launch = [&](auto kern) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, T1_SMEM);
    if (e != cudaSuccess) return e;
    e = launch_pdl(kern, grid, dim3(TC_THREADS), T1_SMEM, stream, p, maps);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
  };
  if (mma_bf16) return convert ? launch(pa_prefill_tc_kernel<true, true>) : launch(pa_prefill_tc_kernel<true, false>);
  return convert ? launch(pa_prefill_tc_kernel<false, true>) : launch(pa_prefill_tc_kernel<false, false>);
}

}  // namespace pa
