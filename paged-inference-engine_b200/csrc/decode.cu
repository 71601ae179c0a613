// Split-K ("flash-decoding") paged attention for short query blocks.
//
// Replaces the q_len == 1 use of flash_attention_kernel
// (kernels/flash_attention.py:19-136), whose grid
// (batch, heads, cdiv(max_q_len, BLOCK_M)) gives one program per (sequence,
// head) that walks the block table serially (:58) with >= 31 of 32 MMA rows
// idle, and reads every KV head once per query head.
//
// Design (B200, HBM-bound):
//  * Work unit = a TILE of 16 keys (32 for int8 pools) of one (sequence, kv head) SEGMENT.  All tiles
//    of all segments form one flat list (segment-major); a persistent grid of
//    W warps gives warp w the contiguous range [w*chunk, (w+1)*chunk) with
//    chunk = ceil(total / W) ("stream-K"): every warp streams the same number
//    of KV bytes however skewed the context lengths are.
//  * Each warp is an independent worker with a private ring of STAGES tiles.
//    Lane 0 fetches a tile's K and V with TMA boxes (4-D tensor maps over the
//    pool [block, slot, head, d], 128-byte swizzle, mbarrier completion) --
//    a handful of bulk copies per 8 KB instead of 512 16-byte requests; pools
//    with block_size < 8 use per-lane cp.async into the same layout.  Loads
//    for the next tiles, also across segment boundaries, are in flight while
//    the current tile is computed.  No CTA barrier in the main loop.
//  * Grouped-query packing: the G = Hq/Hkv query heads (times q_len rows)
//    of a KV head form the N=8*NT columns of a transposed product
//    S^T = K * Q^T (mma.sync m16n8k16, keys in M), so each KV tile is read
//    once per KV head and feeds all its query heads.
//  * Online softmax in base 2 with the softmax scale folded into one multiply;
//    P^T goes through 256 bytes of shared memory (ldmatrix.trans) into the B
//    operand of O^T = V^T * P^T.
//  * INT8 KV: the tile stays int8 in shared memory; fragments are converted
//    with an exact prmt/hsub2 int8->fp16 sequence.  The per-key K scale is
//    applied to the logits and the per-key V scale to P before the PV
//    product -- algebraically the reference's dequantise-then-dot
//    (kernels/flash_attention.py:83-88,113).
//  * A segment split across warps leaves fp32 partials (m, l, o) in the
//    workspace; pa_decode_merge_kernel combines them.  Segments inside one
//    warp's range are written straight to O / L.
#include "pa_common.cuh"

namespace pa {
namespace {

constexpr int NC_MAX = 16;      // max packed columns (q rows x group heads)
// Worker warps per CTA (upper bound): 12 for single-n-tile variants (<= 170
// registers per thread), 8 for the two-n-tile ones.
template <int NT>
constexpr int max_warps() { return NT == 1 ? 12 : 8; }
constexpr int SMEM_LIMIT = 227 * 1024;
constexpr int META_B = 16;      // per stage: [0] fp16 half-select mask of the scale words, [1] missing rows
// Shared-memory bytes of tile ring per warp (16-bit pools / int8 pools).
#ifndef PA_DEC_STAGE_BUDGET
#define PA_DEC_STAGE_BUDGET (22 * 1024)
#endif
#ifndef PA_DEC_STAGE_BUDGET_I8
#define PA_DEC_STAGE_BUDGET_I8 (17 * 1024)
#endif

#ifndef PA_DEC_TILE_I8
#define PA_DEC_TILE_I8 32
#endif
// INT8 pools: S = Q K^T on the integer MMA (PA_DEC_I8_IMMA = 1).  Each packed
// Q column is quantised once per piece to 16-bit fixed point against its own
// absmax (q ~ s_q * (256 * hi + lo), hi and lo int8) and the raw int8 K tile is
// the A operand as it sits in shared memory: two m16n8k32 chains (hi, lo) give
// sum_d k_d * v_d exactly in int32, so no K byte is converted.  Q keeps 15 bits
// against its column maximum (an absolute error of amax / 65024 per element,
// below fp16's 2^-11 relative for every element above amax / 32); the
// reference dots a TF32-rounded Q.  0 keeps the fp16 path with biased operands.
#ifndef PA_DEC_I8_IMMA
#define PA_DEC_I8_IMMA 1
#endif

template <int D, int KVT>
struct DecCfg {
  static constexpr bool INT8 = KVT == KV_I8;
  static constexpr int ELT = INT8 ? 1 : 2;
  // Keys per tile: 16 for 16-bit pools (8 KB of K+V at D=128), 32 for int8
  // pools, so an int8 tile carries as many bytes and twice the independent
  // MMA / conversion chains per softmax step.
  static constexpr int TK = INT8 ? PA_DEC_TILE_I8 : 16;
  static constexpr int KST = TK / 16;                  // 16-key MMA steps per tile
  static constexpr int MAXBOX = TK / 8;                // TMA boxes per tile (block_size >= 8)
  static constexpr int ROWB = D * ELT;                 // bytes of one key row of one head
  static constexpr int CHUNKS = ROWB / 16;
  static constexpr int TILEB = TK * ROWB;              // K (or V) tile bytes, multiple of 1024
  static constexpr int HALVES = ROWB >= 128 ? ROWB / 128 : 1;  // TMA boxes across head_dim
  static constexpr int BOXD = (ROWB >= 128 ? 128 : ROWB) / ELT;
  static constexpr int SCB = (INT8 ? 8 * TK : 0) + META_B;  // K + V scale words, then meta
  static constexpr int STAGE_RAW = 2 * TILEB + SCB + 8;
  static constexpr int STAGES_RAW = (INT8 ? PA_DEC_STAGE_BUDGET_I8 : PA_DEC_STAGE_BUDGET) / STAGE_RAW;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : (STAGES_RAW < 2 ? 2 : STAGES_RAW);
  static constexpr int ROWS_PER_IT = 32 / CHUNKS;
  static constexpr int LOAD_ITS = TK / ROWS_PER_IT;
  static_assert(TK == 16 || TK == 32, "tiles hold 16 or 32 keys");
  static_assert(TILEB % 1024 == 0, "tiles must keep TMA swizzle atoms aligned");
};

template <int D, int KVT, int NT>
struct DecLayout {
  using C = DecCfg<D, KVT>;
  static constexpr int S = C::STAGES;
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = S * C::TILEB;
  static constexpr int SC_OFF = 2 * S * C::TILEB;
  static constexpr int BAR_OFF = SC_OFF + S * C::SCB;
  static constexpr int P_OFF = (BAR_OFF + S * 8 + 15) & ~15;  // ldmatrix rows need 16-byte alignment
  static constexpr int PB = C::TK * 8 * NT * 2;
  static constexpr int WARPB = ((P_OFF + PB) + 1023) & ~1023;
  static_assert(V_OFF % 1024 == 0 && C::TILEB % 1024 == 0, "TMA boxes need 1024-byte aligned tiles");
  static_assert(SC_OFF % 16 == 0 && C::SCB % 16 == 0, "scale words / meta must stay 16-byte aligned");
  static_assert(BAR_OFF % 8 == 0, "mbarriers need 8-byte alignment");
  static_assert(P_OFF % 16 == 0 && WARPB % 1024 == 0, "P buffer / warp regions alignment");
};

// Byte offset of 16-byte chunk `ch` of key row `row` inside a tile of TK
// rows.  This is the layout TMA writes with SWIZZLE_128B (128-byte rows, one
// box column of TK x 128 bytes per 128 bytes of head_dim) or SWIZZLE_64B
// (64-byte rows); the cp.async loader writes the same layout.  The XOR makes
// the ldmatrix / LDS fragment reads bank-conflict free (2-way for INT8 K at
// D=128).
template <int ROWB, int TK>
__device__ __forceinline__ int toff(int row, int ch) {
  if constexpr (ROWB >= 128) return (ch >> 3) * (TK * 128) + row * 128 + (((ch & 7) ^ (row & 7)) << 4);
  else return row * 64 + ((ch ^ ((row >> 1) & 3)) << 4);
}

// Row mask of a whole tile.
template <int TK>
__device__ __forceinline__ unsigned tile_rows() { return TK == 32 ? 0xffffffffu : ((1u << TK) - 1u); }

// Query rows of sequence b, never more than the rows Q holds.
__device__ __forceinline__ int seq_qlen(const AttnParams& p, int b) { return seq_rows(p, b); }

__device__ __forceinline__ int seq_keys(const AttnParams& p, int b) {
  const int q = seq_qlen(p, b);
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

struct Cursor {
  int b, kvh, tile, nt;
  int nkeys;
  const int* bt_row;
};

__device__ __forceinline__ void cursor_seq(const AttnParams& p, const int* ts, Cursor& c) {
  c.nt = ts[c.b + 1] - ts[c.b];
  c.nkeys = seq_keys(p, c.b);
  c.bt_row = p.bt + static_cast<long long>(c.b) * p.bt_ss;
}

__device__ __forceinline__ void cursor_locate(const AttnParams& p, const int* ts, int g, Cursor& c) {
  int lo = 0, hi = p.B - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (ts[mid] * p.Hkv <= g) lo = mid;
    else hi = mid - 1;
  }
  c.b = lo;
  cursor_seq(p, ts, c);
  const int rem = g - ts[lo] * p.Hkv;
  c.kvh = rem / c.nt;
  c.tile = rem - c.kvh * c.nt;
}

__device__ __forceinline__ void cursor_next(const AttnParams& p, const int* ts, Cursor& c) {
  if (++c.tile < c.nt) return;
  c.tile = 0;
  if (++c.kvh < p.Hkv) return;
  c.kvh = 0;
  do {
    ++c.b;
  } while (c.b < p.B && ts[c.b + 1] == ts[c.b]);
  if (c.b < p.B) cursor_seq(p, ts, c);
}

// Scale words of one tile (INT8).  In pass h, lanes 0..15 fetch the K scale
// of rows 16h..16h+15 and lanes 16..31 the V scale, each as the aligned 4-byte
// word holding it; the fp16 half-select bits go to meta words 0 (K) and 2 (V).
// rb[h] is the block id of this lane's row in pass h.
template <int TK>
__device__ __forceinline__ void load_scales(const AttnParams& p, const Cursor& c, unsigned char* sc, unsigned* meta,
                                            int lane, const int (&rb)[TK / 16]) {
  const bool isv = lane >= 16;
  unsigned kmask = 0, vmask = 0;
#pragma unroll
  for (int h = 0; h < TK / 16; ++h) {
    const int row = (lane & 15) + 16 * h;
    const int key = c.tile * TK + row;
    const int blk = rb[h];
    const bool ok = key < c.nkeys && blk >= 0 && blk < p.NB;
    const int slot = key & (p.BS - 1);
    unsigned long long addr = reinterpret_cast<unsigned long long>(isv ? p.vs : p.ks);
    if (ok) {
      const long long off = isv ? (blk * p.vs_sblk + slot * p.vs_sslot + c.kvh * p.vs_shead)
                                : (blk * p.ks_sblk + slot * p.ks_sslot + c.kvh * p.ks_shead);
      addr += static_cast<unsigned long long>(off) * (p.scale_f32 ? 4 : 2);
    }
    const unsigned hi = (!p.scale_f32 && ((addr >> 1) & 1)) ? 1u : 0u;
    const unsigned m = __ballot_sync(0xffffffffu, hi);
    kmask |= (m & 0xffffu) << (16 * h);
    vmask |= (m >> 16) << (16 * h);
    cp_async_4(smem_u32(sc) + (isv ? 4 * TK : 0) + row * 4, reinterpret_cast<const void*>(addr & ~3ull), ok ? 4 : 0);
  }
  if (lane == 0) {
    meta[0] = kmask;
    meta[2] = vmask;
  }
}

// TMA fetch of one tile (lane 0): one box of min(16, block_size) slots per
// block touched and per 128 bytes of head_dim, for K and for V.  bx[j] is
// the block id of box j.  Rows that are not fetched (beyond the sequence, or
// of a block id outside the pool) are recorded in the stage's "missing rows"
// mask.
template <int D, int KVT>
__device__ __forceinline__ void issue_tile_tma(const AttnParams& p, const KvMaps& maps, const Cursor& c,
                                               uint32_t kdst, uint32_t vdst, uint32_t bar, unsigned* meta,
                                               const int (&bx)[DecCfg<D, KVT>::MAXBOX]) {
  using C = DecCfg<D, KVT>;
  constexpr int TK = C::TK;
  constexpr int RB = C::ROWB >= 128 ? 128 : C::ROWB;
  const int key0 = c.tile * TK;
  const int boxs = p.BS < 16 ? p.BS : 16;  // 8 or 16 (TMA mode needs block_size >= 8)
  const int nbox = TK / boxs;
  unsigned missing = 0;
  unsigned fetch = 0;
  uint32_t bytes = 0;
#pragma unroll
  for (int j = 0; j < C::MAXBOX; ++j) {
    if (j >= nbox) break;
    const int k = key0 + j * boxs;
    const unsigned rows = ((1u << boxs) - 1u) << (j * boxs);
    if (k >= c.nkeys) {
      missing |= rows;
      continue;
    }
    if (bx[j] < 0 || bx[j] >= p.NB) {
      set_status(p.status, ST_BAD_BLOCK_ID);
      missing |= rows;
      continue;
    }
    fetch |= 1u << j;
    bytes += 2u * C::HALVES * boxs * RB;
  }
  const int valid = c.nkeys - key0;
  if (valid < TK) missing |= tile_rows<TK>() & ~(valid > 0 ? ((1u << valid) - 1u) : 0u);
  meta[1] = missing;
  mbar_arrive_expect_tx(bar, bytes);
#pragma unroll
  for (int j = 0; j < C::MAXBOX; ++j) {
    if (!((fetch >> j) & 1u)) continue;
    const int slot = (key0 + j * boxs) & (p.BS - 1);
#pragma unroll
    for (int h = 0; h < C::HALVES; ++h) {
      const uint32_t off = h * (TK * 128) + j * boxs * RB;
      tma_load_4d(kdst + off, &maps.k, bar, h * C::BOXD, c.kvh, slot, bx[j]);
      tma_load_4d(vdst + off, &maps.v, bar, h * C::BOXD, c.kvh, slot, bx[j]);
    }
  }
}

// cp.async fetch of one tile (all lanes), for pools TMA boxes cannot cover
// (block_size < 8).  Missing rows are zero-filled.
template <int D, int KVT>
__device__ __forceinline__ void issue_tile_cpasync(const AttnParams& p, const Cursor& c, uint32_t kdst,
                                                   uint32_t vdst, unsigned* meta, int lane) {
  using C = DecCfg<D, KVT>;
  constexpr int TK = C::TK;
  const int key0 = c.tile * TK;
  const char* kbase = static_cast<const char*>(p.k);
  const char* vbase = static_cast<const char*>(p.v);
  const int ch = lane % C::CHUNKS;
#pragma unroll
  for (int it = 0; it < C::LOAD_ITS; ++it) {
    const int row = it * C::ROWS_PER_IT + lane / C::CHUNKS;
    const int key = key0 + row;
    bool ok = key < c.nkeys;
    int blk = 0, slot = 0;
    if (ok) {
      blk = __ldg(c.bt_row + static_cast<long long>(key >> p.log2BS) * p.bt_sc);
      slot = key & (p.BS - 1);
      if (blk < 0 || blk >= p.NB) {
        set_status(p.status, ST_BAD_BLOCK_ID);
        ok = false;
      }
    }
    const char* ksrc = kbase;
    const char* vsrc = vbase;
    if (ok) {
      ksrc = kbase + (blk * p.k_sblk + slot * p.k_sslot + c.kvh * p.k_shead) * C::ELT + ch * 16;
      vsrc = vbase + (blk * p.v_sblk + slot * p.v_sslot + c.kvh * p.v_shead) * C::ELT + ch * 16;
    }
    cp_async_16(kdst + toff<C::ROWB, TK>(row, ch), ksrc, ok ? 16 : 0);
    cp_async_16(vdst + toff<C::ROWB, TK>(row, ch), vsrc, ok ? 16 : 0);
  }
  if (lane == 0) meta[1] = 0u;
}

__device__ __forceinline__ float scale_from_word(uint32_t w, bool hi, int is_f32) {
  if (is_f32) return __uint_as_float(w);
  const unsigned short h = hi ? static_cast<unsigned short>(w >> 16) : static_cast<unsigned short>(w & 0xffffu);
  return __half2float(__ushort_as_half(h));
}

template <int D, int KVT, int QT, int NT, bool TMA>
__global__ void __launch_bounds__(max_warps<NT>() * 32, 1)
    pa_decode_kernel(const AttnParams p, const __grid_constant__ KvMaps maps) {
  pdl_enter();
  using C = DecCfg<D, KVT>;
  using Lay = DecLayout<D, KVT, NT>;
  constexpr int STAGES = C::STAGES;
  constexpr bool INT8 = C::INT8;
  constexpr int TK = C::TK;
  constexpr int KST = C::KST;
  constexpr bool MMA_BF16 = (KVT == KV_BF16);
  constexpr bool QIS_BF16 = (QT == Q_BF16);
  constexpr bool USE_CPASYNC = !TMA || INT8;  // cp.async carries tiles (no TMA) or scale words (INT8)
  constexpr bool IMMA = INT8 && PA_DEC_I8_IMMA;  // integer Q*K^T (see PA_DEC_I8_IMMA)
  constexpr int KS = D / 16;  // k-steps over head_dim / m-tiles of O^T
  constexpr int NC = 8 * NT;

  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int NW = blockDim.x >> 5;
  int* s_ts = reinterpret_cast<int*>(smem_raw);
  const int ts_bytes = ((p.B + 1) * 4 + 127) & ~127;
  // warp regions start on a 1024-byte boundary (TMA swizzle atoms)
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t wbase_u32 = ((raw_u32 + ts_bytes + 1023) & ~1023u) + warp * Lay::WARPB;
  unsigned char* wsm = smem_raw + (wbase_u32 - raw_u32);
  unsigned char* pbuf = wsm + Lay::P_OFF;

  // ---- prologue: tiles per sequence and their exclusive scan -------------
  for (int i = tid; i < p.B; i += NW * 32) {
    const int nk = seq_keys(p, i);
    if (p.nblk[i] > p.bt_cols) set_status(p.status, ST_BAD_NUM_BLOCKS);
    s_ts[i] = (nk + TK - 1) / TK;
  }
  if constexpr (TMA) {
    if (lane == 0) {
      for (int s = 0; s < STAGES; ++s) mbar_init(wbase_u32 + Lay::BAR_OFF + 8 * s, 1);
      fence_mbar_init();
    }
  }
  __syncthreads();
  if (warp == 0) {
    int carry = 0;
    for (int base = 0; base < p.B; base += 32) {
      const int i = base + lane;
      const int v = i < p.B ? s_ts[i] : 0;
      int x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (i < p.B) s_ts[i] = carry + x - v;
      carry += __shfl_sync(0xffffffffu, x, 31);
    }
    if (lane == 0) s_ts[p.B] = carry;
  }
  __syncthreads();
  if (blockIdx.x == 0) {
    for (int i = tid; i <= p.B; i += NW * 32) p.tstart[i] = s_ts[i];
  }

  const int total = s_ts[p.B] * p.Hkv;
  const int W = p.num_warps_total;
  const int chunk = (total + W - 1) / W;
  const int gw = blockIdx.x * NW + warp;
  const int g0 = gw * chunk;
  const int g1 = min(g0 + chunk, total);
  if (total == 0 || g0 >= g1) return;

  const int r = lane >> 2;  // fragment row group
  const int q4 = lane & 3;  // thread in group

  Cursor ld, cp;
  cursor_locate(p, s_ts, g0, ld);
  cp = ld;

  // ---- block-table window (TMA path) ---------------------------------------
  // Lane l holds the block id of box (l mod nbox) of tile win_base + l / nbox
  // of this warp's range; the next window is loaded one window ahead, so no
  // dependent block-table read sits between a tile's issue and its compute.
  const int lnb = (TK == 32 ? 1 : 0) + (p.BS < 16 ? 1 : 0);  // log2(boxes per tile)
  const int lbs = p.BS < 16 ? 3 : 4;                           // log2(box rows)
  const int wt = 32 >> lnb;                                    // tiles per window
  auto fetch_window = [&](int t0) -> int {
    const int g = g0 + t0 + (lane >> lnb);
    int v = 0;
    if (g < g1) {
      Cursor c;
      cursor_locate(p, s_ts, g, c);
      const int key = c.tile * TK + ((lane & ((1 << lnb) - 1)) << lbs);
      if (key < c.nkeys) v = __ldg(c.bt_row + static_cast<long long>(key >> p.log2BS) * p.bt_sc);
    }
    return v;
  };
  int win_base = 0, win_cur = 0, win_nxt = 0;
  if constexpr (TMA) {
    win_cur = fetch_window(0);
    win_nxt = fetch_window(wt);
  }

  auto issue = [&](int ti, int slot_idx) {
    const uint32_t kdst = wbase_u32 + Lay::K_OFF + slot_idx * C::TILEB;
    const uint32_t vdst = wbase_u32 + Lay::V_OFF + slot_idx * C::TILEB;
    unsigned char* sc = wsm + Lay::SC_OFF + slot_idx * C::SCB;
    unsigned* meta = reinterpret_cast<unsigned*>(sc + (INT8 ? 8 * TK : 0));
    int rb[KST];
    if constexpr (TMA) {
      if (ti - win_base >= wt) {
        win_cur = win_nxt;
        win_base += wt;
        win_nxt = fetch_window(win_base + wt);
      }
      const int sl = (ti - win_base) << lnb;
      int bx[C::MAXBOX];
#pragma unroll
      for (int j = 0; j < C::MAXBOX; ++j) bx[j] = __shfl_sync(0xffffffffu, win_cur, (sl + j) & 31);
      if (lane == 0) issue_tile_tma<D, KVT>(p, maps, ld, kdst, vdst, wbase_u32 + Lay::BAR_OFF + 8 * slot_idx, meta, bx);
      if constexpr (INT8) {
#pragma unroll
        for (int h = 0; h < KST; ++h)
          rb[h] = __shfl_sync(0xffffffffu, win_cur, (sl + (((lane & 15) + 16 * h) >> lbs)) & 31);
      }
    } else {
      issue_tile_cpasync<D, KVT>(p, ld, kdst, vdst, meta, lane);
      if constexpr (INT8) {
#pragma unroll
        for (int h = 0; h < KST; ++h) {
          const int key = ld.tile * TK + (lane & 15) + 16 * h;
          rb[h] = key < ld.nkeys ? __ldg(ld.bt_row + static_cast<long long>(key >> p.log2BS) * p.bt_sc) : 0;
        }
      }
    }
    if constexpr (INT8) load_scales<TK>(p, ld, sc, meta, lane, rb);
  };

#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (g0 + s < g1) {
      issue(s, s);
      cursor_next(p, s_ts, ld);
    }
    if constexpr (USE_CPASYNC) cp_async_commit();
  }

  uint32_t qf[NT][KS][2];
  float acc[KS][NT][4];
  float m_run[NT][2], l_run[NT][2];
  int lim[NT][2];
  int lim_min = 0;      // fewest visible keys over the warp's columns (warp-uniform)
  // INT8 (biased operands): I8_BIAS * sum_d q_d of this thread's S columns, and
  // the per-column sum of P' accumulated by an MMA with an all-ones A operand.
  // With the integer Q*K^T (IMMA) qs holds the columns' fixed-point scales instead.
  float qs[NT][2];
  float acc1[NT][4];
  float qscale_own[NT];  // IMMA: this thread's column (nt*8 + r) scale
  int piece_start_tile = 0;
  int qlen_b = 0;
  bool piece_first = true;  // first piece of this warp's range
  bool zeroed_prev = false;

  for (int g = g0; g < g1; ++g) {
    const int i = g - g0;
    // ---- prefetch tile i + STAGES - 1 into the slot freed last iteration --
    if constexpr (TMA) {
      if (zeroed_prev) fence_proxy_async_smem();  // generic zero-fill before the next TMA write
    }
    __syncwarp();
    if (g + STAGES - 1 < g1) {
      issue(i + STAGES - 1, (i + STAGES - 1) % STAGES);
      cursor_next(p, s_ts, ld);
    }
    if constexpr (USE_CPASYNC) cp_async_commit();

    const bool pstart = (g == g0) || (cp.tile == 0);
    const bool pend = (g == g1 - 1) || (cp.tile == cp.nt - 1);
    if (pstart) {
      qlen_b = seq_qlen(p, cp.b);
      piece_start_tile = cp.tile;
      // ---- Q^T fragments of the packed (q row, group head) columns -------
      const int off = p.top_left ? 0 : (p.kvlen[cp.b] - qlen_b);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int col = nt * 8 + r;
        const int qi = col / p.G;
        const int hq = col - qi * p.G;
        const bool valid = qi < qlen_b;
        const unsigned short* qrow = static_cast<const unsigned short*>(p.q) + q_seq_base(p, cp.b) +
                                     (cp.kvh * p.G + hq) * p.q_sh + static_cast<long long>(qi) * p.q_sm;
        if constexpr (!INT8) {
#pragma unroll
          for (int kk = 0; kk < KS; ++kk) {
            uint32_t w0 = 0, w1 = 0;
            if (valid) {
              w0 = *reinterpret_cast<const uint32_t*>(qrow + 16 * kk + 2 * q4);
              w1 = *reinterpret_cast<const uint32_t*>(qrow + 16 * kk + 8 + 2 * q4);
            }
            qf[nt][kk][0] = cvt_pair<QIS_BF16, MMA_BF16>(w0);
            qf[nt][kk][1] = cvt_pair<QIS_BF16, MMA_BF16>(w1);
          }
        } else if constexpr (IMMA) {
          // this thread's 16 values of column nt*8 + r per 64 of head_dim (d = 64 gg + 16 q4 + 0..15)
          float f[D / 64][16];
          float amax = 0.f;
#pragma unroll
          for (int gg = 0; gg < D / 64; ++gg) {
            uint4 a = make_uint4(0, 0, 0, 0), bq = make_uint4(0, 0, 0, 0);
            if (valid) {
              const uint4* src = reinterpret_cast<const uint4*>(qrow + 64 * gg + 16 * q4);
              a = src[0];
              bq = src[1];
            }
            const uint32_t w[8] = {a.x, a.y, a.z, a.w, bq.x, bq.y, bq.z, bq.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float2 v;
              if constexpr (QIS_BF16) v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
              else v = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
              f[gg][2 * j] = v.x;
              f[gg][2 * j + 1] = v.y;
              amax = fmaxf(amax, fmaxf(fabsf(v.x), fabsf(v.y)));
            }
          }
          // the column's absmax over head_dim: the four threads of the row group
          amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
          amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
          const float inv = amax > 0.f ? 32512.f / amax : 0.f;
          qscale_own[nt] = amax * (1.f / 32512.f);
#pragma unroll
          for (int gg = 0; gg < D / 64; ++gg)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint32_t hi = 0, lo = 0;
#pragma unroll
              for (int b8 = 0; b8 < 4; ++b8) {
                const int v = __float2int_rn(f[gg][4 * j + b8] * inv);  // |v| <= 32512
                const int h = (v + 128) >> 8;                             // [-127, 127]
                const int l = v - (h << 8);                               // [-128, 127]
                hi |= static_cast<uint32_t>(h & 0xff) << (8 * b8);
                lo |= static_cast<uint32_t>(l & 0xff) << (8 * b8);
              }
              qf[nt][4 * gg + j][0] = hi;
              qf[nt][4 * gg + j][1] = lo;
            }
        } else {
#pragma unroll
          for (int gg = 0; gg < D / 64; ++gg) {
            uint4 a = make_uint4(0, 0, 0, 0), bq = make_uint4(0, 0, 0, 0);
            if (valid) {
              const uint4* src = reinterpret_cast<const uint4*>(qrow + 64 * gg + 16 * q4);
              a = src[0];
              bq = src[1];
            }
            const uint32_t w[8] = {a.x, a.y, a.z, a.w, bq.x, bq.y, bq.z, bq.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              qf[nt][4 * gg + j][0] = cvt_pair<QIS_BF16, false>(w[2 * j]);
              qf[nt][4 * gg + j][1] = cvt_pair<QIS_BF16, false>(w[2 * j + 1]);
            }
          }
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int c2 = nt * 8 + 2 * q4 + e;
          const int qi2 = c2 / p.G;
          int L = cp.nkeys;
          if (qi2 < qlen_b) {
            const int vis = off + qi2 + 1;
            L = min(L, vis);
          }
          lim[nt][e] = L;
          m_run[nt][e] = -INFINITY;
          l_run[nt][e] = 0.f;
        }
      }
#pragma unroll
      for (int mt = 0; mt < KS; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[mt][nt][c] = 0.f;
      int lm = lim[0][0];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) lm = min(lm, min(lim[nt][0], lim[nt][1]));
      lim_min = __reduce_min_sync(0xffffffffu, lm);
      if constexpr (IMMA) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          // S fragment columns nt*8 + 2 q4 + e: their fixed-point scale, from a thread of that column
#pragma unroll
          for (int e = 0; e < 2; ++e) qs[nt][e] = __shfl_sync(0xffffffffu, qscale_own[nt], (2 * q4 + e) << 2);
#pragma unroll
          for (int c = 0; c < 4; ++c) acc1[nt][c] = 0.f;
        }
      } else if constexpr (INT8) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          // this thread's Q fragments are column nt*8 + r; sum over the four
          // threads of the row group gives the column's sum over head_dim
          float part = 0.f;
#pragma unroll
          for (int kk = 0; kk < KS; ++kk)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&qf[nt][kk][hf]));
              part += f.x + f.y;
            }
          part += __shfl_xor_sync(0xffffffffu, part, 1);
          part += __shfl_xor_sync(0xffffffffu, part, 2);
#pragma unroll
          for (int e = 0; e < 2; ++e) qs[nt][e] = I8_BIAS * __shfl_sync(0xffffffffu, part, (2 * q4 + e) << 2);
#pragma unroll
          for (int c = 0; c < 4; ++c) acc1[nt][c] = 0.f;
        }
      }
    }

    // ---- wait for this tile ----------------------------------------------
    const int slot_idx = i % STAGES;
    if constexpr (USE_CPASYNC) cp_async_wait<STAGES - 1>();
    if constexpr (TMA) {
      if (!mbar_wait(wbase_u32 + Lay::BAR_OFF + 8 * slot_idx, (i / STAGES) & 1) && lane == 0)
        set_status(p.status, ST_WAIT_TIMEOUT);
    }
    __syncwarp();
    unsigned char* kt = wsm + Lay::K_OFF + slot_idx * C::TILEB;
    unsigned char* vt = wsm + Lay::V_OFF + slot_idx * C::TILEB;
    unsigned char* sc = wsm + Lay::SC_OFF + slot_idx * C::SCB;
    const unsigned* meta = reinterpret_cast<const unsigned*>(sc + (INT8 ? 8 * TK : 0));
    const uint32_t sk = smem_u32(kt);
    const uint32_t sv = smem_u32(vt);
    zeroed_prev = false;
    if constexpr (TMA && !INT8) {
      // rows not fetched (or past the sequence) may hold stale or non-finite
      // bytes: zero them in V so that P = 0 really contributes nothing.
      const unsigned missing = meta[1];
      if (missing) {
        for (int idx = lane; idx < TK * C::CHUNKS; idx += 32) {
          const int row = idx / C::CHUNKS;
          if ((missing >> row) & 1u)
            *reinterpret_cast<uint4*>(vt + toff<C::ROWB, TK>(row, idx % C::CHUNKS)) = make_uint4(0, 0, 0, 0);
        }
        zeroed_prev = true;
        __syncwarp();
      }
    }

    // ---- S^T = K * Q^T, one m-tile per 16 keys ------------------------------
    // s / s2: two independent accumulation chains per m-tile (even / odd
    // k-steps) halve the dependent-MMA latency.
    float s[KST][NT][4], s2[KST][NT][4];
#pragma unroll
    for (int mk = 0; mk < KST; ++mk)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[mk][nt][c] = s2[mk][nt][c] = 0.f;
    if constexpr (!INT8) {
      const int j = lane >> 3;
      const int row = (lane & 7) + 8 * (j & 1);
#pragma unroll
      for (int mk = 0; mk < KST; ++mk)
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
          uint32_t a[4];
          ldsm_x4(sk + toff<C::ROWB, TK>(row + 16 * mk, 2 * kk + (j >> 1)), a[0], a[1], a[2], a[3]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            if (kk & 1) mma16816<MMA_BF16>(s2[mk][nt], a, qf[nt][kk][0], qf[nt][kk][1]);
            else mma16816<MMA_BF16>(s[mk][nt], a, qf[nt][kk][0], qf[nt][kk][1]);
          }
        }
    } else if constexpr (IMMA) {
      // raw int8 K rows r / r+8 as A, Q's hi / lo bytes as B: two exact int32 chains
      int sh[KST][NT][4], sl[KST][NT][4];
#pragma unroll
      for (int mk = 0; mk < KST; ++mk)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int c = 0; c < 4; ++c) sh[mk][nt][c] = sl[mk][nt][c] = 0;
#pragma unroll
      for (int gg = 0; gg < D / 64; ++gg) {
        const int chn = 4 * gg + q4;
#pragma unroll
        for (int mk = 0; mk < KST; ++mk) {
          const uint4 w0 = *reinterpret_cast<const uint4*>(kt + toff<C::ROWB, TK>(r + 16 * mk, chn));
          const uint4 w1 = *reinterpret_cast<const uint4*>(kt + toff<C::ROWB, TK>(r + 8 + 16 * mk, chn));
          const uint32_t x0[4] = {w0.x, w0.y, w0.z, w0.w};
          const uint32_t x1[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
          for (int jj = 0; jj < 4; jj += 2) {
            const uint32_t a[4] = {x0[jj], x1[jj], x0[jj + 1], x1[jj + 1]};
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              mma_s8_16832(sh[mk][nt], a, qf[nt][4 * gg + jj][0], qf[nt][4 * gg + jj + 1][0]);
              mma_s8_16832(sl[mk][nt], a, qf[nt][4 * gg + jj][1], qf[nt][4 * gg + jj + 1][1]);
            }
          }
        }
      }
#pragma unroll
      for (int mk = 0; mk < KST; ++mk)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int c = 0; c < 4; ++c) s[mk][nt][c] = __int2float_rn(sh[mk][nt][c] * 256 + sl[mk][nt][c]);
    } else {
#pragma unroll
      for (int gg = 0; gg < D / 64; ++gg) {
        const int chn = 4 * gg + q4;
#pragma unroll
        for (int mk = 0; mk < KST; ++mk) {
          const uint4 w0 = *reinterpret_cast<const uint4*>(kt + toff<C::ROWB, TK>(r + 16 * mk, chn));
          const uint4 w1 = *reinterpret_cast<const uint4*>(kt + toff<C::ROWB, TK>(r + 8 + 16 * mk, chn));
          const uint32_t x0[4] = {w0.x, w0.y, w0.z, w0.w};
          const uint32_t x1[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            uint32_t a[4];
            i8x4_to_f16x4_biased(x0[jj], a[0], a[2]);
            i8x4_to_f16x4_biased(x1[jj], a[1], a[3]);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              if (jj & 1) mma16816<false>(s2[mk][nt], a, qf[nt][4 * gg + jj][0], qf[nt][4 * gg + jj][1]);
              else mma16816<false>(s[mk][nt], a, qf[nt][4 * gg + jj][0], qf[nt][4 * gg + jj][1]);
            }
          }
        }
      }
    }
#pragma unroll
    for (int mk = 0; mk < KST; ++mk)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[mk][nt][c] += s2[mk][nt][c];

    // ---- per-row logit multiplier (K scale x softmax scale) and V scale -----
    // rows r + 8*hh + 16*mk
    float kscl[KST][2], vsc[KST][2];
#pragma unroll
    for (int mk = 0; mk < KST; ++mk)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        kscl[mk][hh] = p.scale_log2;
        vsc[mk][hh] = 1.f;
        if constexpr (INT8) {
          const uint32_t* sw = reinterpret_cast<const uint32_t*>(sc);
          const int row = r + 8 * hh + 16 * mk;
          kscl[mk][hh] = scale_from_word(sw[row], (meta[0] >> row) & 1, p.scale_f32) * p.scale_log2;
          vsc[mk][hh] = scale_from_word(sw[TK + row], (meta[2] >> row) & 1, p.scale_f32);
        }
      }

    // ---- online softmax (base 2) ------------------------------------------
    // The reference max of a column only moves when a logit exceeds it by
    // more than 2^8 (or on the piece's first tile): P stays <= 256, and most
    // tiles skip the cross-lane max, the alpha exponentials and the rescale.
    const int key_r = cp.tile * TK + r;
    const bool full = (cp.tile + 1) * TK <= lim_min;  // every key of the tile visible to every column
    uint32_t* pw = reinterpret_cast<uint32_t*>(pbuf);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float pv[KST][4];
      float x[2][KST][2];
      float tm[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        tm[e] = -INFINITY;
#pragma unroll
        for (int mk = 0; mk < KST; ++mk)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            float sv = s[mk][nt][e + 2 * hh];
            if constexpr (IMMA) sv *= qs[nt][e];
            else if constexpr (INT8) sv -= qs[nt][e];
            float v = sv * kscl[mk][hh];
            if (!full && key_r + 16 * mk + 8 * hh >= lim[nt][e]) v = -INFINITY;
            x[e][mk][hh] = v;
            tm[e] = fmaxf(tm[e], v);
          }
      }
      if (!__all_sync(0xffffffffu, tm[0] <= m_run[nt][0] + 8.f && tm[1] <= m_run[nt][1] + 8.f)) {
        float alpha[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float m_new = fmaxf(m_run[nt][e], warp_max_xor(tm[e], 4));
          const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
          alpha[e] = ex2(m_run[nt][e] - m_use);
          l_run[nt][e] *= alpha[e];
          m_run[nt][e] = m_new;
        }
        if (!__all_sync(0xffffffffu, alpha[0] == 1.f && alpha[1] == 1.f)) {
#pragma unroll
          for (int mt = 0; mt < KS; ++mt) {
            acc[mt][nt][0] *= alpha[0];
            acc[mt][nt][1] *= alpha[1];
            acc[mt][nt][2] *= alpha[0];
            acc[mt][nt][3] *= alpha[1];
          }
          if constexpr (INT8) {
            acc1[nt][0] *= alpha[0];
            acc1[nt][1] *= alpha[1];
            acc1[nt][2] *= alpha[0];
            acc1[nt][3] *= alpha[1];
          }
        }
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float m_use = (m_run[nt][e] == -INFINITY) ? 0.f : m_run[nt][e];
        float ps = 0.f;
#pragma unroll
        for (int mk = 0; mk < KST; ++mk)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const float pe = ex2(x[e][mk][hh] - m_use);
            pv[mk][e + 2 * hh] = pe;
            ps += pe;
          }
        l_run[nt][e] += ps;
      }
      // P^T tile [key][col] (fp16 or bf16, V scale folded in for INT8)
#pragma unroll
      for (int mk = 0; mk < KST; ++mk) {
        pw[((r + 16 * mk) * NC + nt * 8 + 2 * q4) >> 1] =
            pack2<MMA_BF16>(pv[mk][0] * vsc[mk][0], pv[mk][1] * vsc[mk][0]);
        pw[((r + 8 + 16 * mk) * NC + nt * 8 + 2 * q4) >> 1] =
            pack2<MMA_BF16>(pv[mk][2] * vsc[mk][1], pv[mk][3] * vsc[mk][1]);
      }
    }
    __syncwarp();
    uint32_t bp[KST][NT][2];
    {
      const uint32_t pb = smem_u32(pbuf);
      if constexpr (NT == 1) {
        if constexpr (KST == 1) ldsm_x2_t(pb + (lane & 15) * NC * 2, bp[0][0][0], bp[0][0][1]);
        else ldsm_x4_t(pb + lane * NC * 2, bp[0][0][0], bp[0][0][1], bp[1][0][0], bp[1][0][1]);
      } else {
#pragma unroll
        for (int mk = 0; mk < KST; ++mk) {
          const int row = (lane & 15) + 16 * mk;
          const int colb = (lane >> 4) * 8;
          ldsm_x4_t(pb + (row * NC + colb) * 2, bp[mk][0][0], bp[mk][0][1], bp[mk][1][0], bp[mk][1][1]);
        }
      }
    }

    // ---- O^T += V^T * P^T ---------------------------------------------------
    if constexpr (!INT8) {
      const int j = lane >> 3;
      const int row = (lane & 7) + 8 * (j >> 1);
#pragma unroll
      for (int mk = 0; mk < KST; ++mk)
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          uint32_t a[4];
          ldsm_x4_t(sv + toff<C::ROWB, TK>(row + 16 * mk, 2 * mt + (j & 1)), a[0], a[1], a[2], a[3]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) mma16816<MMA_BF16>(acc[mt][nt], a, bp[mk][nt][0], bp[mk][nt][1]);
        }
    } else {
      constexpr int WORDS = D / 32;  // 32-bit words of this thread's d range per key
#pragma unroll
      for (int mk = 0; mk < KST; ++mk) {
        uint32_t R[4][WORDS];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int row = 16 * mk + 2 * q4 + (c & 1) + 8 * (c >> 1);
          if constexpr (D >= 128) {
            const uint4 w = *reinterpret_cast<const uint4*>(vt + toff<C::ROWB, TK>(row, r));
            R[c][0] = w.x;
            R[c][1] = w.y;
            R[c][2] = w.z;
            R[c][3] = w.w;
          } else {
            const uint2 w = *reinterpret_cast<const uint2*>(vt + toff<C::ROWB, TK>(row, r >> 1) + (r & 1) * 8);
            R[c][0] = w.x;
            R[c][1] = w.y;
          }
        }
#pragma unroll
        for (int w = 0; w < WORDS; ++w) {
          const uint32_t x01 = prmt(R[0][w], R[1][w], 0x5140u);
          const uint32_t y01 = prmt(R[0][w], R[1][w], 0x7362u);
          const uint32_t x23 = prmt(R[2][w], R[3][w], 0x5140u);
          const uint32_t y23 = prmt(R[2][w], R[3][w], 0x7362u);
          uint32_t a[4], b2[4];
          i8x4_to_f16x4_biased(x01, a[0], a[1]);
          i8x4_to_f16x4_biased(x23, a[2], a[3]);
          i8x4_to_f16x4_biased(y01, b2[0], b2[1]);
          i8x4_to_f16x4_biased(y23, b2[2], b2[3]);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            mma16816<false>(acc[2 * w][nt], a, bp[mk][nt][0], bp[mk][nt][1]);
            mma16816<false>(acc[2 * w + 1][nt], b2, bp[mk][nt][0], bp[mk][nt][1]);
          }
        }
        // sum over keys of P' per column, accumulated exactly like O'
        const uint32_t ones[4] = {0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u};
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) mma16816<false>(acc1[nt], ones, bp[mk][nt][0], bp[mk][nt][1]);
      }
    }

    // ---- end of a piece: final output or split-K partial ------------------
    if (pend) {
      const bool complete = (piece_start_tile == 0) && (cp.tile == cp.nt - 1);
      if constexpr (INT8) {
        // O' = O + I8_BIAS * sum_k P'_k per column
#pragma unroll
        for (int mt = 0; mt < KS; ++mt)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[mt][nt][c] -= I8_BIAS * acc1[nt][c & 1];
      }
      const int slot = piece_first ? 2 * gw : 2 * gw + 1;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float lt = warp_sum_xor(l_run[nt][e], 4);
          const int col = nt * 8 + 2 * q4 + e;
          const int qi = col / p.G;
          const int hq = col - qi * p.G;
          const bool valid = (qi < qlen_b) && (col < NC);
          if (complete) {
            const float inv = lt > 0.f ? 1.f / lt : 0.f;
            if (valid) {
              const long long orow = o_seq_base(p, cp.b) + (cp.kvh * p.G + hq) * p.o_sh +
                                     static_cast<long long>(qi) * p.o_sm;
#pragma unroll
              for (int mt = 0; mt < KS; ++mt)
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                  const int d = INT8 ? (D / 8) * r + 2 * mt + hf : 16 * mt + r + 8 * hf;
                  store_o(p, orow + d, __float2half_rn(acc[mt][nt][e + 2 * hf] * inv));
                }
              if (r == 0 && p.lse) {
                const float L = lt > 0.f ? (m_run[nt][e] + lg2(lt)) * 0.6931471805599453f : -INFINITY;
                static_cast<__half*>(p.lse)[l_seq_base(p, cp.b) + (cp.kvh * p.G + hq) * p.l_sh +
                                            static_cast<long long>(qi) * p.l_sm] = __float2half_rn(L);
              }
            }
          } else {
            float* po = p.part_o + (static_cast<long long>(slot) * NC_MAX + col) * D;
#pragma unroll
            for (int mt = 0; mt < KS; ++mt)
#pragma unroll
              for (int hf = 0; hf < 2; ++hf) {
                const int d = INT8 ? (D / 8) * r + 2 * mt + hf : 16 * mt + r + 8 * hf;
                po[d] = acc[mt][nt][e + 2 * hf];
              }
            if (r == 0) {
              float* pm = p.part_ml + (static_cast<long long>(slot) * NC_MAX + col) * 2;
              pm[0] = m_run[nt][e];
              pm[1] = lt;
            }
          }
        }
      }
      piece_first = false;
    }
    cursor_next(p, s_ts, cp);
  }
  if constexpr (USE_CPASYNC) cp_async_wait<0>();
  peer_store_fence(p);
}

// Combine the split-K partials of every segment that straddles warp ranges.
// grid (Hkv, B), 128 threads.
template <int D>
__global__ void __launch_bounds__(128) pa_decode_merge_kernel(const AttnParams p) {
  pdl_enter();
  const int kvh = blockIdx.x;
  const int b = blockIdx.y;
  const int qlen = seq_qlen(p, b);
  if (qlen <= 0) return;
  const int ncols = min(qlen * p.G, NC_MAX);
  const int nt_b = p.tstart[b + 1] - p.tstart[b];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (nt_b == 0) {
    // no visible keys: O = 0, L = -inf
    for (int col = warp; col < ncols; col += 4) {
      const int qi = col / p.G, hq = col - (col / p.G) * p.G;
      const long long orow = o_seq_base(p, b) + (kvh * p.G + hq) * p.o_sh + static_cast<long long>(qi) * p.o_sm;
      for (int d = lane; d < D; d += 32) store_o(p, orow + d, __float2half_rn(0.f));
      if (lane == 0 && p.lse)
        static_cast<__half*>(p.lse)[l_seq_base(p, b) + (kvh * p.G + hq) * p.l_sh + static_cast<long long>(qi) * p.l_sm] =
            __float2half_rn(-INFINITY);
    }
    peer_store_fence(p);
    return;
  }
  const int total = p.tstart[p.B] * p.Hkv;
  const int W = p.num_warps_total;
  const int chunk = (total + W - 1) / W;
  const int S0 = p.tstart[b] * p.Hkv + kvh * nt_b;
  const int S1 = S0 + nt_b;
  const int w0 = S0 / chunk;
  const int w1 = (S1 - 1) / chunk;
  if (w0 == w1) return;  // written directly by the split kernel
  // slot of warp w's partial for this segment: its second slot when the segment starts inside w's range
  auto slot_of = [&](int w) { return (w == w0 && w0 * chunk < S0) ? 2 * w + 1 : 2 * w; };
  for (int col = warp; col < ncols; col += 4) {
    const int qi = col / p.G, hq = col - (col / p.G) * p.G;
    // lane i reads partial w0 + i (32 at a time): the maxima and the sums are
    // warp reductions instead of a chain of dependent L2 reads
    float M = -INFINITY;
    for (int w = w0 + lane; w <= w1; w += 32)
      M = fmaxf(M, p.part_ml[(static_cast<long long>(slot_of(w)) * NC_MAX + col) * 2]);
    M = warp_max_xor(M, 1);
    const float Mu = (M == -INFINITY) ? 0.f : M;
    float l = 0.f;
    float o[D / 32];
#pragma unroll
    for (int k = 0; k < D / 32; ++k) o[k] = 0.f;
    for (int base = w0; base <= w1; base += 32) {
      float f = 0.f;
      if (base + lane <= w1) {
        const float* pm = p.part_ml + (static_cast<long long>(slot_of(base + lane)) * NC_MAX + col) * 2;
        f = ex2(pm[0] - Mu);
        l += pm[1] * f;
      }
      const int n = min(32, w1 - base + 1);
#pragma unroll 4
      for (int j = 0; j < n; ++j) {
        const float fj = __shfl_sync(0xffffffffu, f, j);
        const float* po = p.part_o + (static_cast<long long>(slot_of(base + j)) * NC_MAX + col) * D;
#pragma unroll
        for (int k = 0; k < D / 32; ++k) o[k] += po[lane + 32 * k] * fj;
      }
    }
    l = warp_sum_xor(l, 1);
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const long long orow = o_seq_base(p, b) + (kvh * p.G + hq) * p.o_sh + static_cast<long long>(qi) * p.o_sm;
#pragma unroll
    for (int k = 0; k < D / 32; ++k) store_o(p, orow + lane + 32 * k, __float2half_rn(o[k] * inv));
    if (lane == 0 && p.lse) {
      const float L = l > 0.f ? (M + lg2(l)) * 0.6931471805599453f : -INFINITY;
      static_cast<__half*>(p.lse)[l_seq_base(p, b) + (kvh * p.G + hq) * p.l_sh + static_cast<long long>(qi) * p.l_sm] =
          __float2half_rn(L);
    }
  }
  peer_store_fence(p);
}

template <int D, int KVT, int QT, int NT, bool TMA>
struct DecodeInst {
  using Lay = DecLayout<D, KVT, NT>;
  static int plan(int B, DecodeLaunch* out) {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    const int ts_bytes = ((B + 1) * 4 + 127) & ~127;
    const int fixed = ts_bytes + 1024;  // scan + alignment slack
    int nw = (SMEM_LIMIT - fixed) / Lay::WARPB;
    if (nw > max_warps<NT>()) nw = max_warps<NT>();
    if (nw < 1) return -1;
    out->warps_per_cta = nw;
    out->smem = static_cast<size_t>(fixed + nw * Lay::WARPB);
    auto kern = pa_decode_kernel<D, KVT, QT, NT, TMA>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(out->smem)) !=
        cudaSuccess)
      return -1;
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, nw * 32, out->smem);
    if (per_sm < 1) per_sm = 1;
    out->ctas = sms * per_sm;
    return 0;
  }
  static cudaError_t launch(const AttnParams& p, const KvMaps& maps, const DecodeLaunch& pl, int phase,
                            cudaStream_t stream) {
    cudaError_t e;
    if (phase != DECODE_MERGE) {
      auto kern = pa_decode_kernel<D, KVT, QT, NT, TMA>;
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(pl.smem));
      if (e != cudaSuccess) return e;
      e = launch_pdl(kern, dim3(pl.ctas), dim3(pl.warps_per_cta * 32), pl.smem, stream, p, maps);
      if (e != cudaSuccess) return e;
      e = cudaGetLastError();
      if (e != cudaSuccess) return e;
      if (phase == DECODE_SPLIT) return cudaSuccess;
    }
    e = launch_pdl(pa_decode_merge_kernel<D>, dim3(p.Hkv, p.B), dim3(128), 0, stream, p);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
  }
};

template <int D, int KVT, int QT>
struct Sel {
  static int plan(int nt, int B, bool tma, DecodeLaunch* o) {
    if (nt == 1) return tma ? DecodeInst<D, KVT, QT, 1, true>::plan(B, o) : DecodeInst<D, KVT, QT, 1, false>::plan(B, o);
    return tma ? DecodeInst<D, KVT, QT, 2, true>::plan(B, o) : DecodeInst<D, KVT, QT, 2, false>::plan(B, o);
  }
  static cudaError_t launch(const AttnParams& p, const KvMaps& m, int nt, bool tma, const DecodeLaunch& pl, int ph,
                            cudaStream_t s) {
    if (nt == 1)
      return tma ? DecodeInst<D, KVT, QT, 1, true>::launch(p, m, pl, ph, s)
                 : DecodeInst<D, KVT, QT, 1, false>::launch(p, m, pl, ph, s);
    return tma ? DecodeInst<D, KVT, QT, 2, true>::launch(p, m, pl, ph, s)
               : DecodeInst<D, KVT, QT, 2, false>::launch(p, m, pl, ph, s);
  }
};

template <int D>
int plan_kv(int kv, int qbf, int nt, int B, bool tma, DecodeLaunch* o) {
  if (kv == KV_F16) return qbf ? Sel<D, KV_F16, Q_BF16>::plan(nt, B, tma, o) : Sel<D, KV_F16, Q_F16>::plan(nt, B, tma, o);
  if (kv == KV_BF16) return qbf ? Sel<D, KV_BF16, Q_BF16>::plan(nt, B, tma, o) : Sel<D, KV_BF16, Q_F16>::plan(nt, B, tma, o);
  return qbf ? Sel<D, KV_I8, Q_BF16>::plan(nt, B, tma, o) : Sel<D, KV_I8, Q_F16>::plan(nt, B, tma, o);
}
template <int D>
cudaError_t launch_kv(const AttnParams& p, const KvMaps& m, int kv, int qbf, int nt, bool tma, const DecodeLaunch& pl,
                      int ph, cudaStream_t s) {
  if (ph == DECODE_MERGE)  // the merge kernel depends on head_dim only
    return Sel<D, KV_F16, Q_F16>::launch(p, m, nt, tma, pl, ph, s);
  if (kv == KV_F16)
    return qbf ? Sel<D, KV_F16, Q_BF16>::launch(p, m, nt, tma, pl, ph, s)
               : Sel<D, KV_F16, Q_F16>::launch(p, m, nt, tma, pl, ph, s);
  if (kv == KV_BF16)
    return qbf ? Sel<D, KV_BF16, Q_BF16>::launch(p, m, nt, tma, pl, ph, s)
               : Sel<D, KV_BF16, Q_F16>::launch(p, m, nt, tma, pl, ph, s);
  return qbf ? Sel<D, KV_I8, Q_BF16>::launch(p, m, nt, tma, pl, ph, s)
             : Sel<D, KV_I8, Q_F16>::launch(p, m, nt, tma, pl, ph, s);
}

}  // namespace

int decode_plan(int kv_kind, int q_bf16, int D, int nt, int B, int use_tma, DecodeLaunch* out) {
  if (D == 64) return plan_kv<64>(kv_kind, q_bf16, nt, B, use_tma != 0, out);
  if (D == 128) return plan_kv<128>(kv_kind, q_bf16, nt, B, use_tma != 0, out);
  return -1;
}

namespace {
// One CTA: thread t posts `epoch` into slot `rank` of peer t's flags, then
// waits for slot t of this GPU's flags to reach `epoch` (system-scope
// release / acquire; each wait gives up after ~0.4 s with a status bit).
// A peer can pass this barrier as soon as this GPU has posted, run its next
// step and post epoch + 1 before this GPU has read the slot, so any value at
// or past `epoch` ends the wait (a peer is never more than one epoch ahead).
__global__ void __launch_bounds__(32) pa_peer_barrier_kernel(int* local_flags, const PeerFlags peers, int n,
                                                              int rank, int epoch, int* status) {
  pdl_enter();
  const int t = threadIdx.x;
  if (t < n) {
    asm volatile("fence.acq_rel.sys;\n" ::: "memory");
    asm volatile("st.release.sys.global.b32 [%0], %1;\n" ::"l"(peers.flag[t] + rank), "r"(epoch) : "memory");
  }
  __syncwarp();
  if (t < n) {
    bool ok = false;
    for (int i = 0; i < (1 << 22); ++i) {
      int v;
      asm volatile("ld.acquire.sys.global.b32 %0, [%1];\n" : "=r"(v) : "l"(local_flags + t) : "memory");
      if (v - epoch >= 0) {  // epochs only grow; a peer may already have posted the next one
        ok = true;
        break;
      }
      __nanosleep(100);
    }
    if (!ok) set_status(status, ST_PEER_TIMEOUT);
  }
  __syncwarp();
}
}  // namespace

cudaError_t launch_peer_barrier(int* local_flags, const PeerFlags& peers, int n, int rank, int epoch, int* status,
                                cudaStream_t stream) {
  if (n < 1 || n > kMaxPeers) return cudaErrorInvalidValue;
  cudaError_t e = launch_pdl(pa_peer_barrier_kernel, dim3(1), dim3(32), 0, stream, local_flags, peers, n, rank, epoch,
                             status);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_decode(const AttnParams& p, const KvMaps* maps, int kv_kind, int q_bf16, int D, int nt,
                          const DecodeLaunch& plan, cudaStream_t stream, int phase) {
  KvMaps none{};
  const KvMaps& m = maps ? *maps : none;
  const bool tma = maps != nullptr;
  if (D == 64) return launch_kv<64>(p, m, kv_kind, q_bf16, nt, tma, plan, phase, stream);
  if (D == 128) return launch_kv<128>(p, m, kv_kind, q_bf16, nt, tma, plan, phase, stream);
  return cudaErrorInvalidValue;
}

}  // namespace pa
