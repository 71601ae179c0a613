// Tiled causal paged attention for long query blocks (prefill and chunked
// prefill), warp-level mma.sync version.
//
// Replaces the q_len > 1 use of flash_attention_kernel
// (kernels/flash_attention.py:19-136): one CTA per (64 query rows, query
// head, sequence); K/V tiles of 64 keys are gathered through the block table
// row by row (any power-of-two block_size), double-buffered with cp.async,
// and consumed by m16n8k16 tensor-core MMAs with an online softmax
// (kernels/flash_attention.py:102-123) in base 2.  Causal alignment is
// bottom-right (query row m sits at kv_len - q_len + m) unless top_left is
// set; tiles above the diagonal are skipped.
//
// INT8 pools: the int8 tile and its per-key scales are staged, then every
// thread dequantises its share (q * scale in fp32, rounded once to the MMA
// type) into a 16-bit tile, the same value the reference forms before its
// dot product (kernels/flash_attention.py:83-84).
//
// FP32 pools (the reference kernel casts any float pool to fp32,
// kernels/flash_attention.py:79-84, and its tl.dot then runs in TF32 on the
// GPU): the fp32 tile is staged and rounded once to fp16, whose 11-bit
// significand equals TF32's, before the fp16 MMAs.  Values must lie inside
// the fp16 range (|x| < 65520); beyond it the rounding overflows to inf.
#include "pa_common.cuh"

namespace pa {
namespace {

constexpr int PF_BM = 64;
constexpr int PF_BN = 64;
constexpr int PF_THREADS = 128;

__device__ __forceinline__ int pf_seq_qlen(const AttnParams& p, int b) { return seq_rows(p, b); }

__device__ __forceinline__ int pf_seq_keys(const AttnParams& p, int b) {
  const int q = pf_seq_qlen(p, b);
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

template <int D, int KVT>
struct PfCfg {
  static constexpr bool INT8 = KVT == KV_I8;
  static constexpr bool F32 = KVT == KV_F32;
  static constexpr bool CONV = INT8 || F32;  // staged tiles converted to 16-bit operands
  static constexpr int ELT = INT8 ? 1 : F32 ? 4 : 2;
  static constexpr int ROWB = D * 2;  // 16-bit operand rows
  static constexpr int CH = ROWB / 16;
  static constexpr int TB = PF_BN * ROWB;
  static constexpr int QB = PF_BM * ROWB;
  static constexpr int RAWROWB = D * ELT;
  static constexpr int RAWCH = RAWROWB / 16;
  static constexpr int RAWTB = PF_BN * RAWROWB;
  static constexpr int SCB = INT8 ? (2 * PF_BN * 4 + 32) : 0;  // K/V scale words + 4 mask words (+pad)
  static constexpr int STAGEB = 2 * RAWTB + SCB;
  static constexpr int CONVB = CONV ? 2 * TB : 0;
  static constexpr int SMEM = QB + 2 * STAGEB + CONVB;
};

__device__ __forceinline__ int swz16(int row, int c) { return c ^ (row & 7); }

template <int D, int KVT>
__device__ __forceinline__ void pf_load_kv(const AttnParams& p, const int* bt_row, int nkeys, int kvh, int k0,
                                           unsigned char* st, int tid) {
  using C = PfCfg<D, KVT>;
  constexpr int ELT = C::ELT;
  constexpr int TOTAL = PF_BN * C::RAWCH;
  const char* kbase = static_cast<const char*>(p.k);
  const char* vbase = static_cast<const char*>(p.v);
  const uint32_t sk = smem_u32(st);
  const uint32_t sv = sk + C::RAWTB;
#pragma unroll
  for (int it = 0; it < TOTAL / PF_THREADS; ++it) {
    const int c = it * PF_THREADS + tid;
    const int row = c / C::RAWCH;
    const int ch = c % C::RAWCH;
    const int key = k0 + row;
    bool ok = key < nkeys;
    int blk = 0, slot = 0;
    if (ok) {
      blk = __ldg(bt_row + static_cast<long long>(key >> p.log2BS) * p.bt_sc);
      slot = key & (p.BS - 1);
      if (blk < 0 || blk >= p.NB) {
        set_status(p.status, ST_BAD_BLOCK_ID);
        ok = false;
      }
    }
    const char* ksrc = kbase;
    const char* vsrc = vbase;
    if (ok) {
      ksrc = kbase + (blk * p.k_sblk + slot * p.k_sslot + kvh * p.k_shead) * ELT + ch * 16;
      vsrc = vbase + (blk * p.v_sblk + slot * p.v_sslot + kvh * p.v_shead) * ELT + ch * 16;
    }
    const int pc = C::CONV ? ch : swz16(row, ch);
    cp_async_16(sk + row * C::RAWROWB + pc * 16, ksrc, ok ? 16 : 0);
    cp_async_16(sv + row * C::RAWROWB + pc * 16, vsrc, ok ? 16 : 0);
  }
  if constexpr (C::INT8) {
    // threads 0..63: K scale of key row tid; 64..127: V scale of row tid-64
    const int row = tid & (PF_BN - 1);
    const bool isv = tid >= PF_BN;
    const int key = k0 + row;
    bool ok = key < nkeys;
    int blk = 0, slot = 0;
    if (ok) {
      blk = __ldg(bt_row + static_cast<long long>(key >> p.log2BS) * p.bt_sc);
      slot = key & (p.BS - 1);
      ok = blk >= 0 && blk < p.NB;
    }
    unsigned long long addr = reinterpret_cast<unsigned long long>(isv ? p.vs : p.ks);
    if (ok) {
      const long long off = isv ? (blk * p.vs_sblk + slot * p.vs_sslot + kvh * p.vs_shead)
                                : (blk * p.ks_sblk + slot * p.ks_sslot + kvh * p.ks_shead);
      addr += static_cast<unsigned long long>(off) * (p.scale_f32 ? 4 : 2);
    }
    const unsigned hi = (!p.scale_f32 && ((addr >> 1) & 1)) ? 1u : 0u;
    const unsigned mask = __ballot_sync(0xffffffffu, hi);
    const uint32_t ss = sv + C::RAWTB;
    cp_async_4(ss + tid * 4, reinterpret_cast<const void*>(addr & ~3ull), ok ? 4 : 0);
    if ((tid & 31) == 0) *reinterpret_cast<unsigned*>(st + 2 * C::RAWTB + 2 * PF_BN * 4 + (tid >> 5) * 4) = mask;
  }
}

// INT8 stage -> dequantised 16-bit tiles (K and V), swizzled for ldmatrix.
template <int D, bool MB>
__device__ __forceinline__ void pf_convert(const unsigned char* st, unsigned char* conv, int scale_f32, int tid) {
  using C = PfCfg<D, KV_I8>;
  const uint32_t* sw = reinterpret_cast<const uint32_t*>(st + 2 * C::RAWTB);
  const unsigned* masks = reinterpret_cast<const unsigned*>(st + 2 * C::RAWTB + 2 * PF_BN * 4);
  constexpr int TOTAL = 2 * PF_BN * C::RAWCH;  // chunks of 16 int8 over K and V
#pragma unroll
  for (int it = 0; it < TOTAL / PF_THREADS; ++it) {
    const int c = it * PF_THREADS + tid;
    const int isv = c / (PF_BN * C::RAWCH);
    const int cc = c % (PF_BN * C::RAWCH);
    const int row = cc / C::RAWCH;
    const int ch = cc % C::RAWCH;
    const int sidx = isv * PF_BN + row;
    const uint32_t w = sw[sidx];
    const bool hi = (masks[sidx >> 5] >> (sidx & 31)) & 1;
    float sc;
    if (scale_f32) sc = __uint_as_float(w);
    else sc = __half2float(__ushort_as_half(hi ? static_cast<unsigned short>(w >> 16) : static_cast<unsigned short>(w)));
    const uint4 raw = *reinterpret_cast<const uint4*>(st + isv * C::RAWTB + row * C::RAWROWB + ch * 16);
    const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t out[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int8_t* b = reinterpret_cast<const int8_t*>(&rw[k]);
      out[2 * k] = pack2<MB>(static_cast<float>(b[0]) * sc, static_cast<float>(b[1]) * sc);
      out[2 * k + 1] = pack2<MB>(static_cast<float>(b[2]) * sc, static_cast<float>(b[3]) * sc);
    }
    unsigned char* dst = conv + isv * C::TB + row * C::ROWB;
    *reinterpret_cast<uint4*>(dst + swz16(row, 2 * ch) * 16) = make_uint4(out[0], out[1], out[2], out[3]);
    *reinterpret_cast<uint4*>(dst + swz16(row, 2 * ch + 1) * 16) = make_uint4(out[4], out[5], out[6], out[7]);
  }
}

// FP32 stage -> 16-bit tiles (K and V), swizzled for ldmatrix: each thread
// turns two 16-byte chunks of fp32 (8 values) into one chunk of fp16.
template <int D>
__device__ __forceinline__ void pf_convert_f32(const unsigned char* st, unsigned char* conv, int tid) {
  using C = PfCfg<D, KV_F32>;
  constexpr int TOTAL = 2 * PF_BN * C::CH;  // 16-bit output chunks over K and V
#pragma unroll
  for (int it = 0; it < TOTAL / PF_THREADS; ++it) {
    const int c = it * PF_THREADS + tid;
    const int isv = c / (PF_BN * C::CH);
    const int cc = c % (PF_BN * C::CH);
    const int row = cc / C::CH;
    const int ch = cc % C::CH;
    const float4* src = reinterpret_cast<const float4*>(st + isv * C::RAWTB + row * C::RAWROWB + ch * 32);
    const float4 a = src[0];
    const float4 b = src[1];
    unsigned char* dst = conv + isv * C::TB + row * C::ROWB;
    *reinterpret_cast<uint4*>(dst + swz16(row, ch) * 16) =
        make_uint4(pack2<false>(a.x, a.y), pack2<false>(a.z, a.w), pack2<false>(b.x, b.y), pack2<false>(b.z, b.w));
  }
}

template <int D, int KVT, int QT>
__global__ void __launch_bounds__(PF_THREADS) pa_prefill_kernel(const AttnParams p) {
  pdl_enter();
  using C = PfCfg<D, KVT>;
  constexpr bool INT8 = C::INT8;
  constexpr bool MB = (KVT == KV_BF16);
  constexpr bool QB16 = (QT == Q_BF16);
  constexpr int KS = D / 16;  // k-steps over head_dim
  constexpr int NTS = PF_BN / 8;  // n-tiles of S
  constexpr int NTO = D / 8;      // n-tiles of O

  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* sq = smem;
  unsigned char* stage0 = smem + C::QB;
  unsigned char* conv = stage0 + 2 * C::STAGEB;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int r = lane >> 2;
  const int q4 = lane & 3;

  const int mtile = gridDim.x - 1 - blockIdx.x;
  const int hq = blockIdx.y;
  const int b = blockIdx.z;
  const int qlen = pf_seq_qlen(p, b);
  const int m0 = mtile * PF_BM;
  if (m0 >= qlen) return;
  const int kvh = hq / p.G;
  const int nkeys = pf_seq_keys(p, b);
  const int off = p.top_left ? 0 : p.kvlen[b] - qlen;
  const int kend = min(nkeys, off + m0 + PF_BM);
  const int ntile = kend > 0 ? (kend + PF_BN - 1) / PF_BN : 0;
  const int* bt_row = p.bt + static_cast<long long>(b) * p.bt_ss;

  // ---- Q tile ---------------------------------------------------------------
  {
    const unsigned short* qbase = static_cast<const unsigned short*>(p.q) + q_seq_base(p, b) + hq * p.q_sh;
#pragma unroll
    for (int it = 0; it < PF_BM * C::CH / PF_THREADS; ++it) {
      const int c = it * PF_THREADS + tid;
      const int row = c / C::CH;
      const int ch = c % C::CH;
      const int qi = m0 + row;
      const bool ok = qi < qlen;
      const unsigned short* src = ok ? qbase + static_cast<long long>(qi) * p.q_sm + ch * 8 : qbase;
      cp_async_16(smem_u32(sq + row * C::ROWB + swz16(row, ch) * 16), src, ok ? 16 : 0);
    }
  }
  if (ntile > 0) pf_load_kv<D, KVT>(p, bt_row, nkeys, kvh, 0, stage0, tid);
  cp_async_commit();

  if constexpr (QB16 != MB) {
    cp_async_wait<0>();
    __syncthreads();
    // convert the Q tile in place to the MMA element type
    for (int i = tid; i < PF_BM * D / 2; i += PF_THREADS) {
      uint32_t* w = reinterpret_cast<uint32_t*>(sq) + i;
      *w = cvt_pair<QB16, MB>(*w);
    }
  }

  float acc[NTO][4];
#pragma unroll
  for (int n = 0; n < NTO; ++n)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[n][c] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  const int qi_a = m0 + warp * 16 + r;
  const int qi_b = qi_a + 8;
  const int lim_a = min(nkeys, off + qi_a + 1);
  const int lim_b = min(nkeys, off + qi_b + 1);
  uint32_t qa[KS][4];

  for (int t = 0; t < ntile; ++t) {
    if (t + 1 < ntile) pf_load_kv<D, KVT>(p, bt_row, nkeys, kvh, (t + 1) * PF_BN, stage0 + ((t + 1) & 1) * C::STAGEB, tid);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (t == 0) {
      const int j = lane >> 3;
      const int row = warp * 16 + (lane & 7) + 8 * (j & 1);
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        const int ch = 2 * kk + (j >> 1);
        ldsm_x4(smem_u32(sq + row * C::ROWB + swz16(row, ch) * 16), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
      }
    }
    const unsigned char* st = stage0 + (t & 1) * C::STAGEB;
    const unsigned char* kt;
    const unsigned char* vt;
    if constexpr (C::CONV) {
      if constexpr (INT8) pf_convert<D, MB>(st, conv, p.scale_f32, tid);
      else pf_convert_f32<D>(st, conv, tid);
      __syncthreads();
      kt = conv;
      vt = conv + C::TB;
    } else {
      kt = st;
      vt = st + C::RAWTB;
    }
    const int k0 = t * PF_BN;

    // ---- S = Q K^T ---------------------------------------------------------
    float s[NTS][4];
#pragma unroll
    for (int n = 0; n < NTS; ++n)
#pragma unroll
      for (int c = 0; c < 4; ++c) s[n][c] = 0.f;
    {
      const int j = lane >> 3;
#pragma unroll
      for (int np = 0; np < NTS / 2; ++np) {
        const int row = np * 16 + (lane & 7) + 8 * (j >> 1);
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
          uint32_t b0, b1, b2, b3;
          const int ch = 2 * kk + (j & 1);
          ldsm_x4(smem_u32(kt + row * C::ROWB + swz16(row, ch) * 16), b0, b1, b2, b3);
          mma16816<MB>(s[2 * np], qa[kk], b0, b1);
          mma16816<MB>(s[2 * np + 1], qa[kk], b2, b3);
        }
      }
    }

    // ---- online softmax ----------------------------------------------------
    const bool need_mask = (k0 + PF_BN > off + m0 + 1) || (k0 + PF_BN > nkeys);
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < NTS; ++n) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float x = s[n][c] * p.scale_log2;
        if (need_mask) {
          const int key = k0 + 8 * n + 2 * q4 + (c & 1);
          const int lim = (c < 2) ? lim_a : lim_b;
          if (key >= lim) x = -INFINITY;
        }
        s[n][c] = x;
        mx[c >> 1] = fmaxf(mx[c >> 1], x);
      }
    }
    float alpha[2], m_use[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
      const float m_new = fmaxf(m_run[h], mx[h]);
      m_use[h] = (m_new == -INFINITY) ? 0.f : m_new;
      alpha[h] = ex2(m_run[h] - m_use[h]);
      m_run[h] = m_new;
      l_run[h] *= alpha[h];
    }
#pragma unroll
    for (int n = 0; n < NTO; ++n) {
      acc[n][0] *= alpha[0];
      acc[n][1] *= alpha[0];
      acc[n][2] *= alpha[1];
      acc[n][3] *= alpha[1];
    }
    uint32_t pa_[NTS / 2][4];
#pragma unroll
    for (int n = 0; n < NTS; ++n) {
      const float p0 = ex2(s[n][0] - m_use[0]);
      const float p1 = ex2(s[n][1] - m_use[0]);
      const float p2 = ex2(s[n][2] - m_use[1]);
      const float p3 = ex2(s[n][3] - m_use[1]);
      l_run[0] += p0 + p1;
      l_run[1] += p2 + p3;
      pa_[n >> 1][(n & 1) * 2 + 0] = pack2<MB>(p0, p1);
      pa_[n >> 1][(n & 1) * 2 + 1] = pack2<MB>(p2, p3);
    }

    // ---- O += P V ----------------------------------------------------------
    {
      const int j = lane >> 3;
#pragma unroll
      for (int kk = 0; kk < PF_BN / 16; ++kk) {
        const int row = kk * 16 + (lane & 7) + 8 * (j & 1);
#pragma unroll
        for (int np = 0; np < NTO / 2; ++np) {
          uint32_t b0, b1, b2, b3;
          const int ch = 2 * np + (j >> 1);
          ldsm_x4_t(smem_u32(vt + row * C::ROWB + swz16(row, ch) * 16), b0, b1, b2, b3);
          mma16816<MB>(acc[2 * np], pa_[kk], b0, b1);
          mma16816<MB>(acc[2 * np + 1], pa_[kk], b2, b3);
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // ---- epilogue ---------------------------------------------------------------
  float lt[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    lt[h] = l_run[h];
    lt[h] += __shfl_xor_sync(0xffffffffu, lt[h], 1);
    lt[h] += __shfl_xor_sync(0xffffffffu, lt[h], 2);
  }
  __half* obase = static_cast<__half*>(p.o) + o_seq_base(p, b) + hq * p.o_sh;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int qi = h ? qi_b : qi_a;
    if (qi >= qlen) continue;
    const float inv = lt[h] > 0.f ? 1.f / lt[h] : 0.f;
    __half* orow = obase + static_cast<long long>(qi) * p.o_sm;
#pragma unroll
    for (int n = 0; n < NTO; ++n) {
      *reinterpret_cast<uint32_t*>(orow + 8 * n + 2 * q4) = pack_f16(acc[n][2 * h] * inv, acc[n][2 * h + 1] * inv);
    }
    if (q4 == 0 && p.lse) {
      const float L = lt[h] > 0.f ? (m_run[h] + lg2(lt[h])) * 0.6931471805599453f : -INFINITY;
      static_cast<__half*>(p.lse)[l_seq_base(p, b) + hq * p.l_sh + static_cast<long long>(qi) * p.l_sm] =
          __float2half_rn(L);
    }
  }
}

template <int D, int KVT, int QT>
cudaError_t pf_launch(const AttnParams& p, cudaStream_t stream) {
  using C = PfCfg<D, KVT>;
  auto kern = pa_prefill_kernel<D, KVT, QT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const dim3 grid((p.maxq + PF_BM - 1) / PF_BM, p.Hq, p.B);
  const cudaError_t le = launch_pdl(kern, grid, dim3(PF_THREADS), C::SMEM, stream, p);
  if (le != cudaSuccess) return le;
  return cudaGetLastError();
}

template <int D>
cudaError_t pf_dispatch(const AttnParams& p, int kv, cudaStream_t s) {
  const bool qbf = p.q_bf16 != 0;
  if (kv == KV_F16) return qbf ? pf_launch<D, KV_F16, Q_BF16>(p, s) : pf_launch<D, KV_F16, Q_F16>(p, s);
  if (kv == KV_BF16) return qbf ? pf_launch<D, KV_BF16, Q_BF16>(p, s) : pf_launch<D, KV_BF16, Q_F16>(p, s);
  if (kv == KV_F32) return qbf ? pf_launch<D, KV_F32, Q_BF16>(p, s) : pf_launch<D, KV_F32, Q_F16>(p, s);
  return qbf ? pf_launch<D, KV_I8, Q_BF16>(p, s) : pf_launch<D, KV_I8, Q_F16>(p, s);
}

}  // namespace

cudaError_t launch_prefill(const AttnParams& p, int kv_kind, int D, int /*mma_bf16*/, cudaStream_t stream) {
  if (p.B == 0 || p.maxq == 0) return cudaSuccess;
  if (D == 64) return pf_dispatch<64>(p, kv_kind, stream);
  if (D == 128) return pf_dispatch<128>(p, kv_kind, stream);
  return cudaErrorInvalidValue;
}

}  // namespace pa
