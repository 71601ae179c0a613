// Quantise-on-write / copy-on-write of new K/V rows into the paged pool.
//
// Replaces the per-token Python loop of transformer/model.py:85-122 (which
// issues ~12 torch launches and two host syncs per token per layer) with one
// launch: one warp per (token, kv head) row.
//
// INT8 rule (per row of head_dim values, all arithmetic in IEEE fp32):
//   absmax = max_d |x_d|
//   scale  = absmax / 127            (1.0 when absmax == 0,
//                                      tests/pre_quantize_test.py:6-10)
//   q_d    = clamp(round_half_even(x_d / scale), -127, 127)
//                                     (tests/pre_quantize_test.py:11,
//                                      transformer/model.py:105-114)
// scale is the correctly rounded quotient (div127_rn), and each q_d equals
// __float2int_rn(__fdiv_rn(x_d, scale)) (quant_row_fast below), so the int8
// values are bit-identical to torch's round(x / scale).clamp(-127, 127) on the
// same fp32 inputs.  The stored scale is `scale` rounded to the pool's scale
// dtype (fp16 RNE, or fp32 exactly).
#include "pa_common.cuh"
#include "quant.cuh"

#ifndef PA_WRITE_NL
#define PA_WRITE_NL 4
#endif
#ifndef PA_WRITE_MINB
#define PA_WRITE_MINB 4
#endif
#ifndef PA_WRITE_THREADS
#define PA_WRITE_THREADS 256
#endif

namespace pa {
namespace {

// Per-warp geometry for one (input dtype, head_dim): every lane loads 16
// bytes per instruction, LPR lanes cover one row, and a warp owns the K and V
// rows of HG kv heads of one token (NL loads per lane in flight at once).
template <int IN, int D>
struct WCfg {
  static constexpr int ESZ = IN == PA_DTYPE_F32 ? 4 : 2;
  static constexpr int EPL = 16 / ESZ;   // elements per lane per load
  static constexpr int LPR = D / EPL;    // lanes per row
  static constexpr int RPI = 32 / LPR;   // rows per load instruction
  static constexpr int NL = PA_WRITE_NL;  // loads per lane
  static constexpr int HG = NL * RPI / 2;  // kv heads per warp (K and V rows)
  static_assert(LPR >= 1 && LPR <= 32 && 32 % LPR == 0, "row must map onto whole lanes");
};

template <int IN, int EPL>
__device__ __forceinline__ void unpack_row(const uint4& w, float (&f)[EPL]) {
  if constexpr (IN == PA_DTYPE_F32) {
    f[0] = __uint_as_float(w.x);
    f[1] = __uint_as_float(w.y);
    f[2] = __uint_as_float(w.z);
    f[3] = __uint_as_float(w.w);
  } else {
    const uint32_t x[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 v;
      if constexpr (IN == PA_DTYPE_BF16) v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x[i]));
      else v = __half22float2(*reinterpret_cast<const __half2*>(&x[i]));
      f[2 * i] = v.x;
      f[2 * i + 1] = v.y;
    }
  }
}

// Quantise-on-write / copy-on-write.  One warp per (token, group of HG kv
// heads): the group's K and V source rows are loaded before the token's
// block-table entry is known, so the index lookups overlap the row loads.
template <int IN, int D>
__global__ void __launch_bounds__(PA_WRITE_THREADS, PA_WRITE_MINB) kv_write_kernel(const WriteParams p) {
  pdl_enter();
  using C = WCfg<IN, D>;
  constexpr int EPL = C::EPL;
  const int lane = threadIdx.x & 31;
  const int wid = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int groups = (p.Hkv + C::HG - 1) / C::HG;
  if (wid >= p.T * groups) return;  // T * groups < 2^26 (checked on the host)
  const int t = groups == 1 ? wid : wid / groups;
  const int h0 = (wid - t * groups) * C::HG;
  const int part = lane % C::LPR;
  const int sub = lane / C::LPR;

  // ---- 1. source rows (row j of the warp: head h0 + j/2, K for even j) ----
  uint4 raw[C::NL];
#pragma unroll
  for (int it = 0; it < C::NL; ++it) {
    const int j = it * C::RPI + sub;
    const int h = h0 + (j >> 1);
    raw[it] = make_uint4(0, 0, 0, 0);
    if (h < p.Hkv) {
      const char* src = (j & 1) ? static_cast<const char*>(p.v_new) + (t * p.vn_st + h * p.vn_sh) * C::ESZ
                                : static_cast<const char*>(p.k_new) + (t * p.kn_st + h * p.kn_sh) * C::ESZ;
      raw[it] = __ldg(reinterpret_cast<const uint4*>(src) + part);
    }
  }

  // ---- 2. destination block / slot ----------------------------------------
  const int s = p.seq_idx[t];
  const int pos = p.pos[t];
  if (s < 0 || s >= p.num_seqs) {
    if (lane == 0) set_status(p.status, ST_BAD_SEQ_INDEX);
    return;
  }
  const int bi = pos >> p.log2BS;
  if (pos < 0 || bi >= p.bt_cols) {
    if (lane == 0) set_status(p.status, ST_BAD_POSITION);
    return;
  }
  const int blk = p.bt[s * p.bt_ss + bi * p.bt_sc];
  if (blk < 0 || blk >= p.NB) {
    if (lane == 0) set_status(p.status, ST_BAD_BLOCK_ID);
    return;
  }
  const int slot = pos & (p.BS - 1);
  const long long kb = blk * p.k_sblk + slot * p.k_sslot, vb = blk * p.v_sblk + slot * p.v_sslot;
  const long long ksb = blk * p.ks_sblk + slot * p.ks_sslot, vsb = blk * p.vs_sblk + slot * p.vs_sslot;

  // ---- 3. convert and store -------------------------------------------------
  // The NL rows of a lane are independent: each phase runs over all of them
  // before the next, so their latencies overlap.
  if (p.cache_dtype == PA_DTYPE_I8) {
    // rows stay packed; each is unpacked only while it is quantised
    float am[C::NL];
#pragma unroll
    for (int it = 0; it < C::NL; ++it) am[it] = load_absmax<IN>(raw[it]);
#pragma unroll
    for (int o = C::LPR / 2; o >= 1; o >>= 1)
#pragma unroll
      for (int it = 0; it < C::NL; ++it) am[it] = fmaxf(am[it], __shfl_xor_sync(0xffffffffu, am[it], o));
    float sc[C::NL];
    uint32_t w[C::NL][EPL / 4];
    unsigned near = 0;
#pragma unroll
    for (int it = 0; it < C::NL; ++it) {
      sc[it] = (am[it] == 0.f) ? 1.0f : div127_rn(am[it]);
      float f[EPL];
      unpack_row<IN, EPL>(raw[it], f);
      if (quant_row_fast<EPL>(f, rcp_approx(sc[it]), w[it])) near |= 1u << it;
    }
    // rows with a quotient near a rounding boundary: redo with the division
#pragma unroll
    for (int it = 0; it < C::NL; ++it) {
      if (__any_sync(0xffffffffu, (near >> it) & 1u)) {
        float f[EPL];
        unpack_row<IN, EPL>(raw[it], f);
        quant_row_exact<EPL>(f, sc[it], w[it]);
      }
    }
#pragma unroll
    for (int it = 0; it < C::NL; ++it) {
      const int j = it * C::RPI + sub;
      const int h = h0 + (j >> 1);
      if (h >= p.Hkv) continue;
      const bool isv = j & 1;
      int8_t* dst = static_cast<int8_t*>(isv ? p.v : p.k) + (isv ? vb + h * p.v_shead : kb + h * p.k_shead) + part * EPL;
      if constexpr (EPL == 8) *reinterpret_cast<uint2*>(dst) = make_uint2(w[it][0], w[it][1]);
      else *reinterpret_cast<uint32_t*>(dst) = w[it][0];
      if (part == 0) {
        const long long so = isv ? vsb + h * p.vs_shead : ksb + h * p.ks_shead;
        void* sp = isv ? p.vs : p.ks;
        if (p.scale_f32) static_cast<float*>(sp)[so] = sc[it];
        else static_cast<__half*>(sp)[so] = __float2half_rn(sc[it]);
      }
    }
    return;
  }
  if (p.cache_dtype == PA_DTYPE_F32) {
#pragma unroll
    for (int it = 0; it < C::NL; ++it) {
      const int j = it * C::RPI + sub;
      const int h = h0 + (j >> 1);
      if (h >= p.Hkv) continue;
      const bool isv = j & 1;
      float* dst = static_cast<float*>(isv ? p.v : p.k) + (isv ? vb + h * p.v_shead : kb + h * p.k_shead) + part * EPL;
      float f[EPL];
      unpack_row<IN, EPL>(raw[it], f);
#pragma unroll
      for (int i = 0; i < EPL / 4; ++i)
        reinterpret_cast<float4*>(dst)[i] = make_float4(f[4 * i], f[4 * i + 1], f[4 * i + 2], f[4 * i + 3]);
    }
    return;
  }
  const bool bf = p.cache_dtype == PA_DTYPE_BF16;
#pragma unroll
  for (int it = 0; it < C::NL; ++it) {
    const int j = it * C::RPI + sub;
    const int h = h0 + (j >> 1);
    if (h >= p.Hkv) continue;
    const bool isv = j & 1;
    uint16_t* dst = static_cast<uint16_t*>(isv ? p.v : p.k) + (isv ? vb + h * p.v_shead : kb + h * p.k_shead) +
                    part * EPL;
    if constexpr (IN == PA_DTYPE_F16 || IN == PA_DTYPE_BF16) {
      if ((IN == PA_DTYPE_BF16) == bf) {
        *reinterpret_cast<uint4*>(dst) = raw[it];  // same 16-bit type: plain copy
        continue;
      }
    }
    float f[EPL];
    unpack_row<IN, EPL>(raw[it], f);
    uint32_t w[EPL / 2];
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) w[i] = bf ? pack2<true>(f[2 * i], f[2 * i + 1]) : pack2<false>(f[2 * i], f[2 * i + 1]);
    if constexpr (EPL == 8) *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    else *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
  }
}

template <int IN>
cudaError_t launch_in(const WriteParams& p, cudaStream_t stream) {
  auto go = [&](auto kern, int hg) {
    const long long warps = static_cast<long long>(p.T) * ((p.Hkv + hg - 1) / hg);
    const long long blocks = (warps * 32 + PA_WRITE_THREADS - 1) / PA_WRITE_THREADS;
    return launch_pdl(kern, dim3(static_cast<unsigned>(blocks)), dim3(PA_WRITE_THREADS), 0, stream, p);
  };
  if (p.D == 64) return go(kv_write_kernel<IN, 64>, WCfg<IN, 64>::HG);
  if (p.D == 128) return go(kv_write_kernel<IN, 128>, WCfg<IN, 128>::HG);
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_kv_write(const WriteParams& p, cudaStream_t stream) {
  if (static_cast<long long>(p.T) * p.Hkv == 0) return cudaSuccess;
  switch (p.in_dtype) {
    case PA_DTYPE_F32:
      return launch_in<PA_DTYPE_F32>(p, stream);
    case PA_DTYPE_BF16:
      return launch_in<PA_DTYPE_BF16>(p, stream);
    default:
      return launch_in<PA_DTYPE_F16>(p, stream);
  }
}

}  // namespace pa
