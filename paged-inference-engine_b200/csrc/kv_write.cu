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
// The division is the correctly rounded __fdiv_rn and the rounding is
// __float2int_rn, so the int8 values are bit-identical to torch's
// round(x / scale).clamp(-127, 127) on the same fp32 inputs.  The stored scale
// is `scale` rounded to the pool's scale dtype (fp16 RNE, or fp32 exactly).
#include "pa_common.cuh"

namespace pa {
namespace {

// Load EPL consecutive elements of the input dtype into fp32.
template <int EPL, int IN>
__device__ __forceinline__ void load_row(const void* base, float (&f)[EPL]) {
  if constexpr (IN == PA_DTYPE_F32) {
    const float4* p = static_cast<const float4*>(base);
    if constexpr (EPL == 2) {
      float2 v = *static_cast<const float2*>(base);
      f[0] = v.x;
      f[1] = v.y;
    } else {
#pragma unroll
      for (int i = 0; i < EPL / 4; ++i) {
        float4 v = p[i];
        f[4 * i + 0] = v.x;
        f[4 * i + 1] = v.y;
        f[4 * i + 2] = v.z;
        f[4 * i + 3] = v.w;
      }
    }
  } else {
    uint32_t w[EPL / 2];
    if constexpr (EPL == 2) {
      w[0] = *static_cast<const uint32_t*>(base);
    } else if constexpr (EPL == 4) {
      uint2 v = *static_cast<const uint2*>(base);
      w[0] = v.x;
      w[1] = v.y;
    } else {
      uint4 v = *static_cast<const uint4*>(base);
      w[0] = v.x;
      w[1] = v.y;
      w[2] = v.z;
      w[3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < EPL / 2; ++i) {
      if constexpr (IN == PA_DTYPE_BF16) {
        float2 x = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w[i]));
        f[2 * i] = x.x;
        f[2 * i + 1] = x.y;
      } else {
        float2 x = __half22float2(*reinterpret_cast<__half2*>(&w[i]));
        f[2 * i] = x.x;
        f[2 * i + 1] = x.y;
      }
    }
  }
}

template <int EPL>
__device__ __forceinline__ void store_i8(void* dst, const int (&q)[EPL]) {
  uint32_t w[(EPL + 3) / 4] = {};
#pragma unroll
  for (int i = 0; i < EPL; ++i) w[i / 4] |= (static_cast<uint32_t>(q[i]) & 0xffu) << (8 * (i % 4));
  if constexpr (EPL == 2) {
    *static_cast<unsigned short*>(dst) = static_cast<unsigned short>(w[0]);
  } else if constexpr (EPL == 4) {
    *static_cast<uint32_t*>(dst) = w[0];
  } else {
    *static_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
  }
}

template <int EPL, bool BF16>
__device__ __forceinline__ void store_16b(void* dst, const float (&f)[EPL]) {
  uint32_t w[EPL / 2];
#pragma unroll
  for (int i = 0; i < EPL / 2; ++i) w[i] = pack2<BF16>(f[2 * i], f[2 * i + 1]);
  if constexpr (EPL == 2) {
    *static_cast<uint32_t*>(dst) = w[0];
  } else if constexpr (EPL == 4) {
    *static_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
  } else {
    *static_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <int EPL>
__device__ __forceinline__ void write_row(const WriteParams& p, const void* src, void* cache_row, void* scale_ptr,
                                          int lane) {
  float f[EPL];
  const int off = lane * EPL;
  switch (p.in_dtype) {
    case PA_DTYPE_F32:
      load_row<EPL, PA_DTYPE_F32>(static_cast<const float*>(src) + off, f);
      break;
    case PA_DTYPE_BF16:
      load_row<EPL, PA_DTYPE_BF16>(static_cast<const __nv_bfloat16*>(src) + off, f);
      break;
    default:
      load_row<EPL, PA_DTYPE_F16>(static_cast<const __half*>(src) + off, f);
      break;
  }
  if (p.cache_dtype == PA_DTYPE_I8) {
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) amax = fmaxf(amax, fabsf(f[i]));
    amax = warp_max_xor(amax, 1);
    const float scale = (amax == 0.f) ? 1.0f : __fdiv_rn(amax, 127.0f);
    int q[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      int v = __float2int_rn(__fdiv_rn(f[i], scale));
      q[i] = max(-127, min(127, v));
    }
    store_i8<EPL>(static_cast<int8_t*>(cache_row) + off, q);
    if (lane == 0) {
      if (p.scale_f32) *static_cast<float*>(scale_ptr) = scale;
      else *static_cast<__half*>(scale_ptr) = __float2half_rn(scale);
    }
  } else if (p.cache_dtype == PA_DTYPE_BF16) {
    store_16b<EPL, true>(static_cast<__nv_bfloat16*>(cache_row) + off, f);
  } else {
    store_16b<EPL, false>(static_cast<__half*>(cache_row) + off, f);
  }
}

template <int EPL>
__global__ void __launch_bounds__(256) kv_write_kernel(const WriteParams p) {
  const int lane = threadIdx.x & 31;
  const long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (row >= static_cast<long long>(p.T) * p.Hkv) return;
  const int t = static_cast<int>(row / p.Hkv);
  const int h = static_cast<int>(row % p.Hkv);
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
  const int esz = p.in_dtype == PA_DTYPE_F32 ? 4 : 2;
  const int csz = p.cache_dtype == PA_DTYPE_I8 ? 1 : 2;

  const char* ksrc = static_cast<const char*>(p.k_new) + (t * p.kn_st + h * p.kn_sh) * esz;
  const char* vsrc = static_cast<const char*>(p.v_new) + (t * p.vn_st + h * p.vn_sh) * esz;
  char* kdst = static_cast<char*>(p.k) + (blk * p.k_sblk + slot * p.k_sslot + h * p.k_shead) * csz;
  char* vdst = static_cast<char*>(p.v) + (blk * p.v_sblk + slot * p.v_sslot + h * p.v_shead) * csz;
  void* ksc = nullptr;
  void* vsc = nullptr;
  if (p.cache_dtype == PA_DTYPE_I8) {
    const int ssz = p.scale_f32 ? 4 : 2;
    ksc = static_cast<char*>(p.ks) + (blk * p.ks_sblk + slot * p.ks_sslot + h * p.ks_shead) * ssz;
    vsc = static_cast<char*>(p.vs) + (blk * p.vs_sblk + slot * p.vs_sslot + h * p.vs_shead) * ssz;
  }
  write_row<EPL>(p, ksrc, kdst, ksc, lane);
  write_row<EPL>(p, vsrc, vdst, vsc, lane);
}

}  // namespace

cudaError_t launch_kv_write(const WriteParams& p, cudaStream_t stream) {
  const long long rows = static_cast<long long>(p.T) * p.Hkv;
  if (rows == 0) return cudaSuccess;
  const int threads = 256;
  const long long blocks = (rows * 32 + threads - 1) / threads;
  switch (p.D) {
    case 64:
      kv_write_kernel<2><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(p);
      break;
    case 128:
      kv_write_kernel<4><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(p);
      break;
    case 256:
      kv_write_kernel<8><<<static_cast<unsigned>(blocks), threads, 0, stream>>>(p);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace pa
