// Symmetric absmax INT8 quantisation of fp32 rows, bit-identical to the
// reference's rule (tests/pre_quantize_test.py:3-12, transformer/model.py:105-114):
// scale = absmax / 127 (1.0 for an all-zero row), q = clamp(round_half_even(x / scale),
// -127, 127).  Shared by the quantise-on-write kernel (kv_write.cu) and the
// projection kernel that quantises its own output rows (kv_project.cu).
#pragma once

#include "pa_common.cuh"

namespace pa {

// round_half_even(x / s) for |x| <= 127 * s, as the low byte of an fp32 sum.
// inv = rcp.approx(s) (at most 1 ulp off, per the PTX ISA; a relative error
// below 2^-22 is all this needs) and y = x * inv differs from x / s by at most
// |x / s| * (2^-22 + 2^-24), and from the correctly rounded quotient
// fl(x / s) by at most that plus half an ulp of fl(x / s): below 4.3e-5 for
// |x / s| <= 127.  Unless y lies within 1e-4 of a half-integer both round to
// the same integer; rows where some value does are redone with the exact
// division (quant_row_exact).  Adding 1.5 * 2^23 rounds to the nearest
// integer, ties to even, and leaves it in the low mantissa bits, whose low
// byte is the int8 two's complement encoding.  No clamp is needed:
// |x| <= absmax gives |fl(x / s)| <= 127 * (1 + 2^-23) and
// |y| <= 127 * (1 + 2^-21), both rounding to at most 127 in magnitude.
constexpr float RNE_MAGIC = 12582912.0f;  // 1.5 * 2^23

// RN(a / 127) without a division: y = RN(a * c) with c = RN(1 / 127), then
// one FMA correction -- the multiply-and-correct scheme for a divisor known
// in advance (Brisebarre, Muller, Raina, "Accelerating correctly rounded
// floating-point division when the divisor is known in advance", IEEE Trans.
// Computers 53(8), 2004).  For the divisor 127 it returns the correctly
// rounded quotient for every non-negative finite float (checked exhaustively
// against IEEE division; tests/test_div127_cpu.py restates the check).
__device__ __forceinline__ float div127_rn(float a) {
  constexpr float c = 1.0f / 127.0f;
  const float y = __fmul_rn(a, c);
  const float r = __fmaf_rn(-y, 127.0f, a);
  return __fmaf_rn(r, c, y);
}
constexpr float NEAR_HALF = 0.5f - 1.0e-4f;

__device__ __forceinline__ uint32_t q_byte(float y) { return __float_as_uint(y + RNE_MAGIC); }

__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Four quotient bytes (low bytes of b0..b3) -> one int8x4 word.
__device__ __forceinline__ uint32_t pack_bytes(uint32_t b0, uint32_t b1, uint32_t b2, uint32_t b3) {
  return prmt(prmt(b0, b1, 0x0040u), prmt(b2, b3, 0x0040u), 0x5410u);
}

// max |x| over one 16-byte load, from the packed values: |x| and max are
// exact in 16 bits, so this equals the fp32 maximum of the unpacked row.
template <int IN>
__device__ __forceinline__ float load_absmax(const uint4& w) {
  if constexpr (IN == PA_DTYPE_F32) {
    return fmaxf(fmaxf(fabsf(__uint_as_float(w.x)), fabsf(__uint_as_float(w.y))),
                 fmaxf(fabsf(__uint_as_float(w.z)), fabsf(__uint_as_float(w.w))));
  } else if constexpr (IN == PA_DTYPE_BF16) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
    const __nv_bfloat162 m = __hmax2(__hmax2(__habs2(h[0]), __habs2(h[1])), __hmax2(__habs2(h[2]), __habs2(h[3])));
    return fmaxf(__bfloat162float(m.x), __bfloat162float(m.y));
  } else {
    const __half2* h = reinterpret_cast<const __half2*>(&w);
    const __half2 m = __hmax2(__hmax2(__habs2(h[0]), __habs2(h[1])), __hmax2(__habs2(h[2]), __habs2(h[3])));
    return fmaxf(__half2float(m.x), __half2float(m.y));
  }
}

template <int EPL>
__device__ __forceinline__ bool quant_row_fast(const float (&f)[EPL], float inv, uint32_t (&w)[EPL / 4]) {
  bool near = false;
#pragma unroll
  for (int i = 0; i < EPL / 4; ++i) {
    uint32_t b[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float y = f[4 * i + k] * inv;
      const float r = (y + RNE_MAGIC) - RNE_MAGIC;
      near |= fabsf(y - r) > NEAR_HALF;
      b[k] = q_byte(y);
    }
    w[i] = pack_bytes(b[0], b[1], b[2], b[3]);
  }
  return near;
}

template <int EPL>
__device__ __forceinline__ void quant_row_exact(const float (&f)[EPL], float s, uint32_t (&w)[EPL / 4]) {
#pragma unroll
  for (int i = 0; i < EPL / 4; ++i) {
    uint32_t b[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) b[k] = q_byte(__fdiv_rn(f[4 * i + k], s));
    w[i] = pack_bytes(b[0], b[1], b[2], b[3]);
  }
}

}  // namespace pa
