// Shared device helpers for the sm_100a paged-attention kernels.
//
// Everything here is a thin wrapper over a documented PTX instruction
// (mma.sync, ldmatrix, cp.async, ex2.approx, prmt) or plain integer/float
// arithmetic.  No CUDA math-library routine is restated.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <utility>

#include "pa_types.h"

namespace pa {
// Programmatic dependent launch.  Every kernel of this library is launched
// with programmatic stream serialisation (launch_pdl) and starts with
// pdl_enter(): it waits until the previous grid in the stream has completed
// and its writes are visible (so no input is read early), then lets the next
// grid be scheduled.  The next grid's CTAs become resident while this one
// runs and start as soon as it finishes, instead of after a launch gap.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}
}  // namespace pa

namespace pa {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// cp.async (Ampere-style asynchronous global->shared copies).
// src_bytes == 0 zero-fills the destination without touching global memory,
// which is how masked / out-of-range rows become zeros in shared memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_4(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// ---------------------------------------------------------------------------
// ldmatrix / mma.sync (m16n8k16, fp32 accumulate).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}

template <bool BF16>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// D (int32) += A (16x32 s8, row) * B (32x8 s8, col), warp-level.  Thread
// (group g, lane-in-group t) holds A rows g / g+8 at k = 4t..4t+3 (a0 / a1) and
// 16+4t.. (a2 / a3), B column g at k = 4t.. (b0) and 16+4t.. (b1), four
// int8 per register, the lowest k in the lowest byte.
__device__ __forceinline__ void mma_s8_16832(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------
// Scalar helpers.
// ---------------------------------------------------------------------------
// Hardware base-2 exponential (MUFU.EX2); ex2(-inf) == +0.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// Row bases of sequence b in Q, O and L: b * seq_stride for [B, H, maxq, ...]
// tensors, q_start[b] * row_stride for ragged rows packed as [T, H, ...].
__device__ __forceinline__ long long q_seq_base(const AttnParams& p, int b) {
  return p.q_start ? static_cast<long long>(p.q_start[b]) * p.q_sm : static_cast<long long>(b) * p.q_sb;
}
__device__ __forceinline__ long long o_seq_base(const AttnParams& p, int b) {
  return p.q_start ? static_cast<long long>(p.q_start[b]) * p.o_sm : static_cast<long long>(b) * p.o_sb;
}
__device__ __forceinline__ long long l_seq_base(const AttnParams& p, int b) {
  return p.q_start ? static_cast<long long>(p.q_start[b]) * p.l_sm : static_cast<long long>(b) * p.l_sb;
}
// Store one O element at element offset `idx` from p.o: locally, or into
// every GPU of a peer output exchange (NVLink stores to mapped peer memory).
__device__ __forceinline__ void store_o(const AttnParams& p, long long idx, __half v) {
  if (p.n_peers == 0) {
    static_cast<__half*>(p.o)[idx] = v;
    return;
  }
#pragma unroll 1
  for (int r = 0; r < p.n_peers; ++r) static_cast<__half*>(p.o_peer[r])[idx] = v;
}
// End of a kernel that stored O to peers: its stores are performed system-wide
// before the barrier kernel that follows posts its flags.
__device__ __forceinline__ void peer_store_fence(const AttnParams& p) {
  if (p.n_peers) __threadfence_system();
}
// Query rows of sequence b: q_len clamped to max_q_len and, for ragged rows,
// to the rows left in Q after q_start[b] (0 for a start outside [0, T)), so
// bad metadata can never address past Q, O or L.
__device__ __forceinline__ int seq_rows(const AttnParams& p, int b) {
  int q = min(p.qlen[b], p.maxq);
  if (p.q_start) {
    const int s = p.q_start[b];
    q = (s < 0 || s >= p.q_total) ? 0 : min(q, p.q_total - s);
  }
  return q;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Four signed int8 values (bytes 0..3 of `w`) -> two packed fp16 pairs
// {b0,b1} and {b2,b3}.  Exact for every int8 input: the byte is biased to
// unsigned (xor 0x80), placed in the mantissa of 1024.0h (0x64xx) and the
// bias 1024+128 is subtracted.
__device__ __forceinline__ void i8x4_to_f16x4(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  uint32_t a = prmt(u, 0x64646464u, 0x5140u);
  uint32_t b = prmt(u, 0x64646464u, 0x7362u);
  const __half2 bias = __half2half2(__ushort_as_half(0x6480));  // 1152.0
  __half2 ha = __hsub2(*reinterpret_cast<__half2*>(&a), bias);
  __half2 hb = __hsub2(*reinterpret_cast<__half2*>(&b), bias);
  lo = *reinterpret_cast<uint32_t*>(&ha);
  hi = *reinterpret_cast<uint32_t*>(&hb);
}

// Four signed int8 values -> two packed fp16 pairs holding 1152 + b_i (the
// byte biased to unsigned and placed in the mantissa of 1024.0h): exact, and
// one subtraction per pair cheaper than i8x4_to_f16x4.  Callers remove the
// 1152 offset after the dot product (it adds 1152 * sum of the other operand).
constexpr float I8_BIAS = 1152.0f;
__device__ __forceinline__ void i8x4_to_f16x4_biased(uint32_t w, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  lo = prmt(u, 0x64646464u, 0x5140u);
  hi = prmt(u, 0x64646464u, 0x7362u);
}

__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (BF16) return pack_bf16(a, b);
  else return pack_f16(a, b);
}

// Convert a packed pair of 16-bit values of element type SRC_BF16 into the
// MMA element type DST_BF16 (identity when equal).
template <bool SRC_BF16, bool DST_BF16>
__device__ __forceinline__ uint32_t cvt_pair(uint32_t v) {
  if constexpr (SRC_BF16 == DST_BF16) {
    return v;
  } else if constexpr (SRC_BF16) {
    float2 f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&v));
    return pack_f16(f.x, f.y);
  } else {
    float2 f = __half22float2(*reinterpret_cast<__half2*>(&v));
    return pack_bf16(f.x, f.y);
  }
}

__device__ __forceinline__ float warp_max_xor(float v, int first_mask) {
  for (int m = first_mask; m < 32; m <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}
__device__ __forceinline__ float warp_sum_xor(float v, int first_mask) {
  for (int m = first_mask; m < 32; m <<= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

__device__ __forceinline__ void set_status(int* status, int bit) {
  if (status) atomicOr(status, bit);
}

// ---------------------------------------------------------------------------
// mbarrier + TMA (cp.async.bulk.tensor, single-CTA destination only).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::); }
// Orders this thread's generic-proxy shared-memory accesses before later
// async-proxy (TMA) writes to the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after `limit` polls and returns false.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int limit = 1 << 22) {
  for (int i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, uint32_t bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];\n" ::"r"(dst),
      "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          dst),
      "l"(tmap), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

// Fetch a TMA box into L2 only (no shared memory, no completion tracking).
__device__ __forceinline__ void tma_prefetch_4d(const void* tmap, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];\n" ::"l"(tmap), "r"(c0),
               "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
// max of three floats (one instruction on sm_100)
__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;\n" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, TMEM accumulators), cta_group::1.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(dst_smem), "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
// Arrive on `bar` once every tcgen05 operation issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
               : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void tc_mma_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The 8 K16 steps of a head_dim-128 contraction in one block, D (tmem) =
// sum_k A_k B_k with both operands K-major SW128 in shared memory: A_k and B_k
// are the descriptors a0 / b0 advanced by 32 bytes per step within a 64-column
// half and by AH / BH (16-byte units) from the first half to the second.  One
// descriptor pair is computed by the caller; the rest are immediate adds.
template <int AH, int BH>
__device__ __forceinline__ void tc_mma_ss_k128(uint32_t d_tmem, uint64_t a0, uint64_t b0, uint32_t idesc) {
  asm volatile(
      "{\n .reg .pred p0, p1;\n .reg .b64 a1, a2, a3, a4, a5, a6, a7, b1, b2, b3, b4, b5, b6, b7;\n"
      " setp.ne.b32 p0, %3, %3;\n setp.eq.b32 p1, %3, %3;\n"
      " add.s64 a1, %1, 2;\n add.s64 a2, %1, 4;\n add.s64 a3, %1, 6;\n"
      " add.s64 a4, %1, %4;\n add.s64 a5, a4, 2;\n add.s64 a6, a4, 4;\n add.s64 a7, a4, 6;\n"
      " add.s64 b1, %2, 2;\n add.s64 b2, %2, 4;\n add.s64 b3, %2, 6;\n"
      " add.s64 b4, %2, %5;\n add.s64 b5, b4, 2;\n add.s64 b6, b4, 4;\n add.s64 b7, b4, 6;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], a1, b1, %3, p1;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], a2, b2, %3, p1;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], a3, b3, %3, p1;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], a4, b4, %3, p1;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], a5, b5, %3, p1;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], a6, b6, %3, p1;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], a7, b7, %3, p1;\n}\n" ::"r"(d_tmem),
      "l"(a0), "l"(b0), "r"(idesc), "n"(AH), "n"(BH)
      : "memory");
}

// tc_mma_ss_k128 onto an existing accumulator when `accumulate` is non-zero
// (the first of the 8 steps adds to D instead of overwriting it).
template <int AH, int BH>
__device__ __forceinline__ void tc_mma_ss_k128_acc(uint32_t d_tmem, uint64_t a0, uint64_t b0, uint32_t idesc,
                                                   uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p0, p1;\n .reg .b64 a1, a2, a3, a4, a5, a6, a7, b1, b2, b3, b4, b5, b6, b7;\n"
      " setp.ne.b32 p0, %6, 0;\n setp.eq.b32 p1, %3, %3;\n"
      " add.s64 a1, %1, 2;\n add.s64 a2, %1, 4;\n add.s64 a3, %1, 6;\n"
      " add.s64 a4, %1, %4;\n add.s64 a5, a4, 2;\n add.s64 a6, a4, 4;\n add.s64 a7, a4, 6;\n"
      " add.s64 b1, %2, 2;\n add.s64 b2, %2, 4;\n add.s64 b3, %2, 6;\n"
      " add.s64 b4, %2, %5;\n add.s64 b5, b4, 2;\n add.s64 b6, b4, 4;\n add.s64 b7, b4, 6;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], a1, b1, %3, p1;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], a2, b2, %3, p1;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], a3, b3, %3, p1;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], a4, b4, %3, p1;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], a5, b5, %3, p1;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], a6, b6, %3, p1;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], a7, b7, %3, p1;\n}\n" ::"r"(d_tmem),
      "l"(a0), "l"(b0), "r"(idesc), "n"(AH), "n"(BH), "r"(accumulate)
      : "memory");
}

// NK K16 steps (NK = 4 or 8) with A in TMEM (8 columns of packed 16-bit
// values per step) and B an MN-major SW128 descriptor advanced by 16 rows of
// 128 bytes per step: D (tmem) (+)= sum_k A_k B_k; the first step accumulates
// onto D only when `accumulate` is non-zero.
template <int NK>
__device__ __forceinline__ void tc_mma_ts_seq(uint32_t d_tmem, uint32_t a_tmem, uint64_t b0, uint32_t idesc,
                                              uint32_t accumulate) {
  static_assert(NK == 4 || NK == 8, "4 or 8 steps");
  if constexpr (NK == 4) {
    asm volatile(
        "{\n .reg .pred p0, p1;\n .reg .b32 t1, t2, t3;\n .reg .b64 b1, b2, b3;\n"
        " setp.ne.b32 p0, %4, 0;\n setp.eq.b32 p1, %3, %3;\n"
        " add.u32 t1, %1, 8;\n add.u32 t2, %1, 16;\n add.u32 t3, %1, 24;\n"
        " add.s64 b1, %2, 128;\n add.s64 b2, %2, 256;\n add.s64 b3, %2, 384;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [t1], b1, %3, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [t2], b2, %3, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [t3], b3, %3, p1;\n}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b0), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n .reg .pred p0, p1;\n .reg .b32 t1, t2, t3, t4, t5, t6, t7;\n"
        " .reg .b64 b1, b2, b3, b4, b5, b6, b7;\n"
        " setp.ne.b32 p0, %4, 0;\n setp.eq.b32 p1, %3, %3;\n"
        " add.u32 t1, %1, 8;\n add.u32 t2, %1, 16;\n add.u32 t3, %1, 24;\n add.u32 t4, %1, 32;\n"
        " add.u32 t5, %1, 40;\n add.u32 t6, %1, 48;\n add.u32 t7, %1, 56;\n"
        " add.s64 b1, %2, 128;\n add.s64 b2, %2, 256;\n add.s64 b3, %2, 384;\n add.s64 b4, %2, 512;\n"
        " add.s64 b5, %2, 640;\n add.s64 b6, %2, 768;\n add.s64 b7, %2, 896;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [t1], b1, %3, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [t2], b2, %3, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [t3], b3, %3, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [t4], b4, %3, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [t5], b5, %3, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [t6], b6, %3, p1;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [t7], b7, %3, p1;\n}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b0), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// 32 consecutive 32-bit TMEM columns of this thread's lane (32x32b shape).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05): start address, leading / stride
// byte offsets (all >> 4), descriptor version 1, layout type at bits 61..63
// (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16 with fp32 accumulation.
__host__ __device__ constexpr uint32_t instr_desc_f16(bool bf16, bool a_mn_major, bool b_mn_major, int M, int N) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         ((b_mn_major ? 1u : 0u) << 16) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Packed fp32 pairs (sm_100 f32x2 FMA-pipe instructions) and 2^x on the FMA pipe.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};\n" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;\n" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;\n" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;\n" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// 2^x for a pair of floats without the MUFU unit.  Range reduction: adding
// 1.5*2^23 rounds x to the nearest integer n inside the float's mantissa
// (f = x - n in [-1/2, 1/2]); 2^f is a cubic whose coefficients were fitted
// here by iteratively re-weighted least squares on the relative error over
// [-1/2, 1/2] (max relative error 7.6e-5, 13.7 bits -- more than the 11 bits
// an fp16 probability keeps); 2^n is applied by adding n to the exponent
// field.  Inputs below -125 are clamped there (result ~2^-125).
__device__ __forceinline__ void exp2_fma_x2(float& a, float& b) {
  const float kMagic = 12582912.0f;  // 1.5 * 2^23
  a = fmaxf(a, -125.0f);
  b = fmaxf(b, -125.0f);
  const uint64_t x = f2_pack(a, b);
  const uint64_t t = f2_add(x, f2_pack(kMagic, kMagic));
  const uint64_t n = f2_add(t, f2_pack(-kMagic, -kMagic));
  const uint64_t f = f2_fma(n, f2_pack(-1.0f, -1.0f), x);
  uint64_t poly = f2_fma(f2_pack(0.055170249193906784f, 0.055170249193906784f), f,
                         f2_pack(0.24260790646076202f, 0.24260790646076202f));
  poly = f2_fma(poly, f, f2_pack(0.693260908126831f, 0.693260908126831f));
  poly = f2_fma(poly, f, f2_pack(0.9999282956123352f, 0.9999282956123352f));
  float p0, p1, t0, t1;
  f2_unpack(poly, p0, p1);
  f2_unpack(t, t0, t1);
  a = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  b = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

__device__ __forceinline__ float load_scale(const void* base, long long off, int is_f32) {
  return is_f32 ? static_cast<const float*>(base)[off]
                : __half2float(static_cast<const __half*>(base)[off]);
}

}  // namespace pa
