// extern "C" entry points of libpaged_attn_b200.so (declared in
// include/paged_attn_b200.h): argument validation, kernel selection and
// workspace layout.  Nothing here allocates device memory.
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include <cudaTypedefs.h>

#include "pa_types.h"

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(PA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool is_pow2(long long x) { return x > 0 && (x & (x - 1)) == 0; }
int ilog2(long long x) {
  int r = 0;
  while ((1LL << r) < x) ++r;
  return r;
}
bool al(const void* p, unsigned a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
bool row_al(long long stride_elems, int elt, unsigned a) { return ((stride_elems * elt) % a) == 0; }

int elt_size(int dtype) {
  switch (dtype) {
    case PA_DTYPE_F16:
    case PA_DTYPE_BF16:
      return 2;
    case PA_DTYPE_I8:
      return 1;
    case PA_DTYPE_F32:
      return 4;
    default:
      return 0;
  }
}

constexpr int kNcMax = 16;
constexpr int kMaxDecodeSeqs = 8192;

// Validate a KV pool; fills the pool part of AttnParams / WriteParams.
int check_cache(const pa_kv_cache_t* kv) {
  if (!kv) return fail(PA_ERR_INVALID, "kv cache descriptor is NULL");
  if (kv->dtype != PA_DTYPE_F16 && kv->dtype != PA_DTYPE_BF16 && kv->dtype != PA_DTYPE_I8 &&
      kv->dtype != PA_DTYPE_F32)
    return fail(PA_ERR_INVALID, "KV pool dtype %d unsupported (fp16, bf16, int8 or fp32)", kv->dtype);
  if (kv->head_dim != 64 && kv->head_dim != 128)
    return fail(PA_ERR_UNSUPPORTED, "head_dim %d not compiled (64 or 128)", kv->head_dim);
  if (!is_pow2(kv->block_size))
    return fail(PA_ERR_INVALID, "block_size %d must be a power of two", kv->block_size);
  if (kv->num_kv_heads < 1 || kv->num_blocks < 0) return fail(PA_ERR_INVALID, "bad KV pool shape");
  if (!kv->k || !kv->v) return fail(PA_ERR_INVALID, "K/V pool pointer is NULL");
  const int e = elt_size(kv->dtype);
  if (!al(kv->k, 16) || !al(kv->v, 16)) return fail(PA_ERR_INVALID, "K/V pool must be 16-byte aligned");
  const long long ks[6] = {kv->k_stride_block, kv->k_stride_slot, kv->k_stride_head,
                           kv->v_stride_block, kv->v_stride_slot, kv->v_stride_head};
  for (long long s : ks)
    if (!row_al(s, e, 16) || s < 0)
      return fail(PA_ERR_INVALID, "K/V pool strides must be non-negative and keep rows 16-byte aligned");
  if (kv->dtype == PA_DTYPE_I8) {
    if (!kv->k_scale || !kv->v_scale) return fail(PA_ERR_INVALID, "int8 KV pool needs k_scale and v_scale");
    if (kv->scale_dtype != PA_DTYPE_F16 && kv->scale_dtype != PA_DTYPE_F32)
      return fail(PA_ERR_INVALID, "scale dtype must be fp16 or fp32");
    const unsigned sa = kv->scale_dtype == PA_DTYPE_F32 ? 4 : 2;
    if (!al(kv->k_scale, sa) || !al(kv->v_scale, sa)) return fail(PA_ERR_INVALID, "scale tensors misaligned");
  }
  return PA_OK;
}

int check_paging(const pa_paging_t* pg) {
  if (!pg) return fail(PA_ERR_INVALID, "paging descriptor is NULL");
  if (pg->num_seqs < 0 || pg->bt_cols < 0) return fail(PA_ERR_INVALID, "negative num_seqs / block table width");
  if (pg->num_seqs > 0 && (!pg->block_table || !pg->q_len_per_seq || !pg->kv_len_per_seq || !pg->num_blocks_per_seq))
    return fail(PA_ERR_INVALID, "paging metadata pointer is NULL");
  return PA_OK;
}

void fill_cache(pa::AttnParams& p, const pa_kv_cache_t* kv) {
  p.k = kv->k;
  p.v = kv->v;
  p.k_sblk = kv->k_stride_block;
  p.k_sslot = kv->k_stride_slot;
  p.k_shead = kv->k_stride_head;
  p.v_sblk = kv->v_stride_block;
  p.v_sslot = kv->v_stride_slot;
  p.v_shead = kv->v_stride_head;
  p.ks = kv->k_scale;
  p.vs = kv->v_scale;
  p.ks_sblk = kv->ks_stride_block;
  p.ks_sslot = kv->ks_stride_slot;
  p.ks_shead = kv->ks_stride_head;
  p.vs_sblk = kv->vs_stride_block;
  p.vs_sslot = kv->vs_stride_slot;
  p.vs_shead = kv->vs_stride_head;
  p.scale_f32 = kv->scale_dtype == PA_DTYPE_F32;
  p.Hkv = kv->num_kv_heads;
  p.BS = kv->block_size;
  p.log2BS = ilog2(kv->block_size);
  p.NB = kv->num_blocks;
}

int build_attn(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg, int32_t* status,
               pa::AttnParams& p) {
  int rc = check_cache(kv);
  if (rc) return rc;
  rc = check_paging(pg);
  if (rc) return rc;
  if (!io) return fail(PA_ERR_INVALID, "attention io descriptor is NULL");
  if (io->q_dtype != PA_DTYPE_F16 && io->q_dtype != PA_DTYPE_BF16)
    return fail(PA_ERR_INVALID, "Q dtype must be fp16 or bf16");
  if (io->num_q_heads < 1 || io->num_q_heads % kv->num_kv_heads)
    return fail(PA_ERR_INVALID, "num_q_heads (%d) must be a positive multiple of num_kv_heads (%d)",
                io->num_q_heads, kv->num_kv_heads);
  if (io->max_q_len < 0) return fail(PA_ERR_INVALID, "max_q_len < 0");
  if (pg->num_seqs > 0 && io->max_q_len > 0) {
    if (!io->q || !io->o) return fail(PA_ERR_INVALID, "Q / O pointer is NULL");
    if (!al(io->q, 16) || !row_al(io->q_stride_seq, 2, 16) || !row_al(io->q_stride_head, 2, 16) ||
        !row_al(io->q_stride_row, 2, 16))
      return fail(PA_ERR_INVALID, "Q rows must be 16-byte aligned (contiguous head_dim)");
    if (!al(io->o, 4) || !row_al(io->o_stride_seq, 2, 4) || !row_al(io->o_stride_head, 2, 4) ||
        !row_al(io->o_stride_row, 2, 4))
      return fail(PA_ERR_INVALID, "O rows must be 4-byte aligned");
    if (io->lse && !al(io->lse, 2)) return fail(PA_ERR_INVALID, "LSE misaligned");
  }
  p = pa::AttnParams{};
  fill_cache(p, kv);
  p.q = io->q;
  p.q_sb = io->q_stride_seq;
  p.q_sh = io->q_stride_head;
  p.q_sm = io->q_stride_row;
  p.q_bf16 = io->q_dtype == PA_DTYPE_BF16;
  p.bt = pg->block_table;
  p.bt_ss = pg->bt_stride_seq;
  p.bt_sc = pg->bt_stride_col;
  p.bt_cols = pg->bt_cols;
  p.nblk = pg->num_blocks_per_seq;
  p.qlen = pg->q_len_per_seq;
  p.kvlen = pg->kv_len_per_seq;
  p.o = io->o;
  p.o_sb = io->o_stride_seq;
  p.o_sh = io->o_stride_head;
  p.o_sm = io->o_stride_row;
  p.lse = io->lse;
  p.l_sb = io->l_stride_seq;
  p.l_sh = io->l_stride_head;
  p.l_sm = io->l_stride_row;
  p.B = pg->num_seqs;
  p.Hq = io->num_q_heads;
  p.G = io->num_q_heads / kv->num_kv_heads;
  p.maxq = io->max_q_len;
  const float sc = io->softmax_scale > 0.f ? io->softmax_scale : 1.0f / sqrtf(static_cast<float>(kv->head_dim));
  p.sm_scale = sc;
  p.scale_log2 = sc * 1.4426950408889634f;
  p.top_left = io->causal_top_left ? 1 : 0;
  p.status = status;
  return PA_OK;
}

// The split-K decode kernels read 16-bit and int8 pools; fp32 pools (a
// reference-compatible format, not a serving one) always take the tiled kernel.
// Batches of more than kMaxDecodeSeqs sequences decode in launches of at most
// that many (run_decode).
bool use_decode(const pa::AttnParams& p, const pa_kv_cache_t* kv) {
  return p.maxq * p.G <= kNcMax && kv->dtype != PA_DTYPE_F32;
}
int decode_nt(const pa::AttnParams& p) { return p.maxq * p.G <= 8 ? 1 : 2; }
int kv_kind(int dtype) {
  return dtype == PA_DTYPE_F16 ? pa::KV_F16 : dtype == PA_DTYPE_BF16 ? pa::KV_BF16
                                            : dtype == PA_DTYPE_F32 ? pa::KV_F32 : pa::KV_I8;
}

// Persistent decode launch plan, cached per (device, variant, num_seqs).
int cached_plan(int kv, int qbf, int D, int nt, int B, int tma, pa::DecodeLaunch* out) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int, int, int>, pa::DecodeLaunch> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  const auto key = std::make_tuple(dev, kv, qbf, D, nt, B, tma);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return 0;
    }
  }
  if (pa::decode_plan(kv, qbf, D, nt, B, tma, out) != 0) return -1;
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = *out;
  return 0;
}

// cuTensorMapEncodeTiled, fetched through the runtime (no link-time libcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 4-D TMA map over a pool read as [block, slot, head, d]: box = 128 bytes of
// head_dim (64 for 64-byte rows) x 1 head x min(16, block_size) slots x 1 block,
// with the matching shared-memory swizzle.
bool make_pool_map(CUtensorMap* m, void* base, int dtype, int D, int H, int BS, int NB, long long s_head,
                   long long s_slot, long long s_blk) {
  auto enc = encode_fn();
  if (dtype == PA_DTYPE_F32) return false;
  if (!enc || NB < 1 || BS < 8 || s_head <= 0 || s_slot <= 0 || s_blk <= 0) return false;
  const int elt = dtype == PA_DTYPE_I8 ? 1 : 2;
  const int rowb = D * elt;
  if (rowb != 64 && rowb % 128 != 0) return false;
  const cuuint32_t boxd = static_cast<cuuint32_t>((rowb >= 128 ? 128 : rowb) / elt);
  const CUtensorMapSwizzle swz = rowb >= 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(BS),
                              static_cast<cuuint64_t>(NB)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(s_head * elt), static_cast<cuuint64_t>(s_slot * elt),
                                 static_cast<cuuint64_t>(s_blk * elt)};
  const cuuint32_t box[4] = {boxd, 1, static_cast<cuuint32_t>(BS < 16 ? BS : 16), 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  // L2 fills no wider than one box row: a wider promotion drags the next
  // head's row of the same slot out of DRAM with every row.
  const CUtensorMapL2promotion l2 = rowb >= 256 ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B
                                    : rowb >= 128 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B
                                                  : CU_TENSOR_MAP_L2_PROMOTION_L2_64B;
  const CUresult r = enc(m, elt == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, base, dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz, l2, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool encode_kv_maps(const pa_kv_cache_t* kv, pa::KvMaps* maps) {
  return make_pool_map(&maps->k, kv->k, kv->dtype, kv->head_dim, kv->num_kv_heads, kv->block_size, kv->num_blocks,
                       kv->k_stride_head, kv->k_stride_slot, kv->k_stride_block) &&
         make_pool_map(&maps->v, kv->v, kv->dtype, kv->head_dim, kv->num_kv_heads, kv->block_size, kv->num_blocks,
                       kv->v_stride_head, kv->v_stride_slot, kv->v_stride_block);
}

// The pool's TMA maps, remembered per thread for the last few pools: a decode
// loop calls with the same pool every step, and encoding a map is a driver
// call.  A map holds only the pool's address, shape and strides (the key).
bool make_kv_maps(const pa_kv_cache_t* kv, pa::KvMaps* maps) {
  static const bool no_tma = std::getenv("PIE_B200_NO_TMA") != nullptr;
  if (no_tma) return false;
  struct Entry {
    pa_kv_cache_t key;
    int dev;
    pa::KvMaps maps;
    bool ok;
    bool used;
  };
  constexpr int kEntries = 4;
  thread_local Entry cache[kEntries] = {};
  thread_local int next = 0;
  auto same = [&](const pa_kv_cache_t& a) {
    return a.k == kv->k && a.v == kv->v && a.dtype == kv->dtype && a.num_blocks == kv->num_blocks &&
           a.block_size == kv->block_size && a.num_kv_heads == kv->num_kv_heads && a.head_dim == kv->head_dim &&
           a.k_stride_block == kv->k_stride_block && a.k_stride_slot == kv->k_stride_slot &&
           a.k_stride_head == kv->k_stride_head && a.v_stride_block == kv->v_stride_block &&
           a.v_stride_slot == kv->v_stride_slot && a.v_stride_head == kv->v_stride_head;
  };
  int dev = -1;
  cudaGetDevice(&dev);
  for (Entry& e : cache) {
    if (e.used && e.dev == dev && same(e.key)) {
      *maps = e.maps;
      return e.ok;
    }
  }
  Entry& e = cache[next];
  next = (next + 1) % kEntries;
  e.key = *kv;
  e.dev = dev;
  e.ok = encode_kv_maps(kv, &e.maps);
  e.used = true;
  *maps = e.maps;
  return e.ok;
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

struct WsLayout {
  size_t part_o, part_ml, tstart, total;
};
WsLayout ws_layout(int warps, int D, int B) {
  WsLayout l;
  l.part_o = 0;
  l.part_ml = align256(static_cast<size_t>(2) * warps * kNcMax * D * sizeof(float));
  l.tstart = l.part_ml + align256(static_cast<size_t>(2) * warps * kNcMax * 2 * sizeof(float));
  l.total = l.tstart + align256(static_cast<size_t>(B + 1) * sizeof(int));
  return l;
}

int run_decode_launch(pa::AttnParams& p, const pa_kv_cache_t* kv, void* ws, size_t ws_bytes, void* stream,
                      int phase, int plan_B);

// The sequences [first, first + n) of a decode problem as a problem of their
// own: every per-sequence pointer moves to row `first` (ragged rows keep their
// absolute row offsets through q_start).
pa::AttnParams seq_slice(const pa::AttnParams& p, int first, int n) {
  pa::AttnParams c = p;
  const long long f = first;
  c.bt = p.bt + f * p.bt_ss;
  c.nblk = p.nblk + f;
  c.qlen = p.qlen + f;
  c.kvlen = p.kvlen + f;
  if (p.q_start) {
    c.q_start = p.q_start + f;
  } else {
    c.q = static_cast<const unsigned short*>(p.q) + f * p.q_sb;
    c.o = static_cast<uint16_t*>(p.o) + f * p.o_sb;
    for (int r = 0; r < p.n_peers; ++r) c.o_peer[r] = static_cast<uint16_t*>(p.o_peer[r]) + f * p.o_sb;
    if (p.lse) c.lse = static_cast<uint16_t*>(p.lse) + f * p.l_sb;
  }
  c.B = n;
  return c;
}

// Split-K decode of any number of sequences: launches of at most
// kMaxDecodeSeqs sequences (the per-sequence tile scan of one launch lives in
// shared memory), one after another on the stream, sharing the workspace.
// Every launch of a split batch uses the launch plan of a full one, so the
// workspace that paged_attn_workspace_size reports fits each of them.
int run_decode(pa::AttnParams& p, const pa_kv_cache_t* kv, void* ws, size_t ws_bytes, void* stream,
               int phase = pa::DECODE_BOTH) {
  if (p.B <= kMaxDecodeSeqs) return run_decode_launch(p, kv, ws, ws_bytes, stream, phase, p.B);
  if (phase != pa::DECODE_BOTH)
    return fail(PA_ERR_UNSUPPORTED, "split / reduce as separate calls take at most %d sequences", kMaxDecodeSeqs);
  for (int first = 0; first < p.B; first += kMaxDecodeSeqs) {
    pa::AttnParams c = seq_slice(p, first, p.B - first < kMaxDecodeSeqs ? p.B - first : kMaxDecodeSeqs);
    const int rc = run_decode_launch(c, kv, ws, ws_bytes, stream, phase, kMaxDecodeSeqs);
    if (rc) return rc;
  }
  return PA_OK;
}

int run_decode_launch(pa::AttnParams& p, const pa_kv_cache_t* kv, void* ws, size_t ws_bytes, void* stream,
                      int phase, int plan_B) {
  if (p.B > kMaxDecodeSeqs)
    return fail(PA_ERR_UNSUPPORTED, "decode kernel supports at most %d sequences per launch", kMaxDecodeSeqs);
  if (p.maxq * p.G > kNcMax)
    return fail(PA_ERR_UNSUPPORTED, "decode kernel packs at most %d (q rows x group heads) columns", kNcMax);
  if (kv->dtype == PA_DTYPE_F32)
    return fail(PA_ERR_UNSUPPORTED, "the decode kernel reads fp16, bf16 or int8 pools (fp32 pools: paged_attn_forward)");
  if (p.B == 0 || p.maxq == 0) return PA_OK;
  const int nt = decode_nt(p);
  const int kv_k = kv_kind(kv->dtype);
  pa::KvMaps maps;
  const bool tma = make_kv_maps(kv, &maps);
  pa::DecodeLaunch plan;
  if (cached_plan(kv_k, p.q_bf16, kv->head_dim, nt, plan_B, tma, &plan) != 0)
    return fail(PA_ERR_CUDA, "could not plan the decode launch (no CUDA device?)");
  const int warps = plan.ctas * plan.warps_per_cta;
  const WsLayout L = ws_layout(warps, kv->head_dim, plan_B);
  if (!ws || ws_bytes < L.total)
    return fail(PA_ERR_WORKSPACE, "decode workspace needs %zu bytes, got %zu", L.total, ws_bytes);
  if (!al(ws, 256)) return fail(PA_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  char* base = static_cast<char*>(ws);
  p.part_o = reinterpret_cast<float*>(base + L.part_o);
  p.part_ml = reinterpret_cast<float*>(base + L.part_ml);
  p.tstart = reinterpret_cast<int*>(base + L.tstart);
  p.num_warps_total = warps;
  cudaError_t e = pa::launch_decode(p, tma ? &maps : nullptr, kv_k, p.q_bf16, kv->head_dim, nt, plan,
                                    static_cast<cudaStream_t>(stream), phase);
  if (e != cudaSuccess) return cuda_fail(e, "decode launch");
  return PA_OK;
}

// 4-D TMA map over Q [num_seqs, num_q_heads, max_q_len, 128] (d contiguous):
// box = 64 columns x 128 rows, 128-byte swizzle; rows past max_q_len read as zeros.
// Ragged rows (q_total > 0): Q packed as [q_total, num_q_heads, 128], mapped as
// [1, num_q_heads, q_total, 128]; rows past q_total read as zeros.
bool make_q_map(CUtensorMap* m, const pa_attn_io_t* io, int D, int B, int q_total = 0) {
  auto enc = encode_fn();
  if (!enc || D != 128) return false;
  const bool ragged = q_total > 0;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(ragged ? q_total : io->max_q_len),
                              static_cast<cuuint64_t>(io->num_q_heads), static_cast<cuuint64_t>(ragged ? 1 : B)};
  const long long st[3] = {io->q_stride_row, io->q_stride_head,
                           ragged ? io->q_stride_row * static_cast<long long>(q_total) : io->q_stride_seq};
  for (long long x : st)
    if (x <= 0) return false;
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(st[0] * 2), static_cast<cuuint64_t>(st[1] * 2),
                                 static_cast<cuuint64_t>(st[2] * 2)};
  const cuuint32_t box[4] = {64, 128, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, const_cast<void*>(io->q), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Scratch of an INT8 prefill on the tcgen05 kernel: the blocks the call reads,
// dequantised to fp16 (see kv_dequant.cu).  gather when the call's table holds
// fewer blocks than the pool (then a scratch block table too), else a mirror
// of the whole pool.  0 when the tcgen05 kernel cannot take the problem or the
// scratch would exceed kMaxDequantScratch (the mma.sync kernel then reads the
// int8 pool directly).
constexpr size_t kMaxDequantScratch = static_cast<size_t>(16) << 30;
struct DequantLayout {
  size_t dk, dv, dbt, total;
  long long blocks;
  bool gather;
};
DequantLayout dequant_layout(const pa::AttnParams& p, const pa_kv_cache_t* kv) {
  DequantLayout l{};
  if (kv->dtype != PA_DTYPE_I8 || !pa::prefill_tc_supported(pa::KV_F16, kv->head_dim, kv->block_size) ||
      std::getenv("PIE_B200_NO_TCGEN05"))
    return l;
  const long long table_blocks = static_cast<long long>(p.B) * p.bt_cols;
  l.gather = table_blocks <= kv->num_blocks;
  l.blocks = l.gather ? table_blocks : kv->num_blocks;
  const size_t pool = align256(static_cast<size_t>(l.blocks) * kv->block_size * kv->num_kv_heads * kv->head_dim * 2);
  l.dk = 0;
  l.dv = pool;
  l.dbt = 2 * pool;
  l.total = l.dbt + (l.gather ? align256(static_cast<size_t>(table_blocks) * 4) : 0);
  if (l.blocks == 0 || l.total > kMaxDequantScratch) l = DequantLayout{};
  return l;
}

int run_prefill(pa::AttnParams& p, const pa_kv_cache_t* kv, const pa_attn_io_t* io, void* stream,
                void* ws = nullptr, size_t ws_bytes = 0) {
  if (p.B == 0 || p.maxq == 0) return PA_OK;
  if (p.B > 65535) return fail(PA_ERR_UNSUPPORTED, "prefill kernel supports at most 65535 sequences per call");
  const int kvk = kv_kind(kv->dtype);
  const DequantLayout dq = dequant_layout(p, kv);
  if (dq.total && ws && ws_bytes >= dq.total && al(ws, 256) && al(io->o, 16) && row_al(io->o_stride_seq, 2, 16) &&
      row_al(io->o_stride_head, 2, 16) && row_al(io->o_stride_row, 2, 16)) {
    // INT8 pool: dequantise the blocks the call reads once, then the fp16 tcgen05 kernel over them
    char* base = static_cast<char*>(ws);
    __half* dk = reinterpret_cast<__half*>(base + dq.dk);
    __half* dv = reinterpret_cast<__half*>(base + dq.dv);
    int* dbt = dq.gather ? reinterpret_cast<int*>(base + dq.dbt) : nullptr;
    cudaError_t e = pa::launch_kv_dequant(p, dk, dv, dbt, dq.gather ? 1 : 0, kv->head_dim,
                                          static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "INT8 prefill dequantisation launch");
    pa_kv_cache_t f = *kv;
    f.k = dk;
    f.v = dv;
    f.dtype = PA_DTYPE_F16;
    f.num_blocks = static_cast<int32_t>(dq.blocks);
    f.k_stride_head = f.v_stride_head = kv->head_dim;
    f.k_stride_slot = f.v_stride_slot = static_cast<int64_t>(kv->num_kv_heads) * kv->head_dim;
    f.k_stride_block = f.v_stride_block = static_cast<int64_t>(kv->block_size) * kv->num_kv_heads * kv->head_dim;
    f.k_scale = f.v_scale = nullptr;
    pa::AttnParams q = p;
    fill_cache(q, &f);
    q.status = p.status;
    if (dq.gather) {
      q.bt = dbt;
      q.bt_ss = p.bt_cols;
      q.bt_sc = 1;
    }
    pa::KvMaps maps;
    CUtensorMap qmap;
    if (make_kv_maps(&f, &maps) && make_q_map(&qmap, io, kv->head_dim, p.B, p.q_start ? p.q_total : 0)) {
      e = pa::launch_prefill_tc(q, maps.k, maps.v, qmap, pa::KV_F16, static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) return cuda_fail(e, "prefill (tcgen05, dequantised INT8) launch");
      return PA_OK;
    }
    return fail(PA_ERR_CUDA, "could not encode the TMA maps of the dequantised INT8 pool");
  }
  if (pa::prefill_tc_supported(kvk, kv->head_dim, kv->block_size) && !std::getenv("PIE_B200_NO_TCGEN05") &&
      al(io->o, 16) && row_al(io->o_stride_seq, 2, 16) && row_al(io->o_stride_head, 2, 16) &&
      row_al(io->o_stride_row, 2, 16)) {
    pa::KvMaps maps;
    CUtensorMap qmap;
    if (make_kv_maps(kv, &maps) && make_q_map(&qmap, io, kv->head_dim, p.B, p.q_start ? p.q_total : 0)) {
      cudaError_t e = pa::launch_prefill_tc(p, maps.k, maps.v, qmap, kvk, static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) return cuda_fail(e, "prefill (tcgen05) launch");
      return PA_OK;
    }
  }
  cudaError_t e = pa::launch_prefill(p, kvk, kv->head_dim, kv->dtype == PA_DTYPE_BF16,
                                     static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
  return PA_OK;
}

int build_write(const pa_kv_new_t* nw, const pa_kv_cache_t* kv, const pa_paging_t* pg, int32_t* status,
                pa::WriteParams& w) {
  int rc = check_cache(kv);
  if (rc) return rc;
  if (!pg) return fail(PA_ERR_INVALID, "paging descriptor is NULL");
  if (!nw) return fail(PA_ERR_INVALID, "new K/V descriptor is NULL");
  if (nw->dtype != PA_DTYPE_F16 && nw->dtype != PA_DTYPE_BF16 && nw->dtype != PA_DTYPE_F32)
    return fail(PA_ERR_INVALID, "new K/V dtype must be fp16, bf16 or fp32");
  if (nw->num_tokens < 0) return fail(PA_ERR_INVALID, "num_tokens < 0");
  if (static_cast<long long>(nw->num_tokens) * kv->num_kv_heads > (1LL << 26))
    return fail(PA_ERR_UNSUPPORTED, "write of more than 2^26 (token, kv head) rows in one call");
  const int e = elt_size(nw->dtype);
  if (nw->num_tokens > 0) {
    if (!nw->k_new || !nw->v_new || !nw->seq_index || !nw->positions || !pg->block_table)
      return fail(PA_ERR_INVALID, "write: NULL pointer");
    if (!al(nw->k_new, 16) || !al(nw->v_new, 16) || !row_al(nw->k_stride_token, e, 16) ||
        !row_al(nw->k_stride_head, e, 16) || !row_al(nw->v_stride_token, e, 16) || !row_al(nw->v_stride_head, e, 16))
      return fail(PA_ERR_INVALID, "new K/V rows must be 16-byte aligned (contiguous head_dim)");
  }
  w = pa::WriteParams{};
  w.k_new = nw->k_new;
  w.v_new = nw->v_new;
  w.kn_st = nw->k_stride_token;
  w.kn_sh = nw->k_stride_head;
  w.vn_st = nw->v_stride_token;
  w.vn_sh = nw->v_stride_head;
  w.in_dtype = nw->dtype;
  w.seq_idx = nw->seq_index;
  w.pos = nw->positions;
  w.T = nw->num_tokens;
  w.bt = pg->block_table;
  w.bt_ss = pg->bt_stride_seq;
  w.bt_sc = pg->bt_stride_col;
  w.bt_cols = pg->bt_cols;
  w.num_seqs = pg->num_seqs;
  w.k = kv->k;
  w.v = kv->v;
  w.k_sblk = kv->k_stride_block;
  w.k_sslot = kv->k_stride_slot;
  w.k_shead = kv->k_stride_head;
  w.v_sblk = kv->v_stride_block;
  w.v_sslot = kv->v_stride_slot;
  w.v_shead = kv->v_stride_head;
  w.cache_dtype = kv->dtype;
  w.ks = kv->k_scale;
  w.vs = kv->v_scale;
  w.ks_sblk = kv->ks_stride_block;
  w.ks_sslot = kv->ks_stride_slot;
  w.ks_shead = kv->ks_stride_head;
  w.vs_sblk = kv->vs_stride_block;
  w.vs_sslot = kv->vs_stride_slot;
  w.vs_shead = kv->vs_stride_head;
  w.scale_f32 = kv->scale_dtype == PA_DTYPE_F32;
  w.Hkv = kv->num_kv_heads;
  w.D = kv->head_dim;
  w.BS = kv->block_size;
  w.log2BS = ilog2(kv->block_size);
  w.NB = kv->num_blocks;
  w.status = status;
  return PA_OK;
}

// ---------------------------------------------------------------------------
// Split-K scratch for paged_attn_decode_noalloc: a fixed array that every GPU
// loading this library holds in device memory until the process exits, so the
// entry point never allocates.  Host code cannot use the symbol's name as a
// device address (on the host it names a shadow variable), so the address is
// looked up once per device with cudaGetSymbolAddress while that device is
// current.
// ---------------------------------------------------------------------------
constexpr size_t kStaticScratchBytes = static_cast<size_t>(24) << 20;  // 24 MiB per device
static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

// Device address of g_decode_scratch on the current device (set up on first
// use per device).
int static_scratch_address(void** out) {
  static std::mutex mu;
  static std::map<int, void*> addr;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lk(mu);
  auto it = addr.find(dev);
  if (it != addr.end()) {
    *out = it->second;
    return PA_OK;
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_decode_scratch);
  if (e != cudaSuccess || p == nullptr) return cuda_fail(e, "cudaGetSymbolAddress(decode scratch)");
  addr[dev] = p;
  *out = p;
  return PA_OK;
}

}  // namespace

extern "C" {

int paged_attn_workspace_size(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg,
                              size_t* bytes) {
  g_err[0] = 0;
  if (!bytes) return fail(PA_ERR_INVALID, "bytes is NULL");
  *bytes = 0;
  pa::AttnParams p;
  int rc = build_attn(io, kv, pg, nullptr, p);
  if (rc) return rc;
  if (p.B == 0 || p.maxq == 0) return PA_OK;
  if (!use_decode(p, kv)) {
    *bytes = dequant_layout(p, kv).total;  // 0 unless an INT8 pool takes the tcgen05 prefill
    return PA_OK;
  }
  const int per_launch = p.B < kMaxDecodeSeqs ? p.B : kMaxDecodeSeqs;
  pa::KvMaps maps;
  const bool tma = make_kv_maps(kv, &maps);
  pa::DecodeLaunch plan;
  if (cached_plan(kv_kind(kv->dtype), p.q_bf16, kv->head_dim, decode_nt(p), per_launch, tma, &plan) != 0)
    return fail(PA_ERR_CUDA, "could not plan the decode launch (no CUDA device?)");
  *bytes = ws_layout(plan.ctas * plan.warps_per_cta, kv->head_dim, per_launch).total;
  return PA_OK;
}

int paged_attn_forward(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg, void* workspace,
                       size_t workspace_bytes, int32_t* status, void* stream) {
  g_err[0] = 0;
  pa::AttnParams p;
  int rc = build_attn(io, kv, pg, status, p);
  if (rc) return rc;
  if (use_decode(p, kv)) return run_decode(p, kv, workspace, workspace_bytes, stream);
  return run_prefill(p, kv, io, stream, workspace, workspace_bytes);
}

int paged_attn_decode(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg, void* workspace,
                      size_t workspace_bytes, int32_t* status, void* stream) {
  g_err[0] = 0;
  pa::AttnParams p;
  int rc = build_attn(io, kv, pg, status, p);
  if (rc) return rc;
  return run_decode(p, kv, workspace, workspace_bytes, stream);
}

int paged_attn_decode_split(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg, void* workspace,
                            size_t workspace_bytes, int32_t* status, void* stream) {
  g_err[0] = 0;
  pa::AttnParams p;
  int rc = build_attn(io, kv, pg, status, p);
  if (rc) return rc;
  return run_decode(p, kv, workspace, workspace_bytes, stream, pa::DECODE_SPLIT);
}

int paged_attn_reduce(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg, void* workspace,
                      size_t workspace_bytes, int32_t* status, void* stream) {
  g_err[0] = 0;
  pa::AttnParams p;
  int rc = build_attn(io, kv, pg, status, p);
  if (rc) return rc;
  return run_decode(p, kv, workspace, workspace_bytes, stream, pa::DECODE_MERGE);
}

int paged_attn_varlen(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg, const int32_t* q_start,
                      int32_t total_q_rows, void* workspace, size_t workspace_bytes, int32_t* status, void* stream) {
  g_err[0] = 0;
  if (!q_start) return fail(PA_ERR_INVALID, "q_start is NULL");
  if (total_q_rows < 0) return fail(PA_ERR_INVALID, "total_q_rows < 0");
  pa::AttnParams p;
  int rc = build_attn(io, kv, pg, status, p);
  if (rc) return rc;
  if (total_q_rows == 0) return PA_OK;
  p.q_start = q_start;
  p.q_total = total_q_rows;
  if (use_decode(p, kv)) return run_decode(p, kv, workspace, workspace_bytes, stream);
  return run_prefill(p, kv, io, stream, workspace, workspace_bytes);
}

int paged_attn_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  g_err[0] = 0;
  if (!ptr || !ipc_handle || bytes == 0) return fail(PA_ERR_INVALID, "peer_alloc: NULL argument or zero size");
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "peer_alloc: cudaMalloc");
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "peer_alloc: IPC handle");
  }
  *ptr = p;
  return PA_OK;
}

int paged_attn_peer_free(void* ptr) {
  g_err[0] = 0;
  if (!ptr) return PA_OK;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? PA_OK : cuda_fail(e, "peer_free");
}

int paged_attn_peer_open(const void* ipc_handle, void** ptr) {
  g_err[0] = 0;
  if (!ptr || !ipc_handle) return fail(PA_ERR_INVALID, "peer_open: NULL argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? PA_OK : cuda_fail(e, "peer_open: cudaIpcOpenMemHandle");
}

int paged_attn_peer_close(void* ptr) {
  g_err[0] = 0;
  if (!ptr) return PA_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? PA_OK : cuda_fail(e, "peer_close");
}

int paged_attn_decode_peers(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg, void* workspace,
                            size_t workspace_bytes, void* const* o_peers, int32_t n_peers, int32_t* status,
                            void* stream) {
  g_err[0] = 0;
  if (!o_peers || n_peers < 1 || n_peers > pa::kMaxPeers)
    return fail(PA_ERR_INVALID, "decode_peers: 1..%d output pointers required", pa::kMaxPeers);
  pa::AttnParams p;
  int rc = build_attn(io, kv, pg, status, p);
  if (rc) return rc;
  for (int r = 0; r < n_peers; ++r) {
    if (!o_peers[r] || !al(o_peers[r], 2)) return fail(PA_ERR_INVALID, "decode_peers: output %d NULL or misaligned", r);
    p.o_peer[r] = o_peers[r];
  }
  p.n_peers = n_peers;
  if (!use_decode(p, kv))
    return fail(PA_ERR_UNSUPPORTED, "decode_peers: max_q_len * (num_q_heads / num_kv_heads) must be <= %d", kNcMax);
  return run_decode(p, kv, workspace, workspace_bytes, stream);
}

int paged_attn_peer_barrier(int32_t* local_flags, int32_t* const* peer_flags, int32_t n_peers, int32_t rank,
                            int32_t epoch, int32_t* status, void* stream) {
  g_err[0] = 0;
  if (!local_flags || !peer_flags || n_peers < 1 || n_peers > pa::kMaxPeers || rank < 0 || rank >= n_peers)
    return fail(PA_ERR_INVALID, "peer_barrier: bad arguments");
  pa::PeerFlags pf{};
  for (int r = 0; r < n_peers; ++r) {
    if (!peer_flags[r]) return fail(PA_ERR_INVALID, "peer_barrier: flag pointer %d is NULL", r);
    pf.flag[r] = peer_flags[r];
  }
  cudaError_t e = pa::launch_peer_barrier(local_flags, pf, n_peers, rank, epoch, status,
                                          static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? PA_OK : cuda_fail(e, "peer barrier launch");
}

int paged_attn_prefill(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg, int32_t* status,
                       void* stream) {
  g_err[0] = 0;
  pa::AttnParams p;
  int rc = build_attn(io, kv, pg, status, p);
  if (rc) return rc;
  return run_prefill(p, kv, io, stream);
}

int kv_write_quant(const pa_kv_new_t* nw, const pa_kv_cache_t* kv, const pa_paging_t* pg, int32_t* status,
                   void* stream) {
  g_err[0] = 0;
  pa::WriteParams w;
  int rc = build_write(nw, kv, pg, status, w);
  if (rc) return rc;
  if (kv->dtype != PA_DTYPE_I8) return fail(PA_ERR_INVALID, "kv_write_quant needs an int8 pool");
  cudaError_t e = pa::launch_kv_write(w, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "kv_write_quant launch");
  return PA_OK;
}

int kv_write_copy(const pa_kv_new_t* nw, const pa_kv_cache_t* kv, const pa_paging_t* pg, int32_t* status,
                  void* stream) {
  g_err[0] = 0;
  pa::WriteParams w;
  int rc = build_write(nw, kv, pg, status, w);
  if (rc) return rc;
  if (kv->dtype == PA_DTYPE_I8) return fail(PA_ERR_INVALID, "kv_write_copy needs an fp16 / bf16 pool");
  cudaError_t e = pa::launch_kv_write(w, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "kv_write_copy launch");
  return PA_OK;
}

// Decode with the split-K scratch taken from the library's own static device
// array (see paged_attn_b200.h).  The persistent grid keeps every SM but may use
// fewer warps per CTA so that the partials fit the fixed scratch.
int paged_attn_decode_noalloc(const pa_attn_io_t* io, const pa_kv_cache_t* kv, const pa_paging_t* pg,
                              int32_t* status, void* stream) {
  g_err[0] = 0;
  pa::AttnParams p;
  int rc = build_attn(io, kv, pg, status, p);
  if (rc) return rc;
  if (p.B > kMaxDecodeSeqs)
    return fail(PA_ERR_UNSUPPORTED, "decode (no-alloc) supports at most %d sequences per call", kMaxDecodeSeqs);
  if (p.maxq * p.G > kNcMax)
    return fail(PA_ERR_UNSUPPORTED, "decode (no-alloc) packs at most %d (q rows x group heads) columns", kNcMax);
  if (kv->dtype == PA_DTYPE_F32)
    return fail(PA_ERR_UNSUPPORTED, "decode (no-alloc) reads fp16, bf16 or int8 pools");
  if (p.B == 0 || p.maxq == 0) return PA_OK;
  void* scratch = nullptr;
  rc = static_scratch_address(&scratch);
  if (rc) return rc;
  const int nt = decode_nt(p);
  const int kv_k = kv_kind(kv->dtype);
  pa::KvMaps maps;
  const bool tma = make_kv_maps(kv, &maps);
  pa::DecodeLaunch plan;
  if (cached_plan(kv_k, p.q_bf16, kv->head_dim, nt, p.B, tma, &plan) != 0)
    return fail(PA_ERR_CUDA, "could not plan the decode launch (no CUDA device?)");
  // dynamic shared memory = fixed part + warps * per-warp ring
  const size_t fixed = static_cast<size_t>(((p.B + 1) * 4 + 127) & ~127) + 1024;
  const size_t warp_bytes = (plan.smem - fixed) / plan.warps_per_cta;
  int nw = plan.warps_per_cta;
  while (nw > 0 && ws_layout(plan.ctas * nw, kv->head_dim, p.B).total > kStaticScratchBytes) --nw;
  if (nw < 1)
    return fail(PA_ERR_UNSUPPORTED, "decode (no-alloc): %d CTAs x 1 warp need more than the %zu-byte static scratch",
                plan.ctas, kStaticScratchBytes);
  const WsLayout L = ws_layout(plan.ctas * nw, kv->head_dim, p.B);
  char* base = static_cast<char*>(scratch);
  p.part_o = reinterpret_cast<float*>(base + L.part_o);
  p.part_ml = reinterpret_cast<float*>(base + L.part_ml);
  p.tstart = reinterpret_cast<int*>(base + L.tstart);
  p.num_warps_total = plan.ctas * nw;
  pa::DecodeLaunch pl = plan;
  pl.warps_per_cta = nw;
  pl.smem = fixed + nw * warp_bytes;
  cudaError_t e = pa::launch_decode(p, tma ? &maps : nullptr, kv_k, p.q_bf16, kv->head_dim, nt, pl,
                                    static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "decode (no-alloc) launch");
  return PA_OK;
}

// 2-D TMA map over a row-major [rows, cols] 16-bit matrix: box of 64 columns x 128 rows, 128-byte swizzle.
static bool make_rows_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long row_stride,
                          unsigned box_rows) {
  auto enc = encode_fn();
  if (!enc || rows < 1 || cols < 64) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride * 2)};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int kv_project_write(const pa_kv_proj_t* pj, const pa_kv_cache_t* kv, const pa_paging_t* pg, int32_t* status,
                     void* stream) {
  g_err[0] = 0;
  if (!pj) return fail(PA_ERR_INVALID, "projection descriptor is NULL");
  if (!pg) return fail(PA_ERR_INVALID, "paging descriptor is NULL");
  int rc = check_cache(kv);
  if (rc) return rc;
  if (kv->dtype == PA_DTYPE_F32) return fail(PA_ERR_UNSUPPORTED, "kv_project_write writes int8, fp16 or bf16 pools");
  if (kv->head_dim != 128) return fail(PA_ERR_UNSUPPORTED, "kv_project_write needs head_dim 128");
  if (pj->dtype != PA_DTYPE_F16 && pj->dtype != PA_DTYPE_BF16)
    return fail(PA_ERR_INVALID, "x / w must be fp16 or bf16");
  if (pj->num_tokens < 0) return fail(PA_ERR_INVALID, "num_tokens < 0");
  if (pj->d_model <= 0 || pj->d_model % 128) return fail(PA_ERR_UNSUPPORTED, "d_model must be a positive multiple of 128");
  if (kv->dtype == PA_DTYPE_I8 && kv->ks_stride_slot == 0 && kv->block_size > 1)
    return fail(PA_ERR_INVALID, "an int8 pool written per token needs per-token scales");
  if (pj->num_tokens == 0) return PA_OK;
  if (!pj->x || !pj->w || !pj->seq_index || !pj->positions || !pg->block_table)
    return fail(PA_ERR_INVALID, "kv_project_write: NULL pointer");
  if (!al(pj->x, 16) || !al(pj->w, 16) || !row_al(pj->x_stride, 2, 16) || !row_al(pj->w_stride, 2, 16) ||
      pj->x_stride < pj->d_model || pj->w_stride < pj->d_model)
    return fail(PA_ERR_INVALID, "x / w rows must be 16-byte aligned and hold d_model values");
  if (pj->bias && !al(pj->bias, 4)) return fail(PA_ERR_INVALID, "bias misaligned");
  pa::ProjParams p{};
  p.k = kv->k;
  p.v = kv->v;
  p.k_sblk = kv->k_stride_block;
  p.k_sslot = kv->k_stride_slot;
  p.k_shead = kv->k_stride_head;
  p.v_sblk = kv->v_stride_block;
  p.v_sslot = kv->v_stride_slot;
  p.v_shead = kv->v_stride_head;
  p.cache_dtype = kv->dtype;
  p.ks = kv->k_scale;
  p.vs = kv->v_scale;
  p.ks_sblk = kv->ks_stride_block;
  p.ks_sslot = kv->ks_stride_slot;
  p.ks_shead = kv->ks_stride_head;
  p.vs_sblk = kv->vs_stride_block;
  p.vs_sslot = kv->vs_stride_slot;
  p.vs_shead = kv->vs_stride_head;
  p.scale_f32 = kv->scale_dtype == PA_DTYPE_F32;
  p.Hkv = kv->num_kv_heads;
  p.D = kv->head_dim;
  p.BS = kv->block_size;
  p.log2BS = ilog2(kv->block_size);
  p.NB = kv->num_blocks;
  p.seq_idx = pj->seq_index;
  p.pos = pj->positions;
  p.T = pj->num_tokens;
  p.bt = pg->block_table;
  p.bt_ss = pg->bt_stride_seq;
  p.bt_sc = pg->bt_stride_col;
  p.bt_cols = pg->bt_cols;
  p.num_seqs = pg->num_seqs;
  p.status = status;
  p.d_model = pj->d_model;
  p.bias = pj->bias;
  CUtensorMap xmap, wmap;
  // boxes: 64 columns x 128 tokens of x, 64 columns x 256 outputs (two heads) of w
  if (!make_rows_map(&xmap, pj->x, pj->num_tokens, pj->d_model, pj->x_stride, 128) ||
      !make_rows_map(&wmap, pj->w, 2LL * kv->num_kv_heads * kv->head_dim, pj->d_model, pj->w_stride, 256))
    return fail(PA_ERR_CUDA, "could not encode the TMA maps of x / w");
  cudaError_t e = pa::launch_kv_project(p, xmap, wmap, pj->dtype == PA_DTYPE_BF16, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? PA_OK : cuda_fail(e, "kv_project_write launch");
}

static int block_pool_check(const pa_block_pool_t* pool, pa::PoolParams& p) {
  if (!pool) return fail(PA_ERR_INVALID, "block pool descriptor is NULL");
  if (pool->num_blocks < 0 || pool->max_seqs < 0 || pool->max_blocks_per_seq < 0)
    return fail(PA_ERR_INVALID, "block pool sizes must be non-negative");
  if (pool->table_stride < pool->max_blocks_per_seq)
    return fail(PA_ERR_INVALID, "table_stride %lld is narrower than max_blocks_per_seq %d",
                static_cast<long long>(pool->table_stride), pool->max_blocks_per_seq);
  if (!pool->free_stack || !pool->free_top || !pool->count || (!pool->table && pool->max_seqs > 0))
    return fail(PA_ERR_INVALID, "block pool array pointer is NULL");
  p.free_stack = pool->free_stack;
  p.free_top = pool->free_top;
  p.table = pool->table;
  p.count = pool->count;
  p.table_stride = pool->table_stride;
  p.num_blocks = pool->num_blocks;
  p.max_seqs = pool->max_seqs;
  p.max_blocks_per_seq = pool->max_blocks_per_seq;
  return PA_OK;
}

int block_pool_init(const pa_block_pool_t* pool, void* stream) {
  g_err[0] = 0;
  pa::PoolParams p;
  int rc = block_pool_check(pool, p);
  if (rc) return rc;
  cudaError_t e = pa::launch_block_pool_init(p, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? PA_OK : cuda_fail(e, "block_pool_init launch");
}

int block_pool_apply(const pa_block_pool_t* pool, const int32_t* ops, int32_t n_ops, int32_t* results, void* stream) {
  g_err[0] = 0;
  pa::PoolParams p;
  int rc = block_pool_check(pool, p);
  if (rc) return rc;
  if (n_ops < 0) return fail(PA_ERR_INVALID, "n_ops < 0");
  if (n_ops > 0 && !ops) return fail(PA_ERR_INVALID, "ops is NULL");
  cudaError_t e = pa::launch_block_pool_apply(p, ops, n_ops, results, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? PA_OK : cuda_fail(e, "block_pool_apply launch");
}

int block_pool_step(const pa_block_pool_t* pool, const int32_t* seq_slot, const int32_t* q_len, const int32_t* kv_len,
                    const int32_t* cu_seqlens, int32_t num_seqs, int32_t* block_table, int64_t bt_stride,
                    int32_t bt_cols, int32_t* num_blocks, int32_t* positions, int32_t* token_seq,
                    int32_t total_tokens, int32_t* status, void* stream) {
  g_err[0] = 0;
  pa::PoolParams p;
  int rc = block_pool_check(pool, p);
  if (rc) return rc;
  if (num_seqs < 0 || bt_cols < 0 || total_tokens < 0) return fail(PA_ERR_INVALID, "negative step size");
  if (num_seqs == 0) return PA_OK;
  if (!seq_slot || !q_len || !kv_len || !cu_seqlens || !num_blocks || (!block_table && bt_cols > 0))
    return fail(PA_ERR_INVALID, "block_pool_step: NULL argument");
  if (bt_cols > 0 && bt_stride < bt_cols) return fail(PA_ERR_INVALID, "bt_stride narrower than bt_cols");
  pa::StepParams s{};
  s.seq_slot = seq_slot;
  s.q_len = q_len;
  s.kv_len = kv_len;
  s.cu_seqlens = cu_seqlens;
  s.num_seqs = num_seqs;
  s.block_table = block_table;
  s.bt_stride = bt_stride;
  s.bt_cols = bt_cols;
  s.num_blocks = num_blocks;
  s.positions = positions;
  s.token_seq = token_seq;
  s.total_tokens = total_tokens;
  s.status = status;
  cudaError_t e = pa::launch_block_pool_step(p, s, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? PA_OK : cuda_fail(e, "block_pool_step launch");
}

const char* paged_attn_error_string(void) { return g_err; }

const char* paged_attn_version(void) { return "0.1.0"; }

}  // extern "C"
