// fa8_api.cu — C-ABI host side of the sm_100a FP8 attention forward.
//
// Replaces the reference's host path (csrc/flash_attention.cu:462-543:
// fill_params, launch_flash_attn_fp8_kernel, flash_attn_fp8_forward) with a
// status-returning, non-blocking launcher:
//   * no cudaDeviceSynchronize after the launch (reference :539) and no
//     exit() on error (reference include/attention_api.cuh:28-37);
//   * the dynamic shared-memory attribute is set once per device and kernel
//     instead of on every call (reference :503);
//   * operands are described to the kernel as TMA tensor maps (4-D:
//     innermost dim, rows, heads, batch) so ragged sequence ends are
//     zero-filled by hardware instead of requiring S % 64 == 0 (reference
//     F7: no load predicates).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <map>
#include <mutex>
#include <utility>

#include "../../include/fa8.h"
#include "fa8_fwd_kernel.cuh"

namespace {

thread_local char g_last_msg[512] = "";
std::atomic<uint64_t> g_launches{0};

int set_cuda_error(cudaError_t e, const char* where) {
  snprintf(g_last_msg, sizeof(g_last_msg), "%s: %s", where, cudaGetErrorString(e));
  return FA8_ERR_CUDA;
}
int set_msg(int status, const char* msg) {
  snprintf(g_last_msg, sizeof(g_last_msg), "%s", msg);
  return status;
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 4-D byte tensor map: dims {inner, rows, heads, batch}, box {box_inner, box_rows, 1, 1}.
int make_map_u8(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows,
                uint64_t heads, uint64_t batch, uint64_t row_stride, uint64_t head_stride,
                uint64_t batch_stride, uint32_t box_inner, uint32_t box_rows,
                CUtensorMapSwizzle swz) {
  auto enc = get_encode_fn();
  if (!enc) return set_msg(FA8_ERR_DRIVER, "cuTensorMapEncodeTiled entry point not found");
  cuuint64_t dims[4] = {inner, rows, heads, batch};
  cuuint64_t strides[3] = {row_stride, head_stride, batch_stride};  // bytes
  cuuint32_t box[4] = {box_inner, box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    snprintf(g_last_msg, sizeof(g_last_msg), "cuTensorMapEncodeTiled failed (CUresult %d)",
             (int)r);
    return FA8_ERR_ALIGNMENT;
  }
  return FA8_OK;
}

template <int D, bool kVmn>
int setup_kernel_attr(int dev) {
  static std::once_flag flags[64];
  static cudaError_t errs[64];
  if (dev < 0 || dev >= 64) return set_msg(FA8_ERR_INVALID_ARG, "device index out of range");
  std::call_once(flags[dev], [dev] {
    errs[dev] = cudaFuncSetAttribute(fa8::fa8_fwd_kernel<D, kVmn>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     fa8::TileCfg<D>::kSmemAlloc);
  });
  if (errs[dev] != cudaSuccess) return set_cuda_error(errs[dev], "cudaFuncSetAttribute");
  return FA8_OK;
}

// SM budget: a stream of a green context that owns `want` SMs (a multiple of
// 8, the partition granularity on sm_90+), created once per (device, count)
// and kept for the life of the process. *out = nullptr when the budget covers
// the whole GPU (launch on the caller's stream).
template <typename F>
F driver_fn(const char* name) {
  void* ptr = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion(name, &ptr, 12080, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<F>(ptr);
}

int budget_stream(int dev, int n_sms, cudaStream_t* out) {
  *out = nullptr;
  int total = 0;
  cudaError_t ce = cudaDeviceGetAttribute(&total, cudaDevAttrMultiProcessorCount, dev);
  if (ce != cudaSuccess) return set_cuda_error(ce, "cudaDeviceGetAttribute (SM count)");
  const int want = (n_sms + 7) / 8 * 8;
  if (want >= total) return FA8_OK;
  static std::mutex mu;
  static std::map<std::pair<int, int>, cudaStream_t> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find({dev, want});
  if (it != cache.end()) {
    *out = it->second;
    return FA8_OK;
  }
  auto get_dev = driver_fn<decltype(&cuDeviceGet)>("cuDeviceGet");
  auto get_res = driver_fn<decltype(&cuDeviceGetDevResource)>("cuDeviceGetDevResource");
  auto split = driver_fn<decltype(&cuDevSmResourceSplitByCount)>("cuDevSmResourceSplitByCount");
  auto gen = driver_fn<decltype(&cuDevResourceGenerateDesc)>("cuDevResourceGenerateDesc");
  auto mk_ctx = driver_fn<decltype(&cuGreenCtxCreate)>("cuGreenCtxCreate");
  auto mk_stream = driver_fn<decltype(&cuGreenCtxStreamCreate)>("cuGreenCtxStreamCreate");
  if (!get_dev || !get_res || !split || !gen || !mk_ctx || !mk_stream)
    return set_msg(FA8_ERR_DRIVER, "sm_budget: green-context driver entry points not found");
  CUdevice cu_dev;
  CUdevResource all, grp, rem;
  CUdevResourceDesc desc;
  CUgreenCtx gctx;
  CUstream cs;
  unsigned int n_groups = 1;
  CUresult r = get_dev(&cu_dev, dev);
  if (r == CUDA_SUCCESS) r = get_res(cu_dev, &all, CU_DEV_RESOURCE_TYPE_SM);
  if (r == CUDA_SUCCESS) r = split(&grp, &n_groups, &all, &rem, 0, (unsigned)want);
  if (r == CUDA_SUCCESS && n_groups < 1) r = CUDA_ERROR_INVALID_VALUE;
  if (r == CUDA_SUCCESS) r = gen(&desc, &grp, 1);
  if (r == CUDA_SUCCESS) r = mk_ctx(&gctx, desc, cu_dev, CU_GREEN_CTX_DEFAULT_STREAM);
  if (r == CUDA_SUCCESS) r = mk_stream(&cs, gctx, CU_STREAM_NON_BLOCKING, 0);
  if (r != CUDA_SUCCESS) {
    snprintf(g_last_msg, sizeof(g_last_msg), "sm_budget: green context of %d SMs failed (CUresult %d)",
             want, (int)r);
    return FA8_ERR_DRIVER;
  }
  cache[{dev, want}] = reinterpret_cast<cudaStream_t>(cs);
  *out = reinterpret_cast<cudaStream_t>(cs);
  return FA8_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Split-KV plan of a call: shares per query tile and the workspace layout
// [counters (qtiles x 4 B, padded to 256 B) | part_lse | part_o].
struct SplitPlan {
  int splits = 1;
  int64_t qtiles = 0, cnt_bytes = 0, lse_bytes = 0, o_bytes = 0;
  int64_t bytes() const { return splits > 1 ? cnt_bytes + lse_bytes + o_bytes : 0; }
};
constexpr int kSmCount = 148;
constexpr int kMaxSplits = fa8::kMaxKvSplits;
constexpr int64_t kMinTilesPerSplit = 8;

SplitPlan plan_splits(const fa8_fwd_params* p, int splits_req) {
  SplitPlan sp;
  if (p->cu_seqlens_q || p->batch <= 0 || p->heads <= 0 || p->seqlen_q <= 0 ||
      p->seqlen_kv <= 0 || splits_req == 1)
    return sp;
  const int64_t nq = (p->seqlen_q + fa8::kBlockM - 1) / fa8::kBlockM;
  const int64_t n_kv = (p->seqlen_kv + fa8::kBlockN - 1) / fa8::kBlockN;
  sp.qtiles = p->batch * p->heads * nq;
  int64_t ns;
  if (splits_req > 1) {
    ns = splits_req;
  } else {
    // Split only when the grid would not fill the GPU and every share keeps
    // at least kMinTilesPerSplit K/V tiles: each split CTA pays a partial
    // round trip through the workspace and the last one a merge, which short
    // shares do not earn back (B1 H8 S512: 13.7 us unsplit, 19-21 us split).
    if (sp.qtiles >= kSmCount) return sp;  // the grid fills the GPU already
    ns = std::min<int64_t>((2 * kSmCount + sp.qtiles - 1) / sp.qtiles,  // two CTAs per SM
                           n_kv / kMinTilesPerSplit);
  }
  ns = std::min<int64_t>(std::min<int64_t>(ns, n_kv), kMaxSplits);
  if (ns < 2 || p->batch * ns > 65535) return sp;
  sp.splits = (int)ns;
  const int64_t units = sp.qtiles * ns;
  sp.cnt_bytes = (sp.qtiles * 4 + 255) / 256 * 256;
  sp.lse_bytes = (units * fa8::kBlockM * 4 + 255) / 256 * 256;
  sp.o_bytes = units * fa8::kBlockM * p->head_dim * 4;
  return sp;
}

template <int D>
int launch(const fa8_fwd_params* p, cudaStream_t stream, int dev, const SplitPlan& sp) {
  using C = fa8::TileCfg<D>;
  int st = setup_kernel_attr<D, false>(dev);
  if (!st) st = setup_kernel_attr<D, true>(dev);
  if (st) return st;
  const CUtensorMapSwizzle swz_qk =
      (D == 128) ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUtensorMap tq, tk, tv;
  memset(&tk, 0, sizeof(tk));
  memset(&tv, 0, sizeof(tv));
  // Packed variable-length layout: one "batch" of total rows per map.
  const bool varlen = p->cu_seqlens_q != nullptr;
  const uint64_t nb = varlen ? 1 : (uint64_t)p->batch;
  const uint64_t qsb = varlen ? 16 : (uint64_t)p->q_stride_b;
  const uint64_t ksb = varlen ? 16 : (uint64_t)p->k_stride_b;
  const uint64_t vsb = varlen ? 16 : (uint64_t)p->v_stride_b;
  st = make_map_u8(&tq, p->q, D, p->seqlen_q, p->heads, nb, p->q_stride_s, p->q_stride_h, qsb, D,
                   fa8::kBlockM, swz_qk);
  if (st) return st;
  if (p->seqlen_kv > 0)
    st = make_map_u8(&tk, p->k, D, p->seqlen_kv, p->heads_kv, nb, p->k_stride_s, p->k_stride_h,
                     ksb, D, fa8::kBlockN, swz_qk);
  if (st) return st;
  // V^T (BHDS): innermost = keys, rows = d. V (BHSD): innermost = d, rows =
  // keys — a V tile is then shaped and swizzled like a K tile.
  const bool v_bhsd = p->v_layout == FA8_V_BHSD;
  if (p->seqlen_kv > 0 && !v_bhsd)
    st = make_map_u8(&tv, p->v, p->seqlen_kv, D, p->heads_kv, nb, p->v_stride_r, p->v_stride_h,
                     vsb, fa8::kBlockN, D, CU_TENSOR_MAP_SWIZZLE_128B);
  else if (p->seqlen_kv > 0)
    st = make_map_u8(&tv, p->v, D, p->seqlen_kv, p->heads_kv, nb, p->v_stride_r, p->v_stride_h,
                     vsb, D, fa8::kBlockN, swz_qk);
  if (st) return st;
  // O as a 4-D fp16 map {D, rows, heads, batch}, box 64 x 128, 128B swizzle.
  CUtensorMap to;
  memset(&to, 0, sizeof(to));
  bool o_tma = false;
  if (p->out_dtype == FA8_OUT_F16 && (p->o_stride_s * 2) % 16 == 0 && (p->o_stride_h * 2) % 16 == 0 &&
      (varlen || (p->o_stride_b * 2) % 16 == 0) && p->o_stride_h > 0 && p->o_stride_s > 0) {
    auto enc = get_encode_fn();
    if (enc) {
      cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)p->seqlen_q, (cuuint64_t)p->heads, nb};
      cuuint64_t strides[3] = {(cuuint64_t)p->o_stride_s * 2, (cuuint64_t)p->o_stride_h * 2,
                               varlen ? 16ull : (cuuint64_t)(p->o_stride_b > 0 ? p->o_stride_b * 2 : 16)};
      cuuint32_t box[4] = {64, (cuuint32_t)fa8::kBlockM, 1, 1};
      cuuint32_t estr[4] = {1, 1, 1, 1};
      o_tma = enc(&to, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, p->o, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
  }

  fa8::KernelParams kp;
  kp.batch = (int)p->batch;
  kp.heads = (int)p->heads;
  kp.heads_kv = (int)p->heads_kv;
  kp.seqlen_q = (int)p->seqlen_q;
  kp.seqlen_kv = (int)p->seqlen_kv;
  kp.head_group = (int)(p->heads / p->heads_kv);
  kp.causal = p->causal ? 1 : 0;
  kp.out_kind = p->out_dtype;
  kp.o_esize = p->out_dtype == FA8_OUT_E4M3 ? 1 : (p->out_dtype == FA8_OUT_F32 ? 4 : 2);
  kp.split_keys = p->split_keys < 0 ? fa8::kDefaultSplitKeys : p->split_keys;
  const int rows_per_cta = fa8::kBlockM;
  const int64_t rows = varlen ? p->max_seqlen_q : p->seqlen_q;
  kp.n_qblocks = (int)((rows + rows_per_cta - 1) / rows_per_cta);
  kp.cu_seqlens_q = p->cu_seqlens_q;
  kp.cu_seqlens_kv = p->cu_seqlens_kv;
  kp.o_tma = o_tma ? 1 : 0;
  kp.scale_log2 = p->softmax_scale * p->descale_q * p->descale_k * 1.4426950408889634f;
  kp.o_scale = p->descale_v;
  kp.q_offset = p->q_offset;
  kp.kv_offset = p->kv_offset;
  kp.o = p->o;
  kp.o_sb = p->o_stride_b;
  kp.o_sh = p->o_stride_h;
  kp.o_ss = p->o_stride_s;
  kp.lse = p->lse;
  kp.lse_sb = p->lse_stride_b;
  kp.lse_sh = p->lse_stride_h;
  kp.status = p->status;
  kp.timeout_cycles = p->wait_timeout_cycles > 0 ? p->wait_timeout_cycles : fa8::kTimeoutCycles;
  kp.debug_skip_kv_loads = p->debug_skip_kv_loads;
  kp.dq_bh = p->descale_q_bh;
  kp.dk_bh = p->descale_k_bh;
  kp.dv_bh = p->descale_v_bh;
  kp.dq_sb = p->descale_q_stride_b;
  kp.dq_sh = p->descale_q_stride_h;
  kp.dkv_sb = p->descale_kv_stride_b;
  kp.dkv_sh = p->descale_kv_stride_h;
  kp.kv_splits = sp.splits;
  kp.part_o = nullptr;
  kp.part_lse = nullptr;
  kp.split_cnt = nullptr;
  if (sp.splits > 1) {
    char* ws = static_cast<char*>(p->workspace);
    kp.split_cnt = reinterpret_cast<unsigned int*>(ws);
    kp.part_lse = reinterpret_cast<float*>(ws + sp.cnt_bytes);
    kp.part_o = reinterpret_cast<float*>(ws + sp.cnt_bytes + sp.lse_bytes);
  }
  if (varlen) {  // sequences are addressed by their packed row offsets
    kp.o_sb = 0;
    kp.lse_sb = 0;
  }

  dim3 grid(kp.n_qblocks, (unsigned)p->heads, (unsigned)(p->batch * sp.splits));
  if (v_bhsd)
    fa8::fa8_fwd_kernel<D, true><<<grid, fa8::kThreads, C::kSmemAlloc, stream>>>(tq, tk, tv, to, kp);
  else
    fa8::fa8_fwd_kernel<D, false><<<grid, fa8::kThreads, C::kSmemAlloc, stream>>>(tq, tk, tv, to, kp);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "fa8_fwd_kernel launch");
  return FA8_OK;
}

}  // namespace

extern "C" {

void fa8_fwd_params_init(fa8_fwd_params* p, int64_t batch, int64_t heads, int64_t heads_kv,
                         int64_t seqlen_q, int64_t seqlen_kv, int64_t head_dim) {
  memset(p, 0, sizeof(*p));
  p->batch = batch;
  p->heads = heads;
  p->heads_kv = heads_kv;
  p->seqlen_q = seqlen_q;
  p->seqlen_kv = seqlen_kv;
  p->head_dim = head_dim;
  p->q_stride_s = head_dim;
  p->q_stride_h = seqlen_q * head_dim;
  p->q_stride_b = heads * seqlen_q * head_dim;
  p->k_stride_s = head_dim;
  p->k_stride_h = seqlen_kv * head_dim;
  p->k_stride_b = heads_kv * seqlen_kv * head_dim;
  p->v_stride_r = seqlen_kv;  // BHDS: d rows of seqlen_kv keys
  p->v_stride_h = head_dim * seqlen_kv;
  p->v_stride_b = heads_kv * head_dim * seqlen_kv;
  p->o_stride_s = head_dim;
  p->o_stride_h = seqlen_q * head_dim;
  p->o_stride_b = heads * seqlen_q * head_dim;
  p->lse_stride_h = seqlen_q;
  p->lse_stride_b = heads * seqlen_q;
  p->softmax_scale = head_dim > 0 ? 1.0f / sqrtf((float)head_dim) : 1.0f;
  p->causal = 0;
  p->v_layout = FA8_V_BHDS;
  p->out_dtype = FA8_OUT_F16;
  p->split_keys = -1;
  p->descale_q = 1.0f;
  p->descale_k = 1.0f;
  p->descale_v = 1.0f;
  p->descale_q_stride_b = heads;
  p->descale_q_stride_h = 1;
  p->descale_kv_stride_b = heads_kv;
  p->descale_kv_stride_h = 1;
}

int fa8_fwd(const fa8_fwd_params* p, void* stream) {
  if (!p) return set_msg(FA8_ERR_INVALID_ARG, "params is NULL");
  if (p->batch < 0 || p->heads < 0 || p->heads_kv < 0 || p->seqlen_q < 0 || p->seqlen_kv < 0)
    return set_msg(FA8_ERR_INVALID_ARG, "negative size");
  if (p->head_dim != 64 && p->head_dim != 128)
    return set_msg(FA8_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (p->v_layout != FA8_V_BHDS && p->v_layout != FA8_V_BHSD)
    return set_msg(FA8_ERR_INVALID_ARG, "v_layout must be FA8_V_BHDS or FA8_V_BHSD");
  if (p->out_dtype != FA8_OUT_F16 && p->out_dtype != FA8_OUT_E4M3 && p->out_dtype != FA8_OUT_F32)
    return set_msg(FA8_ERR_INVALID_ARG, "out_dtype must be FA8_OUT_F16, FA8_OUT_E4M3 or FA8_OUT_F32");
  if (p->batch == 0 || p->heads == 0 || p->seqlen_q == 0) return FA8_OK;
  if (p->cu_seqlens_q || p->cu_seqlens_kv) {
    if (!p->cu_seqlens_q || !p->cu_seqlens_kv)
      return set_msg(FA8_ERR_INVALID_ARG, "varlen needs both cu_seqlens_q and cu_seqlens_kv");
    if (p->max_seqlen_q <= 0 || p->max_seqlen_q > p->seqlen_q)
      return set_msg(FA8_ERR_INVALID_ARG, "varlen needs 0 < max_seqlen_q <= total query rows");
    if (p->q_offset || p->kv_offset)
      return set_msg(FA8_ERR_UNSUPPORTED, "varlen does not take context-parallel offsets");
  }
  if (p->heads_kv <= 0 || p->heads % p->heads_kv != 0)
    return set_msg(FA8_ERR_UNSUPPORTED, "heads must be a multiple of heads_kv");
  if (p->batch > 65535 || p->heads > 65535 || p->seqlen_q > (1ll << 30) ||
      p->seqlen_kv > (1ll << 30))
    return set_msg(FA8_ERR_UNSUPPORTED, "size exceeds the supported grid / index range");
  if (!p->q || !p->o || (p->seqlen_kv > 0 && (!p->k || !p->v)))
    return set_msg(FA8_ERR_INVALID_ARG, "null tensor pointer");
  if (!(p->softmax_scale > 0.f) || !std::isfinite(p->softmax_scale))
    return set_msg(FA8_ERR_INVALID_ARG, "softmax_scale must be positive and finite");
  for (float d : {p->descale_q, p->descale_k, p->descale_v})
    if (!(d > 0.f) || !std::isfinite(d))
      return set_msg(FA8_ERR_INVALID_ARG, "descale factors must be positive and finite");
  if (!aligned16(p->q) || !aligned16(p->o) ||
      (p->seqlen_kv > 0 && (!aligned16(p->k) || !aligned16(p->v))))
    return set_msg(FA8_ERR_ALIGNMENT, "tensor base addresses must be 16-byte aligned");
  const int64_t osz = p->out_dtype == FA8_OUT_E4M3 ? 1 : (p->out_dtype == FA8_OUT_F32 ? 4 : 2);
  const int64_t s16[] = {p->q_stride_b, p->q_stride_h, p->q_stride_s, p->k_stride_b,
                         p->k_stride_h, p->k_stride_s, p->v_stride_b, p->v_stride_h,
                         p->v_stride_r};
  const int n_checked = p->seqlen_kv > 0 ? 9 : 3;  // no K/V access without keys
  for (int j = 0; j < n_checked; ++j) {
    const int64_t s = s16[j];
    if (s <= 0 || (s % 16) != 0)
      return set_msg(FA8_ERR_ALIGNMENT,
                     "Q/K/V strides must be positive multiples of 16 elements (TMA); for BHDS V "
                     "this means seqlen_kv % 16 == 0");
  }
  if (p->v_layout == FA8_V_BHSD && p->seqlen_kv > 0 && p->v_stride_r < p->head_dim) {
    return set_msg(FA8_ERR_INVALID_ARG, "BHSD V rows overlap (v_stride_r < head_dim)");
  }
  if ((p->o_stride_s * osz) % 16 || (p->o_stride_h * osz) % 16 || (p->o_stride_b * osz) % 16)
    return set_msg(FA8_ERR_ALIGNMENT, "O strides must be multiples of 16 bytes");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaGetDevice");
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0)
    return set_msg(FA8_ERR_NO_DEVICE, "the current device is not sm_100 (B200)");

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (p->kv_splits < 0) return set_msg(FA8_ERR_INVALID_ARG, "kv_splits must be >= 0");
  SplitPlan sp = plan_splits(p, p->kv_splits);
  if (sp.splits > 1) {
    const bool fits = p->workspace && p->workspace_bytes >= sp.bytes() &&
                      (reinterpret_cast<uintptr_t>(p->workspace) & 255) == 0;
    if (!fits) {
      if (p->kv_splits > 1)
        return set_msg(FA8_ERR_INVALID_ARG,
                       "kv_splits > 1 needs a 256-byte aligned workspace of "
                       "fa8_fwd_workspace_size() bytes");
      sp = SplitPlan();  // automatic: run without splitting
    }
  }
  if (p->sm_budget < 0) return set_msg(FA8_ERR_INVALID_ARG, "sm_budget must be >= 0");
  cudaStream_t ls = nullptr;
  if (p->sm_budget > 0) {
    const int rc = budget_stream(dev, p->sm_budget, &ls);
    if (rc != FA8_OK) return rc;
  }
  if (!ls) return p->head_dim == 128 ? launch<128>(p, s, dev, sp) : launch<64>(p, s, dev, sp);
  // Budgeted launch: ordered after the caller's stream and before its next work.
  cudaEvent_t e_in = nullptr, e_out = nullptr;
  e = cudaEventCreateWithFlags(&e_in, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&e_out, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventRecord(e_in, s);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(ls, e_in, 0);
  int rc = FA8_ERR_CUDA;
  if (e == cudaSuccess) {
    rc = p->head_dim == 128 ? launch<128>(p, ls, dev, sp) : launch<64>(p, ls, dev, sp);
    e = cudaEventRecord(e_out, ls);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, e_out, 0);
  }
  if (e_in) cudaEventDestroy(e_in);
  if (e_out) cudaEventDestroy(e_out);
  if (e != cudaSuccess) return set_cuda_error(e, "sm_budget stream ordering");
  return rc;
}

int64_t fa8_fwd_workspace_size(const fa8_fwd_params* p) {
  if (!p || p->kv_splits < 0 || (p->head_dim != 64 && p->head_dim != 128)) return 0;
  return plan_splits(p, p->kv_splits).bytes();
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Forward for callers that cannot allocate device memory.
//
// Split-KV needs scratch (the shares' partial outputs and the per-tile
// counters). fa8_fwd takes it from the caller; some callers have no way to
// provide it: code running inside a framework that owns the device memory
// pool, plugins that may not call cudaMalloc (or may not call it from the
// thread that launches), and runtimes whose launch path must not allocate.
// fa8_fwd_static_scratch gives them the same forward with the scratch taken
// from this fixed-size array, which is part of the library's image: every GPU
// that loads the library holds it until the process exits.
namespace {

constexpr int64_t kStaticScratchBytes = 8ll << 20;  // 8 MiB
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch on `dev`, looked up once per device with
// that device current. In host code the symbol itself is only a host-side
// stand-in: it must never be passed to a kernel as a pointer.
int static_scratch_ptr(int dev, void** out) {
  static std::once_flag flags[64];
  static void* ptrs[64];
  static cudaError_t errs[64];
  if (dev < 0 || dev >= 64) return set_msg(FA8_ERR_INVALID_ARG, "device index out of range");
  std::call_once(flags[dev], [dev] {
    errs[dev] = cudaGetSymbolAddress(&ptrs[dev], g_static_scratch);
  });
  if (errs[dev] != cudaSuccess) return set_cuda_error(errs[dev], "cudaGetSymbolAddress");
  *out = ptrs[dev];
  return FA8_OK;
}

}  // namespace

extern "C" {

int fa8_fwd_static_scratch(const fa8_fwd_params* p, void* stream) {
  if (!p) return set_msg(FA8_ERR_INVALID_ARG, "params is NULL");
  if (p->kv_splits < 0) return set_msg(FA8_ERR_INVALID_ARG, "kv_splits must be >= 0");
  fa8_fwd_params q = *p;
  q.workspace = nullptr;
  q.workspace_bytes = 0;
  const int64_t need = fa8_fwd_workspace_size(&q);
  if (need > kStaticScratchBytes) {
    snprintf(g_last_msg, sizeof(g_last_msg),
             "fa8_fwd_static_scratch: this call's split-KV plan needs %lld bytes of scratch, "
             "more than the library's fixed %lld; pass kv_splits = 1 (no split) or call "
             "fa8_fwd with a workspace",
             (long long)need, (long long)kStaticScratchBytes);
    return FA8_ERR_INVALID_ARG;
  }
  if (need > 0) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_cuda_error(e, "cudaGetDevice");
    void* ptr = nullptr;
    const int st = static_scratch_ptr(dev, &ptr);
    if (st) return st;
    // The array keeps the previous call's contents; the split counters at its
    // start must be zero (a call that timed out can leave them set).
    const SplitPlan sp = plan_splits(&q, q.kv_splits);
    e = cudaMemsetAsync(ptr, 0, (size_t)sp.cnt_bytes, reinterpret_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return set_cuda_error(e, "cudaMemsetAsync (split counters)");
    q.workspace = ptr;
    q.workspace_bytes = kStaticScratchBytes;
  }
  return fa8_fwd(&q, stream);
}

int64_t fa8_static_scratch_bytes(void) { return kStaticScratchBytes; }

const char* fa8_status_string(int status) {
  switch (status) {
    case FA8_OK: return "ok";
    case FA8_ERR_INVALID_ARG: return "invalid argument";
    case FA8_ERR_UNSUPPORTED: return "unsupported configuration";
    case FA8_ERR_ALIGNMENT: return "alignment / stride requirement violated";
    case FA8_ERR_CUDA: return "CUDA runtime error";
    case FA8_ERR_DRIVER: return "CUDA driver entry point unavailable";
    case FA8_ERR_NO_DEVICE: return "no sm_100 device";
    default: return "unknown status";
  }
}

const char* fa8_last_error_message(void) { return g_last_msg; }

uint64_t fa8_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

}  // extern "C"

#ifdef FA8_TRACE
extern "C" int fa8_trace_cta_fetch(long long* host_buf) {
  return cudaMemcpyFromSymbol(host_buf, fa8::fa8_trace_cta, sizeof(fa8::fa8_trace_cta)) ==
                 cudaSuccess
             ? 0
             : 1;
}
extern "C" int fa8_trace_fetch(long long* host_buf) {
  return cudaMemcpyFromSymbol(host_buf, fa8::fa8_trace_buf, sizeof(fa8::fa8_trace_buf)) ==
                 cudaSuccess
             ? 0
             : 1;
}
#endif

// Used by the auxiliary kernels' translation unit.
void fa8_note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
int fa8_note_cuda_error(cudaError_t e, const char* where) { return set_cuda_error(e, where); }
int fa8_note_error(int status, const char* msg) { return set_msg(status, msg); }
